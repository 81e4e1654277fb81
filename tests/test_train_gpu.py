"""The MLP training step on the device against the
oracle's CPU port of the same step, at a reduced width where the CPU finishes
in seconds, and the README quick-start chain (config 1) against the oracle."""

from __future__ import annotations

import pytest
import torch

import oracle as O
from conftest import assert_close, assert_close_terms

pytestmark = pytest.mark.gpu


def test_training_step_matches_the_cpu_step(backend):
    from tensorplay_mlu_b200.train import DataParallelMLP, MLPConfig, init_params_host, make_batch_host

    cfg = MLPConfig(d_in=256, d_hidden=1024, batch=128, lr=0.05)
    params = init_params_host(cfg, seed=0)
    x, t = make_batch_host(cfg, seed=0)
    model = DataParallelMLP(cfg, device=0, host_params=params)
    ops = backend.ops
    loss = model.step(ops.to_device(x), ops.to_device(t))
    got_loss = ops.item(loss)
    ref = [p.clone() for p in params]
    want_loss = O.mlp_step(x, t, ref[0], ref[1], ref[2], ref[3], cfg.lr)
    assert abs(got_loss - want_loss) <= 1e-2 * max(1.0, abs(want_loss))
    for dev_p, want in zip(model.params(), ref):
        # bf16 parameters after one step: within bf16 tolerance of the CPU step.
        assert_close(ops.to_host(dev_p), want, torch.bfloat16)
    # The step really moved the weights.
    assert not torch.equal(ops.to_host(model.w1), params[0])


def test_training_steps_reduce_the_loss(backend):
    from tensorplay_mlu_b200.train import DataParallelMLP, MLPConfig, make_batch_host

    cfg = MLPConfig(d_in=256, d_hidden=1024, batch=256, lr=0.5)
    model = DataParallelMLP(cfg, device=0)
    x, t = make_batch_host(cfg, seed=0)
    dx, dt = backend.ops.to_device(x), backend.ops.to_device(t)
    losses = [backend.ops.item(model.step(dx, dt)) for _ in range(5)]
    assert losses[-1] < losses[0]


def test_quick_start_chain(backend):
    """README quick-start: y = x @ w; z = relu(y).softmax(-1);
    loss = z.sum(); backward -- gradients of x and w, fp32 [256, 256]."""
    ops = backend.ops
    g = torch.Generator().manual_seed(0)
    x = torch.randn(256, 256, generator=g)
    w = torch.randn(256, 256, generator=g)
    dx_, dw_ = ops.to_device(x), ops.to_device(w)
    y = ops.mm(dx_, dw_)
    r = ops.relu(y)
    z = ops.softmax(r, -1)
    loss = ops.sum(z)
    dz = ops.fill_(torch.empty_like(z), 1.0)          # d loss / d z
    dr = ops._softmax_backward_data(dz, z, -1, torch.float32)
    dy = ops.threshold_backward(dr, y, 0.0)
    gx = ops.mm(dy, dw_.t())
    gw = ops.mm(dx_.t(), dy)
    # oracle chain
    yo = O.gemm(x, w)
    ro = O.unary(O.RELU, yo)
    zo = O.softmax(ro, -1)
    lo = O.reduce(O.SUM, zo, None, torch.float32)
    dro = O.softmax_backward(torch.ones(256, 256), zo, -1)
    dyo = O.unary_backward(O.THRESHOLD_BACKWARD, dro, yo, 0.0)
    # Sums and products within fp32's 1e-5 of their terms' magnitude (the
    # loss sums 65536 positive softmax values; the gradients are products).
    assert_close_terms(loss, lo, O.reduce(O.SUM, zo.abs(), None, torch.float32))
    assert_close_terms(gx, O.gemm(dyo, w.t()), O.gemm(dyo.abs(), w.t().abs()))
    assert_close_terms(gw, O.gemm(x.t(), dyo), O.gemm(x.t().abs(), dyo.abs()))
