"""BASELINE config 4 at its own size: one training step of Linear 4096 ->
16384, GELU, Linear 16384 -> 4096 on a batch of 8192 (bf16, nn.Linear init
from seed 0, inputs ~N(0, 1), MSE loss, SGD lr 1e-3), checked piece by piece
against the CPU oracle -- the full-size counterpart of the reference's
device-versus-host training-step test (tests/test_mlu.py:363-378 of
tensorplay-mlu).

* each of the five products is checked on 4096 sampled outputs, computed in
  float64 from the device's own inputs to that product;
* gelu, gelu_backward, the MSE gradient, the bias gradients and the SGD
  update are checked over every element;
* the loss is checked against a float64 mean over the device's output.

Tolerances are the north-star bf16 bound (1e-2 relative), against the
magnitude of the summed terms for products and sums
(conftest.assert_close_terms).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle as O
from conftest import assert_close, assert_close_terms

pytestmark = pytest.mark.gpu

SAMPLES = 4096


@pytest.fixture(scope="module")
def step(backend):
    from tensorplay_mlu_b200.train import DataParallelMLP, MLPConfig, init_params_host, make_batch_host

    ops = backend.ops
    cfg = MLPConfig()
    assert (cfg.d_in, cfg.d_hidden, cfg.batch) == (4096, 16384, 8192)
    params = init_params_host(cfg, seed=0)
    x, t = make_batch_host(cfg, seed=0)
    model = DataParallelMLP(cfg, device=0, host_params=params)
    model.trace = {}
    loss = model.step(ops.to_device(x), ops.to_device(t))
    torch.cuda.synchronize()
    tr = {k: (ops.to_host(v) if isinstance(v, torch.Tensor) else v) for k, v in model.trace.items()}
    tr["loss"] = ops.item(loss)
    tr["params_before"] = params
    tr["params_after"] = [ops.to_host(p) for p in model.params()]
    tr["grads"] = [ops.to_host(g) for g in model.grads()]  # dW1, db1, dW2, db2
    tr["cfg"] = cfg
    del model
    torch.cuda.empty_cache()
    return tr


def _sample(m, n, seed):
    rng = np.random.default_rng(seed)
    idx = np.zeros((SAMPLES, 3), dtype=np.int64)
    idx[:, 1] = rng.integers(0, m, SAMPLES)
    idx[:, 2] = rng.integers(0, n, SAMPLES)
    return idx


def _check_product(got_full, a, b, seed, bias=None):
    """got_full [M, N] (bf16, host) against a @ b (+ bias) on sampled outputs."""
    M, N = got_full.shape
    idx = _sample(M, N, seed)
    c = bias.view(1, -1).expand(M, N) if bias is not None else None
    want = O.gemm_sampled(a, b, idx, c, 1.0, 1.0 if c is not None else 0.0)
    terms = O.gemm_sampled(a.abs(), b.abs(), idx, c.abs() if c is not None else None, 1.0,
                           1.0 if c is not None else 0.0)
    got = got_full[idx[:, 1], idx[:, 2]]
    assert_close_terms(got, torch.from_numpy(want), torch.from_numpy(terms), torch.bfloat16)


def test_forward_products(step):
    w1, b1, w2, b2 = step["params_before"]
    _check_product(step["h"], step["x"], w1.t(), 1, b1)          # h = x W1^T + b1
    if "out" in step:
        _check_product(step["out"], step["a"], w2.t(), 2, b2)    # out = a W2^T + b2


def test_gelu_over_every_element(step):
    assert_close(step["a"], O.unary(O.GELU, step["h"]), torch.bfloat16)


def test_mse_gradient_and_loss(step):
    n = step["t"].numel()
    out, t = step["out"], step["t"]
    diff = O.binary(O.SUB, out, t)
    want = O.binary_scalar(O.MUL, diff, 2.0 / n)
    assert_close(step["d_out"], want, torch.bfloat16)
    # loss = mean((out - t)^2), in float64 over the device's output.
    ref = ((out.double() - t.double()) ** 2).mean().item()
    assert abs(step["loss"] - ref) <= 1e-2 * max(1.0, abs(ref)), (step["loss"], ref)


def test_backward_products(step):
    w1, b1, w2, b2 = step["params_before"]
    dw1, db1, dw2, db2 = step["grads"]
    _check_product(dw2, step["d_out"].t(), step["a"], 3)         # dW2 = d_out^T a
    if "d_a" in step:
        _check_product(step["d_a"], step["d_out"], w2, 4)        # d_a = d_out W2
    _check_product(dw1, step["d_h"].t(), step["x"], 5)           # dW1 = d_h^T x


def test_gelu_backward_over_every_element(step):
    if "d_a" in step:
        want = O.unary_backward(O.GELU_BACKWARD, step["d_a"], step["h"])
        assert_close(step["d_h"], want, torch.bfloat16)
    else:
        # d_a was never stored: recompute it on sampled entries in float64,
        # round it to bf16 as the step does, and apply gelu_backward there.
        w2 = step["params_before"][2]
        idx = _sample(*step["d_h"].shape, 6)
        d_a = torch.from_numpy(O.gemm_sampled(step["d_out"], w2, idx)).to(torch.bfloat16)
        h = step["h"][idx[:, 1], idx[:, 2]]
        want = O.unary_backward(O.GELU_BACKWARD, d_a, h)
        assert_close(step["d_h"][idx[:, 1], idx[:, 2]], want, torch.bfloat16)


def test_bias_gradients_over_every_element(step):
    dw1, db1, dw2, db2 = step["grads"]
    for got, src in ((db2, step["d_out"]), (db1, step["d_h"])):
        want = O.reduce(O.SUM, src, [0], torch.bfloat16)
        terms = O.reduce(O.SUM, O.unary(O.ABS, src.float()), [0], torch.float32)
        assert_close_terms(got, want, terms, torch.bfloat16)


def test_sgd_update_over_every_element(step):
    lr = step["cfg"].lr
    for before, g, after in zip(step["params_before"], step["grads"], step["params_after"]):
        # At this config (MSE averaged over 33.5M outputs, lr 1e-3) lr * g is
        # mostly below the weights' bf16 resolution, so most weights keep
        # their bits; the check is that every element is the oracle's.
        want = O.binary(O.ADD, before, g, alpha=-lr)
        assert_close(after, want, torch.bfloat16)
