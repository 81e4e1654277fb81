"""The CPU port of the MLP step (oracle/mlp.c), which is both the checker of
the device step and the timed CPU baseline: its blocked matrix product
against float64 sums on ragged shapes and transposed operands, and one whole
step against the same step written out in PyTorch CPU operations (bf16
storage between operators, fp32 arithmetic inside them)."""

from __future__ import annotations

import pytest
import torch

import oracle as O
from conftest import assert_close, assert_close_terms


@pytest.mark.parametrize("m,n,k", [(1, 1, 1), (7, 33, 5), (129, 257, 300), (64, 4100, 513), (300, 31, 1030)])
@pytest.mark.parametrize("layout", ["nn", "tn", "nt"])
def test_blocked_product(m, n, k, layout):
    g = torch.Generator().manual_seed(m * 7 + n)
    a = torch.randn(m, k, generator=g)
    b = torch.randn(k, n, generator=g)
    if layout[0] == "t":
        a = a.t().contiguous().t()
    if layout[1] == "t":
        b = b.t().contiguous().t()
    want = a.double() @ b.double()
    terms = a.double().abs() @ b.double().abs()
    assert_close_terms(O.gemm_blocked(a, b), want, terms, torch.float32)


def _torch_step(x, t, w1, b1, w2, b2, lr):
    """The step in PyTorch CPU operations, rounding to bf16 after each operator."""
    bf, f = torch.bfloat16, torch.float32
    h = (x.float() @ w1.float().t() + b1.float()).to(bf)
    a = torch.nn.functional.gelu(h.float()).to(bf)
    out = (a.float() @ w2.float().t() + b2.float()).to(bf)
    diff = (out.float() - t.float()).to(bf)
    loss = (diff.float() ** 2).to(bf).double().mean().item()
    d_out = (diff.float() * (2.0 / diff.numel())).to(bf)
    d_a = (d_out.float() @ w2.float()).to(bf)
    hf = h.float()
    grad = 0.5 * (1 + torch.erf(hf * 0.70710678)) + hf * torch.exp(-0.5 * hf * hf) * 0.39894228
    d_h = (d_a.float() * grad).to(bf)
    dw2 = (d_out.float().t() @ a.float()).to(bf)
    db2 = d_out.float().sum(0).to(bf)
    dw1 = (d_h.float().t() @ x.float()).to(bf)
    db1 = d_h.float().sum(0).to(bf)
    new = [(p.float() - lr * g.float()).to(bf) for p, g in ((w1, dw1), (b1, db1), (w2, dw2), (b2, db2))]
    return loss, new


def test_mlp_step_matches_its_pytorch_restatement():
    from tensorplay_mlu_b200.train import MLPConfig, init_params_host, make_batch_host

    cfg = MLPConfig(d_in=96, d_hidden=200, batch=40, lr=0.5)
    params = [p.contiguous() for p in init_params_host(cfg, seed=0)]
    x, t = make_batch_host(cfg, seed=0)
    want_loss, want = _torch_step(x, t, *params, cfg.lr)
    got = [p.clone() for p in params]
    loss = O.mlp_step(x, t, *got, cfg.lr)
    assert abs(loss - want_loss) <= 1e-2 * max(1.0, abs(want_loss))
    for g_, w_ in zip(got, want):
        assert_close(g_, w_, torch.bfloat16)
    assert not torch.equal(got[0], params[0])


def test_thread_count_can_be_set():
    before = O.num_threads()
    O.set_num_threads(2)
    assert O.num_threads() == 2
    O.set_num_threads(before)
    assert O.num_threads() == before
