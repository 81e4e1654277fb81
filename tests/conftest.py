"""Shared test setup: the ``gpu`` marker, backend loading, tolerances.

CPU tests (``-m "not gpu"``) check the oracle against the golden fixtures,
the host-side logic and the C ABI's exports.  GPU tests (``-m gpu``) run the
sm_100a kernels through the C ABI and compare them with the oracle; they fail
(never skip) when the native library or the GPU is missing, so a silent
fallback cannot pass.
"""

from __future__ import annotations

import os
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

# Relative tolerances: max|got - want| <= TOL * max(max|want|, 1) * scale.
# fp32 1e-5 and bf16 1e-2 are the north-star bounds; fp16 and fp64 follow the
# same rule with their own precisions.
TOL = {
    torch.float32: 1e-5,
    torch.bfloat16: 1e-2,
    torch.float16: 2e-3,
    torch.float64: 1e-12,
}


def assert_close(got: torch.Tensor, want: torch.Tensor, dtype=None, scale: float = 1.0) -> None:
    dtype = dtype or want.dtype
    got = got.detach().cpu()
    want = want.detach().cpu()
    assert tuple(got.shape) == tuple(want.shape), (tuple(got.shape), tuple(want.shape))
    if got.numel() == 0:
        return
    if not dtype.is_floating_point:
        assert torch.equal(got, want), "integer results differ"
        return
    g, w = got.double(), want.double()
    both_nan = torch.isnan(g) & torch.isnan(w)
    assert torch.equal(torch.isnan(g), torch.isnan(w)), "NaN positions differ"
    g = torch.where(both_nan, torch.zeros_like(g), g)
    w = torch.where(both_nan, torch.zeros_like(w), w)
    err = (g - w).abs().max().item()
    ref = max(w.abs().max().item(), 1.0) * scale
    assert err <= TOL[dtype] * ref, f"max error {err} > {TOL[dtype] * ref} ({dtype})"


def assert_close_terms(got: torch.Tensor, want: torch.Tensor, terms, dtype=None) -> None:
    """The bound for results that are sums -- reductions, products, scans,
    scatter-adds: max|got - want| <= TOL * max(max(terms), 1), where `terms`
    is the magnitude of what was summed into each result (sum |x_i| for a
    sum, sum |a_k b_k| for a product; a tensor shaped like `want`, or a
    number).  Rounding errors of a sum scale with its terms, not with its
    value, which cancellation can make arbitrarily small; so this is the same
    relative tolerance (fp32 1e-5, bf16 1e-2) taken against the terms,
    with no extra factor."""
    dtype = dtype or want.dtype
    got = got.detach().cpu()
    want = want.detach().cpu()
    assert tuple(got.shape) == tuple(want.shape), (tuple(got.shape), tuple(want.shape))
    if got.numel() == 0:
        return
    g, w = got.double(), want.double()
    assert torch.equal(torch.isnan(g), torch.isnan(w)), "NaN positions differ"
    nan = torch.isnan(g)
    g = torch.where(nan, torch.zeros_like(g), g)
    w = torch.where(nan, torch.zeros_like(w), w)
    err = (g - w).abs().max().item()
    t = terms.detach().double().abs().max().item() if isinstance(terms, torch.Tensor) else abs(float(terms))
    ref = max(t, w.abs().max().item(), 1.0)
    assert err <= TOL[dtype] * ref, f"max error {err} > {TOL[dtype] * ref} ({dtype}, terms {t})"


def assert_equal(got: torch.Tensor, want: torch.Tensor) -> None:
    got, want = got.detach().cpu(), want.detach().cpu()
    assert got.dtype == want.dtype, (got.dtype, want.dtype)
    assert tuple(got.shape) == tuple(want.shape), (tuple(got.shape), tuple(want.shape))
    if got.dtype.is_floating_point:
        same = (got == want) | (torch.isnan(got) & torch.isnan(want))
        assert bool(same.all()), "values differ"
    else:
        assert torch.equal(got, want), "values differ"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU and the built CUDA library")


@pytest.fixture(scope="session")
def backend():
    """The loaded backend on a GPU box (fails, does not skip, without one)."""
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    import tensorplay_mlu_b200 as tpb

    tpb.load()
    return tpb
