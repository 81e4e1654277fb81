"""Indexing, scatter, scans and where (tensorplay-mlu IndexKernels.cpp:
352-367) against the oracle over every dtype: exact for integers, gathers,
selects, replacement, amax / amin and where; within the dtype's tolerance
for floating sums and products (atomic accumulation order)."""

from __future__ import annotations

import pytest
import torch

import oracle as O
from conftest import assert_close_terms, assert_equal

pytestmark = pytest.mark.gpu

FLOATS = [torch.float32, torch.bfloat16, torch.float16, torch.float64]
INTS = [torch.int64, torch.int32, torch.int16, torch.int8, torch.uint8]


def values(*shape, dtype, seed=0, lo=-40, hi=40):
    g = torch.Generator().manual_seed(seed)
    if dtype.is_floating_point:
        return (torch.randn(*shape, generator=g) * 3).to(dtype)
    if dtype == torch.bool:
        return torch.randint(0, 2, shape, generator=g).bool()
    if dtype == torch.uint8:
        lo = max(lo, 0)
    return torch.randint(lo, hi, shape, generator=g).to(dtype)


def indices(*shape, high, seed=1, low=0):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(low, high, shape, generator=g)


@pytest.fixture(scope="module")
def ops(backend):
    return backend.ops


# Unit roundoff of each floating type (half its machine epsilon).
UNIT = {torch.float32: 2.0 ** -24, torch.bfloat16: 2.0 ** -8, torch.float16: 2.0 ** -11, torch.float64: 2.0 ** -53}


def check(got, want, dtype, exact=False, terms=None):
    """Integers and exact ops bit for bit; a sum within the dtype's tolerance
    of the magnitude of its terms (`terms`: the same op on |values|)."""
    if exact or not dtype.is_floating_point:
        assert_equal(got.cpu() if got.device.type != "cpu" else got, want)
    else:
        assert_close_terms(got, want, terms if terms is not None else want.abs(), dtype)


def check_product(got, want, dtype, factors, per_step_rounding=None):
    """A product of up to `factors` values, formed in any order with a
    rounding after each multiply, is within gamma_n |exact| of the exact
    product (Higham, Accuracy and Stability of Numerical Algorithms, 3.1:
    gamma_n = n u / (1 - n u)), plus the oracle's own final rounding (u) --
    elementwise and relative, so near-zero products need no absolute floor.
    `per_step_rounding` is the type each multiply rounds to: the accumulation
    type (fp32, fp64 for fp64) for a scan, which rounds to the storage type
    once at the end; the storage type itself for atomic scatter updates."""
    got = got.cpu().double()
    want = want.double()
    step = per_step_rounding or (torch.float64 if dtype == torch.float64 else torch.float32)
    acc_u = UNIT[step]
    n = factors
    gamma = n * acc_u / (1 - n * acc_u) + 2 * UNIT[dtype]
    assert torch.equal(torch.isnan(got), torch.isnan(want))
    ok = (got - want).abs() <= gamma * want.abs() + 1e-30
    assert bool(ok.all()), f"max relative error {((got - want).abs() / want.abs()).max().item()} > {gamma}"


@pytest.mark.parametrize("dtype", FLOATS + INTS + [torch.bool])
def test_gather_and_backward(ops, dtype):
    x = values(30, 17, dtype=dtype)
    for dim, idx in ((0, indices(12, 17, high=30)), (1, indices(30, 9, high=17, low=-17)), (-1, indices(5, 4, high=17))):
        got = ops.gather(ops.to_device(x), dim, ops.to_device(idx))
        check(got, O.gather(x, dim, idx), dtype, exact=True)
    # A transposed (non-contiguous) input.
    base = values(17, 30, dtype=dtype, seed=2)
    idx = indices(30, 5, high=17, seed=3)
    got = ops.gather(ops.to_device(base).t(), 1, ops.to_device(idx))
    check(got, O.gather(base.t(), 1, idx), dtype, exact=True)
    if dtype != torch.bool:
        idx = indices(40, 17, high=30, seed=4)  # duplicates accumulate
        grad = values(40, 17, dtype=dtype, seed=5)
        got = ops.gather_backward(ops.to_device(grad), ops.to_device(x), 0, ops.to_device(idx))
        want = O.scatter(torch.zeros_like(x), 0, idx, grad, "add")
        terms = O.scatter(torch.zeros_like(x), 0, idx, grad.abs(), "add") if dtype.is_floating_point else None
        check(got, want, dtype, terms=terms)


@pytest.mark.parametrize("dtype", FLOATS + INTS)
def test_index_select_and_backward(ops, dtype):
    for shape, dim, n in (((50, 64), 0, 37), ((7, 33, 5), 1, 11), ((3, 4, 130), 2, 9), ((1000, 256), 0, 4096)):
        x = values(*shape, dtype=dtype, seed=6)
        idx = indices(n, high=shape[dim], seed=7)
        got = ops.index_select(ops.to_device(x), dim, ops.to_device(idx))
        check(got, O.index_select(x, dim, idx), dtype, exact=True)
        gshape = list(shape)
        gshape[dim] = n
        grad = values(*gshape, dtype=dtype, seed=8, lo=-5, hi=5)
        got = ops.index_select_backward(ops.to_device(grad), list(shape), dim, ops.to_device(idx))
        terms = O.index_add_zeros(list(shape), dim, idx, grad.abs()) if dtype.is_floating_point else None
        check(got, O.index_add_zeros(list(shape), dim, idx, grad), dtype, terms=terms)


@pytest.mark.parametrize("dtype", FLOATS + INTS)
def test_scatter_modes(ops, dtype):
    x = values(20, 9, dtype=dtype, seed=9, lo=-6, hi=6)
    src = values(30, 9, dtype=dtype, seed=10, lo=-3, hi=4)
    idx = indices(30, 9, high=20, seed=11)  # duplicates
    d = ops.to_device
    # Replacement without duplicates (torch.randperm columns).
    g = torch.Generator().manual_seed(12)
    perm = torch.stack([torch.randperm(20, generator=g)[:15] for _ in range(9)], 1)
    check(ops.scatter_reduce_op(d(x), 0, d(perm), d(src)), O.scatter(x, 0, perm, src[:15]), dtype, exact=True)
    fl = dtype.is_floating_point
    check(ops.scatter_add(d(x), 0, d(idx), d(src)), O.scatter(x, 0, idx, src, "add"), dtype,
          terms=O.scatter(x.abs(), 0, idx, src.abs(), "add") if fl else None)
    # The most factors any output of a prod reduction multiplies: its own
    # value and every source row that lands on it.
    factors = 1 + int(torch.bincount(idx[:, 0], minlength=20).max())
    for c in range(idx.shape[1]):
        factors = max(factors, 1 + int(torch.bincount(idx[:, c], minlength=20).max()))
    for red in ("sum", "prod", "amax", "amin", "mean"):
        for inc in (True, False):
            got = ops.scatter_reduce(d(x), 0, d(idx), d(src), red, inc)
            want = O.scatter(x, 0, idx, src, red, inc)
            if red in ("amax", "amin") or not fl:
                check(got, want, dtype, exact=True)
            elif red == "prod":
                check_product(got, want, dtype, factors, per_step_rounding=dtype)
            else:
                check(got, want, dtype, terms=O.scatter(x.abs(), 0, idx, src.abs(), red, inc))
    # In place, and the scatter.reduce spellings.
    y = d(x)
    ops.scatter_add_(y, 1, d(indices(20, 4, high=9, seed=13)), d(src[:20, :4]))
    check(y, O.scatter(x, 1, indices(20, 4, high=9, seed=13), src[:20, :4], "add"), dtype,
          terms=O.scatter(x.abs(), 1, indices(20, 4, high=9, seed=13), src[:20, :4].abs(), "add") if fl else None)
    y = d(x)
    ops.scatter_reduce_op_(y, 0, d(idx), d(src), "amax")
    check(y, O.scatter(x, 0, idx, src, "amax"), dtype, exact=True)


def test_scatter_bool_replace_and_rejects_bool_sums(ops):
    x = values(6, 4, dtype=torch.bool)
    src = values(6, 4, dtype=torch.bool, seed=3)
    perm = torch.stack([torch.randperm(6)[:6] for _ in range(4)], 1)
    check(ops.scatter_reduce_op(ops.to_device(x), 0, ops.to_device(perm), ops.to_device(src)),
          O.scatter(x, 0, perm, src), torch.bool, exact=True)
    with pytest.raises(RuntimeError, match="bool"):
        ops.scatter_add(ops.to_device(x), 0, ops.to_device(perm), ops.to_device(src))


@pytest.mark.parametrize("dtype", FLOATS + [torch.int64, torch.int32, torch.int16, torch.int8])
def test_cumsum_cumprod(ops, dtype):
    d = ops.to_device
    for shape, dim in (((13, 700), 1), ((700, 13), 0), ((4, 5, 6), 1), ((2, 100000), -1), ((5000, 3), 1)):
        x = values(*shape, dtype=dtype, seed=14, lo=-3, hi=4)
        got = ops.cumsum(d(x), dim)
        want = O.scan(x, dim, False)
        fl = dtype.is_floating_point
        check(got, want, dtype, terms=O.scan(x.abs(), dim, False) if fl else None)
        xs = values(*shape, dtype=dtype, seed=15, lo=-1, hi=2)
        if fl:
            xs = (1 + xs.double() / 50).to(dtype)
        got = ops.cumprod(d(xs), dim)
        if fl:
            check_product(got, O.scan(xs, dim, True), dtype, shape[dim if dim >= 0 else len(shape) + dim])
        else:
            check(got, O.scan(xs, dim, True), dtype)
    y = d(values(6, 8, dtype=dtype, seed=16, lo=-3, hi=4))
    yh = ops.to_host(y)
    want = O.scan(yh, 1, False)
    ops.cumsum_(y, 1)
    check(y, want, dtype, terms=O.scan(yh.abs(), 1, False) if dtype.is_floating_point else None)


def test_int32_cumsum_wraps_like_the_host(ops):
    x = torch.tensor([[2**31 - 1, 1, 5]], dtype=torch.int32)
    assert_equal(ops.to_host(ops.cumsum(ops.to_device(x), 1)), O.scan(x, 1, False))


@pytest.mark.parametrize("dtype", FLOATS + INTS + [torch.bool])
def test_where(ops, dtype):
    g = torch.Generator().manual_seed(17)
    cond = torch.rand(7, 1, 5, generator=g) > 0.4
    a = values(1, 6, 5, dtype=dtype, seed=18)
    b = values(7, 6, 1, dtype=dtype, seed=19)
    got = ops.where_self(ops.to_device(cond), ops.to_device(a), ops.to_device(b))
    check(got, O.where(cond, a, b), dtype, exact=True)


def test_out_of_range_index_sets_the_error_word(ops, backend):
    lib = backend._native.lib()
    dev = torch.cuda.current_device()
    lib.tp_b200_take_device_error(dev)
    x = ops.to_device(torch.arange(10.0))
    ops.index_select(x, 0, ops.to_device(torch.tensor([1, 10, 2])))
    torch.cuda.synchronize()
    assert lib.tp_b200_take_device_error(dev) != 0
    got = ops.gather(x, 0, ops.to_device(torch.tensor([-1, 3])))  # negative counts from the end
    assert_equal(ops.to_host(got), torch.tensor([9.0, 3.0]))
    assert lib.tp_b200_take_device_error(dev) == 0
