"""BASELINE config 2 -- the memory-bound op sweep -- checked in full at the
sizes the benchmark times, against the CPU oracle on the same seeded inputs.

fp32 / bf16 [8192, 8192] ~N(0, 2): broadcast add / mul / div with an [8192]
row vector (divisor |b| + 1), exp / gelu / sigmoid forward and backward (dy
~N(0, 1); exp's backward is dy * exp(x), the mul autograd records), sum /
mean / amax / amin over dim -1 and over everything; softmax / log_softmax
forward and backward on [32768, 4096]; int32 add and amax on [8192, 8192]
uniform [-1e6, 1e6], bit-exact.  The reference's own device-versus-host checks
of these operators are tests/test_mlu.py:303-350 of tensorplay-mlu.

Every element of every result is compared: elementwise results within the
north-star tolerance of the result (fp32 1e-5, bf16 1e-2 relative), sums
within the same tolerance of the summed terms (conftest.assert_close_terms),
amax / amin and integer work bit-exact.
"""

from __future__ import annotations

import pytest
import torch

import oracle as O
from conftest import assert_close, assert_close_terms, assert_equal

pytestmark = pytest.mark.gpu

M = N = 8192
SR, SC = 32768, 4096


def _randn(shape, seed, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(shape, generator=g) * scale


@pytest.fixture(scope="module")
def ops(backend):
    return backend.ops


@pytest.fixture(scope="module", params=[torch.float32, torch.bfloat16], ids=["f32", "bf16"])
def sweep(request, ops):
    """Host and device copies of config 2's [8192, 8192] inputs in one dtype."""
    dt = request.param
    a = (_randn((M, N), 0, 2.0)).to(dt)
    b = (_randn((N,), 1, 2.0)).to(dt)
    dy = _randn((M, N), 2).to(dt)
    bpos = O.binary_scalar(O.ADD, O.unary(O.ABS, b), 1)
    d = {"dt": dt, "a": a, "b": b, "dy": dy, "bpos": bpos}
    for k in ("a", "b", "dy", "bpos"):
        d["d_" + k] = ops.to_device(d[k])
    yield d
    d.clear()
    torch.cuda.empty_cache()


@pytest.mark.parametrize("name,op", [("add", O.ADD), ("mul", O.MUL), ("div", O.DIV)])
def test_row_broadcast_binary(ops, sweep, name, op):
    fn = {"add": ops.add_Tensor, "mul": ops.mul_Tensor, "div": ops.div_Tensor}[name]
    rhs = "bpos" if name == "div" else "b"
    got = fn(sweep["d_a"], sweep["d_" + rhs])
    assert_close(ops.to_host(got), O.binary(op, sweep["a"], sweep[rhs]), sweep["dt"])


@pytest.mark.parametrize("name,code", [("exp", O.EXP), ("gelu", O.GELU), ("sigmoid", O.SIGMOID)])
def test_unary_forward_and_backward(ops, sweep, name, code):
    dt = sweep["dt"]
    a, dy = sweep["a"], sweep["dy"]
    y = getattr(ops, name)(sweep["d_a"])
    want_y = O.unary(code, a)
    assert_close(ops.to_host(y), want_y, dt)
    if name == "exp":
        got = ops.mul_Tensor(sweep["d_dy"], y)
        want = O.binary(O.MUL, dy, want_y)
    elif name == "gelu":
        got = ops.gelu_backward(sweep["d_dy"], sweep["d_a"])
        want = O.unary_backward(O.GELU_BACKWARD, dy, a)
    else:
        # sigmoid_backward takes the forward output; both sides get the device's.
        yh = ops.to_host(y)
        got = ops.sigmoid_backward(sweep["d_dy"], y)
        want = O.unary_backward(O.SIGMOID_BACKWARD, dy, yh)
    assert_close(ops.to_host(got), want, dt)


@pytest.mark.parametrize("op_name", ["sum", "mean", "amax", "amin"])
@pytest.mark.parametrize("over", ["dim-1", "all"])
def test_reductions(ops, sweep, op_name, over):
    dt = sweep["dt"]
    a = sweep["a"]
    code = {"sum": O.SUM, "mean": O.MEAN, "amax": O.AMAX, "amin": O.AMIN}[op_name]
    dims = [-1] if over == "dim-1" else None
    if op_name == "sum":
        got = ops.sum_dim_IntList(sweep["d_a"], [-1]) if dims else ops.sum(sweep["d_a"])
    elif op_name == "mean":
        got = ops.mean_dim(sweep["d_a"], [-1]) if dims else ops.mean(sweep["d_a"])
    else:
        got = getattr(ops, op_name)(sweep["d_a"], [-1]) if dims else getattr(ops, op_name)(sweep["d_a"])
    want = O.reduce(code, a, dims, dt)
    got = ops.to_host(got)
    if op_name in ("amax", "amin"):
        assert_equal(got, want)
        return
    terms = O.reduce(code, O.unary(O.ABS, a.float()), dims, torch.float32)
    assert_close_terms(got, want, terms, dt)


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16], ids=["f32", "bf16"])
def test_softmax_family_32768x4096(ops, dt):
    x = _randn((SR, SC), 5, 2.0).to(dt)
    dy = _randn((SR, SC), 6).to(dt)
    dx_, ddy = ops.to_device(x), ops.to_device(dy)
    for log in (False, True):
        y = (ops.log_softmax if log else ops.softmax)(dx_, -1)
        yh = ops.to_host(y)
        assert_close(yh, O.softmax(x, -1, log=log), dt)
        back = (ops._log_softmax_backward_data if log else ops._softmax_backward_data)(ddy, y, -1, dt)
        assert_close(ops.to_host(back), O.softmax_backward(dy, yh, -1, log=log), dt)
        del y, back
    del dx_, ddy


def test_int32_add_and_amax_are_bit_exact(ops):
    g = torch.Generator().manual_seed(3)
    ia = torch.randint(-1000000, 1000000, (M, N), generator=g, dtype=torch.int32)
    g.manual_seed(4)
    ib = torch.randint(-1000000, 1000000, (M, N), generator=g, dtype=torch.int32)
    da, db = ops.to_device(ia), ops.to_device(ib)
    assert_equal(ops.to_host(ops.add_Tensor(da, db)), O.binary(O.ADD, ia, ib))
    assert_equal(ops.to_host(ops.amax(da)), O.reduce(O.AMAX, ia, None, torch.int32))
    assert_equal(ops.to_host(ops.amax(da, [-1])), O.reduce(O.AMAX, ia, [-1], torch.int32))
    # The integer sum is exact too (int64 accumulation).
    assert_equal(ops.to_host(ops.sum(da)), O.reduce(O.SUM, ia, None, torch.int64))
