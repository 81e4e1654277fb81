"""Kernel-versus-oracle parity on a B200, operator family by operator family.

The structure follows tensorplay-mlu's tests/test_mlu.py (round trips,
strided and broadcasting copies, casts, fills, binary/scalar/in-place forms,
unary and activation kernels, products, reductions, softmax): every device
result is compared with the CPU oracle on the same seeded host inputs --
bit-exact for integer, copy, cast, fill and amax/amin work; within the
relative tolerances of conftest.TOL (fp32 1e-5, bf16 1e-2) for float math.
All device work goes through tensorplay_mlu_b200.ops and the C ABI.
"""

from __future__ import annotations

import pytest
import torch

import oracle as O
from conftest import assert_close, assert_close_terms, assert_equal

pytestmark = pytest.mark.gpu

FLOATS = [torch.float32, torch.bfloat16, torch.float16]
ALL = FLOATS + [torch.float64, torch.int64, torch.int32, torch.int16, torch.int8, torch.uint8,
                torch.bool]


def rand(*shape, dtype=torch.float32, seed=0, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).to(dtype)


def randint(*shape, low=-1000, high=1000, dtype=torch.int32, seed=0):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(low, high, shape, generator=g).to(dtype)


def close_sum(got, a, dims, dtype, keepdim=False):
    """A device sum against the oracle's, within the dtype's tolerance of the
    magnitude of the summed terms (the same sum of |a|)."""
    want = O.reduce(O.SUM, a, dims, dtype, keepdim)
    wide = torch.float64 if dtype == torch.float64 else torch.float32
    terms = O.reduce(O.SUM, a.to(wide).abs(), dims, wide, keepdim)
    assert_close_terms(got, want, terms, dtype)


@pytest.fixture(scope="module")
def ops(backend):
    return backend.ops


def dev(ops, t):
    return ops.to_device(t)


def host(ops, t):
    return ops.to_host(t)


# ---------------------------------------------------------------- copies --

@pytest.mark.parametrize("dtype", ALL)
def test_round_trip(ops, dtype):
    x = (rand(5, 7) * 10).to(dtype)
    y = dev(ops, x)
    assert y.is_cuda and y.dtype == dtype
    assert_equal(host(ops, y), x)


def test_strided_copies_both_ways(ops):
    x = rand(6, 8)
    assert_equal(host(ops, dev(ops, x.t())), x.t().contiguous())
    d = dev(ops, x)
    assert_equal(host(ops, d.t()), x.t().contiguous())
    assert_equal(host(ops, d[:, 1::3]), x[:, 1::3].contiguous())
    out = ops.zero_(torch.empty(8, 6, device="cuda"))
    ops.copy_(out, d.t())
    assert_equal(host(ops, out), x.t().contiguous())


def test_large_transpose_copy(ops):
    x = rand(257, 1031)
    d = dev(ops, x)
    assert_equal(host(ops, ops.contiguous(d.t())), x.t().contiguous())


def test_broadcasting_copy_on_device(ops):
    row = dev(ops, rand(1, 5))
    out = torch.empty(4, 5, device="cuda")
    ops.copy_(out, row)
    assert_equal(host(ops, out), host(ops, row).expand(4, 5).contiguous())


CAST_PAIRS = [(torch.float32, torch.float16), (torch.float16, torch.float32),
              (torch.float32, torch.bfloat16), (torch.float16, torch.bfloat16),
              (torch.float32, torch.int32), (torch.int64, torch.float32),
              (torch.float64, torch.float32), (torch.float32, torch.float64),
              (torch.float64, torch.bfloat16), (torch.int32, torch.bool), (torch.bool, torch.float32),
              (torch.bfloat16, torch.int64), (torch.uint8, torch.float16), (torch.int64, torch.int8)]


@pytest.mark.parametrize("src,dst", CAST_PAIRS)
def test_casts_on_device(ops, src, dst):
    x = (rand(3, 9) * 4).to(src) if src != torch.uint8 else (rand(3, 9) * 4).abs().to(src)
    y = ops._to_dtype(dev(ops, x), dst)
    assert y.dtype == dst
    assert_equal(host(ops, y), O.cast(x, dst))


def test_host_to_device_with_cast_and_broadcast(ops):
    src = rand(1, 6, dtype=torch.float64)
    out = torch.empty(3, 6, dtype=torch.bfloat16, device="cuda")
    ops.copy_(out, src)
    assert_equal(host(ops, out), O.cast(src.expand(3, 6).contiguous(), torch.bfloat16))


@pytest.mark.parametrize("dtype", FLOATS + [torch.int32, torch.int64, torch.float64, torch.bool])
def test_fill_and_factories(ops, dtype):
    value = 2.5 if dtype.is_floating_point else (True if dtype == torch.bool else 3)
    t = ops.fill_(torch.empty(3, 4, dtype=dtype, device="cuda"), value)
    assert_equal(host(ops, t), torch.full((3, 4), value, dtype=dtype))
    d = ops.zero_(torch.empty(2, 3, dtype=dtype, device="cuda"))
    assert_equal(host(ops, d), torch.zeros(2, 3, dtype=dtype))
    for like, v in ((ops.ones_like(d), 1), (ops.zeros_like(d), 0), (ops.full_like(d, 7), 7)):
        assert like.is_cuda and like.dtype == dtype
        assert_equal(host(ops, like), torch.full((2, 3), v, dtype=dtype))
    assert ops.ones_like(d, dtype=torch.float32).dtype == torch.float32
    assert not ops.ones_like(d, device="cpu").is_cuda


def test_strided_fill(ops):
    d = dev(ops, rand(6, 8))
    ops.fill_(d[:, ::2], 1.5)
    want = rand(6, 8)
    want[:, ::2] = 1.5
    assert_equal(host(ops, d), want)


def test_item(ops):
    for dtype, v in ((torch.float32, 3.25), (torch.int64, -7), (torch.bfloat16, 1.5), (torch.float64, 0.1)):
        t = ops.fill_(torch.empty((), dtype=dtype, device="cuda"), v)
        assert ops.item(t) == torch.tensor(v, dtype=dtype).item()


# ------------------------------------------------------------ arithmetic --

BIN_OPS = {"add": O.ADD, "sub": O.SUB, "mul": O.MUL, "div": O.DIV}


@pytest.mark.parametrize("dtype", FLOATS + [torch.float64])
def test_binary_with_broadcasting(ops, dtype):
    a, b = rand(4, 1, 5, dtype=dtype), rand(3, 1, dtype=dtype, seed=1)
    da, db = dev(ops, a), dev(ops, b)
    assert_close(ops.add_Tensor(da, db), O.binary(O.ADD, a, b), dtype)
    assert_close(ops.sub_Tensor(da, ops.mul_Scalar(db, 0.5)), O.binary(O.SUB, a, b, 0.5), dtype)
    assert_close(ops.sub_Tensor(da, db, alpha=2), O.binary(O.SUB, a, b, 2), dtype)
    assert_close(ops.mul_Tensor(da, db), O.binary(O.MUL, a, b), dtype)
    denom = O.binary_scalar(O.ADD, O.unary(O.ABS, b), 1.0)
    assert_close(ops.div_Tensor(da, ops.add_Scalar(ops.abs(db), 1)), O.binary(O.DIV, a, denom), dtype)


@pytest.mark.parametrize("dtype", [torch.int32, torch.int64, torch.int16, torch.int8, torch.uint8])
def test_integer_binary_is_exact(ops, dtype):
    lo, hi = (0, 100) if dtype == torch.uint8 else (-100, 100)
    a, b = randint(37, 19, low=lo, high=hi, dtype=dtype), randint(19, low=lo, high=hi, dtype=dtype, seed=1)
    da, db = dev(ops, a), dev(ops, b)
    assert_equal(host(ops, ops.add_Tensor(da, db, alpha=3)), O.binary(O.ADD, a, b, 3))
    assert_equal(host(ops, ops.sub_Tensor(da, db)), O.binary(O.SUB, a, b))
    assert_equal(host(ops, ops.mul_Tensor(da, db)), O.binary(O.MUL, a, b))


def test_int32_wraps_like_the_host(ops):
    a = torch.tensor([2**31 - 1, -2**31, 123456789], dtype=torch.int32)
    b = torch.tensor([1, -1, 987654321], dtype=torch.int32)
    assert_equal(host(ops, ops.add_Tensor(dev(ops, a), dev(ops, b))), a + b)
    assert_equal(host(ops, ops.mul_Tensor(dev(ops, a), dev(ops, b))), a * b)


def test_integer_division_promotes(ops):
    a, b = randint(5, 6, low=1, high=50), randint(5, 6, low=1, high=50, seed=1)
    got = ops.div_Tensor(dev(ops, a), dev(ops, b))
    assert got.dtype == torch.float32
    assert_close(got, O.binary(O.DIV, a.float(), b.float()))


@pytest.mark.parametrize("dtype", FLOATS)
def test_scalar_forms_and_host_scalars(ops, dtype):
    a = rand(8, 3, dtype=dtype)
    d = dev(ops, a)
    assert_close(ops.add_Scalar(d, 2), O.binary_scalar(O.ADD, a, 2.0), dtype)
    assert_close(ops.mul_Scalar(d, 3), O.binary_scalar(O.MUL, a, 3.0), dtype)
    assert_close(ops.div_Scalar(d, 4), O.binary_scalar(O.DIV, a, 4.0), dtype)
    assert_close(ops.rsub_Scalar(d, 1), O.binary_scalar(O.RSUB, a, 1.0), dtype)
    assert_close(ops.mul_Tensor(d, torch.tensor(2.0)), O.binary_scalar(O.MUL, a, 2.0), dtype)
    assert_close(ops.add_Tensor(torch.tensor(2.0), d), O.binary_scalar(O.ADD, a, 2.0), dtype)
    assert_close(ops.sub_Tensor(torch.tensor(2.0), d), O.binary_scalar(O.RSUB, a, 2.0), dtype)


@pytest.mark.parametrize("dtype", FLOATS)
def test_in_place(ops, dtype):
    a, b = rand(6, 4, dtype=dtype), rand(4, dtype=dtype, seed=2)
    d, db = dev(ops, a), dev(ops, b)
    ops.add__Tensor(d, db, alpha=0.5)
    ops.mul__Scalar(d, 2)
    ops.sub__Tensor(d, db)
    ops.div__Scalar(d, 3)
    want = O.binary_scalar(O.DIV, O.binary(O.SUB, O.binary_scalar(O.MUL, O.binary(O.ADD, a, b, 0.5), 2.0), b), 3.0)
    assert_close(d, want, dtype, scale=2)


@pytest.mark.parametrize("dtype", FLOATS)
def test_scalar_forms_of_strided_operands(ops, dtype):
    base = rand(1, 5, dtype=dtype)
    expanded = dev(ops, base).expand(4, 5)
    assert_close(ops.mul_Scalar(expanded, 3), O.binary_scalar(O.MUL, base.expand(4, 5), 3.0), dtype)
    assert_close(ops.add_Scalar(expanded, 2), O.binary_scalar(O.ADD, base.expand(4, 5), 2.0), dtype)
    a = rand(6, 8, dtype=dtype)
    d = dev(ops, a)
    ops.mul__Scalar(d.t(), 0.5)
    ops.add__Scalar(d[:, ::2], 1.0)
    want = O.binary_scalar(O.MUL, a, 0.5)
    want[:, ::2] = O.binary_scalar(O.ADD, want[:, ::2].contiguous(), 1.0)
    assert_close(d, want, dtype)


def test_strided_operands(ops):
    a = rand(5, 7)
    d = dev(ops, a)
    assert_close(ops.add_Tensor(d.t(), d.t()), O.binary(O.ADD, a.t(), a.t()))
    assert_close(ops.mul_Tensor(d[:, ::2][:, :3], d[:, 1::2]), O.binary(O.MUL, a[:, ::2][:, :3], a[:, 1::2]))


def test_integer_math_on_device(ops):
    # tensorplay-mlu runs this on the host fallback (test_mlu.py:196-198).
    x = dev(ops, torch.arange(10))
    assert_equal(host(ops, ops.add_Scalar(ops.mul_Scalar(x, 3), 1)), torch.arange(10) * 3 + 1)


def test_row_broadcast_fast_path_shapes(ops):
    # [M, N] (+) [N] -- the bias pattern the vectorised kernel takes -- and odd N.
    for n in (8192, 1000, 7):
        a, b = rand(33, n, seed=4), rand(n, seed=5)
        assert_close(ops.add_Tensor(dev(ops, a), dev(ops, b)), O.binary(O.ADD, a, b))
        assert_close(ops.mul_Tensor(dev(ops, b), dev(ops, a)), O.binary(O.MUL, b.expand(33, n), a))


@pytest.mark.parametrize("dtype", FLOATS + [torch.float64, torch.int32])
def test_row_broadcast_long_rows_both_orders(ops, dtype):
    # Rows of at least half a block of vectors take the 2-d kernel (one row
    # read per several outputs); outer counts not a multiple of its row group,
    # and the row as first and as second operand of non-commuting ops.
    for outer, n in ((37, 1024), (5, 4096), (2, 8192), (9, 2048)):
        if dtype.is_floating_point:
            a, b = rand(outer, n, dtype=dtype, seed=6), (rand(n, dtype=dtype, seed=7).abs() + 0.5).to(dtype)
        else:
            a, b = randint(outer, n, dtype=dtype, seed=6), randint(n, low=1, high=50, dtype=dtype, seed=7)
        da, db = dev(ops, a), dev(ops, b)
        assert_close(ops.sub_Tensor(da, db), O.binary(O.SUB, a, b.expand(outer, n)), dtype)
        assert_close(ops.sub_Tensor(db, da), O.binary(O.SUB, b.expand(outer, n), a), dtype)
        if dtype.is_floating_point:
            apos = (a.abs() + 0.5).to(dtype)  # divisor away from zero
            assert_close(ops.div_Tensor(da, db), O.binary(O.DIV, a, b.expand(outer, n)), dtype)
            assert_close(ops.div_Tensor(db, dev(ops, apos)), O.binary(O.DIV, b.expand(outer, n), apos), dtype)


# ----------------------------------------------------------------- unary --

UN = {"exp": O.EXP, "log": O.LOG, "sqrt": O.SQRT, "rsqrt": O.RSQRT, "neg": O.NEG, "abs": O.ABS,
      "relu": O.RELU, "sigmoid": O.SIGMOID, "tanh": O.TANH, "silu": O.SILU}


@pytest.mark.parametrize("dtype", FLOATS + [torch.float64])
@pytest.mark.parametrize("name", list(UN))
def test_unary(ops, dtype, name):
    a = rand(33, 17, dtype=dtype)
    if name in ("log", "sqrt", "rsqrt"):
        a = (a.abs() + 0.1).to(dtype)
    got = getattr(ops, name)(dev(ops, a))
    assert_close(got, O.unary(UN[name], a), dtype)


@pytest.mark.parametrize("dtype", [torch.int32, torch.int64])
def test_integer_unary(ops, dtype):
    a = randint(7, 5, low=-9, high=9, dtype=dtype)
    d = dev(ops, a)
    assert_equal(host(ops, ops.neg(d)), O.unary(O.NEG, a))
    assert_equal(host(ops, ops.abs(d)), O.unary(O.ABS, a))
    assert_equal(host(ops, ops.relu(d)), O.unary(O.RELU, a))
    assert_equal(host(ops, ops.pow_Tensor_Scalar(d, 3)), O.unary(O.POW, a, 3))
    got = ops.exp(d)
    assert got.dtype == torch.float32
    assert_close(got, O.unary(O.EXP, a.float()))


@pytest.mark.parametrize("dtype", FLOATS)
@pytest.mark.parametrize("exponent", [2, 1, 0, 0.5, -0.5, 3, 1.7])
def test_pow_scalar(ops, dtype, exponent):
    a = (rand(6, 9).abs() + 0.5).to(dtype)
    assert_close(ops.pow_Tensor_Scalar(dev(ops, a), exponent), O.unary(O.POW, a, exponent), dtype)


@pytest.mark.parametrize("dtype", FLOATS + [torch.float64])
def test_activations(ops, dtype):
    a = rand(16, 32, dtype=dtype)
    d = dev(ops, a)
    assert_close(ops.gelu(d), O.unary(O.GELU, a), dtype)
    assert_close(ops.gelu(d, approximate="tanh"), O.unary(O.GELU_TANH, a), dtype)
    assert_close(ops.silu(d), O.unary(O.SILU, a), dtype)
    r = dev(ops, a)
    ops.relu_(r)
    assert_close(r, O.unary(O.RELU, a), dtype)


@pytest.mark.parametrize("dtype", FLOATS + [torch.float64])
def test_activation_backward(ops, dtype):
    x, dy = rand(16, 32, dtype=dtype, seed=2), rand(16, 32, dtype=dtype, seed=3)
    dx_, ddy = dev(ops, x), dev(ops, dy)
    y = O.unary(O.SIGMOID, x)
    assert_close(ops.sigmoid_backward(ddy, dev(ops, y)), O.unary_backward(O.SIGMOID_BACKWARD, dy, y), dtype)
    y = O.unary(O.TANH, x)
    assert_close(ops.tanh_backward(ddy, dev(ops, y)), O.unary_backward(O.TANH_BACKWARD, dy, y), dtype)
    assert_close(ops.gelu_backward(ddy, dx_), O.unary_backward(O.GELU_BACKWARD, dy, x), dtype)
    assert_close(ops.gelu_backward(ddy, dx_, "tanh"), O.unary_backward(O.GELU_TANH_BACKWARD, dy, x), dtype)
    assert_close(ops.silu_backward(ddy, dx_), O.unary_backward(O.SILU_BACKWARD, dy, x), dtype)
    assert_equal(host(ops, ops.threshold_backward(ddy, dx_, 0.0)),
                 O.unary_backward(O.THRESHOLD_BACKWARD, dy, x, 0.0))


def test_squared_error_backward(ops):
    x, t = rand(8, 5), rand(8, 5, seed=1)
    diff = ops.sub_Tensor(dev(ops, x), dev(ops, t))
    grad = ops.mul_Scalar(diff, 2.0 / diff.numel())
    assert_close(grad, O.binary_scalar(O.MUL, O.binary(O.SUB, x, t), 2.0 / 40))


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_large_narrow_float_elementwise(ops, dtype):
    a = rand(4096, 8192, dtype=dtype)  # 64 MiB
    d = dev(ops, a)
    assert_close(ops.add_Tensor(d, d), O.binary(O.ADD, a, a), dtype)
    assert_close(ops.sigmoid(d), O.unary(O.SIGMOID, a), dtype)
    assert_close(ops.gelu(d), O.unary(O.GELU, a), dtype)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_narrow_gelu_over_its_range(ops, dtype):
    # Both lanes of the packed (two-at-a-time) form and the tail, over the
    # negative tail where Phi is tiny, zero, the saturated side, inf and NaN.
    a = torch.linspace(-12, 12, 4001).to(dtype)
    a = torch.cat([a, torch.tensor([0.0, -0.0, float("inf"), float("-inf"), float("nan"), 1e-6, -1e-6]).to(dtype)])
    dy = torch.ones_like(a)
    for got, want in ((host(ops, ops.gelu(dev(ops, a))), O.unary(O.GELU, a)),
                      (host(ops, ops.gelu_backward(dev(ops, dy), dev(ops, a))),
                       O.unary_backward(O.GELU_BACKWARD, dy, a))):
        finite = torch.isfinite(want)
        assert_close(got[finite], want[finite], dtype)
        g, w = got[~finite], want[~finite]
        assert bool(((g == w) | (torch.isnan(g) & torch.isnan(w))).all()), (g, w)


# --------------------------------------------------- reductions, softmax --

@pytest.mark.parametrize("dtype", FLOATS + [torch.float64])
def test_reductions(ops, dtype):
    a = rand(6, 7, 8, dtype=dtype)
    d = dev(ops, a)
    close_sum(ops.sum(d), a, None, dtype)
    close_sum(ops.sum_dim_IntList(d, [1]), a, [1], dtype)
    close_sum(ops.sum_dim_IntList(d, [0, 2], keepdim=True), a, [0, 2], dtype, keepdim=True)
    assert_close(ops.mean(d), O.reduce(O.MEAN, a, None, dtype), dtype)
    assert_close(ops.mean_dim(d, [-1]), O.reduce(O.MEAN, a, [2], dtype), dtype)
    assert_equal(host(ops, ops.amax(d, [-1])), O.reduce(O.AMAX, a, [2], dtype))
    assert_equal(host(ops, ops.amin(d, [0, 1])), O.reduce(O.AMIN, a, [0, 1], dtype))


@pytest.mark.parametrize("dtype", FLOATS)
def test_long_reductions(ops, dtype):
    for shape in ((2, 4096), (2, 65536), (16, 8192), (3, 32768), (4096, 2)):
        a = rand(*shape, dtype=dtype)
        d = dev(ops, a)
        close_sum(ops.sum(d), a, None, dtype)
        assert_close(ops.mean(d), O.reduce(O.MEAN, a, None, dtype), dtype)
        close_sum(ops.sum_dim_IntList(d, [1]), a, [1], dtype)
        assert_close(ops.mean_dim(d, [0]), O.reduce(O.MEAN, a, [0], dtype), dtype)
    a = rand(65537, dtype=dtype)
    close_sum(ops.sum(dev(ops, a)), a, None, dtype)
    a = rand(2, 4096, 2, dtype=dtype)
    close_sum(ops.sum_dim_IntList(dev(ops, a), [1]), a, [1], dtype)
    a = rand(16, 8192, dtype=dtype)
    assert_equal(host(ops, ops.amax(dev(ops, a), [-1])), O.reduce(O.AMAX, a, [1], dtype))
    assert_equal(host(ops, ops.amin(dev(ops, a), [-1])), O.reduce(O.AMIN, a, [1], dtype))


@pytest.mark.parametrize("dtype", [torch.int32, torch.int64, torch.int8, torch.bool])
def test_integer_reductions_are_exact(ops, dtype):
    a = randint(16, 3000, low=-100, high=100, dtype=dtype) if dtype != torch.bool else \
        randint(16, 3000, low=0, high=2).bool()
    d = dev(ops, a)
    s = ops.sum(d)
    assert s.dtype == torch.int64
    assert_equal(host(ops, s), O.reduce(O.SUM, a, None, torch.int64))
    assert_equal(host(ops, ops.sum_dim_IntList(d, [0])), O.reduce(O.SUM, a, [0], torch.int64))
    if dtype != torch.bool:
        assert_equal(host(ops, ops.amax(d, [-1])), O.reduce(O.AMAX, a, [1], dtype))
        assert_equal(host(ops, ops.amin(d)), O.reduce(O.AMIN, a, None, dtype))


def test_reduction_nan_and_empty(ops):
    a = rand(4, 9)
    a[2, 3] = float("nan")
    d = dev(ops, a)
    assert_equal(host(ops, ops.amax(d, [1])), O.reduce(O.AMAX, a, [1], torch.float32))
    empty = torch.empty(0, 5, device="cuda")
    assert_equal(host(ops, ops.sum_dim_IntList(empty, [0])), torch.zeros(5))
    with pytest.raises(RuntimeError):
        ops.amax(torch.empty(0, device="cuda"))


@pytest.mark.parametrize("dtype", FLOATS + [torch.float64])
@pytest.mark.parametrize("dim", [0, 1, -1])
def test_softmax_and_log_softmax(ops, dtype, dim):
    a = rand(5, 6, 7, dtype=dtype)
    d = dev(ops, a)
    y = ops.softmax(d, dim)
    ly = ops.log_softmax(d, dim)
    assert_close(y, O.softmax(a, dim, False), dtype)
    assert_close(ly, O.softmax(a, dim, True), dtype)
    dy = rand(5, 6, 7, dtype=dtype, seed=7)
    yh, lyh = host(ops, y), host(ops, ly)
    assert_close(ops._softmax_backward_data(dev(ops, dy), y, dim, dtype),
                 O.softmax_backward(dy, yh, dim, False), dtype)
    assert_close(ops._log_softmax_backward_data(dev(ops, dy), ly, dim, dtype),
                 O.softmax_backward(dy, lyh, dim, True), dtype)


@pytest.mark.parametrize("D", [1, 37, 1000, 4096, 8192, 20000])
def test_softmax_row_lengths(ops, D):
    a = rand(9, D, scale=3.0)
    for dtype in (torch.float32, torch.bfloat16):
        x = a.to(dtype)
        assert_close(ops.softmax(dev(ops, x), -1), O.softmax(x, -1), dtype)
        assert_close(ops._log_softmax(dev(ops, x), -1), O.softmax(x, -1, True), dtype)


@pytest.mark.parametrize("dtype", FLOATS + [torch.float64])
@pytest.mark.parametrize("rows,D", [(297, 8), (640, 1000), (333, 2048), (400, 3000), (1200, 4096), (301, 8192)])
def test_softmax_many_rows(ops, dtype, rows, D):
    # Enough rows for the persistent kernel that stages rows in shared memory.
    a = rand(rows, D, dtype=dtype, scale=3.0)
    d = dev(ops, a)
    assert_close(ops.softmax(d, -1), O.softmax(a, -1), dtype)
    assert_close(ops._log_softmax(d, -1), O.softmax(a, -1, True), dtype)


def test_full_reductions_on_concurrent_streams(ops):
    # Full reductions split over the grid finish in their last block, which
    # counts the blocks in on a per-stream ticket: launches queued on two
    # streams at once, several times in a row, each keep their own count.
    a = rand(4096, 4096, seed=11)
    b = rand(4096, 4096, seed=12, scale=3.0)
    da, db = dev(ops, a), dev(ops, b)
    want_a, want_b = O.reduce(O.SUM, a, None, torch.float32), O.reduce(O.AMAX, b, None, torch.float32)
    s1, s2 = torch.cuda.Stream(), torch.cuda.Stream()
    torch.cuda.synchronize()
    outs = []
    for _ in range(4):
        with torch.cuda.stream(s1):
            ra = ops.sum(da)
        with torch.cuda.stream(s2):
            rb = ops.amax(db)
        outs.append((ra, rb))
    torch.cuda.synchronize()
    for ra, rb in outs:
        assert_close_terms(ra, want_a, O.reduce(O.SUM, a.abs(), None, torch.float32), torch.float32)
        assert_equal(host(ops, rb), want_b)


@pytest.mark.parametrize("dtype", FLOATS + [torch.float64, torch.int32])
def test_many_row_reductions(ops, dtype):
    # Enough rows for one warp per row, including rows that start off a
    # 16-byte boundary (a column slice) and rows shorter than a warp.
    for shape, sl in (((5000, 37), None), ((6000, 1000), None), ((4800, 131), 1), ((8192, 4096), None)):
        if dtype.is_floating_point:
            full = rand(*shape, dtype=dtype)
        else:
            full = randint(*shape, low=-1000, high=1000, dtype=dtype)
        a = full[:, sl:] if sl else full
        d = dev(ops, full)
        d = d[:, sl:] if sl else d
        if dtype.is_floating_point:
            close_sum(ops.sum_dim_IntList(d, [1]), a, [1], dtype)
            assert_close(ops.mean_dim(d, [-1]), O.reduce(O.MEAN, a, [1], dtype), dtype)
        else:
            assert_equal(host(ops, ops.sum_dim_IntList(d, [1])), O.reduce(O.SUM, a, [1], torch.int64))
        assert_equal(host(ops, ops.amax(d, [-1])), O.reduce(O.AMAX, a, [1], dtype))
        assert_equal(host(ops, ops.amin(d, [1])), O.reduce(O.AMIN, a, [1], dtype))


def test_memory_statistics(backend, ops):
    if not backend.allocator_installed():
        pytest.skip("caching allocator not installed as the tensor allocator in this process")
    rt = backend.runtime
    rt.empty_cache()
    before = rt.memory_allocated()
    x = torch.empty(1 << 20, device="cuda")
    assert rt.memory_allocated() >= before + (4 << 20)
    assert rt.max_memory_allocated() >= rt.memory_allocated()
    del x
    assert rt.memory_allocated() == before
    assert rt.memory_reserved() >= before
    free, total = rt.mem_get_info()
    assert 0 < free <= total
