"""Matrix products on a B200 against the oracle (tensorplay-mlu
tests/test_mlu.py:238-300 structure): transposes read in place, addmm / bmm /
matmul / linear, the reference's shape list, the TF32 switch, and the
BASELINE GEMM shapes checked on sampled outputs.  bf16/f16 products run on
the tcgen05 kernel, exact fp32 / f64 / integer on the CUDA-core kernel."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle as O
from conftest import TOL, assert_close_terms, assert_equal

pytestmark = pytest.mark.gpu

FLOATS = [torch.float32, torch.bfloat16, torch.float16]


def rand(*shape, dtype=torch.float32, seed=0, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).to(dtype)


@pytest.fixture(scope="module")
def ops(backend):
    return backend.ops


def dev(ops, t):
    return ops.to_device(t)


def close_product(got, a, b, dtype, c=None, alpha=1.0, beta=0.0):
    """got against alpha * a @ b + beta * c from the oracle, within the
    dtype's tolerance of the summed terms' magnitude (|alpha| |a| @ |b| +
    |beta| |c|; conftest.assert_close_terms)."""
    want = O.gemm(a, b, c, alpha, beta)
    terms = O.gemm(a.abs(), b.abs(), c.abs() if c is not None else None, abs(alpha), abs(beta))
    assert_close_terms(got, want, terms, dtype)


def check_sampled(got_dev, a, b, c=None, alpha=1.0, beta=0.0, flags=0, samples=4096, seed=0):
    """Compare `samples` random outputs of a large product with the oracle
    (float64 accumulation), relative to the largest |reference| sampled."""
    got = got_dev.cpu() if got_dev.device.type != "cpu" else got_dev
    rng = np.random.default_rng(seed)
    if got.dim() == 2:
        idx = np.stack([np.zeros(samples, np.int64), rng.integers(0, got.shape[0], samples),
                        rng.integers(0, got.shape[1], samples)], 1)
        vals = got[idx[:, 1], idx[:, 2]]
    else:
        idx = np.stack([rng.integers(0, got.shape[0], samples), rng.integers(0, got.shape[1], samples),
                        rng.integers(0, got.shape[2], samples)], 1)
        vals = got[idx[:, 0], idx[:, 1], idx[:, 2]]
    want = O.gemm_sampled(a, b, idx, c, alpha, beta, flags)
    terms = O.gemm_sampled(a.abs(), b.abs(), idx, c.abs() if c is not None else None, abs(alpha), abs(beta), flags)
    err = np.abs(vals.double().numpy() - want).max()
    ref = max(np.abs(terms).max(), np.abs(want).max(), 1.0)
    return err / ref


@pytest.mark.parametrize("dtype", FLOATS + [torch.float64])
@pytest.mark.parametrize("ta,tb", [(False, False), (True, False), (False, True), (True, True)])
def test_mm_transposes(ops, dtype, ta, tb):
    a, b = rand(37, 19, dtype=dtype), rand(19, 23, dtype=dtype, seed=3)
    da = dev(ops, a.t().contiguous()).t() if ta else dev(ops, a)
    db = dev(ops, b.t().contiguous()).t() if tb else dev(ops, b)
    close_product(ops.mm(da, db), a, b, dtype)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("ta,tb", [(False, False), (True, False), (False, True), (True, True)])
def test_tensor_core_transposes(ops, dtype, ta, tb):
    # Aligned shapes so every transpose combination takes the tcgen05 path
    # (K-major and MN-major shared-memory operands), with M, N, K tails.
    M, N, K = 200, 328, 136
    a, b = rand(M, K, dtype=dtype, seed=1), rand(K, N, dtype=dtype, seed=2)
    da = dev(ops, a.t().contiguous()).t() if ta else dev(ops, a)
    db = dev(ops, b.t().contiguous()).t() if tb else dev(ops, b)
    close_product(ops.mm(da, db), a, b, dtype)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("ta,tb", [(False, False), (True, False), (False, True), (True, True)])
def test_cta_pair_kernel_transposes_and_tails(ops, dtype, ta, tb):
    # M, N >= 256 take the 2-SM (cta_group::2) kernel: 256 x 256 tiles with
    # tails in M, N and K, every operand major, and a batched case.
    M, N, K = 520, 776, 200
    a, b = rand(M, K, dtype=dtype, seed=1), rand(K, N, dtype=dtype, seed=2)
    da = dev(ops, a.t().contiguous()).t() if ta else dev(ops, a)
    db = dev(ops, b.t().contiguous()).t() if tb else dev(ops, b)
    close_product(ops.mm(da, db), a, b, dtype)
    x, y = rand(3, 300, 136, dtype=dtype, seed=3), rand(3, 136, 264, dtype=dtype, seed=4)
    dx_ = dev(ops, x.transpose(1, 2).contiguous()).transpose(1, 2) if ta else dev(ops, x)
    dy_ = dev(ops, y.transpose(1, 2).contiguous()).transpose(1, 2) if tb else dev(ops, y)
    close_product(ops.bmm(dx_, dy_), x, y, dtype)
    bias = rand(N, dtype=dtype, seed=5)
    close_product(ops.addmm(dev(ops, bias), da, db, beta=1.0, alpha=0.5), a, b, dtype, bias, 0.5, 1.0)


@pytest.mark.parametrize("dtype", [torch.int32, torch.int64, torch.int8])
def test_integer_mm_is_exact(ops, dtype):
    g = torch.Generator().manual_seed(0)
    a = torch.randint(-9, 9, (37, 19), generator=g).to(dtype)
    b = torch.randint(-9, 9, (19, 23), generator=g).to(dtype)
    assert_equal(ops.mm(dev(ops, a), dev(ops, b)).cpu(), O.gemm(a, b))


def test_gemm_sm_limit_changes_the_grid_not_the_result(ops, backend):
    # Each output tile is computed the same way whichever CTA takes it, so a
    # lower SM budget (fewer persistent CTAs / pairs) gives identical bits,
    # for the CTA-pair kernel (1024 x 768) and the 1-SM kernel (200 x 300).
    lib = backend._native.lib()
    device = torch.cuda.current_device()
    cases = [(rand(1024, 512, dtype=torch.bfloat16, seed=1), rand(512, 768, dtype=torch.bfloat16, seed=2)),
             (rand(200, 256, dtype=torch.bfloat16, seed=3), rand(256, 300, dtype=torch.bfloat16, seed=4))]
    for a, b in cases:
        want = ops.to_host(ops.mm(dev(ops, a), dev(ops, b)))
        for sms in (2, 10, 37, 132):
            assert lib.tp_b200_set_gemm_sm_limit(device, sms) == 0
            try:
                got = ops.to_host(ops.mm(dev(ops, a), dev(ops, b)))
            finally:
                assert lib.tp_b200_set_gemm_sm_limit(device, 0) == 0
            assert_equal(got, want)
    assert lib.tp_b200_set_gemm_sm_limit(-1, 8) != 0


def test_small_products_split_k_on_cuda_cores(ops):
    # Products too small to fill the SMs are split along K on the CUDA-core
    # kernel and the splits combined in order: exact fp32 (the README chain's
    # 256^3), f64 with alpha / beta and a broadcast addend, integers exactly,
    # a batch, and transposed views.
    a, b = rand(256, 256, seed=1), rand(256, 256, seed=2)
    close_product(ops.mm(dev(ops, a), dev(ops, b)), a, b, torch.float32)
    close_product(ops.mm(dev(ops, a.t().contiguous()).t(), dev(ops, b.t().contiguous()).t()), a, b, torch.float32)
    a, b, c = (rand(40, 3000, dtype=torch.float64, seed=3), rand(3000, 50, dtype=torch.float64, seed=4),
               rand(50, dtype=torch.float64, seed=5))
    close_product(ops.addmm(dev(ops, c), dev(ops, a), dev(ops, b), beta=0.5, alpha=-2.0), a, b, torch.float64, c,
                  -2.0, 0.5)
    g = torch.Generator().manual_seed(6)
    ia = torch.randint(-50, 50, (30, 5000), generator=g, dtype=torch.int32)
    ib = torch.randint(-50, 50, (5000, 20), generator=g, dtype=torch.int32)
    assert_equal(ops.mm(dev(ops, ia), dev(ops, ib)).cpu(), O.gemm(ia, ib))
    x, y = rand(3, 64, 700, seed=7), rand(3, 700, 48, seed=8)
    close_product(ops.bmm(dev(ops, x), dev(ops, y)), x, y, torch.float32)


@pytest.mark.parametrize("dtype", FLOATS)
def test_addmm_bmm_matmul(ops, dtype):
    bias, a, b = rand(23, dtype=dtype), rand(37, 19, dtype=dtype, seed=1), rand(19, 23, dtype=dtype, seed=2)
    close_product(ops.addmm(dev(ops, bias), dev(ops, a), dev(ops, b), beta=0.5, alpha=2.0), a, b, dtype, bias,
                  2.0, 0.5)
    x, y = rand(4, 9, 6, dtype=dtype), rand(4, 6, 5, dtype=dtype, seed=4)
    close_product(ops.bmm(dev(ops, x), dev(ops, y)), x, y, dtype)
    w = rand(6, 5, dtype=dtype, seed=5)
    close_product(ops.matmul(dev(ops, x), dev(ops, w)).reshape(-1, 5), x.reshape(-1, 6), w, dtype)
    v = rand(2, 1, 6, 3, dtype=dtype, seed=6)
    xa = x.unsqueeze(0).expand(2, 4, 9, 6).reshape(8, 9, 6).contiguous()
    va = v.expand(2, 4, 6, 3).reshape(8, 6, 3).contiguous()
    close_product(ops.matmul(dev(ops, x), dev(ops, v)).reshape(8, 9, 3), xa, va, dtype)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("M,N,K", [(256, 384, 128), (600, 1000, 256), (300, 520, 64)])
def test_addmm_bias_in_epilogue_on_tensor_cores(ops, dtype, M, N, K):
    # Whole 32-column chunks read the addend as 16-byte vectors; ragged N
    # (1000, 520) and an offset (unaligned) bias exercise the element path.
    bias, a, b = rand(N, dtype=dtype), rand(M, K, dtype=dtype, seed=1), rand(K, N, dtype=dtype, seed=2)
    close_product(ops.addmm(dev(ops, bias), dev(ops, a), dev(ops, b)), a, b, dtype, bias, 1.0, 1.0)
    full = rand(M, N, dtype=dtype, seed=3)
    close_product(ops.addmm(dev(ops, full), dev(ops, a), dev(ops, b), beta=0.25, alpha=-1.0), a, b, dtype, full,
                  -1.0, 0.25)
    wide = rand(N + 1, dtype=dtype, seed=4)
    close_product(ops.addmm(dev(ops, wide)[1:], dev(ops, a), dev(ops, b)), a, b, dtype, wide[1:].contiguous(),
                  1.0, 1.0)


@pytest.mark.parametrize("dtype", FLOATS)
@pytest.mark.parametrize("m,k,n", [(2, 1024, 1024), (128, 1024, 256), (256, 4096, 1024),
                                   (1024, 4096, 128), (4096, 4096, 4096)])
def test_mm_shapes(ops, dtype, m, k, n):
    a, b = rand(m, k, dtype=dtype, seed=1), rand(k, n, dtype=dtype, seed=2)
    got = ops.mm(dev(ops, a), dev(ops, b))
    rel = check_sampled(got, a, b)
    assert rel <= TOL[dtype], rel


@pytest.mark.parametrize("dtype", FLOATS)
def test_linear(ops, dtype):
    x, w, b = rand(3, 5, 64, dtype=dtype), rand(48, 64, dtype=dtype, seed=1), rand(48, dtype=dtype, seed=2)
    xd, wd, bd = dev(ops, x), dev(ops, w), dev(ops, b)
    x2, wt = x.reshape(15, 64), w.t().contiguous()
    close_product(ops.linear(xd, wd, bd).reshape(15, 48), x2, wt, dtype, b, 1.0, 1.0)
    close_product(ops.linear(xd, wd).reshape(15, 48), x2, wt, dtype)
    close_product(ops.linear(xd[0, 0], wd, bd).reshape(1, 48), x2[:1], wt, dtype, b, 1.0, 1.0)


@pytest.mark.parametrize("dtype", FLOATS)
def test_bmm_shapes(ops, dtype):
    for (bt, m, k, n) in ((32, 512, 64, 512), (1, 256, 4096, 1024), (3, 1, 7, 5)):
        a, b = rand(bt, m, k, dtype=dtype, seed=1), rand(bt, k, n, dtype=dtype, seed=2)
        got = ops.bmm(dev(ops, a), dev(ops, b))
        assert check_sampled(got, a, b) <= TOL[dtype]
    a, b = rand(4, 9, 6, dtype=dtype), rand(4, 5, 6, dtype=dtype, seed=3)
    close_product(ops.bmm(dev(ops, a), dev(ops, b).transpose(1, 2)), a, b.transpose(1, 2).contiguous(), dtype)


def test_float32_matmul_precision_selects_tf32(ops):
    a, b = rand(512, 512, seed=1), rand(512, 512, seed=2)
    want = O.gemm(a.double(), b.double())
    da, db = dev(ops, a), dev(ops, b)
    previous = torch.get_float32_matmul_precision()
    torch.set_float32_matmul_precision("highest")
    try:
        exact = (ops.mm(da, db).cpu().double() - want).abs().max().item()
        torch.set_float32_matmul_precision("high")
        fast = (ops.mm(da, db).cpu().double() - want).abs().max().item()
    finally:
        torch.set_float32_matmul_precision(previous)
    assert exact < 1e-3, exact
    assert fast < 0.5, fast  # TF32 keeps 10 mantissa bits
    assert fast > exact  # the switch really selected another path


class _Highest:
    """fp32 products at full precision (no TF32) inside the block."""

    def __enter__(self):
        self.previous = torch.get_float32_matmul_precision()
        torch.set_float32_matmul_precision("highest")

    def __exit__(self, *exc):
        torch.set_float32_matmul_precision(self.previous)


def test_fp32_split_tf32_batches_and_batch_broadcast(ops):
    # Full-precision batched products: two real batch members on the split-TF32
    # tensor-core path (bit-identical to the single product), and operands
    # broadcast over the batch (stride 0), which take the CUDA-core kernel.
    with _Highest():
        a, b = rand(384, 3072, seed=21), rand(3072, 320, seed=22)
        da, db = dev(ops, a), dev(ops, b)
        one = ops.to_host(ops.mm(da, db))
        two = ops.to_host(ops.bmm(dev(ops, a.unsqueeze(0).repeat(2, 1, 1)), dev(ops, b.unsqueeze(0).repeat(2, 1, 1))))
        assert_equal(one, two[0])
        assert_equal(one, two[1])
        assert check_sampled(ops.mm(da, db), a, b) <= 1e-5
        bc = ops.bmm(da.unsqueeze(0).expand(2, -1, -1), db.unsqueeze(0).expand(2, -1, -1))
        assert check_sampled(bc, a.expand(2, -1, -1), b.expand(2, -1, -1)) <= 1e-5


def test_fp32_split_tf32_layouts_and_epilogue(ops):
    # Large enough for the split-TF32 tensor-core path: transposed operands
    # (copied K-major first), an operand broadcast over the batch, and the
    # addmm epilogue (alpha, beta, bias).
    with _Highest():
        a, b = rand(640, 384, seed=1), rand(384, 520, seed=2)
        got = ops.mm(dev(ops, a.t().contiguous()).t(), dev(ops, b.t().contiguous()).t())
        assert check_sampled(got, a, b) <= 1e-5
        a2, b2 = rand(512, 256, seed=3), rand(4, 256, 512, seed=4)
        got = ops.matmul(dev(ops, a2), dev(ops, b2))
        assert check_sampled(got, a2.expand(4, 512, 256), b2) <= 1e-5
        bias = rand(520, seed=5)
        got = ops.addmm(dev(ops, bias), dev(ops, a), dev(ops, b), beta=0.5, alpha=2.0)
        assert check_sampled(got, a, b, bias, 2.0, 0.5) <= 1e-5


def test_fp32_split_tf32_non_finite_inputs(ops):
    # inf and NaN keep fp32 semantics (inf * finite = inf, not the NaN a
    # zero low part would give); every other output stays exact.
    a, b = rand(512, 512, seed=1), rand(512, 512, seed=2)
    a[3, 7] = float("inf")
    a[100, 5] = float("nan")
    b[9, 200] = -float("inf")
    b[:, 300] = 1.0  # exactly representable: zero low parts in that column
    a[50, 11] = float("inf")
    with _Highest():
        got = ops.mm(dev(ops, a), dev(ops, b)).cpu()
    want = O.gemm(a.double(), b.double()).float()
    assert torch.equal(torch.isnan(got), torch.isnan(want))
    assert torch.equal(torch.isinf(got), torch.isinf(want))
    inf = torch.isinf(want)
    assert torch.equal(got[inf], want[inf])
    fin = torch.isfinite(want)
    assert (got[fin] - want[fin]).abs().max().item() <= 1e-5 * max(want[fin].abs().max().item(), 1.0)


# ------------------------------------------------- BASELINE GEMM shapes --

def test_baseline_mm_8192_bf16(ops):
    n = 8192
    a, b = rand(n, n, dtype=torch.bfloat16, seed=1, scale=n ** -0.5), rand(n, n, dtype=torch.bfloat16, seed=2)
    got = ops.mm(dev(ops, a), dev(ops, b))
    assert check_sampled(got, a, b) <= 1e-2


def test_baseline_addmm_and_linear_bf16(ops):
    M, K, N = 16384, 4096, 11008
    a = rand(M, K, dtype=torch.bfloat16, seed=1)
    w = rand(N, K, dtype=torch.bfloat16, seed=2, scale=K ** -0.5)
    bias = rand(N, dtype=torch.bfloat16, seed=3)
    da, dw, db = dev(ops, a), dev(ops, w), dev(ops, bias)
    lin = ops.linear(da, dw, db)          # weight [N, K] read transposed in place
    assert check_sampled(lin, a, w.t(), bias, 1.0, 1.0) <= 1e-2
    b = w.t().contiguous()
    add = ops.addmm(db, da, dev(ops, b))  # [K, N] row-major
    assert check_sampled(add, a, b, bias, 1.0, 1.0) <= 1e-2


def test_baseline_bmm_bf16(ops):
    a = rand(64, 2048, 128, dtype=torch.bfloat16, seed=1, scale=128 ** -0.5)
    b = rand(64, 128, 2048, dtype=torch.bfloat16, seed=2)
    got = ops.bmm(dev(ops, a), dev(ops, b))
    assert check_sampled(got, a, b) <= 1e-2


def test_baseline_mm_4096_fp32_highest(ops):
    n = 4096
    a, b = rand(n, n, seed=1, scale=n ** -0.5), rand(n, n, seed=2)
    previous = torch.get_float32_matmul_precision()
    torch.set_float32_matmul_precision("highest")
    try:
        got = ops.mm(dev(ops, a), dev(ops, b))
    finally:
        torch.set_float32_matmul_precision(previous)
    assert check_sampled(got, a, b) <= 1e-5
