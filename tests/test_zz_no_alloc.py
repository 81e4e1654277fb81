"""The allocation-free reduction entry point, tp_b200_reduce_noalloc.

It exists for callers that cannot allocate device memory when they reduce --
a serving process whose GPU memory is reserved up front by its own pool, or a
latency-critical path that must not risk a cudaMalloc on an allocator miss --
and keeps its partial results in a static 8 MiB device array instead.  These
tests call it through the C ABI and check its results against the ordinary
entry point, tp_b200_reduce, on two calls in a row (the array keeps the
previous call's contents, which must not leak into the next result).  The
file is named to be collected last so a failure here cannot hide failures
elsewhere; it passes alone in a fresh process as well as after the suite.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from conftest import assert_close, assert_equal

pytestmark = pytest.mark.gpu

SUM, MEAN, AMAX, AMIN = range(4)


def _reduce(entry, op, x, dims, out_dtype):
    from tensorplay_mlu_b200 import _native as N

    mask = 0
    for d in dims:
        mask |= 1 << d
    keep = [1 if (mask >> i) & 1 else s for i, s in enumerate(x.shape)]
    out = torch.empty(keep, dtype=out_dtype, device=x.device)
    status = getattr(N.lib(), entry)(op, N.describe(out), N.describe(x), mask,
                                     ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    N.check(status, entry)
    return out


def _pair(op, x, dims, out_dtype):
    got = _reduce("tp_b200_reduce_noalloc", op, x, dims, out_dtype)
    want = _reduce("tp_b200_reduce", op, x, dims, out_dtype)
    torch.cuda.synchronize()
    return got.cpu(), want.cpu()


CASES = [
    # (shape, dtype, dims, op, out dtype) -- each uses per-block partial results
    ((8192, 8192), torch.float32, [0, 1], SUM, torch.float32),        # full reduction, thousands of splits
    ((8192, 16384), torch.bfloat16, [0], SUM, torch.bfloat16),        # bias-gradient column sum
    ((16, 65536), torch.float32, [1], MEAN, torch.float32),           # few long rows
    ((2, 4096, 2), torch.float16, [1], SUM, torch.float16),           # [O, R, K] columns
    ((4096, 4096), torch.int32, [0, 1], SUM, torch.int64),            # exact integer sum
    ((3, 100000), torch.bfloat16, [1], AMAX, torch.bfloat16),         # exact max
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"{c[1]}-{c[0]}-{c[3]}")
def test_matches_the_allocating_entry_point_on_two_calls(backend, case):
    shape, dtype, dims, op, out_dtype = case
    g = torch.Generator(device="cuda")
    results = []
    for seed in (1, 2):  # two calls in a row, different inputs
        g.manual_seed(seed)
        if dtype.is_floating_point:
            x = (torch.randn(shape, generator=g, device="cuda") * 2).to(dtype)
        else:
            x = torch.randint(-1000, 1000, shape, generator=g, device="cuda", dtype=dtype)
        got, want = _pair(op, x, dims, out_dtype)
        if op in (AMAX, AMIN) or not out_dtype.is_floating_point:
            assert_equal(got, want)
        else:
            assert_close(got, want, out_dtype)
        results.append(got)
    assert not torch.equal(results[0], results[1])


def test_wide_column_sums_fit_the_static_scratch(backend):
    # The column plan combines 8 row lanes per block in shared memory, so its
    # partial results stay near (resident blocks x 32 column vectors) however
    # wide the rows are: a 1.2M-column sum, whose per-split partials would
    # take 9.7 MB under a one-lane-per-block plan, runs inside the 8 MiB array.
    g = torch.Generator(device="cuda").manual_seed(3)
    big = torch.randn(32, 591 * 2048, generator=g, device="cuda").to(torch.bfloat16)
    for _ in range(2):
        got, want = _pair(SUM, big, [0], torch.bfloat16)
        assert_equal(got, want)


def test_rejects_what_needs_more_than_the_static_scratch(backend):
    from tensorplay_mlu_b200 import _native as N

    # A layout whose reduced dimensions are not contiguous needs a gathered copy.
    x = torch.randn(6, 7, 8, device="cuda")
    with pytest.raises(RuntimeError, match="gathered copy"):
        _reduce("tp_b200_reduce_noalloc", SUM, x, [0, 2], torch.float32)
    # A result dtype that would need a conversion buffer.
    with pytest.raises(RuntimeError, match="conversion buffer"):
        _reduce("tp_b200_reduce_noalloc", SUM, torch.ones(4, 4, device="cuda"), [0, 1], torch.float16)
    assert N.lib().tp_b200_take_device_error(torch.cuda.current_device()) == 0
