"""The allocation-free reduction entry point, tp_b200_reduce_noalloc.

It exists for callers that cannot allocate device memory when they reduce --
a serving process whose GPU memory is reserved up front by its own pool, or a
latency-critical path that must not risk a cudaMalloc on an allocator miss --
and keeps its partial results in a static 8 MiB device array instead.  These
tests call it through the C ABI and check its results against the ordinary
entry point, tp_b200_reduce, and against the CPU oracle, on two calls in a row
(the array keeps the previous call's contents, which must not leak into the
next result); they check that a call leaves the caching allocator's
statistics and, once the first call on the device has done its set-up, the
driver's free-memory count unchanged.  The file is named to be collected last
so a failure here cannot hide failures elsewhere; it passes alone in a fresh
process as well as after the suite.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
import sys

import pytest
import torch

import oracle as O
from conftest import ROOT, assert_close, assert_equal

pytestmark = pytest.mark.gpu

SUM, MEAN, AMAX, AMIN = range(4)


def _reduce(entry, op, x, dims, out_dtype, out=None):
    from tensorplay_mlu_b200 import _native as N

    mask = 0
    for d in dims:
        mask |= 1 << d
    keep = [1 if (mask >> i) & 1 else s for i, s in enumerate(x.shape)]
    if out is None:
        out = torch.empty(keep, dtype=out_dtype, device=x.device)
    status = getattr(N.lib(), entry)(op, N.describe(out), N.describe(x), mask,
                                     ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    N.check(status, entry)
    return out


CASES = [
    # (shape, dtype, dims, op, out dtype) -- each uses per-block partial results
    ((8192, 8192), torch.float32, [0, 1], SUM, torch.float32),        # full reduction, thousands of splits
    ((8192, 16384), torch.bfloat16, [0], SUM, torch.bfloat16),        # bias-gradient column sum
    ((16, 65536), torch.float32, [1], MEAN, torch.float32),           # few long rows
    ((2, 4096, 2), torch.float16, [1], SUM, torch.float16),           # [O, R, K] columns
    ((4096, 4096), torch.int32, [0, 1], SUM, torch.int64),            # exact integer sum
    ((3, 100000), torch.bfloat16, [1], AMAX, torch.bfloat16),         # exact max
    ((64, 1), torch.int32, [1], SUM, torch.int64),                    # nothing to reduce (R == 1)
]


def _host_input(shape, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    if dtype.is_floating_point:
        return (torch.randn(shape, generator=g) * 2).to(dtype)
    return torch.randint(-1000, 1000, shape, generator=g, dtype=dtype)


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"{c[1]}-{c[0]}-{c[3]}")
def test_matches_the_allocating_entry_point_and_the_oracle_on_two_calls(backend, case):
    shape, dtype, dims, op, out_dtype = case
    results = []
    for seed in (1, 2):  # two calls in a row, different inputs
        xh = _host_input(shape, dtype, seed)
        x = backend.ops.to_device(xh)
        mask_keep = [1 if i in dims else s for i, s in enumerate(shape)]
        out = torch.empty(mask_keep, dtype=out_dtype, device="cuda")
        torch.cuda.synchronize()
        stats0 = backend.runtime.memory_stats()
        _reduce("tp_b200_reduce_noalloc", op, x, dims, out_dtype, out=out)
        torch.cuda.synchronize()
        # The call itself takes nothing from the caching allocator.
        assert backend.runtime.memory_stats() == stats0
        got = out.cpu()
        want = _reduce("tp_b200_reduce", op, x, dims, out_dtype).cpu()
        ref = O.reduce(op, xh, dims, out_dtype, keepdim=True)
        if op in (AMAX, AMIN) or not out_dtype.is_floating_point:
            assert_equal(got, want)
            assert_equal(got, ref)
        else:
            assert_close(got, want, out_dtype)
            assert_close(got, ref, out_dtype)
        results.append(got)
    assert not torch.equal(results[0], results[1])


def test_wide_column_sums_fit_the_static_scratch(backend):
    # The column plan combines 8 row lanes per block in shared memory, so its
    # partial results stay near (resident blocks x 32 column vectors) however
    # wide the rows are: a 1.2M-column sum, whose per-split partials would
    # take 9.7 MB under a one-lane-per-block plan, runs inside the 8 MiB array.
    xh = _host_input((32, 591 * 2048), torch.bfloat16, 3)
    big = backend.ops.to_device(xh)
    ref = O.reduce(SUM, xh, [0], torch.bfloat16, keepdim=True)
    for _ in range(2):
        got = _reduce("tp_b200_reduce_noalloc", SUM, big, [0], torch.bfloat16).cpu()
        assert_equal(got, _reduce("tp_b200_reduce", SUM, big, [0], torch.bfloat16).cpu())
        assert_close(got, ref, torch.bfloat16)


def test_rejects_what_needs_more_than_the_static_scratch(backend):
    from tensorplay_mlu_b200 import _native as N

    # A layout whose reduced dimensions are not contiguous needs a gathered copy.
    x = torch.randn(6, 7, 8, device="cuda")
    with pytest.raises(RuntimeError, match="gathered copy"):
        _reduce("tp_b200_reduce_noalloc", SUM, x, [0, 2], torch.float32)
    # A result dtype that would need a conversion buffer.
    with pytest.raises(RuntimeError, match="conversion buffer"):
        _reduce("tp_b200_reduce_noalloc", SUM, torch.ones(4, 4, device="cuda"), [0, 1], torch.float16)
    # A column reduction under 65536 outer rows (the column kernel's grid).
    cols = torch.zeros(65536, 2, 8, device="cuda")
    with pytest.raises(RuntimeError, match="outer rows"):
        _reduce("tp_b200_reduce_noalloc", SUM, cols, [1], torch.float32)
    # tp_b200_reduce takes the same input (through a gathered copy).
    _reduce("tp_b200_reduce", SUM, cols, [1], torch.float32)
    torch.cuda.synchronize()
    assert N.lib().tp_b200_take_device_error(torch.cuda.current_device()) == 0


def _run_fresh(script: str, env_extra=None) -> str:
    env = dict(os.environ)
    env.update(env_extra or {})
    proc = subprocess.run([sys.executable, "-c", script], cwd=ROOT, env=env, capture_output=True, text=True,
                          timeout=300)
    assert proc.returncode == 0, proc.stdout + proc.stderr
    return proc.stdout


_FRESH_PRELUDE = r"""
import ctypes, sys, torch
sys.path.insert(0, '.')
import tensorplay_mlu_b200 as tpb
from tensorplay_mlu_b200 import _native as N
tpb.load()
torch.cuda.set_device(0)

def call(op, x, dims, out):
    mask = 0
    for d in dims:
        mask |= 1 << d
    N.check(N.lib().tp_b200_reduce_noalloc(op, N.describe(out), N.describe(x), mask,
            ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)), 'reduce_noalloc')
"""


def test_no_device_memory_is_taken_after_the_first_call_in_a_fresh_process(backend):
    # The first call on a device is the set-up (the array and every kernel
    # the entry point can launch are loaded); afterwards calls over other
    # dtypes, ops and layouts leave the driver's free-memory count as it was.
    script = _FRESH_PRELUDE + r"""
g = torch.Generator(device='cuda').manual_seed(0)
cases = []
def case(x, dims, op, out_dtype):
    keep = [1 if i in dims else s for i, s in enumerate(x.shape)]
    cases.append((op, x, dims, torch.empty(keep, dtype=out_dtype, device='cuda')))
case(torch.randn(4096, 4096, generator=g, device='cuda').to(torch.bfloat16), [1], 0, torch.bfloat16)
case(torch.randn(4096, 4096, generator=g, device='cuda'), [0], 1, torch.float32)
case(torch.randn(1 << 22, generator=g, device='cuda').double(), [0], 0, torch.float64)
case(torch.randint(-9, 9, (2048, 2048), generator=g, device='cuda', dtype=torch.int32), [0, 1], 0, torch.int64)
case(torch.randint(-9, 9, (8, 300000), generator=g, device='cuda', dtype=torch.int16), [1], 2, torch.int16)
case(torch.randn(3, 5000, 7, generator=g, device='cuda').half(), [1], 3, torch.float16)
case(torch.randint(0, 2, (1000, 33), generator=g, device='cuda', dtype=torch.uint8).bool(), [1], 0, torch.int64)
first = torch.randn(64, 64, device='cuda')
call(0, first, [1], torch.empty(64, 1, device='cuda'))   # set-up on device 0
torch.cuda.synchronize()
free0 = torch.cuda.mem_get_info()[0]
stats0 = tpb.runtime.memory_stats()
for _ in range(2):
    for op, x, dims, out in cases:
        call(op, x, dims, out)
torch.cuda.synchronize()
free1 = torch.cuda.mem_get_info()[0]
assert tpb.runtime.memory_stats() == stats0, (tpb.runtime.memory_stats(), stats0)
assert free1 == free0, (free0, free1)
print('free unchanged', free0)
"""
    assert "free unchanged" in _run_fresh(script)


def test_partials_over_the_static_scratch_are_rejected_in_a_fresh_process(backend):
    # On the default plans the partial results stay far below 8 MiB; the
    # forced shared-memory ring plan keeps one partial per 16 KB chunk of each
    # row, so 524288 rows of 8 chunks (rows expanded from one, no memory)
    # need 16 MiB and must be refused, not written past the array.
    script = _FRESH_PRELUDE + r"""
row = torch.randn(1, 8 * 4096, device='cuda')
x = row.expand(1 << 19, 8 * 4096)
out = torch.empty(1 << 19, 1, device='cuda')
try:
    call(0, x, [1], out)
except RuntimeError as e:
    assert 'partial results' in str(e), str(e)
    print('rejected')
assert N.lib().tp_b200_take_device_error(0) == 0
"""
    assert "rejected" in _run_fresh(script, {"TPB200_REDUCE_ROWS": "ring"})
