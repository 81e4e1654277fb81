"""Host-side operator logic without a GPU: dtype promotion, result shapes and
argument checks mirror the host framework's (PyTorch CPU stands in for
TensorPlay's), and the collective helpers' split arithmetic."""

from __future__ import annotations

import itertools

import pytest
import torch

from tensorplay_mlu_b200 import distributed as D
from tensorplay_mlu_b200 import ops

DTYPES = [torch.uint8, torch.int8, torch.int16, torch.int32, torch.int64, torch.float16,
          torch.bfloat16, torch.float32, torch.float64, torch.bool]


@pytest.mark.parametrize("da,db", list(itertools.product(DTYPES, DTYPES)))
def test_binary_promotion_matches_host(da, db):
    a = torch.zeros(3, 2, dtype=da)
    b = torch.zeros(2, dtype=db)
    assert ops.binary_result_dtype(a, b) == torch.result_type(a, b)
    s = torch.zeros((), dtype=db)
    assert ops.binary_result_dtype(a, s) == torch.result_type(a, s)


@pytest.mark.parametrize("dt", DTYPES)
@pytest.mark.parametrize("value", [2, 2.5, True])
def test_scalar_promotion_matches_host(dt, value):
    a = torch.zeros(3, dtype=dt)
    assert ops.scalar_result_dtype(dt, value) == torch.result_type(a, value)


def test_dims_normalisation():
    t = torch.zeros(2, 3, 4)
    assert ops._dims(t, -1) == [2]
    assert ops._dims(t, [0, -1]) == [0, 2]
    assert ops._dims(t, None) == [0, 1, 2]
    with pytest.raises(IndexError):
        ops._dims(t, 3)
    with pytest.raises(RuntimeError):
        ops._dims(t, [1, -2])


def test_device_operators_reject_host_tensors():
    with pytest.raises(RuntimeError):
        ops.exp(torch.zeros(3))
    with pytest.raises(RuntimeError):
        ops.mm(torch.zeros(2, 2), torch.zeros(2, 2))


def test_all_to_all_split_arithmetic():
    t = torch.zeros(6, 4)
    assert D._element_counts(t, [1, 2, 3], 3) == [4, 8, 12]
    assert D._element_counts(t, None, 2) == [12, 12]
    assert D._prefix_offsets([4, 8, 12]) == [0, 4, 12]


def test_reduction_table_matches_the_reference():
    # AVG is SUM plus a 1/world scale (tensorplay_mlu/distributed.py:48-58).
    assert D._REDUCTIONS[D.ReduceOp.AVG] == (0, None)
    assert D._REDUCTIONS[D.ReduceOp.MAX][0] == 2 and D._REDUCTIONS[D.ReduceOp.MIN][0] == 3


@pytest.mark.parametrize("d_in,d_hidden,slices", [(4096, 16384, 1), (4096, 16384, 2), (4096, 16384, 4),
                                                  (256, 512, 2), (256, 1000, 3), (64, 24, 8)])
def test_bucket_b_slices_tile_the_bucket(d_in, d_hidden, slices):
    # The data-parallel step exchanges bucket B = (db1, dW1) in row slices of
    # dW1: together they cover the flat bucket exactly once, in order, db1
    # with the first, and every slice of d_h's columns starts 16-byte aligned.
    from tensorplay_mlu_b200.train import bucket_b_slices

    parts = bucket_b_slices(d_in, d_hidden, slices)
    assert parts[0][2] == 0
    offset = 0
    rows = 0
    for r0, r1, lo, length in parts:
        assert lo == offset and length > 0 and r0 == rows and r1 > r0
        assert (r0 * 2) % 16 == 0  # bf16 column offset of d_h
        offset += length
        rows = r1
    assert rows == d_hidden and offset == d_hidden + d_hidden * d_in
    assert len(parts) <= slices


@pytest.mark.parametrize("rows,slices", [(8192, 1), (8192, 2), (4096, 2), (64, 3), (256, 3), (8, 4), (12, 2)])
def test_row_slices_cover_the_rows_on_aligned_bounds(rows, slices):
    # The products beside an exchange run in row slices: in order, covering
    # every row once, each slice non-empty and starting on a multiple of 8
    # (16 bytes of bf16); at most `slices` of them.
    from tensorplay_mlu_b200.train import row_slices

    parts = row_slices(rows, slices)
    assert 1 <= len(parts) <= slices
    assert parts[0][0] == 0 and parts[-1][1] == rows
    for (a0, a1), (b0, _) in zip(parts, parts[1:]):
        assert a1 == b0
    for r0, r1 in parts:
        assert r1 > r0 and r0 % 8 == 0
    if rows % (8 * slices) == 0:
        assert all(r1 - r0 == rows // slices for r0, r1 in parts)


@pytest.mark.parametrize("dtype", [torch.bool, torch.uint8, torch.int8, torch.int16, torch.int32, torch.int64,
                                   torch.float16, torch.bfloat16, torch.float32, torch.float64])
def test_reduction_result_dtypes_match_the_host(dtype):
    # An explicit dtype wins, else the input's (ReduceKernels.cpp:86-88); the
    # reference sends integer inputs to the host kernels (:97-103), where a
    # sum of integers (bool included) accumulates in int64 and mean refuses
    # integer inputs unless a floating dtype is given -- the device path here
    # keeps those host results.
    from tensorplay_mlu_b200 import ops

    x = torch.zeros(3, dtype=dtype)
    assert ops._sum_dtype(x, None) == torch.sum(x).dtype
    assert ops._sum_dtype(x, torch.float64) == torch.float64
    if dtype.is_floating_point:
        assert ops._mean_dtype(x, None) == torch.mean(x).dtype
    else:
        with pytest.raises(RuntimeError, match="could not infer output dtype"):
            ops._mean_dtype(x, None)
        assert ops._mean_dtype(x, torch.float32) == torch.float32


@pytest.mark.parametrize("self_dtype,result,ok", [
    (torch.float32, torch.float32, True), (torch.float32, torch.int64, True),
    (torch.int64, torch.float32, False), (torch.int32, torch.bool, True),
    (torch.bool, torch.int32, False), (torch.bfloat16, torch.float32, True),
])
def test_in_place_results_cast_like_the_host(self_dtype, result, ok):
    # An in-place operator may not write a result type the output cannot
    # hold (an integer tensor receiving a float result), as on the host.
    from tensorplay_mlu_b200 import ops

    if ok:
        ops._check_inplace(self_dtype, result)
    else:
        with pytest.raises(RuntimeError, match="can't be cast"):
            ops._check_inplace(self_dtype, result)


def test_layer_norm_statistics_type():
    from tensorplay_mlu_b200 import ops

    assert ops._stats_dtype(torch.float64) == torch.float64
    for dt in (torch.float32, torch.bfloat16, torch.float16):
        assert ops._stats_dtype(dt) == torch.float32
