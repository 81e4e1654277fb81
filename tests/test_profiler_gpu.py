"""Per-operation device time (tensorplay-mlu: MLUProfiler.cpp:20-80; the
reference's test_mlu.py:381-401 checks the same rows through TensorPlay's
profiler): every registered operator called in the block gets a row with its
call count and device time, the device timer gives back every pooled event,
and a device timing covers the work between its two records."""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_profile_reports_device_time_per_operator(backend):
    from tensorplay_mlu_b200.profiler import ProfilerActivity, profile
    from tensorplay_mlu_b200 import _native as N

    ops = backend.ops
    a = ops.to_device(torch.randn(512, 512))
    ops.mm(a, a)
    pooled = N.lib().tp_b200_timer_pooled()
    with profile(activities=[ProfilerActivity.CPU, ProfilerActivity.PrivateUse1]) as prof:
        for _ in range(3):
            ops.relu(ops.mm(a, a))
    rows = {r.key: r for r in prof.key_averages()}
    assert rows["mm"].count == 3 and rows["mm"].device_time_total > 0
    assert rows["relu"].count == 3 and rows["relu"].device_time_total > 0
    assert rows["mm"].cpu_time_total > 0
    assert "B200" in prof.key_averages().table(sort_by="device_time_total", row_limit=5)
    # Every event taken for the session is back in the pool.
    assert N.lib().tp_b200_timer_pooled() >= pooled + 2
    # Outside the block the operators are the plain functions again.
    assert ops.mm is backend.ops.KERNELS["mm"]


def test_device_timer_measures_the_bracketed_work(backend):
    from tensorplay_mlu_b200.profiler import DeviceTimer

    ops = backend.ops
    timer = DeviceTimer()
    dev = timer.current_device()
    a = ops.to_device(torch.randn(4096, 4096).to(torch.bfloat16))
    ops.mm(a, a)  # first use of this product shape: host set-up outside the timing
    torch.cuda.synchronize()
    lib = backend._native.lib()
    previous = lib.tp_b200_get_stream(dev)
    lib.tp_b200_set_stream(dev, backend._native.stream_of(dev))
    try:
        t0 = timer.record(dev)
        ops.mm(a, a)
        t1 = timer.record(dev)
        for _ in range(20):
            ops.mm(a, a)
        t2 = timer.record(dev)
    finally:
        lib.tp_b200_set_stream(dev, previous)
    one, twenty = timer.elapsed_ms(t0, t1), timer.elapsed_ms(t1, t2)
    assert one is not None and twenty is not None and one > 0
    assert twenty > 5 * one  # twenty products take longer than one
    for e in (t0, t1, t2):
        timer.release(e)
    assert timer.record(10 ** 6) is None  # an invalid device gives no event
