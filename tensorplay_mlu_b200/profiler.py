"""Per-operation device time (tensorplay-mlu: MLUProfiler.cpp:20-80).

``DeviceTimer`` is the device-timer hook set TensorPlay's profiler calls
around every operation (``current_device``, ``record``, ``elapsed_ms``,
``release``), over pooled CUDA timing events recorded on the device's current
stream (``tp_b200_timer_*``).  ``profile`` is the same measurement for this
package's operator functions when TensorPlay's profiler is not there: inside
the ``with`` block every registered operator (``ops.KERNELS``) is bracketed
by two records, and ``key_averages()`` reports per operator the call count,
device time and host time, like ``profile(activities=[PrivateUse1])``.

    with profile() as prof:
        for _ in range(3):
            ops.relu(ops.mm(a, a))
    rows = {r.key: r for r in prof.key_averages()}
    rows["mm"].count, rows["mm"].device_time_total   # 3, microseconds
"""

from __future__ import annotations

import ctypes
import time
from dataclasses import dataclass, field

from . import _native as N

__all__ = ["DeviceTimer", "profile", "ProfilerActivity"]


class DeviceTimer:
    """The device-timer hooks (MLUProfiler.cpp:20-62) over pooled CUDA events."""

    def current_device(self) -> int:
        return int(N.lib().tp_b200_timer_current_device())

    def record(self, device: int):
        """A timing event recorded on ``device``'s current library stream, or None."""
        return N.lib().tp_b200_timer_record(device)

    def elapsed_ms(self, start, end):
        """Milliseconds between two records (waits for ``end``), or None."""
        if start is None or end is None:
            return None
        ms = ctypes.c_float()
        if N.lib().tp_b200_timer_elapsed_ms(start, end, ctypes.byref(ms)) != 0:
            return None
        return float(ms.value)

    def release(self, event) -> None:
        if event is not None:
            N.lib().tp_b200_timer_release(event)


class ProfilerActivity:
    CPU = "cpu"
    PrivateUse1 = "privateuse1"


@dataclass
class FunctionEvent:
    key: str
    count: int = 0
    device_time_total: float = 0.0  # microseconds
    cpu_time_total: float = 0.0     # microseconds

    @property
    def device_time(self) -> float:
        return self.device_time_total / self.count if self.count else 0.0

    @property
    def cpu_time(self) -> float:
        return self.cpu_time_total / self.count if self.count else 0.0


class EventList(list):
    def table(self, sort_by: str = "device_time_total", row_limit: int = 100) -> str:
        rows = sorted(self, key=lambda r: getattr(r, sort_by), reverse=True)[:row_limit]
        head = f"{'Name':<32s}{'# of Calls':>12s}{'B200 total (us)':>18s}{'B200 avg (us)':>16s}{'CPU total (us)':>16s}"
        lines = [head, "-" * len(head)]
        for r in rows:
            lines.append(f"{r.key:<32s}{r.count:>12d}{r.device_time_total:>18.1f}{r.device_time:>16.1f}"
                         f"{r.cpu_time_total:>16.1f}")
        return "\n".join(lines)


@dataclass
class _Record:
    key: str
    device: int
    start: object
    end: object
    cpu_us: float


def _key(schema: str) -> str:
    return schema.split(".")[0]


@dataclass
class profile:
    """Time every registered operator called inside the block on the device."""

    activities: list = field(default_factory=lambda: [ProfilerActivity.CPU, ProfilerActivity.PrivateUse1])

    def __post_init__(self):
        self._records: list[_Record] = []
        self._patched: list[tuple[str, object]] = []
        self._timer = DeviceTimer()
        self._rows: EventList | None = None

    def __enter__(self):
        from . import ops

        import torch

        by_function = {}
        for schema, fn in ops.KERNELS.items():
            by_function.setdefault(id(fn), _key(schema))
        timed = ProfilerActivity.PrivateUse1 in self.activities
        lib = N.lib()
        for name in dir(ops):
            fn = getattr(ops, name)
            if not callable(fn) or id(fn) not in by_function:
                continue
            key = by_function[id(fn)]

            def wrapper(*args, __fn=fn, __key=key, **kwargs):
                dev = torch.cuda.current_device()
                previous = lib.tp_b200_get_stream(dev)
                lib.tp_b200_set_stream(dev, N.stream_of(dev))
                start = self._timer.record(dev) if timed else None
                t0 = time.perf_counter()
                try:
                    return __fn(*args, **kwargs)
                finally:
                    cpu_us = (time.perf_counter() - t0) * 1e6
                    end = self._timer.record(dev) if timed else None
                    lib.tp_b200_set_stream(dev, previous)
                    self._records.append(_Record(__key, dev, start, end, cpu_us))

            self._patched.append((name, fn))
            setattr(ops, name, wrapper)
        return self

    def __exit__(self, *exc):
        from . import ops

        for name, fn in self._patched:
            setattr(ops, name, fn)
        self._patched.clear()
        rows: dict[str, FunctionEvent] = {}
        for r in self._records:
            row = rows.setdefault(r.key, FunctionEvent(r.key))
            row.count += 1
            row.cpu_time_total += r.cpu_us
            ms = self._timer.elapsed_ms(r.start, r.end)
            if ms is not None:
                row.device_time_total += ms * 1000.0
            self._timer.release(r.start)
            self._timer.release(r.end)
        self._records.clear()
        self._rows = EventList(rows.values())
        return False

    def key_averages(self) -> EventList:
        if self._rows is None:
            raise RuntimeError("the profile has not finished")
        return self._rows
