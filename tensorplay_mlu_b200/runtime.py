"""``tensorplay.b200``: device management and memory statistics.

Mirrors tensorplay-mlu's device module (tensorplay_mlu/runtime.py:12-102):
the same function names, the same memory-statistics keys, backed by the
native runtime and caching allocator instead of CNRT.
"""

from __future__ import annotations

import contextlib
import ctypes

from . import _native

__all__ = [
    "current_device", "device", "device_count", "empty_cache", "is_available",
    "is_initialized", "max_memory_allocated", "max_memory_reserved", "mem_get_info",
    "memory_allocated", "memory_reserved", "memory_stats", "reset_peak_memory_stats",
    "set_device", "synchronize",
]


def is_available() -> bool:
    try:
        return _native.lib().tp_b200_device_count() > 0
    except Exception:
        return False


def is_initialized() -> bool:
    return True


def device_count() -> int:
    return _native.lib().tp_b200_device_count()


def current_device() -> int:
    dev = _native.lib().tp_b200_current_device()
    _native.check(dev, "current_device")
    return dev


def _index(device=None) -> int:
    if device is None:
        return current_device()
    if isinstance(device, int):
        return device
    index = getattr(device, "index", None)
    if index is None and isinstance(device, str) and ":" in device:
        index = int(device.rsplit(":", 1)[1])
    return current_device() if index is None or index < 0 else index


def set_device(device) -> None:
    _native.check(_native.lib().tp_b200_set_device(_index(device)), "set_device")


@contextlib.contextmanager
def device(index):
    """Context manager: B200 ``index`` is the current device while the
    ``with`` body runs; the previous device is restored afterwards."""
    previous = current_device()
    set_device(index)
    try:
        yield
    finally:
        set_device(previous)


def synchronize(device=None) -> None:
    _native.check(_native.lib().tp_b200_synchronize(_index(device)), "synchronize")


def memory_stats(device=None) -> dict[str, int]:
    out = (ctypes.c_int64 * 4)()
    _native.lib().tp_b200_memory_stats(_index(device), out)
    return {
        "allocated_bytes": out[0],
        "reserved_bytes": out[1],
        "peak_allocated_bytes": out[2],
        "peak_reserved_bytes": out[3],
    }


def memory_allocated(device=None) -> int:
    return memory_stats(device)["allocated_bytes"]


def memory_reserved(device=None) -> int:
    return memory_stats(device)["reserved_bytes"]


def max_memory_allocated(device=None) -> int:
    return memory_stats(device)["peak_allocated_bytes"]


def max_memory_reserved(device=None) -> int:
    return memory_stats(device)["peak_reserved_bytes"]


def reset_peak_memory_stats(device=None) -> None:
    _native.lib().tp_b200_reset_peak_memory_stats(_index(device))


def empty_cache() -> None:
    """Free the caching allocator's idle blocks (cudaFree), keeping blocks
    that tensors still hold."""
    _native.lib().tp_b200_empty_cache()


def mem_get_info(device=None) -> tuple[int, int]:
    """cudaMemGetInfo for the device: a (free_bytes, total_bytes) tuple."""
    free = ctypes.c_size_t()
    total = ctypes.c_size_t()
    _native.check(_native.lib().tp_b200_mem_get_info(_index(device), ctypes.byref(free),
                                                      ctypes.byref(total)), "mem_get_info")
    return free.value, total.value
