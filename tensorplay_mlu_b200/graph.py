"""Recording a fixed sequence of device work and replaying it in one launch.

Mirror of ``tensorplay_mlu/graph.py:38-92`` (``Graph`` with ``capture``,
``replay``, ``reset``, ``stats`` and ``ready``) over CUDA stream capture.

    graph = Graph()
    loss = graph.capture(lambda: model.step(x, target))
    x.copy_(next_batch)          # the recorded work reads x's buffer again
    graph.replay()               # loss now holds the replayed step's value

The body runs on a stream created for the recording (the default stream
cannot be captured); the library's kernels and the caching allocator see it
as the current stream.  The values a capture returns are kept by the graph,
because the recorded work reads and writes those buffers on every replay.
A body may only queue device work: a host read-back or synchronisation
inside it invalidates the recording and raises.
"""

from __future__ import annotations

import ctypes

import torch

from . import _native as N

__all__ = ["Graph"]


def _check(status: int) -> None:
    N.check(status, "recording")


class Graph:
    """A recorded sequence of device work that replays in one call."""

    def __init__(self) -> None:
        self._outputs = None
        self._ready = False
        self._device = None
        self._stream = None

    @property
    def ready(self) -> bool:
        return bool(N.lib().tp_b200_capture_ready())

    def capture(self, body):
        """Record what one call to ``body`` queues, and return its value."""
        lib = N.lib()
        index = torch.cuda.current_device()
        torch.cuda.synchronize(index)
        stream = torch.cuda.Stream(device=index)
        previous = lib.tp_b200_get_stream(index)
        _check(lib.tp_b200_set_stream(index, stream.cuda_stream))
        try:
            _check(lib.tp_b200_capture_begin(index))
            try:
                with torch.cuda.stream(stream):
                    outputs = body()
            except BaseException:
                self._abandon()
                raise
            try:
                _check(lib.tp_b200_capture_end(index))
            except BaseException:
                self._abandon()
                raise
        finally:
            lib.tp_b200_set_stream(index, previous)
        self._outputs = outputs
        self._ready = True
        self._device = index
        self._stream = stream
        return outputs

    def replay(self) -> None:
        """Queue another run of the recording on the current stream."""
        if not self._ready:
            raise RuntimeError("nothing has been recorded yet")
        lib = N.lib()
        index = self._device
        previous = lib.tp_b200_get_stream(index)
        _check(lib.tp_b200_set_stream(index, N.stream_of(index)))
        try:
            _check(lib.tp_b200_capture_invoke(index))
        finally:
            lib.tp_b200_set_stream(index, previous)

    def reset(self) -> None:
        """Drop the recording and give back the blocks it held.  The values
        the capture returned are released first, so their blocks go back in
        the same reset unless the caller still holds them."""
        self._outputs = None
        self._ready = False
        _check(N.lib().tp_b200_capture_reset())

    def stats(self) -> tuple[int, int]:
        """Blocks handed out while recording, and blocks the recording holds."""
        out = (ctypes.c_int64 * 2)()
        N.lib().tp_b200_capture_stats(out)
        return int(out[0]), int(out[1])

    def _abandon(self) -> None:
        try:
            N.lib().tp_b200_capture_reset()
        except Exception:  # noqa: BLE001 - the original failure is the one to raise
            pass
        self._outputs = None
        self._ready = False
