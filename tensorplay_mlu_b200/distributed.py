"""NCCL process group for B200 tensors (the ``nccl_b200`` backend).

The host-side mirror of tensorplay-mlu's CNCL process group
(tensorplay_mlu/distributed.py:158-591): the same provider protocol
(``ensure``/``destroy``/``allreduce``/``allgather``/... each returning a work
object with ``is_completed``/``wait``/``abort``), the same dtype and
reduction codes, and the same rendezvous -- rank 0 creates the communicator id
and publishes it as hex in the process store, the other ranks read it with a
timeout (:169-197).  The collectives run over NCCL through the C ABI
(``tp_b200_nccl_*``), one process per GPU, over NVLink / NVSwitch.

Differences, by design for B200:
  * collectives are enqueued on PyTorch's current stream of the device, so a
    caller can run the gradient exchange on a side stream and overlap it with
    the rest of the backward pass;
  * AVG is a SUM followed by one scale kernel, as in the reference
    (:220-229); the data-parallel trainer folds that scale into its SGD
    update instead of launching it (see ``train.py``);
  * ``create(...)`` accepts any store with ``set``/``get`` (a
    ``torch.distributed`` TCPStore here; TensorPlay's store when present);
  * communicator creation can be bounded by a timeout, so a rank that never
    joins turns into an error instead of a hang.
"""

from __future__ import annotations

import ctypes
import time
from typing import Any, List, Optional

import torch

from . import _native as N

__all__ = ["is_available", "ProcessGroupB200", "create", "register", "ReduceOp"]


class ReduceOp:
    """TensorPlay's ReduceOp values (the keys of tensorplay_mlu/distributed.py:53-58)."""

    SUM = 0
    AVG = 1
    PRODUCT = 2
    MIN = 3
    MAX = 4


# ReduceOp value -> (NCCL reduction code, post-scale); None = 1/world (AVG).
_SUM_CODE, _PROD_CODE, _MAX_CODE, _MIN_CODE = 0, 1, 2, 3
_REDUCTIONS = {
    ReduceOp.SUM: (_SUM_CODE, 1.0),
    ReduceOp.AVG: (_SUM_CODE, None),
    ReduceOp.PRODUCT: (_PROD_CODE, 1.0),
    ReduceOp.MIN: (_MIN_CODE, 1.0),
    ReduceOp.MAX: (_MAX_CODE, 1.0),
}


def _check(code: int) -> None:
    if code >= 0:
        return
    message = N.lib().tp_b200_nccl_last_error()
    raise RuntimeError(message.decode() if message else "NCCL call failed")


def _ptr(t: torch.Tensor) -> ctypes.c_void_p:
    return ctypes.c_void_p(int(t.data_ptr()))


def _dtype_code(t: torch.Tensor) -> int:
    try:
        code = N.DTYPE_CODES[t.dtype]
    except KeyError as error:
        raise TypeError(f"NCCL does not support {t.dtype} tensors") from error
    if t.dtype == torch.int16:
        raise TypeError("NCCL does not support torch.int16 tensors")
    return code


def _flat(t: torch.Tensor) -> torch.Tensor:
    """A contiguous 1-D view of ``t`` (a device copy when it is strided)."""
    from . import ops

    if t.dim() == 1 and t.is_contiguous():
        return t
    return ops.contiguous(t).reshape(-1)


class _Work:
    """Handle for collectives enqueued on a stream that has not drained yet.

    ``wait()`` without a timeout makes the caller's current stream wait for
    the collective (no host block), as a CUDA process group's work does.
    ``wait(timeout)`` also bounds it on the host: it polls the collective's
    completion and the communicator's asynchronous error until the deadline,
    and a collective that has not finished by then aborts the communicator
    and raises ``TimeoutError`` -- a stuck peer becomes an error instead of
    a hang (tensorplay-mlu's wait ignores its timeout,
    tensorplay_mlu/distributed.py:113-118)."""

    POLL_S = 0.001

    def __init__(self, device: int, stream, done=None, group=None, event=None) -> None:
        self._device = device
        if event is None:
            event = torch.cuda.Event()
            event.record(stream)
        self._event = event
        self._done = done
        self._group = group
        self._finished = False

    def _finish(self) -> None:
        if not self._finished:
            self._finished = True
            if self._done is not None:
                self._done()

    def is_completed(self) -> bool:
        if self._finished:
            return True
        if self._event.query():
            self._finish()
            return True
        return False

    def wait(self, timeout=None) -> bool:
        seconds = _seconds(timeout)
        if seconds is not None and seconds > 0:
            deadline = time.monotonic() + seconds
            while not self._event.query():
                if self._group is not None:
                    self._group.check()  # raises on an asynchronous NCCL error
                if time.monotonic() > deadline:
                    if self._group is not None:
                        self._group.abort()
                    raise TimeoutError(f"collective did not complete within {seconds} s; "
                                       "the communicator was aborted")
                time.sleep(self.POLL_S)
            self._finish()
            return True
        torch.cuda.current_stream(self._device).wait_event(self._event)
        self._finish()
        return True

    def synchronize(self) -> None:
        self._event.synchronize()
        self._finish()

    def abort(self) -> None:
        raise RuntimeError("abort is unavailable for an individual NCCL work item; "
                           "abort the process group's communicator instead")


def _seconds(timeout) -> Optional[float]:
    """A work timeout in seconds: a number of seconds or a timedelta."""
    if timeout is None:
        return None
    if hasattr(timeout, "total_seconds"):
        return float(timeout.total_seconds())
    return float(timeout)


class ProcessGroupB200:
    """Collective provider for one ``nccl_b200`` group (one rank per GPU)."""

    def __init__(self, store, rank: int, size: int, device: Optional[int] = None,
                 group_name: str = "default", timeout_s: float = 300.0, max_ctas: int = 0) -> None:
        self._store = store
        self._rank = rank
        self._size = size
        self._device = torch.cuda.current_device() if device is None else device
        self._group_name = group_name
        self._timeout_s = timeout_s
        self._comm: Optional[ctypes.c_void_p] = None
        self._barrier_flag: Optional[torch.Tensor] = None
        # Bound on the CTAs (SMs) NCCL's kernels take (0: NCCL's choice).
        self._max_ctas = int(max_ctas)

    # -- lifecycle ---------------------------------------------------------
    def rank(self) -> int:
        return self._rank

    def size(self) -> int:
        return self._size

    def ensure(self) -> None:
        """Create the communicator, rendezvousing through the store."""
        if self._comm is not None:
            return
        lib = N.lib()
        nbytes = lib.tp_b200_nccl_unique_id_bytes()
        key = f"tensorplay_distributed/nccl_b200_unique_id/{self._group_name}"
        if self._rank == 0:
            buf = ctypes.create_string_buffer(nbytes)
            _check(lib.tp_b200_nccl_get_unique_id(buf))
            self._store.set(key, buf.raw.hex())
        else:
            raw = _store_get(self._store, key, self._timeout_s)
            buf = ctypes.create_string_buffer(bytes.fromhex(raw.decode() if isinstance(raw, bytes) else raw), nbytes)
        comm = ctypes.c_void_p()
        timeout_ms = int(self._timeout_s * 1000)
        _check(lib.tp_b200_nccl_comm_init_ctas(self._rank, self._size, self._device, buf, timeout_ms, 0,
                                               self._max_ctas, ctypes.byref(comm)))
        self._comm = comm

    def destroy(self) -> None:
        if self._comm is None:
            return
        torch.cuda.synchronize(self._device)
        _check(N.lib().tp_b200_nccl_comm_destroy(self._comm))
        self._comm = None

    def abort(self) -> None:
        if self._comm is not None:
            _check(N.lib().tp_b200_nccl_comm_abort(self._comm))
            self._comm = None

    def check(self) -> None:
        """Raise when the communicator has reported an asynchronous error."""
        if self._comm is not None:
            _check(N.lib().tp_b200_nccl_comm_check(self._comm))

    def set_timeout(self, timeout_ms: int) -> None:
        self._timeout_s = timeout_ms / 1000.0

    # -- plumbing ----------------------------------------------------------
    def _enter(self) -> tuple[Any, torch.cuda.Stream]:
        """Point the library's current stream at PyTorch's current stream."""
        self.ensure()
        stream = torch.cuda.current_stream(self._device)
        _check(N.lib().tp_b200_set_stream(self._device, ctypes.c_void_p(stream.cuda_stream)))
        return N.lib(), stream

    def _work(self, stream) -> _Work:
        return _Work(self._device, stream, group=self)

    def _reduction(self, op: int):
        try:
            code, scale = _REDUCTIONS[int(op)]
        except KeyError:
            raise RuntimeError(f"NCCL does not support reduction {op}")
        if scale is None:
            scale = 1.0 / self._size
        return code, scale

    def _scale(self, tensor: torch.Tensor, scale: float) -> None:
        if scale != 1.0:
            from . import ops

            ops.mul__Scalar(tensor, scale)

    # -- collectives -------------------------------------------------------
    def allreduce(self, tensors: List[torch.Tensor], op: int = ReduceOp.SUM, timeout_ms: int = 0):
        lib, stream = self._enter()
        tensor = tensors[0]
        code, scale = self._reduction(op)
        count = int(tensor.numel())
        if count:
            _check(lib.tp_b200_nccl_all_reduce(_ptr(tensor), _ptr(tensor), count, _dtype_code(tensor),
                                               code, self._device, self._comm))
            self._scale(tensor, scale)
        return self._work(stream)

    def allreduce_coalesced(self, tensors: List[torch.Tensor], op: int = ReduceOp.SUM,
                            timeout_ms: int = 0):
        lib, stream = self._enter()
        code, scale = self._reduction(op)
        _check(lib.tp_b200_nccl_group_start())
        for tensor in tensors:
            count = int(tensor.numel())
            if count:
                _check(lib.tp_b200_nccl_all_reduce(_ptr(tensor), _ptr(tensor), count,
                                                   _dtype_code(tensor), code, self._device, self._comm))
        _check(lib.tp_b200_nccl_group_end())
        for tensor in tensors:
            self._scale(tensor, scale)
        return self._work(stream)

    def broadcast(self, tensors: List[torch.Tensor], root: int = 0, root_tensor: int = 0,
                  timeout_ms: int = 0):
        lib, stream = self._enter()
        tensor = tensors[0]
        count = int(tensor.numel())
        if count:
            _check(lib.tp_b200_nccl_broadcast(_ptr(tensor), _ptr(tensor), count, _dtype_code(tensor),
                                              root, self._device, self._comm))
        return self._work(stream)

    def reduce(self, tensors: List[torch.Tensor], root: int = 0, op: int = ReduceOp.SUM,
               root_tensor: int = 0, timeout_ms: int = 0):
        lib, stream = self._enter()
        tensor = tensors[0]
        code, scale = self._reduction(op)
        count = int(tensor.numel())
        if count:
            _check(lib.tp_b200_nccl_reduce(_ptr(tensor), _ptr(tensor), count, _dtype_code(tensor),
                                           code, root, self._device, self._comm))
            if self._rank == root:
                self._scale(tensor, scale)
        return self._work(stream)

    def _into_buffer(self, chunks: List[torch.Tensor]) -> torch.Tensor:
        """A dense buffer holding ``chunks`` end to end."""
        from . import ops

        total = 0
        for c in chunks:
            total += int(c.numel())
        buffer = torch.empty((total,), dtype=chunks[0].dtype, device=chunks[0].device)
        offset = 0
        for chunk in chunks:
            n = int(chunk.numel())
            if n:
                ops.copy_(buffer.narrow(0, offset, n), _flat(chunk))
            offset += n
        return buffer

    def _scatter_from(self, flat: torch.Tensor, chunks: List[torch.Tensor]) -> None:
        from . import ops

        offset = 0
        for chunk in chunks:
            n = int(chunk.numel())
            if n:
                ops.copy_(chunk, flat.narrow(0, offset, n).reshape(chunk.shape))
            offset += n

    def allgather(self, output_lists, input_tensors: List[torch.Tensor], timeout_ms: int = 0):
        lib, stream = self._enter()
        outputs = output_lists[0]
        tensor = input_tensors[0]
        count = int(tensor.numel())
        if count:
            flat = self._into_buffer(outputs)
            _check(lib.tp_b200_nccl_all_gather(_ptr(tensor), _ptr(flat), count, _dtype_code(tensor),
                                               self._device, self._comm))
            self._scatter_from(flat, outputs)
        return self._work(stream)

    def all_gather_single(self, output: torch.Tensor, input_tensor: torch.Tensor, timeout_ms: int = 0):
        lib, stream = self._enter()
        count = int(input_tensor.numel())
        if count:
            _check(lib.tp_b200_nccl_all_gather(_ptr(input_tensor), _ptr(output), count,
                                               _dtype_code(input_tensor), self._device, self._comm))
        return self._work(stream)

    def reduce_scatter(self, recv_tensors: List[torch.Tensor], input_lists, op: int = ReduceOp.SUM,
                       timeout_ms: int = 0):
        lib, stream = self._enter()
        output = recv_tensors[0]
        code, scale = self._reduction(op)
        count = int(output.numel())
        if count:
            send = self._into_buffer(input_lists[0])
            _check(lib.tp_b200_nccl_reduce_scatter(_ptr(send), _ptr(output), count, _dtype_code(output),
                                                   code, self._device, self._comm))
            self._scale(output, scale)
        return self._work(stream)

    def reduce_scatter_single(self, output: torch.Tensor, input_tensor: torch.Tensor,
                              op: int = ReduceOp.SUM, timeout_ms: int = 0):
        lib, stream = self._enter()
        code, scale = self._reduction(op)
        count = int(output.numel())
        if count:
            _check(lib.tp_b200_nccl_reduce_scatter(_ptr(input_tensor), _ptr(output), count,
                                                   _dtype_code(output), code, self._device, self._comm))
            self._scale(output, scale)
        return self._work(stream)

    def reduce_scatter_single_coalesced(self, outputs: List[torch.Tensor], inputs: List[torch.Tensor],
                                        op: int = ReduceOp.SUM, timeout_ms: int = 0):
        """One reduce-scatter per (output, input) pair, issued as one NCCL
        group (tensorplay_mlu/distributed.py:391-407)."""
        lib, stream = self._enter()
        code, scale = self._reduction(op)
        _check(lib.tp_b200_nccl_group_start())
        for output, input_tensor in zip(outputs, inputs):
            count = int(output.numel())
            if count:
                _check(lib.tp_b200_nccl_reduce_scatter(_ptr(input_tensor), _ptr(output), count,
                                                       _dtype_code(output), code, self._device, self._comm))
        _check(lib.tp_b200_nccl_group_end())
        for output in outputs:
            self._scale(output, scale)
        return self._work(stream)

    def all_gather_single_coalesced(self, outputs: List[torch.Tensor], inputs: List[torch.Tensor],
                                    timeout_ms: int = 0):
        """One all-gather per (output, input) pair, issued as one NCCL group
        (tensorplay_mlu/distributed.py:328-340)."""
        lib, stream = self._enter()
        _check(lib.tp_b200_nccl_group_start())
        for output, input_tensor in zip(outputs, inputs):
            count = int(input_tensor.numel())
            if count:
                _check(lib.tp_b200_nccl_all_gather(_ptr(input_tensor), _ptr(output), count,
                                                   _dtype_code(input_tensor), self._device, self._comm))
        _check(lib.tp_b200_nccl_group_end())
        return self._work(stream)

    def allgather_coalesced(self, output_lists, input_tensors: List[torch.Tensor], timeout_ms: int = 0):
        """All-gather of each input into the per-rank lists
        (``output_lists[rank][index]``), issued as one NCCL group
        (tensorplay_mlu/distributed.py:342-363); each tensor's rank chunks
        go through one dense buffer, copied out once the group has run."""
        lib, stream = self._enter()
        staged = []
        _check(lib.tp_b200_nccl_group_start())
        for index, tensor in enumerate(input_tensors):
            count = int(tensor.numel())
            if not count:
                continue
            chunks = [rank_outputs[index] for rank_outputs in output_lists]
            flat = torch.empty((count * self._size,), dtype=tensor.dtype, device=tensor.device)
            _check(lib.tp_b200_nccl_all_gather(_ptr(_flat(tensor)), _ptr(flat), count, _dtype_code(tensor),
                                               self._device, self._comm))
            staged.append((flat, chunks))
        _check(lib.tp_b200_nccl_group_end())
        for flat, chunks in staged:
            self._scatter_from(flat, chunks)
        return self._work(stream)

    def gather(self, output_lists, input_tensors: List[torch.Tensor], root: int = 0, timeout_ms: int = 0):
        """Every rank's ``input_tensors[0]`` into ``output_lists[0][rank]`` on
        ``root``, over point-to-point sends (tensorplay_mlu/distributed.py:410-431)."""
        from . import ops

        lib, stream = self._enter()
        tensor = input_tensors[0]
        count = int(tensor.numel())
        dtype = _dtype_code(tensor)
        staged = []
        _check(lib.tp_b200_nccl_group_start())
        if self._rank == root:
            for peer in range(self._size):
                target = output_lists[0][peer]
                if peer == root:
                    if count:
                        ops.copy_(target, _flat(tensor).reshape(target.shape))
                elif count:
                    buf = target if target.is_contiguous() else torch.empty_like(target)
                    _check(lib.tp_b200_nccl_recv(_ptr(buf), count, dtype, peer, self._device, self._comm))
                    if buf is not target:
                        staged.append((target, buf))
        elif count:
            _check(lib.tp_b200_nccl_send(_ptr(_flat(tensor)), count, dtype, root, self._device, self._comm))
        _check(lib.tp_b200_nccl_group_end())
        for target, buf in staged:
            ops.copy_(target, buf)
        return self._work(stream)

    def gather_single(self, output: torch.Tensor, input_tensor: torch.Tensor, root: int = 0,
                      timeout_ms: int = 0):
        """Rank r's input into elements [r * n, (r + 1) * n) of ``output`` on
        ``root`` (tensorplay_mlu/distributed.py:433-452)."""
        from . import ops

        lib, stream = self._enter()
        count = int(input_tensor.numel())
        dtype = _dtype_code(input_tensor)
        if self._rank == root:
            flat_out = _flat(output)
            _check(lib.tp_b200_nccl_group_start())
            for peer in range(self._size):
                if peer != root and count:
                    _check(lib.tp_b200_nccl_recv(_ptr(flat_out.narrow(0, peer * count, count)), count, dtype,
                                                 peer, self._device, self._comm))
            _check(lib.tp_b200_nccl_group_end())
            if count:
                ops.copy_(flat_out.narrow(0, root * count, count), _flat(input_tensor))
            self._write_back(output, flat_out)
        elif count:
            _check(lib.tp_b200_nccl_group_start())
            _check(lib.tp_b200_nccl_send(_ptr(_flat(input_tensor)), count, dtype, root, self._device,
                                         self._comm))
            _check(lib.tp_b200_nccl_group_end())
        return self._work(stream)

    def scatter(self, recv_tensors: List[torch.Tensor], input_lists, root: int = 0, timeout_ms: int = 0):
        """``input_lists[0][r]`` on ``root`` into rank r's ``recv_tensors[0]``
        (tensorplay_mlu/distributed.py:454-470)."""
        from . import ops

        lib, stream = self._enter()
        output = recv_tensors[0]
        count = int(output.numel())
        dtype = _dtype_code(output)
        buf = output if output.is_contiguous() else torch.empty_like(output)
        _check(lib.tp_b200_nccl_group_start())
        if self._rank == root:
            for peer in range(self._size):
                if peer != root and count:
                    _check(lib.tp_b200_nccl_send(_ptr(_flat(input_lists[0][peer])), count, dtype, peer,
                                                 self._device, self._comm))
        elif count:
            _check(lib.tp_b200_nccl_recv(_ptr(buf), count, dtype, root, self._device, self._comm))
        _check(lib.tp_b200_nccl_group_end())
        if self._rank == root and count:
            ops.copy_(output, _flat(input_lists[0][root]).reshape(output.shape))
        elif buf is not output:
            ops.copy_(output, buf)
        return self._work(stream)

    def all_to_all_single(self, output: torch.Tensor, input_tensor: torch.Tensor,
                          output_split_sizes=None, input_split_sizes=None, timeout_ms: int = 0):
        from . import ops

        lib, stream = self._enter()
        dtype = _dtype_code(input_tensor)
        world, rank = self._size, self._rank
        flat_in, flat_out = _flat(input_tensor), _flat(output)
        if not output_split_sizes and not input_split_sizes:
            if world == 1:
                ops.copy_(flat_out, flat_in)
            elif flat_in.numel():
                _check(lib.tp_b200_nccl_all_to_all(_ptr(flat_in), _ptr(flat_out),
                                                   int(flat_in.numel()) // world, dtype, self._device,
                                                   self._comm))
            self._write_back(output, flat_out)
            return self._work(stream)
        in_counts = _element_counts(input_tensor, input_split_sizes, world)
        out_counts = _element_counts(output, output_split_sizes, world)
        in_off, out_off = _prefix_offsets(in_counts), _prefix_offsets(out_counts)
        if world > 1:
            _check(lib.tp_b200_nccl_group_start())
            for peer in range(world):
                if peer != rank and in_counts[peer]:
                    _check(lib.tp_b200_nccl_send(_ptr(flat_in.narrow(0, in_off[peer], in_counts[peer])),
                                                 in_counts[peer], dtype, peer, self._device, self._comm))
            for peer in range(world):
                if peer != rank and out_counts[peer]:
                    _check(lib.tp_b200_nccl_recv(_ptr(flat_out.narrow(0, out_off[peer], out_counts[peer])),
                                                 out_counts[peer], dtype, peer, self._device, self._comm))
            _check(lib.tp_b200_nccl_group_end())
        if in_counts[rank] and out_counts[rank]:
            ops.copy_(flat_out.narrow(0, out_off[rank], out_counts[rank]),
                      flat_in.narrow(0, in_off[rank], in_counts[rank]))
        self._write_back(output, flat_out)
        return self._work(stream)

    def alltoall(self, outputs: List[torch.Tensor], inputs: List[torch.Tensor], timeout_ms: int = 0):
        from . import ops

        lib, stream = self._enter()
        rank, world = self._rank, self._size
        if world > 1:
            _check(lib.tp_b200_nccl_group_start())
            for peer, tensor in enumerate(inputs):
                if tensor.numel() and peer != rank:
                    _check(lib.tp_b200_nccl_send(_ptr(tensor), int(tensor.numel()), _dtype_code(tensor),
                                                 peer, self._device, self._comm))
            for peer, tensor in enumerate(outputs):
                if tensor.numel() and peer != rank:
                    _check(lib.tp_b200_nccl_recv(_ptr(tensor), int(tensor.numel()), _dtype_code(tensor),
                                                 peer, self._device, self._comm))
            _check(lib.tp_b200_nccl_group_end())
        if inputs[rank].numel() and outputs[rank].numel():
            ops.copy_(outputs[rank], _flat(inputs[rank]).reshape(outputs[rank].shape))
        return self._work(stream)

    def _write_back(self, output: torch.Tensor, flat_out: torch.Tensor) -> None:
        from . import ops

        if flat_out.data_ptr() != output.data_ptr() or not output.is_contiguous():
            ops.copy_(output, flat_out.reshape(output.shape))

    def send(self, tensors: List[torch.Tensor], dst: int, tag: int = 0):
        lib, stream = self._enter()
        tensor = tensors[0]
        if tensor.numel():
            _check(lib.tp_b200_nccl_send(_ptr(tensor), int(tensor.numel()), _dtype_code(tensor), dst,
                                         self._device, self._comm))
        return self._work(stream)

    def recv(self, tensors: List[torch.Tensor], src: int, tag: int = 0):
        lib, stream = self._enter()
        tensor = tensors[0]
        if tensor.numel():
            _check(lib.tp_b200_nccl_recv(_ptr(tensor), int(tensor.numel()), _dtype_code(tensor), src,
                                         self._device, self._comm))
        return self._work(stream)

    def recv_anysource(self, tensors, tag: int = 0):
        raise RuntimeError("receiving from any source is unavailable for NCCL")

    def barrier(self, timeout_ms: int = 0):
        lib, stream = self._enter()
        if self._barrier_flag is None:
            from . import ops

            self._barrier_flag = ops.zero_(torch.empty(1, dtype=torch.float32,
                                                       device=f"cuda:{self._device}"))
        _check(lib.tp_b200_nccl_all_reduce(_ptr(self._barrier_flag), _ptr(self._barrier_flag), 1,
                                           N.DTYPE_CODES[torch.float32], _SUM_CODE, self._device,
                                           self._comm))
        return self._work(stream)

    def monitored_barrier(self, timeout_ms: int = 0, wait_all_ranks: bool = False):
        raise RuntimeError("monitored_barrier is unavailable for NCCL")


def _store_get(store, key: str, timeout_s: float):
    """``store.get(key)`` bounded by ``timeout_s`` (TensorPlay's store takes a
    timeout argument; a torch store is polled with ``check``)."""
    try:
        return store.get(key, timeout=timeout_s)
    except TypeError:
        pass
    deadline = time.monotonic() + timeout_s
    while True:
        try:
            if store.check([key]):
                return store.get(key)
        except Exception:
            pass
        if time.monotonic() > deadline:
            raise TimeoutError(f"rendezvous key {key!r} not published within {timeout_s} s "
                               "(rank 0 did not create the communicator)")
        time.sleep(0.01)


def _prefix_offsets(sizes):
    offsets, total = [], 0
    for size in sizes:
        offsets.append(total)
        total += int(size)
    return offsets


def _element_counts(tensor, split_sizes, world: int):
    """Per-peer element counts for ``all_to_all`` split sizes (which count
    leading-dimension rows, tensorplay_mlu/distributed.py:607-620)."""
    dim0 = int(tensor.shape[0]) if tensor.dim() > 0 else 1
    row = int(tensor.numel()) // dim0 if dim0 else 0
    if split_sizes:
        return [int(s) * row for s in split_sizes]
    return [(dim0 // world) * row] * world


def is_available() -> bool:
    try:
        from . import is_loaded, runtime

        return is_loaded() and runtime.device_count() > 0
    except Exception:
        return False


def create(store, rank: int, size: int, device: Optional[int] = None, group_name: str = "default",
           timeout_s: float = 300.0, max_ctas: int = 0) -> ProcessGroupB200:
    """A ready process group (communicator created); `max_ctas` bounds the
    SMs its collectives' kernels occupy (0: NCCL's choice)."""
    pg = ProcessGroupB200(store, rank, size, device, group_name, timeout_s, max_ctas)
    pg.ensure()
    return pg


def create_process_group(pg):
    """TensorPlay device-backend factory (tensorplay_mlu/distributed.py:628-632)."""
    from tensorplay.distributed import distributed_core as dc  # type: ignore

    impl = ProcessGroupB200(dc._current_store(), pg.group_rank(dc._global_rank()), pg.size(),
                            group_name=pg.group_name, timeout_s=pg._timeout_s)
    impl.ensure()
    return impl


def register() -> None:
    """Register ``nccl_b200`` with ``tensorplay.distributed`` when TensorPlay is
    importable (tensorplay_mlu/distributed.py:635-648); idempotent."""
    try:
        from tensorplay.distributed import distributed_core as dc  # type: ignore
    except Exception:
        return
    from . import BACKEND_NAME, DEVICE_NAME

    if BACKEND_NAME not in dc.Backend.backend_list:
        dc.Backend.register_backend(BACKEND_NAME, create_process_group, devices=[DEVICE_NAME],
                                    _backend_type=BACKEND_NAME)
    dc.register_device_backend(BACKEND_NAME, create_process_group)
