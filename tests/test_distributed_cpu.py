"""The multi-rank host logic on CPU (gloo, world size 2, no GPU): the NCCL
rendezvous of the process group through the job store (rank 0 publishes the
communicator id, the others read it -- tensorplay_mlu/distributed.py:169-197),
the bench's host-side barrier / max-over-ranks, and failure detection when a
rank never joins (a store timeout, not a hang).  The native NCCL entry points
are replaced by a recording fake, so nothing touches a GPU."""

from __future__ import annotations

import ctypes
import os
import socket
import sys
import time

import pytest
import torch
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as sock:
        sock.bind(("127.0.0.1", 0))
        return sock.getsockname()[1]


class FakeNccl:
    """The tp_b200_nccl_* entry points the rendezvous uses, recording what they see."""

    ID_BYTES = 128

    def __init__(self, rank):
        self.rank = rank
        self.seen_id = None
        self.init_args = None

    def tp_b200_nccl_unique_id_bytes(self):
        return self.ID_BYTES

    def tp_b200_nccl_get_unique_id(self, buf):
        ctypes.memmove(buf, bytes((i * 7 + 3) % 256 for i in range(self.ID_BYTES)), self.ID_BYTES)
        return 0

    def tp_b200_nccl_comm_init_ctas(self, rank, nranks, dev, buf, timeout_ms, min_ctas, max_ctas, comm_ref):
        self.seen_id = bytes(buf.raw[: self.ID_BYTES])
        self.init_args = (rank, nranks, dev, timeout_ms, max_ctas)
        return 0

    def tp_b200_nccl_last_error(self):
        return b""


def _worker(rank: int, port: int, out_dir: str) -> None:
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE="2")
    import bench
    from tensorplay_mlu_b200 import _native
    from tensorplay_mlu_b200 import distributed as D

    fake = FakeNccl(rank)
    _native.lib = lambda: fake  # the rendezvous goes through the fake entry points
    host = bench.HostGroup(rank, 2)
    got_max = host.max(float(rank) + 0.5)
    host.barrier()
    pg = D.ProcessGroupB200(bench._PrefixStore("nccl_b200", host.store), rank, 2, device=rank,
                            group_name="g", timeout_s=30, max_ctas=16)
    pg.ensure()
    host.barrier()
    host.close()
    torch.save({"max": got_max, "id": fake.seen_id, "args": fake.init_args},
               os.path.join(out_dir, f"r{rank}.pt"))


def test_rendezvous_and_host_group_with_two_gloo_ranks(tmp_path):
    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_worker, args=(r, port, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert [p.exitcode for p in procs] == [0, 0]
    r0, r1 = torch.load(tmp_path / "r0.pt"), torch.load(tmp_path / "r1.pt")
    assert r0["max"] == r1["max"] == 1.5
    assert r0["id"] == r1["id"] and len(r0["id"]) == FakeNccl.ID_BYTES
    assert r0["args"] == (0, 2, 0, 30000, 16) and r1["args"] == (1, 2, 1, 30000, 16)


def test_rank_without_rendezvous_times_out():
    """Rank 1 of a group whose rank 0 never creates the communicator gets a
    TimeoutError after the group timeout instead of waiting for ever."""
    from tensorplay_mlu_b200 import _native
    from tensorplay_mlu_b200 import distributed as D

    store = torch.distributed.TCPStore("127.0.0.1", _free_port(), 1, True)
    fake = FakeNccl(1)
    real = _native.lib
    _native.lib = lambda: fake
    try:
        pg = D.ProcessGroupB200(store, 1, 2, device=0, group_name="lonely", timeout_s=1.0)
        t0 = time.monotonic()
        with pytest.raises(TimeoutError):
            pg.ensure()
        assert time.monotonic() - t0 < 10
        assert fake.init_args is None  # never reached communicator creation
    finally:
        _native.lib = real


def test_native_errors_surface_as_exceptions():
    from tensorplay_mlu_b200 import _native
    from tensorplay_mlu_b200 import distributed as D

    class Failing(FakeNccl):
        def tp_b200_nccl_comm_init_ctas(self, *args):
            return -1

        def tp_b200_nccl_last_error(self):
            return b"NCCL: communicator of rank 0/2 not ready after 1000 ms (a peer did not join)"

    store = torch.distributed.TCPStore("127.0.0.1", _free_port(), 1, True)
    real = _native.lib
    _native.lib = lambda: Failing(0)
    try:
        pg = D.ProcessGroupB200(store, 0, 2, device=0, group_name="failing", timeout_s=1.0)
        with pytest.raises(RuntimeError, match="did not join"):
            pg.ensure()
    finally:
        _native.lib = real


class _NeverDone:
    """A collective's completion event that never fires (a stuck peer)."""

    def query(self):
        return False


class _Group:
    def __init__(self, error_after=None):
        self.aborted = False
        self.checks = 0
        self.error_after = error_after

    def check(self):
        self.checks += 1
        if self.error_after is not None and self.checks >= self.error_after:
            raise RuntimeError("NCCL asynchronous error: remote process exited")

    def abort(self):
        self.aborted = True


def test_work_wait_with_a_timeout_aborts_a_stuck_collective():
    import datetime

    from tensorplay_mlu_b200.distributed import _Work

    group = _Group()
    work = _Work(0, None, group=group, event=_NeverDone())
    start = time.monotonic()
    with pytest.raises(TimeoutError):
        work.wait(timeout=datetime.timedelta(milliseconds=200))
    assert 0.2 <= time.monotonic() - start < 5.0
    assert group.aborted and group.checks > 0
    assert not work.is_completed()


def test_work_wait_surfaces_an_asynchronous_communicator_error():
    from tensorplay_mlu_b200.distributed import _Work

    group = _Group(error_after=3)
    work = _Work(0, None, group=group, event=_NeverDone())
    with pytest.raises(RuntimeError, match="asynchronous error"):
        work.wait(timeout=30.0)
    assert not group.aborted


def test_work_wait_returns_once_the_collective_completes():
    from tensorplay_mlu_b200.distributed import _Work

    class DoneAfter:
        def __init__(self, n):
            self.n = n

        def query(self):
            self.n -= 1
            return self.n <= 0

    finished = []
    work = _Work(0, None, done=lambda: finished.append(1), group=_Group(), event=DoneAfter(5))
    assert work.wait(timeout=5.0) and work.is_completed() and finished == [1]


def test_forms_nccl_does_not_offer_raise_before_touching_the_communicator():
    # tensorplay_mlu/distributed.py:578-591: receiving from any source and the
    # monitored barrier are refused with a RuntimeError, not an AttributeError.
    from tensorplay_mlu_b200 import distributed as D

    store = torch.distributed.TCPStore("127.0.0.1", _free_port(), 1, True)
    pg = D.ProcessGroupB200(store, 0, 2, device=0, group_name="refusals", timeout_s=1.0)
    with pytest.raises(RuntimeError, match="any source"):
        pg.recv_anysource([torch.zeros(1)])
    with pytest.raises(RuntimeError, match="monitored_barrier"):
        pg.monitored_barrier()


def test_set_timeout_bounds_the_rendezvous():
    # The provider's set_timeout (tensorplay_mlu/distributed.py:206) takes
    # milliseconds and bounds the wait for the communicator id.
    from tensorplay_mlu_b200 import _native
    from tensorplay_mlu_b200 import distributed as D

    store = torch.distributed.TCPStore("127.0.0.1", _free_port(), 1, True)
    fake = FakeNccl(1)
    real = _native.lib
    _native.lib = lambda: fake
    try:
        pg = D.ProcessGroupB200(store, 1, 2, device=0, group_name="short", timeout_s=60.0)
        pg.set_timeout(300)
        t0 = time.monotonic()
        with pytest.raises(TimeoutError):
            pg.ensure()
        assert time.monotonic() - t0 < 10
    finally:
        _native.lib = real
