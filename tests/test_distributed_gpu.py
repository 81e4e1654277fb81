"""The nccl_b200 process group on one GPU rank (tensorplay-mlu
tests/test_mlu_distributed.py:57-157, with NCCL in place of CNCL): every
collective against its hand-computed single-rank result, through the process
group object, the C ABI and NCCL.  The rendezvous goes through a real TCP
store."""

from __future__ import annotations

import contextlib
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as sock:
        sock.bind(("127.0.0.1", 0))
        return sock.getsockname()[1]


@contextlib.contextmanager
def single_rank(backend):
    from tensorplay_mlu_b200 import distributed as D

    store = torch.distributed.TCPStore("127.0.0.1", _free_port(), 1, True)
    pg = D.create(store, 0, 1, device=0, timeout_s=60)
    try:
        yield pg
    finally:
        pg.destroy()


def t(backend, values, dtype=torch.float32):
    return backend.ops.to_device(torch.tensor(values, dtype=dtype))


def host(backend, x):
    torch.cuda.synchronize()
    return backend.ops.to_host(x).tolist()


def test_backend_names_are_distinct_from_cuda(backend):
    from tensorplay_mlu_b200 import distributed as D

    assert backend.BACKEND_NAME != "nccl" and backend.DEVICE_NAME not in ("cuda", "mlu")
    assert D.is_available()


def test_all_reduce_sum_avg_max_bf16(backend):
    from tensorplay_mlu_b200.distributed import ReduceOp

    with single_rank(backend) as pg:
        x = t(backend, [1.0, 2.0, 3.0])
        pg.allreduce([x], ReduceOp.SUM).wait()
        assert host(backend, x) == [1.0, 2.0, 3.0]
        x = t(backend, [2.0, 4.0])
        pg.allreduce([x], ReduceOp.AVG).wait()
        assert host(backend, x) == [2.0, 4.0]
        x = t(backend, [1.5, 2.5], torch.bfloat16)
        pg.allreduce([x], ReduceOp.SUM).wait()
        assert host(backend, x) == [1.5, 2.5]
        x = t(backend, [1.0])
        pg.allreduce([x], ReduceOp.MAX).wait()
        pg.barrier().wait()
        assert host(backend, x) == [1.0]


def test_all_reduce_coalesced(backend):
    with single_rank(backend) as pg:
        a, b = t(backend, [1.0, 2.0]), t(backend, [3.0])
        pg.allreduce_coalesced([a, b], 0).wait()
        assert host(backend, a) == [1.0, 2.0] and host(backend, b) == [3.0]


def test_broadcast_reduce(backend):
    with single_rank(backend) as pg:
        x = t(backend, [5.0, 6.0])
        pg.broadcast([x], 0).wait()
        assert host(backend, x) == [5.0, 6.0]
        y = t(backend, [7.0, 8.0])
        pg.reduce([y], 0, 0).wait()
        assert host(backend, y) == [7.0, 8.0]


def test_all_gather_reduce_scatter(backend):
    with single_rank(backend) as pg:
        send = t(backend, [1.0, 2.0])
        outputs = [t(backend, [0.0, 0.0])]
        pg.allgather([outputs], [send]).wait()
        assert host(backend, outputs[0]) == [1.0, 2.0]
        out = t(backend, [0.0, 0.0])
        pg.all_gather_single(out, send).wait()
        assert host(backend, out) == [1.0, 2.0]
        inputs = [t(backend, [1.0, 2.0])]
        output = t(backend, [0.0, 0.0])
        pg.reduce_scatter([output], [inputs], 0).wait()
        assert host(backend, output) == [1.0, 2.0]


def test_all_to_all(backend):
    with single_rank(backend) as pg:
        send, recv = t(backend, [1.0, 2.0, 3.0, 4.0]), t(backend, [0.0] * 4)
        pg.all_to_all_single(recv, send).wait()
        assert host(backend, recv) == [1.0, 2.0, 3.0, 4.0]
        send = t(backend, [[1.0, 2.0], [3.0, 4.0]])
        recv = t(backend, [[0.0, 0.0], [0.0, 0.0]])
        pg.all_to_all_single(recv, send, [2], [2]).wait()
        assert host(backend, recv) == [[1.0, 2.0], [3.0, 4.0]]
        sends, recvs = [t(backend, [1.0, 2.0])], [t(backend, [0.0, 0.0])]
        pg.alltoall(recvs, sends).wait()
        assert host(backend, recvs[0]) == [1.0, 2.0]


def test_large_bf16_all_reduce_is_identity_on_one_rank(backend):
    from tensorplay_mlu_b200.distributed import ReduceOp

    with single_rank(backend) as pg:
        g = torch.Generator().manual_seed(0)
        h = torch.randn(1 << 22, generator=g).bfloat16()
        x = backend.ops.to_device(h)
        work = pg.allreduce([x], ReduceOp.SUM)
        work.synchronize()
        assert work.is_completed()
        assert torch.equal(backend.ops.to_host(x), h)


def test_gather_scatter_and_coalesced_forms(backend):
    # tensorplay_mlu/distributed.py:328-470: on one rank every form is the identity.
    from tensorplay_mlu_b200.distributed import ReduceOp

    with single_rank(backend) as pg:
        x = t(backend, [1.0, 2.0, 3.0])
        out = [backend.ops.zero_(torch.empty(3, device="cuda"))]
        pg.gather([out], [x], 0).wait()
        assert host(backend, out[0]) == [1.0, 2.0, 3.0]
        flat = backend.ops.zero_(torch.empty(3, device="cuda"))
        pg.gather_single(flat, x, 0).wait()
        assert host(backend, flat) == [1.0, 2.0, 3.0]
        recv = backend.ops.zero_(torch.empty(3, device="cuda"))
        pg.scatter([recv], [[x]], 0).wait()
        assert host(backend, recv) == [1.0, 2.0, 3.0]
        ys = [t(backend, [5.0]), t(backend, [6.0, 7.0], torch.bfloat16)]
        outs = [[backend.ops.zero_(torch.empty(1, device="cuda")),
                 backend.ops.zero_(torch.empty(2, dtype=torch.bfloat16, device="cuda"))]]
        pg.allgather_coalesced(outs, ys).wait()
        assert host(backend, outs[0][0]) == [5.0] and host(backend, outs[0][1]) == [6.0, 7.0]
        singles = [backend.ops.zero_(torch.empty(1, device="cuda")),
                   backend.ops.zero_(torch.empty(2, dtype=torch.bfloat16, device="cuda"))]
        pg.all_gather_single_coalesced(singles, ys).wait()
        assert host(backend, singles[0]) == [5.0] and host(backend, singles[1]) == [6.0, 7.0]
        reds = [backend.ops.zero_(torch.empty(1, device="cuda")),
                backend.ops.zero_(torch.empty(2, dtype=torch.bfloat16, device="cuda"))]
        pg.reduce_scatter_single_coalesced(reds, ys, ReduceOp.AVG).wait(timeout=30)
        assert host(backend, reds[0]) == [5.0] and host(backend, reds[1]) == [6.0, 7.0]
