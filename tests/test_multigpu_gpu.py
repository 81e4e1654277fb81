"""Two ranks on two GPUs (one process per GPU, NCCL through the nccl_b200
process group): collectives against hand-computed results, and one
data-parallel MLP step against the single-GPU step on the concatenated batch
(the DP step averages per-rank mean-loss gradients, which equals the gradient
of the global mean loss).  Needs at least two visible B200s."""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

WORLD = 2


def _free_port() -> int:
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as sock:
        sock.bind(("127.0.0.1", 0))
        return sock.getsockname()[1]


def _worker(rank: int, port: int, result_dir: str) -> None:
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    import tensorplay_mlu_b200 as tpb
    from tensorplay_mlu_b200 import distributed as D
    from tensorplay_mlu_b200.distributed import ReduceOp
    from tensorplay_mlu_b200.train import DataParallelMLP, MLPConfig, init_params_host, make_batch_host

    tpb.load()
    assert tpb.allocator_installed()
    torch.cuda.set_device(rank)
    ops = tpb.ops
    store = torch.distributed.TCPStore("127.0.0.1", port, WORLD, rank == 0, timeout=__import__("datetime").timedelta(seconds=60))
    pg = D.create(store, rank, WORLD, device=rank, timeout_s=60)
    out = {}
    # all_reduce SUM / AVG / MAX
    x = ops.to_device(torch.tensor([1.0 + rank, 10.0 * (rank + 1)]))
    pg.allreduce([x], ReduceOp.SUM).wait()
    out["sum"] = ops.to_host(x).tolist()
    x = ops.to_device(torch.tensor([2.0 + 2 * rank]))
    pg.allreduce([x], ReduceOp.AVG).wait()
    out["avg"] = ops.to_host(x).tolist()
    x = ops.to_device(torch.tensor([float(rank)], dtype=torch.bfloat16))
    pg.allreduce([x], ReduceOp.MAX).wait()
    out["max"] = ops.to_host(x).float().tolist()
    # all_gather / reduce_scatter / all_to_all / broadcast
    send = ops.to_device(torch.tensor([float(rank), float(rank) + 0.5]))
    gathered = torch.empty(4, device="cuda")
    pg.all_gather_single(gathered, send).wait()
    out["gather"] = ops.to_host(gathered).tolist()
    inp = ops.to_device(torch.arange(4, dtype=torch.float32) + 100 * rank)
    red = torch.empty(2, device="cuda")
    pg.reduce_scatter_single(red, inp, ReduceOp.SUM).wait()
    out["reduce_scatter"] = ops.to_host(red).tolist()
    a2a_in = ops.to_device(torch.tensor([10.0 * rank, 10.0 * rank + 1]))
    a2a_out = torch.empty(2, device="cuda")
    pg.all_to_all_single(a2a_out, a2a_in).wait()
    out["all_to_all"] = ops.to_host(a2a_out).tolist()
    b = ops.to_device(torch.tensor([float(rank + 7)]))
    pg.broadcast([b], 1).wait()
    out["broadcast"] = ops.to_host(b).tolist()
    # one DP step of a small MLP
    cfg = MLPConfig(d_in=256, d_hidden=512, batch=64, lr=0.1)
    params = init_params_host(cfg, seed=0)
    model = DataParallelMLP(cfg, device=rank, pg=pg, host_params=params)
    xh, th = make_batch_host(cfg, seed=rank)
    model.step(ops.to_device(xh), ops.to_device(th))
    torch.cuda.synchronize()
    out["params"] = [ops.to_host(p) for p in model.params()]
    pg.barrier().wait()
    torch.cuda.synchronize()
    pg.destroy()
    torch.save(out, os.path.join(result_dir, f"rank{rank}.pt"))


def test_two_rank_collectives_and_dp_step(backend, tmp_path):
    if torch.cuda.device_count() < WORLD:
        pytest.skip("needs two GPUs")
    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_worker, args=(r, port, str(tmp_path))) for r in range(WORLD)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    r0 = torch.load(tmp_path / "rank0.pt")
    r1 = torch.load(tmp_path / "rank1.pt")
    for r in (r0, r1):
        assert r["sum"] == [3.0, 30.0]
        assert r["avg"] == [3.0]
        assert r["max"] == [1.0]
        assert r["gather"] == [0.0, 0.5, 1.0, 1.5]
        assert r["broadcast"] == [8.0]
    assert r0["reduce_scatter"] == [100.0, 102.0] and r1["reduce_scatter"] == [104.0, 106.0]
    assert r0["all_to_all"] == [0.0, 10.0] and r1["all_to_all"] == [1.0, 11.0]
    # Both ranks hold identical parameters, equal to the single-GPU step on
    # the concatenated batch.
    for a, b in zip(r0["params"], r1["params"]):
        assert torch.equal(a, b)
    from tensorplay_mlu_b200.train import DataParallelMLP, MLPConfig, init_params_host, make_batch_host

    ops = backend.ops
    cfg = MLPConfig(d_in=256, d_hidden=512, batch=64, lr=0.1)
    params = init_params_host(cfg, seed=0)
    x0, t0 = make_batch_host(cfg, seed=0)
    x1, t1 = make_batch_host(cfg, seed=1)
    big = MLPConfig(d_in=256, d_hidden=512, batch=128, lr=0.1)
    single = DataParallelMLP(big, device=0, host_params=params)
    single.step(ops.to_device(torch.cat([x0, x1])), ops.to_device(torch.cat([t0, t1])))
    for got, want in zip(r0["params"], single.params()):
        want = ops.to_host(want).float()
        err = (got.float() - want).abs().max().item()
        assert err <= 1e-2 * max(want.abs().max().item(), 1.0), err
