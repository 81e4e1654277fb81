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
    # point to point: rank 0 sends then receives, rank 1 the mirror image
    mine = ops.to_device(torch.tensor([100.0 * (rank + 1), 100.0 * (rank + 1) + 1], dtype=torch.bfloat16))
    theirs = torch.zeros(2, dtype=torch.bfloat16, device="cuda")
    peer = 1 - rank
    if rank == 0:
        pg.send([mine], peer).wait()
        pg.recv([theirs], peer).wait()
    else:
        pg.recv([theirs], peer).wait()
        pg.send([mine], peer).wait()
    out["p2p"] = ops.to_host(theirs).float().tolist()
    # gather / gather_single / scatter to and from rank 1, and the coalesced forms
    g_in = ops.to_device(torch.tensor([10.0 + rank, 20.0 + rank]))
    g_out = [torch.zeros(2, device="cuda") for _ in range(WORLD)]
    pg.gather([g_out], [g_in], 1).wait(timeout=60)
    out["gather_list"] = [ops.to_host(t).tolist() for t in g_out]
    g_flat = torch.zeros(2 * WORLD, device="cuda")
    pg.gather_single(g_flat, g_in, 1).wait()
    out["gather_single"] = ops.to_host(g_flat).tolist()
    s_in = [ops.to_device(torch.tensor([100.0 * r + rank])) for r in range(WORLD)]
    s_out = torch.zeros(1, device="cuda")
    pg.scatter([s_out], [s_in], 1).wait()
    out["scatter"] = ops.to_host(s_out).tolist()
    c_in = [ops.to_device(torch.tensor([1.0 + rank])), ops.to_device(torch.tensor([5.0, 6.0]) * (rank + 1))]
    c_out = [[torch.zeros(1, device="cuda"), torch.zeros(2, device="cuda")] for _ in range(WORLD)]
    pg.allgather_coalesced(c_out, c_in).wait()
    out["allgather_coalesced"] = [[ops.to_host(t).tolist() for t in r] for r in c_out]
    singles = [torch.zeros(WORLD, device="cuda"), torch.zeros(2 * WORLD, device="cuda")]
    pg.all_gather_single_coalesced(singles, c_in).wait()
    out["all_gather_single_coalesced"] = [ops.to_host(t).tolist() for t in singles]
    rs_in = [ops.to_device(torch.arange(WORLD, dtype=torch.float32) + rank),
             ops.to_device(torch.arange(2 * WORLD, dtype=torch.float32) * (rank + 1))]
    rs_out = [torch.zeros(1, device="cuda"), torch.zeros(2, device="cuda")]
    pg.reduce_scatter_single_coalesced(rs_out, rs_in, ReduceOp.SUM).wait()
    out["reduce_scatter_single_coalesced"] = [ops.to_host(t).tolist() for t in rs_out]
    # two DP steps of a small MLP, in both schedules of the last bucket, with
    # the products beside an exchange in two and three (ragged) row slices,
    # and in the other backward order
    for key, overlap, split, order in (("params_overlap0", False, 1, "w1_first"),
                                       ("params_overlap1", True, 1, "w1_first"),
                                       ("params_split2", True, 2, "w1_first"),
                                       ("params_split3", False, 3, "w1_first"),
                                       ("params_w2first0", False, 1, "w2_first"),
                                       ("params_w2first1", True, 1, "w2_first")):
        cfg = MLPConfig(d_in=256, d_hidden=512, batch=64, lr=0.1, dw1_slices=2, overlap_next_step=overlap,
                        beside_slices=split, dp_order=order)
        params = init_params_host(cfg, seed=0)
        model = DataParallelMLP(cfg, device=rank, pg=pg, host_params=params)
        xh, th = make_batch_host(cfg, seed=rank)
        for _ in range(2):
            model.step(ops.to_device(xh), ops.to_device(th))
        model.flush()
        torch.cuda.synchronize()
        out[key] = [ops.to_host(p) for p in model.params()]
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
    assert r0["p2p"] == [200.0, 201.0] and r1["p2p"] == [100.0, 101.0]
    assert r0["all_to_all"] == [0.0, 10.0] and r1["all_to_all"] == [1.0, 11.0]
    # tensorplay_mlu/distributed.py:328-470
    assert r1["gather_list"] == [[10.0, 20.0], [11.0, 21.0]]
    assert r1["gather_single"] == [10.0, 20.0, 11.0, 21.0]
    assert r0["scatter"] == [1.0] and r1["scatter"] == [101.0]
    for r in (r0, r1):
        assert r["allgather_coalesced"] == [[[1.0], [5.0, 6.0]], [[2.0], [10.0, 12.0]]]
        assert r["all_gather_single_coalesced"] == [[1.0, 2.0], [5.0, 6.0, 10.0, 12.0]]
    # rank r gets elements [r] of (arange(2) + 0) + (arange(2) + 1), and
    # [2r, 2r + 2) of arange(4) * 1 + arange(4) * 2
    assert r0["reduce_scatter_single_coalesced"] == [[1.0], [0.0, 3.0]]
    assert r1["reduce_scatter_single_coalesced"] == [[3.0], [6.0, 9.0]]
    # Both ranks hold identical parameters, equal to the single-GPU steps on
    # the concatenated batch, in every schedule (bit for bit across them: a
    # row slice of a product has the bits of the same rows of the whole).
    schedules = ("params_overlap0", "params_overlap1", "params_split2", "params_split3", "params_w2first0",
                 "params_w2first1")
    for key in schedules:
        for a, b in zip(r0[key], r1[key]):
            assert torch.equal(a, b)
    for key in schedules[1:]:
        for a, b in zip(r0["params_overlap0"], r0[key]):
            assert torch.equal(a, b), key
    r0["params"] = r0["params_overlap0"]
    from tensorplay_mlu_b200.train import DataParallelMLP, MLPConfig, init_params_host, make_batch_host

    ops = backend.ops
    cfg = MLPConfig(d_in=256, d_hidden=512, batch=64, lr=0.1)
    params = init_params_host(cfg, seed=0)
    x0, t0 = make_batch_host(cfg, seed=0)
    x1, t1 = make_batch_host(cfg, seed=1)
    big = MLPConfig(d_in=256, d_hidden=512, batch=128, lr=0.1)
    single = DataParallelMLP(big, device=0, host_params=params)
    for _ in range(2):
        single.step(ops.to_device(torch.cat([x0, x1])), ops.to_device(torch.cat([t0, t1])))
    for got, want in zip(r0["params"], single.params()):
        want = ops.to_host(want).float()
        err = (got.float() - want).abs().max().item()
        assert err <= 1e-2 * max(want.abs().max().item(), 1.0), err
