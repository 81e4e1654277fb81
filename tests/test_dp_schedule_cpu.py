"""The data-parallel step's schedule on CPU (gloo, world size 2, no GPU).

`DataParallelMLP.step` is run as written -- bucket order, the row slices of
bucket B and of the products beside an exchange, deferred updates and
`flush()`, the SM reserve around the products beside a collective -- with
its device kernels replaced by CPU stand-ins (test-only fakes: a float32
matmul rounded to the step's dtype, gelu, the MSE pass, a column sum, the
SGD add) and its process group by gloo all-reduces.  Checked, for every
combination of backward order, update schedule, bucket-B slices and
beside-exchange slices:

* both ranks end with identical parameters, bit for bit equal across the
  schedules (the same sums in every schedule);
* they match the single-process step on the concatenated batch (the DP step
  averages per-rank mean-loss gradients: the gradient of the global mean);
* each step all-reduces bucket A once and bucket B once per slice, covering
  the flat gradient buffer exactly once;
* every SM reserve set for a product beside a collective is lifted again.

The kernels themselves are checked against the oracle on the GPU; this file
covers the host-side schedule around them."""

from __future__ import annotations

import contextlib
import itertools
import os
import socket
import sys
import types

import pytest
import torch
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

SMALL = dict(d_in=64, d_hidden=192, batch=48, lr=0.05)
SCHEDULES = list(itertools.product(("w1_first", "w2_first"), (False, True), (1, 2, 3), (1, 2, 3)))


def _free_port() -> int:
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as sock:
        sock.bind(("127.0.0.1", 0))
        return sock.getsockname()[1]


# ----------------------------------------------------------------- fakes

def _mm(a, b, dtype):
    return (a.float() @ b.float()).to(dtype)


def _gelu(x):
    return torch.nn.functional.gelu(x)


def _gelu_backward(d, x):
    cdf = 0.5 * (1.0 + torch.erf(x * 0.7071067811865476))
    pdf = torch.exp(-0.5 * x * x) * 0.3989422804014327
    return d * (cdf + x * pdf)


class FakeLib:
    """The tp_b200_* entry points the step calls, on CPU tensors (N.describe
    is the identity under these fakes), recording the SM-limit calls."""

    def __init__(self):
        self.sm_limits = []

    def tp_b200_reduce(self, op, out, x, mask, stream):
        assert mask == 1  # the bias gradients: a sum over dim 0
        out.copy_(x.float().sum(0, keepdim=True).to(out.dtype))
        return 0

    def tp_b200_gemm_epilogue(self, epi, out, aux, a, b, c, alpha, beta, flags, stream):
        from tensorplay_mlu_b200 import _native as N

        if epi == N.EPI_GELU:
            pre = a.float() @ b.float() + (c.float() if c is not None else 0.0)
            aux.copy_(pre.to(aux.dtype))
            out.copy_(_gelu(aux.float()).to(out.dtype))
        else:
            d = _mm(a, b, out.dtype)
            out.copy_(_gelu_backward(d.float(), aux.float()).to(out.dtype))
        return 0

    def tp_b200_mse_loss(self, loss, grad, out, target, scale, stream):
        diff = (out.float() - target.float()).to(out.dtype)
        grad.copy_((diff.float() * scale).to(grad.dtype))
        loss.copy_((diff.float() ** 2).mean().to(loss.dtype))
        return 0

    def tp_b200_set_gemm_sm_limit(self, dev, sms):
        self.sm_limits.append(sms)
        return 0

    def tp_b200_set_gemm_tile_order(self, dev, dynamic):
        return 0


class _FakeStream:
    def wait_event(self, event):
        pass


class _FakeEvent:
    def __init__(self, *args, **kwargs):
        pass

    def record(self, stream=None):
        pass


def _fake_cuda():
    return types.SimpleNamespace(
        Stream=lambda device=None, priority=0: _FakeStream(),
        Event=_FakeEvent,
        stream=lambda s: contextlib.nullcontext(),
        get_device_properties=lambda dev: types.SimpleNamespace(multi_processor_count=148),
        synchronize=lambda *a: None,
    )


class _TorchOnCpu:
    """`torch` as train.py sees it under the fakes: CUDA devices, streams and
    events become CPU / no-ops; everything else is torch."""

    def __init__(self):
        self.cuda = _fake_cuda()

    def __getattr__(self, name):
        return getattr(torch, name)

    @staticmethod
    def device(*args, **kwargs):
        return torch.device("cpu")

    @staticmethod
    def empty(*args, device=None, **kwargs):
        return torch.empty(*args, **kwargs)


class GlooGroup:
    """The process group the step uses (size, allreduce) over gloo, recording
    each all-reduce's span of the flat gradient buffer."""

    def __init__(self, world, grad_flat_of):
        self.world = world
        self.grad_flat_of = grad_flat_of
        self.spans = []

    def size(self):
        return self.world

    def allreduce(self, tensors, op=0):
        (t,) = tensors
        base = self.grad_flat_of()
        offset = (t.data_ptr() - base.data_ptr()) // t.element_size()
        self.spans.append((offset, t.numel()))
        torch.distributed.all_reduce(t)
        return types.SimpleNamespace(wait=lambda *a, **k: True)


@contextlib.contextmanager
def cpu_step():
    """Install the fakes into train.py's view of the library (restored after)."""
    from tensorplay_mlu_b200 import _native as N
    from tensorplay_mlu_b200 import ops
    from tensorplay_mlu_b200 import train

    lib = FakeLib()
    saved = {
        (N, "lib"): N.lib, (N, "describe"): N.describe, (N, "stream_of"): N.stream_of,
        (ops, "copy_"): ops.copy_, (ops, "to_device"): ops.to_device, (ops, "_gemm"): ops._gemm,
        (ops, "linear"): ops.linear, (ops, "add__Tensor"): ops.add__Tensor, (train, "torch"): train.torch,
    }

    def add_(p, g, alpha=1):
        p.copy_((p.float() + alpha * g.float()).to(p.dtype))
        return p

    N.lib = lambda: lib
    N.describe = lambda t: t
    N.stream_of = lambda dev: None
    ops.copy_ = lambda dst, src: dst.copy_(src)
    ops.to_device = lambda t, dev=None: t.clone()
    ops._gemm = lambda out, a, b, c=None, alpha=1.0, beta=0.0: out.copy_(_mm(a, b, out.dtype))
    ops.linear = lambda a, w, b=None: (a.float() @ w.float().t() + (b.float() if b is not None else 0.0)).to(a.dtype)
    ops.add__Tensor = add_
    train.torch = _TorchOnCpu()
    try:
        yield lib
    finally:
        for (mod, name), value in saved.items():
            setattr(mod, name, value)


def _run(cfg_kwargs, world, rank, batches, steps=2, pg_factory=None):
    from tensorplay_mlu_b200.train import DataParallelMLP, MLPConfig, init_params_host

    cfg = MLPConfig(**cfg_kwargs)
    with cpu_step() as lib:
        holder = {}
        pg = pg_factory(lambda: holder["model"].grad_flat) if pg_factory else None
        model = DataParallelMLP(cfg, device=rank, pg=pg, host_params=init_params_host(cfg, seed=0))
        holder["model"] = model
        x, t = batches
        for _ in range(steps):
            model.step(x, t)
        model.flush()
        return [p.clone() for p in model.params()], lib.sm_limits, (pg.spans if pg else []), model


# ---------------------------------------------------------------- workers

def _worker(rank: int, port: int, out_dir: str) -> None:
    sys.path.insert(0, ROOT)
    for key in ("TPB200_DP_ORDER", "TPB200_BESIDE_SLICES", "TPB200_COMM_SMS", "TPB200_COMM_DYNAMIC"):
        os.environ.pop(key, None)
    torch.distributed.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=2)
    from tensorplay_mlu_b200.train import MLPConfig, make_batch_host

    results = {}
    for order, overlap, dw1, beside in SCHEDULES:
        kw = dict(SMALL, dp_order=order, overlap_next_step=overlap, dw1_slices=dw1, beside_slices=beside)
        batches = make_batch_host(MLPConfig(**kw), seed=rank)
        params, limits, spans, model = _run(kw, 2, rank, batches,
                                            pg_factory=lambda flat: GlooGroup(2, flat))
        results[(order, overlap, dw1, beside)] = {
            "params": params, "limits": limits, "spans": spans,
            "n_a": model.n_a, "n_total": model.grad_flat.numel(),
        }
    torch.distributed.destroy_process_group()
    torch.save(results, os.path.join(out_dir, f"rank{rank}.pt"))


@pytest.fixture(scope="module")
def two_rank_results(tmp_path_factory):
    out = tmp_path_factory.mktemp("dp_schedule")
    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_worker, args=(r, port, str(out))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    assert [p.exitcode for p in procs] == [0, 0]
    return torch.load(out / "rank0.pt"), torch.load(out / "rank1.pt")


def test_ranks_agree_and_every_schedule_gives_the_same_bits(two_rank_results):
    r0, r1 = two_rank_results
    first = r0[SCHEDULES[0]]["params"]
    for key in SCHEDULES:
        for a, b in zip(r0[key]["params"], r1[key]["params"]):
            assert torch.equal(a, b), key
        for a, b in zip(first, r0[key]["params"]):
            assert torch.equal(a, b), key


def test_data_parallel_equals_the_single_process_step_on_the_whole_batch(two_rank_results):
    from tensorplay_mlu_b200.train import MLPConfig, make_batch_host

    r0, _ = two_rank_results
    x0, t0 = make_batch_host(MLPConfig(**SMALL), seed=0)
    x1, t1 = make_batch_host(MLPConfig(**SMALL), seed=1)
    whole = dict(SMALL, batch=2 * SMALL["batch"])
    params, limits, _, _ = _run(whole, 1, 0, (torch.cat([x0, x1]), torch.cat([t0, t1])))
    assert limits == []  # no collective, no reserve
    for got, want in zip(r0[SCHEDULES[0]]["params"], params):
        # bf16 storage: the two sums of the batch's gradient differ in
        # rounding only (the per-rank halves are rounded before the exchange)
        err = (got.float() - want.float()).abs().max().item()
        assert err <= 2e-2 * max(want.float().abs().max().item(), 1.0), err


def test_every_gradient_element_is_exchanged_once_per_step(two_rank_results):
    r0, _ = two_rank_results
    for key, res in r0.items():
        order, overlap, dw1, beside = key
        spans = res["spans"]
        per_step = 1 + dw1
        assert len(spans) == 2 * per_step, key
        for step in range(2):
            covered = sorted(spans[step * per_step:(step + 1) * per_step])
            pos = 0
            for offset, length in covered:
                assert offset == pos, (key, covered)
                pos += length
            assert pos == res["n_total"], key
            assert (0, res["n_a"]) in covered  # bucket A in one piece


def test_every_sm_reserve_is_lifted(two_rank_results):
    r0, _ = two_rank_results
    for key, res in r0.items():
        limits = res["limits"]
        assert limits, key  # products did run beside exchanges
        assert limits[-1] == 0, key
        for set_, lift in zip(limits[0::2], limits[1::2]):
            assert set_ == 148 - 24 and lift == 0, (key, limits)
