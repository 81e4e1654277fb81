"""Benchmark of the B200 backend on BASELINE.json's workloads.

Headline (one JSON line on rank 0): the data-parallel MLP training step
-- Linear 4096->16384, GELU, Linear 16384->4096, bf16,
per-rank batch 8192, MSE loss, full backward and SGD -- run on N GPUs, one
process per GPU (torchrun), gradients all-reduced over NCCL.  ``value`` is
the whole-job throughput in samples/s (8192 * N samples per step), with the
inputs already resident in HBM; ``e2e`` is the same step fed from pinned host
memory every step (host->device copies and the loss read-back inside the
timed region).  At N=1 rank 0 also reports the memory-bound operator sweep
(config 2) and the GEMM set (config 3), and times the CPU port of the step
(``cpu_baseline``).

``--impl reference`` times the reference's CPU path of the same step (the
oracle's port of it: tensorplay-mlu's host path is TensorPlay's CPU kernels,
not installable here) on the host cores, rank 0 only.

Usage:  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
"""

from __future__ import annotations

import argparse
import json
import os
import re
import statistics
import subprocess
import sys
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

PER_RANK_BATCH = 8192
D_IN, D_HIDDEN = 4096, 16384
METRIC = "dp_mlp_train_throughput"
UNIT = "samples/s"
WORKLOAD = "dp_mlp_4096x16384x4096_bf16_b8192_per_rank"


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), float(p["bf16_tflops_sustained"]), "measured"
    except Exception:
        return 6650.0, 1590.0, 1400.0, "fallback"


# DRAM bytes per launch (dram__bytes_read.sum + dram__bytes_write.sum) of
# each of the step's five products, from one ncu capture of the five
# gemm_tc2_kernel launches of a full-size step (`ncu --metrics
# dram__bytes_read.sum,dram__bytes_write.sum --clock-control none -k
# regex:gemm_tc2 -s 5 -c 5` of `bench.py --only mlp_step --steps 2`; its
# summary is kept with the profiles).  Algorithmic bytes per launch:
# A + B read once, C written once.
GEMM_NAMES = ("h=xW1^T", "out=aW2^T", "dW2=dout^T a", "dh=gelu'(dout W2)", "dW1=dh^T x")
GEMM_DRAM_BYTES = {
    "h=xW1^T": 1099996416,
    "out=aW2^T": 1697812224,
    "dW2=dout^T a": 1157644544,
    "dh=gelu'(dout W2)": 1154491136,
    "dW1=dh^T x": 1428218880,
}
GEMM_ALGORITHMIC_BYTES = {
    "h=xW1^T": (8192 * 4096 + 16384 * 4096 + 2 * 8192 * 16384 + 16384) * 2,
    "out=aW2^T": (8192 * 16384 + 4096 * 16384 + 8192 * 4096 + 4096) * 2,
    "dW2=dout^T a": (8192 * 4096 + 8192 * 16384 + 4096 * 16384) * 2,
    "dh=gelu'(dout W2)": (8192 * 4096 + 4096 * 16384 + 8192 * 16384 * 2) * 2,
    "dW1=dh^T x": (8192 * 16384 + 8192 * 4096 + 16384 * 4096) * 2,
}


# ------------------------------------------------------------------ clocks

class ClockSampler:
    """SM clock and throttle reasons sampled during the timed region.

    NVML is polled from a thread every 5 ms (the timed regions last from
    ~0.1 s), the device found by its PCI bus id; nvidia-smi at 20 ms is the
    fallback where NVML cannot be loaded."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    NAMES = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]

    def __init__(self, device: int, period_s: float = 0.005):
        self.device = device
        self.period = period_s
        self.proc = None
        self.thread = None
        self.rows = []  # (sm_mhz, max_mhz, [flag per NAMES])

    def _nvml_handle(self):
        import pynvml

        pynvml.nvmlInit()
        try:
            bus = torch.cuda.get_device_properties(self.device).pci_bus_id
            dom = torch.cuda.get_device_properties(self.device).pci_domain_id
            dev = torch.cuda.get_device_properties(self.device).pci_device_id
            return pynvml, pynvml.nvmlDeviceGetHandleByPciBusId(f"{dom:08x}:{bus:02x}:{dev:02x}.0")
        except Exception:
            return pynvml, pynvml.nvmlDeviceGetHandleByIndex(self.device)

    def __enter__(self):
        import threading

        try:
            nv, handle = self._nvml_handle()
            bits = [nv.nvmlClocksEventReasonHwSlowdown, nv.nvmlClocksEventReasonHwThermalSlowdown,
                    nv.nvmlClocksEventReasonSwThermalSlowdown, nv.nvmlClocksEventReasonSwPowerCap]
            max_mhz = nv.nvmlDeviceGetMaxClockInfo(handle, nv.NVML_CLOCK_SM)
            self.stop = threading.Event()

            def poll():
                while not self.stop.is_set():
                    try:
                        mhz = nv.nvmlDeviceGetClockInfo(handle, nv.NVML_CLOCK_SM)
                        reasons = nv.nvmlDeviceGetCurrentClocksEventReasons(handle)
                        self.rows.append((float(mhz), float(max_mhz), [bool(reasons & b) for b in bits]))
                    except Exception:
                        pass
                    self.stop.wait(self.period)

            self.thread = threading.Thread(target=poll, daemon=True)
            self.thread.start()
            self.source = "nvml"
            return self
        except Exception:
            self.thread = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.device}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "20"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            # Wait (up to ~5 s) for the first sample, so the sampler is running
            # before the timed region starts; that sample itself is pre-region.
            import select

            if select.select([self.proc.stdout], [], [], 5.0)[0]:
                self.proc.stdout.readline()
            self.source = "nvidia-smi"
        except OSError:
            self.proc = None
            self.source = None
        return self

    def __exit__(self, *exc):
        if self.thread is not None:
            self.stop.set()
            self.thread.join(timeout=5)
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.add_smi_lines(out.splitlines())
        return False

    def add_smi_lines(self, lines):
        """Samples from nvidia-smi's csv lines (FIELDS, no header, no units)."""
        for line in lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                self.rows.append((float(parts[1]), float(parts[2]), [f.lower() == "active" for f in parts[5:9]]))
            except ValueError:
                continue

    def summary(self):
        rows = list(self.rows)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0,
                    "source": getattr(self, "source", None)}
        reasons = sorted({self.NAMES[i] for _, _, flags in rows for i, f in enumerate(flags) if f})
        return {"sm_mhz": statistics.median(r[0] for r in rows), "sm_max_mhz": max(r[1] for r in rows),
                "sm_mhz_min": min(r[0] for r in rows), "reasons": reasons, "samples": len(rows),
                "source": self.source}


# ------------------------------------------------------- NCCL's choices

NCCL_LOG = re.compile(r"AllReduce: (\d+) Bytes -> Algo (\w+) proto (\w+) channel\{Lo\.\.Hi\}=\{(\d+)\.\.(\d+)\}")


def nccl_log_setup(rank: int):
    """Point NCCL's INFO / TUNING log at a file of this rank, so the line can
    report the algorithm NCCL chose for the step's all-reduces.  A quiet level
    the environment already sets (VERSION, WARN) is replaced, since the log
    goes to a file rather than the console; a user who asked for INFO or TRACE
    themselves, or who set NCCL_DEBUG_FILE, keeps their own log and the line
    reports nothing.  Must run before the first communicator is made."""
    level = os.environ.get("NCCL_DEBUG", "").strip().upper()
    if level not in ("", "VERSION", "WARN") or "NCCL_DEBUG_FILE" in os.environ:
        return None
    path = f"/tmp/tpb200_nccl_rank{rank}_{os.getpid()}.log"
    os.environ.update(NCCL_DEBUG="INFO", NCCL_DEBUG_SUBSYS="INIT,TUNING", NCCL_DEBUG_FILE=path)
    return path


def nccl_choices(lines, sizes):
    """{bytes: {"algo", "proto", "channels", "calls"}} for the all-reduces of
    the given sizes, from NCCL TUNING lines; plus whether NVLS was available."""
    out = {}
    nvls = False
    for line in lines:
        if "NVLS multicast support is available" in line:
            nvls = True
        m = NCCL_LOG.search(line)
        if m is None or int(m.group(1)) not in sizes:
            continue
        key = str(int(m.group(1)))
        entry = out.setdefault(key, {"algo": m.group(2), "proto": m.group(3),
                                     "channels": int(m.group(5)) - int(m.group(4)) + 1, "calls": 0})
        entry["calls"] += 1
        if entry["algo"] != m.group(2) or entry["proto"] != m.group(3):
            entry["algo"], entry["proto"] = "mixed", "mixed"
    return {"nvls_available": nvls, "allreduce": out}


# ----------------------------------------------------------- distributed

def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    return rank, world, local


class HostGroup:
    """Host-side plumbing across ranks (gloo): barrier, max, store."""

    def __init__(self, rank: int, world: int):
        self.rank, self.world = rank, world
        self.active = world > 1
        if self.active:
            import datetime
            import torch.distributed as dist

            dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=600))
            self.dist = dist
            self.store = dist.distributed_c10d._get_default_store()

    def barrier(self):
        if self.active:
            self.dist.barrier()

    def max(self, value: float) -> float:
        if not self.active:
            return value
        t = torch.tensor([value], dtype=torch.float64)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.active:
            self.dist.destroy_process_group()


# ------------------------------------------------------------- reference arm

def workload_config(world: int) -> dict:
    """The `config` object of both arms' lines (identical, so the two arms
    are the same workload)."""
    return {"workload": WORKLOAD, "model": "MLP 4096-16384-4096 gelu, MSE loss, SGD lr 1e-3",
            "global_batch": PER_RANK_BATCH * world, "per_rank_batch": PER_RANK_BATCH, "seq_len": None,
            "parallelism": f"dp{world}",
            "l2": "inputs larger than L2 (per-step working set ~1.9 GB > 126 MB)"}


def host_threads() -> int:
    """The host cores this process may run on."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_mlp_throughput(steps: int, warmup: int, rows: int = PER_RANK_BATCH):
    """The CPU port of the step (oracle/mlp.c: blocked fp32 products over
    bf16 tensors) on `rows` rows per step with the full-size weights, on
    every host core.  Returns (samples/s, threads, seconds, GFLOP/s)."""
    import oracle as O
    from tensorplay_mlu_b200.train import MLPConfig, init_params_host, make_batch_host

    threads = host_threads()
    O.set_num_threads(threads)  # torchrun exports OMP_NUM_THREADS=1
    cfg = MLPConfig(d_in=D_IN, d_hidden=D_HIDDEN, batch=rows)
    w1, b1, w2, b2 = [p.contiguous() for p in init_params_host(cfg, seed=0)]
    x, t = make_batch_host(cfg, seed=0)
    for _ in range(warmup):
        O.mlp_step(x, t, w1, b1, w2, b2, cfg.lr)
    start = time.perf_counter()
    for _ in range(steps):
        O.mlp_step(x, t, w1, b1, w2, b2, cfg.lr)
    elapsed = time.perf_counter() - start
    gflops = 5 * 2.0 * rows * D_IN * D_HIDDEN * steps / elapsed / 1e9
    return rows * steps / elapsed, O.num_threads(), elapsed, gflops


def run_reference(args, rank: int, world: int) -> None:
    """The reference's CPU path of the step: TensorPlay's CPU kernels are not
    installable here, so its port (oracle/mlp.c) runs the full 8192-row step
    on rank 0's host cores; the other ranks exit without work."""
    if rank != 0:
        return
    value, threads, elapsed, gflops = cpu_mlp_throughput(args.steps, args.warmup)
    line = {
        "impl": "reference",
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1000.0 * elapsed / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": workload_config(world),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                         "gflop_s": round(gflops, 1),
                         "sample": f"the full {PER_RANK_BATCH}-row step (forward, backward, SGD over the "
                                   "134M-parameter weights), every step; oracle/mlp.c's blocked fp32 products "
                                   "on the host cores, rank 0 only"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------- our arm

def time_events(fn, iters: int, warmup: int = 3, preroll: int = 2) -> float:
    """Mean milliseconds of `fn` over `iters`, CUDA events on the current stream.

    `preroll` calls are queued (not waited for) just before the start event,
    so the device is busy when the event is reached and the timed calls run
    back to back, as in a model's step, rather than each run starting on an
    idle device behind the host's first launch."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for _ in range(preroll):
        fn()
    start.record()
    for _ in range(iters):
        fn()
    end.record()
    end.synchronize()
    return start.elapsed_time(end) / iters


def op_sweep(ops, hbm_peak: float, iters: int = 20, passes: int = 3):
    """memory-bound kernels, achieved GB/s and fraction of HBM.

    The whole sweep runs `passes` times; each kernel is timed over `iters`
    back-to-back launches (CUDA events) per pass and its median pass is
    reported, with `spread` = slowest / fastest pass.  Passes are seconds
    apart, so a disturbance of the device that lasts a while spoils one pass
    of a row, not its figure."""
    runs = [_op_sweep_pass(ops, iters) for _ in range(passes)]
    res = {}
    for name in runs[0]:
        times = sorted(r[name][0] for r in runs)
        ms, nbytes = statistics.median(times), runs[0][name][1]
        gbs = nbytes / (ms * 1e-3) / 1e9
        res[name] = {"ms": round(ms, 4), "gb_s": round(gbs, 1), "frac": round(gbs / hbm_peak, 3),
                     "spread": round(times[-1] / times[0], 2)}
    return res


def _op_sweep_pass(ops, iters: int):
    """One pass of the sweep: {row: (ms per launch, algorithmic bytes)}."""
    g = torch.Generator(device="cuda").manual_seed(0)
    res = {}
    _time_events = globals()["time_events"]

    def time_events(fn, n):  # noqa: F811 -- the sweep's own iteration count
        return _time_events(fn, iters)

    def record(name, ms, nbytes):
        res[name] = (ms, nbytes)

    M = N = 8192
    for dt, tag in ((torch.float32, "f32"), (torch.bfloat16, "bf16")):
        es = torch.finfo(dt).bits // 8
        a = (torch.randn(M, N, generator=g, device="cuda") * 2).to(dt)
        b = (torch.randn(N, generator=g, device="cuda") * 2).to(dt)
        bpos = ops.add_Scalar(ops.abs(b), 1)
        n = M * N
        record(f"add_row_{tag}", time_events(lambda: ops.add_Tensor(a, b), 10), (2 * n + N) * es)
        record(f"mul_row_{tag}", time_events(lambda: ops.mul_Tensor(a, b), 10), (2 * n + N) * es)
        record(f"div_row_{tag}", time_events(lambda: ops.div_Tensor(a, bpos), 10), (2 * n + N) * es)
        record(f"exp_{tag}", time_events(lambda: ops.exp(a), 10), 2 * n * es)
        record(f"gelu_{tag}", time_events(lambda: ops.gelu(a), 10), 2 * n * es)
        record(f"sigmoid_{tag}", time_events(lambda: ops.sigmoid(a), 10), 2 * n * es)
        dy = torch.randn(M, N, generator=g, device="cuda").to(dt)
        sy = ops.sigmoid(a)
        record(f"gelu_backward_{tag}", time_events(lambda: ops.gelu_backward(dy, a), 10), 3 * n * es)
        record(f"sigmoid_backward_{tag}", time_events(lambda: ops.sigmoid_backward(dy, sy), 10), 3 * n * es)
        for name, fn in (("sum", ops.sum), ("mean", ops.mean)):
            record(f"{name}_all_{tag}", time_events(lambda: fn(a), 10), n * es)
        record(f"sum_dim-1_{tag}", time_events(lambda: ops.sum_dim_IntList(a, [-1]), 10), n * es + M * es)
        record(f"amax_dim-1_{tag}", time_events(lambda: ops.amax(a, [-1]), 10), n * es + M * es)
        record(f"amin_all_{tag}", time_events(lambda: ops.amin(a), 10), n * es)
        del a, b, bpos, dy, sy
        R, C = 32768, 4096
        x = (torch.randn(R, C, generator=g, device="cuda") * 2).to(dt)
        dx = torch.randn(R, C, generator=g, device="cuda").to(dt)
        y = ops.softmax(x, -1)
        ly = ops.log_softmax(x, -1)
        m = R * C
        record(f"softmax_{tag}", time_events(lambda: ops.softmax(x, -1), 10), 2 * m * es)
        record(f"log_softmax_{tag}", time_events(lambda: ops.log_softmax(x, -1), 10), 2 * m * es)
        record(f"softmax_backward_{tag}",
               time_events(lambda: ops._softmax_backward_data(dx, y, -1, dt), 10), 3 * m * es)
        record(f"log_softmax_backward_{tag}",
               time_events(lambda: ops._log_softmax_backward_data(dx, ly, -1, dt), 10), 3 * m * es)
        del x, dx, y, ly
    ia = torch.randint(-1000000, 1000000, (M, N), generator=g, device="cuda", dtype=torch.int32)
    ib = torch.randint(-1000000, 1000000, (M, N), generator=g, device="cuda", dtype=torch.int32)
    record("add_int32", time_events(lambda: ops.add_Tensor(ia, ib), 10), 3 * M * N * 4)
    record("amax_all_int32", time_events(lambda: ops.amax(ia), 10), M * N * 4)
    del ia, ib
    # The MLP's bias gradient: [8192, 16384] bf16 summed over dim 0.
    hb = torch.randn(8192, 16384, generator=g, device="cuda").to(torch.bfloat16)
    record("sum_dim0_8192x16384_bf16", time_events(lambda: ops.sum_dim_IntList(hb, [0]), 10),
           (8192 * 16384 + 16384) * 2)
    return res


def quick_start(ops, iters: int = 200):
    """BASELINE config 1, the README quick-start chain on fp32 [256, 256]:
    y = x @ w; z = relu(y).softmax(-1); loss = z.sum(); backward to x and w.
    Latency-bound: milliseconds per chain run eagerly (one launch per
    operator) and replayed from one recording (graph.py's Graph)."""
    from tensorplay_mlu_b200 import _native as N
    from tensorplay_mlu_b200.graph import Graph

    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(256, 256, generator=g, device="cuda")
    w = torch.randn(256, 256, generator=g, device="cuda")
    ones = ops.fill_(torch.empty_like(x), 1.0)

    def chain():
        y = ops.mm(x, w)
        z = ops.softmax(ops.relu(y), -1)
        loss = ops.sum(z)
        dr = ops._softmax_backward_data(ones, z, -1, torch.float32)
        dy = ops.threshold_backward(dr, y, 0.0)
        return loss, ops.mm(dy, w.t()), ops.mm(x.t(), dy)

    launches0 = N.lib().tp_b200_launch_count()
    chain()
    per_chain = N.lib().tp_b200_launch_count() - launches0
    eager_ms = time_events(chain, iters)
    t0 = time.perf_counter()
    for _ in range(iters):
        chain()
    torch.cuda.synchronize()
    eager_wall_ms = (time.perf_counter() - t0) * 1e3 / iters
    graph = Graph()
    try:
        graph.capture(chain)
        replay_ms = time_events(graph.replay, iters)
    finally:
        graph.reset()
    return {"eager_ms": round(eager_ms, 4), "eager_wall_ms": round(eager_wall_ms, 4),
            "graph_replay_ms": round(replay_ms, 4), "launches_per_chain": int(per_chain),
            "note": "fp32 [256,256], forward + backward; eager_ms / graph_replay_ms are CUDA-event "
                    "times per chain on the stream, eager_wall_ms the host wall clock"}


def gemm_set(ops, bf16_peak: float, hbm_peak: float = None):
    """achieved TFLOP/s of the GEMM shapes; for the bmm
    (K = 128, below the ridge: bound by HBM) also its algorithmic bytes --
    A, B and C once each -- per second against the HBM copy peak."""
    g = torch.Generator(device="cuda").manual_seed(0)
    res = {}

    def rnd(*shape, k, dt=torch.bfloat16):
        return (torch.randn(*shape, generator=g, device="cuda") * k ** -0.5).to(dt)

    def record(name, ms, flops, peak):
        tf = flops / (ms * 1e-3) / 1e12
        res[name] = {"ms": round(ms, 4), "tflops": round(tf, 1), "frac": round(tf / peak, 3) if peak else None}

    n = 8192
    a, b = rnd(n, n, k=n), rnd(n, n, k=n)
    record("mm_8192_bf16", time_events(lambda: ops.mm(a, b), 10), 2 * n ** 3, bf16_peak)
    del a, b
    M, K, N = 16384, 4096, 11008
    x, w, bias = rnd(M, K, k=K), rnd(N, K, k=K), rnd(N, k=1)
    wt = ops.contiguous(w.t())
    record("addmm_16384x4096x11008_bf16", time_events(lambda: ops.addmm(bias, x, wt), 10), 2 * M * K * N,
           bf16_peak)
    record("linear_16384x4096x11008_bf16", time_events(lambda: ops.linear(x, w, bias), 10), 2 * M * K * N,
           bf16_peak)
    del x, w, bias, wt
    ba, bb = rnd(64, 2048, 128, k=128), rnd(64, 128, 2048, k=128)
    ms = time_events(lambda: ops.bmm(ba, bb), 10)
    record("bmm_64x2048x128x2048_bf16", ms, 2 * 64 * 2048 * 128 * 2048, bf16_peak)
    bytes_bmm = (64 * 2048 * 128 + 64 * 128 * 2048 + 64 * 2048 * 2048) * 2
    gbs = bytes_bmm / (ms * 1e-3) / 1e9
    res["bmm_64x2048x128x2048_bf16"].update(
        bound="hbm", hbm_gb_s=round(gbs, 1), hbm_frac=round(gbs / hbm_peak, 3) if hbm_peak else None)
    del ba, bb
    n = 4096
    fa, fb = rnd(n, n, k=n, dt=torch.float32), rnd(n, n, k=n, dt=torch.float32)
    prev = torch.get_float32_matmul_precision()
    torch.set_float32_matmul_precision("highest")
    try:
        # Full fp32 precision runs as three TF32 tensor-core products (the
        # split-precision method): its ceiling is a third of the TF32 peak.
        record("mm_4096_fp32_highest", time_events(lambda: ops.mm(fa, fb), 5), 2 * n ** 3, bf16_peak / 2 / 3)
        torch.set_float32_matmul_precision("high")
        record("mm_4096_fp32_tf32", time_events(lambda: ops.mm(fa, fb), 10), 2 * n ** 3, bf16_peak / 2)
    finally:
        torch.set_float32_matmul_precision(prev)
    return res


# NVLink 5 per GPU and direction (18 links through NVSwitch), the roofline of
# the collective sweep's bus bandwidth.
NVLINK_GBS = 900.0


def collective_sweep(pg, host, ops, world: int, max_bytes: int = 1 << 30):
    """BASELINE config 5b: NCCL collectives through the nccl_b200 process group,
    bus bandwidth by the nccl-tests convention (all_reduce 2(n-1)/n, others
    (n-1)/n), time = max over ranks of CUDA-event time; nvlink_frac = bus
    bandwidth / 900 GB/s (NVLink 5 per GPU and direction)."""
    res = {}
    sizes = []
    s = 4096
    while s <= max_bytes:
        sizes.append(s)
        s *= 4
    for dt, tag in ((torch.float32, "f32"), (torch.bfloat16, "bf16")):
        es = torch.finfo(dt).bits // 8
        for nbytes in sizes:
            n = (nbytes // es) // world * world
            buf = torch.ones(n, dtype=dt, device="cuda")
            out = torch.empty(n, dtype=dt, device="cuda")
            part = torch.empty(n // world, dtype=dt, device="cuda")
            cases = {
                "all_reduce": (lambda: pg.allreduce([buf], 0), 2.0 * (world - 1) / world),
                "all_gather": (lambda: pg.all_gather_single(out, buf[: n // world]), (world - 1) / world),
                "reduce_scatter": (lambda: pg.reduce_scatter_single(part, buf, 0), (world - 1) / world),
                "all_to_all": (lambda: pg.all_to_all_single(out, buf), (world - 1) / world),
            }
            for name, (fn, factor) in cases.items():
                iters = 5 if nbytes >= (64 << 20) else 20
                for _ in range(2):
                    fn()
                torch.cuda.synchronize()
                host.barrier()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                for _ in range(iters):
                    fn()
                e1.record()
                e1.synchronize()
                ms = host.max(e0.elapsed_time(e1) / iters)
                algbw = n * es / (ms * 1e-3) / 1e9
                res.setdefault(f"{name}_{tag}", []).append(
                    {"bytes": n * es, "ms": round(ms, 4), "algbw_gb_s": round(algbw, 1),
                     "busbw_gb_s": round(algbw * factor, 1),
                     "nvlink_frac": round(algbw * factor / NVLINK_GBS, 3)})
            del buf, out, part
    return res


def nccl_summary(path, model):
    """NCCL's algorithm / protocol / channels for the step's exchanges, from
    this rank's log (None when the log was not ours to read)."""
    if path is None:
        return None
    try:
        with open(path, errors="replace") as f:
            lines = f.readlines()
    except OSError:
        return None
    if not lines:
        return None
    es = model.bucket_a.element_size()
    sizes = {model.bucket_a.numel() * es} | {length * es for _, _, _, length in model._bucket_b_slices}
    return nccl_choices(lines, sizes)


def exchange_ms(pg, bucket, host, iters: int = 5) -> float:
    """Milliseconds of one SUM all-reduce of `bucket` on `pg`, nothing beside
    it (CUDA events, max over ranks)."""
    for _ in range(2):
        pg.allreduce([bucket], 0)
    torch.cuda.synchronize()
    host.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        pg.allreduce([bucket], 0)
    e1.record()
    e1.synchronize()
    return host.max(e0.elapsed_time(e1) / iters)


def h2d_only_ms(upload, copy_stream, steps: int, host) -> float:
    """Milliseconds per step of the e2e leg's host->device copies alone
    (both slots' batches, pinned memory, the copy stream), max over ranks."""
    for slot in (0, 1):
        upload(slot)
    copy_stream.synchronize()
    host.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(copy_stream)
    for i in range(steps):
        upload(i % 2)
    e1.record(copy_stream)
    e1.synchronize()
    return host.max(e0.elapsed_time(e1) / steps)


def run_ours(args, rank: int, world: int, local: int) -> None:
    import tensorplay_mlu_b200 as tpb
    from tensorplay_mlu_b200 import _native as N
    from tensorplay_mlu_b200 import distributed as D
    from tensorplay_mlu_b200.train import DataParallelMLP, MLPConfig, init_params_host, make_batch_host

    tpb.load()  # before any CUDA call, so the caching allocator backs every tensor
    assert tpb.allocator_installed(), "the B200 caching allocator must back the benchmark's tensors"
    torch.cuda.set_device(local)
    ops = tpb.ops
    nccl_log = nccl_log_setup(rank) if world > 1 else None
    host = HostGroup(rank, world)
    hbm_peak, bf16_peak, bf16_sustained, peak_kind = peaks()
    # The training step's collectives take at most as many CTAs as the
    # products beside them leave SMs free (MLPConfig.comm_sms; TPB200_COMM_SMS).
    # TPB200_NCCL_MAX_CTAS sets the bound apart from the reserve (A/B).
    comm_sms = int(os.environ.get("TPB200_COMM_SMS", MLPConfig.comm_sms))
    max_ctas = int(os.environ.get("TPB200_NCCL_MAX_CTAS", comm_sms))
    pg = D.create(_PrefixStore("nccl_b200", host.store), rank, world, device=local, timeout_s=300,
                  max_ctas=max_ctas) if world > 1 else None

    # Kernel-level extras (op sweep, GEMM set) at N = 1: measured before the
    # training loop by default, so their kernels run at the clocks a kernel
    # gets on its own rather than just after seconds at the power cap.
    pre = {}
    if world == 1 and not args.no_extras and args.extras_order == "first":
        with ClockSampler(local) as extra_clocks:
            pre["op_sweep"] = op_sweep(ops, hbm_peak)
            pre["gemm_set"] = gemm_set(ops, bf16_peak, hbm_peak)
            pre["quick_start"] = quick_start(ops)
        pre["extras_clocks"] = extra_clocks.summary()
        torch.cuda.empty_cache()
        tpb.runtime.empty_cache()

    # TPB200_DW1_SLICES overrides how many slices the last gradient bucket is
    # exchanged in (A/B measurements; the default is MLPConfig's).
    slices = int(os.environ.get("TPB200_DW1_SLICES", MLPConfig.dw1_slices))
    # Bucket B's update deferred into the next step (TPB200_OVERLAP_NEXT=0
    # applies it at the end of each step instead, for A/B measurements);
    # flush() inside each timed region completes the last step's update.
    overlap = os.environ.get("TPB200_OVERLAP_NEXT", "1") != "0"
    cfg = MLPConfig(d_in=D_IN, d_hidden=D_HIDDEN, batch=PER_RANK_BATCH, dw1_slices=slices,
                    overlap_next_step=overlap)
    model = DataParallelMLP(cfg, device=local, pg=pg, host_params=init_params_host(cfg, seed=0))
    xh, th = make_batch_host(cfg, seed=rank)
    x, t = ops.to_device(xh), ops.to_device(th)

    # ---- device-resident timing (the headline value)
    for _ in range(args.warmup):
        model.step(x, t)
    model.flush()
    torch.cuda.synchronize()
    host.barrier()
    launches0 = N.lib().tp_b200_launch_count()
    model.gemm_events = []
    with ClockSampler(local) as clocks:
        torch.cuda.synchronize()
        host.barrier()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(args.steps):
            loss = model.step(x, t)
        model.flush()
        end.record()
        end.synchronize()
        host.barrier()
    launches = N.lib().tp_b200_launch_count() - launches0
    ms_local = start.elapsed_time(end) / args.steps
    ms = host.max(ms_local)
    gemm_ms = [s.elapsed_time(e) for s, e in model.gemm_events]
    model.gemm_events = None
    gemm_avg_ms = sum(gemm_ms) / len(gemm_ms)
    # Average per GEMM of the step, in step order: h = x W1^T, out = a W2^T,
    # dW2 = dout^T a, d_a = dout W2, dW1 = dh^T x.
    per_gemm = [sum(gemm_ms[i::5]) / len(gemm_ms[i::5]) for i in range(5)]
    loss_value = ops.item(loss)

    # ---- end to end: pinned host batches, copies and the loss read-back timed
    xp, tp_ = xh.pin_memory(), th.pin_memory()
    h2d = xp.numel() * xp.element_size() + tp_.numel() * tp_.element_size()
    copy_stream = torch.cuda.Stream()
    bufs = [(torch.empty_like(x), torch.empty_like(t)) for _ in range(2)]
    # One pinned slot per step: every step's loss is copied to the host
    # without stalling the host on it (as a training loop logs its loss);
    # the slots are checked once the timed region has ended.
    # NaN until a step's copy lands, so a slot that was never written fails
    # the check after the timed region.
    loss_host = torch.full((max(args.steps, args.warmup, 1),), float("nan"), dtype=torch.float32).pin_memory()
    loss_keep = []

    def upload(slot):
        with torch.cuda.stream(copy_stream):
            for dst, src in zip(bufs[slot], (xp, tp_)):
                N.check(N.lib().tp_b200_memcpy(dst.data_ptr(), src.data_ptr(), src.numel() * src.element_size(),
                                               1, local, -1, copy_stream.cuda_stream, 0), "h2d")
            ev = torch.cuda.Event()
            ev.record(copy_stream)
        return ev

    def e2e_steps(n):
        ready = upload(0)
        for i in range(n):
            torch.cuda.current_stream().wait_event(ready)
            xs, ts = bufs[i % 2]
            if i + 1 < n:
                copy_stream.wait_stream(torch.cuda.current_stream())
                ready = upload((i + 1) % 2)
            l = model.step(xs, ts)
            l32 = ops._to_dtype(l, torch.float32)
            loss_keep.append(l32)  # the source stays alive until the copy has run
            N.check(N.lib().tp_b200_memcpy(loss_host.data_ptr() + 4 * i, l32.data_ptr(), 4, 2, local, -1,
                                           N.stream_of(local), 0), "d2h")

    e2e_steps(max(1, args.warmup // 2))
    model.flush()
    torch.cuda.synchronize()
    host.barrier()
    t0 = time.perf_counter()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    e2e_steps(args.steps)
    model.flush()
    e1.record()
    e1.synchronize()
    e2e_ms = host.max(e0.elapsed_time(e1) / args.steps)
    host.barrier()
    read_back = loss_host[:args.steps]
    assert bool(torch.isfinite(read_back).all()), "a step's loss read back from the device is not finite"
    last_dev = loss_keep[-1].item()
    assert read_back[-1].item() == last_dev, (read_back[-1].item(), last_dev)
    loss_keep.clear()

    # ---- the end-to-end ceiling: the same per-step host->device copies alone
    h2d_ms = h2d_only_ms(upload, copy_stream, args.steps, host)

    # ---- one bucket's exchange alone, on the step's (CTA-bounded) communicator
    exchange = None
    if world > 1:
        exchange = {"bucket_bytes": model.bucket_a.numel() * model.bucket_a.element_size(),
                    "ms_bounded": round(exchange_ms(pg, model.bucket_a, host), 4)}

    # ---- data parallelism kept every rank's parameters identical
    params_identical = None
    if world > 1:
        import hashlib

        digest = hashlib.sha256()
        for p in model.params():
            digest.update(ops.to_host(p).view(torch.int16).numpy().tobytes())
        digests = [None] * world
        host.dist.all_gather_object(digests, digest.hexdigest())
        params_identical = len(set(digests)) == 1
        assert params_identical, "data-parallel ranks hold different parameters"

    samples = PER_RANK_BATCH * world
    value = samples / (ms * 1e-3)
    e2e_value = samples / (e2e_ms * 1e-3)
    gemm_flops = 2.0 * PER_RANK_BATCH * D_IN * D_HIDDEN
    achieved = gemm_flops / (gemm_avg_ms * 1e-3) / 1e12
    traffic_by_gemm = {k: GEMM_DRAM_BYTES.get(k) for k in GEMM_NAMES}
    known = [v for v in traffic_by_gemm.values() if v is not None]
    traffic = sum(known) / len(known) if len(known) == len(GEMM_NAMES) else None

    line = None
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic: inputs/targets N(0,1) seeded by rank, nn.Linear-init weights seed 0",
            "config": workload_config(world),
            "steps_per_s": round(1000.0 / ms, 2),
            "step_tflops": round(model.flops_per_step() / (ms * 1e-3) / 1e12, 1),
            "train_loss": loss_value,
            "roofline": {"bound": "tensor", "kernel": "gemm_tc2_kernel (tcgen05 cta_group::2, bf16 -> fp32)",
                         "achieved": round(achieved, 1), "peak": bf16_peak, "unit": "TFLOP/s",
                         "frac": round(achieved / bf16_peak, 3), "traffic": traffic,
                         "peak_kind": f"{peak_kind} burst bf16 (the timed region lasts well under a second)",
                         "frac_of_sustained": round(achieved / bf16_sustained, 3),
                         "per_launch_flops": gemm_flops, "avg_launch_ms": round(gemm_avg_ms, 4),
                         "launches_timed": len(gemm_ms),
                         "per_gemm_ms": {k: round(v, 4) for k, v in zip(model.gemm_names(), per_gemm)},
                         "traffic_by_gemm": traffic_by_gemm,
                         "algorithmic_bytes_by_gemm": GEMM_ALGORITHMIC_BYTES},
            "e2e": {"value": round(e2e_value, 1), "unit": UNIT, "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": 4, "ms_per_step": round(e2e_ms, 4),
                    "path": "pinned host batch -> tp_b200_memcpy (copy stream, next batch prefetched) "
                            "-> step -> loss -> tp_b200_memcpy into that step's pinned host slot "
                            "(not waited on per step; all slots checked after the timed region)",
                    "h2d_only_ms_per_step": round(h2d_ms, 4),
                    "h2d_ceiling_gb_s": round(h2d * world / (h2d_ms * 1e-3) / 1e9, 1),
                    "ceiling_note": "the same per-step host->device copies with no compute, on every rank at "
                                    "once (max over ranks): aggregate GB/s; the e2e step cannot be shorter "
                                    "than h2d_only_ms_per_step"},
            "dp_params_identical": params_identical,
            "dp_exchange": exchange,
            "dp_nccl": nccl_summary(nccl_log, model) if world > 1 else None,
            "dp_schedule": {"order": model._order, "dw1_slices": cfg.dw1_slices,
                            "overlap_next_step": cfg.overlap_next_step,
                            "beside_slices": model._beside_slices,
                            "gemm_sms_beside_collective": model._overlap_sms or None,
                            "dynamic_tiles_beside_collective": model._overlap_dynamic,
                            "nccl_max_ctas": max_ctas or None,
                            "nccl_env": {k: v for k, v in os.environ.items() if k.startswith("NCCL_")}}
            if world > 1 else None,
            "gpu_launches": int(launches),
            "clocks": clocks.summary(),
        }
    del x, t, bufs
    if pg is not None:
        torch.cuda.synchronize()
        if not args.no_extras:
            # The sweep measures NCCL unbounded, on a communicator of its own.
            sweep_pg = D.create(_PrefixStore("nccl_b200_sweep", host.store), rank, world, device=local,
                                timeout_s=300, group_name="sweep")
            sweep = collective_sweep(sweep_pg, host, ops, world)
            bucket = torch.empty(model.bucket_a.numel(), dtype=model.bucket_a.dtype, device="cuda")
            unbounded = exchange_ms(sweep_pg, ops.zero_(bucket), host)
            if rank == 0:
                line["dp_exchange"]["ms_unbounded"] = round(unbounded, 4)
            del bucket
            torch.cuda.synchronize()
            sweep_pg.destroy()
            if rank == 0:
                line["collectives"] = sweep
                # The largest size of each row, last in the line.
                line["collectives_summary"] = {
                    k: {"bytes": v[-1]["bytes"], "busbw_gb_s": v[-1]["busbw_gb_s"], "nvlink_frac": v[-1]["nvlink_frac"]}
                    for k, v in sweep.items()}
        torch.cuda.synchronize()
        host.barrier()
        pg.destroy()
    if rank == 0 and world == 1 and not args.no_extras:
        del model
        torch.cuda.empty_cache()
        tpb.runtime.empty_cache()
        if pre:
            line.update(pre)
        else:
            with ClockSampler(local) as extra_clocks:
                line["op_sweep"] = op_sweep(ops, hbm_peak)
                line["gemm_set"] = gemm_set(ops, bf16_peak, hbm_peak)
                line["quick_start"] = quick_start(ops)
            line["extras_clocks"] = extra_clocks.summary()
        cpu_value, threads, _, gflops = cpu_mlp_throughput(2, 1)
        line["cpu_baseline"] = {"value": round(cpu_value, 2), "unit": UNIT, "cores": threads, "kind": "port",
                                "gflop_s": round(gflops, 1),
                                "sample": f"the full {PER_RANK_BATCH}-row step, 2 timed steps after 1 warm-up "
                                          "(oracle/mlp.c's blocked fp32 products, every host core)"}
        line["peaks"] = {"hbm_gbs": hbm_peak, "bf16_tflops": bf16_peak, "bf16_tflops_sustained": bf16_sustained,
                         "kind": peak_kind}
    if rank == 0:
        print(json.dumps(line), flush=True)
    host.close()


def run_only(args) -> None:
    """One kernel's workload, `--steps` launches (for ncu captures of a single kernel)."""
    import tensorplay_mlu_b200 as tpb

    tpb.load()
    torch.cuda.set_device(0)
    ops = tpb.ops
    g = torch.Generator(device="cuda").manual_seed(0)

    def rnd(*shape, dt=torch.bfloat16, scale=1.0):
        return (torch.randn(*shape, generator=g, device="cuda") * scale).to(dt)

    name = args.only
    if name == "gemm_mlp":        # the MLP's forward GEMM: [8192,4096] @ W1[16384,4096]^T
        a, w = rnd(8192, 4096), rnd(16384, 4096, scale=4096 ** -0.5)
        fn = lambda: ops.linear(a, w)
    elif name == "gemm_mlp_dw":   # weight-gradient GEMM: d_out^T [4096,8192] @ a [8192,16384]
        a, b = rnd(8192, 4096), rnd(8192, 16384)
        fn = lambda: ops.mm(a.t(), b)
    elif name == "gemm_mm8192":
        a, b = rnd(8192, 8192, scale=8192 ** -0.5), rnd(8192, 8192)
        fn = lambda: ops.mm(a, b)
    elif name == "bmm":
        a, b = rnd(64, 2048, 128, scale=128 ** -0.5), rnd(64, 128, 2048)
        fn = lambda: ops.bmm(a, b)
    elif name == "gelu_bf16":
        a = rnd(8192, 8192)
        fn = lambda: ops.gelu(a)
    elif name == "exp_bf16":
        a = rnd(8192, 8192)
        fn = lambda: ops.exp(a)
    elif name == "sum_bf16":
        a = rnd(8192, 8192)
        fn = lambda: ops.sum(a)
    elif name == "amax_rows_bf16":
        a = rnd(8192, 8192)
        fn = lambda: ops.amax(a, [-1])
    elif name == "sum_dim0_bf16":  # the MLP's bias gradient: a column sum
        a = rnd(8192, 16384)
        fn = lambda: ops.sum_dim_IntList(a, [0])
    elif name == "softmax_bf16":
        a = rnd(32768, 4096)
        fn = lambda: ops.softmax(a, -1)
    elif name in ("gemm_gelu", "gemm_gelu_bwd", "gemm_linear_h"):
        # the step's first / fourth product with and without the fused epilogue
        from tensorplay_mlu_b200 import _native as N

        x, w, bias = rnd(8192, 4096), rnd(16384, 4096, scale=4096 ** -0.5), rnd(16384)
        h, a = torch.empty(8192, 16384, dtype=torch.bfloat16, device="cuda"), torch.empty(
            8192, 16384, dtype=torch.bfloat16, device="cuda")
        d_out, w2 = rnd(8192, 4096, scale=1e-3), rnd(4096, 16384, scale=4096 ** -0.5)

        def epi(code, out, aux, A, B, c=None):
            N.check(N.lib().tp_b200_gemm_epilogue(code, N.describe(out), N.describe(aux), N.describe(A),
                                                  N.describe(B), N.describe(c) if c is not None else None, 1.0,
                                                  1.0 if c is not None else 0.0, 0, N.stream_of(out.device)),
                    "gemm_epilogue")

        if name == "gemm_gelu":
            fn = lambda: epi(N.EPI_GELU, a, h, x, w.t(), bias)
        elif name == "gemm_gelu_bwd":
            fn = lambda: epi(N.EPI_GELU_BACKWARD, a, h, d_out, w2)
        else:
            fn = lambda: ops.linear(x, w, bias)
    elif name == "mlp_step":       # one full-size training step per launch of fn (five products)
        from tensorplay_mlu_b200.train import DataParallelMLP, MLPConfig, init_params_host, make_batch_host

        cfg = MLPConfig(d_in=D_IN, d_hidden=D_HIDDEN, batch=PER_RANK_BATCH)
        model = DataParallelMLP(cfg, device=0, host_params=init_params_host(cfg, seed=0))
        xh, th = make_batch_host(cfg, seed=0)
        x, t = ops.to_device(xh), ops.to_device(th)
        fn = lambda: model.step(x, t)
    elif name == "add_row_f32":
        a, b = rnd(8192, 8192, dt=torch.float32), rnd(8192, dt=torch.float32)
        fn = lambda: ops.add_Tensor(a, b)
    else:
        raise SystemExit(f"unknown --only workload {name}")
    for _ in range(args.steps):
        fn()
    torch.cuda.synchronize()
    print(json.dumps({"only": name, "launches": args.steps,
                      "device_error": tpb._native.lib().tp_b200_take_device_error(0)}))


class _PrefixStore:
    """Keys of the NCCL rendezvous under their own prefix in the job store."""

    def __init__(self, prefix, store):
        self.prefix, self.store = prefix, store

    def set(self, key, value):
        self.store.set(f"{self.prefix}/{key}", value)

    def get(self, key, timeout=None):
        return self.store.get(f"{self.prefix}/{key}")

    def check(self, keys):
        return self.store.check([f"{self.prefix}/{k}" for k in keys])


def main() -> None:
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=100)
    p.add_argument("--warmup", type=int, default=10)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--no-extras", action="store_true", help="skip the op sweep, GEMM set and CPU baseline")
    p.add_argument("--extras-order", choices=["first", "last"], default="first",
                   help="run the op sweep and GEMM set before (default) or after the training loop")
    p.add_argument("--only", default=None,
                   help="run one kernel workload --steps times and exit (for ncu captures)")
    p.add_argument("--sweep-only", action="store_true",
                   help="only the memory-bound op sweep (config 2), --steps iterations per kernel")
    p.add_argument("--gemm-only", action="store_true", help="only the GEMM set (config 3)")
    args = p.parse_args()
    if args.only:
        run_only(args)
        return
    if args.gemm_only:
        import tensorplay_mlu_b200 as tpb

        tpb.load()
        print(json.dumps({"gemm_set": gemm_set(tpb.ops, peaks()[1], peaks()[0])}), flush=True)
        return
    if args.sweep_only:
        import tensorplay_mlu_b200 as tpb

        tpb.load()
        hbm_peak = peaks()[0]
        with ClockSampler(0) as clocks:
            sweep = op_sweep(tpb.ops, hbm_peak, iters=args.steps)
            chain = quick_start(tpb.ops)
        print(json.dumps({"op_sweep": sweep, "quick_start": chain, "clocks": clocks.summary()}), flush=True)
        return
    if args.warmup < 3:
        args.warmup = 3
    rank, world, local = dist_env()
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    run_ours(args, rank, world, local)


if __name__ == "__main__":
    main()
