"""Data-parallel MLP training step on the B200 backend.

The model of tensorplay-mlu's README distributed benchmark, at the sizes the
B200 build is measured on: Linear(4096 -> 16384), GELU, Linear(16384 -> 4096),
bf16 weights with PyTorch's nn.Linear initialisation (Kaiming-uniform, bound
1/sqrt(fan_in)) from seed 0, loss = mean((out - target)^2), full backward
(no input gradient) and an SGD update.  The step computes what TensorPlay's
autograd engine computes for this model with its operators (linear, gelu,
sub, pow, mean, mul, mm on transposed views, sum over dim 0, gelu_backward,
add_), rounding every intermediate where those operators round, with the
memory-bound operators fused into their producers:

  h = x W1^T + b1, a = gelu(h)      one product, gelu in its epilogue
                                    (h kept for the backward pass)
  out = a W2^T + b2                 product, bias in the epilogue
  loss, d_out = mse(out, t)         one pass: sub, pow, mean and the 2/n mul
  dW2 = d_out^T a, db2 = sum(d_out) product (transposes read in place), sum
  d_h = gelu_backward(d_out W2, h)  one product, gelu_backward in its epilogue
  dW1 = d_h^T x, db1 = sum(d_h)     product, sum
  p += -lr * g                      one launch per gradient bucket (the
                                    parameters share the gradients' layout)

Data parallelism (one rank per GPU): gradients live in one flat buffer split
into two buckets in backward order, A = (dW2, db2) and B = (db1, dW1), and
the parameters in one flat buffer of the same layout.  Each bucket is
all-reduced (SUM) on a side stream as soon as backward has produced it.  In
the default order (`dp_order = "w1_first"`) backward runs d_h, then dW1 in
`dw1_slices` row slices (db1 travels with the first), each slice's exchange
beside the next product, then dW2 beside bucket B's last slice; bucket B is
applied at the end of the step, and bucket A's exchange runs beside the next
step's h = x W1^T product (with `overlap_next_step`; `flush()` applies what
is still pending) and is applied before out = a W2^T.  In the "w2_first"
order dW2 comes first (bucket A beside d_h and dW1) and bucket B's slices
are applied ahead of the next step's h product, slice by slice.  Every
product that runs while an exchange is in flight leaves `comm_sms` SMs to
the collective's kernels (the communicator is bounded to as many CTAs);
the next step's h product and dW2 run in `beside_slices` row slices with
only the first beside the exchange; with `comm_dynamic_tiles` those
products claim their tiles at run time instead of in a fixed order.  The
AVG's 1/world scale is folded into the SGD step
(p -= lr/world * g_sum), not launched as its own pass as
tensorplay_mlu/distributed.py:241-242 does.
"""

from __future__ import annotations

import contextlib
import math
import os
from dataclasses import dataclass
from typing import Optional

import torch

from . import _native as N
from . import ops


@dataclass
class MLPConfig:
    d_in: int = 4096
    d_hidden: int = 16384
    batch: int = 8192
    lr: float = 1e-3
    dtype: torch.dtype = torch.bfloat16
    # Data-parallel: the last gradient bucket (db1, dW1) is produced and
    # all-reduced in this many row slices of dW1, so each slice's exchange
    # overlaps the next slice's product.
    dw1_slices: int = 2
    # Data-parallel: defer an exchange's SGD update into the next step (call
    # flush() after the last step).  False: every step ends with its
    # parameters updated.
    overlap_next_step: bool = False
    # Data-parallel order of the backward products.  "w1_first": d_h, dW1
    # (bucket B exchanged beside dW2), then dW2 (bucket A exchanged beside
    # the next step's first product, applied before its second).
    # "w2_first": dW2 (bucket A beside d_h and dW1), then d_h and dW1
    # (bucket B applied slice by slice ahead of the next step's first
    # product).  The gradients are the same either way.
    dp_order: str = "w1_first"
    # Data-parallel: SMs left free for the collective's kernels by every
    # product that runs while an all-reduce is in flight (d_h, the dW1
    # slices, the next step's h slices).  The products are persistent and
    # hold one CTA per SM, so without a reserve the collective's kernels
    # find no SM until a product ends; the process group is created with
    # its collectives bounded to as many CTAs (create(max_ctas=...)).
    # 0: the products take every SM.
    comm_sms: int = 24
    # Data-parallel: those products claim their tiles at run time
    # (tp_b200_set_gemm_tile_order), so clusters that start late behind the
    # collective's kernels take fewer tiles.
    comm_dynamic_tiles: bool = False
    # Data-parallel (w1_first order): the products that run beside an
    # exchange with nothing after it in the step to overlap -- the next
    # step's h = x W1^T beside bucket A, dW2 beside bucket B's last slice --
    # in this many row slices, only the first leaving comm_sms SMs free, so
    # the reserve lasts about as long as the exchange rather than the whole
    # product.  1: the whole product beside the exchange (measured the
    # better default: 2 gained 0.7% per step at two GPUs and lost 2.3% at
    # four, where the second dW2 slice started while the exchange still
    # held its SMs).
    beside_slices: int = 1


def init_params_host(cfg: MLPConfig, seed: int = 0):
    """Host weights, nn.Linear's default init: U(-1/sqrt(fan_in), 1/sqrt(fan_in))."""
    g = torch.Generator().manual_seed(seed)

    def uniform(shape, fan_in):
        bound = 1.0 / math.sqrt(fan_in)
        return (torch.rand(shape, generator=g, dtype=torch.float32) * 2 - 1) * bound

    w1 = uniform((cfg.d_hidden, cfg.d_in), cfg.d_in).to(cfg.dtype)
    b1 = uniform((cfg.d_hidden,), cfg.d_in).to(cfg.dtype)
    w2 = uniform((cfg.d_in, cfg.d_hidden), cfg.d_hidden).to(cfg.dtype)
    b2 = uniform((cfg.d_in,), cfg.d_hidden).to(cfg.dtype)
    return w1, b1, w2, b2


def make_batch_host(cfg: MLPConfig, seed: int):
    """Synthetic input and target, ~N(0, 1), from ``seed`` (the rank)."""
    g = torch.Generator().manual_seed(1000 + seed)
    x = torch.randn((cfg.batch, cfg.d_in), generator=g, dtype=torch.float32).to(cfg.dtype)
    t = torch.randn((cfg.batch, cfg.d_in), generator=g, dtype=torch.float32).to(cfg.dtype)
    return x, t


def bucket_b_slices(d_in: int, d_hidden: int, slices: int):
    """The row slices bucket B = (db1 [H], dW1 [H, D]) is exchanged in:
    [(r0, r1, offset, length)] -- dW1 rows [r0, r1) and the slice's span of
    the flat bucket (db1 travels with the first).  Row bounds are multiples
    of 8, so every slice of d_h's columns starts on a 16-byte boundary."""
    H, D = d_hidden, d_in
    n = max(1, int(slices))
    bounds = [(H * i // n) // 8 * 8 for i in range(n)] + [H]
    out = []
    for i in range(n):
        r0, r1 = bounds[i], bounds[i + 1]
        if r1 <= r0:
            continue
        lo = 0 if not out else H + r0 * D
        out.append((r0, r1, lo, H + r1 * D - lo))
    return out


def row_slices(rows: int, slices: int):
    """[(r0, r1)]: `rows` split into `slices` parts (empty ones dropped) whose
    bounds are multiples of 8, so a slice of a bf16 operand's columns starts
    on a 16-byte boundary."""
    n = max(1, int(slices))
    bounds = [(rows * i // n) // 8 * 8 for i in range(n)] + [rows]
    return [(bounds[i], bounds[i + 1]) for i in range(n) if bounds[i + 1] > bounds[i]]


class DataParallelMLP:
    """Parameters, gradient buckets and the training step of one rank."""

    def __init__(self, cfg: MLPConfig, device: int = 0, pg=None, host_params=None):
        self.cfg = cfg
        self.device = torch.device("cuda", device)
        self.pg = pg
        self.world = pg.size() if pg is not None else 1
        w1, b1, w2, b2 = host_params if host_params is not None else init_params_host(cfg)
        dev = self.device
        # One flat gradient buffer, bucket A = (dW2, db2), bucket B = (dW1,
        # db1), and one flat parameter buffer with the same layout, so the
        # SGD update of a bucket is one launch over one slice.
        H, D = cfg.d_hidden, cfg.d_in
        n_a = D * H + D
        n_b = H * D + H
        self.n_a = n_a
        self.grad_flat = torch.empty(n_a + n_b, dtype=cfg.dtype, device=dev)
        self.param_flat = torch.empty(n_a + n_b, dtype=cfg.dtype, device=dev)
        self.bucket_a = self.grad_flat.narrow(0, 0, n_a)
        self.bucket_b = self.grad_flat.narrow(0, n_a, n_b)
        self.dw2 = self.bucket_a.narrow(0, 0, D * H).view(D, H)
        self.db2 = self.bucket_a.narrow(0, D * H, D)
        self.db1 = self.bucket_b.narrow(0, 0, H)
        self.dw1 = self.bucket_b.narrow(0, H, H * D).view(H, D)
        self.params_a = self.param_flat.narrow(0, 0, n_a)
        self.params_b = self.param_flat.narrow(0, n_a, n_b)
        self.w2 = self.params_a.narrow(0, 0, D * H).view(D, H)
        self.b2 = self.params_a.narrow(0, D * H, D)
        self.b1 = self.params_b.narrow(0, 0, H)
        self.w1 = self.params_b.narrow(0, H, H * D).view(H, D)
        for dst, src in ((self.w1, w1), (self.b1, b1), (self.w2, w2), (self.b2, b2)):
            ops.copy_(dst, ops.to_device(src.contiguous(), dev))
        # The exchange runs on a high-priority stream, so when SMs free up the
        # collective's CTAs are dispatched ahead of the compute stream's
        # (TPB200_COMM_PRIORITY=0: default priority, for A/B measurements).
        prio = -1 if os.environ.get("TPB200_COMM_PRIORITY", "1") != "0" else 0
        self.comm_stream = (torch.cuda.Stream(device=dev, priority=prio)
                            if pg is not None and self.world > 1 else None)
        # TPB200_COMM_SMS / TPB200_COMM_DYNAMIC override cfg.comm_sms /
        # cfg.comm_dynamic_tiles (A/B measurements).
        reserve = int(os.environ.get("TPB200_COMM_SMS", cfg.comm_sms))
        total = torch.cuda.get_device_properties(dev).multi_processor_count
        self._overlap_sms = total - reserve if self.comm_stream is not None and 0 < reserve < total else 0
        dyn = os.environ.get("TPB200_COMM_DYNAMIC")
        self._overlap_dynamic = self.comm_stream is not None and (
            cfg.comm_dynamic_tiles if dyn is None else dyn not in ("", "0"))
        # When a list, every GEMM of the step appends a (start, end) pair of
        # CUDA events recorded around its launch on the current stream.
        self.gemm_events: Optional[list] = None
        # When a dict, the step stores its intermediates in it (for checks).
        self.trace: Optional[dict] = None
        # Bucket B slices whose SGD update is deferred: (start, length, work).
        self._pending: list = []
        # Bucket A's exchange whose SGD update is deferred (w1_first order).
        self._pending_a = None
        self._order = os.environ.get("TPB200_DP_ORDER", cfg.dp_order)
        # TPB200_BESIDE_SLICES overrides cfg.beside_slices (A/B measurements).
        self._beside_slices = int(os.environ.get("TPB200_BESIDE_SLICES", cfg.beside_slices))
        self._bucket_b_slices = bucket_b_slices(D, H, cfg.dw1_slices)
        self._slices = [(r0, r1) for r0, r1, _, _ in self._bucket_b_slices]

    def _timed(self, fn, *args):
        if self.gemm_events is None:
            return fn(*args)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        out = fn(*args)
        end.record()
        self.gemm_events.append((start, end))
        return out

    def params(self):
        return [self.w1, self.b1, self.w2, self.b2]

    def grads(self):
        return [self.dw1, self.db1, self.dw2, self.db2]

    # -- kernels with preallocated outputs ----------------------------------
    @staticmethod
    def _mm_into(out, a, b):
        return ops._gemm(out, a, b)

    @staticmethod
    def _colsum_into(out, x):
        """sum(x, dim=0) written into ``out`` (the bias gradient)."""
        N.check(N.lib().tp_b200_reduce(N.SUM, N.describe(out.view(1, -1)), N.describe(x), 1,
                                       N.stream_of(x.device)), "sum")
        return out

    @staticmethod
    def _gemm_epilogue(epilogue, out, aux, a, b, c=None):
        """out (and aux) from a @ b with gelu / gelu_backward fused in."""
        N.check(N.lib().tp_b200_gemm_epilogue(epilogue, N.describe(out), N.describe(aux), N.describe(a),
                                              N.describe(b), N.describe(c) if c is not None else None, 1.0,
                                              1.0 if c is not None else 0.0, 0, N.stream_of(out.device)),
                "gemm_epilogue")
        return out

    @staticmethod
    def _mse_into(loss, grad, out, target):
        """loss = mean((out - target)^2), grad = 2 (out - target) / numel."""
        N.check(N.lib().tp_b200_mse_loss(N.describe(loss), N.describe(grad), N.describe(out), N.describe(target),
                                         2.0 / out.numel(), N.stream_of(out.device)), "mse_loss")
        return loss

    def _gemm_sm_limit(self, sms: int) -> None:
        N.check(N.lib().tp_b200_set_gemm_sm_limit(self.device.index, sms), "set_gemm_sm_limit")

    @contextlib.contextmanager
    def _beside_collective(self):
        """Products launched inside run beside an all-reduce: they leave
        comm_sms SMs free (and claim tiles at run time when configured)."""
        if self.comm_stream is None:
            yield
            return
        dev = self.device.index
        if self._overlap_sms:
            self._gemm_sm_limit(self._overlap_sms)
        if self._overlap_dynamic:
            N.check(N.lib().tp_b200_set_gemm_tile_order(dev, 1), "set_gemm_tile_order")
        try:
            yield
        finally:
            if self._overlap_sms:
                self._gemm_sm_limit(0)
            if self._overlap_dynamic:
                N.check(N.lib().tp_b200_set_gemm_tile_order(dev, 0), "set_gemm_tile_order")

    def _allreduce_async(self, bucket, ready_event):
        """SUM all-reduce of ``bucket`` on the comm stream after ``ready_event``."""
        self.comm_stream.wait_event(ready_event)
        with torch.cuda.stream(self.comm_stream):
            work = self.pg.allreduce([bucket], op=0)
        return work

    def step(self, x: torch.Tensor, target: torch.Tensor) -> torch.Tensor:
        """One forward + backward + SGD step; returns the loss (device 0-d tensor)."""
        cfg = self.cfg
        B, D, H = x.shape[0], cfg.d_in, cfg.d_hidden
        dt, dev = cfg.dtype, x.device
        # forward: h = x W1^T + b1 and a = gelu(h) from one product
        h = torch.empty((B, H), dtype=dt, device=dev)
        a = torch.empty((B, H), dtype=dt, device=dev)
        if self._pending:
            # The previous step's bucket B, slice by slice: update the rows of
            # W1 (and b1, first slice) once their exchange is in, then the
            # columns of h and a those rows produce.
            with self._beside_collective():
                self._timed(self._forward_sliced, x, h, a)
        elif self._pending_a is not None:
            # The previous step's bucket A is still being exchanged: the
            # first row slice beside it, the rest on every SM.
            self._timed(self._forward_beside, x, h, a)
        else:
            self._timed(self._gemm_epilogue, N.EPI_GELU, a, h, x, self.w1.t(), self.b1)
        self._apply_pending_a()  # W2, b2 before the product that reads them
        out = self._timed(ops.linear, a, self.w2, self.b2)
        # loss = mean((out - t)^2) and d out = 2 (out - t) / numel in one pass
        loss = torch.empty((), dtype=dt, device=dev)
        d_out = torch.empty_like(out)
        self._mse_into(loss, d_out, out, target)
        work_a = None
        if self.comm_stream is None or self._order != "w1_first":
            self._timed(self._mm_into, self.dw2, d_out.t(), a)
            self._colsum_into(self.db2, d_out)
            if self.comm_stream is not None:
                ev = torch.cuda.Event()
                ev.record()
                work_a = self._allreduce_async(self.bucket_a, ev)
        # d_h = gelu_backward(d_out W2, h) from one product
        d_h = torch.empty((B, H), dtype=dt, device=dev)
        beside = self._beside_collective() if work_a is not None else contextlib.nullcontext()
        with beside:
            self._timed(self._gemm_epilogue, N.EPI_GELU_BACKWARD, d_h, h, d_out, self.w2)
        if self.trace is not None:
            self.trace.update(x=x, t=target, h=h, a=a, out=out, d_out=d_out, d_h=d_h, loss=loss)
        if self.comm_stream is None:
            self._timed(self._mm_into, self.dw1, d_h.t(), x)
            self._colsum_into(self.db1, d_h)
            # SGD: p += -lr * g over the whole flat buffer
            ops.add__Tensor(self.param_flat, self.grad_flat, alpha=-cfg.lr)
            return loss
        if self._order == "w1_first":
            return self._backward_w1_first(x, a, d_out, d_h, loss)
        # Bucket B in row slices of dW1 (db1 travels with the first); each
        # slice's SUM all-reduce starts once its product is done.
        self._colsum_into(self.db1, d_h)
        pending = self._dw1_sliced(d_h, x, beside_from=0)
        # SGD: p += (-lr / world) * g_sum, bucket A as soon as it is in.
        work_a.wait()
        ops.add__Tensor(self.params_a, self.bucket_a, alpha=self._sgd_scale())
        self._pending = pending
        if not cfg.overlap_next_step:
            self.flush()
        return loss

    def _sgd_scale(self) -> float:
        return -self.cfg.lr / self.world

    def _apply_pending_a(self) -> None:
        if self._pending_a is not None:
            self._pending_a.wait()
            ops.add__Tensor(self.params_a, self.bucket_a, alpha=self._sgd_scale())
            self._pending_a = None

    def _backward_w1_first(self, x, a, d_out, d_h, loss):
        """dW1 (bucket B's exchange beside dW2), then dW2 (bucket A's exchange
        beside the next step's first product)."""
        self._colsum_into(self.db1, d_h)
        pending_b = self._dw1_sliced(d_h, x, beside_from=1)
        self._timed(self._dw2_beside, d_out, a)
        self._colsum_into(self.db2, d_out)
        ev = torch.cuda.Event()
        ev.record()
        self._pending_a = self._allreduce_async(self.bucket_a, ev)
        for start, length, work in pending_b:
            work.wait()
            ops.add__Tensor(self.params_b.narrow(0, start, length), self.bucket_b.narrow(0, start, length),
                            alpha=self._sgd_scale())
        if not self.cfg.overlap_next_step:
            self._apply_pending_a()
        return loss

    def flush(self) -> None:
        """Apply every SGD update still pending (the last step's, with
        overlap_next_step); a no-op otherwise."""
        self._apply_pending_a()
        for start, length, work in self._pending:
            work.wait()
            ops.add__Tensor(self.params_b.narrow(0, start, length), self.bucket_b.narrow(0, start, length),
                            alpha=self._sgd_scale())
        self._pending = []

    def _forward_sliced(self, x, h, a):
        """h = x W1^T + b1 and a = gelu(h) in the column slices matching the
        pending bucket-B slices, each after its slice's update."""
        for (start, length, work), (r0, r1) in zip(self._pending, self._slices):
            work.wait()
            ops.add__Tensor(self.params_b.narrow(0, start, length), self.bucket_b.narrow(0, start, length),
                            alpha=self._sgd_scale())
            self._gemm_epilogue(N.EPI_GELU, a[:, r0:r1], h[:, r0:r1], x, self.w1[r0:r1].t(), self.b1[r0:r1])
        self._pending = []

    def _first_beside(self, i: int):
        return self._beside_collective() if i == 0 else contextlib.nullcontext()

    def _forward_beside(self, x, h, a):
        """h = x W1^T + b1 and a = gelu(h) in `beside_slices` row slices of
        the batch, the first beside the exchange in flight."""
        for i, (r0, r1) in enumerate(row_slices(x.shape[0], self._beside_slices)):
            with self._first_beside(i):
                self._gemm_epilogue(N.EPI_GELU, a[r0:r1], h[r0:r1], x[r0:r1], self.w1.t(), self.b1)

    def _dw2_beside(self, d_out, a):
        """dW2 = d_out^T a in `beside_slices` row slices of dW2, the first
        beside the exchange in flight."""
        for i, (r0, r1) in enumerate(row_slices(self.cfg.d_in, self._beside_slices)):
            with self._first_beside(i):
                self._mm_into(self.dw2[r0:r1], d_out[:, r0:r1].t(), a)

    def _dw1_sliced(self, d_h, x, beside_from: int = 0):
        """dW1 = d_h^T x in row slices (one timed GEMM region), each slice's
        all-reduce issued as soon as the slice is written; slices from
        `beside_from` on run beside a collective.  Returns the slices as
        (offset in bucket B, length, work)."""
        pending = []
        start = end = None
        if self.gemm_events is not None:
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record()
        for i, (r0, r1, lo, length) in enumerate(self._bucket_b_slices):
            with self._beside_collective() if i >= beside_from else contextlib.nullcontext():
                self._mm_into(self.dw1[r0:r1], d_h[:, r0:r1].t(), x)
            ev = torch.cuda.Event()
            ev.record()
            pending.append((lo, length, self._allreduce_async(self.bucket_b.narrow(0, lo, length), ev)))
        if start is not None:
            end.record()
            self.gemm_events.append((start, end))
        return pending

    def gemm_names(self):
        """The step's products in the order their timing events are recorded."""
        h, o, w2, dh, w1 = ("h=xW1^T", "out=aW2^T", "dW2=dout^T a", "dh=gelu'(dout W2)", "dW1=dh^T x")
        if self.comm_stream is not None and self._order == "w1_first":
            return (h, o, dh, w1, w2)
        return (h, o, w2, dh, w1)

    def flops_per_step(self) -> float:
        """Five GEMMs of 2 * B * D * H each (forward 2, backward 3, no dX)."""
        c = self.cfg
        return 5 * 2.0 * c.batch * c.d_in * c.d_hidden
