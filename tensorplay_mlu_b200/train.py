"""Data-parallel MLP training step on the B200 backend.

The model of tensorplay-mlu's README distributed benchmark, at the sizes the
B200 build is measured on: Linear(4096 -> 16384), GELU, Linear(16384 -> 4096),
bf16 weights with PyTorch's nn.Linear initialisation (Kaiming-uniform, bound
1/sqrt(fan_in)) from seed 0, loss = mean((out - target)^2), full backward
(no input gradient) and an SGD update.  Every step is a sequence of the
backend's own operators -- the ones TensorPlay's autograd engine would call
for this model (linear, gelu, sub, pow, mean, mul, mm on transposed views,
sum over dim 0, gelu_backward, add_) -- so the step exercises the claimed
kernels end to end.

Data parallelism (one rank per GPU): gradients live in one flat buffer split
into two buckets in backward order, (dW2, db2) then (dW1, db1).  Each bucket
is all-reduced (SUM) on a side stream as soon as backward has produced it,
so the first exchange overlaps the dh / dW1 GEMMs (the GEMM running beside
it leaves `comm_sms` SMs to the collective's kernels); the AVG's 1/world scale is
folded into the SGD step (p -= lr/world * g_sum), not launched as its own
pass as tensorplay_mlu/distributed.py:241-242 does.
"""

from __future__ import annotations

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
    # Data-parallel: the last gradient bucket (dW1, db1) is produced and
    # all-reduced in this many row slices, so each slice's exchange overlaps
    # the next slice's GEMM.
    dw1_slices: int = 1
    # Data-parallel: SMs left free for the collective's kernels while the
    # d_a GEMM overlaps the first bucket's all-reduce (the GEMM is persistent
    # with statically scheduled tiles, so SMs taken by the collective would
    # otherwise delay its last tiles).  0: the GEMM takes every SM.
    comm_sms: int = 32


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


class DataParallelMLP:
    """Parameters, gradient buckets and the training step of one rank."""

    def __init__(self, cfg: MLPConfig, device: int = 0, pg=None, host_params=None):
        self.cfg = cfg
        self.device = torch.device("cuda", device)
        self.pg = pg
        self.world = pg.size() if pg is not None else 1
        w1, b1, w2, b2 = host_params if host_params is not None else init_params_host(cfg)
        dev = self.device
        # Parameters.
        self.w1 = ops.to_device(w1, dev)
        self.b1 = ops.to_device(b1, dev)
        self.w2 = ops.to_device(w2, dev)
        self.b2 = ops.to_device(b2, dev)
        # One flat gradient buffer, bucket A = (dW2, db2), bucket B = (dW1, db1).
        H, D = cfg.d_hidden, cfg.d_in
        n_a = D * H + D
        n_b = H * D + H
        self.grad_flat = torch.empty(n_a + n_b, dtype=cfg.dtype, device=dev)
        self.bucket_a = self.grad_flat.narrow(0, 0, n_a)
        self.bucket_b = self.grad_flat.narrow(0, n_a, n_b)
        self.dw2 = self.bucket_a.narrow(0, 0, D * H).view(D, H)
        self.db2 = self.bucket_a.narrow(0, D * H, D)
        self.dw1 = self.bucket_b.narrow(0, 0, H * D).view(H, D)
        self.db1 = self.bucket_b.narrow(0, H * D, H)
        self.comm_stream = torch.cuda.Stream(device=dev) if pg is not None and self.world > 1 else None
        # TPB200_COMM_SMS overrides cfg.comm_sms (A/B measurements).
        reserve = int(os.environ.get("TPB200_COMM_SMS", cfg.comm_sms))
        total = torch.cuda.get_device_properties(dev).multi_processor_count
        self._overlap_sms = total - reserve if self.comm_stream is not None and 0 < reserve < total else 0
        # When a list, every GEMM of the step appends a (start, end) pair of
        # CUDA events recorded around its launch on the current stream.
        self.gemm_events: Optional[list] = None
        # When a dict, the step stores its intermediates in it (for checks).
        self.trace: Optional[dict] = None

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

    def _gemm_sm_limit(self, sms: int) -> None:
        N.check(N.lib().tp_b200_set_gemm_sm_limit(self.device.index, sms), "set_gemm_sm_limit")

    def _allreduce_async(self, bucket, ready_event):
        """SUM all-reduce of ``bucket`` on the comm stream after ``ready_event``."""
        self.comm_stream.wait_event(ready_event)
        with torch.cuda.stream(self.comm_stream):
            work = self.pg.allreduce([bucket], op=0)
        return work

    def step(self, x: torch.Tensor, target: torch.Tensor) -> torch.Tensor:
        """One forward + backward + SGD step; returns the loss (device 0-d tensor)."""
        cfg = self.cfg
        # forward
        h = self._timed(ops.linear, x, self.w1, self.b1)
        a = ops.gelu(h)
        out = self._timed(ops.linear, a, self.w2, self.b2)
        diff = ops.sub_Tensor(out, target)
        loss = ops.mean(ops.pow_Tensor_Scalar(diff, 2))
        # backward of mean((out - t)^2): d out = 2 (out - t) / numel
        d_out = ops.mul_Scalar(diff, 2.0 / diff.numel())
        self._timed(self._mm_into, self.dw2, d_out.t(), a)
        self._colsum_into(self.db2, d_out)
        work_a = None
        if self.comm_stream is not None:
            ev = torch.cuda.Event()
            ev.record()
            work_a = self._allreduce_async(self.bucket_a, ev)
        if self._overlap_sms:
            self._gemm_sm_limit(self._overlap_sms)
            try:
                d_a = self._timed(ops.mm, d_out, self.w2)
            finally:
                self._gemm_sm_limit(0)
        else:
            d_a = self._timed(ops.mm, d_out, self.w2)
        d_h = ops.gelu_backward(d_a, h)
        if self.trace is not None:
            self.trace.update(x=x, t=target, h=h, a=a, out=out, d_out=d_out, d_a=d_a, d_h=d_h, loss=loss)
        if self.comm_stream is None:
            self._timed(self._mm_into, self.dw1, d_h.t(), x)
            self._colsum_into(self.db1, d_h)
            # SGD: p += -lr * g
            for p, g in zip(self.params(), self.grads()):
                ops.add__Tensor(p, g, alpha=-cfg.lr)
            return loss
        # Bucket B in row slices of dW1 (db1 travels with the last slice);
        # each slice's SUM all-reduce starts once its GEMM is done.
        self._colsum_into(self.db1, d_h)
        works_b = self._dw1_sliced(d_h, x)
        # SGD: p += (-lr / world) * g_sum, W2/b2 as soon as bucket A is in.
        scale = -cfg.lr / self.world
        work_a.wait()
        ops.add__Tensor(self.w2, self.dw2, alpha=scale)
        ops.add__Tensor(self.b2, self.db2, alpha=scale)
        for w in works_b:
            w.wait()
        ops.add__Tensor(self.w1, self.dw1, alpha=scale)
        ops.add__Tensor(self.b1, self.db1, alpha=scale)
        return loss

    def _dw1_sliced(self, d_h, x):
        """dW1 = d_h^T x as `dw1_slices` row slices (one timed GEMM region),
        each slice's all-reduce issued as soon as the slice is written."""
        H, D = self.cfg.d_hidden, self.cfg.d_in
        n = max(1, int(self.cfg.dw1_slices))
        bounds = [(H * i // n) // 8 * 8 for i in range(n)] + [H]  # 16-byte-aligned column offsets of d_h
        works = []
        start = end = None
        if self.gemm_events is not None:
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record()
        for i in range(n):
            r0, r1 = bounds[i], bounds[i + 1]
            self._mm_into(self.dw1[r0:r1], d_h[:, r0:r1].t(), x)
            ev = torch.cuda.Event()
            ev.record()
            length = (r1 - r0) * D if i < n - 1 else self.bucket_b.numel() - r0 * D  # + db1
            works.append(self._allreduce_async(self.bucket_b.narrow(0, r0 * D, length), ev))
        if start is not None:
            end.record()
            self.gemm_events.append((start, end))
        return works

    def flops_per_step(self) -> float:
        """Five GEMMs of 2 * B * D * H each (forward 2, backward 3, no dX)."""
        c = self.cfg
        return 5 * 2.0 * c.batch * c.d_in * c.d_hidden
