"""CPU oracle for the B200 backend's operators -- TEST INFRASTRUCTURE ONLY.

Python face of ``oracle.c`` / ``mlp.c`` (see the header of oracle.c for what
is restated from the reference and how it is pinned).  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm
may import this package, and only as the checker or the timed CPU path --
never as part of the product.

Inputs and outputs are host (CPU) torch tensors; any strides are accepted.
Operator codes are the C ABI's (``include/tpb200.h``).
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIBRARY = os.path.join(HERE, "liboracle.so")
MAX_DIMS = 8

DTYPE_CODES = {
    torch.uint8: 0, torch.int8: 1, torch.int16: 2, torch.int32: 3, torch.int64: 4,
    torch.float16: 5, torch.float32: 6, torch.bfloat16: 7, torch.float64: 8, torch.bool: 9,
}

ADD, SUB, MUL, DIV, RSUB = range(5)
(EXP, LOG, SQRT, RSQRT, NEG, ABS, POW, RELU, SIGMOID, TANH, SILU, GELU, GELU_TANH,
 SQUARE) = range(14)
(THRESHOLD_BACKWARD, SIGMOID_BACKWARD, TANH_BACKWARD, GELU_BACKWARD, GELU_TANH_BACKWARD,
 SILU_BACKWARD) = range(6)
SUM, MEAN, AMAX, AMIN = range(4)
GEMM_ALLOW_TF32 = 1


class _Desc(ctypes.Structure):
    _fields_ = [
        ("data", ctypes.c_void_p),
        ("dtype", ctypes.c_int32),
        ("ndim", ctypes.c_int32),
        ("sizes", ctypes.c_int64 * MAX_DIMS),
        ("strides", ctypes.c_int64 * MAX_DIMS),
    ]


def _d(t: torch.Tensor) -> _Desc:
    assert t.device.type == "cpu", "the oracle works on host tensors"
    d = _Desc()
    d.data = t.data_ptr() if t.numel() else None
    d.dtype = DTYPE_CODES[t.dtype]
    d.ndim = t.dim()
    for i, (s, st) in enumerate(zip(t.shape, t.stride())):
        d.sizes[i] = s
        d.strides[i] = st
    return d


_LIB = None


def build() -> str:
    """Compile liboracle.so (make -C oracle)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIBRARY


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        if not os.path.isfile(LIBRARY):
            build()
        handle = ctypes.CDLL(LIBRARY)
        T = ctypes.POINTER(_Desc)
        D, I, I64 = ctypes.c_double, ctypes.c_int, ctypes.c_int64
        sig = {
            "orc_copy": [T, T],
            "orc_fill": [T, D, I64],
            "orc_binary": [I, T, T, T, D],
            "orc_binary_scalar": [I, T, T, D, I64, D],
            "orc_unary": [I, T, T, D],
            "orc_unary_backward": [I, T, T, T, D],
            "orc_reduce": [I, T, T, ctypes.c_uint32],
            "orc_softmax": [I, T, T, I],
            "orc_softmax_backward": [I, T, T, T, I],
            "orc_gemm": [T, T, T, T, D, D, I],
            "orc_dropout": [T, T, T, D, ctypes.c_uint64, ctypes.c_uint64],
            "orc_gather": [T, T, T, I],
            "orc_index_select": [T, T, T, I],
            "orc_index_add": [T, T, T, I],
            "orc_scatter": [T, T, T, I, I, I],
            "orc_scan": [I, T, T, I],
            "orc_where": [T, T, T, T],
            "orc_layer_norm": [T, T, T, T, T, T, I64, D],
            "orc_layer_norm_backward": [T, T, T, T, T, T, T, T, I64],
            "orc_nll_loss": [T, T, T, T, T, I, I64],
            "orc_nll_loss_backward": [T, T, T, T, T, I, I64],
            "orc_gemm_sampled": [ctypes.c_void_p, ctypes.c_void_p, I64, T, T, T, D, D, I],
            "orc_mlp_step": [I, I, I, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                             ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_float,
                             ctypes.POINTER(ctypes.c_float)],
            "orc_num_threads": [],
            "orc_set_num_threads": [I],
            "orc_gemm_blocked": [I64, I64, I64, ctypes.c_void_p, I64, I64, ctypes.c_void_p, I64, I64,
                                 ctypes.c_void_p],
        }
        for name, args in sig.items():
            fn = getattr(handle, name)
            fn.argtypes = args
            fn.restype = ctypes.c_int
        _LIB = handle
    return _LIB


def _ok(status: int, what: str) -> None:
    if status != 0:
        raise RuntimeError(f"oracle {what} failed ({status})")


def copy(dst: torch.Tensor, src: torch.Tensor) -> torch.Tensor:
    _ok(lib().orc_copy(_d(dst), _d(src)), "copy")
    return dst


def cast(src: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    return copy(torch.empty(src.shape, dtype=dtype), src)


def fill(dst: torch.Tensor, value) -> torch.Tensor:
    if dst.dtype.is_floating_point:
        _ok(lib().orc_fill(_d(dst), float(value), 0), "fill")
    else:
        _ok(lib().orc_fill(_d(dst), float(int(value)), int(value)), "fill")
    return dst


def binary(op: int, a: torch.Tensor, b: torch.Tensor, alpha=1.0) -> torch.Tensor:
    assert a.dtype == b.dtype
    out = torch.empty(torch.broadcast_shapes(a.shape, b.shape), dtype=a.dtype)
    _ok(lib().orc_binary(op, _d(out), _d(a), _d(b), float(alpha)), "binary")
    return out


def binary_scalar(op: int, a: torch.Tensor, s, alpha=1.0) -> torch.Tensor:
    out = torch.empty(a.shape, dtype=a.dtype)
    si = int(s) if not a.dtype.is_floating_point else 0
    _ok(lib().orc_binary_scalar(op, _d(out), _d(a), float(s), si, float(alpha)), "binary_scalar")
    return out


def unary(op: int, x: torch.Tensor, p: float = 0.0) -> torch.Tensor:
    out = torch.empty(x.shape, dtype=x.dtype)
    _ok(lib().orc_unary(op, _d(out), _d(x), float(p)), "unary")
    return out


def unary_backward(op: int, dy: torch.Tensor, z: torch.Tensor, p: float = 0.0) -> torch.Tensor:
    out = torch.empty(dy.shape, dtype=dy.dtype)
    _ok(lib().orc_unary_backward(op, _d(out), _d(dy), _d(z), float(p)), "unary_backward")
    return out


def reduce(op: int, x: torch.Tensor, dims, out_dtype: torch.dtype, keepdim: bool = False) -> torch.Tensor:
    dims = [d % max(x.dim(), 1) for d in (dims if dims is not None else range(x.dim()))]
    if not dims:
        dims = list(range(x.dim()))
    mask = 0
    for d in dims:
        mask |= 1 << d
    keep = [1 if (mask >> i) & 1 else s for i, s in enumerate(x.shape)]
    out = torch.empty(keep, dtype=out_dtype)
    _ok(lib().orc_reduce(op, _d(out), _d(x), mask), "reduce")
    if keepdim:
        return out
    return out.reshape([s for i, s in enumerate(x.shape) if not (mask >> i) & 1])


def softmax(x: torch.Tensor, dim: int, log: bool = False) -> torch.Tensor:
    x = x.contiguous()
    out = torch.empty(x.shape, dtype=x.dtype)
    _ok(lib().orc_softmax(int(log), _d(out), _d(x), dim), "softmax")
    return out


def softmax_backward(dy: torch.Tensor, y: torch.Tensor, dim: int, log: bool = False) -> torch.Tensor:
    dy, y = dy.contiguous(), y.contiguous()
    out = torch.empty(dy.shape, dtype=dy.dtype)
    _ok(lib().orc_softmax_backward(int(log), _d(out), _d(dy), _d(y), dim), "softmax_backward")
    return out


def gemm(a: torch.Tensor, b: torch.Tensor, c=None, alpha=1.0, beta=0.0, flags: int = 0) -> torch.Tensor:
    shape = list(a.shape[:-1]) + [b.shape[-1]]
    if a.dim() == 3:
        shape[0] = max(a.shape[0], b.shape[0])
    out = torch.empty(shape, dtype=a.dtype)
    _ok(lib().orc_gemm(_d(out), _d(a), _d(b), _d(c) if c is not None else None, float(alpha),
                       float(beta), flags), "gemm")
    return out


def gemm_sampled(a: torch.Tensor, b: torch.Tensor, idx: np.ndarray, c=None, alpha=1.0, beta=0.0,
                 flags: int = 0) -> np.ndarray:
    """alpha * (a @ b) + beta * c at the (batch, m, n) rows of ``idx``, in float64."""
    idx = np.ascontiguousarray(idx, dtype=np.int64)
    vals = np.empty(idx.shape[0], dtype=np.float64)
    _ok(lib().orc_gemm_sampled(vals.ctypes.data, idx.ctypes.data, idx.shape[0], _d(a), _d(b),
                               _d(c) if c is not None else None, float(alpha), float(beta), flags),
        "gemm_sampled")
    return vals


def mlp_step(x, t, w1, b1, w2, b2, lr: float) -> float:
    """One SGD step of the BASELINE MLP on bf16 host tensors (weights updated in place)."""
    for tensor in (x, t, w1, b1, w2, b2):
        assert tensor.dtype == torch.bfloat16 and tensor.is_contiguous()
    loss = ctypes.c_float()
    _ok(lib().orc_mlp_step(x.shape[0], x.shape[1], w1.shape[0], x.data_ptr(), t.data_ptr(),
                           w1.data_ptr(), b1.data_ptr(), w2.data_ptr(), b2.data_ptr(), float(lr),
                           ctypes.byref(loss)), "mlp_step")
    return loss.value


def num_threads() -> int:
    return lib().orc_num_threads()


def set_num_threads(n: int) -> None:
    """OpenMP threads of the oracle's parallel loops (torchrun exports
    OMP_NUM_THREADS=1, so the CPU baseline sets its count explicitly)."""
    lib().orc_set_num_threads(int(n))


def gemm_blocked(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """fp32 a @ b through mlp.c's blocked product (any strides)."""
    assert a.dtype == b.dtype == torch.float32 and a.dim() == b.dim() == 2
    out = torch.empty(a.shape[0], b.shape[1], dtype=torch.float32)
    _ok(lib().orc_gemm_blocked(a.shape[0], b.shape[1], a.shape[1], a.data_ptr(), a.stride(0), a.stride(1),
                               b.data_ptr(), b.stride(0), b.stride(1), out.data_ptr()), "gemm_blocked")
    return out


# ---------------------------------------------------------------------- NN

def _stats_dtype(dtype):
    return torch.float64 if dtype == torch.float64 else torch.float32


def _numel(shape):
    n = 1
    for s in shape:
        n *= int(s)
    return n


def layer_norm(x: torch.Tensor, normalized_shape, w=None, b=None, eps: float = 1e-5):
    """(y, mean, rstd) of native_layer_norm; mean / rstd flat over the rows."""
    x = x.contiguous()
    D = _numel(normalized_shape)
    rows = x.numel() // D
    y = torch.empty(x.shape, dtype=x.dtype)
    mean = torch.empty([rows], dtype=_stats_dtype(x.dtype))
    rstd = torch.empty([rows], dtype=_stats_dtype(x.dtype))
    _ok(lib().orc_layer_norm(_d(y), _d(mean), _d(rstd), _d(x), _d(w.contiguous()) if w is not None else None,
                             _d(b.contiguous()) if b is not None else None, D, float(eps)), "layer_norm")
    return y, mean, rstd


def layer_norm_backward(dy, x, normalized_shape, mean, rstd, w=None):
    """(dx, dweight, dbias) of native_layer_norm_backward."""
    x, dy = x.contiguous(), dy.contiguous()
    D = _numel(normalized_shape)
    dx = torch.empty(x.shape, dtype=x.dtype)
    dw = torch.empty(list(normalized_shape), dtype=x.dtype)
    db = torch.empty(list(normalized_shape), dtype=x.dtype)
    _ok(lib().orc_layer_norm_backward(_d(dx), _d(dw), _d(db), _d(dy), _d(x), _d(mean.contiguous()),
                                      _d(rstd.contiguous()), _d(w.contiguous()) if w is not None else None, D),
        "layer_norm_backward")
    return dx, dw, db


def nll_loss(x: torch.Tensor, target: torch.Tensor, w=None, reduction: int = 1, ignore_index: int = -100):
    """(output, total_weight) of nll_loss."""
    out = torch.empty([x.shape[0]] if reduction == 0 else [], dtype=x.dtype)
    total = torch.empty([], dtype=x.dtype)
    _ok(lib().orc_nll_loss(_d(out), _d(total), _d(x), _d(target), _d(w) if w is not None else None,
                           int(reduction), int(ignore_index)), "nll_loss")
    return out, total


def nll_loss_backward(dy, x, target, w, reduction, ignore_index, total):
    dx = torch.empty(x.shape, dtype=x.dtype)
    _ok(lib().orc_nll_loss_backward(_d(dx), _d(dy.contiguous()), _d(target), _d(w) if w is not None else None,
                                    _d(total), int(reduction), int(ignore_index)), "nll_loss_backward")
    return dx


# -------------------------------------------------------------------- index

SCATTER_MODES = {None: 0, "add": 1, "sum": 1, "multiply": 2, "prod": 2, "amax": 3, "amin": 4, "mean": 5}


def gather(self: torch.Tensor, dim: int, index: torch.Tensor) -> torch.Tensor:
    out = torch.empty(index.shape, dtype=self.dtype)
    _ok(lib().orc_gather(_d(out), _d(self), _d(index), dim % max(self.dim(), 1)), "gather")
    return out


def index_select(self: torch.Tensor, dim: int, index: torch.Tensor) -> torch.Tensor:
    x = self.contiguous()
    d = dim % max(self.dim(), 1)
    shape = list(self.shape)
    shape[d] = index.numel()
    out = torch.empty(shape, dtype=self.dtype)
    _ok(lib().orc_index_select(_d(out), _d(x), _d(index.reshape(-1)), d), "index_select")
    return out


def index_add_zeros(shape, dim: int, index: torch.Tensor, src: torch.Tensor) -> torch.Tensor:
    out = torch.zeros(shape, dtype=src.dtype)
    _ok(lib().orc_index_add(_d(out), _d(src.contiguous()), _d(index.reshape(-1)), dim % max(len(shape), 1)),
        "index_add")
    return out


def scatter(self: torch.Tensor, dim: int, index: torch.Tensor, src: torch.Tensor, reduce=None,
            include_self: bool = True) -> torch.Tensor:
    out = self.clone().contiguous()
    _ok(lib().orc_scatter(_d(out), _d(index), _d(src), dim % max(self.dim(), 1), SCATTER_MODES[reduce],
                          int(include_self)), "scatter")
    return out


def scan(x: torch.Tensor, dim: int, product: bool = False) -> torch.Tensor:
    x = x.contiguous()
    out = torch.empty(x.shape, dtype=x.dtype)
    _ok(lib().orc_scan(int(product), _d(out), _d(x), dim % max(x.dim(), 1)), "scan")
    return out


def where(cond: torch.Tensor, a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    out = torch.empty(torch.broadcast_shapes(cond.shape, a.shape, b.shape), dtype=a.dtype)
    _ok(lib().orc_where(_d(out), _d(cond), _d(a), _d(b)), "where")
    return out


# ------------------------------------------------------------------ dropout

def philox4x32_10(ctr, key):
    """Philox-4x32-10 block for four 32-bit counter words and two key words."""
    c = (ctypes.c_uint32 * 4)(*ctr)
    k = (ctypes.c_uint32 * 2)(*key)
    out = (ctypes.c_uint32 * 4)()
    fn = lib().orc_philox4x32_10
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    fn.restype = None
    fn(ctypes.addressof(c), ctypes.addressof(k), ctypes.addressof(out))
    return list(out)


def dropout(x: torch.Tensor, p: float, seed: int, offset: int = 0):
    """(output, mask) of the device dropout kernel's element -> random-word mapping."""
    x = x.contiguous()
    out = torch.empty(x.shape, dtype=x.dtype)
    mask = torch.empty(x.shape, dtype=torch.bool)
    _ok(lib().orc_dropout(_d(out), _d(mask), _d(x), float(p), int(seed), int(offset)), "dropout")
    return out, mask
