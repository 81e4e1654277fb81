"""The operators the B200 backend claims, one function per registered schema.

This is the host-side mirror of tensorplay-mlu's operator registrations
(``TENSORPLAY_LIBRARY_IMPL(PrivateUse1, ...)`` blocks in
tensorplay_mlu/csrc/CopyKernels.cpp:349-364, BinaryKernels.cpp:252-269,
UnaryKernels.cpp:291-310, ReduceKernels.cpp:267-282, BlasKernels.cpp:416-422):
the same operator names (``KERNELS`` maps each schema name to its function),
argument meaning, dtype rules and error behaviour.  Each function decides
shapes and dtypes on the host and runs one or more sm_100a kernels through the
C ABI (``include/tpb200.h``); none of them computes on the host.  Where the
reference falls back to the host (integers, float64, unsupported casts) these
run on the device too.

Device tensors are PyTorch CUDA tensors standing in for TensorPlay
PrivateUse1 tensors; a host tensor is a CPU tensor.  Kernels are enqueued on
PyTorch's current stream of the tensor's device.
"""

from __future__ import annotations

import ctypes
import math
from typing import Optional, Sequence

import torch

from . import _native as N
from ._native import describe

__all__ = ["KERNELS"]


# ------------------------------------------------------------------ helpers

def _lib():
    return N.lib()


def _stream(t: torch.Tensor) -> int:
    return N.stream_of(t.device)


def _is_device(t) -> bool:
    return isinstance(t, torch.Tensor) and t.is_cuda


def _is_host_scalar(t) -> bool:
    """A 0-d host tensor (BinaryKernels.cpp:25-27 is_host_scalar)."""
    return isinstance(t, torch.Tensor) and not t.is_cuda and t.numel() == 1 and t.dim() == 0


def _default_float() -> torch.dtype:
    return torch.get_default_dtype()


def _is_float(dtype: torch.dtype) -> bool:
    return dtype.is_floating_point


def _is_integral(dtype: torch.dtype, include_bool: bool = True) -> bool:
    if dtype == torch.bool:
        return include_bool
    return not dtype.is_floating_point and not dtype.is_complex


def _empty(shape, dtype, device) -> torch.Tensor:
    return torch.empty(tuple(shape), dtype=dtype, device=device)


def _require_device(*tensors) -> None:
    for t in tensors:
        if not _is_device(t):
            raise RuntimeError(f"expected a {'b200'} device tensor, got {getattr(t, 'device', type(t))}")


def _to_dtype(t: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """``t`` converted on its device (CopyKernels.cpp:268-273 to_dtype)."""
    if t.dtype == dtype:
        return t
    out = _empty(t.shape, dtype, t.device)
    if out.numel():
        N.check(_lib().tp_b200_copy(describe(out), describe(t), _stream(t)), "cast")
    return out


def _dense(t: torch.Tensor) -> torch.Tensor:
    """``t`` itself when contiguous, otherwise a contiguous device copy."""
    return t if t.is_contiguous() else clone(t)


def _scalar_value(v):
    if isinstance(v, torch.Tensor):
        return v.item()
    return v


def _scalar_args(value, dtype: torch.dtype):
    """(double, int64) forms of a scalar for a kernel computing in ``dtype``."""
    value = _scalar_value(value)
    if _is_integral(dtype):
        return float(int(value)), int(value)
    return float(value), 0


def binary_result_dtype(a, b) -> torch.dtype:
    """Promotion of two tensor operands (Cnnl.cpp:178-192 binary_result_dtype):
    a dimensioned operand's dtype wins over a 0-d one of the same kind (and a
    floating full tensor over an integral 0-d one); otherwise the usual
    promotion."""
    if a.dtype == b.dtype:
        return a.dtype
    a_scalar, b_scalar = a.dim() == 0, b.dim() == 0
    if a_scalar != b_scalar:
        full, scalar = (b, a) if a_scalar else (a, b)
        same_kind = (_is_float(full.dtype) == _is_float(scalar.dtype)
                     and (full.dtype == torch.bool) == (scalar.dtype == torch.bool))
        if same_kind or (_is_float(full.dtype) and not _is_float(scalar.dtype)):
            return full.dtype
    return torch.promote_types(a.dtype, b.dtype)


def scalar_result_dtype(dtype: torch.dtype, value) -> torch.dtype:
    """Result dtype of ``tensor (op) python scalar``."""
    value = _scalar_value(value)
    if isinstance(value, bool):
        return dtype
    if isinstance(value, float) and not _is_float(dtype):
        return _default_float()
    if isinstance(value, int) and dtype == torch.bool:
        return torch.int64
    return dtype


def _check_inplace(self_dtype: torch.dtype, result: torch.dtype) -> None:
    if not torch.can_cast(result, self_dtype):
        raise RuntimeError(f"result type {str(result).split('.')[-1].capitalize()} can't be cast to "
                           f"the desired output type {str(self_dtype).split('.')[-1].capitalize()}")


# --------------------------------------------------------- copy / factories

def empty(size, dtype: Optional[torch.dtype] = None, device=None, pin_memory: bool = False,
          **_ignored) -> torch.Tensor:
    """``empty`` (CopyKernels.cpp:301-307)."""
    if pin_memory:
        raise RuntimeError("B200 tensors cannot be pinned host memory")
    if any(int(s) < 0 for s in size):
        raise RuntimeError(f"negative dimension in requested size {tuple(size)}")
    return _empty(size, dtype or _default_float(), device if device is not None else "cuda")


def empty_memory_format(size, dtype=None, layout=None, device=None, pin_memory=None,
                        memory_format=None) -> torch.Tensor:
    """``empty.memory_format`` (CopyKernels.cpp:309-316)."""
    return empty(size, dtype, device, bool(pin_memory))


def empty_like(self: torch.Tensor, dtype: Optional[torch.dtype] = None, device=None) -> torch.Tensor:
    """``empty_like`` (CopyKernels.cpp:318-325): a host device keeps the host."""
    return torch.empty(self.shape, dtype=dtype or self.dtype,
                       device=device if device is not None else self.device)


def full_like(self: torch.Tensor, value, dtype=None, device=None) -> torch.Tensor:
    """``full_like`` (CopyKernels.cpp:327-334): allocate, then fill on the result's device."""
    result = empty_like(self, dtype, device)
    if result.is_cuda:
        fill_(result, value)
    else:
        result.fill_(value)
    return result


def zeros_like(self, dtype=None, device=None) -> torch.Tensor:
    return full_like(self, 0, dtype, device)


def ones_like(self, dtype=None, device=None) -> torch.Tensor:
    return full_like(self, 1, dtype, device)


def fill_(self: torch.Tensor, value) -> torch.Tensor:
    """``fill_.Scalar`` on the device for every dtype (CopyKernels.cpp:266-299
    stages float64 and 16-bit-plus integer fills through the host)."""
    _require_device(self)
    if self.numel() == 0:
        return self
    value = _scalar_value(value)
    if self.dtype == torch.bool:
        fv, iv = float(bool(value)), int(bool(value))
    elif _is_integral(self.dtype):
        fv, iv = float(int(value)), int(value)
    else:
        fv, iv = float(value), 0
    N.check(_lib().tp_b200_fill(describe(self), fv, iv, _stream(self)), "fill_")
    return self


def zero_(self: torch.Tensor) -> torch.Tensor:
    return fill_(self, 0)


def clone(self: torch.Tensor, memory_format=None) -> torch.Tensor:
    """``clone`` (CopyKernels.cpp:303-308): dense copy on the device."""
    out = _empty(self.shape, self.dtype, self.device)
    if out.numel():
        N.check(_lib().tp_b200_copy(describe(out), describe(self), _stream(self)), "clone")
    return out


def contiguous(self: torch.Tensor, memory_format=None) -> torch.Tensor:
    return self if self.is_contiguous() else clone(self)


def _host_to_device(self: torch.Tensor, src: torch.Tensor) -> None:
    # Only dense source bytes cross PCIe; broadcast, cast and strides are
    # applied on the device (CopyKernels.cpp:169-184 does them on the host).
    host = src if src.is_contiguous() else src.contiguous()
    staging = self if (self.is_contiguous() and host.dtype == self.dtype
                       and tuple(host.shape) == tuple(self.shape)) else \
        _empty(host.shape, host.dtype, self.device)
    nbytes = host.numel() * host.element_size()
    dev = self.device.index if self.device.index is not None else torch.cuda.current_device()
    N.check(_lib().tp_b200_memcpy(staging.data_ptr(), host.data_ptr(), nbytes, 1, dev, -1,
                                  _stream(self), 1), "copy_ host->device")
    if staging is not self:
        N.check(_lib().tp_b200_copy(describe(self), describe(staging), _stream(self)), "copy_")


def _device_to_host(self: torch.Tensor, src: torch.Tensor) -> None:
    direct = (self.is_contiguous() and src.is_contiguous() and self.dtype == src.dtype
              and tuple(self.shape) == tuple(src.shape))
    dense = src if direct else _empty(self.shape, self.dtype, src.device)
    if not direct:
        N.check(_lib().tp_b200_copy(describe(dense), describe(src), _stream(src)), "copy_")
    target = self if direct else torch.empty(self.shape, dtype=self.dtype)
    dev = src.device.index if src.device.index is not None else torch.cuda.current_device()
    N.check(_lib().tp_b200_memcpy(target.data_ptr(), dense.data_ptr(),
                                  dense.numel() * dense.element_size(), 2, dev, -1, _stream(src), 1),
            "copy_ device->host")
    if target is not self:
        self.copy_(target)  # host tensor into host tensor


def _device_to_device(self: torch.Tensor, src: torch.Tensor) -> None:
    if self.device == src.device:
        N.check(_lib().tp_b200_copy(describe(self), describe(src), _stream(self)), "copy_")
        return
    # Between devices: dense bytes peer-to-peer over NVLink, then layout/cast
    # on the destination (MLUHooks.cpp:34-37 bounces through the host).
    dense = _dense(src.expand(self.shape) if tuple(src.shape) != tuple(self.shape) else src)
    staging = _empty(dense.shape, dense.dtype, self.device)
    dst_dev, src_dev = self.device.index, dense.device.index
    torch.cuda.current_stream(src.device).synchronize()
    N.check(_lib().tp_b200_memcpy(staging.data_ptr(), dense.data_ptr(),
                                  dense.numel() * dense.element_size(), 3, dst_dev, src_dev,
                                  _stream(self), 0), "copy_ peer")
    N.check(_lib().tp_b200_copy(describe(self), describe(staging), _stream(self)), "copy_")


def copy_(self: torch.Tensor, src: torch.Tensor, non_blocking: bool = False) -> torch.Tensor:
    """``copy_`` between the device and the host, or on / between devices
    (CopyKernels.cpp:236-264 copy_kernel)."""
    if self.numel() == 0:
        return self
    if not (self.is_cuda or self.device.type == "cpu") or not (src.is_cuda or src.device.type == "cpu"):
        raise RuntimeError(f"B200 copies run between B200 devices and the host, not "
                           f"{src.device} -> {self.device}")
    if self.is_cuda and src.is_cuda:
        _device_to_device(self, src)
    elif self.is_cuda:
        _host_to_device(self, src)
    elif src.is_cuda:
        _device_to_host(self, src)
    else:
        self.copy_(src)
    return self


def to_device(host: torch.Tensor, device="cuda", dtype: Optional[torch.dtype] = None) -> torch.Tensor:
    """``tensor.to(device)``: allocate on the device and ``copy_`` into it."""
    out = _empty(host.shape, dtype or host.dtype, device)
    return copy_(out, host)


def to_host(t: torch.Tensor) -> torch.Tensor:
    """``tensor.cpu()``."""
    out = torch.empty(t.shape, dtype=t.dtype)
    return copy_(out, t)


def item(self: torch.Tensor):
    """``item`` / ``_local_scalar_dense`` (CopyKernels.cpp:341-345): one element to the host."""
    if self.numel() != 1:
        raise RuntimeError("a Tensor with %d elements cannot be converted to Scalar" % self.numel())
    return to_host(self.reshape(())).item()


_local_scalar_dense = item


# ------------------------------------------------------------------- binary

def _binary(a, b, alpha, op: int, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """BinaryKernels.cpp:89-146 binary(): broadcasting a (op) alpha*b."""
    a_dev, b_dev = _is_device(a), _is_device(b)
    if not (a_dev or _is_host_scalar(a)) or not (b_dev or _is_host_scalar(b)) or not (a_dev or b_dev):
        raise RuntimeError("expected device tensors (or a 0-d host scalar) as operands")
    anchor = a if a_dev else b
    dtype = binary_result_dtype(a, b)
    if op == N.DIV and _is_integral(dtype):
        dtype = _default_float()
    shape = torch.broadcast_shapes(tuple(a.shape), tuple(b.shape))
    if out is not None:
        _check_inplace(out.dtype, dtype)
        if tuple(out.shape) != tuple(shape):
            raise RuntimeError(f"output with shape {list(out.shape)} doesn't match the broadcast "
                               f"shape {list(shape)}")
    result = out if (out is not None and out.dtype == dtype) else _empty(shape, dtype, anchor.device)
    if result.numel():
        s = _stream(anchor)
        if not a_dev or not b_dev:
            # A host scalar: the scalar form of the kernel on the device operand.
            value = (b if a_dev else a).item()
            x = _to_dtype(a if a_dev else b, dtype)
            fv, iv = _scalar_args(value, dtype)
            if a_dev:
                N.check(_lib().tp_b200_binary_scalar(op, describe(result), describe(x.expand(shape)),
                                                     fv, iv, float(alpha), s), "binary")
            else:
                # s (op) alpha*x
                if op == N.ADD:
                    tmp = x if alpha == 1 else _mul_scalar_into(x, alpha, dtype)
                    N.check(_lib().tp_b200_binary_scalar(N.ADD, describe(result), describe(tmp.expand(shape)),
                                                         fv, iv, 1.0, s), "binary")
                elif op == N.SUB:
                    N.check(_lib().tp_b200_binary_scalar(N.RSUB, describe(result), describe(x.expand(shape)),
                                                         fv, iv, float(alpha), s), "binary")
                else:
                    sc = fill_(_empty((), dtype, anchor.device), value)
                    N.check(_lib().tp_b200_binary(op, describe(result), describe(sc), describe(x),
                                                  float(alpha), s), "binary")
        else:
            N.check(_lib().tp_b200_binary(op, describe(result), describe(_to_dtype(a, dtype)),
                                          describe(_to_dtype(b, dtype)), float(alpha), s), "binary")
    if out is not None and result is not out:
        copy_(out, result)
        return out
    return result


def _mul_scalar_into(x, alpha, dtype):
    out = _empty(x.shape, dtype, x.device)
    fv, iv = _scalar_args(alpha, dtype)
    N.check(_lib().tp_b200_binary_scalar(N.MUL, describe(out), describe(x), fv, iv, 1.0, _stream(x)),
            "mul")
    return out


def add_Tensor(self, other, alpha=1):
    return _binary(self, other, alpha, N.ADD)


def sub_Tensor(self, other, alpha=1):
    return _binary(self, other, alpha, N.SUB)


def mul_Tensor(self, other):
    return _binary(self, other, 1, N.MUL)


def div_Tensor(self, other):
    return _binary(self, other, 1, N.DIV)


def add__Tensor(self, other, alpha=1):
    return _binary(self, other, alpha, N.ADD, out=self)


def sub__Tensor(self, other, alpha=1):
    return _binary(self, other, alpha, N.SUB, out=self)


def mul__Tensor(self, other):
    return _binary(self, other, 1, N.MUL, out=self)


def div__Tensor(self, other):
    return _binary(self, other, 1, N.DIV, out=self)


def _scalar_op(self, other, alpha, op: int, out=None):
    """The .Scalar forms (BinaryKernels.cpp:204-248, one affine transform
    there; one scalar-operand kernel here)."""
    _require_device(self)
    dtype = scalar_result_dtype(self.dtype, other)
    if op == N.DIV and _is_integral(dtype):
        dtype = _default_float()
    if out is not None:
        _check_inplace(out.dtype, dtype)
    result = out if (out is not None and out.dtype == dtype) else _empty(self.shape, dtype, self.device)
    if result.numel():
        fv, iv = _scalar_args(other, dtype)
        N.check(_lib().tp_b200_binary_scalar(op, describe(result), describe(_to_dtype(self, dtype)),
                                             fv, iv, float(_scalar_value(alpha)), _stream(self)),
                "binary_scalar")
    if out is not None and result is not out:
        copy_(out, result)
        return out
    return result


def add_Scalar(self, other, alpha=1):
    return _scalar_op(self, other, alpha, N.ADD)


def sub_Scalar(self, other, alpha=1):
    return _scalar_op(self, other, alpha, N.SUB)


def rsub_Scalar(self, other, alpha=1):
    return _scalar_op(self, other, alpha, N.RSUB)


def mul_Scalar(self, other):
    return _scalar_op(self, other, 1, N.MUL)


def div_Scalar(self, other):
    return _scalar_op(self, other, 1, N.DIV)


def add__Scalar(self, other, alpha=1):
    return _scalar_op(self, other, alpha, N.ADD, out=self)


def mul__Scalar(self, other):
    return _scalar_op(self, other, 1, N.MUL, out=self)


def div__Scalar(self, other):
    return _scalar_op(self, other, 1, N.DIV, out=self)


# -------------------------------------------------------------------- unary

def _unary(op: int, self: torch.Tensor, p: float = 0.0, floating: bool = True,
           out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """UnaryKernels.cpp:29-50 unary<>: integer inputs of the floating ops are
    promoted to the default float type, as the host framework does."""
    _require_device(self)
    x = self
    if floating and not _is_float(x.dtype):
        x = _to_dtype(x, _default_float())
    y = out if out is not None else _empty(x.shape, x.dtype, x.device)
    if y.numel():
        N.check(_lib().tp_b200_unary(op, describe(y), describe(x), float(p), _stream(x)), "unary")
    return y


def exp(self):
    return _unary(N.EXP, self)


def log(self):
    return _unary(N.LOG, self)


def sqrt(self):
    return _unary(N.SQRT, self)


def rsqrt(self):
    return _unary(N.RSQRT, self)


def neg(self):
    if self.dtype == torch.bool:
        raise RuntimeError("Negation, the `-` operator, on a bool tensor is not supported.")
    return _unary(N.NEG, self, floating=False)


def abs(self):
    return _unary(N.ABS, self, floating=False)


def pow_Tensor_Scalar(self, exponent):
    """``pow.Tensor_Scalar`` (UnaryKernels.cpp:140-186)."""
    exponent = _scalar_value(exponent)
    if _is_integral(self.dtype) and not isinstance(exponent, float):
        if exponent < 0:
            raise RuntimeError("Integers to negative integer powers are not allowed.")
        return _unary(N.POW, self, float(exponent), floating=False)
    return _unary(N.POW, self, float(exponent))


def relu(self):
    return _unary(N.RELU, self, floating=False)


def relu_(self):
    return _unary(N.RELU, self, floating=False, out=self)


def sigmoid(self):
    return _unary(N.SIGMOID, self)


def tanh(self):
    return _unary(N.TANH, self)


def silu(self):
    return _unary(N.SILU, self)


def gelu(self, approximate: str = "none"):
    if approximate not in ("none", "tanh"):
        raise RuntimeError(f"approximate argument must be either none or tanh, got {approximate}")
    return _unary(N.GELU_TANH if approximate == "tanh" else N.GELU, self)


def _unary_backward(op: int, grad: torch.Tensor, other: torch.Tensor, p: float = 0.0) -> torch.Tensor:
    """UnaryKernels.cpp:82-104 activation_backward and the *_backward kernels."""
    _require_device(grad, other)
    if tuple(grad.shape) != tuple(other.shape):
        raise RuntimeError("backward: grad_output and input shapes differ")
    dtype = torch.promote_types(grad.dtype, other.dtype)
    dx = _empty(grad.shape, dtype, grad.device)
    if dx.numel():
        N.check(_lib().tp_b200_unary_backward(op, describe(dx), describe(_to_dtype(grad, dtype)),
                                              describe(_to_dtype(other, dtype)), float(p), _stream(grad)),
                "unary_backward")
    return dx


def threshold_backward(grad_output, self, threshold):
    return _unary_backward(N.THRESHOLD_BACKWARD, grad_output, self, float(_scalar_value(threshold)))


def sigmoid_backward(grad_output, output):
    return _unary_backward(N.SIGMOID_BACKWARD, grad_output, output)


def tanh_backward(grad_output, output):
    return _unary_backward(N.TANH_BACKWARD, grad_output, output)


def gelu_backward(grad_output, self, approximate: str = "none"):
    op = N.GELU_TANH_BACKWARD if approximate == "tanh" else N.GELU_BACKWARD
    return _unary_backward(op, grad_output, self)


def silu_backward(grad_output, self):
    return _unary_backward(N.SILU_BACKWARD, grad_output, self)


# ------------------------------------------------------ reductions, softmax

def _dims(self: torch.Tensor, dim) -> list[int]:
    nd = max(self.dim(), 1)
    if dim is None:
        return list(range(self.dim()))
    if isinstance(dim, int):
        dim = [dim]
    dims = []
    for d in dim:
        if not -nd <= d < nd:
            raise IndexError(f"Dimension out of range (expected to be in range of [{-nd}, {nd - 1}], but got {d})")
        dims.append(d % nd if self.dim() else 0)
    if len(set(dims)) != len(dims):
        raise RuntimeError("dim appears multiple times in the list of dims")
    return dims if dims else list(range(self.dim()))


def _reduce(op: int, self: torch.Tensor, dims: Sequence[int], keepdim: bool,
            out_dtype: torch.dtype) -> torch.Tensor:
    """ReduceKernels.cpp:46-95 reduce(): keepdim-shaped result, then a view."""
    _require_device(self)
    mask = 0
    for d in dims:
        mask |= 1 << d
    keep_shape = [1 if (mask >> i) & 1 else s for i, s in enumerate(self.shape)]
    out = _empty(keep_shape, out_dtype, self.device)
    if out.numel():
        N.check(_lib().tp_b200_reduce(op, describe(out), describe(self), mask, _stream(self)), "reduce")
    if keepdim:
        return out
    final = [s for i, s in enumerate(self.shape) if not (mask >> i) & 1]
    return out.view(final)


def _sum_dtype(self, dtype):
    if dtype is not None:
        return dtype
    return torch.int64 if _is_integral(self.dtype) else self.dtype


def _mean_dtype(self, dtype):
    out = dtype or self.dtype
    if not _is_float(out):
        raise RuntimeError("mean(): could not infer output dtype. Input dtype must be either a "
                           f"floating point or complex dtype. Got: {str(out).split('.')[-1].capitalize()}")
    return out


def sum(self, dtype: Optional[torch.dtype] = None):
    """``sum`` (ReduceKernels.cpp:97-103); integral inputs sum into int64."""
    return _reduce(N.SUM, self, list(range(self.dim())), False, _sum_dtype(self, dtype))


def sum_dim_IntList(self, dim, keepdim: bool = False, dtype: Optional[torch.dtype] = None):
    return _reduce(N.SUM, self, _dims(self, dim), keepdim, _sum_dtype(self, dtype))


def mean(self, dtype: Optional[torch.dtype] = None):
    return _reduce(N.MEAN, self, list(range(self.dim())), False, _mean_dtype(self, dtype))


def mean_dim(self, dim, keepdim: bool = False, dtype: Optional[torch.dtype] = None):
    return _reduce(N.MEAN, self, _dims(self, dim), keepdim, _mean_dtype(self, dtype))


def amax(self, dim=(), keepdim: bool = False):
    if self.numel() == 0 and (not dim or any(self.shape[d] == 0 for d in _dims(self, dim))):
        raise RuntimeError("amax(): Expected reduction dim to be specified for input.numel() == 0.")
    return _reduce(N.AMAX, self, _dims(self, dim if dim != () else None), keepdim, self.dtype)


def amin(self, dim=(), keepdim: bool = False):
    if self.numel() == 0 and (not dim or any(self.shape[d] == 0 for d in _dims(self, dim))):
        raise RuntimeError("amin(): Expected reduction dim to be specified for input.numel() == 0.")
    return _reduce(N.AMIN, self, _dims(self, dim if dim != () else None), keepdim, self.dtype)


def _softmax_impl(self: torch.Tensor, dim: int, log: bool) -> torch.Tensor:
    _require_device(self)
    x = self if _is_float(self.dtype) else _to_dtype(self, _default_float())
    y = _empty(x.shape, x.dtype, x.device)
    if y.numel():
        N.check(_lib().tp_b200_softmax(int(log), describe(y), describe(x), int(dim), _stream(x)),
                "softmax")
    return y


def softmax(self, dim: int, dtype: Optional[torch.dtype] = None):
    """``softmax`` (ReduceKernels.cpp:221-224): the result takes ``dtype``."""
    return _softmax_impl(_to_dtype(self, dtype) if dtype is not None else self, dim, False)


def log_softmax(self, dim: int, dtype: Optional[torch.dtype] = None):
    return _softmax_impl(_to_dtype(self, dtype) if dtype is not None else self, dim, True)


def _softmax(self, dim: int, half_to_float: bool = False):
    return _softmax_impl(_to_dtype(self, torch.float32) if half_to_float else self, dim, False)


def _log_softmax(self, dim: int, half_to_float: bool = False):
    return _softmax_impl(_to_dtype(self, torch.float32) if half_to_float else self, dim, True)


def _softmax_backward_common(grad_output, output, dim, input_dtype, log: bool):
    _require_device(grad_output, output)
    dx = _empty(grad_output.shape, grad_output.dtype, grad_output.device)
    if dx.numel():
        N.check(_lib().tp_b200_softmax_backward(int(log), describe(dx), describe(grad_output),
                                                describe(_to_dtype(output, grad_output.dtype)),
                                                int(dim), _stream(grad_output)), "softmax_backward")
    if input_dtype is not None and input_dtype != dx.dtype:
        return _to_dtype(dx, input_dtype)
    return dx


def _softmax_backward_data(grad_output, output, dim, input_dtype=None):
    return _softmax_backward_common(grad_output, output, dim, input_dtype, False)


def _log_softmax_backward_data(grad_output, output, dim, input_dtype=None):
    return _softmax_backward_common(grad_output, output, dim, input_dtype, True)


# --------------------------------------------------------------------- BLAS

def _gemm_flags(dtype: torch.dtype) -> int:
    """TF32 for fp32 unless the float32 matmul precision is "highest"
    (BlasKernels.cpp:63-66 allow_tf32)."""
    if dtype == torch.float32 and torch.get_float32_matmul_precision() != "highest":
        return N.GEMM_ALLOW_TF32
    return 0


def _gemm(out, a, b, c=None, alpha=1.0, beta=0.0):
    N.check(_lib().tp_b200_gemm(describe(out), describe(a), describe(b),
                                describe(c) if c is not None else None, float(alpha), float(beta),
                                _gemm_flags(out.dtype), _stream(out)), "gemm")
    return out


def _native_pair(a, b, what: str) -> None:
    _require_device(a, b)
    if a.dtype != b.dtype:
        raise RuntimeError(f"{what}: expected m1 and m2 to have the same dtype, but got: "
                           f"{a.dtype} != {b.dtype}")
    if a.device != b.device:
        raise RuntimeError(f"{what}: operands are on different devices")


def mm(self, mat2):
    """``mm`` (BlasKernels.cpp:273-283)."""
    _native_pair(self, mat2, "mm")
    if self.dim() != 2 or mat2.dim() != 2:
        raise RuntimeError("mm: both arguments must be 2-d")
    if self.shape[1] != mat2.shape[0]:
        raise RuntimeError(f"mat1 and mat2 shapes cannot be multiplied ({self.shape[0]}x{self.shape[1]} "
                           f"and {mat2.shape[0]}x{mat2.shape[1]})")
    out = _empty((self.shape[0], mat2.shape[1]), self.dtype, self.device)
    return _gemm(out, self, mat2) if out.numel() else out


def bmm(self, mat2):
    """``bmm`` (BlasKernels.cpp:285-294)."""
    _native_pair(self, mat2, "bmm")
    if self.dim() != 3 or mat2.dim() != 3:
        raise RuntimeError("bmm: both arguments must be 3-d")
    if self.shape[0] != mat2.shape[0] or self.shape[2] != mat2.shape[1]:
        raise RuntimeError("bmm: batch or inner dimensions do not match")
    out = _empty((self.shape[0], self.shape[1], mat2.shape[2]), self.dtype, self.device)
    return _gemm(out, self, mat2) if out.numel() else out


def addmm(self, mat1, mat2, beta=1, alpha=1):
    """``addmm`` (BlasKernels.cpp:296-336): the addend is read in the GEMM
    epilogue instead of being copied into the output first."""
    _native_pair(mat1, mat2, "addmm")
    _require_device(self)
    if mat1.dim() != 2 or mat2.dim() != 2:
        raise RuntimeError("addmm: matrices expected")
    if mat1.shape[1] != mat2.shape[0]:
        raise RuntimeError("addmm: shapes cannot be multiplied")
    if self.dtype != mat1.dtype:
        raise RuntimeError("addmm: self and mat1 must have the same dtype")
    M, Nn = mat1.shape[0], mat2.shape[1]
    torch.broadcast_shapes(tuple(self.shape), (M, Nn))
    out = _empty((M, Nn), mat1.dtype, mat1.device)
    if not out.numel():
        return out
    beta, alpha = _scalar_value(beta), _scalar_value(alpha)
    return _gemm(out, mat1, mat2, self if beta != 0 else None, alpha, beta)


def linear(input, weight, bias=None):
    """``linear`` (BlasKernels.cpp:338-358): input [..., K] @ weight[N, K].t()
    + bias, the weight read transposed in place and the bias added in the
    epilogue."""
    _native_pair(input, weight, "linear")
    if input.dim() == 0 or weight.dim() != 2:
        raise RuntimeError("linear: unsupported operand ranks")
    K, Nn = weight.shape[1], weight.shape[0]
    if input.shape[-1] != K:
        raise RuntimeError(f"linear: mat1 and mat2 shapes cannot be multiplied "
                           f"({input.shape[-1]} and {K})")
    if bias is not None:
        _require_device(bias)
        if bias.dtype != input.dtype:
            raise RuntimeError("linear: bias dtype must match the input")
    rows = input.numel() // max(K, 1) if K else math.prod(input.shape[:-1])
    x2 = _dense(input).reshape(rows, K)
    out = _empty((rows, Nn), input.dtype, input.device)
    if out.numel():
        _gemm(out, x2, weight.t(), bias, 1.0, 1.0 if bias is not None else 0.0)
    return out.reshape(*input.shape[:-1], Nn)


def matmul(self, other):
    """``matmul`` (BlasKernels.cpp:360-412): every case becomes one mm or one
    bmm on dense operands."""
    _native_pair(self, other, "matmul")
    da, db = self.dim(), other.dim()
    if da == 0 or db == 0:
        raise RuntimeError("both arguments to matmul need to be at least 1D")
    if da <= 2 and db <= 2:
        a = self.reshape(1, -1) if da == 1 else self
        b = other.reshape(-1, 1) if db == 1 else other
        if a.shape[1] != b.shape[0]:
            raise RuntimeError("matmul: inner dimensions do not match")
        out = mm(a, b)
        shape = ([a.shape[0]] if da == 2 else []) + ([b.shape[1]] if db == 2 else [])
        return out.reshape(shape)
    if db <= 2 and da >= 3:
        K = self.shape[-1]
        b = other.reshape(-1, 1) if db == 1 else other
        if b.shape[0] != K:
            raise RuntimeError("matmul: inner dimensions do not match")
        out = mm(_dense(self).reshape(-1, K), b)
        shape = list(self.shape[:-1]) + ([b.shape[1]] if db == 2 else [])
        return out.reshape(shape)
    a = self.reshape(1, -1) if da == 1 else self
    b = other.reshape(-1, 1) if db == 1 else other
    M, K, Nn = a.shape[-2], a.shape[-1], b.shape[-1]
    if b.shape[-2] != K:
        raise RuntimeError("matmul: inner dimensions do not match")
    batch = torch.broadcast_shapes(tuple(a.shape[:-2]), tuple(b.shape[:-2]))
    B = math.prod(batch)
    ae = _dense(a.expand(*batch, M, K)).reshape(B, M, K)
    be = _dense(b.expand(*batch, K, Nn)).reshape(B, K, Nn)
    out = bmm(ae, be)
    shape = list(batch) + ([M] if da > 1 else []) + ([Nn] if db > 1 else [])
    return out.reshape(shape)


# ----------------------------------------------------------------------- NN

def _stats_dtype(dtype: torch.dtype) -> torch.dtype:
    """Statistics type of layer_norm (NNKernels.cpp:53-57)."""
    return torch.float64 if dtype == torch.float64 else torch.float32


def _optional(t):
    return t if isinstance(t, torch.Tensor) and t.numel() > 0 else None


def native_layer_norm(input, normalized_shape, weight=None, bias=None, eps: float = 1e-5):
    """``native_layer_norm`` (NNKernels.cpp:59-107): (y, mean, rstd), the
    statistics flat over the leading dimensions, in fp32 for 16-bit inputs."""
    _require_device(input)
    normalized_shape = [int(s) for s in normalized_shape]
    axis = input.dim() - len(normalized_shape)
    if not normalized_shape or axis < 0 or list(input.shape[axis:]) != normalized_shape:
        raise RuntimeError(f"native_layer_norm: normalized_shape {normalized_shape} does not match "
                           f"the trailing dimensions of {list(input.shape)}")
    if not input.dtype.is_floating_point:
        raise RuntimeError(f"native_layer_norm: expected a floating input, got {input.dtype}")
    w, b = _optional(weight), _optional(bias)
    for p in (w, b):
        if p is not None:
            _require_device(p)
            if p.dtype != input.dtype or list(p.shape) != normalized_shape:
                raise RuntimeError("native_layer_norm: weight / bias must have the input dtype and the normalized shape")
    x = _dense(input)
    outer = 1
    for d in input.shape[:axis]:
        outer *= int(d)
    d_norm = 1
    for d in normalized_shape:
        d_norm *= d
    y = _empty(input.shape, input.dtype, input.device)
    sd = _stats_dtype(input.dtype)
    mean = _empty([outer], sd, input.device)
    rstd = _empty([outer], sd, input.device)
    if x.numel():
        N.check(_lib().tp_b200_layer_norm(describe(y), describe(mean), describe(rstd), describe(x),
                                          describe(_dense(w)) if w is not None else None,
                                          describe(_dense(b)) if b is not None else None,
                                          int(d_norm), float(eps), _stream(x)), "native_layer_norm")
    return y, mean, rstd


def native_layer_norm_backward(grad_out, input, normalized_shape, mean, rstd, weight=None, bias=None,
                               output_mask=(True, True, True)):
    """``native_layer_norm_backward`` (NNKernels.cpp:109-161): (dx, dweight,
    dbias), each None where ``output_mask`` says so."""
    _require_device(grad_out, input, mean, rstd)
    normalized_shape = [int(s) for s in normalized_shape]
    if list(grad_out.shape) != list(input.shape):
        raise RuntimeError("native_layer_norm_backward: grad and input shapes differ")
    d_norm = 1
    for d in normalized_shape:
        d_norm *= d
    w = _optional(weight)
    mask = list(output_mask) + [True] * (3 - len(output_mask))
    dx = _empty(input.shape, input.dtype, input.device) if mask[0] else None
    dw = _empty(normalized_shape, input.dtype, input.device) if mask[1] else None
    db = _empty(normalized_shape, input.dtype, input.device) if mask[2] else None
    if input.numel() and (dx is not None or dw is not None or db is not None):
        sd = _stats_dtype(input.dtype)
        N.check(_lib().tp_b200_layer_norm_backward(
            describe(dx) if dx is not None else None, describe(dw) if dw is not None else None,
            describe(db) if db is not None else None, describe(_dense(_to_dtype(grad_out, input.dtype))),
            describe(_dense(input)), describe(_dense(_to_dtype(mean, sd))), describe(_dense(_to_dtype(rstd, sd))),
            describe(_dense(w)) if w is not None else None, int(d_norm), _stream(input)),
            "native_layer_norm_backward")
    elif input.numel() == 0:
        if dw is not None:
            fill_(dw, 0)
        if db is not None:
            fill_(db, 0)
    return dx, dw, db


def _nll_target(target):
    _require_device(target)
    if target.dtype not in (torch.int64, torch.int32):
        raise RuntimeError(f"nll_loss: expected int64 or int32 targets, got {target.dtype}")
    return _dense(target)


def nll_loss(self, target, weight=None, reduction: int = 1, ignore_index: int = -100):
    """``nll_loss`` (NNKernels.cpp:322-360) for (N, C) input and (N) targets:
    (output, total_weight); reduction 0 none, 1 mean, 2 sum.  A target
    outside [0, C) other than ignore_index sets the device error word."""
    _require_device(self)
    if self.dim() != 2 or target.dim() != 1 or target.shape[0] != self.shape[0]:
        raise RuntimeError("nll_loss: expected (N, C) input and (N) targets")
    if reduction not in (0, 1, 2):
        raise RuntimeError(f"nll_loss: reduction must be 0, 1 or 2, got {reduction}")
    t = _nll_target(target)
    w = _optional(weight)
    if w is not None:
        _require_device(w)
        w = _dense(_to_dtype(w, self.dtype))
    out = _empty([self.shape[0]] if reduction == 0 else [], self.dtype, self.device)
    total = _empty([], self.dtype, self.device)
    N.check(_lib().tp_b200_nll_loss(describe(out), describe(total), describe(self), describe(t),
                                    describe(w) if w is not None else None, int(reduction), int(ignore_index),
                                    _stream(self)), "nll_loss")
    return out, total


def nll_loss_backward(grad_output, self, target, weight, reduction: int, ignore_index: int, total_weight):
    """``nll_loss_backward`` (NNKernels.cpp:362-397): d input, zero except at
    each sample's target."""
    _require_device(grad_output, self, total_weight)
    t = _nll_target(target)
    w = _optional(weight)
    if w is not None:
        _require_device(w)
        w = _dense(_to_dtype(w, self.dtype))
    dx = _empty(self.shape, self.dtype, self.device)
    if dx.numel():
        N.check(_lib().tp_b200_nll_loss_backward(
            describe(dx), describe(_dense(_to_dtype(grad_output, self.dtype))), describe(t),
            describe(w) if w is not None else None, describe(_to_dtype(total_weight, self.dtype)),
            int(reduction), int(ignore_index), _stream(self)), "nll_loss_backward")
    return dx


def _dropout_seed() -> int:
    """A 64-bit Philox key drawn from PyTorch's default host generator, so
    torch.manual_seed reproduces the masks."""
    return int(torch.randint(0, 2 ** 62, (1,)).item())


def native_dropout(input, p: float, train=True):
    """``native_dropout`` (NNKernels.cpp:164-196): (output, mask); kept
    elements scaled by 1 / (1 - p)."""
    _require_device(input)
    if not input.dtype.is_floating_point:
        raise RuntimeError(f"native_dropout: expected a floating input, got {input.dtype}")
    if not 0.0 <= p <= 1.0:
        raise RuntimeError(f"native_dropout: probability must be in [0, 1], got {p}")
    if train is False or p == 0.0:
        return clone(input), full_like(input, True, dtype=torch.bool)
    if p == 1.0:
        return zeros_like(input), full_like(input, False, dtype=torch.bool)
    x = _dense(input)
    out = _empty(input.shape, input.dtype, input.device)
    mask = _empty(input.shape, torch.bool, input.device)
    if x.numel():
        N.check(_lib().tp_b200_dropout(describe(out), describe(mask), describe(x), float(p), _dropout_seed(), 0,
                                       _stream(input)), "native_dropout")
    return out, mask


def native_dropout_backward(grad_output, mask, scale: float):
    """``native_dropout_backward`` (NNKernels.cpp:222-236): grad * mask * scale."""
    _require_device(grad_output, mask)
    dx = _empty(grad_output.shape, grad_output.dtype, grad_output.device)
    if dx.numel():
        N.check(_lib().tp_b200_masked_scale(describe(dx), describe(_dense(grad_output)),
                                            describe(_dense(_to_dtype(mask, torch.bool))), float(scale),
                                            _stream(grad_output)), "native_dropout_backward")
    return dx


def embedding(weight, indices, padding_idx: int = -1, scale_grad_by_freq: bool = False, sparse: bool = False):
    """``embedding`` (NNKernels.cpp:242-267): rows of ``weight`` at ``indices``
    (index_select's row-vector copies)."""
    _require_device(weight)
    _index_tensor(indices, "embedding")
    if weight.dim() != 2:
        raise RuntimeError("embedding: weight must be 2-d")
    rows = index_select(weight, 0, indices.reshape(-1))
    return rows.reshape(list(indices.shape) + [weight.shape[1]])


def embedding_dense_backward(grad_output, indices, num_weights: int, padding_idx: int = -1,
                             scale_grad_by_freq: bool = False):
    """``embedding_dense_backward`` (NNKernels.cpp:269-300): gradient rows
    summed into their index (the padding row stays zero); with
    scale_grad_by_freq each row divided by how often its index occurs."""
    _require_device(grad_output)
    _index_tensor(indices, "embedding_dense_backward")
    dim = grad_output.shape[-1]
    g = grad_output.reshape(-1, dim)
    idx = indices.reshape(-1)
    out = index_select_backward(g, [int(num_weights), int(dim)], 0, idx)
    if scale_grad_by_freq:
        ones = full_like(idx, 1, dtype=torch.float32).reshape(-1, 1)
        counts = index_select_backward(ones, [int(num_weights), 1], 0, idx)
        counts = where_self(gt_zero(counts), counts, full_like(counts, 1.0))
        out = div_Tensor(out, _to_dtype(counts, out.dtype))
    if 0 <= padding_idx < num_weights:
        fill_(out[padding_idx], 0)
    return out


def gt_zero(t):
    """t > 0 as bool, on the device (sign test through the unary kernels)."""
    return _to_dtype(relu(t), torch.bool)


def cross_entropy(input, target, weight=None, reduction: int = 1, ignore_index: int = -100):
    """cross_entropy over class dimension 1 of an (N, C) input, as TensorPlay
    composes it: nll_loss(log_softmax(input, 1), target)."""
    return nll_loss(_log_softmax(input, 1), target, weight, reduction, ignore_index)[0]


def layer_norm(input, normalized_shape, weight=None, bias=None, eps: float = 1e-5):
    return native_layer_norm(input, normalized_shape, weight, bias, eps)[0]


# -------------------------------------------------------------------- index

_SCATTER_MODES = {None: 0, "": 0, "add": 1, "sum": 1, "multiply": 2, "prod": 2, "amax": 3, "amin": 4,
                  "mean": 5}


def _index_tensor(index, what):
    _require_device(index)
    if index.dtype not in (torch.int64, torch.int32):
        raise RuntimeError(f"{what}: index must be int64 or int32, got {index.dtype}")
    return index


def _norm_dim(dim: int, nd: int, what: str) -> int:
    n = max(nd, 1)
    if not -n <= dim < n:
        raise IndexError(f"{what}: dimension {dim} out of range for a {nd}-d tensor")
    return dim % n


def gather(self, dim: int, index, sparse_grad: bool = False):
    """``gather`` (IndexKernels.cpp:45-69, 167-172): result shaped like index."""
    _require_device(self)
    _index_tensor(index, "gather")
    d = _norm_dim(dim, self.dim(), "gather")
    out = _empty(index.shape, self.dtype, self.device)
    if out.numel():
        N.check(_lib().tp_b200_gather(describe(out), describe(self), describe(index), d, _stream(self)),
                "gather")
    return out


def _scatter_into(out, dim, index, src, mode: int, include_self: bool, what: str):
    if index.numel():
        N.check(_lib().tp_b200_scatter(describe(out), describe(index), describe(src), int(dim), int(mode),
                                       int(include_self), _stream(out)), what)
    return out


def gather_backward(grad, self, dim: int, index, sparse_grad: bool = False):
    """``gather_backward`` (IndexKernels.cpp:151-182): zeros of self's shape
    accumulating grad at index."""
    _require_device(grad)
    _index_tensor(index, "gather_backward")
    d = _norm_dim(dim, self.dim(), "gather_backward")
    out = zeros_like(self, dtype=grad.dtype)
    return _scatter_into(out, d, index, grad, 1, True, "gather_backward")


def index_select(self, dim: int, index):
    """``index_select`` (IndexKernels.cpp:184-209)."""
    _require_device(self)
    _index_tensor(index, "index_select")
    if index.dim() > 1:
        raise RuntimeError("index_select: index must be 0-d or 1-d")
    d = _norm_dim(dim, self.dim(), "index_select")
    x = _dense(self)
    shape = list(self.shape)
    if shape:
        shape[d] = index.numel()
    out = _empty(shape, self.dtype, self.device)
    if out.numel():
        N.check(_lib().tp_b200_index_select(describe(out), describe(x), describe(index), d, _stream(self)),
                "index_select")
    return out


def index_select_backward(grad, self_sizes, dim: int, index):
    """``index_select_backward`` (IndexKernels.cpp:211-219): zeros of
    self_sizes with grad's slices added at index."""
    _require_device(grad)
    _index_tensor(index, "index_select_backward")
    d = _norm_dim(dim, len(self_sizes), "index_select_backward")
    out = torch.empty(tuple(int(x) for x in self_sizes), dtype=grad.dtype, device=grad.device)
    fill_(out, 0)
    g = _dense(grad)
    if g.numel():
        N.check(_lib().tp_b200_index_add(describe(out), describe(g), describe(index), d, _stream(grad)),
                "index_select_backward")
    return out


def _scatter_common(self, dim, index, src, reduce, include_self, what):
    _require_device(self, src)
    _index_tensor(index, what)
    if reduce not in _SCATTER_MODES:
        raise RuntimeError(f"{what}: unknown reduction {reduce!r}")
    dt = binary_result_dtype(self, src)
    d = _norm_dim(dim, self.dim(), what)
    out = clone(_to_dtype(self, dt))
    if not out.is_contiguous():
        out = contiguous(out)
    return _scatter_into(out, d, index, _to_dtype(src, dt), _SCATTER_MODES[reduce], include_self, what)


def _scatter_inplace(self, dim, index, src, reduce, what):
    _require_device(self, src)
    _index_tensor(index, what)
    if reduce not in _SCATTER_MODES:
        raise RuntimeError(f"{what}: unknown reduction {reduce!r}")
    if binary_result_dtype(self, src) != self.dtype:
        raise RuntimeError(f"{what}: result type {binary_result_dtype(self, src)} can't be cast to {self.dtype}")
    d = _norm_dim(dim, self.dim(), what)
    mode = _SCATTER_MODES[reduce]
    target = self if (mode != 5 or self.is_contiguous()) else contiguous(self)
    _scatter_into(target, d, index, _to_dtype(src, self.dtype), mode, True, what)
    if target is not self:
        copy_(self, target)
    return self


def scatter_add(self, dim: int, index, src):
    """``scatter_add`` (IndexKernels.cpp:221-227)."""
    return _scatter_common(self, dim, index, src, "add", True, "scatter_add")


def scatter_add_(self, dim: int, index, src):
    """``scatter_add_`` (IndexKernels.cpp:229-237)."""
    return _scatter_inplace(self, dim, index, src, "add", "scatter_add_")


def scatter_reduce_op(self, dim: int, index, src, reduce=None):
    """``scatter.reduce`` (IndexKernels.cpp:239-249): replace when reduce is
    None, else add / multiply / amax / amin / mean including self."""
    return _scatter_common(self, dim, index, src, reduce, True, "scatter")


def scatter_reduce_op_(self, dim: int, index, src, reduce=None):
    """``scatter_.reduce`` (IndexKernels.cpp:251-264)."""
    return _scatter_inplace(self, dim, index, src, reduce, "scatter_")


def scatter_reduce(self, dim: int, index, src, reduce: str, include_self: bool = True):
    """``scatter_reduce.two`` (IndexKernels.cpp:266-275): sum / prod / mean /
    amax / amin, with or without self."""
    if reduce not in ("sum", "prod", "mean", "amax", "amin"):
        raise RuntimeError(f"scatter_reduce: reduce must be sum, prod, mean, amax or amin, got {reduce!r}")
    return _scatter_common(self, dim, index, src, reduce, include_self, "scatter_reduce")


def _scan(self, dim, dtype, product: bool, what: str):
    _require_device(self)
    out_dtype = dtype if dtype is not None else self.dtype
    d = _norm_dim(dim, self.dim(), what)
    x = _dense(_to_dtype(self, out_dtype))
    out = _empty(self.shape, out_dtype, self.device)
    if out.numel():
        N.check(_lib().tp_b200_scan(int(product), describe(out), describe(x), d, _stream(self)), what)
    return out


def cumsum(self, dim: int, dtype=None):
    """``cumsum`` (IndexKernels.cpp:277-283): result in ``dtype`` or self's dtype."""
    return _scan(self, dim, dtype, False, "cumsum")


def cumsum_(self, dim: int, dtype=None):
    if dtype is not None and dtype != self.dtype:
        raise RuntimeError("cumsum_: dtype must match the tensor")
    return copy_(self, _scan(self, dim, None, False, "cumsum_"))


def cumprod(self, dim: int, dtype=None):
    """``cumprod`` (IndexKernels.cpp:295-301)."""
    return _scan(self, dim, dtype, True, "cumprod")


def cumprod_(self, dim: int, dtype=None):
    if dtype is not None and dtype != self.dtype:
        raise RuntimeError("cumprod_: dtype must match the tensor")
    return copy_(self, _scan(self, dim, None, True, "cumprod_"))


def where_self(condition, self, other):
    """``where.self`` (IndexKernels.cpp:313-349): broadcast select, operands
    promoted to their common dtype."""
    _require_device(condition, self, other)
    if condition.dtype != torch.bool:
        raise RuntimeError(f"where: expected a bool condition, got {condition.dtype}")
    dt = binary_result_dtype(self, other)
    shape = torch.broadcast_shapes(condition.shape, self.shape, other.shape)
    out = _empty(shape, dt, self.device)
    if out.numel():
        N.check(_lib().tp_b200_where(describe(out), describe(condition), describe(_to_dtype(self, dt)),
                                     describe(_to_dtype(other, dt)), _stream(self)), "where")
    return out


# ---------------------------------------------------------------- registry

# Schema name -> kernel, in the reference's registration order.
KERNELS = {
    # CopyKernels.cpp:350-363
    "empty_like": empty_like,
    "zeros_like": zeros_like,
    "ones_like": ones_like,
    "full_like": full_like,
    "item": item,
    "_local_scalar_dense": _local_scalar_dense,
    "empty": empty,
    "empty.memory_format": empty_memory_format,
    "copy_": copy_,
    "fill_.Scalar": fill_,
    "zero_": zero_,
    "clone": clone,
    "contiguous": contiguous,
    # BinaryKernels.cpp:253-268
    "add.Tensor": add_Tensor,
    "sub.Tensor": sub_Tensor,
    "mul.Tensor": mul_Tensor,
    "div.Tensor": div_Tensor,
    "add_.Tensor": add__Tensor,
    "sub_.Tensor": sub__Tensor,
    "mul_.Tensor": mul__Tensor,
    "div_.Tensor": div__Tensor,
    "add.Scalar": add_Scalar,
    "sub.Scalar": sub_Scalar,
    "rsub.Scalar": rsub_Scalar,
    "mul.Scalar": mul_Scalar,
    "div.Scalar": div_Scalar,
    "add_.Scalar": add__Scalar,
    "mul_.Scalar": mul__Scalar,
    "div_.Scalar": div__Scalar,
    # UnaryKernels.cpp:292-309
    "exp": exp,
    "log": log,
    "sqrt": sqrt,
    "rsqrt": rsqrt,
    "neg": neg,
    "abs": abs,
    "pow.Tensor_Scalar": pow_Tensor_Scalar,
    "relu": relu,
    "relu_": relu_,
    "sigmoid": sigmoid,
    "tanh": tanh,
    "silu": silu,
    "gelu": gelu,
    "threshold_backward": threshold_backward,
    "sigmoid_backward": sigmoid_backward,
    "tanh_backward": tanh_backward,
    "gelu_backward": gelu_backward,
    "silu_backward": silu_backward,
    # ReduceKernels.cpp:268-281
    "sum": sum,
    "sum.dim_IntList": sum_dim_IntList,
    "amax": amax,
    "amin": amin,
    "mean": mean,
    "mean.dim": mean_dim,
    "softmax": softmax,
    "log_softmax": log_softmax,
    "_softmax": _softmax,
    "_log_softmax": _log_softmax,
    "_softmax_backward_data": _softmax_backward_data,
    "_log_softmax_backward_data": _log_softmax_backward_data,
    # BlasKernels.cpp:417-421
    "mm": mm,
    "bmm": bmm,
    "addmm": addmm,
    "matmul": matmul,
    "linear": linear,
    # NNKernels.cpp:399-410 (normalisation and loss)
    "native_layer_norm": native_layer_norm,
    "native_layer_norm_backward": native_layer_norm_backward,
    "nll_loss": nll_loss,
    "nll_loss_backward": nll_loss_backward,
    # IndexKernels.cpp:352-367
    "gather": gather,
    "gather_backward": gather_backward,
    "index_select": index_select,
    "index_select_backward": index_select_backward,
    "scatter_add": scatter_add,
    "scatter_add_": scatter_add_,
    "scatter.reduce": scatter_reduce_op,
    "scatter_.reduce": scatter_reduce_op_,
    "scatter_reduce.two": scatter_reduce,
    "cumsum": cumsum,
    "cumsum_": cumsum_,
    "cumprod": cumprod,
    "cumprod_": cumprod_,
    "where.self": where_self,
    "native_dropout": native_dropout,
    "native_dropout_backward": native_dropout_backward,
    "embedding": embedding,
    "embedding_dense_backward": embedding_dense_backward,
}
