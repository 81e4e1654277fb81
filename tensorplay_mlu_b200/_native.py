"""ctypes binding of ``libtpb200.so`` (declared in ``include/tpb200.h``).

Tensors cross the boundary as ``tpb_tensor`` descriptors: data pointer,
dtype code, rank, sizes and element strides.  Host tensors (torch CPU
tensors standing in for TensorPlay's) and device tensors are described the
same way; which side a pointer lives on is the entry point's contract.
"""

from __future__ import annotations

import ctypes
import os
import threading

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIBRARY_PATH = os.path.join(HERE, "libtpb200.so")
MAX_DIMS = 8

# dtype codes shared with the C ABI (tpb_dtype); 0..7 are tensorplay-mlu's
# collective codes (tensorplay_mlu/distributed.py:37-46).
DTYPE_CODES = {
    torch.uint8: 0,
    torch.int8: 1,
    torch.int16: 2,
    torch.int32: 3,
    torch.int64: 4,
    torch.float16: 5,
    torch.float32: 6,
    torch.bfloat16: 7,
    torch.float64: 8,
    torch.bool: 9,
}
CODE_DTYPES = {v: k for k, v in DTYPE_CODES.items()}

# Operator codes (tpb_binary_op, tpb_unary_op, tpb_unary_backward_op, tpb_reduce_op).
ADD, SUB, MUL, DIV, RSUB = range(5)
(EXP, LOG, SQRT, RSQRT, NEG, ABS, POW, RELU, SIGMOID, TANH, SILU, GELU, GELU_TANH,
 SQUARE) = range(14)
(THRESHOLD_BACKWARD, SIGMOID_BACKWARD, TANH_BACKWARD, GELU_BACKWARD, GELU_TANH_BACKWARD,
 SILU_BACKWARD) = range(6)
SUM, MEAN, AMAX, AMIN = range(4)
EPI_GELU, EPI_GELU_BACKWARD = 1, 2  # tp_b200_gemm_epilogue
GEMM_ALLOW_TF32 = 1


class TpbTensor(ctypes.Structure):
    _fields_ = [
        ("data", ctypes.c_void_p),
        ("dtype", ctypes.c_int32),
        ("ndim", ctypes.c_int32),
        ("sizes", ctypes.c_int64 * MAX_DIMS),
        ("strides", ctypes.c_int64 * MAX_DIMS),
    ]


def describe(t: torch.Tensor) -> TpbTensor:
    """Descriptor of a strided tensor (device or host memory)."""
    if t.dim() > MAX_DIMS:
        raise RuntimeError(f"at most {MAX_DIMS} dimensions are supported, got {t.dim()}")
    try:
        code = DTYPE_CODES[t.dtype]
    except KeyError as error:
        raise TypeError(f"dtype {t.dtype} is not supported by the B200 backend") from error
    d = TpbTensor()
    d.data = t.data_ptr() if t.numel() else None
    d.dtype = code
    d.ndim = t.dim()
    for i, (s, st) in enumerate(zip(t.shape, t.stride())):
        d.sizes[i] = s
        d.strides[i] = st
    return d


_LOCK = threading.Lock()
_LIB: ctypes.CDLL | None = None

_P = ctypes.c_void_p
_T = ctypes.POINTER(TpbTensor)
_I = ctypes.c_int
_SZ = ctypes.c_size_t
_I64 = ctypes.c_int64
_D = ctypes.c_double

_SIGNATURES = {
    "tp_b200_init": ([], _I),
    "tp_b200_device_count": ([], _I),
    "tp_b200_current_device": ([], _I),
    "tp_b200_set_device": ([_I], _I),
    "tp_b200_capability": ([_I], _I),
    "tp_b200_synchronize": ([_I], _I),
    "tp_b200_set_stream": ([_I, _P], _I),
    "tp_b200_get_stream": ([_I], _P),
    "tp_b200_memcpy": ([_P, _P, _SZ, _I, _I, _I, _P, _I], _I),
    "tp_b200_mem_get_info": ([_I, ctypes.POINTER(_SZ), ctypes.POINTER(_SZ)], _I),
    "tp_b200_last_error": ([], ctypes.c_char_p),
    "tp_b200_take_device_error": ([_I], _I),
    "tp_b200_launch_count": ([], _I64),
    "tp_b200_set_gemm_sm_limit": ([_I, _I], _I),
    "tp_b200_set_gemm_tile_order": ([_I, _I], _I),
    "tp_b200_capture_ready": ([], _I),
    "tp_b200_capture_stats": ([ctypes.POINTER(ctypes.c_int64)], None),
    "tp_b200_capture_begin": ([_I], _I),
    "tp_b200_capture_end": ([_I], _I),
    "tp_b200_capture_invoke": ([_I], _I),
    "tp_b200_capture_reset": ([], _I),
    "tp_b200_timer_current_device": ([], _I),
    "tp_b200_timer_record": ([_I], _P),
    "tp_b200_timer_elapsed_ms": ([_P, _P, ctypes.POINTER(ctypes.c_float)], _I),
    "tp_b200_timer_release": ([_P], None),
    "tp_b200_timer_pooled": ([], _I64),
    "tp_b200_malloc": ([_SZ, _I, _P], _P),
    "tp_b200_free": ([_P, _SZ, _I, _P], None),
    "tp_b200_memory_stats": ([_I, ctypes.POINTER(_I64)], None),
    "tp_b200_reset_peak_memory_stats": ([_I], None),
    "tp_b200_empty_cache": ([], None),
    "tp_b200_copy": ([_T, _T, _P], _I),
    "tp_b200_fill": ([_T, _D, _I64, _P], _I),
    "tp_b200_binary": ([_I, _T, _T, _T, _D, _P], _I),
    "tp_b200_binary_scalar": ([_I, _T, _T, _D, _I64, _D, _P], _I),
    "tp_b200_unary": ([_I, _T, _T, _D, _P], _I),
    "tp_b200_unary_backward": ([_I, _T, _T, _T, _D, _P], _I),
    "tp_b200_reduce": ([_I, _T, _T, ctypes.c_uint32, _P], _I),
    "tp_b200_reduce_noalloc": ([_I, _T, _T, ctypes.c_uint32, _P], _I),
    "tp_b200_softmax": ([_I, _T, _T, _I, _P], _I),
    "tp_b200_softmax_backward": ([_I, _T, _T, _T, _I, _P], _I),
    "tp_b200_gemm": ([_T, _T, _T, _T, _D, _D, _I, _P], _I),
    "tp_b200_gemm_epilogue": ([_I, _T, _T, _T, _T, _T, _D, _D, _I, _P], _I),
    "tp_b200_mse_loss": ([_T, _T, _T, _T, _D, _P], _I),
    "tp_b200_gather": ([_T, _T, _T, _I, _P], _I),
    "tp_b200_index_select": ([_T, _T, _T, _I, _P], _I),
    "tp_b200_index_add": ([_T, _T, _T, _I, _P], _I),
    "tp_b200_scatter": ([_T, _T, _T, _I, _I, _I, _P], _I),
    "tp_b200_scan": ([_I, _T, _T, _I, _P], _I),
    "tp_b200_where": ([_T, _T, _T, _T, _P], _I),
    "tp_b200_layer_norm": ([_T, _T, _T, _T, _T, _T, _I64, _D, _P], _I),
    "tp_b200_layer_norm_backward": ([_T, _T, _T, _T, _T, _T, _T, _T, _I64, _P], _I),
    "tp_b200_nll_loss": ([_T, _T, _T, _T, _T, _I, _I64, _P], _I),
    "tp_b200_nll_loss_backward": ([_T, _T, _T, _T, _T, _I, _I64, _P], _I),
    "tp_b200_dropout": ([_T, _T, _T, _D, ctypes.c_uint64, ctypes.c_uint64, _P], _I),
    "tp_b200_masked_scale": ([_T, _T, _T, _D, _P], _I),
    "tp_b200_nccl_last_error": ([], ctypes.c_char_p),
    "tp_b200_nccl_unique_id_bytes": ([], _I),
    "tp_b200_nccl_get_unique_id": ([_P], _I),
    "tp_b200_nccl_comm_init": ([_I, _I, _I, _P, ctypes.POINTER(_P)], _I),
    "tp_b200_nccl_comm_init_timeout": ([_I, _I, _I, _P, _I, ctypes.POINTER(_P)], _I),
    "tp_b200_nccl_comm_init_ctas": ([_I, _I, _I, _P, _I, _I, _I, ctypes.POINTER(_P)], _I),
    "tp_b200_nccl_comm_destroy": ([_P], _I),
    "tp_b200_nccl_comm_abort": ([_P], _I),
    "tp_b200_nccl_comm_rank": ([_P, ctypes.POINTER(_I)], _I),
    "tp_b200_nccl_comm_count": ([_P, ctypes.POINTER(_I)], _I),
    "tp_b200_nccl_comm_check": ([_P], _I),
    "tp_b200_nccl_all_reduce": ([_P, _P, _SZ, _I, _I, _I, _P], _I),
    "tp_b200_nccl_broadcast": ([_P, _P, _SZ, _I, _I, _I, _P], _I),
    "tp_b200_nccl_reduce": ([_P, _P, _SZ, _I, _I, _I, _I, _P], _I),
    "tp_b200_nccl_all_gather": ([_P, _P, _SZ, _I, _I, _P], _I),
    "tp_b200_nccl_reduce_scatter": ([_P, _P, _SZ, _I, _I, _I, _P], _I),
    "tp_b200_nccl_all_to_all": ([_P, _P, _SZ, _I, _I, _P], _I),
    "tp_b200_nccl_send": ([_P, _SZ, _I, _I, _I, _P], _I),
    "tp_b200_nccl_recv": ([_P, _SZ, _I, _I, _I, _P], _I),
    "tp_b200_nccl_group_start": ([], _I),
    "tp_b200_nccl_group_end": ([], _I),
    "tp_b200_nccl_synchronize": ([_I], _I),
    "tp_b200_nccl_queue_idle": ([_I], _I),
}


def exported_symbols() -> list[str]:
    return list(_SIGNATURES)


def lib() -> ctypes.CDLL:
    """The loaded native library (loaded on first use; fails loudly when absent)."""
    global _LIB
    if _LIB is not None:
        return _LIB
    with _LOCK:
        if _LIB is None:
            if not os.path.isfile(LIBRARY_PATH):
                raise RuntimeError(
                    f"the B200 native library is not built ({LIBRARY_PATH} missing); "
                    "run `python -m tensorplay_mlu_b200._build` or __graft_entry__.build()")
            handle = ctypes.CDLL(LIBRARY_PATH)
            for name, (args, res) in _SIGNATURES.items():
                fn = getattr(handle, name)
                fn.argtypes = args
                fn.restype = res
            _LIB = handle
    return _LIB


def check(status: int, what: str = "") -> None:
    """Raise with the library's message when ``status`` is an error."""
    if status >= 0:
        return
    message = lib().tp_b200_last_error()
    text = message.decode() if message else "B200 backend call failed"
    raise RuntimeError(f"{what}: {text}" if what else text)


def stream_of(device: torch.device | int | None = None) -> int:
    """Handle of PyTorch's current stream on ``device`` (ordering matches torch)."""
    return torch.cuda.current_stream(device).cuda_stream
