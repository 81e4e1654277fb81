"""The drop-in boundary without a GPU: the C-ABI library loads, exports
every entry point include/tpb200.h declares, and rejects malformed calls with
a negative status and a message (never an exception across the boundary).
No kernel is launched here."""

from __future__ import annotations

import ctypes
import os
import re
import subprocess

import torch

import tensorplay_mlu_b200 as tpb
from tensorplay_mlu_b200 import _native as N

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "tpb200.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"\b(tp_b200_\w+)\s*\(", text)))


def test_header_declares_the_reference_surface():
    names = declared_symbols()
    # The collective ABI of tensorplay-mlu (Cncl.cpp:71-387), renamed.
    for ref in ("last_error", "unique_id_bytes", "get_unique_id", "comm_init", "comm_destroy",
                "comm_abort", "comm_rank", "comm_count", "all_reduce", "broadcast", "reduce",
                "all_gather", "reduce_scatter", "all_to_all", "send", "recv", "group_start",
                "group_end", "synchronize", "queue_idle"):
        assert f"tp_b200_nccl_{ref}" in names
    # Module.cpp:13-37
    for ref in ("init", "device_count", "memory_stats", "reset_peak_memory_stats", "empty_cache",
                "last_error"):
        assert f"tp_b200_{ref}" in names


def test_library_exports_every_declared_symbol():
    lib = N.lib()
    exported = subprocess.run(["nm", "-D", "--defined-only", N.LIBRARY_PATH], capture_output=True,
                              text=True, check=True).stdout
    for name in declared_symbols():
        assert re.search(rf"\bT {name}$", exported, re.M), f"{name} not exported"
        assert getattr(lib, name) is not None


def test_binding_covers_the_header():
    assert sorted(N.exported_symbols()) == declared_symbols()


def test_library_is_built_for_sm100a():
    # Every object is compiled with exactly one -gencode pair, for sm_100a
    # (no PTX for other targets, no other SASS); the GPU tests then run the
    # kernels on a B200.
    from tensorplay_mlu_b200 import _build

    assert _build.ARCH == ["-gencode", "arch=compute_100a,code=sm_100a"]
    src = open(_build.__file__).read()
    assert src.count('"-gencode"') == 1 and "*ARCH" in src


def test_init_and_device_count_without_crashing():
    lib = N.lib()
    assert lib.tp_b200_init() == 0
    assert lib.tp_b200_device_count() >= 0


def test_malformed_calls_return_errors():
    lib = N.lib()
    assert lib.tp_b200_copy(None, None, None) == -1
    assert b"null tensor descriptor" in lib.tp_b200_last_error()
    d = N.TpbTensor()
    d.ndim = 12
    assert lib.tp_b200_fill(ctypes.byref(d), 0.0, 0, None) == -1
    assert b"dimensions" in lib.tp_b200_last_error()
    d.ndim = 1
    d.dtype = 42
    assert lib.tp_b200_unary(0, ctypes.byref(d), ctypes.byref(d), 0.0, None) == -1
    assert b"dtype" in lib.tp_b200_last_error()
    assert lib.tp_b200_nccl_all_reduce(None, None, 1, 6, 0, 0, None) == -1
    assert b"null communicator" in lib.tp_b200_nccl_last_error()
    assert lib.tp_b200_nccl_all_reduce(None, None, 1, 2, 0, 0, ctypes.c_void_p(1)) == -1
    assert b"data type" in lib.tp_b200_nccl_last_error()


def test_descriptor_layout_matches_the_header():
    # data pointer, dtype, ndim, 8 sizes, 8 strides
    assert ctypes.sizeof(N.TpbTensor) == 8 + 4 + 4 + 8 * 8 + 8 * 8
    t = torch.arange(24, dtype=torch.float32).reshape(2, 3, 4).transpose(0, 2)
    d = N.describe(t)
    assert d.ndim == 3 and d.dtype == 6
    assert list(d.sizes)[:3] == [4, 3, 2] and list(d.strides)[:3] == [1, 4, 12]


def test_kernel_registry_matches_the_reference_registrations():
    # Exact schema names of the TENSORPLAY_LIBRARY_IMPL blocks (CopyKernels.cpp:350-363,
    # BinaryKernels.cpp:253-268, UnaryKernels.cpp:292-309, ReduceKernels.cpp:268-281,
    # BlasKernels.cpp:417-421).
    expected = {
        "empty_like", "zeros_like", "ones_like", "full_like", "item", "_local_scalar_dense", "empty",
        "empty.memory_format", "copy_", "fill_.Scalar", "zero_", "clone", "contiguous",
        "add.Tensor", "sub.Tensor", "mul.Tensor", "div.Tensor", "add_.Tensor", "sub_.Tensor",
        "mul_.Tensor", "div_.Tensor", "add.Scalar", "sub.Scalar", "rsub.Scalar", "mul.Scalar",
        "div.Scalar", "add_.Scalar", "mul_.Scalar", "div_.Scalar",
        "exp", "log", "sqrt", "rsqrt", "neg", "abs", "pow.Tensor_Scalar", "relu", "relu_", "sigmoid",
        "tanh", "silu", "gelu", "threshold_backward", "sigmoid_backward", "tanh_backward",
        "gelu_backward", "silu_backward",
        "sum", "sum.dim_IntList", "amax", "amin", "mean", "mean.dim", "softmax", "log_softmax",
        "_softmax", "_log_softmax", "_softmax_backward_data", "_log_softmax_backward_data",
        "mm", "bmm", "addmm", "matmul", "linear",
    }
    # NNKernels.cpp:399-410.
    expected |= {"native_layer_norm", "native_layer_norm_backward", "nll_loss", "nll_loss_backward",
                 "native_dropout", "native_dropout_backward", "embedding", "embedding_dense_backward"}
    # IndexKernels.cpp:352-367.
    expected |= {"gather", "gather_backward", "index_select", "index_select_backward", "scatter_add",
                 "scatter_add_", "scatter.reduce", "scatter_.reduce", "scatter_reduce.two", "cumsum", "cumsum_",
                 "cumprod", "cumprod_", "where.self"}
    assert set(tpb.ops.KERNELS) == expected


def test_product_code_does_not_import_the_oracle():
    pkg = os.path.join(ROOT, "tensorplay_mlu_b200")
    for dirpath, _, files in os.walk(pkg):
        for f in files:
            if f.endswith((".py", ".cpp", ".cu", ".h", ".cuh")):
                text = open(os.path.join(dirpath, f)).read()
                assert "import oracle" not in text and "from oracle" not in text, f
                assert "liboracle" not in text, f
