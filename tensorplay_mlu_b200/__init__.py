"""B200 (sm_100a) device backend for TensorPlay.

The backend fills TensorPlay's out-of-tree device slot the way tensorplay-mlu
does (tensorplay_mlu/__init__.py:66-104): memory comes from a stream-ordered
caching allocator, every operator it registers runs a hand-written sm_100a
kernel (there is no host fallback for a claimed operator), and collectives run
over NCCL.  The device is named ``"b200"`` and the process-group backend
``"nccl_b200"``: TensorPlay already has an in-tree CUDA backend named
"cuda"/"nccl", so the plugin must not reuse those names.

Where TensorPlay itself is not installed (this repository's test and bench
environment), PyTorch CUDA tensors stand in for TensorPlay device tensors:
the operators in :mod:`tensorplay_mlu_b200.ops` take and return them, and
:func:`load` installs the caching allocator as PyTorch's CUDA allocator so
every such tensor's memory comes from it, as every MLU tensor's memory comes
from tensorplay-mlu's allocator.

    import tensorplay_mlu_b200 as tpb
    tpb.load()
    y = tpb.ops.relu(tpb.ops.mm(x, w))
"""

from __future__ import annotations

import os
import threading
import warnings

from . import _native

__all__ = ["is_loaded", "load", "allocator_installed", "DEVICE_NAME", "BACKEND_NAME"]

DEVICE_NAME = "b200"
BACKEND_NAME = "nccl_b200"

_LOCK = threading.Lock()
_LOADED = False
_ALLOCATOR_INSTALLED = False


def is_loaded() -> bool:
    return _LOADED


def allocator_installed() -> bool:
    """Whether the caching allocator backs PyTorch's CUDA tensors in this process."""
    return _ALLOCATOR_INSTALLED


def _library():
    if not _LOADED:
        raise RuntimeError("the B200 backend is not loaded; call tensorplay_mlu_b200.load()")
    return _native.lib()


def _install_allocator() -> bool:
    import torch

    if not torch.cuda.is_available():
        return False
    try:
        alloc = torch.cuda.memory.CUDAPluggableAllocator(
            _native.LIBRARY_PATH, "tp_b200_malloc", "tp_b200_free")
        torch.cuda.memory.change_current_allocator(alloc)
        return True
    except RuntimeError as error:
        # PyTorch refuses once its own allocator has handed out memory.
        warnings.warn(f"B200 caching allocator not installed for PyTorch tensors: {error}")
        return False


def load(install_allocator: bool | None = None) -> None:
    """Load the native backend once, then name the device (when TensorPlay exists).

    ``install_allocator`` (default: on unless ``TPB200_TORCH_ALLOCATOR=0``) makes
    the backend's caching allocator PyTorch's CUDA allocator; it must happen
    before the process's first CUDA allocation.
    """
    global _LOADED, _ALLOCATOR_INSTALLED
    with _LOCK:
        if _LOADED:
            return
        lib = _native.lib()
        if lib.tp_b200_init() != 0:
            raise RuntimeError(f"B200 backend initialisation failed: {lib.tp_b200_last_error().decode()}")
        if install_allocator is None:
            install_allocator = os.environ.get("TPB200_TORCH_ALLOCATOR", "1") != "0"
        if install_allocator:
            _ALLOCATOR_INSTALLED = _install_allocator()
        _LOADED = True
        _register_with_tensorplay()

        from . import distributed as _distributed

        _distributed.register()


def _register_with_tensorplay() -> None:
    """Name the PrivateUse1 device and register the device module, as
    tensorplay_mlu/__init__.py:95-99 does, when TensorPlay is importable."""
    try:
        import tensorplay as tp  # type: ignore
    except Exception:
        return
    tp.utils.rename_privateuse1_backend(DEVICE_NAME)
    tp.utils.generate_methods_for_privateuse1_backend()
    from . import runtime

    tp._register_device_module(DEVICE_NAME, runtime)


def _autoload() -> None:
    """``tensorplay.backends`` entry point: load when a B200 is visible."""
    try:
        if _native.lib().tp_b200_device_count() > 0:
            load()
    except Exception:
        pass


from . import ops  # noqa: E402  (the operator surface, importable before load())
from . import runtime  # noqa: E402
