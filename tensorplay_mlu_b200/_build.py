"""Build the native library ``libtpb200.so`` in-tree for sm_100a.

Every ``csrc/*.cu`` / ``csrc/*.cpp`` is compiled by nvcc with
``-gencode arch=compute_100a,code=sm_100a`` (objects under ``_build/``, rebuilt
when the source or any header is newer) and linked with the static CUDA
runtime and the NCCL that ships with PyTorch (rpath set, so the library loads
the same NCCL as the process's PyTorch).  No GPU is needed to build.
"""

from __future__ import annotations

import glob
import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(ROOT, "include")
OBJDIR = os.path.join(HERE, "_build")
LIBRARY = os.path.join(HERE, "libtpb200.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    return os.path.join(home, "bin", "nvcc")


def nccl_dirs() -> tuple[str, str]:
    """(include, lib) of the NCCL PyTorch loads (the nvidia-nccl wheel)."""
    import nvidia.nccl  # type: ignore

    base = list(nvidia.nccl.__path__)[0]
    return os.path.join(base, "include"), os.path.join(base, "lib")


def _headers() -> list[str]:
    return (glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh"))
            + glob.glob(os.path.join(INCLUDE, "*.h")))


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd: list[str], verbose: bool) -> None:
    if verbose:
        print(" ".join(cmd), flush=True)
    proc = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"command failed ({proc.returncode}): {' '.join(cmd)}\n{proc.stdout}")
    if verbose and proc.stdout.strip():
        print(proc.stdout, flush=True)


def build(verbose: bool = False, jobs: int | None = None) -> str:
    """Compile and link the library if anything changed; returns its path."""
    os.makedirs(OBJDIR, exist_ok=True)
    nccl_inc, nccl_lib = nccl_dirs()
    sources = sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))
    headers = _headers()
    common = [nvcc(), "-std=c++17", "-O3", "-lineinfo", *ARCH, "-Xcompiler", "-fPIC,-Wall",
              "-Xcompiler", "-Wno-unused-function", f"-I{INCLUDE}", f"-I{CSRC}", f"-I{nccl_inc}"]
    jobs_todo = []
    objects = []
    for src in sources:
        obj = os.path.join(OBJDIR, os.path.basename(src) + ".o")
        objects.append(obj)
        if _stale(obj, [src, *headers]):
            jobs_todo.append(common + ["-c", src, "-o", obj])
    if jobs_todo:
        with ThreadPoolExecutor(max_workers=jobs or os.cpu_count() or 4) as pool:
            list(pool.map(lambda c: _run(c, verbose), jobs_todo))
    if jobs_todo or _stale(LIBRARY, objects):
        _run([nvcc(), "-shared", *ARCH, "-cudart", "static", "-o", LIBRARY, *objects,
              f"-L{nccl_lib}", "-l:libnccl.so.2", f"-Xlinker=-rpath={nccl_lib}"], verbose)
    return LIBRARY


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
