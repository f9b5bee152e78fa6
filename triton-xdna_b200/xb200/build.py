"""Build ``libxb200.so`` (the C-ABI operator library) in-tree with nvcc.

Every ``csrc/*.cu`` file is compiled for sm_100a only
(``-gencode arch=compute_100a,code=sm_100a``) into an object under
``csrc/_build/`` and linked into ``xb200/libxb200.so`` next to this file.
The CUDA runtime is linked statically, so the library depends on nothing but
the driver; the tensor-map encoder is fetched through
``cudaGetDriverEntryPoint`` instead of linking libcuda.

Rebuilds are incremental on file modification times (any header change
rebuilds everything).
"""

from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG_DIR)  # triton-xdna_b200/
CSRC = os.path.join(ROOT, "csrc")
BUILD = os.path.join(CSRC, "_build")
INCLUDE = os.path.join(os.path.dirname(ROOT), "include")
LIB_PATH = os.path.join(PKG_DIR, "libxb200.so")

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH_FLAGS + [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    "-I" + INCLUDE,
    "-I" + CSRC,
]


def _nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the xb200 CUDA library cannot be built")


def _sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _headers() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(INCLUDE, "*.h")))


def _compile(src: str, extra: list[str]) -> str:
    obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
    newest_dep = max([os.path.getmtime(src)] + [os.path.getmtime(h) for h in _headers()])
    if os.path.exists(obj) and os.path.getmtime(obj) >= newest_dep and not extra:
        return obj
    cmd = [_nvcc(), *NVCC_FLAGS, *extra, "-c", src, "-o", obj]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed on {os.path.basename(src)}:\n{res.stdout}\n{res.stderr}")
    return obj


def build(verbose: bool = False, extra_flags: list[str] | None = None) -> str:
    """Compile and link the library; returns the path of ``libxb200.so``."""
    os.makedirs(BUILD, exist_ok=True)
    extra = list(extra_flags or [])
    srcs = _sources()
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        objs = list(ex.map(lambda s: _compile(s, extra), srcs))
    if os.path.exists(LIB_PATH) and not extra:
        lib_m = os.path.getmtime(LIB_PATH)
        if all(os.path.getmtime(o) <= lib_m for o in objs):
            return LIB_PATH
    tmp = LIB_PATH + ".tmp"
    cmd = [_nvcc(), *ARCH_FLAGS, "-shared", "-o", tmp, *objs, "-lpthread", "-ldl"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc link failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, LIB_PATH)
    if verbose:
        print(f"built {LIB_PATH}")
    return LIB_PATH


if __name__ == "__main__":
    build(verbose=True, extra_flags=sys.argv[1:])
