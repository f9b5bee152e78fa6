"""ORACLE (test infrastructure): build and call the C integer-GEMM restatement.

``build()`` compiles ``int_gemm.c`` with gcc (-O3, OpenMP when available)
into ``oracle/_build/liboracle_int_gemm.so``; ``gemm_int(a, b)`` runs it on
int8 / int16 CPU tensors and returns the int32 product (mod 2^32).
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "int_gemm.c")
OUT_DIR = os.path.join(HERE, "_build")
LIB = os.path.join(OUT_DIR, "liboracle_int_gemm.so")

_lib = None


def build() -> str:
    os.makedirs(OUT_DIR, exist_ok=True)
    if os.path.exists(LIB) and os.path.getmtime(LIB) >= os.path.getmtime(SRC):
        return LIB
    base = ["gcc", "-O3", "-shared", "-fPIC", SRC, "-o", LIB]
    res = subprocess.run(base[:2] + ["-fopenmp"] + base[2:], capture_output=True, text=True)
    if res.returncode != 0:
        res = subprocess.run(base, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"gcc failed on int_gemm.c:\n{res.stderr}")
    return LIB


def _load():
    global _lib
    if _lib is None:
        _lib = ctypes.CDLL(build())
        for name in ("oracle_gemm_i8_i32", "oracle_gemm_i16_i32"):
            fn = getattr(_lib, name)
            fn.restype = None
            fn.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int64] * 6
    return _lib


def gemm_int(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """int32 C = A @ B (mod 2^32) for int8 or int16 row-major CPU tensors."""
    assert a.dtype == b.dtype and a.dtype in (torch.int8, torch.int16)
    a = a.contiguous()
    b = b.contiguous()
    M, K = a.shape
    K2, N = b.shape
    assert K == K2
    c = torch.empty((M, N), dtype=torch.int32)
    fn = _load().oracle_gemm_i8_i32 if a.dtype == torch.int8 else _load().oracle_gemm_i16_i32
    fn(a.data_ptr(), b.data_ptr(), c.data_ptr(), M, N, K, K, N, N)
    return c
