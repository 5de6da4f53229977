"""Build the oracle's C restatement (TEST INFRASTRUCTURE ONLY).

    python -m oracle.build        ->  oracle/_build/liboracle_int.so

Also exposes ``int_gemm(...)`` — a ctypes wrapper used by tests/ as an
independent checker of the integer path.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "int_gemm_ref.c")
OUT_DIR = os.path.join(HERE, "_build")
LIB = os.path.join(OUT_DIR, "liboracle_int.so")

_CODES = {"int8": 5, "uint8": 6, "int16": 7, "int32": 8, "int64": 9}


def build(force: bool = False) -> str:
    if not force and os.path.exists(LIB) and os.path.getmtime(LIB) >= os.path.getmtime(SRC):
        return LIB
    os.makedirs(OUT_DIR, exist_ok=True)
    subprocess.run(["gcc", "-O2", "-fPIC", "-shared", "-o", LIB, SRC], check=True)
    return LIB


_lib = None


def _load():
    global _lib
    if _lib is None:
        _lib = ctypes.CDLL(build())
        i64, vp, ci = ctypes.c_int64, ctypes.c_void_p, ctypes.c_int
        _lib.mb_ref_int_gemm.argtypes = [ci, i64, i64, i64, vp, i64, i64, vp, i64, i64, vp, i64, i64,
                                         ci, vp, i64, i64, i64, i64, ci, ci]
        _lib.mb_ref_int_gemm.restype = ci
    return _lib


def int_gemm(a: np.ndarray, b: np.ndarray, dtype: str, bias=None, alpha=1, beta=1, epilogue=False):
    """C[m,n] per the reference's int_gemm semantics for 2-D numpy inputs of ``dtype``."""
    lib = _load()
    npdt = np.dtype(dtype)
    a = np.ascontiguousarray(a, npdt)
    b = np.ascontiguousarray(b, npdt)
    M, K = a.shape
    N = b.shape[1]
    c = np.zeros((M, N), npdt)
    if epilogue and beta != 0:
        bias_b = np.ascontiguousarray(np.broadcast_to(np.asarray(bias, npdt), (M, N)))
        bptr, brs, bcs = bias_b.ctypes.data, N, 1
    else:
        bias_b, bptr, brs, bcs = None, None, 0, 0
    rc = lib.mb_ref_int_gemm(_CODES[dtype], M, N, K, a.ctypes.data, K, 1, b.ctypes.data, N, 1,
                             c.ctypes.data, N, 1, int(epilogue), bptr, brs, bcs,
                             int(alpha), int(beta), int(alpha != 0), int(beta != 0))
    assert rc == 0
    return c


if __name__ == "__main__":
    print(build(force=True))
