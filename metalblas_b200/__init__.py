"""metalblas_b200 — B200 (sm_100a) matmul / addmm / bmm with the metalBLAS API.

Drop-in for the reference's public names (metalblas/__init__.py:1-19):

    import metalblas_b200 as metalblas
    c = metalblas.matmul(a, b)          # a, b are CUDA tensors

The compute runs in ``libmetalblas_b200.so`` through the C ABI declared in
``include/metalblas_b200.h``; there is no CPU fallback.
"""
from . import kernels
from .dispatch import (
    addbmm,
    addmm,
    baddbmm,
    bmm,
    dot,
    gemm,
    ger,
    matmul,
    mv,
    outer,
    vdot,
)

__all__ = [
    "matmul", "gemm", "addmm", "bmm", "baddbmm", "addbmm",
    "dot", "vdot", "outer", "ger", "mv", "kernels",
]
