"""``import metalblas`` for the B200 build: the reference's package name
(metalblas/__init__.py:1-19 of Isalia20/metalBLAS) bound to this repository's
CUDA implementation, so code written against the reference runs unchanged on
CUDA tensors.  Every name is the object from ``metalblas_b200``; the library
behind them is ``libmetalblas_b200.so`` (there is no CPU or Metal path).
"""
from metalblas_b200 import (  # noqa: F401
    addbmm,
    addmm,
    baddbmm,
    bmm,
    dot,
    gemm,
    ger,
    kernels,
    matmul,
    mv,
    outer,
    vdot,
)
from metalblas_b200 import __all__  # noqa: F401
