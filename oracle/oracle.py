"""CPU oracle for the matmul / addmm / bmm path — TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg may import this module; the product (``metalblas_b200``) never does.

It restates the reference's own correctness oracle, tests/test_basic.py, in
numpy, and tightens it the way the north star asks (fp64 reference and relative
Frobenius error):

* integers: exact product, then wrap to the dtype's width in two's complement
  (tests/test_basic.py:27-34 ``_wrap``; :37-39 ``_product`` computes in int64);
* complex: the reference upcasts to complex64 (tests/test_basic.py:40-41); we
  use complex128;
* floats: the reference computes ``a.float() @ b.float()`` (tests/test_basic.py:42);
  we use float64;
* fused ops: ``alpha * product + beta * bias`` with alpha==0 meaning "no
  product" and beta==0 meaning "bias never read"
  (tests/test_basic.py:110-121 ``_fused_ref``; metalblas/shaders/mb_epi.h:16-26).

Inputs are numpy arrays of the storage values (bf16 values held exactly in
float32, complex32 in complex64).  Parity is pinned by tests/golden/, generated
from the reference's own oracle functions (tests/golden/make_golden.py).
"""
from __future__ import annotations

import numpy as np

INT_BITS = {"int8": 8, "uint8": 8, "int16": 16, "int32": 32, "int64": 64}
SIGNED = {"int8", "int16", "int32", "int64"}
FLOAT_NAMES = ("float32", "float16", "bfloat16")
COMPLEX_NAMES = ("complex64", "complex32")
INT_NAMES = tuple(INT_BITS)


def wrap(x, dtype: str) -> np.ndarray:
    """Two's-complement wrap of an exact integer array to ``dtype``
    (tests/test_basic.py:27-34)."""
    x = np.asarray(x)
    bits = INT_BITS[dtype]
    if bits == 64:
        return x.astype(np.int64)
    mod = 1 << bits
    x = np.mod(x.astype(np.int64), mod)
    if dtype in SIGNED:
        x = np.where(x >= mod // 2, x - mod, x)
    return x.astype({"int8": np.int8, "uint8": np.uint8, "int16": np.int16, "int32": np.int32}[dtype])


def _int_matmul(a, b) -> np.ndarray:
    """Exact int64 product (mod 2^64 like torch's long matmul).  When every
    partial sum fits in 53 bits the fp64 BLAS product is exact and fast."""
    a = np.asarray(a, dtype=np.int64)
    b = np.asarray(b, dtype=np.int64)
    k = a.shape[-1]
    bound = (float(np.abs(a).max(initial=0)) * float(np.abs(b).max(initial=0)) * max(k, 1))
    if bound < 2.0 ** 52:
        return np.rint(np.matmul(a.astype(np.float64), b.astype(np.float64))).astype(np.int64)
    with np.errstate(over="ignore"):
        return np.matmul(a, b)  # numpy integer matmul wraps mod 2^64


def product(a, b, dtype: str) -> np.ndarray:
    """The reference's ``_product`` (tests/test_basic.py:37-42) in wider precision:
    int64 (exact) for integers, complex128 for complex, float64 for floats."""
    if dtype in INT_BITS:
        return _int_matmul(a, b)
    if dtype in COMPLEX_NAMES:
        return np.matmul(np.asarray(a, np.complex128), np.asarray(b, np.complex128))
    return np.matmul(np.asarray(a, np.float64), np.asarray(b, np.float64))


def fused(bias, a, b, beta, alpha, dtype: str, reduce: bool = False) -> np.ndarray:
    """``_fused_ref`` (tests/test_basic.py:110-121): alpha*product + beta*bias,
    with addbmm's batch reduction when ``reduce``."""
    p = product(a, b, dtype)
    if reduce:
        p = p.sum(0)
    if dtype in INT_BITS:
        bias_w = np.asarray(bias, np.int64)
        with np.errstate(over="ignore"):
            r = np.int64(int(alpha)) * p if alpha != 0 else np.zeros_like(p)
            if beta != 0:
                r = r + np.int64(int(beta)) * np.broadcast_to(bias_w, p.shape)
        return r
    wide = np.complex128 if dtype in COMPLEX_NAMES else np.float64
    bias_w = np.asarray(bias, wide)
    r = alpha * p if alpha != 0 else np.zeros_like(p)
    if beta != 0:
        r = r + beta * np.broadcast_to(bias_w, p.shape)
    return r


def expected(ref, dtype: str) -> np.ndarray:
    """Integers: the wrapped result in the output dtype; others unchanged."""
    if dtype in INT_BITS:
        return wrap(ref, dtype)
    return ref


def rel_frobenius(got, ref) -> float:
    """||got - ref||_F / ||ref||_F in float64 / complex128."""
    got = np.asarray(got)
    ref = np.asarray(ref)
    wide = np.complex128 if np.iscomplexobj(got) or np.iscomplexobj(ref) else np.float64
    g, r = got.astype(wide), ref.astype(wide)
    den = np.linalg.norm(r.ravel())
    num = np.linalg.norm((g - r).ravel())
    if den == 0:
        return float(num)
    return float(num / den)


# Tolerances ------------------------------------------------------------------
# Relative Frobenius bounds of the north star: 1e-2 for 16-bit floats and
# complex32, 1e-5 for float32 and complex64, exact for integers.
FROB_TOL = {"bfloat16": 1e-2, "float16": 1e-2, "complex32": 1e-2, "float32": 1e-5, "complex64": 1e-5}


def ref_atol(dtype: str, k: int, strict: bool = False) -> float:
    """Absolute tolerance of the reference's ``_atol`` (tests/test_basic.py:45-50)."""
    if dtype == "float32":
        return max(1e-3, 1e-5 * k) if strict else max(0.1, 5e-3 * k ** 0.5)
    if dtype == "bfloat16":
        return max(0.5, 3e-2 * k ** 0.5)
    return max(5e-2, 1e-2 * k ** 0.5)


def ref_check(got, ref, dtype: str, k: int, scale: float = 1.0, strict: bool = False):
    """The reference's ``_check`` acceptance rule (tests/test_basic.py:53-69).

    ``ref`` is this oracle's wide result; ``got`` the kernel's output values.
    Returns (ok, measured_error, limit).
    """
    got = np.asarray(got)
    if dtype in INT_BITS:
        exp = wrap(ref, dtype)
        ok = got.shape == exp.shape and np.array_equal(got.astype(np.int64), exp.astype(np.int64))
        return ok, 0.0 if ok else 1.0, 0.0
    if dtype in COMPLEX_NAMES:
        g = got.astype(np.complex128)
        r = np.asarray(ref, np.complex128)
        rel = float(np.abs(g - r).max(initial=0) / (np.abs(r).max(initial=0) + 1e-9))
        limit = 3e-2 if dtype == "complex32" else 5e-3
        return rel <= limit, rel, limit
    # floats: reference compares against ref rounded to the dtype
    r = round_to(np.asarray(ref, np.float64), dtype)
    err = float(np.abs(got.astype(np.float64) - r).max(initial=0))
    limit = scale * ref_atol(dtype, k, strict)
    return err <= limit, err, limit


def round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round float64 values to the storage dtype (round-to-nearest-even)."""
    x = np.asarray(x, np.float64)
    if dtype == "float32":
        return x.astype(np.float32).astype(np.float64)
    if dtype == "float16":
        return x.astype(np.float16).astype(np.float64)
    if dtype == "bfloat16":
        f = x.astype(np.float32)
        u = f.view(np.uint32).astype(np.uint64)
        rounding = ((u >> 16) & 1) + 0x7FFF
        u = ((u + rounding) >> 16) << 16
        out = u.astype(np.uint32).view(np.float32).astype(np.float64)
        return np.where(np.isnan(f), np.nan, out)
    raise ValueError(dtype)


def check(got, ref, dtype: str) -> tuple[bool, float]:
    """North-star acceptance: exact for integers, relative Frobenius otherwise."""
    if dtype in INT_BITS:
        exp = wrap(ref, dtype)
        got = np.asarray(got)
        ok = got.shape == exp.shape and np.array_equal(got.astype(np.int64), exp.astype(np.int64))
        return ok, 0.0 if ok else 1.0
    err = rel_frobenius(got, ref)
    return err <= FROB_TOL[dtype], err
