"""Parity of the CUDA path with the oracle on every case of the reference's test
suite (tests/test_basic.py:166-255), through the public API and the C ABI.

Each case is checked twice: with the reference's own acceptance rule
(tests/test_basic.py:53-69 ``_check``: exact for integers, max-abs for floats,
max-relative for complex) and with the north star's (relative Frobenius error
against an fp64 product: <= 1e-2 for bf16/fp16/complex32, <= 1e-5 for
fp32/complex64; integers bit-exact).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import oracle as orc
from tests.helpers import ALL, COMPLEX, FLOATS, INTS, NAME, rand, to_np

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def mb():
    import metalblas_b200
    metalblas_b200.kernels.load()
    return metalblas_b200


def _gen():
    return torch.Generator().manual_seed(0)


def _verify(got, ref, dtype, k, tag, scale=1.0, strict=False):
    name = NAME[dtype]
    assert got.dtype == dtype, f"{tag}: dtype {got.dtype} != {dtype}"
    assert tuple(got.shape) == tuple(np.shape(ref)), f"{tag}: shape {tuple(got.shape)} != {np.shape(ref)}"
    g = to_np(got)
    ok, err, lim = orc.ref_check(g, ref, name, k, scale=scale, strict=strict)
    assert ok, f"{tag}: reference rule violated (error {err:.3e} > {lim:.3e})"
    ok2, rel = orc.check(g, ref, name)
    assert ok2, f"{tag}: relative Frobenius {rel:.3e} > {orc.FROB_TOL.get(name, 0)}"


def _matrices(M, N, K, dtype, layout, gen):
    """tests/test_basic.py:72-82 ``_matrices``."""
    a = rand((K, M), dtype, gen).t() if layout in ("ta", "tr") else rand((M, K), dtype, gen)
    b = rand((N, K), dtype, gen).t() if layout == "tr" else rand((K, N), dtype, gen)
    if layout == "conj":
        a = a.conj()
    elif layout == "strided":
        if N == 1:
            b = rand((K, 2), dtype, gen)[:, :1]
        else:
            a = rand((K, 2), dtype, gen)[:, :1].t()
    return a, b


def check_mm(mb, M, N, K, dtype, backend=None, layout="rm"):
    gen = _gen()
    a, b = _matrices(M, N, K, dtype, layout, gen)
    kwargs = {"backend": backend} if backend else {}
    got = mb.matmul(a, b, **kwargs)
    ref = orc.product(to_np(a), to_np(b), NAME[dtype])
    _verify(got, ref, dtype, K, f"matmul {dtype} {layout} {backend or 'auto'} {M}x{N}x{K}",
            strict=backend not in (None, "mpp"))


# ----------------------------------------------------------------- matmul cases
_BASE = [(64, 64, 64), (128, 128, 128), (256, 256, 256), (513, 257, 129), (1024, 1024, 256)]
MM_CASES = []
for _dt in FLOATS:
    for _be in ("simd", "mpp"):
        for _s in _BASE + ([(33, 33, 33)] if _dt is torch.float32 and _be == "simd" else []):
            MM_CASES.append((*_s, _dt, _be, "rm"))
    for _s in [(128, 128, 128), (513, 257, 129), (1024, 1024, 256), (1, 4096, 4096), (4096, 1, 4096)]:
        MM_CASES.append((*_s, _dt, None, "tr"))
    for _s in [(1, 4096, 4096), (4096, 1, 4096), (1, 1024, 1024), (1024, 1, 1024)]:
        MM_CASES.append((*_s, _dt, "gemv", "rm"))
    for _s in [(1, 1024, 256), (1, 4096, 1024), (64, 1, 256), (1024, 1, 1024)]:
        MM_CASES.append((*_s, _dt, "gemv", "strided"))
for _s in [(64, 64, 64), (128, 128, 128), (256, 256, 256), (512, 512, 512), (1024, 1024, 1024),
           (513, 257, 129), (333, 444, 555), (2, 64, 128), (1, 4096, 4096), (4096, 1, 4096),
           (1, 1024, 1024), (1024, 1, 1024), (1, 1, 512), (1, 17, 33)]:
    MM_CASES.append((*_s, torch.complex64, None, "rm"))
for _s in [(256, 256, 256), (513, 257, 129)]:
    MM_CASES.append((*_s, torch.complex64, None, "ta"))
    MM_CASES.append((*_s, torch.complex64, None, "conj"))
for _s in [(256, 256, 256), (512, 512, 512), (1, 2048, 2048), (2048, 1, 2048)]:
    MM_CASES.append((*_s, torch.complex32, None, "rm"))
for _dt in INTS:
    for _s in [(64, 64, 64), (256, 256, 256), (513, 257, 129), (333, 444, 555), (1024, 1024, 1024),
               (96, 4096, 512), (33, 33, 33), (1, 4096, 4096), (4096, 1, 4096), (1, 1024, 257),
               (300, 1, 1024)]:
        MM_CASES.append((*_s, _dt, None, "rm"))
    MM_CASES.append((256, 256, 256, _dt, None, "ta"))


@pytest.mark.parametrize("M,N,K,dtype,backend,layout", MM_CASES,
                         ids=[f"{NAME[c[3]]}-{c[4]}-{c[5]}-{c[0]}x{c[1]}x{c[2]}" for c in MM_CASES])
def test_matmul(mb, M, N, K, dtype, backend, layout):
    check_mm(mb, M, N, K, dtype, backend, layout)


# ----------------------------------------------------------------- fused ops
def _fused_ref(bias, a, b, beta, alpha, dtype, reduce):
    return orc.fused(to_np(bias), to_np(a), to_np(b), beta, alpha, NAME[dtype], reduce)


def check_fused(mb, op, shape, dtype, bshape, beta=1, alpha=1):
    gen = _gen()
    if op == "addmm":
        M, N, K = shape
        a, b = rand((M, K), dtype, gen), rand((K, N), dtype, gen)
    else:
        B, M, N, K = shape
        a, b = rand((B, M, K), dtype, gen), rand((B, K, N), dtype, gen)
    bias = rand(bshape, dtype, gen)
    got = getattr(mb, op)(bias, a, b, beta=beta, alpha=alpha)
    ref = _fused_ref(bias, a, b, beta, alpha, dtype, op == "addbmm")
    _verify(got, ref, dtype, K * (shape[0] if op == "addbmm" else 1),
            f"{op} {dtype} {shape} bias={bshape} beta={beta} alpha={alpha}", scale=abs(alpha) + abs(beta))


FUSED = []
for _dt in ALL:
    for _bs in [(128, 96), (1, 96), (128, 1), (96,), (1,), ()]:
        FUSED.append(("addmm", (128, 96, 256), _dt, _bs, 1, 1))
    for _be, _al in [(2, 3), (0, 1), (1, 0), (0, 0)]:
        FUSED.append(("addmm", (128, 96, 256), _dt, (96,), _be, _al))
    FUSED.append(("addmm", (1, 4096, 4096), _dt, (4096,), 1, 1))
    FUSED.append(("addmm", (4096, 1, 4096), _dt, (1,), 1, 1))
for _dt in FLOATS:
    for _M, _N, _K in [(130, 100, 200), (257, 257, 257), (333, 444, 555)]:
        for _bs in [(_M, _N), (1, _N), (_M, 1), (_N,), (1,), ()]:
            FUSED.append(("addmm", (_M, _N, _K), _dt, _bs, 1, 1))
for _dt in ALL:
    for _bs in [(4, 128, 96), (4, 1, 96), (4, 128, 1), (1, 128, 96), (128, 96), (96,), (1,), ()]:
        FUSED.append(("baddbmm", (4, 128, 96, 256), _dt, _bs, 1, 1))
    for _be, _al in [(2, 3), (0, 1), (1, 0), (0, 0)]:
        FUSED.append(("baddbmm", (4, 128, 96, 256), _dt, (96,), _be, _al))
    for _bs in [(128, 96), (1, 96), (128, 1), (96,), (1,), ()]:
        FUSED.append(("addbmm", (8, 128, 96, 256), _dt, _bs, 1, 1))
    for _sh in [(32, 64, 64, 64), (4, 256, 256, 512)]:
        FUSED.append(("addbmm", _sh, _dt, (_sh[2],), 1, 1))
    for _be, _al in [(1, 1), (2, 3), (0, 1), (1, 0)]:
        FUSED.append(("addbmm", (8, 128, 96, 256), _dt, (96,), _be, _al))
for _dt in FLOATS:
    for _M, _N, _K in [(130, 100, 200), (257, 129, 257)]:
        for _bs in [(4, _M, _N), (_N,), ()]:
            FUSED.append(("baddbmm", (4, _M, _N, _K), _dt, _bs, 1, 1))


@pytest.mark.parametrize("op,shape,dtype,bshape,beta,alpha", FUSED,
                         ids=[f"{c[0]}-{NAME[c[2]]}-{'x'.join(map(str, c[1]))}-b{c[3]}-{c[4]}-{c[5]}"
                              for c in FUSED])
def test_fused(mb, op, shape, dtype, bshape, beta, alpha):
    check_fused(mb, op, shape, dtype, bshape, beta, alpha)


@pytest.mark.parametrize("dtype", FLOATS, ids=[NAME[d] for d in FLOATS])
def test_addmm_beta0_no_nan(mb, dtype):
    """beta=0 never reads bias (tests/test_basic.py:214-217)."""
    gen = _gen()
    a, b = rand((128, 256), dtype, gen), rand((256, 96), dtype, gen)
    got = mb.addmm(torch.full((128, 96), float("nan"), dtype=dtype, device="cuda"), a, b, beta=0)
    assert not torch.isnan(got).any().item(), f"addmm beta=0 leaked NaN for {dtype}"


# ----------------------------------------------------------------- bmm
BMM_SHAPES = [(8, 128, 128, 128), (32, 256, 256, 256), (4, 512, 512, 512), (96, 512, 512, 64),
              (16, 64, 4096, 512), (128, 4096, 64, 256), (512, 64, 64, 64), (2048, 64, 64, 32),
              (3, 130, 100, 200), (8, 1, 512, 256), (8, 512, 1, 256)]
BMM = [(s, dt, "rm") for dt in ALL for s in BMM_SHAPES] + [((8, 256, 256, 256), dt, "tr") for dt in ALL]


@pytest.mark.parametrize("shape,dtype,layout", BMM,
                         ids=[f"{NAME[c[1]]}-{c[2]}-{'x'.join(map(str, c[0]))}" for c in BMM])
def test_bmm(mb, shape, dtype, layout):
    B, M, N, K = shape
    gen = _gen()
    if layout == "tr":
        a = rand((B, K, M), dtype, gen).transpose(-2, -1)
        b = rand((B, N, K), dtype, gen).transpose(-2, -1)
    else:
        a, b = rand((B, M, K), dtype, gen), rand((B, K, N), dtype, gen)
    got = mb.bmm(a, b)
    ref = orc.product(to_np(a), to_np(b), NAME[dtype])
    _verify(got, ref, dtype, K, f"bmm {dtype} {layout} {shape}")


# ----------------------------------------------------------------- N-D / vectors
ND = [((64,), (64,)), ((32,), (32, 48)), ((40, 32), (32,)), ((32,), (8, 32, 48)), ((6, 40, 32), (32,)),
      ((8, 40, 32), (8, 32, 48)), ((8, 40, 32), (32, 48)), ((40, 32), (8, 32, 48)),
      ((2, 3, 40, 32), (2, 3, 32, 48)), ((3, 1, 64, 32), (1, 5, 32, 48))]
ND_DT = (torch.float32, torch.bfloat16, torch.float16, torch.complex64, torch.int32, torch.int8, torch.int64)
ND_CASES = [(s, dt) for dt in ND_DT for s in ND]


@pytest.mark.parametrize("shapes,dtype", ND_CASES, ids=[f"{NAME[c[1]]}-{c[0]}" for c in ND_CASES])
def test_nd(mb, shapes, dtype):
    a_shape, b_shape = shapes
    gen = _gen()
    a, b = rand(a_shape, dtype, gen), rand(b_shape, dtype, gen)
    k = a_shape[0] if len(a_shape) == 1 else a_shape[-1]
    got = mb.matmul(a, b)
    ref = orc.product(to_np(a), to_np(b), NAME[dtype])
    _verify(got, ref, dtype, k, f"matmul {dtype} {a_shape} @ {b_shape}")


VEC_DT = (torch.float32, torch.bfloat16, torch.float16, torch.complex64, torch.complex32,
          torch.int8, torch.int32, torch.int64)


@pytest.mark.parametrize("dtype", VEC_DT, ids=[NAME[d] for d in VEC_DT])
def test_vectors(mb, dtype):
    """dot / vdot / outer / mv (tests/test_basic.py:148-163)."""
    gen = _gen()
    name = NAME[dtype]
    for k in (4096, 7, 1):
        a, b = rand((k,), dtype, gen), rand((k,), dtype, gen)
        ref = orc.product(to_np(a), to_np(b), name)
        _verify(mb.dot(a, b), ref, dtype, k, f"dot {dtype} {k}")
        vref = orc.product(np.conj(to_np(a)), to_np(b), name) if dtype in COMPLEX else ref
        _verify(mb.vdot(a, b), vref, dtype, k, f"vdot {dtype} {k}")
    a, b = rand((128,), dtype, gen), rand((96,), dtype, gen)
    if dtype in INTS:
        ref = to_np(a).astype(np.int64)[:, None] * to_np(b).astype(np.int64)[None, :]
    else:
        ref = np.outer(to_np(a).astype(np.complex128 if dtype in COMPLEX else np.float64), to_np(b))
    _verify(mb.outer(a, b), ref, dtype, 1, f"outer {dtype}")
    a, b = rand((256, 512), dtype, gen), rand((512,), dtype, gen)
    _verify(mb.mv(a, b), orc.product(to_np(a), to_np(b), name), dtype, 512, f"mv {dtype}")


def test_device_status_clean(mb):
    """No bounded device wait gave up during the parity cases above."""
    assert mb.kernels.device_status() == 0
