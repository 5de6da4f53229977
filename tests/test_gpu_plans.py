"""Every plan of the sm_100a tile table gives the oracle's answer, whatever plan
ran before it on the same (shared, cached) split-K workspace.

This pins the workspace contract of include/metalblas_b200.h: ticket counters
live at a fixed offset for every plan and are returned to zero by the kernel
that used them, so a split-K launch never reads counters or partials left by
a different plan.
"""
from __future__ import annotations

import itertools

import numpy as np
import pytest
import torch

from oracle import oracle as orc
from metalblas_b200 import _lib, dispatch
from tests.helpers import NAME, rand, to_np

pytestmark = pytest.mark.gpu

SHAPES = [(128, 8192, 4096), (64, 2048, 8192), (256, 512, 16384), (4, 4096, 4096), (16, 1024, 2048),
          (520, 1000, 1024)]
# (tile_n, split_k, swap_ab, cta_pair)
VARIANTS = [(0, 0, 0, 0), (64, 1, -1, 1), (64, 4, -1, 0), (128, 2, -1, 0), (256, 4, -1, 0), (256, 8, -1, 0),
            (128, 3, -1, 0), (0, 0, 1, 0), (32, 4, 1, 0), (16, 2, 1, 0), (64, 1, 1, 0),
            (256, 1, -1, 2), (128, 1, -1, 2), (256, 0, -1, 2),
            # stream-K tail (forced), plain and swapped
            (0, 0, -1, 0, 2), (64, 0, -1, 0, 2), (256, 0, -1, 0, 2), (16, 0, 1, 0, 2), (128, 0, 1, 0, 2),
            # stream-K tail on CTA pairs (each CTA of a pair reduces its own 128 rows)
            (256, 0, -1, 2, 2), (128, 0, -1, 2, 2),
            # 512-wide CTA-pair tile (two N = 256 MMAs per K-step, one accumulator)
            (512, 1, -1, 2)]


def _run(a, b, tile_n, split, swap, pair=0, sk=0, epilogue=None):
    M, K = a.shape
    N = b.shape[1]
    c = torch.empty(M, N, dtype=a.dtype, device=a.device)
    try:
        dispatch._launch(a, b, c, M, N, K, 1, (a.stride(0), a.stride(1), 0), (b.stride(0), b.stride(1), 0),
                         (c.stride(0), c.stride(1), 0), epilogue=epilogue, backend=_lib.MB_BACKEND_TC,
                         tile_n=tile_n, split_k=split, swap_ab=swap, cta_pair=pair, stream_k=sk, autotune=False)
    except NotImplementedError:
        return None  # this layout cannot take the forced variant (e.g. MN-major B with a narrow tile)
    return c


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.int8], ids=NAME.get)
def test_interleaved_plans_share_workspace(dtype):
    gen = torch.Generator().manual_seed(7)
    cases = []
    for (M, N, K) in SHAPES:
        a = rand((M, K), dtype, gen, full_range=dtype is torch.int8)
        b = rand((K, N), dtype, gen, full_range=dtype is torch.int8)
        cases.append((a, b, orc.product(to_np(a), to_np(b), NAME[dtype])))
    ran = 0
    # round-robin over shapes so consecutive launches always switch plan and shape
    for v, (a, b, ref) in itertools.product(VARIANTS, cases):
        c = _run(a, b, *v)
        if c is None:
            continue
        ran += 1
        ok, err = orc.check(to_np(c), ref, NAME[dtype])
        assert ok, f"{dtype} {tuple(a.shape)}x{b.shape[1]} variant={v} plan err={err}"
    assert ran >= len(cases) * 8


def test_split_k_epilogue_int8_wraps():
    """Split-K partials are summed as int32 with wraparound, then alpha/beta/bias."""
    gen = torch.Generator().manual_seed(8)
    a = rand((128, 8192), torch.int8, gen, full_range=True)
    b = rand((8192, 384), torch.int8, gen, full_range=True)
    bias = rand((384,), torch.int8, gen, full_range=True)
    for split in (1, 2, 4, 8):
        c = _run(a, b, 128, split, -1, epilogue=(bias, (0, 1, 0), 3, -7, True, True))
        ref = orc.fused(to_np(bias), to_np(a), to_np(b), 3, -7, "int8")
        ok, _ = orc.check(to_np(c), ref, "int8")
        assert ok, f"split={split}"
    for bn in (64, 128):  # stream-K tail: 3..6 K-ordered partials per tile
        c = _run(a, b, bn, 0, -1, sk=2, epilogue=(bias, (0, 1, 0), 3, -7, True, True))
        ref = orc.fused(to_np(bias), to_np(a), to_np(b), 3, -7, "int8")
        ok, _ = orc.check(to_np(c), ref, "int8")
        assert ok, f"stream-K bn={bn}"
    for pair in (1, 2):
        c = _run(a, b, 256, 1, -1, pair=pair, epilogue=(bias, (0, 1, 0), 3, -7, True, True))
        ref = orc.fused(to_np(bias), to_np(a), to_np(b), 3, -7, "int8")
        ok, _ = orc.check(to_np(c), ref, "int8")
        assert ok, f"pair={pair}"


def test_stream_k_many_parts_and_repeat():
    """One tile cut into one piece per SM (its last piece sums ~148 partials),
    run twice so the tickets must have been returned to zero, plus a batched
    bf16 case with an alpha/beta epilogue."""
    from metalblas_b200 import kernels
    gen = torch.Generator().manual_seed(11)
    a = rand((128, 65536), torch.bfloat16, gen)
    b = rand((65536, 128), torch.bfloat16, gen)
    ref = orc.product(to_np(a), to_np(b), "bfloat16")
    for _ in range(2):
        c = _run(a, b, 128, 0, -1, sk=2)
        ok, err = orc.check(to_np(c), ref, "bfloat16")
        assert ok, f"many parts err={err}"
    A = rand((3, 200, 3000), torch.float16, gen)
    B = rand((3, 3000, 72), torch.float16, gen)
    bias = rand((3, 200, 72), torch.float16, gen)
    C = torch.empty(3, 200, 72, dtype=torch.float16, device="cuda")
    dispatch._launch(A, B, C, 200, 72, 3000, 3, (3000, 1, 200 * 3000), (72, 1, 3000 * 72), (72, 1, 200 * 72),
                     epilogue=(bias, (72, 1, 200 * 72), 0.5, 2.0, True, True), backend=_lib.MB_BACKEND_TC,
                     tile_n=32, stream_k=2, autotune=False)
    fref = orc.fused(to_np(bias), to_np(A), to_np(B), 0.5, 2.0, "float16")
    ok, err = orc.check(to_np(C), fref, "float16")
    assert ok, f"batched stream-K baddbmm err={err}"
    assert kernels.device_status() == 0


def _plan(a, b, **ov):
    """The plan mb_gemm runs for a @ b on the tensor-core backend with these
    overrides (forced variants must really run, not fall back to CUDA cores)."""
    M, K = a.shape
    N = b.shape[1]
    d = _lib.new_desc()
    d.dtype, d.backend = _lib.DTYPE_CODE[a.dtype], _lib.MB_BACKEND_TC
    d.M, d.N, d.K = M, N, K
    d.A, d.B, d.C = a.data_ptr(), b.data_ptr(), a.data_ptr()
    d.a_rs, d.a_cs = a.stride()
    d.b_rs, d.b_cs = b.stride()
    d.c_rs, d.c_cs = N, 1
    for k, v in ov.items():
        setattr(d, k, v)
    d.workspace_bytes = -1
    return _lib.plan_query(d)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.int8], ids=NAME.get)
def test_pair_stream_k(dtype):
    """Stream-K tails on CTA pairs: the BASELINE config-1 shape (64 256-row tiles
    on 74 pairs, all in the tail), a tile cut into one piece per pair, a shape
    with whole-tile waves before the tail, and an epilogue with a bias row;
    each run twice so the tickets must have returned to zero."""
    from metalblas_b200 import kernels
    gen = torch.Generator().manual_seed(12)
    full = dtype is torch.int8
    # (8-bit: a 128-wide pair tile would give each CTA 64 bytes of a row-major
    # B, narrower than one TMA box, so the ragged case uses 256 there)
    for (M, N, K, bn) in ((2048, 2048, 4096, 256), (256, 256, 65536, 256), (4096, 4096, 1024, 256),
                          (1000, 1000, 3000, 256 if full else 128)):
        a = rand((M, K), dtype, gen, full_range=full)
        b = rand((K, N), dtype, gen, full_range=full)
        ref = orc.product(to_np(a), to_np(b), NAME[dtype])
        plan = _plan(a, b, tile_n=bn, cta_pair=2, stream_k=2, swap_ab=-1)
        assert "pair=2 sk=1" in plan, plan
        for _ in range(2):
            c = _run(a, b, bn, 0, -1, pair=2, sk=2)
            assert c is not None
            ok, err = orc.check(to_np(c), ref, NAME[dtype])
            assert ok, f"{dtype} {M}x{N}x{K} bn={bn} pair stream-K err={err}"
    a = rand((2048, 4096), dtype, gen, full_range=full)
    b = rand((4096, 2048), dtype, gen, full_range=full)
    bias = rand((2048,), dtype, gen, full_range=full)
    beta, alpha = (3, -2) if full else (0.5, 2.0)
    c = _run(a, b, 256, 0, -1, pair=2, sk=2, epilogue=(bias, (0, 1, 0), beta, alpha, True, True))
    ref = orc.fused(to_np(bias), to_np(a), to_np(b), beta, alpha, NAME[dtype])
    ok, err = orc.check(to_np(c), ref, NAME[dtype])
    assert ok, f"pair stream-K addmm err={err}"
    d = _lib.new_desc()
    d.dtype, d.backend = _lib.DTYPE_CODE[dtype], _lib.MB_BACKEND_TC
    d.M, d.N, d.K = 2048, 2048, 4096
    d.A, d.B, d.C = a.data_ptr(), b.data_ptr(), c.data_ptr()
    d.a_rs, d.a_cs, d.b_rs, d.b_cs, d.c_rs, d.c_cs = 4096, 1, 2048, 1, 2048, 1
    d.tile_n, d.cta_pair, d.stream_k, d.workspace_bytes = 256, 2, 2, -1
    assert "pair=2 sk=1" in _lib.plan_query(d)
    assert kernels.device_status() == 0


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.int8], ids=NAME.get)
def test_pair_wide_tile(dtype):
    """The 512-wide CTA-pair tile: several tiles per pair (accumulator reuse
    across tiles), ragged edges in M, N and K, B read K-major (x @ W^T) and
    MN-major, an addmm epilogue and a batched, broadcast product."""
    gen = torch.Generator().manual_seed(13)
    full = dtype is torch.int8
    for (M, N, K) in ((4096, 4096, 1024), (1000, 1500, 3000), (2304, 8192, 512)):
        a = rand((M, K), dtype, gen, full_range=full)
        for b in (rand((K, N), dtype, gen, full_range=full), rand((N, K), dtype, gen, full_range=full).t()):
            ref = orc.product(to_np(a), to_np(b), NAME[dtype])
            plan = _plan(a, b, tile_n=512, cta_pair=2, split_k=1, swap_ab=-1)
            assert "bn=512" in plan and "pair=2" in plan, plan
            c = _run(a, b, 512, 1, -1, pair=2)
            assert c is not None
            ok, err = orc.check(to_np(c), ref, NAME[dtype])
            assert ok, f"{dtype} {M}x{N}x{K} b_strides={b.stride()} wide tile err={err}"
    a = rand((2048, 2048), dtype, gen, full_range=full)
    b = rand((2048, 4096), dtype, gen, full_range=full)
    bias = rand((4096,), dtype, gen, full_range=full)
    beta, alpha = (3, -2) if full else (0.5, 2.0)
    c = _run(a, b, 512, 1, -1, pair=2, epilogue=(bias, (0, 1, 0), beta, alpha, True, True))
    ref = orc.fused(to_np(bias), to_np(a), to_np(b), beta, alpha, NAME[dtype])
    ok, err = orc.check(to_np(c), ref, NAME[dtype])
    assert ok, f"wide tile addmm err={err}"
    A = rand((6, 600, 700), dtype, gen, full_range=full)
    B = rand((1, 700, 1100), dtype, gen, full_range=full)
    C = torch.empty(6, 600, 1100, dtype=dtype, device="cuda")
    dispatch._launch(A, B, C, 600, 1100, 700, 6, (700, 1, 600 * 700), (1100, 1, 0), (1100, 1, 600 * 1100),
                     backend=_lib.MB_BACKEND_TC, tile_n=512, cta_pair=2, autotune=False)
    ref = orc.product(to_np(A), np.broadcast_to(to_np(B), (6, 700, 1100)), NAME[dtype])
    ok, err = orc.check(to_np(C), ref, NAME[dtype])
    assert ok, f"wide tile broadcast bmm err={err}"


def test_complex32_workspace_does_not_clobber_tickets():
    """complex32 on the tensor cores keeps its expanded B' in the shared
    workspace; split-K plans that run after it must still find zeroed tickets."""
    import metalblas_b200 as mb
    gen = torch.Generator().manual_seed(9)
    ca = rand((512, 640), torch.complex32, gen)
    cb = rand((640, 384), torch.complex32, gen)
    cref = orc.product(to_np(ca), to_np(cb), "complex32")
    x = rand((1, 8192), torch.bfloat16, gen)
    w = rand((8192, 4096), torch.bfloat16, gen)
    gref = orc.product(to_np(x), to_np(w), "bfloat16")
    a = rand((128, 8192), torch.bfloat16, gen)
    b = rand((8192, 512), torch.bfloat16, gen)
    sref = orc.product(to_np(a), to_np(b), "bfloat16")
    for _ in range(3):
        ok, err = orc.check(to_np(mb.matmul(ca, cb)), cref, "complex32")
        assert ok, f"complex32 {err}"
        ok, err = orc.check(to_np(mb.matmul(x, w)), gref, "bfloat16")   # K-split GEMV
        assert ok, f"gemv after complex32 {err}"
        ok, err = orc.check(to_np(_run(a, b, 128, 4, -1)), sref, "bfloat16")  # split-K tensor-core
        assert ok, f"split-K after complex32 {err}"


def _gemv_rows(x, w, split, epilogue=None):
    """y[b] = W[b] x[b] with W rows contiguous along K (the x @ W^T layout),
    through the GEMV backend with a forced K split."""
    B, N, K = w.shape
    c = torch.empty(B, 1, N, dtype=x.dtype, device=x.device)
    dispatch._launch(x, w, c, 1, N, K, B, (K, 1, K), (1, K, N * K), (N, 1, N), epilogue=epilogue,
                     backend=_lib.MB_BACKEND_GEMV, split_k=split, autotune=False)
    return c


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32, torch.complex64,
                                   torch.int32], ids=NAME.get)
def test_gemv_rows_k_split(dtype):
    """The staged-x rows GEMV split along K: ragged K (not a multiple of the
    chunk), batches, the alpha/beta epilogue, and two calls in a row with the
    same tickets."""
    gen = torch.Generator().manual_seed(10)
    for (B, N, K) in [(1, 1000, 5000), (3, 77, 12288), (2, 4096, 3000)]:
        x = rand((B, 1, K), dtype, gen)
        w = rand((B, N, K), dtype, gen)
        bias = rand((B, 1, N), dtype, gen)
        ref = orc.product(to_np(x), to_np(w).transpose(0, 2, 1), NAME[dtype])
        fref = orc.fused(to_np(bias), to_np(x), to_np(w).transpose(0, 2, 1), 2, 3, NAME[dtype])
        for split in (1, 2, 3, 7):
            for _ in range(2):
                got = _gemv_rows(x, w, split)
                ok, err = orc.check(to_np(got), ref, NAME[dtype])
                assert ok, f"{(B, N, K)} split={split} err={err}"
            got = _gemv_rows(x, w, split, epilogue=(bias, (N, 1, N), 2, 3, True, True))
            ok, err = orc.check(to_np(got), fref, NAME[dtype])
            assert ok, f"{(B, N, K)} split={split} addmv err={err}"


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32], ids=NAME.get)
def test_gemv_thin_rows(dtype):
    """Thin products on the column GEMV with several x rows sharing each load
    of W (M = 2..4 with W row-major, and the mirrored N = 2..4 with A
    column-major): batches, K splits (ragged chunks), full and broadcast bias
    epilogues, and an N that is not a multiple of the vector width (no thin
    plan: the library falls back to another kernel); fp32 also with row
    blocks."""
    gen = torch.Generator().manual_seed(12)
    # fp32 takes up to 32 rows, in blocks of 8 (9 and 20: ragged last block)
    for M in (2, 3, 4) + ((7, 9, 20) if dtype == torch.float32 else ()):
        for (B, K, N) in [(1, 5000, 1000), (3, 1000, 2056), (2, 4096, 333)]:
            x = rand((B, M, K), dtype, gen)
            w = rand((B, K, N), dtype, gen)
            bias = rand((B, M, N), dtype, gen)
            bvec = rand((N,), dtype, gen)
            ref = orc.product(to_np(x), to_np(w), NAME[dtype])
            fref = orc.fused(to_np(bias), to_np(x), to_np(w), 2, 3, NAME[dtype])
            vref = orc.fused(to_np(bvec), to_np(x), to_np(w), 0.5, 1, NAME[dtype])
            a3, b3, c3 = (K, 1, M * K), (N, 1, K * N), (N, 1, M * N)
            for split in (0, 1, 2, 5):
                for be in (_lib.MB_BACKEND_GEMV, _lib.MB_BACKEND_AUTO):
                    c = torch.empty(B, M, N, dtype=dtype, device=x.device)
                    dispatch._launch(x, w, c, M, N, K, B, a3, b3, c3, backend=be, split_k=split if be else 0,
                                     autotune=False)
                    ok, err = orc.check(to_np(c), ref, NAME[dtype])
                    assert ok, f"M={M} {(B, K, N)} split={split} backend={be} err={err}"
                c = torch.empty(B, M, N, dtype=dtype, device=x.device)
                dispatch._launch(x, w, c, M, N, K, B, a3, b3, c3, epilogue=(bias, (N, 1, M * N), 2, 3, True, True),
                                 backend=_lib.MB_BACKEND_GEMV, split_k=split, autotune=False)
                ok, err = orc.check(to_np(c), fref, NAME[dtype])
                assert ok, f"M={M} {(B, K, N)} split={split} addmm err={err}"
                dispatch._launch(x, w, c, M, N, K, B, a3, b3, c3, epilogue=(bvec, (0, 1, 0), 0.5, 1, True, True),
                                 backend=_lib.MB_BACKEND_GEMV, split_k=split, autotune=False)
                ok, err = orc.check(to_np(c), vref, NAME[dtype])
                assert ok, f"M={M} {(B, K, N)} split={split} bias-vector err={err}"
            # mirrored: C[N, M] = A[N, K] @ x^T with A column-major (stored [K, N])
            at = rand((B, K, N), dtype, gen)
            xt = rand((B, K, M), dtype, gen)
            ref_t = orc.product(to_np(at).transpose(0, 2, 1), to_np(xt), NAME[dtype])
            for split in (0, 3):
                c = torch.empty(B, N, M, dtype=dtype, device=x.device)
                dispatch._launch(at, xt, c, N, M, K, B, (1, N, K * N), (M, 1, K * M), (M, 1, N * M),
                                 backend=_lib.MB_BACKEND_GEMV, split_k=split, autotune=False)
                ok, err = orc.check(to_np(c), ref_t, NAME[dtype])
                assert ok, f"thin N={M} {(B, K, N)} split={split} err={err}"


def test_no_device_timeouts():
    from metalblas_b200 import kernels
    assert kernels.device_status() == 0


def _offset(t):
    """[1:, 1:] of a buffer one row and one column larger (lda = cols + 1, storage
    offset > 0): the reference's "offset" layout, which TMA cannot address."""
    big = torch.zeros(*t.shape[:-2], t.shape[-2] + 1, t.shape[-1] + 1, dtype=t.dtype, device=t.device)
    big[..., 1:, 1:] = t
    return big[..., 1:, 1:]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.int8, torch.uint8], ids=NAME.get)
def test_packed_operands_on_tensor_cores(dtype):
    """Views TMA cannot load in place are packed into the workspace and run on
    the tensor cores (plan "tc_packed"); results match the oracle for plain,
    thin-M (swapped), batched/broadcast and epilogue cases."""
    import metalblas_b200 as mb
    gen = torch.Generator().manual_seed(14)
    full = dtype in (torch.int8, torch.uint8)
    for (M, N, K) in [(512, 640, 768), (16, 1000, 2048), (1000, 96, 1100)]:
        a = rand((M, K), dtype, gen, full_range=full)
        b = rand((K, N), dtype, gen, full_range=full)
        ref = orc.product(to_np(a), to_np(b), NAME[dtype])
        # row-major offset views, and a column-major one (lda = M + 1)
        for av, bv in ((_offset(a), b), (a, _offset(b)), (_offset(a), _offset(b)), (_offset(a.t().contiguous()).t(), b)):
            expect = "tc_packed" if M * N * K >= 1e8 else "simt"  # small products stay on CUDA cores
            assert mb.kernels.plan(av, bv).startswith(expect), mb.kernels.plan(av, bv)
            ok, err = orc.check(to_np(mb.matmul(av, bv)), ref, NAME[dtype])
            assert ok, f"{(M, N, K)} err={err}"
    # batched with a broadcast B, and addmm
    A = rand((5, 300, 520), dtype, gen, full_range=full)
    B = rand((1, 520, 260), dtype, gen, full_range=full)
    ref = orc.product(to_np(A), np.broadcast_to(to_np(B), (5, 520, 260)), NAME[dtype])
    ok, err = orc.check(to_np(mb.matmul(_offset(A), _offset(B))), ref, NAME[dtype])
    assert ok, f"batched err={err}"
    a = rand((700, 900), dtype, gen, full_range=full)
    b = rand((900, 500), dtype, gen, full_range=full)
    bias = rand((500,), dtype, gen, full_range=full)
    beta, alpha = (3, -2) if full else (0.5, 2.0)
    got = mb.addmm(bias, _offset(a), b, beta=beta, alpha=alpha)
    ok, err = orc.check(to_np(got), orc.fused(to_np(bias), to_np(a), to_np(b), beta, alpha, NAME[dtype]), NAME[dtype])
    assert ok, f"addmm err={err}"


def test_fp32_3xtf32_matches_oracle():
    """fp32 on the tensor cores (3xTF32: tf32 high/low split, three MMAs per
    K-step) stays inside the north star's 1e-5 relative-Frobenius bound across
    layouts, thin M (swap), split / stream-K tails, batches with a broadcast
    operand and the alpha/beta/bias epilogue."""
    import metalblas_b200 as mb
    gen = torch.Generator().manual_seed(15)
    # backend="mpp_tensor" puts any fp32 product on the tensor cores; the planner
    # chooses them by itself for compute-heavy shapes (2048^3 here)
    for (M, N, K) in [(512, 640, 768), (1000, 1000, 1000), (64, 4096, 2048), (256, 512, 16384), (2048, 2048, 2048)]:
        a = rand((M, K), torch.float32, gen)
        b = rand((K, N), torch.float32, gen)
        ref = orc.product(to_np(a), to_np(b), "float32")
        for av, bv in ((a, b), (a.t().contiguous().t(), b), (a, b.t().contiguous().t()), (_offset(a), _offset(b))):
            plan = mb.kernels.plan(av, bv, backend="mpp_tensor")
            assert plan.startswith("tc_3xtf32"), plan
            ok, err = orc.check(to_np(mb.matmul(av, bv, backend="mpp_tensor")), ref, "float32")
            assert ok, f"{(M, N, K)} err={err}"
        if M * N * K >= 512 * (M * K + K * N):
            assert mb.kernels.plan(a, b).startswith("tc_3xtf32")
    A = rand((8, 1024, 1024), torch.float32, gen)
    B = rand((1, 1024, 1024), torch.float32, gen)
    bias = rand((8, 1024, 1024), torch.float32, gen)
    assert mb.kernels.plan(A, B).startswith("tc_3xtf32")  # compute-heavy: the planner's own choice
    got = mb.baddbmm(bias, A, B.expand(8, 1024, 1024), beta=0.5, alpha=-2.0)
    ref = orc.fused(to_np(bias), to_np(A), np.broadcast_to(to_np(B), (8, 1024, 1024)), 0.5, -2.0, "float32")
    ok, err = orc.check(to_np(got), ref, "float32")
    assert ok, f"baddbmm err={err}"
    # non-finite inputs propagate like the CUDA-core kernel's
    a = rand((256, 512), torch.float32, gen)
    b = rand((512, 384), torch.float32, gen)
    a[3, 7] = float("inf")
    a[5, 1] = float("nan")
    got = mb.matmul(a, b, backend="mpp_tensor")
    simd = mb.matmul(a, b, backend="simd")
    assert torch.equal(torch.isnan(got), torch.isnan(simd)) and torch.equal(torch.isinf(got), torch.isinf(simd))


def test_complex64_3xtf32_matches_oracle():
    """complex64 on the tensor cores: one real 3xTF32 GEMM in the block form
    C' = A' B' (A' the interleaved storage of A, B' the 2x2 real blocks of B),
    with the split pass reading the complex operands in place.  Checked within
    the 1e-5 bound across layouts, conj(A) / conj(B), thin M, batches with a
    broadcast operand, real alpha/beta with a bias (on the tensor cores) and a
    complex alpha (the FFMA kernel), and non-finite inputs."""
    import metalblas_b200 as mb
    gen = torch.Generator().manual_seed(16)
    for (M, N, K) in [(512, 640, 768), (1000, 1000, 1000), (3, 2048, 512), (256, 96, 4096)]:
        a = rand((M, K), torch.complex64, gen)
        b = rand((K, N), torch.complex64, gen)
        for av, bv in ((a, b), (a.t().contiguous().t(), b), (a, b.t().contiguous().t()), (a.conj(), b),
                       (a, b.conj()), (a.conj(), b.conj()), (_offset(a), _offset(b))):
            ref = orc.product(to_np(av.resolve_conj()), to_np(bv.resolve_conj()), "complex64")
            plan = mb.kernels.plan(av, bv, backend="mpp_tensor")
            assert plan.startswith("tc_c64x3"), plan
            ok, err = orc.check(to_np(mb.matmul(av, bv, backend="mpp_tensor")), ref, "complex64")
            assert ok, f"{(M, N, K)} conj=({av.is_conj()}, {bv.is_conj()}) err={err}"
            ok, err = orc.check(to_np(mb.matmul(av, bv)), ref, "complex64")
            assert ok, f"{(M, N, K)} auto err={err}"
    a = rand((2048, 1024), torch.complex64, gen)
    b = rand((1024, 1024), torch.complex64, gen)
    assert mb.kernels.plan(a, b).startswith("tc_c64x3")  # compute-heavy: the planner's own choice
    bias = rand((1024,), torch.complex64, gen)
    for beta, alpha in ((0.5, -2.0), (0.0, 1.0), (1.5, 0.0), (0.5, complex(2.0, 1.0)), (complex(0, 1), 1.0)):
        got = mb.addmm(bias, a, b, beta=beta, alpha=alpha)
        ref = orc.fused(to_np(bias), to_np(a), to_np(b), beta, alpha, "complex64")
        ok, err = orc.check(to_np(got), ref, "complex64")
        assert ok, f"addmm beta={beta} alpha={alpha} err={err}"
    A = rand((6, 256, 384), torch.complex64, gen)
    B = rand((1, 384, 320), torch.complex64, gen)
    bias3 = rand((6, 256, 320), torch.complex64, gen)
    got = mb.baddbmm(bias3, A, B.expand(6, 384, 320), beta=0.5, alpha=2.0)
    ref = orc.fused(to_np(bias3), to_np(A), np.broadcast_to(to_np(B), (6, 384, 320)), 0.5, 2.0, "complex64")
    ok, err = orc.check(to_np(got), ref, "complex64")
    assert ok, f"baddbmm err={err}"
    # non-finite inputs propagate like the CUDA-core kernel's
    a = rand((256, 512), torch.complex64, gen)
    b = rand((512, 384), torch.complex64, gen)
    a[3, 7] = complex(float("inf"), 0.0)
    a[5, 1] = complex(0.0, float("nan"))
    got = mb.matmul(a, b, backend="mpp_tensor")
    simd = mb.matmul(a, b, backend="simd")
    assert torch.equal(torch.isnan(got), torch.isnan(simd)) and torch.equal(torch.isinf(got), torch.isinf(simd))


@pytest.mark.parametrize("dtype", [torch.int16, torch.int32, torch.int64], ids=NAME.get)
def test_integer_byte_planes_bit_exact(dtype):
    """16/32/64-bit integer products on the 8-bit tensor cores (byte planes,
    one u8 GEMM per shift accumulated into C with wrapping arithmetic) are
    bit-exact against the oracle over the full type range: layouts, thin M,
    K not a multiple of 16, K long enough for several exact chunks (int64),
    the alpha/beta/bias epilogue including alpha == 0, and batches with a
    broadcast operand."""
    import metalblas_b200 as mb
    name = NAME[dtype]
    gen = torch.Generator().manual_seed(17)
    # K = 17000 runs in several exact chunks for every width (int16 2, int32 3, int64 5)
    for (M, N, K) in [(256, 320, 768), (1000, 1000, 1000), (130, 70, 5000), (4, 600, 300), (300, 200, 17),
                      (40, 48, 17000)]:
        a = rand((M, K), dtype, gen, full_range=True)
        b = rand((K, N), dtype, gen, full_range=True)
        ref = orc.product(to_np(a), to_np(b), name)
        for av, bv in ((a, b), (a.t().contiguous().t(), b), (a, b.t().contiguous().t()), (_offset(a), _offset(b))):
            plan = mb.kernels.plan(av, bv, backend="mpp_tensor")
            assert plan.startswith("tc_int_planes"), plan
            ok, err = orc.check(to_np(mb.matmul(av, bv, backend="mpp_tensor")), ref, name)
            assert ok, f"{(M, N, K)} err={err}"
        ok, err = orc.check(to_np(mb.matmul(a, b)), ref, name)
        assert ok, f"{(M, N, K)} auto err={err}"
    a = rand((512, 384), dtype, gen, full_range=True)
    b = rand((384, 640), dtype, gen, full_range=True)
    bias = rand((640,), dtype, gen, full_range=True)
    for beta, alpha in ((3, -7), (0, 1), (1, 0), (-2, 5)):
        got = mb.addmm(bias, a, b, beta=beta, alpha=alpha)
        ref = orc.fused(to_np(bias), to_np(a), to_np(b), beta, alpha, name)
        ok, err = orc.check(to_np(got), ref, name)
        assert ok, f"addmm beta={beta} alpha={alpha} err={err}"
    A = rand((5, 200, 300), dtype, gen, full_range=True)
    B = rand((1, 300, 260), dtype, gen, full_range=True)
    bias3 = rand((5, 200, 260), dtype, gen, full_range=True)
    got = mb.baddbmm(bias3, A, B.expand(5, 300, 260), beta=2, alpha=-3)
    ref = orc.fused(to_np(bias3), to_np(A), np.broadcast_to(to_np(B), (5, 300, 260)), 2, -3, name)
    ok, err = orc.check(to_np(got), ref, name)
    assert ok, f"baddbmm err={err}"


def test_nd_broadcast_batches_read_operands_in_place(monkeypatch):
    """matmul over multi-dim broadcast batches (the reference reshapes, which copies): when the
    expanded batch dims cannot be flattened into one stride, the leading dim is
    walked instead of copying the operand; every launch reads the caller's own
    storage."""
    import metalblas_b200 as mb
    from metalblas_b200 import dispatch
    gen = torch.Generator().manual_seed(16)
    cases = [((2, 3, 64, 96), (3, 96, 80)), ((2, 1, 64, 96), (1, 3, 96, 80)), ((4, 64, 96), (96, 80)),
             ((2, 3, 64, 96), (2, 3, 96, 80)), ((5, 1, 33, 40), (1, 7, 40, 20))]
    real_bmm = dispatch.bmm
    for dtype in (torch.bfloat16, torch.float32, torch.int32):
        for sa, sb in cases:
            a = rand(sa, dtype, gen)
            b = rand(sb, dtype, gen)
            storages = {a.untyped_storage().data_ptr(), b.untyped_storage().data_ptr()}
            seen = []

            def spy(x, y, *, out=None):
                seen.append((x.untyped_storage().data_ptr(), y.untyped_storage().data_ptr()))
                return real_bmm(x, y, out=out)
            monkeypatch.setattr(dispatch, "bmm", spy)
            got = mb.matmul(a, b)
            monkeypatch.setattr(dispatch, "bmm", real_bmm)
            assert seen and all(p in storages and q in storages for p, q in seen), (sa, sb)
            ref = orc.product(np.broadcast_to(to_np(a), got.shape[:-2] + a.shape[-2:]),
                              np.broadcast_to(to_np(b), got.shape[:-2] + b.shape[-2:]), NAME[dtype])
            ok, err = orc.check(to_np(got), ref, NAME[dtype])
            assert ok, f"{dtype} {sa} @ {sb} err={err}"
