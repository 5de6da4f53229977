"""The BASELINE configurations at full size.

Small configs are checked against the full fp64 / exact oracle.  Where the full
oracle would take minutes on the host, a seeded sample of rows (or columns, or
batches) of the output is checked exactly against the oracle computed for that
sample only; the sample is drawn independently of the kernel's tiling, so a
tile-level error anywhere is caught with high probability.  Tolerances are the
north star's: integers bit-exact, relative Frobenius <= 1e-2 for bf16 / fp16 /
complex32 and <= 1e-5 for fp32 / complex64.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import oracle as orc
from tests.helpers import NAME, rand, to_np

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def mb():
    import metalblas_b200
    return metalblas_b200


def _check(got, ref, dtype, tag):
    ok, err = orc.check(got, ref, NAME[dtype])
    assert ok, f"{tag}: error {err:.3e}"


def _gpu_randn(shape, dtype, seed, std=1.0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return (std * torch.randn(shape, generator=g, device="cuda")).to(dtype)


# ------------------------------------------------------------------ config 1
def test_config1_gemm_and_addmm(mb):
    """A[2048,4096] @ B[4096,2048] bf16, N(0,1) seed 0; addmm bias[2048], beta=0.5, alpha=2."""
    g = torch.Generator().manual_seed(0)
    a = torch.randn(2048, 4096, generator=g).to(torch.bfloat16)
    b = torch.randn(4096, 2048, generator=g).to(torch.bfloat16)
    bias = torch.randn(2048, generator=g).to(torch.bfloat16)
    ad, bd, biasd = a.cuda(), b.cuda(), bias.cuda()
    ref = orc.product(a.float().numpy(), b.float().numpy(), "bfloat16")
    _check(to_np(mb.matmul(ad, bd)), ref, torch.bfloat16, "config1 matmul")
    ref2 = orc.fused(bias.float().numpy(), a.float().numpy(), b.float().numpy(), 0.5, 2.0, "bfloat16")
    _check(to_np(mb.addmm(biasd, ad, bd, beta=0.5, alpha=2.0)), ref2, torch.bfloat16, "config1 addmm")


# ------------------------------------------------------------------ config 2
GEMV = [(M, K, N) for M in (1, 4, 16) for K in (4096, 8192, 16384) for N in (4096, 14336, 28672)]
GEMV_CASES = [(s, dt, lay) for dt in (torch.bfloat16, torch.float16) for s in GEMV
              for lay in ("x@W", "x@Wt", "x@Wcm")]


@pytest.mark.parametrize("shape,dtype,layout", GEMV_CASES,
                         ids=[f"{NAME[c[1]]}-{c[2]}-{c[0][0]}x{c[0][1]}x{c[0][2]}" for c in GEMV_CASES])
def test_config2_gemv_sweep(mb, shape, dtype, layout):
    """M in {1,4,16} x K in {4096,8192,16384} x N in {4096,14336,28672}; W ~ N(0,0.02), x ~ N(0,1), seed 1.
    x@W: W [K,N] row-major; x@Wt: W stored [N,K] (the product reads it transposed);
    x@Wcm: W [K,N] column-major view."""
    M, K, N = shape
    x = _gpu_randn((M, K), dtype, 1)
    if layout == "x@W":
        W = _gpu_randn((K, N), dtype, 2, 0.02)
    else:
        W = _gpu_randn((N, K), dtype, 2, 0.02).t()   # both "Wt" and "cm" read a [K,N] column-major view
    y = mb.matmul(x, W)
    cols = torch.randperm(N, generator=torch.Generator().manual_seed(3))[:256].sort().values
    ref = orc.product(to_np(x), to_np(W[:, cols.cuda()]), NAME[dtype])
    _check(to_np(y[:, cols.cuda()]), ref, dtype, f"gemv {shape} {layout}")


# Batched thin products, the reference's batched gemv_bt layout
# (metalblas/shaders/gemv_bt.h:67-74: a batch of [M <= 16, K] @ [K, N] with W
# row-major, or read transposed from [N, K] storage).
BATCHED_THIN = [(B, M, K, N, dt, lay) for dt in (torch.bfloat16, torch.float16) for (B, M, K, N) in
                ((8, 4, 4096, 4096), (8, 16, 4096, 4096), (4, 4, 8192, 14336), (4, 16, 8192, 14336))
                for lay in ("W", "Wt")]


@pytest.mark.parametrize("B,M,K,N,dtype,layout", BATCHED_THIN,
                         ids=[f"{NAME[c[4]]}-{c[5]}-{c[0]}x{c[1]}x{c[2]}x{c[3]}" for c in BATCHED_THIN])
def test_config2_batched_thin(mb, B, M, K, N, dtype, layout):
    """[B, M, K] @ [B, K, N] with M in {4, 16}: W ~ N(0, 0.02), x ~ N(0, 1), seed 1;
    "Wt": each batch's W stored [N, K] and read transposed."""
    x = _gpu_randn((B, M, K), dtype, 1)
    if layout == "W":
        W = _gpu_randn((B, K, N), dtype, 2, 0.02)
    else:
        W = _gpu_randn((B, N, K), dtype, 2, 0.02).transpose(1, 2)
    y = mb.bmm(x, W)
    cols = torch.randperm(N, generator=torch.Generator().manual_seed(3))[:256].sort().values.cuda()
    for b in (0, B - 1):
        ref = orc.product(to_np(x[b]), to_np(W[b][:, cols]), NAME[dtype])
        _check(to_np(y[b][:, cols]), ref, dtype, f"batched thin {B}x{M}x{K}x{N} {layout} batch {b}")


def test_config2_w_at_x(mb):
    """y = W @ x (the gemv_nt orientation, metalblas/shaders/gemv_nt.h:16-101):
    W [N, K] row-major, bf16 and fp16, through mv."""
    for dtype in (torch.bfloat16, torch.float16):
        for (N, K) in ((4096, 4096), (14336, 8192), (28672, 16384)):
            W = _gpu_randn((N, K), dtype, 2, 0.02)
            x = _gpu_randn((K,), dtype, 1)
            y = mb.mv(W, x)
            rows = torch.randperm(N, generator=torch.Generator().manual_seed(3))[:256].sort().values.cuda()
            ref = orc.product(to_np(W[rows]), to_np(x)[:, None], NAME[dtype])[:, 0]
            _check(to_np(y[rows]), ref, dtype, f"W@x {N}x{K}")


# ------------------------------------------------------------------ config 3
BMM = [((8, 512, 256), (8, 256, 512)), ((64, 2048, 128), (64, 128, 2048)), ((256, 1024, 1024), (256, 1024, 1024)),
       ((64, 512, 256), (1, 256, 512))]


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16], ids=NAME.get)
@pytest.mark.parametrize("shapes", BMM, ids=lambda s: f"{s[0]}@{s[1]}")
def test_config3_bmm(mb, shapes, dtype):
    sa, sb = shapes
    a = _gpu_randn(sa, dtype, 2)
    b = _gpu_randn(sb, dtype, 3)
    bb = b.expand(sa[0], *sb[1:]) if sb[0] == 1 else b
    c = mb.bmm(a, bb)
    idx = torch.randperm(sa[0], generator=torch.Generator().manual_seed(4))[:4].tolist()
    for i in idx:
        ref = orc.product(to_np(a[i]), to_np(bb[i]), NAME[dtype])
        _check(to_np(c[i]), ref, dtype, f"bmm {shapes} batch {i}")


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16], ids=NAME.get)
@pytest.mark.parametrize("layout", ["transposed", "sliced", "offset"])
def test_config3_bmm_views(mb, dtype, layout):
    B, M, N, K = 16, 384, 320, 256
    if layout == "transposed":
        a = _gpu_randn((B, K, M), dtype, 5).transpose(1, 2)
        b = _gpu_randn((B, N, K), dtype, 6).transpose(1, 2)
    elif layout == "sliced":
        a = _gpu_randn((B, 2 * M, K), dtype, 5)[:, ::2]
        b = _gpu_randn((B, 2 * K, N), dtype, 6)[:, ::2]
    else:
        a = _gpu_randn((B, M + 1, K + 1), dtype, 5)[:, 1:, 1:]
        b = _gpu_randn((B, K + 1, N + 1), dtype, 6)[:, 1:, 1:]
    c = mb.bmm(a, b)
    ref = orc.product(to_np(a), to_np(b), NAME[dtype])
    _check(to_np(c), ref, dtype, f"bmm {layout}")


# ------------------------------------------------------------------ config 4
def _int_inputs(shape, dtype, seed, full_range, lo=-1000, hi=1001):
    g = torch.Generator().manual_seed(seed)
    if full_range:
        info = torch.iinfo(dtype)
        return torch.randint(info.min, info.max + 1, shape, dtype=dtype, generator=g)
    return torch.randint(lo, hi, shape, dtype=dtype, generator=g)


def _layout(t, lay):
    """rm: row-major; cm: column-major view of the same values; offset: [1:,1:] view (ld+1)."""
    if lay == "rm":
        return t.cuda()
    if lay == "cm":
        return t.t().contiguous().t().cuda()
    big = torch.zeros(t.shape[0] + 1, t.shape[1] + 1, dtype=t.dtype)
    big[1:, 1:] = t
    return big.cuda()[1:, 1:]


INT_GEMM = ([(dt, n, lays) for dt in (torch.int8, torch.uint8) for n in (4096, 8192)
             for lays in (("rm", "rm"), ("rm", "cm"), ("cm", "cm"), ("offset", "offset"))]
            + [(dt, 2048, lays) for dt in (torch.int16, torch.int32, torch.int64)
               for lays in (("rm", "rm"), ("rm", "cm"), ("cm", "cm"), ("offset", "offset"))])


@pytest.mark.parametrize("dtype,n,lays", INT_GEMM, ids=[f"{NAME[c[0]]}-{c[1]}-{c[2][0]}_{c[2][1]}" for c in INT_GEMM])
def test_config4_integer_gemm(mb, dtype, n, lays):
    full = dtype in (torch.int8, torch.uint8)
    a = _int_inputs((n, n), dtype, 3 if full else 4, full)
    b = _int_inputs((n, n), dtype, 13 if full else 14, full)
    c = mb.matmul(_layout(a, lays[0]), _layout(b, lays[1]))
    assert c.dtype == dtype
    rows = torch.randperm(n, generator=torch.Generator().manual_seed(5))[:64].sort().values
    ref = orc.product(a[rows].numpy(), b.numpy(), NAME[dtype])
    _check(c[rows.cuda()].cpu().numpy(), ref, dtype, f"int gemm {dtype} {n} {lays}")


@pytest.mark.parametrize("lay", ["rm", "cm", "offset"])
def test_config4_int32_gemv(mb, lay):
    x = _int_inputs((1, 8192), torch.int32, 4, False)
    W = _int_inputs((8192, 8192), torch.int32, 14, False)
    y = mb.matmul(x.cuda(), _layout(W, lay))
    _check(y.cpu().numpy(), orc.product(x.numpy(), W.numpy(), "int32"), torch.int32, f"int32 gemv {lay}")


# ------------------------------------------------------------------ config 5
@pytest.mark.parametrize("dtype", [torch.complex64, torch.complex32], ids=NAME.get)
@pytest.mark.parametrize("form", ["A@B", "conj(A)@B", "At@B", "gemv"])
def test_config5_complex(mb, dtype, form):
    n = 4096
    g = torch.Generator().manual_seed(5)
    m = 1 if form == "gemv" else n
    a = torch.complex(torch.randn(m, n, generator=g), torch.randn(m, n, generator=g)).to(dtype)
    b = torch.complex(torch.randn(n, n, generator=g), torch.randn(n, n, generator=g)).to(dtype)
    ad, bd = a.cuda(), b.cuda()
    if form == "conj(A)@B":
        ad = ad.conj()
    elif form == "At@B":
        ad = ad.t().contiguous().t()
    c = mb.matmul(ad, bd)
    rows = torch.arange(0, m, max(1, m // 48))
    an = to_np(ad)[rows.numpy()]
    ref = orc.product(an, to_np(b), NAME[dtype])
    _check(to_np(c)[rows.numpy()], ref, dtype, f"complex {form}")


def test_config5_large_bf16(mb):
    """bf16 16384^3, N(0,1), seed 6 (row-sampled oracle)."""
    n = 16384
    a = _gpu_randn((n, n), torch.bfloat16, 6)
    b = _gpu_randn((n, n), torch.bfloat16, 7)
    c = mb.matmul(a, b)
    rows = torch.randperm(n, generator=torch.Generator().manual_seed(6))[:48].sort().values.cuda()
    ref = orc.product(to_np(a[rows]), to_np(b), "bfloat16")
    _check(to_np(c[rows]), ref, torch.bfloat16, "bf16 16384^3")


def test_config5_skinny_split_k(mb):
    """bf16 128 x 8192 x 65536 (split-K regime), N(0,1), seed 6."""
    a = _gpu_randn((128, 65536), torch.bfloat16, 6)
    b = _gpu_randn((65536, 8192), torch.bfloat16, 7)
    c = mb.matmul(a, b)
    rows = torch.arange(0, 128, 8).cuda()
    ref = orc.product(to_np(a[rows]), to_np(b), "bfloat16")
    _check(to_np(c[rows]), ref, torch.bfloat16, "skinny")
    assert mb.kernels.device_status() == 0
