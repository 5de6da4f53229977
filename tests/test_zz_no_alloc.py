"""The allocation-free entry point, mb_gemm_noalloc, against mb_gemm.

mb_gemm_noalloc serves callers that cannot allocate device memory and have no
workspace to pass (inference runtimes that fix their memory at start-up and
forbid allocation on the request path, plugin hosts that hand over only the
input/output buffers and a stream, C-ABI callers without a CUDA allocator).  It
runs the same plan as mb_gemm, but its split-K scratch is a buffer built into
the library, of MB_NOALLOC_SCRATCH_BYTES per GPU, shared by every call.

These tests call both entry points through the C ABI on shapes whose plans use
split-K scratch (tensor-core split-K, the K-split GEMV) and on one that uses
none, twice in a row for the new entry point, and compare with mb_gemm's output
using the same tolerances as the rest of the suite (integers bit-exact,
relative Frobenius <= 1e-2 for bf16).  The file runs last in the suite and also
passes alone in a fresh process: the reference result uses its own zero-filled
workspace, not any cache.
"""
from __future__ import annotations

import ctypes

import pytest
import torch

from metalblas_b200 import _lib
from oracle import oracle as orc
from tests.helpers import NAME, rand, to_np

pytestmark = pytest.mark.gpu

CAPACITY = 16 * 1024 * 1024   # MB_NOALLOC_SCRATCH_BYTES in include/metalblas_b200.h


def _desc(a, b, c, tile_n=0, split_k=0, epilogue=None):
    M, K = a.shape
    N = b.shape[1]
    d = _lib.new_desc()
    d.dtype = _lib.DTYPE_CODE[a.dtype]
    d.backend = _lib.MB_BACKEND_AUTO
    d.M, d.N, d.K, d.batch = M, N, K, 1
    d.A, d.B, d.C = a.data_ptr(), b.data_ptr(), c.data_ptr()
    d.a_rs, d.a_cs = a.stride()
    d.b_rs, d.b_cs = b.stride()
    d.c_rs, d.c_cs = c.stride()
    d.tile_n, d.split_k = tile_n, split_k
    if epilogue is not None:
        bias, beta, alpha = epilogue
        d.epilogue, d.alpha_nz, d.beta_nz = 1, 1, 1
        d.bias, d.bias_rs, d.bias_cs = bias.data_ptr(), 0, 1
        d.alpha_re, d.beta_re = float(alpha), float(beta)
        d.ialpha, d.ibeta = int(alpha), int(beta)
    return d


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _with_mb_gemm(a, b, **kw):
    """The existing entry point, with a caller-allocated zero-filled workspace."""
    lib = _lib.load()
    c = torch.empty(a.shape[0], b.shape[1], dtype=a.dtype, device="cuda")
    d = _desc(a, b, c, **kw)
    n = int(lib.mb_gemm_workspace_size(ctypes.byref(d)))
    ws = torch.zeros(max(n, 1), dtype=torch.uint8, device="cuda")
    d.workspace, d.workspace_bytes = ws.data_ptr(), ws.numel()
    _lib.raise_for(lib.mb_gemm(ctypes.byref(d), _stream()))
    torch.cuda.synchronize()
    return c, n, _lib.plan_query(d)


def _with_noalloc(a, b, **kw):
    lib = _lib.load()
    c = torch.full((a.shape[0], b.shape[1]), 77, dtype=a.dtype, device="cuda")
    d = _desc(a, b, c, **kw)
    _lib.raise_for(lib.mb_gemm_noalloc(ctypes.byref(d), _stream()), "mb_gemm_noalloc")
    torch.cuda.synchronize()
    return c


CASES = [
    # (tag, dtype, M, N, K, tile_n, split_k, epilogue)
    ("tc-split-bf16", torch.bfloat16, 128, 8192, 8192, 128, 2, False),
    ("tc-split-bf16-addmm", torch.bfloat16, 256, 1024, 16384, 64, 4, True),
    ("tc-split-int8", torch.int8, 128, 2048, 8192, 128, 4, True),
    ("gemv-ksplit-bf16", torch.bfloat16, 1, 4096, 16384, 0, 0, False),
    ("no-scratch-bf16", torch.bfloat16, 512, 512, 512, 0, 1, False),
]


@pytest.mark.parametrize("tag,dtype,M,N,K,tile_n,split_k,epi", CASES, ids=[c[0] for c in CASES])
def test_noalloc_matches_mb_gemm_twice(tag, dtype, M, N, K, tile_n, split_k, epi):
    gen = torch.Generator().manual_seed(11)
    full = dtype is torch.int8
    a = rand((M, K), dtype, gen, full_range=full)
    b = rand((K, N), dtype, gen, full_range=full)
    epilogue = (rand((N,), dtype, gen, full_range=full), 2, 3) if epi else None
    ref, need, plan = _with_mb_gemm(a, b, tile_n=tile_n, split_k=split_k, epilogue=epilogue)
    if tag != "no-scratch-bf16":
        assert need > 0, f"{tag}: expected a plan that uses scratch, got {plan}"
    assert need <= CAPACITY
    for call in range(2):
        got = _with_noalloc(a, b, tile_n=tile_n, split_k=split_k, epilogue=epilogue)
        ok, err = orc.check(to_np(got), to_np(ref).astype("float64") if not full else to_np(ref).astype("int64"),
                            NAME[dtype])
        assert ok, f"{tag} call {call}: differs from mb_gemm (error {err:.3e}; plan {plan})"


def test_noalloc_rejects_plans_beyond_capacity():
    lib = _lib.load()
    gen = torch.Generator().manual_seed(12)
    a = rand((128, 8192), torch.bfloat16, gen)
    b = rand((8192, 8192), torch.bfloat16, gen)
    c = torch.empty(128, 8192, dtype=torch.bfloat16, device="cuda")
    d = _desc(a, b, c, tile_n=256, split_k=8)      # 32 tiles x 8 splits x 128 KiB of partials
    d.workspace_bytes = -1
    assert lib.mb_gemm_workspace_size(ctypes.byref(d)) > CAPACITY
    rc = lib.mb_gemm_noalloc(ctypes.byref(d), _stream())
    assert rc == _lib.MB_ERR_WORKSPACE
    msg = _lib.last_error()
    assert "split_k=1" in msg and str(CAPACITY) in msg
    # the suggested fix works
    d.split_k = 1
    _lib.raise_for(lib.mb_gemm_noalloc(ctypes.byref(d), _stream()), "mb_gemm_noalloc")
    torch.cuda.synchronize()
    ref = orc.product(to_np(a[:8]), to_np(b), "bfloat16")
    ok, err = orc.check(to_np(c[:8]), ref, "bfloat16")
    assert ok, err


def test_noalloc_replans_auto_shapes_beyond_capacity():
    """A decode-sized bf16 product whose first-choice plan (a split-K tail)
    needs more than the built-in scratch: with no split asked for, the call is
    planned again without scratch and must still run, matching mb_gemm and the
    oracle on a row sample."""
    lib = _lib.load()
    gen = torch.Generator().manual_seed(13)
    a = rand((128, 16384), torch.bfloat16, gen)
    b = rand((16384, 8192), torch.bfloat16, gen)
    c = torch.empty(128, 8192, dtype=torch.bfloat16, device="cuda")
    d = _desc(a, b, c)
    d.workspace_bytes = -1
    need = int(lib.mb_gemm_workspace_size(ctypes.byref(d)))
    assert need > CAPACITY, f"expected a first-choice plan beyond the scratch, got {need} bytes"
    ref, _, plan = _with_mb_gemm(a, b)
    for call in range(2):
        got = _with_noalloc(a, b)
        ok, err = orc.check(to_np(got), to_np(ref).astype("float64"), "bfloat16")
        assert ok, f"call {call}: differs from mb_gemm (error {err:.3e}; mb_gemm plan {plan})"
    rows = [0, 37, 127]
    want = orc.product(to_np(a[rows]), to_np(b), "bfloat16")
    ok, err = orc.check(to_np(got[rows]), want, "bfloat16")
    assert ok, f"oracle row sample: error {err:.3e}"


def test_noalloc_fp32_cuda_core_fallback_against_oracle():
    """fp32 at 1024^3 runs as 3xTF32 in mb_gemm, whose split operands need
    more than the built-in scratch; under backend AUTO the allocation-free call
    computes it on the CUDA-core FFMA kernel instead, within the fp32 bound
    (relative Frobenius <= 1e-5 against the fp64 oracle)."""
    lib = _lib.load()
    gen = torch.Generator().manual_seed(14)
    a = rand((1024, 1024), torch.float32, gen)
    b = rand((1024, 1024), torch.float32, gen)
    c = torch.empty(1024, 1024, dtype=torch.float32, device="cuda")
    d = _desc(a, b, c)
    d.workspace_bytes = -1
    assert int(lib.mb_gemm_workspace_size(ctypes.byref(d))) > CAPACITY
    want = orc.product(to_np(a), to_np(b), "float32")
    for call in range(2):
        got = _with_noalloc(a, b)
        ok, err = orc.check(to_np(got), want, "float32")
        assert ok, f"call {call}: error {err:.3e}"


def test_noalloc_direct_oracle_check_with_epilogue():
    """One split-K addmm through the allocation-free entry point checked against
    the oracle itself (not only against mb_gemm)."""
    gen = torch.Generator().manual_seed(15)
    a = rand((256, 16384), torch.bfloat16, gen)
    b = rand((16384, 1024), torch.bfloat16, gen)
    bias = rand((1024,), torch.bfloat16, gen)
    got = _with_noalloc(a, b, tile_n=64, split_k=4, epilogue=(bias, 0.5, 2.0))
    want = orc.fused(to_np(bias)[None, :], to_np(a), to_np(b), 0.5, 2.0, "bfloat16")
    ok, err = orc.check(to_np(got), want, "bfloat16")
    assert ok, f"error {err:.3e}"
