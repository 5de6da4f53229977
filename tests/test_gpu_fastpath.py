"""The host fast path of repeated calls (csrc/fastpath.cpp) against the Python
path: the same outputs, bit for bit, for matmul / bmm with and without out=,
fresh operand buffers on every call (only the cached descriptor is reused),
strided outputs, conjugated complex operands, and after the caches are reset."""
from __future__ import annotations

import pytest
import torch

import metalblas_b200 as mb
from metalblas_b200 import _lib, dispatch
from oracle import oracle as orc
from tests.helpers import NAME, rand, to_np

pytestmark = pytest.mark.gpu


def _fast_hits(fn):
    """Run fn twice; the second call must be served by the fast path."""
    fast = _lib.fast()
    assert fast is not None
    fn()
    return fn()


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.int8, torch.float32, torch.complex64],
                         ids=NAME.get)
@pytest.mark.parametrize("shape", [(1, 4096, 1024), (256, 512, 384), (1000, 1000, 600)])
def test_matmul_fast_path_matches(dtype, shape):
    M, N, K = shape
    gen = torch.Generator().manual_seed(21)
    for call in range(3):
        a = rand((M, K), dtype, gen, full_range=dtype is torch.int8)
        b = rand((K, N), dtype, gen, full_range=dtype is torch.int8)
        c1 = mb.matmul(a, b)
        out = torch.empty(M, N, dtype=dtype, device="cuda")
        c2 = mb.matmul(a, b, out=out)
        assert c2 is out
        assert torch.equal(c1, c2), f"call {call}"
        ok, err = orc.check(to_np(c1), orc.product(to_np(a), to_np(b), NAME[dtype]), NAME[dtype])
        assert ok, f"call {call}: err {err}"
    # a strided output view and a conjugated operand
    if dtype is torch.complex64:
        a = rand((M, K), dtype, gen).conj()
        b = rand((K, N), dtype, gen)
        big = torch.empty(M, N + 8, dtype=dtype, device="cuda")
        for _ in range(2):
            mb.matmul(a, b, out=big[:, 3:3 + N])
        ok, err = orc.check(to_np(big[:, 3:3 + N]), orc.product(to_np(a), to_np(b), "complex64"), "complex64")
        assert ok, err


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=NAME.get)
def test_bmm_fast_path_matches(dtype):
    gen = torch.Generator().manual_seed(22)
    for call in range(3):
        a = rand((8, 512, 256), dtype, gen)
        b = rand((8, 256, 512), dtype, gen)
        c1 = mb.bmm(a, b)
        c2 = mb.bmm(a, b, out=torch.empty_like(c1))
        assert torch.equal(c1, c2), f"call {call}"
        ok, err = orc.check(to_np(c1), orc.product(to_np(a), to_np(b), NAME[dtype]), NAME[dtype])
        assert ok, err
    # broadcast B (batch stride 0)
    a = rand((4, 64, 96), dtype, gen)
    b = rand((1, 96, 80), dtype, gen).expand(4, 96, 80)
    for _ in range(2):
        c = mb.bmm(a, b)
    ok, err = orc.check(to_np(c), orc.product(to_np(a), to_np(b), NAME[dtype]), NAME[dtype])
    assert ok, err


def test_fast_path_after_reset_and_overrides():
    gen = torch.Generator().manual_seed(23)
    a = rand((128, 256), torch.bfloat16, gen)
    b = rand((256, 192), torch.bfloat16, gen)
    ref = mb.matmul(a, b)
    dispatch.reset_caches()
    assert torch.equal(mb.matmul(a, b), ref)
    assert torch.equal(mb.matmul(a, b), ref)
    # overrides bypass the fast path and still give the product
    c = mb.matmul(a, b, backend="simd")
    ok, err = orc.check(to_np(c), orc.product(to_np(a), to_np(b), "bfloat16"), "bfloat16")
    assert ok, err
    # mismatched shapes still raise from the Python path
    with pytest.raises(AssertionError):
        mb.matmul(a, rand((255, 192), torch.bfloat16, gen))
