"""CPU: host-side logic of the public API that runs before any device work —
layout classification, scalar casting, tile/backend validation and the error
types the reference raises (metalblas/dispatch.py, float_dispatch.py)."""
from __future__ import annotations

import pytest
import torch

import metalblas_b200 as mb
from metalblas_b200 import dispatch


def test_public_names_match_reference():
    assert mb.__all__ == ["matmul", "gemm", "addmm", "bmm", "baddbmm", "addbmm",
                          "dot", "vdot", "outer", "ger", "mv", "kernels"]
    assert mb.gemm is mb.matmul and mb.ger is mb.outer


@pytest.mark.parametrize("shape,transpose,expect", [
    ((8, 16), False, (False, 16)),
    ((8, 16), True, (True, 16)),
])
def test_unit_lead(shape, transpose, expect):
    t = torch.empty(shape)
    if transpose:
        t = t.t()
        rows, cols = shape[1], shape[0]
    else:
        rows, cols = shape
    assert dispatch._unit_lead(t, rows, cols) == expect


def test_unit_lead_rejects_fully_strided_and_copies():
    t = torch.empty(8, 32)[:, ::2]          # stride (32, 2): neither stride is 1
    assert dispatch._unit_lead(t, 8, 16) is None
    v = dispatch._matrix_view(t, 8, 16)
    assert v.is_contiguous()


def test_offset_view_is_kept():
    t = torch.empty(9, 17)[1:, 1:]          # lda = 17 (reference "offset" layout)
    assert dispatch._unit_lead(t, 8, 16) == (False, 17)
    assert dispatch._matrix_view(t, 8, 16) is t


def test_scalars_cast_like_reference():
    assert dispatch._scalars(torch.int8, 2.7, 1.2) == (2, 1, True, True)
    assert dispatch._scalars(torch.float16, 0, 1) == (0.0, 1.0, False, True)
    beta, alpha, bnz, anz = dispatch._scalars(torch.complex64, 1j, 0)
    assert beta == 1j and alpha == 0 and bnz and not anz


def test_int64_scalar_wraps():
    assert dispatch._int64(2 ** 64 + 3) == 3
    assert dispatch._int64(-1) == -1
    assert dispatch._int64(2 ** 63) == -(2 ** 63)


def test_parse_tile():
    assert dispatch._parse_tile("mpp_tensor", (128, 256)) == (256, 0)
    # the reference's (BM, BN, NSG) tuples map to the nearest sm_100a N-tile
    assert dispatch._parse_tile("mpp_tensor", (128, 64, 4)) == (64, 0)
    assert dispatch._parse_tile("mpp_tensor", (64, 64, 2)) == (64, 0)
    assert dispatch._parse_tile("mpp_tensor", (48, 128, 4)) == (128, 0)
    assert dispatch._parse_tile("mpp_tensor", (32, 32, 4)) == (32, 0)
    assert dispatch._parse_tile("mpp_tensor", (16, 96, 2)) == (128, 0)
    assert dispatch._parse_tile("mpp_tensor", (128, 512, 8)) == (256, 0)
    # a fourth entry is the split-K override
    assert dispatch._parse_tile("mpp_tensor", (128, 64, 4, 3)) == (64, 3)
    assert dispatch._parse_tile(None, None) == (0, 0)
    with pytest.raises(ValueError):
        dispatch._parse_tile("mpp_tensor", (64, 64))       # (BM, BN) form needs BM = 128
    with pytest.raises(ValueError):
        dispatch._parse_tile("mpp_tensor", (64, 0, 2))
    with pytest.raises(AssertionError):
        dispatch._parse_tile("simd", (64, 64))


def test_cpu_tensors_are_rejected():
    a, b = torch.randn(4, 4), torch.randn(4, 4)
    with pytest.raises(AssertionError):
        mb.matmul(a, b)
    with pytest.raises(AssertionError):
        mb.addmm(torch.randn(4), a, b)
    with pytest.raises(AssertionError):
        mb.bmm(a[None], b[None])


def test_vector_argument_checks():
    with pytest.raises(AssertionError):
        mb.dot(torch.randn(3), torch.randn(4))
    with pytest.raises(AssertionError):
        mb.outer(torch.randn(3, 1), torch.randn(4))
    with pytest.raises(AssertionError):
        mb.mv(torch.randn(3, 4), torch.randn(5))


def test_outer_is_broadcast_multiply_on_host_types():
    a, b = torch.arange(3.0), torch.arange(4.0)
    assert torch.equal(mb.outer(a, b), torch.outer(a, b))


def test_metalblas_alias_module():
    """``import metalblas`` binds the reference's package name to this build."""
    import metalblas
    import metalblas_b200
    for name in metalblas_b200.__all__:
        assert getattr(metalblas, name) is getattr(metalblas_b200, name)
    assert metalblas.kernels.plan is metalblas_b200.kernels.plan
