"""CPU: pin the oracle against the golden fixtures made from the reference's own
oracle (tests/golden/make_golden.py), and cross-check the C restatement of the
integer arithmetic (oracle/int_gemm_ref.c) against both."""
from __future__ import annotations

import numpy as np
import pytest

from oracle import build as oracle_build
from oracle import oracle as orc
from tests import golden_io

CASES = golden_io.cases()


def _oracle(case):
    op, dt = case["op"], case["dtype"]
    a, b = golden_io.get(case, "a"), golden_io.get(case, "b")
    if op == "matmul":
        if case.get("layout") == "conj":
            a = np.conj(a)
        return orc.product(a, b, dt)
    if op == "bmm":
        return orc.product(a, b, dt)
    if op == "bmm_bcast_b":
        return orc.product(a, np.broadcast_to(b, (case["B"],) + b.shape[1:]), dt)
    bias = golden_io.get(case, "bias")
    return orc.fused(bias, a, b, case["beta"], case["alpha"], dt, reduce=(op == "addbmm"))


@pytest.mark.parametrize("case", CASES, ids=[f"{c['id']}-{c['op']}-{c['dtype']}" for c in CASES])
def test_oracle_matches_reference_oracle(case):
    ref = _oracle(case)
    exp = golden_io.get(case, "expected")
    dt = case["dtype"]
    if dt in orc.INT_BITS:
        assert np.array_equal(orc.wrap(ref, dt).astype(np.int64), exp.astype(np.int64))
    else:
        # the reference's oracle runs in fp32 / complex64; ours in fp64 / complex128
        assert orc.rel_frobenius(exp, ref) < 2e-6


INT_CASES = [c for c in CASES if c["dtype"] in orc.INT_BITS and c["op"] in ("matmul", "addmm")]


@pytest.mark.parametrize("case", INT_CASES, ids=[f"{c['id']}-{c['op']}-{c['dtype']}" for c in INT_CASES])
def test_c_restatement_matches_reference_oracle(case):
    dt = case["dtype"]
    a, b = golden_io.get(case, "a"), golden_io.get(case, "b")
    if case["op"] == "matmul":
        got = oracle_build.int_gemm(a, b, dt)
    else:
        got = oracle_build.int_gemm(a, b, dt, bias=golden_io.get(case, "bias"), alpha=case["alpha"],
                                    beta=case["beta"], epilogue=True)
    assert np.array_equal(got.astype(np.int64), golden_io.get(case, "expected").astype(np.int64))


def test_wrap_matches_twos_complement():
    x = np.array([127, 128, 255, 256, -129, -1, 2 ** 40 + 5], dtype=np.int64)
    assert orc.wrap(x, "int8").tolist() == [127, -128, -1, 0, 127, -1, 5]
    assert orc.wrap(x, "uint8").tolist() == [127, 128, 255, 0, 127, 255, 5]


def test_bf16_rounding_is_nearest_even():
    x = np.array([1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8, -2.5, 0.0])
    assert orc.round_to(x, "bfloat16").tolist() == [1.0, 1.0 + 2 ** -6, -2.5, 0.0]


def test_frobenius_tolerances_follow_north_star():
    assert orc.FROB_TOL["bfloat16"] == 1e-2 and orc.FROB_TOL["float32"] == 1e-5
    assert orc.FROB_TOL["complex32"] == 1e-2 and orc.FROB_TOL["complex64"] == 1e-5
