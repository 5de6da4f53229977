"""Run the CUDA path on the golden fixtures and compare with the outputs the
reference's own oracle produced for them (tests/golden/make_golden.py).

Integers must match bit for bit (full-range 8/16-bit cases exercise wraparound);
floats and complex must meet the reference's tolerance rule
(tests/test_basic.py:53-69) against the golden value.
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle import oracle as orc
from tests import golden_io
from tests.helpers import to_np

pytestmark = pytest.mark.gpu

CASES = golden_io.cases()


@pytest.fixture(scope="module")
def mb():
    import metalblas_b200
    return metalblas_b200


def _run(mb, case):
    op = case["op"]
    a = golden_io.tensor(case, "a")
    b = golden_io.tensor(case, "b")
    if op == "matmul":
        if case.get("layout") == "ta":
            a = a.t().contiguous().t()
        elif case.get("layout") == "conj":
            a = a.conj()
        return mb.matmul(a, b)
    if op in ("bmm", "bmm_bcast_b"):
        if op == "bmm_bcast_b":
            b = b.expand(case["B"], *b.shape[1:])
        return mb.bmm(a, b)
    bias = golden_io.tensor(case, "bias")
    return getattr(mb, op)(bias, a, b, beta=case["beta"], alpha=case["alpha"])


@pytest.mark.parametrize("case", CASES, ids=[f"{c['id']}-{c['op']}-{c['dtype']}" for c in CASES])
def test_golden(mb, case):
    got = to_np(_run(mb, case))
    exp = golden_io.get(case, "expected")
    dtype = case["dtype"]
    assert got.shape == exp.shape
    if dtype in orc.INT_BITS:
        assert np.array_equal(got.astype(np.int64), exp.astype(np.int64)), f"{case['id']}: integer mismatch"
        return
    k = case["K"] * (case["B"] if case["op"] == "addbmm" else 1)
    scale = abs(case.get("alpha", 1)) + abs(case.get("beta", 0)) if "beta" in case else 1.0
    ok, err, lim = orc.ref_check(got, exp.astype(np.complex128 if np.iscomplexobj(exp) else np.float64),
                                 dtype, k, scale=scale)
    assert ok, f"{case['id']}: error {err:.3e} > {lim:.3e}"
