"""Generate the golden fixtures in this directory from the REFERENCE's own oracle.

The reference (Isalia20/metalBLAS) ships no fixtures; its correctness oracle is
the set of CPU functions in its tests/test_basic.py: ``_product`` (:37-42),
``_wrap`` (:27-34) and ``_fused_ref`` (:110-121).  Its Metal kernels cannot run
off macOS, but those oracle functions run on any CPU.  This script imports that
file from a reference checkout (``--reference`` or the METALBLAS_REFERENCE
environment variable, required),
draws seeded CPU inputs with the reference's distributions (``_rand``,
tests/test_basic.py:20-24: integers in [-4,4) or [0,4) for uint8, N(0,1)
otherwise) plus full-range 8-bit integers (the BASELINE integer config, which
exercises wraparound), and stores inputs and the reference oracle's outputs.

Run it where the reference checkout exists (it is not needed at test time):

    python tests/golden/make_golden.py [--reference /path/to/metalBLAS]

Output: golden_cases.npz (arrays) + golden_index.json (case metadata).
bfloat16 values are stored exactly as float32; complex32 as complex64.
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
INTS = (torch.int8, torch.uint8, torch.int16, torch.int32, torch.int64)
FLOATS = (torch.float32, torch.float16, torch.bfloat16)
COMPLEX = (torch.complex64, torch.complex32)
ALL = FLOATS + COMPLEX + INTS
NAME = {torch.float32: "float32", torch.float16: "float16", torch.bfloat16: "bfloat16",
        torch.complex64: "complex64", torch.complex32: "complex32", torch.int8: "int8",
        torch.uint8: "uint8", torch.int16: "int16", torch.int32: "int32", torch.int64: "int64"}


def load_reference_oracle(ref_root):
    sys.path.insert(0, ref_root)
    path = os.path.join(ref_root, "tests", "test_basic.py")
    spec = importlib.util.spec_from_file_location("reference_test_basic", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


class Gen:
    def __init__(self, seed):
        self.g = torch.Generator().manual_seed(seed)

    def rand(self, shape, dtype, full_range=False):
        """CPU version of the reference's _rand (tests/test_basic.py:20-24)."""
        if dtype in INTS:
            if full_range:
                info = torch.iinfo(dtype)
                return torch.randint(info.min, info.max + 1, shape, dtype=dtype, generator=self.g)
            lo = 0 if dtype is torch.uint8 else -4
            return torch.randint(lo, 4, shape, dtype=dtype, generator=self.g)
        if dtype in COMPLEX:
            re = torch.randn(shape, generator=self.g)
            im = torch.randn(shape, generator=self.g)
            return torch.complex(re, im).to(dtype)
        return torch.randn(shape, generator=self.g).to(dtype)


def to_np(t):
    if t.dtype is torch.bfloat16:
        return t.float().numpy()
    if t.dtype is torch.complex32:
        return t.to(torch.complex64).numpy()
    return t.resolve_conj().numpy()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("METALBLAS_REFERENCE"),
                    help="path of a metalBLAS checkout (or set METALBLAS_REFERENCE)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("--reference (or METALBLAS_REFERENCE) is required")
    ref = load_reference_oracle(args.reference)
    gen = Gen(1234)
    arrays, index = {}, []

    def add(case, **tensors):
        cid = f"c{len(index):04d}"
        for k, v in tensors.items():
            arrays[f"{cid}_{k}"] = v
        case["id"] = cid
        index.append(case)

    def expected_plain(a, b, dtype):
        out = ref._product(a, b)
        return ref._wrap(out, dtype) if dtype in INTS else out

    # matmul: every dtype, edge shapes (ragged, GEMV, K=1)
    mm_shapes = [(33, 17, 45), (1, 40, 64), (40, 1, 64), (7, 9, 1), (20, 24, 129)]
    for dtype in ALL:
        for (M, N, K) in mm_shapes:
            for layout in ("rm", "ta", "conj") if dtype in COMPLEX else ("rm", "ta"):
                a = gen.rand((M, K), dtype)
                b = gen.rand((K, N), dtype)
                a_use = a.conj() if layout == "conj" else a
                exp = expected_plain(a_use, b, dtype)
                add({"op": "matmul", "dtype": NAME[dtype], "M": M, "N": N, "K": K, "layout": layout},
                    a=to_np(a), b=to_np(b), expected=to_np(exp))
    # full-range 8-bit (wraparound; BASELINE integer config distribution)
    for dtype in (torch.int8, torch.uint8, torch.int16):
        for (M, N, K) in [(64, 48, 80), (33, 40, 257)]:
            a = gen.rand((M, K), dtype, full_range=True)
            b = gen.rand((K, N), dtype, full_range=True)
            add({"op": "matmul", "dtype": NAME[dtype], "M": M, "N": N, "K": K, "layout": "rm",
                 "full_range": True}, a=to_np(a), b=to_np(b), expected=to_np(expected_plain(a, b, dtype)))

    # addmm: bias shapes and beta/alpha grid (tests/test_basic.py:202-213)
    M, N, K = 24, 20, 36
    grid = [(bs, 1, 1) for bs in [(M, N), (1, N), (M, 1), (N,), (1,), ()]]
    grid += [((N,), be, al) for be, al in [(2, 3), (0, 1), (1, 0), (0, 0), (0.5, 2.0)]]
    for dtype in ALL:
        for bshape, beta, alpha in grid:
            if dtype in INTS and isinstance(beta, float):
                continue
            a, b = gen.rand((M, K), dtype), gen.rand((K, N), dtype)
            bias = gen.rand(bshape, dtype)
            out = ref._fused_ref(bias, a, b, beta, alpha, False)
            exp = ref._wrap(out, dtype) if dtype in INTS else out
            add({"op": "addmm", "dtype": NAME[dtype], "M": M, "N": N, "K": K, "bshape": list(bshape),
                 "beta": beta, "alpha": alpha},
                a=to_np(a), b=to_np(b), bias=to_np(bias), expected=to_np(exp))

    # bmm / baddbmm / addbmm (tests/test_basic.py:219-242), incl. broadcast batch
    Bb, M, N, K = 3, 20, 24, 16
    for dtype in ALL:
        a, b = gen.rand((Bb, M, K), dtype), gen.rand((Bb, K, N), dtype)
        add({"op": "bmm", "dtype": NAME[dtype], "B": Bb, "M": M, "N": N, "K": K},
            a=to_np(a), b=to_np(b), expected=to_np(expected_plain(a, b, dtype)))
        b1 = gen.rand((1, K, N), dtype)
        exp = expected_plain(a, b1.expand(Bb, K, N), dtype)
        add({"op": "bmm_bcast_b", "dtype": NAME[dtype], "B": Bb, "M": M, "N": N, "K": K},
            a=to_np(a), b=to_np(b1), expected=to_np(exp))
        for bshape in [(Bb, M, N), (1, N), (M, 1), (N,), ()]:
            bias = gen.rand(bshape, dtype)
            out = ref._fused_ref(bias, a, b, 2, 3, False)
            exp = ref._wrap(out, dtype) if dtype in INTS else out
            add({"op": "baddbmm", "dtype": NAME[dtype], "B": Bb, "M": M, "N": N, "K": K,
                 "bshape": list(bshape), "beta": 2, "alpha": 3},
                a=to_np(a), b=to_np(b), bias=to_np(bias), expected=to_np(exp))
        bias = gen.rand((N,), dtype)
        out = ref._fused_ref(bias, a, b, 1, 1, True)
        exp = ref._wrap(out, dtype) if dtype in INTS else out
        add({"op": "addbmm", "dtype": NAME[dtype], "B": Bb, "M": M, "N": N, "K": K, "bshape": [N],
             "beta": 1, "alpha": 1}, a=to_np(a), b=to_np(b), bias=to_np(bias), expected=to_np(exp))

    np.savez_compressed(os.path.join(HERE, "golden_cases.npz"), **arrays)
    with open(os.path.join(HERE, "golden_index.json"), "w") as f:
        json.dump({"generator": "tests/golden/make_golden.py",
                   "oracle": "reference tests/test_basic.py _product/_wrap/_fused_ref",
                   "torch": torch.__version__, "cases": index}, f, indent=1)
    print(f"{len(index)} cases")


if __name__ == "__main__":
    main()
