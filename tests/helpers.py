"""Shared test helpers: seeded inputs and torch <-> oracle conversion."""
from __future__ import annotations

import numpy as np
import torch

INTS = (torch.int8, torch.uint8, torch.int16, torch.int32, torch.int64)
FLOATS = (torch.float32, torch.float16, torch.bfloat16)
COMPLEX = (torch.complex64, torch.complex32)
ALL = FLOATS + COMPLEX + INTS
NAME = {torch.float32: "float32", torch.float16: "float16", torch.bfloat16: "bfloat16",
        torch.complex64: "complex64", torch.complex32: "complex32", torch.int8: "int8",
        torch.uint8: "uint8", torch.int16: "int16", torch.int32: "int32", torch.int64: "int64"}
BY_NAME = {v: k for k, v in NAME.items()}


def rand(shape, dtype, gen, device="cuda", full_range=False, lo=None, hi=None):
    """Seeded CPU draw, then moved to ``device``.

    Distributions follow the reference's _rand (tests/test_basic.py:20-24):
    integers in [-4, 4) ([0, 4) for uint8), N(0,1) for floats; complex parts
    N(0,1).  ``full_range`` draws integers over the whole type; lo/hi override.
    """
    if dtype in INTS:
        if full_range:
            info = torch.iinfo(dtype)
            # randint's exclusive bound must itself fit the type's C range
            lo, hi = info.min, (info.max if dtype is torch.int64 else info.max + 1)
        elif lo is None:
            lo, hi = (0 if dtype is torch.uint8 else -4), 4
        t = torch.randint(lo, hi, tuple(shape), dtype=dtype, generator=gen)
    elif dtype in COMPLEX:
        t = torch.complex(torch.randn(tuple(shape), generator=gen),
                          torch.randn(tuple(shape), generator=gen)).to(dtype)
    else:
        t = torch.randn(tuple(shape), generator=gen).to(dtype)
    return t.to(device)


def to_np(t: torch.Tensor) -> np.ndarray:
    """Values of a (possibly conj / strided / cuda) tensor as numpy, exactly."""
    t = t.detach()
    if t.is_conj():
        t = t.resolve_conj()
    if t.is_neg():
        t = t.resolve_neg()
    t = t.cpu()
    if t.dtype is torch.bfloat16:
        return t.float().numpy()
    if t.dtype is torch.complex32:
        return t.to(torch.complex64).numpy()
    return t.numpy()
