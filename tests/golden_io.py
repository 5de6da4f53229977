"""Load the golden fixtures (tests/golden/, made by tests/golden/make_golden.py
from the reference's own oracle functions)."""
from __future__ import annotations

import json
import os

import numpy as np
import torch

from tests.helpers import BY_NAME

HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def cases():
    with open(os.path.join(HERE, "golden_index.json")) as f:
        return json.load(f)["cases"]


_arrays = None


def arrays():
    global _arrays
    if _arrays is None:
        _arrays = dict(np.load(os.path.join(HERE, "golden_cases.npz")))
    return _arrays


def get(case, name):
    return arrays()[f"{case['id']}_{name}"]


def tensor(case, name, device="cuda"):
    """The fixture array as a tensor of the case's dtype (exact values)."""
    dtype = BY_NAME[case["dtype"]]
    x = torch.from_numpy(np.ascontiguousarray(get(case, name)))
    return x.to(dtype).to(device)
