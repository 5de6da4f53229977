"""CPU baseline of the hot path — TEST/BENCH INFRASTRUCTURE ONLY.

The reference has no CPU implementation of matmul (its kernels are Metal); its
correctness oracle and the north star's stated CPU baseline are host-CPU
``torch.matmul`` on the same inputs (tests/test_basic.py:37-42), timed on the
host's own cores.  ``bench.py`` times this function for its ``cpu_baseline`` object and
for ``--impl reference``; nothing in the product imports it.
"""
from __future__ import annotations

import time

import torch


def cpu_matmul(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """Host torch.matmul in the operands' dtype (all host threads)."""
    return torch.matmul(a, b)


def time_rows(a: torch.Tensor, b: torch.Tensor, rows: int, reps: int) -> tuple[float, int]:
    """Time ``reps`` products of the first ``rows`` rows of ``a`` with ``b``.

    Returns (seconds per product, rows used).
    """
    rows = max(1, min(rows, a.shape[0]))
    sub = a[:rows].contiguous()
    cpu_matmul(sub, b)  # warm-up (thread pool, packing buffers)
    t0 = time.perf_counter()
    for _ in range(reps):
        cpu_matmul(sub, b)
    return (time.perf_counter() - t0) / reps, rows


def calibrate_rows(a: torch.Tensor, b: torch.Tensor, seconds_per_product: float) -> int:
    """Rows of ``a`` whose product with ``b`` takes about ``seconds_per_product``."""
    probe = max(16, min(256, a.shape[0]))
    t, probe = time_rows(a, b, probe, 1)
    rows = int(probe * seconds_per_product / max(t, 1e-6))
    return max(16, min(a.shape[0], rows))
