"""Split-K of thin tiles reduced inside a thread-block cluster.

When every K split of a tile runs on the CTAs of one cluster, ranks 1.. hand
their partial sums to rank 0 through distributed shared memory instead of the
workspace, and rank 0 adds them in K order.  These products must give the
oracle's answer and, since the order of the additions is the same, the same
bits as the workspace reduction (METALBLAS_CLUSTER_SPLIT=0, in a child
process: the switch is read once when the library loads).  Cases cover bf16,
fp16 and int8 (wrapping int32 sums), 2, 3 and 4 splits, ragged M and N, an
alpha/beta/bias epilogue and repeated calls.
"""
from __future__ import annotations

import multiprocessing as mp

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

# (dtype name, M, N, K, split_k, epilogue?)
CASES = [("bfloat16", 4, 4096, 4096, 4, False), ("bfloat16", 16, 1000, 3000, 3, True),
         ("float16", 5, 2048, 8192, 2, False), ("float16", 16, 4096, 2048, 4, True),
         ("int8", 16, 1536, 4096, 4, True), ("int8", 3, 777, 2048, 3, False)]
DT = {"bfloat16": torch.bfloat16, "float16": torch.float16, "int8": torch.int8}


def _inputs(i, name, M, N, K):
    g = torch.Generator().manual_seed(100 + i)
    dt = DT[name]
    if dt is torch.int8:
        a = torch.randint(-128, 128, (M, K), generator=g, dtype=dt)
        b = torch.randint(-128, 128, (K, N), generator=g, dtype=dt)
        bias = torch.randint(-128, 128, (N,), generator=g, dtype=dt)
    else:
        a = torch.randn(M, K, generator=g).to(dt)
        b = torch.randn(K, N, generator=g).mul(0.05).to(dt)
        bias = torch.randn(N, generator=g).to(dt)
    return a, b, bias


def _compute():
    """Every case through the forced swapped split plan, twice; CPU results."""
    from metalblas_b200 import _lib, dispatch
    out = []
    for i, (name, M, N, K, split, epi) in enumerate(CASES):
        a, b, bias = (t.cuda() for t in _inputs(i, name, M, N, K))
        alpha, beta = (3, -2) if name == "int8" else (2.0, 0.5)
        e = (bias, (0, 1, 0), beta, alpha, True, True) if epi else None
        res = []
        for _ in range(2):
            c = torch.empty(M, N, dtype=a.dtype, device="cuda")
            dispatch._launch(a, b, c, M, N, K, 1, (K, 1, 0), (N, 1, 0), (N, 1, 0), epilogue=e,
                             backend=_lib.MB_BACKEND_TC, split_k=split, swap_ab=1, autotune=False)
            res.append(c)
        torch.cuda.synchronize()
        out.append([r.cpu() for r in res])
    return out


def _bits(c):
    """The result's bit patterns as a plain numpy array (picklable)."""
    return (c.view(torch.int16) if c.element_size() == 2 else c).numpy()


def _child(q):
    import os
    os.environ["METALBLAS_CLUSTER_SPLIT"] = "0"
    try:
        q.put(("ok", [_bits(r[0]) for r in _compute()]))
    except Exception as ex:  # noqa: BLE001 - reported to the parent
        q.put(("error", repr(ex)))


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")
def test_cluster_split_matches_oracle_and_workspace_reduction():
    from oracle import oracle as orc
    got = _compute()
    for i, (name, M, N, K, split, epi) in enumerate(CASES):
        a, b, bias = _inputs(i, name, M, N, K)
        if name == "int8":
            an, bn, biasn = a.numpy(), b.numpy(), bias.numpy()
        else:
            an, bn, biasn = a.float().numpy(), b.float().numpy(), bias.float().numpy()
        if epi:
            alpha, beta = (3, -2) if name == "int8" else (2.0, 0.5)
            ref = orc.fused(biasn, an, bn, beta, alpha, name)
        else:
            ref = orc.product(an, bn, name)
        for c in got[i]:
            cn = c.numpy() if name == "int8" else c.float().numpy()
            ok, err = orc.check(cn, ref, name)
            assert ok, f"case {i} {name} {M}x{N}x{K} split={split}: err={err}"
        assert torch.equal(got[i][0], got[i][1]), f"case {i}: repeated call differs"
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_child, args=(q,))
    p.start()
    status, ws = q.get(timeout=300)
    p.join(timeout=60)
    assert status == "ok", ws
    for i in range(len(CASES)):
        x = got[i][0]
        xb, yb = _bits(x), ws[i]
        if not np.array_equal(xb, yb):
            # only the sign of a zero may differ (the workspace sum starts from +0)
            y = torch.from_numpy(yb.copy())
            y = y.view(x.dtype) if x.element_size() == 2 else y
            assert torch.equal(x, y), f"case {i}: cluster and workspace reductions differ"
        assert np.isfinite(x.float().numpy()).all()
