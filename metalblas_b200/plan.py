"""Per-shape autotune cache over the sm_100a tile table.

The tile table itself is the C planner (``mb_plan_query`` prints its choice):
GEMV kernels for M==1/N==1, the tcgen05 kernel with an N-tile and split-K picked
by a wave-quantisation cost model, Cᵀ=BᵀAᵀ for thin M, CUDA cores otherwise.
This module keeps the reference's autotuning contract on top of it
(metalblas/float_dispatch.py:152-158, 411-505):

* ``METALBLAS_AUTOTUNE`` ("0" disables; default on);
* the table's primary choice is kept unless a rival is faster by 3 % (1 % for
  tall/narrow shapes) — ``_fastest``, metalblas/float_dispatch.py:421-436;
* a rival is accepted only if it agrees with the primary within
  0.02 * max|ref| (bit-exact for integers) — metalblas/float_dispatch.py:464-468;
* results are cached per shape in the library's table (mb_autotune_record /
  mb_autotune_lookup, so C callers of mb_gemm get the tuned plans too), keyed
  by GPU name, dtype, M, N, K, batch, broadcast flags, layout and alignment
  class and epilogue flag; with ``METALBLAS_AUTOTUNE_CACHE=<file>`` the table
  persists across processes (mb_autotune_cache_load / _save).  A missing or
  unreadable file means re-tune.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

from . import _lib

AUTOTUNE = os.environ.get("METALBLAS_AUTOTUNE", "1") != "0"
MARGIN = 0.03
TALL_NARROW_MARGIN = 0.01
MIN_FLOPS = 4e9          # below this the table's choice stands (launch-bound)
_TC_CODES = (_lib.MB_BF16, _lib.MB_F16, _lib.MB_I8, _lib.MB_U8)

_lock = threading.Lock()
_loaded = False


def _cache_path():
    return os.environ.get("METALBLAS_AUTOTUNE_CACHE")


def _load_cache():
    """Merge the cache file into the library's table once per process; a
    missing or unreadable file means re-tune."""
    global _loaded
    if _loaded:
        return
    _loaded = True
    path = _cache_path()
    if path and os.path.exists(path):
        _lib.load().mb_autotune_cache_load(path.encode())


def _save_cache():
    path = _cache_path()
    if path:
        _lib.load().mb_autotune_cache_save(path.encode())


def _candidates(primary: str, d):
    """Rivals worth timing against the table's choice (backend, tile_n, split_k, swap)."""
    if not primary.startswith("tc"):
        return []
    f = dict(kv.split("=") for kv in primary.split()[1:] if "=" in kv)
    if "bn" not in f:
        return []
    bn, split, swap = int(f["bn"]), int(f.get("split", 1)), int(f.get("swap", 0))
    tc = _lib.MB_BACKEND_TC
    out = []
    for obn in (64, 128, 256):
        if obn != bn:
            out.append((tc, obn, 0, 1 if swap else -1))
    if split > 1:
        out.append((tc, bn, 1, 1 if swap else -1))
        out.append((tc, bn, max(2, split // 2), 1 if swap else -1))
        out.append((tc, bn, split * 2, 1 if swap else -1))
    elif d.K >= 8 * max(d.M, d.N):
        out.append((tc, bn, 2, 1 if swap else -1))
        out.append((tc, bn, 4, 1 if swap else -1))
    out.append((tc, 0, 0, -1 if swap else 1))
    return list(dict.fromkeys(out))


def _probe_params(flops):
    """Fewer probe iterations for longer kernels (metalblas/float_dispatch.py:411-418)."""
    if flops <= 2e9:
        return 3, 10, 3
    if flops <= 5e10:
        return 2, 5, 3
    return 1, 3, 3


def _run(d, stream):
    lib = _lib.load()
    nbytes = int(lib.mb_gemm_workspace_size(ctypes.byref(d)))
    keep = None
    if nbytes > 0:
        from .dispatch import _workspace
        dev = torch.device("cuda", torch.cuda.current_device())
        keep = _workspace(dev, stream, nbytes)
        d.workspace, d.workspace_bytes = keep.data_ptr(), keep.numel()
    else:
        d.workspace, d.workspace_bytes = None, 0
    return lib.mb_gemm(ctypes.byref(d), ctypes.c_void_p(stream))


def _tune(d, C, stream):
    primary = _lib.plan_query(d)
    cands = _candidates(primary, d)
    if not cands:
        return None
    tall_narrow = min(d.M, d.N) <= 256 and max(d.M, d.N) >= 1024
    margin = TALL_NARROW_MARGIN if tall_narrow else MARGIN
    # scratch output with C's element size; packed row-major [batch, M, N]
    scratch = torch.empty((max(d.batch, 1), d.M, d.N), dtype=C.dtype, device=C.device)
    ref = torch.empty_like(scratch)

    def desc_for(choice, out):
        q = _lib.GemmDesc()
        ctypes.pointer(q)[0] = d
        q.C = out.data_ptr()
        q.c_rs, q.c_cs, q.sC = d.N, 1, d.M * d.N if d.batch > 1 else 0
        if choice is not None:
            q.backend, q.tile_n, q.split_k, q.swap_ab = choice
        return q

    if _run(desc_for(None, ref), stream) != _lib.MB_OK:
        return None
    torch.cuda.synchronize()
    is_int = C.dtype in (torch.int8, torch.uint8)
    scale = 0.0 if is_int else float(ref.float().abs().max()) + 1e-6
    runs = [desc_for(None, scratch)]
    labels = [None]
    for c in cands:
        q = desc_for(c, scratch)
        try:
            if _lib.plan_query(q) == primary:
                continue
        except (ValueError, NotImplementedError, RuntimeError):
            continue
        if _run(q, stream) != _lib.MB_OK:
            continue
        torch.cuda.synchronize()
        if is_int:
            ok = torch.equal(scratch, ref)
        else:
            ok = float((scratch.float() - ref.float()).abs().max()) <= 0.02 * scale
        if ok:
            runs.append(q)
            labels.append(c)
    if len(runs) == 1:
        return None
    flops = 2.0 * d.M * d.N * d.K * max(d.batch, 1)
    warmup, iters, reps = _probe_params(flops)
    s = torch.cuda.current_stream()
    times = [float("inf")] * len(runs)
    for q in runs:
        for _ in range(warmup):
            _run(q, stream)
    for _ in range(reps):
        for i, q in enumerate(runs):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(s)
            for _ in range(iters):
                _run(q, stream)
            e1.record(s)
            e1.synchronize()
            times[i] = min(times[i], e0.elapsed_time(e1) / iters)
    best = min(range(len(times)), key=times.__getitem__)
    if best and times[best] < times[0] * (1.0 - margin):
        return labels[best]
    return None


def wants(d) -> bool:
    """Whether the autotuner would time rivals for this descriptor's shape."""
    if not AUTOTUNE or d.dtype not in _TC_CODES or d.M <= 1 or d.N <= 1 or d.K == 0:
        return False
    return 2.0 * d.M * d.N * d.K * max(d.batch, 1) >= MIN_FLOPS


def choose(d, A, B, C, stream):
    """Return (backend, tile_n, split_k, swap_ab) to override the table, or None."""
    if not wants(d):
        return None
    if torch.cuda.is_current_stream_capturing():
        return None
    with _lock:
        _load_cache()
        hit = _lib.autotune_lookup(d)
    if hit is not None:
        return None if hit == "keep" else hit
    choice = _tune(d, C, stream)
    with _lock:
        _lib.autotune_record(d, choice)
        _save_cache()
    return choice


def clear():
    """Forget every tuned shape (the library's table, and this thread's cached
    descriptors that carry a tuned plan)."""
    with _lock:
        _lib.load().mb_autotune_cache_clear()
    from . import dispatch
    dispatch._fast_cache().clear()
