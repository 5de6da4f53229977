"""Sharding of the hot path over the GPUs of one node (one process per GPU).

The reference is single-device (no torch.distributed anywhere in it); these
helpers spread its products over N GPUs the way the north star asks:

* ``sharded_bmm``     — the batch is independent: rank r computes its contiguous
  slice of batches with no communication; ``gather=True`` all-gathers the slabs
  over NCCL (NVLink) into the full [B, M, N] output, optionally in pipelined
  rounds that overlap the exchange with the next round's products.
* ``sharded_matmul_n`` — large GEMMs split along N: rank r holds all of A and its
  column block of B and computes C[:, block r]; ``gather=True`` all-gathers the
  blocks and lays them out as one row-major C.
* ``sharded_matmul_k`` — skinny long-K GEMMs split along K: rank r multiplies its
  K-slice (fp32 accumulation, rounded to the input dtype), the partials are
  summed in fp32 with one all-reduce, then rounded to the output dtype.

Only the exchange steps (gather, reduce) use a collective; the products run
locally through the tcgen05 / GEMV kernels.  ``local_mm`` / ``local_bmm`` default
to this package's matmul / bmm and can be replaced (the CPU test suite runs the
same plumbing with torch's CPU products over gloo).
"""
from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.distributed as dist


def shard_range(n: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous [start, stop) of ``n`` items for ``rank`` of ``world``; the first
    ``n % world`` ranks take one extra item."""
    if world <= 0 or not (0 <= rank < world):
        raise ValueError(f"bad rank {rank} of world {world}")
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def _world(group):
    """(world size, rank); a single process without a process group is world 1."""
    if group is None and not (dist.is_available() and dist.is_initialized()):
        return 1, 0
    return dist.get_world_size(group), dist.get_rank(group)


def _default_mm(a, b):
    from . import matmul
    return matmul(a, b)


def _default_bmm(a, b):
    from . import bmm
    return bmm(a, b)


def _all_gather_rows(local: torch.Tensor, n_total: int, group, world: int) -> torch.Tensor:
    """All-gather slabs along dim 0 whose sizes follow shard_range (ragged ok)."""
    sizes = [shard_range(n_total, world, r) for r in range(world)]
    maxn = max(b - a for a, b in sizes)
    pad = torch.zeros((maxn,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    pad[: local.shape[0]].copy_(local)
    out = torch.empty((world * maxn,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(out, pad, group=group)
    parts = [out[r * maxn: r * maxn + (b - a)] for r, (a, b) in enumerate(sizes)]
    return torch.cat(parts, dim=0)


def sharded_bmm(a: torch.Tensor, b: torch.Tensor, *, group=None, gather: bool = False,
                local_bmm: Optional[Callable] = None, chunks: int = 1) -> torch.Tensor:
    """Batch-sharded bmm.  ``a``: [B, M, K] and ``b``: [B, K, N] (or [1, K, N],
    broadcast) on every rank; returns this rank's [B_r, M, N] slab (its
    shard_range of the batches), or the whole [B, M, N] when ``gather``.

    ``chunks > 1`` with ``gather`` pipelines the exchange: the batches are
    dealt out in ``chunks`` rounds (round c holds ranks' blocks side by side),
    each round's all-gather is issued asynchronously on NCCL's stream as soon
    as its products are done and runs while the next round computes, and each
    gathers straight into its contiguous slice of the output (no assembly
    copy).  This needs B divisible by world * chunks; otherwise one exchange
    after all products is used."""
    world, rank = _world(group)
    bsz = a.shape[0]
    bb = b.expand(bsz, *b.shape[1:]) if b.shape[0] == 1 and bsz > 1 else b
    mm = local_bmm or _default_bmm
    if gather and chunks > 1 and world > 1 and bsz % (world * chunks) == 0:
        cb = bsz // (world * chunks)                 # batches per rank and round
        out = torch.empty((bsz,) + tuple(a.shape[1:2]) + tuple(bb.shape[2:]), dtype=a.dtype, device=a.device)
        works = []
        for c in range(chunks):
            lo = (c * world + rank) * cb             # this rank's block of round c
            slab = mm(a[lo:lo + cb], bb[lo:lo + cb]).contiguous()
            dst = out[c * world * cb:(c + 1) * world * cb]
            works.append((dist.all_gather_into_tensor(dst, slab, group=group, async_op=True), slab))
        for w, _ in works:
            w.wait()
        return out
    s, e = shard_range(bsz, world, rank)
    local = mm(a[s:e], bb[s:e])
    if not gather:
        return local
    return _all_gather_rows(local.contiguous(), bsz, group, world)


def sharded_matmul_n(a: torch.Tensor, b_block: torch.Tensor, n_total: int, *, group=None,
                     gather: bool = False, local_mm: Optional[Callable] = None) -> torch.Tensor:
    """N-sharded GEMM.  ``a``: [M, K] replicated; ``b_block``: this rank's
    [K, N_r] column block of B (blocks follow shard_range(n_total)).  Returns
    C[:, block r] ([M, N_r]) or, with ``gather``, the row-major [M, n_total]."""
    world, rank = _world(group)
    s, e = shard_range(n_total, world, rank)
    if b_block.shape[1] != e - s:
        raise ValueError(f"rank {rank} expects a B block of {e - s} columns, got {b_block.shape[1]}")
    local = (local_mm or _default_mm)(a, b_block)
    if not gather:
        return local
    # gather column blocks as rows of C^T, then transpose back into row-major C
    cols = _all_gather_rows(local.t().contiguous(), n_total, group, world)
    return cols.t().contiguous()


def sharded_matmul_k(a_block: torch.Tensor, b_block: torch.Tensor, *, group=None,
                     local_mm: Optional[Callable] = None, out_dtype=None) -> torch.Tensor:
    """K-sharded (split-K) GEMM.  ``a_block``: [M, K_r], ``b_block``: [K_r, N]
    (this rank's K slice).  Each rank's product accumulates in fp32 and is
    rounded to the input dtype; the partials are summed in fp32 (16-bit inputs)
    or in the integer dtype (wrapping) by one all-reduce, and the sum is cast to
    ``out_dtype`` (default: a's)."""
    out_dtype = out_dtype or a_block.dtype
    part = (local_mm or _default_mm)(a_block, b_block)
    if a_block.dtype in (torch.float16, torch.bfloat16):
        part = part.float()
    dist.all_reduce(part, op=dist.ReduceOp.SUM, group=group)
    return part.to(out_dtype)
