"""Sharding of the hot path over the GPUs of one node (one process per GPU).

The reference is single-device (no torch.distributed anywhere in it); these
helpers spread its products over N GPUs the way the north star asks:

* ``sharded_bmm``     — the batch is independent: rank r computes its contiguous
  slice of batches with no communication; ``gather=True`` returns the full
  [B, M, N] on every rank.
* ``sharded_matmul_n`` — large GEMMs split along N: rank r holds all of A and its
  column block of B and computes C[:, block r]; ``gather=True`` returns the
  row-major [M, N] on every rank.
* ``sharded_matmul_k`` — skinny long-K GEMMs split along K: rank r multiplies its
  K-slice (fp32 accumulation, rounded to the input dtype), the partials are
  summed in fp32 with one all-reduce, then rounded to the output dtype.

The gather is fused into the product: on CUDA tensors of the tensor-core
dtypes (bf16, fp16, int8, uint8) the kernel's epilogue stores each finished
tile into every rank's output at once (``mb_gemm_peer``; plain peer stores over
NVLink into buffers mapped by CUDA IPC, ``peer.py``), so the transfer overlaps
the math tile by tile, and one stream-ordered barrier ends the step.  The
result is a view of a two-slot peer buffer (``peer.arena``), valid until the
second sharded call after it on the same group and device; copy it to keep
it.  Other cases (other dtypes, a custom ``local_mm``, ``fused=False``) gather
with NCCL all-gathers after the products.  ``local_mm`` / ``local_bmm`` default
to this package's matmul / bmm and can be replaced (the CPU test suite runs the
same plumbing with torch's CPU products over gloo).
"""
from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.distributed as dist

from . import peer as _peer

FUSED_DTYPES = (torch.bfloat16, torch.float16, torch.int8, torch.uint8)


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
    return _peer.world_of(group)


def _default_mm(a, b):
    from . import matmul
    return matmul(a, b)


def _default_bmm(a, b):
    from . import bmm
    return bmm(a, b)


# Fusability agreed by all ranks once per call signature: every rank must take
# the same path (the fused step ends in a barrier, the NCCL one in all-gathers).
_AGREED: dict = {}


def _agree(key, local_ok: bool, group, device) -> bool:
    hit = _AGREED.get(key)
    if hit is not None:
        return hit
    dev = _peer._comm_device(group, device)
    t = torch.tensor([1 if local_ok else 0], dtype=torch.int32, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MIN, group=group)
    ok = bool(int(t.item()))
    _AGREED[key] = ok
    return ok


def _fusable(tensors, local_fn, fused, world) -> bool:
    if fused is False or local_fn is not None or world < 2 or world - 1 > 7:
        return False
    return all(t.is_cuda and t.dtype in FUSED_DTYPES for t in tensors)


def _plans_tc(a, b, batched: bool) -> bool:
    """Whether this rank's product plans on the tensor-core kernel (the only
    plan mb_gemm_peer runs)."""
    from . import kernels
    try:
        return kernels.plan(a, b).startswith("tc ")
    except (ValueError, NotImplementedError, RuntimeError, AssertionError):
        return False


def _all_gather_rows(local: torch.Tensor, n_total: int, group, world: int) -> torch.Tensor:
    """All-gather slabs along dim 0 whose sizes follow shard_range (ragged ok)."""
    sizes = [shard_range(n_total, world, r) for r in range(world)]
    maxn = max(b - a for a, b in sizes)
    if all(b - a == maxn for a, b in sizes):
        out = torch.empty((n_total,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
        dist.all_gather_into_tensor(out, local.contiguous(), group=group)
        return out
    pad = torch.zeros((maxn,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    pad[: local.shape[0]].copy_(local)
    out = torch.empty((world * maxn,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(out, pad, group=group)
    parts = [out[r * maxn: r * maxn + (b - a)] for r, (a, b) in enumerate(sizes)]
    return torch.cat(parts, dim=0)


def sharded_bmm(a: torch.Tensor, b: torch.Tensor, *, group=None, gather: bool = False,
                local_bmm: Optional[Callable] = None, chunks: int = 1, fused: Optional[bool] = None) -> torch.Tensor:
    """Batch-sharded bmm.  ``a``: [B, M, K] and ``b``: [B, K, N] (or [1, K, N],
    broadcast) on every rank; returns this rank's [B_r, M, N] slab (its
    shard_range of the batches), or the whole [B, M, N] when ``gather``.

    With ``gather`` on CUDA tensor-core dtypes the product writes its slab into
    every rank's copy of the output (see the module docstring).  Otherwise
    ``chunks > 1`` pipelines NCCL all-gathers: the batches are dealt out in
    ``chunks`` rounds, each round's all-gather issued asynchronously as soon as
    its products are done (this needs B divisible by world * chunks; else one
    exchange after all products)."""
    world, rank = _world(group)
    bsz = a.shape[0]
    bb = b.expand(bsz, *b.shape[1:]) if b.shape[0] == 1 and bsz > 1 else b
    s, e = shard_range(bsz, world, rank)
    if gather and _fusable((a, b), local_bmm, fused, world):
        M, N = a.shape[1], bb.shape[2]
        key = ("bmm", tuple(a.shape), tuple(a.stride()), tuple(bb.shape), tuple(bb.stride()), a.dtype,
               a.data_ptr() & 15, bb.data_ptr() & 15, id(group), a.device.index)
        if _agree(key, e == s or _plans_tc(a[s:e], bb[s:e], True), group, a.device):
            from .dispatch import _bmm
            esz = a.element_size()
            buf = _peer.arena(bsz * M * N * esz, a.device, group)
            slot = buf.next_slot()
            out = buf.view(slot, a.dtype, (bsz, M, N))
            if e > s:
                off = s * M * N * esz
                _bmm(a[s:e], bb[s:e], out[s:e], peers=(buf.peer_addrs(slot, off), buf.mc_addr(slot, off)))
            _peer.barrier(group, a.device)
            return out
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
    local = mm(a[s:e], bb[s:e])
    if not gather or world == 1:
        return local
    return _all_gather_rows(local.contiguous(), bsz, group, world)


def sharded_matmul_n(a: torch.Tensor, b_block: torch.Tensor, n_total: int, *, group=None,
                     gather: bool = False, local_mm: Optional[Callable] = None,
                     fused: Optional[bool] = None) -> torch.Tensor:
    """N-sharded GEMM.  ``a``: [M, K] replicated; ``b_block``: this rank's
    [K, N_r] column block of B (blocks follow shard_range(n_total)).  Returns
    C[:, block r] ([M, N_r]) or, with ``gather``, the row-major [M, n_total] on
    every rank.

    With ``gather`` on CUDA tensor-core dtypes the block is computed straight
    into columns [s, e) of a row-major [M, n_total] peer buffer and every other
    rank's copy of it (the fused gather); otherwise the blocks are all-gathered
    over NCCL as rows of Cᵀ and laid out once."""
    world, rank = _world(group)
    s, e = shard_range(n_total, world, rank)
    if b_block.shape[1] != e - s:
        raise ValueError(f"rank {rank} expects a B block of {e - s} columns, got {b_block.shape[1]}")
    M = a.shape[0]
    if gather and _fusable((a, b_block), local_mm, fused, world):
        key = ("mm_n", tuple(a.shape), tuple(a.stride()), tuple(b_block.shape), tuple(b_block.stride()), n_total,
               a.dtype, a.data_ptr() & 15, b_block.data_ptr() & 15, id(group), a.device.index)
        if _agree(key, e == s or _plans_tc(a, b_block, False), group, a.device):
            from .dispatch import _mm2d
            esz = a.element_size()
            buf = _peer.arena(M * n_total * esz, a.device, group)
            slot = buf.next_slot()
            out = buf.view(slot, a.dtype, (M, n_total))
            if e > s:
                _mm2d(a, b_block, out[:, s:e], peers=(buf.peer_addrs(slot, s * esz), buf.mc_addr(slot, s * esz)))
            _peer.barrier(group, a.device)
            return out
    local = (local_mm or _default_mm)(a, b_block)
    if not gather or world == 1:
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
    ``out_dtype`` (default: a's).  The reference's single-device split-K
    (metalblas/float_dispatch.py:183-219, metalblas/shaders/splitk.h:21-82)
    sums fp32 partials the same way, over K chunks of one GPU."""
    out_dtype = out_dtype or a_block.dtype
    part = (local_mm or _default_mm)(a_block, b_block)
    if a_block.dtype in (torch.float16, torch.bfloat16):
        part = part.float()
    dist.all_reduce(part, op=dist.ReduceOp.SUM, group=group)
    return part.to(out_dtype)
