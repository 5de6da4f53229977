"""CPU: the multi-GPU sharding plumbing (metalblas_b200/shard.py) at world size 2
over gloo, with torch's CPU products standing in for the CUDA kernels."""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from metalblas_b200 import shard


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(0)
        # bmm, ragged batch (5 over 2 ranks), broadcast B
        a = torch.randn(5, 6, 7, generator=g)
        b = torch.randn(1, 7, 4, generator=g)
        full = shard.sharded_bmm(a, b, gather=True, local_bmm=torch.bmm)
        ok_bmm = torch.allclose(full, torch.bmm(a, b.expand(5, 7, 4)), atol=1e-5)
        s, e = shard.shard_range(5, world, rank)
        part = shard.sharded_bmm(a, b, gather=False, local_bmm=torch.bmm)
        ok_part = part.shape[0] == e - s
        # N-sharded GEMM with gather (ragged N = 9)
        A = torch.randn(6, 8, generator=g)
        B = torch.randn(8, 9, generator=g)
        s, e = shard.shard_range(9, world, rank)
        C = shard.sharded_matmul_n(A, B[:, s:e].contiguous(), 9, gather=True, local_mm=torch.matmul)
        ok_n = torch.allclose(C, A @ B, atol=1e-5) and C.is_contiguous()
        # K-sharded with all-reduce
        s, e = shard.shard_range(8, world, rank)
        Ck = shard.sharded_matmul_k(A[:, s:e].contiguous(), B[s:e].contiguous(), local_mm=torch.matmul)
        ok_k = torch.allclose(Ck, A @ B, atol=1e-5)
        # pipelined exchange: bmm in rounds gathered straight into the output
        # (8 batches = 2 ranks x 4 rounds)
        a8 = torch.randn(8, 6, 7, generator=g)
        b8 = torch.randn(8, 7, 5, generator=g)
        ok_pipe = torch.allclose(shard.sharded_bmm(a8, b8, gather=True, local_bmm=torch.bmm, chunks=4),
                                 torch.bmm(a8, b8), atol=1e-5)
        results[rank] = (ok_bmm, ok_part, ok_n, ok_k and ok_pipe)
    finally:
        dist.destroy_process_group()


def test_shard_range_partitions():
    for n in (0, 1, 5, 8, 9, 64):
        for world in (1, 2, 3, 8):
            ranges = [shard.shard_range(n, world, r) for r in range(world)]
            assert ranges[0][0] == 0 and ranges[-1][1] == n
            assert all(ranges[i][1] == ranges[i + 1][0] for i in range(world - 1))
            sizes = [b - a for a, b in ranges]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard.shard_range(4, 2, 2)


def test_sharded_products_world2_gloo():
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, results)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert dict(results) == {0: (True, True, True, True), 1: (True, True, True, True)}


def _peer_worker(rank, world, port, results):
    """The IPC-handle exchange and the fused-path agreement of peer.py / shard.py
    over gloo (no CUDA needed: handles are opaque bytes here)."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from metalblas_b200 import peer
        handle = bytes((rank * 37 + i) % 256 for i in range(peer.HANDLE_BYTES))
        recs = peer.exchange(peer.pack_payload(handle, 4096 * (rank + 1) + 7), None, torch.device("cpu"))
        got = [peer.unpack_payload(r) for r in recs]
        want = [(bytes((r * 37 + i) % 256 for i in range(peer.HANDLE_BYTES)), 4096 * (r + 1) + 7)
                for r in range(world)]
        ok_exchange = got == want
        # every rank must take the same path: the agreement is the minimum
        ok_agree = shard._agree(("k", 1), rank == 0, None, torch.device("cpu")) is False
        ok_cached = shard._agree(("k", 1), True, None, torch.device("cpu")) is False   # decided once
        ok_agree2 = shard._agree(("k", 2), True, None, torch.device("cpu")) is True
        results[rank] = (ok_exchange, ok_agree and ok_cached and ok_agree2)
    finally:
        dist.destroy_process_group()


def test_peer_exchange_world2_gloo():
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_peer_worker, args=(r, 2, port, results)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert dict(results) == {0: (True, True), 1: (True, True)}


def _multicast_worker(rank, world, port, results):
    """peer.PeerBuffer._init_multicast over gloo with torch's symmetric-memory
    calls replaced by fakes: a failure on one rank alone (allocation, or no
    multicast address) must send every rank to the IPC fallback, and success
    must give each rank the same multicast base."""
    import types
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import torch.distributed._symmetric_memory as symm_mem
        from metalblas_b200 import peer
        mode = {}

        def fake_empty(n, dtype=None, device=None):
            if mode["fail_alloc_rank"] == rank:
                raise RuntimeError("no symmetric memory here")
            return torch.empty(n, dtype=dtype)

        def fake_rendezvous(t, group):
            ptrs = [0x10000000 * (r + 1) for r in range(world)]
            ptrs[rank] = t.data_ptr()
            mc = 0 if mode["no_mc_rank"] == rank else 0x7000000000
            return types.SimpleNamespace(buffer_ptrs=ptrs, multicast_ptr=mc)

        symm_mem.empty, symm_mem.rendezvous = fake_empty, fake_rendezvous

        def attempt(fail_alloc_rank, no_mc_rank):
            mode.update(fail_alloc_rank=fail_alloc_rank, no_mc_rank=no_mc_rank)
            buf = object.__new__(peer.PeerBuffer)
            buf.slot, buf.nslots, buf.device = 4096, 2, torch.device("cpu")
            buf.world, buf.rank = world, rank
            buf._symm, buf.local, buf.mc_base = None, None, 0
            buf._base_addr = [0] * world
            buf._init_multicast(None)
            return buf

        b1 = attempt(fail_alloc_rank=1, no_mc_rank=-1)
        ok_alloc = b1._symm is None and b1.mc_base == 0 and b1.mc_addr(1) == 0
        b2 = attempt(fail_alloc_rank=-1, no_mc_rank=0)
        ok_nomc = b2._symm is None and b2.mc_base == 0
        b3 = attempt(fail_alloc_rank=-1, no_mc_rank=-1)
        ok_mc = (b3._symm is not None and b3.mc_base == 0x7000000000 and
                 b3.mc_addr(1, 32) == 0x7000000000 + 4096 + 32 and
                 b3.addr(0, rank) == b3.local.data_ptr())
        results[rank] = (ok_alloc, ok_nomc, ok_mc)
    finally:
        dist.destroy_process_group()


def test_multicast_setup_falls_back_together_world2_gloo():
    ctx = mp.get_context("spawn")
    results = ctx.Manager().dict()
    port = _free_port()
    procs = [ctx.Process(target=_multicast_worker, args=(r, 2, port, results)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert dict(results) == {0: (True, True, True), 1: (True, True, True)}


def test_multicast_policy(monkeypatch):
    from metalblas_b200 import peer
    monkeypatch.delenv("METALBLAS_NVLS", raising=False)
    assert not peer._multicast_wanted(2) and not peer._multicast_wanted(3)
    assert peer._multicast_wanted(peer.MULTICAST_MIN_WORLD) and peer._multicast_wanted(8)
    monkeypatch.setenv("METALBLAS_NVLS", "1")
    assert peer._multicast_wanted(2)
    monkeypatch.setenv("METALBLAS_NVLS", "0")
    assert not peer._multicast_wanted(8)


def test_peer_payload_and_slots():
    from metalblas_b200 import peer
    h = bytes(range(64))
    t = peer.pack_payload(h, -12345)
    assert t.dtype == torch.uint8 and t.numel() == peer.HANDLE_BYTES + 8
    assert peer.unpack_payload(t) == (h, -12345)
    with pytest.raises(ValueError):
        peer.pack_payload(b"short", 0)
    assert peer.slot_bytes(1) == peer.SLOT_ALIGN
    assert peer.slot_bytes(peer.SLOT_ALIGN) == peer.SLOT_ALIGN
    assert peer.slot_bytes(peer.SLOT_ALIGN + 1) == 2 * peer.SLOT_ALIGN
    # without a process group the world is one rank and the barrier is a no-op
    assert peer.world_of(None) == (1, 0)
    peer.barrier(None)


def test_fused_gather_needs_cuda_and_the_default_product():
    a = torch.zeros(4, 4, dtype=torch.bfloat16)
    assert not shard._fusable((a, a), None, None, 2)              # CPU tensors
    assert not shard._fusable((a, a), torch.matmul, None, 2)      # custom local product
    assert not shard._fusable((a, a), None, None, 1)              # one rank: nothing to gather
    assert not shard._fusable((a, a), None, None, 9)              # more peers than the kernel's table
