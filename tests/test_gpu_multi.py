"""Multi-GPU: the sharded products on 2 GPUs (skipped with fewer), one process
per GPU, every gathered or reduced result checked against the fp64 oracle.

The fused gather (mb_gemm_peer: the tcgen05 epilogue stores each tile into
every rank's output over NVLink, through CUDA-IPC mappings) is covered on each
store path of the kernel: whole tiles staged for TMA stores (peer copies of
the staged boxes), split-K / stream-K finishes and direct stores at a column
offset that is not 16-byte aligned (peer copies from registers), for bf16,
fp16 and int8 (bit-exact); two calls in a row exercise both slots of the peer
buffer.  The fused cases run twice: with the NVSwitch multicast buffer
(multimem.st, where the GPUs support it) and with plain CUDA-IPC peer
mappings (METALBLAS_NVLS=0; the default at two ranks).  The NCCL gather (fused=False) and the K-sharded
all-reduce are checked too.  NCCL's own NVLS is off; the peer buffers are
released on every exit path before the process group is destroyed."""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, results):
    import datetime
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    out = {}
    from metalblas_b200 import peer
    try:
        from metalblas_b200 import shard
        from oracle import oracle as orc

        def host(t):
            return t.float().cpu().numpy() if t.dtype in (torch.bfloat16, torch.float16) else t.cpu().numpy()

        def check(got, a, b, name):
            ok, err = orc.check(host(got), orc.product(host(a), host(b), name), name)
            return bool(ok)

        g = torch.Generator().manual_seed(0)

        def rnd(*shape, dt=torch.bfloat16):
            if dt is torch.int8:
                return torch.randint(-128, 128, shape, dtype=dt, generator=g)
            return torch.randn(*shape, generator=g).to(dt)

        def mm_n(name, M, n_total, K, dt, fused=None, calls=1):
            ok = True
            keep = []
            for _ in range(calls):
                A, B = rnd(M, K, dt=dt), rnd(K, n_total, dt=dt)
                s, e = shard.shard_range(n_total, world, rank)
                C = shard.sharded_matmul_n(A.to(dev), B[:, s:e].contiguous().to(dev), n_total, gather=True,
                                           fused=fused)
                keep.append((C, A, B))
            torch.cuda.synchronize()
            for C, A, B in keep:   # every call's result, both peer-buffer slots
                ok = ok and C.shape == (M, n_total) and check(C, A, B, name)
            return ok

        def fused_cases(tag):
            # whole tiles, TMA-staged epilogue (CTA-pair 256-wide tiles), two calls in a row
            out[f"{tag}mm_n_bf16_tiles"] = mm_n("bfloat16", 2048, 4096, 2048, torch.bfloat16, calls=2)
            # split-K finishes; rank 1's block starts at column 500 (1000 bytes: direct stores)
            out[f"{tag}mm_n_bf16_ragged_split"] = mm_n("bfloat16", 512, 1000, 1024, torch.bfloat16)
            # stream-K tail on a skinny block
            out[f"{tag}mm_n_bf16_skinny_sk"] = mm_n("bfloat16", 128, 2048, 16384, torch.bfloat16)
            out[f"{tag}mm_n_fp16_tiles"] = mm_n("float16", 2048, 4096, 1024, torch.float16)
            out[f"{tag}mm_n_int8_exact"] = mm_n("int8", 1024, 1024, 2048, torch.int8)
            a = rnd(7, 384, 256)
            b = rnd(7, 256, 320)
            c = shard.sharded_bmm(a.to(dev), b.to(dev), gather=True)
            out[f"{tag}bmm_fused"] = check(c, a, b, "bfloat16")

        os.environ["METALBLAS_NVLS"] = "1"   # multicast buffer, forced at two ranks
        fused_cases("")
        multicast = any(buf.mc_base for buf in peer._ARENAS.values())
        # the same with plain CUDA-IPC peer mappings
        torch.cuda.synchronize()
        peer.release_arenas()
        os.environ["METALBLAS_NVLS"] = "0"
        fused_cases("ipc_")
        os.environ.pop("METALBLAS_NVLS")
        # the unfused NCCL gather
        out["mm_n_bf16_nccl"] = mm_n("bfloat16", 512, 1000, 1024, torch.bfloat16, fused=False)

        # batch-sharded bmm, ragged batch (7 over 2), NCCL
        a = rnd(7, 384, 256)
        b = rnd(7, 256, 320)
        c = shard.sharded_bmm(a.to(dev), b.to(dev), gather=True, fused=False)
        out["bmm_nccl"] = check(c, a, b, "bfloat16")
        a8, b8 = rnd(8, 384, 256), rnd(8, 256, 320)
        c8 = shard.sharded_bmm(a8.to(dev), b8.to(dev), gather=True, chunks=4, fused=False)
        out["bmm_nccl_pipelined"] = check(c8, a8, b8, "bfloat16")

        # K-sharded with the fp32 all-reduce
        A, B = rnd(512, 1024), rnd(1024, 1000)
        s, e = shard.shard_range(1024, world, rank)
        Ck = shard.sharded_matmul_k(A[:, s:e].contiguous().to(dev), B[s:e].contiguous().to(dev))
        out["mm_k"] = check(Ck, A, B, "bfloat16")
        torch.cuda.synchronize()
        results[rank] = out
        results[f"multicast{rank}"] = multicast
    finally:
        torch.cuda.synchronize()
        peer.release_arenas()
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_sharded_products_two_gpus():
    ctx = mp.get_context("spawn")
    results = ctx.Manager().dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, results)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = dict(results)
    print("multicast buffers:", res.pop("multicast0", None), res.pop("multicast1", None))
    assert set(res) == {0, 1}, res
    for r in (0, 1):
        bad = [k for k, v in res[r].items() if not v]
        assert not bad, f"rank {r}: {bad}"
