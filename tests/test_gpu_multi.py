"""Multi-GPU: the sharded products over NCCL on 2 GPUs (skipped with fewer),
one process per GPU, results checked against the fp64 oracle."""
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
    try:
        import numpy as np
        from metalblas_b200 import shard
        from oracle import oracle as orc
        g = torch.Generator().manual_seed(0)
        a = torch.randn(7, 384, 256, generator=g).to(torch.bfloat16)
        b = torch.randn(7, 256, 320, generator=g).to(torch.bfloat16)
        c = shard.sharded_bmm(a.to(dev), b.to(dev), gather=True)
        ok1, _ = orc.check(c.float().cpu().numpy(), orc.product(a.float().numpy(), b.float().numpy(), "bfloat16"),
                           "bfloat16")
        A = torch.randn(512, 1024, generator=g).to(torch.bfloat16)
        B = torch.randn(1024, 1000, generator=g).to(torch.bfloat16)
        s, e = shard.shard_range(1000, world, rank)
        C = shard.sharded_matmul_n(A.to(dev), B[:, s:e].contiguous().to(dev), 1000, gather=True)
        ref = orc.product(A.float().numpy(), B.float().numpy(), "bfloat16")
        ok2, _ = orc.check(C.float().cpu().numpy(), ref, "bfloat16")
        s, e = shard.shard_range(1024, world, rank)
        Ck = shard.sharded_matmul_k(A[:, s:e].contiguous().to(dev), B[s:e].contiguous().to(dev))
        ok3, _ = orc.check(Ck.float().cpu().numpy(), ref, "bfloat16")
        # pipelined exchange: bmm in 4 rounds (8 batches over 2 ranks)
        a8 = torch.randn(8, 384, 256, generator=g).to(torch.bfloat16)
        b8 = torch.randn(8, 256, 320, generator=g).to(torch.bfloat16)
        c8 = shard.sharded_bmm(a8.to(dev), b8.to(dev), gather=True, chunks=4)
        ok4, _ = orc.check(c8.float().cpu().numpy(), orc.product(a8.float().numpy(), b8.float().numpy(), "bfloat16"),
                           "bfloat16")
        results[rank] = (bool(ok1), bool(ok2), bool(ok3 and ok4))
    finally:
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
    assert dict(results) == {0: (True, True, True), 1: (True, True, True)}
