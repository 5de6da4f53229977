"""Benchmark of the matmul hot path on B200 (driver contract: one JSON line).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload NAME]

Headline workload (BASELINE.json metric "bf16 GEMM TFLOP/s at 4096^3"): one
step = one bf16 GEMM C[4096,4096] = A[4096,4096] @ B[4096,4096], both row-major,
N(0,1) inputs from seed 0, through metalblas_b200.matmul (tcgen05 kernel).
With N ranks (torchrun, one process per GPU, NCCL) the GEMM is N-sharded with
fixed per-rank work (weak scaling): rank r computes C[:, r] = A @ B[:, r] of a
global [4096, 4096*N] product; the value keeps the output sharded, and a second
timing that all-gathers the shards over NVLink is reported as "gathered".

value      device time (CUDA events on the launching stream, barrier + sync on
           both sides, max over ranks), inputs resident in HBM, rotating over 4
           input sets (256 MB > 2 x L2) so operands come from HBM each step.
e2e        the same metric through the public API with the step's inputs copied
           from pinned host memory and the result copied back, every step.
roofline   tcgen05 kernel: 2*M*N*K FLOP per launch / average launch time, against
           the measured dense bf16 peak (MEASURED_PEAKS.json).
cpu_baseline  host torch.matmul (the reference's CPU oracle path) on a bounded
           row sample of the same product, rank 0 at N=1.
--impl reference  the reference's CPU path alone (host torch.matmul, all threads).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

PUBLISHED_M5_MAX_4096 = 42.95   # the reference's published bf16 4096^3 rate, Apple M5 Max (perf_benchs/M5_Max.md:17)


def _peaks():
    """(bf16 burst TFLOP/s, HBM GB/s, source) from MEASURED_PEAKS.json, else the
    pool's fallback figures."""
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p["bf16_tflops"]), float(p.get("hbm_gbs", 6650.0)), "measured"
    except (OSError, ValueError, KeyError):
        return 1590.0, 6650.0, "fallback"


def _sustained_peak():
    """bf16 TFLOP/s of a seconds-long GEMM loop under the power cap (the
    denominator for kernels timed inside long runs), or None."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["bf16_tflops_sustained"])
    except (OSError, ValueError, KeyError):
        return None


def _profile_traffic(name):
    """dram bytes per launch recorded from an ncu capture in profiles/<name>."""
    path = os.path.join(ROOT, "profiles", name)
    try:
        for line in open(path):
            if line.startswith("traffic_bytes_per_launch:"):
                return float(line.split(":", 1)[1].split()[0])
    except OSError:
        pass
    return None


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled while the timed region runs."""

    Q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index):
        self.dev = device_index
        self.samples = []
        self.proc = None
        self.active = False
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits", "-lms", "50",
                 "-i", str(self.dev)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 7:
                self.samples.append((time.time(), self.active, parts))

    def mark(self, active):
        self.active = active

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        if self.thread is not None:
            self.thread.join(timeout=5)

    def summary(self):
        rows = [p for (_, act, p) in self.samples if act] or [p for (_, _, p) in self.samples]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}

        def num(x):
            try:
                return float(x)
            except ValueError:
                return None
        sm = [num(r[0]) for r in rows if num(r[0]) is not None]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[3 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": num(rows[0][1]), "reasons": reasons, "samples": len(rows),
                "power_w_max": max((num(r[2]) or 0.0) for r in rows)}


def _host_cores() -> int:
    """CPU cores this process may run on (its affinity mask), else os.cpu_count()."""
    try:
        return max(1, len(os.sched_getaffinity(0)))
    except (AttributeError, OSError):
        return os.cpu_count() or 1


def _dist():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    return rank, world, local


def _max_over_ranks(x, world, device):
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _barrier(world, device):
    if world > 1:
        import torch.distributed as dist
        dist.barrier(device_ids=[device.index])
    torch.cuda.synchronize(device)


# --------------------------------------------------------------------------- workloads
WORKLOADS = {
    "bf16_gemm_4096": dict(M=4096, N=4096, K=4096, dtype=torch.bfloat16,
                           desc="bf16 GEMM 4096x4096x4096, A row-major @ B row-major"),
    "bf16_gemm_2048x2048x4096": dict(M=2048, N=2048, K=4096, dtype=torch.bfloat16,
                                     desc="bf16 GEMM config 1: A[2048,4096] @ B[4096,2048]"),
    "bf16_gemm_8192": dict(M=8192, N=8192, K=8192, dtype=torch.bfloat16, desc="bf16 GEMM 8192^3"),
    "fp16_gemm_4096": dict(M=4096, N=4096, K=4096, dtype=torch.float16, desc="fp16 GEMM 4096^3"),
    "int8_gemm_4096": dict(M=4096, N=4096, K=4096, dtype=torch.int8, desc="int8 GEMM 4096^3 full range"),
}


def _global_inputs(w, world):
    """Host A [M, K] and the global B [K, N * world] of the weak-scaling run
    (seed 0; A drawn first)."""
    g = torch.Generator().manual_seed(0)
    M, N, K, dt = w["M"], w["N"], w["K"], w["dtype"]
    if dt in (torch.int8, torch.uint8):
        info = torch.iinfo(dt)
        a = torch.randint(info.min, info.max + 1, (M, K), dtype=dt, generator=g)
        b = torch.randint(info.min, info.max + 1, (K, N * world), dtype=dt, generator=g)
    else:
        a = torch.randn(M, K, generator=g).to(dt)
        b = torch.randn(K, N * world, generator=g).to(dt)
    return a, b


def _inputs(w, rank, world):
    """Host A and this rank's column block of the global B."""
    a, b = _global_inputs(w, world)
    N = w["N"]
    return a, (b[:, rank * N:(rank + 1) * N].contiguous() if world > 1 else b)


def run_ours(args, w, rank, world, device):
    import metalblas_b200 as mb
    M, N, K, dt = w["M"], w["N"], w["K"], w["dtype"]
    flops = 2.0 * M * N * K
    a_h, b_h = _inputs(w, rank, world)
    a_pin, b_pin = a_h.pin_memory(), b_h.pin_memory()
    SETS = 4
    As = [a_pin.to(device) for _ in range(SETS)]
    Bs = [b_pin.to(device) for _ in range(SETS)]
    Cs = [torch.empty(M, N, dtype=dt, device=device) for _ in range(SETS)]
    stream = torch.cuda.current_stream(device)

    plan = mb.kernels.plan(As[0], Bs[0])
    # warm-up (also runs the autotuner once for this shape)
    for i in range(max(args.warmup, 3)):
        mb.matmul(As[i % SETS], Bs[i % SETS], out=Cs[i % SETS])
    torch.cuda.synchronize(device)

    sampler = ClockSampler(device.index)
    if rank == 0:
        sampler.start()
        time.sleep(0.3)
    _barrier(world, device)
    sampler.mark(True)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(args.steps):
        mb.matmul(As[i % SETS], Bs[i % SETS], out=Cs[i % SETS])
    e1.record(stream)
    e1.synchronize()
    sampler.mark(False)
    _barrier(world, device)
    ms = e0.elapsed_time(e1) / args.steps
    ms = _max_over_ranks(ms, world, device)
    if rank == 0:
        time.sleep(0.2)
        sampler.stop()
    value = flops * world / (ms * 1e-3) / 1e12

    # correctness guard on the timed output (row sample vs fp64 oracle)
    ok_rows = None
    if rank == 0:
        from oracle import oracle as orc
        idx = torch.arange(0, M, max(1, M // 64))
        ref = orc.product(a_h[idx].float().numpy(), b_h.float().numpy(),
                          "int8" if dt is torch.int8 else "bfloat16")
        got = Cs[(args.steps - 1) % SETS][idx.to(device)].cpu()
        name = {torch.bfloat16: "bfloat16", torch.float16: "float16", torch.int8: "int8"}[dt]
        ok_rows, err = orc.check(got.float().numpy() if dt is not torch.int8 else got.numpy(), ref, name)
        ok_rows = {"ok": bool(ok_rows), "rel_frobenius_or_mismatch": err, "rows_checked": int(len(idx))}

    bmm_line = run_bmm_sharded(args, rank, world, device) if not args.no_bmm else None
    large = run_large_nshard(args, rank, world, device) if not args.no_multi else None
    skinny = run_skinny(args, rank, world, device) if not args.no_multi else None

    # gathered variants (N > 1): the whole row-major C [M, N * ranks] on every
    # rank after every step.  "gathered": the product writes its column block
    # into every rank's copy of C from its epilogue (fused peer stores over
    # NVLink) and one barrier ends the step; "gathered_nccl": the product, then
    # a NCCL all-gather of the blocks (the unfused baseline).
    gathered = gathered_nccl = None
    if world > 1:
        from metalblas_b200 import shard
        n_total = N * world
        gms = _timed(lambda i: shard.sharded_matmul_n(As[i % SETS], Bs[i % SETS], n_total, gather=True),
                     args.steps, world, device)
        Cg = shard.sharded_matmul_n(As[0], Bs[0], n_total, gather=True)
        chk = _check_gathered(Cg, a_h, lambda cols: _weak_b_cols(w, cols, world), dt, world, device, rank,
                              row_step=max(1, M // 32), col_step=max(1, n_total // 2048))
        gathered = {"value": flops * world / (gms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": gms,
                    "layout": f"row-major C [{M}, {n_total}] on every rank",
                    "collective": "fused: tcgen05 epilogue stores each tile into every rank's C over NVLink "
                                  "(mb_gemm_peer), then one barrier", "peer_stores": _peer_mode(),
                    "roofline": _fused_roofline(flops, M * n_total * As[0].element_size(), world, gms), "check": chk}
        nms = _timed(lambda i: shard.sharded_matmul_n(As[i % SETS], Bs[i % SETS], n_total, gather=True,
                                                      fused=False), args.steps, world, device)
        gathered_nccl = {"value": flops * world / (nms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": nms,
                         "collective": "product, then NCCL all_gather_into_tensor of the blocks (unfused)"}

    # e2e: host buffers -> public API -> host result, every step.  Three streams
    # (copy-in, compute, copy-out) and two device buffer sets, so step i's
    # host-to-device copy overlaps step i-1's product and step i-2's read-back;
    # every step still copies its own inputs and reads its own result.  With N
    # ranks A (the same on every rank) is loaded once per step for the job:
    # each rank copies its 1/N of A's rows from host memory and the slices are
    # all-gathered over NVLink; each rank copies its own block of B.
    e2e_steps = max(1, min(args.steps, 100))
    elt = a_h.element_size()
    s_in, s_out = torch.cuda.Stream(device), torch.cuda.Stream(device)
    split_a = world > 1 and M % world == 0
    ma = M // world if split_a else M
    a_src = a_pin[rank * ma:(rank + 1) * ma] if split_a else a_pin
    a_part = [torch.empty(ma, K, dtype=dt, device=device) for _ in range(2)] if split_a else None
    a_d = [torch.empty(M, K, dtype=dt, device=device) for _ in range(2)]
    b_d = [torch.empty(K, N, dtype=dt, device=device) for _ in range(2)]
    c_d = [torch.empty(M, N, dtype=dt, device=device) for _ in range(2)]
    c_pin = [torch.empty(M, N, dtype=dt).pin_memory() for _ in range(2)]
    in_done = [torch.cuda.Event() for _ in range(2)]
    mm_done = [torch.cuda.Event() for _ in range(2)]
    out_done = [torch.cuda.Event() for _ in range(2)]

    def e2e_step(i):
        j = i % 2
        with torch.cuda.stream(s_in):
            s_in.wait_event(mm_done[j])          # buffer set j free (product i-2 consumed it)
            (a_part[j] if split_a else a_d[j]).copy_(a_src, non_blocking=True)
            b_d[j].copy_(b_pin, non_blocking=True)
            in_done[j].record(s_in)
        stream.wait_event(in_done[j])
        stream.wait_event(out_done[j])           # c_d[j] read back (step i-2)
        if split_a:
            import torch.distributed as dist
            dist.all_gather_into_tensor(a_d[j], a_part[j])
        mb.matmul(a_d[j], b_d[j], out=c_d[j])
        mm_done[j].record(stream)
        with torch.cuda.stream(s_out):
            s_out.wait_event(mm_done[j])
            c_pin[j].copy_(c_d[j], non_blocking=True)
            out_done[j].record(s_out)

    for i in range(4):
        e2e_step(i)
    torch.cuda.synchronize(device)
    _barrier(world, device)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(s_in)
    for i in range(e2e_steps):
        e2e_step(i)
    t1.record(s_out)
    t1.synchronize()
    _barrier(world, device)
    ems = _max_over_ranks(t0.elapsed_time(t1) / e2e_steps, world, device)
    e2e = {"value": flops * world / (ems * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": ems,
           "h2d_bytes_per_step": (ma * K + K * N) * elt, "d2h_bytes_per_step": M * N * elt, "steps": e2e_steps,
           "pipelining": "copy-in / compute / copy-out streams, 2 device buffer sets" +
                         ("; A's rows loaded 1/N per rank and all-gathered over NVLink" if split_a else "")}

    peak, hbm, src = _peaks()
    achieved = flops / (ms * 1e-3) / 1e12
    traffic = _profile_traffic((f"tc_gemm_{w['dtype_name']}_wide512_{M}x{N}x{K}.txt" if "bn=512" in plan
                                else f"tc_gemm_{w['dtype_name']}_{M}x{N}x{K}.txt"))
    roofline = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                "frac": achieved / peak, "peak_source": f"{src} bf16_tflops (burst)",
                "traffic": traffic, "kernel": "mb::tc::tc_gemm_kernel", "per_launch_flop": flops}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle import cpu_baseline as cb
        torch.set_num_threads(_host_cores())
        rows = cb.calibrate_rows(a_h, b_h, 2.0)
        reps = 5
        sec, rows = cb.time_rows(a_h, b_h, rows, reps)
        cpu = {"value": 2.0 * rows * N * K / sec / 1e12, "unit": "TFLOP/s", "cores": torch.get_num_threads(),
               "kind": "port", "sample": f"host torch.matmul {dt} A[:{rows}] @ B[{K},{N}], {reps} reps"}

    return {
        "metric": "bf16 GEMM TFLOP/s at 4096^3" if dt is torch.bfloat16 else f"{w['dtype_name']} GEMM TFLOP/s",
        "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": (value / PUBLISHED_M5_MAX_4096) if w["name"] == "bf16_gemm_4096" else None,
        "dtype": w["dtype_name"], "data": "synthetic N(0,1) seed 0 (full-range uniform for int8)",
        "config": {"workload": w["desc"], "M": M, "N": N, "K": K, "global_N": N * world,
                   "sharding": "N-sharded over ranks, output sharded in value" if world > 1 else "single GPU",
                   "l2": "inputs rotate over 4 sets (256 MB > 2 x 126 MB L2)", "plan": plan,
                   "vs_baseline_ref": "Apple M5 Max 42.95 TFLOP/s (perf_benchs/M5_Max.md:17)"},
        "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "gathered": gathered,
        "gathered_nccl": gathered_nccl,
        "gpu_launches": args.steps, "check": ok_rows, "clocks": sampler.summary() if rank == 0 else None,
        "bmm": bmm_line, "large": large, "skinny": skinny,
    }


def run_bmm_sharded(args, rank, world, device):
    """BASELINE's "bmm TFLOP/s at 1-8 GPUs": bf16 bmm [256,1024,1024] @
    [256,1024,1024] (N(0,1), seed 2) with the batch sharded over the ranks
    (strong scaling: the 256 batches are split, metalblas_b200.shard.shard_range).
    `value` keeps each rank's output slab local; `gathered` returns the full
    [256, 1024, 1024] on every rank every step (pipelined NCCL all-gathers).
    Device time, max over ranks, 2 input sets (1.5 GB > L2)."""
    import metalblas_b200 as mb
    from metalblas_b200 import shard
    Bt, M, N, K = 256, 1024, 1024, 1024
    s, e = shard.shard_range(Bt, world, rank)
    nb = e - s
    g = torch.Generator(device=device).manual_seed(2)  # the same full operands on every rank
    As = [torch.randn(Bt, M, K, generator=g, device=device, dtype=torch.bfloat16) for _ in range(2)]
    Bs = [torch.randn(Bt, K, N, generator=g, device=device, dtype=torch.bfloat16) for _ in range(2)]
    steps = max(5, min(args.steps, 50))
    ms = _timed(lambda i: shard.sharded_bmm(As[i % 2], Bs[i % 2], gather=False), steps, world, device)
    flops = 2.0 * Bt * M * N * K
    out = {"workload": "bf16 bmm [256,1024,1024]@[256,1024,1024], batch sharded over ranks (strong scaling)",
           "value": flops / (ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": ms, "steps": steps,
           "batches_per_rank": nb, "plan": mb.kernels.plan(As[0][s:e], Bs[0][s:e]),
           "api": "metalblas_b200.shard.sharded_bmm"}
    if world > 1:
        gms = _timed(lambda i: shard.sharded_bmm(As[i % 2], Bs[i % 2], gather=True), steps, world, device)
        Cg = shard.sharded_bmm(As[0], Bs[0], gather=True)
        # one batch from every rank's slab, checked against the oracle on rank 0;
        # every rank's copy of the sample must hold the same bytes
        pick = [shard.shard_range(Bt, world, r)[0] for r in range(world)]
        chk = _check_batches(Cg, As[0], Bs[0], pick, world, device, rank)
        out["gathered"] = {"value": flops / (gms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": gms,
                           "collective": "fused: each rank's bmm epilogue stores its slab into every rank's "
                                         "[256,1024,1024] output over NVLink (mb_gemm_peer), then one barrier",
                           "peer_stores": _peer_mode(),
                           "roofline": _fused_roofline(flops / world, Bt * M * N * 2, world, gms), "check": chk}
        nms = _timed(lambda i: shard.sharded_bmm(As[i % 2], Bs[i % 2], gather=True, chunks=4, fused=False),
                     steps, world, device)
        out["gathered_nccl"] = {"value": flops / (nms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": nms,
                                "collective": "NCCL all_gather_into_tensor in 4 rounds, each overlapping the "
                                              "next round's products (unfused)"}
    return out


def run_large_nshard(args, rank, world, device):
    """BASELINE config 5, large GEMM: bf16 16384 x 16384 x 16384 (N(0,1), seed 6)
    with N sharded over the ranks (strong scaling: rank r computes the
    16384 x 16384/N column block).  "value" keeps the output sharded;
    "gathered" returns the row-major 16384 x 16384 C on every rank each step,
    the gather fused into the product's epilogue.  At N = 1 both are the plain
    GEMM.  Inputs 1 GiB > L2."""
    import metalblas_b200 as mb
    from metalblas_b200 import shard
    Mx = Nx = Kx = 16384
    g = torch.Generator(device=device).manual_seed(6)
    A = torch.randn(Mx, Kx, generator=g, device=device, dtype=torch.bfloat16)
    B = torch.randn(Kx, Nx, generator=g, device=device, dtype=torch.bfloat16)
    s, e = shard.shard_range(Nx, world, rank)
    Bb = B[:, s:e]                       # this rank's column block, read in place (ldb = 16384)
    C = torch.empty(Mx, e - s, dtype=torch.bfloat16, device=device)
    steps = max(3, min(args.steps, 20))
    flops = 2.0 * Mx * Nx * Kx
    ms = _timed(lambda i: mb.matmul(A, Bb, out=C), steps, world, device)
    out = {"workload": "bf16 GEMM 16384^3, N sharded over ranks (strong scaling)",
           "value": flops / (ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": ms, "steps": steps,
           "columns_per_rank": e - s, "plan": mb.kernels.plan(A, Bb), "l2": "inputs 1 GiB > L2"}
    if world == 1:
        Cg, gms = C, ms
    else:
        gms = _timed(lambda i: shard.sharded_matmul_n(A, Bb, Nx, gather=True), steps, world, device)
        Cg = shard.sharded_matmul_n(A, Bb, Nx, gather=True)
    chk = _check_gathered(Cg, A, lambda cols: B[:, cols], torch.bfloat16, world, device, rank,
                          row_step=1024, col_step=8)
    out["gathered"] = {"value": flops / (gms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": gms,
                       "layout": "row-major C [16384, 16384] on every rank",
                       "collective": ("fused: tcgen05 epilogue stores each tile into every rank's C over "
                                      "NVLink (mb_gemm_peer), then one barrier") if world > 1 else "none (1 GPU)",
                       "peer_stores": _peer_mode(),
                       "roofline": _fused_roofline(flops / world, Mx * Nx * 2, world, gms), "check": chk}
    del A, B, C
    return out


def run_skinny(args, rank, world, device):
    """BASELINE config 5, skinny: bf16 128 x 8192 x 65536 (N(0,1), seed 6),
    HBM-bound (reads B, 1 GiB, once).  Two shardings over the ranks:
    "n_sharded" — N split, the 128 x 8192 output gathered to every rank by the
    fused epilogue (the north star's "N sharded ... output gathered");
    "k_sharded" — K split, each rank's 128 x 8192 partial summed in fp32 by one
    NCCL all-reduce (the reference's split-K, float_dispatch.py:183-219, across
    GPUs).  At N = 1 both are the plain GEMM."""
    import metalblas_b200 as mb
    from metalblas_b200 import shard
    Mx, Nx, Kx = 128, 8192, 65536
    g = torch.Generator(device=device).manual_seed(6)
    A = torch.randn(Mx, Kx, generator=g, device=device, dtype=torch.bfloat16)
    B = torch.randn(Kx, Nx, generator=g, device=device, dtype=torch.bfloat16)
    steps = max(5, min(args.steps, 50))
    flops = 2.0 * Mx * Nx * Kx
    byts = 2.0 * (Mx * Kx + Kx * Nx + Mx * Nx)
    out = {"workload": "bf16 skinny GEMM 128x8192x65536", "unit": "GB/s", "steps": steps,
           "bytes_per_step": byts, "l2": "B 1 GiB > L2"}
    s, e = shard.shard_range(Nx, world, rank)
    if world == 1:
        C = torch.empty(Mx, Nx, dtype=torch.bfloat16, device=device)
        ms = _timed(lambda i: mb.matmul(A, B, out=C), steps, world, device)
        Cn = Ck = C
        kms = ms
        out["plan"] = mb.kernels.plan(A, B)
    else:
        Bb = B[:, s:e]
        ms = _timed(lambda i: shard.sharded_matmul_n(A, Bb, Nx, gather=True), steps, world, device)
        Cn = shard.sharded_matmul_n(A, Bb, Nx, gather=True).clone()
        ks, ke = shard.shard_range(Kx, world, rank)
        Ak, Bk = A[:, ks:ke], B[ks:ke]
        kms = _timed(lambda i: shard.sharded_matmul_k(Ak, Bk), steps, world, device)
        Ck = shard.sharded_matmul_k(Ak, Bk)
        out["plan"] = mb.kernels.plan(A, Bb)
        out["plan_k"] = mb.kernels.plan(Ak, Bk)
    cn = _check_gathered(Cn, A, lambda cols: B[:, cols], torch.bfloat16, world, device, rank, row_step=8,
                         col_step=16)
    ck = _check_gathered(Ck, A, lambda cols: B[:, cols], torch.bfloat16, world, device, rank, row_step=8,
                         col_step=16)
    out["n_sharded"] = {"value": byts / (ms * 1e-3) / 1e9, "ms_per_step": ms,
                        "tflops": flops / (ms * 1e-3) / 1e12,
                        "collective": "fused gather (mb_gemm_peer) + barrier" if world > 1 else "none (1 GPU)",
                        "peer_stores": _peer_mode(), "check": cn}
    out["k_sharded"] = {"value": byts / (kms * 1e-3) / 1e9, "ms_per_step": kms,
                        "tflops": flops / (kms * 1e-3) / 1e12,
                        "collective": "NCCL all_reduce of fp32 partials" if world > 1 else "none (1 GPU)",
                        "check": ck}
    del A, B
    return out


# Measured NVLink peer-copy rate per direction per GPU on this pool (GB/s).
NVLINK_GBS = 770.0


def _fused_roofline(flops_per_rank, out_bytes, world, ms):
    """Roofline of a product fused with its output gather: the target time is
    the slower of the rank's math at the dense bf16 peak and the bytes each GPU
    must receive over NVLink, (N-1)/N of the gathered output, at the measured
    peer-copy rate; frac = target / measured step time."""
    peak, _, src = _peaks()
    t_math = flops_per_rank / (peak * 1e12)
    t_link = (world - 1) / world * out_bytes / (NVLINK_GBS * 1e9)
    target = max(t_math, t_link)
    return {"bound": "tensor" if t_math >= t_link else "nvlink", "target_ms": target * 1e3,
            "math_ms": t_math * 1e3, "link_ms": t_link * 1e3, "peak_tflops": peak, "peak_source": src,
            "nvlink_gbs": NVLINK_GBS, "frac": target / (ms * 1e-3)}


def _peer_mode():
    """How the fused gather's peer stores travelled: through the NVSwitch
    multicast buffer or plain CUDA-IPC peer mappings ("none" at one rank)."""
    from metalblas_b200 import peer
    bufs = list(peer._ARENAS.values())
    if not bufs:
        return "none"
    if any(b.mc_base for b in bufs):
        return "multicast: one multimem.st per 16 bytes, replicated by NVSwitch"
    return "CUDA-IPC: one st.global per peer per 16 bytes"


def _timed(fn, steps, world, device, warm=3):
    """Device time per call of fn(i): warm-up calls, then `steps` calls between
    CUDA events on the current stream, barrier + synchronize on both sides, max
    over ranks."""
    stream = torch.cuda.current_stream(device)
    for i in range(warm):
        fn(i)
    _barrier(world, device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(steps):
        fn(i)
    e1.record(stream)
    e1.synchronize()
    _barrier(world, device)
    return _max_over_ranks(e0.elapsed_time(e1) / steps, world, device)


def _rank_consistency(sample, world, device):
    """Every rank's copy of a gathered sample holds the same values: a weighted
    float64 checksum, all-gathered and compared."""
    if world == 1:
        return True
    import torch.distributed as dist
    x = sample.double()
    wts = torch.arange(1, x.numel() + 1, dtype=torch.float64, device=x.device).reshape(x.shape)
    cs = torch.stack([x.sum(), (x * wts).sum()]).reshape(1, 2)
    allc = torch.empty(world, 2, dtype=torch.float64, device=device)
    dist.all_gather_into_tensor(allc, cs)
    return bool(torch.equal(allc, allc[:1].expand(world, 2)))


def _check_gathered(C, A, b_cols, dt, world, device, rank, row_step, col_step):
    """Oracle check (rank 0) of a row x column sample of a gathered product
    C = A @ B, the sample spanning every rank's block; plus the cross-rank
    consistency of the same sample.  b_cols(cols) returns B[:, cols]."""
    from oracle import oracle as orc
    rows = torch.arange(0, C.shape[0], row_step, device=C.device)
    cols = torch.arange(0, C.shape[1], col_step, device=C.device)
    sample = C[rows][:, cols]
    same = _rank_consistency(sample, world, device)
    res = {"rows_checked": int(len(rows)), "cols_checked": int(len(cols)), "ranks_identical": same}
    if rank == 0:
        name = {torch.bfloat16: "bfloat16", torch.float16: "float16", torch.int8: "int8"}[dt]
        a_s = A[rows.to(A.device)].cpu() if A.is_cuda else A[rows.cpu()]
        b_s = b_cols(cols.to(A.device) if A.is_cuda else cols.cpu())
        b_s = b_s.cpu()
        as_np = a_s.float().numpy() if dt is not torch.int8 else a_s.numpy()
        bs_np = b_s.float().numpy() if dt is not torch.int8 else b_s.numpy()
        got = sample.cpu()
        ok, err = orc.check(got.float().numpy() if dt is not torch.int8 else got.numpy(),
                            orc.product(as_np, bs_np, name), name)
        res.update({"ok": bool(ok) and same, "rel_frobenius_or_mismatch": float(err)})
    return res


def _check_batches(C, A, B, pick, world, device, rank):
    """Oracle check (rank 0) of whole batches `pick` of a gathered bmm, plus
    cross-rank consistency of those batches."""
    from oracle import oracle as orc
    idx = torch.tensor(pick, device=C.device)
    sample = C[idx]
    same = _rank_consistency(sample, world, device)
    res = {"batches_checked": list(map(int, pick)), "ranks_identical": same}
    if rank == 0:
        ref = orc.product(A[idx].float().cpu().numpy(), B[idx].float().cpu().numpy(), "bfloat16")
        ok, err = orc.check(sample.float().cpu().numpy(), ref, "bfloat16")
        res.update({"ok": bool(ok) and same, "rel_frobenius_or_mismatch": float(err)})
    return res


def _weak_b_cols(w, cols, world):
    """Columns `cols` of the weak-scaling run's global B [K, N * world] (host)."""
    return _global_inputs(w, world)[1][:, cols.cpu()]


def run_reference(args, w, rank, world):
    """The reference's path on the host: torch.matmul on the CPU, all threads, on
    a bounded row sample of the same product per step."""
    from oracle import cpu_baseline as cb
    M, N, K, dt = w["M"], w["N"], w["K"], w["dtype"]
    # torch.distributed.run sets OMP_NUM_THREADS=1 for every rank; the
    # reference's CPU path runs on rank 0 alone, with every core this process
    # may run on
    torch.set_num_threads(_host_cores())
    a, b = _inputs(w, 0, 1)
    budget = 90.0  # seconds for the whole run
    per_step = budget / max(1, args.steps + args.warmup)
    rows = cb.calibrate_rows(a, b, min(per_step, 2.0))
    sub = a[:rows].contiguous()
    for _ in range(args.warmup):
        cb.cpu_matmul(sub, b)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        cb.cpu_matmul(sub, b)
    sec = (time.perf_counter() - t0) / args.steps
    value = 2.0 * rows * N * K / sec / 1e12
    sample = f"host torch.matmul {dt} A[:{rows}] @ B[{K},{N}] per step"
    return {
        "impl": "reference",
        "metric": "bf16 GEMM TFLOP/s at 4096^3" if dt is torch.bfloat16 else f"{w['dtype_name']} GEMM TFLOP/s",
        "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": sec * 1e3, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": w["dtype_name"], "data": "synthetic N(0,1) seed 0",
        "config": {"workload": w["desc"], "M": M, "N": N, "K": K, "rows_per_step": rows},
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": torch.get_num_threads(), "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


# --------------------------------------------------------------------------- suite
# `bench.py --suite`: every BASELINE.json config (C1-C5) on one GPU, one JSON
# line per case: the value, its roofline fraction against the bound that
# applies (dense tensor peak, CUDA-core multiply-add peak measured by
# mb_peak_probe, or HBM), an oracle check on a row or column sample, and where
# stated a host-CPU torch timing of a bounded sample of the same product.
L2_BYTES = 126 * 2 ** 20


def _suite_time(fn, nsets, min_ms=150.0, max_iters=2000):
    """Average device time of fn(i) (i cycles over nsets input sets), CUDA
    events on the current stream after 3 warm-up calls."""
    for i in range(3):
        fn(i % nsets)
    torch.cuda.synchronize()
    s = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    fn(0)
    e1.record(s)
    e1.synchronize()
    one = max(e0.elapsed_time(e1), 1e-3)
    n = int(max(5, min(max_iters, min_ms / one)))
    e0.record(s)
    for i in range(n):
        fn(i % nsets)
    e1.record(s)
    e1.synchronize()
    return e0.elapsed_time(e1) / n


def _graph_time(fn, nsets, calls=None):
    """Device time per call with the calls replayed from a CUDA graph (one
    graph of `calls` calls cycling over the input sets), so that a kernel of a
    few microseconds is not hidden behind the host's per-call dispatch cost.
    Returns None if the calls cannot be captured."""
    calls = calls or max(nsets, 32)
    try:
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for i in range(3):
                fn(i % nsets)         # plans, autotune and this stream's workspace before capture
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(side):
            with torch.cuda.graph(g, stream=side):
                for i in range(calls):
                    fn(i % nsets)
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        for _ in range(2):
            g.replay()
        torch.cuda.synchronize()
        s = torch.cuda.current_stream()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 10
        e0.record(s)
        for _ in range(reps):
            g.replay()
        e1.record(s)
        e1.synchronize()
        return e0.elapsed_time(e1) / (reps * calls)
    except RuntimeError:
        torch.cuda.synchronize()
        return None


def _nsets(bytes_per_set, cap=32):
    """Input sets to rotate so that one pass over them exceeds 2 x L2."""
    return int(max(1, min(cap, -(-int(2.2 * L2_BYTES) // max(1, int(bytes_per_set))))))


def _copies(t, n):
    return [t] + [t.clone() for _ in range(n - 1)]


def _int_range(dt):
    info = torch.iinfo(dt)
    return info.min, info.max + 1


def _cpu_rows(fn_rows, rows_total, seconds=1.0):
    """Host time of a bounded row sample: fn_rows(r) computes the first r rows.
    Returns (seconds per call, rows)."""
    r = max(1, min(rows_total, 16))
    t0 = time.perf_counter()
    fn_rows(r)
    t = max(time.perf_counter() - t0, 1e-6)
    r = int(max(1, min(rows_total, r * seconds / t)))
    fn_rows(r)
    t0 = time.perf_counter()
    fn_rows(r)
    return time.perf_counter() - t0, r


class _Suite:
    def __init__(self, args):
        import metalblas_b200 as mb
        from metalblas_b200 import _lib
        from oracle import oracle as orc
        self.mb, self.lib, self.orc = mb, _lib, orc
        self.args = args
        self.dev = torch.device("cuda", 0)
        self.bf16_peak, self.hbm, self.peak_src = _peaks()
        self.ffma = _lib.peak_probe(0)
        self.imad = _lib.peak_probe(1)
        self.imad64 = _lib.peak_probe(2)
        self.int8_peak = self._int8_peak()
        self.threads = torch.get_num_threads()
        self.emit({"suite": "peaks", "bf16_dense_tflops": self.bf16_peak, "bf16_source": self.peak_src,
                   "hbm_gbs": self.hbm, "int8_dense_tops_cublaslt": self.int8_peak,
                   "ffma_tflops_probe": self.ffma, "imad32_tops_probe": self.imad,
                   "mad64_tops_probe": self.imad64, "host_threads": self.threads,
                   "gpu": torch.cuda.get_device_name(0)})

    @staticmethod
    def emit(d):
        print(json.dumps(d), flush=True)

    def _int8_peak(self):
        """Dense int8 rate of cuBLASLt (torch._int_mm, 8192^3, best of 5): the
        measured counterpart of MEASURED_PEAKS.json's bf16 figure."""
        try:
            a = torch.randint(-128, 128, (8192, 8192), dtype=torch.int8, device=self.dev)
            b = torch.randint(-128, 128, (8192, 8192), dtype=torch.int8, device=self.dev)
            best = min(_suite_time(lambda i: torch._int_mm(a, b), 1, min_ms=50) for _ in range(5))
            return 2.0 * 8192 ** 3 / (best * 1e-3) / 1e12
        except RuntimeError:
            return 4500.0

    def check_rows(self, got, a_h, b_h, name, rows=64, bias=None, beta=None, alpha=None):
        """Oracle on a sample of output rows (2-D product a_h @ b_h)."""
        orc = self.orc
        M = a_h.shape[0]
        idx = torch.arange(0, M, max(1, M // rows))
        a_s = _to_np(a_h[idx])
        ref = (orc.product(a_s, _to_np(b_h), name) if bias is None else
               orc.fused(_to_np(bias)[idx] if bias.dim() == 2 else _to_np(bias), a_s, _to_np(b_h), beta, alpha, name))
        ok, err = orc.check(_to_np(got[idx.to(got.device)]), ref, name)
        return {"ok": bool(ok), "err": float(err), "rows": int(len(idx))}

    # ------------------------------------------------------------------ GEMM
    def gemm_case(self, suite, case, a_h, b_h, name, peak, peak_name, *, bias_h=None, beta=1.0, alpha=1.0,
                  a_view=None, b_view=None, make_a=None, flops_mult=2.0, cpu=True, check_name=None):
        """a_h/b_h: logical host operands (what the product means; a_h may be a
        conj or transposed view); a_view / b_view map a device copy of the
        logical operand to the tested layout; make_a builds the device A
        operand directly (for conj / transposed storage)."""
        mb = self.mb
        dt = a_h.dtype
        M, K = a_h.shape
        N = b_h.shape[1]
        set_bytes = (M * K + K * N + M * N) * a_h.element_size()
        n = _nsets(set_bytes, cap=8)
        if make_a is None:
            make_a = lambda: (a_view(a_h.to(self.dev)) if a_view else a_h.to(self.dev))
        make_b = lambda: (b_view(b_h.to(self.dev)) if b_view else b_h.to(self.dev))
        As = [make_a() for _ in range(n)]
        Bs = [make_b() for _ in range(n)]
        Cs = [torch.empty(M, N, dtype=dt, device=self.dev) for _ in range(n)]
        bias = bias_h.to(self.dev) if bias_h is not None else None
        if bias is None:
            fn = lambda i: mb.matmul(As[i], Bs[i], out=Cs[i])
        else:
            fn = lambda i: mb.addmm(bias, As[i], Bs[i], beta=beta, alpha=alpha, out=Cs[i])
        ms = _suite_time(fn, n)
        fn(0)
        torch.cuda.synchronize()
        flops = flops_mult * M * N * K
        value = flops / (ms * 1e-3) / 1e12
        chk = self.check_rows(Cs[0], a_h, b_h, check_name or {torch.bfloat16: "bfloat16"}.get(dt, str(dt)[6:]),
                              bias=bias_h, beta=beta, alpha=alpha)
        line = {"suite": suite, "case": case, "metric": "TFLOP/s" if dt.is_floating_point or dt.is_complex else "TOPS",
                "value": value, "ms": ms, "roofline": {"bound": peak_name, "peak": peak, "frac": value / peak},
                "check": chk, "plan": mb.kernels.plan(As[0], Bs[0]), "l2": f"{n} rotating input sets"}
        if cpu:
            line["cpu"] = self.cpu_gemm(a_h, b_h, flops_mult)
        self.emit(line)

    def cpu_gemm(self, a_h, b_h, flops_mult=2.0):
        a, b = a_h, b_h
        label = ""
        if a.dtype is torch.complex32:
            a, b = a.to(torch.complex64), b.to(torch.complex64)
            label = " (complex64 upcast: CPU has no complex32 matmul)"
        N, K = b.shape[1], b.shape[0]
        sec, rows = _cpu_rows(lambda r: torch.matmul(a[:r].contiguous(), b), a.shape[0], self.args.cpu_seconds)
        v = flops_mult * rows * N * K / sec / 1e12
        return {"value": v, "unit": "TFLOP/s" if a.dtype.is_floating_point or a.dtype.is_complex else "TOPS",
                "cores": self.threads, "kind": "port", "sample": f"host torch.matmul A[:{rows}] @ B{label}"}

    # ------------------------------------------------------------------ suites
    def c1(self):
        g = torch.Generator().manual_seed(0)
        a = torch.randn(2048, 4096, generator=g).to(torch.bfloat16)
        b = torch.randn(4096, 2048, generator=g).to(torch.bfloat16)
        bias = torch.randn(2048, generator=g).to(torch.bfloat16)
        self.gemm_case("C1", "bf16 matmul A[2048,4096]@B[4096,2048]", a, b, "bfloat16", self.bf16_peak,
                       "tensor bf16 dense")
        self.gemm_case("C1", "bf16 addmm bias[2048] beta=0.5 alpha=2", a, b, "bfloat16", self.bf16_peak,
                       "tensor bf16 dense", bias_h=bias, beta=0.5, alpha=2.0, cpu=False)
        g = torch.Generator().manual_seed(0)
        a = torch.randn(4096, 4096, generator=g).to(torch.bfloat16)
        b = torch.randn(4096, 4096, generator=g).to(torch.bfloat16)
        self.gemm_case("headline", "bf16 4096^3", a, b, "bfloat16", self.bf16_peak, "tensor bf16 dense")

    def c2(self):
        """GEMV / thin-matrix sweep: bytes 2(KN + MK + MN) against HBM."""
        mb, orc = self.mb, self.orc
        for K in (4096, 8192, 16384):
            for N in (4096, 14336, 28672):
                g = torch.Generator().manual_seed(1)
                w32 = torch.randn(K, N, generator=g) * 0.02
                xs32 = {M: torch.randn(M, K, generator=g) for M in (1, 4, 16)}
                cols = torch.randperm(N, generator=g)[:256].sort().values
                for dt, name in ((torch.bfloat16, "bfloat16"), (torch.float16, "float16")):
                    w_h = w32.to(dt)
                    W = w_h.to(self.dev)
                    Wt = W.t().contiguous()   # [N, K] storage, used as its transpose
                    nW = _nsets(W.numel() * W.element_size(), cap=16)
                    for layout in ("x@W", "x@Wt"):
                        base = W if layout == "x@W" else Wt.t()
                        ops = [base] + [(W.clone() if layout == "x@W" else Wt.clone().t()) for _ in range(nW - 1)]
                        for M in (1, 4, 16):
                            x_h = xs32[M].to(dt)
                            X = [x_h.to(self.dev) for _ in range(nW)]
                            Y = [torch.empty(M, N, dtype=dt, device=self.dev) for _ in range(nW)]
                            ms = _suite_time(lambda i: mb.matmul(X[i], ops[i], out=Y[i]), nW, min_ms=60)
                            byts = 2.0 * (K * N + M * K + M * N)
                            gbs = byts / (ms * 1e-3) / 1e9
                            gms = (_graph_time(lambda i: mb.matmul(X[i], ops[i], out=Y[i]), nW)
                                   if ms < 0.05 else None)
                            ref = orc.product(_to_np(x_h), _to_np(w_h[:, cols]), name)
                            ok, err = orc.check(_to_np(Y[0][:, cols.to(self.dev)]), ref, name)
                            line = {"suite": "C2", "case": f"{name} M={M} K={K} N={N} {layout}", "metric": "GB/s",
                                    "value": gbs, "ms": ms,
                                    "roofline": {"bound": "hbm", "peak": self.hbm, "frac": gbs / self.hbm},
                                    "check": {"ok": bool(ok), "err": float(err), "cols": 256},
                                    "plan": mb.kernels.plan(X[0], ops[0]), "l2": f"{nW} rotating weight copies"}
                            if gms:
                                line["graph"] = {"value": byts / (gms * 1e-3) / 1e9, "ms": gms,
                                                 "frac": byts / (gms * 1e-3) / 1e9 / self.hbm,
                                                 "note": "calls replayed from a CUDA graph (no host dispatch)"}
                            if M == 1 and dt is torch.bfloat16 and layout == "x@W":
                                x1 = x_h.contiguous()
                                t0 = time.perf_counter()
                                torch.matmul(x1, w_h)
                                reps = 3
                                t0 = time.perf_counter()
                                for _ in range(reps):
                                    torch.matmul(x1, w_h)
                                sec = (time.perf_counter() - t0) / reps
                                line["cpu"] = {"value": byts / sec / 1e9, "unit": "GB/s", "cores": self.threads,
                                               "kind": "port", "sample": "host torch.matmul, whole product"}
                            self.emit(line)
                        del ops
                    del W, Wt

    def c3(self):
        """Batched / broadcast bmm: roofline time = max(FLOP / tensor peak, bytes / HBM)."""
        mb, orc = self.mb, self.orc
        for dt, name in ((torch.float16, "float16"), (torch.bfloat16, "bfloat16")):
            cases = [("[8,512,256]@[8,256,512]", (8, 512, 256), (8, 256, 512), None),
                     ("[64,2048,128]@[64,128,2048]", (64, 2048, 128), (64, 128, 2048), None),
                     ("[256,1024,1024]@[256,1024,1024]", (256, 1024, 1024), (256, 1024, 1024), None),
                     ("broadcast [64,2048,128]@[1,128,2048]", (64, 2048, 128), (1, 128, 2048), None),
                     ("transposed A^T: [64,128,2048]^T@[64,128,2048]", (64, 128, 2048), (64, 128, 2048), "at"),
                     ("sliced A[:, :, :128] of [64,2048,256] (lda=2K)", (64, 2048, 256), (64, 128, 2048), "slice"),
                     ("offset A[:, 1:, 1:] of [64,2049,129]", (64, 2049, 129), (64, 128, 2048), "offset")]
            for label, sa, sb, kind in cases:
                g = torch.Generator().manual_seed(2)
                a_h = torch.randn(*sa, generator=g).to(dt)
                b_h = torch.randn(*sb, generator=g).to(dt)
                if kind == "at":
                    view = lambda t: t.transpose(1, 2)
                elif kind == "slice":
                    view = lambda t: t[:, :, :128]
                elif kind == "offset":
                    view = lambda t: t[:, 1:, 1:]
                else:
                    view = lambda t: t
                A_log = view(a_h)
                Bt, M, K = sb[0], A_log.shape[1], A_log.shape[2]
                Bsz, N = A_log.shape[0], sb[2]
                set_bytes = (a_h.numel() + b_h.numel() + Bsz * M * N) * a_h.element_size()
                n = _nsets(set_bytes, cap=64)
                As = [view(a_h.to(self.dev)) for _ in range(n)]
                Bs = [b_h.to(self.dev) for _ in range(n)]
                Cs = [torch.empty(Bsz, M, N, dtype=dt, device=self.dev) for _ in range(n)]
                if Bt == 1:
                    fn = lambda i: mb.matmul(As[i], Bs[i], out=Cs[i])  # broadcast batch, written in place
                else:
                    fn = lambda i: mb.bmm(As[i], Bs[i], out=Cs[i])
                ms = _suite_time(fn, n)
                gms = _graph_time(fn, n) if ms < 0.05 else None
                flops = 2.0 * Bsz * M * N * K
                byts = (Bsz * M * K + Bt * K * N + Bsz * M * N) * a_h.element_size()
                t_roof = max(flops / (self.bf16_peak * 1e12), byts / (self.hbm * 1e9))
                fn(0)
                torch.cuda.synchronize()
                bi = [0, Bsz - 1]
                ref = orc.product(_to_np(A_log[bi]), _to_np(b_h[[0, 0]] if Bt == 1 else b_h[bi]), name)
                ok, err = orc.check(_to_np(Cs[0][bi]), ref, name)
                sec, nb = _cpu_rows(lambda r: torch.matmul(A_log[:r], b_h if Bt == 1 else b_h[:r]), Bsz,
                                    self.args.cpu_seconds)
                line = {"suite": "C3", "case": f"{name} {label}", "metric": "TFLOP/s",
                           "value": flops / (ms * 1e-3) / 1e12, "ms": ms,
                           "roofline": {"bound": "max(tensor, hbm)", "roofline_ms": t_roof * 1e3,
                                        "frac": t_roof * 1e3 / ms,
                                        "tensor_frac": flops / (ms * 1e-3) / 1e12 / self.bf16_peak,
                                        "hbm_frac": byts / (ms * 1e-3) / 1e9 / self.hbm},
                           "check": {"ok": bool(ok), "err": float(err), "batches": bi},
                           "plan": mb.kernels.plan(As[0], Bs[0]), "l2": f"{n} rotating input sets",
                           "cpu": {"value": 2.0 * nb * M * N * K / sec / 1e12, "unit": "TFLOP/s",
                                   "cores": self.threads, "kind": "port",
                                   "sample": f"host torch.matmul, {nb} of {Bsz} batches"}}
                if gms:
                    line["graph"] = {"value": flops / (gms * 1e-3) / 1e12, "ms": gms, "frac": t_roof * 1e3 / gms,
                                     "note": "calls replayed from a CUDA graph (no host dispatch)"}
                self.emit(line)

    def c4(self):
        """Integers, bit-exact: 8-bit on the int8 tensor cores; 16/32/64-bit as
        byte planes on them too (L(L+1)/2 u8 GEMM-equivalents for L-byte
        integers, so the ceiling is the measured int8 rate / 3, / 10, / 36)."""
        mb = self.mb
        layouts = {
            "rm_rm": (None, None),
            "rm_cm": (None, lambda t: t.t().contiguous().t()),
            "cm_cm": (lambda t: t.t().contiguous().t(), lambda t: t.t().contiguous().t()),
            "offset": (lambda t: _offset_view(t), lambda t: _offset_view(t)),
        }
        for n in (4096, 8192):
            for dt, name in ((torch.int8, "int8"), (torch.uint8, "uint8")):
                g = torch.Generator().manual_seed(3)
                lo, hi = _int_range(dt)
                a = torch.randint(lo, hi, (n, n), dtype=dt, generator=g)
                b = torch.randint(lo, hi, (n, n), dtype=dt, generator=g)
                lays = ("rm_rm", "rm_cm", "cm_cm", "offset") if (n == 4096 and dt is torch.int8) else ("rm_rm",)
                for lay in lays:
                    av, bv = layouts[lay]
                    self.gemm_case("C4", f"{name} {n}^3 {lay} full range", a, b, name, self.int8_peak,
                                   "tensor int8 dense (cuBLASLt measured)", a_view=av, b_view=bv,
                                   cpu=(lay == "rm_rm" and n == 4096), check_name=name)
        for dt, name, peak, pname in ((torch.int16, "int16", self.int8_peak / 3.0, "int8 tensor / 3 (byte planes)"),
                                      (torch.int32, "int32", self.int8_peak / 10.0, "int8 tensor / 10 (byte planes)"),
                                      (torch.int64, "int64", self.int8_peak / 36.0, "int8 tensor / 36 (byte planes)")):
            g = torch.Generator().manual_seed(4)
            a = torch.randint(-1000, 1000, (2048, 2048), dtype=dt, generator=g)
            b = torch.randint(-1000, 1000, (2048, 2048), dtype=dt, generator=g)
            lays = ("rm_rm", "rm_cm", "cm_cm", "offset") if dt is torch.int32 else ("rm_rm",)
            for lay in lays:
                av, bv = layouts[lay]
                self.gemm_case("C4", f"{name} 2048^3 {lay}", a, b, name, peak, pname, a_view=av, b_view=bv,
                               cpu=(lay == "rm_rm"), check_name=name)
        # int32 GEMV 1 x 8192 x 8192
        g = torch.Generator().manual_seed(4)
        w = torch.randint(-1000, 1000, (8192, 8192), dtype=torch.int32, generator=g)
        x = torch.randint(-1000, 1000, (1, 8192), dtype=torch.int32, generator=g)
        self.gemv_case("C4", "int32 GEMV 1x8192x8192 x@W", x, w, "int32")

    def gemv_case(self, suite, case, x_h, w_h, name):
        mb, orc = self.mb, self.orc
        M, K = x_h.shape
        N = w_h.shape[1]
        elt = w_h.element_size()
        n = _nsets(K * N * elt, cap=16)
        W = [w_h.to(self.dev) for _ in range(n)]
        X = [x_h.to(self.dev) for _ in range(n)]
        Y = [torch.empty(M, N, dtype=w_h.dtype, device=self.dev) for _ in range(n)]
        ms = _suite_time(lambda i: mb.matmul(X[i], W[i], out=Y[i]), n)
        byts = elt * (K * N + M * K + M * N)
        gbs = byts / (ms * 1e-3) / 1e9
        ok, err = orc.check(_to_np(Y[0]), orc.product(_to_np(x_h), _to_np(w_h), name), name)
        self.emit({"suite": suite, "case": case, "metric": "GB/s", "value": gbs, "ms": ms,
                   "roofline": {"bound": "hbm", "peak": self.hbm, "frac": gbs / self.hbm},
                   "check": {"ok": bool(ok), "err": float(err)}, "plan": mb.kernels.plan(X[0], W[0]),
                   "l2": f"{n} rotating weight copies"})

    def c5(self):
        mb = self.mb
        # complex64 runs as one real 3xTF32 GEMM on the tensor cores: three tf32
        # MMAs per K-step at half the bf16 rate, so its ceiling is the measured
        # bf16 dense peak / 6 (the FFMA probe stays in the peaks line)
        for dt, name, peak, pname in ((torch.complex64, "complex64", self.bf16_peak / 6.0,
                                       "tensor 3xTF32 (bf16 dense / 6; 8MNK real ops)"),
                                      (torch.complex32, "complex32", self.bf16_peak, "tensor fp16 dense")):
            g = torch.Generator().manual_seed(5)
            a = torch.complex(torch.randn(4096, 4096, generator=g), torch.randn(4096, 4096, generator=g)).to(dt)
            b = torch.complex(torch.randn(4096, 4096, generator=g), torch.randn(4096, 4096, generator=g)).to(dt)
            self.gemm_case("C5", f"{name} 4096^3", a, b, name, peak, pname, flops_mult=8.0, check_name=name)
            # conj(A) @ B: A passed as a lazy conj view (conj bit, read in place)
            self.gemm_case("C5", f"{name} conj(A)@B 4096^3", a.conj(), b, name, peak, pname,
                           make_a=lambda: a.to(self.dev).conj(), flops_mult=8.0, cpu=False, check_name=name)
            # A^T @ B: A stored row-major, passed transposed (column-major read)
            self.gemm_case("C5", f"{name} A^T@B 4096^3", a.t(), b, name, peak, pname,
                           make_a=lambda: a.to(self.dev).t(), flops_mult=8.0, cpu=False, check_name=name)
            x = torch.complex(torch.randn(1, 8192, generator=g), torch.randn(1, 8192, generator=g)).to(dt)
            w = torch.complex(torch.randn(8192, 8192, generator=g), torch.randn(8192, 8192, generator=g)).to(dt)
            self.gemv_case("C5", f"{name} GEMV 1x8192x8192 x@W", x, w, name)
        g = torch.Generator().manual_seed(6)
        a = torch.randn(16384, 16384, generator=g).to(torch.bfloat16)
        b = torch.randn(16384, 16384, generator=g).to(torch.bfloat16)
        # 8 ms per launch, timed back to back for seconds: the power-capped
        # sustained rate is the roofline that applies (the burst one if absent)
        sus = _sustained_peak()
        self.gemm_case("C5", "bf16 16384^3", a, b, "bfloat16", sus or self.bf16_peak,
                       "tensor bf16 dense, sustained" if sus else "tensor bf16 dense")
        del a, b
        g = torch.Generator().manual_seed(6)
        a = torch.randn(128, 65536, generator=g).to(torch.bfloat16)
        b = torch.randn(65536, 8192, generator=g).to(torch.bfloat16)
        self._skinny(a, b)

    def _skinny(self, a_h, b_h):
        """128 x 8192 x 65536 bf16: HBM-bound (reads B once)."""
        mb = self.mb
        M, K = a_h.shape
        N = b_h.shape[1]
        As = [a_h.to(self.dev) for _ in range(2)]
        Bs = [b_h.to(self.dev) for _ in range(2)]
        Cs = [torch.empty(M, N, dtype=torch.bfloat16, device=self.dev) for _ in range(2)]
        ms = _suite_time(lambda i: mb.matmul(As[i], Bs[i], out=Cs[i]), 2)
        byts = 2.0 * (M * K + K * N + M * N)
        gbs = byts / (ms * 1e-3) / 1e9
        chk = self.check_rows(Cs[0], a_h, b_h, "bfloat16", rows=16)
        self.emit({"suite": "C5", "case": "bf16 skinny split-K 128x8192x65536", "metric": "GB/s", "value": gbs,
                   "ms": ms, "tflops": 2.0 * M * N * K / (ms * 1e-3) / 1e12,
                   "roofline": {"bound": "hbm", "peak": self.hbm, "frac": gbs / self.hbm}, "check": chk,
                   "plan": mb.kernels.plan(As[0], Bs[0]), "l2": "inputs 1.1 GB > L2",
                   "cpu": self.cpu_gemm(a_h, b_h)})


def _to_np(t):
    """Values of a (possibly conj / strided / cuda) tensor as numpy, exactly."""
    t = t.detach()
    if t.dtype is torch.complex32:
        t = t.to(torch.complex64)
    if t.is_conj():
        t = t.resolve_conj()
    if t.is_neg():
        t = t.resolve_neg()
    t = t.cpu()
    if t.dtype is torch.bfloat16:
        t = t.float()
    return t.numpy()


def _offset_view(t):
    """The reference's "offset" layout: [1:, 1:] of a (rows+1) x (cols+1) buffer
    (lda = cols + 1, storage offset > 0)."""
    big = torch.zeros(t.shape[0] + 1, t.shape[1] + 1, dtype=t.dtype, device=t.device)
    big[1:, 1:] = t
    return big[1:, 1:]


# `bench.py --one CASE`: one product, a few warm-up calls and `--steps` timed
# calls (CUDA events), one JSON line.  Small enough to run under ncu; the
# profiles/ summaries name these commands.
ONE_CASES = {
    "bf16_gemm_4096": ("gemm", torch.bfloat16, 4096, 4096, 4096, None),
    "fp16_gemm_4096": ("gemm", torch.float16, 4096, 4096, 4096, None),
    "c32_gemm_4096": ("gemm", torch.complex32, 4096, 4096, 4096, None),
    "c64_gemm_4096": ("gemm", torch.complex64, 4096, 4096, 4096, None),
    "fp32_gemm_4096": ("gemm", torch.float32, 4096, 4096, 4096, None),
    "gemv_bf16_1x4096x4096": ("gemm", torch.bfloat16, 1, 4096, 4096, None),
    "gemv_bf16_1x4096x4096_wt": ("gemm", torch.bfloat16, 1, 4096, 4096, "wt"),
    "gemv_bf16_16x4096x4096": ("gemm", torch.bfloat16, 16, 4096, 4096, None),
    # the CUDA-core kernels (backend="simd": FFMA for fp32, IMAD for int32)
    "simt_fp32_gemm_2048": ("gemm", torch.float32, 2048, 2048, 2048, None, "simd"),
    "simt_int32_gemm_2048": ("gemm", torch.int32, 2048, 2048, 2048, None, "simd"),
}


def run_one(args):
    import metalblas_b200 as mb
    kind, dt, M, N, K, lay, backend = (ONE_CASES[args.one] + (None,))[:7]
    kw = {"backend": backend} if backend else {}
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)

    def rnd(*shape):
        if not dt.is_floating_point and not dt.is_complex:
            return torch.randint(-1000, 1000, shape, generator=g, device=dev, dtype=dt)
        if dt.is_complex:
            return torch.complex(torch.randn(*shape, generator=g, device=dev),
                                 torch.randn(*shape, generator=g, device=dev)).to(dt)
        return torch.randn(*shape, generator=g, device=dev).to(dt)
    byts = (M * K + K * N + M * N) * torch.empty((), dtype=dt).element_size()
    sets = _nsets(byts, cap=16)
    A = [rnd(M, K) for _ in range(sets)]
    B = [(rnd(N, K).t() if lay == "wt" else rnd(K, N)) for _ in range(sets)]
    C = [torch.empty(M, N, dtype=dt, device=dev) for _ in range(sets)]
    for i in range(max(args.warmup, 3)):
        mb.matmul(A[i % sets], B[i % sets], out=C[i % sets], **kw)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(args.steps):
        mb.matmul(A[i % sets], B[i % sets], out=C[i % sets], **kw)
    e1.record()
    e1.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    flops = (8.0 if dt.is_complex else 2.0) * M * N * K
    print(json.dumps({"one": args.one, "ms": ms, "tflops": flops / (ms * 1e-3) / 1e12,
                      "gbs": byts / (ms * 1e-3) / 1e9, "plan": mb.kernels.plan(A[0], B[0], **kw),
                      "l2": f"{sets} rotating input sets"}), flush=True)


def run_suite(args):
    assert torch.cuda.is_available(), "bench.py --suite needs a CUDA device"
    torch.cuda.set_device(0)
    s = _Suite(args)
    for c in args.configs.split(","):
        getattr(s, c.lower())()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="bf16_gemm_4096", choices=sorted(WORKLOADS))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-bmm", action="store_true", help="skip the batch-sharded bmm measurement")
    ap.add_argument("--no-multi", action="store_true",
                    help="skip the 16384^3 N-sharded and skinny 128x8192x65536 measurements")
    ap.add_argument("--suite", action="store_true",
                    help="measure every BASELINE config on one GPU, one JSON line per case")
    ap.add_argument("--configs", default="C1,C2,C3,C4,C5")
    ap.add_argument("--cpu-seconds", type=float, default=1.0, help="host time per CPU-baseline sample")
    ap.add_argument("--one", choices=sorted(ONE_CASES), help="time one product (small enough to run under ncu)")
    args = ap.parse_args()
    if args.suite:
        run_suite(args)
        return
    if args.one:
        torch.cuda.set_device(0)
        run_one(args)
        return
    w = dict(WORKLOADS[args.workload])
    w["name"] = args.workload
    w["dtype_name"] = {torch.bfloat16: "bf16", torch.float16: "fp16", torch.int8: "int8"}[w["dtype"]]
    rank, world, local = _dist()

    if args.impl == "reference":
        if rank != 0:
            return
        print(json.dumps(run_reference(args, w, rank, world)), flush=True)
        return

    assert torch.cuda.is_available(), "bench.py --impl ours needs a CUDA device"
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
    try:
        res = run_ours(args, w, rank, world, device)
        if rank == 0:
            print(json.dumps(res), flush=True)
    finally:
        if world > 1:
            import torch.distributed as dist
            from metalblas_b200 import peer
            torch.cuda.synchronize(device)
            peer.release_arenas()
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
