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

PUBLISHED_M5_MAX_4096 = 42.95   # bf16 4096^3, Apple M5 Max, perf_benchs/M5_Max.md:17


def _peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p["bf16_tflops"]), float(p.get("hbm_gbs", 6650.0)), "measured"
    except (OSError, ValueError, KeyError):
        return 1590.0, 6650.0, "fallback"


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


def _inputs(w, rank, world):
    g = torch.Generator().manual_seed(0)
    M, N, K, dt = w["M"], w["N"], w["K"], w["dtype"]
    if dt in (torch.int8, torch.uint8):
        info = torch.iinfo(dt)
        a = torch.randint(info.min, info.max + 1, (M, K), dtype=dt, generator=g)
        b_full = torch.randint(info.min, info.max + 1, (K, N * world), dtype=dt, generator=g) if world > 1 else None
        b = torch.randint(info.min, info.max + 1, (K, N), dtype=dt, generator=g) if world == 1 else None
    else:
        a = torch.randn(M, K, generator=g).to(dt)
        b_full = torch.randn(K, N * world, generator=g).to(dt) if world > 1 else None
        b = torch.randn(K, N, generator=g).to(dt) if world == 1 else None
    if world > 1:
        b = b_full[:, rank * N:(rank + 1) * N].contiguous()
    return a, b


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

    # gathered variant (N > 1): all-gather the output shards over NVLink each step
    gathered = None
    if world > 1:
        import torch.distributed as dist
        G = torch.empty(world, M, N, dtype=dt, device=device)
        for i in range(3):
            mb.matmul(As[i % SETS], Bs[i % SETS], out=Cs[i % SETS])
            dist.all_gather_into_tensor(G, Cs[i % SETS])
        _barrier(world, device)
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        g0.record(stream)
        for i in range(args.steps):
            mb.matmul(As[i % SETS], Bs[i % SETS], out=Cs[i % SETS])
            dist.all_gather_into_tensor(G, Cs[i % SETS])
        g1.record(stream)
        g1.synchronize()
        _barrier(world, device)
        gms = _max_over_ranks(g0.elapsed_time(g1) / args.steps, world, device)
        gathered = {"value": flops * world / (gms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": gms,
                    "layout": "[N_ranks, M, N/N_ranks] via NCCL all_gather_into_tensor"}

    # e2e: host buffers -> public API -> host result, every step.  Three streams
    # (copy-in, compute, copy-out) and two device buffer sets, so step i's
    # host-to-device copy overlaps step i-1's product and step i-2's read-back;
    # every step still copies its own inputs and reads its own result.
    e2e_steps = max(1, min(args.steps, 100))
    elt = a_h.element_size()
    s_in, s_out = torch.cuda.Stream(device), torch.cuda.Stream(device)
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
            a_d[j].copy_(a_pin, non_blocking=True)
            b_d[j].copy_(b_pin, non_blocking=True)
            in_done[j].record(s_in)
        stream.wait_event(in_done[j])
        stream.wait_event(out_done[j])           # c_d[j] read back (step i-2)
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
           "h2d_bytes_per_step": (M * K + K * N) * elt, "d2h_bytes_per_step": M * N * elt, "steps": e2e_steps,
           "pipelining": "copy-in / compute / copy-out streams, 2 device buffer sets"}

    peak, hbm, src = _peaks()
    achieved = flops / (ms * 1e-3) / 1e12
    traffic = _profile_traffic(f"tc_gemm_{w['dtype_name']}_{M}x{N}x{K}.txt")
    roofline = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                "frac": achieved / peak, "peak_source": f"{src} bf16_tflops (burst)",
                "traffic": traffic, "kernel": "mb::tc::tc_gemm_kernel", "per_launch_flop": flops}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle import cpu_baseline as cb
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
        "gpu_launches": args.steps, "check": ok_rows, "clocks": sampler.summary() if rank == 0 else None,
    }


def run_reference(args, w, rank, world):
    """The reference's path on the host: torch.matmul on the CPU, all threads, on
    a bounded row sample of the same product per step."""
    from oracle import cpu_baseline as cb
    M, N, K, dt = w["M"], w["N"], w["K"], w["dtype"]
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


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="bf16_gemm_4096", choices=sorted(WORKLOADS))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
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
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
