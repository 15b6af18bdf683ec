"""Benchmark of the B200 hot path (one JSON line on rank 0).

Workload `q8_gemm_layer_sweep` (the Q8_0 GEMM shape sweep of one
FastConformer layer): shapes QKV (K=1024, N=3072), out-proj (1024, 1024),
FFN-up (1024, 4096) and FFN-down (4096, 1024) at M = 1, 8, 32 and 128 frames,
seeded ~N(0, 1) activations and ~N(0, 0.02) weights quantised to Q8_0.  One
step runs every (M, shape) GEMM over 24 distinct layer copies of the weights
(321 MB, like the encoder's 24 layers), M-major, so every weight byte comes
from HBM, not L2 (126 MB).  The step is captured once in a CUDA graph and
replayed.  value = algorithmic bytes (weights N*K*34/32 + f32 x 4*M*K + f32 y
4*M*N per GEMM) of all ranks / max-over-ranks device time.

Multi-GPU: one process per GPU (torchrun), every rank runs the same sweep on
its own weight replica (no data-path collective; weak scaling).

`--impl reference` times the reference's CPU path (the oracle's AVX2+threads
restatement of q8_gemm) on a bounded sample (layer copy 0 only) of the same
workload, rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

SHAPES = [("qkv", 1024, 3072), ("out", 1024, 1024), ("ffn_up", 1024, 4096), ("ffn_down", 4096, 1024)]
MS = [1, 8, 32, 128]
LAYERS = 24
METRIC = "Q8_0 GEMM HBM GB/s (FastConformer layer shape sweep)"


def gemm_bytes(m, k, n):
    return n * k * 34 // 32 + 4 * m * k + 4 * m * n


def kernel_bytes(m, k, n):
    # the GEMM kernel alone reads quantised activations (int8 + f32 block scales)
    return n * k * 34 // 32 + m * k + 4 * m * (k // 32) + 4 * m * n


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--e2e-steps", type=int, default=3)
    ap.add_argument("--profile", default=None, choices=["gemm", "attn", "tc"],
                    help="small eager case for ncu captures (no timing, no JSON line)")
    return ap.parse_args()


# ---------------------------------------------------------------- clocks ---
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"], stdout=self.f,
                                         stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.f.close()
        rows = [r.split(",") for r in open(self.path).read().strip().splitlines() if r.strip()]
        os.unlink(self.path)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].strip().replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].strip().replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if len(r) > 5 + i and "Active" in r[5 + i]
                          and "Not" not in r[5 + i]})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


# ------------------------------------------------------------ CPU paths ---
def cpu_sample(layer_weights_host, threads=0, reps=1):
    """The reference CPU path (oracle restatement of q8_gemm) over one layer
    copy: every (M, shape) GEMM once.  Returns (GB/s, seconds, bytes)."""
    import oracle

    xs = {}
    tot_bytes = 0
    t0 = time.perf_counter()
    for _ in range(reps):
        for m in MS:
            for name, k, n in SHAPES:
                if (m, k) not in xs:
                    from stealcode_b200 import synth

                    xs[(m, k)] = np.ascontiguousarray(synth.normal(synth.SEED_BASE + 100 + m + k, (m, k)).T)
                oracle.q8_gemm(n, k, m, layer_weights_host[name], (k // 32) * 34, 34, 2, xs[(m, k)],
                               nthreads=threads)
                tot_bytes += gemm_bytes(m, k, n)
    dt = time.perf_counter() - t0
    return tot_bytes / dt / 1e9, dt, tot_bytes


def host_weights():
    from stealcode_b200 import synth

    return {name: synth.q8_weights(synth.SEED_BASE + 1 + i, n, k) for i, (name, k, n) in enumerate(SHAPES)}


def run_reference(args, rank):
    if rank != 0:
        return
    import oracle

    w = host_weights()
    for _ in range(args.warmup):
        cpu_sample(w)
    times, gbs = [], []
    total_bytes = 0
    for _ in range(args.steps):
        g, dt, b = cpu_sample(w)
        times.append(dt)
        gbs.append(g)
        total_bytes += b
    value = total_bytes / sum(times) / 1e9
    cores = oracle.num_cpus()
    sample = "layer copy 0 of 24: the 16 (M, shape) GEMMs once per step"
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * sum(times) / len(times),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": "q8_gemm_layer_sweep", "shapes": SHAPES, "m": MS, "sample": sample},
            "cpu_baseline": {"value": value, "unit": "GB/s", "cores": cores, "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------ GPU path ---
def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    from stealcode_b200 import _lib, synth
    from stealcode_b200._lib import SC_LAYOUT_FEATURE_MAJOR, SC_LAYOUT_TIME_MAJOR, check
    from stealcode_b200.ops import Q8Mat

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    lib = _lib.lib
    wh = host_weights()
    mats = [{name: Q8Mat(wh[name], n, k) for name, k, n in SHAPES} for _ in range(LAYERS)]
    xs = {(m, k): torch.from_numpy(synth.normal(synth.SEED_BASE + 100 + m + k, (m, k))).to(dev)
          for m in MS for k in (1024, 4096)}
    ys = {(m, n): torch.empty((m, n), dtype=torch.float32, device=dev) for m in MS for n in (1024, 3072, 4096)}
    ws_bytes = int(lib.sc_q8_gemm_workspace_bytes(max(MS), 4096))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    # pre-quantised activations for the kernel-only (roofline) pass
    xq = {}
    for m in MS:
        for k in (1024, 4096):
            q = torch.zeros((m, k), dtype=torch.int8, device=dev)
            d = torch.zeros((k // 32, m), dtype=torch.float32, device=dev)
            check(lib.sc_q8_quantize(xs[(m, k)].data_ptr(), m, k, SC_LAYOUT_TIME_MAJOR, 0, q.data_ptr(),
                                     d.data_ptr(), torch.cuda.current_stream().cuda_stream))
            xq[(m, k)] = (q, d)
    torch.cuda.synchronize()

    def step_calls(stream, kernel_only=False, only_m=None):
        n_launch = 0
        for m in MS if only_m is None else [only_m]:
            for layer in mats:
                for name, k, n in SHAPES:
                    y = ys[(m, n)]
                    if kernel_only:
                        q, d = xq[(m, k)]
                        check(lib.sc_q8_gemm_q(layer[name].handle, q.data_ptr(), d.data_ptr(), m, m, None,
                                               y.data_ptr(), SC_LAYOUT_TIME_MAJOR, 0, stream))
                        n_launch += 1
                    else:
                        check(lib.sc_q8_gemm(layer[name].handle, xs[(m, k)].data_ptr(), m, SC_LAYOUT_TIME_MAJOR,
                                             0, None, y.data_ptr(), SC_LAYOUT_TIME_MAJOR, 0, ws.data_ptr(),
                                             ws_bytes, stream))
                        n_launch += 1
        return n_launch

    def capture(**kw):
        s = torch.cuda.Stream(device=dev)
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            step_calls(s.cuda_stream, **kw)  # warm: sets smem attributes outside capture
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            n = step_calls(torch.cuda.current_stream().cuda_stream, **kw)
        return g, n

    def time_graph(g, steps, warmup):
        for _ in range(warmup):
            g.replay()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            g.replay()
        e1.record()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        ms = e0.elapsed_time(e1)
        if world > 1:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms / steps

    g_step, launches_per_step = capture()
    step_bytes = sum(gemm_bytes(m, k, n) for m in MS for _ in range(LAYERS) for _, k, n in SHAPES)

    clocks = ClockSampler(local_rank)
    clocks.start()
    time.sleep(0.3)  # the sampler's first reading lands inside the timed region
    ms_step = time_graph(g_step, args.steps, args.warmup)
    clk = clocks.stop()
    value = world * step_bytes / (ms_step * 1e-3) / 1e9

    # roofline: the GEMM kernel alone, per M and over the whole sweep
    g_k, n_k = capture(kernel_only=True)
    ms_k = time_graph(g_k, max(3, args.steps // 2), 2)
    kbytes = sum(kernel_bytes(m, k, n) for m in MS for _ in range(LAYERS) for _, k, n in SHAPES)
    peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json"))) if os.path.exists(
        os.path.join(ROOT, "MEASURED_PEAKS.json")) else {}
    peak = peaks.get("hbm_gbs", 6650.0)
    peak_src = "measured" if "hbm_gbs" in peaks else "fallback"
    by_m = {}
    for m in MS:
        g_m, n_m = capture(kernel_only=True, only_m=m)
        ms_m = time_graph(g_m, max(3, args.steps // 2), 2)
        b_m = sum(kernel_bytes(m, k, n) for _, k, n in SHAPES) * LAYERS
        by_m[str(m)] = {"us_per_launch": 1e3 * ms_m / n_m, "gbs": b_m / (ms_m * 1e-3) / 1e9,
                        "frac": b_m / (ms_m * 1e-3) / 1e9 / peak}
        del g_m
    achieved = kbytes / (ms_k * 1e-3) / 1e9
    roofline = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                "peak_source": peak_src, "kernel": "q8_gemm_small_kernel",
                "bytes_per_launch_avg": kbytes / n_k, "us_per_launch_avg": 1e3 * ms_k / n_k,
                "traffic": None, "by_m": by_m}

    # e2e: the reference-facing host-buffer call (Q8Mat::gemm_t twin), pinned host x/y
    hx = {key: torch.empty((key[1], key[0]), dtype=torch.float32).pin_memory() for key in xs}
    for key, t in xs.items():
        hx[key].copy_(t.t().cpu())
    hy = {(m, n): torch.empty((n, m), dtype=torch.float32).pin_memory() for m in MS for n in (1024, 3072, 4096)}
    h2d = sum(4 * m * k for m in MS for _ in range(LAYERS) for _, k, n in SHAPES)
    d2h = sum(4 * m * n for m in MS for _ in range(LAYERS) for _, k, n in SHAPES)

    def e2e_step():
        for m in MS:
            for layer in mats:
                for name, k, n in SHAPES:
                    check(lib.sc_q8mat_gemm_t(layer[name].handle, hx[(m, k)].data_ptr(), m, hy[(m, n)].data_ptr()))

    e2e_step()
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(args.e2e_steps):
        e2e_step()
    e2e_s = (time.perf_counter() - t0) / args.e2e_steps
    if world > 1:
        t = torch.tensor([e2e_s], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    e2e = {"value": world * step_bytes / e2e_s / 1e9, "unit": "GB/s", "h2d_bytes_per_step": h2d,
           "d2h_bytes_per_step": d2h, "api": "sc_q8mat_gemm_t (host x [k,t], host y [n,t], pinned)"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        import oracle

        g, dt, b = cpu_sample(wh)
        cpu = {"value": g, "unit": "GB/s", "cores": oracle.num_cpus(), "kind": "port",
               "sample": f"layer copy 0 of 24: the 16 (M, shape) GEMMs once ({dt:.1f} s)"}
    del g_step, g_k
    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "int8", "data": "synthetic",
                "config": {"workload": "q8_gemm_layer_sweep", "shapes": SHAPES, "m": MS, "layers": LAYERS,
                           "parallelism": f"replicas x{world}",
                           "l2": "inputs larger than L2: 24 distinct layer weight copies (321 MB) per M pass"},
                "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e,
                "gpu_launches": launches_per_step * args.steps, "clocks": clk}
        print(json.dumps(line), flush=True)


def run_profile(args):
    """A few eager launches of one kernel family on a small case, for ncu."""
    import math

    import torch

    from stealcode_b200 import synth
    from stealcode_b200.ops import SC_LAYOUT_TIME_MAJOR, Q8Mat, attn_stream_ring

    dev = torch.device("cuda", 0)
    if args.profile in ("gemm", "tc"):
        wh = host_weights()
        for name, k, n in SHAPES:
            mat = Q8Mat(wh[name], n, k)
            for m in ((8, 128) if args.profile == "gemm" else (1792,)):
                x = torch.from_numpy(synth.normal(synth.SEED_BASE + 100 + m + k, (m, k))).to(dev)
                for _ in range(3):
                    mat.gemm(x, x_layout=SC_LAYOUT_TIME_MAJOR, y_layout=SC_LAYOUT_TIME_MAJOR)
    else:
        ns, c, d, nh, chunk, lc, cap, s = 64, 8, 1024, 8, 7, 10, 84, 140
        k_lo = (s // chunk - lc) * chunk
        z = lambda *shape: torch.from_numpy(synth.normal(7 + len(shape), shape)).to(dev)
        q, kn, vn = z(ns * c, d), z(ns * c, d), z(ns * c, d)
        rk, rv = z(ns, cap, d), z(ns, cap, d)
        pos = z((lc + 2) * chunk - 1, d)
        u, v = z(d) * 0.02, z(d) * 0.02
        for _ in range(3):
            attn_stream_ring(q, kn, vn, rk, rv, pos, u, v, c=c, d=d, n_heads=nh, scale=1 / math.sqrt(128), s=s,
                             k_lo=k_lo, chunk=chunk, left_chunks=lc, pos_off=chunk - 1)
    torch.cuda.synchronize()
    print("profile case done")


def main():
    args = parse()
    if args.profile:
        run_profile(args)
        return
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
