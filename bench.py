"""Benchmark of the B200 hot path (one JSON line on rank 0).

Headline workload `streaming_encoder_24l` (the full streaming encoder): a
random-init 24-layer FastConformer (d_model 1024, 8 heads, macaron FFN 4096,
depthwise causal conv kernel 9, pointwise 1024 -> 2048 GLU, every linear
Q8_0 from ~N(0, 0.02) weights) streaming 256 concurrent streams of seeded
~N(0, 1) 128-bin log-mel.  One step is one encode_new call that advances
every stream by one 560 ms chunk (56 mel frames -> 7 encoder frames) with
70 frames of left context; the first 11 steps (untimed priming) bring the
attention band to its steady 77 frames.  value = audio seconds encoded per
second of device time over all ranks: n_gpus * streams * 0.56 * K / (max
over ranks of the K steps' CUDA-event time).  The f16 weight tiles a step
streams (1.1 GB; 587 MB as Q8_0) are larger than L2 (126 MB).

Also in the line:
  roofline      the tcgen05 GEMM (the step's dominant kernel: kind::f16
                on the int8 codes held as f16, exact per-block f32 drain) at
                the step's shapes (the encoder's two halves of the streams,
                896 frames each at 256 streams, in flight on two CUDA
                streams), over the 24 layers' own weights, timed with CUDA
                events, against the dense f16 tensor peak; drain_issue is the
                same time against the kernel's own floor, 3 f32 operations
                per (output, 32-deep block) at 128 per SM per clock;
  gemm_sweep    the Q8_0 GEMM shape sweep of one layer (M = 1, 8, 32, 128;
                QKV, out-proj, FFN-up, FFN-down; 24 weight copies, 321 MB)
                as HBM GB/s, and its weight-streaming kernel's roofline;
                config0 is the single streaming chunk (M 8, K 1024, N 4096)
                on its own; batched is the sweep for M = 1 and 8 as one
                sc_q8_gemm_batch call per M (96 GEMMs streamed in one pass);
  e2e           the same metric through the C ABI with host mel buffers:
                pinned host -> device copy of each step's mel, encode_new,
                device -> pinned host copy of the step's output frames;
  prefill       a 750-frame (60 s) prefill of 64 streams: the same device
                encoder given 56 encoder frames (448 mel) per encode_new call
                (13 calls + a 22-frame tail), so every GEMM sees M = 64 * 56
                frames; audio seconds per second of CUDA-event time;
  box_scale     the box-scale streaming batch: 8192 concurrent streams
                sharded by stream over the GPUs (8192 / N per GPU, each
                rank's shard in one encoder; a shard that does not fit in
                device memory is halved, and the streams actually resident
                are reported), audio seconds per second over all ranks;
  transcriber   the streaming transcriber's whole step (LiveTranscriber::
                process): encode_new, then the RNN-T greedy decode of each
                stream's 7 new frames (random-init 2 x 640 LSTM predictor,
                joint 640, 1025 classes) straight from the encoder's device
                output; CUDA-event time per step, the decoder's share, and
                the tokens emitted per frame;
  cpu_baseline  the reference CPU path (the oracle's restatement with the
                reference's threading -- rayon over 256-row GEMM chunks,
                conv output positions and attention queries -- and AVX2
                lanes, one StreamingEncoder per stream) on a bounded sample
                of the same workload with its host seconds by phase, and the
                reference CPU GEMM on one streaming chunk (M 8, K 1024,
                N 4096) with all host threads and with one.

Multi-GPU: one process per GPU (torchrun); every rank encodes its own 256
streams with its own weight copy (streams are independent: no collective on
the data path; weak scaling).

`--impl reference` times the reference's CPU path (the oracle port above,
all host threads) on a bounded sample per step, rank 0 only.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "encoder audio-sec/sec (24-layer streaming FastConformer, 560 ms chunks)"
UNIT = "audio-s/s"
WORKLOAD = "streaming_encoder_24l"
MEL_PER_STEP = 56          # 560 ms of 10 ms mel frames -> 7 encoder frames
AUDIO_S_PER_STEP = 0.56
PRIME_STEPS = 11           # band reaches its steady 77 frames
N_LAYERS = 24
MODEL_SEED = 0x5EED0000 + 3
MEL_POOL = 8               # distinct mel chunks cycled through the steps
DECODER_BLANK_BIAS = 0.9   # random decoder's blank bias: ~0.5 tokens / frame on the encoder's output

SHAPES = [("qkv", 1024, 3072), ("out", 1024, 1024), ("ffn_up", 1024, 4096), ("ffn_down", 4096, 1024)]
MS = [1, 8, 32, 128]
SWEEP_LAYERS = 24


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--streams", type=int, default=256, help="streams per GPU")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-sweep", action="store_true", help="skip the GEMM shape sweep block")
    ap.add_argument("--e2e-steps", type=int, default=10)
    ap.add_argument("--no-decoder", action="store_true", help="skip the transcriber (encoder + decoder) block")
    ap.add_argument("--no-prefill", action="store_true", help="skip the 750-frame prefill block")
    ap.add_argument("--no-graphs", action="store_true",
                    help="launch every kernel of a step separately instead of replaying the step's CUDA graph")
    ap.add_argument("--box-streams", type=int, default=8192,
                    help="global streams of the box-scale block (sharded over the GPUs); 0 skips it")
    ap.add_argument("--box-steps", type=int, default=3)
    ap.add_argument("--profile", default=None, choices=["gemm", "attn", "tc", "encoder", "breakdown", "batch"],
                    help="small eager case for ncu captures (no timing, no JSON line); breakdown: per-kernel "
                         "device time of 3 steady headline steps (CUPTI through torch.profiler)")
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


def reduce_max(value: float, device) -> float:
    """Max of `value` over the ranks of the default process group (the value
    itself without one); every rank must call it at the same point."""
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return value
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def stream_shard(global_streams: int, world: int, rank: int):
    """Contiguous streams [lo, hi) of `rank` when `global_streams` independent
    streams are spread over `world` GPUs (the first ranks take the remainder)."""
    from stealcode_b200 import shards

    return shards.stream_shard(global_streams, world, rank)


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    return json.load(open(p)) if os.path.exists(p) else {}


def encoder_config():
    from stealcode_b200 import model

    return model.EncoderConfig(n_layers=N_LAYERS)


def encoder_model():
    from stealcode_b200 import model

    return model.random_model(encoder_config(), seed=MODEL_SEED)


# ------------------------------------------------------------ CPU paths ---
def cpu_encoder_sample(m, n_streams, n_steps, budget_s=None):
    """The reference CPU path for n_streams streams x up to n_steps chunks
    from t = 0: one oracle StreamingEncoder per stream in its fast mode --
    the reference's threading (rayon over 256-row chunks, output positions
    and queries, on all host threads) and AVX2 lanes, bit-identical to the
    serial restatement -- with the reference's Q8 GEMM dispatch.  Returns
    (audio-s/s, seconds, audio seconds, steps, host seconds by phase)."""
    import oracle
    from stealcode_b200 import model

    mel = model.mel_stream(MODEL_SEED + 1, n_streams, MEL_PER_STEP * n_steps, m.config.feat_in)
    encs = [oracle.StreamingEncoder(m) for _ in range(n_streams)]
    t0 = time.perf_counter()
    done = 0
    for i in range(n_steps):
        a, b = MEL_PER_STEP * i, MEL_PER_STEP * (i + 1)
        for z in range(n_streams):
            assert encs[z].encode_new(mel[z, :b], a, b) == 0
        done += 1
        if budget_s is not None and time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    audio = n_streams * done * AUDIO_S_PER_STEP
    return audio / dt, dt, audio, done, phase_sum(encs)


def phase_sum(encs):
    """Host seconds by phase summed over the oracle encoders, with the rest."""
    tot = {"pre_encode": 0.0, "linears": 0.0, "attention": 0.0, "total": 0.0}
    for e in encs:
        for k, v in e.phase_times().items():
            tot[k] += v
    tot["rest"] = tot["total"] - tot["pre_encode"] - tot["linears"] - tot["attention"]
    return tot


def cpu_gemm_sample(budget_s=2.0):
    """The reference CPU GEMM on the single streaming-chunk workload (8
    frames x K 1024 through a 4096-row Q8_0 matrix, weights ~N(0, 0.02)
    quantised to Q8_0, activations ~N(0, 1), seeded): the oracle's AVX2
    restatement of q8_gemm's SIMD dispatch (simd_kernel.rs:96-394), with all
    host threads and with one.  Returns µs per GEMM and GEMM GB/s for each."""
    import oracle
    from stealcode_b200 import synth

    m, k, n = 4096, 1024, 8
    w = synth.q8_weights(synth.SEED_BASE, m, k)
    x = synth.normal(synth.SEED_BASE + 1, (k, n))
    y = np.zeros((m, n), dtype=np.float32)
    nbytes = m * (k // 32) * 34 + 4 * k * n + 4 * m * n
    out = {"workload": "q8_gemm M=8 K=1024 N=4096 (one streaming chunk)", "bytes_per_gemm": nbytes}
    for label, threads in (("all_threads", 0), ("one_thread", 1)):
        oracle.q8_gemm(m, k, n, w, (k // 32) * 34, 34, 2, x, nthreads=threads, y=y)
        reps, t0 = 0, time.perf_counter()
        while True:
            oracle.q8_gemm(m, k, n, w, (k // 32) * 34, 34, 2, x, nthreads=threads, y=y)
            reps += 1
            dt = time.perf_counter() - t0
            if dt > budget_s:
                break
        out[label] = {"us_per_gemm": 1e6 * dt / reps, "gbs": nbytes * reps / dt / 1e9,
                      "threads": oracle.num_cpus() if threads == 0 else 1}
    return out


def run_reference(args, rank):
    if rank != 0:
        return
    import oracle

    m = encoder_model()
    n_streams = 2
    # one reference step = one 560 ms chunk for 2 streams (the GPU arm's step
    # for 256 streams, sampled); state carries across steps like a stream
    encs = [oracle.StreamingEncoder(m) for _ in range(n_streams)]
    from stealcode_b200 import model

    total = args.warmup + args.steps
    mel = model.mel_stream(MODEL_SEED + 1, n_streams, MEL_PER_STEP * total, m.config.feat_in)
    times = []
    for i in range(total):
        a, b = MEL_PER_STEP * i, MEL_PER_STEP * (i + 1)
        if i == args.warmup:
            before = phase_sum(encs)
        t0 = time.perf_counter()
        for z in range(n_streams):
            assert encs[z].encode_new(mel[z, :b], a, b) == 0
        if i >= args.warmup:
            times.append(time.perf_counter() - t0)
    after = phase_sum(encs)
    phases = {k: after[k] - before[k] for k in after}
    value = n_streams * AUDIO_S_PER_STEP * len(times) / sum(times)
    cores = oracle.num_cpus()
    sample = (f"{n_streams} streams x 1 chunk per step (steps {args.warmup}..{total - 1} of the streams), "
              "oracle StreamingEncoder per stream with the reference's threading, AVX2 lanes and GEMM dispatch")
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * sum(times) / len(times),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8+f32",
            "data": "synthetic", "config": {"workload": WORKLOAD, "streams_per_step": n_streams,
                                            "chunk_ms": 560, "layers": N_LAYERS},
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample,
                             "phases_s": phases},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------ GPU path ---
class _DevArray:
    """A device pointer viewed as a torch tensor (no copy)."""

    def __init__(self, ptr, shape):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": "<f4", "data": (ptr, False),
                                         "version": 3, "strides": None}


def time_steps(fn, steps, warmup, world, dev, stream):
    import torch
    import torch.distributed as dist

    for _ in range(warmup):
        fn()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        fn()
    e1.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms = reduce_max(e0.elapsed_time(e1), dev)
    return ms / steps


def step_halves(streams, frames=7):
    """Frames per GEMM of the encoder step's sub-batches: the encoder runs
    two halves of the streams in flight, split where the 128-frame tiles of
    its GEMM inputs split (sc_stream_encoder_set_concurrency)."""
    unit = 128 // math.gcd(frames, 128)
    z0 = (streams // 2) // unit * unit
    return [z0 * frames, (streams - z0) * frames] if 0 < z0 < streams else [streams * frames]


def tc_roofline(m, streams, dev, stream):
    """The tcgen05 int8 GEMM at the encoder step's shapes over the 24
    layers' own Q8_0 weights, in the step's order, with the step's two
    sub-batches (halves of the streams, 896 frames each at 256 streams) in
    flight on two CUDA streams as the encoder runs them.  The GEMM kernel's
    time is (quantise + GEMM) minus quantise, each timed with CUDA events
    over the same sequence."""
    import torch

    from stealcode_b200 import _lib
    from stealcode_b200._lib import SC_LAYOUT_TIME_MAJOR, check
    from stealcode_b200.ops import Q8Mat

    lib = _lib.lib
    T = {t.name: t for t in m.tensors}
    # the step's linears in its order; q, k and v run as one fused GEMM
    names = ["feed_forward1.linear1", "feed_forward1.linear2", ("self_attn.linear_q", "self_attn.linear_k",
             "self_attn.linear_v"), "self_attn.linear_out", "conv.pointwise_conv1", "conv.pointwise_conv2",
             "feed_forward2.linear1", "feed_forward2.linear2"]
    halves = step_halves(streams)
    side = torch.cuda.Stream(device=dev)
    sts = [stream, side][:len(halves)]
    mats = []
    for li in range(m.config.n_layers):
        for nm in names:
            parts = [T[f"encoder.layers.{li}.{x}.weight"] for x in (nm if isinstance(nm, tuple) else (nm,))]
            blocks = np.concatenate([w.data for w in parts], axis=0)
            rows, k = blocks.shape[0], int(parts[0].dims[0])
            mats.append((Q8Mat(blocks, rows, k), rows, k))
    ks = sorted({k for _, _, k in mats})
    # per half its own inputs, outputs, workspace and codes (the halves run at once)
    bufs = []
    for t in halves:
        ws_bytes = max(mt.workspace_bytes(t) for mt, _, _ in mats)
        bufs.append({"x": {k: torch.randn(t, k, device=dev) for k in ks},
                     "y": {r: torch.empty(t, r, device=dev) for r in sorted({r for _, r, _ in mats})},
                     "ws": torch.empty(ws_bytes, dtype=torch.uint8, device=dev), "ws_bytes": ws_bytes,
                     "q": {k: (torch.empty(t, k, dtype=torch.int8, device=dev), torch.empty(k // 32, t, device=dev))
                           for k in ks}})

    def gemms():
        for mt, rows, k in mats:
            for t, b, st in zip(halves, bufs, sts):
                check(lib.sc_q8_gemm(mt.handle, b["x"][k].data_ptr(), t, SC_LAYOUT_TIME_MAJOR, 0, None,
                                     b["y"][rows].data_ptr(), SC_LAYOUT_TIME_MAJOR, 0, b["ws"].data_ptr(),
                                     b["ws_bytes"], st.cuda_stream))

    def quants():
        for mt, rows, k in mats:
            for t, b, st in zip(halves, bufs, sts):
                q, d = b["q"][k]
                check(lib.sc_q8_quantize(b["x"][k].data_ptr(), t, k, SC_LAYOUT_TIME_MAJOR, 0, q.data_ptr(),
                                         d.data_ptr(), st.cuda_stream))

    def timed(fn, reps=3):
        fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for st in sts[1:]:
            st.wait_event(e0)
        for _ in range(reps):
            fn()
        for st in sts[1:]:
            ev = torch.cuda.Event()
            ev.record(st)
            stream.wait_event(ev)
        e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / reps

    ms_all = timed(gemms)
    ms_q = timed(quants)
    ms_tc = ms_all - ms_q
    ops = sum(2.0 * t * rows * k for t in halves for _, rows, k in mats)
    p = peaks()
    bf16 = p.get("bf16_tflops")
    # the MMAs run kind::f16 on the int8 codes held as f16 (exact), so the
    # tensor roofline is the dense f16 / bf16 rate
    peak = bf16 if bf16 else 1590.0
    achieved = ops / (ms_tc * 1e-3) / 1e12
    n = len(mats) * len(halves)
    # The exact per-block scaling drains every 32-deep block of every output
    # from TMEM through 3 f32 operations (s = dw*dx, p = s*dot, acc += p):
    # at 128 f32 operations per SM per clock that is the kernel's issue floor.
    blocks = sum(t * rows * (k // 32) for t in halves for _, rows, k in mats)
    clk_ghz = float(p.get("sm_max_mhz") or 1965.0) / 1e3
    drain_floor_ms = 3.0 * blocks / (148 * 128 * clk_ghz * 1e9) * 1e3
    del mats, bufs
    return {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
            "frac_of_nominal_2250": achieved / 2250.0,
            "peak_source": ("measured dense bf16 TFLOP/s (the kind::f16 rate)" if bf16 else "fallback bf16"),
            "kernel": "q8_gemm_tc_kernel (tcgen05 kind::f16, int8 codes held as f16, exact per-block f32 drain)",
            "traffic": None, "frames": halves, "launches": n, "us_per_launch": 1e3 * ms_tc / n,
            "ops_per_launch": ops / n,
            "note": "the step's sub-batches in flight on two streams: us_per_launch is step GEMM time / launches",
            "drain_issue": {"element_blocks_per_step": blocks, "ops_per_element_block": 3,
                            "floor_ms_per_step": drain_floor_ms, "measured_ms_per_step": ms_tc,
                            "frac": drain_floor_ms / ms_tc,
                            "basis": f"148 SMs x 128 f32 ops per clock at {clk_ghz:.3f} GHz"},
            "linear_incl_quantize": {"tflops": ops / (ms_all * 1e-3) / 1e12, "us_per_launch": 1e3 * ms_all / n}}


def gemm_sweep(args, dev, world, stream):
    """The Q8_0 GEMM shape sweep of one layer (M = 1, 8, 32, 128) over 24
    weight copies, graph-captured: whole-sweep GB/s and the weight-streaming
    kernel's HBM roofline per M."""
    import torch

    from stealcode_b200 import _lib, synth
    from stealcode_b200._lib import SC_LAYOUT_TIME_MAJOR, check
    from stealcode_b200.ops import Q8Mat

    lib = _lib.lib

    def gemm_bytes(m, k, n):
        return n * k * 34 // 32 + 4 * m * k + 4 * m * n

    def kernel_bytes(m, k, n):
        return n * k * 34 // 32 + m * k + 4 * m * (k // 32) + 4 * m * n

    wh = {name: synth.q8_weights(synth.SEED_BASE + 1 + i, n, k) for i, (name, k, n) in enumerate(SHAPES)}
    mats = [{name: Q8Mat(wh[name], n, k) for name, k, n in SHAPES} for _ in range(SWEEP_LAYERS)]
    xs = {(m, k): torch.from_numpy(synth.normal(synth.SEED_BASE + 100 + m + k, (m, k))).to(dev)
          for m in MS for k in (1024, 4096)}
    ys = {(m, n): torch.empty((m, n), dtype=torch.float32, device=dev) for m in MS for n in (1024, 3072, 4096)}
    ws_bytes = int(lib.sc_q8_gemm_workspace_bytes(max(MS), 4096))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    xq = {}
    for m in MS:
        for k in (1024, 4096):
            q = torch.zeros((m, k), dtype=torch.int8, device=dev)
            d = torch.zeros((k // 32, m), dtype=torch.float32, device=dev)
            check(lib.sc_q8_quantize(xs[(m, k)].data_ptr(), m, k, SC_LAYOUT_TIME_MAJOR, 0, q.data_ptr(),
                                     d.data_ptr(), torch.cuda.current_stream().cuda_stream))
            xq[(m, k)] = (q, d)
    torch.cuda.synchronize()

    def calls(sp, kernel_only=False, only_m=None):
        n = 0
        for m in MS if only_m is None else [only_m]:
            for layer in mats:
                for name, k, nn in SHAPES:
                    y = ys[(m, nn)]
                    if kernel_only:
                        q, d = xq[(m, k)]
                        check(lib.sc_q8_gemm_q(layer[name].handle, q.data_ptr(), d.data_ptr(), m, m, None,
                                               y.data_ptr(), SC_LAYOUT_TIME_MAJOR, 0, sp))
                    else:
                        check(lib.sc_q8_gemm(layer[name].handle, xs[(m, k)].data_ptr(), m, SC_LAYOUT_TIME_MAJOR,
                                             0, None, y.data_ptr(), SC_LAYOUT_TIME_MAJOR, 0, ws.data_ptr(),
                                             ws_bytes, sp))
                    n += 1
        return n

    def capture(**kw):
        s = torch.cuda.Stream(device=dev)
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            calls(s.cuda_stream, **kw)  # sets kernel attributes outside capture
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            n = calls(torch.cuda.current_stream().cuda_stream, **kw)
        return g, n

    def time_graph(g, steps):
        g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            g.replay()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / steps

    reps = 10
    g, n_launch = capture()
    ms = time_graph(g, reps)
    step_bytes = sum(gemm_bytes(m, k, n) for m in MS for _ in range(SWEEP_LAYERS) for _, k, n in SHAPES)
    del g
    p = peaks()
    peak = p.get("hbm_gbs", 6650.0)
    by_m = {}
    for m in MS:
        g_m, n_m = capture(kernel_only=True, only_m=m)
        ms_m = time_graph(g_m, reps)
        b_m = sum(kernel_bytes(m, k, n) for _, k, n in SHAPES) * SWEEP_LAYERS
        by_m[str(m)] = {"us_per_launch": 1e3 * ms_m / n_m, "gbs": b_m / (ms_m * 1e-3) / 1e9,
                        "frac": b_m / (ms_m * 1e-3) / 1e9 / peak}
        del g_m
    g_k, n_k = capture(kernel_only=True)
    ms_k = time_graph(g_k, reps)
    kb = sum(kernel_bytes(m, k, n) for m in MS for _ in range(SWEEP_LAYERS) for _, k, n in SHAPES)
    del g_k
    achieved = kb / (ms_k * 1e-3) / 1e9
    # the single streaming chunk (M 8, K 1024, N 4096) on its own, over 64
    # weight copies (285 MB, larger than L2), through sc_q8_gemm (the
    # streaming kernel quantises the activations itself)
    c0 = [Q8Mat(wh["ffn_up"], 4096, 1024) for _ in range(64)]
    x0, y0 = xs[(8, 1024)], ys[(8, 4096)]

    def calls0(sp):
        for mt in c0:
            check(lib.sc_q8_gemm(mt.handle, x0.data_ptr(), 8, SC_LAYOUT_TIME_MAJOR, 0, None, y0.data_ptr(),
                                 SC_LAYOUT_TIME_MAJOR, 0, ws.data_ptr(), ws_bytes, sp))
        return len(c0)

    s0 = torch.cuda.Stream(device=dev)
    s0.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s0):
        calls0(s0.cuda_stream)
    torch.cuda.current_stream().wait_stream(s0)
    torch.cuda.synchronize()
    g0 = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g0):
        n0 = calls0(torch.cuda.current_stream().cuda_stream)
    ms0 = time_graph(g0, reps)
    del g0
    b0 = gemm_bytes(8, 1024, 4096)
    config0 = {"workload": "q8_gemm M=8 K=1024 N=4096 (one streaming chunk), 64 weight copies in a graph",
               "us_per_gemm": 1e3 * ms0 / n0, "bytes_per_gemm": b0, "gbs": b0 * n0 / (ms0 * 1e-3) / 1e9,
               "frac": b0 * n0 / (ms0 * 1e-3) / 1e9 / peak, "peak_source": "measured" if "hbm_gbs" in p else "fallback"}
    # the same sweep per M in batched calls (sc_q8_gemm_batch: every GEMM of
    # the 24 layer copies in one streaming pass, quantisation included)
    from stealcode_b200.ops import q8_gemm_batch

    batched = {}
    flat = [(layer[name], k, n) for layer in mats for name, k, n in SHAPES]
    bws_n = len(flat)
    hw = (ctypes.c_void_p * bws_n)(*[mt.handle.value for mt, _, _ in flat])
    bws_bytes = int(lib.sc_q8_gemm_batch_workspace_bytes(hw, bws_n))
    bws = torch.empty(bws_bytes, dtype=torch.uint8, device=dev)
    for m in (1, 8):
        xb = [xs[(m, k)] for _, k, _ in flat]
        yb = [ys[(m, n)] for _, _, n in flat]

        def callb():
            q8_gemm_batch([mt for mt, _, _ in flat], xb, outs=yb, workspace=bws)
            return 2

        sb = torch.cuda.Stream(device=dev)
        sb.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(sb):
            callb()
        torch.cuda.current_stream().wait_stream(sb)
        torch.cuda.synchronize()
        gb_ = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gb_):
            callb()
        ms_b = time_graph(gb_, reps)
        del gb_
        bb = sum(gemm_bytes(m, k, n) for _, k, n in flat)
        batched[str(m)] = {"ms_per_sweep": ms_b, "gbs": bb / (ms_b * 1e-3) / 1e9,
                           "frac": bb / (ms_b * 1e-3) / 1e9 / peak, "gemms_per_call": bws_n, "launches": 2}
    del bws
    # config 0 the batched way: the 64 single-chunk GEMMs (M 8, K 1024,
    # N 4096, own weights and outputs) as one sc_q8_gemm_batch call
    h0 = (ctypes.c_void_p * len(c0))(*[mt.handle.value for mt in c0])
    ws0 = torch.empty(int(lib.sc_q8_gemm_batch_workspace_bytes(h0, len(c0))), dtype=torch.uint8, device=dev)
    y0s = [torch.empty((8, 4096), dtype=torch.float32, device=dev) for _ in c0]

    def call0b():
        q8_gemm_batch(c0, [x0] * len(c0), outs=y0s, workspace=ws0)

    s0b = torch.cuda.Stream(device=dev)
    s0b.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s0b):
        call0b()
    torch.cuda.current_stream().wait_stream(s0b)
    torch.cuda.synchronize()
    g0b = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g0b):
        call0b()
    ms0b = time_graph(g0b, reps)
    del g0b, c0, ws0, y0s
    config0["batched"] = {"api": "sc_q8_gemm_batch, the 64 GEMMs in one call", "us_per_gemm": 1e3 * ms0b / n0,
                          "gbs": b0 * n0 / (ms0b * 1e-3) / 1e9, "frac": b0 * n0 / (ms0b * 1e-3) / 1e9 / peak}
    return {"metric": "Q8_0 GEMM HBM GB/s (FastConformer layer shape sweep)", "value": step_bytes / (ms * 1e-3) / 1e9,
            "unit": "GB/s", "shapes": SHAPES, "m": MS, "weight_copies": SWEEP_LAYERS, "ms_per_sweep": ms,
            "launches_per_sweep": n_launch,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_source": "measured" if "hbm_gbs" in p else "fallback",
                         "frac_of_spec_8000_gbs": achieved / 8000.0,
                         "kernel": "q8_gemm_stream_kernel", "bytes_per_launch_avg": kb / n_k,
                         "us_per_launch_avg": 1e3 * ms_k / n_k, "traffic": None, "by_m": by_m},
            "config0": config0, "batched": batched}


def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    from stealcode_b200 import _lib
    from stealcode_b200.ops import StreamEncoder

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    stream = torch.cuda.Stream(device=dev)
    Z = args.streams
    m = encoder_model()
    cfg = m.config
    enc = StreamEncoder(m, Z)
    if args.no_graphs:
        enc.set_graphs(False)
    gen = torch.Generator(device=dev)
    gen.manual_seed(MODEL_SEED + 7 + rank)
    pool = [torch.randn((Z, MEL_PER_STEP, cfg.feat_in), device=dev, generator=gen) for _ in range(MEL_POOL)]
    state = {"i": 0}

    def step():
        i = state["i"]
        enc.encode_new(pool[i % MEL_POOL], MEL_PER_STEP * i, MEL_PER_STEP * (i + 1), stream=stream)
        state["i"] = i + 1

    with torch.cuda.stream(stream):
        for _ in range(PRIME_STEPS):
            step()
    torch.cuda.synchronize()

    clocks = ClockSampler(local_rank)
    clocks.start()
    time.sleep(0.3)  # the sampler's first reading lands inside the timed region
    n0 = _lib.launch_count()
    ms_step = time_steps(step, args.steps, args.warmup, world, dev, stream)
    launches = _lib.launch_count() - n0
    clk = clocks.stop()
    launches_timed = launches * args.steps // (args.steps + args.warmup)
    value = world * Z * AUDIO_S_PER_STEP / (ms_step * 1e-3)
    g_on, g_cap, g_launch = enc.graph_stats()
    graphs = {"on": g_on, "captured": g_cap, "graph_launches": g_launch,
              "note": "steady steps replay a CUDA graph of the whole step (both sub-batches) after a one-thread "
                      "store of the frame shift; the warm-up captures them"}

    # e2e through the C ABI with host buffers: mel in, output frames out
    rows = Z * 7
    h_mel = [torch.empty((Z, MEL_PER_STEP, cfg.feat_in), dtype=torch.float32).pin_memory() for _ in range(2)]
    for h, p in zip(h_mel, pool):
        h.copy_(p.cpu())
    d_mel = torch.empty((Z, MEL_PER_STEP, cfg.feat_in), device=dev)
    h_out = torch.empty((rows, cfg.d_model), dtype=torch.float32).pin_memory()
    h_out_full = torch.empty((Z * cfg.max_frames, cfg.d_model), dtype=torch.float32).pin_memory()

    def e2e_step_host():
        # sc_stream_encoder_encode_new_host: each half of the streams is
        # copied in, encoded and copied out on its own CUDA stream
        i = state["i"]
        r = enc.encode_new_host_ptr(h_mel[i % 2].data_ptr(), MEL_PER_STEP * i, MEL_PER_STEP * (i + 1), False,
                                    h_out_full.data_ptr(), stream=stream)
        state["i"] = i + 1
        assert r == rows

    def e2e_step_dev():
        i = state["i"]
        with torch.cuda.stream(stream):
            d_mel.copy_(h_mel[i % 2], non_blocking=True)
            enc.encode_new(d_mel, MEL_PER_STEP * i, MEL_PER_STEP * (i + 1), stream=stream)
            ptr, r, d = enc.output()
            out = torch.as_tensor(_DevArray(ptr, (r, d)), device=dev)
            h_out.copy_(out, non_blocking=True)
        stream.synchronize()
        state["i"] = i + 1

    e2e_step, api = e2e_step_host, ("sc_stream_encoder_encode_new_host: pinned host mel in / frames out, each "
                                     "half of the streams copied in, encoded and copied out on its own CUDA "
                                     "stream, synchronous every step")
    try:
        e2e_step()
    except Exception as exc:  # measure through the device-pointer entry point instead
        print(f"e2e: host entry point failed ({exc}); timing the device-pointer path", file=sys.stderr)
        e2e_step, api = e2e_step_dev, ("sc_stream_encoder_encode_new + sc_stream_encoder_output, pinned host mel "
                                       "in / frames out, synchronised every step")
        e2e_step()
    # the same warm-up as the device-timed steps: the host entry's step
    # geometry differs from the device entry's, so its step graphs are
    # captured here, outside the timed steps
    for _ in range(max(args.warmup, 3)):
        e2e_step()
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(args.e2e_steps):
        e2e_step()
    e2e_s = reduce_max((time.perf_counter() - t0) / args.e2e_steps, dev)
    e2e = {"value": world * Z * AUDIO_S_PER_STEP / e2e_s, "unit": UNIT,
           "h2d_bytes_per_step": Z * MEL_PER_STEP * cfg.feat_in * 4, "d2h_bytes_per_step": rows * cfg.d_model * 4,
           "api": api}
    trans = None if args.no_decoder else transcriber_leg(args, enc, pool, state, Z, world, dev, stream)
    enc.close()
    del pool, enc
    torch.cuda.empty_cache()

    prefill = None if args.no_prefill else prefill_leg(m, world, dev, stream)
    box = box_leg(args, m, world, rank, dev, stream) if args.box_streams > 0 else None
    roof = tc_roofline(m, Z, dev, stream)
    sweep = None if args.no_sweep else gemm_sweep(args, dev, world, stream)
    if world > 1:
        dist.barrier()

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        import oracle

        v, dt, audio, steps, phases = cpu_encoder_sample(m, 4, 8, budget_s=15.0)
        cpu = {"value": v, "unit": UNIT, "cores": oracle.num_cpus(), "kind": "port",
               "sample": f"4 streams x {steps} chunks from t=0 ({audio:.2f} audio s in {dt:.1f} s), oracle "
                         "StreamingEncoder per stream with the reference's threading, AVX2 lanes and GEMM "
                         "dispatch", "phases_s": phases, "gemm": cpu_gemm_sample()}
    if rank == 0:
        p = peaks()
        line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "int8+f32", "data": "synthetic",
                "config": {"workload": WORKLOAD, "encoder": "random-init FastConformer, 24 layers, d 1024, "
                                                            "8 heads, FFN 4096, conv 9, Q8_0 linears",
                           "streams_per_gpu": Z, "global_streams": Z * world, "chunk_ms": 560,
                           "frames_per_step": 7, "left_context_frames": 70, "prime_steps": PRIME_STEPS,
                           "frames_per_gemm": step_halves(Z), "sub_batches": len(step_halves(Z)),
                           "step_graphs": graphs,
                           "parallelism": f"streams sharded, {world} independent ranks",
                           "l2": "inputs larger than L2: each step streams the 24 layers' f16 weight tiles, 1.1 GB (587 MB as Q8_0), L2 126 MB"},
                "realtime_streams_per_gpu": value / world,
                "roofline": roof, "gemm_sweep": sweep, "cpu_baseline": cpu, "e2e": e2e, "transcriber": trans, "prefill": prefill, "box_scale": box,
                "gpu_launches": launches_timed, "launches_per_step": launches / (args.steps + args.warmup),
                "clocks": clk, "peaks_file": {k: p.get(k) for k in ("hbm_gbs", "bf16_tflops")}}
        print(json.dumps(line), flush=True)


PREFILL_STREAMS = 64
PREFILL_MEL = 6000          # 60 s of 10 ms mel frames -> 750 encoder frames
PREFILL_CALL_MEL = 448      # 56 encoder frames per encode_new call


def prefill_leg(m, world, dev, stream):
    """A 750-frame (60 s) per-stream prefill at batch 64: the device encoder
    fed 448 mel frames (56 encoder frames) per encode_new call, so the
    GEMMs run at M = 64 * 56; the first prefill (on a separate encoder)
    warms the kernels, a fresh encoder is timed."""
    import torch

    from stealcode_b200 import model
    from stealcode_b200.ops import StreamEncoder

    cfg = model.EncoderConfig(**{**m.config.__dict__, "max_frames": PREFILL_CALL_MEL // 8})
    pm = model.Model(cfg, m.tensors)
    Z = PREFILL_STREAMS
    gen = torch.Generator(device=dev)
    gen.manual_seed(MODEL_SEED + 11)
    mel = torch.randn((Z, PREFILL_MEL, cfg.feat_in), device=dev, generator=gen)
    calls = [(a, min(a + PREFILL_CALL_MEL, PREFILL_MEL)) for a in range(0, PREFILL_MEL, PREFILL_CALL_MEL)]
    chunks = [mel[:, a:b].contiguous() for a, b in calls]

    def run(enc):
        for (a, b), x in zip(calls, chunks):
            enc.encode_new(x, a, b, stream=stream)

    warm = StreamEncoder(pm, Z)
    with torch.cuda.stream(stream):
        run(warm)
    torch.cuda.synchronize()
    warm.close()
    enc = StreamEncoder(pm, Z)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        run(enc)
        e1.record(stream)
    torch.cuda.synchronize()
    frames = enc.total()
    enc.close()
    del chunks, mel
    torch.cuda.empty_cache()
    ms = reduce_max(e0.elapsed_time(e1), dev)
    audio = Z * PREFILL_MEL * 0.01
    return {"value": world * audio / (ms * 1e-3), "unit": UNIT, "ms": ms, "streams_per_gpu": Z,
            "frames_per_stream": frames, "calls": len(calls), "frames_per_call": PREFILL_CALL_MEL // 8,
            "frames_per_gemm": step_halves(Z, PREFILL_CALL_MEL // 8),
            "note": "same encoder and bits as streaming; long calls, attention run chunk by chunk inside a call"}


def box_leg(args, m, world, rank, dev, stream):
    """The box-scale streaming batch: `--box-streams` concurrent streams (8192)
    sharded by stream over the ranks, each rank's shard in one encoder (its
    two halves in flight), no collective on the data path.  A rank whose
    shard does not fit in device memory halves it until it does (the line
    reports the streams actually resident).  Steady state after the priming
    steps; value = resident streams x 0.56 s / max-over-ranks step time."""
    import torch
    import torch.distributed as dist

    from stealcode_b200 import _lib
    from stealcode_b200.ops import StreamEncoder

    lo, hi = stream_shard(args.box_streams, world, rank)
    want = hi - lo
    Z, enc = want, None
    free0, total = torch.cuda.mem_get_info(dev)
    while Z > 0 and enc is None:
        try:
            enc = StreamEncoder(m, Z)
        except _lib.ScError as exc:
            if exc.code != _lib.SC_ERR_ALLOC:
                raise
            Z = Z // 2 // 128 * 128 if Z > 256 else Z // 2
    used = free0 - torch.cuda.mem_get_info(dev)[0]
    cfg = m.config
    gen = torch.Generator(device=dev)
    gen.manual_seed(MODEL_SEED + 13 + rank)
    pool = [torch.randn((Z, MEL_PER_STEP, cfg.feat_in), device=dev, generator=gen) for _ in range(2)]
    state = {"i": 0}

    def step():
        i = state["i"]
        enc.encode_new(pool[i % 2], MEL_PER_STEP * i, MEL_PER_STEP * (i + 1), stream=stream)
        state["i"] = i + 1

    with torch.cuda.stream(stream):
        for _ in range(PRIME_STEPS):
            step()
    torch.cuda.synchronize()
    n0 = _lib.launch_count()
    # two warm-up steps: the first steady steps capture the step graphs (one
    # per mel-history buffer), so the timed steps all replay
    ms = time_steps(step, args.box_steps, 2, world, dev, stream)
    launches = (_lib.launch_count() - n0) / (args.box_steps + 2)
    enc.close()
    del pool, enc
    torch.cuda.empty_cache()
    resident = Z
    if world > 1:
        t = torch.tensor([Z], dtype=torch.float64, device=dev)
        dist.all_reduce(t)
        resident = int(t.item())
    return {"value": resident * AUDIO_S_PER_STEP / (ms * 1e-3), "unit": UNIT, "ms_per_step": ms,
            "global_streams_requested": args.box_streams, "global_streams_resident": resident,
            "streams_per_gpu": Z, "requested_per_gpu": want, "frames_per_gemm": step_halves(Z),
            "device_bytes_used": used, "device_bytes_total": total, "steps": args.box_steps,
            "prime_steps": PRIME_STEPS, "launches_per_step": launches,
            "realtime_streams_per_gpu": resident * AUDIO_S_PER_STEP / (ms * 1e-3) / world,
            "note": "the headline encoder, 8192 streams sharded by stream over the GPUs (no collective)"}


def transcriber_leg(args, enc, pool, state, Z, world, dev, stream):
    """LiveTranscriber::process for every stream (live.rs:336-375):
    encode_new of the step's 56 mel frames, then decode_frames over the 7 new
    encoder frames of each stream, read from the encoder's device output."""
    import torch

    from stealcode_b200 import model
    from stealcode_b200.ops import RnntDecoder

    dcfg = model.RnntConfig()
    # blank bias 0.9: about 0.5 tokens per frame on this encoder's output
    # frames (a speech-like rate; 80 ms frames)
    dec = RnntDecoder(model.random_decoder(dcfg, blank_bias=DECODER_BLANK_BIAS), Z, max_frames=8)
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    emitted = torch.zeros(Z, dtype=torch.int64)

    def one(e=None):
        i = state["i"]
        if e:
            e[0].record(stream)
        enc.encode_new(pool[i % MEL_POOL], MEL_PER_STEP * i, MEL_PER_STEP * (i + 1), stream=stream)
        if e:
            e[1].record(stream)
        ptr, r, _ = enc.output()
        dec.decode_frames((ptr, r // Z), stream=stream)
        if e:
            e[2].record(stream)
        state["i"] = i + 1

    for _ in range(args.warmup):
        one()
    frames = 0
    for k in range(args.steps):
        one(ev[k])
        emitted += torch.as_tensor(dec.emitted())
        frames += 7 * Z
    torch.cuda.synchronize()
    enc_ms = sum(e[0].elapsed_time(e[1]) for e in ev) / args.steps
    dec_ms = sum(e[1].elapsed_time(e[2]) for e in ev) / args.steps
    step_ms = reduce_max(enc_ms + dec_ms, dev)
    dec.close()
    return {"value": world * Z * AUDIO_S_PER_STEP / (step_ms * 1e-3), "unit": UNIT, "ms_per_step": step_ms,
            "encoder_ms_per_step": enc_ms, "decoder_ms_per_step": dec_ms,
            "tokens_per_frame": float(emitted.sum()) / frames, "steps": args.steps,
            "decoder": f"random-init RNN-T: {dcfg.n_layers} x {dcfg.hidden} LSTM, joint {dcfg.joint}, "
                       f"{dcfg.vocab} classes, greedy, max_symbols {dcfg.max_symbols}; per-stream state carried",
            "api": "sc_stream_encoder_encode_new, then sc_rnnt_decode_frames on sc_stream_encoder_output"}


def run_profile(args):
    """A few eager launches of one kernel family on a small case, for ncu."""
    import math

    import torch

    from stealcode_b200 import synth
    from stealcode_b200.ops import SC_LAYOUT_TIME_MAJOR, Q8Mat, StreamEncoder, attn_stream_ring

    dev = torch.device("cuda", 0)
    if args.profile in ("gemm", "tc"):
        for i, (name, k, n) in enumerate(SHAPES):
            mat = Q8Mat(synth.q8_weights(synth.SEED_BASE + 1 + i, n, k), n, k)
            for m in ((8, 128) if args.profile == "gemm" else (1792,)):
                x = torch.from_numpy(synth.normal(synth.SEED_BASE + 100 + m + k, (m, k))).to(dev)
                for _ in range(3):
                    mat.gemm(x, x_layout=SC_LAYOUT_TIME_MAJOR, y_layout=SC_LAYOUT_TIME_MAJOR)
    elif args.profile == "attn":
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
    elif args.profile == "batch":
        # one sc_q8_gemm_batch call over the layer sweep's 96 GEMMs (24
        # weight copies of the four shapes, 321 MB), M = 1 then M = 8
        from stealcode_b200.ops import q8_gemm_batch

        wh = {name: synth.q8_weights(synth.SEED_BASE + 1 + i, n, k) for i, (name, k, n) in enumerate(SHAPES)}
        flat = [(Q8Mat(wh[name], n, k), k, n) for _ in range(SWEEP_LAYERS) for name, k, n in SHAPES]
        for m in (1, 8):
            xs = {k: torch.from_numpy(synth.normal(synth.SEED_BASE + 100 + m + k, (m, k))).to(dev)
                  for k in (1024, 4096)}
            ys = [torch.empty((m, n), dtype=torch.float32, device=dev) for _, _, n in flat]
            for _ in range(3):
                q8_gemm_batch([mt for mt, _, _ in flat], [xs[k] for _, k, _ in flat], outs=ys)
    elif args.profile == "breakdown":
        import collections

        from torch.profiler import ProfilerActivity, profile

        m = encoder_model()
        enc = StreamEncoder(m, args.streams)
        enc.set_concurrency(1)  # kernels one after another: durations add up to the step
        mel = torch.randn((args.streams, MEL_PER_STEP, m.config.feat_in), device=dev)
        for i in range(PRIME_STEPS + 2):
            enc.encode_new(mel, MEL_PER_STEP * i, MEL_PER_STEP * (i + 1))
        torch.cuda.synchronize()
        steps = 3
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            for i in range(PRIME_STEPS + 2, PRIME_STEPS + 2 + steps):
                enc.encode_new(mel, MEL_PER_STEP * i, MEL_PER_STEP * (i + 1))
            torch.cuda.synchronize()
        tot, cnt = collections.defaultdict(float), collections.Counter()
        for ev in prof.events():
            if ev.device_type == torch.autograd.DeviceType.CUDA:
                name = ev.name.split("(")[0].replace("void ", "")
                tot[name] += ev.device_time_total
                cnt[name] += 1
        total = sum(tot.values())
        print(f"{args.streams} streams, {N_LAYERS} layers: kernel time per step {total / steps / 1e3:.2f} ms")
        for k, v in sorted(tot.items(), key=lambda x: -x[1]):
            print(f"{k[:56]:56s} launches/step {cnt[k] // steps:4d}  us/step {v / steps:9.1f}  "
                  f"share {100 * v / total:5.1f}%  us/launch {v / cnt[k]:8.2f}")
        enc.close()
    else:
        # the encoder step with 2 layers at the headline's stream count
        from stealcode_b200 import model

        cfg = model.EncoderConfig(n_layers=2)
        m = model.random_model(cfg, seed=MODEL_SEED)
        enc = StreamEncoder(m, args.streams)
        mel = torch.randn((args.streams, MEL_PER_STEP, cfg.feat_in), device=dev)
        for i in range(PRIME_STEPS + 2):
            enc.encode_new(mel, MEL_PER_STEP * i, MEL_PER_STEP * (i + 1))
        enc.close()
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

        # rank 0 prints exactly one line: keep NCCL's version banner off stdout
        if os.environ.get("NCCL_DEBUG", "").upper() in ("", "VERSION"):
            os.environ["NCCL_DEBUG"] = "WARN"
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
    try:
        run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
