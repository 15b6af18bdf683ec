"""Writes tests/golden/golden.npz: the oracle's outputs on the inputs of the
reference's own GEMM, quantiser and streaming-attention tests.

The reference (a Rust nightly crate) cannot be built in this image and its
tests store no expected outputs (each compares two in-tree paths), so these
fixtures are the oracle's outputs on the reference tests' generators
(tests/refcases.py), frozen: tests/test_golden.py checks that the oracle
still reproduces them bit for bit, tests/test_golden_gpu.py checks the CUDA
path against them.

    python tests/golden/make_golden.py

Cases (reference paths relative to crates/audio_engine/src/):
- pattern_<m>_<k>_<n>[_simd]: run_case's integer-pattern Q8_0 GEMM
  (sgemm_kernel.rs:223-270, simd_kernel.rs:1325-1383) through
  q8_gemm_scalar and through the SIMD kernel's accumulation order;
- mid_128_1024_40, tc_128_1024_136: the same generator at 40 and 136
  frames (more than 16 frames: the reference runs q8_gemm_scalar);
- wgsl_37_1024_13: q8_gemm_matches_reference's random-u16-scale blocks
  (gpu/kernels.rs:1562-1627) through q8_gemm_scalar;
- quant_2048_16_q / _d: quantize_col over the 2048 x 16 pattern activations;
- attn_ref: attn_stream_matches_reference's case (gpu/kernels.rs:1878-1988)
  through the CPU attention of block_new (streaming.rs:492-589).
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

import oracle  # noqa: E402
from tests import refcases  # noqa: E402

ATTN_KEYS = ("q", "kv", "vv", "pos_p", "q_bias", "v_bias", "c", "d", "n_heads", "scale", "s", "k_lo", "band",
             "chunk", "left_chunks", "k_hi", "pos_off")
MID_CASES = [(128, 1024, 40), (128, 1024, 136)]


def pattern_cases():
    return sorted(set(refcases.VNNI_CASES + refcases.SIMD_CASES))


def compute() -> dict:
    out = {}
    for m, k, n in pattern_cases():
        w, pr, x = refcases.gemm_pattern_case(m, k, n)
        out[f"pattern_{m}_{k}_{n}"] = oracle.q8_gemm_scalar(m, k, n, w, pr, 34, 2, x)
        out[f"pattern_{m}_{k}_{n}_simd"] = oracle.q8_gemm_simd_order(m, k, n, w, pr, 34, 2, x)
    for (m, k, n), name in zip(MID_CASES, ("mid", "tc")):
        w, pr, x = refcases.gemm_pattern_case(m, k, n)
        out[f"{name}_{m}_{k}_{n}"] = oracle.q8_gemm_scalar(m, k, n, w, pr, 34, 2, x)
    raw, t, k, n, x_tk = refcases.wgsl_gemm_case()
    out[f"wgsl_{n}_{k}_{t}"] = oracle.q8_gemm_scalar(n, k, t, raw, (k // 32) * 34, 34, 2,
                                                     np.ascontiguousarray(x_tk.T))
    _, _, x = refcases.gemm_pattern_case(8, 2048, 16)
    q, d = oracle.quantize(x)
    out["quant_2048_16_q"], out["quant_2048_16_d"] = q, d
    cs = refcases.attn_case()
    out["attn_ref"] = oracle.attn_stream(*[cs[a] for a in ATTN_KEYS])
    return {key: np.ascontiguousarray(v) for key, v in out.items()}


def main():
    np.savez_compressed(os.path.join(HERE, "golden.npz"), **compute())


if __name__ == "__main__":
    main()
