"""Input generators of the reference's own tests, restated in numpy.

Each generator reproduces the inputs of one reference test bit for bit, so
the CUDA kernels are checked on the same cases the reference checks its own
kernels on.  Paths are relative to crates/audio_engine/src/.
"""
from __future__ import annotations

import math

import numpy as np

MASK64 = (1 << 64) - 1


class XorShift:
    """The xorshift64 closure of the reference GPU tests (gpu/kernels.rs:1566-1577)."""

    def __init__(self, seed: int):
        self.s = seed & MASK64

    def next(self) -> int:
        s = self.s
        s ^= (s << 13) & MASK64
        s ^= s >> 7
        s ^= (s << 17) & MASK64
        self.s = s
        return s

    def f32(self) -> np.float32:
        # (seed >> 33) as f32 / u32::MAX as f32 * 2.0 - 1.0, all in f32
        a = np.float32(self.next() >> 33)
        b = np.float32(4294967295.0)
        return np.float32(np.float32(np.float32(a / b) * np.float32(2.0)) - np.float32(1.0))

    def u16(self) -> int:
        return self.next() >> 48


def half_f32_to_u16(v: float) -> int:
    """sgemm_kernel.rs:209-221 (truncating f32 -> f16 bits)."""
    bits = int(np.array([v], dtype=np.float32).view(np.uint32)[0])
    sign = (bits >> 16) & 0x8000
    exp = ((bits >> 23) & 0xFF) - 127 + 15
    mant = (bits >> 13) & 0x3FF
    if exp <= 0:
        return sign
    if exp >= 31:
        return sign | 0x7C00
    return sign | (exp << 10) | mant


def gemm_pattern_case(m: int, k: int, n: int):
    """Inputs of run_case (sgemm_kernel.rs:223-247, simd_kernel.rs:1325-1344):
    integer-pattern Q8 blocks and x = ((i*3) % 101)/17 - 1 in feature-major [k, n].
    Returns (w bytes [m, padded_row], padded_row, x [k, n])."""
    nb = (k + 31) // 32
    padded_row = nb * 34
    w = np.zeros((m, padded_row), dtype=np.uint8)
    s_even = half_f32_to_u16(0.0125)
    s_odd = half_f32_to_u16(0.03125)
    i = np.arange(m)[:, None]
    b = np.arange(nb)[None, :]
    sc = np.where((i + b) % 2 == 0, s_even, s_odd).astype(np.uint16)
    blk = w.reshape(m, nb, 34)
    blk[:, :, 0] = (sc & 0xFF).astype(np.uint8)
    blk[:, :, 1] = (sc >> 8).astype(np.uint8)
    j = np.arange(32)[None, None, :]
    blk[:, :, 2:] = ((i[:, :, None] * 31 + b[:, :, None] * 7 + j * 13) % 251).astype(np.uint8)
    idx = np.arange(k * n)
    x = (((idx * 3) % 101).astype(np.float32) / np.float32(17.0) - np.float32(1.0)).astype(np.float32)
    return w, padded_row, x.reshape(k, n)


# (m, k, n) of vnni_matches_scalar (sgemm_kernel.rs:260-270) and
# simd_matches_scalar (simd_kernel.rs:1375-1383).
VNNI_CASES = [(8, 64, 1), (16, 128, 2), (32, 512, 4), (64, 512, 8), (128, 768, 14), (128, 2048, 16),
              (512, 2048, 1), (512, 4352, 16)]
SIMD_CASES = [(8, 64, 1), (16, 128, 4), (64, 512, 8), (128, 2048, 16), (512, 2048, 16)]


def wgsl_gemm_case():
    """Inputs of q8_gemm_matches_reference (gpu/kernels.rs:1562-1590): t=13,
    k=1024, n=37 rows of random-u16-scale blocks, x time-major [t, k].  The
    two closures each copy the seed (Rust `move` of a Copy u64), so the f32
    and u16 streams restart from the same state."""
    seed = 0x9E3779B97F4A7C15
    rf, ru = XorShift(seed), XorShift(seed)
    t, k, n = 13, 1024, 37
    kb = (k + 31) // 32
    raw = np.zeros((n, kb * 34), dtype=np.uint8)
    for r in range(n):
        for b in range(kb):
            base = b * 34
            u = ru.u16()
            raw[r, base] = u & 0xFF
            raw[r, base + 1] = u >> 8
            for i in range(32):
                v = float(np.float32(rf.f32() * np.float32(127.0)))
                raw[r, base + 2 + i] = np.uint8(np.int8(int(v)) if -128 < v < 128 else (127 if v > 0 else -128))
    x = np.array([rf.f32() for _ in range(t * k)], dtype=np.float32).reshape(t, k)
    return raw, t, k, n, x


def attn_case():
    """Inputs of attn_stream_matches_reference (gpu/kernels.rs:1878-1918)."""
    rf = XorShift(0x5150_1503_7265_616D)
    d, n_heads = 1024, 8
    head_dim = d // n_heads
    scale = float(np.float32(1.0) / np.float32(math.sqrt(head_dim)))
    chunk, left_chunks, pos_off = 4, 2, 3
    s, c, k_lo, k_hi = 16, 8, 8, 24
    band = k_hi - k_lo
    n_pos = 2 * chunk * left_chunks + chunk - 1 + 1

    def mk(nv):
        return np.array([rf.f32() for _ in range(nv)], dtype=np.float32)

    q = mk(c * d).reshape(c, d)
    kv = mk(band * d).reshape(band, d)
    vv = mk(band * d).reshape(band, d)
    pos_p = mk(n_pos * d).reshape(n_pos, d)
    q_bias = mk(d)
    v_bias = mk(d)
    return dict(q=q, kv=kv, vv=vv, pos_p=pos_p, q_bias=q_bias, v_bias=v_bias, c=c, d=d, n_heads=n_heads,
                scale=scale, s=s, k_lo=k_lo, band=band, chunk=chunk, left_chunks=left_chunks, k_hi=k_hi,
                pos_off=pos_off)


def score_case(head_dim: int):
    """Inputs of score_run_case (simd_kernel.rs:1500-1519)."""
    i = np.arange(head_dim)
    f = lambda mul, mod, div, off: (((i * mul) % mod).astype(np.float32) / np.float32(div)
                                    - np.float32(off)).astype(np.float32)
    return (f(3, 101, 11, 1.0), f(5, 97, 13, 2.0), f(7, 89, 17, 1.5), f(9, 83, 19, 0.5),
            f(13, 79, 23, 1.0), f(17, 73, 29, 2.0))


def softmax_case(band: int, head_dim: int, n_heads: int):
    """Inputs of softmax_v_run_case (simd_kernel.rs:1537-1556)."""
    k1 = band
    k0 = band // 3
    h = (band // 2) % n_heads
    srow = ((np.arange(k1 * n_heads) * 19 % 71).astype(np.float32) / np.float32(31.0)
            - np.float32(1.0)).astype(np.float32)
    v = ((np.arange(band * head_dim) * 23 % 67).astype(np.float32) / np.float32(37.0)
         - np.float32(0.5)).astype(np.float32).reshape(band, head_dim)
    return srow, k0, k1, h, v
