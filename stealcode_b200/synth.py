"""Seeded synthetic inputs for the hot-path workloads.

Random numbers: a splitmix64 stream (state advanced by 0x9E3779B97F4A7C15 per
draw) turned into normals by Box-Muller, so every consumer (tests, bench,
smoke) regenerates bit-identical inputs from a seed.  Q8_0 weights are drawn
~N(0, 0.02) and quantised per 32-wide block along K into GGUF's 34-byte
``[f16 d][32 x i8]`` blocks (the layout the reference loads as ``Q8F16``,
nemotron/weights.rs:47-62; GGUF dtype 8, gguf.rs:355-356).
"""
from __future__ import annotations

import numpy as np

GAMMA = np.uint64(0x9E3779B97F4A7C15)
_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)

SEED_BASE = 0x5EED0000


def splitmix64(seed: int, n: int, offset: int = 0) -> np.ndarray:
    """The n draws of splitmix64 seeded with `seed`, starting at draw `offset`."""
    with np.errstate(over="ignore"):
        i = np.arange(offset + 1, offset + n + 1, dtype=np.uint64)
        z = np.uint64(seed & 0xFFFFFFFFFFFFFFFF) + i * GAMMA
        z = (z ^ (z >> np.uint64(30))) * _M1
        z = (z ^ (z >> np.uint64(27))) * _M2
        z = z ^ (z >> np.uint64(31))
    return z


def normal(seed: int, shape, std: float = 1.0, mean: float = 0.0) -> np.ndarray:
    """Seeded N(mean, std^2) f32 array of `shape` (Box-Muller on splitmix64)."""
    n = int(np.prod(shape))
    m = (n + 1) // 2
    z = splitmix64(seed, 2 * m)
    u = ((z >> np.uint64(11)).astype(np.float64) + 0.5) * (1.0 / 9007199254740992.0)
    u1, u2 = u[0::2], u[1::2]
    r = np.sqrt(-2.0 * np.log(u1))
    out = np.empty(2 * m, dtype=np.float64)
    out[0::2] = r * np.cos(2.0 * np.pi * u2)
    out[1::2] = r * np.sin(2.0 * np.pi * u2)
    return (out[:n] * std + mean).astype(np.float32).reshape(shape)


def round_half_away(v: np.ndarray) -> np.ndarray:
    return np.sign(v) * np.floor(np.abs(v) + 0.5)


def quantize_q8_0(w: np.ndarray) -> np.ndarray:
    """[rows, k] f32 -> GGUF Q8_0 bytes [rows, ceil(k/32)*34] (f16 scale first).

    Per block: d = amax / 127 (stored as f16), q = round-half-away(w / d)
    saturated to +-127; an all-zero block stores d = 0 and zero quants.  K is
    zero-padded to a multiple of 32, as GGUF pads rows.
    """
    rows, k = w.shape
    nb = (k + 31) // 32
    wp = np.zeros((rows, nb * 32), dtype=np.float32)
    wp[:, :k] = w
    blk = wp.reshape(rows, nb, 32)
    amax = np.abs(blk).max(axis=2)
    d = (amax / np.float32(127.0)).astype(np.float32)
    safe = np.where(d > 0, d, np.float32(1.0))
    inv = np.where(d > 0, np.float32(1.0) / safe, np.float32(0.0)).astype(np.float32)
    q = np.clip(round_half_away(blk * inv[:, :, None]), -127, 127).astype(np.int8)
    out = np.empty((rows, nb, 34), dtype=np.uint8)
    out[:, :, 0:2] = d.astype(np.float16).view(np.uint8).reshape(rows, nb, 2)
    out[:, :, 2:] = q.view(np.uint8)
    return out.reshape(rows, nb * 34)


def q8_weights(seed: int, rows: int, k: int, std: float = 0.02) -> np.ndarray:
    """Seeded ~N(0, std) weights quantised to Q8_0 GGUF bytes [rows, nb*34]."""
    return quantize_q8_0(normal(seed, (rows, k), std=std))


def dequant_q8_0(blocks: np.ndarray, k: int) -> np.ndarray:
    """GGUF Q8_0 bytes [rows, nb*34] -> f32 [rows, k] (d * q, gguf.rs:425-440)."""
    rows = blocks.shape[0]
    nb = (k + 31) // 32
    b = np.ascontiguousarray(blocks).reshape(rows, nb, 34)
    d = np.ascontiguousarray(b[:, :, 0:2]).view(np.float16).astype(np.float32)
    q = np.ascontiguousarray(b[:, :, 2:]).view(np.int8).astype(np.float32)
    return (d * q).reshape(rows, nb * 32)[:, :k]
