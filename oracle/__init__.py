"""CPU oracle for the stealcode_b200 hot path -- TEST INFRASTRUCTURE ONLY.

A ctypes binding of ``oracle/liboracle.so``, a plain-C restatement of the
reference's CPU operators (see ``oracle/sc_oracle.h`` for the file:line each
function restates).  Only the tests, ``__graft_entry__.smoke()`` and
``bench.py``'s CPU-baseline leg use it, as the checker and the timed CPU
baseline; the product never imports it.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from ctypes import c_float, c_int, c_size_t, c_uint16, c_void_p

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")


def build() -> None:
    """Compile liboracle.so with gcc (make -C oracle)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)


if not os.path.exists(LIB_PATH):
    build()

lib = ctypes.CDLL(LIB_PATH)
_P = c_void_p
_S = c_size_t
for _name, _res, _args in [
    ("orc_f16_to_f32", c_float, [c_uint16]),
    ("orc_half_from_f32_trunc", c_uint16, [c_float]),
    ("orc_quantize_col", None, [_P, _S, _S, _S, _S, _P, _P]),
    ("orc_q8_gemm_scalar", None, [_S, _S, _S, _P, _S, _S, _S, _P, _P]),
    ("orc_q8_gemm_simd_order", None, [_S, _S, _S, _P, _S, _S, _S, _P, _P]),
    ("orc_q8_gemm", None, [_S, _S, _S, _P, _S, _S, _S, _P, _P, c_int]),
    ("orc_q8_gemm_order", None, [_S, _S, _S, _P, _S, _S, _S, _P, _P, c_int, c_int]),
    ("orc_q8_block_dots", None, [_S, _S, _S, _P, _S, _S, _S, _P, _P]),
    ("orc_score_dot", c_float, [_P, _P, _P, _P, _P, _P, _S, c_float]),
    ("orc_softmax_v", None, [_P, _S, _S, _S, _S, _P, _S, _P]),
    ("orc_attn_stream", None, [_P, _P, _P, _P, _P, _P, _S, _S, _S, c_float, _S, _S, _S, _S, _S, _S,
                               _S, _P]),
    ("orc_attn_stream_testloop", None, [_P, _P, _P, _P, _P, _P, _S, _S, _S, c_float, _S, _S, _S, _S,
                                        _S, _S, _P]),
    ("orc_num_cpus", c_int, []),
    ("orc_enc_create", c_void_p, [_P, _P, c_int, ctypes.c_char_p, _S]),
    ("orc_enc_destroy", None, [_P]),
    ("orc_enc_encode_new", c_int, [_P, _P, _S, _S, _S, _S, c_int]),
    ("orc_enc_total", _S, [_P]),
    ("orc_enc_frames", c_int, [_P, _S, _S, _P]),
    ("orc_enc_last", c_int, [_P, c_int, _P, ctypes.POINTER(_S)]),
    ("orc_enc_set_dump", None, [_P, c_int]),
    ("orc_enc_set_gemm_order", None, [_P, c_int]),
    ("orc_enc_set_exp_mode", None, [_P, c_int]),
    ("orc_enc_set_prompt", c_int, [_P, c_int]),
    ("orc_rnnt_create", c_void_p, [_P, _P, c_int, ctypes.c_char_p, _S]),
    ("orc_rnnt_destroy", None, [_P]),
    ("orc_rnnt_set_order", None, [_P, c_int, c_int]),
    ("orc_rnnt_state_new", c_void_p, [_P]),
    ("orc_rnnt_state_free", None, [_P]),
    ("orc_rnnt_state_get", None, [_P, _P, _P, _P]),
    ("orc_rnnt_decode_frames", c_int, [_P, _P, _P, _S, _P, _P, c_int]),
    ("orc_tanhf", c_float, [c_float]),
    ("orc_set_exp_mode", None, [c_int]),
    ("orc_get_exp_mode", c_int, []),
    ("orc_expf", c_float, [c_float]),
    ("orc_enc_dump", c_int, [_P, c_int, _P, ctypes.POINTER(_S)]),
    ("orc_ln_forward", None, [_P, _P, _P, c_float, _P, _S]),
    ("orc_dwconv_forward", None, [_P, _S, _S, _S, _S, _S, _P, _P]),
    ("orc_glu_from", None, [_P, _S, _S, _P]),
    ("orc_silu_inplace", None, [_P, _S]),
    ("orc_gemm_simd_into", None, [_S, _S, _S, _P, _P, _P, _P]),
    ("orc_set_fast", None, [c_int]),
    ("orc_get_fast", c_int, []),
    ("orc_have_avx2", c_int, []),
    ("orc_enc_phase_times", None, [_P, _P]),
]:
    _f = getattr(lib, _name)
    _f.restype = _res
    _f.argtypes = _args


def _p(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


def f16_to_f32(h: int) -> float:
    return lib.orc_f16_to_f32(h)


def half_from_f32_trunc(v: float) -> int:
    return lib.orc_half_from_f32_trunc(v)


def quantize(x_km: np.ndarray):
    """quantize_col over every column of feature-major x [k, n]:
    returns (xq [n, k] int8, dx [n, nblocks] f32)."""
    x = np.ascontiguousarray(x_km, dtype=np.float32)
    k, n = x.shape
    nb = (k + 31) // 32
    xq = np.zeros((n, k), dtype=np.int8)
    dx = np.zeros((n, nb), dtype=np.float32)
    for nj in range(n):
        lib.orc_quantize_col(_p(x), nj, k, n, nb, xq[nj:].ctypes.data, dx[nj:].ctypes.data)
    return xq, dx


def q8_gemm_scalar(m, k, n, w, padded_row, block_bytes, qoff, x_km):
    """q8_gemm_scalar: y [m, n] from weight bytes and feature-major x [k, n]."""
    w = np.ascontiguousarray(w, dtype=np.uint8)
    x = np.ascontiguousarray(x_km, dtype=np.float32)
    y = np.zeros((m, n), dtype=np.float32)
    lib.orc_q8_gemm_scalar(m, k, n, _p(w), padded_row, block_bytes, qoff, _p(x), _p(y))
    return y


def q8_gemm_simd_order(m, k, n, w, padded_row, block_bytes, qoff, x_km):
    w = np.ascontiguousarray(w, dtype=np.uint8)
    x = np.ascontiguousarray(x_km, dtype=np.float32)
    y = np.zeros((m, n), dtype=np.float32)
    lib.orc_q8_gemm_simd_order(m, k, n, _p(w), padded_row, block_bytes, qoff, _p(x), _p(y))
    return y


def q8_gemm(m, k, n, w, padded_row, block_bytes, qoff, x_km, nthreads: int = 0, y=None):
    """The threaded AVX2 dispatcher (timed CPU baseline); same bits as above."""
    w = np.ascontiguousarray(w, dtype=np.uint8)
    x = np.ascontiguousarray(x_km, dtype=np.float32)
    if y is None:
        y = np.zeros((m, n), dtype=np.float32)
    lib.orc_q8_gemm(m, k, n, _p(w), padded_row, block_bytes, qoff, _p(x), _p(y), nthreads)
    return y


def q8_block_dots(m, k, n, w, padded_row, block_bytes, qoff, x_km):
    w = np.ascontiguousarray(w, dtype=np.uint8)
    x = np.ascontiguousarray(x_km, dtype=np.float32)
    nb = (k + 31) // 32
    dots = np.zeros((m, n, nb), dtype=np.int32)
    lib.orc_q8_block_dots(m, k, n, _p(w), padded_row, block_bytes, qoff, _p(x), _p(dots))
    return dots


def gemm_simd_into(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """The reference's f32 GEMM c[m, n] = a[m, k] @ b[k, n] with its rounding
    (simd_kernel.rs:448-727 gemm_simd_into)."""
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    m, k = a.shape
    k2, n = b.shape
    assert k == k2
    c = np.zeros((m, n), np.float32)
    bt = np.zeros((max(n * k, 1),), np.float32)
    lib.orc_gemm_simd_into(m, k, n, _p(a), _p(b), _p(c), _p(bt))
    return c


def score_dot(qu, uh, qv, vh, kk, p, scale):
    arrs = [np.ascontiguousarray(a, dtype=np.float32) for a in (qu, uh, qv, vh, kk, p)]
    return lib.orc_score_dot(*[_p(a) for a in arrs], arrs[0].size, scale)


def softmax_v(srow, k0, k1, n_heads, h, v_rows, head_dim):
    """v_rows: array [k1, head_dim] (row kk = v_at(kk))."""
    srow = np.ascontiguousarray(srow, dtype=np.float32)
    v = np.ascontiguousarray(v_rows, dtype=np.float32)
    ptrs = (c_void_p * max(k1, 1))(*[v.ctypes.data + kk * head_dim * 4 for kk in range(k1)])
    out = np.zeros(head_dim, dtype=np.float32)
    lib.orc_softmax_v(_p(srow), k0, k1, n_heads, h, ctypes.cast(ptrs, c_void_p), head_dim, _p(out))
    return out


def attn_stream(q, kv, vv, pos_p, q_bias, v_bias, c, d, n_heads, scale, s, k_lo, band, chunk,
                left_chunks, k_hi, pos_off):
    arrs = [np.ascontiguousarray(a, dtype=np.float32) for a in (q, kv, vv, pos_p, q_bias, v_bias)]
    out = np.zeros((c, d), dtype=np.float32)
    lib.orc_attn_stream(*[_p(a) for a in arrs], c, d, n_heads, scale, s, k_lo, band, chunk,
                        left_chunks, k_hi, pos_off, _p(out))
    return out


def attn_stream_testloop(q, kv, vv, pos_p, q_bias, v_bias, c, d, n_heads, scale, s, k_lo, chunk,
                         left_chunks, k_hi, pos_off):
    arrs = [np.ascontiguousarray(a, dtype=np.float32) for a in (q, kv, vv, pos_p, q_bias, v_bias)]
    out = np.zeros((c, d), dtype=np.float32)
    lib.orc_attn_stream_testloop(*[_p(a) for a in arrs], c, d, n_heads, scale, s, k_lo, chunk,
                                 left_chunks, k_hi, pos_off, _p(out))
    return out


def set_exp_mode(correctly_rounded: bool) -> None:
    """Exp of the standalone softmax/attention/SiLU functions in this thread
    (False: libm expf as the reference; True: correctly rounded)."""
    lib.orc_set_exp_mode(1 if correctly_rounded else 0)


def expf(x: float, correctly_rounded: bool = False) -> float:
    saved = lib.orc_get_exp_mode()
    lib.orc_set_exp_mode(1 if correctly_rounded else 0)
    try:
        return lib.orc_expf(x)
    finally:
        lib.orc_set_exp_mode(saved)


def num_cpus() -> int:
    return lib.orc_num_cpus()


def set_fast(on: bool) -> None:
    """True (the default): the reference's threading and AVX2 lanes; False:
    every operator serial and scalar.  Outputs are bit-identical."""
    lib.orc_set_fast(1 if on else 0)


def get_fast() -> bool:
    return bool(lib.orc_get_fast())


def have_avx2() -> bool:
    return bool(lib.orc_have_avx2())


class OrcEncConfig(ctypes.Structure):
    _fields_ = [("d_model", ctypes.c_int32), ("n_layers", ctypes.c_int32), ("n_heads", ctypes.c_int32),
                ("d_ff", ctypes.c_int32), ("feat_in", ctypes.c_int32), ("conv_channels", ctypes.c_int32),
                ("conv_kernel", ctypes.c_int32), ("conv_left", ctypes.c_int32), ("att_left", ctypes.c_int32),
                ("att_right", ctypes.c_int32), ("ln_eps", ctypes.c_float)]


class StreamingEncoder:
    """The reference's single-stream CPU StreamingEncoder (streaming.rs:42-383),
    restated in C.  `model` is a stealcode_b200.model.Model."""

    def __init__(self, model):
        c = model.config
        self.model = model
        self._table = model.table()
        self._cfg = OrcEncConfig(c.d_model, c.n_layers, c.n_heads, c.d_ff, c.feat_in, c.conv_channels,
                                 c.conv_kernel, c.conv_left, c.att_left, c.att_right, c.ln_eps)
        err = ctypes.create_string_buffer(256)
        self._destroy = lib.orc_enc_destroy
        self._h = lib.orc_enc_create(ctypes.byref(self._cfg), self._table, len(model.tensors), err, 256)
        if not self._h:
            raise RuntimeError(err.value.decode())
        self.d = c.d_model

    def encode_new(self, mel: np.ndarray, t0: int, t1: int, fin: bool = False) -> int:
        """mel: all mel frames of the stream so far, [n_frames, n_mels]."""
        mel = np.ascontiguousarray(mel, dtype=np.float32)
        return lib.orc_enc_encode_new(self._h, _p(mel), mel.shape[0], mel.shape[1], t0, t1, int(fin))

    def total(self) -> int:
        return lib.orc_enc_total(self._h)

    def frames(self, frm: int, to: int) -> np.ndarray:
        out = np.empty((to - frm, self.d), dtype=np.float32)
        if lib.orc_enc_frames(self._h, frm, to, _p(out)):
            raise ValueError("frames out of range")
        return out

    def last(self, which: int) -> np.ndarray:
        c = ctypes.c_size_t()
        out = np.empty((16, self.d), dtype=np.float32)
        if lib.orc_enc_last(self._h, which, _p(out), ctypes.byref(c)):
            raise ValueError("no such stage")
        return out[: c.value].copy()

    def phase_times(self) -> dict:
        """Host seconds spent in encode_new so far, by phase."""
        out = np.zeros(4, np.float64)
        lib.orc_enc_phase_times(self._h, _p(out))
        return {"pre_encode": float(out[0]), "linears": float(out[1]), "attention": float(out[2]),
                "total": float(out[3])}

    def set_gemm_order(self, scalar: bool) -> None:
        """False: the reference's GEMM dispatch (8-lane SIMD order for chunks
        of <= 16 frames); True: q8_gemm_scalar's arithmetic for every linear."""
        lib.orc_enc_set_gemm_order(self._h, 1 if scalar else 0)

    def set_exp_mode(self, correctly_rounded: bool) -> None:
        """False: libm expf (the reference on glibc); True: correctly rounded
        exp, as the device computes it."""
        lib.orc_enc_set_exp_mode(self._h, 1 if correctly_rounded else 0)

    def set_device_rounding(self) -> None:
        """Scalar-order linears and correctly rounded exp: the device's
        rounding, one ulp away from the reference's dispatch in rare places."""
        self.set_gemm_order(True)
        self.set_exp_mode(True)

    def set_prompt(self, prompt_id) -> None:
        """Prompt of the multilingual prompt MLP (streaming.rs:320-342);
        None = no prompt.  Raises when the model has no prompt MLP or the id
        is out of range."""
        if lib.orc_enc_set_prompt(self._h, -1 if prompt_id is None else int(prompt_id)):
            raise ValueError(f"prompt {prompt_id}: no prompt MLP or out of range")

    def set_dump(self, layer: int) -> None:
        lib.orc_enc_set_dump(self._h, layer)

    def dump(self, stage: int) -> np.ndarray:
        c = ctypes.c_size_t()
        out = np.empty((16, self.d), dtype=np.float32)
        if lib.orc_enc_dump(self._h, stage, _p(out), ctypes.byref(c)):
            raise ValueError("no dump recorded")
        return out[: c.value].copy()

    def __del__(self):
        # the destroy function is held by the instance: module globals may
        # already be gone when this runs at interpreter exit
        h, destroy = getattr(self, "_h", None), getattr(self, "_destroy", None)
        if h and destroy:
            destroy(h)
            self._h = None


class OrcRnntConfig(ctypes.Structure):
    _fields_ = [("d_enc", ctypes.c_int32), ("hidden", ctypes.c_int32), ("n_layers", ctypes.c_int32),
                ("joint", ctypes.c_int32), ("vocab", ctypes.c_int32), ("blank", ctypes.c_int32),
                ("max_symbols", ctypes.c_int32)]


class RnntState:
    """StreamState (live.rs:24-50) of one stream: LSTM h/c per layer and the
    last emitted token."""

    def __init__(self, dec: "RnntDecoder"):
        self._dec = dec
        self._free = lib.orc_rnnt_state_free
        self._h = lib.orc_rnnt_state_new(dec._h)

    def get(self):
        c = self._dec.config
        h = np.empty((c.n_layers, c.hidden), dtype=np.float32)
        cc = np.empty_like(h)
        last = ctypes.c_int32()
        lib.orc_rnnt_state_get(self._h, _p(h), _p(cc), ctypes.byref(last))
        return h, cc, last.value

    def __del__(self):
        h, free = getattr(self, "_h", None), getattr(self, "_free", None)
        if h and free:
            free(h)
            self._h = None


class RnntDecoder:
    """The reference's greedy RNN-T decoder (nemotron/decoder.rs:75-235,
    live.rs:56-145) restated in C.  `model` is a stealcode_b200.model.Model
    whose config is an RnntConfig."""

    def __init__(self, model):
        c = model.config
        self.config = c
        self.model = model
        self._table = model.table()
        self._cfg = OrcRnntConfig(c.d_enc, c.hidden, c.n_layers, c.joint, c.vocab, c.blank, c.max_symbols)
        err = ctypes.create_string_buffer(256)
        self._destroy = lib.orc_rnnt_destroy
        self._h = lib.orc_rnnt_create(ctypes.byref(self._cfg), self._table, len(model.tensors), err, 256)
        if not self._h:
            raise RuntimeError(err.value.decode())

    def set_order(self, scalar_gemm: bool = False, exp_cr: bool = False) -> None:
        """scalar_gemm: q8_gemm_scalar's arithmetic for every matvec instead
        of the reference's dispatch; exp_cr: correctly rounded exp/tanh."""
        lib.orc_rnnt_set_order(self._h, int(scalar_gemm), int(exp_cr))

    def new_state(self) -> RnntState:
        return RnntState(self)

    def decode_frames(self, frames: np.ndarray, state: RnntState):
        """decode_frames (live.rs:56-145) over frames [n, d_enc]: returns
        the (ids, steps) emitted; raises on the iteration cap."""
        frames = np.ascontiguousarray(frames, dtype=np.float32)
        n = frames.shape[0]
        cap = 16 * n + 64
        ids = np.empty(cap, dtype=np.int32)
        steps = np.empty(cap, dtype=np.int32)
        k = lib.orc_rnnt_decode_frames(self._h, state._h, _p(frames), n, _p(ids), _p(steps), cap)
        if k < 0:
            raise RuntimeError("rnnt decode: iteration cap hit")
        return ids[:k].copy(), steps[:k].copy()

    def __del__(self):
        h, destroy = getattr(self, "_h", None), getattr(self, "_destroy", None)
        if h and destroy:
            destroy(h)
            self._h = None
