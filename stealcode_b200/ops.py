"""Host-side mirror of the reference's operator interface over the C ABI.

Names, argument order and meaning follow the reference's Rust operators so
that code written against them reads the same:

* ``q8_gemm(m, k, n, w, padded_row, block_bytes, qoff, x, y)`` --
  sgemm_kernel.rs:99-127 (host buffers, weights repacked per call);
* ``Q8Mat`` -- nemotron/weights.rs:69-232 (``gemm_t`` keeps the repacked
  weights resident on the device);
* ``Lin.forward_t`` -- nemotron/weights.rs:305-337 (GEMM + bias);
* ``AttnStreamKernel.forward`` -- gpu/kernels.rs:1137-1156.

Device-side entry points take ``torch`` CUDA tensors (PyTorch is used only
for device memory and streams) and launch the library's kernels on the
current torch stream.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import numpy as np

from . import _lib
from ._lib import SC_LAYOUT_FEATURE_MAJOR, SC_LAYOUT_TIME_MAJOR, check, lib


def _hp(a: np.ndarray) -> int:
    if not a.flags["C_CONTIGUOUS"]:
        raise ValueError("host buffers must be C-contiguous")
    return a.ctypes.data


def _stream_ptr(stream=None) -> int:
    import torch

    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def _dp(t) -> int:
    return 0 if t is None else t.data_ptr()


def q8_gemm(m: int, k: int, n: int, w: np.ndarray, padded_row: int, block_bytes: int, qoff: int,
            x: np.ndarray, y: np.ndarray) -> None:
    """Twin of the reference ``q8_gemm``: y [m, n] = W [m, k] @ x [k, n] (host)."""
    if m == 0 or k == 0 or n == 0:
        return
    w = np.ascontiguousarray(w, dtype=np.uint8)
    if x.dtype != np.float32 or y.dtype != np.float32 or x.size != k * n or y.size != m * n:
        raise ValueError("x must be f32 [k, n] and y f32 [m, n]")
    check(lib.sc_q8_gemm_host(m, k, n, _hp(w), padded_row, block_bytes, qoff, _hp(x), _hp(y)))


class Q8Mat:
    """A Q8_0 matrix repacked once into device memory (``Q8Mat``, weights.rs:69-232)."""

    def __init__(self, blocks: np.ndarray, rows: int, row_len: int, block_bytes: int = 34,
                 qoff: int = 2):
        blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
        padded_row = (row_len + 31) // 32 * block_bytes
        if blocks.size != rows * padded_row:
            raise ValueError(f"Q8Mat: {blocks.size} bytes != {rows} rows x {padded_row}")
        h = ctypes.c_void_p()
        check(lib.sc_q8_repack(_hp(blocks), rows, row_len, block_bytes, qoff, ctypes.byref(h)))
        self._h = h
        self.rows = rows
        self.row_len = row_len
        self.padded_row = padded_row

    @property
    def handle(self) -> ctypes.c_void_p:
        return self._h

    def free(self) -> None:
        if self._h:
            lib.sc_q8w_free(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass

    def gemm_t(self, x: np.ndarray, t: int) -> np.ndarray:
        """y [rows, t] = W @ x [row_len, t] with host arrays (``Q8Mat::gemm_t``)."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        y = np.empty((self.rows, t), dtype=np.float32)
        check(lib.sc_q8mat_gemm_t(self._h, _hp(x), t, _hp(y)))
        return y

    def gemm(self, x, *, x_layout: int = SC_LAYOUT_TIME_MAJOR, bias=None, out=None,
             y_layout: int = SC_LAYOUT_TIME_MAJOR, ldx: int = 0, ldy: int = 0, workspace=None,
             stream=None):
        """Device GEMM on torch CUDA tensors; returns ``out``.

        TIME_MAJOR: x [t, row_len] -> y [t, rows]; FEATURE_MAJOR: x [row_len, t] ->
        y [rows, t].  ``workspace`` is an optional uint8 CUDA tensor of at least
        ``workspace_bytes(t)`` bytes."""
        import torch

        if x_layout == SC_LAYOUT_TIME_MAJOR:
            t = x.shape[0]
        else:
            t = x.shape[1]
        if out is None:
            shape = (t, self.rows) if y_layout == SC_LAYOUT_TIME_MAJOR else (self.rows, t)
            out = torch.empty(shape, dtype=torch.float32, device=x.device)
        ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
        check(lib.sc_q8_gemm(self._h, x.data_ptr(), t, x_layout, ldx, _dp(bias), out.data_ptr(), y_layout,
                             ldy, _dp(workspace), ws_bytes, _stream_ptr(stream)))
        return out

    def workspace_bytes(self, t: int) -> int:
        return int(lib.sc_q8_gemm_workspace_bytes(t, self.row_len))

    def block_dots(self, x, *, x_layout: int = SC_LAYOUT_TIME_MAJOR, stream=None):
        """int32 per-block dots [rows, t, nblocks] of the quantised frames."""
        import torch

        t = x.shape[0] if x_layout == SC_LAYOUT_TIME_MAJOR else x.shape[1]
        nb = (self.row_len + 31) // 32
        dots = torch.zeros((self.rows, t, nb), dtype=torch.int32, device=x.device)
        check(lib.sc_q8_block_dots(self._h, x.data_ptr(), t, x_layout, 0, dots.data_ptr(),
                                   _stream_ptr(stream)))
        return dots


class Lin:
    """A Q8_0 linear layer with optional bias (``Lin``, weights.rs:241-337)."""

    def __init__(self, q: Q8Mat, bias: Optional[np.ndarray] = None):
        self.q = q
        self.out = q.rows
        self.inp = q.row_len
        self.bias_host = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
        self._bias_dev = {}

    def forward_t(self, x_t: np.ndarray, t: int) -> np.ndarray:
        """y_t [out, t] = W @ x_t [inp, t] + bias (host arrays)."""
        y = self.q.gemm_t(x_t, t)
        if self.bias_host is not None:
            y += self.bias_host[:, None]
        return y

    def forward(self, x, **kw):
        """Device forward (bias fused into the GEMM epilogue)."""
        import torch

        bias = None
        if self.bias_host is not None:
            dev = x.device
            if dev not in self._bias_dev:
                self._bias_dev[dev] = torch.from_numpy(self.bias_host).to(dev)
            bias = self._bias_dev[dev]
        return self.q.gemm(x, bias=bias, **kw)


def quantize(x, *, x_layout: int = SC_LAYOUT_TIME_MAJOR, stream=None):
    """Device activation quantiser: returns (xq [t, k_pad] int8, dx [nb, t] f32)."""
    import torch

    if x_layout == SC_LAYOUT_TIME_MAJOR:
        t, k = x.shape
    else:
        k, t = x.shape
    nb = (k + 31) // 32
    xq = torch.zeros((t, nb * 32), dtype=torch.int8, device=x.device)
    dx = torch.zeros((nb, t), dtype=torch.float32, device=x.device)
    check(lib.sc_q8_quantize(x.data_ptr(), t, k, x_layout, 0, xq.data_ptr(), dx.data_ptr(),
                             _stream_ptr(stream)))
    return xq, dx


class AttnStreamKernel:
    """Streaming rel-pos attention operator (``AttnStreamKernel``, gpu/kernels.rs:1057-1326)."""

    @staticmethod
    def forward(q, kv, vv, pos_p, q_bias, v_bias, c, d, n_heads, scale, s, k_lo, band, chunk,
                left_chunks, k_hi, pos_off) -> np.ndarray:
        """Host-buffer twin of ``forward``: returns out [c, d]."""
        arrs = [np.ascontiguousarray(a, dtype=np.float32) for a in (q, kv, vv, pos_p, q_bias, v_bias)]
        n_pos = arrs[3].size // d
        out = np.zeros((c, d), dtype=np.float32)
        check(lib.sc_attn_stream_host(*[_hp(a) for a in arrs[:4]], n_pos, _hp(arrs[4]), _hp(arrs[5]), c, d,
                                      n_heads, scale, s, k_lo, band, chunk, left_chunks, k_hi, pos_off,
                                      _hp(out)))
        return out

    @staticmethod
    def forward_device(q, kv, vv, pos_p, q_bias, v_bias, c, d, n_heads, scale, s, k_lo, band, chunk,
                       left_chunks, k_hi, pos_off, out=None, stream=None):
        import torch

        if out is None:
            out = torch.empty((c, d), dtype=torch.float32, device=q.device)
        n_pos = pos_p.numel() // d
        check(lib.sc_attn_stream(q.data_ptr(), kv.data_ptr(), vv.data_ptr(), pos_p.data_ptr(), n_pos,
                                 q_bias.data_ptr(), v_bias.data_ptr(), c, d, n_heads, scale, s, k_lo, band,
                                 chunk, left_chunks, k_hi, pos_off, out.data_ptr(), _stream_ptr(stream)))
        return out


def attn_stream_ring(q, k_new, v_new, k_ring, v_ring, pos_p, q_bias, v_bias, *, c, d, n_heads, scale, s,
                     k_lo, chunk, left_chunks, pos_off, out=None, ldq=0, ld_new=0, ldo=0, stream=None):
    """Batched ring-cache attention over ``k_ring.shape[0]`` streams (torch CUDA tensors).

    k_ring/v_ring: [n_streams, cap, d]; q/k_new/v_new: [n_streams * c, ld] rows."""
    import torch

    n_streams, cap = k_ring.shape[0], k_ring.shape[1]
    if out is None:
        out = torch.empty((n_streams * c, d), dtype=torch.float32, device=q.device)
    n_pos = pos_p.numel() // d
    check(lib.sc_attn_stream_ring(q.data_ptr(), ldq, k_new.data_ptr(), v_new.data_ptr(), ld_new,
                                  k_ring.data_ptr(), v_ring.data_ptr(), cap, n_streams, pos_p.data_ptr(), n_pos,
                                  q_bias.data_ptr(), v_bias.data_ptr(), c, d, n_heads, scale, s, k_lo, chunk,
                                  left_chunks, s + c, pos_off, out.data_ptr(), ldo, _stream_ptr(stream)))
    return out


class StreamEncoder:
    """Device streaming encoder for n_streams lockstep streams -- the
    StreamEncoder trait (streaming.rs:687-704): encode_new, frames, total."""

    def __init__(self, model, n_streams: int):
        from .model import ScEncoderConfig

        self.model = model
        self._table = model.table()
        self._cfg = ScEncoderConfig.of(model.config)
        h = ctypes.c_void_p()
        check(lib.sc_stream_encoder_create(ctypes.byref(self._cfg), self._table, len(model.tensors), n_streams,
                                           ctypes.byref(h)))
        self._h = h
        self.n_streams = n_streams
        self.d = model.config.d_model

    def encode_new(self, mel_new, t0: int, t1: int, fin: bool = False, stream=None) -> None:
        """mel_new: CUDA tensor [n_streams, t1 - t0, feat_in] (f32)."""
        check(lib.sc_stream_encoder_encode_new(self._h, mel_new.data_ptr() if mel_new is not None else None, t0, t1,
                                               int(fin), _stream_ptr(stream)))

    def encode_new_host(self, mel_new: np.ndarray, t0: int, t1: int, fin: bool = False, out=None,
                        stream=None):
        """encode_new with host buffers (the reference's call shape): mel_new
        is a host float32 array [n_streams, t1 - t0, feat_in]; returns the
        call's output frames [n_streams * c, d] in `out` (a host float32
        array of at least n_streams * max_frames rows, page-locked for
        overlapped copies) or a new array.  Synchronous."""
        mel = np.ascontiguousarray(mel_new, dtype=np.float32)
        if mel.shape[0] != self.n_streams or (mel.ndim == 3 and mel.shape[1] != t1 - t0):
            raise ValueError(f"encode_new_host: mel shape {mel.shape} for {self.n_streams} streams x {t1 - t0}")
        cap = self.n_streams * self.model.config.max_frames
        if out is None:
            out = np.empty((cap, self.d), dtype=np.float32)
        if isinstance(out, np.ndarray):
            if out.dtype != np.float32 or not out.flags.c_contiguous or out.size < cap * self.d:
                raise ValueError("encode_new_host: out must be C-contiguous float32 with n_streams * max_frames rows")
            optr = _hp(out)
        else:  # a page-locked torch CPU tensor
            if out.numel() < cap * self.d:
                raise ValueError("encode_new_host: out too small")
            optr = out.data_ptr()
        rows = ctypes.c_int64()
        check(lib.sc_stream_encoder_encode_new_host(self._h, _hp(mel) if mel.size else None, t0, t1, int(fin),
                                                    optr, ctypes.byref(rows), _stream_ptr(stream)))
        return out[: rows.value]

    def encode_new_host_ptr(self, mel_ptr: int, t0: int, t1: int, fin: bool, out_ptr: int, stream=None) -> int:
        """encode_new_host on raw host pointers (page-locked buffers the caller
        owns); returns the rows written."""
        rows = ctypes.c_int64()
        check(lib.sc_stream_encoder_encode_new_host(self._h, mel_ptr, t0, t1, int(fin), out_ptr,
                                                    ctypes.byref(rows), _stream_ptr(stream)))
        return rows.value

    @classmethod
    def from_gguf(cls, path: str, n_streams: int, max_frames: int = 8) -> "StreamEncoder":
        """Build from a GGUF checkpoint in the reference's layout
        (`Encoder::load`, nemotron/encoder.rs:249-282): the file is memory-
        mapped and its tensors go to the device without a host copy."""
        from . import gguf

        g = gguf.open_gguf(path)
        enc = cls(gguf.model_from_gguf(g, max_frames), n_streams)
        enc._gguf = g  # the mapping backs the model's arrays
        return enc

    def total(self) -> int:
        return int(lib.sc_stream_encoder_total(self._h))

    def frames(self, stream_idx: int, frm: int, to: int) -> np.ndarray:
        out = np.empty((to - frm, self.d), dtype=np.float32)
        check(lib.sc_stream_encoder_frames(self._h, stream_idx, frm, to, _hp(out)))
        return out

    def output(self):
        """(device pointer, rows, d) of the last step's frames [n_streams * c, d]."""
        ptr, rows, d = ctypes.c_void_p(), ctypes.c_int64(), ctypes.c_int64()
        check(lib.sc_stream_encoder_output(self._h, ctypes.byref(ptr), ctypes.byref(rows), ctypes.byref(d)))
        return ptr.value, rows.value, d.value

    def set_prompts(self, prompt_ids) -> None:
        """Prompt of each stream for the prompt MLP (the prompt_id argument of
        encode_new, streaming.rs:687-699); None / < 0 / out of range: none."""
        ids = np.array([-1 if p is None else int(p) for p in prompt_ids], dtype=np.int32)
        if ids.shape != (self.n_streams,):
            raise ValueError(f"set_prompts: {ids.shape[0]} ids for {self.n_streams} streams")
        check(lib.sc_stream_encoder_set_prompts(self._h, _hp(ids)))

    @property
    def n_prompts(self) -> int:
        return int(lib.sc_stream_encoder_n_prompts(self._h))

    def set_concurrency(self, n_batches: int) -> None:
        """Sub-batches of streams in flight per encode_new (1 or 2; same bits)."""
        check(lib.sc_stream_encoder_set_concurrency(self._h, n_batches))

    def set_graphs(self, enable: bool) -> None:
        """Step graphs on (the default) or off: steady steps replay one CUDA
        graph of the whole step, else every kernel launches separately (same
        bits)."""
        check(lib.sc_stream_encoder_set_graphs(self._h, 1 if enable else 0))

    def graph_stats(self) -> tuple:
        """(graphs on, graphs captured, graph launches) so far."""
        cap, lau = ctypes.c_int64(), ctypes.c_int64()
        rc = lib.sc_stream_encoder_graph_stats(self._h, ctypes.byref(cap), ctypes.byref(lau))
        check(min(rc, 0))
        return bool(rc), int(cap.value), int(lau.value)

    def set_dump(self, layer: int) -> None:
        check(lib.sc_stream_encoder_set_dump(self._h, layer))

    def dump(self, stage: int) -> np.ndarray:
        rows = ctypes.c_int64()
        out = np.empty((self.n_streams * 16, self.d), dtype=np.float32)
        check(lib.sc_stream_encoder_dump(self._h, stage, _hp(out), ctypes.byref(rows)))
        return out[: rows.value].copy()

    def close(self):
        if getattr(self, "_h", None):
            lib.sc_stream_encoder_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class RnntDecoder:
    """Device greedy RNN-T decoder for n_streams streams, each with its own
    carried state: decode_frames (live.rs:56-145) over the predictor LSTM
    and joint network (nemotron/decoder.rs:75-235)."""

    def __init__(self, model, n_streams: int, max_frames: int = 16):
        from .model import ScRnntConfig

        self.model = model
        self.config = model.config
        self._table = model.table()
        self._cfg = ScRnntConfig.of(model.config, max_frames)
        h = ctypes.c_void_p()
        check(lib.sc_rnnt_create(ctypes.byref(self._cfg), self._table, len(model.tensors), n_streams,
                                 ctypes.byref(h)))
        self._h = h
        self.n_streams = n_streams
        self.cap = 16 * max_frames + 64

    @classmethod
    def from_gguf(cls, path: str, n_streams: int, max_frames: int = 16) -> "RnntDecoder":
        """Build from a GGUF checkpoint in the reference's layout
        (GreedyDecoder::load, nemotron/decoder.rs:238-247), memory-mapped."""
        from . import gguf

        g = gguf.open_gguf(path)
        dec = cls(gguf.decoder_from_gguf(g), n_streams, max_frames)
        dec._gguf = g  # the mapping backs the model's arrays
        return dec

    def decode_frames(self, frames, stream=None) -> None:
        """frames: CUDA tensor [n_streams, n, d_enc] (f32) or a raw device
        pointer with n given as (ptr, n).  Synchronises the stream."""
        if isinstance(frames, tuple):
            ptr, n = frames
        else:
            if frames.dim() != 3 or frames.shape[0] != self.n_streams or frames.shape[2] != self.config.d_enc:
                raise ValueError(f"frames must be [{self.n_streams}, n, {self.config.d_enc}]")
            import torch

            if not frames.is_contiguous() or frames.dtype != torch.float32:
                raise ValueError("frames must be contiguous f32")
            ptr, n = frames.data_ptr(), frames.shape[1]
        check(lib.sc_rnnt_decode_frames(self._h, ptr, n, _stream_ptr(stream)))

    def tokens(self, stream_idx: int):
        """(ids, steps) the last decode_frames emitted for one stream."""
        ids = np.empty(self.cap, dtype=np.int32)
        steps = np.empty(self.cap, dtype=np.int32)
        cnt = ctypes.c_int32()
        check(lib.sc_rnnt_tokens(self._h, stream_idx, _hp(ids), _hp(steps), self.cap, ctypes.byref(cnt)))
        return ids[: cnt.value].copy(), steps[: cnt.value].copy()

    def last_rounds(self) -> int:
        """Loop rounds the last decode_frames ran (diagnostic)."""
        return int(lib.sc_rnnt_last_rounds(self._h))

    def emitted(self) -> np.ndarray:
        """Tokens each stream emitted in the last decode_frames, [n_streams]."""
        out = np.empty(self.n_streams, dtype=np.int32)
        check(lib.sc_rnnt_emitted(self._h, _hp(out)))
        return out

    def state(self, stream_idx: int):
        """(h, c, last_token) of one stream; h, c: [n_layers, hidden]."""
        c = self.config
        h = np.empty((c.n_layers, c.hidden), dtype=np.float32)
        cc = np.empty_like(h)
        last = ctypes.c_int32()
        check(lib.sc_rnnt_state(self._h, stream_idx, _hp(h), _hp(cc), ctypes.byref(last)))
        return h, cc, last.value

    def reset(self, stream_idx: int = -1) -> None:
        check(lib.sc_rnnt_reset(self._h, stream_idx))

    def close(self):
        if getattr(self, "_h", None):
            lib.sc_rnnt_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


__all__ = ["StreamEncoder", "RnntDecoder", "q8_gemm", "Q8Mat", "Lin", "quantize", "AttnStreamKernel", "attn_stream_ring",
           "SC_LAYOUT_FEATURE_MAJOR", "SC_LAYOUT_TIME_MAJOR", "_lib"]


def q8_gemm_batch(mats, xs, *, biases=None, outs=None, x_layout: int = SC_LAYOUT_TIME_MAJOR,
                  y_layout: int = SC_LAYOUT_TIME_MAJOR, workspace=None, stream=None):
    """Independent GEMMs y[i] = mats[i] x[i] (+ biases[i]) of the same frame
    count (<= 16) in one streaming pass (sc_q8_gemm_batch); torch CUDA
    tensors; returns the outputs."""
    import torch

    n = len(mats)
    t = xs[0].shape[0] if x_layout == SC_LAYOUT_TIME_MAJOR else xs[0].shape[1]
    if outs is None:
        outs = [torch.empty((t, m.rows) if y_layout == SC_LAYOUT_TIME_MAJOR else (m.rows, t), dtype=torch.float32,
                            device=xs[0].device) for m in mats]
    P = ctypes.c_void_p
    hw = (P * n)(*[m.handle.value for m in mats])
    hx = (P * n)(*[x.data_ptr() for x in xs])
    hy = (P * n)(*[y.data_ptr() for y in outs])
    hb = (P * n)(*[(b.data_ptr() if b is not None else None) for b in biases]) if biases is not None else None
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    check(lib.sc_q8_gemm_batch(hw, hx, hb, hy, n, t, x_layout, y_layout, _dp(workspace), ws_bytes,
                               _stream_ptr(stream)))
    return outs
