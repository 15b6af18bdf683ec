"""GGUF checkpoints in the layout the reference reads (gguf.rs:1-440).

The reference's converter writes a GGUF variant, and its loader reads it so:
  * header `<IIQQ`: magic 0x46554747, version, n_tensors, n_kv;
  * KV pairs: key (u64 length + bytes), value type u32, value; types
    2 | 8 string, 4 u32, 5 i32, 6 f32, 7 u8 (bool), 3 | 9 array (element
    type u32, count u64, elements of type 4 / 5 / 6 / 8);
  * tensor table: name, n_dims u32, dims u64[n] (fastest axis first), dtype
    u32 (after the dims), offset u64 relative to the data start;
  * tensor data starts at the table's end rounded up to 32 bytes;
  * dtypes 0 f32, 1 f16, 7 Q8_0 with an f32 scale (36-byte blocks), 8 Q8_0
    with an f16 scale (34-byte blocks; this model's linears).

`open_gguf` memory-maps a file and returns zero-copy views of the tensor
bytes; `model_from_gguf` builds the encoder's tensor table from them (the
device repacks the Q8_0 bytes once at `StreamEncoder` creation, the load-
time repack of the reference's `pack_q8`), and `write_gguf` writes the same
layout (synthetic checkpoints for tests and benchmarks).
"""
from __future__ import annotations

import mmap
import struct
from dataclasses import dataclass

import numpy as np

from . import model as _model

GGUF_MAGIC = 0x46554747
F32, F16, Q8_0_F32, Q8_0_F16 = 0, 1, 7, 8


class GgufError(ValueError):
    pass


@dataclass
class TensorMeta:
    name: str
    dims: tuple     # fastest axis first
    dtype: int
    offset: int     # relative to the data start


def tensor_bytes(dims, dtype: int) -> int:
    """Stored size of a tensor (gguf.rs:312-337): rows of dims[0] elements
    padded to whole 32-blocks for the Q8 types."""
    n = 1
    for d in dims:
        n *= int(d)
    row = int(dims[0]) if len(dims) else 1
    if dtype == F32:
        return n * 4
    if dtype == F16:
        return n * 2
    if dtype in (Q8_0_F32, Q8_0_F16):
        blocks = (n // row) * ((row + 31) // 32)
        return blocks * (36 if dtype == Q8_0_F32 else 34)
    raise GgufError(f"unsupported tensor dtype {dtype}")


class _Reader:
    def __init__(self, buf):
        self.buf, self.pos = buf, 0

    def take(self, fmt):
        size = struct.calcsize(fmt)
        if self.pos + size > len(self.buf):
            raise GgufError("unexpected end of file")
        v = struct.unpack_from(fmt, self.buf, self.pos)
        self.pos += size
        return v[0] if len(v) == 1 else v

    def string(self):
        n = self.take("<Q")
        if self.pos + n > len(self.buf):
            raise GgufError("string out of range")
        s = bytes(self.buf[self.pos:self.pos + n]).decode("utf-8", errors="replace")
        self.pos += n
        return s

    def array(self):
        et, count = self.take("<I"), self.take("<Q")
        if et in (4, 5, 6):
            fmt = {4: "<I", 5: "<i", 6: "<f"}[et]
            return [self.take(fmt) for _ in range(count)]
        if et == 8:
            return [self.string() for _ in range(count)]
        raise GgufError(f"unsupported array element type {et}")

    def value(self, t, key):
        if t in (2, 8):
            return self.string()
        if t == 4:
            return self.take("<I")
        if t == 5:
            return self.take("<i")
        if t == 6:
            return self.take("<f")
        if t == 7:
            return self.take("<B")
        if t in (3, 9):
            return self.array()
        raise GgufError(f"unsupported KV value type {t} for key {key}")


class GgufFile:
    """A memory-mapped GGUF file: `kv`, `tensors`, zero-copy `tensor_data`."""

    def __init__(self, path: str):
        self._f = open(path, "rb")
        try:
            self._mm = mmap.mmap(self._f.fileno(), 0, access=mmap.ACCESS_READ)
        except ValueError as e:  # empty file
            self._f.close()
            raise GgufError("not a GGUF file (empty)") from e
        self.kv, self.tensors, self.data_start = self._parse(memoryview(self._mm))
        self._by_name = {t.name: t for t in self.tensors}

    @staticmethod
    def _parse(buf):
        r = _Reader(buf)
        if r.take("<I") != GGUF_MAGIC:
            raise GgufError("not a GGUF file (bad magic)")
        r.take("<I")  # version
        n_tensors, n_kv = r.take("<Q"), r.take("<Q")
        kv = {}
        for _ in range(n_kv):
            key = r.string()
            kv[key] = r.value(r.take("<I"), key)
        tensors = []
        for _ in range(n_tensors):
            name = r.string()
            n_dims = r.take("<I")
            dims = tuple(r.take("<Q") for _ in range(n_dims))
            dtype, offset = r.take("<I"), r.take("<Q")
            tensors.append(TensorMeta(name, dims, dtype, offset))
        return kv, tensors, (r.pos + 31) & ~31

    def tensor(self, name: str) -> TensorMeta:
        try:
            return self._by_name[name]
        except KeyError:
            raise GgufError(f"tensor {name} not in the file") from None

    def tensor_data(self, meta: TensorMeta) -> np.ndarray:
        """The stored bytes of a tensor as a read-only uint8 view of the map."""
        base = self.data_start + meta.offset
        end = base + tensor_bytes(meta.dims, meta.dtype)
        if end > len(self._mm):
            raise GgufError(f"tensor {meta.name} data out of range")
        return np.frombuffer(self._mm, dtype=np.uint8, count=end - base, offset=base)

    def read_f32(self, meta: TensorMeta) -> np.ndarray:
        """Values as f32 in stored order (gguf.rs:270-309): f32, f16, and both
        Q8_0 block formats (value = scale * q, rows padded to 32)."""
        raw = self.tensor_data(meta)
        n = int(np.prod(meta.dims)) if meta.dims else 1
        if meta.dtype == F32:
            return raw.view("<f4").copy()
        if meta.dtype == F16:
            return raw.view("<f2").astype(np.float32)
        row = int(meta.dims[0])
        nb = (row + 31) // 32
        bb = 36 if meta.dtype == Q8_0_F32 else 34
        blocks = raw.reshape(-1, bb)
        if meta.dtype == Q8_0_F32:
            scale = np.ascontiguousarray(blocks[:, :4]).view("<f4")[:, 0]
        else:
            scale = np.ascontiguousarray(blocks[:, :2]).view("<f2")[:, 0].astype(np.float32)
        q = blocks[:, bb - 32:].view(np.int8).astype(np.float32)
        vals = (scale[:, None] * q).reshape(-1, nb * 32)[:, :row]
        return np.ascontiguousarray(vals).reshape(-1)[:n]

    def close(self):
        """Unmap the file; views handed out by tensor_data keep the mapping
        alive until they are released."""
        if getattr(self, "_mm", None) is not None:
            try:
                self._mm.close()
            except BufferError:
                return
            self._mm = None
            self._f.close()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


def open_gguf(path: str) -> GgufFile:
    return GgufFile(path)


# ---------------------------------------------------------------- writer ---
def _w_str(out, s: str):
    b = s.encode()
    out += struct.pack("<Q", len(b)) + b


def _w_value(out, v):
    if isinstance(v, bool):
        out += struct.pack("<IB", 7, int(v))
    elif isinstance(v, int):
        out += struct.pack("<Ii", 5, v) if v < 0 else struct.pack("<II", 4, v)
    elif isinstance(v, float):
        out += struct.pack("<If", 6, v)
    elif isinstance(v, str):
        out += struct.pack("<I", 8)
        _w_str(out, v)
    elif isinstance(v, (list, tuple)):
        if all(isinstance(e, str) for e in v):
            out += struct.pack("<IIQ", 9, 8, len(v))
            for e in v:
                _w_str(out, e)
        elif all(isinstance(e, float) for e in v):
            out += struct.pack("<IIQ", 9, 6, len(v)) + struct.pack(f"<{len(v)}f", *v)
        else:
            out += struct.pack("<IIQ", 9, 5, len(v)) + struct.pack(f"<{len(v)}i", *v)
    else:
        raise GgufError(f"cannot write KV value {v!r}")


def write_gguf(path: str, kv: dict, tensors) -> None:
    """Write `tensors` (objects with name, dtype, dims, data: the stored
    bytes or f32 values) and `kv` in the reference's layout."""
    head = bytearray(struct.pack("<IIQQ", GGUF_MAGIC, 3, len(tensors), len(kv)))
    for k, v in kv.items():
        _w_str(head, k)
        _w_value(head, v)
    blobs, off = [], 0
    for t in tensors:
        data = np.ascontiguousarray(t.data)
        blob = data.view(np.uint8).reshape(-1) if t.dtype != F32 else data.astype("<f4").view(np.uint8).reshape(-1)
        if blob.size != tensor_bytes(t.dims, t.dtype):
            raise GgufError(f"tensor {t.name}: {blob.size} bytes, expected {tensor_bytes(t.dims, t.dtype)}")
        _w_str(head, t.name)
        head += struct.pack("<I", len(t.dims)) + struct.pack(f"<{len(t.dims)}Q", *t.dims)
        head += struct.pack("<IQ", t.dtype, off)
        blobs.append((off, blob))
        off = (off + blob.size + 31) & ~31
    data_start = (len(head) + 31) & ~31
    with open(path, "wb") as f:
        f.write(head)
        f.write(b"\0" * (data_start - len(head)))
        pos = 0
        for o, blob in blobs:
            f.write(b"\0" * (o - pos))
            f.write(blob.tobytes())
            pos = o + blob.size


# ------------------------------------------------------- encoder models ---
ENCODER_KEYS = {
    "d_model": "asr.encoder.d_model", "n_layers": "asr.encoder.n_layers", "n_heads": "asr.encoder.n_heads",
    "d_ff": "asr.encoder.d_ff", "feat_in": "asr.encoder.feat_in",
    "conv_channels": "asr.encoder.subsampling_conv_channels", "conv_kernel": "asr.encoder.conv_kernel_size",
    "att_left": "asr.encoder.offline_left_ctx",
}


def encoder_config(g: GgufFile, max_frames: int = 8) -> "_model.EncoderConfig":
    """EncoderConfig from the metadata (nemotron/config.rs:93-190): the
    streaming chunk is fixed at 7 frames (att_right 6) as in the reference;
    only causal convolution context is supported on the streaming path."""
    def u32(key):
        v = g.kv.get(key)
        if not isinstance(v, int):
            raise GgufError(f"GGUF metadata: missing u32 {key}")
        return v

    ctx = g.kv.get("asr.encoder.conv_context", "causal")
    if ctx != "causal":
        raise GgufError(f"GGUF metadata: conv_context {ctx} is not causal (streaming needs causal)")
    vals = {f: u32(k) for f, k in ENCODER_KEYS.items()}
    n_prompts = g.kv.get("asr.rnnt.num_prompts", 0) if "prompt_kernel.0.weight" in g._by_name else 0
    return _model.EncoderConfig(att_right=6, max_frames=max_frames, n_prompts=int(n_prompts), **vals)


def model_from_gguf(g: GgufFile, max_frames: int = 8) -> "_model.Model":
    """The encoder's tensors (every `encoder.*` tensor of the file and the
    prompt MLP's `prompt_kernel.*`) as a Model whose arrays are zero-copy
    views of the map (f32 tensors are viewed as f32, Q8_0 tensors as their
    stored blocks)."""
    cfg = encoder_config(g, max_frames)
    return _model.Model(cfg, _views(g, ("encoder.", "prompt_kernel.")))


def _views(g: GgufFile, prefixes) -> list:
    out = []
    for t in g.tensors:
        if not t.name.startswith(prefixes):
            continue
        raw = g.tensor_data(t)
        if t.dtype == F32:
            data = raw.view("<f4")
        elif t.dtype == Q8_0_F16:
            data = raw.reshape(-1, (int(t.dims[0]) + 31) // 32 * 34)
        else:
            raise GgufError(f"tensor {t.name}: dtype {t.dtype} not supported on the device path")
        out.append(_model.Tensor(t.name, t.dtype, tuple(int(d) for d in t.dims), data))
    return out


# ------------------------------------------------------- RNN-T decoder ---
RNNT_KEYS = {
    "vocab": "asr.rnnt.vocab_size", "blank": "asr.rnnt.blank_id", "hidden": "asr.rnnt.pred_hidden",
    "n_layers": "asr.rnnt.pred_num_layers", "joint": "asr.rnnt.joint_dim",
    "max_symbols": "asr.rnnt.max_symbols_per_step",
}


def rnnt_config(g: GgufFile) -> "_model.RnntConfig":
    """RnntConfig from the metadata (nemotron/config.rs:171-186); the joint's
    encoder width is the encoder's d_model (joint.enc, decoder.rs:219-221)."""
    vals = {}
    for f, k in RNNT_KEYS.items():
        v = g.kv.get(k)
        if not isinstance(v, int):
            raise GgufError(f"GGUF metadata: missing u32 {k}")
        vals[f] = v
    d_enc = g.kv.get("asr.encoder.d_model", 1024)
    return _model.RnntConfig(d_enc=int(d_enc), **vals)


def decoder_from_gguf(g: GgufFile) -> "_model.Model":
    """The RNN-T decoder's tensors (`decoder.*`, `joint.*`) as a Model of
    zero-copy views of the map."""
    return _model.Model(rnnt_config(g), _views(g, ("decoder.", "joint.")))


def save_model(m: "_model.Model", path: str, extra_kv: dict | None = None,
               decoder: "_model.Model | None" = None) -> None:
    """Write a Model (e.g. a seeded random-init one) as a GGUF checkpoint
    with the encoder metadata the reference reads, and optionally the RNN-T
    decoder's tensors and metadata in the same file."""
    c = m.config
    kv = {k: int(getattr(c, f)) for f, k in ENCODER_KEYS.items()}
    kv.update({"asr.encoder.conv_context": "causal", "asr.encoder.xscaling": False, "asr.encoder.use_bias": True,
               "asr.encoder.subsampling_factor": 8, "asr.encoder.pos_emb_max_len": 5000,
               "asr.rnnt.num_prompts": int(c.n_prompts)})
    tensors = list(m.tensors)
    if decoder is not None:
        dc = decoder.config
        kv.update({k: int(getattr(dc, f)) for f, k in RNNT_KEYS.items()})
        kv.update({"asr.rnnt.pred_embed_dim": int(dc.hidden)})
        tensors += decoder.tensors
    kv.update(extra_kv or {})
    write_gguf(path, kv, tensors)
