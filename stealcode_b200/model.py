"""Seeded random-init FastConformer encoder weights with the reference's GGUF
tensor names, and the tensor table (`sc_tensor`) that hands them to the C ABI.

Tensor names and shapes follow what the reference loads
(nemotron/encoder.rs:89-245, weights.rs:640-790): linears are Q8_0 with f16
block scales (GGUF dtype 8, dims [in, out]); LayerNorms, biases, pos_bias_u/v,
the depthwise conv (dims [k, 1, d]) and the pre-encode convs (dims [kw, kh,
in/groups, out]) are f32.  Value distributions: linear weights ~N(0, 0.02)
then Q8_0, biases and LN shifts ~N(0, 0.02), LN scales 1 + N(0, 0.02),
pos_bias_u/v ~N(0, 0.02); convolution weights are scaled by 1/sqrt(fan-in)
so activations keep unit scale through the pre-encode stack.
"""
from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass, field

import numpy as np

from . import synth


@dataclass
class EncoderConfig:
    """EncoderConfig (nemotron/config.rs:19-39) of the streaming Nemotron
    encoder; att_right = 6 is the reference's fixed chunk of 7 frames
    (nemotron/config.rs:164)."""
    d_model: int = 1024
    n_layers: int = 24
    n_heads: int = 8
    d_ff: int = 4096
    feat_in: int = 128
    conv_channels: int = 256
    conv_kernel: int = 9
    att_left: int = 70
    att_right: int = 6
    ln_eps: float = 1e-5
    max_frames: int = 8
    n_prompts: int = 0      # asr.rnnt.num_prompts: > 0 adds the prompt MLP

    @property
    def conv_left(self) -> int:
        return self.conv_kernel - 1

    @property
    def chunk(self) -> int:
        return self.att_right + 1


class ScEncoderConfig(ctypes.Structure):
    _fields_ = [("d_model", ctypes.c_int32), ("n_layers", ctypes.c_int32), ("n_heads", ctypes.c_int32),
                ("d_ff", ctypes.c_int32), ("feat_in", ctypes.c_int32), ("conv_channels", ctypes.c_int32),
                ("conv_kernel", ctypes.c_int32), ("conv_left", ctypes.c_int32), ("att_left", ctypes.c_int32),
                ("att_right", ctypes.c_int32), ("ln_eps", ctypes.c_float), ("max_frames", ctypes.c_int32)]

    @classmethod
    def of(cls, c: EncoderConfig) -> "ScEncoderConfig":
        return cls(c.d_model, c.n_layers, c.n_heads, c.d_ff, c.feat_in, c.conv_channels, c.conv_kernel,
                   c.conv_left, c.att_left, c.att_right, c.ln_eps, c.max_frames)


class ScTensor(ctypes.Structure):
    """sc_tensor / orc_tensor: {name, dtype, n_dims, dims[4], data}."""
    _fields_ = [("name", ctypes.c_char_p), ("dtype", ctypes.c_int32), ("n_dims", ctypes.c_int32),
                ("dims", ctypes.c_int64 * 4), ("data", ctypes.c_void_p)]


@dataclass
class Tensor:
    name: str
    dtype: int          # 0 f32, 8 Q8_0 (f16 scales)
    dims: tuple         # GGUF order, fastest axis first
    data: np.ndarray    # f32 values, or uint8 Q8_0 blocks


@dataclass
class Model:
    config: EncoderConfig
    tensors: list = field(default_factory=list)

    def table(self):
        """ctypes array of ScTensor pointing into this model's arrays (keep
        the Model alive while the table is in use)."""
        arr = (ScTensor * len(self.tensors))()
        self._names = [t.name.encode() for t in self.tensors]
        for i, t in enumerate(self.tensors):
            dims = (ctypes.c_int64 * 4)(*(list(t.dims) + [1] * (4 - len(t.dims))))
            arr[i] = ScTensor(self._names[i], t.dtype, len(t.dims), dims, t.data.ctypes.data)
        return arr

    def get(self, name: str) -> Tensor:
        for t in self.tensors:
            if t.name == name:
                return t
        raise KeyError(name)


PROMPT_HIDDEN = 2048  # prompt_intermediate (nemotron/config.rs:181, encoder.rs:268)


def random_model(cfg: EncoderConfig, seed: int = synth.SEED_BASE + 3, linear_pos_bias: bool = False) -> Model:
    """Random-init model of `cfg`, bit-identical for a given seed.  With
    cfg.n_prompts > 0 it also holds the multilingual prompt MLP
    prompt_kernel.0 [d + n_prompts -> 2048] and prompt_kernel.2 [2048 -> d]
    (nemotron/encoder.rs:260-270)."""
    d, dff, C, k = cfg.d_model, cfg.d_ff, cfg.conv_channels, cfg.conv_kernel
    m = Model(cfg)
    ctr = [seed * 1000]

    def nxt():
        ctr[0] += 1
        return ctr[0]

    def f32(name, dims, std, mean=0.0):
        n = int(np.prod(dims))
        m.tensors.append(Tensor(name, 0, tuple(dims), synth.normal(nxt(), (n,), std=std, mean=mean)))

    def lin(name, inp, out, bias=True):
        q = synth.q8_weights(nxt(), out, inp)
        m.tensors.append(Tensor(name + ".weight", 8, (inp, out), np.ascontiguousarray(q)))
        if bias:
            f32(name + ".bias", (out,), 0.02)

    def ln(name, dim):
        f32(name + ".weight", (dim,), 0.02, 1.0)
        f32(name + ".bias", (dim,), 0.02)

    pc = "encoder.pre_encode.conv."
    f32(pc + "0.weight", (3, 3, 1, C), 1.0 / 3.0)
    f32(pc + "0.bias", (C,), 0.02)
    f32(pc + "2.weight", (3, 3, 1, C), 1.0 / 3.0)
    f32(pc + "2.bias", (C,), 0.02)
    f32(pc + "3.weight", (1, 1, C, C), 1.0 / math.sqrt(C))
    f32(pc + "3.bias", (C,), 0.02)
    f32(pc + "5.weight", (3, 3, 1, C), 1.0 / 3.0)
    f32(pc + "5.bias", (C,), 0.02)
    f32(pc + "6.weight", (1, 1, C, C), 1.0 / math.sqrt(C))
    f32(pc + "6.bias", (C,), 0.02)
    f_final = cfg.feat_in
    for _ in range(3):
        f_final = (f_final + 3 - 3) // 2 + 1
    lin("encoder.pre_encode.out", f_final * C, d)
    for i in range(cfg.n_layers):
        p = f"encoder.layers.{i}."
        ln(p + "norm_feed_forward1", d)
        lin(p + "feed_forward1.linear1", d, dff)
        lin(p + "feed_forward1.linear2", dff, d)
        ln(p + "norm_self_att", d)
        lin(p + "self_attn.linear_q", d, d)
        lin(p + "self_attn.linear_k", d, d)
        lin(p + "self_attn.linear_v", d, d)
        lin(p + "self_attn.linear_pos", d, d, bias=linear_pos_bias)
        lin(p + "self_attn.linear_out", d, d)
        f32(p + "self_attn.pos_bias_u", (cfg.n_heads * (d // cfg.n_heads),), 0.02)
        f32(p + "self_attn.pos_bias_v", (cfg.n_heads * (d // cfg.n_heads),), 0.02)
        ln(p + "norm_conv", d)
        lin(p + "conv.pointwise_conv1", d, 2 * d)
        f32(p + "conv.depthwise_conv.weight", (k, 1, d), 1.0 / math.sqrt(k))
        ln(p + "conv.batch_norm", d)
        lin(p + "conv.pointwise_conv2", d, d)
        ln(p + "norm_feed_forward2", d)
        lin(p + "feed_forward2.linear1", d, dff)
        lin(p + "feed_forward2.linear2", dff, d)
        ln(p + "norm_out", d)
    if cfg.n_prompts > 0:
        lin("prompt_kernel.0", d + cfg.n_prompts, PROMPT_HIDDEN)
        lin("prompt_kernel.2", PROMPT_HIDDEN, d)
    return m


@dataclass
class RnntConfig:
    """RnntConfig (nemotron/config.rs:41-53) of the greedy RNN-T decoder:
    the predictor's embedding and LSTM width `hidden`, its layers, the joint
    width, the classes (vocabulary + blank) and max symbols per frame."""
    d_enc: int = 1024
    hidden: int = 640
    n_layers: int = 2
    joint: int = 640
    vocab: int = 1025
    blank: int = 1024
    max_symbols: int = 10


class ScRnntConfig(ctypes.Structure):
    _fields_ = [("d_enc", ctypes.c_int32), ("hidden", ctypes.c_int32), ("n_layers", ctypes.c_int32),
                ("joint", ctypes.c_int32), ("vocab", ctypes.c_int32), ("blank", ctypes.c_int32),
                ("max_symbols", ctypes.c_int32), ("max_frames", ctypes.c_int32)]

    @classmethod
    def of(cls, c: "RnntConfig", max_frames: int) -> "ScRnntConfig":
        return cls(c.d_enc, c.hidden, c.n_layers, c.joint, c.vocab, c.blank, c.max_symbols, max_frames)


def random_decoder(cfg: RnntConfig, seed: int = synth.SEED_BASE + 5, blank_bias: float = 1.3,
                   lstm_std: float = 0.08, pred_std: float = 0.1) -> Model:
    """Random-init RNN-T decoder with the reference's tensor names
    (nemotron/decoder.rs:75-235): embedding ~N(0, 1) (f32), LSTM linears
    Q8_0 ~N(0, lstm_std), joint.pred ~N(0, pred_std), joint.enc and the
    output linear ~N(0, 0.02), biases ~N(0, 0.02).  The wider LSTM and
    joint.pred weights give the predictor's output a weight in the joint
    comparable to the encoder frame's, as in a trained model; `blank_bias`
    is added to the blank class's output bias so that greedy decoding of
    N(0, 1) frames mixes blanks and emissions (random weights otherwise
    almost never pick the blank class)."""
    H, J = cfg.hidden, cfg.joint
    m = Model(cfg)
    ctr = [seed * 1000]

    def nxt():
        ctr[0] += 1
        return ctr[0]

    def f32(name, dims, std, add=None):
        n = int(np.prod(dims))
        v = synth.normal(nxt(), (n,), std=std)
        if add is not None:
            v[add[0]] += np.float32(add[1])
        m.tensors.append(Tensor(name, 0, tuple(dims), v))

    def lin(name, inp, out, bias=True, bias_add=None, std=0.02):
        q = synth.q8_weights(nxt(), out, inp, std=std)
        m.tensors.append(Tensor(name + ".weight", 8, (inp, out), np.ascontiguousarray(q)))
        if bias:
            f32(name + ".bias", (out,), 0.02, bias_add)

    f32("decoder.prediction.embed.weight", (H, cfg.vocab), 1.0)
    for i in range(cfg.n_layers):
        p = f"decoder.prediction.dec_rnn.lstm."
        lin(p + f"ih_l{i}", H, 4 * H, std=lstm_std)
        lin(p + f"hh_l{i}", H, 4 * H, std=lstm_std)
    lin("joint.enc", cfg.d_enc, J)
    lin("joint.pred", H, J, std=pred_std)
    lin("joint.joint_net.2", J, cfg.vocab, bias_add=(cfg.blank, blank_bias))
    return m


def mel_stream(seed: int, n_streams: int, n_frames: int, n_mels: int = 128) -> np.ndarray:
    """Seeded ~N(0, 1) log-mel input, [n_streams, n_frames, n_mels]."""
    return synth.normal(seed, (n_streams, n_frames, n_mels))
