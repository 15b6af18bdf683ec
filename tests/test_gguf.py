"""GGUF checkpoints in the reference's layout (gguf.rs): writer/reader round
trips, the reference's dtype quirks, metadata -> EncoderConfig, and an
encoder built from a file computing the same bits as one built in memory
(oracle, CPU)."""
import struct

import numpy as np
import pytest

import oracle
from stealcode_b200 import gguf, model, synth

SMALL = dict(d_model=256, n_layers=1, n_heads=4, d_ff=512, feat_in=64, conv_channels=16, conv_kernel=9)


@pytest.fixture(scope="module")
def small_model():
    return model.random_model(model.EncoderConfig(**SMALL), seed=21)


def test_model_round_trip(tmp_path, small_model):
    path = str(tmp_path / "enc.gguf")
    gguf.save_model(small_model, path)
    with gguf.open_gguf(path) as g:
        m2 = gguf.model_from_gguf(g)
        assert m2.config == small_model.config
        assert [t.name for t in m2.tensors] == [t.name for t in small_model.tensors]
        for a, b in zip(small_model.tensors, m2.tensors):
            assert a.dtype == b.dtype and tuple(a.dims) == b.dims
            assert np.array_equal(np.ascontiguousarray(a.data).view(np.uint8).reshape(-1),
                                  np.ascontiguousarray(b.data).view(np.uint8).reshape(-1))
        assert g.data_start % 32 == 0 and all(t.offset % 32 == 0 for t in g.tensors)
        del m2


def test_q8_f16_dequant_matches_synth(tmp_path):
    k, rows = 80, 6  # rows padded to 3 blocks
    w = synth.normal(5, (rows, k), std=0.02)
    blocks = synth.quantize_q8_0(w)
    t = model.Tensor("encoder.w", gguf.Q8_0_F16, (k, rows), blocks)
    path = str(tmp_path / "q.gguf")
    gguf.write_gguf(path, {}, [t])
    with gguf.open_gguf(path) as g:
        got = g.read_f32(g.tensor("encoder.w")).reshape(rows, k)
    assert np.array_equal(got, synth.dequant_q8_0(blocks, k))


def test_q8_f32_and_f16_dtypes(tmp_path):
    # Q8_0 with an f32 scale (36-byte blocks) and a plain f16 tensor
    rng = np.random.default_rng(1)
    q = rng.integers(-127, 128, size=(2, 32)).astype(np.int8)
    scale = np.array([0.5, -0.25], dtype="<f4")
    blk = np.concatenate([scale.view(np.uint8).reshape(2, 4), q.view(np.uint8)], axis=1)
    h = np.array([1.0, -2.5, 65504.0, 2.0 ** -24], dtype="<f2")
    tensors = [model.Tensor("a", gguf.Q8_0_F32, (32, 2), blk), model.Tensor("b", gguf.F16, (4,), h.view(np.uint8))]
    path = str(tmp_path / "t.gguf")
    gguf.write_gguf(path, {}, tensors)
    with gguf.open_gguf(path) as g:
        assert np.array_equal(g.read_f32(g.tensor("a")).reshape(2, 32), scale[:, None] * q.astype(np.float32))
        assert np.array_equal(g.read_f32(g.tensor("b")), h.astype(np.float32))


def test_kv_value_types(tmp_path):
    kv = {"u": 7, "i": -3, "f": 1.5, "b": True, "s": "causal", "as": ["auto:0", "en:1"], "ai": [1, 2, 3],
          "af": [0.5, 0.25]}
    path = str(tmp_path / "kv.gguf")
    gguf.write_gguf(path, kv, [])
    with gguf.open_gguf(path) as g:
        assert g.kv == {"u": 7, "i": -3, "f": 1.5, "b": 1, "s": "causal", "as": ["auto:0", "en:1"],
                        "ai": [1, 2, 3], "af": [0.5, 0.25]}


def test_reference_quirks_dtype_after_dims(tmp_path):
    # hand-built file: one f32 tensor, dtype written after the dims, data at
    # the table end rounded up to 32
    name = b"x"
    head = struct.pack("<IIQQ", gguf.GGUF_MAGIC, 3, 1, 0) + struct.pack("<Q", 1) + name
    head += struct.pack("<I", 2) + struct.pack("<QQ", 3, 2) + struct.pack("<IQ", 0, 0)
    pad = (-len(head)) % 32
    vals = np.arange(6, dtype="<f4")
    p = tmp_path / "h.gguf"
    p.write_bytes(head + b"\0" * pad + vals.tobytes())
    with gguf.open_gguf(str(p)) as g:
        t = g.tensor("x")
        assert t.dims == (3, 2) and t.dtype == 0 and g.data_start == len(head) + pad
        assert np.array_equal(g.read_f32(t), vals)


def test_errors(tmp_path):
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"NOPE" + b"\0" * 28)
    with pytest.raises(gguf.GgufError, match="magic"):
        gguf.open_gguf(str(bad))
    short = tmp_path / "short.gguf"
    short.write_bytes(struct.pack("<IIQQ", gguf.GGUF_MAGIC, 3, 5, 0))
    with pytest.raises(gguf.GgufError, match="end of file"):
        gguf.open_gguf(str(short))
    empty = tmp_path / "empty.gguf"
    empty.write_bytes(b"")
    with pytest.raises(gguf.GgufError):
        gguf.open_gguf(str(empty))
    with pytest.raises(gguf.GgufError, match="bytes"):
        gguf.write_gguf(str(tmp_path / "w.gguf"), {}, [model.Tensor("w", gguf.F32, (4,), np.zeros(3, np.float32))])


def test_encoder_config_from_metadata(tmp_path, small_model):
    path = str(tmp_path / "enc.gguf")
    gguf.save_model(small_model, path, extra_kv={"asr.encoder.conv_context": "same"})
    with gguf.open_gguf(path) as g, pytest.raises(gguf.GgufError, match="causal"):
        gguf.encoder_config(g)


def test_oracle_encoder_from_file_matches_memory(tmp_path, small_model):
    path = str(tmp_path / "enc.gguf")
    gguf.save_model(small_model, path)
    mel = model.mel_stream(3, 1, 112, small_model.config.feat_in)[0]
    with gguf.open_gguf(path) as g:
        m2 = gguf.model_from_gguf(g)
        a, b = oracle.StreamingEncoder(small_model), oracle.StreamingEncoder(m2)
        for t0, t1 in ((0, 56), (56, 112)):
            assert a.encode_new(mel[:t1], t0, t1) == 0 and b.encode_new(mel[:t1], t0, t1) == 0
        assert np.array_equal(a.frames(0, a.total()), b.frames(0, b.total()))
        del a, b, m2


def test_encoder_decoder_checkpoint(tmp_path):
    """One file with the encoder (prompt MLP included) and the RNN-T decoder:
    configs from the metadata, and the oracle decoder built from the file
    emits what the in-memory one does."""
    enc = model.random_model(model.EncoderConfig(**SMALL, n_prompts=32), seed=22)
    dcfg = model.RnntConfig(d_enc=256, hidden=128, n_layers=2, joint=128, vocab=65, blank=64, max_symbols=4)
    dec = model.random_decoder(dcfg, blank_bias=0.21)
    path = str(tmp_path / "asr.gguf")
    gguf.save_model(enc, path, decoder=dec)
    with gguf.open_gguf(path) as g:
        e2, d2 = gguf.model_from_gguf(g), gguf.decoder_from_gguf(g)
        assert e2.config == enc.config and e2.config.n_prompts == 32
        assert d2.config == dcfg
        assert {t.name for t in e2.tensors} == {t.name for t in enc.tensors}
        assert {t.name for t in d2.tensors} == {t.name for t in dec.tensors}
        fr = synth.normal(23, (12, 256))
        a, b = oracle.RnntDecoder(dec), oracle.RnntDecoder(d2)
        ra, rb = a.decode_frames(fr, a.new_state()), b.decode_frames(fr, b.new_state())
        assert ra[0].tolist() == rb[0].tolist() and ra[1].tolist() == rb[1].tolist()
        del a, b, e2, d2
