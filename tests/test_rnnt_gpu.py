"""GPU parity of the device RNN-T greedy decoder (decode_frames, live.rs:56-145,
over the predictor LSTM and joint of nemotron/decoder.rs:75-235) against the
oracle decoder, one oracle state per stream, on seeded random-init weights
and N(0, 1) encoder frames.

The device follows the reference's GEMM dispatch (the 8-lane SIMD order for
n <= 16 GEMMs with rows % 8 == 0, q8_gemm_scalar's order otherwise) and
rounds exp and tanh correctly; the oracle in that mode (exp_cr) must agree
bit for bit: the same tokens at the same steps and the same LSTM state.
Against the oracle with glibc's expf/tanhf (the reference's libm) the
tokens may differ only where a logit margin is within those last-ulp
differences; that rate is reported, not asserted."""
import numpy as np
import pytest

import oracle
from stealcode_b200 import _lib, model, synth

pytestmark = pytest.mark.gpu

FULL = model.RnntConfig()  # hidden 640, 2 layers, joint 640, 1025 classes
SMALL = model.RnntConfig(d_enc=256, hidden=128, n_layers=2, joint=128, vocab=65, blank=64, max_symbols=4)


@pytest.fixture(scope="module")
def torch():
    import torch as _t

    assert _t.cuda.is_available()
    return _t


def run(torch, m, n_streams, chunks, seed, libm_too=False, max_frames=16):
    """Decodes the same frames on the device and per-stream oracles; chunks
    is the list of frame counts per call.  Returns the per-call token lists
    and the mismatch count against the glibc-libm oracle."""
    from stealcode_b200.ops import RnntDecoder

    cfg = m.config
    dev = RnntDecoder(m, n_streams, max_frames=max_frames)
    ref = oracle.RnntDecoder(m)
    ref.set_order(scalar_gemm=False, exp_cr=True)
    states = [ref.new_state() for _ in range(n_streams)]
    alt = oracle.RnntDecoder(m) if libm_too else None
    alt_states = [alt.new_state() for _ in range(n_streams)] if libm_too else []
    diff, out = 0, []
    for ci, n in enumerate(chunks):
        fr = synth.normal(seed + ci, (n_streams, n, cfg.d_enc))
        dev.decode_frames(torch.from_numpy(fr).cuda())
        call = []
        for z in range(n_streams):
            ids, steps = dev.tokens(z)
            rids, rsteps = ref.decode_frames(fr[z], states[z])
            assert ids.tolist() == rids.tolist(), (ci, z)
            assert steps.tolist() == rsteps.tolist(), (ci, z)
            h, c, last = dev.state(z)
            rh, rc, rlast = states[z].get()
            assert last == rlast
            np.testing.assert_array_equal(h, rh)
            np.testing.assert_array_equal(c, rc)
            if libm_too:
                a, _ = alt.decode_frames(fr[z], alt_states[z])
                diff += a.tolist() != rids.tolist()
            call.append(ids.tolist())
        out.append(call)
    dev.close()
    return out, diff


def test_small_decoder_matches_oracle(torch):
    """6 streams, 7-frame calls (the encoder's chunk), a short final call."""
    m = model.random_decoder(SMALL, blank_bias=0.21)
    out, _ = run(torch, m, 6, [7] * 8 + [3], seed=100)
    assert sum(len(t) for call in out for t in call) > 10


def test_full_decoder_matches_oracle(torch):
    """The Nemotron decoder's shapes (2 x 640 LSTM, joint 640, 1025 classes:
    joint.out in q8_gemm_scalar's order since 1025 % 8 != 0), 5 streams."""
    m = model.random_decoder(FULL)
    out, diff = run(torch, m, 5, [7] * 6, seed=200, libm_too=True)
    emitted = sum(len(t) for call in out for t in call)
    print(f"full decoder: {emitted} tokens; calls differing from the glibc-libm oracle: {diff} of {6 * 5}")
    assert emitted > 10


def test_long_calls_use_scalar_enc_order(torch):
    """n > 16 frames in one call: joint.enc takes q8_gemm_scalar's order."""
    m = model.random_decoder(SMALL, blank_bias=0.21)
    run(torch, m, 3, [17, 5, 20], seed=300, max_frames=20)


def test_all_blank_and_symbol_cap(torch):
    """A dominant blank emits nothing; a suppressed blank emits exactly
    max_symbols tokens per frame (every stream in lockstep)."""
    m = model.random_decoder(SMALL, blank_bias=100.0)
    out, _ = run(torch, m, 3, [7, 7], seed=400)
    assert all(t == [] for call in out for t in call)
    m = model.random_decoder(SMALL, blank_bias=-100.0)
    out, _ = run(torch, m, 3, [5], seed=401)
    assert all(len(t) == 5 * SMALL.max_symbols for t in out[0])


def test_iteration_cap_is_an_error(torch):
    """max_symbols 0 with a suppressed blank runs into 16 n + 64 iterations:
    SC_ERR_STATE, as the reference's bail."""
    from stealcode_b200.ops import RnntDecoder

    cfg = model.RnntConfig(**{**SMALL.__dict__, "max_symbols": 0})
    dev = RnntDecoder(model.random_decoder(cfg, blank_bias=-100.0), 2, max_frames=8)
    with pytest.raises(_lib.ScError) as e:
        dev.decode_frames(torch.from_numpy(synth.normal(500, (2, 3, cfg.d_enc))).cuda())
    assert e.value.code == _lib.SC_ERR_STATE and "iteration cap" in str(e.value)
    ids, _ = dev.tokens(0)
    assert len(ids) == 16 * 3 + 64
    dev.close()


def test_reset_one_stream(torch):
    """reset(z) restarts one stream's state (StreamState::new) and leaves
    the others alone."""
    from stealcode_b200.ops import RnntDecoder

    m = model.random_decoder(SMALL, blank_bias=0.21)
    dev = RnntDecoder(m, 3)
    ref = oracle.RnntDecoder(m)
    ref.set_order(exp_cr=True)
    st = [ref.new_state() for _ in range(3)]
    for ci in range(4):
        fr = synth.normal(600 + ci, (3, 7, SMALL.d_enc))
        if ci == 2:
            dev.reset(1)
            st[1] = ref.new_state()
        dev.decode_frames(torch.from_numpy(fr).cuda())
        for z in range(3):
            assert dev.tokens(z)[0].tolist() == ref.decode_frames(fr[z], st[z])[0].tolist()
    dev.close()


def test_encoder_to_decoder_on_device(torch):
    """The device pipeline: encoder output frames straight into the decoder
    (no host copy), against the oracle encoder (device rounding) feeding the
    oracle decoder."""
    from stealcode_b200.ops import RnntDecoder, StreamEncoder

    ecfg = model.EncoderConfig(n_layers=2)
    em = model.random_model(ecfg, seed=31)
    dm = model.random_decoder(FULL)
    Z = 3
    mel = model.mel_stream(32, Z, 56 * 4, ecfg.feat_in)
    enc = StreamEncoder(em, Z)
    dec = RnntDecoder(dm, Z, max_frames=ecfg.max_frames)
    oenc = [oracle.StreamingEncoder(em) for _ in range(Z)]
    for e in oenc:
        e.set_device_rounding()
    odec = oracle.RnntDecoder(dm)
    odec.set_order(exp_cr=True)
    ost = [odec.new_state() for _ in range(Z)]
    for i in range(4):
        t0, t1 = 56 * i, 56 * (i + 1)
        s = enc.total()
        enc.encode_new(torch.from_numpy(np.ascontiguousarray(mel[:, t0:t1])).cuda(), t0, t1)
        ptr, rows, _ = enc.output()
        dec.decode_frames((ptr, rows // Z))
        for z in range(Z):
            assert oenc[z].encode_new(mel[z, :t1], t0, t1) == 0
            fr = oenc[z].frames(s, oenc[z].total())
            assert dec.tokens(z)[0].tolist() == odec.decode_frames(fr, ost[z])[0].tolist()
    enc.close()
    dec.close()


def test_decoder_from_gguf_matches_memory(torch, tmp_path):
    """A device decoder built from a GGUF checkpoint emits what one built in
    memory does."""
    from stealcode_b200 import gguf
    from stealcode_b200.ops import RnntDecoder

    em = model.random_model(model.EncoderConfig(n_layers=0), seed=41)
    dm = model.random_decoder(FULL)
    path = str(tmp_path / "asr.gguf")
    gguf.save_model(em, path, decoder=dm)
    a, b = RnntDecoder(dm, 2, max_frames=8), RnntDecoder.from_gguf(path, 2, max_frames=8)
    for ci in range(3):
        fr = torch.from_numpy(synth.normal(700 + ci, (2, 7, FULL.d_enc))).cuda()
        a.decode_frames(fr)
        b.decode_frames(fr)
        assert a.emitted().tolist() == b.emitted().tolist()
        for z in range(2):
            assert a.tokens(z)[0].tolist() == b.tokens(z)[0].tolist()
    a.close()
    b.close()
