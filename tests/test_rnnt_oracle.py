"""CPU checks of the oracle's RNN-T greedy decoder (nemotron/decoder.rs:75-235,
live.rs:56-145) and of the encoder's prompt MLP (streaming.rs:320-342)
against float64 numpy restatements and the properties of the loop."""
import numpy as np
import pytest

import oracle
from stealcode_b200 import model, synth

SMALL = model.RnntConfig(d_enc=256, hidden=128, n_layers=2, joint=128, vocab=65, blank=64, max_symbols=4)


def _deq(t):
    inp, out = t.dims
    return synth.dequant_q8_0(t.data.reshape(out, -1), inp).astype(np.float64)


def _weights(m):
    return {t.name: (_deq(t) if t.dtype == 8 else t.data.astype(np.float64)) for t in m.tensors}


def _sig(x):
    return 1.0 / (1.0 + np.exp(-x))


def _np_pred_step(W, cfg, tok, h, c):
    """Predictor::step (decoder.rs:142-205) in float64."""
    H = cfg.hidden
    x = W["decoder.prediction.embed.weight"].reshape(cfg.vocab, H)[tok] if tok >= 0 else np.zeros(H)
    nh, nc = [], []
    for l in range(cfg.n_layers):
        p = "decoder.prediction.dec_rnn.lstm."
        g = (W[p + f"ih_l{l}.weight"] @ x + W[p + f"hh_l{l}.weight"] @ h[l] + W[p + f"ih_l{l}.bias"] +
             W[p + f"hh_l{l}.bias"])
        i, f, gg, o = np.split(g, 4)
        cn = _sig(f) * c[l] + _sig(i) * np.tanh(gg)
        nh.append(_sig(o) * np.tanh(cn))
        nc.append(cn)
        x = nh[-1]
    return nh, nc


def _frames(seed, n, d):
    return synth.normal(seed, (n, d))


@pytest.fixture(scope="module")
def small_dec():
    return model.random_decoder(SMALL, blank_bias=0.21)


def test_predictor_state_matches_float64(small_dec):
    """After a decode, h/c equal a float64 replay of the emitted tokens'
    predictor steps (the state only advances on emissions)."""
    dec = oracle.RnntDecoder(small_dec)
    st = dec.new_state()
    ids, _ = dec.decode_frames(_frames(11, 12, SMALL.d_enc), st)
    assert len(ids) > 0
    W = _weights(small_dec)
    h = [np.zeros(SMALL.hidden)] * SMALL.n_layers
    c = [np.zeros(SMALL.hidden)] * SMALL.n_layers
    tok = -1
    for t in ids:
        h, c = _np_pred_step(W, SMALL, tok, h, c)
        tok = int(t)
    hg, cg, last = st.get()
    assert last == ids[-1]
    np.testing.assert_allclose(hg, np.array(h), atol=2e-2)
    np.testing.assert_allclose(cg, np.array(c), atol=2e-2)


def test_greedy_choice_matches_float64(small_dec):
    """The first emission decision of a fresh stream follows the float64
    joint: argmax of joint_net.2(relu(enc(x) + pred(h))) at frame 0 (only
    checked when the float64 margin is clear of rounding)."""
    W = _weights(small_dec)
    fr = _frames(12, 7, SMALL.d_enc)
    nh, _ = _np_pred_step(W, SMALL, -1, [np.zeros(SMALL.hidden)] * 2, [np.zeros(SMALL.hidden)] * 2)
    enc = W["joint.enc.weight"] @ fr[0] + W["joint.enc.bias"]
    pred = W["joint.pred.weight"] @ nh[-1] + W["joint.pred.bias"]
    logits = W["joint.joint_net.2.weight"] @ np.maximum(enc + pred, 0) + W["joint.joint_net.2.bias"]
    top2 = np.sort(logits)[-2:]
    if top2[1] - top2[0] < 1e-3:
        pytest.skip("float64 margin too small for this seed")
    best = int(np.argmax(logits))
    dec = oracle.RnntDecoder(small_dec)
    ids, steps = dec.decode_frames(fr[:1], dec.new_state())
    if best == SMALL.blank:
        assert len(ids) == 0
    else:
        assert ids[0] == best and steps[0] == 0


@pytest.mark.parametrize("scalar", [False, True])
def test_split_calls_equal_one_call(small_dec, scalar):
    """decode_frames carries its state: frames decoded as 5 + 6 emit what one
    call over 11 does (both <= 16 frames: the same GEMM order), with the
    steps of the second call counted from its own start."""
    fr = _frames(13, 11, SMALL.d_enc)
    dec = oracle.RnntDecoder(small_dec)
    dec.set_order(scalar_gemm=scalar, exp_cr=True)
    st1 = dec.new_state()
    ids1, steps1 = dec.decode_frames(fr, st1)
    st2 = dec.new_state()
    a, sa = dec.decode_frames(fr[:5], st2)
    b, sb = dec.decode_frames(fr[5:], st2)
    assert ids1.tolist() == a.tolist() + b.tolist()
    assert steps1.tolist() == sa.tolist() + (sb + 5).tolist()
    for x, y in zip(st1.get(), st2.get()):
        np.testing.assert_array_equal(x, y)


def test_all_blank_and_max_symbols():
    """A dominant blank emits nothing and leaves the state untouched; a
    suppressed blank emits exactly max_symbols tokens per frame."""
    fr = _frames(14, 6, SMALL.d_enc)
    dec = oracle.RnntDecoder(model.random_decoder(SMALL, blank_bias=100.0))
    st = dec.new_state()
    ids, _ = dec.decode_frames(fr, st)
    h, c, last = st.get()
    assert len(ids) == 0 and last == -1 and not h.any() and not c.any()
    dec = oracle.RnntDecoder(model.random_decoder(SMALL, blank_bias=-100.0))
    ids, steps = dec.decode_frames(fr, dec.new_state())
    assert len(ids) == 6 * SMALL.max_symbols
    assert steps.tolist() == [f for f in range(6) for _ in range(SMALL.max_symbols)]


def test_iteration_cap_raises():
    """With max_symbols 0 (no per-frame cap) and a suppressed blank the loop
    runs into 16 n + 64 iterations and fails like the reference's bail."""
    cfg = model.RnntConfig(**{**SMALL.__dict__, "max_symbols": 0})
    dec = oracle.RnntDecoder(model.random_decoder(cfg, blank_bias=-100.0))
    with pytest.raises(RuntimeError, match="iteration cap"):
        dec.decode_frames(_frames(15, 3, SMALL.d_enc), dec.new_state())


def test_missing_tensor_is_an_error():
    m = model.random_decoder(SMALL)
    m.tensors = [t for t in m.tensors if t.name != "joint.pred.weight"]
    with pytest.raises(RuntimeError, match="joint.pred"):
        oracle.RnntDecoder(m)


def test_tanh_modes_within_two_ulp():
    """libm tanhf (glibc 2.39 here) is not correctly rounded: it differs from
    the correctly rounded tanh by up to 2 ulp on about one input in eight."""
    xs = synth.normal(16, (2000,), std=3.0)
    lib = oracle.lib
    saved = lib.orc_get_exp_mode()
    try:
        lib.orc_set_exp_mode(0)
        a = np.array([lib.orc_tanhf(float(x)) for x in xs], dtype=np.float32)
        lib.orc_set_exp_mode(1)
        b = np.array([lib.orc_tanhf(float(x)) for x in xs], dtype=np.float32)
    finally:
        lib.orc_set_exp_mode(saved)
    ulps = np.abs(a.view(np.int32).astype(np.int64) - b.view(np.int32).astype(np.int64))
    assert ulps.max() <= 2


# ---- prompt MLP ----------------------------------------------------------
ENC = model.EncoderConfig(d_model=256, n_layers=1, n_heads=4, d_ff=512, conv_channels=32, att_left=14,
                          n_prompts=32)


@pytest.fixture(scope="module")
def prompt_model():
    return model.random_model(ENC)


def _run(m, prompt):
    e = oracle.StreamingEncoder(m)
    e.set_prompt(prompt)
    mel = model.mel_stream(21, 1, 64, ENC.feat_in)[0]
    for t0 in range(0, 64, 56):
        e.encode_new(mel[: min(t0 + 56, 64)], t0, min(t0 + 56, 64))
    return e.frames(0, e.total())


def test_prompt_none_is_identity(prompt_model):
    plain = model.Model(ENC, [t for t in prompt_model.tensors if not t.name.startswith("prompt_kernel")])
    np.testing.assert_array_equal(_run(prompt_model, None), _run(plain, None))


def test_prompt_mlp_matches_float64(prompt_model):
    """out = prompt2(relu(prompt0([x ; onehot(id)]))) over the frames the
    blocks produced (float64 restatement from the same x)."""
    x = _run(prompt_model, None).astype(np.float64)
    y = _run(prompt_model, 5)
    W = _weights(prompt_model)
    onehot = np.zeros((x.shape[0], ENC.n_prompts))
    onehot[:, 5] = 1.0
    h = np.maximum(np.concatenate([x, onehot], 1) @ W["prompt_kernel.0.weight"].T + W["prompt_kernel.0.bias"], 0)
    ref = h @ W["prompt_kernel.2.weight"].T + W["prompt_kernel.2.bias"]
    rms = np.sqrt(np.mean(ref ** 2))
    assert np.abs(y - ref).max() < 0.05 * rms


def test_prompt_out_of_range(prompt_model):
    e = oracle.StreamingEncoder(prompt_model)
    with pytest.raises(ValueError):
        e.set_prompt(ENC.n_prompts)
