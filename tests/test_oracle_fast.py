"""The oracle's fast mode -- the reference's threading (rayon over 256-row
chunks, output positions and queries) and AVX2 lanes for the f32 GEMM,
score_dot and softmax_v -- against its serial scalar restatement: every
output bit for bit.  The fast mode is what the timed CPU baseline runs."""
import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.skipif(not oracle.have_avx2(), reason="host without AVX2 + FMA")


def _both(fn):
    saved = oracle.get_fast()
    try:
        oracle.set_fast(False)
        slow = fn()
        oracle.set_fast(True)
        fast = fn()
    finally:
        oracle.set_fast(saved)
    return slow, fast


def _bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


@pytest.mark.parametrize("m,k,n", [(256, 256, 693), (256, 256, 187), (264, 48, 35), (13, 40, 7),
                                   (520, 33, 48), (300, 19, 3)])
def test_gemm_simd_into_fast_equals_serial(m, k, n):
    rng = np.random.default_rng(m * 7 + k + n)
    a = (rng.standard_normal((m, k)) * 0.06).astype(np.float32)
    b = np.maximum(rng.standard_normal((k, n)), 0).astype(np.float32)
    slow, fast = _both(lambda: oracle.gemm_simd_into(a, b))
    assert np.array_equal(_bits(slow), _bits(fast))


@pytest.mark.parametrize("hd", [64, 128, 72])
def test_score_dot_fast_equals_serial(hd):
    rng = np.random.default_rng(hd)
    vecs = [rng.standard_normal(hd).astype(np.float32) for _ in range(6)]
    for scale in (0.088388, 1.0):
        slow, fast = _both(lambda: oracle.score_dot(*vecs, scale))
        assert np.float32(slow).view(np.uint32) == np.float32(fast).view(np.uint32)


@pytest.mark.parametrize("hd", [128, 40])
def test_softmax_v_fast_equals_serial(hd):
    rng = np.random.default_rng(hd + 1)
    nh, band = 8, 77
    srow = rng.standard_normal(band * nh).astype(np.float32) * 3
    v_rows = rng.standard_normal((band, hd)).astype(np.float32)
    for k0, k1, h in [(0, 77, 0), (7, 70, 5)]:
        slow, fast = _both(lambda: oracle.softmax_v(srow, k0, k1, nh, h, v_rows, hd))
        assert np.array_equal(_bits(slow), _bits(fast))


def test_encoder_fast_equals_serial():
    """A 2-layer encoder for 12 chunks of one stream: the direct convs on
    the pool, the pointwise convs through the AVX2 GEMM, the attention over
    queries once c * band * n_heads >= 2048 (band 37+, from the 6th chunk),
    the Q8 linears on all threads -- every output frame and the phase timers
    against the serial scalar run."""
    from stealcode_b200 import model

    m = model.random_model(model.EncoderConfig(n_layers=2), seed=5)
    steps, per = 12, 56
    mel = model.mel_stream(6, 1, per * steps, m.config.feat_in)[0]

    def run():
        enc = oracle.StreamingEncoder(m)
        for i in range(steps):
            assert enc.encode_new(mel[:per * (i + 1)], per * i, per * (i + 1)) == 0
        out = enc.frames(0, enc.total())
        times = enc.phase_times()
        return out, times

    (slow, t_slow), (fast, t_fast) = _both(run)
    assert slow.shape == fast.shape == (7 * steps, m.config.d_model)
    assert np.array_equal(_bits(slow), _bits(fast))
    for t in (t_slow, t_fast):
        assert t["total"] > 0 and 0 < t["pre_encode"] < t["total"]
        assert t["linears"] > 0 and t["attention"] > 0
        assert t["pre_encode"] + t["linears"] + t["attention"] <= t["total"] * 1.001
