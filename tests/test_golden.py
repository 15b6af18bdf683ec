"""The committed golden fixtures (tests/golden/golden.npz, written by
tests/golden/make_golden.py from the reference tests' input generators) are
reproduced bit for bit by the oracle, so the oracle the GPU tests check
against has not drifted from what was frozen."""
import numpy as np

from tests.golden import make_golden


def test_oracle_reproduces_golden_fixtures():
    frozen = np.load(make_golden.os.path.join(make_golden.HERE, "golden.npz"))
    now = make_golden.compute()
    assert sorted(frozen.files) == sorted(now)
    for key in frozen.files:
        a, b = frozen[key], now[key]
        assert a.shape == b.shape and a.dtype == b.dtype, key
        assert np.array_equal(a.view(np.uint8), b.view(np.uint8)), key


def test_golden_fixture_sanity():
    """Properties of the frozen outputs themselves: the SIMD and scalar
    orders agree within the reference tests' bar, the quantiser's codes stay
    in [-127, 127] with positive scales, the attention output is finite."""
    g = np.load(make_golden.os.path.join(make_golden.HERE, "golden.npz"))
    for m, k, n in make_golden.pattern_cases():
        s, v = g[f"pattern_{m}_{k}_{n}"], g[f"pattern_{m}_{k}_{n}_simd"]
        assert np.all(np.abs(v - s) <= 1e-3 * (1 + np.abs(s)))
    q, d = g["quant_2048_16_q"], g["quant_2048_16_d"]
    assert q.dtype == np.int8 and int(np.abs(q.astype(np.int32)).max()) <= 127 and np.all(d > 0)
    assert np.all(np.isfinite(g["attn_ref"]))
