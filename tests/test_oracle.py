"""CPU tests of the oracle: pinned against the reference's own test cases and
against known answers derived by hand from the reference's arithmetic.

The reference stores no golden outputs (its tests compare two in-tree
implementations) and it cannot be built here (Rust nightly, no cargo), so
the oracle is pinned by (a) reproducing each of those self-consistency
tests with the reference's generators and tolerances, (b) analytic
known-answer cases, and (c) the committed fixtures in tests/golden/.
"""
import math

import numpy as np
import pytest

import oracle
from tests import refcases

TOL = 1e-3  # the reference tests' |d| <= 1e-3 * (1 + |ref|)


# ---- f16 decode (gguf.rs:365-397) ----------------------------------------
def test_f16_to_f32_all_values():
    h = np.arange(65536, dtype=np.uint32)
    want = h.astype(np.uint16).view(np.float16).astype(np.float32)
    got = np.array([oracle.f16_to_f32(int(v)) for v in h], dtype=np.float32)
    nan = np.isnan(want)
    assert np.array_equal(np.isnan(got), nan)
    assert np.array_equal(got[~nan].view(np.uint32), want[~nan].view(np.uint32))
    # NaN payload rule of the reference: quiet bit set, mantissa << 13
    assert np.float32(oracle.f16_to_f32(0x7C01)).view(np.uint32) == 0x7FC02000


def test_half_from_f32_trunc():
    assert oracle.half_from_f32_trunc(0.0125) == refcases.half_f32_to_u16(0.0125)
    assert oracle.half_from_f32_trunc(0.03125) == 0x2800
    assert oracle.half_from_f32_trunc(1e-9) == 0  # flushed below the normal range


# ---- quantize_col known answers (sgemm_kernel.rs:57-90) -------------------
def _quant_col(vals):
    x = np.asarray(vals, dtype=np.float32).reshape(-1, 1)
    xq, dx = oracle.quantize(x)
    return xq[0], dx[0]


def test_quantize_zero_block():
    xq, dx = _quant_col([0.0] * 32)
    assert dx[0] == 1.0 and not xq.any()


def test_quantize_half_away_from_zero():
    # amax 127 -> s = 1, inv = 1: codes are round-half-away of x itself
    vals = [127.0, -63.5, 0.5, -0.5, 2.5, -2.5, 1.49, -126.5] + [0.0] * 24
    xq, dx = _quant_col(vals)
    assert dx[0] == 1.0
    assert list(xq[:8]) == [127, -64, 1, -1, 3, -3, 1, -127]


def test_quantize_nan_and_inf():
    xq, dx = _quant_col([np.nan, 3.0, -6.35] + [0.0] * 29)
    assert dx[0] == np.float32(6.35) / np.float32(127.0)
    assert xq[0] == 0 and xq[2] == -127
    xq, dx = _quant_col([np.inf, 1.0] + [0.0] * 30)
    assert np.isinf(dx[0]) and not xq.any()  # inv = 0: finite -> 0, inf*0 = NaN -> 0
    xq, dx = _quant_col([np.nan] * 32)
    assert dx[0] == 1.0 and not xq.any()


def test_quantize_denormal_block():
    # s = amax/127 is subnormal and 1/s overflows to inf: x*inf saturates.
    xq, dx = _quant_col([1e-40, -1e-40] + [0.0] * 30)
    assert dx[0] == np.float32(1e-40) / np.float32(127.0)
    assert xq[0] == 127 and xq[1] == -128 and xq[2] == 0


def test_quantize_ragged_tail():
    x = np.linspace(-1, 1, 45, dtype=np.float32).reshape(45, 1)
    xq, dx = oracle.quantize(x)
    assert xq.shape == (1, 45) and dx.shape == (1, 2)
    tail = x[32:, 0]
    s = np.float32(np.abs(tail).max()) / np.float32(127.0)
    assert dx[0, 1] == s


# ---- GEMM: the reference's vnni_matches_scalar / simd_matches_scalar ------
@pytest.mark.parametrize("m,k,n", refcases.VNNI_CASES)
def test_vnni_matches_scalar(m, k, n):
    w, pr, x = refcases.gemm_pattern_case(m, k, n)
    ref = oracle.q8_gemm_scalar(m, k, n, w, pr, 34, 2, x)
    got = oracle.q8_gemm(m, k, n, w, pr, 34, 2, x)
    assert np.all(np.abs(got - ref) <= TOL * (1 + np.abs(ref)))
    # the threaded AVX2 baseline reproduces the SIMD accumulation order exactly
    assert np.array_equal(got, oracle.q8_gemm_simd_order(m, k, n, w, pr, 34, 2, x))


@pytest.mark.parametrize("m,k,n", refcases.SIMD_CASES)
def test_simd_matches_scalar(m, k, n):
    w, pr, x = refcases.gemm_pattern_case(m, k, n)
    ref = oracle.q8_gemm_scalar(m, k, n, w, pr, 34, 2, x)
    got = oracle.q8_gemm_simd_order(m, k, n, w, pr, 34, 2, x)
    assert np.all(np.abs(got - ref) <= TOL * (1 + np.abs(ref)))


def test_gemm_thread_counts_agree():
    w, pr, x = refcases.gemm_pattern_case(512, 2048, 16)
    one = oracle.q8_gemm(512, 2048, 16, w, pr, 34, 2, x, nthreads=1)
    for t in (2, 3, 0):
        assert np.array_equal(one, oracle.q8_gemm(512, 2048, 16, w, pr, 34, 2, x, nthreads=t))


def test_scalar_is_sum_of_block_dots():
    m, k, n = 16, 100, 3  # ragged k, scalar path
    w, pr, x = refcases.gemm_pattern_case(m, k, n)
    dots = oracle.q8_block_dots(m, k, n, w, pr, 34, 2, x)
    xq, dx = oracle.quantize(x)
    nb = (k + 31) // 32
    sc = w.reshape(m, nb, 34)[:, :, :2].copy().view(np.float16).reshape(m, nb).astype(np.float32)
    y = np.zeros((m, n), dtype=np.float32)
    for i in range(m):
        for j in range(n):
            acc = np.float32(0)
            for b in range(nb):
                acc = np.float32(acc + np.float32(sc[i, b] * dx[j, b]) * np.float32(dots[i, j, b]))
            y[i, j] = acc
    assert np.array_equal(y, oracle.q8_gemm_scalar(m, k, n, w, pr, 34, 2, x))


def test_gemm_zero_dims_noop():
    y = oracle.q8_gemm(0, 64, 1, np.zeros(0, np.uint8), 68, 34, 2, np.zeros((64, 1), np.float32))
    assert y.size == 0


# ---- attention helpers: helpers_match_scalar (simd_kernel.rs:1432-1688) ---
@pytest.mark.parametrize("hd", [64, 512, 128, 37])
def test_score_dot(hd):
    qu, uh, qv, vh, kk, p = refcases.score_case(hd)
    got = oracle.score_dot(qu, uh, qv, vh, kk, p, 0.125)
    acc = np.float32(0)
    for i in range(hd):
        acc = np.float32(acc + np.float32(np.float32(qu[i] + uh[i]) * kk[i])
                         + np.float32(np.float32(qv[i] + vh[i]) * p[i]))
    want = np.float32(acc * np.float32(0.125))
    assert abs(got - want) <= TOL * (1 + abs(want))


@pytest.mark.parametrize("band,hd,nh", [(16, 64, 8), (61, 64, 8), (96, 64, 8), (128, 512, 8)])
def test_softmax_v(band, hd, nh):
    srow, k0, k1, h, v = refcases.softmax_case(band, hd, nh)
    got = oracle.softmax_v(srow, k0, k1, nh, h, v, hd)
    s = srow.reshape(k1, nh)[k0:k1, h].astype(np.float64)
    e = np.exp(s - s.max())
    want = (e / e.sum()) @ v[k0:k1].astype(np.float64)
    assert np.all(np.abs(got - want) <= TOL * (1 + np.abs(want)))


def test_attn_matches_reference_testloop():
    """attn_stream_matches_reference (gpu/kernels.rs:1878-1988): the block_new
    restatement against the test's own CPU loop, tolerance 1e-4 abs."""
    cs = refcases.attn_case()
    args = [cs[k] for k in ("q", "kv", "vv", "pos_p", "q_bias", "v_bias", "c", "d", "n_heads", "scale",
                            "s", "k_lo")]
    a = oracle.attn_stream(*args, cs["band"], cs["chunk"], cs["left_chunks"], cs["k_hi"], cs["pos_off"])
    b = oracle.attn_stream_testloop(*args, cs["chunk"], cs["left_chunks"], cs["k_hi"], cs["pos_off"])
    assert np.max(np.abs(a - b)) < 1e-4


def test_attn_band_mask_is_exact():
    """Changing K/V outside a query's band must not change that query's output."""
    cs = refcases.attn_case()
    a = oracle.attn_stream(*[cs[k] for k in ("q", "kv", "vv", "pos_p", "q_bias", "v_bias", "c", "d",
                                               "n_heads", "scale", "s", "k_lo", "band", "chunk",
                                               "left_chunks", "k_hi", "pos_off")])
    kv2, vv2 = cs["kv"].copy(), cs["vv"].copy()
    # queries 16..19 (chunk 4) attend to frames [8, 20): frames 20..23 are masked for them
    kv2[12:] = 1e3
    vv2[12:] = -1e3
    b = oracle.attn_stream(cs["q"], kv2, vv2, *[cs[k] for k in ("pos_p", "q_bias", "v_bias", "c", "d",
                                                                 "n_heads", "scale", "s", "k_lo", "band",
                                                                 "chunk", "left_chunks", "k_hi",
                                                                 "pos_off")])
    assert np.array_equal(a[:4], b[:4])
    assert not np.allclose(a[4:], b[4:])


def test_exp_modes():
    """orc_expf: mode 0 is libm expf (the reference's f32::exp on glibc), mode
    1 the correctly rounded exp; they agree except in rare last-ulp cases."""
    import ctypes

    libm = ctypes.CDLL("libm.so.6")
    libm.expf.restype = ctypes.c_float
    libm.expf.argtypes = [ctypes.c_float]
    xs = np.random.default_rng(5).uniform(-20, 20, 20000).astype(np.float32)
    differ = 0
    for x in xs:
        x = float(x)
        glibc = oracle.expf(x, correctly_rounded=False)
        cr = oracle.expf(x, correctly_rounded=True)
        assert glibc == libm.expf(x)
        assert cr == np.float32(np.exp(np.float64(np.float32(x))))
        if glibc != cr:
            assert abs(np.float32(glibc).view(np.int32) - np.float32(cr).view(np.int32)) == 1
            differ += 1
    assert differ < 0.005 * len(xs)
    assert oracle.lib.orc_get_exp_mode() == 0


# ---- the pointwise convs' f32 GEMM (simd_kernel.rs:448-727) ----------------
def _fma32(a, b, c):
    """Correctly rounded f32 fused multiply-add of float32 arrays: the
    product is exact in float64, the sum's rounding error comes from
    TwoSum, and it decides the one case where rounding the float64 sum to
    f32 differs from rounding the exact sum (an exact f32 halfway point)."""
    a64, b64, c64 = (np.asarray(v, np.float32).astype(np.float64) for v in (a, b, c))
    p = a64 * b64
    s = p + c64
    bb = s - p
    err = (p - (s - bb)) + (c64 - bb)
    r = s.astype(np.float32)
    r64 = r.astype(np.float64)
    up = np.nextafter(r, np.float32(np.inf))
    dn = np.nextafter(r, np.float32(-np.inf))
    half_up = (up.astype(np.float64) - r64) / 2
    half_dn = (r64 - dn.astype(np.float64)) / 2
    d = s - r64
    above = (d == half_up) & (err != 0)   # s is the midpoint between r and up
    below = (d == -half_dn) & (err != 0)  # s is the midpoint between dn and r
    r = np.where(above & (err > 0), up, np.where(above & (err < 0), r, r))
    r = np.where(below & (err < 0), dn, r)
    return r.astype(np.float32)


def _gemm_tile8_cols_tail(a, b):
    """gemm_tile8 (simd_kernel.rs:560-627) for m % 8 == 0, k % 16 == 0, m <=
    256, with gemm_cols_tail (:688-727) for the last n % 16 columns, written
    out loop by loop in numpy."""
    m, k = a.shape
    n = b.shape[1]
    assert m % 8 == 0 and k % 16 == 0 and m <= 256
    n_main = n // 16 * 16
    c = np.zeros((m, n), np.float32)
    acc = np.zeros((m, n_main), np.float32)
    for kk in range(k):  # acc[r] = splat(a[r][kk]).mul_add(b row kk, acc[r])
        acc = _fma32(a[:, kk:kk + 1], b[kk:kk + 1, :n_main], acc)
    c[:, :n_main] = acc + np.float32(0.0)  # + ktail (empty: k % 16 == 0)
    if n > n_main:
        bt = b[:, n_main:].T  # [tail columns, k]
        lanes = np.zeros((m, n - n_main, 16), np.float32)
        for kk in range(0, k, 16):  # acc = av.mul_add(bv, acc), 16 lanes
            lanes = _fma32(a[:, None, kk:kk + 16], bt[None, :, kk:kk + 16], lanes)
        r = np.full((m, n - n_main), -0.0, np.float32)
        for l in range(16):  # reduce_sum: ordered lane sum
            r = (r + lanes[:, :, l]).astype(np.float32)
        c[:, n_main:] = r + np.float32(0.0)
    return c


def test_fma32_emulation_known_answers():
    one = np.float32(1.0)
    eps = np.float32(2.0 ** -23)
    # (1 + 2^-23)(1 - 2^-23) = 1 - 2^-46: a separately rounded product gives 1
    assert _fma32(one + eps, one - eps, np.float32(-1.0)) == np.float32(-(2.0 ** -46))
    # 1 + 2^-23 + (2^-24 - 2^-70): float64 rounds the sum onto the f32
    # halfway point 1 + 2^-23 + 2^-24 (where ties-to-even goes up); the exact
    # sum is below it, so the fused result is 1 + 2^-23
    a = np.float32(2.0 ** -24) * (one + eps)
    b = one - eps
    assert _fma32(a, b, one + eps) == one + eps
    x = np.float32(1.0) + np.float32(2.0 ** -22)
    got = _fma32(np.float32(2.0 ** -24), np.float32(1.0 + 2.0 ** -20), x)
    assert got == np.nextafter(x, np.float32(2))


@pytest.mark.parametrize("t,f", [(21, 33), (11, 17)])
def test_pointwise_conv_gemm_matches_restatement(t, f):
    """The oracle's f32 GEMM, through which its pointwise convs run, equals
    the reference's gemm_tile8 + gemm_cols_tail written out in numpy, bit
    for bit, at the pre-encode's conv.3 / conv.6 window shapes (spatial =
    693 = 21 x 33, 187 = 11 x 17: 5 and 11 tail columns), 256 -> 256
    channels; and the tail columns' lane order is not the one-chain order."""
    rng = np.random.default_rng(t * 100 + f)
    spatial = t * f
    w = (rng.standard_normal((256, 256)) * 0.06).astype(np.float32)
    x = np.maximum(rng.standard_normal((256, spatial)), 0).astype(np.float32)
    got = oracle.gemm_simd_into(w, x)
    want = _gemm_tile8_cols_tail(w, x)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    n_main = spatial // 16 * 16
    chain = np.zeros((256, spatial - n_main), np.float32)
    for kk in range(256):
        chain = _fma32(w[:, kk:kk + 1], x[kk:kk + 1, n_main:], chain)
    assert not np.array_equal(chain, want[:, n_main:])


def test_gemm_simd_into_rows_and_k_tails():
    """Shapes off the fast tile: m % 8 != 0 (gemm_row), k % 16 != 0 (the
    separately rounded k tail), n < 16: against float64 within the f32
    error bound, and the tiled part against the numpy restatement."""
    rng = np.random.default_rng(3)
    for m, k, n in [(13, 40, 7), (264, 48, 35), (8, 16, 16), (300, 19, 3)]:
        a = rng.standard_normal((m, k)).astype(np.float32)
        b = rng.standard_normal((k, n)).astype(np.float32)
        got = oracle.gemm_simd_into(a, b)
        ref = a.astype(np.float64) @ b.astype(np.float64)
        bound = 2 * k * 2.0 ** -24 * (np.abs(a).astype(np.float64) @ np.abs(b).astype(np.float64))
        assert np.all(np.abs(got - ref) <= bound + 1e-30)
        if m % 8 == 0 and k % 16 == 0 and m <= 256:
            want = _gemm_tile8_cols_tail(a, b)
            assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
