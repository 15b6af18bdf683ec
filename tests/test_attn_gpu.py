"""GPU parity tests of the fused streaming attention, through the C ABI,
against the oracle (block_new's attention, streaming.rs:492-589).
Bar: max|d| <= 1e-4 * RMS(out)."""
import math

import numpy as np
import pytest

import oracle
from stealcode_b200 import _lib, synth
from stealcode_b200.ops import AttnStreamKernel, attn_stream_ring
from tests import refcases

pytestmark = pytest.mark.gpu
TOL_RMS = 1e-4


@pytest.fixture(scope="module")
def torch():
    import torch as _t

    assert _t.cuda.is_available()
    return _t


def rms_err(got, ref):
    ref = np.asarray(ref, np.float64)
    return float(np.max(np.abs(np.asarray(got, np.float64) - ref)) / np.sqrt(np.mean(ref ** 2)))


def band_bounds(s, c, chunk, left_chunks):
    k_lo = max(s // chunk - left_chunks, 0) * chunk
    return k_lo, s + c


def test_reference_case_host_and_device(torch):
    cs = refcases.attn_case()
    keys = ("q", "kv", "vv", "pos_p", "q_bias", "v_bias", "c", "d", "n_heads", "scale", "s", "k_lo", "band",
            "chunk", "left_chunks", "k_hi", "pos_off")
    args = [cs[k] for k in keys]
    ref = oracle.attn_stream(*args)
    got = AttnStreamKernel.forward(*args)
    assert rms_err(got, ref) <= TOL_RMS
    assert np.max(np.abs(got - ref)) < 1e-4  # the reference test's own bar
    dev = [torch.from_numpy(np.ascontiguousarray(a)).cuda() if isinstance(a, np.ndarray) else a for a in args]
    got_d = AttnStreamKernel.forward_device(*dev)
    torch.cuda.synchronize()
    assert np.array_equal(got_d.cpu().numpy(), got)


def make_stream_case(seed, n_streams, s, c, d, n_heads, chunk, left_chunks, cap):
    """Per-stream history [0, s) plus c new frames; returns arrays and the ring."""
    k_lo, k_hi = band_bounds(s, c, chunk, left_chunks)
    n_pos = (left_chunks + 2) * chunk - 1 + 8
    hist_k = synth.normal(seed, (n_streams, s + c, d))
    hist_v = synth.normal(seed + 1, (n_streams, s + c, d))
    q = synth.normal(seed + 2, (n_streams, c, d))
    pos_p = synth.normal(seed + 3, (n_pos, d))
    u = synth.normal(seed + 4, (d,), std=0.02)
    v = synth.normal(seed + 5, (d,), std=0.02)
    ring_k = np.full((n_streams, cap, d), np.nan, np.float32)  # slots outside the band are never read
    ring_v = np.full((n_streams, cap, d), np.nan, np.float32)
    for fr in range(k_lo, s):
        ring_k[:, fr % cap] = hist_k[:, fr]
        ring_v[:, fr % cap] = hist_v[:, fr]
    return dict(k_lo=k_lo, k_hi=k_hi, n_pos=n_pos, hist_k=hist_k, hist_v=hist_v, q=q, pos_p=pos_p, u=u, v=v,
                ring_k=ring_k, ring_v=ring_v)


@pytest.mark.parametrize("s,c,cap", [(140, 8, 84), (147, 7, 80), (0, 7, 84), (14, 7, 78), (70, 16, 96)])
def test_ring_batched_matches_oracle(torch, s, c, cap):
    """Config-2 shape: 64 streams, 8 heads x 128, chunk 7, left_chunks 10."""
    d, nh, chunk, lc, ns = 1024, 8, 7, 10, 64
    if s == 0 or s == 14:
        ns = 4
    cs = make_stream_case(1000 + s + c, ns, s, c, d, nh, chunk, lc, cap)
    k_lo, k_hi = cs["k_lo"], cs["k_hi"]
    scale = 1.0 / math.sqrt(d // nh)
    pos_off = chunk - 1
    q = torch.from_numpy(cs["q"].reshape(ns * c, d)).cuda()
    kn = torch.from_numpy(np.ascontiguousarray(cs["hist_k"][:, s:s + c]).reshape(ns * c, d)).cuda()
    vn = torch.from_numpy(np.ascontiguousarray(cs["hist_v"][:, s:s + c]).reshape(ns * c, d)).cuda()
    rk = torch.from_numpy(cs["ring_k"]).cuda()
    rv = torch.from_numpy(cs["ring_v"]).cuda()
    pos = torch.from_numpy(cs["pos_p"]).cuda()
    u = torch.from_numpy(cs["u"]).cuda()
    v = torch.from_numpy(cs["v"]).cuda()
    out = attn_stream_ring(q, kn, vn, rk, rv, pos, u, v, c=c, d=d, n_heads=nh, scale=scale, s=s, k_lo=k_lo,
                           chunk=chunk, left_chunks=lc, pos_off=pos_off)
    torch.cuda.synchronize()
    out = out.cpu().numpy().reshape(ns, c, d)
    for z in range(ns):
        kv = cs["hist_k"][z, k_lo:k_hi]
        vv = cs["hist_v"][z, k_lo:k_hi]
        ref = oracle.attn_stream(cs["q"][z], kv, vv, cs["pos_p"], cs["u"], cs["v"], c, d, nh, scale, s, k_lo,
                                 k_hi - k_lo, chunk, lc, k_hi, pos_off)
        assert rms_err(out[z], ref) <= TOL_RMS, z
    # the new frames were appended to the rings
    rk = rk.cpu().numpy()
    for fr in range(s, s + c):
        assert np.array_equal(rk[:, fr % cap], cs["hist_k"][:, fr])


def test_ring_multi_step_stream(torch):
    """Five consecutive 7-frame chunks through one ring equal the oracle on
    the full history at every step (the cache slide of streaming.rs:263-277)."""
    d, nh, chunk, lc, cap, c, ns = 1024, 8, 7, 10, 77, 7, 3
    scale = 1.0 / math.sqrt(128)
    steps = 14
    hist_k = synth.normal(5, (ns, steps * c, d))
    hist_v = synth.normal(6, (ns, steps * c, d))
    qs = synth.normal(7, (ns, steps * c, d))
    pos_p = synth.normal(8, ((lc + 2) * chunk - 1, d))
    u = synth.normal(9, (d,), std=0.02)
    v = synth.normal(10, (d,), std=0.02)
    rk = torch.zeros((ns, cap, d), device="cuda")
    rv = torch.zeros((ns, cap, d), device="cuda")
    pos = torch.from_numpy(pos_p).cuda()
    ud, vd = torch.from_numpy(u).cuda(), torch.from_numpy(v).cuda()
    for step in range(steps):
        s = step * c
        k_lo, k_hi = band_bounds(s, c, chunk, lc)
        q = torch.from_numpy(np.ascontiguousarray(qs[:, s:s + c]).reshape(ns * c, d)).cuda()
        kn = torch.from_numpy(np.ascontiguousarray(hist_k[:, s:s + c]).reshape(ns * c, d)).cuda()
        vn = torch.from_numpy(np.ascontiguousarray(hist_v[:, s:s + c]).reshape(ns * c, d)).cuda()
        out = attn_stream_ring(q, kn, vn, rk, rv, pos, ud, vd, c=c, d=d, n_heads=nh, scale=scale, s=s,
                               k_lo=k_lo, chunk=chunk, left_chunks=lc, pos_off=chunk - 1)
        out = out.cpu().numpy().reshape(ns, c, d)
        for z in range(ns):
            ref = oracle.attn_stream(qs[z, s:s + c], hist_k[z, k_lo:k_hi], hist_v[z, k_lo:k_hi], pos_p, u, v, c,
                                     d, nh, scale, s, k_lo, k_hi - k_lo, chunk, lc, k_hi, chunk - 1)
            assert rms_err(out[z], ref) <= TOL_RMS, (step, z)


@pytest.mark.parametrize("c", [1, 5, 16])
def test_band_mode_shapes_head_dim_64(torch, c):
    d, nh, chunk, lc = 512, 8, 4, 2
    s = 16
    k_lo, k_hi = band_bounds(s, c, chunk, lc)
    band = k_hi - k_lo
    n_pos = s + c + 8
    q = synth.normal(20 + c, (c, d))
    kv = synth.normal(21 + c, (band, d))
    vv = synth.normal(22 + c, (band, d))
    pos_p = synth.normal(23 + c, (n_pos, d))
    u = synth.normal(24, (d,), std=0.02)
    v = synth.normal(25, (d,), std=0.02)
    scale = 1.0 / math.sqrt(d // nh)
    args = (q, kv, vv, pos_p, u, v, c, d, nh, scale, s, k_lo, band, chunk, lc, k_hi, chunk - 1)
    assert rms_err(AttnStreamKernel.forward(*args), oracle.attn_stream(*args)) <= TOL_RMS


def test_attn_error_paths(torch):
    cs = refcases.attn_case()
    keys = ("q", "kv", "vv", "pos_p", "q_bias", "v_bias", "c", "d", "n_heads", "scale", "s", "k_lo", "band",
            "chunk", "left_chunks", "k_hi", "pos_off")
    args = [cs[k] for k in keys]
    bad = list(args)
    bad[-1] = 40  # pos_off pushes pos rows past pos_p
    with pytest.raises(_lib.ScError) as e:
        AttnStreamKernel.forward(*bad)
    assert e.value.code == _lib.SC_ERR_INVALID and "pos rows" in str(e.value)
    bad = list(args)
    bad[11] = 12  # k_lo above the first query's band start
    bad[12] = 12
    with pytest.raises(_lib.ScError):
        AttnStreamKernel.forward(*bad)
    # ring capacity smaller than the band
    d = 1024
    t = lambda *s: torch.zeros(s, device="cuda")
    with pytest.raises(_lib.ScError) as e:
        attn_stream_ring(t(8, d), t(8, d), t(8, d), t(1, 40, d), t(1, 40, d), t(83, d), t(d), t(d), c=8, d=d,
                         n_heads=8, scale=0.1, s=140, k_lo=70, chunk=7, left_chunks=10, pos_off=6)
    assert "ring cap" in str(e.value)
