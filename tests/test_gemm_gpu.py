"""GPU parity tests of the Q8_0 GEMM, through the C ABI, against the oracle.

Bars (from the hot-path spec): activation Q8 codes and scales and the int32
block dots bit-exact; f32 outputs within max|d| <= 1e-4 * RMS(out).
"""
import ctypes

import numpy as np
import pytest

import oracle
from stealcode_b200 import _lib, synth
from stealcode_b200.ops import SC_LAYOUT_FEATURE_MAJOR, SC_LAYOUT_TIME_MAJOR, Q8Mat, q8_gemm
from tests import refcases

pytestmark = pytest.mark.gpu
TOL_RMS = 1e-4


@pytest.fixture(scope="module")
def torch():
    import torch as _t

    assert _t.cuda.is_available()
    return _t


def rms_err(got, ref):
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    assert got.shape == ref.shape
    fin = np.isfinite(ref)
    assert np.array_equal(np.isnan(got), np.isnan(ref))
    assert np.array_equal(np.isinf(got), np.isinf(ref))
    assert np.array_equal(got[np.isinf(ref)], ref[np.isinf(ref)])
    if not fin.any():
        return 0.0
    rms = np.sqrt(np.mean(ref[fin] ** 2))
    return np.max(np.abs(got[fin] - ref[fin])) / max(rms, 1e-30)


def dev_gemm(torch, mat, x_km, bias=None, y_layout=SC_LAYOUT_FEATURE_MAJOR):
    """Run the device GEMM on feature-major x [k, t]; returns y [rows, t]."""
    xd = torch.from_numpy(np.ascontiguousarray(x_km)).cuda()
    b = None if bias is None else torch.from_numpy(bias).cuda()
    y = mat.gemm(xd, x_layout=SC_LAYOUT_FEATURE_MAJOR, bias=b, y_layout=y_layout)
    torch.cuda.synchronize()
    y = y.cpu().numpy()
    return y if y_layout == SC_LAYOUT_FEATURE_MAJOR else y.T


def edge_activations(k, t, seed):
    x = synth.normal(seed, (t, k))
    x[0, :32] = 0.0                                # zero block
    x[1, :32] = [127.0, -63.5, 0.5, -0.5, 2.5, -2.5] + [0.25] * 26  # ties
    x[2, 5] = np.nan                               # NaN ignored by amax
    x[3 % t, 40] = np.inf                          # inf block
    x[4 % t, 64:96] = 1e-40                        # subnormal block
    x[5 % t, 96:128] = -3.0e38                     # near-overflow block
    return x


@pytest.mark.parametrize("layout", [SC_LAYOUT_TIME_MAJOR, SC_LAYOUT_FEATURE_MAJOR])
@pytest.mark.parametrize("k,t", [(1024, 8), (1000, 13), (4352, 3)])
def test_quantize_bit_exact(torch, layout, k, t):
    x_tk = edge_activations(k, t, 11 + k + t)
    xq_ref, dx_ref = oracle.quantize(np.ascontiguousarray(x_tk.T))   # [t, k], [t, nb]
    xd = torch.from_numpy(x_tk if layout == SC_LAYOUT_TIME_MAJOR else np.ascontiguousarray(x_tk.T)).cuda()
    from stealcode_b200.ops import quantize

    xq, dx = quantize(xd, x_layout=layout)
    torch.cuda.synchronize()
    xq = xq.cpu().numpy()[:, :k]
    dx = dx.cpu().numpy().T
    assert np.array_equal(xq, xq_ref)
    assert np.array_equal(dx.view(np.uint32), dx_ref.view(np.uint32))


@pytest.mark.parametrize("m,k,n", [(128, 768, 14), (37, 100, 5), (512, 4352, 16)])
def test_block_dots_bit_exact(torch, m, k, n):
    w, pr, x = refcases.gemm_pattern_case(m, k, n)
    x = x + synth.normal(5 + m, x.shape, std=0.3)
    ref = oracle.q8_block_dots(m, k, n, w, pr, 34, 2, x)
    mat = Q8Mat(w, m, k)
    got = mat.block_dots(torch.from_numpy(np.ascontiguousarray(x)).cuda(), x_layout=SC_LAYOUT_FEATURE_MAJOR)
    torch.cuda.synchronize()
    assert np.array_equal(got.cpu().numpy(), ref)


@pytest.mark.parametrize("m,k,n", sorted(set(refcases.VNNI_CASES + refcases.SIMD_CASES)))
def test_reference_pattern_cases(torch, m, k, n):
    w, pr, x = refcases.gemm_pattern_case(m, k, n)
    ref_s = oracle.q8_gemm_scalar(m, k, n, w, pr, 34, 2, x)
    ref_v = oracle.q8_gemm_simd_order(m, k, n, w, pr, 34, 2, x)
    got = dev_gemm(torch, Q8Mat(w, m, k), x)
    assert rms_err(got, ref_s) <= TOL_RMS
    assert rms_err(got, ref_v) <= TOL_RMS
    # the reference tests' own bar, too
    assert np.all(np.abs(got - ref_s) <= 1e-3 * (1 + np.abs(ref_s)))


def test_config0_single_chunk(torch):
    """One streaming chunk: x [8, 1024] ~ N(0,1), W [4096, 1024] Q8_0 ~ N(0, 0.02)."""
    seed = synth.SEED_BASE + 0
    w = synth.q8_weights(seed, 4096, 1024)
    x_tk = synth.normal(seed + 1, (8, 1024))
    ref = oracle.q8_gemm_scalar(4096, 1024, 8, w, 32 * 34, 34, 2, np.ascontiguousarray(x_tk.T))
    mat = Q8Mat(w, 4096, 1024)
    got = dev_gemm(torch, mat, np.ascontiguousarray(x_tk.T))
    assert rms_err(got, ref) <= TOL_RMS
    xd = torch.from_numpy(x_tk).cuda()
    y_tm = mat.gemm(xd, x_layout=SC_LAYOUT_TIME_MAJOR, y_layout=SC_LAYOUT_TIME_MAJOR)
    torch.cuda.synchronize()
    assert rms_err(y_tm.cpu().numpy().T, ref) <= TOL_RMS


@pytest.mark.parametrize("kn", [(1024, 3072), (1024, 1024), (1024, 4096), (4096, 1024)])
@pytest.mark.parametrize("mm", [1, 8, 32, 128])
def test_config1_layer_shapes(torch, kn, mm):
    k, n = kn
    seed = synth.SEED_BASE + 1
    w = synth.q8_weights(seed + k + n, n, k)
    x_tk = synth.normal(seed + 7 * mm, (mm, k))
    bias = synth.normal(seed + 3, (n,), std=0.02)
    ref = oracle.q8_gemm(n, k, mm, w, (k // 32) * 34, 34, 2, np.ascontiguousarray(x_tk.T)) + bias[:, None]
    mat = Q8Mat(w, n, k)
    got = dev_gemm(torch, mat, np.ascontiguousarray(x_tk.T), bias=bias, y_layout=SC_LAYOUT_TIME_MAJOR)
    assert rms_err(got, ref) <= TOL_RMS


def test_wgsl_random_scale_case(torch):
    """q8_gemm_matches_reference's inputs (random u16 f16 scales, so NaN/inf
    scales occur), under the CPU path's semantics."""
    raw, t, k, n, x_tk = refcases.wgsl_gemm_case()
    ref = oracle.q8_gemm_scalar(n, k, t, raw, (k // 32) * 34, 34, 2, np.ascontiguousarray(x_tk.T))
    got = dev_gemm(torch, Q8Mat(raw, n, k), np.ascontiguousarray(x_tk.T))
    assert rms_err(got, ref) <= TOL_RMS


def test_ragged_shapes_and_strides(torch):
    m, k, t = 37, 100, 5
    w = synth.q8_weights(91, m, k)
    x_tk = synth.normal(92, (t, k))
    ref = oracle.q8_gemm_scalar(m, k, t, w, 4 * 34, 34, 2, np.ascontiguousarray(x_tk.T))
    mat = Q8Mat(w, m, k)
    # time-major x with a padded row stride, time-major y with a padded stride
    xpad = np.zeros((t, 160), np.float32)
    xpad[:, :k] = x_tk
    y = torch.full((t, 64), 7.0, device="cuda")
    mat.gemm(torch.from_numpy(xpad).cuda(), x_layout=SC_LAYOUT_TIME_MAJOR, ldx=160, out=y,
             y_layout=SC_LAYOUT_TIME_MAJOR, ldy=64)
    torch.cuda.synchronize()
    yn = y.cpu().numpy()
    assert rms_err(yn[:, :m].T, ref) <= TOL_RMS
    assert np.all(yn[:, m:] == 7.0)  # nothing written past the rows


def test_host_twins_match_device(torch):
    m, k, n = 256, 1024, 8
    w = synth.q8_weights(31, m, k)
    x = synth.normal(32, (k, n))
    y = np.zeros((m, n), np.float32)
    q8_gemm(m, k, n, w, 32 * 34, 34, 2, x, y)
    mat = Q8Mat(w, m, k)
    y2 = mat.gemm_t(x, n)
    y3 = dev_gemm(torch, mat, x)
    assert np.array_equal(y, y2) and np.array_equal(y2, y3)  # one kernel, deterministic
    assert rms_err(y, oracle.q8_gemm_scalar(m, k, n, w, 32 * 34, 34, 2, x)) <= TOL_RMS


@pytest.mark.parametrize("t", [8, 128])
def test_full_size_properties(torch, t):
    """Size-independent properties at full layer sizes (K=4096, N=1024):
    scaling x by 2 leaves the codes unchanged and doubles every scale, so y
    doubles bit for bit; permuting frames permutes columns bit for bit."""
    k, n = 4096, 1024
    mat = Q8Mat(synth.q8_weights(41, n, k), n, k)
    x = torch.from_numpy(synth.normal(42, (t, k))).cuda()
    y1 = mat.gemm(x)
    y2 = mat.gemm(2 * x)
    perm = torch.randperm(t, generator=torch.Generator().manual_seed(0)).cuda()
    y3 = mat.gemm(x[perm].contiguous())
    torch.cuda.synchronize()
    assert torch.equal(y2, 2 * y1)
    assert torch.equal(y3, y1[perm])


def test_deterministic_across_calls(torch):
    mat = Q8Mat(synth.q8_weights(51, 3072, 1024), 3072, 1024)
    x = torch.from_numpy(synth.normal(52, (32, 1024))).cuda()
    a = mat.gemm(x).clone()
    for _ in range(3):
        assert torch.equal(mat.gemm(x), a)


def test_error_paths(torch):
    w = synth.q8_weights(61, 64, 64)
    h = ctypes.c_void_p()
    # 36-byte f32-scale blocks are rejected with a clear code
    rc = _lib.lib.sc_q8_repack(np.zeros(64 * 2 * 36, np.uint8).ctypes.data, 64, 64, 36, 4, ctypes.byref(h))
    assert rc == _lib.SC_ERR_UNSUPPORTED and "34-byte" in _lib.last_error()
    mat = Q8Mat(w, 64, 64)
    x = torch.zeros((4, 64), device="cuda")
    y = torch.zeros((4, 64), device="cuda")
    small = torch.zeros(16, dtype=torch.uint8, device="cuda")
    rc = _lib.lib.sc_q8_gemm(mat.handle, x.data_ptr(), 4, 1, 0, None, y.data_ptr(), 1, 0, small.data_ptr(), 16,
                             None)
    assert rc == _lib.SC_ERR_INVALID and "workspace" in _lib.last_error()
    rc = _lib.lib.sc_q8_gemm(mat.handle, x.data_ptr(), 4, 7, 0, None, y.data_ptr(), 1, 0, None, 0, None)
    assert rc == _lib.SC_ERR_INVALID
    # t == 0 is a no-op (q8_gemm returns early on zero dims)
    assert _lib.lib.sc_q8_gemm(mat.handle, x.data_ptr(), 0, 1, 0, None, y.data_ptr(), 1, 0, None, 0,
                               None) == _lib.SC_OK


def test_caller_workspace(torch):
    mat = Q8Mat(synth.q8_weights(71, 1024, 1024), 1024, 1024)
    x = torch.from_numpy(synth.normal(72, (8, 1024))).cuda()
    ws = torch.empty(mat.workspace_bytes(8), dtype=torch.uint8, device="cuda")
    assert torch.equal(mat.gemm(x, workspace=ws), mat.gemm(x))


def test_no_device_wait_timed_out(torch):
    """No bounded device-side wait gave up during the tests above."""
    torch.cuda.synchronize()
    assert _lib.device_status() == 0


# ---- mid-size path (17..128 frames): q8_gemm_scalar's order, bit-exact ----
@pytest.mark.parametrize("t,k,n", [(17, 1024, 256), (40, 1000, 37), (100, 4096, 128), (128, 1024, 384),
                                   (33, 4352, 1024)])
@pytest.mark.parametrize("layout", [SC_LAYOUT_TIME_MAJOR, SC_LAYOUT_FEATURE_MAJOR])
def test_mid_path_bit_exact_scalar_order(torch, t, k, n, layout):
    """More than 16 frames is where the reference runs q8_gemm_scalar
    (simd_kernel.rs:111-125); the mid-size kernel reproduces it bit for bit,
    bias added after."""
    w = synth.q8_weights(4000 + t + k, n, k)
    x_tk = edge_activations(k, t, 5000 + t)
    x_tk = np.nan_to_num(x_tk, nan=0.0, posinf=0.0, neginf=0.0)
    bias = synth.normal(6000 + n, (n,), std=0.02)
    ref = oracle.q8_gemm_scalar(n, k, t, w, ((k + 31) // 32) * 34, 34, 2, np.ascontiguousarray(x_tk.T))
    ref = (ref + bias[:, None]).astype(np.float32)
    mat = Q8Mat(w, n, k)
    xd = torch.from_numpy(x_tk if layout == SC_LAYOUT_TIME_MAJOR else np.ascontiguousarray(x_tk.T)).cuda()
    y = mat.gemm(xd, x_layout=layout, bias=torch.from_numpy(bias).cuda(), y_layout=layout)
    torch.cuda.synchronize()
    y = y.cpu().numpy()
    got = y.T if layout == SC_LAYOUT_TIME_MAJOR else y
    assert np.array_equal(got, ref)


# ---- tensor-core path (tcgen05 kind::i8), t > 16 frames -------------------
@pytest.mark.parametrize("t,k,n", [(17, 1024, 256), (33, 1000, 37), (64, 1024, 384), (100, 4096, 128),
                                   (129, 1024, 256), (300, 4352, 128), (1000, 1024, 640)])
@pytest.mark.parametrize("layout", [SC_LAYOUT_TIME_MAJOR, SC_LAYOUT_FEATURE_MAJOR])
def test_tensor_core_path_matches_oracle(torch, t, k, n, layout):
    w = synth.q8_weights(1000 + t + k, n, k)
    x_tk = synth.normal(2000 + t, (t, k))
    bias = synth.normal(3000 + n, (n,), std=0.02)
    ref = oracle.q8_gemm(n, k, t, w, ((k + 31) // 32) * 34, 34, 2, np.ascontiguousarray(x_tk.T)) + bias[:, None]
    mat = Q8Mat(w, n, k)
    xd = torch.from_numpy(x_tk if layout == SC_LAYOUT_TIME_MAJOR else np.ascontiguousarray(x_tk.T)).cuda()
    y = mat.gemm(xd, x_layout=layout, bias=torch.from_numpy(bias).cuda(), y_layout=layout)
    torch.cuda.synchronize()
    y = y.cpu().numpy()
    got = y.T if layout == SC_LAYOUT_TIME_MAJOR else y
    assert rms_err(got, ref) <= TOL_RMS


def test_tensor_core_path_config3_frames(torch):
    """M = 256 streams x 7 frames = 1792 (the batched encoder step), full
    FFN-up shape; checked on a column subset against the oracle plus the
    size-independent scaling and permutation properties on all of it."""
    t, k, n = 1792, 1024, 4096
    mat = Q8Mat(synth.q8_weights(77, n, k), n, k)
    x = torch.from_numpy(synth.normal(78, (t, k))).cuda()
    y1 = mat.gemm(x)
    y2 = mat.gemm(2 * x)
    perm = torch.randperm(t, generator=torch.Generator().manual_seed(1)).cuda()
    y3 = mat.gemm(x[perm].contiguous())
    torch.cuda.synchronize()
    assert torch.equal(y2, 2 * y1)
    assert torch.equal(y3, y1[perm])
    cols = [0, 1, 127, 128, 1000, 1791]
    xs = x[cols].cpu().numpy()
    w = synth.q8_weights(77, n, k)
    ref = oracle.q8_gemm(n, k, len(cols), w, 32 * 34, 34, 2, np.ascontiguousarray(xs.T))
    assert rms_err(y1[cols].cpu().numpy().T, ref) <= TOL_RMS


def test_tensor_core_no_timeouts(torch):
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
