"""The CUDA path through the C ABI against the committed golden fixtures
(tests/golden/golden.npz: the oracle's frozen outputs on the inputs of the
reference's own GEMM, quantiser and streaming-attention tests).

Bars: activation codes and scales bit-exact; GEMMs over more than 16
frames (q8_gemm_scalar's order, which is the reference's dispatch there)
bit-exact; the small-M GEMM and the attention within max|d| <= 1e-4 x RMS
and the reference tests' own bars."""
import os

import numpy as np
import pytest

from stealcode_b200.ops import SC_LAYOUT_FEATURE_MAJOR, AttnStreamKernel, Q8Mat, quantize
from tests import refcases
from tests.golden import make_golden

pytestmark = pytest.mark.gpu
TOL_RMS = 1e-4


@pytest.fixture(scope="module")
def torch():
    import torch as _t

    assert _t.cuda.is_available()
    return _t


@pytest.fixture(scope="module")
def golden():
    return np.load(os.path.join(make_golden.HERE, "golden.npz"))


def rms_err(got, ref):
    """max |got - ref| / RMS(ref) over finite references; NaN and inf (from
    NaN / inf f16 block scales) must match exactly."""
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


def dev_gemm(torch, w, m, k, x_km):
    """Device GEMM of GGUF blocks w [m, k/32*34] and feature-major x [k, t]."""
    mat = Q8Mat(w, m, k)
    xd = torch.from_numpy(np.ascontiguousarray(x_km)).cuda()
    y = mat.gemm(xd, x_layout=SC_LAYOUT_FEATURE_MAJOR, y_layout=SC_LAYOUT_FEATURE_MAJOR)
    torch.cuda.synchronize()
    return y.cpu().numpy()


@pytest.mark.parametrize("m,k,n", make_golden.pattern_cases())
def test_pattern_cases_match_golden(torch, golden, m, k, n):
    w, _, x = refcases.gemm_pattern_case(m, k, n)
    ref = golden[f"pattern_{m}_{k}_{n}"]
    got = dev_gemm(torch, w, m, k, x)
    assert rms_err(got, ref) <= TOL_RMS
    assert rms_err(got, golden[f"pattern_{m}_{k}_{n}_simd"]) <= TOL_RMS
    assert np.all(np.abs(got - ref) <= 1e-3 * (1 + np.abs(ref)))  # the reference tests' own bar


@pytest.mark.parametrize("name,case", [("mid", make_golden.MID_CASES[0]), ("tc", make_golden.MID_CASES[1])])
def test_scalar_order_paths_match_golden_bit_exact(torch, golden, name, case):
    """40 frames (mid-size kernel) and 136 frames (tensor-core kernel)."""
    m, k, n = case
    w, _, x = refcases.gemm_pattern_case(m, k, n)
    got = dev_gemm(torch, w, m, k, x)
    assert np.array_equal(got.view(np.uint32), golden[f"{name}_{m}_{k}_{n}"].view(np.uint32))


def test_random_scale_case_matches_golden(torch, golden):
    raw, t, k, n, x_tk = refcases.wgsl_gemm_case()
    got = dev_gemm(torch, raw, n, k, np.ascontiguousarray(x_tk.T))
    assert rms_err(got, golden[f"wgsl_{n}_{k}_{t}"]) <= TOL_RMS


def test_quantiser_matches_golden(torch, golden):
    _, _, x = refcases.gemm_pattern_case(8, 2048, 16)  # feature-major [2048, 16]
    xq, dx = quantize(torch.from_numpy(np.ascontiguousarray(x)).cuda(), x_layout=SC_LAYOUT_FEATURE_MAJOR)
    torch.cuda.synchronize()
    xq = xq.cpu().numpy()[:, :2048]
    dx = dx.cpu().numpy().T
    assert np.array_equal(xq, golden["quant_2048_16_q"])
    assert np.array_equal(dx.view(np.uint32), golden["quant_2048_16_d"].view(np.uint32))


def test_attention_matches_golden(torch, golden):
    cs = refcases.attn_case()
    got = AttnStreamKernel.forward(*[cs[a] for a in make_golden.ATTN_KEYS])
    ref = golden["attn_ref"]
    assert rms_err(got, ref) <= TOL_RMS
    assert np.max(np.abs(got - ref)) < 1e-4  # the reference test's own bar
