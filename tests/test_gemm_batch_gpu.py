"""GPU parity of the batched streaming GEMM (sc_q8_gemm_batch): several
independent Q8_0 GEMMs of one small frame count in one pass, against the
oracle (q8_gemm_simd_order: the reference's dispatch for up to 16 frames,
simd_kernel.rs:96-394) and against sc_q8_gemm one call at a time.  Bar: the
f32 GEMM tolerance, max |d| <= 1e-4 x RMS."""
import numpy as np
import pytest

import oracle
from stealcode_b200 import _lib, synth
from stealcode_b200.ops import SC_LAYOUT_FEATURE_MAJOR, SC_LAYOUT_TIME_MAJOR, Q8Mat, q8_gemm_batch

pytestmark = pytest.mark.gpu
TOL = 1e-4


@pytest.fixture(scope="module")
def torch():
    import torch as _t

    assert _t.cuda.is_available()
    return _t


def _rms_err(got, ref):
    ref = np.asarray(ref, np.float64)
    return float(np.max(np.abs(np.asarray(got, np.float64) - ref)) / np.sqrt(np.mean(ref ** 2)))


SHAPES = [(1024, 3072), (1024, 1024), (1024, 4096), (4096, 1024), (96, 200), (4352, 1024)]


@pytest.mark.parametrize("t", [1, 2, 7, 8, 16])
def test_batch_matches_oracle_and_single_calls(torch, t):
    mats, xs, bs, blocks = [], [], [], []
    for i, (k, n) in enumerate(SHAPES):
        wb = synth.q8_weights(500 + 10 * t + i, n, k)
        blocks.append(wb)
        mats.append(Q8Mat(wb, n, k))
        xs.append(torch.from_numpy(synth.normal(600 + 10 * t + i, (t, k))).cuda())
        bs.append(torch.from_numpy(synth.normal(700 + i, (n,), std=0.1)).cuda() if i % 2 == 0 else None)
    ys = q8_gemm_batch(mats, xs, biases=bs)
    singles = [m.gemm(x, bias=b) for m, x, b in zip(mats, xs, bs)]
    torch.cuda.synchronize()
    for i, (k, n) in enumerate(SHAPES):
        got = ys[i].cpu().numpy()
        x = xs[i].cpu().numpy()
        ref = oracle.q8_gemm_simd_order(n, k, t, blocks[i], (k + 31) // 32 * 34, 34, 2,
                                        np.ascontiguousarray(x.T)).T
        if bs[i] is not None:
            ref = ref + bs[i].cpu().numpy()[None, :]
        assert got.shape == (t, n)
        assert _rms_err(got, ref) <= TOL, (i, _rms_err(got, ref))
        assert _rms_err(got, singles[i].cpu().numpy()) <= TOL


def test_batch_feature_major_and_workspace(torch):
    """Feature-major x [k, t] and y [rows, t] (the reference CPU layout), a
    caller workspace, two calls in a row over it, 128 GEMMs (the most)."""
    t = 8
    mats = [Q8Mat(synth.q8_weights(800 + i, 256, 512), 256, 512) for i in range(128)]
    xs = [torch.from_numpy(synth.normal(900 + i, (512, t))).cuda() for i in range(128)]
    hw = (_lib.ctypes.c_void_p * 128)(*[m.handle.value for m in mats])
    ws_bytes = _lib.lib.sc_q8_gemm_batch_workspace_bytes(hw, 128)
    assert ws_bytes > 0
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    for _ in range(2):
        ys = q8_gemm_batch(mats, xs, x_layout=SC_LAYOUT_FEATURE_MAJOR, y_layout=SC_LAYOUT_FEATURE_MAJOR,
                           workspace=ws)
    singles = [m.gemm(x, x_layout=SC_LAYOUT_FEATURE_MAJOR, y_layout=SC_LAYOUT_FEATURE_MAJOR) for m, x in zip(mats, xs)]
    torch.cuda.synchronize()
    for y, s in zip(ys, singles):
        assert y.shape == (256, t)
        assert _rms_err(y.cpu().numpy(), s.cpu().numpy()) <= TOL
    assert _lib.device_status() == 0


def test_batch_rejects_bad_calls(torch):
    m = Q8Mat(synth.q8_weights(990, 128, 64), 128, 64)
    x = torch.zeros((17, 64), device="cuda")
    y = torch.zeros((17, 128), device="cuda")
    with pytest.raises(_lib.ScError) as e:
        q8_gemm_batch([m], [x], outs=[y])  # 17 frames: more than the streaming batch takes
    assert e.value.code == _lib.SC_ERR_INVALID
