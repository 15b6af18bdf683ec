"""sc_q8_gemm_noalloc, the GEMM entry point for callers that cannot allocate
device memory (a plugin inside someone else's CUDA-graph capture, a
real-time audio callback that must not stall in cudaMalloc, a host that owns
all device memory).  Its scratch is a fixed device array inside the library.

Checked through the C ABI against sc_q8_gemm (the entry point that takes a
workspace) on two calls in a row, so the second call runs over the first
call's leftovers in the shared array, and against the oracle's
q8_gemm_scalar (the reference's arithmetic for more than 16 frames, which
the mid-size and tensor-core kernels reproduce bit for bit) for every frame
count class: the streaming kernel (8 frames), the mid-size kernel (64) and
the tensor-core kernel (256, and 384 frames at k = 4096, the largest batch
of whole 128-frame tiles the fixed array holds).  This file is collected last, and it passes both on
its own in a fresh process and after the other tests.
"""
import numpy as np
import pytest

import oracle
from stealcode_b200 import _lib, synth
from stealcode_b200.ops import SC_LAYOUT_FEATURE_MAJOR, SC_LAYOUT_TIME_MAJOR, Q8Mat

pytestmark = pytest.mark.gpu
TOL_RMS = 1e-4  # the GEMM parity bar used by every GPU test
SCRATCH = 4 << 20


def _rms_err(got, ref):
    ref = ref.astype(np.float64)
    return float(np.max(np.abs(got.astype(np.float64) - ref)) / np.sqrt(np.mean(ref ** 2)))


def _with_workspace(torch, mat, x, t, layout):
    y = torch.empty((t, mat.rows), dtype=torch.float32, device="cuda")
    _lib.check(_lib.lib.sc_q8_gemm(mat.handle, x.data_ptr(), t, layout, 0, None, y.data_ptr(),
                                   SC_LAYOUT_TIME_MAJOR, 0, None, 0, None))
    return y


def _no_alloc(torch, mat, x, t, layout):
    y = torch.full((t, mat.rows), float("nan"), dtype=torch.float32, device="cuda")
    _lib.check(_lib.lib.sc_q8_gemm_noalloc(mat.handle, x.data_ptr(), t, layout, 0, None, y.data_ptr(),
                                           SC_LAYOUT_TIME_MAJOR, 0, None))
    return y


def test_noalloc_matches_workspace_gemm_on_two_calls():
    import torch

    # first call: a large frame batch that fills much of the scratch
    mat = Q8Mat(synth.q8_weights(901, 1024, 4096), 1024, 4096)
    x1 = torch.from_numpy(synth.normal(902, (256, 4096))).cuda()
    a1 = _no_alloc(torch, mat, x1, 256, SC_LAYOUT_TIME_MAJOR)
    r1 = _with_workspace(torch, mat, x1, 256, SC_LAYOUT_TIME_MAJOR)
    # second call, right after: fewer frames, another matrix and layout, so
    # the array still holds the first call's codes beyond this call's range
    mat2 = Q8Mat(synth.q8_weights(903, 3072, 1024), 3072, 1024)
    x2 = torch.from_numpy(synth.normal(904, (1024, 8))).cuda()  # feature-major [k, t]
    a2 = _no_alloc(torch, mat2, x2, 8, SC_LAYOUT_FEATURE_MAJOR)
    r2 = _with_workspace(torch, mat2, x2, 8, SC_LAYOUT_FEATURE_MAJOR)
    torch.cuda.synchronize()
    for got, ref in ((a1, r1), (a2, r2)):
        got, ref = got.cpu().numpy(), ref.cpu().numpy()
        assert np.isfinite(got).all()
        assert _rms_err(got, ref) <= TOL_RMS


def test_noalloc_rejects_frames_beyond_the_scratch():
    import torch

    mat = Q8Mat(synth.q8_weights(905, 128, 4096), 128, 4096)
    t = 1024  # 1024 x 4096 codes alone are 4 MiB: over the fixed array
    assert _lib.lib.sc_q8_gemm_workspace_bytes(t, 4096) > SCRATCH
    x = torch.zeros((t, 4096), device="cuda")
    y = torch.zeros((t, 128), device="cuda")
    rc = _lib.lib.sc_q8_gemm_noalloc(mat.handle, x.data_ptr(), t, SC_LAYOUT_TIME_MAJOR, 0, None, y.data_ptr(),
                                     SC_LAYOUT_TIME_MAJOR, 0, None)
    assert rc == _lib.SC_ERR_INVALID
    assert "scratch" in _lib.last_error()
    assert _lib.lib.sc_q8_gemm_noalloc(None, None, 1, 0, 0, None, None, 0, 0, None) == _lib.SC_ERR_INVALID


def _oracle_scalar(w_blocks, rows, k, x_tk):
    """q8_gemm_scalar (sgemm_kernel.rs:132-202) on host: y [t, rows]."""
    t = x_tk.shape[0]
    y = oracle.q8_gemm_scalar(rows, k, t, w_blocks, (k // 32) * 34, 34, 2, np.ascontiguousarray(x_tk.T))
    return np.ascontiguousarray(y.T)


@pytest.mark.parametrize("t,rows,k", [(8, 1024, 1024), (64, 1024, 1024), (256, 512, 4096), (384, 256, 4096)])
def test_noalloc_matches_oracle_in_every_frame_class(t, rows, k):
    import torch

    assert _lib.lib.sc_q8_gemm_workspace_bytes(t, k) <= SCRATCH
    wb = synth.q8_weights(910 + t, rows, k)
    mat = Q8Mat(wb, rows, k)
    x = synth.normal(911 + t, (t, k))
    xd = torch.from_numpy(x).cuda()
    outs = [_no_alloc(torch, mat, xd, t, SC_LAYOUT_TIME_MAJOR) for _ in range(2)]  # two calls in a row
    torch.cuda.synchronize()
    ref = _oracle_scalar(wb, rows, k, x)
    for y in outs:
        got = y.cpu().numpy()
        assert np.isfinite(got).all()
        if t > 16:  # the reference's scalar order: bit for bit
            assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
        else:       # the SIMD dispatch's order differs in the last bits
            assert _rms_err(got, ref) <= TOL_RMS
