"""Failure paths of the C ABI on the GPU, made on the host (no GPU fault):
device allocations refused by the library's allocation cap
(sc_debug_set_device_alloc_cap) must surface as SC_ERR_ALLOC from the entry
point that needed them, free what that call had allocated, and leave the
library usable.  The reference degrades the same way: a failed GPU set-up is
an error value, not an abort (gpu/context.rs:43-87)."""
import numpy as np
import pytest

from stealcode_b200 import _lib, model, synth
from stealcode_b200.ops import Q8Mat, StreamEncoder

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch():
    import torch as _t

    assert _t.cuda.is_available()
    return _t


def _free_bytes(torch):
    torch.cuda.synchronize()
    return torch.cuda.mem_get_info()[0]


@pytest.mark.parametrize("cap_mb", [0, 1, 60, 160])
def test_encoder_create_under_allocation_cap(torch, cap_mb):
    """A 2-layer encoder needs ~180 MB of device memory: every cap below that
    fails at a different allocation (the first one, inside the weights, at
    the step buffers), and each failure returns SC_ERR_ALLOC with nothing
    left allocated."""
    cfg = model.EncoderConfig(n_layers=2)
    m = model.random_model(cfg, seed=41)
    before = _free_bytes(torch)
    _lib.check(_lib.lib.sc_debug_set_device_alloc_cap(cap_mb << 20))
    try:
        with pytest.raises(_lib.ScError) as e:
            StreamEncoder(m, 4)
        assert e.value.code == _lib.SC_ERR_ALLOC, str(e.value)
    finally:
        _lib.check(_lib.lib.sc_debug_set_device_alloc_cap(-1))
    after = _free_bytes(torch)
    assert abs(after - before) < (8 << 20), (before, after)
    enc = StreamEncoder(m, 4)  # the cap is gone: the same call succeeds
    mel = torch.zeros((4, 56, cfg.feat_in), device="cuda")
    enc.encode_new(mel, 0, 56)
    assert enc.total() == 7
    enc.close()


def test_repack_under_allocation_cap(torch):
    blocks = synth.q8_weights(43, 1024, 1024)
    _lib.check(_lib.lib.sc_debug_set_device_alloc_cap(1 << 20))
    try:
        with pytest.raises(_lib.ScError) as e:
            Q8Mat(blocks, 1024, 1024)
        assert e.value.code == _lib.SC_ERR_ALLOC
    finally:
        _lib.check(_lib.lib.sc_debug_set_device_alloc_cap(-1))
    mat = Q8Mat(blocks, 1024, 1024)
    x = torch.from_numpy(synth.normal(44, (8, 1024))).cuda()
    y = mat.gemm(x)
    torch.cuda.synchronize()
    assert np.isfinite(y.cpu().numpy()).all()
    mat.free()
