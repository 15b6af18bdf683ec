"""GPU parity of the device streaming encoder (one encode_new call = one
streaming step for all streams) against the oracle StreamingEncoder
(streaming.rs:137-680), one oracle instance per stream, on the same seeded
random-init model and mel input."""
import numpy as np
import pytest

import oracle
from stealcode_b200 import _lib, model

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch():
    import torch as _t

    assert _t.cuda.is_available()
    return _t


def _err(got, ref):
    ref = ref.astype(np.float64)
    d = np.abs(got.astype(np.float64) - ref)
    rms = np.sqrt(np.mean(ref ** 2))
    return float(d.max() / rms), float(d.mean() / rms)


def run_steps(torch, cfg, n_streams, n_steps, tail=0, seed=11):
    from stealcode_b200.ops import StreamEncoder

    m = model.random_model(cfg, seed=seed)
    n_mel = 56 * n_steps + tail
    mel = model.mel_stream(seed + 1, n_streams, n_mel, cfg.feat_in)
    dev = StreamEncoder(m, n_streams)
    refs = [oracle.StreamingEncoder(m) for _ in range(n_streams)]
    stats = []
    batches = [(56 * i, 56 * (i + 1), False) for i in range(n_steps)]
    if tail:
        batches.append((56 * n_steps, 56 * n_steps + tail, True))
    for (t0, t1, fin) in batches:
        dev.encode_new(torch.from_numpy(np.ascontiguousarray(mel[:, t0:t1])).cuda(), t0, t1, fin)
        torch.cuda.synchronize()
        s = t0 // 8
        for z in range(n_streams):
            assert refs[z].encode_new(mel[z, :t1], t0, t1, fin) == 0
            assert dev.total() == refs[z].total()
            got = dev.frames(z, s, dev.total())
            ref = refs[z].frames(s, refs[z].total())
            stats.append((t0, z) + _err(got, ref))
    dev.close()
    return stats


def test_encoder_two_layers_matches_oracle(torch):
    """2 conformer blocks at full width (d 1024, 8 heads, FF 4096, conv 9):
    13 steady 56-mel steps (the band reaches its 77-frame steady state at
    step 11) and a 24-mel final tail."""
    cfg = model.EncoderConfig(n_layers=2)
    stats = run_steps(torch, cfg, 3, 13, tail=24)
    worst = max(s[2] for s in stats)
    mean = max(s[3] for s in stats)
    print("encoder 2-layer: worst max/RMS %.3g, worst mean/RMS %.3g" % (worst, mean))
    for s in stats:
        print("step t0=%d stream %d: max/RMS %.3g mean/RMS %.3g" % s)
    assert mean <= 1e-4
    assert worst <= 1e-2


def test_encoder_out_of_sync_is_rejected(torch):
    from stealcode_b200.ops import StreamEncoder

    cfg = model.EncoderConfig(n_layers=1)
    dev = StreamEncoder(model.random_model(cfg, seed=3), 2)
    mel = torch.zeros((2, 56, cfg.feat_in), device="cuda")
    with pytest.raises(_lib.ScError) as e:
        dev.encode_new(mel, 56, 112)  # first call must start at frame 0
    assert e.value.code == _lib.SC_ERR_STATE and "out of sync" in str(e.value)
    dev.encode_new(mel, 0, 56)
    assert dev.total() == 7
    with pytest.raises(_lib.ScError):
        dev.frames(0, 0, 8)  # past the encoded frames
    dev.close()
