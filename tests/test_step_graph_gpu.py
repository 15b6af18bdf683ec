"""GPU tests of the encoder's step graphs (sc_stream_encoder_set_graphs):
steady steps replayed from one CUDA graph of the whole step give the bits of
the same steps launched kernel by kernel.  Covered: both entry points, new
or rotating input buffers every step (the copy nodes re-pointed per
replay), ring slots that wrap while graphs replay (the device frame shift),
two sub-batches or one, 7-frame steps and 56-frame calls, a step that
cannot use a graph between replays, and the launch count a replay reports.
The replayed steps are also checked against the oracle (the reference's
StreamingEncoder, streaming.rs:137-680, with the device's rounding)."""
import numpy as np
import pytest

import oracle
from stealcode_b200 import _lib, model

pytestmark = pytest.mark.gpu

TOL = 1e-4  # max |d| / RMS(reference), f32 outputs


@pytest.fixture(scope="module")
def torch():
    import torch as _t

    assert _t.cuda.is_available()
    return _t


class _DevRows:
    """A device pointer [rows, d] f32 viewed as a torch tensor (no copy)."""

    def __init__(self, ptr, rows, d):
        self.__cuda_array_interface__ = {"shape": (rows, d), "typestr": "<f4", "data": (ptr, False),
                                         "version": 3, "strides": None}


def _rows(torch, enc):
    return torch.as_tensor(_DevRows(*enc.output()), device="cuda").cpu().numpy()


def _err(got, ref):
    ref = ref.astype(np.float64)
    return float(np.abs(got.astype(np.float64) - ref).max() / np.sqrt(np.mean(ref ** 2)))


@pytest.mark.parametrize("n_streams", [256, 3])
def test_step_graphs_match_separate_launches(torch, n_streams):
    """20 streaming steps of 7 frames, 2 blocks at full width.  The band is
    steady (77 keys) from step 10, so steps 11 and 12 are captured (one graph
    per mel-history buffer) and steps 13-19 replay them; 256 streams run as
    two halves, 3 as one batch.  Every step's frames equal those of the same
    encoder with graphs off, bit for bit; each step's mel is a new device
    buffer; the K/V (84 slots), GLU (16) and output (64) rings wrap while
    graphs replay; a graph step reports the separate launches' count plus
    the frame-shift store; the first and last streams match the oracle."""
    from stealcode_b200.ops import StreamEncoder

    cfg = model.EncoderConfig(n_layers=2)
    m = model.random_model(cfg, seed=31)
    n_steps = 20
    mel = model.mel_stream(32, n_streams, 56 * n_steps, cfg.feat_in)
    g, e = StreamEncoder(m, n_streams), StreamEncoder(m, n_streams)
    e.set_graphs(False)
    refs = {z: oracle.StreamingEncoder(m) for z in sorted({0, n_streams - 1})}
    for r in refs.values():
        r.set_device_rounding()
    worst = 0.0
    for i in range(n_steps):
        t0, t1 = 56 * i, 56 * (i + 1)
        x = torch.from_numpy(np.ascontiguousarray(mel[:, t0:t1])).cuda()
        s = g.total()
        n0 = _lib.launch_count()
        g.encode_new(x, t0, t1)
        n_graph = _lib.launch_count() - n0
        a = _rows(torch, g)
        n0 = _lib.launch_count()
        e.encode_new(x.clone(), t0, t1)
        n_sep = _lib.launch_count() - n0
        b = _rows(torch, e)
        assert np.array_equal(a, b), f"step {i}: graph replay differs from separate launches"
        if i >= 11:
            assert n_graph == n_sep + 1, (i, n_graph, n_sep)
        for z, r in refs.items():
            assert r.encode_new(mel[z, :t1], t0, t1, False) == 0
            worst = max(worst, _err(a[z * 7:(z + 1) * 7], r.frames(s, r.total())))
        del x
    assert g.graph_stats() == (True, 2, n_steps - 11)
    assert e.graph_stats() == (False, 0, 0)
    print("%d streams: %d steps, graphs == separate launches; oracle worst max/RMS %.3g" % (n_streams, n_steps, worst))
    assert worst <= TOL
    g.close()
    e.close()


def test_step_graphs_host_entry(torch):
    """encode_new_host through step graphs with page-locked buffers: three
    mel buffers used in turn (so a graph meets a different buffer at each
    replay) and one output buffer, 256 streams, 18 steps; the frames equal
    those of encode_new with graphs off.  Step 16 passes a pageable mel
    array: it launches kernel by kernel (no graph launch) with the same
    bits, and step 17 replays again."""
    from stealcode_b200.ops import StreamEncoder

    n_streams, n_steps = 256, 18
    cfg = model.EncoderConfig(n_layers=2)
    m = model.random_model(cfg, seed=37)
    mel = model.mel_stream(38, n_streams, 56 * n_steps, cfg.feat_in)
    g, e = StreamEncoder(m, n_streams), StreamEncoder(m, n_streams)
    e.set_graphs(False)
    h_mel = [torch.empty((n_streams, 56, cfg.feat_in), dtype=torch.float32).pin_memory() for _ in range(3)]
    out = torch.empty((n_streams * cfg.max_frames, cfg.d_model), dtype=torch.float32).pin_memory()
    for i in range(n_steps):
        t0, t1 = 56 * i, 56 * (i + 1)
        x = np.ascontiguousarray(mel[:, t0:t1])
        before = g.graph_stats()[2]
        if i == 16:
            got = np.array(g.encode_new_host(x.copy(), t0, t1, out=out))
            assert g.graph_stats()[2] == before, "a pageable buffer must not go through a graph"
        else:
            h = h_mel[i % 3]
            h.copy_(torch.from_numpy(x))
            rows = g.encode_new_host_ptr(h.data_ptr(), t0, t1, False, out.data_ptr())
            got = out[:rows].numpy().copy()
        e.encode_new(torch.from_numpy(x).cuda(), t0, t1)
        ref = _rows(torch, e)
        assert got.shape == ref.shape
        assert np.array_equal(got, ref), f"step {i}: host entry through graphs differs"
    # graphs launched at steps 11-15 and 17
    assert g.graph_stats() == (True, 2, n_steps - 11 - 1)
    g.close()
    e.close()


def test_step_graphs_long_calls(torch):
    """56-frame calls (eight attention launches per call), 2 streams: every
    launch's band is steady from call 2, so calls 3 and 4 are captured and
    5-7 replay; same bits as separate launches.  Then graphs off and on
    again mid-stream: the next steps still match."""
    from stealcode_b200.ops import StreamEncoder

    cfg = model.EncoderConfig(n_layers=2, max_frames=64)
    m = model.random_model(cfg, seed=41)
    n_calls = 10
    mel = model.mel_stream(42, 2, 448 * n_calls, cfg.feat_in)
    g, e = StreamEncoder(m, 2), StreamEncoder(m, 2)
    e.set_graphs(False)
    for i in range(n_calls):
        if i == 8:
            g.set_graphs(False)
            assert g.graph_stats()[0] is False
            g.set_graphs(True)
        t0, t1 = 448 * i, 448 * (i + 1)
        x = torch.from_numpy(np.ascontiguousarray(mel[:, t0:t1])).cuda()
        g.encode_new(x, t0, t1)
        e.encode_new(x, t0, t1)
        assert np.array_equal(_rows(torch, g), _rows(torch, e)), f"call {i}"
    # calls 3-7 through graphs; after the reset, call 9 repeats call 8's
    # geometry and is captured (and launched) afresh
    assert g.graph_stats() == (True, 3, 6)
    g.close()
    e.close()


def test_step_graphs_prompt_mlp(torch):
    """The prompt MLP inside replayed step graphs: 3 streams with prompts
    (one none), 2 blocks, 128 prompts, 16 steps; at step 14, while graphs
    replay, the prompts change (the graph reads the per-stream prompt ids
    from device memory when it runs).  Every step equals the same encoder
    with graphs off."""
    from stealcode_b200.ops import StreamEncoder

    cfg = model.EncoderConfig(n_layers=2, n_prompts=128)
    m = model.random_model(cfg, seed=43)
    n_steps = 16
    mel = model.mel_stream(44, 3, 56 * n_steps, cfg.feat_in)
    g, e = StreamEncoder(m, 3), StreamEncoder(m, 3)
    e.set_graphs(False)
    for enc in (g, e):
        enc.set_prompts([None, 3, 127])
    for i in range(n_steps):
        if i == 14:
            for enc in (g, e):
                enc.set_prompts([5, None, 2])
        t0, t1 = 56 * i, 56 * (i + 1)
        x = torch.from_numpy(np.ascontiguousarray(mel[:, t0:t1])).cuda()
        g.encode_new(x, t0, t1)
        e.encode_new(x, t0, t1)
        assert np.array_equal(_rows(torch, g), _rows(torch, e)), f"step {i}"
    assert g.graph_stats() == (True, 2, n_steps - 11)
    g.close()
    e.close()
