"""Rank-failure handling of the multi-GPU driver's stream shards, on CPU
(processes and a TCPStore; no GPU): a rank that leaves between steps, or
hangs past the heartbeat timeout, is dropped and the survivors take over its
streams, every stream owned by exactly one rank at every step."""
import socket
import time

import pytest
import torch.multiprocessing as mp

from stealcode_b200 import shards


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, streams, behaviour, out):
    import datetime

    from torch.distributed import TCPStore

    store = TCPStore("127.0.0.1", port, world, rank == 0, timeout=datetime.timedelta(seconds=30))
    sh = shards.StreamShards(store, rank, world, streams, timeout_s=1.0)
    log = []
    try:
        for step in range(3):
            if step == 1 and behaviour == "leave":
                out.put((rank, "left", log))
                return
            if step == 1 and behaviour == "hang":
                time.sleep(2.5)  # misses the heartbeat window, then comes back
            lo, hi, taken = sh.step(step)
            log.append((step, lo, hi, taken, list(sh.live)))
        out.put((rank, "ok", log))
    except RuntimeError as exc:
        out.put((rank, "dropped: " + str(exc), log))
    finally:
        if rank == 0:
            time.sleep(1.0)  # the store's host outlives the other ranks' last reads


def _run(world, streams, behaviours):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, streams, behaviours.get(r, ""), q))
             for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in procs:
        r, status, log = q.get(timeout=120)
        res[r] = (status, log)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    return res


def _check_cover(spans, streams):
    owned = sorted(z for lo, hi in spans for z in range(lo, hi))
    assert owned == list(range(streams))


def test_rank_leaving_between_steps_is_taken_over():
    streams = 1000
    res = _run(3, streams, {2: "leave"})
    assert res[2][0] == "left"
    assert res[0][0] == "ok" and res[1][0] == "ok"
    step0 = {r: res[r][1][0] for r in (0, 1)}
    assert step0[0][1:3] == shards.stream_shard(streams, 3, 0)
    old2 = range(*shards.stream_shard(streams, 3, 2))
    for step in (1, 2):
        spans = [res[r][1][step][1:3] for r in (0, 1)]
        _check_cover(spans, streams)
        assert all(res[r][1][step][4] == [0, 1] for r in (0, 1))
    taken = sorted(res[0][1][1][3] + res[1][1][1][3])
    assert set(old2) <= set(taken)  # rank 2's streams moved to the survivors
    assert res[0][1][2][3] == [] and res[1][1][2][3] == []  # nothing moves once settled


def test_rank_hanging_past_the_timeout_is_dropped():
    streams = 64
    res = _run(2, streams, {1: "hang"})
    assert res[1][0].startswith("dropped"), res[1][0]
    assert res[0][0] == "ok"
    for step in (1, 2):
        assert res[0][1][step][1:3] == (0, streams)
        assert res[0][1][step][4] == [0]


@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_plans_cover_every_stream_once(world):
    for streams in (256, 8192, 1001):
        for live in ([*range(world)], [r for r in range(world) if r != world // 2] or [0]):
            _check_cover(shards.plan(streams, live).values(), streams)
