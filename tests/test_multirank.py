"""Multi-rank host logic of the benchmark on CPU (gloo, world size 2): the
max-over-ranks timing reduction, the stream sharding of independent streams
over GPUs, and the reference arm printing on rank 0 only.  No GPU."""
import os
import socket

import pytest
import torch.multiprocessing as mp

import bench


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out):
    import datetime

    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        got = bench.reduce_max(1.5 + rank, "cpu")
        lo, hi = bench.stream_shard(8192, world, rank)
        out.put((rank, got, lo, hi))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_reduce_max_and_shards_over_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert [r[1] for r in res] == [2.5, 2.5]  # every rank sees the max
    assert res[0][2:] == (0, 4096) and res[1][2:] == (4096, 8192)


@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_stream_shard_covers_every_stream_once(world):
    for total in (256, 8192, 1000):
        spans = [bench.stream_shard(total, world, r) for r in range(world)]
        assert spans[0][0] == 0 and spans[-1][1] == total
        assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
        sizes = [hi - lo for lo, hi in spans]
        assert max(sizes) - min(sizes) <= 1


def test_reduce_max_without_process_group_is_identity():
    assert bench.reduce_max(3.25, "cpu") == 3.25


def test_reference_arm_prints_on_rank_zero_only(capsys):
    class A:
        warmup, steps, gpus = 1, 1, 2

    bench.run_reference(A(), rank=1)
    assert capsys.readouterr().out == ""
