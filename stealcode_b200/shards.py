"""Stream shards over ranks, with rank-failure detection on the host.

Audio streams are independent, so a multi-GPU run gives each rank (one
process per GPU) a contiguous span of the global streams and needs no
collective on the data path.  Before each step every rank posts a heartbeat
for that step to a shared key-value store (torch.distributed's TCPStore); a
rank whose heartbeat has not arrived within the timeout is taken as gone
(it crashed, hung, or left between steps), and the survivors split the
global streams over the live ranks again.  The streams a rank takes over
start from fresh encoder state on it (their caches were in the lost rank's
GPU memory), like a stream that has just connected.

The reference runs one stream per StreamingEncoder on one machine and has no
multi-process driver (its failure handling is a CPU fallback when the GPU
context cannot be created, gpu/context.rs:43-87); this module is the
B200 build's multi-GPU host logic.
"""
from __future__ import annotations

import time
from typing import Dict, List, Sequence, Tuple


def stream_shard(global_streams: int, world: int, rank: int) -> Tuple[int, int]:
    """Span [lo, hi) of the global streams that rank `rank` of `world`
    encodes; the first ranks take the remainder."""
    base, extra = divmod(global_streams, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def plan(global_streams: int, live: Sequence[int]) -> Dict[int, Tuple[int, int]]:
    """Spans of every live rank (in rank order) covering all streams once."""
    live = sorted(live)
    return {r: stream_shard(global_streams, len(live), i) for i, r in enumerate(live)}


class StreamShards:
    """This rank's stream span, kept consistent across ranks by heartbeats.

    step(s) posts this rank's heartbeat for step s, waits up to `timeout_s`
    for the others' and returns (lo, hi, taken_over): this rank's span for
    step s and the streams in it that another rank held at step s - 1.  A
    rank that misses a step's heartbeat is dropped for good; every survivor
    sees the same set (a late rank that posts after the others gave up on
    it is still dropped: it finds itself missing from the step's member list
    and must stop)."""

    def __init__(self, store, rank: int, world: int, global_streams: int, timeout_s: float = 5.0,
                 prefix: str = "shards"):
        self.store, self.rank, self.world = store, rank, world
        self.global_streams, self.timeout_s, self.prefix = global_streams, timeout_s, prefix
        self.live: List[int] = list(range(world))
        self.spans = plan(global_streams, self.live)

    def _key(self, step: int, r: int) -> str:
        return f"{self.prefix}/hb/{step}/{r}"

    def step(self, step: int) -> Tuple[int, int, List[int]]:
        self.store.set(self._key(step, self.rank), "1")
        deadline = time.monotonic() + self.timeout_s
        seen = {self.rank}
        while len(seen) < len(self.live):
            for r in self.live:
                if r not in seen and self.store.check([self._key(step, r)]):
                    seen.add(r)
            if len(seen) == len(self.live) or time.monotonic() > deadline:
                break
            time.sleep(0.005)
        # the step's members are decided once, by the lowest live rank that
        # saw them; everyone else adopts that list, so all survivors agree
        members_key = f"{self.prefix}/members/{step}"
        leader = min(seen)
        if self.rank == leader:
            self.store.compare_set(members_key, "", ",".join(str(r) for r in sorted(seen)))
        self.store.wait([members_key], _timedelta(self.timeout_s * 4))
        members = [int(v) for v in self.store.get(members_key).decode().split(",")]
        if self.rank not in members:
            raise RuntimeError(f"rank {self.rank} was dropped at step {step}")
        old = self.spans
        self.live = members
        self.spans = plan(self.global_streams, members)
        lo, hi = self.spans[self.rank]
        olo, ohi = old.get(self.rank, (0, 0))
        taken = [z for z in range(lo, hi) if not (olo <= z < ohi)]
        return lo, hi, taken


def _timedelta(seconds: float):
    import datetime

    return datetime.timedelta(seconds=seconds)
