"""Failure detection among serving ranks, on the host: heartbeats in the process group's store and bounded waits.

Every rank publishes ``(step, time)`` after each round; before launching the next round's kernels (which wait on
peers) a rank checks that every peer has reached the previous step within ``timeout`` seconds, and raises
:class:`PeerFailure` naming the late ranks otherwise. A rank that crashed or hung is so detected between rounds, with
none of its collectives in flight, instead of inside a peer-memory wait. The device side is bounded too: the fused
collectives give up after one second and record ``kErrTimeoutPeer`` in the error word (``native.check_errors``).
"""

from __future__ import annotations

import time
from typing import Iterable, List, Optional

import torch.distributed as dist


class PeerFailure(RuntimeError):
    def __init__(self, ranks: List[int], step: int):
        super().__init__(f"ranks {ranks} did not reach step {step} in time (crashed, hung or partitioned)")
        self.ranks, self.step = ranks, step


class Heartbeat:
    """Per-rank step counters in a ``torch.distributed`` store (``TCPStore`` / ``FileStore``)."""

    def __init__(self, store: dist.Store, rank: int, world: int, *, prefix: str = "e4hb"):
        self.store, self.rank, self.world, self.prefix = store, rank, world, prefix
        self.step = 0

    def _key(self, r: int) -> str:
        return f"{self.prefix}/{r}"

    def beat(self, step: Optional[int] = None) -> None:
        self.step = self.step + 1 if step is None else step
        self.store.set(self._key(self.rank), f"{self.step}:{time.time():.6f}")

    def peer_step(self, r: int) -> int:
        try:
            self.store.wait([self._key(r)], _td(0.001))
        except Exception:  # noqa: BLE001 - a rank that never beat is at step -1
            return -1
        return int(self.store.get(self._key(r)).decode().split(":")[0])

    def check(self, step: int, timeout: float, ranks: Optional[Iterable[int]] = None, poll: float = 0.01) -> None:
        """Wait (at most ``timeout`` s) until every peer reports ``step``; raise :class:`PeerFailure` otherwise."""
        peers = [r for r in (ranks if ranks is not None else range(self.world)) if r != self.rank]
        deadline = time.monotonic() + timeout
        late = peers
        while True:
            late = [r for r in late if self.peer_step(r) < step]
            if not late:
                return
            if time.monotonic() > deadline:
                raise PeerFailure(late, step)
            time.sleep(poll)


def _td(seconds: float):
    import datetime

    return datetime.timedelta(seconds=seconds)


def process_group_heartbeat(group=None) -> Optional[Heartbeat]:
    """A :class:`Heartbeat` in the default process group's store (None without a multi-rank group)."""
    if not dist.is_initialized() or dist.get_world_size(group) < 2:
        return None
    from torch.distributed import distributed_c10d

    store = distributed_c10d._get_default_store()
    return Heartbeat(store, dist.get_rank(group), dist.get_world_size(group))
