"""Tensor-parallel serving: rank 0's scheduler commands mirrored on every rank.

Under tensor parallelism every rank runs the same engine rounds over its weight shard, so every rank must admit the
same requests in the same order and step the same rounds. Rank 0 owns the request queue (the HTTP front end); before
each step it broadcasts one :class:`Command` (the requests submitted since the last step, or stop) over a separate
gloo group, and every other rank applies it to its own
:class:`~eagle4_b200.runtime.scheduler.Scheduler` (:func:`follow`).
The schedulers then stay identical without further messages: admission and retirement depend only on the submitted
requests and the emitted tokens, which every rank computes alike (the greedy head's argmax is exchanged between
ranks), and the engine's timing-based round choices take the maximum over ranks before deciding.

While rank 0 is idle it broadcasts an empty command every ``beat_s`` seconds, so a follower waiting longer than the
control group's timeout has lost its leader and ends with an error instead of waiting forever. An engine error on
any rank ends serving on that rank (the process exits non-zero and the launcher tears the group down): ranks whose
collectives may be out of step are not resumed; a restart is the recovery path.
"""

from __future__ import annotations

import datetime
from dataclasses import dataclass, field
from typing import List, Optional, Sequence, Tuple, Union

import torch.distributed as dist

from eagle4_b200.runtime.scheduler import Request, RequestParams, Scheduler


@dataclass
class Command:
    submit: List[Tuple[Sequence[int], RequestParams]] = field(default_factory=list)
    stop: bool = False


class Lockstep:
    """The control channel: a gloo group over the default group's ranks (created collectively, on every rank)."""

    def __init__(self, *, timeout_s: float = 60.0, beat_s: float = 1.0):
        if beat_s >= timeout_s:
            raise ValueError("the idle beat must come well within the control timeout")
        self.rank = dist.get_rank()
        self.world = dist.get_world_size()
        self.group = dist.new_group(backend="gloo", timeout=datetime.timedelta(seconds=timeout_s))
        self.beat_s = beat_s
        self.sent = 0

    @property
    def leader(self) -> bool:
        return self.rank == 0

    def exchange(self, cmd: Optional[Command] = None) -> Command:
        """Rank 0 sends ``cmd``; every rank returns it."""
        if self.leader and cmd is None:
            raise ValueError("rank 0 sends a command")
        box = [cmd if self.leader else None]
        dist.broadcast_object_list(box, src=0, group=self.group)
        self.sent += 1
        return box[0]


def apply(sched: Scheduler, cmd: Command) -> List[Union[Request, ValueError]]:
    """Submit a command's requests: the queued request, or the refusal (the same on every rank) for each."""
    out: List[Union[Request, ValueError]] = []
    for prompt, params in cmd.submit:
        try:
            out.append(sched.submit(prompt, params))
        except ValueError as e:
            out.append(e)
    return out


def follow(engine, lockstep: Lockstep, *, speculative: bool = True, detokenize=None,
           batch_prefill: bool = False) -> int:
    """A non-leader rank's serving loop: apply each command, step while requests run, return on stop.
    ``detokenize`` and ``batch_prefill`` must be the leader's (stop strings end requests, and prefills group, on
    every rank alike)."""
    if lockstep.leader:
        raise ValueError("rank 0 leads; follow() runs on the other ranks")
    sched = Scheduler(engine, speculative=speculative, detokenize=detokenize, batch_prefill=batch_prefill)
    rounds = 0
    while True:
        cmd = lockstep.exchange()
        if cmd.stop:
            return rounds
        apply(sched, cmd)
        if not sched.idle:
            sched.step()
            rounds += 1
