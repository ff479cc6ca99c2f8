"""Round policy of the serving loop: the fixed tree shape, or the measured cost model fed by live costs.

Mirrors the reference drafter's policy choice (``eagle_harness/sglang/drafter.py:315-389``): a round uses the cost
model once its batch bucket is priced, else the fixed shape (static mode, or the live seed sweep, which forces each
captured verify width for a few rounds so every width of the bucket gets timed). Live cells are refreshed into the
cost model's tables when a bucket becomes ready and every ``LIVE_REFRESH_ROUNDS`` rounds; buckets whose measured
costs the cost model's checks refuse keep the fixed shape.
"""

from __future__ import annotations

import logging
import math
import os
from collections import Counter
from typing import List, Optional, Sequence

from eagle4_b200.core.config import HarnessConfig, Mode, build_cost_model
from eagle4_b200.core.cost_model import CostModel, FixedShapePolicy, depth_loss_ratio
from eagle4_b200.core.cost_table import cost_model_problem
from eagle4_b200.core.limits import verify_buckets
from eagle4_b200.core.live_costs import DRAFT_WIDTH, CostKey, LiveCosts

log = logging.getLogger(__name__)

LIVE_REFRESH_ROUNDS = 64


def round_up_width(width: int, widths: Sequence[int]) -> int:
    """The smallest captured width ``>= width`` (the widest when none is)."""
    up = [w for w in widths if w >= width]
    return min(up) if up else max(widths)


def fit_width(width: int, widths: Sequence[int], available: int) -> int:
    """The captured verify width for a requested ``width`` with ``available`` tree tokens (root included): the
    smallest captured width >= width if the tree fills it, else the widest one it fills."""
    up = round_up_width(width, widths)
    if up <= available:
        return up
    return max(w for w in widths if w <= available)


class RoundPolicy:
    def __init__(self, config: HarnessConfig, *, top_k: int, steps: int, verify_tokens: int,
                 target_is_moe: bool = False, key: Optional[CostKey] = None):
        self.config = config
        self.top_k, self.steps, self.verify_tokens = top_k, steps, verify_tokens
        self.fixed = FixedShapePolicy(config.intensity, top_k, steps, verify_tokens)
        self.cost: Optional[CostModel] = None
        self.live: Optional[LiveCosts] = None
        self.visits: Counter = Counter()
        self.rounds = 0
        self.unpriced: set = set()
        self.key = key
        if not config.mode.uses_cost_model:
            return
        if config.data_path:
            self.cost = build_cost_model(config, node_top_k=top_k, tree_depth=steps, verify_num=verify_tokens,
                                         target_is_moe=target_is_moe, key=key)
            return
        loss = depth_loss_ratio(config.draft_family.value, target_is_moe=target_is_moe, intensity=config.intensity)
        self.cost = CostModel(tables={}, params=config.cost_model.params(loss), intensity=config.intensity,
                              node_top_k=top_k, tree_depth=steps, verify_num=verify_tokens,
                              target_is_moe=target_is_moe)
        self.live = LiveCosts(self.widths, key=key, draft_shape=(top_k, steps))
        if key is not None and self.live.load(self.cache_path):
            self._refresh()

    # ------------------------------------------------------------------ shapes
    def widths(self, bucket: int) -> List[int]:
        """Verify widths with a graph at ``bucket``: the calibrated buckets up to the configured draft tokens, plus
        the configured width itself; widest first."""
        ws = {w for w in verify_buckets(bucket, self.config.intensity) if w <= self.verify_tokens}
        ws.update({1, self.verify_tokens})
        return sorted(ws, reverse=True)

    @property
    def cache_path(self) -> str:
        return os.path.join(self.config.cost_cache_dir, f"{self.key.digest}.json")

    # ------------------------------------------------------------------ rounds
    def begin_round(self, bs: int):
        """The policy object of this round (``CostModel`` or ``FixedShapePolicy``)."""
        self.rounds += 1
        if self.cost is None:
            return self.fixed
        if self.live is None:
            return self.cost
        self.visits[bs] += 1
        ready = self.live.ready(bs)
        if ready and (bs not in self.cost.tables or self.rounds % LIVE_REFRESH_ROUNDS == 0):
            self._refresh()
        if ready and bs in self.cost.tables and bs not in self.unpriced:
            self.fixed.force_width = None
            return self.cost
        self.fixed.force_width = self.live.seed_width(bs)
        return self.fixed

    def _refresh(self) -> None:
        tables = self.live.tables(also=tuple(self.visits))
        for b, t in tables.items():
            problem = cost_model_problem(t, target_is_moe=self.cost.target_is_moe)
            if problem is None:
                self.unpriced.discard(b)
            elif b not in self.unpriced:
                self.unpriced.add(b)
                log.warning("eagle4_b200: batch bucket %d keeps the fixed draft shape: %s", b, problem)
        self.cost.set_tables(tables, refused=self.unpriced)
        if self.key is not None:
            try:
                self.live.save(self.cache_path)
            except OSError as e:  # a read-only cache directory only costs a re-measurement next start
                log.info("live cost cache not saved: %s", e)

    def record(self, bs: int, width: int, context: int, verify_us: float, steps: int, draft_us: float,
               settled: bool = True) -> None:
        """One served round's timings: the verify at ``width`` and the mean draft step. A round that ran eagerly or
        captured a graph (``settled`` False) is not a cost sample."""
        if self.live is None or not settled:
            return
        self.live.record(bs, width, context, verify_us)
        if steps > 0:
            self.live.record(bs, DRAFT_WIDTH, context, draft_us / steps)


class _ServedSearch:
    """Chooses one action per batch bucket from tokens per microsecond measured on served rounds.

    Exploration serves the actions in interleaved blocks of ``block`` rounds until each has ``explore`` settled
    periods, so every action sees the same load. A period is settled when nothing but serving happened inside it: a
    round that ran a kernel sequence eagerly or captured a CUDA graph is counted as served but never priced (a
    capture costs as much as dozens of rounds). Periods longer than ``stall`` times the action's median are dropped
    too. The rate of an action is the ratio of its token and time sums (ratio estimator, with its variance); the
    decision is served for ``interval`` rounds, then the bucket explores again from fresh samples. The interval
    doubles while the decision stays the same (up to ``max_interval``) and falls back to ``refresh`` when it changes,
    so a change of acceptance moves the choice while a steady workload pays for exploration ever more rarely.
    (Behaviour of the reference's served choices, ``eagle_harness/sglang/chain_rounds.py:232-628``: settled periods
    only, a stall filter, a ratio estimator with a standard-error margin; its decisions are permanent, these are
    re-checked.)
    """

    def __init__(self, actions: Sequence[int], *, block: int = 4, explore: int = 8, stall: float = 3.0,
                 refresh: int = 256, max_interval: int = 8192):
        self.actions = list(actions)
        if not self.actions:
            raise ValueError("a served search needs at least one action")
        self.block, self.explore, self.stall = max(1, block), max(2, explore), stall
        self.refresh, self.max_interval = refresh, max(refresh, max_interval)
        self.samples: dict = {}  # (bucket, action) -> [(us, tokens)] settled periods of the current exploration
        self.served: Counter = Counter()  # (bucket, action) -> rounds served
        self.rounds: Counter = Counter()  # bucket -> rounds served
        self.decided: dict = {}  # bucket -> action
        self._since: Counter = Counter()  # bucket -> rounds served since the decision
        self._interval: dict = {}  # bucket -> rounds until the next exploration
        self._explored: Counter = Counter()  # bucket -> rounds of the current exploration
        self._last: dict = {}  # bucket -> the previous decision

    @staticmethod
    def bucket(bs: int) -> int:
        return 1 << max(bs - 1, 0).bit_length()

    def action(self, bs: int) -> int:
        b = self.bucket(bs)
        if len(self.actions) == 1:
            return self.actions[0]
        if b in self.decided and (not self.refresh or self._since[b] < self._interval[b]):
            return self.decided[b]
        if b in self.decided:  # the interval ran out: explore again from fresh samples
            del self.decided[b]
            self._explored[b] = 0
            for a in self.actions:
                self.samples.pop((b, a), None)
        return self.actions[(self._explored[b] // self.block) % len(self.actions)]

    def record(self, bs: int, action: int, round_us: float, tokens_per_request: float, settled: bool = True) -> None:
        b = self.bucket(bs)
        self.rounds[b] += 1
        self.served[(b, action)] += 1
        if b in self.decided:
            self._since[b] += 1
            return
        self._explored[b] += 1
        if settled and round_us > 0:
            self.samples.setdefault((b, action), []).append((float(round_us), float(tokens_per_request)))
        have = [len(self._settled(b, a)) for a in self.actions]
        # an exploration whose rounds keep being unsettled still ends (every action priced from what it has)
        if min(have) >= self.explore or self._explored[b] >= 8 * self.explore * len(self.actions):
            self._decide(b)

    def _settled(self, b: int, a: int) -> List[tuple]:
        s = self.samples.get((b, a), [])
        if len(s) < 2:
            return list(s)
        us = sorted(u for u, _ in s)
        limit = self.stall * us[len(us) // 2]
        return [x for x in s if x[0] <= limit]

    def rate(self, bucket: int, action: int) -> tuple:
        """``(tokens per us, variance)`` of the action's settled periods; ``(-1, inf)`` without any."""
        s = self._settled(bucket, action)
        n, us = len(s), sum(u for u, _ in s)
        if n == 0 or us <= 0:
            return -1.0, math.inf
        r = sum(t for _, t in s) / us
        if n < 2:
            return r, math.inf
        mean_us = us / n
        return r, sum((t - r * u) ** 2 for u, t in s) / (n * (n - 1) * mean_us ** 2)

    def _winner(self, b: int) -> int:
        return max(self.actions, key=lambda a: (self.rate(b, a)[0], -a))

    def _decide(self, b: int) -> None:
        win = self._winner(b)
        previous, self._last[b] = self._last.get(b), win
        if previous != win:
            self._interval[b] = self.refresh
        else:
            self._interval[b] = min(self.max_interval, 2 * self._interval.get(b, self.refresh))
        self.decided[b] = win
        self._since[b] = 0
        log.info("served choice at batch bucket %d: %s (tokens/us %s)", b, win,
                 {a: round(self.rate(b, a)[0], 6) for a in self.actions})

    def share(self, action: int) -> float:
        """The fraction of served rounds that took ``action`` (all buckets)."""
        total = sum(self.served.values())
        return sum(v for (_, a), v in self.served.items() if a == action) / total if total else 0.0


class ServedChainPolicy(_ServedSearch):
    """Chain width per batch bucket for chain rounds (top-k 1), chosen on served rounds.

    A calibrated schedule (``core.chain_width.chain_widths``: served round times or cost tables, with the acceptance
    profile) fixes the width per batch size when one is given. Otherwise each bucket explores the candidate widths
    on served rounds and serves the one with the most tokens per microsecond (``(1 + accepted) / round_us``, the rule
    of ``core.chain_width``); see :class:`_ServedSearch` for how periods are priced and when the choice is
    re-checked (reference ``eagle_harness/sglang/chain_rounds.py:232``: served chain choices per batch key).
    """

    def __init__(self, widths: Sequence[int], *, schedule: Optional[List[tuple]] = None, **kw):
        widths = sorted(set(int(w) for w in widths if w >= 1))
        if not widths:
            raise ValueError("a chain policy needs at least one width")
        super().__init__(widths, **kw)
        self.widths, self.schedule = widths, schedule

    def width(self, bs: int) -> int:
        if self.schedule:
            from eagle4_b200.core.chain_width import width_at

            return max(1, width_at(self.schedule, bs))
        return self.action(bs)

    def best(self, bucket: int) -> int:
        return self._winner(bucket)


class ServedTreeChoice(_ServedSearch):
    """Per batch bucket: speculate (1) or decode natively (0), chosen on served rounds.

    The cost model prices a tree from draft and verify costs and an acceptance prior; what a round actually yields
    depends on the draft. So each bucket explores both on served rounds (see :class:`_ServedSearch`) and speculates
    only when its tokens per microsecond beat native decode's by ``margin_se`` standard errors: a tie serves native
    decode, which spends no draft work. A measured schedule (``rounds/tree.json`` reduced to 0 / 1 per batch key, or
    packaged served choices) fixes the choice instead (reference served tree choices:
    ``eagle_harness/core/cost_profiles.py:packaged_served_choices`` and ``ServedTreePolicy`` in
    ``eagle_harness/sglang/chain_rounds.py:556``).
    """

    SPECULATE, NATIVE = 1, 0

    def __init__(self, *, margin_se: float = 2.0, choices: Optional[dict] = None, **kw):
        super().__init__([self.SPECULATE, self.NATIVE], **kw)
        self.margin_se, self.choices = margin_se, choices

    def choice(self, bs: int) -> int:
        if self.choices:
            b = self.bucket(bs)
            keys = sorted(self.choices)
            return self.choices[min(keys, key=lambda k: (abs(k - b), -k))]
        return self.action(bs)

    def _winner(self, b: int) -> int:
        (rs, vs), (rn, vn) = self.rate(b, self.SPECULATE), self.rate(b, self.NATIVE)
        margin = self.margin_se * math.sqrt(vs + vn) if math.isfinite(vs + vn) else 0.0
        return self.SPECULATE if rs - rn > margin else self.NATIVE

    def best(self, bucket: int) -> int:
        return self._winner(bucket)
