"""Round policy of the serving loop: the fixed tree shape, or the measured cost model fed by live costs.

Mirrors the reference drafter's policy choice (``eagle_harness/sglang/drafter.py:315-389``): a round uses the cost
model once its batch bucket is priced, else the fixed shape (static mode, or the live seed sweep, which forces each
captured verify width for a few rounds so every width of the bucket gets timed). Live cells are refreshed into the
cost model's tables when a bucket becomes ready and every ``LIVE_REFRESH_ROUNDS`` rounds; buckets whose measured
costs the cost model's checks refuse keep the fixed shape.
"""

from __future__ import annotations

import logging
import os
from collections import Counter
from typing import Callable, List, Optional, Sequence

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

    def record(self, bs: int, width: int, context: int, verify_us: float, steps: int, draft_us: float) -> None:
        """One served round's timings: the verify at ``width`` and the mean draft step."""
        if self.live is None:
            return
        self.live.record(bs, width, context, verify_us)
        if steps > 0:
            self.live.record(bs, DRAFT_WIDTH, context, draft_us / steps)


class ServedChainPolicy:
    """Chain width per batch bucket for chain rounds (top-k 1), chosen on served rounds.

    A calibrated schedule (``core.chain_width.chain_widths``: served round times or cost tables, with the acceptance
    profile) fixes the width per batch size when one is given. Otherwise each batch bucket first serves every
    candidate width for ``probe_rounds`` rounds, measuring the round period and the tokens a request gains per round,
    then serves the width with the most tokens per microsecond (``(1 + accepted) / round_us``, the rule of
    ``core.chain_width``), re-probing the other widths every ``refresh`` rounds so a changed acceptance moves it
    (reference ``eagle_harness/sglang/chain_rounds.py``: served chain choices, searched per batch key).
    """

    def __init__(self, widths: Sequence[int], *, probe_rounds: int = 4, refresh: int = 256,
                 schedule: Optional[List[tuple]] = None):
        self.widths = sorted(set(int(w) for w in widths if w >= 1))
        if not self.widths:
            raise ValueError("a chain policy needs at least one width")
        self.probe_rounds, self.refresh, self.schedule = probe_rounds, refresh, schedule
        self.samples: dict = {}  # (bucket, width) -> [round_us sum, tokens sum, rounds]
        self.rounds: Counter = Counter()

    @staticmethod
    def bucket(bs: int) -> int:
        return 1 << max(bs - 1, 0).bit_length()

    def width(self, bs: int) -> int:
        if self.schedule:
            from eagle4_b200.core.chain_width import width_at

            return max(1, width_at(self.schedule, bs))
        b = self.bucket(bs)
        n = self.rounds[b]
        period = len(self.widths) * self.probe_rounds
        if n < period or (self.refresh and n % self.refresh < period):
            return self.widths[(n % period) // self.probe_rounds]
        return self.best(b)

    def best(self, bucket: int) -> int:
        def rate(w):
            us, tok, r = self.samples.get((bucket, w), (0.0, 0.0, 0))
            return (tok / r) / (us / r) if r and us > 0 else -1.0

        return max(self.widths, key=lambda w: (rate(w), -w))

    def record(self, bs: int, width: int, round_us: float, tokens_per_request: float) -> None:
        b = self.bucket(bs)
        self.rounds[b] += 1
        us, tok, r = self.samples.get((b, width), (0.0, 0.0, 0))
        self.samples[(b, width)] = (us + round_us, tok + tokens_per_request, r + 1)


class ServedTreeChoice:
    """Per batch bucket: speculate (1) or decode natively (0), chosen on served rounds.

    The cost model prices a tree from draft and verify costs and an acceptance prior; what a round actually yields
    depends on the draft. So each bucket serves ``probe_rounds`` speculative rounds and ``probe_rounds`` native
    rounds, compares tokens per microsecond (tokens a request gains per round over the round period), serves the
    better choice, and probes again every ``refresh`` rounds. A measured schedule (``rounds/tree.json`` reduced to
    0 / 1 per batch key, or packaged served choices) fixes the choice instead (reference served tree choices:
    ``eagle_harness/core/cost_profiles.py:packaged_served_choices`` and the served-round search of
    ``eagle_harness/sglang/chain_rounds.py``).
    """

    SPECULATE, NATIVE = 1, 0

    def __init__(self, *, probe_rounds: int = 4, refresh: int = 256, choices: Optional[dict] = None):
        self.probe_rounds, self.refresh, self.choices = probe_rounds, refresh, choices
        self.samples: dict = {}
        self.rounds: Counter = Counter()

    @staticmethod
    def bucket(bs: int) -> int:
        return 1 << max(bs - 1, 0).bit_length()

    def choice(self, bs: int) -> int:
        b = self.bucket(bs)
        if self.choices:
            keys = sorted(self.choices)
            return self.choices[min(keys, key=lambda k: (abs(k - b), -k))]
        n = self.rounds[b]
        period = 2 * self.probe_rounds
        if n < period or (self.refresh and n % self.refresh < period):
            return self.SPECULATE if (n % period) < self.probe_rounds else self.NATIVE
        return self.best(b)

    def best(self, bucket: int) -> int:
        def rate(c):
            us, tok, r = self.samples.get((bucket, c), (0.0, 0.0, 0))
            return tok / us if r and us > 0 else -1.0

        return self.SPECULATE if rate(self.SPECULATE) >= rate(self.NATIVE) else self.NATIVE

    def record(self, bs: int, choice: int, round_us: float, tokens_per_request: float) -> None:
        b = self.bucket(bs)
        self.rounds[b] += 1
        us, tok, r = self.samples.get((b, choice), (0.0, 0.0, 0))
        self.samples[(b, choice)] = (us + round_us, tok + tokens_per_request, r + 1)
