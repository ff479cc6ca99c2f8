"""Per-round records of the serving loop, exported as JSON lines (observability; the reference's round recorder).

Each record: round index, batch size, round kind (``tree`` / ``chain`` / ``native`` / ``plain``), drafted depth and
verify width, tokens emitted per request, and the round's device time when it was timed. ``summary()`` gives tokens
per round, acceptance histogram and time shares over the most recent ``keep`` rounds (a long-running server keeps a
bounded window in memory; the file has every round). Enable with ``Engine.recorder = RoundRecorder(path)``.
"""

from __future__ import annotations

import json
import os
from collections import Counter, deque
from typing import List, Optional


class RoundRecorder:
    def __init__(self, path: Optional[str] = None, flush_every: int = 256, keep: int = 65536):
        self.path, self.flush_every = path, flush_every
        self.records: "deque[dict]" = deque(maxlen=keep)
        self._pending: List[dict] = []
        self.rounds = 0

    def record(self, *, bs: int, kind: str, depth: int, width: int, tokens: List[int],
               round_us: Optional[float] = None) -> None:
        rec = {"round": self.rounds, "bs": bs, "kind": kind, "depth": depth, "width": width,
               "tokens_per_request": sum(tokens) / max(1, len(tokens)), "accepted_hist": dict(Counter(tokens))}
        if round_us is not None:
            rec["round_us"] = round(round_us, 2)
        self.rounds += 1
        self.records.append(rec)
        self._pending.append(rec)
        if self.path and len(self._pending) >= self.flush_every:
            self.flush()

    def flush(self) -> None:
        if not self.path or not self._pending:
            return
        os.makedirs(os.path.dirname(self.path) or ".", exist_ok=True)
        with open(self.path, "a", encoding="utf-8") as f:
            for rec in self._pending:
                f.write(json.dumps(rec) + "\n")
        self._pending.clear()

    def summary(self) -> dict:
        kinds = Counter(r["kind"] for r in self.records)
        timed = [r for r in self.records if "round_us" in r]
        toks = sum(r["tokens_per_request"] for r in self.records)
        return {"rounds": len(self.records), "kinds": dict(kinds),
                "tokens_per_round": toks / max(1, len(self.records)),
                "mean_round_us": sum(r["round_us"] for r in timed) / max(1, len(timed)) if timed else None}
