"""Per-batch answers the vLLM speculator gives through vLLM's optional speculator hooks, from host tables only.

* ``suspend_drafting(num_reqs, req_ids)``: decode the batch natively (no draft, no verify) when it is above the verify
  batch limit (``max_verify_batch_size``, or the serve-mode default: 32 requests for trees, 48 for chains) or inside a
  batch-size range where the calibrated chain schedule chose width 0 (speculation does not pay there);
* ``verify_budget(req_ids, num_draft_tokens)``: verify at most the drafts the schedule gives the batch size being
  verified (width - 1 per request). vLLM sizes a request's drafts at the step that drafted them; trimming here makes a
  changed batch size's width apply from its first step. A tree's verify rows put parents before children, so a
  prefix of them is still a tree.

The hook names and parameters are vLLM's (the reference's ``eagle_harness/vllm/batch_policy.py`` answers the same
two). Decisions are counted; ``summary()`` reports them.
"""

from __future__ import annotations

from typing import Optional, Sequence, Tuple

import numpy as np

SPECULATOR_HOOKS = {"suspend_drafting": ("num_reqs", "req_ids"), "verify_budget": ("req_ids", "num_draft_tokens")}


class BatchPolicy:
    def __init__(self, *, verify_batch_limit: Optional[int] = None,
                 schedule: Optional[Sequence[Tuple[int, int, int]]] = None, max_num_reqs: int = 512):
        """``schedule``: (first batch size, last batch size, verify width) rows; width 0 decodes natively."""
        self.limit = verify_batch_limit
        self.native = tuple((int(a), int(b)) for a, b, w in (schedule or ()) if int(w) == 0)
        self.drafts: Optional[np.ndarray] = None
        if schedule:
            d = np.full(max_num_reqs + 1, np.iinfo(np.int64).max, dtype=np.int64)
            for a, b, w in schedule:
                d[max(int(a), 0):min(int(b), max_num_reqs) + 1] = max(int(w) - 1, 0)
            self.drafts = d
        self.batches = self.suspended = self.trimmed = 0

    def suspend_drafting(self, num_reqs: int, req_ids=None) -> bool:
        over = self.limit is not None and num_reqs > self.limit
        native = over or any(a <= num_reqs <= b for a, b in self.native)
        self.suspended += native
        return native

    def verify_budget(self, req_ids, num_draft_tokens):
        """``num_draft_tokens`` (per request) capped at the scheduled drafts of this batch size; the input itself when
        nothing is cut."""
        self.batches += 1
        n = np.asarray(num_draft_tokens)
        if self.drafts is None or n.size == 0:
            return num_draft_tokens
        cap = self.drafts[min(len(n), len(self.drafts) - 1)]
        if int(n.max()) <= cap:
            return num_draft_tokens
        self.trimmed += 1
        return np.minimum(n, cap)

    def summary(self) -> dict:
        return {"batches": self.batches, "trimmed": self.trimmed, "suspended": self.suspended}
