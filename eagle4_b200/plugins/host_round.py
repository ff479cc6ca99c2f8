"""The draft half of EAGLE-4 rounds over a serving host's target, shared by the engine adapters.

A host (SGLang, vLLM, TokenSpeed) keeps its scheduler, KV pools and target model. Around its target forwards it needs
the draft side of every round: take each new request's prompt rows (the target's aux hidden states and first token),
draft a tree per running request and hand back the verify rows (tokens, parent rows), and after the host's verify and
accept, take the accepted path. :class:`HostDrafter` runs exactly the engine's draft half on the host's requests:
draft KV in its own page pool, pending rows (the accepted tokens and their aux states awaiting the next extend), the
draft tree, and the round policy (cost model, live costs) deciding depth and verify width. The verify rows it returns
are those the engine itself would verify, so a host that verifies and accepts them greedily emits exactly plain
greedy decoding (tested against the engine with fake hosts).

Reference counterparts: the drafter inside each adapter (``eagle_harness/sglang/drafter.py:482-691``,
``eagle_harness/vllm/tree_drafter.py:155``, ``eagle_harness/tokenspeed/drafter.py:49``).
"""

from __future__ import annotations

from typing import Dict, Hashable, List, Optional, Sequence, Tuple

import torch

from eagle4_b200.models.configs import TargetConfig
from eagle4_b200.models.draft import DraftModel
from eagle4_b200.runtime.engine import Engine


class _HostTarget:
    """Stands in for the target inside the drafter's engine: no layers (the host owns the target and its caches)."""

    def __init__(self, draft: DraftModel):
        c = draft.cfg
        self.cfg = TargetConfig(family="llama", hidden_size=c.target_hidden_size, vocab_size=c.vocab_size,
                                layers=[], intermediate_size=0)
        self.device = draft.device
        self.dtype = draft.w["fc"].dtype
        self.tp = None


class HostDrafter:
    def __init__(self, draft: DraftModel, *, max_reqs: int, max_len: int, page: int = 16, steps: int = 12,
                 top_k: int = 4, verify_tokens: int = 16, config=None, temperature: float = 0.0, seed: int = 0):
        self.engine = Engine(_HostTarget(draft), draft, max_reqs=max_reqs, max_len=max_len, page=page, steps=steps,
                             top_k=top_k, verify_tokens=verify_tokens, config=config, temperature=temperature,
                             seed=seed)
        self.order: List[Hashable] = []  # request id of each engine batch row
        self.slot_of: Dict[Hashable, int] = {}
        self.free = list(range(max_reqs - 1, -1, -1))

    @property
    def top_k(self) -> int:
        return self.engine.top_k

    # ------------------------------------------------------------------ requests
    def admit(self, rid: Hashable, prompt: torch.Tensor, aux: torch.Tensor, first_token) -> None:
        """A request the host prefilled: its prompt ids, the target's aux hidden states of the prompt rows
        ``[n, num_aux * H_target]`` and the first generated token."""
        eng = self.engine
        if rid in self.slot_of:
            raise ValueError(f"request {rid!r} is already admitted")
        if not self.free:
            raise RuntimeError("every draft row is in use")
        b = len(self.order)
        slot = self.free.pop()
        self.slot_of[rid] = slot
        self.order.append(rid)
        n = int(prompt.shape[0])
        eng.slot[b] = slot
        eng.pages.release(slot)
        eng.pages.reserve(slot, eng.max_len)
        first = torch.as_tensor(first_token, dtype=torch.int64, device=eng.device).view(1)
        eng.L[b] = n
        eng.root[b] = first[0]
        eng._draft_prefill(b, prompt.to(eng.device), aux.to(eng.device), first)
        if eng.tree is not None and len(self.order) == 1:
            eng.lagged_scores = None

    def release(self, rid: Hashable) -> None:
        """A finished request: its row is filled by the last row, its draft pages return to the pool."""
        eng = self.engine
        b = self.order.index(rid)
        last = len(self.order) - 1
        if b != last:
            for t in (eng.L, eng.root, eng.slot, eng.ext_tok, eng.ext_cnt, eng.ext_aux):
                t[b] = t[last]
            self.order[b] = self.order[last]
        self.order.pop()
        slot = self.slot_of.pop(rid)
        eng.pages.release(slot)
        self.free.append(slot)

    def _arrange(self, rids: Sequence[Hashable]) -> int:
        """Put the requests in the host's batch order (the engine rows [0, bs)); returns bs."""
        rids = list(rids)
        if rids != self.order[:len(rids)]:
            missing = [r for r in rids if r not in self.slot_of]
            if missing:
                raise KeyError(f"requests {missing} were never admitted")
            rest = [r for r in self.order if r not in set(rids)]
            perm = torch.tensor([self.order.index(r) for r in rids + rest], device=self.engine.device)
            eng = self.engine
            for t in (eng.L, eng.root, eng.slot, eng.ext_tok, eng.ext_cnt, eng.ext_aux):
                t[:len(perm)] = t.index_select(0, perm)
            self.order = rids + rest
        return len(rids)

    # ------------------------------------------------------------------ rounds
    def propose(self, rids: Sequence[Hashable], context: Optional[int] = None
                ) -> Tuple[torch.Tensor, torch.Tensor]:
        """Draft the round's trees for ``rids`` (the host's batch order). Returns the verify rows: tokens
        ``[bs, w]`` (the committed root first) and parent rows ``[bs, w]`` (-1 for the root), w chosen by the round
        policy."""
        eng = self.engine
        bs = self._arrange(rids)
        rows = eng.bucket(bs)
        eng._pad(bs, rows)
        ctx = context if context is not None else int(eng.L[:bs].float().mean().item())
        policy = eng.policy.begin_round(rows)
        width, _ = eng._draft_round(rows, ctx, policy)
        if width > 1:
            toks, prow = eng.tree.verify_rows(rows, eng.steps, width - 1)
            tokens = torch.cat([eng.root[:rows, None], toks], dim=1)
        else:
            tokens = eng.root[:rows, None].clone()
            prow = torch.full((rows, 1), -1, dtype=torch.int32, device=eng.device)
        self._rows, self._width = rows, width
        return tokens[:bs], prow[:bs]

    def tree_nodes(self, bs: int) -> torch.Tensor:
        """Tree node of every verify row of the last proposal (-1: root), for a sampled accept."""
        if self._width > 1:
            return self.engine.tree.last_nodes[:bs]
        return torch.full((bs, 1), -1, dtype=torch.int64, device=self.engine.device)

    def accept(self, rids: Sequence[Hashable], tokens: torch.Tensor, accepted: torch.Tensor, counts: torch.Tensor,
               bonus: torch.Tensor, aux: Optional[torch.Tensor]) -> List[List[int]]:
        """The host's verdict on the proposed rows: accepted row indices ``[bs, w]`` (-1 pad), counts ``[bs]``, bonus
        tokens ``[bs]`` and the verify rows' aux hidden states ``[bs * w, A]``. Returns each request's emitted tokens
        (its accepted drafted tokens, then the bonus)."""
        eng = self.engine
        bs = self._arrange(rids)
        w = tokens.shape[1]
        eng._record_accept(bs, w, tokens, accepted, counts, bonus, aux)
        if eng.policy.cost is not None and eng.tree is not None:
            _, cum = eng.tree.rank_reference(bs, eng.steps, eng.verify_tokens - 1)
            eng.lagged_scores = cum.mean(dim=0).tolist()
        cnt = eng.out_cnt[:bs].tolist()
        out = eng.out_tok[:bs].tolist()
        return [row[:c] for row, c in zip(out, cnt)]


class ServedTreeRounds:
    """Served rounds' periods per (batch size, verify width), written to ``<data_path>/rounds/tree.json`` (the served
    tree schedule's input, ``core.chain_width.served_tree_schedule``): mean round period, mean tokens emitted per
    request and round, and the round count of every cell. ``flush`` merges the cells into the file (other cells kept);
    it runs every ``flush_every`` rounds and when the host closes the method."""

    def __init__(self, data_path: str, flush_every: int = 256):
        self.data_path, self.flush_every = data_path, flush_every
        self.cells: Dict[Tuple[int, int], List[float]] = {}  # (bs, width) -> [sum us, sum tokens, rounds]
        self._since = 0

    def record(self, batch_size: int, width: int, round_us: float, tokens_per_request: float) -> None:
        c = self.cells.setdefault((int(batch_size), int(width)), [0.0, 0.0, 0])
        c[0] += float(round_us)
        c[1] += float(tokens_per_request)
        c[2] += 1
        self._since += 1
        if self._since >= self.flush_every:
            self.flush()

    def flush(self) -> Optional[str]:
        from eagle4_b200.core.chain_width import merge_tree_rounds

        self._since = 0
        rows = [{"batch_size": b, "width": w, "round_us": s / n, "accept": max(1.0, a / n), "count": n}
                for (b, w), (s, a, n) in sorted(self.cells.items()) if n and s > 0]
        return merge_tree_rounds(self.data_path, rows) if rows else None
