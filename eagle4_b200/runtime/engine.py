"""The serving loop: prefill, plain decode and EAGLE tree rounds over one target and one draft head.

Round structure (the reference's SGLang worker, ``eagle_harness/sglang/worker.py:532-616`` and
``sglang/drafter.py:482-600``, re-planned around this package's kernels):

1. **draft extend** over the previous round's accepted rows (target aux hidden states, next tokens); its last row's
   top-``K`` seeds the tree (depth 1);
2. **draft steps**: ``K`` frontier rows per request attend to the frozen draft window plus their ancestors;
   ``DraftTree.step`` keeps the best ``K`` of the ``K*K`` children;
3. **verify**: the best ``N-1`` nodes plus the root, in node order, through the target in one forward;
4. **accept**: greedy walk over the rows (bonus = target token at the last accepted row);
5. **commit**: recurrent states replay the accepted path, attention KV of accepted rows moves to chain positions.

Invariants: the draft KV and the target KV both hold positions ``[0, L)`` of a request; rows of a round live past
``L`` (physical position ``L + row``) until commit. Plain decode is step 3-5 with one row, so every target op runs
the same arithmetic in both modes and greedy output is identical.
"""

from __future__ import annotations

import time
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence

import torch

from eagle4_b200 import ops
from eagle4_b200.core.draft_tree import DraftTree, TreeShape, rows_meta
from eagle4_b200.models.draft import DraftCache, DraftModel
from eagle4_b200.models.target import Records, RowBatch, TargetCache, TargetModel


@dataclass
class Request:
    prompt: List[int]
    max_new: int
    slot: int = -1
    out: List[int] = field(default_factory=list)
    L: int = 0  # committed positions in target and draft KV
    root: int = -1  # emitted token not yet run through the target
    ext_tokens: Optional[torch.Tensor] = None  # pending draft-extend tokens [n]
    ext_aux: Optional[torch.Tensor] = None  # pending draft-extend target features [n, n_aux*H]

    @property
    def done(self) -> bool:
        return len(self.out) >= self.max_new


@dataclass
class RoundStats:
    rounds: int = 0
    emitted: int = 0
    accepted_hist: Dict[int, int] = field(default_factory=dict)

    def record(self, accepted: Sequence[int]) -> None:
        self.rounds += 1
        for a in accepted:
            self.emitted += a
            self.accepted_hist[a] = self.accepted_hist.get(a, 0) + 1

    @property
    def mean_accept(self) -> float:
        n = sum(self.accepted_hist.values())
        return self.emitted / n if n else 0.0


class Engine:
    def __init__(self, target: TargetModel, draft: Optional[DraftModel], *, max_reqs: int, max_len: int,
                 page: int = 16, steps: int = 4, top_k: int = 2, verify_tokens: int = 8):
        self.target, self.draft = target, draft
        self.device = target.device
        self.dtype = target.dtype
        self.page = page
        self.steps, self.top_k, self.verify_tokens = steps, top_k, verify_tokens
        span = max(verify_tokens, steps * top_k) + 1
        self.max_len = max_len + span
        self.tcache = TargetCache.allocate(target.cfg, max_reqs=max_reqs, max_len=self.max_len, page=page,
                                           device=self.device, dtype=self.dtype)
        self.dcache = None
        self.tree = None
        if draft is not None:
            self.dcache = DraftCache.allocate(draft.cfg, self.tcache.block_table, page, self.device, self.dtype)
            shape = TreeShape(top_k=top_k, max_depth=steps)
            self.tree = DraftTree(shape, max_reqs, draft.cfg.hidden_size, self.dtype, self.device,
                                  max_verify=min(verify_tokens, shape.work_cap))
        self.free_slots = list(range(max_reqs))
        self.stats = RoundStats()

    # ------------------------------------------------------------------ helpers
    def _slot(self, req: int, pos: torch.Tensor) -> torch.Tensor:
        bt = self.tcache.block_table
        pos = pos.long()
        return bt[req, pos // self.page].long() * self.page + pos % self.page

    def _t(self, data, dtype) -> torch.Tensor:
        return torch.as_tensor(data, dtype=dtype, device=self.device)

    def admit(self, req: Request) -> None:
        req.slot = self.free_slots.pop(0)
        self.tcache.reset_slot(req.slot)

    def release(self, req: Request) -> None:
        self.free_slots.append(req.slot)
        self.free_slots.sort()

    # ------------------------------------------------------------------ prefill
    def prefill(self, reqs: List[Request]) -> None:
        """Run the prompts through the target (recurrent layers in scan mode); emit the first token."""
        for req in reqs:
            n = len(req.prompt)
            pos = torch.arange(n, device=self.device)
            slots = self._slot(req.slot, pos)
            one = lambda v: torch.full((n,), v, dtype=torch.int32, device=self.device)  # noqa: E731
            rb = RowBatch(
                ids=self._t(req.prompt, torch.int64), pos=pos, req=one(req.slot), write_slot=slots,
                ctx_start=one(0), ctx_len=(pos + 1).int(), extra=torch.zeros(n, 1, dtype=torch.int32,
                                                                             device=self.device),
                n_extra=one(0), parent=(pos - 1).int(), state_slot=one(req.slot), scan=True,
            )
            out, aux = self.target.forward(rb, self.tcache)
            ids, _ = self.target.greedy(out[-1:])
            req.root = int(ids[0])
            req.out.append(req.root)
            req.L = n
            if self.draft is not None:
                req.ext_tokens = torch.cat([self._t(req.prompt[1:], torch.int64), ids.view(1)])
                req.ext_aux = aux

    # ------------------------------------------------------------------ plain decode
    def plain_step(self, reqs: List[Request]) -> None:
        """One token per request: a one-row verify plus its commit."""
        bs = len(reqs)
        L = self._t([r.L for r in reqs], torch.int64)
        slots = torch.stack([self._slot(r.slot, L[i:i + 1])[0] for i, r in enumerate(reqs)])
        rb = RowBatch(
            ids=self._t([r.root for r in reqs], torch.int64), pos=L, req=self._t([r.slot for r in reqs], torch.int32),
            write_slot=slots, ctx_start=torch.zeros(bs, dtype=torch.int32, device=self.device), ctx_len=L.int(),
            extra=slots.int().view(bs, 1), n_extra=torch.ones(bs, dtype=torch.int32, device=self.device),
            parent=torch.full((bs,), -1, dtype=torch.int32, device=self.device),
            state_slot=self._t([r.slot for r in reqs], torch.int32),
        )
        rec = Records()
        out, _ = self.target.forward(rb, self.tcache, rec)
        ids, _ = self.target.greedy(out)
        rows = torch.arange(bs, dtype=torch.int32, device=self.device).view(bs, 1)
        self.target.commit(self.tcache, rec, rows, torch.ones(bs, dtype=torch.int32, device=self.device),
                           rb.state_slot, slots, slots)
        for r, t in zip(reqs, ids.tolist()):
            r.L += 1
            r.root = t
            r.out.append(t)

    # ------------------------------------------------------------------ speculative round
    def _draft_extend(self, reqs: List[Request]) -> None:
        draft, cfg = self.draft, self.draft.cfg
        ids, aux, pos, req_idx, last = [], [], [], [], []
        total = 0
        for r in reqs:
            n = r.ext_tokens.shape[0]
            ids.append(r.ext_tokens)
            aux.append(r.ext_aux)
            pos.append(torch.arange(r.L - n, r.L, device=self.device))
            req_idx.append(torch.full((n,), r.slot, dtype=torch.int32, device=self.device))
            total += n
            last.append(total - 1)
        ids, aux, pos, req_idx = torch.cat(ids), torch.cat(aux), torch.cat(pos), torch.cat(req_idx)
        t = ids.shape[0]
        w = cfg.sliding_window
        start = (pos - w + 1).clamp(min=0) if w else torch.zeros_like(pos)
        hidden = draft.project(aux)
        slots = self.tcache.block_table[req_idx.long(), pos // self.page].long() * self.page + pos % self.page
        normed, nh = draft.forward(ids, hidden, pos, req_idx, slots, start.int(), (pos + 1).int(),
                                   torch.zeros(t, 1, dtype=torch.int32, device=self.device),
                                   torch.zeros(t, dtype=torch.int32, device=self.device), self.dcache)
        sel = self._t(last, torch.int64)
        probs, toks = draft.candidates(normed.index_select(0, sel), self.top_k)
        self.tree.stage_root(len(reqs), probs, toks, nh.index_select(0, sel))
        for r in reqs:
            r.ext_tokens = r.ext_aux = None

    def _draft_steps(self, reqs: List[Request]) -> None:
        bs, k, tree, draft = len(reqs), self.top_k, self.tree, self.draft
        w = draft.cfg.sliding_window
        L = self._t([r.L for r in reqs], torch.int64)
        req_idx = self._t([r.slot for r in reqs], torch.int32).repeat_interleave(k)
        lane = torch.arange(k, device=self.device).repeat(bs)
        Lr = L.repeat_interleave(k)
        tree.begin(bs)
        for s in range(1, self.steps):
            phys = Lr + (s - 1) * k + lane
            slots = self.tcache.block_table[req_idx.long(), phys // self.page].long() * self.page + phys % self.page
            tree.set_step_slots(bs, s, slots.view(bs, k))
            extra = tree.ancestors[:bs, :, :s].reshape(bs * k, s).contiguous()
            n_extra = torch.full((bs * k,), s, dtype=torch.int32, device=self.device)
            start = (Lr - w).clamp(min=0) if w else torch.zeros_like(Lr)
            normed, nh = draft.forward(tree.front_tokens[: bs * k], tree.front_hidden[: bs * k], Lr - 1 + s, req_idx,
                                       slots, start.int(), Lr.int(), extra, n_extra, self.dcache)
            probs, toks = draft.candidates(normed, k)
            tree.step(bs, s, probs, toks, nh)

    def spec_round(self, reqs: List[Request]) -> None:
        bs, n = len(reqs), self.verify_tokens
        self._draft_extend(reqs)
        self._draft_steps(reqs)
        toks, prow = self.tree.verify_rows(bs, self.steps, n - 1)
        roots = self._t([r.root for r in reqs], torch.int64).view(bs, 1)
        tokens = torch.cat([roots, toks], dim=1)  # [bs, n]
        depth, mask = rows_meta(prow)
        L = self._t([r.L for r in reqs], torch.int64)
        sl = self._t([r.slot for r in reqs], torch.int32)
        rowidx = torch.arange(n, device=self.device)
        phys = L[:, None] + rowidx[None, :]
        slots = self.tcache.block_table[sl.long()[:, None], phys // self.page].long() * self.page + phys % self.page
        # extra slots: the row's ancestors and itself, in row order
        bits = ((mask[:, :, None] >> rowidx[None, None, :]) & 1).bool()  # [bs, n(row), n(j)]
        n_extra = bits.sum(-1).int()
        order = torch.argsort((~bits).int() * n + rowidx, dim=-1)  # set bits first, ascending j
        extra = torch.gather(slots[:, None, :].expand(bs, n, n), 2, order).int()
        parent = torch.where(prow >= 0, prow + torch.arange(bs, device=self.device)[:, None] * n, prow)
        rb = RowBatch(
            ids=tokens.reshape(-1), pos=(L[:, None] + depth).reshape(-1), req=sl.repeat_interleave(n),
            write_slot=slots.reshape(-1), ctx_start=torch.zeros(bs * n, dtype=torch.int32, device=self.device),
            ctx_len=L.int().repeat_interleave(n), extra=extra.reshape(bs * n, n), n_extra=n_extra.reshape(-1),
            parent=parent.reshape(-1).int(), state_slot=sl.repeat_interleave(n),
        )
        rec = Records()
        out, aux = self.target.forward(rb, self.tcache, rec)
        tid, _ = self.target.greedy(out)
        tid = tid.view(bs, n)
        acc, cnt, bonus = ops.accept_greedy(tid, tokens, prow, torch.full((bs,), n, dtype=torch.int32,
                                                                          device=self.device))
        acc_c, cnt_c, bonus_c = acc.cpu(), cnt.cpu(), bonus.cpu()
        base = torch.arange(bs, device=self.device)[:, None] * n
        rows = torch.where(acc >= 0, acc + base, torch.zeros_like(acc)).int()
        src = torch.gather(slots, 1, acc.clamp(min=0).long())
        dst = slots  # position L + d
        valid = rowidx[None, :] < cnt.to(self.device)[:, None]
        self.target.commit(self.tcache, rec, rows, cnt.to(self.device).int(), sl, src[valid], dst[valid])
        accepted = []
        for b, r in enumerate(reqs):
            c = int(cnt_c[b])
            path = acc_c[b, :c].tolist()
            new = [int(tokens[b, j]) for j in path[1:]] + [int(bonus_c[b])]
            room = r.max_new - len(r.out)
            r.out.extend(new[:room])
            accepted.append(min(len(new), room))
            keep = self._t(path, torch.int64) + b * n
            r.ext_tokens = self._t(new, torch.int64)
            r.ext_aux = aux.index_select(0, keep)
            r.L += c
            r.root = new[-1]
        self.stats.record(accepted)

    # ------------------------------------------------------------------ driver
    def generate(self, prompts: Sequence[Sequence[int]], max_new_tokens: int, *, speculative: bool = True
                 ) -> List[List[int]]:
        reqs = [Request(list(p), max_new_tokens) for p in prompts]
        for r in reqs:
            self.admit(r)
        self.prefill(reqs)
        active = [r for r in reqs if not r.done]
        while active:
            if speculative and self.draft is not None:
                self.spec_round(active)
            else:
                self.plain_step(active)
            active = [r for r in active if not r.done]
        for r in reqs:
            self.release(r)
        return [r.out[:max_new_tokens] for r in reqs]
