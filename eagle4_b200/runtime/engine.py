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

Every step of a round reads and writes *device state* (committed lengths, roots, pending draft-extend rows, emitted
tokens) with fixed shapes, so on a GPU one round is one CUDA-graph replay per batch size and the host reads only the
emitted tokens once per round. Invariants: draft and target KV hold positions ``[0, L)`` of a request; a round's rows
live past ``L`` (physical position ``L + row``) until commit. Plain decode is steps 3-5 with one row, so every target
op runs the same arithmetic in both modes and greedy output is identical.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence

import torch

from eagle4_b200 import ops
from eagle4_b200.core.config import HarnessConfig, Mode
from eagle4_b200.core.cost_model import CostModel
from eagle4_b200.core.draft_tree import DraftTree, TreeShape
from eagle4_b200.core.limits import COST_BATCH_SIZES
from eagle4_b200.runtime.pages import PagePool
from eagle4_b200.runtime.policy import RoundPolicy, ServedChainPolicy, ServedTreeChoice, fit_width
from eagle4_b200.runtime.round_plan import DECIDE, KIND as PLAN_KIND, LAST, LAUNCH, RoundCheck, round_plan
from eagle4_b200.models.draft import DraftCache, DraftModel
from eagle4_b200.models.target import Records, RowBatch, TargetCache, TargetModel


@dataclass
class RoundStats:
    rounds: int = 0
    emitted: int = 0
    accepted_hist: Dict[int, int] = field(default_factory=dict)
    # natively decoded positions left without draft KV (the draft's attention reads stale KV there until its window
    # moves past them); the reference counts the same slots (``StaleDraftKV``, ``eagle_harness/sglang/draft_kv.py:90``)
    draft_kv_holes: int = 0

    def record(self, accepted: Sequence[int]) -> None:
        self.rounds += 1
        for a in accepted:
            self.emitted += a
            self.accepted_hist[a] = self.accepted_hist.get(a, 0) + 1

    @property
    def mean_accept(self) -> float:
        n = sum(self.accepted_hist.values())
        return self.emitted / n if n else 0.0


def tree_rows_meta(prow: torch.Tensor):
    """Device-side verify-row structure from parent rows ``[bs, n]`` (row 0 the root with -1).

    Returns ``(depth [bs, n] int64, anc [bs, n, n] bool)`` where ``anc[b, r, j]`` says row ``j`` is ``r`` or one of
    its ancestors (path doubling over the parent relation; no host synchronisation).
    """
    bs, n = prow.shape
    dev = prow.device
    eye = torch.eye(n, dtype=torch.float32, device=dev).expand(bs, n, n)
    par = torch.zeros(bs, n, n, dtype=torch.float32, device=dev)
    par.scatter_(2, prow.clamp(min=0).long()[:, :, None], 1.0)
    par[:, 0, :] = 0.0
    anc = eye + par
    reach = 1
    while reach < n:
        anc = ((anc + torch.bmm(anc, anc)) > 0).float()
        reach *= 2
    depth = anc.sum(-1).long() - 1
    return depth, anc > 0


def _launch_count() -> int:
    if not torch.cuda.is_available():
        return 0
    from eagle4_b200.ops import native

    return native.LAUNCHES[0]


def _count_launches(n: int) -> None:
    """Account this package's kernels launched by a graph replay (recorded at capture) in ``native.LAUNCHES``."""
    if torch.cuda.is_available():
        from eagle4_b200.ops import native

        native.LAUNCHES[0] += n


class _Stamp:
    """A CUDA event on a GPU, a host clock reading on the CPU (the CPU path has no asynchrony)."""

    def __init__(self, device: torch.device):
        self.cuda = device.type == "cuda"
        self.ev = torch.cuda.Event(enable_timing=True) if self.cuda else None
        self.t = 0.0

    def record(self) -> None:
        if self.cuda:
            self.ev.record()
        else:
            import time

            self.t = time.perf_counter()

    def elapsed_us(self, later: "_Stamp") -> float:
        if self.cuda:
            return self.ev.elapsed_time(later.ev) * 1e3
        return (later.t - self.t) * 1e6


SAMPLED_STREAM = 0x10000  # random stream of the tree walk's coins (draft steps use streams 0..steps-1)


class Engine:
    def __init__(self, target: TargetModel, draft: Optional[DraftModel], *, max_reqs: int, max_len: int,
                 page: int = 16, steps: int = 4, top_k: int = 2, verify_tokens: int = 8, use_graphs: bool = True,
                 config: Optional[HarnessConfig] = None, temperature: float = 0.0, seed: int = 0,
                 kv_tokens: Optional[int] = None):
        """``temperature > 0`` samples: draft children are drawn without replacement from the draft's candidate
        distribution and verified by recursive tree rejection, so the output follows the target's distribution at
        that temperature (``temperature == 0``: greedy, equal to plain greedy decoding). ``kv_tokens``: positions
        the attention caches hold over all requests (default ``max_reqs * max_len``); a request's pages are mapped
        when it is admitted, for the positions it can reach."""
        self.target, self.draft = target, draft
        self.temperature, self.seed = float(temperature), int(seed)
        self.device = target.device
        self.dtype = target.dtype
        self.page = page
        self.steps, self.top_k, self.verify_tokens = steps, top_k, verify_tokens
        self.max_reqs = max_reqs
        span = max(verify_tokens, steps * top_k) + 1
        self.max_len = max_len + span
        self.span = span
        row_pages = -(-self.max_len // page)  # a row reaching max_len holds whole pages
        kv_pages = (kv_tokens // page if kv_tokens is not None else max_reqs * row_pages) + 2  # + trash page
        # one cache row beyond the requests' rows: batch rows that pad a round up to its graph bucket use it (its
        # block-table row maps only the trash page, its recurrent state belongs to no request)
        self.pad_slot = max_reqs
        # prompts longer than this prefill in chunks (the recurrent states and the KV carry over between chunks)
        self.prefill_chunk = 8192
        self.tcache = TargetCache.allocate(target.cfg, max_reqs=max_reqs + 1, max_len=self.max_len, page=page,
                                           device=self.device, dtype=self.dtype, kv_pages=kv_pages)
        self.pages = PagePool(self.tcache.block_table, kv_pages, page)
        self.dcache = None
        self.tree = None
        if draft is not None:
            self.dcache = DraftCache.allocate(draft.cfg, self.tcache.block_table, page, self.device, self.dtype,
                                              pages=kv_pages)
            shape = TreeShape(top_k=top_k, max_depth=steps)
        self.config = config or HarnessConfig(mode=Mode.STATIC)
        self.policy = RoundPolicy(self.config, top_k=top_k, steps=steps, verify_tokens=verify_tokens,
                                  target_is_moe=target.cfg.is_moe)
        # chain rounds (top-k 1): the width per batch bucket is chosen on served rounds (or a calibrated schedule)
        self.chain_policy = None
        if draft is not None and top_k == 1 and self.config.mode.uses_cost_model:
            schedule = None
            if self.config.data_path:
                from eagle4_b200.core.chain_width import chain_widths

                schedule = chain_widths(self.config.data_path, verify_tokens, max_reqs)
            self.chain_policy = ServedChainPolicy(range(2, verify_tokens + 1), schedule=schedule)
        # batches above the verify limit decode natively (reference default: 32 requests for trees, 48 for chains,
        # in serve mode; an explicit max_verify_batch_size applies in every mode)
        limit = self.config.max_verify_batch_size
        if limit is None and self.config.mode.uses_cost_model:
            limit = 48 if top_k == 1 else 32
        self.verify_batch_limit = limit
        # failure detection among tensor-parallel ranks: a Heartbeat (parallel.health) beats and checks every
        # ``heartbeat_every`` rounds, before the round's collectives
        self.heartbeat = None
        self.heartbeat_every, self.heartbeat_timeout = 64, 30.0
        self._rounds_served = 0
        # serve mode: per batch bucket, speculate or decode natively, whichever yields more tokens per microsecond
        self.tree_choice = None
        if draft is not None and top_k > 1 and self.config.mode.uses_cost_model:
            self.tree_choice = ServedTreeChoice()
        if draft is not None:
            # work deltas are only read by the cost model's decisions
            slots = None if self.policy.cost is not None else ()
            budget = max(verify_tokens, self.policy.cost.max_history_verify_num if self.policy.cost else 1)
            self.tree = DraftTree(shape, max_reqs, draft.cfg.hidden_size, self.dtype, self.device,
                                  max_verify=min(budget, shape.work_cap), delta_slots=slots)
        dev, n = self.device, verify_tokens
        i64, i32 = torch.int64, torch.int32
        self.round_ctr = torch.zeros(1, dtype=i32, device=dev)
        # plain sampling reads one (empty) candidate set per request
        self.plain_q = torch.zeros(max_reqs, 1, 1, dtype=torch.float32, device=dev)
        self.plain_ids = torch.zeros(max_reqs, 1, 1, dtype=i32, device=dev)
        self.plain_slot = torch.zeros(max_reqs, 1, dtype=i32, device=dev)
        if self.sampled and draft is not None:
            cap = self.tree.shape.capacity
            self.cands = draft.cfg.num_candidates if draft.cfg.low_rank else min(256, draft.cfg.draft_vocab_size)
            self.q_store = torch.zeros(max_reqs, 1 + cap, self.cands, dtype=torch.float32, device=dev)
            self.q_ids = torch.zeros(max_reqs, 1 + cap, self.cands, dtype=i32, device=dev)
            self.node_slot = torch.zeros(max_reqs, cap, dtype=i32, device=dev)
            self.tree.keep_draw_order = True
        # device state, one row per batch position
        self.L = torch.zeros(max_reqs, dtype=i64, device=dev)
        self.root = torch.zeros(max_reqs, dtype=i64, device=dev)
        self.slot = torch.arange(max_reqs, dtype=i32, device=dev)
        self.ext_tok = torch.zeros(max_reqs, n, dtype=i64, device=dev)
        self.ext_cnt = torch.zeros(max_reqs, dtype=i32, device=dev)
        # host mirror of ext_cnt (prefills and the rounds' read-back counts set it): a native round on a request
        # whose ring is full drops its oldest pending row, a position that never gets draft KV
        self.pending_host = [0] * max_reqs
        aux_w = (draft.cfg.num_aux * draft.cfg.target_hidden_size) if draft is not None else 1
        self.ext_aux = torch.zeros(max_reqs, n, aux_w, dtype=self.dtype, device=dev)
        self.out_tok = torch.zeros(max_reqs, n, dtype=i64, device=dev)
        self.out_cnt = torch.zeros(max_reqs, dtype=i32, device=dev)
        pin = dev.type == "cuda"
        self.host_tok = torch.zeros(max_reqs, n, dtype=i64, pin_memory=pin)
        self.host_cnt = torch.zeros(max_reqs, dtype=i32, pin_memory=pin)
        self.use_graphs = use_graphs and dev.type == "cuda"
        # rounds run at graph buckets (the calibration batch grid up to max_reqs): a batch of bs requests replays the
        # graph of the smallest bucket >= bs, its extra rows padding on the spare cache row
        self.buckets = sorted({b for b in COST_BATCH_SIZES if b < max_reqs} | {max_reqs})
        self.graphs: Dict[tuple, torch.cuda.CUDAGraph] = {}
        self.pool = torch.cuda.graph_pool_handle() if self.use_graphs else None
        self.graph_launches: Dict[tuple, int] = {}
        self._captured = False  # a graph was captured during the current round
        self.last_timing: Dict[str, float] = {}
        self.stats = RoundStats()
        # set to a RoundCheck to compare every planned DECIDE stop with the cost model's own decision
        self.round_check: Optional[RoundCheck] = None
        self.recorder = None  # a runtime.recorder.RoundRecorder to keep per-round records
        if self.tree is not None:
            self.host_deltas = torch.zeros(tuple(self.tree.deltas.shape), dtype=torch.float32, pin_memory=pin)
            self.host_scores = torch.zeros(n, dtype=torch.float32, pin_memory=pin)
            self.lagged_scores: Optional[List[float]] = None
            self.last_depth = self.last_width = 0

    # ------------------------------------------------------------------ helpers
    @property
    def sampled(self) -> bool:
        return self.temperature > 0

    def _sample(self, normed: torch.Tensor, front_nodes: Optional[torch.Tensor], lanes: int, stream: int,
                child_base: int):
        """Sampled children of the rows of ``normed`` (see ``ops.sample_children``)."""
        ids, logit = self.draft.candidate_logits(normed)
        if logit.shape[1] > self.cands:  # full-vocabulary head: its top candidates are the proposal's support
            logit, pick = ops.topk_rows(logit, self.cands)
            ids = ids.gather(1, pick)
        return ops.sample_children(logit, ids, self.top_k, self.temperature, self.seed, self.round_ctr, stream,
                                   front_nodes, lanes, self.q_store, self.q_ids, self.node_slot, child_base)

    def _slots(self, slot: torch.Tensor, pos: torch.Tensor) -> torch.Tensor:
        """Physical KV slots of positions ``pos`` in the block-table rows ``slot`` (broadcasting)."""
        pos = pos.long()
        return self.tcache.block_table[slot.long(), pos // self.page].long() * self.page + pos % self.page

    def _segments(self, n: int) -> torch.Tensor:
        """The scan segment table of one request's ``n`` rows, built on the device (no host round trip)."""
        seg = torch.full((2,), n, dtype=torch.int32, device=self.device)
        seg[0] = 0
        return seg

    def _i32(self, n: int, v: int) -> torch.Tensor:
        return torch.full((n,), v, dtype=torch.int32, device=self.device)

    # ------------------------------------------------------------------ prefill (eager)
    def prefill(self, b: int, prompt: torch.Tensor, reserve_tokens: Optional[int] = None):
        """Prompt of batch row ``b`` through the target (recurrent layers in scan mode); the first token becomes the
        root; the draft consumes all but the last ``N`` prompt rows now and the rest at the first round. The row's
        KV pages are mapped first, for ``reserve_tokens`` positions (default: the engine's ``max_len``). Returns
        (first token [1], the prompt rows' aux hidden states or None)."""
        n = prompt.shape[0]
        slot = int(self.slot[b])
        self.pages.release(slot)
        self.pages.reserve(slot, reserve_tokens if reserve_tokens is not None else self.max_len)
        self.tcache.reset_slot(slot)
        auxes = []
        for s in range(0, n, self.prefill_chunk):  # long prompts in chunks: bounded activations, same results
            e = min(n, s + self.prefill_chunk)
            t = e - s
            pos = torch.arange(s, e, device=self.device)
            slots = self._slots(torch.tensor(slot, device=self.device), pos)
            rb = RowBatch(ids=prompt[s:e].to(self.device), pos=pos, req=self._i32(t, slot), write_slot=slots,
                          ctx_start=self._i32(t, 0), ctx_len=(pos + 1).int(),
                          extra=torch.zeros(t, 1, dtype=torch.int32, device=self.device), n_extra=self._i32(t, 0),
                          parent=torch.arange(-1, t - 1, device=self.device, dtype=torch.int32),
                          state_slot=self._i32(t, slot), scan=True, max_keys=e, segments=self._segments(t))
            out, aux = self.target.forward(rb, self.tcache)
            auxes.append(aux)
        aux = auxes[0] if len(auxes) == 1 else (None if auxes[0] is None else torch.cat(auxes))
        if self.sampled:
            dev = self.device
            _, _, first = self.target.sampled_accept(out[-1:], self.temperature,
                                             torch.full((1, 1), -1, dtype=torch.int32, device=dev),
                                             torch.zeros(1, 1, dtype=torch.int64, device=dev),
                                             torch.full((1, 1), -1, dtype=torch.int64, device=dev), self.plain_q[:1],
                                             self.plain_ids[:1], self.plain_slot[:1], 1, self.seed, self.round_ctr,
                                             SAMPLED_STREAM + 2)
            ops.advance_round(self.round_ctr)
        else:
            first, _ = self.target.greedy(out[-1:])
        self.L[b] = n
        self.root[b] = first[0]
        self.out_tok[b, 0] = first[0]
        self.out_cnt[b] = 1
        if self.draft is not None:
            self._draft_prefill(b, prompt, aux, first)
        return first, aux

    def prefill_many(self, rows: List[int], prompts: List[torch.Tensor],
                     reserve_tokens: Optional[List[int]] = None) -> List[torch.Tensor]:
        """Several requests' prompts through the target in one scan-mode forward (each request its own segment of
        contiguous rows; per-row attention, per-segment recurrences and row-independent GEMMs make every request's
        result the one ``prefill`` gives it alone), then each request's first token and draft share as in
        ``prefill``. ``rows``: the batch rows (their ``slot`` set). Returns the first tokens, in order."""
        if len(rows) == 1:
            return [self.prefill(rows[0], prompts[0], reserve_tokens[0] if reserve_tokens else None)[0]]
        dev = self.device
        lens = [int(p.shape[0]) for p in prompts]
        slots_of = [int(self.slot[b]) for b in rows]
        for i, slot in enumerate(slots_of):
            self.pages.release(slot)
            self.pages.reserve(slot, reserve_tokens[i] if reserve_tokens is not None else self.max_len)
            self.tcache.reset_slot(slot)
        pos = torch.cat([torch.arange(n, device=dev) for n in lens])
        slot_rows = torch.cat([self._i32(n, s) for n, s in zip(lens, slots_of)])
        starts = [0]
        for n in lens:
            starts.append(starts[-1] + n)
        parent = torch.arange(starts[-1], device=dev, dtype=torch.int32) - 1
        parent[torch.tensor(starts[:-1], device=dev)] = -1
        t = starts[-1]
        rb = RowBatch(ids=torch.cat([p.to(dev) for p in prompts]), pos=pos, req=slot_rows,
                      write_slot=self._slots(slot_rows.long(), pos), ctx_start=self._i32(t, 0),
                      ctx_len=(pos + 1).int(), extra=torch.zeros(t, 1, dtype=torch.int32, device=dev),
                      n_extra=self._i32(t, 0), parent=parent, state_slot=slot_rows, scan=True, max_keys=max(lens),
                      segments=torch.tensor(starts, dtype=torch.int32, device=dev))
        out, aux = self.target.forward(rb, self.tcache)
        last = torch.tensor([s - 1 for s in starts[1:]], device=dev)
        firsts: List[torch.Tensor] = []
        if self.sampled:  # one draw per request, in order, as ``prefill`` draws them
            for i in range(len(rows)):
                _, _, first = self.target.sampled_accept(
                    out[last[i]:last[i] + 1], self.temperature,
                    torch.full((1, 1), -1, dtype=torch.int32, device=dev), torch.zeros(1, 1, dtype=torch.int64,
                                                                                      device=dev),
                    torch.full((1, 1), -1, dtype=torch.int64, device=dev), self.plain_q[:1], self.plain_ids[:1],
                    self.plain_slot[:1], 1, self.seed, self.round_ctr, SAMPLED_STREAM + 2)
                ops.advance_round(self.round_ctr)
                firsts.append(first.view(1))
        else:
            ids, _ = self.target.greedy(out.index_select(0, last))
            firsts = [ids[i:i + 1] for i in range(len(rows))]
        for i, b in enumerate(rows):
            first = firsts[i]
            self.L[b] = lens[i]
            self.root[b] = first[0]
            self.out_tok[b, 0] = first[0]
            self.out_cnt[b] = 1
            if self.draft is not None:
                self._draft_prefill(b, prompts[i], aux[starts[i]:starts[i + 1]], first)
        return firsts

    def _draft_prefill(self, b: int, prompt: torch.Tensor, aux: torch.Tensor, first: torch.Tensor) -> None:
        """The draft's share of a prefill: the prompt's leading rows through the draft now (their draft KV), the last
        ``N`` rows (tokens shifted by one, with their aux hidden states) left pending for the first round's extend."""
        n = prompt.shape[0]
        slot = int(self.slot[b])
        pos = torch.arange(n, device=self.device)
        nxt = torch.cat([prompt.to(self.device)[1:], first.to(self.device).view(1)])  # token after each position
        keep = min(n, self.verify_tokens)
        lead = n - keep
        if lead:  # the leading rows' outputs are never read: only their draft KV is written
            if self.device.type == "cuda":  # prefill GEMM launches
                from eagle4_b200.ops import native

                with native.prefill_gemms():
                    self._draft_kv(nxt[:lead], self.draft.project(aux[:lead]), pos[:lead], slot)
            else:
                self._draft_kv(nxt[:lead], self.draft.project(aux[:lead]), pos[:lead], slot)
        self.ext_tok[b, :keep] = nxt[lead:]
        self.ext_aux[b, :keep] = aux[lead:]
        self.ext_cnt[b] = keep
        self.pending_host[b] = keep

    def _track_pending(self, bs: int, counts: List[int], native: bool) -> None:
        n = self.verify_tokens
        for b in range(bs):
            if not native:
                self.pending_host[b] = min(counts[b], n)
            elif self.pending_host[b] >= n:
                self.stats.draft_kv_holes += 1
            else:
                self.pending_host[b] += 1

    def _draft_kv(self, ids, hidden, pos, slot: int) -> None:
        self.draft.write_kv(ids, hidden, pos, self._slots(torch.tensor(slot, device=self.device), pos), self.dcache)

    # ------------------------------------------------------------------ device-state rounds
    def _plain_round(self, bs: int) -> None:
        """One token per request: a one-row verify plus its commit, all on device state."""
        L, sl = self.L[:bs], self.slot[:bs]
        slots = self._slots(sl, L)
        rb = RowBatch(ids=self.root[:bs].clone(), pos=L.clone(), req=sl, write_slot=slots,
                      ctx_start=torch.zeros(bs, dtype=torch.int32, device=self.device), ctx_len=L.int(),
                      extra=slots.int().view(bs, 1), n_extra=torch.ones(bs, dtype=torch.int32, device=self.device),
                      parent=torch.full((bs,), -1, dtype=torch.int32, device=self.device), state_slot=sl,
                      max_keys=self.max_len)
        rec = Records()
        out, aux = self.target.forward(rb, self.tcache, rec)
        if self.sampled:  # plain sampling: the walk with no children draws from p
            dev = self.device
            _, _, ids = self.target.sampled_accept(out, self.temperature,
                                           torch.full((bs, 1), -1, dtype=torch.int32, device=dev), self.root[:bs, None],
                                           torch.full((bs, 1), -1, dtype=torch.int64, device=dev), self.plain_q,
                                           self.plain_ids, self.plain_slot, 1, self.seed, self.round_ctr,
                                           SAMPLED_STREAM)
            ops.advance_round(self.round_ctr)
        else:
            ids, _ = self.target.greedy(out)
        rows = torch.arange(bs, dtype=torch.int32, device=self.device).view(bs, 1)
        self.target.commit(self.tcache, rec, rows, torch.ones(bs, dtype=torch.int32, device=self.device), sl,
                           slots, slots)
        self.L[:bs] += 1
        self.root[:bs] = ids
        self.out_tok[:bs, 0] = ids
        self.out_cnt[:bs] = 1
        if self.draft is not None and aux is not None:
            # keep the draft's pending rows (the most recent N) so a later speculative round extends from here
            n = self.verify_tokens
            cnt = self.ext_cnt[:bs].long()
            full = (cnt >= n)[:, None]
            self.ext_tok[:bs] = torch.where(full, torch.roll(self.ext_tok[:bs], -1, 1), self.ext_tok[:bs])
            self.ext_aux[:bs] = torch.where(full[:, :, None], torch.roll(self.ext_aux[:bs], -1, 1), self.ext_aux[:bs])
            at = cnt.clamp(max=n - 1)
            b = torch.arange(bs, device=self.device)
            self.ext_tok[b, at] = ids
            self.ext_aux[b, at] = aux
            self.ext_cnt[:bs] = (cnt + 1).clamp(max=n).int()

    def _draft_extend(self, bs: int) -> None:
        """Pending rows (``ext_cnt <= N`` per request, padded to N) through the draft; the last valid row's top-K
        seeds the tree. Padded rows write draft KV into the tree region past L, which the steps overwrite."""
        n, dev = self.verify_tokens, self.device
        draft, w = self.draft, self.draft.cfg.sliding_window
        cnt = self.ext_cnt[:bs].long()
        d = torch.arange(n, device=dev)
        pos = (self.L[:bs, None] - cnt[:, None] + d[None, :]).clamp(min=0)  # [bs, n]
        sl = self.slot[:bs]
        slots = self._slots(sl[:, None], pos)
        start = (pos - w + 1).clamp(min=0) if w else torch.zeros_like(pos)
        hidden = draft.project(self.ext_aux[:bs].reshape(bs * n, -1))
        t = bs * n
        normed, nh = draft.forward(self.ext_tok[:bs].reshape(-1), hidden, pos.reshape(-1),
                                   sl.repeat_interleave(n), slots.reshape(-1), start.reshape(-1).int(),
                                   (pos + 1).reshape(-1).int(), torch.zeros(t, 1, dtype=torch.int32, device=dev),
                                   torch.zeros(t, dtype=torch.int32, device=dev), self.dcache,
                                   max_keys=self.max_len)
        last = torch.arange(bs, device=dev) * n + (cnt - 1).clamp(min=0)
        if self.sampled:
            probs, toks = self._sample(normed.index_select(0, last), None, 1, 0, 0)
        else:
            probs, toks = draft.candidates(normed.index_select(0, last), self.top_k,
                                           pos.reshape(-1).index_select(0, last))
        self.tree.stage_root(bs, probs, toks, nh.index_select(0, last))

    def _phase_begin(self, bs: int) -> None:
        """Draft extend, then depth 1 of a fresh tree (its work deltas copied to the host)."""
        self._draft_extend(bs)
        self.tree.scores[:bs].zero_()  # undrafted depths rank last in the verify selection
        self.tree.begin(bs)
        if 0 in self.tree.delta_slots:
            self.host_deltas[0].copy_(self.tree.deltas[0], non_blocking=True)

    def _phase_step(self, bs: int, s: int) -> None:
        """Draft step ``s``: the depth-``s`` frontier through the draft head; adds depth ``s + 1``."""
        k, tree, draft, dev = self.top_k, self.tree, self.draft, self.device
        w = draft.cfg.sliding_window
        keys = min(w, self.max_len) + self.steps if w else self.max_len + self.steps
        if dev.type == "cuda":  # all the rows' metadata in one launch
            from eagle4_b200.ops import native

            pos, req, slots, start, ctx, extra, n_extra = native._C.draft_step_rows(
                self.L, self.slot, self.tcache.block_table, tree.ancestors, bs, k, s, self.page, w or 0)
        else:
            Lr = self.L[:bs].repeat_interleave(k)
            req = self.slot[:bs].repeat_interleave(k)
            lane = torch.arange(k, device=dev).repeat(bs)
            start = ((Lr - w).clamp(min=0) if w else torch.zeros_like(Lr)).int()
            slots = self._slots(req, Lr + (s - 1) * k + lane)
            tree.set_step_slots(bs, s, slots.view(bs, k))
            extra = tree.ancestors[:bs, :, :s].reshape(bs * k, s).contiguous()
            n_extra = torch.full((bs * k,), s, dtype=torch.int32, device=dev)
            pos, ctx = Lr - 1 + s, Lr.int()
        normed, nh = draft.forward(tree.front_tokens[: bs * k], tree.front_hidden[: bs * k], pos, req,
                                   slots, start, ctx, extra, n_extra, self.dcache, max_keys=keys)
        if self.sampled:
            probs, toks = self._sample(normed, tree.front_nodes[:bs].reshape(-1), k, s, tree.shape.layer_start(s + 1))
        else:
            probs, toks = draft.candidates(normed, k, pos)
        tree.step(bs, s, probs, toks, nh)
        if s in tree.delta_slots:
            self.host_deltas[s].copy_(tree.deltas[s], non_blocking=True)

    def _phase_verify(self, bs: int, n: int) -> None:
        """Verify the root and the best ``n - 1`` drafted nodes, accept, commit; rank this round's tree for the
        next round's verify-width decision."""
        dev = self.device
        tree = self.tree
        if n > 1:
            toks, prow = tree.verify_rows(bs, self.steps, n - 1)
        else:
            toks = None
            prow = torch.full((bs, 1), -1, dtype=torch.int32, device=dev)
        nodes = tree.last_nodes if n > 1 else torch.full((bs, 1), -1, dtype=torch.int64, device=dev)
        tokens, acc, cnt, bonus, aux = self._verify_forward(bs, n, toks, prow, nodes)
        self._record_accept(bs, n, tokens, acc, cnt, bonus, aux)
        if self.policy.cost is not None:
            # cumulative decayed scores of this round's best nodes (root first), batch mean: the next round's
            # lagged verify-width input
            count = self.verify_tokens - 1
            _, cum = tree.rank_reference(bs, self.steps, count)
            self.host_scores[: cum.shape[1]].copy_(cum.mean(dim=0), non_blocking=True)

    def _verify_forward(self, bs: int, n: int, toks: Optional[torch.Tensor], prow: torch.Tensor,
                        nodes: Optional[torch.Tensor] = None, accept=None):
        """The target half of a round: rows [root, toks...] per request (``prow``: parent rows, -1 for the root) through
        the target, accepted (greedy, or the sampled tree walk over ``nodes``; ``accept(hidden, tokens)`` replaces
        this engine's accept, as a host's rejection sampler does), the accepted rows' recurrent states and KV
        committed. Returns (tokens [bs, n], accepted rows [bs, n] (-1 pad), counts [bs] int32, bonus [bs],
        aux hidden [bs * n, A] or None)."""
        dev = self.device
        if dev.type == "cuda":  # the rows' structure in one launch
            from eagle4_b200.ops import native

            tokens, pos, slots, extra, n_extra, parent, req, ctx = native._C.verify_rows_meta(
                prow.contiguous(), toks.contiguous() if n > 1 else self.root[:bs, None], self.root[:bs].contiguous(),
                self.L[:bs].contiguous(), self.slot[:bs].contiguous(), self.tcache.block_table, self.page)
            rb = RowBatch(ids=tokens.reshape(-1), pos=pos, req=req, write_slot=slots.reshape(-1),
                          ctx_start=torch.zeros(bs * n, dtype=torch.int32, device=dev), ctx_len=ctx, extra=extra,
                          n_extra=n_extra, parent=parent, state_slot=req, max_keys=self.max_len)
        else:
            tokens = torch.cat([self.root[:bs, None], toks], dim=1) if n > 1 else self.root[:bs, None].clone()
            L, sl = self.L[:bs], self.slot[:bs]
            rowidx = torch.arange(n, device=dev)
            base = (torch.arange(bs, device=dev) * n)[:, None]
            depth, anc = tree_rows_meta(prow)
            slots = self._slots(sl[:, None], L[:, None] + rowidx[None, :])  # [bs, n] physical slot of row r at L + r
            key = (~anc).long() * n + rowidx[None, None, :]
            order = torch.argsort(key, dim=-1)
            extra = torch.gather(slots[:, None, :].expand(bs, n, n), 2, order).int()
            parent = torch.where(prow >= 0, prow + base, prow)
            rb = RowBatch(ids=tokens.reshape(-1), pos=(L[:, None] + depth).reshape(-1), req=sl.repeat_interleave(n),
                          write_slot=slots.reshape(-1), ctx_start=torch.zeros(bs * n, dtype=torch.int32, device=dev),
                          ctx_len=L.int().repeat_interleave(n), extra=extra.reshape(bs * n, n),
                          n_extra=anc.sum(-1).int().reshape(-1), parent=parent.reshape(-1).int(),
                          state_slot=sl.repeat_interleave(n), max_keys=self.max_len)
        rec = Records()
        out, aux = self.target.forward(rb, self.tcache, rec)
        if accept is not None:
            acc, cnt, bonus = accept(out, tokens)
        elif self.sampled:
            acc, cnt, bonus = self.target.sampled_accept(out, self.temperature, prow, tokens, nodes,
                                                 self.q_store, self.q_ids, self.node_slot, self.top_k, self.seed,
                                                 self.round_ctr, SAMPLED_STREAM)
            ops.advance_round(self.round_ctr)
        else:
            tid, _ = self.target.greedy(out)
            acc, cnt, bonus = ops.accept_greedy(tid.view(bs, n), tokens, prow,
                                                torch.full((bs,), n, dtype=torch.int32, device=dev))
        cnt = cnt.to(torch.int32)
        accc = acc.long().clamp(min=0)
        rowidx = torch.arange(n, device=dev)
        base = (torch.arange(bs, device=dev) * n)[:, None]
        valid = rowidx[None, :] < cnt[:, None]
        rows = torch.where(valid, accc + base, torch.zeros_like(accc)).int()
        src = torch.gather(slots, 1, accc)
        dst = torch.where(valid, slots, src)  # invalid entries copy a slot onto itself (skipped)
        self.target.commit(self.tcache, rec, rows, cnt, self.slot[:bs], src.reshape(-1), dst.reshape(-1))
        return tokens, acc, cnt, bonus, aux

    def _record_accept(self, bs: int, n: int, tokens: torch.Tensor, acc: torch.Tensor, cnt: torch.Tensor,
                       bonus: torch.Tensor, aux: Optional[torch.Tensor]) -> None:
        """The draft side of an accepted round: the emitted tokens (accepted drafted tokens, then the bonus) become
        the round's output and the next extend's pending rows (with the accepted rows' aux hidden states); committed
        lengths advance and the bonus becomes the next root."""
        dev = self.device
        rowidx = torch.arange(n, device=dev)
        base = (torch.arange(bs, device=dev) * n)[:, None]
        accc = acc.long().clamp(min=0)
        cnt = cnt.to(torch.int32)
        path_tok = torch.gather(tokens, 1, accc)
        shifted = torch.cat([path_tok[:, 1:], torch.zeros_like(path_tok[:, :1])], dim=1)
        c1 = (cnt - 1)[:, None]
        emitted = torch.where(rowidx[None, :] < c1, shifted,
                              torch.where(rowidx[None, :] == c1, bonus[:, None], torch.zeros_like(shifted)))
        self.out_tok[:bs, :n] = emitted
        self.out_cnt[:bs] = cnt
        self.ext_tok[:bs, :n] = emitted
        self.ext_cnt[:bs] = cnt
        if aux is not None:
            self.ext_aux[:bs, :n] = aux.index_select(0, (accc + base).reshape(-1)).view(bs, n, -1)
        self.L[:bs] += cnt.long()
        self.root[:bs] = bonus

    def _graph(self, key: tuple, fn, *args) -> None:
        """Run ``fn(*args)``; on a GPU the first call of a key runs eagerly (sizing lazily allocated workspaces)
        and is then captured into a CUDA graph that later calls replay."""
        g = self.graphs.get(key)
        if g is not None:
            if self.device.type == "cuda":
                torch.cuda.nvtx.range_push(f"e4.{key[0]}")
                g.replay()
                torch.cuda.nvtx.range_pop()
            else:
                g.replay()
            _count_launches(self.graph_launches[key])
            return
        fn(*args)
        if self.use_graphs:
            self._captured = True  # this round's period holds an eager run and a capture: not a cost sample
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            before = _launch_count()
            with torch.cuda.graph(g, pool=self.pool):
                fn(*args)  # recorded, not executed
            self.graph_launches[key] = _launch_count() - before
            _count_launches(-self.graph_launches[key])  # recorded launches run at replay
            self.graphs[key] = g

    def _spec_round(self, bs: int, context: int) -> int:
        """One speculative round driven by the round policy (the reference drafter's decision loop,
        ``eagle_harness/sglang/drafter.py:482-691``): the draft half, then the verify. Returns the verify width."""
        policy = self.policy.begin_round(bs)
        timed = self.policy.live is not None
        if timed:
            ev = [_Stamp(self.device) for _ in range(3)]
            ev[0].record()
        width, depth = self._draft_round(bs, context, policy)
        if timed:
            ev[1].record()
        self._graph(("verify", bs, width), self._phase_verify, bs, width)
        if timed:
            ev[2].record()
            self._pending_timing = (bs, width, context, ev, depth)
        return width

    def _draft_round(self, bs: int, context: int, policy) -> tuple:
        """The draft half of a round: extend and depth 1, then steps until a DECIDE depth's work deltas say stop;
        the verify width comes from the previous round's scores. Returns (verify width, last step depth)."""
        self._graph(("begin", bs), self._phase_begin, bs)
        past = policy.history_verify_num(bs)
        # a cost-model tree round fixes its stop rule up front (RoundPlan); chains and the fixed shape ask per depth
        # (the cost row is read before the plan: a DECIDE changes the size tier the row depends on)
        is_cost = isinstance(policy, CostModel)
        row = policy.draft_cost_row(bs, context) if not is_cost or self.round_check is not None else None
        if is_cost and self.round_check is not None:
            self.round_check.begin(policy)
        plan = round_plan(policy, bs, context, self.steps - 1) if is_cost else None
        if is_cost and plan is None:  # chain rounds: the cost model decides per depth
            row = policy.draft_cost_row(bs, context)
        deltas_ready = torch.cuda.Event() if self.device.type == "cuda" else None
        slot = 0
        depth = 0
        while depth < self.steps - 1:
            kind = plan.kind[depth] if plan is not None else PLAN_KIND[policy.width_step(depth)]
            if kind == LAST:
                break
            if kind == LAUNCH:
                if deltas_ready is not None:
                    deltas_ready.record()
                slot = depth
            elif kind == DECIDE:
                if deltas_ready is not None:
                    deltas_ready.synchronize()
                if plan is not None:
                    deltas = self.host_deltas[slot, plan.budget].tolist()
                    stop = plan.stop(depth, deltas)
                    if self.round_check is not None:
                        self.round_check.compare(policy, plan, depth, bs, past, row, deltas)
                else:
                    deltas = self.host_deltas[slot, policy.deltas_budget(past) - 1].tolist()
                    stop = policy.tree_width(depth, bs, past, row, deltas).stop
                if stop:
                    break
            depth += 1
            self._graph(("step", bs, depth), self._phase_step, bs, depth)
        levels = depth + 1
        nodes = self.tree.shape.num_nodes(levels)
        widths = self.policy.widths(bs)
        verify_count = policy.verify_count(bs, nodes + 1)
        if self.lagged_scores is not None:
            req = verify_count
            if not policy.verifies_whole_draft:
                req, _ = policy.verify_num_paged(self.lagged_scores[:verify_count], verify_count, bs, context,
                                                 lagged=True)
                policy.record_verify_num(bs, req)
                req = min(req, verify_count)
            width = fit_width(req, widths, nodes + 1)
        else:
            width = fit_width(verify_count, widths, nodes + 1)
        self.last_depth, self.last_width = levels, width
        return width, depth

    def _chain_round(self, bs: int, width: int) -> int:
        """One chain round of verify width ``width`` (``width - 1`` drafted tokens, one per depth; width 1 verifies
        the root only, after the draft extend)."""
        self._graph(("begin", bs), self._phase_begin, bs)
        for depth in range(1, width - 1):
            self._graph(("step", bs, depth), self._phase_step, bs, depth)
        self._graph(("verify", bs, width), self._phase_verify, bs, width)
        self.last_depth, self.last_width = width - 1, width
        return width

    def _plain(self, bs: int) -> None:
        self._graph(("plain", bs), self._plain_round, bs)

    # ------------------------------------------------------------------ driver
    def bucket(self, bs: int) -> int:
        """The graph batch size a round of ``bs`` requests runs at."""
        for b in self.buckets:
            if b >= bs:
                return b
        raise ValueError(f"batch {bs} exceeds max_reqs {self.max_reqs}")

    def _pad(self, bs: int, rows: int) -> None:
        """Batch rows [bs, rows) as inert padding: the spare cache row, one committed position, token 0."""
        if rows > bs:
            self.slot[bs:rows] = self.pad_slot
            self.L[bs:rows] = 1
            self.root[bs:rows] = 0
            self.ext_tok[bs:rows] = 0
            self.ext_cnt[bs:rows] = 1

    def serve_round(self, bs: int, context: int, *, speculative: bool = True,
                    room: Optional[Sequence[int]] = None):
        """One serving round over batch rows [0, bs) (padded to the round's graph bucket): a speculative tree or
        chain round, or a native decode round when the served choice or the verify batch limit says so; then the
        rows' emitted tokens are read back (one device-to-host copy). ``context``: the batch's mean context length
        (cost-model input). ``room[b]``: at most this many tokens are taken for row b. Returns (tokens taken per
        row, tokens emitted per row)."""
        rows = self.bucket(bs)
        self._pad(bs, rows)
        spec = speculative and self.draft is not None
        over_limit = spec and self.verify_batch_limit is not None and bs > self.verify_batch_limit
        self._pending_timing = None
        self._captured = False
        self._rounds_served += 1
        if self.heartbeat is not None and self._rounds_served % self.heartbeat_every == 0:
            # every rank reaches this round; a peer that crashed or hung is named here, before any collective
            step = self._rounds_served // self.heartbeat_every
            self.heartbeat.beat(step)
            self.heartbeat.check(step, self.heartbeat_timeout)
        chain_t0 = None
        tree_t0 = None
        choice = ServedTreeChoice.SPECULATE
        if spec and self.tree_choice is not None and not over_limit:
            choice = self.tree_choice.choice(rows)
            tree_t0 = _Stamp(self.device)
            tree_t0.record()
        if over_limit:  # above the verify batch limit: native decode (the draft keeps its pending rows)
            choice = ServedTreeChoice.NATIVE
            self._plain(rows)
        elif spec and choice == ServedTreeChoice.NATIVE:
            self._plain(rows)
        elif spec and self.chain_policy is not None:
            chain_w = self.chain_policy.width(rows)
            chain_t0 = _Stamp(self.device)
            chain_t0.record()
            self._chain_round(rows, chain_w)
            chain_t1 = _Stamp(self.device)
            chain_t1.record()
        elif spec:
            self._spec_round(rows, context)
        else:
            self._plain(rows)
        if tree_t0 is not None:
            tree_t1 = _Stamp(self.device)
            tree_t1.record()
        self.host_tok[:bs].copy_(self.out_tok[:bs], non_blocking=True)
        self.host_cnt[:bs].copy_(self.out_cnt[:bs], non_blocking=True)
        if self.device.type == "cuda":
            torch.cuda.current_stream().synchronize()
        if spec and self.policy.cost is not None:
            self.lagged_scores = self.host_scores.tolist()
        if self._pending_timing is not None:
            b_, w_, c_, ev, nsteps = self._pending_timing
            verify_us, draft_us = ev[1].elapsed_us(ev[2]), ev[0].elapsed_us(ev[1])
            if self.target.tp is not None:  # every rank must record the same costs to decide alike
                verify_us, draft_us = self.target.tp.max_over_ranks([verify_us, draft_us])
            self.policy.record(b_, w_, c_, verify_us, nsteps, draft_us, settled=not self._captured)
        taken, counts = [], []
        for b in range(bs):
            c = int(self.host_cnt[b])
            take = c if room is None else min(c, room[b])
            taken.append(self.host_tok[b, :take].tolist())
            counts.append(c)
        got = [len(t) for t in taken]
        if spec:
            self.stats.record(got)
        if self.draft is not None:
            self._track_pending(bs, counts, native=not spec or choice == ServedTreeChoice.NATIVE or over_limit)
        if self.recorder is not None:
            kind = "plain" if not spec else ("native" if choice == ServedTreeChoice.NATIVE else
                                             ("chain" if chain_t0 is not None else "tree"))
            t_us = tree_t0.elapsed_us(tree_t1) if tree_t0 is not None else (
                chain_t0.elapsed_us(chain_t1) if chain_t0 is not None else None)
            self.recorder.record(bs=bs, kind=kind, depth=self.last_depth if spec else 0,
                                 width=self.last_width if spec else 1, tokens=got, round_us=t_us)
        if tree_t0 is not None:
            us = tree_t0.elapsed_us(tree_t1)
            if self.target.tp is not None:
                us = self.target.tp.max_over_ranks([us])[0]
            self.tree_choice.record(rows, choice, us, sum(got) / len(got), settled=not self._captured)
        if chain_t0 is not None:
            us = chain_t0.elapsed_us(chain_t1)
            if self.target.tp is not None:
                us = self.target.tp.max_over_ranks([us])[0]
            self.chain_policy.record(rows, chain_w, us, sum(got) / len(got), settled=not self._captured)
        return taken, counts

    def generate(self, prompts, max_new_tokens: int, *, speculative: bool = True) -> List[List[int]]:
        """Static batch: all prompts prefill, then rounds until every request has ``max_new_tokens`` tokens."""
        prompts = [p if torch.is_tensor(p) else torch.tensor(list(p), dtype=torch.int64) for p in prompts]
        bs = len(prompts)
        if bs > self.max_reqs:
            raise ValueError(f"batch {bs} exceeds max_reqs {self.max_reqs}")
        outs: List[List[int]] = [[] for _ in range(bs)]
        ctx = [int(p.shape[0]) for p in prompts]
        marks = [_Stamp(self.device) for _ in range(3)]  # start, prefill done, rounds done
        marks[0].record()
        self.slot[:bs] = torch.arange(bs, dtype=torch.int32, device=self.device)
        for b, p in enumerate(prompts):
            need = int(p.shape[0]) + max_new_tokens + self.span
            if need > self.max_len:
                raise ValueError(f"request {b}: prompt {int(p.shape[0])} + {max_new_tokens} new tokens + {self.span} "
                                 f"tree rows exceed max_len {self.max_len - self.span}")
            self.prefill(b, p, reserve_tokens=need)
        if self.tree is not None:
            self.lagged_scores = None
        marks[1].record()
        self.host_tok[:bs].copy_(self.out_tok[:bs])
        for b in range(bs):
            outs[b].append(int(self.host_tok[b, 0]))
        while min(len(o) for o in outs) < max_new_tokens:
            taken, counts = self.serve_round(bs, sum(ctx) // bs, speculative=speculative,
                                             room=[max_new_tokens - len(o) for o in outs])
            for b in range(bs):
                outs[b].extend(taken[b])
                ctx[b] += counts[b]
        marks[2].record()
        if self.device.type == "cuda":
            torch.cuda.current_stream().synchronize()
        # device time of this call's prefill (every prompt) and of its decode rounds
        self.last_timing = {"prefill_ms": marks[0].elapsed_us(marks[1]) / 1e3,
                            "decode_ms": marks[1].elapsed_us(marks[2]) / 1e3}
        return [o[:max_new_tokens] for o in outs]
