"""Continuous batching over the engine: requests are admitted between rounds and retire on their own stop condition.

    sched = Scheduler(llm.engine)
    a = sched.submit(prompt_ids, RequestParams(max_new_tokens=64, stop_token_ids=(271,), eos_token_id=2))
    b = sched.submit(other_ids, RequestParams(max_new_tokens=512, ignore_eos=True))
    sched.run()                      # or sched.step() from a serving loop
    a.output, a.finish_reason        # tokens, "length" / "stop" / "eos"

The engine's batch rows [0, bs) hold the running requests; each request keeps its own cache row (KV pages in the page
pool, recurrent state slot) for its whole life. A round emits 1..N tokens per row; the host walks each row's tokens
in order and ends the request at the first token that meets its stop condition (the length limit, one of its stop
tokens, its EOS unless ``ignore_eos``, or a stop string in the detokenised text), so a speculative round that accepts
tokens past a stop never leaks them, and one request's stop set never ends another. A retired request frees its
row: the last running row moves into the hole (its device state is copied; its cache row stays), its pages return to
the pool, and waiting requests are admitted into free rows while the pool has pages for them (prompt, new tokens and
one round's tree rows). Per-request stop handling under batched speculation is what the reference's
``tools/stop_check.py`` checks against live servers; ``eagle4_b200.tools.stop_check`` does the same against this
package's HTTP server (``eagle4_b200.serve``).

Greedy outputs do not depend on the batch: every target op computes a row independently of the other rows of its
launch, so a request produces the same tokens whether it runs alone, in a static batch, or joins and leaves a
continuously changing one.
"""

from __future__ import annotations

import itertools
from collections import deque
from dataclasses import dataclass, field
from typing import Callable, Deque, List, Optional, Sequence

import torch

from eagle4_b200.runtime.pages import OutOfPages


@dataclass(frozen=True)
class RequestParams:
    """Per-request generation limits and stop conditions."""

    max_new_tokens: int = 128
    stop_token_ids: Sequence[int] = ()
    eos_token_id: Optional[int] = None
    ignore_eos: bool = False
    stop: Sequence[str] = ()  # stop strings (need the scheduler's detokenizer); kept in the output

    def __post_init__(self):
        if self.max_new_tokens < 1:
            raise ValueError(f"max_new_tokens must be positive, got {self.max_new_tokens}")


@dataclass
class Request:
    rid: int
    prompt: torch.Tensor
    params: RequestParams
    output: List[int] = field(default_factory=list)
    finish_reason: Optional[str] = None  # "length", "stop" (stop token or string), "eos"
    slot: int = -1  # engine cache row while running
    rounds: int = 0

    @property
    def finished(self) -> bool:
        return self.finish_reason is not None


class Scheduler:
    def __init__(self, engine, *, speculative: bool = True, detokenize: Optional[Callable[[List[int]], str]] = None,
                 batch_prefill: bool = False, prefill_tokens: int = 8192):
        """``detokenize``: token ids -> text, needed only for requests with stop strings. ``batch_prefill``: the
        requests admitted in one step prefill together, in groups of up to ``prefill_tokens`` prompt tokens (one
        target forward per group instead of one per request; the results are each request's alone)."""
        self.engine = engine
        self.batch_prefill, self.prefill_tokens = batch_prefill, prefill_tokens
        self.speculative = speculative
        self.detokenize = detokenize
        self.waiting: Deque[Request] = deque()
        self.running: List[Request] = []  # index = engine batch row
        self.free_slots: List[int] = list(range(engine.max_reqs - 1, -1, -1))
        for slot in self.free_slots:  # the scheduler owns the engine: pages a static generate left mapped return
            engine.pages.release(slot)
        self._ids = itertools.count()
        self.ctx: List[int] = []  # context length per running row

    # ------------------------------------------------------------------ admission
    def submit(self, prompt, params: RequestParams = RequestParams()) -> Request:
        prompt = prompt if torch.is_tensor(prompt) else torch.tensor(list(prompt), dtype=torch.int64)
        if prompt.dim() != 1 or prompt.numel() == 0:
            raise ValueError("a prompt is a non-empty 1-D sequence of token ids")
        if params.stop and self.detokenize is None:
            raise ValueError("stop strings need a scheduler with a detokenizer")
        need = self._need(prompt, params)
        if need > self.engine.max_len:
            raise ValueError(f"prompt {prompt.numel()} + {params.max_new_tokens} new tokens + {self.engine.span} tree "
                             f"rows exceed max_len {self.engine.max_len - self.engine.span}")
        req = Request(next(self._ids), prompt, params)
        self.waiting.append(req)
        return req

    def _started(self, req: Request, b: int, done: List[Request]) -> None:
        """A prefilled request joins the running batch at row ``b`` with its first token."""
        self.running.append(req)
        self.ctx.append(int(req.prompt.numel()))
        if self._take(req, [int(self.engine.out_tok[b, 0])]):
            done.append(req)

    def _prefill_group(self, group: List[tuple], done: List[Request]) -> None:
        self.engine.prefill_many([b for b, _, _ in group], [r.prompt for _, r, _ in group],
                                 [need for _, _, need in group])
        for b, req, _ in group:
            self._started(req, b, done)

    def _need(self, prompt: torch.Tensor, params: RequestParams) -> int:
        return int(prompt.numel()) + params.max_new_tokens + self.engine.span

    def _admit(self) -> List[Request]:
        """Prefill waiting requests into free rows while rows and pages last (first come, first served)."""
        eng = self.engine
        done = []
        fresh = not self.running
        group: List[tuple] = []  # (row, request, need) admitted and waiting for a batched prefill
        planned = 0  # pages the group will take
        while self.waiting and self.free_slots:
            req = self.waiting[0]
            need = self._need(req.prompt, req.params)
            if eng.pages.pages_for(need) > eng.pages.free_pages - planned:
                if not self.running and not group:
                    raise OutOfPages(f"request {req.rid} needs {eng.pages.pages_for(need)} pages; the pool has "
                                     f"{eng.pages.free_pages} with nothing running")
                break
            self.waiting.popleft()
            b = len(self.running) + len(group)
            req.slot = self.free_slots.pop()
            eng.slot[b] = req.slot
            if not self.batch_prefill:
                eng.prefill(b, req.prompt, reserve_tokens=need)
                self._started(req, b, done)
                continue
            if group and sum(int(r.prompt.numel()) for _, r, _ in group) + int(req.prompt.numel()) > \
                    self.prefill_tokens:
                self._prefill_group(group, done)
                group, planned = [], 0
                b = len(self.running)
                eng.slot[b] = req.slot
            group.append((b, req, need))
            planned += eng.pages.pages_for(need)
        if group:
            self._prefill_group(group, done)
        if done:
            self._retire(done)
        if fresh and eng.tree is not None:
            eng.lagged_scores = None  # a new batch: no previous round's ranking to lag
        return done

    # ------------------------------------------------------------------ stop conditions
    def _take(self, req: Request, tokens: List[int]) -> bool:
        """Append ``tokens`` up to the first that ends ``req``; True if it ended."""
        p = req.params
        stops = set(p.stop_token_ids)
        for t in tokens:
            req.output.append(t)
            if t in stops:
                req.finish_reason = "stop"
            elif p.eos_token_id is not None and t == p.eos_token_id and not p.ignore_eos:
                req.finish_reason = "eos"
            elif p.stop and any(s in self.detokenize(req.output) for s in p.stop):
                req.finish_reason = "stop"
            elif len(req.output) >= p.max_new_tokens:
                req.finish_reason = "length"
            if req.finished:
                return True
        return False

    # ------------------------------------------------------------------ retirement
    def _retire(self, done: Sequence[Request]) -> None:
        """Remove finished requests from the batch: the last running row moves into each hole."""
        eng = self.engine
        for req in done:
            b = self.running.index(req)
            last = len(self.running) - 1
            if b != last:
                self._move_row(last, b)
                self.running[b] = self.running[last]
                self.ctx[b] = self.ctx[last]
            self.running.pop()
            self.ctx.pop()
            eng.pages.release(req.slot)
            self.free_slots.append(req.slot)
            req.slot = -1

    def _move_row(self, src: int, dst: int) -> None:
        """Batch row ``src``'s per-request device state into row ``dst`` (the request keeps its cache row)."""
        eng = self.engine
        for t in (eng.L, eng.root, eng.slot, eng.ext_tok, eng.ext_cnt, eng.ext_aux):
            t[dst] = t[src]
        eng.pending_host[dst] = eng.pending_host[src]

    # ------------------------------------------------------------------ rounds
    def step(self) -> List[Request]:
        """Admit what fits, run one round over the running requests, retire the ones that ended. Returns the
        requests that finished during this step."""
        finished = self._admit()
        if not self.running:
            return finished
        bs = len(self.running)
        room = [r.params.max_new_tokens - len(r.output) for r in self.running]
        taken, counts = self.engine.serve_round(bs, sum(self.ctx) // bs, speculative=self.speculative, room=room)
        done = []
        for b, req in enumerate(self.running):
            req.rounds += 1
            self.ctx[b] += counts[b]
            if self._take(req, taken[b]):
                done.append(req)
        self._retire(done)
        return finished + done

    @property
    def idle(self) -> bool:
        return not self.waiting and not self.running

    def run(self) -> List[Request]:
        """Step until every submitted request has finished; returns them in finishing order."""
        out: List[Request] = []
        while not self.idle:
            out.extend(self.step())
        return out
