"""Calibration driver of this package's engine: times target verify forwards and draft steps, then fits cost tables.

The engine exposes whole forwards, not attention-only timers, so the driver records whole-step timings per
(batch size, query length, context length) and lets :func:`eagle4_b200.core.calibration.fit_step_timings` split
them into attention and non-attention costs (the reference's path for engines that time whole steps,
``eagle_harness/core/calibration.py:540-624``). Each timed shape is one CUDA graph whose context length lives in a
device tensor, so a context sweep replays the same graph after an in-place update, and the time is the median of
``repeats`` replays (CUDA events around each replay).

Target rows of one request form a chain of ``q`` tokens after ``ctx`` committed tokens (the verify layout of a
chain; tree layouts of the same width cost the same: the row count, the keys each row reads and the recurrent path
lengths are what the kernels pay for). Draft rows are ``q`` siblings per request at the same depth. Nothing is
committed: KV rows are written at positions past the context, recurrent states are only read.
"""

from __future__ import annotations

import logging
import os
import statistics
from typing import Callable, Dict, List, Optional, Sequence, Tuple

import torch

from eagle4_b200.core.calibration import (AttentionShape, CalibrationPaths, MeasureParams, StepTiming,
                                          fit_step_timings, query_lens)
from eagle4_b200.core.cost_table import cost_model_problem, load_cost_tables
from eagle4_b200.core.limits import ComputeIntensity
from eagle4_b200.core.live_costs import CostKey, write_key
from eagle4_b200.models.target import RowBatch

log = logging.getLogger(__name__)


class _Shape:
    """Static inputs and (on a GPU) a captured graph of one timed forward; ``ctx`` is updated in place."""

    def __init__(self, build: Callable[[], None], ctx: torch.Tensor, use_graph: bool):
        self.ctx, self.build = ctx, build
        self.graph = None
        build()  # eager run sizes lazily allocated workspaces
        if use_graph:
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                build()
            self.graph = g

    def run(self) -> None:
        if self.graph is not None:
            self.graph.replay()
        else:
            self.build()


def _gen(dev, bs: int, q: int) -> torch.Generator:
    """The timed rows' random inputs: the same on every tensor-parallel rank."""
    return torch.Generator(device=dev).manual_seed(1009 * bs + q)


class ForwardTimer:
    """Times target and draft forwards of an :class:`~eagle4_b200.runtime.engine.Engine` at any (bs, q, ctx)."""

    def __init__(self, engine, repeats: int = 10):
        self.eng = engine
        self.repeats = repeats
        for row in range(engine.max_reqs):  # timed contexts read real pages, not the trash page
            engine.pages.reserve(row, engine.max_len)
        self.shapes: Dict[tuple, _Shape] = {}
        self.cuda = engine.device.type == "cuda"

    # ------------------------------------------------------------------ layouts
    def _target(self, bs: int, q: int) -> _Shape:
        eng, dev = self.eng, self.eng.device
        n = bs * q
        req = eng.slot[:bs].repeat_interleave(q)
        ctx = torch.zeros(bs, dtype=torch.int64, device=dev)
        r = torch.arange(q, device=dev)
        ids = torch.randint(0, eng.target.cfg.vocab_size, (n,), device=dev, generator=_gen(dev, bs, q))
        tri = (r[None, :] <= r[:, None])  # [q, q] row i sees rows 0..i
        parent = (torch.arange(n, device=dev) - 1).int()
        parent[::q] = -1

        def build():
            pos = (ctx[:, None] + r[None, :]).reshape(-1)
            slots = eng._slots(req, pos)
            sl = slots.view(bs, q)
            extra = torch.where(tri[None], sl[:, None, :], sl[:, :, None]).reshape(n, q).int()
            rb = RowBatch(ids=ids, pos=pos, req=req, write_slot=slots,
                          ctx_start=torch.zeros(n, dtype=torch.int32, device=dev),
                          ctx_len=ctx.int().repeat_interleave(q), extra=extra,
                          n_extra=(r + 1).int().repeat(bs), parent=parent, state_slot=req, max_keys=eng.max_len)
            out, _ = eng.target.forward(rb, eng.tcache)
            eng.target.greedy(out)

        return _Shape(build, ctx, self.cuda)

    def _draft(self, bs: int, q: int) -> _Shape:
        eng, dev = self.eng, self.eng.device
        draft = eng.draft
        n = bs * q
        req = eng.slot[:bs].repeat_interleave(q)
        ctx = torch.zeros(bs, dtype=torch.int64, device=dev)
        lane = torch.arange(q, device=dev).repeat(bs)
        g = _gen(dev, bs, q)
        ids = torch.randint(0, eng.target.cfg.vocab_size, (n,), device=dev, generator=g)
        hidden = (torch.randn(n, draft.cfg.hidden_size, device=dev, generator=g) * 0.5).to(eng.dtype)
        w = draft.cfg.sliding_window
        k = max(q, eng.top_k)

        def build():
            Lr = ctx.repeat_interleave(q)
            slots = eng._slots(req, Lr + lane)
            start = ((Lr - w).clamp(min=0) if w else torch.zeros_like(Lr)).int()
            extra = slots.view(n, 1).int()
            normed, _ = draft.forward(ids, hidden, Lr, req, slots, start, Lr.int(), extra,
                                      torch.ones(n, dtype=torch.int32, device=dev), eng.dcache,
                                      max_keys=(min(w, eng.max_len) if w else eng.max_len) + 1)
            draft.candidates(normed, k, Lr)

        return _Shape(build, ctx, self.cuda)

    # ------------------------------------------------------------------ timing
    def time_us(self, model: str, bs: int, q: int, ctx: int) -> float:
        key = (model, bs, q)
        shape = self.shapes.get(key)
        if shape is None:
            shape = self.shapes[key] = (self._target if model == "llm" else self._draft)(bs, q)
        shape.ctx.fill_(ctx)
        shape.run()  # warm
        samples = []
        for _ in range(self.repeats):
            if self.cuda:
                s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s.record()
                shape.run()
                e.record()
                e.synchronize()
                samples.append(s.elapsed_time(e) * 1e3)
            else:
                import time
                t0 = time.perf_counter()
                shape.run()
                samples.append((time.perf_counter() - t0) * 1e6)
        med = statistics.median(samples)
        tp = self.eng.target.tp
        # tensor parallel: a step takes as long as its slowest rank, and every rank must fit the same tables
        return tp.max_over_ranks([med])[0] if tp is not None and tp.world > 1 else med


def engine_attention_shapes(engine) -> Tuple[AttentionShape, AttentionShape]:
    """(draft, target) attention layer counts of the engine's models."""
    dcfg = engine.draft.cfg
    draft = AttentionShape(1, 1 if dcfg.sliding_window else 0, dcfg.sliding_window or 0)
    target = AttentionShape(max(1, len(engine.target.cfg.layer_ids("attn"))))
    return draft, target


def calibrate(engine, data_path: str, *, batch_sizes: Sequence[int], context_step: int = 256,
              context_stop: int = 4096, intensity: ComputeIntensity = ComputeIntensity.HIGH, repeats: int = 10,
              key: Optional[CostKey] = None, progress: Callable[[str], None] = print) -> Dict[int, Optional[str]]:
    """Measure and fit every batch size into ``data_path``; returns ``{batch size: problem or None}`` from the cost
    model's table checks. Under tensor parallelism every rank runs the same timed forwards (each time is the maximum
    over the ranks), rank 0 alone writes the files (fitted with the TP size) and every rank returns its checks."""
    if engine.draft is None:
        raise ValueError("calibration needs a draft model")
    if max(batch_sizes) > engine.max_reqs:
        raise ValueError(f"batch sizes up to {max(batch_sizes)} need an engine with max_reqs >= that")
    if context_stop + 2 * engine.verify_tokens > engine.max_len:
        raise ValueError(f"context_stop {context_stop} does not fit the engine's max_len {engine.max_len}")
    paths = CalibrationPaths(data_path)
    world, writer = _tp_role(engine)
    if not writer:
        progress = _quiet
    timer = ForwardTimer(engine, repeats)
    draft_shape, target_shape = engine_attention_shapes(engine)
    contexts = list(range(context_step, context_stop + 1, context_step))
    for bs in batch_sizes:
        params = MeasureParams(context_step=context_step, context_stop=context_stop, batch_size=bs,
                               verify_num=engine.verify_tokens, node_top_k=engine.top_k,
                               loop_top_m=engine.verify_tokens, repeat_cnt=repeats)
        timings = {}
        for model, max_q in (("slm", params.node_top_k), ("llm", params.verify_num)):
            qs = query_lens(f"x_{model}", bs, intensity, max_q)
            timings[model] = [StepTiming(q, c, timer.time_us(model, bs, q, c)) for q in qs for c in contexts]
            progress(f"bs {bs} {model}: " + ", ".join(
                f"q{q}={statistics.median(t.time_us for t in timings[model] if t.query_length == q):.0f}us"
                for q in qs))
        if writer:
            fit_step_timings(paths, params, intensity, (draft_shape, timings["slm"]), (target_shape, timings["llm"]),
                             tp_size=world)
    if key is not None and writer:
        write_key(data_path, key)
    _files_written(engine)
    tables = load_cost_tables(paths.cost)
    return {bs: cost_model_problem(t, target_is_moe=engine.target.cfg.is_moe) for bs, t in tables.items()}


def calibrate_chain(engine, data_path: str, *, batch_sizes: Sequence[int], prompt_len: int = 256,
                    new_tokens: int = 128, widths: Optional[Sequence[int]] = None, seed: int = 0,
                    key: Optional[CostKey] = None, progress: Callable[[str], None] = print) -> str:
    """Served-chain calibration (the reference's SGLang calibration driver): serve generation at every chain width
    and batch size, store the median round period per (batch size, width) as ``rounds/chain.json`` and the
    acceptance by draft position, measured at the widest chain, as ``accept/chain.json``; returns ``data_path``.

    ``engine`` must be a chain engine (top-k 1); width 1 is root-only verification."""
    from eagle4_b200.core.chain_width import save_accept_profile, save_round_times

    _, writer = _tp_role(engine)
    if not writer:
        progress = _quiet
    if engine.draft is None or engine.top_k != 1:
        raise ValueError("chain calibration needs a draft and a top-k 1 (chain) engine")
    widths = sorted(widths or range(1, engine.verify_tokens + 1))
    gen = torch.Generator().manual_seed(seed)
    rows, drafts, accepted = [], 0, [0] * (max(widths) - 1)
    saved_policy = engine.chain_policy
    try:
        for bs in batch_sizes:
            prompts = torch.randint(0, engine.target.cfg.vocab_size, (bs, prompt_len), generator=gen)
            for w in widths:
                engine.chain_policy = _FixedChain(w)
                engine.generate(prompts, new_tokens)
                us = sorted(engine.chain_policy.round_us)
                if not us:
                    continue
                rows.append({"batch_size": bs, "width": w, "round_us": us[len(us) // 2], "count": len(us)})
                if w == max(widths):
                    for got in engine.chain_policy.emitted:
                        drafts += 1
                        for d in range(min(got - 1, len(accepted))):
                            accepted[d] += 1
                progress(f"bs {bs} width {w}: {rows[-1]['round_us']:.0f} us per round")
    finally:
        engine.chain_policy = saved_policy
    if writer:  # round periods are already the maximum over the ranks (the engine reduces them before recording)
        save_round_times(data_path, rows)
        if drafts:
            save_accept_profile(data_path, drafts, accepted)
        if key is not None:
            write_key(data_path, key)
    _files_written(engine)
    return data_path


def _tp_role(engine) -> Tuple[int, bool]:
    """(tensor-parallel world size, whether this rank writes the calibration files)."""
    tp = engine.target.tp
    return (tp.world, tp.rank == 0) if tp is not None else (1, True)


def _files_written(engine) -> None:
    """Every rank waits until rank 0's files are on disk."""
    tp = engine.target.tp
    if tp is not None and tp.world > 1:
        import torch.distributed as dist

        dist.barrier(group=tp.group)


def _quiet(msg: str) -> None:
    pass


class _FixedChain:
    """A chain policy that serves one width and keeps every round's period and per-request tokens."""

    def __init__(self, width: int):
        self.w = width
        self.round_us: List[float] = []
        self.emitted: List[int] = []

    def width(self, bs: int) -> int:
        return self.w

    def record(self, bs: int, width: int, round_us: float, tokens_per_request: float, settled: bool = True) -> None:
        if not settled:  # an eager run and a graph capture sit inside this period
            return
        self.round_us.append(round_us)
        self.emitted.append(int(round(tokens_per_request)))
