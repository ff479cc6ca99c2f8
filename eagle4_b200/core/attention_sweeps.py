"""Attention cost vs context length on the GPU (calibration step 1), timing this package's tree-attention kernel.

:func:`sweep` times every (query length, context length) of a :class:`~eagle4_b200.core.calibration.CacheSweepPlan`
through a :class:`Timer` and writes the ``cache_qo_len_<q>.jsonl`` records the cache fit reads (reference
``eagle_harness/core/attention_sweeps.py:28-140``, whose timer drives FlashInfer's paged prefill; here the timed
kernel is the one the verify forward runs: paged tree attention with each query row's ancestor chain as extras).
"""

from __future__ import annotations

import logging
import os
from dataclasses import dataclass
from typing import List, Protocol, Sequence

import torch

from eagle4_b200.core.calibration import CacheSweepPlan, MeasureRecord, save_jsonl

log = logging.getLogger(__name__)


@dataclass(frozen=True)
class HeadLayout:
    """Attention heads of one tensor-parallel rank."""

    num_qo_heads: int
    num_kv_heads: int
    head_dim: int

    @classmethod
    def for_rank(cls, num_qo_heads_total: int, num_kv_heads_total: int, head_dim: int, tp_size: int, *,
                 replicate_kv: bool = True) -> "HeadLayout":
        """With ``replicate_kv``, KV heads fewer than the ranks are replicated (one per rank)."""
        if num_qo_heads_total % tp_size:
            raise ValueError("the query heads do not split evenly over tp_size ranks")
        kv_total = num_kv_heads_total
        if replicate_kv:
            if kv_total % tp_size and tp_size % kv_total:
                raise ValueError("neither the KV heads nor tp_size divides the other")
        elif kv_total % tp_size:
            raise ValueError("the KV heads do not split evenly over tp_size ranks")
        return cls(num_qo_heads_total // tp_size, max(1, kv_total // tp_size), head_dim)


class Timer(Protocol):
    def time_us(self, batch_size: int, qo_len: int, kv_len: int, num_layers: int) -> int:
        """The time in microseconds of ``num_layers`` attention launches of this shape."""


def time_calls(fn, calls: int) -> int:
    """Microseconds of ``calls`` back-to-back calls of ``fn`` (CUDA events, synchronised on both sides)."""
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    start.record()
    for _ in range(calls):
        fn()
    end.record()
    torch.cuda.synchronize()
    return int(start.elapsed_time(end) * 1000)


class TreeAttentionTimer:
    """Times ``eagle4_b200.ops.attention`` on a paged cache: every request has ``kv_len - qo_len`` committed tokens
    and ``qo_len`` verify rows forming a chain (row ``i`` sees the committed context and rows ``0..i``)."""

    def __init__(self, heads: HeadLayout, device: str = "cuda", page: int = 64, dtype=torch.bfloat16):
        self.heads, self.device, self.page, self.dtype = heads, device, page, dtype

    def inputs(self, batch_size: int, qo_len: int, kv_len: int):
        h, dev, page = self.heads, self.device, self.page
        pages = (kv_len + page - 1) // page
        slots = batch_size * pages * page
        k = torch.randn(slots, h.num_kv_heads, h.head_dim, device=dev).to(self.dtype)
        v = torch.randn_like(k)
        table = torch.arange(batch_size * pages, device=dev, dtype=torch.int32).view(batch_size, pages)
        t = batch_size * qo_len
        req = torch.arange(batch_size, device=dev, dtype=torch.int32).repeat_interleave(qo_len)
        ctx = max(kv_len - qo_len, 0)
        ctx_start = torch.zeros(t, dtype=torch.int32, device=dev)
        ctx_len = torch.full((t,), ctx, dtype=torch.int32, device=dev)
        i = torch.arange(qo_len, device=dev)
        base = (req.long() * pages * page + ctx).view(batch_size, qo_len)  # tree rows sit after the context
        extra = torch.where(i[None, :] <= i[:, None], i[None, :], 0)  # [q, q]: row i -> positions 0..i
        extra = (base[:, :, None] + extra[None]).view(t, qo_len).to(torch.int32)
        n_extra = (i + 1).repeat(batch_size).to(torch.int32)
        q = torch.randn(t, h.num_qo_heads, h.head_dim, device=dev).to(self.dtype)
        return q, k, v, table, req, ctx_start, ctx_len, extra, n_extra

    def time_us(self, batch_size: int, qo_len: int, kv_len: int, num_layers: int) -> int:
        from eagle4_b200 import ops

        q, k, v, table, req, s0, s1, extra, ne = self.inputs(batch_size, qo_len, kv_len)
        scale = self.heads.head_dim ** -0.5
        run = lambda: ops.attention(q, k, v, table, self.page, req, s0, s1, extra, ne, scale, max_keys=kv_len)
        run()  # warm-up
        return time_calls(run, num_layers)


def sweep(timer: Timer, *, category: str, batch_size: int, qo_lens: Sequence[int], plan: CacheSweepPlan,
          save_dir: str, device: str = "cuda") -> List[str]:
    """Time every (qo_len, kv_len) of ``plan``; lengths below ``plan.kv_step`` are warm-up and not recorded."""
    written = []
    for q in qo_lens:
        records = []
        for kv in plan.cache_lengths():
            kv = max(kv, 1)
            us = timer.time_us(batch_size, q, kv, plan.num_layers)
            if kv >= plan.kv_step:
                records.append(MeasureRecord(us, plan.num_layers, q, kv, category, batch_size))
            _warn_if_low(device)
        if not records:
            raise RuntimeError(f"query length {q}: every timing of the sweep was invalid")
        path = os.path.join(save_dir, f"cache_qo_len_{q}.jsonl")
        save_jsonl(path, records)
        written.append(path)
    return written


def _warn_if_low(device: str) -> None:
    if not torch.cuda.is_available():
        return
    free, total = torch.cuda.mem_get_info(device)
    if free < 0.05 * total:
        log.warning("the attention sweep runs short of device memory; its timings may read slow")
        torch.cuda.empty_cache()
