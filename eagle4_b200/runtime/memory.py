"""Device memory of a serving configuration, per GPU, before anything is allocated.

The plan builds the same tensors the engine builds, on PyTorch's ``meta`` device (shapes, no storage): the target and
draft weights as this rank keeps them under tensor parallelism (shared tensors counted once), the target's paged KV
cache and recurrent states, the draft's KV cache. Everything scales with the KV token budget except the weights and
the per-request states, so the plan also answers the largest ``kv_tokens`` that fits a memory budget (the server's
``--kv-tokens``). ``prefill`` estimates the largest transient of a prefill: one piece of ``prefill_chunk`` rows
through the widest projection plus a few hidden-size buffers, and the aux hidden states of a whole ``max_len``
prompt kept for the draft. ``reserve_gb`` stands for what the plan does not count: decode activations, CUDA graph
pools, the tensor-parallel buffers, the CUDA context (a few GB at the flagship shapes; measure with
``torch.cuda.mem_get_info`` on the target GPU for a tighter figure).
"""

from __future__ import annotations

from dataclasses import asdict, dataclass
from typing import Dict, Optional

import torch

GB = 1e9
B200_GB = 183359 * 2 ** 20 / GB  # nvidia-smi's 183,359 MiB


@dataclass
class MemoryPlan:
    weights: int             # bytes of this rank's target and draft weights
    kv_bytes_per_token: int  # target attention K/V plus draft K/V per token position
    state_bytes: int         # recurrent states (conv windows, SSM states) of every cache row
    kv_tokens: int
    reserve: int
    prefill: int = 0         # bytes of the largest prefill transient (one piece's activations, the prompt's aux rows)

    @property
    def kv(self) -> int:
        return self.kv_bytes_per_token * self.kv_tokens

    @property
    def total(self) -> int:
        return self.weights + self.kv + self.state_bytes + self.reserve + self.prefill

    def kv_tokens_within(self, budget_bytes: float) -> int:
        """The largest KV token budget (a multiple of 1024) whose plan fits ``budget_bytes``."""
        free = budget_bytes - self.weights - self.state_bytes - self.reserve - self.prefill
        return max(0, int(free // self.kv_bytes_per_token) // 1024 * 1024)

    def summary(self, budget_gb: Optional[float] = None) -> Dict[str, float]:
        out = {k: round(v / GB, 3) for k, v in asdict(self).items() if k not in ("kv_bytes_per_token", "kv_tokens")}
        out.update(kv_tokens=self.kv_tokens, kv_bytes_per_token=self.kv_bytes_per_token, kv=round(self.kv / GB, 3),
                   total=round(self.total / GB, 3))
        if budget_gb is not None:
            out.update(budget=budget_gb, fits=self.total <= budget_gb * GB,
                       max_kv_tokens=self.kv_tokens_within(budget_gb * GB))
        return out


def _bytes(tensors) -> int:
    seen, n = set(), 0
    for t in tensors:
        if id(t) not in seen and torch.is_tensor(t):
            seen.add(id(t))
            n += t.numel() * t.element_size()
    return n


def plan(target_cfg, draft_cfg=None, *, tp: int = 1, max_batch: int = 1, max_len: int = 4096, page: int = 16,
         tree=(12, 4, 16), kv_tokens: Optional[int] = None, dtype=torch.bfloat16, reserve_gb: float = 4.0,
         prefill_chunk: int = 8192) -> MemoryPlan:
    """The memory of rank 0 of a ``tp``-way engine (ranks differ at most by a vocabulary shard's rounding)."""
    from eagle4_b200.models import weights
    from eagle4_b200.models.draft import DraftCache
    from eagle4_b200.models.target import TargetCache
    from eagle4_b200.parallel.sharding import shard_draft, shard_target

    meta = torch.device("meta")
    tw = weights.init_target(target_cfg, device=meta, dtype=dtype)
    dw = weights.init_draft(draft_cfg, device=meta, dtype=dtype, embed=tw["embed"], lm_head=tw["lm_head"]) \
        if draft_cfg is not None else {}
    ltc, ltw = shard_target(target_cfg, tw, tp, 0)
    ldc, ldw = shard_draft(draft_cfg, dw, tp, 0) if draft_cfg is not None else (None, {})
    w_bytes = _bytes(list(ltw.values()) + list(ldw.values()))
    steps, top_k, verify = tree
    span = max(verify, steps * top_k) + 1  # the engine's room for one round's rows past a request's length
    row_len = max_len + span
    tokens = kv_tokens if kv_tokens is not None else max_batch * (-(-row_len // page)) * page
    one = TargetCache.allocate(ltc, max_reqs=max_batch + 1, max_len=row_len, page=page, device=meta, dtype=dtype,
                               kv_pages=1)
    kv_page = _bytes(one.k + one.v)
    state = _bytes(one.conv + one.ssm)
    if ldc is not None:
        kv_page += _bytes([DraftCache.allocate(ldc, one.block_table, page, meta, dtype, pages=1).k]) * 2
    esize = torch.empty(0, dtype=dtype).element_size()
    widest = max((t.shape[0] for name, t in ltw.items() if t.dim() == 2 and name not in ("embed", "lm_head")),
                 default=0)
    hidden = target_cfg.hidden_size
    aux = len(draft_cfg.aux_layer_ids) * hidden if draft_cfg is not None else 0
    prefill = (min(prefill_chunk, max_len) * (widest + 4 * hidden) + max_len * aux) * esize
    return MemoryPlan(weights=w_bytes, kv_bytes_per_token=kv_page // page, state_bytes=state,
                      kv_tokens=int(tokens), reserve=int(reserve_gb * GB), prefill=int(prefill))
