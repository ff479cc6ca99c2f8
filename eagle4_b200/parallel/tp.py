"""Tensor parallelism: one rank per GPU, ``torch.distributed`` for setup, and two data paths for the collectives.

``backend="fused"`` (the B200 path): a row-parallel linear is ONE GEMM launch whose epilogue stores each finished
fp32 tile straight into this rank's slot of every rank's receive buffer over NVLink (peer pointers from CUDA IPC)
as (value, call tag) pairs; a second kernel sums each element over the ranks in rank order as soon as its pairs
carry this call's tag, adds the residual and applies the next RMSNorm. The greedy head's vocabulary-parallel (max, argmax) is
exchanged the same way by one small kernel. Both kernels are captured in the engine's CUDA graphs.

``backend="torch"``: the same math through ``torch.distributed.all_reduce`` / ``all_gather`` (NCCL on GPUs, gloo on
CPU): the baseline the fused path is measured against, and the CPU oracle of the multi-process tests.

Every rank sums partials in rank order and applies identical elementwise math, so all ranks hold bit-identical
hidden states, greedy tokens and draft trees, and take the same host decisions without exchanging them.
"""

from __future__ import annotations

import os
from typing import List, Optional, Tuple

import torch
import torch.distributed as dist

from eagle4_b200 import ops

MAX_RANKS = 8
_CH0, _CH1 = 0, 256  # channel words: GEMM -> reduce, greedy-head exchange
_RECV = 4096


class TensorParallel:
    def __init__(self, group=None, *, backend: str = "fused", max_rows: int = 1024, max_cols: int = 8192,
                 device: Optional[torch.device] = None):
        if backend not in ("fused", "torch"):
            raise ValueError(f"unknown tensor-parallel backend {backend!r}")
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if self.world > MAX_RANKS:
            raise ValueError(f"at most {MAX_RANKS} tensor-parallel ranks")
        self.device = device or (torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available()
                                 else torch.device("cpu"))
        self.backend = backend if self.device.type == "cuda" else "torch"
        self.max_rows, self.max_cols = max_rows, max_cols
        self.base = 0
        self.peers: List[int] = []
        # one rank may still run the fused kernels (signalling only itself): measures their cost without NVLink
        self.force_fused = self.world == 1 and os.environ.get("E4_TP_FORCE_FUSED") == "1"
        if self.backend == "fused" and (self.world > 1 or self.force_fused):
            self._open()

    # ------------------------------------------------------------------ symmetric buffer
    def _open(self) -> None:
        from eagle4_b200.ops import native

        C = native._C
        dev = self.device.index
        self.slot = self.max_rows * self.max_cols  # (value, tag) pairs of 8 bytes
        recv_bytes = 2 * self.world * self.slot * 8
        self.xbuf_off = _RECV + recv_bytes
        total = self.xbuf_off + 2 * MAX_RANKS * self.max_rows * 16
        self.base = C.sym_alloc(total, dev)
        handle = C.sym_handle(self.base)
        handles: List[Optional[torch.Tensor]] = [None] * self.world
        dist.all_gather_object(handles, handle, group=self.group)
        self.peers = [self.base if r == self.rank else C.sym_open(handles[r], dev) for r in range(self.world)]
        self.err = native.error_word(self.device)
        dist.barrier(group=self.group)

    def close(self) -> None:
        """Unmap the peers' buffers and free this rank's (after a barrier: no peer may still write into it)."""
        if not self.base:
            return
        from eagle4_b200.ops import native

        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        for r, p in enumerate(self.peers):
            if r != self.rank:
                native._C.sym_close(p)
        native._C.sym_free(self.base)
        self.base = 0

    # ------------------------------------------------------------------ ops
    def row_linear(self, x: torch.Tensor, w: torch.Tensor, residual: torch.Tensor,
                   norm_w: Optional[torch.Tensor] = None, eps: float = 1e-6, offset: bool = False
                   ) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
        """``h = residual + all_reduce(x @ w^T)``; ``x_next = rmsnorm(h, norm_w)`` when a norm weight is given."""
        if self.world == 1 and not self.force_fused:
            h = ops.linear_residual(x, w, residual)
            return h, (ops.rmsnorm(h, norm_w, eps, offset) if norm_w is not None else None)
        if self.backend == "torch":
            # the NCCL baseline: a bf16 partial and a bf16 all-reduce (what an engine's all-reduce moves)
            part = ops.linear(x, w)
            dist.all_reduce(part, group=self.group)
            h = (residual.float() + part.float()).to(residual.dtype)
            return h, (ops.rmsnorm(h, norm_w, eps, offset) if norm_w is not None else None)
        t, n = residual.shape
        if n > self.max_cols:
            raise ValueError(f"row_linear: {n} features exceed the receive buffer's {self.max_cols}")
        h = torch.empty_like(residual)
        xn = torch.empty_like(residual) if norm_w is not None else None
        C = _native()
        for r0 in range(0, t, self.max_rows):
            r1 = min(t, r0 + self.max_rows)
            C.gemm_scatter(x[r0:r1], w, [p + _RECV for p in self.peers], self.base + _CH0 + 4, self.rank, self.slot)
            C.tp_reduce(self.base + _RECV, self.world, self.slot, residual[r0:r1], norm_w, eps, offset, h[r0:r1],
                        xn[r0:r1] if xn is not None else None, self.base + _CH0, self.err)
        return h, xn

    def lm_head_argmax(self, x: torch.Tensor, w_shard: torch.Tensor, lo: int) -> Tuple[torch.Tensor, torch.Tensor]:
        """Greedy ids over the whole vocabulary from this rank's row range ``[lo, lo + rows)`` of the LM head."""
        ids, val = ops.lm_head_argmax(x, w_shard)
        if self.world == 1 and not self.force_fused:
            return ids + lo, val
        if self.backend == "torch":
            both = torch.stack([val.double(), (ids + lo).double()], dim=1)
            parts = [torch.empty_like(both) for _ in range(self.world)]
            dist.all_gather(parts, both, group=self.group)
            stack = torch.stack(parts)  # [W, T, 2]
            best_val = stack[..., 0].amax(dim=0)
            cand = torch.where(stack[..., 0] == best_val[None], stack[..., 1], torch.full_like(stack[..., 1], 2 ** 40))
            return cand.amin(dim=0).long(), best_val.float()
        t = ids.shape[0]
        out_ids = torch.empty_like(ids)
        out_val = torch.empty_like(val)
        C = _native()
        for r0 in range(0, t, self.max_rows):
            r1 = min(t, r0 + self.max_rows)
            C.tp_argmax(ids[r0:r1], val[r0:r1], int(lo), [p + self.xbuf_off for p in self.peers], self.rank,
                        self.max_rows, self.base + _CH1, out_ids[r0:r1], out_val[r0:r1], self.err)
        return out_ids, out_val

    def gather_logits(self, local: torch.Tensor, vocab: int) -> torch.Tensor:
        """Full-vocabulary logits from the vocabulary-parallel shards (host-synchronising; not on the greedy path)."""
        parts = [torch.empty(local.shape[0], _shard_rows(vocab, self.world, r), dtype=local.dtype,
                             device=local.device) for r in range(self.world)]
        dist.all_gather(parts, local.contiguous(), group=self.group)
        return torch.cat(parts, dim=1)

    def max_over_ranks(self, values: List[float]) -> List[float]:
        """Host floats reduced by MAX over the ranks (measured timings, so every rank decides alike)."""
        if self.world == 1:
            return values
        t = torch.tensor(values, dtype=torch.float64, device=self.device if self.device.type == "cuda" else "cpu")
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self.group)
        return t.tolist()


def _shard_rows(vocab: int, world: int, rank: int) -> int:
    from eagle4_b200.parallel.sharding import vocab_range

    lo, hi = vocab_range(vocab, world, rank)
    return hi - lo


def _native():
    from eagle4_b200.ops import native

    return native._C


def init_distributed(timeout_s: int = 60) -> Tuple[int, int]:
    """Join the process group torchrun describes (NCCL on GPUs, gloo otherwise); returns ``(rank, world)``."""
    import datetime

    if not dist.is_initialized():
        backend = "nccl" if torch.cuda.is_available() else "gloo"
        if torch.cuda.is_available():
            torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s))
    return dist.get_rank(), dist.get_world_size()
