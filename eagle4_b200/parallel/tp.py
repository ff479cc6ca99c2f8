"""Tensor parallelism: one rank per GPU, ``torch.distributed`` for setup, and two data paths for the collectives.

``backend="fused"`` (the B200 path): a row-parallel linear is ONE GEMM launch whose epilogue does the all-reduce
over NVLink peer memory (CUDA IPC mappings of one symmetric buffer per rank) and adds the residual: each finished
tile leaves as bf16 while the next tiles' MMAs run, the CTA that finished a tile sums it over the ranks in rank order
once every rank's copy has landed (per-tile release / acquire flags tagged with the call number), and the kernel
returns only when this rank holds the whole result. Up to ``two_shot_rows`` tokens per launch every rank receives
every partial (one-shot: one NVLink hop); above it a tile goes only to its home rank (reduce-scatter), which reduces
it and pushes the result to the others (all-gather), so each rank sends 2 (w-1)/w of the output instead of w-1 times
it. The greedy head's vocabulary-parallel argmax is the LM-head GEMM's per-tile (max, argmax) epilogue plus one
kernel that reduces the tiles and exchanges (max, id) pairs across the ranks. All of it is captured in the engine's
CUDA graphs.

``backend="torch"``: the same math through ``torch.distributed.all_reduce`` / ``all_gather`` (NCCL on GPUs, gloo on
CPU) over bf16 partials: the baseline the fused path is measured against, and the CPU oracle of the multi-process
tests.

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
TP_ROWS = 256  # tokens per GEMM launch (the GEMM splits larger inputs into launches of at most this many)
TP_TILES = 64  # 128-row weight tiles per launch: output features up to 8192
# symmetric buffer layout (bytes): control words, arrival flags, partial areas, gathered areas, argmax exchange
_CTRL_GEMM, _CTRL_ARGMAX = 0, 256  # GEMM: (calls, done); argmax exchange: (done, calls)
_FLAGS = 4096
_FLAG_BYTES = (2 * TP_TILES * MAX_RANKS + 2 * TP_TILES) * 4
_PART = 16384


class TensorParallel:
    def __init__(self, group=None, *, backend: str = "fused", max_rows: int = 1024, max_cols: int = 8192,
                 device: Optional[torch.device] = None, two_shot_rows: Optional[int] = None):
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
        self.max_rows, self.max_cols = (max_rows + 255) // 256 * 256, max_cols
        if two_shot_rows is None:
            two_shot_rows = int(os.environ.get("E4_TP_TWO_SHOT_ROWS", "48"))
        self.two_shot_rows = two_shot_rows
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
        self.ldp = (self.max_cols + 7) // 8 * 8
        part_bytes = 2 * MAX_RANKS * TP_ROWS * self.ldp * 2
        gath_bytes = 2 * TP_ROWS * self.ldp * 2
        self.gath_off = _PART + part_bytes
        self.xbuf_off = self.gath_off + gath_bytes
        total = self.xbuf_off + 2 * MAX_RANKS * self.max_rows * 16
        self.base = C.sym_alloc(total, dev)  # zero-filled: no flag carries a tag yet
        handle = C.sym_handle(self.base)
        handles: List[Optional[torch.Tensor]] = [None] * self.world
        dist.all_gather_object(handles, handle, group=self.group)
        self.peers = [self.base if r == self.rank else C.sym_open(handles[r], dev) for r in range(self.world)]
        self.err = native.error_word(self.device)
        dist.barrier(group=self.group)

    def nvlink_bytes(self, tokens: int, features: int) -> int:
        """Bytes one rank sends over NVLink for one row-parallel projection of ``tokens`` x ``features``."""
        if self.world == 1:
            return 0
        el = 2 * features
        total = 0
        for r0 in range(0, tokens, TP_ROWS):
            t = min(TP_ROWS, tokens - r0)
            if t > self.two_shot_rows:  # reduce-scatter then all-gather of this rank's home tiles
                tiles = (features + 127) // 128
                home = len([i for i in range(tiles) if i % self.world == self.rank])
                total += t * 128 * 2 * (tiles - home) + t * 128 * 2 * home * (self.world - 1)
            else:
                total += t * el * (self.world - 1)
        return total

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
            raise ValueError(f"row_linear: {n} features exceed the peer areas' {self.max_cols}")
        h = torch.empty_like(residual)
        C = _native()
        part = [p + _PART for p in self.peers]
        gath = [p + self.gath_off for p in self.peers]
        flags = [p + _FLAGS for p in self.peers]
        C.gemm_allreduce(_rows16(x), w, residual.contiguous(), h, part, gath, flags, self.base + _CTRL_GEMM,
                         self.ldp, self.rank, self.two_shot_rows)
        return h, (ops.rmsnorm(h, norm_w, eps, offset) if norm_w is not None else None)

    def lm_head_argmax(self, x: torch.Tensor, w_shard: torch.Tensor, lo: int) -> Tuple[torch.Tensor, torch.Tensor]:
        """Greedy ids over the whole vocabulary from this rank's row range ``[lo, lo + rows)`` of the LM head."""
        if self.backend == "torch" or (self.world == 1 and not self.force_fused):
            ids, val = ops.lm_head_argmax(x, w_shard)
            if self.world == 1:
                return ids + lo, val
            both = torch.stack([val.double(), (ids + lo).double()], dim=1)
            parts = [torch.empty_like(both) for _ in range(self.world)]
            dist.all_gather(parts, both, group=self.group)
            stack = torch.stack(parts)  # [W, T, 2]
            best_val = stack[..., 0].amax(dim=0)
            cand = torch.where(stack[..., 0] == best_val[None], stack[..., 1], torch.full_like(stack[..., 1], 2 ** 40))
            return cand.amin(dim=0).long(), best_val.float()
        from eagle4_b200.ops import native

        val, idx, n_tiles = native.lm_head_partials(x, w_shard)
        t = x.shape[0]
        out_ids = torch.empty(t, dtype=torch.int64, device=x.device)
        out_val = torch.empty(t, dtype=torch.float32, device=x.device)
        C = _native()
        for r0 in range(0, t, self.max_rows):
            r1 = min(t, r0 + self.max_rows)
            # partials of rows [r0, r1): whole 256-row chunks of the GEMM's layout (max_rows is a multiple of 256)
            c0 = r0 // 256
            C.tp_argmax(val[c0 * 256 * n_tiles:], idx[c0 * 256 * n_tiles:], n_tiles, int(lo),
                        [p + self.xbuf_off for p in self.peers], self.rank, self.max_rows, self.base + _CTRL_ARGMAX,
                        out_ids[r0:r1], out_val[r0:r1], self.err)
        return out_ids, out_val

    def gather_logits(self, local: torch.Tensor, vocab: int) -> torch.Tensor:
        """Full-vocabulary logits from the vocabulary-parallel shards (host-synchronising; not on the greedy path)."""
        parts = [torch.empty(local.shape[0], _shard_rows(vocab, self.world, r), dtype=local.dtype,
                             device=local.device) for r in range(self.world)]
        dist.all_gather(parts, local.contiguous(), group=self.group)
        return torch.cat(parts, dim=1)

    def sampled_accept(self, local: torch.Tensor, lo: int, temperature: float, row_parent, row_tok, row_node, q_store,
                       q_ids, node_slot, k: int, seed: int, round_ctr, stream: int):
        """Recursive tree rejection over vocabulary-parallel logits (``local``: this rank's fp32 shard of the verify
        rows' logits, vocabulary ids ``[lo, lo + Vl)``), exchanging a few floats per row instead of the logits:

        1. row statistics: each rank's max and sum of exp over its shard, all-gathered (2 floats per row and rank),
           combined in rank order into the global max and normaliser;
        2. the target probabilities at each row's draft candidates, computed by the rank owning each id and
           sum-reduced ([rows, C] floats);
        3. the walk, identical on every rank, from those probabilities; it leaves each request's final row and the
           residual at its candidates;
        4. the final draw: each rank's residual mass of the final rows (one float per request and rank), then the
           rank whose cumulative mass passes the target searches its shard; the token is max-reduced.

        Returns (accepted rows [bs, n], counts [bs], final token [bs]) on every rank."""
        from eagle4_b200.core import sampled_tree as st

        bs, n = row_parent.shape
        S, C = q_store.shape[1], q_store.shape[2]
        vl = local.shape[1]
        cuda = local.is_cuda
        lg = local.float() * (1.0 / temperature)
        mx_l = lg.amax(dim=-1)
        z_l = torch.exp(lg - mx_l[:, None]).sum(dim=-1)
        stats = torch.stack([mx_l, z_l], dim=1).contiguous()
        parts = [torch.empty_like(stats) for _ in range(self.world)]
        dist.all_gather(parts, stats, group=self.group)
        allst = torch.stack(parts)  # [W, T, 2]
        mx = allst[..., 0].amax(dim=0)
        z = (allst[..., 1] * torch.exp(allst[..., 0] - mx[None])).sum(dim=0)
        node = row_node.reshape(-1)
        req = torch.arange(bs, device=local.device).repeat_interleave(n)
        qrow = req * S + torch.where(node < 0, torch.zeros_like(node), node + 1)
        ids = q_ids.reshape(bs * S, C).index_select(0, qrow).long()
        own = (ids >= lo) & (ids < lo + vl)
        vals = lg.gather(1, (ids - lo).clamp(0, vl - 1))
        p = torch.where(own, torch.exp(vals - mx[:, None]) / z[:, None], torch.zeros_like(vals)).contiguous()
        dist.all_reduce(p, op=dist.ReduceOp.SUM, group=self.group)
        if cuda:
            C_ = _native()
            acc, cnt, final, r_final = C_.sampled_walk_sparse(p, row_parent, row_tok, row_node, q_store, q_ids,
                                                              node_slot, k, seed, round_ctr, stream)
            mass = C_.shard_residual_mass(local.float().contiguous(), lo, temperature, mx.contiguous(),
                                          z.contiguous(), final, row_node, q_ids, r_final.contiguous(), S, n)
        else:
            rnd = int(round_ctr[0])
            acc, cnt, final, r_final = st.sampled_walk_sparse_reference(p, row_parent, row_node, q_store, q_ids,
                                                                        node_slot, k, seed, rnd, stream)
            resid = st.shard_residual(local.float(), lo, temperature, mx, z, final, row_node, q_ids, r_final, n)
            mass = resid.sum(dim=1).float()
        masses = [torch.empty_like(mass) for _ in range(self.world)]
        dist.all_gather(masses, mass.contiguous(), group=self.group)
        masses = torch.stack(masses).contiguous()
        if cuda:
            tok = _native().shard_draw(local.float().contiguous(), lo, temperature, mx.contiguous(), z.contiguous(),
                                       final, row_node, q_ids, r_final.contiguous(), S, n, masses, self.rank, seed,
                                       round_ctr, stream)
        else:
            tok = st.shard_draw_reference(resid, lo, masses, self.rank, seed, int(round_ctr[0]), stream)
        dist.all_reduce(tok, op=dist.ReduceOp.MAX, group=self.group)
        return acc, cnt, tok

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


def _rows16(x: torch.Tensor) -> torch.Tensor:
    """``x`` as a 2-D tensor with contiguous 16-byte-aligned rows (the GEMM's TMA operand)."""
    from eagle4_b200.ops import native

    return native._c2(x)


def init_distributed(timeout_s: int = 60) -> Tuple[int, int]:
    """Join the process group torchrun describes (NCCL on GPUs, gloo otherwise); returns ``(rank, world)``."""
    import datetime

    if not dist.is_initialized():
        backend = "nccl" if torch.cuda.is_available() else "gloo"
        if torch.cuda.is_available():
            torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s))
    return dist.get_rank(), dist.get_world_size()
