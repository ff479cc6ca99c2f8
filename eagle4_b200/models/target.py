"""Target language models for verification and plain decode.

One class serves the three target families of the configs (see ``configs.TargetConfig``). Weights are held as plain
tensors in fused layouts chosen for the sm_100a kernels:

* GDN ``in_proj``: ``[qkv | z | b | a]`` rows in one matrix (one GEMM per layer);
* attention ``qkv``: ``[q | gate | k | v]`` (the Qwen3.5 per-head ``[q_h, gate_h]`` interleave is undone at load);
* MLP ``gate_up``: gate and up rows interleaved in 64-row blocks so the GEMM epilogue applies SwiGLU in-tile;
* the block's output projection (``o_proj`` / ``out_proj`` / ``down``) adds the residual in its epilogue.

Every forward takes a ``RowBatch`` (the rows' positions, KV slots, visible context and tree links), so prefill,
tree verify and plain decode are the same code; plain decode is a verify of one row.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, List, Optional

import torch

from eagle4_b200 import ops
from eagle4_b200.models.configs import TargetConfig


@dataclass
class RowBatch:
    """Per-row metadata of one forward (T rows). All tensors live on the model's device."""

    ids: torch.Tensor  # [T] int64 token ids
    pos: torch.Tensor  # [T] int64 logical positions (RoPE)
    req: torch.Tensor  # [T] int32 request row in the block table
    write_slot: torch.Tensor  # [T] int64 physical KV slot this row writes
    ctx_start: torch.Tensor  # [T] int32 first visible committed position
    ctx_len: torch.Tensor  # [T] int32 end of the visible committed positions
    extra: torch.Tensor  # [T, X] int32 extra visible physical slots (ancestors, then itself)
    n_extra: torch.Tensor  # [T] int32
    parent: torch.Tensor  # [T] int32 parent row inside this forward (-1: the committed state)
    state_slot: torch.Tensor  # [T] int32 recurrent-state slot of the row's request
    scan: bool = False  # recurrent layers update their state in place row by row (prefill chains)
    max_keys: Optional[int] = None  # bound on any row's visible keys (lets attention skip a host read)
    segments: Optional[torch.Tensor] = None  # scan mode: request boundaries [0, ..., T] int32 on the device

    @property
    def num_rows(self) -> int:
        return self.ids.shape[0]


@dataclass
class TargetCache:
    """KV pages for attention layers and per-slot recurrent state for GDN / Mamba2 layers."""

    block_table: torch.Tensor  # [max_reqs, max_blocks] int32
    page: int
    k: List[torch.Tensor]  # per attention layer [slots, Hkv, D]
    v: List[torch.Tensor]
    conv: List[torch.Tensor]  # per recurrent layer [state_slots, C, K-1]
    ssm: List[torch.Tensor]  # per recurrent layer, fp32 ([slots, HV, V, K] GDN or [slots, H, P, N] Mamba2)

    @classmethod
    def allocate(cls, cfg: TargetConfig, *, max_reqs: int, max_len: int, page: int, device, dtype,
                 state_slots: Optional[int] = None, kv_pages: Optional[int] = None) -> "TargetCache":
        """Caches for ``max_reqs`` block-table rows of up to ``max_len`` positions. Without ``kv_pages`` every row
        owns ``max_len`` positions (an identity block table); with it the attention caches hold ``kv_pages`` pages
        that a :class:`~eagle4_b200.runtime.pages.PagePool` maps into the rows (all entries start at page 0)."""
        blocks_per_req = (max_len + page - 1) // page
        if kv_pages is None:
            nblocks = max_reqs * blocks_per_req
            bt = torch.arange(nblocks, dtype=torch.int32, device=device).view(max_reqs, blocks_per_req)
        else:
            nblocks = kv_pages
            bt = torch.zeros(max_reqs, blocks_per_req, dtype=torch.int32, device=device)
        slots = nblocks * page
        nattn = len(cfg.layer_ids("attn"))
        k = [torch.zeros(slots, cfg.num_kv_heads, cfg.head_dim, dtype=dtype, device=device) for _ in range(nattn)]
        v = [torch.zeros_like(t) for t in k]
        ns = state_slots or max_reqs
        conv, ssm = [], []
        kw = cfg.conv_kernel
        for m, _ in cfg.layers:
            if m == "gdn":
                conv.append(torch.zeros(ns, cfg.gdn_conv_dim, kw - 1, dtype=dtype, device=device))
                ssm.append(torch.zeros(ns, cfg.gdn_v_heads, cfg.gdn_v_dim, cfg.gdn_k_dim, dtype=torch.float32,
                                       device=device))
            elif m == "mamba":
                conv.append(torch.zeros(ns, cfg.mamba_conv_dim, kw - 1, dtype=dtype, device=device))
                ssm.append(torch.zeros(ns, cfg.mamba_heads, cfg.mamba_head_dim, cfg.mamba_state,
                                       dtype=torch.float32, device=device))
        return cls(bt, page, k, v, conv, ssm)

    def reset_slot(self, slot: int) -> None:
        for t in self.conv:
            t[slot].zero_()
        for t in self.ssm:
            t[slot].zero_()


@dataclass
class Records:
    """What a tree verify keeps per recurrent layer so the accepted path can be committed afterwards."""

    layer: List[int] = field(default_factory=list)  # model layer of each entry
    x_pre: List[torch.Tensor] = field(default_factory=list)  # GDN: the whole in_proj output; Mamba2: conv inputs
    conv_out: List[torch.Tensor] = field(default_factory=list)  # post-conv [T, C]
    gate_a: List[torch.Tensor] = field(default_factory=list)  # Mamba2 raw dt [T, H] (None for GDN)


FOLDED = "__input_norms_folded__"  # marks a weight dict whose projections carry their input norm weights

# the projection that consumes each sub-block's input norm
_CONSUMER = {"attn": "qkv", "gdn": "in_proj", "mamba": "in_proj", "swiglu": "gate_up", "relu2": "up"}


def fold_input_norms(cfg: TargetConfig, weights: Dict[str, torch.Tensor]) -> None:
    """Multiply every sub-block's input-norm weight into the columns of the projection that consumes it (once per
    dict: the dict is marked), so the projection can take the raw residual stream and apply the norm's per-token
    scale in its epilogue. The final norm before the LM head stays a separate op."""
    if FOLDED in weights:
        return
    for i, (mixer, mlp) in enumerate(cfg.layers):
        for kind, norm in ((mixer, "norm1"), (mlp, "norm2")):
            if kind is None:
                continue
            name = f"l{i}.{_CONSUMER[kind]}"
            weights[name] = ops.fold_norm_weight(weights[name], weights[f"l{i}.{norm}"], cfg.norm_offset)
    weights[FOLDED] = torch.ones(())


class TargetModel:
    def __init__(self, cfg: TargetConfig, weights: Dict[str, torch.Tensor], *, aux_layer_ids=(), tp=None,
                 fold_norms: bool = True):
        """``cfg`` / ``weights`` are this rank's shard under tensor parallelism (``tp``: a
        :class:`~eagle4_b200.parallel.tp.TensorParallel`; None on one GPU). With ``fold_norms`` (the default) the
        sub-blocks' input norms are folded into their first projections (``weights`` is updated in place, once)."""
        self.cfg = cfg
        self.w = weights
        self.fold = fold_norms
        if fold_norms:
            fold_input_norms(cfg, weights)
        elif FOLDED in weights:
            raise ValueError("these weights carry folded input norms: build the model with fold_norms=True")
        self.fold_eps = cfg.rms_norm_eps if fold_norms else None
        self.tp = tp
        self.lm_lo = int(weights["lm_head_lo"]) if "lm_head_lo" in weights else 0
        self.aux_layer_ids = tuple(aux_layer_ids)
        self.device = weights["embed"].device
        self.dtype = weights["embed"].dtype
        # cache index of each layer inside its kind's list
        self.attn_index: Dict[int, int] = {}
        self.rec_index: Dict[int, int] = {}
        for i, (m, _) in enumerate(cfg.layers):
            if m == "attn":
                self.attn_index[i] = len(self.attn_index)
            elif m in ("gdn", "mamba"):
                self.rec_index[i] = len(self.rec_index)
        # the norm applied to the residual stream after each sub-block (the next sub-block's input norm)
        norms = [f"l{i}.{n}" for i, (m, f) in enumerate(cfg.layers) for n, on in (("norm1", m), ("norm2", f)) if on]
        self.next_norm = dict(zip(norms, norms[1:] + ["norm"]))

    def _row(self, y: torch.Tensor, w_out: torch.Tensor, h: torch.Tensor, after: str):
        """Row-parallel output projection + residual, then the next sub-block's input: ``(h, x_next)``. With folded
        norms ``x_next`` is ``h`` itself (the next projection normalises), except before the LM head."""
        nxt = self.next_norm[after]
        nw = None if (self.fold and nxt != "norm") else self.w[nxt]
        if self.tp is not None:
            h, xn = self.tp.row_linear(y, w_out, h, nw, self.cfg.rms_norm_eps, self.cfg.norm_offset)
            return h, (h if nw is None else xn)
        h = ops.linear_residual(y, w_out, h)
        return h, (h if nw is None else ops.rmsnorm(h, nw, self.cfg.rms_norm_eps, self.cfg.norm_offset))

    # ------------------------------------------------------------------ blocks
    def _attn(self, i: int, x: torch.Tensor, h: torch.Tensor, rb: RowBatch, cache: TargetCache) -> torch.Tensor:
        cfg, w = self.cfg, self.w
        li = self.attn_index[i]
        qkv = ops.linear(x, w[f"l{i}.qkv"], self.fold_eps)
        q, gate = ops.qkv_prepare(qkv, cfg, rb.pos, rb.write_slot, cache.k[li], cache.v[li],
                                  w.get(f"l{i}.q_norm"), w.get(f"l{i}.k_norm"))
        o = ops.attention(q, cache.k[li], cache.v[li], cache.block_table, cache.page, rb.req, rb.ctx_start,
                          rb.ctx_len, rb.extra, rb.n_extra, cfg.head_dim ** -0.5, rb.max_keys, gate)
        return self._row(o, w[f"l{i}.o_proj"], h, f"l{i}.norm1")

    def _gdn(self, i: int, x: torch.Tensor, h: torch.Tensor, rb: RowBatch, cache: TargetCache,
             rec: Optional[Records]) -> torch.Tensor:
        cfg, w = self.cfg, self.w
        ri = self.rec_index[i]
        cd, vd, hv = cfg.gdn_conv_dim, cfg.gdn_value_dim, cfg.gdn_v_heads
        proj = ops.linear(x, w[f"l{i}.in_proj"], self.fold_eps)
        x_pre = proj[:, :cd]
        conv = ops.causal_conv_tree(x_pre, cache.conv[ri], rb.state_slot, rb.parent, w[f"l{i}.conv"])
        y = ops.gdn_mixer(conv, proj, cfg, w[f"l{i}.A_log"], w[f"l{i}.dt_bias"], w[f"l{i}.gnorm"], cache.ssm[ri],
                          rb.state_slot, rb.parent, rb.scan, rb.segments)
        if rb.scan:
            ops.conv_commit_scan(cache.conv[ri], x_pre, rb.state_slot, cfg.conv_kernel, rb.segments)
        elif rec is not None:
            rec.layer.append(i)
            rec.x_pre.append(proj)
            rec.conv_out.append(conv)
            rec.gate_a.append(None)
        return self._row(y, w[f"l{i}.out_proj"], h, f"l{i}.norm1")

    def _mamba(self, i: int, x: torch.Tensor, h: torch.Tensor, rb: RowBatch, cache: TargetCache,
               rec: Optional[Records]) -> torch.Tensor:
        cfg, w = self.cfg, self.w
        ri = self.rec_index[i]
        inner, cd, nh = cfg.mamba_inner, cfg.mamba_conv_dim, cfg.mamba_heads
        proj = ops.linear(x, w[f"l{i}.in_proj"], self.fold_eps)
        z = proj[:, :inner]
        x_pre = proj[:, inner: inner + cd]
        dt = proj[:, inner + cd: inner + cd + nh]
        conv = ops.causal_conv_tree(x_pre, cache.conv[ri], rb.state_slot, rb.parent, w[f"l{i}.conv"],
                                    w.get(f"l{i}.conv_bias"))
        y = ops.mamba_tree(conv, dt, w[f"l{i}.A_log"], w[f"l{i}.dt_bias"], w[f"l{i}.D"], cache.ssm[ri],
                           rb.state_slot, rb.parent, cfg, rb.scan, rb.segments)
        if rb.scan:
            ops.conv_commit_scan(cache.conv[ri], x_pre, rb.state_slot, cfg.conv_kernel, rb.segments)
        elif rec is not None:
            rec.layer.append(i)
            rec.x_pre.append(x_pre)
            rec.conv_out.append(conv)
            rec.gate_a.append(dt)
        group = cfg.mamba_inner // cfg.mamba_groups
        y = ops.gated_rmsnorm(y.reshape(y.shape[0], cfg.mamba_groups, group), z, w[f"l{i}.gnorm"], cfg.rms_norm_eps,
                              cfg.mamba_gate_first)
        return self._row(y, w[f"l{i}.out_proj"], h, f"l{i}.norm1")

    def _mlp(self, i: int, x: torch.Tensor, h: torch.Tensor, kind: str) -> torch.Tensor:
        w = self.w
        if kind == "swiglu":
            a = ops.linear_swiglu(x, w[f"l{i}.gate_up"], self.fold_eps)
        else:
            a = ops.linear_relu2(x, w[f"l{i}.up"], self.fold_eps)
        return self._row(a, w[f"l{i}.down"], h, f"l{i}.norm2")

    # ------------------------------------------------------------------ forward
    def forward(self, rb: RowBatch, cache: TargetCache, rec: Optional[Records] = None):
        """Returns ``(final normed hidden [T, H], aux hidden [T, n_aux * H] or None)``. Scan-mode (prefill) forwards
        on a GPU run their GEMMs as prefill launches (``native.prefill_gemms``)."""
        if rb.scan and rb.ids.is_cuda:
            from eagle4_b200.ops import native

            with native.prefill_gemms():
                return self._forward(rb, cache, rec)
        return self._forward(rb, cache, rec)

    def _forward(self, rb: RowBatch, cache: TargetCache, rec: Optional[Records] = None):
        cfg, w = self.cfg, self.w
        eps, off = cfg.rms_norm_eps, cfg.norm_offset
        h = ops.embedding(rb.ids, w["embed"])
        first = next(iter(self.next_norm))
        # each sub-block returns the next one's input (normed, or raw when the next projection folds the norm)
        x = h if self.fold else ops.rmsnorm(h, w[first], eps, off)
        saved: Dict[int, torch.Tensor] = {}
        for i, (mixer, mlp) in enumerate(cfg.layers):
            if mixer is not None:
                if mixer == "attn":
                    h, x = self._attn(i, x, h, rb, cache)
                elif mixer == "gdn":
                    h, x = self._gdn(i, x, h, rb, cache, rec)
                else:
                    h, x = self._mamba(i, x, h, rb, cache, rec)
            if mlp is not None:
                h, x = self._mlp(i, x, h, mlp)
            if i in self.aux_layer_ids:
                saved[i] = h
        aux = [saved[i] for i in self.aux_layer_ids if i in saved]
        return x, (torch.cat(aux, dim=-1) if aux else None)

    def greedy(self, hidden: torch.Tensor):
        if self.tp is not None:
            return self.tp.lm_head_argmax(hidden, self.w["lm_head"], self.lm_lo)
        return ops.lm_head_argmax(hidden, self.w["lm_head"])

    def sampled_accept(self, hidden: torch.Tensor, temperature: float, row_parent, row_tok, row_node, q_store, q_ids,
                       node_slot, k: int, seed: int, round_ctr, stream: int):
        """Recursive tree rejection of the rows of ``hidden`` (``ops.sampled_accept``); under tensor parallelism the
        vocabulary-parallel form, which exchanges row statistics and candidate probabilities instead of logits."""
        if self.tp is not None and self.tp.world > 1:
            local = ops.logits(hidden, self.w["lm_head"])
            return self.tp.sampled_accept(local, self.lm_lo, temperature, row_parent, row_tok, row_node, q_store,
                                          q_ids, node_slot, k, seed, round_ctr, stream)
        return ops.sampled_accept(self.logits(hidden), temperature, row_parent, row_tok, row_node, q_store, q_ids,
                                  node_slot, k, seed, round_ctr, stream)

    def logits(self, hidden: torch.Tensor) -> torch.Tensor:
        local = ops.logits(hidden, self.w["lm_head"])
        if self.tp is not None and self.tp.world > 1:
            return self.tp.gather_logits(local, self.cfg.vocab_size)
        return local

    # ------------------------------------------------------------------ commit
    def commit(self, cache: TargetCache, rec: Records, rows: torch.Tensor, n_rows: torch.Tensor,
               slots: torch.Tensor, src_kv: torch.Tensor, dst_kv: torch.Tensor) -> None:
        """Commit the accepted rows: recurrent state replay along the path and KV moves in attention layers."""
        cfg, w = self.cfg, self.w
        gdn = [(j, li) for j, li in enumerate(rec.layer) if cfg.layers[li][0] == "gdn"]
        if gdn:
            ops.gdn_commit_all([rec.conv_out[j] for j, _ in gdn], [rec.x_pre[j] for j, _ in gdn],
                               [cache.ssm[self.rec_index[li]] for _, li in gdn],
                               [cache.conv[self.rec_index[li]] for _, li in gdn],
                               [w[f"l{li}.A_log"] for _, li in gdn], [w[f"l{li}.dt_bias"] for _, li in gdn],
                               slots, rows, n_rows, cfg)
        for j, li in enumerate(rec.layer):
            if cfg.layers[li][0] != "mamba":
                continue
            ri = self.rec_index[li]
            ops.mamba_commit(rec.conv_out[j], rec.gate_a[j], w[f"l{li}.A_log"], w[f"l{li}.dt_bias"], w[f"l{li}.D"],
                             rec.x_pre[j], cache.ssm[ri], cache.conv[ri], slots, rows, n_rows, cfg)
        if cache.k:
            ops.kv_commit(cache.k, cache.v, src_kv, dst_kv)
