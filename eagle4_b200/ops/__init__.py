"""Op entry points used by the models and runtime.

Tensors on a CUDA device run this package's sm_100a kernels (``eagle4_b200/csrc``, loaded by
``eagle4_b200.ops.native``); CPU tensors run the PyTorch definitions in ``eagle4_b200.ops.reference``, which are also
the oracle of the kernel tests. There is no other backend: on a GPU a missing extension is an error, never a silent
fallback.
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch

from eagle4_b200.ops import reference as ref


def _cuda(x: torch.Tensor) -> bool:
    return x.is_cuda


def _nat():
    from eagle4_b200.ops import native

    return native


# dense -----------------------------------------------------------------------------------------------------------
def linear(x: torch.Tensor, w: torch.Tensor, fold_eps: Optional[float] = None) -> torch.Tensor:
    """``x @ w^T``; with ``fold_eps`` the RMSNorm of ``x``'s rows is folded in (``w`` made by ``fold_norm_weight``)."""
    return _nat().linear(x, w, fold_eps) if _cuda(x) else ref.linear(x, w, fold_eps)


def linear_residual(x: torch.Tensor, w: torch.Tensor, residual: torch.Tensor) -> torch.Tensor:
    return _nat().linear_residual(x, w, residual) if _cuda(x) else ref.linear_residual(x, w, residual)


def linear_swiglu(x: torch.Tensor, w_gu: torch.Tensor, fold_eps: Optional[float] = None) -> torch.Tensor:
    return _nat().linear_swiglu(x, w_gu, fold_eps) if _cuda(x) else ref.linear_swiglu(x, w_gu, fold_eps)


def linear_relu2(x: torch.Tensor, w: torch.Tensor, fold_eps: Optional[float] = None) -> torch.Tensor:
    return _nat().linear_relu2(x, w, fold_eps) if _cuda(x) else ref.linear_relu2(x, w, fold_eps)


def fold_norm_weight(w: torch.Tensor, norm_w: torch.Tensor, offset: bool) -> torch.Tensor:
    """``w`` with an RMSNorm weight multiplied into its input columns (computed in float64, rounded once)."""
    return ref.fold_norm_weight(w, norm_w, offset)


def lm_head_argmax(x: torch.Tensor, w: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    return _nat().lm_head_argmax(x, w) if _cuda(x) else ref.lm_head_argmax(x, w)


def logits(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    return _nat().logits(x, w) if _cuda(x) else ref.logits(x, w)


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float, offset: bool) -> torch.Tensor:
    return _nat().rmsnorm(x, w, eps, offset) if _cuda(x) else ref.rmsnorm(x, w, eps, offset)


def embedding(ids: torch.Tensor, table: torch.Tensor) -> torch.Tensor:
    return _nat().embedding(ids, table) if _cuda(table) else ref.embedding(ids, table)


def concat_norms(e, h, we, wh, eps: float) -> torch.Tensor:
    return _nat().concat_norms(e, h, we, wh, eps) if _cuda(e) else ref.concat_norms(e, h, we, wh, eps)


# attention -------------------------------------------------------------------------------------------------------
def qkv_prepare(qkv, cfg, pos, write_slot, k_cache, v_cache, q_norm, k_norm):
    if _cuda(qkv):
        return _nat().qkv_prepare(qkv, cfg, pos, write_slot, k_cache, v_cache, q_norm, k_norm)
    return ref.qkv_prepare(qkv, cfg, pos, write_slot, k_cache, v_cache, q_norm, k_norm)


def attention(q, k_cache, v_cache, block_table, page, req, ctx_start, ctx_len, extra, n_extra, scale,
              max_keys=None, gate=None):
    """Tree attention; returns ``[T, Hq*D]`` (times ``sigmoid(gate)`` when a gate ``[T, Hq*D]`` is given).
    ``max_keys`` bounds every row's context + extras (required inside CUDA graphs: no host read)."""
    if _cuda(q):
        return _nat().attention(q, k_cache, v_cache, block_table, page, req, ctx_start, ctx_len, extra, n_extra,
                                scale, max_keys, gate)
    o = ref.attention(q, k_cache, v_cache, block_table, page, req, ctx_start, ctx_len, extra, n_extra, scale)
    o = o.reshape(o.shape[0], -1)
    return ref.sigmoid_gate(o, gate) if gate is not None else o


# recurrent -------------------------------------------------------------------------------------------------------
def causal_conv_tree(x, conv_state, state_slot, parent, weight, bias=None):
    """Tree causal conv + SiLU; ``bias`` ``[C]`` (optional) is added before the SiLU."""
    fn = _nat().causal_conv_tree if _cuda(x) else ref.causal_conv_tree
    return fn(x, conv_state, state_slot, parent, weight, bias)


def gdn_mixer(conv, proj, cfg, a_log, dt_bias, norm_w, state, state_slot, parent, scan: bool, segments=None):
    """Fused GDN token mixer after the conv: gates, tree recurrence and gated RMSNorm -> ``[T, HV*V]``.
    ``segments``: scan mode's request boundaries on the device (spares a device-to-host read)."""
    if _cuda(conv):
        return _nat().gdn_mixer(conv, proj, cfg, a_log, dt_bias, norm_w, state, state_slot, parent, scan, segments)
    return ref.gdn_mixer(conv, proj, cfg, a_log, dt_bias, norm_w, state, state_slot, parent, scan)


def gdn_commit_all(convs, projs, states, conv_states, a_logs, dt_biases, slots, rows, n_rows, cfg):
    """Commit accepted rows in every GDN layer at once (state replay and conv windows)."""
    if not convs:
        return
    fn = _nat().gdn_commit_all if _cuda(slots) else ref.gdn_commit_all
    return fn(convs, projs, states, conv_states, a_logs, dt_biases, slots, rows, n_rows, cfg)


def gdn_tree(qkv, g, beta, state, state_slot, parent, cfg, scan: bool):
    """Unfused gated delta rule (float64 definition; the CUDA path is ``gdn_mixer`` / ``gdn_recurrence``)."""
    return ref.gdn_tree(qkv, g, beta, state, state_slot, parent, cfg, scan)


def gdn_recurrence(qkv, a, b, a_log, dt_bias, state, state_slot, parent, cfg):
    """Tree gated delta rule from raw gates, no output norm: ``[T, HV * V]`` (host adapters apply their own norm)."""
    if _cuda(qkv):
        return _nat().gdn_recurrence(qkv, a, b, a_log, dt_bias, state, state_slot, parent, cfg)
    g, beta = ref.gdn_gates(a, b, a_log, dt_bias)
    return ref.gdn_tree(qkv, g, beta, state, state_slot, parent, cfg, False).reshape(qkv.shape[0], -1)


def gdn_commit(qkv, g, beta, x_pre, state, conv_state, slots, rows, n_rows, cfg):
    """Unfused commit (float64 definition; the CUDA path is ``gdn_commit_all``)."""
    return ref.gdn_commit(qkv, g, beta, x_pre, state, conv_state, slots, rows, n_rows, cfg)


def conv_commit_scan(conv_state, x_pre, state_slot, kw, segments=None):
    if _cuda(x_pre):
        return _nat().conv_commit_scan(conv_state, x_pre, state_slot, kw, segments)
    return ref.conv_commit_scan(conv_state, x_pre, state_slot, kw)


def gated_rmsnorm(o, z, w, eps, gate_first: bool = False):
    """``rmsnorm(o) * w * silu(z)`` per group of ``o [T, G, D]``, or with ``gate_first`` ``rmsnorm(o * silu(z)) * w``
    (Mamba2's form); ``w`` is one ``[D]`` row shared by the groups or ``G * D`` values."""
    fn = _nat().gated_rmsnorm if _cuda(o) else ref.gated_rmsnorm
    return fn(o, z, w, eps, gate_first)


def mamba_tree(xbc, dt_raw, a_log, dt_bias, d_skip, state, state_slot, parent, cfg, scan: bool, segments=None):
    if _cuda(xbc):
        return _nat().mamba_tree(xbc, dt_raw, a_log, dt_bias, d_skip, state, state_slot, parent, cfg, scan, segments)
    return ref.mamba_tree(xbc, dt_raw, a_log, dt_bias, d_skip, state, state_slot, parent, cfg, scan)


def mamba_commit(xbc, dt_raw, a_log, dt_bias, d_skip, x_pre, state, conv_state, slots, rows, n_rows, cfg):
    fn = _nat().mamba_commit if _cuda(xbc) else ref.mamba_commit
    return fn(xbc, dt_raw, a_log, dt_bias, d_skip, x_pre, state, conv_state, slots, rows, n_rows, cfg)


def kv_commit(k_caches, v_caches, src_slots, dst_slots):
    fn = _nat().kv_commit if _cuda(src_slots) else ref.kv_commit
    return fn(k_caches, v_caches, src_slots, dst_slots)


# draft head ------------------------------------------------------------------------------------------------------
def candidate_head(h, down, scores_w, lm_head, num_candidates: int, k: int):
    fn = _nat().candidate_head if _cuda(h) else ref.candidate_head
    return fn(h, down, scores_w, lm_head, num_candidates, k)


def candidate_logits(h, down, scores_w, lm_head, num_candidates: int):
    fn = _nat().candidate_logits if _cuda(h) else ref.candidate_logits
    return fn(h, down, scores_w, lm_head, num_candidates)


def full_head_topk(h, lm_head, k: int):
    return _nat().full_head_topk(h, lm_head, k) if _cuda(h) else ref.full_head_topk(h, lm_head, k)


def topk_rows(scores, k: int):
    return _nat().topk_rows(scores, k) if _cuda(scores) else ref.topk_rows(scores, k)


# acceptance ------------------------------------------------------------------------------------------------------
def accept_greedy(target_ids, tokens, parent_rows, n_rows):
    fn = _nat().accept_greedy if _cuda(tokens) else ref.accept_greedy
    return fn(target_ids, tokens, parent_rows, n_rows)


# sampled trees ------------------------------------------------------------------------------------------------------
def sample_children(logits, cand_ids, k, temperature, seed, round_ctr, stream, front_nodes, lanes, q_store, q_ids,
                    node_slot, child_base):
    """K children per row drawn without replacement (Gumbel-top-k) from ``softmax(logits / T)`` over the row's
    candidates; writes the rows' q and candidate ids to the q store and the children's slots to ``node_slot``.
    Returns ``(child probs [R, K] fp32, child ids [R, K] int64)``."""
    if _cuda(logits):
        return _nat().sample_children(logits, cand_ids, k, temperature, seed, round_ctr, stream, front_nodes, lanes,
                                      q_store, q_ids, node_slot, child_base)
    from eagle4_b200.core.sampled_tree import sample_children_reference

    r, c = logits.shape
    q, cp, ct, slots = sample_children_reference(logits, cand_ids, k, temperature, seed, int(round_ctr[0]), stream)
    b = torch.arange(r) // lanes
    lane = torch.arange(r) % lanes
    qrow = torch.zeros(r, dtype=torch.long) if front_nodes is None else 1 + front_nodes.reshape(-1).long()
    q_store[b, qrow] = q.to(q_store.dtype)
    q_ids[b, qrow] = cand_ids.to(q_ids.dtype)
    node_slot[b[:, None], child_base + lane[:, None] * k + torch.arange(k)[None, :]] = slots.to(node_slot.dtype)
    return cp.float(), ct.long()


def sampled_accept(logits, temperature, row_parent, row_tok, row_node, q_store, q_ids, node_slot, k, seed, round_ctr,
                   stream):
    """Recursive tree rejection over the verify rows: ``(accepted rows [bs, n], counts [bs], final token [bs])``."""
    if _cuda(logits):
        return _nat().sampled_accept(logits, temperature, row_parent, row_tok, row_node, q_store, q_ids, node_slot, k,
                                     seed, round_ctr, stream)
    from eagle4_b200.core.sampled_tree import sampled_walk_reference

    return sampled_walk_reference(logits, temperature, row_parent, row_node, q_store, q_ids, node_slot, k, seed,
                                  int(round_ctr[0]), stream)


def advance_round(round_ctr):
    if _cuda(round_ctr):
        _nat().advance_round(round_ctr)
    else:
        round_ctr += 1


# latent MoE MLP ---------------------------------------------------------------------------------------------------
def latent_moe(x: torch.Tensor, w: dict, moe: dict, residual: torch.Tensor) -> torch.Tensor:
    """``residual + fc2_latent(routed) + shared(x)`` of a latent ReLU^2 MoE (the Nemotron-H block a Nemotron-class
    EAGLE-4 draft uses): fp32 sigmoid router with bias-corrected choice, the routed experts in the latent space
    between ``fc1_latent`` and ``fc2_latent`` weighted by ``scale`` times the routing weights, plus the ReLU^2 shared
    expert (``eagle_harness/sglang/models/llama_eagle4.py:125-145``)."""
    chosen, wts = ref.moe_route(x, w["moe_gate"], w["moe_bias"], moe["top_k"], moe.get("n_group", 1),
                                moe.get("topk_group", 1), moe.get("norm_topk_prob", True))
    wts = wts * float(moe.get("scale", 1.0))
    latent = linear(x, w["fc1_latent"])
    experts = _nat().moe_experts if _cuda(x) else ref.moe_experts
    routed = experts(latent, chosen, wts, w["experts_up"], w["experts_down"])
    out = linear_residual(routed, w["fc2_latent"], residual)
    if "shared_up" in w:
        out = linear_residual(linear_relu2(x, w["shared_up"]), w["shared_down"], out)
    return out
