"""CUDA entry points: thin wrappers over the in-tree sm_100a extension (``eagle4_b200/csrc``).

Importing this module on a machine with a GPU loads the extension; if it cannot be loaded the import fails loudly
(there is no fallback path for CUDA tensors).
"""

from __future__ import annotations

import contextlib
from typing import Dict, Optional, Tuple

import torch

from eagle4_b200.ops.build import load


class _Counted:
    """The extension module with a count of kernel-launching calls (``LAUNCHES[0]``), for benchmark reports."""

    _QUIET = {"error_word"}

    def __init__(self, mod):
        self._mod = mod

    def __getattr__(self, name):
        fn = getattr(self._mod, name)
        if name in self._QUIET or not callable(fn):
            return fn

        def call(*a, **k):
            LAUNCHES[0] += 1
            return fn(*a, **k)

        return call


LAUNCHES = [0]
if torch.cuda.is_available():  # refuse a GPU the sm_100a kernels cannot run on, with the reason
    from eagle4_b200.utils.arch import require_sm100

    require_sm100()
_C = _Counted(load())

EPI_PLAIN, EPI_RESIDUAL, EPI_SWIGLU, EPI_RELU2, EPI_F32, EPI_ARGMAX = range(6)
_NONE = torch.Tensor()


def error_word(device=None) -> torch.Tensor:
    """The device word the kernels record their first error code in (0: none)."""
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    return _C.error_word(dev.index if dev.index is not None else torch.cuda.current_device())


def check_errors(device=None) -> None:
    w = error_word(device)
    code = int(w.item())
    if code:
        w.zero_()
        raise RuntimeError(f"eagle4_b200 kernel reported error code {code}")


def _c2(x: torch.Tensor) -> torch.Tensor:
    if x.dim() != 2:
        x = x.reshape(-1, x.shape[-1])
    if x.stride(-1) != 1 or (x.stride(0) * 2) % 16 or x.data_ptr() % 16:
        x = x.contiguous()
    return x


# dense ------------------------------------------------------------------------------------------------------------
@contextlib.contextmanager
def prefill_gemms():
    """GEMMs inside run as prefill launches: every token in one launch of whole (weight tile, 256-token chunk) units
    (no split tiles, no merges). Only for forwards whose outputs both the speculative and the plain path share
    (prompt prefill): decode and verify launches keep the partition that is independent of the token count."""
    _C.gemm_prefill_mode(True)
    try:
        yield
    finally:
        _C.gemm_prefill_mode(False)


def _fold(fold_eps: Optional[float]) -> float:
    return -1.0 if fold_eps is None else float(fold_eps)


def linear(x: torch.Tensor, w: torch.Tensor, fold_eps: Optional[float] = None) -> torch.Tensor:
    """``x @ w^T``; with ``fold_eps`` the RMSNorm of ``x`` is folded in (``w`` carries the norm weight)."""
    x = _c2(x)
    y = torch.empty(x.shape[0], w.shape[0], dtype=x.dtype, device=x.device)
    _C.gemm(x, w, EPI_PLAIN, y, _NONE, _NONE, _NONE, _NONE, _fold(fold_eps))
    return y


def linear_residual(x: torch.Tensor, w: torch.Tensor, residual: torch.Tensor) -> torch.Tensor:
    x = _c2(x)
    y = torch.empty(x.shape[0], w.shape[0], dtype=x.dtype, device=x.device)
    _C.gemm(x, w, EPI_RESIDUAL, y, _NONE, residual.contiguous(), _NONE, _NONE, -1.0)
    return y


def linear_swiglu(x: torch.Tensor, w_gu: torch.Tensor, fold_eps: Optional[float] = None) -> torch.Tensor:
    x = _c2(x)
    if w_gu.shape[0] % 128:
        raise ValueError("fused gate/up weight needs a multiple of 128 rows")
    y = torch.empty(x.shape[0], w_gu.shape[0] // 2, dtype=x.dtype, device=x.device)
    _C.gemm(x, w_gu, EPI_SWIGLU, y, _NONE, _NONE, _NONE, _NONE, _fold(fold_eps))
    return y


def linear_relu2(x: torch.Tensor, w: torch.Tensor, fold_eps: Optional[float] = None) -> torch.Tensor:
    x = _c2(x)
    y = torch.empty(x.shape[0], w.shape[0], dtype=x.dtype, device=x.device)
    _C.gemm(x, w, EPI_RELU2, y, _NONE, _NONE, _NONE, _NONE, _fold(fold_eps))
    return y


def moe_experts(latent: torch.Tensor, chosen: torch.Tensor, weights: torch.Tensor, up: torch.Tensor,
                down: torch.Tensor) -> torch.Tensor:
    """Routed latent-MoE experts: route by expert, grouped up / down GEMVs, weighted mix (``csrc/moe.cu``)."""
    return _C.moe_experts(latent.contiguous(), chosen, weights, up, down)


def logits(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    x = _c2(x)
    y = torch.empty(x.shape[0], w.shape[0], dtype=torch.float32, device=x.device)
    _C.gemm(x, w, EPI_F32, _NONE, y, _NONE, _NONE, _NONE, -1.0)
    return y


def lm_head_argmax(x: torch.Tensor, w: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    x = _c2(x)
    t = x.shape[0]
    n_tiles = (w.shape[0] + 127) // 128
    chunks = (t + 255) // 256
    val = torch.empty(chunks * 256 * n_tiles, dtype=torch.float32, device=x.device)
    idx = torch.empty(chunks * 256 * n_tiles, dtype=torch.int32, device=x.device)
    _C.gemm(x, w, EPI_ARGMAX, _NONE, _NONE, _NONE, val, idx, -1.0)
    ids, best = _C.argmax_reduce(val, idx, n_tiles, t)
    return ids, best


def lm_head_partials(x: torch.Tensor, w: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor, int]:
    """The LM-head GEMM's per-tile (max, argmax) partials ``(val, idx, n_tiles)`` (layout: see ``tp_argmax``)."""
    x = _c2(x)
    t = x.shape[0]
    n_tiles = (w.shape[0] + 127) // 128
    chunks = (t + 255) // 256
    val = torch.empty(chunks * 256 * n_tiles, dtype=torch.float32, device=x.device)
    idx = torch.empty(chunks * 256 * n_tiles, dtype=torch.int32, device=x.device)
    _C.gemm(x, w, EPI_ARGMAX, _NONE, _NONE, _NONE, val, idx, -1.0)
    return val, idx, n_tiles


# row ops ----------------------------------------------------------------------------------------------------------
def rmsnorm(x, w, eps, offset):
    return _C.rmsnorm(x, w, float(eps), bool(offset))


def embedding(ids, table):
    return _C.embedding(ids, table)


def concat_norms(e, h, we, wh, eps):
    return _C.concat_norms(e, h, we, wh, float(eps))


def gated_rmsnorm(o, z, w, eps, gate_first: bool = False):
    return _C.gated_rmsnorm(o, z, w, float(eps), bool(gate_first))


# attention --------------------------------------------------------------------------------------------------------
_ROPE: Dict[tuple, Tuple[torch.Tensor, torch.Tensor]] = {}


def rope_tables(rot: int, theta: float, device, max_pos: int = 1 << 17) -> Tuple[torch.Tensor, torch.Tensor]:
    """cos/sin of ``pos * theta^(-i/half)``, computed in float64 and stored as fp32 ``[max_pos, half]``."""
    key = (rot, float(theta), str(device), max_pos)
    if key not in _ROPE:
        half = max(rot // 2, 1)
        inv = 1.0 / (theta ** (torch.arange(0, half, dtype=torch.float64) / half))
        ang = torch.arange(max_pos, dtype=torch.float64)[:, None] * inv[None, :]
        _ROPE[key] = (ang.cos().float().to(device), ang.sin().float().to(device))
    return _ROPE[key]


def qkv_prepare(qkv, cfg, pos, write_slot, k_cache, v_cache, q_norm, k_norm):
    cos_t, sin_t = rope_tables(cfg.rotary_dim, cfg.rope_theta, qkv.device)
    q = _C.qkv_prepare(qkv, pos.long().contiguous(), write_slot.long().contiguous(), k_cache, v_cache, q_norm,
                       k_norm, bool(cfg.norm_offset), cos_t, sin_t, cfg.num_heads, cfg.num_kv_heads, cfg.head_dim,
                       cfg.rotary_dim, bool(cfg.attn_output_gate), float(cfg.rms_norm_eps))
    gate = None
    if cfg.attn_output_gate:
        hd = cfg.num_heads * cfg.head_dim
        gate = qkv[:, hd: 2 * hd]
    return q, gate


def attention(q, k_cache, v_cache, block_table, page, req, ctx_start, ctx_len, extra, n_extra, scale,
              max_keys: Optional[int] = None, gate: Optional[torch.Tensor] = None):
    if max_keys is None:
        max_keys = int(((ctx_len - ctx_start).clamp(min=0) + n_extra).max().item()) if q.shape[0] else 0
    o = _C.attention(q.contiguous(), k_cache, v_cache, block_table, int(page), req, ctx_start, ctx_len, extra,
                     n_extra, float(scale), int(max_keys), gate)
    return o.reshape(o.shape[0], -1)


# recurrent --------------------------------------------------------------------------------------------------------
def causal_conv_tree(x, conv_state, state_slot, parent, weight, bias=None):
    return _C.conv_tree(x, conv_state, state_slot, parent, weight, _NONE if bias is None else bias)


def _gdn_offsets(cfg):
    cd, vd, hv = cfg.gdn_conv_dim, cfg.gdn_value_dim, cfg.gdn_v_heads
    return cd, cd + vd, cd + vd + hv


def gdn_mixer(conv, proj, cfg, a_log, dt_bias, norm_w, state, state_slot, parent, scan: bool, segments=None):
    """``segments``: scan mode's request boundaries as a device table ([0, ..., T] int32); without it the boundaries
    are found from the slots on the host (a device-to-host read)."""
    z_off, b_off, a_off = _gdn_offsets(cfg)
    return _C.gdn_tree(conv, proj, z_off, b_off, a_off, a_log, dt_bias, state, state_slot, parent, norm_w,
                       float(cfg.rms_norm_eps), cfg.gdn_k_heads, cfg.gdn_v_heads, cfg.gdn_k_dim, cfg.gdn_v_dim,
                       bool(scan), _NONE if segments is None else segments)


def gdn_recurrence(qkv, a, b, a_log, dt_bias, state, state_slot, parent, cfg):
    """Tree gated delta rule from raw gate inputs ``a`` / ``b`` ``[T, HV]``, without the output norm."""
    hv = cfg.gdn_v_heads
    raw = torch.cat([b, a], dim=1).contiguous()
    return _C.gdn_tree(qkv, raw, 0, 0, hv, a_log, dt_bias, state, state_slot, parent, _NONE,
                       float(cfg.rms_norm_eps), cfg.gdn_k_heads, hv, cfg.gdn_k_dim, cfg.gdn_v_dim, False, _NONE)


def gdn_commit_all(convs, projs, states, conv_states, a_logs, dt_biases, slots, rows, n_rows, cfg):
    _, b_off, a_off = _gdn_offsets(cfg)
    _C.gdn_commit_all(list(convs), list(projs), list(states), list(conv_states), list(a_logs), list(dt_biases),
                      b_off, a_off, slots, rows, n_rows, cfg.gdn_k_heads, cfg.gdn_v_heads, cfg.gdn_k_dim,
                      cfg.gdn_v_dim, cfg.gdn_conv_dim, cfg.conv_kernel)


def conv_commit_scan(conv_state, x_pre, state_slot, kw, segments=None):
    _C.conv_commit_scan(conv_state, x_pre, state_slot, int(kw), _NONE if segments is None else segments)


def mamba_tree(xbc, dt_raw, a_log, dt_bias, d_skip, state, state_slot, parent, cfg, scan: bool, segments=None):
    return _C.mamba_tree(xbc, dt_raw, a_log, dt_bias, d_skip, state, state_slot, parent, cfg.mamba_heads,
                         cfg.mamba_head_dim, cfg.mamba_state, cfg.mamba_groups, bool(scan),
                         _NONE if segments is None else segments)


def mamba_commit(xbc, dt_raw, a_log, dt_bias, d_skip, x_pre, state, conv_state, slots, rows, n_rows, cfg):
    _C.mamba_commit(xbc, dt_raw, a_log, dt_bias, d_skip, state, slots, rows, n_rows, cfg.mamba_heads,
                    cfg.mamba_head_dim, cfg.mamba_state, cfg.mamba_groups)
    _C.conv_commit(x_pre, conv_state, slots, rows, n_rows, cfg.conv_kernel)


_PTRS: Dict[tuple, Tuple[torch.Tensor, torch.Tensor]] = {}


def kv_commit(k_caches, v_caches, src_slots, dst_slots):
    if src_slots.numel() == 0:
        return
    key = tuple(t.data_ptr() for t in k_caches)
    if key not in _PTRS:
        dev = src_slots.device
        _PTRS[key] = (torch.tensor([t.data_ptr() for t in k_caches], dtype=torch.int64, device=dev),
                      torch.tensor([t.data_ptr() for t in v_caches], dtype=torch.int64, device=dev))
    kp, vp = _PTRS[key]
    row = k_caches[0].shape[1] * k_caches[0].shape[2]
    _C.kv_commit(kp, vp, src_slots.long().contiguous(), dst_slots.long().contiguous(), row)


# draft head -------------------------------------------------------------------------------------------------------
def topk_rows(scores: torch.Tensor, k: int):
    """Top-k per row (value desc, index asc) by a two-stage radix select."""
    v, i = _C.topk_large(scores.float().contiguous(), int(k))
    return v, i


def candidate_logits(h, down, scores_w, lm_head, num_candidates: int):
    lr = linear(h, down)
    s = logits(lr, scores_w)
    _, idx = topk_rows(s, num_candidates)
    return idx, _C.gather_dot(h.contiguous(), lm_head, idx)


def candidate_head(h, down, scores_w, lm_head, num_candidates: int, k: int):
    idx, lg = candidate_logits(h, down, scores_w, lm_head, num_candidates)
    probs, ids = _C.softmax_topk(lg, idx, int(k), 1.0)
    return probs, ids


def full_head_topk(h, lm_head, k: int):
    lg = logits(h, lm_head)
    if lg.shape[1] <= 1024:
        probs, ids = _C.softmax_topk(lg, None, int(k), 1.0)
        return probs, ids
    p = torch.softmax(lg, dim=-1)
    return torch.topk(p, k, dim=-1)


def accept_greedy(target_ids, tokens, parent_rows, n_rows):
    acc, cnt, bonus = _C.accept_greedy(target_ids, tokens, parent_rows, n_rows)
    return acc, cnt, bonus


# sampled trees -----------------------------------------------------------------------------------------------------
def sample_children(logits, cand_ids, k, temperature, seed, round_ctr, stream, front_nodes, lanes, q_store, q_ids,
                    node_slot, child_base):
    return _C.sample_children(logits.float().contiguous(), cand_ids.long().contiguous(), int(k), float(temperature),
                              int(seed), round_ctr, int(stream), front_nodes, int(lanes), q_store, q_ids, node_slot,
                              int(child_base))


def sampled_accept(logits, temperature, row_parent, row_tok, row_node, q_store, q_ids, node_slot, k, seed, round_ctr,
                   stream):
    return _C.sampled_accept(logits, float(temperature), row_parent.int().contiguous(), row_tok.long().contiguous(),
                             row_node.long().contiguous(), q_store, q_ids, node_slot, int(k), int(seed), round_ctr,
                             int(stream))


def advance_round(round_ctr):
    _C.advance_round(round_ctr)
