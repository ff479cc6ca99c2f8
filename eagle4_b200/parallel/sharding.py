"""Tensor-parallel sharding of the target and draft weights (Megatron layout, one rank per GPU).

Column-parallel (output features split, no communication): attention q/gate/k/v by heads, GDN and Mamba2 in_proj by
heads (their conv channels, gates and per-head parameters follow), MLP gate/up by intermediate channels. Row-parallel
(input features split, partial sums all-reduced): attention o_proj, GDN / Mamba2 out_proj, MLP down. KV heads fewer
than the ranks are replicated, one per rank. The LM head is vocabulary-parallel: rank ``r`` owns a contiguous row
range whose boundaries are multiples of 128 (the GEMM's weight tile), and the greedy head exchanges (max, argmax)
across ranks. The embedding, the norms and the draft's candidate head are replicated.

A sharded rank runs the unchanged layer code on a config whose head / channel counts are the local ones
(:func:`local_target_config`); the fused in-projection layouts keep their order, so every offset the kernels use
comes out right for the local sizes. Shards are contiguous copies (TMA needs 16-byte aligned rows).
"""

from __future__ import annotations

import dataclasses
from typing import Dict, List, Tuple

import torch

from eagle4_b200.models.configs import DraftConfig, TargetConfig

LM_TILE = 128
MLP_BLOCK = 64  # gate/up rows are interleaved in blocks of 64 channels


def _check(cond: bool, what: str) -> None:
    if not cond:
        raise ValueError(f"tensor parallelism: {what}")


def kv_layout(num_heads: int, num_kv_heads: int, world: int, rank: int) -> Tuple[int, int]:
    """``(local kv heads, first kv head)`` of ``rank``; KV heads fewer than the ranks are replicated."""
    _check(num_heads % world == 0, f"{num_heads} query heads do not split over {world} ranks")
    if num_kv_heads >= world:
        _check(num_kv_heads % world == 0, f"{num_kv_heads} kv heads do not split over {world} ranks")
        n = num_kv_heads // world
        return n, rank * n
    _check(world % num_kv_heads == 0, f"{world} ranks do not replicate {num_kv_heads} kv heads evenly")
    return 1, rank // (world // num_kv_heads)


def vocab_range(vocab: int, world: int, rank: int) -> Tuple[int, int]:
    """Rows ``[lo, hi)`` of the vocabulary-parallel LM head owned by ``rank`` (boundaries on 128-row tiles)."""
    chunk = -(-vocab // world)
    chunk = -(-chunk // LM_TILE) * LM_TILE
    lo = min(vocab, rank * chunk)
    return lo, min(vocab, lo + chunk)


def local_target_config(cfg: TargetConfig, world: int, rank: int) -> TargetConfig:
    if world == 1:
        return cfg
    upd = {}
    if cfg.layer_ids("attn"):
        kv, _ = kv_layout(cfg.num_heads, cfg.num_kv_heads, world, rank)
        upd.update(num_heads=cfg.num_heads // world, num_kv_heads=kv)
    if cfg.layer_ids("gdn"):
        _check(cfg.gdn_k_heads % world == 0 and cfg.gdn_v_heads % world == 0,
               f"GDN heads {cfg.gdn_k_heads}/{cfg.gdn_v_heads} do not split over {world} ranks")
        upd.update(gdn_k_heads=cfg.gdn_k_heads // world, gdn_v_heads=cfg.gdn_v_heads // world)
    if cfg.layer_ids("mamba"):
        _check(cfg.mamba_heads % world == 0 and cfg.mamba_groups % world == 0,
               f"Mamba2 heads {cfg.mamba_heads} / groups {cfg.mamba_groups} do not split over {world} ranks")
        upd.update(mamba_heads=cfg.mamba_heads // world, mamba_groups=cfg.mamba_groups // world)
    _check(cfg.intermediate_size % (world * MLP_BLOCK) == 0,
           f"intermediate size {cfg.intermediate_size} does not split over {world} ranks in {MLP_BLOCK}-blocks")
    upd["intermediate_size"] = cfg.intermediate_size // world
    return dataclasses.replace(cfg, **upd)


def _rows(w: torch.Tensor, pieces: List[Tuple[int, int]]) -> torch.Tensor:
    return torch.cat([w[a:b] for a, b in pieces], dim=0).contiguous()


def _cols(w: torch.Tensor, a: int, b: int) -> torch.Tensor:
    return w[:, a:b].contiguous()


def shard_target(cfg: TargetConfig, w: Dict[str, torch.Tensor], world: int, rank: int
                 ) -> Tuple[TargetConfig, Dict[str, torch.Tensor]]:
    """``(local config, local weights)`` of ``rank``; the LM head keeps its global row range in ``lm_head_lo``."""
    if world == 1:
        return cfg, w
    loc = local_target_config(cfg, world, rank)
    out: Dict[str, torch.Tensor] = {"embed": w["embed"], "norm": w["norm"]}
    lo, hi = vocab_range(cfg.vocab_size, world, rank)
    out["lm_head"] = w["lm_head"][lo:hi].contiguous()
    out["lm_head_lo"] = torch.tensor(lo)
    from eagle4_b200.models.target import FOLDED

    if FOLDED in w:  # the column-parallel shards of folded projections are folded too
        out[FOLDED] = w[FOLDED]
    d = cfg.head_dim
    for i, (mixer, mlp) in enumerate(cfg.layers):
        p = f"l{i}."
        for k in ("norm1", "norm2", "q_norm", "k_norm", "gnorm"):
            if p + k in w:
                out[p + k] = w[p + k]
        if mixer == "attn":
            h, hk = cfg.num_heads, cfg.num_kv_heads
            hl = h // world
            nkv, kv0 = kv_layout(h, hk, world, rank)
            q0 = rank * hl * d
            pieces = [(q0, q0 + hl * d)]
            off = h * d
            if cfg.attn_output_gate:
                pieces.append((off + q0, off + q0 + hl * d))
                off += h * d
            pieces += [(off + kv0 * d, off + (kv0 + nkv) * d), (off + hk * d + kv0 * d, off + hk * d + (kv0 + nkv) * d)]
            out[p + "qkv"] = _rows(w[p + "qkv"], pieces)
            out[p + "o_proj"] = _cols(w[p + "o_proj"], q0, q0 + hl * d)
        elif mixer == "gdn":
            kh, vh, kd, vd = cfg.gdn_k_heads, cfg.gdn_v_heads, cfg.gdn_k_dim, cfg.gdn_v_dim
            kl, vl = kh // world, vh // world
            key, val = kh * kd, vh * vd
            k0, v0 = rank * kl * kd, rank * vl * vd
            conv_pieces = [(k0, k0 + kl * kd), (key + k0, key + k0 + kl * kd), (2 * key + v0, 2 * key + v0 + vl * vd)]
            cd = 2 * key + val
            h0 = rank * vl
            out[p + "in_proj"] = _rows(w[p + "in_proj"], conv_pieces + [
                (cd + v0, cd + v0 + vl * vd), (cd + val + h0, cd + val + h0 + vl), (cd + val + vh + h0,
                                                                                      cd + val + vh + h0 + vl)])
            out[p + "conv"] = _rows(w[p + "conv"], conv_pieces)
            out[p + "A_log"] = w[p + "A_log"][h0:h0 + vl].contiguous()
            out[p + "dt_bias"] = w[p + "dt_bias"][h0:h0 + vl].contiguous()
            out[p + "out_proj"] = _cols(w[p + "out_proj"], v0, v0 + vl * vd)
        elif mixer == "mamba":
            nh, hp, g, n = cfg.mamba_heads, cfg.mamba_head_dim, cfg.mamba_groups, cfg.mamba_state
            inner = nh * hp
            hl, gl = nh // world, g // world
            x0, g0 = rank * hl * hp, rank * gl * n
            conv_pieces = [(x0, x0 + hl * hp), (inner + g0, inner + g0 + gl * n),
                           (inner + g * n + g0, inner + g * n + g0 + gl * n)]
            cd = inner + 2 * g * n
            out[p + "in_proj"] = _rows(w[p + "in_proj"], [(x0, x0 + hl * hp)] + [
                (inner + a, inner + b) for a, b in conv_pieces] + [(inner + cd + rank * hl, inner + cd + (rank + 1) * hl)])
            out[p + "conv"] = _rows(w[p + "conv"], conv_pieces)
            if p + "conv_bias" in w:
                out[p + "conv_bias"] = torch.cat([w[p + "conv_bias"][a:b] for a, b in conv_pieces]).contiguous()
            if w[p + "gnorm"].numel() == inner:  # one weight row per group: this rank's groups
                out[p + "gnorm"] = w[p + "gnorm"][x0:x0 + hl * hp].contiguous()
            for k in ("A_log", "dt_bias", "D"):
                out[p + k] = w[p + k][rank * hl:(rank + 1) * hl].contiguous()
            out[p + "out_proj"] = _cols(w[p + "out_proj"], x0, x0 + hl * hp)
        if mlp is not None:
            il = cfg.intermediate_size // world
            if mlp == "swiglu":
                out[p + "gate_up"] = w[p + "gate_up"][2 * rank * il:2 * (rank + 1) * il].contiguous()
            else:
                out[p + "up"] = w[p + "up"][rank * il:(rank + 1) * il].contiguous()
            out[p + "down"] = _cols(w[p + "down"], rank * il, (rank + 1) * il)
    return loc, out


def local_draft_config(cfg: DraftConfig, world: int, rank: int) -> DraftConfig:
    if world == 1:
        return cfg
    kv, _ = kv_layout(cfg.num_heads, cfg.num_kv_heads, world, rank)
    if cfg.moe:  # a latent-MoE MLP is replicated (its output needs no collective)
        return dataclasses.replace(cfg, num_heads=cfg.num_heads // world, num_kv_heads=kv)
    _check(cfg.intermediate_size % (world * MLP_BLOCK) == 0,
           f"draft intermediate size {cfg.intermediate_size} does not split over {world} ranks")
    return dataclasses.replace(cfg, num_heads=cfg.num_heads // world, num_kv_heads=kv,
                               intermediate_size=cfg.intermediate_size // world)


def shard_draft(cfg: DraftConfig, w: Dict[str, torch.Tensor], world: int, rank: int
                ) -> Tuple[DraftConfig, Dict[str, torch.Tensor]]:
    """The draft layer is sharded like a target attention + MLP layer; ``fc``, ``eh_proj``, norms, the head and a
    latent-MoE MLP are replicated."""
    if world == 1:
        return cfg, w
    loc = local_draft_config(cfg, world, rank)
    out = dict(w)
    d, h, hk = cfg.head_dim, cfg.num_heads, cfg.num_kv_heads
    hl = h // world
    nkv, kv0 = kv_layout(h, hk, world, rank)
    q0 = rank * hl * d
    off = h * d
    out["qkv"] = _rows(w["qkv"], [(q0, q0 + hl * d), (off + kv0 * d, off + (kv0 + nkv) * d),
                                  (off + hk * d + kv0 * d, off + hk * d + (kv0 + nkv) * d)])
    out["o_proj"] = _cols(w["o_proj"], q0, q0 + hl * d)
    if cfg.moe:
        return loc, out
    il = cfg.intermediate_size // world
    out["gate_up"] = w["gate_up"][2 * rank * il:2 * (rank + 1) * il].contiguous()
    out["down"] = _cols(w["down"], rank * il, (rank + 1) * il)
    return loc, out
