"""Plain PyTorch definitions of every op (the CPU path and the oracle the CUDA kernels are tested against).

Reductions run in float64 and round once to the output dtype, so a row's result does not depend on which other rows
share the call: plain decode (one row) and tree verify (many rows) give identical results on CPU, the property the
greedy-equality tests rely on. Shapes follow the CUDA ops in ``eagle4_b200/csrc``.
"""

from __future__ import annotations

import math
from typing import Optional, Tuple

import torch
import torch.nn.functional as F


# ----------------------------------------------------------------------------------------------- dense ops
def _matmul(x: torch.Tensor, w: torch.Tensor, fold_eps: Optional[float]) -> torch.Tensor:
    """``x @ w^T`` in float64; with ``fold_eps`` each row is scaled by ``rsqrt(mean(x_row^2) + fold_eps)`` (an RMSNorm
    of ``x`` folded into the product, ``w`` carrying the norm weight in its columns)."""
    xd = x.double()
    y = xd @ w.double().t()
    if fold_eps is not None:
        y = y * torch.rsqrt(xd.square().mean(-1, keepdim=True) + fold_eps)
    return y


def linear(x: torch.Tensor, w: torch.Tensor, fold_eps: Optional[float] = None) -> torch.Tensor:
    """``x [T, K] @ w[N, K]^T``."""
    return _matmul(x, w, fold_eps).to(x.dtype)


def linear_residual(x: torch.Tensor, w: torch.Tensor, residual: torch.Tensor) -> torch.Tensor:
    """``residual + x @ w^T`` rounded once."""
    return (residual.double() + x.double() @ w.double().t()).to(residual.dtype)


def linear_swiglu(x: torch.Tensor, w_gu: torch.Tensor, fold_eps: Optional[float] = None) -> torch.Tensor:
    """``silu(x @ g^T) * (x @ u^T)`` with ``w_gu`` holding gate and up rows interleaved in blocks of 64:
    rows ``[128i, 128i+64)`` are gate rows ``[64i, 64i+64)`` and rows ``[128i+64, 128i+128)`` the matching up rows."""
    y = _matmul(x, w_gu, fold_eps)
    t, n2 = y.shape
    y = y.view(t, n2 // 128, 2, 64)
    g, u = y[:, :, 0], y[:, :, 1]
    return (F.silu(g) * u).reshape(t, n2 // 2).to(x.dtype)


def linear_relu2(x: torch.Tensor, w: torch.Tensor, fold_eps: Optional[float] = None) -> torch.Tensor:
    y = _matmul(x, w, fold_eps)
    return torch.relu(y).square().to(x.dtype)


def fold_norm_weight(w: torch.Tensor, norm_w: torch.Tensor, offset: bool) -> torch.Tensor:
    """``w`` [N, K] with the RMSNorm weight (``1 + norm_w`` with ``offset``) multiplied into its columns."""
    # a bf16 x bf16 product is exact in float32; wider weights use float64 (either way one rounding to w's dtype)
    ct = torch.float32 if w.dtype in (torch.bfloat16, torch.float16) else torch.float64
    scale = norm_w.to(ct) + 1.0 if offset else norm_w.to(ct)
    return (w.to(ct) * scale[None, :]).to(w.dtype)


def interleave_gate_up(gate: torch.Tensor, up: torch.Tensor, block: int = 64) -> torch.Tensor:
    """Stack gate and up weights ``[F, H]`` as ``[2F, H]`` in the block-interleaved layout of ``linear_swiglu``."""
    f, h = gate.shape
    if f % block:
        raise ValueError(f"intermediate size {f} must be a multiple of {block}")
    return torch.stack([gate.view(f // block, block, h), up.view(f // block, block, h)], dim=1).reshape(2 * f, h)


def lm_head_argmax(x: torch.Tensor, w: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """Greedy token per row: ``(argmax ids int64 [T], max logit fp32 [T])``; ties go to the lower id."""
    logits = x.double() @ w.double().t()
    logits = logits.float()  # the GPU kernel compares fp32 logits
    m, idx = logits.max(dim=-1)
    return idx, m


def logits(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    return (x.double() @ w.double().t()).float()


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float, offset: bool) -> torch.Tensor:
    xd = x.double()
    r = torch.rsqrt(xd.square().mean(-1, keepdim=True) + eps)
    scale = w.double() + 1.0 if offset else w.double()
    return (xd * r * scale).to(x.dtype)


def add_rmsnorm(x: torch.Tensor, residual: torch.Tensor, w: torch.Tensor, eps: float,
                offset: bool) -> Tuple[torch.Tensor, torch.Tensor]:
    """``h = x + residual`` (rounded to the dtype), returns ``(rmsnorm(h), h)``."""
    h = (x.double() + residual.double()).to(x.dtype)
    return rmsnorm(h, w, eps, offset), h


def embedding(ids: torch.Tensor, table: torch.Tensor) -> torch.Tensor:
    return table.index_select(0, ids.long())


# ----------------------------------------------------------------------------------------------- attention
def rope(x: torch.Tensor, pos: torch.Tensor, rotary_dim: int, theta: float) -> torch.Tensor:
    """NeoX-style rotary embedding on the first ``rotary_dim`` dims of ``x [T, H, D]``."""
    if rotary_dim == 0:
        return x
    half = rotary_dim // 2
    inv = 1.0 / (theta ** (torch.arange(0, half, dtype=torch.float64) / half))
    ang = pos.double()[:, None] * inv[None, :]
    cos, sin = ang.cos()[:, None, :], ang.sin()[:, None, :]
    xd = x.double()
    a, b = xd[..., :half], xd[..., half:rotary_dim]
    out = xd.clone()
    out[..., :half] = a * cos - b * sin
    out[..., half:rotary_dim] = b * cos + a * sin
    return out.to(x.dtype)


def slots_of(block_table: torch.Tensor, req: torch.Tensor, positions: torch.Tensor, page: int) -> torch.Tensor:
    return block_table[req.long(), positions.long() // page].long() * page + positions.long() % page


def qkv_prepare(qkv: torch.Tensor, cfg, pos: torch.Tensor, write_slot: torch.Tensor, k_cache: torch.Tensor,
                v_cache: torch.Tensor, q_norm: Optional[torch.Tensor], k_norm: Optional[torch.Tensor]
                ) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
    """Split the fused projection, apply q/k norms and RoPE, write K/V at ``write_slot``; return ``(q, gate)``.

    Fused projection layout per row: ``[q (H*D) | gate (H*D) if gated | k (Hkv*D) | v (Hkv*D)]``.
    """
    t = qkv.shape[0]
    h, hk, d = cfg.num_heads, cfg.num_kv_heads, cfg.head_dim
    o = 0
    q = qkv[:, o: o + h * d].reshape(t, h, d); o += h * d
    gate = None
    if cfg.attn_output_gate:
        gate = qkv[:, o: o + h * d]; o += h * d
    k = qkv[:, o: o + hk * d].reshape(t, hk, d); o += hk * d
    v = qkv[:, o: o + hk * d].reshape(t, hk, d)
    if q_norm is not None:
        q = rmsnorm(q, q_norm, cfg.rms_norm_eps, cfg.norm_offset)
        k = rmsnorm(k, k_norm, cfg.rms_norm_eps, cfg.norm_offset)
    q = rope(q, pos, cfg.rotary_dim, cfg.rope_theta)
    k = rope(k, pos, cfg.rotary_dim, cfg.rope_theta)
    k_cache[write_slot.long()] = k.to(k_cache.dtype)
    v_cache[write_slot.long()] = v.to(v_cache.dtype)
    return q.contiguous(), gate


def attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, block_table: torch.Tensor, page: int,
              req: torch.Tensor, ctx_start: torch.Tensor, ctx_len: torch.Tensor, extra: torch.Tensor,
              n_extra: torch.Tensor, scale: float) -> torch.Tensor:
    """Each row attends to context positions ``[ctx_start, ctx_len)`` of its request (through the block table) and
    then to its ``n_extra`` extra physical slots (tree ancestors and itself), in that logical order.

    ``q [T, Hq, D]``, caches ``[slots, Hkv, D]``; returns ``[T, Hq, D]`` in q's dtype.
    """
    t, hq, d = q.shape
    hk = k_cache.shape[1]
    grp = hq // hk
    out = torch.empty_like(q)
    for r in range(t):
        b = int(req[r])
        s0, s1 = int(ctx_start[r]), int(ctx_len[r])
        pos = torch.arange(s0, s1)
        slots = [slots_of(block_table, torch.full_like(pos, b), pos, page)] if s1 > s0 else []
        ne = int(n_extra[r])
        if ne:
            slots.append(extra[r, :ne].long())
        sl = torch.cat(slots) if slots else torch.zeros(0, dtype=torch.long)
        kk = k_cache[sl].double()  # [S, Hkv, D]
        vv = v_cache[sl].double()
        qq = q[r].double().view(hk, grp, d)
        s = torch.einsum("hgd,shd->hgs", qq, kk) * scale
        p = torch.softmax(s, dim=-1)
        o = torch.einsum("hgs,shd->hgd", p, vv)
        out[r] = o.reshape(hq, d).to(q.dtype)
    return out


# ----------------------------------------------------------------------------------------------- GDN
def _walk(parent: torch.Tensor, r: int, limit: int):
    """Rows on the path from the committed state to ``r`` (ancestors first), at most ``limit`` rows."""
    path = []
    cur = r
    while cur >= 0 and len(path) < limit:
        path.append(cur)
        cur = int(parent[cur])
    return path[::-1]


def causal_conv_tree(x: torch.Tensor, conv_state: torch.Tensor, state_slot: torch.Tensor, parent: torch.Tensor,
                     weight: torch.Tensor, bias: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Width-``K`` causal depthwise conv (plus ``bias [C]`` when given) + SiLU over a forest of rows.

    ``x [T, C]`` pre-conv inputs; ``conv_state [slots, C, K-1]`` the committed last inputs (oldest first);
    ``parent [T]`` the parent row of each row (``-1``: the committed state); ``weight [C, K]``.
    """
    t, c = x.shape
    kw = weight.shape[1]
    out = torch.empty_like(x)
    wd = weight.double()
    for r in range(t):
        path = _walk(parent, r, kw)
        win = [x[j].double() for j in path]
        need = kw - len(win)
        if need > 0:
            st = conv_state[int(state_slot[r])].double()  # [C, K-1]
            win = [st[:, kw - 1 - need + i] for i in range(need)] + win
        acc = torch.zeros(c, dtype=torch.float64) if bias is None else bias.double().clone()
        for j in range(kw):
            acc = acc + wd[:, j] * win[j]
        out[r] = F.silu(acc).to(x.dtype)
    return out


def l2norm(x: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    return x * torch.rsqrt((x * x).sum(-1, keepdim=True) + eps)


def gdn_gates(a: torch.Tensor, b: torch.Tensor, a_log: torch.Tensor, dt_bias: torch.Tensor
              ) -> Tuple[torch.Tensor, torch.Tensor]:
    """``g = -exp(A_log) * softplus(a + dt_bias)`` and ``beta = sigmoid(b)`` in fp32 ``[T, HV]``."""
    g = -a_log.float().exp() * F.softplus(a.float() + dt_bias.float())
    beta = torch.sigmoid(b.float())
    return g, beta


def _gdn_step(s: torch.Tensor, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, g: torch.Tensor,
              beta: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """One gated-delta-rule step on state ``s [HV, V, K]`` (fp64 math, state rounded to fp32 afterwards)."""
    s = s * torch.exp(g)[:, None, None]
    kv = (s * k[:, None, :]).sum(-1)  # [HV, V]
    delta = (v - kv) * beta[:, None]
    s = s + delta[:, :, None] * k[:, None, :]
    o = (s * q[:, None, :]).sum(-1)
    return s.float().double(), o


def _gdn_inputs(qkv: torch.Tensor, cfg) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    t = qkv.shape[0]
    kd, vd = cfg.gdn_key_dim, cfg.gdn_value_dim
    q = qkv[:, :kd].double().view(t, cfg.gdn_k_heads, cfg.gdn_k_dim)
    k = qkv[:, kd: 2 * kd].double().view(t, cfg.gdn_k_heads, cfg.gdn_k_dim)
    v = qkv[:, 2 * kd: 2 * kd + vd].double().view(t, cfg.gdn_v_heads, cfg.gdn_v_dim)
    rep = cfg.gdn_v_heads // cfg.gdn_k_heads
    q = l2norm(q).repeat_interleave(rep, dim=1) * (cfg.gdn_k_dim ** -0.5)
    k = l2norm(k).repeat_interleave(rep, dim=1)
    return q, k, v


def gdn_tree(qkv: torch.Tensor, g: torch.Tensor, beta: torch.Tensor, state: torch.Tensor,
             state_slot: torch.Tensor, parent: torch.Tensor, cfg, scan: bool) -> torch.Tensor:
    """Gated delta rule over a forest of rows; returns ``o [T, HV, V]`` in qkv's dtype.

    Tree mode (``scan=False``): each row replays its path from the committed state; the state is not written.
    Scan mode (prefill chains): rows of a request are processed in order and the state is updated in place.
    ``state [slots, HV, V, K]`` fp32.
    """
    t = qkv.shape[0]
    q, k, v = _gdn_inputs(qkv, cfg)
    gd, bd = g.double(), beta.double()
    out = torch.empty(t, cfg.gdn_v_heads, cfg.gdn_v_dim, dtype=qkv.dtype)
    if scan:
        for r in range(t):
            slot = int(state_slot[r])
            s, o = _gdn_step(state[slot].double(), q[r], k[r], v[r], gd[r], bd[r])
            state[slot] = s.float()
            out[r] = o.to(qkv.dtype)
        return out
    for r in range(t):
        s = state[int(state_slot[r])].double()
        o = None
        for j in _walk(parent, r, 1 << 30):
            s, o = _gdn_step(s, q[j], k[j], v[j], gd[j], bd[j])
        out[r] = o.to(qkv.dtype)
    return out


def gdn_commit(qkv: torch.Tensor, g: torch.Tensor, beta: torch.Tensor, x_pre: torch.Tensor, state: torch.Tensor,
               conv_state: torch.Tensor, slots: torch.Tensor, rows: torch.Tensor, n_rows: torch.Tensor, cfg) -> None:
    """Apply the accepted rows ``rows[b, :n_rows[b]]`` of each request to its committed state and conv window."""
    q, k, v = _gdn_inputs(qkv, cfg)
    gd, bd = g.double(), beta.double()
    kw = cfg.conv_kernel
    for b in range(rows.shape[0]):
        n = int(n_rows[b])
        if n == 0:
            continue
        slot = int(slots[b])
        s = state[slot].double()
        for j in rows[b, :n].tolist():
            s, _ = _gdn_step(s, q[j], k[j], v[j], gd[j], bd[j])
        state[slot] = s.float()
        _shift_conv(conv_state, slot, x_pre, rows[b, :n], kw)


def _shift_conv(conv_state: torch.Tensor, slot: int, x_pre: torch.Tensor, rows: torch.Tensor, kw: int) -> None:
    hist = [conv_state[slot, :, i] for i in range(kw - 1)] + [x_pre[j].to(conv_state.dtype) for j in rows.tolist()]
    hist = hist[-(kw - 1):]
    conv_state[slot] = torch.stack(hist, dim=-1)


def conv_commit_scan(conv_state: torch.Tensor, x_pre: torch.Tensor, state_slot: torch.Tensor, kw: int) -> None:
    """After a scan (prefill) the conv window of each request is its last ``K-1`` inputs."""
    for slot in torch.unique(state_slot).tolist():
        rows = (state_slot == slot).nonzero().flatten()
        _shift_conv(conv_state, slot, x_pre, rows, kw)


def gated_rmsnorm(o: torch.Tensor, z: torch.Tensor, w: torch.Tensor, eps: float, gate_first: bool = False
                  ) -> torch.Tensor:
    """Per-head RMSNorm of ``o [T, H, D]`` times ``silu(z)`` (``gate_first``: the RMSNorm of ``o * silu(z)``); returns
    ``[T, H*D]``. ``w``: one ``[D]`` weight shared by the heads, or ``H * D`` values (one row per head)."""
    od = o.double()
    gz = F.silu(z.double().reshape(od.shape))
    if gate_first:
        od = od * gz
    r = torch.rsqrt(od.square().mean(-1, keepdim=True) + eps)
    n = od * r * w.double().reshape(-1, o.shape[-1])
    return (n if gate_first else n * gz).reshape(o.shape[0], -1).to(o.dtype)


# ----------------------------------------------------------------------------------------------- Mamba2
def mamba_inputs(xbc: torch.Tensor, dt_raw: torch.Tensor, cfg, a_log: torch.Tensor, dt_bias: torch.Tensor):
    t = xbc.shape[0]
    hd, ns, ng = cfg.mamba_head_dim, cfg.mamba_state, cfg.mamba_groups
    x = xbc[:, : cfg.mamba_inner].double().view(t, cfg.mamba_heads, hd)
    bmat = xbc[:, cfg.mamba_inner: cfg.mamba_inner + ng * ns].double().view(t, ng, ns)
    cmat = xbc[:, cfg.mamba_inner + ng * ns:].double().view(t, ng, ns)
    rep = cfg.mamba_heads // ng
    bmat = bmat.repeat_interleave(rep, dim=1)
    cmat = cmat.repeat_interleave(rep, dim=1)
    dt = F.softplus(dt_raw.double() + dt_bias.double())  # [T, H]
    a = -a_log.double().exp()
    return x, bmat, cmat, dt, a


def _ssu_step(s, x, bm, cm, dt, a, d):
    da = torch.exp(dt * a)  # [H]
    s = s * da[:, None, None] + (dt[:, None] * x)[:, :, None] * bm[:, None, :]
    s = s.float().double()
    y = (s * cm[:, None, :]).sum(-1) + d[:, None] * x
    return s, y


def mamba_tree(xbc: torch.Tensor, dt_raw: torch.Tensor, a_log, dt_bias, d_skip, state, state_slot, parent, cfg,
               scan: bool) -> torch.Tensor:
    """Mamba2 selective-state update over a forest of rows: ``state [slots, H, P, N]`` fp32; returns ``y [T, H, P]``."""
    t = xbc.shape[0]
    x, bm, cm, dt, a = mamba_inputs(xbc, dt_raw, cfg, a_log, dt_bias)
    d = d_skip.double()
    out = torch.empty(t, cfg.mamba_heads, cfg.mamba_head_dim, dtype=xbc.dtype)
    if scan:
        for r in range(t):
            slot = int(state_slot[r])
            s, y = _ssu_step(state[slot].double(), x[r], bm[r], cm[r], dt[r], a, d)
            state[slot] = s.float()
            out[r] = y.to(xbc.dtype)
        return out
    for r in range(t):
        s = state[int(state_slot[r])].double()
        y = None
        for j in _walk(parent, r, 1 << 30):
            s, y = _ssu_step(s, x[j], bm[j], cm[j], dt[j], a, d)
        out[r] = y.to(xbc.dtype)
    return out


def mamba_commit(xbc, dt_raw, a_log, dt_bias, d_skip, x_pre, state, conv_state, slots, rows, n_rows, cfg) -> None:
    x, bm, cm, dt, a = mamba_inputs(xbc, dt_raw, cfg, a_log, dt_bias)
    d = d_skip.double()
    for b in range(rows.shape[0]):
        n = int(n_rows[b])
        if n == 0:
            continue
        slot = int(slots[b])
        s = state[slot].double()
        for j in rows[b, :n].tolist():
            s, _ = _ssu_step(s, x[j], bm[j], cm[j], dt[j], a, d)
        state[slot] = s.float()
        _shift_conv(conv_state, slot, x_pre, rows[b, :n], cfg.conv_kernel)


# ----------------------------------------------------------------------------------------------- KV commit
def kv_commit(k_caches, v_caches, src_slots: torch.Tensor, dst_slots: torch.Tensor) -> None:
    """Move accepted tree rows' K/V to their chain positions in every attention layer (in list order)."""
    src, dst = src_slots.long(), dst_slots.long()
    keep = src != dst
    src, dst = src[keep], dst[keep]
    for kc, vc in zip(k_caches, v_caches):
        for s, t in zip(src.tolist(), dst.tolist()):
            kc[t] = kc[s]
            vc[t] = vc[s]


# ----------------------------------------------------------------------------------------------- candidates
def topk_rows(scores: torch.Tensor, k: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """Top-``k`` per row, best first, ties to the lower index (values fp32, indices int64)."""
    order = torch.sort(scores.float(), dim=-1, descending=True, stable=True)
    return order.values[:, :k], order.indices[:, :k]


def gather_dot(h: torch.Tensor, w: torch.Tensor, idx: torch.Tensor) -> torch.Tensor:
    """``logit[r, c] = w[idx[r, c]] . h[r]`` in fp32."""
    return torch.einsum("rcd,rd->rc", w[idx.long()].double(), h.double()).float()


def softmax_topk(logit: torch.Tensor, ids: torch.Tensor, k: int, temperature: float = 1.0
                 ) -> Tuple[torch.Tensor, torch.Tensor]:
    """Softmax over each row's candidates then the top ``k`` (probabilities fp32, token ids int64)."""
    p = torch.softmax(logit.double() / temperature, dim=-1).float()
    v, i = topk_rows(p, k)
    return v, torch.gather(ids.long(), 1, i)


# ----------------------------------------------------------------------------------------------- accept
def accept_greedy(target_ids: torch.Tensor, tokens: torch.Tensor, parent_rows: torch.Tensor, n_rows: torch.Tensor
                  ) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Greedy walk of each request's verify rows.

    ``target_ids [bs, N]`` the target's argmax per row, ``tokens [bs, N]`` row tokens (row 0 the root),
    ``parent_rows [bs, N]`` (row 0: -1). Returns ``(accepted rows [bs, N] (row 0 first, -1 padded),
    accepted count [bs] (root included), bonus token [bs])``.
    """
    bs, n = tokens.shape
    acc = torch.full((bs, n), -1, dtype=torch.int32)
    cnt = torch.zeros(bs, dtype=torch.int32)
    bonus = torch.zeros(bs, dtype=torch.int64)
    for b in range(bs):
        nr = int(n_rows[b])
        cur = 0
        acc[b, 0] = 0
        c = 1
        while True:
            want = int(target_ids[b, cur])
            nxt = -1
            for r in range(1, nr):
                if int(parent_rows[b, r]) == cur and int(tokens[b, r]) == want:
                    nxt = r
                    break
            if nxt < 0:
                bonus[b] = want
                break
            acc[b, c] = nxt
            c += 1
            cur = nxt
        cnt[b] = c
    return acc, cnt, bonus


# ----------------------------------------------------------------------------------------------- small fused ops
def sigmoid_gate(o: torch.Tensor, gate: torch.Tensor) -> torch.Tensor:
    return (o.double() * torch.sigmoid(gate.double())).to(o.dtype)


def concat_norms(e: torch.Tensor, h: torch.Tensor, we: torch.Tensor, wh: torch.Tensor, eps: float) -> torch.Tensor:
    """``cat(rmsnorm(e, we), rmsnorm(h, wh))`` (the draft layer's ``2H`` input)."""
    return torch.cat([rmsnorm(e, we, eps, False), rmsnorm(h, wh, eps, False)], dim=-1)


def candidate_logits(h: torch.Tensor, down: torch.Tensor, scores_w: torch.Tensor, lm_head: torch.Tensor,
                     num_candidates: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """Low-rank shortlist then exact logits: ``(ids int64 [T, C], fp32 logits [T, C])``."""
    lr = linear(h, down)
    s = (lr.double() @ scores_w.double().t()).float()
    _, idx = topk_rows(s, num_candidates)
    return idx, gather_dot(h, lm_head, idx)


def candidate_head(h, down, scores_w, lm_head, num_candidates: int, k: int):
    idx, lg = candidate_logits(h, down, scores_w, lm_head, num_candidates)
    return softmax_topk(lg, idx, k)


def full_head_topk(h: torch.Tensor, lm_head: torch.Tensor, k: int):
    lg = logits(h, lm_head)
    ids = torch.arange(lg.shape[1]).expand_as(lg)
    return softmax_topk(lg, ids, k)


# ----------------------------------------------------------------------------------------------- fused GDN mixer
def gdn_offsets(cfg):
    """Column offsets of z, b and a in the fused GDN in_proj output ``[qkv | z | b | a]``."""
    cd, vd, hv = cfg.gdn_conv_dim, cfg.gdn_value_dim, cfg.gdn_v_heads
    return cd, cd + vd, cd + vd + hv


def gdn_mixer(conv, proj, cfg, a_log, dt_bias, norm_w, state, state_slot, parent, scan: bool):
    """Gates from the raw projection, the gated delta rule over the row forest, then the per-head gated RMSNorm:
    ``[T, HV*V]``."""
    z_off, b_off, a_off = gdn_offsets(cfg)
    hv = cfg.gdn_v_heads
    g, beta = gdn_gates(proj[:, a_off: a_off + hv], proj[:, b_off: b_off + hv], a_log, dt_bias)
    o = gdn_tree(conv, g, beta, state, state_slot, parent, cfg, scan)
    return gated_rmsnorm(o, proj[:, z_off: z_off + cfg.gdn_value_dim], norm_w, cfg.rms_norm_eps)


def gdn_commit_all(convs, projs, states, conv_states, a_logs, dt_biases, slots, rows, n_rows, cfg) -> None:
    z_off, b_off, a_off = gdn_offsets(cfg)
    hv = cfg.gdn_v_heads
    for conv, proj, st, cs, al, dtb in zip(convs, projs, states, conv_states, a_logs, dt_biases):
        g, beta = gdn_gates(proj[:, a_off: a_off + hv], proj[:, b_off: b_off + hv], al, dtb)
        gdn_commit(conv, g, beta, proj[:, : cfg.gdn_conv_dim], st, cs, slots, rows, n_rows, cfg)


# latent MoE (EAGLE-4 Nemotron-class drafts) --------------------------------------------------------------------
def moe_route(x: torch.Tensor, gate: torch.Tensor, bias: torch.Tensor, top_k: int, n_group: int = 1,
              topk_group: int = 1, norm_topk_prob: bool = True) -> Tuple[torch.Tensor, torch.Tensor]:
    """Sigmoid router over bias-corrected scores, in fp32: experts are chosen by ``sigmoid(x gate^T) + bias`` (with
    ``n_group`` > 1 only inside the ``topk_group`` groups whose two best biased scores sum highest), weighted by their
    unbiased scores, renormalised over the chosen when ``norm_topk_prob``. Returns (chosen [T, k] int64, best first;
    weights [T, k] fp32)."""
    scores = torch.sigmoid(x.float() @ gate.float().t())
    biased = scores + bias.float()
    if n_group > 1:
        T, E = biased.shape
        per = E // n_group
        group_score = biased.view(T, n_group, per).topk(min(2, per), dim=-1).values.sum(-1)
        keep = torch.zeros(T, n_group, dtype=torch.bool, device=x.device)
        keep.scatter_(1, group_score.topk(topk_group, dim=-1).indices, True)
        biased = biased.masked_fill(~keep.repeat_interleave(per, dim=1), float("-inf"))
    chosen = biased.topk(top_k, dim=-1).indices
    w = scores.gather(1, chosen)
    if norm_topk_prob:
        w = w / w.sum(-1, keepdim=True)
    return chosen, w


def moe_experts(latent: torch.Tensor, chosen: torch.Tensor, weights: torch.Tensor, up: torch.Tensor,
                down: torch.Tensor) -> torch.Tensor:
    """``sum_j weights[t, j] down_e (relu(up_e latent_t)^2)`` over each token's chosen experts e (j in routing order);
    the ReLU^2 activations are rounded to the latent's dtype, as the kernel stores them."""
    lat = latent.float()
    out = torch.zeros(latent.shape[0], latent.shape[1], dtype=torch.float32, device=latent.device)
    for j in range(chosen.shape[1]):
        e = chosen[:, j].long()
        h = torch.relu(torch.einsum("tfl,tl->tf", up[e].float(), lat)) ** 2
        h = h.to(latent.dtype).float()
        out = out + weights[:, j:j + 1].float() * torch.einsum("tlf,tf->tl", down[e].float(), h)
    return out.to(latent.dtype)
