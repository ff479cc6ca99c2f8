"""GDN and Mamba2 layers of a vLLM hybrid target under tree verify, on this package's tree kernels.

vLLM (Model Runner V2 builds with the linear-attention verify hook) hands each GDN layer's speculative rows
(``GDNSpecRows``) and each Mamba2 layer's (``Mamba2SpecRows``) to the method's ``LinearAttnVerifyExtension`` in place
of its own conv and recurrence kernels. vLLM's own verify is a chain with one state slot per verify row: the
recurrent state a step resumes from is ``ssm_state[state_indices[b, num_accepted - 1]]`` and the conv window is the
``K - 1`` columns of ``conv_state[state_indices[b, 0]]`` starting at column ``num_accepted - 1``.

A tree keeps those two reading rules and nothing else of the chain kernels:

* ``forward_*``: each request's committed state and window are gathered once into contiguous buffers; the tree conv
  (each row's window is its ancestors' inputs, the committed window below the root) and the tree recurrence (each
  row from its parent's state, nothing stored) run over the row forest staged by the speculator
  (:func:`stage_tree`: the verify rows' parents, a prefix of the staged tree where vLLM verifies fewer rows);
* ``commit`` (from the speculator's ``post_accept``, :func:`commit_accepted`): the accepted path of every layer is
  replayed from the gathered state (one launch for all GDN layers) and written where vLLM resumes: the state into
  ``state_indices[b, accepted - 1]``, the last ``K - 1`` conv inputs into the window at column ``accepted - 1``.

Nothing is written during verify, so a round costs the tree passes plus one state write per request and layer,
against one state per verify row for vLLM's chain kernels. The speculative output stays the plain greedy output
because every row's state is the result of the same steps as plain decoding.

Reference counterparts: ``eagle_harness/vllm/gdn_tree_verify.py:55,151,176,251`` (``TreeVerify``,
``check_tree_verifiable``, ``create_extension``, ``LinearStateCommit``) and ``eagle_harness/vllm/round_commit.py``
(the accepted rows in chain order); the hook and field names are vLLM's.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, List, Optional, Sequence

import torch

from eagle4_b200 import ops
from eagle4_b200.plugins.common import GdnShape, host_base
from eagle4_b200.plugins.vllm.hooks import VERIFY_EXTENSION_MODULES

_Extension = host_base(" | ".join(f"{m}:LinearAttnVerifyExtension" for m in VERIFY_EXTENSION_MODULES))

NULL_BLOCK_ID = 0  # vLLM's padded-request state slot
TREE_LAYERS = ("QwenGatedDeltaNetAttention", "MambaMixer2")  # the vLLM layers that hand over their rows


@dataclass
class MambaShape:
    mamba_heads: int
    mamba_head_dim: int
    mamba_state: int
    mamba_groups: int
    conv_kernel: int = 4

    @property
    def mamba_inner(self) -> int:
        return self.mamba_heads * self.mamba_head_dim


@dataclass
class _Record:
    """What one layer's commit needs from its verify forward."""

    kind: str  # "gdn" | "mamba2"
    shape: Any
    x_pre: torch.Tensor        # [T, C] conv inputs
    conv: torch.Tensor         # [T, C] conv outputs
    gate_a: torch.Tensor       # GDN: a [T, HV]; Mamba2: raw dt [T, H]
    gate_b: Optional[torch.Tensor]
    a_log: torch.Tensor
    dt_bias: torch.Tensor
    d_skip: Optional[torch.Tensor]
    state: torch.Tensor        # [bs, ...] gathered committed states (replayed in place at commit)
    window: torch.Tensor       # [bs, C, K - 1] gathered committed windows
    ssm_state: torch.Tensor    # vLLM's state pool of the layer
    conv_state: torch.Tensor   # vLLM's conv pool of the layer
    state_indices: torch.Tensor
    query_start_loc: torch.Tensor


@dataclass
class VerifyStage:
    """The round's tree (local parents per request, ``-1`` for the root) and the layers' records."""

    parents: Optional[torch.Tensor] = None  # [bs, w] int32
    records: List[_Record] = field(default_factory=list)


_STAGE = VerifyStage()


def stage_tree(parent_rows: Optional[torch.Tensor]) -> None:
    """Before the verify forward: the verify rows' parents (``[bs, w]`` local, ``-1`` at the root; None: chains)."""
    _STAGE.parents = None if parent_rows is None else parent_rows.int()
    _STAGE.records.clear()


def _rows(query_start_loc: torch.Tensor, tokens: int, device) -> tuple:
    """(request of every token, global parent row of every token) from the staged tree (chains when unstaged)."""
    qsl = query_start_loc.long().to(device)
    t = torch.arange(tokens, device=device)
    req = torch.bucketize(t, qsl[1:], right=True)
    local = t - qsl[:-1][req]
    if _STAGE.parents is None:
        lp = local - 1
    else:
        staged = _STAGE.parents.to(device).long()
        if int((qsl[1:] - qsl[:-1]).max()) > staged.shape[1]:
            raise RuntimeError("a request verifies more rows than the staged tree has")
        lp = staged[req, local]
    parent = torch.where(lp >= 0, lp + qsl[:-1][req], lp)
    return req.int(), parent.int()


def _window_view(conv_state: torch.Tensor, slots: torch.Tensor, start: torch.Tensor, width: int, channels: int):
    """Index tensors of the ``width`` window columns per request, for either conv layout (``[slots, C, L]``, channel
    first, or ``[slots, L, C]``)."""
    cols = start.long()[:, None] + torch.arange(width, device=start.device)[None, :]  # [bs, W]
    dim_first = conv_state.shape[1] == channels
    return cols, dim_first


def _gather_window(conv_state, slots, start, width, channels) -> torch.Tensor:
    cols, dim_first = _window_view(conv_state, slots, start, width, channels)
    s = slots.long()[:, None]
    win = conv_state[s, :, cols] if dim_first else conv_state[s, cols, :]  # [bs, W, C]
    return win.permute(0, 2, 1).contiguous()  # [bs, C, W]


def _scatter_window(conv_state, slots, start, window, channels) -> None:
    cols, dim_first = _window_view(conv_state, slots, start, window.shape[2], channels)
    s = slots.long()[:, None]
    vals = window.permute(0, 2, 1).to(conv_state.dtype)  # [bs, W, C]
    if dim_first:
        conv_state[s, :, cols] = vals
    else:
        conv_state[s, cols, :] = vals


def _bias(rows, x: torch.Tensor) -> Optional[torch.Tensor]:
    """The layer's conv bias (Nemotron-H's Mamba2 has one) in the inputs' dtype, or None."""
    b = getattr(rows, "conv_bias", None)
    return None if b is None else b.to(x.dtype).contiguous()


class TreeVerify(_Extension):
    """The method's ``LinearAttnVerifyExtension``: tree conv + tree recurrence for GDN and Mamba2 spec rows."""

    def __init__(self, vllm_config: Any = None):
        self.vllm_config = vllm_config

    def _committed(self, rows, channels: int, kw: int):
        bs = rows.state_indices.shape[0]
        last = (rows.num_accepted_tokens[:bs].long() - 1).clamp(min=0)  # padded requests: column 0, ignored
        src = rows.state_indices.gather(1, last[:, None]).flatten()
        window = _gather_window(rows.conv_state, rows.state_indices[:, 0], last, kw - 1, channels)
        state = rows.ssm_state[src.long()].float().contiguous()
        return state, window

    def forward_spec_rows(self, rows) -> None:
        """A GDN layer's rows: writes ``rows.out`` ``[T, HV * V]``."""
        x = rows.mixed_qkv
        tokens, channels = x.shape
        shape = GdnShape(rows.num_k_heads, rows.num_v_heads, rows.head_k_dim, rows.head_v_dim,
                         int(rows.conv_weight.shape[-1]))
        weight = rows.conv_weight.reshape(channels, -1)
        state, window = self._committed(rows, channels, shape.conv_kernel)
        req, parent = _rows(rows.query_start_loc, tokens, x.device)
        conv = ops.causal_conv_tree(x, window, req, parent, weight, _bias(rows, x))
        out = ops.gdn_recurrence(conv, rows.a, rows.b, rows.A_log, rows.dt_bias, state, req, parent, shape)
        rows.out.view(tokens, -1).copy_(out.view(tokens, -1))
        _STAGE.records.append(_Record("gdn", shape, x.clone(), conv, rows.a.clone(), rows.b.clone(), rows.A_log,
                                      rows.dt_bias, None, state, window, rows.ssm_state, rows.conv_state,
                                      rows.state_indices.clone(), rows.query_start_loc.clone()))

    def forward_mamba2_spec_rows(self, rows) -> None:
        """A Mamba2 layer's rows: writes ``rows.out`` ``[T, H * P]`` (the SSM output with the D skip; vLLM gates and
        normalises it afterwards)."""
        x = rows.hidden_states_B_C
        tokens, channels = x.shape
        shape = MambaShape(rows.num_heads, rows.head_dim, rows.ssm_state_size, rows.n_groups,
                           int(rows.conv_weight.shape[-1]))
        weight = rows.conv_weight.reshape(channels, -1)
        state, window = self._committed(rows, channels, shape.conv_kernel)
        req, parent = _rows(rows.query_start_loc, tokens, x.device)
        conv = ops.causal_conv_tree(x, window, req, parent, weight, _bias(rows, x))
        a_log = torch.log(-rows.A.float())  # vLLM passes A = -exp(A_log)
        dt = rows.dt.reshape(tokens, -1)
        y = ops.mamba_tree(conv, dt, a_log, rows.dt_bias.float(), rows.D.float(), state, req, parent, shape, False)
        rows.out.view(tokens, -1).copy_(y.reshape(tokens, -1))
        _STAGE.records.append(_Record("mamba2", shape, x.clone(), conv, dt.clone(), None, a_log,
                                      rows.dt_bias.float(), rows.D.float(), state, window, rows.ssm_state,
                                      rows.conv_state, rows.state_indices.clone(), rows.query_start_loc.clone()))


def commit_accepted(accepted: torch.Tensor, counts: torch.Tensor) -> int:
    """After the accept: ``accepted [bs, w]`` local verify rows of each request's path (root first, ``-1`` padding),
    ``counts [bs]`` their number. Replays the path of every recorded layer and writes the state and the window where
    vLLM resumes. Returns the number of layers committed."""
    recs = _STAGE.records
    if not recs:
        return 0
    dev = recs[0].x_pre.device
    cnt = counts.to(dev).long()
    bs = cnt.shape[0]
    qsl = recs[0].query_start_loc.to(dev).long()
    path = accepted.to(dev).long()[:, : max(1, int(cnt.max()))]
    rows = torch.where(path >= 0, path + qsl[:bs, None], torch.zeros_like(path)).int()
    slots = torch.arange(bs, dtype=torch.int32, device=dev)
    gdn = [r for r in recs if r.kind == "gdn"]
    if gdn:
        shape = gdn[0].shape
        projs = []
        for r in gdn:  # the commit reads pre-conv inputs and the raw gates from one projection-shaped row
            cd, vd, hv = shape.gdn_conv_dim, shape.gdn_value_dim, shape.gdn_v_heads
            proj = torch.zeros(r.x_pre.shape[0], cd + vd + 2 * hv, dtype=r.x_pre.dtype, device=dev)
            proj[:, :cd] = r.x_pre
            proj[:, cd + vd: cd + vd + hv] = r.gate_b
            proj[:, cd + vd + hv:] = r.gate_a
            projs.append(proj)
        ops.gdn_commit_all([r.conv for r in gdn], projs, [r.state for r in gdn], [r.window for r in gdn],
                           [r.a_log for r in gdn], [r.dt_bias for r in gdn], slots, rows, cnt.int(), shape)
    for r in recs:
        if r.kind == "mamba2":
            ops.mamba_commit(r.conv, r.gate_a, r.a_log, r.dt_bias, r.d_skip, r.x_pre, r.state, r.window, slots, rows,
                             cnt.int(), r.shape)
    live = (r.state_indices[:bs, 0] != NULL_BLOCK_ID) & (cnt > 0)
    keep = live.nonzero().flatten()
    for r in recs:
        if keep.numel() == 0:
            break
        si = r.state_indices[keep]
        dst = si.gather(1, (cnt[keep] - 1)[:, None]).flatten().long()
        r.ssm_state[dst] = r.state[keep].to(r.ssm_state.dtype)
        _scatter_window(r.conv_state, si[:, 0], cnt[keep] - 1, r.window[keep], r.x_pre.shape[1])
    n = len(recs)
    recs.clear()
    return n


def check_tree_verifiable(layers: Sequence[Any]) -> None:
    """Refuse a target with linear-attention layers that do not hand their rows to the extension (their own kernels
    would verify every tree as a chain)."""
    unhandled = sorted({type(layer).__name__ for layer in layers if type(layer).__name__ not in TREE_LAYERS})
    if unhandled:
        raise RuntimeError(f"eagle4_b200: tree verify cannot run on {', '.join(unhandled)} layers; only "
                           f"{', '.join(TREE_LAYERS)} hand their rows to the verify extension")


def create_extension(vllm_config: Any) -> Optional[TreeVerify]:
    """The method's extension factory: chains (``node_top_k`` 1) keep vLLM's own verify kernels."""
    from eagle4_b200.plugins.vllm.config import parse_method_config

    spec = getattr(vllm_config, "speculative_config", None)
    if parse_method_config(getattr(spec, "method_config", None)).node_top_k == 1:
        return None
    return TreeVerify(vllm_config)
