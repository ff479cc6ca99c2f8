"""Host-independent pieces the serving-host adapters share: the round's draft tree and accept step on host tensors,
GDN / Mamba2 tree-verify state updates on host state pools, and the base-class lookup that lets the adapters import
(and have their override signatures checked) without the host installed.

A host hands the adapter flat token batches: ``T`` verify rows, each with its request's state slot and its parent row
(``-1`` = the request's committed state). These helpers turn the host's tree layout into that form and call this
package's kernels (``eagle4_b200.ops``: sm_100a kernels on CUDA tensors, float64 definitions on CPU).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch

from eagle4_b200 import ops
from eagle4_b200.plugins.contract import resolve


def host_base(path: str):
    """The host class at ``path`` to subclass, or ``object`` when the host is not installed (the adapter module still
    imports, and its overrides' signatures are checked against the hook table)."""
    try:
        return resolve(path)
    except (ImportError, AttributeError):
        return object


def parent_rows(parent_token: torch.Tensor, query_start_loc: torch.Tensor) -> torch.Tensor:
    """Global parent row of every token from per-request local parents (``-1``: the committed state).

    ``parent_token[t]`` is the parent's index inside the token's request (the host's tree layout); the request of a
    token follows from ``query_start_loc`` (``[bs + 1]`` row offsets)."""
    t = parent_token.shape[0]
    starts = query_start_loc.long()
    req = torch.bucketize(torch.arange(t, device=parent_token.device), starts[1:], right=True)
    base = starts[:-1][req]
    local = parent_token.long()
    return torch.where(local >= 0, local + base, local).int()


def token_slots(cache_indices: torch.Tensor, query_start_loc: torch.Tensor) -> torch.Tensor:
    """State slot of every token from the per-request slots."""
    counts = (query_start_loc[1:] - query_start_loc[:-1]).long()
    return cache_indices.int().repeat_interleave(counts)


@dataclass
class GdnShape:
    """What the tree kernels read of a GDN layer's configuration (the host layer's attributes)."""

    gdn_k_heads: int
    gdn_v_heads: int
    gdn_k_dim: int
    gdn_v_dim: int
    conv_kernel: int = 4
    rms_norm_eps: float = 1e-6

    @property
    def gdn_key_dim(self) -> int:
        return self.gdn_k_heads * self.gdn_k_dim

    @property
    def gdn_value_dim(self) -> int:
        return self.gdn_v_heads * self.gdn_v_dim

    @property
    def gdn_conv_dim(self) -> int:
        return 2 * self.gdn_key_dim + self.gdn_value_dim

    @classmethod
    def of(cls, layer) -> "GdnShape":
        return cls(layer.num_k_heads, layer.num_v_heads, layer.head_k_dim, layer.head_v_dim,
                   getattr(layer, "conv_kernel_size", 4), getattr(layer, "rms_norm_eps", 1e-6))


class TreeVerifyRows:
    """The verify forward's row structure, derived once per forward (``begin``) and read by every layer."""

    def __init__(self):
        self.parent: Optional[torch.Tensor] = None
        self.slots: Optional[torch.Tensor] = None

    def begin(self, parent_token: torch.Tensor, query_start_loc: torch.Tensor, cache_indices: torch.Tensor) -> None:
        self.parent = parent_rows(parent_token, query_start_loc)
        self.slots = token_slots(cache_indices, query_start_loc)

    def clear(self) -> None:
        self.parent = self.slots = None

    @property
    def active(self) -> bool:
        return self.parent is not None


def gdn_conv(rows: TreeVerifyRows, mixed_qkv: torch.Tensor, conv_states: torch.Tensor,
             weight: torch.Tensor, bias: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Tree causal conv1d (plus the layer's conv bias, if any): each row's window is its ancestors' inputs, the
    committed window below the root."""
    if bias is not None:
        bias = bias.to(mixed_qkv.dtype).contiguous()
    return ops.causal_conv_tree(mixed_qkv, conv_states, rows.slots, rows.parent, weight, bias)


def gdn_recurrence(rows: TreeVerifyRows, qkv: torch.Tensor, a: torch.Tensor, b: torch.Tensor, a_log: torch.Tensor,
                   dt_bias: torch.Tensor, ssm_states: torch.Tensor, shape: GdnShape) -> torch.Tensor:
    """Gated delta rule over the row forest from the committed states (no state written): ``[T, HV * V]``."""
    return ops.gdn_recurrence(qkv, a, b, a_log, dt_bias, ssm_states, rows.slots, rows.parent, shape)


def accept_greedy_rows(target_ids: torch.Tensor, draft_tokens: torch.Tensor, parent_rows_: torch.Tensor):
    """Fused greedy accept over ``[bs, n]`` verify rows: ``(accepted rows, counts, bonus tokens)``."""
    bs, n = draft_tokens.shape
    return ops.accept_greedy(target_ids.view(bs, n), draft_tokens, parent_rows_,
                             torch.full((bs,), n, dtype=torch.int32, device=draft_tokens.device))
