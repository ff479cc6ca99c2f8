"""Shape caps, calibration batch grid and verify-width buckets.

These numbers are part of the public contract (cost-table directory names, graph buckets, config validation),
so they equal the reference's: ``eagle_harness/core/limits.py:20-53`` (caps and the batch grid),
``:78-99`` (verify buckets), ``:102-110`` (draft query lengths), ``:113-124`` (block-table span) and
``:127-147`` (``check_shape``).
"""

from __future__ import annotations

import enum
from typing import Iterable, List, Tuple


class ComputeIntensity(str, enum.Enum):
    """How wide the served draft shapes are; serialized by value in configs and cost keys."""

    HIGH = "high_intensity"
    LOW = "low_intensity"
    CHAIN = "chain_intensity"


MAX_BATCH_SIZE_CHAIN = 512
MAX_BATCH_SIZE_TREE = 512
MAX_VERIFY_TOKENS = 4096
MAX_TREE_DEPTH = 31
MAX_CHAIN_DEPTH = 15
MAX_NODE_TOP_K = 8
TAIL_MASK_BITS = 64  # every verify row carries one 64-bit ancestor word
MAX_VERIFY_NUM = 64
MAX_CHAIN_VERIFY_NUM = 16
assert MAX_VERIFY_NUM <= TAIL_MASK_BITS

# Batch sizes the offline calibration measures (the ``bs_<N>`` directories).
COST_BATCH_SIZES: Tuple[int, ...] = (
    1, 2, 3, 4, 5, 6, 7, 8, 12, 16, 24, 32, 48, 64, 96, 128, 192, 256, 384, 512,
)

# Verify widths with a graph per batch class, widest first.
_TREE_BUCKETS_SMALL = (64, 32, 16, 8, 1)
_TREE_BUCKETS_MID_LOW = (32, 16, 8, 4, 1)
_TREE_BUCKETS_LARGE_LOW = (16, 8, 4, 2, 1)
_CHAIN_BUCKETS = (16, 14, 12, 10, 8, 6, 4, 2, 1)


def max_batch_size(intensity: ComputeIntensity) -> int:
    """Largest batch that drafts at ``intensity``."""
    return MAX_BATCH_SIZE_CHAIN if intensity is ComputeIntensity.CHAIN else MAX_BATCH_SIZE_TREE


def cost_batch_sizes(max_bs: int, start_bs: int = 1) -> List[int]:
    """The calibration grid restricted to ``[start_bs, max_bs]``."""
    return [b for b in COST_BATCH_SIZES if start_bs <= b <= max_bs]


def nearest_cost_batch_size(batch_size: int, measured: Iterable[int]) -> int:
    """Closest measured batch size; on a tie the larger one wins."""
    pool = sorted(measured)
    if not pool:
        raise ValueError("the cost data measures no batch size")
    best = pool[0]
    for b in pool[1:]:
        if abs(b - batch_size) <= abs(best - batch_size):
            best = b
    return best


def verify_buckets(batch_size: int, intensity: ComputeIntensity) -> List[int]:
    """Verify widths (tokens per request) that get a target graph and a cost curve, widest first."""
    if batch_size <= 0:
        raise ValueError(f"batch size {batch_size} is not positive")
    if batch_size > MAX_BATCH_SIZE_CHAIN:
        raise NotImplementedError(f"batch size {batch_size} is above the {MAX_BATCH_SIZE_CHAIN} requests chain rounds serve")
    if intensity is ComputeIntensity.CHAIN:
        return list(_CHAIN_BUCKETS)
    if batch_size > MAX_BATCH_SIZE_TREE:
        raise NotImplementedError(f"batch size {batch_size} is above the {MAX_BATCH_SIZE_TREE} requests tree rounds serve")
    high = intensity is ComputeIntensity.HIGH
    if batch_size <= 2 or (batch_size <= 8 and high):
        return list(_TREE_BUCKETS_SMALL)
    if batch_size <= 8 or high:
        return list(_TREE_BUCKETS_MID_LOW)
    return list(_TREE_BUCKETS_LARGE_LOW)


def draft_query_lens(batch_size: int, intensity: ComputeIntensity) -> List[int]:
    """Tree widths (rows per request) the calibration times for one draft step."""
    if intensity is ComputeIntensity.CHAIN:
        return [1]
    if batch_size <= 32:
        return [1, 2, 4, 8]
    return [1, 2, 4] if batch_size <= 64 else [1, 2]


def req_to_token_span(node_top_k: int, tree_depth: int, verify_num: int, page_size: int) -> int:
    """Widest span of block-table entries past ``seq_len`` that one round writes (draft, verify, shared chain)."""
    chain = node_top_k == 1
    draft = node_top_k * tree_depth
    verify = min(verify_num, tree_depth + 1) if chain else verify_num
    shared = tree_depth + 1 if chain and page_size > 1 else 0
    return max(draft, verify, shared)


def check_shape(
    intensity: ComputeIntensity, node_top_k: int, tree_depth: int, verify_num: int, max_running_requests: int
) -> None:
    """Refuse a draft shape the kernels cannot serve."""
    chain = intensity is ComputeIntensity.CHAIN
    cap = max_batch_size(intensity)
    if max_running_requests > cap:
        kind = "chain" if chain else "tree"
        raise ValueError(f"max_running_requests {max_running_requests} is above the {cap} requests {kind} rounds serve")
    if tree_depth > (MAX_CHAIN_DEPTH if chain else MAX_TREE_DEPTH):
        raise NotImplementedError(f"{intensity.value} rounds do not draft {tree_depth} levels deep")
    if node_top_k > MAX_NODE_TOP_K:
        raise NotImplementedError(f"--speculative-eagle-topk is at most {MAX_NODE_TOP_K}")
    if chain and node_top_k > 1:
        raise NotImplementedError("chain_intensity drafts one child per node: --speculative-eagle-topk must be 1")
    if verify_num > (MAX_CHAIN_VERIFY_NUM if chain else MAX_VERIFY_NUM):
        raise NotImplementedError(f"{intensity.value} rounds do not verify {verify_num} tokens")
    if verify_num <= 1:
        raise ValueError("a verify of one token or fewer drafts nothing")
