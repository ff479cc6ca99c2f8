"""Prompt sets for the checking tools: a JSONL file of ``{"id": ..., "prompt_ids": [...]}`` rows, or synthetic
uniform-random token ids (no tokenizer or dataset is needed offline)."""

from __future__ import annotations

import json
from typing import List, Tuple

import torch


def load(path: str) -> List[Tuple[str, List[int]]]:
    rows = []
    with open(path, encoding="utf-8") as f:
        for i, line in enumerate(f):
            if line.strip():
                r = json.loads(line)
                rows.append((str(r.get("id", i)), [int(t) for t in r["prompt_ids"]]))
    return rows


def synthetic(n: int, *, lo: int, hi: int, vocab: int, seed: int = 0) -> List[Tuple[str, List[int]]]:
    """``n`` prompts of lengths uniform in [lo, hi] over token ids [1, vocab)."""
    g = torch.Generator().manual_seed(seed)
    out = []
    for i in range(n):
        length = int(torch.randint(lo, hi + 1, (1,), generator=g))
        out.append((f"p{i}", torch.randint(1, vocab, (length,), generator=g).tolist()))
    return out
