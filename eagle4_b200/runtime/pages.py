"""The KV page pool: attention caches hold a fixed number of pages shared by every request's block-table row.

A request's row maps its logical pages (``position // page``) to physical pages of the pool. Pages are handed out on
admission for the tokens the request may reach (prompt, new tokens and one round's tree rows past its committed
length) and returned when it leaves, so the cache holds what the admitted requests need instead of ``max_len`` per
row. Every entry that maps no page points at page 0, a trash page no request owns: a kernel that reads or writes past
a row's mapped range (a padding row of a batch bucket, a stale tree row) touches valid memory whose contents nobody
reads.
"""

from __future__ import annotations

from typing import Dict, List

import torch


class OutOfPages(RuntimeError):
    """The pool has fewer free pages than a request needs."""


class PagePool:
    TRASH = 0

    def __init__(self, block_table: torch.Tensor, num_pages: int, page: int):
        """``block_table``: ``[rows, max_blocks]`` int32 (device), rewritten in place; ``num_pages`` includes the
        trash page."""
        if num_pages < 2:
            raise ValueError("a page pool needs the trash page and at least one page")
        self.block_table, self.num_pages, self.page = block_table, num_pages, page
        self.max_blocks = block_table.shape[1]
        self._free: List[int] = list(range(num_pages - 1, 0, -1))  # a stack: low pages first
        self._owned: Dict[int, List[int]] = {}
        block_table.fill_(self.TRASH)

    @property
    def free_pages(self) -> int:
        return len(self._free)

    def pages_for(self, tokens: int) -> int:
        return (tokens + self.page - 1) // self.page

    def owned(self, row: int) -> int:
        return len(self._owned.get(row, ()))

    def reserve(self, row: int, tokens: int) -> None:
        """Back positions ``[0, tokens)`` of block-table row ``row`` with pages (adding to what it holds)."""
        need = self.pages_for(tokens)
        if need > self.max_blocks:
            raise ValueError(f"{tokens} tokens need {need} pages; a block-table row maps {self.max_blocks}")
        have = self._owned.setdefault(row, [])
        extra = need - len(have)
        if extra <= 0:
            return
        if extra > len(self._free):
            raise OutOfPages(f"row {row} needs {extra} more pages; {len(self._free)} of {self.num_pages} are free")
        new = [self._free.pop() for _ in range(extra)]
        start = len(have)
        have.extend(new)
        self.block_table[row, start:start + extra] = torch.tensor(new, dtype=self.block_table.dtype).to(
            self.block_table.device, non_blocking=True)

    def release(self, row: int) -> None:
        """Return row ``row``'s pages to the pool and point the row at the trash page."""
        pages = self._owned.pop(row, [])
        if pages:
            self._free.extend(reversed(pages))
            self.block_table[row, :len(pages)] = self.TRASH
