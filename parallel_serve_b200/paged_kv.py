"""Paged KV cache bookkeeping for the two-model decode loop (host side).

The reference keeps one contiguous cache per sequence (its decode benchmarks
size the cache per batch, kernel/FRIDAY_REPORT.md:131 lists paging as the
production layout to come). Here each model's K and V live in page pools
``[pages, n_heads, page_size, 128]`` and a block table ``[B, max_pages]``
(int32, rows in routed order, -1 = no page) maps a sequence's positions
``[i*page_size, (i+1)*page_size)`` to a page of its model's pool. The kernels
(``ps_paged_decode_attention`` and the QKV epilogue's KV append) read the
table on the device; this module hands out pages and keeps the table.
"""
from __future__ import annotations

import random

import numpy as np
import torch


class PageAllocator:
    """Free list of one pool's page ids. ``shuffle`` hands pages out in a
    random order (the kernels take any order; tests use it to make sure)."""

    def __init__(self, n_pages: int, shuffle_seed: int | None = None):
        if n_pages < 0:
            raise ValueError("n_pages must be >= 0")
        self.n_pages = n_pages
        self.free = list(range(n_pages))
        if shuffle_seed is not None:
            random.Random(shuffle_seed).shuffle(self.free)
        self.free.reverse()                     # pop() from the end = first in order

    def alloc(self, n: int) -> list[int]:
        if n > len(self.free):
            raise MemoryError(f"KV page pool exhausted: need {n}, {len(self.free)} free")
        return [self.free.pop() for _ in range(n)]

    def release(self, pages) -> None:
        for p in pages:
            if not 0 <= p < self.n_pages:
                raise ValueError(f"page {p} is not in this pool")
        self.free.extend(reversed(list(pages)))

    @property
    def n_free(self) -> int:
        return len(self.free)


class BlockTable:
    """Block table of a batch whose routed row j belongs to model ``row_model[j]``.

    ``ensure(rows, n_positions)`` gives each row pages for positions
    ``< n_positions``; ``release(rows)`` returns a row's pages. ``device``
    holds the int32 table the kernels read; ``sync()`` copies the host table
    there (only when it changed).
    """

    def __init__(self, row_model, allocators: tuple, max_pages: int, page_size: int,
                 device: torch.device | str = "cpu"):
        self.row_model = [int(m) for m in row_model]
        self.alloc = allocators
        self.max_pages = max_pages
        self.page_size = page_size
        self.host = np.full((len(self.row_model), max_pages), -1, dtype=np.int32)
        self.n_pages = np.zeros(len(self.row_model), dtype=np.int64)
        self.device = torch.full((len(self.row_model), max_pages), -1, dtype=torch.int32,
                                 device=device)
        self._dirty = False

    def ensure(self, rows, n_positions: int) -> None:
        need = -(-int(n_positions) // self.page_size)
        if need > self.max_pages:
            raise ValueError(f"{n_positions} positions exceed the table ({self.max_pages} pages "
                             f"of {self.page_size})")
        for j in rows:
            have = int(self.n_pages[j])
            if have < need:
                pages = self.alloc[self.row_model[j]].alloc(need - have)
                self.host[j, have:need] = pages
                self.n_pages[j] = need
                self._dirty = True

    def release(self, rows) -> None:
        for j in rows:
            have = int(self.n_pages[j])
            if have:
                self.alloc[self.row_model[j]].release(self.host[j, :have].tolist())
                self.host[j, :] = -1
                self.n_pages[j] = 0
                self._dirty = True

    def pages_of(self, j: int) -> list[int]:
        return self.host[j, :int(self.n_pages[j])].tolist()

    def sync(self) -> None:
        if self._dirty:
            self.device.copy_(torch.from_numpy(self.host), non_blocking=False)
            self._dirty = False
