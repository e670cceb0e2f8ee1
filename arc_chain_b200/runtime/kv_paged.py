"""Paged KV cache.

The reference keeps an unbounded ``Vec<i64>`` per layer for K and V
(crates/arc-inference/src/cached_integer_model.rs:89-121).  Here K/V live in
fixed 16-token pages shared by all requests: per layer a device tensor
[n_pages, n_kv_heads_local, 16, d_head] int64 (full i64 precision, as in the
reference), a host-side free list, and per-request page tables.  Page ids are
the same in every layer.
"""
from __future__ import annotations

from typing import Dict, List

import torch

PAGE = 16


class PagePool:
    def __init__(self, n_pages: int):
        self.n_pages = n_pages
        self.free: List[int] = list(range(n_pages - 1, -1, -1))

    def alloc(self, n: int) -> List[int]:
        if n > len(self.free):
            raise MemoryError(f"KV cache out of pages: need {n}, have {len(self.free)}")
        return [self.free.pop() for _ in range(n)]

    def release(self, pages: List[int]) -> None:
        self.free.extend(reversed(pages))

    @property
    def used(self) -> int:
        return self.n_pages - len(self.free)


class PagedKV:
    def __init__(self, n_layers: int, n_pages: int, n_kv: int, d_head: int, device, max_pages_per_seq: int,
                 with_v: bool = True):
        self.n_layers, self.n_pages, self.n_kv, self.d_head = n_layers, n_pages, n_kv, d_head
        self.max_pages_per_seq = max_pages_per_seq
        self.K = [torch.zeros(n_pages, n_kv, PAGE, d_head, dtype=torch.int64, device=device) for _ in range(n_layers)]
        # MLA keeps one latent row per token (values alias it): no V planes
        self.V = [torch.zeros(n_pages, n_kv, PAGE, d_head, dtype=torch.int64, device=device)
                  for _ in range(n_layers)] if with_v else self.K
        self.pool = PagePool(n_pages)
        self.tables: Dict[int, List[int]] = {}

    @staticmethod
    def bytes_per_page(n_layers: int, n_kv: int, d_head: int) -> int:
        return 2 * n_layers * n_kv * PAGE * d_head * 8

    def reserve(self, rid: int, n_tokens: int) -> List[int]:
        """Ensure request `rid` has pages for positions [0, n_tokens)."""
        need = (n_tokens + PAGE - 1) // PAGE
        if need > self.max_pages_per_seq:
            raise ValueError(f"sequence of {n_tokens} tokens exceeds {self.max_pages_per_seq} pages")
        t = self.tables.setdefault(rid, [])
        if need > len(t):
            t.extend(self.pool.alloc(need - len(t)))
        return t

    def release(self, rid: int) -> None:
        t = self.tables.pop(rid, None)
        if t:
            self.pool.release(t)

    def table_row(self, rid: int) -> List[int]:
        t = self.tables.get(rid, [])
        return t + [0] * (self.max_pages_per_seq - len(t))
