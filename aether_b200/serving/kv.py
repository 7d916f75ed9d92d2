"""Paged KV cache: a page pool per layer, a device page table, and a host-side
page allocator with reference counts, prefix sharing and LRU reuse.

Reference: the paged KV path (paged_append_kv / paged decode attention,
runtime/src/cuda.rs:440-451, 1126), ``SharedKvPool`` (per-layer K/V block
pools shared across sessions, runtime/src/serving.rs:1011-1080) and the host
block allocator with LRU eviction, page tables and admission/reap
(``aether_pkv_*``, runtime/src/lib.rs:5550-5720).

Layout: per layer K and V pools [num_pages, page_size, Hkv, D] bf16; the page
table [rows, max_pages] int32 lives on the device, so the decode kernels (and
a captured CUDA graph) read it there; row ``r`` is one sequence. A full page of
prompt tokens is keyed by a hash chained over all tokens before it, so two
requests with the same prefix share those pages (their K/V are identical);
released pages keep their key and are reused LRU-first, so a later request with
the same prefix can still hit them.
"""
from __future__ import annotations

from collections import OrderedDict

import torch


class NoPages(RuntimeError):
    pass


class PageAllocator:
    def __init__(self, num_pages: int, page_size: int, reserved: int = 0):
        self.num_pages, self.page_size = num_pages, page_size
        self.ref = [0] * num_pages
        self.free = list(range(num_pages - 1, reserved - 1, -1))  # stack; pages < reserved are never handed out
        self.cached: "OrderedDict[int, int]" = OrderedDict()  # key -> page with ref 0 (LRU order)
        self.key_page: dict = {}  # key -> page (live or cached)
        self.page_key: dict = {}
        self.hits = 0

    def available(self) -> int:
        return len(self.free) + len(self.cached)

    def allocate(self) -> int:
        if self.free:
            p = self.free.pop()
        elif self.cached:
            key, p = self.cached.popitem(last=False)  # least recently released
            del self.key_page[key]
            del self.page_key[p]
        else:
            raise NoPages("KV page pool exhausted")
        self.ref[p] = 1
        return p

    def lookup(self, key) -> int | None:
        p = self.key_page.get(key)
        if p is None:
            return None
        if self.ref[p] == 0:
            del self.cached[key]
        self.ref[p] += 1
        self.hits += 1
        return p

    def register(self, page: int, key) -> None:
        if key in self.key_page or page in self.page_key:
            return
        self.key_page[key] = page
        self.page_key[page] = key

    def release(self, page: int) -> None:
        self.ref[page] -= 1
        assert self.ref[page] >= 0
        if self.ref[page] == 0:
            key = self.page_key.get(page)
            if key is not None:
                self.cached[key] = page
            else:
                self.free.append(page)


def prefix_keys(tokens: list, page_size: int) -> list:
    """One key per full page: a hash chained over every token up to its end."""
    keys, h = [], 0
    for i in range(len(tokens) // page_size):
        h = hash((h, tuple(tokens[i * page_size : (i + 1) * page_size])))
        keys.append(h)
    return keys


class PagedKVCache:
    def __init__(self, n_layers: int, n_kv_heads: int, head_dim: int, num_pages: int, page_size: int, rows: int,
                 max_seq: int, device):
        assert page_size & (page_size - 1) == 0, "page size must be a power of two"
        self.page_size, self.rows, self.max_seq = page_size, rows, max_seq
        self.max_pages = (max_seq + page_size - 1) // page_size
        shape = (num_pages, page_size, n_kv_heads, head_dim)
        self.k = [torch.zeros(shape, dtype=torch.bfloat16, device=device) for _ in range(n_layers)]
        self.v = [torch.zeros(shape, dtype=torch.bfloat16, device=device) for _ in range(n_layers)]
        # page 0 is the scratch page: unused table entries and padded batch rows point at it
        self.alloc = PageAllocator(num_pages, page_size, reserved=1)
        self.table = torch.zeros(rows, self.max_pages, dtype=torch.int32, device=device)
        self.pages: list = [[] for _ in range(rows)]
        self.device = torch.device(device)

    def bytes(self) -> int:
        return sum(t.numel() * 2 for t in self.k + self.v)

    def pages_for(self, n_tokens: int) -> int:
        return (n_tokens + self.page_size - 1) // self.page_size

    def _write_row(self, row: int, start: int) -> None:
        new = self.pages[row][start:]
        if new:
            self.table[row, start : start + len(new)].copy_(torch.tensor(new, dtype=torch.int32), non_blocking=False)

    def match_prefix(self, row: int, tokens: list) -> int:
        """Shares cached full pages of ``tokens``' prefix into the (empty) row;
        returns how many tokens they cover. The last prompt token is never
        covered, so the prefill always has at least one token to run."""
        assert not self.pages[row]
        n = 0
        for key in prefix_keys(tokens[:-1], self.page_size):
            p = self.alloc.lookup(key)
            if p is None:
                break
            self.pages[row].append(p)
            n += self.page_size
        self._write_row(row, 0)
        return n

    def ensure(self, row: int, n_tokens: int) -> None:
        """Gives the row pages for positions [0, n_tokens)."""
        have = len(self.pages[row])
        need = self.pages_for(n_tokens)
        if need > self.max_pages:
            raise ValueError("sequence longer than the cache's max_seq")
        for _ in range(have, need):
            self.pages[row].append(self.alloc.allocate())
        self._write_row(row, have)

    def register_prompt(self, row: int, tokens: list) -> None:
        """After prefill: makes the row's full prompt pages shareable."""
        for i, key in enumerate(prefix_keys(tokens, self.page_size)):
            self.alloc.register(self.pages[row][i], key)

    def release(self, row: int) -> None:
        for p in self.pages[row]:
            self.alloc.release(p)
        self.pages[row] = []
        self.table[row].zero_()
