"""Paged KV memory: page allocator with reference counts, a page-granular prefix cache, and the device
tensors (target KV, draft KV and the per-slot target hidden states used by the EAGLE head).

Layout: K and V are [L, pages, Hkv, page_size, head_dim] bf16, so one (page, kv head) block is a
contiguous page_size x head_dim tile that the attention kernel copies in one pass. A slot is
page * page_size + offset. The draft model's KV uses the same page table as the target (separate
tensors), so prefix-cache hits serve both.

The prefix cache is a hash chain over full pages: the key of page i of a prompt is
hash(key of page i-1, tokens of page i). It plays the role of SGLang's radix cache that the reference
relies on for shared prefixes (configuration.yaml:54, docker/opt/v5/casc/README.md:3-4). Pages are
reference counted; unreferenced cached pages are evicted LRU when the free list runs dry.
"""
from __future__ import annotations

from collections import OrderedDict
from typing import Dict, List, Optional, Sequence, Tuple

import torch


class PageAllocator:
    def __init__(self, num_pages: int, reserved: int = 1):
        self.num_pages = num_pages
        # page 0.. reserved-1 are never handed out (slot 0 holds the zero hidden row)
        self.free: List[int] = list(range(num_pages - 1, reserved - 1, -1))
        self.ref = [0] * num_pages

    def available(self) -> int:
        return len(self.free)

    def alloc(self, n: int) -> List[int]:
        if n > len(self.free):
            raise MemoryError(f"out of KV pages: need {n}, have {len(self.free)}")
        out = [self.free.pop() for _ in range(n)]
        for p in out:
            self.ref[p] = 1
        return out

    def incref(self, pages: Sequence[int]) -> None:
        for p in pages:
            self.ref[p] += 1

    def decref(self, pages: Sequence[int]) -> List[int]:
        """Drop one reference; returns pages whose count reached zero (the caller frees or caches them)."""
        dead = []
        for p in pages:
            self.ref[p] -= 1
            assert self.ref[p] >= 0
            if self.ref[p] == 0:
                dead.append(p)
        return dead

    def release(self, pages: Sequence[int]) -> None:
        self.free.extend(pages)


class PrefixCache:
    """Full-page prefix cache keyed by a hash chain of page contents."""

    def __init__(self, alloc: PageAllocator, page_size: int):
        self.alloc = alloc
        self.ps = page_size
        self.table: Dict[int, int] = {}            # chain key -> page
        self.lru: "OrderedDict[int, int]" = OrderedDict()  # unreferenced cached pages: key -> page
        self.key_of: Dict[int, int] = {}           # page -> chain key

    @staticmethod
    def chain_keys(tokens: Sequence[int], page_size: int, n_pages: int) -> List[int]:
        keys, prev = [], 0x9E3779B97F4A7C15
        for i in range(n_pages):
            prev = hash((prev, tuple(tokens[i * page_size:(i + 1) * page_size])))
            keys.append(prev)
        return keys

    def match(self, tokens: Sequence[int], max_tokens: int) -> List[int]:
        """Longest cached page chain covering at most max_tokens tokens; takes a reference on each."""
        n = max_tokens // self.ps
        pages = []
        for k in self.chain_keys(tokens, self.ps, n):
            p = self.table.get(k)
            if p is None:
                break
            pages.append(p)
        for p in pages:
            k = self.key_of[p]
            if k in self.lru:
                del self.lru[k]
        self.alloc.incref(pages)
        return pages

    def insert(self, tokens: Sequence[int], pages: Sequence[int], n_full: int) -> None:
        """Register the first n_full pages of a sequence whose KV is now written."""
        for k, p in zip(self.chain_keys(tokens, self.ps, n_full), pages[:n_full]):
            if k not in self.table and p not in self.key_of:
                self.table[k] = p
                self.key_of[p] = k

    def release(self, pages: Sequence[int]) -> None:
        for p in self.alloc.decref(pages):
            k = self.key_of.get(p)
            if k is not None:
                self.lru[k] = p
            else:
                self.alloc.release([p])

    def evict(self, n: int) -> int:
        freed = 0
        while freed < n and self.lru:
            k, p = self.lru.popitem(last=False)
            del self.table[k]
            del self.key_of[p]
            self.alloc.release([p])
            freed += 1
        return freed

    def obtainable(self) -> int:
        """Pages an allocation can get now: free ones plus unreferenced cached ones (evicted on demand)."""
        return self.alloc.available() + len(self.lru)

    def alloc_pages(self, n: int) -> List[int]:
        if self.alloc.available() < n:
            self.evict(n - self.alloc.available())
        return self.alloc.alloc(n)


class KVPool:
    def __init__(self, num_layers: int, num_pages: int, kv_heads: int, page_size: int, head_dim: int, device,
                 draft_layers: int = 0, hidden: int = 0, dtype=torch.bfloat16):
        self.page_size = page_size
        self.num_pages = num_pages
        self.k = torch.zeros(num_layers, num_pages, kv_heads, page_size, head_dim, dtype=dtype, device=device)
        self.v = torch.zeros_like(self.k)
        self.dk = self.dv = None
        if draft_layers:
            self.dk = torch.zeros(draft_layers, num_pages, kv_heads, page_size, head_dim, dtype=dtype, device=device)
            self.dv = torch.zeros_like(self.dk)
        # target hidden state per slot (EAGLE input); slot 0 stays zero (feature "before position 0")
        self.hidden = torch.zeros(num_pages * page_size, hidden, dtype=dtype, device=device) if hidden else None
        self.alloc = PageAllocator(num_pages, reserved=1)
        self.prefix = PrefixCache(self.alloc, page_size)

    @staticmethod
    def bytes_per_page(num_layers, kv_heads, page_size, head_dim, draft_layers=0, hidden=0):
        return 2 * (num_layers + draft_layers) * kv_heads * page_size * head_dim * 2 + page_size * hidden * 2

    def move_slots(self, src: torch.Tensor, dst: torch.Tensor) -> None:
        """Copy KV rows (all layers, target and draft) and hidden rows from slots src to dst."""
        if src.numel() == 0:
            return
        ps = self.page_size
        sp, so = src // ps, src % ps
        dp, do = dst // ps, dst % ps
        for t in (self.k, self.v):
            t[:, dp, :, do, :] = t[:, sp, :, so, :]
        if self.hidden is not None:
            self.hidden[dst] = self.hidden[src]
