"""Paged TurboQuant KV cache for serving: sequences of independent lengths share page pools.

Every layer keeps a K pool and a V pool, uint8 [num_pages, n_kv_heads, page_size,
head_dim / 32, block_bytes] (TQ3_0 or TQ4_0 keys, TQ4_0 values).  A page holds
page_size consecutive tokens of one sequence for every KV head; page p of sequence s
is pool page table[s, p], the same page in every layer's pools.  New rows are
Hadamard-rotated and quantized straight into their pages (tq_kv_append_paged_cuda)
and decode attention reads the pages in place (tq_decode_attention_paged_cuda): the
cache is never dequantized.  This is the paged form of the packed cache that
prototype/turboquant/kv_cache.py:109-204 keeps per layer.

A decode step:

    cache = PagedKVCache(n_layers, n_kv_heads=8, head_dim=128, num_pages=4096)
    a, b = cache.add_sequence(), cache.add_sequence()
    step = cache.batch([a, b], n_new=1)          # reserves pages, gathers the page rows
    for layer in range(n_layers):
        cache.append(step, layer, k, v)          # [2, n_kv_heads, 1, head_dim]
        out = cache.attention(step, layer, q)    # [2, n_q_heads, head_dim], sees the new rows
    cache.commit(step)                           # the sequences are one token longer
    cache.free_sequence(a)                       # its pages return to the pool

Page bookkeeping (PageTable) is host-side and needs no GPU.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Sequence

import numpy as np

NO_PAGE = -1   # page-table entry of a page not allocated (appends there are skipped and counted)


class PageTable:
    """Host-side page allocation: a free list of pool pages and one page-table row per sequence slot."""

    def __init__(self, num_pages: int, page_size: int, max_seqs: int, max_pages_per_seq: int):
        if page_size < 16 or page_size & (page_size - 1):
            raise ValueError("page_size must be a power of two >= 16")
        if num_pages <= 0 or max_seqs <= 0 or max_pages_per_seq <= 0:
            raise ValueError("num_pages, max_seqs and max_pages_per_seq must be positive")
        self.num_pages, self.page_size = num_pages, page_size
        self.max_seqs, self.max_pages_per_seq = max_seqs, max_pages_per_seq
        self.table = np.full((max_seqs, max_pages_per_seq), NO_PAGE, dtype=np.int32)
        self.lens = np.zeros(max_seqs, dtype=np.int64)
        self.n_pages = np.zeros(max_seqs, dtype=np.int64)   # pages held per sequence
        self.active = np.zeros(max_seqs, dtype=bool)
        self._free = list(range(num_pages - 1, -1, -1))     # pop() hands out low pages first
        self.dirty: set = set()                             # sequence rows changed since the last sync

    @property
    def free_pages(self) -> int:
        return len(self._free)

    @property
    def capacity(self) -> int:
        """Tokens one sequence can hold."""
        return self.max_pages_per_seq * self.page_size

    def add_sequence(self) -> int:
        idle = np.flatnonzero(~self.active)
        if idle.size == 0:
            raise RuntimeError(f"all {self.max_seqs} sequence slots are in use")
        s = int(idle[0])
        self.active[s] = True
        self.lens[s] = 0
        return s

    def free_sequence(self, s: int) -> None:
        self._check(s)
        held = self.table[s, : self.n_pages[s]]
        self._free.extend(int(p) for p in held[::-1])
        self.table[s, :] = NO_PAGE
        self.n_pages[s] = 0
        self.lens[s] = 0
        self.active[s] = False
        self.dirty.add(s)

    def reserve(self, seqs: Sequence[int], n_new: int) -> None:
        """Give every sequence in seqs pages for n_new more tokens (all or nothing)."""
        need = []
        for s in seqs:
            self._check(s)
            total = int(self.lens[s]) + n_new
            if total > self.capacity:
                raise ValueError(f"sequence {s} would hold {total} tokens; the limit is {self.capacity}")
            need.append(max(0, -(-total // self.page_size) - int(self.n_pages[s])))
        if sum(need) > len(self._free):
            raise MemoryError(f"{sum(need)} pages needed, {len(self._free)} free")
        for s, n in zip(seqs, need):
            for _ in range(n):
                self.table[s, self.n_pages[s]] = self._free.pop()
                self.n_pages[s] += 1
            if n:
                self.dirty.add(s)

    def commit(self, seqs: Sequence[int], n_new: int) -> None:
        for s in seqs:
            self._check(s)
            if self.lens[s] + n_new > self.n_pages[s] * self.page_size:
                raise ValueError(f"sequence {s}: {n_new} tokens were not reserved")
            self.lens[s] += n_new

    def _check(self, s: int) -> None:
        if not (0 <= s < self.max_seqs) or not self.active[s]:
            raise ValueError(f"sequence {s} is not active")


@dataclass
class Batch:
    """One step's sequences: their page-table rows, append positions and attention lengths (device)."""
    seqs: List[int]
    n_new: int
    table: "object"      # int32 [B, max_pages_per_seq]
    pos: "object"        # int32 [B]: the first slot the step writes
    kv_len: "object"     # int32 [B]: pos + n_new
    max_kv_len: int


class PagedKVCache:
    """Per-layer TurboQuant page pools with fused paged append and decode attention."""

    def __init__(self, n_layers: int, n_kv_heads: int, head_dim: int, num_pages: int, page_size: int = 16,
                 max_seqs: int = 64, max_pages_per_seq: int | None = None, k_bits: int = 3, k_opt_passes: int = 0,
                 device: str = "cuda"):
        import torch
        if head_dim not in (128, 256):
            raise ValueError("head_dim must be 128 or 256 (fused decode attention)")
        if k_bits not in (2, 3, 4):
            raise ValueError("keys are TQ2_0, TQ3_0 or TQ4_0")
        if k_opt_passes and k_bits != 3:
            raise ValueError("optimal rounding applies to TQ3_0 keys")
        max_pages_per_seq = max_pages_per_seq or num_pages
        self.pages = PageTable(num_pages, page_size, max_seqs, max_pages_per_seq)
        self.n_layers, self.n_kv_heads, self.head_dim = n_layers, n_kv_heads, head_dim
        self.k_bits, self.k_opt_passes = k_bits, k_opt_passes
        self.device = torch.device(device)
        kb = {2: 10, 3: 14, 4: 18}[k_bits]
        shape = (num_pages, n_kv_heads, page_size, head_dim // 32)
        self.k = [torch.zeros(shape + (kb,), dtype=torch.uint8, device=self.device) for _ in range(n_layers)]
        self.v = [torch.zeros(shape + (18,), dtype=torch.uint8, device=self.device) for _ in range(n_layers)]
        self._table = torch.full((max_seqs, max_pages_per_seq), NO_PAGE, dtype=torch.int32, device=self.device)
        self._lens = torch.zeros(max_seqs, dtype=torch.int32, device=self.device)

    # sequence management (host bookkeeping; page-table rows reach the device in batch())
    def add_sequence(self) -> int:
        s = self.pages.add_sequence()
        self._lens[s] = 0
        return s

    def free_sequence(self, s: int) -> None:
        self.pages.free_sequence(s)

    def seq_len(self, s: int) -> int:
        return int(self.pages.lens[s])

    def batch(self, seqs: Sequence[int], n_new: int = 1) -> Batch:
        """Reserve pages for n_new tokens of every sequence and gather the step's device views."""
        import torch
        seqs = [int(s) for s in seqs]
        if len(set(seqs)) != len(seqs):
            raise ValueError("a sequence may appear once per batch")
        self.pages.reserve(seqs, n_new)
        self._sync()
        idx = torch.tensor(seqs, dtype=torch.int64, device=self.device)
        pos = self._lens.index_select(0, idx)
        lens = self.pages.lens[seqs] + n_new
        return Batch(seqs, n_new, self._table.index_select(0, idx).contiguous(), pos.contiguous(),
                     (pos + n_new).contiguous(), int(lens.max()) if len(seqs) else 0)

    def append(self, step: Batch, layer: int, k, v) -> None:
        """Quantize-on-write of the step's new rows k, v [B, n_kv_heads, n_new, head_dim]."""
        from . import ops
        B = len(step.seqs)
        for t, name in ((k, "k"), (v, "v")):
            if tuple(t.shape) != (B, self.n_kv_heads, step.n_new, self.head_dim):
                raise ValueError(f"{name} must be [{B}, {self.n_kv_heads}, {step.n_new}, {self.head_dim}]")
        ops.kv_append_paged(k.contiguous(), self.k[layer], step.table, step.pos, qtype=self.k_bits,
                            opt_passes=self.k_opt_passes)
        ops.kv_append_paged(v.contiguous(), self.v[layer], step.table, step.pos, qtype=4)

    def attention(self, step: Batch, layer: int, q, sm_scale: float | None = None, out_dtype=None, out=None):
        """Decode attention of q [B, n_q_heads, head_dim] over each sequence's tokens, this step's included."""
        from . import attention as A
        return A.decode_attention_paged(q.contiguous(), self.k[layer], self.v[layer], step.table, step.kv_len,
                                        max_kv_len=step.max_kv_len, sm_scale=sm_scale,
                                        out_dtype=out_dtype or q.dtype, out=out)

    def commit(self, step: Batch) -> None:
        """The step's rows are part of the sequences from now on."""
        import torch
        self.pages.commit(step.seqs, step.n_new)
        idx = torch.tensor(step.seqs, dtype=torch.int64, device=self.device)
        self._lens.index_copy_(0, idx, step.kv_len)

    def _sync(self) -> None:
        import torch
        if not self.pages.dirty:
            return
        rows = sorted(self.pages.dirty)
        self.pages.dirty.clear()
        idx = torch.tensor(rows, dtype=torch.int64, device=self.device)
        self._table.index_copy_(0, idx, torch.from_numpy(self.pages.table[rows]).to(self.device))
        for s in rows:
            if not self.pages.active[s]:
                self._lens[s] = 0

    def memory_summary(self) -> dict:
        pool = sum(t.numel() for t in self.k) + sum(t.numel() for t in self.v)
        used = self.pages.num_pages - self.pages.free_pages
        return {"pool_bytes": pool, "pages": self.pages.num_pages, "pages_used": used,
                "page_size": self.pages.page_size, "bytes_per_page_all_layers": pool // self.pages.num_pages,
                "tokens_cached": int(self.pages.lens[self.pages.active].sum())}
