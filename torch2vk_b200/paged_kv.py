"""Paged KV cache: a pool of fixed-size pages shared by the sequences of a
runner, with per-sequence block tables (logical page -> physical page).

Each layer has one K and one V pool [num_pages, page_size, kv_heads, head_dim]
fp16; page p of sequence s holds positions [p * page_size, (p + 1) * page_size).
Pages are handed out from a free list as sequences grow and returned when a
sequence is released; the device block table [max_seqs, max_pages_per_seq]
int32 is what the paged kernels (t2c_attn_decode_paged,
t2c_kv_cache_write_paged) read.  Host code owns the bookkeeping: reserve()
before a step needs the positions, release() when a sequence ends.
"""

from __future__ import annotations

import torch


class PagedKVCache:
    def __init__(self, *, layers: int, num_pages: int, page_size: int, kv_heads: int, head_dim: int, max_seqs: int,
                 max_pages_per_seq: int, device: torch.device | str = "cuda") -> None:
        if page_size <= 0 or page_size & (page_size - 1):
            raise ValueError(f"page_size {page_size} must be a power of two")
        self.page_size, self.num_pages = page_size, num_pages
        self.max_pages_per_seq = max_pages_per_seq
        self.device = torch.device(device)
        shape = (num_pages, page_size, kv_heads, head_dim)
        self.k = [torch.zeros(shape, dtype=torch.float16, device=self.device) for _ in range(layers)]
        self.v = [torch.zeros(shape, dtype=torch.float16, device=self.device) for _ in range(layers)]
        self.block_table = torch.zeros(max_seqs, max_pages_per_seq, dtype=torch.int32, device=self.device)
        self._free = list(range(num_pages - 1, -1, -1))
        self._pages: dict[int, list[int]] = {}

    @property
    def free_pages(self) -> int:
        return len(self._free)

    def pages(self, seq: int) -> list[int]:
        return list(self._pages.get(seq, []))

    def reserve(self, seq: int, positions: int) -> None:
        """Grows sequence `seq` to hold `positions` positions (pages from the free list)."""
        have = self._pages.setdefault(seq, [])
        need = -(-positions // self.page_size)
        if need > self.max_pages_per_seq:
            raise ValueError(f"{positions} positions exceed {self.max_pages_per_seq} pages of {self.page_size}")
        if need - len(have) > len(self._free):
            raise RuntimeError(f"KV pool exhausted: {need - len(have)} pages wanted, {len(self._free)} free")
        new = [self._free.pop() for _ in range(max(0, need - len(have)))]
        if new:
            row = torch.tensor(new, dtype=torch.int32)
            self.block_table[seq, len(have):len(have) + len(new)].copy_(row, non_blocking=False)
            have.extend(new)

    def release(self, seq: int) -> None:
        """Returns the pages of `seq` to the free list."""
        for p in reversed(self._pages.pop(seq, [])):
            self._free.append(p)
        self.block_table[seq].zero_()
