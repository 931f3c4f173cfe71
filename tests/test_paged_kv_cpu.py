"""Host bookkeeping of the paged KV pool (torch2vk_b200.paged_kv.PagedKVCache), on CPU tensors."""

from __future__ import annotations

import pytest
import torch

from torch2vk_b200.paged_kv import PagedKVCache


def _pool(num_pages=8, page_size=16, max_pages_per_seq=4):
    return PagedKVCache(layers=2, num_pages=num_pages, page_size=page_size, kv_heads=2, head_dim=8, max_seqs=3,
                        max_pages_per_seq=max_pages_per_seq, device="cpu")


def test_reserve_grows_and_fills_block_table():
    pool = _pool()
    pool.reserve(0, 1)
    pool.reserve(1, 17)
    pool.reserve(0, 33)
    assert pool.pages(0) == [0, 3, 4] and pool.pages(1) == [1, 2]
    assert pool.block_table[0, :3].tolist() == [0, 3, 4] and pool.block_table[1, :2].tolist() == [1, 2]
    assert pool.free_pages == 3
    pool.reserve(0, 20)  # never shrinks
    assert pool.pages(0) == [0, 3, 4]
    assert pool.k[0].shape == (8, 16, 2, 8) and pool.k[0].dtype == torch.float16


def test_release_returns_pages_and_clears_row():
    pool = _pool()
    pool.reserve(0, 40)
    pool.reserve(1, 10)
    pool.release(0)
    assert pool.free_pages == 7 and pool.pages(0) == []
    assert pool.block_table[0].tolist() == [0, 0, 0, 0]
    pool.reserve(2, 64)
    assert sorted(pool.pages(2)) == [0, 1, 2, 4]


def test_limits():
    with pytest.raises(ValueError, match="power of two"):
        _pool(page_size=24)
    pool = _pool(num_pages=3)
    with pytest.raises(ValueError, match="exceed"):
        pool.reserve(0, 65)
    pool.reserve(0, 48)
    with pytest.raises(RuntimeError, match="exhausted"):
        pool.reserve(1, 1)
    assert pool.pages(1) == [] and pool.free_pages == 0
