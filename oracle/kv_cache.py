"""Oracle: the paged KV cache bookkeeping and slot writes (test infrastructure only).

Restates TensorPagedKV, worker/llama.py:13-55, and the slot writes of
PagedLlama (decode :171-172, prefill :139-140):
  - pool [layers, blocks, block_size, kv_heads, head_dim], zero-initialised
  - LIFO free list starting [blocks-1, ..., 0]; reserve() takes whole pages
    for the request up front, release() returns them without clearing
  - slots(): (table[pos // bs], pos % bs) per position, as int64
  - metadata(): int32 tables cut/padded with block 0 to ceil(max_len / bs)
    columns, int32 lengths and the host max_length
"""
from __future__ import annotations

import math

import torch


class PagedKVCache:
    def __init__(self, layers: int, kv_heads: int, head_dim: int, blocks: int = 256,
                 block_size: int = 16, device="cpu", dtype=torch.float32):
        self.block_size = block_size
        self.total_blocks = blocks
        self.free = list(range(blocks - 1, -1, -1))
        self.tables: dict = {}
        self.lengths: dict = {}
        shape = (layers, blocks, block_size, kv_heads, head_dim)
        self.keys = torch.zeros(shape, device=device, dtype=dtype)
        self.values = torch.zeros_like(self.keys)

    def reserve(self, request_id, tokens: int) -> bool:
        if request_id in self.tables:
            raise ValueError("duplicate request ID")
        count = math.ceil(tokens / self.block_size)
        if count > len(self.free):
            return False
        self.tables[request_id] = [self.free.pop() for _ in range(count)]
        self.lengths[request_id] = 0
        return True

    def release(self, request_id) -> None:
        self.free.extend(self.tables.pop(request_id, []))
        self.lengths.pop(request_id, None)

    def slots(self, ids, positions):
        physical, offsets = [], []
        for rid, seq_positions in zip(ids, positions):
            for p in seq_positions:
                physical.append(self.tables[rid][p // self.block_size])
                offsets.append(p % self.block_size)
        dev = self.keys.device
        return (torch.tensor(physical, device=dev, dtype=torch.long),
                torch.tensor(offsets, device=dev, dtype=torch.long))

    def metadata(self, ids):
        lengths = [self.lengths[i] for i in ids]
        max_length = max(lengths)
        width = math.ceil(max_length / self.block_size)
        tables = [self.tables[i][:width] + [0] * max(0, width - len(self.tables[i])) for i in ids]
        dev = self.keys.device
        return (torch.tensor(tables, device=dev, dtype=torch.int32),
                torch.tensor(lengths, device=dev, dtype=torch.int32), max_length)


def write_decode(pool: torch.Tensor, physical: torch.Tensor, offsets: torch.Tensor,
                 rows: torch.Tensor) -> None:
    """pool[physical, offsets] = rows   (worker/llama.py:171-172, rows [B, KVH, D])."""
    pool[physical, offsets] = rows


def write_prefill(pool: torch.Tensor, physical: torch.Tensor, offsets: torch.Tensor,
                  x: torch.Tensor, valid: torch.Tensor) -> None:
    """pool[slots] = x[valid]   (worker/llama.py:139-140, x [B, W, KVH, D])."""
    pool[physical, offsets] = x[valid]
