"""Paged KV cache with the decode batch's metadata resident on the GPU.

``DevicePagedKV`` keeps everything ``TensorPagedKV`` (worker/llama.py:13-55)
has — zero-initialised pools ``keys``/``values`` [layers, blocks, block_size,
kv_heads, head_dim], the LIFO free list, per-request page lists ``tables``
and token counts ``lengths`` on the host, and ``reserve``/``release``/
``slots``/``metadata`` with the same behaviour — and adds the decode batch's
block tables and lengths as int32 device tensors [max_batch, width] and
[max_batch]. ``bind(ids)`` makes device rows 0..B-1 describe ``ids`` and
uploads only the rows whose request, page list or length changed since the
device last saw them; within a decode step the first layer's prologue
advances the device lengths itself (``rope_kv_write_decode(advance=True)``)
while ``advance(ids)`` advances the host copy, so a steady batch costs no
host-to-device metadata traffic at all and the step can be replayed as one
CUDA graph.

The host lists remain the allocator's truth (reserve/release never touch
the GPU); stale pool cells are never read because lengths bound all reads,
as in the reference.
"""
from __future__ import annotations

import math

import torch


class DevicePagedKV:
    """TensorPagedKV plus device-resident decode metadata (width = max_tokens / block_size)."""

    def __init__(self, config, blocks: int = 256, block_size: int = 16, device="cuda",
                 dtype=torch.float16, max_batch: int = 256, max_tokens: int = 8192,
                 keys: torch.Tensor | None = None, values: torch.Tensor | None = None):
        self.block_size = block_size
        self.total_blocks = blocks
        self.free = list(range(blocks - 1, -1, -1))
        self.tables: dict = {}
        self.lengths: dict = {}
        if keys is None:
            head_dim = getattr(config, "head_dim", None) or (
                config.hidden_size // config.num_attention_heads)
            shape = (config.num_hidden_layers, blocks, block_size, config.num_key_value_heads,
                     head_dim)
            keys = torch.zeros(shape, device=device, dtype=dtype)
            values = torch.zeros_like(keys)
        self.keys, self.values = keys, values
        self.device = self.keys.device
        self.width = math.ceil(max_tokens / block_size)
        self.max_batch = max_batch
        self.max_tokens = self.width * block_size
        self.dev_tables = torch.zeros((max_batch, self.width), dtype=torch.int32,
                                      device=self.device)
        self.dev_lengths = torch.zeros(max_batch, dtype=torch.int32, device=self.device)
        # What device row i holds: (request id, its page list object, page count,
        # length) or None. Holding the list object keeps its identity unique, so
        # a request id reserved again (a new list) is never mistaken for the old.
        self._rows: list = [None] * max_batch
        self.uploaded_rows = 0  # rows copied to the device so far (for tests and stats)

    @classmethod
    def adopt(cls, cache, max_batch: int = 256, max_tokens: int = 8192) -> "DevicePagedKV":
        """Wrap an existing TensorPagedKV: share its pools, free list, tables and lengths."""
        obj = cls(None, cache.total_blocks, cache.block_size, max_batch=max_batch,
                  max_tokens=max_tokens, keys=cache.keys, values=cache.values)
        obj.free, obj.tables, obj.lengths = cache.free, cache.tables, cache.lengths
        return obj

    # ---- TensorPagedKV interface (worker/llama.py:26-55) --------------------
    def reserve(self, request_id, tokens) -> bool:
        if request_id in self.tables:
            raise ValueError("duplicate request ID")
        count = math.ceil(tokens / self.block_size)
        if count > len(self.free):
            return False
        if count > self.width:
            raise ValueError(f"request needs {count} pages; device tables hold {self.width}")
        self.tables[request_id] = [self.free.pop() for _ in range(count)]
        self.lengths[request_id] = 0
        return True

    def release(self, request_id) -> None:
        # Stale cells are never read: lengths bound all reads.
        self.free.extend(self.tables.pop(request_id, []))
        self.lengths.pop(request_id, None)

    def slots(self, ids, positions):
        physical, offsets = [], []
        for request_id, sequence_positions in zip(ids, positions):
            for position in sequence_positions:
                physical.append(self.tables[request_id][position // self.block_size])
                offsets.append(position % self.block_size)
        return (torch.tensor(physical, device=self.device, dtype=torch.long),
                torch.tensor(offsets, device=self.device, dtype=torch.long))

    def metadata(self, ids):
        lengths = [self.lengths[i] for i in ids]
        max_length = max(lengths)
        width = math.ceil(max_length / self.block_size)
        tables = [self.tables[i][:width] + [0] * max(0, width - len(self.tables[i]))
                  for i in ids]
        return (torch.tensor(tables, device=self.device, dtype=torch.int32),
                torch.tensor(lengths, device=self.device, dtype=torch.int32), max_length)

    # ---- device-resident decode metadata ------------------------------------
    def bind(self, ids) -> tuple[torch.Tensor, torch.Tensor]:
        """Device rows 0..B-1 describe ``ids`` (host lengths = tokens cached so far).

        Returns views ``(tables [B, width], lengths [B])`` of the resident
        tensors. Rows already holding the right request, page count and length
        are left alone; the others are written with one pinned host-to-device
        copy and one scatter, ordered on the current stream."""
        B = len(ids)
        if B > self.max_batch:
            raise ValueError(f"batch {B} exceeds max_batch {self.max_batch}")
        stale = []
        for i, rid in enumerate(ids):
            pages, row = self.tables[rid], self._rows[i]
            if (row is None or row[0] != rid or row[1] is not pages or row[2] != len(pages)
                    or row[3] != self.lengths[rid]):
                stale.append(i)
        if stale:
            pin = self.device.type == "cuda"
            host = torch.zeros((len(stale), self.width + 1), dtype=torch.int32)
            host = host.pin_memory() if pin else host
            for j, i in enumerate(stale):
                rid = ids[i]
                pages = self.tables[rid]
                if pages:
                    host[j, :len(pages)] = torch.tensor(pages, dtype=torch.int32)
                host[j, self.width] = self.lengths[rid]
                self._rows[i] = (rid, pages, len(pages), self.lengths[rid])
            dev = host.to(self.device, non_blocking=True)
            index = torch.tensor(stale, dtype=torch.long)
            index = (index.pin_memory() if pin else index).to(self.device, non_blocking=True)
            self.dev_tables.index_copy_(0, index, dev[:, :self.width])
            self.dev_lengths.index_copy_(0, index, dev[:, self.width])
            self.uploaded_rows += len(stale)
        return self.dev_tables[:B], self.dev_lengths[:B]

    def advance(self, ids) -> int:
        """Host side of a decode step: every sequence gains its new token
        (PagedLlama.decode, worker/llama.py:157-158); the device lengths are
        advanced by the step's first prologue. Returns the new max length."""
        for i, rid in enumerate(ids):
            self.lengths[rid] += 1
            row = self._rows[i]
            if row is not None and row[0] == rid:
                self._rows[i] = (rid, row[1], row[2], row[3] + 1)
        return max(self.lengths[r] for r in ids)
