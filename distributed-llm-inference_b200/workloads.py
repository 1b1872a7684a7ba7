"""Seeded synthetic decode / prefill workloads with the reference's shapes.

There is no dataset in this path: every input is synthetic. Shapes, sizes and
value distributions follow the five configurations the decode path is
measured on:

  smollm_cpu     SmolLM2-135M attention shape, 1 layer, FP32, batch 4, 9/3 heads,
                 head_dim 64, block 16, 256-block pool, len ~ U[1, 512], theta 1e5
  smollm_fp16    same shape, FP16, batch 64, len ~ U[128, 2048], 30 layers, pool =
                 1.25 x blocks needed, unused blocks hold stale N(0, 4) values
  smollm_fp32    the same batch, lengths and tables in FP32 (the CPU shape's
                 dtype at GPU size)
  llama3_8b      32/8 heads, head_dim 128, 32 layers, FP16, batch 256,
                 len ~ lognormal(median 1024, sigma 0.8) clipped to [16, 8192],
                 theta 5e5, fragmented tables, sequences sharded over ranks
  prefill        SmolLM2 shape FP16, 16 prompts, len ~ U[64, 1024], 4096-block
                 pool, positions 0..len-1, theta 1e5
  (the model-level decode tick is built in the bench harness)

Tables follow worker/llama.py: a sequence's blocks are drawn without
replacement from a seeded permutation of the pool (the LIFO free list of
TensorPagedKV hands out arbitrary physical blocks, worker/llama.py:17,31), and
tables are padded with block 0 to ceil(max_length / block_size) columns
(worker/llama.py:49-55).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

from .sharding import shard_indices


@dataclass
class DecodeWorkload:
    name: str
    batch: int
    heads: int
    kv_heads: int
    head_dim: int
    layers: int
    block_size: int
    dtype: torch.dtype
    theta: float
    seed: int
    lengths: torch.Tensor          # int32 [B], CPU: tokens attended (new token included)
    tables: torch.Tensor           # int32 [B, W], CPU, padded with block 0
    num_blocks: int
    used_blocks: torch.Tensor      # int64 [n_used], CPU
    stale_scale: float = 1.0       # std of unused pool blocks
    meta: dict = field(default_factory=dict)

    @property
    def max_length(self) -> int:
        return int(self.lengths.max())

    @property
    def table_width(self) -> int:
        return self.tables.shape[1]

    @property
    def group(self) -> int:
        return self.heads // self.kv_heads

    @property
    def elem_bytes(self) -> int:
        return torch.finfo(self.dtype).bits // 8

    def positions(self) -> torch.Tensor:
        """Position of the new token: len - 1 (worker/llama.py:154-156)."""
        return (self.lengths.to(torch.int64) - 1).unsqueeze(1)

    def slots(self) -> tuple[torch.Tensor, torch.Tensor]:
        """(physical block, offset) of the new token (worker/llama.py:40-47)."""
        pos = self.lengths.to(torch.int64) - 1
        phys = self.tables.to(torch.int64).gather(1, (pos // self.block_size).unsqueeze(1))[:, 0]
        return phys, pos % self.block_size

    def attention_bytes(self) -> int:
        """Algorithmic HBM bytes of one paged_attention launch (one layer).

        K and V rows read once (2*len*KVH*D*e), one int32 table entry per page
        touched, the length, q read and out written. GQA re-reads and split
        partials are not counted.
        """
        e = self.elem_bytes
        lens = self.lengths.to(torch.int64)
        pages = (lens + self.block_size - 1) // self.block_size
        kv = int(2 * lens.sum()) * self.kv_heads * self.head_dim * e
        return kv + 4 * int(pages.sum()) + 4 * self.batch + 2 * self.batch * self.heads * self.head_dim * e

    def prologue_bytes(self) -> int:
        """Algorithmic bytes of one rope_kv_write launch: q,k,v read, q,k written,
        k,v written to their slots, positions/slots/inv_freq read."""
        e = self.elem_bytes
        per_row = (self.heads + 2 * self.kv_heads) * self.head_dim * e
        writes = (self.heads + 3 * self.kv_heads) * self.head_dim * e
        return self.batch * (per_row + writes + 3 * 8) + 4 * (self.head_dim // 2)

    def fused_bytes(self) -> int:
        """Algorithmic bytes of one decode_attention launch (RoPE + slot write +
        attention of one layer): the attention bytes, plus each sequence's new
        k and v read and written to its slot, plus inv_freq. The fused launch
        writes no rotated q or k outputs."""
        e = self.elem_bytes
        return (self.attention_bytes() + 4 * self.batch * self.kv_heads * self.head_dim * e
                + 4 * (self.head_dim // 2))

    def seq_step_bytes(self) -> int:
        """Per decode step, all layers: prologue + attention bytes."""
        return self.layers * (self.attention_bytes() + self.prologue_bytes())

    def shard(self, rank: int, world: int, mode: str = "balanced") -> "DecodeWorkload":
        """The sequences rank `rank` owns (sharding.shard_indices), with a pool
        of the shard's own size: each rank owns its KV pool and block tables,
        renumbered into that pool."""
        idx = shard_indices(self.lengths, world, rank, mode)
        lengths = self.lengths[torch.tensor(idx, dtype=torch.int64)].clone()
        sub = make_decode_tables(lengths, self.block_size, self.seed * 1000 + rank,
                                 self.meta.get("pool_factor", 1.25), None)
        return DecodeWorkload(
            name=f"{self.name}[{mode} {rank}/{world}]", batch=len(idx), heads=self.heads,
            kv_heads=self.kv_heads, head_dim=self.head_dim, layers=self.layers,
            block_size=self.block_size, dtype=self.dtype, theta=self.theta,
            seed=self.seed * 1000 + rank, lengths=lengths, tables=sub[0], num_blocks=sub[1],
            used_blocks=sub[2], stale_scale=self.stale_scale,
            meta=dict(self.meta, shard=(rank, world, mode, idx)))


def make_decode_tables(lengths: torch.Tensor, block_size: int, seed: int,
                       pool_factor: float | None, num_blocks: int | None):
    """Fragmented tables from a seeded permutation of the pool.

    Returns (tables int32 [B, W], num_blocks, used block ids int64).
    """
    g = torch.Generator().manual_seed(seed)
    need = (lengths.to(torch.int64) + block_size - 1) // block_size
    total = int(need.sum())
    if num_blocks is None:
        num_blocks = max(1, math.ceil(pool_factor * total))
    if total > num_blocks:
        raise ValueError("pool too small for the requested lengths")
    perm = torch.randperm(num_blocks, generator=g)
    width = max(1, math.ceil(int(lengths.max()) / block_size))
    tables = torch.zeros(len(lengths), width, dtype=torch.int32)
    off = 0
    for b, n in enumerate(need.tolist()):
        tables[b, :n] = perm[off:off + n].to(torch.int32)
        off += n
    return tables, num_blocks, perm[:total].clone()


def smollm_cpu(seed: int = 1) -> DecodeWorkload:
    """SmolLM2-135M shape, one FP32 decode step on one layer (CPU-runnable)."""
    g = torch.Generator().manual_seed(seed)
    lengths = torch.randint(1, 513, (4,), generator=g, dtype=torch.int64).to(torch.int32)
    tables, n, used = make_decode_tables(lengths, 16, seed + 100, None, 256)
    return DecodeWorkload("smollm2-135m-cpu-fp32", 4, 9, 3, 64, 1, 16, torch.float32, 1e5, seed,
                          lengths, tables, n, used, stale_scale=1.0)


def smollm_fp16(seed: int = 2, batch: int = 64, layers: int = 30,
                dtype: torch.dtype = torch.float16) -> DecodeWorkload:
    """SmolLM2-135M shape in FP16: batch 64, len ~ U[128, 2048], 30 layers."""
    g = torch.Generator().manual_seed(seed)
    lengths = torch.randint(128, 2049, (batch,), generator=g, dtype=torch.int64).to(torch.int32)
    tables, n, used = make_decode_tables(lengths, 16, seed + 100, 1.25, None)
    name = "smollm2-135m-fp16" if dtype == torch.float16 else "smollm2-135m-fp32"
    return DecodeWorkload(name, batch, 9, 3, 64, layers, 16, dtype, 1e5,
                          seed, lengths, tables, n, used, stale_scale=2.0,
                          meta={"pool_factor": 1.25})


def smollm_fp32(seed: int = 2, batch: int = 64, layers: int = 30) -> DecodeWorkload:
    """The FP32 decode of the SmolLM2-135M CPU shape (9/3 heads, head_dim 64,
    FP32) at the FP16 configuration's GPU size: batch 64, len ~ U[128, 2048],
    30 layers, the same lengths and tables as smollm_fp16."""
    return smollm_fp16(seed, batch, layers, dtype=torch.float32)


def llama3_8b(seed: int = 3, batch: int = 256, layers: int = 32) -> DecodeWorkload:
    """Llama-3-8B attention shape: 32/8 heads, D 128, lognormal lengths."""
    g = torch.Generator().manual_seed(seed)
    raw = torch.empty(batch, dtype=torch.float64).log_normal_(math.log(1024.0), 0.8, generator=g)
    lengths = raw.round().clamp(16, 8192).to(torch.int32)
    tables, n, used = make_decode_tables(lengths, 16, seed + 100, 1.25, None)
    return DecodeWorkload("llama3-8b-decode", batch, 32, 8, 128, layers, 16, torch.float16, 5e5,
                          seed, lengths, tables, n, used, stale_scale=2.0,
                          meta={"pool_factor": 1.25})


@dataclass
class DecodeTensors:
    """Device tensors of a DecodeWorkload: per-layer pools and new-token q/k/v."""
    k_pools: list
    v_pools: list
    q: list
    k: list
    v: list
    tables: torch.Tensor
    lengths: torch.Tensor
    positions: torch.Tensor
    physical: torch.Tensor
    offsets: torch.Tensor
    inv_freq: torch.Tensor


def inv_freq(theta: float, head_dim: int) -> torch.Tensor:
    """1 / theta^(arange(0, D, 2) / D) in fp32, evaluated on the CPU
    (worker/llama.py:105-106); both sides of a comparison use these values."""
    return 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim))


def materialize(w: DecodeWorkload, device: torch.device | str, layers: int | None = None,
                seed_offset: int = 0) -> DecodeTensors:
    """Create the pools and new-token inputs on `device` from a seeded generator
    of that device. Used blocks ~ N(0, 1); unused blocks ~ N(0, stale_scale^2)."""
    device = torch.device(device)
    layers = w.layers if layers is None else layers
    g = torch.Generator(device=device).manual_seed(w.seed * 7919 + seed_offset)
    shape = (w.num_blocks, w.block_size, w.kv_heads, w.head_dim)
    unused = None
    if w.stale_scale != 1.0:
        mask = torch.ones(w.num_blocks, dtype=torch.bool)
        mask[w.used_blocks] = False
        unused = mask.nonzero()[:, 0].to(device)
    kp, vp, qs, ks, vs = [], [], [], [], []
    for _ in range(layers):
        for lst in (kp, vp):
            t = torch.randn(shape, generator=g, device=device, dtype=w.dtype)
            if unused is not None and unused.numel():
                t[unused] *= w.stale_scale
            lst.append(t)
        qs.append(torch.randn(w.batch, w.heads, w.head_dim, generator=g, device=device, dtype=w.dtype))
        ks.append(torch.randn(w.batch, w.kv_heads, w.head_dim, generator=g, device=device, dtype=w.dtype))
        vs.append(torch.randn(w.batch, w.kv_heads, w.head_dim, generator=g, device=device, dtype=w.dtype))
    phys, off = w.slots()
    return DecodeTensors(kp, vp, qs, ks, vs, w.tables.to(device), w.lengths.to(device),
                         w.positions().to(device), phys.to(device), off.to(device),
                         inv_freq(w.theta, w.head_dim).to(device))


def compact_pages(tables: torch.Tensor, lengths: torch.Tensor, pools, block_size: int):
    """Copy only the pages the given sequences use to the CPU and renumber the
    tables into the compact copy (CPU checks and CPU baselines of large pools).

    Returns (tables int32 [B, W] with W unchanged, [cpu pool copies])."""
    lengths = lengths.cpu().to(torch.int64)
    tables = tables.cpu().to(torch.int64)
    need = (lengths + block_size - 1) // block_size
    used = torch.cat([tables[b, :n] for b, n in enumerate(need.tolist())]).unique()
    remap = torch.zeros(int(tables.max()) + 1, dtype=torch.int64)
    remap[used] = torch.arange(used.numel())
    new_tables = torch.zeros_like(tables)
    for b, n in enumerate(need.tolist()):
        new_tables[b, :n] = remap[tables[b, :n]]
    idx = used.to(pools[0].device)
    return new_tables.to(torch.int32), [p.index_select(0, idx).cpu() for p in pools]


@dataclass
class PrefillWorkload:
    name: str
    lengths: torch.Tensor          # int64 [B]
    heads: int
    kv_heads: int
    head_dim: int
    block_size: int
    num_blocks: int
    dtype: torch.dtype
    theta: float
    seed: int
    tables: list                   # per prompt list of physical blocks

    @property
    def width(self) -> int:
        return int(self.lengths.max())

    def valid(self) -> torch.Tensor:
        return torch.arange(self.width)[None, :] < self.lengths[:, None]

    def slots(self) -> tuple[torch.Tensor, torch.Tensor]:
        """Slots of positions 0..len-1 of every prompt, prompt-major
        (worker/llama.py:128 with TensorPagedKV.slots, :40-47)."""
        phys, offs = [], []
        for tab, n in zip(self.tables, self.lengths.tolist()):
            p = torch.arange(n)
            phys.append(torch.tensor(tab, dtype=torch.int64)[p // self.block_size])
            offs.append(p % self.block_size)
        return torch.cat(phys), torch.cat(offs)


def prefill_smollm(seed: int = 4) -> PrefillWorkload:
    g = torch.Generator().manual_seed(seed)
    lengths = torch.randint(64, 1025, (16,), generator=g, dtype=torch.int64)
    need = ((lengths + 15) // 16).tolist()
    perm = torch.randperm(4096, generator=g).tolist()
    tables, off = [], 0
    for n in need:
        tables.append(perm[off:off + n])
        off += n
    return PrefillWorkload("smollm2-135m-prefill-fp16", lengths, 9, 3, 64, 16, 4096,
                           torch.float16, 1e5, seed, tables)


def materialize_prefill(w: PrefillWorkload, device: torch.device | str) -> dict:
    device = torch.device(device)
    g = torch.Generator(device=device).manual_seed(w.seed * 7919)
    B, W = len(w.lengths), w.width
    shape = (w.num_blocks, w.block_size, w.kv_heads, w.head_dim)
    phys, offs = w.slots()
    return {
        "q": torch.randn(B, W, w.heads, w.head_dim, generator=g, device=device, dtype=w.dtype),
        "k": torch.randn(B, W, w.kv_heads, w.head_dim, generator=g, device=device, dtype=w.dtype),
        "v": torch.randn(B, W, w.kv_heads, w.head_dim, generator=g, device=device, dtype=w.dtype),
        "k_pool": torch.randn(shape, generator=g, device=device, dtype=w.dtype) * 2,
        "v_pool": torch.randn(shape, generator=g, device=device, dtype=w.dtype) * 2,
        "valid": w.valid().to(device),
        "positions": torch.arange(W, device=device)[None, :].expand(B, -1),
        "physical": phys.to(device),
        "offsets": offs.to(device),
        "inv_freq": inv_freq(w.theta, w.head_dim).to(device),
    }


# --------------------------------------------------------------------------
# Decode tick of the SmolLM2-135M architecture (the model runner's workload)
# --------------------------------------------------------------------------
def smollm2_135m_config():
    """SmolLM2-135M architecture: hidden 576, 30 layers, 9/3 heads, head_dim 64,
    MLP 1536, RMSNorm eps 1e-5, vocab 49152, RoPE theta 1e5, tied embeddings."""
    from transformers import LlamaConfig
    return LlamaConfig(vocab_size=49152, hidden_size=576, intermediate_size=1536,
                       num_hidden_layers=30, num_attention_heads=9, num_key_value_heads=3,
                       head_dim=64, max_position_embeddings=8192, rms_norm_eps=1e-5,
                       rope_theta=1e5, tie_word_embeddings=True)


def seeded_llama(config, seed: int, dtype=torch.float16, device="cuda"):
    """Random-init LlamaForCausalLM (no checkpoint here): initialised on the
    CPU from ``seed``, then cast and moved; no gradients."""
    from transformers import LlamaForCausalLM
    torch.manual_seed(seed)
    model = LlamaForCausalLM(config).eval()
    for prm in model.parameters():
        prm.requires_grad_(False)
    return model.to(dtype=dtype, device=device)


def tick_blocks(batch: int = 128, seed: int = 5, max_len: int = 4096, extra: int = 256,
                block_size: int = 16) -> int:
    """Pool blocks for decode_tick_state: 1.25 x the pages the batch reserves."""
    g = torch.Generator().manual_seed(seed)
    lengths = torch.randint(16, max_len + 1, (batch,), generator=g)
    pages = int(((lengths + extra + block_size - 1) // block_size).sum())
    return math.ceil(1.25 * pages)


def decode_tick_state(cache, batch: int = 128, seed: int = 5, max_len: int = 4096,
                      extra: int = 256):
    """Serving state of a decode tick on a TensorPagedKV-like ``cache``:
    ``batch`` sequences with lengths U[16, max_len] (seeded), each holding the
    pages for its length + ``extra`` tokens, taken from a shuffled free list
    (pages freed and reused in arbitrary order, as after many requests), and
    every pool byte set to seeded N(0, 1) values (the sequences' cached K/V
    and the stale cells of freed pages alike). Returns (ids, lengths)."""
    g = torch.Generator().manual_seed(seed)
    lengths = torch.randint(16, max_len + 1, (batch,), generator=g)
    order = torch.randperm(len(cache.free), generator=g).tolist()
    cache.free[:] = [cache.free[i] for i in order]
    ids = [f"seq{i}" for i in range(batch)]
    for rid, n in zip(ids, lengths.tolist()):
        if not cache.reserve(rid, n + extra):
            raise RuntimeError("pool too small for the tick workload")
        cache.lengths[rid] = n
    gen = torch.Generator(device=cache.keys.device).manual_seed(seed + 1)
    for pool in (cache.keys, cache.values):
        pool.normal_(0.0, 1.0, generator=gen)
    return ids, lengths
