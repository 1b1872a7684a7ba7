"""C-ABI checks that need no GPU: the library loads, exports every symbol the
header declares, validates arguments like cuda/binding.cpp:8-22, and the
fast kernel's work partition covers every unit exactly once."""
from __future__ import annotations

import ctypes
import re

import numpy as np
import pytest
import torch

from conftest import REPO, import_module

_lib = import_module("_lib")
build = import_module("build")

HEADER = REPO / "include" / "paged_decode_b200.h"


@pytest.fixture(scope="module")
def lib():
    build.build_library()
    return _lib.load()


def declared_symbols():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(pdb_[a-z0-9_]+)\s*\(", text)))


def test_exports_every_declared_symbol(lib):
    names = declared_symbols()
    assert len(names) >= 10
    for name in names:
        assert hasattr(lib, name), name
        assert name in _lib.SIGNATURES, f"{name} lacks a ctypes signature"
    assert set(_lib.SIGNATURES) == set(names)


def test_version(lib):
    assert b"sm_100a" in lib.pdb_version()


def attn(lib, **kw):
    a = dict(B=2, H=4, D=32, N=12, bs=16, KVH=2, Dk=32, W=3, max_length=35, dtype=0)
    a.update(kw)
    return lib.pdb_paged_attention(None, None, None, None, None, None, a["B"], a["H"], a["D"],
                                   a["N"], a["bs"], a["KVH"], a["Dk"], a["W"], a["max_length"],
                                   a["dtype"], None, 0, None)


@pytest.mark.parametrize("kw,msg", [
    (dict(B=0), "invalid query shape"),
    (dict(D=257, Dk=257), "invalid query shape"),
    (dict(H=0), "invalid query shape"),
    (dict(N=0), "invalid cache shape"),
    (dict(Dk=16), "invalid cache shape"),
    (dict(KVH=3), "query heads must be a multiple of KV heads"),
    (dict(dtype=7), "use FP32 or FP16"),
    (dict(max_length=0), "invalid context bound"),
    (dict(max_length=8193, W=600), "invalid context bound"),
    (dict(max_length=49), "invalid context bound"),
])
def test_argument_checks_match_reference_messages(lib, kw, msg):
    assert attn(lib, **kw) == 1
    assert _lib.last_error() == msg


def test_null_pointers_rejected_after_shape_checks(lib):
    assert attn(lib) == 1
    assert _lib.last_error() == "null tensor pointer"


def test_rope_argument_checks(lib):
    rc = lib.pdb_rope_kv_write(None, None, None, None, None, None, None, None, 0, 0, None, None,
                               None, 2, None, 2, 1, 4, 2, 63, 8, 16, 1, None, 0, None)
    assert rc == 1 and "even" in _lib.last_error()
    rc = lib.pdb_rope_kv_write(None, None, None, None, None, None, None, None, 0, 0, None, None,
                               None, 3, None, 2, 1, 4, 2, 64, 8, 16, 1, None, 0, None)
    assert rc == 1 and "slots" in _lib.last_error()
    assert lib.pdb_rope_kv_write_workspace_size(4, 100, 1) >= 400
    assert lib.pdb_rope_kv_write_workspace_size(4, 100, 0) == 0


def rope_write(lib, **kw):
    a = dict(num_slots=8, B=2, S=4, H=4, KVH=2, D=64, N=8, bs=16, dtype=0)
    a.update(kw)
    return lib.pdb_rope_kv_write(None, None, None, None, None, None, None, None, 0, 0, None, None,
                                 None, a["num_slots"], None, a["B"], a["S"], a["H"], a["KVH"],
                                 a["D"], a["N"], a["bs"], a["dtype"], None, 0, None)


@pytest.mark.parametrize("kw,msg", [
    (dict(B=0), "invalid q/k/v shapes"),
    (dict(S=0), "invalid q/k/v shapes"),
    (dict(KVH=0), "invalid q/k/v shapes"),
    (dict(D=63), "head_dim must be even for rotate-half RoPE"),
    (dict(N=0), "invalid cache shape"),
    (dict(bs=0), "invalid cache shape"),
    (dict(dtype=7), "use FP32 or FP16"),
    (dict(num_slots=7), "number of slots must match the rows written"),
    (dict(num_slots=-1), "number of slots must match the rows written"),
    # the kernels index rows in 32 bits
    (dict(B=1 << 31, S=1, num_slots=1 << 31), "shape too large"),
    (dict(B=2, S=1 << 30, num_slots=1 << 31), "shape too large"),
    (dict(), "null tensor pointer"),
])
def test_rope_write_argument_checks(lib, kw, msg):
    """pdb_rope_kv_write validates shapes, slot count and row count (rows are
    indexed in 32 bits on the device) before any pointer or CUDA call."""
    assert rope_write(lib, **kw) == 1
    assert _lib.last_error() == msg


def rope_decode(lib, **kw):
    a = dict(W=4, B=2, H=4, KVH=2, D=64, N=8, bs=16, dtype=0)
    a.update(kw)
    return lib.pdb_rope_kv_write_decode(None, None, None, None, None, None, None, None, a["W"],
                                        None, 0, None, a["B"], a["H"], a["KVH"], a["D"], a["N"],
                                        a["bs"], a["dtype"], None)


@pytest.mark.parametrize("kw,msg", [
    (dict(B=0), "invalid q/k/v shapes"),
    (dict(D=65), "head_dim must be even for rotate-half RoPE"),
    (dict(bs=0), "invalid cache shape"),
    (dict(W=0), "invalid table width"),
    (dict(dtype=7), "use FP32 or FP16"),
    (dict(B=1 << 31), "shape too large"),
    (dict(W=1 << 27, bs=16), "shape too large"),
    (dict(), "null tensor pointer"),
])
def test_rope_decode_argument_checks(lib, kw, msg):
    """pdb_rope_kv_write_decode validates its shapes, table width and the
    table's token capacity (positions are formed in 32 bits) first."""
    assert rope_decode(lib, **kw) == 1
    assert _lib.last_error() == msg


def partition(lib, lengths, kvh, grid):
    lens = np.asarray(lengths, dtype=np.int32)
    ranges = np.zeros(2 * grid, dtype=np.int64)
    total = lib.pdb_debug_partition(lens.ctypes.data, len(lens), kvh, grid, ranges.ctypes.data)
    return total, ranges.reshape(grid, 2)


@pytest.mark.parametrize("seed", range(5))
def test_partition_covers_units_once_and_balances(lib, seed):
    rng = np.random.default_rng(seed)
    B = int(rng.integers(1, 300))
    lengths = np.clip(np.round(rng.lognormal(np.log(1024), 0.8, B)), 0, 8192).astype(np.int32)
    lengths[rng.random(B) < 0.1] = 0
    kvh = int(rng.choice([1, 2, 3, 8]))
    grid = int(rng.integers(1, 600))
    total, r = partition(lib, lengths, kvh, grid)
    assert total == kvh * int(np.sum((lengths.astype(np.int64) + 15) // 16))
    assert r[0, 0] == 0 and r[-1, 1] == total
    assert np.all(r[1:, 0] == r[:-1, 1])             # contiguous, no gap, no overlap
    working = min(grid, min(total, max(1, total // 16)))  # >= 16 units per working CTA
    sizes = r[:working, 1] - r[:working, 0]
    assert total == 0 or sizes.min() >= min(16, total // working)  # no shredding
    assert sizes.max() - sizes.min() <= 1            # equal shares of 16-token units
    assert np.all(r[working:, 0] == r[working:, 1])


def test_partition_owner_formula(lib):
    """part_owner(u) (used by the combining CTA) is the CTA whose range holds u."""
    lengths = [37, 0, 1000, 16, 17, 5000]
    for grid in (1, 3, 7, 148, 592, 5000):
        total, r = partition(lib, lengths, 8, grid)
        g = min(grid, min(total, max(1, total // 16)))
        for u in range(0, total, max(1, total // 97)):
            owner = ((u + 1) * g + total - 1) // total - 1
            assert r[owner, 0] <= u < r[owner, 1]


def test_workspace_size_without_device(lib):
    # No GPU here: the fast-kernel part needs the device, the generic part does not.
    n = lib.pdb_paged_attention_workspace_size(256, 32, 8, 128, 8192, 1)
    assert n >= 256 * 32 * 16 * 130 * 4
    assert lib.pdb_paged_attention_workspace_size(0, 32, 8, 128, 8192, 1) == 0


def test_ops_reject_cpu_tensors(pkg):
    q = torch.zeros(2, 4, 32)
    k = torch.zeros(3, 16, 2, 32)
    with pytest.raises(RuntimeError, match="query must be on CUDA"):
        pkg.paged_attention(q, k, k, torch.zeros(2, 1, dtype=torch.int32),
                            torch.zeros(2, dtype=torch.int32), 16)
    with pytest.raises(RuntimeError, match="query must be on CUDA"):
        pkg.rope_kv_write(q, k[0], k[0], k, k, torch.zeros(2, dtype=torch.long),
                          torch.zeros(2, dtype=torch.long), torch.zeros(2, 1, dtype=torch.long),
                          torch.zeros(16))


def test_install_rebinds_module_global(pkg):
    import types
    mod = types.ModuleType("fake_llama")
    mod.cuda_paged_attention = None
    pkg.install(mod)
    assert mod.cuda_paged_attention is pkg.cuda_paged_attention


@pytest.mark.parametrize("units,launched", [(1, 296), (15, 296), (16, 296), (2048, 296),
                                            (9472, 296), (28415, 296), (28416, 296), (40000, 296),
                                            (163000, 296), (20000, 148), (7, 1), (100000, 1)])
def test_dynamic_partition_covers_units(lib, units, launched):
    """Static ranges + tail chunks partition [0, units) into non-empty,
    ordered ranges (no division by an empty tail), tail chunks >= one tile."""
    ranges = np.zeros(3 * launched * 6, dtype=np.int64)
    gs = lib.pdb_debug_dyn_partition(units, launched, ranges.ctypes.data, launched * 6)
    assert gs >= 1
    r = ranges.reshape(-1, 3)
    nw = int(np.count_nonzero(r[:, 1]))
    r = r[:nw]
    assert r[0, 0] == 0 and r[-1, 1] == units
    assert np.all(r[1:, 0] == r[:-1, 1])
    assert np.all(r[:, 1] > r[:, 0])
    assert np.all(r[:gs, 2] == 0) and np.all(r[gs:, 2] == 1)
    tail = r[gs:]
    if len(tail):
        assert np.all(tail[:, 1] - tail[:, 0] >= 16)  # four 64-token tiles
        assert tail[0, 0] == units - units // 16
    # short static shares (under 24 tiles of 4 units per launched CTA) get no tail
    if units < 24 * 4 * launched:
        assert len(tail) == 0


def test_prefill_and_decode_selector_checks(lib):
    """Kernel selectors and flags are validated before any CUDA call."""
    args = [None] * 6 + [2, 8, 4, 64, 16, 16, 2, 1, 1, None]
    assert lib.pdb_prefill_attention_impl(*args, 3) == 1
    assert "unknown prefill kernel" in _lib.last_error()
    assert lib.pdb_prefill_attention_impl(*args, -1) == 1
    dec = [None] * 9 + [2, 4, 64, 16, 16, 2, 1, 16, 0, 0, 1, None, 0, None]
    assert lib.pdb_decode_attention_ex(*dec, 4) == 1
    assert "unknown decode attention flags" in _lib.last_error()
    assert lib.pdb_decode_attention_ex(*dec, _lib.DECODE_STABLE_POOLS) == 1
    assert "requires PDB_DECODE_STABLE_METADATA" in _lib.last_error()


def prefill(lib, ptrs=None, **kw):
    a = dict(B=2, S=40, H=8, D=64, N=64, bs=16, KVH=2, W=4, dtype=1, impl=_lib.PREFILL_AUTO)
    a.update(kw)
    p = ptrs or [None] * 6
    return lib.pdb_prefill_attention_impl(*p, a["B"], a["S"], a["H"], a["D"], a["N"], a["bs"],
                                          a["KVH"], a["W"], a["dtype"], None, a["impl"])


@pytest.mark.parametrize("kw,msg", [
    (dict(dtype=0), "prefill attention takes FP16"),
    (dict(B=0), "invalid q shape"),
    (dict(S=0), "invalid q shape"),
    (dict(D=96), "prefill attention supports head_dim 64 and 128"),
    (dict(KVH=3), "query heads must be a multiple of KV heads"),
    (dict(W=0), "invalid cache shape"),
    (dict(bs=0), "invalid cache shape"),
    (dict(B=65536), "shape too large"),
    (dict(S=64 * 65535 + 1), "shape too large"),
    (dict(), "null tensor pointer"),
])
def test_prefill_argument_checks(lib, kw, msg):
    """pdb_prefill_attention_impl validates dtype, shapes, head_dim, the head
    grouping, the cache shape and the grid limits before its pointers."""
    assert prefill(lib, **kw) == 1
    assert _lib.last_error() == msg


@pytest.mark.skipif(torch.cuda.is_available(),
                    reason="uses made-up addresses: host-only checks, never a GPU")
@pytest.mark.parametrize("kw,ptrs,msg", [
    (dict(), [16, 8, 32, 48, 64, 80], "tensors must be 16-byte aligned"),
    (dict(bs=8, impl=_lib.PREFILL_TCGEN05), [16] * 6,
     "the tcgen05 prefill kernel needs block_size % 16 == 0"),
    (dict(N=1 << 27, impl=_lib.PREFILL_TCGEN05), [16] * 6,
     "the tcgen05 prefill kernel needs under 2^31 pool rows and query rows"),
])
def test_prefill_pointer_and_kernel_checks(lib, kw, ptrs, msg):
    """Past the null check: unaligned tensors, and a pinned tcgen05 kernel
    outside its block-size and row-count limits, are rejected on the host
    (the addresses are never dereferenced; no CUDA call is made)."""
    assert prefill(lib, ptrs, **kw) == 1
    assert _lib.last_error() == msg


def attn_impl(lib, ptrs=None, impl=0, **kw):
    a = dict(B=2, H=4, D=32, N=12, bs=16, KVH=2, Dk=32, W=3, max_length=35, dtype=0)
    a.update(kw)
    p = ptrs or [None] * 6
    return lib.pdb_paged_attention_impl(*p, a["B"], a["H"], a["D"], a["N"], a["bs"], a["KVH"],
                                        a["Dk"], a["W"], a["max_length"], a["dtype"], None, 0,
                                        None, impl)


def test_attention_impl_and_wrappers_checks(lib):
    """The kernel-pinned attention entry point and the decode / prefill
    wrappers run the same argument checks as the entry points they share
    them with; the support query rejects invalid shapes on any device."""
    assert attn_impl(lib, dtype=7) == 1 and _lib.last_error() == "use FP32 or FP16"
    assert attn_impl(lib, KVH=3) == 1
    assert _lib.last_error() == "query heads must be a multiple of KV heads"
    assert attn_impl(lib) == 1 and _lib.last_error() == "null tensor pointer"
    dec = [None] * 9 + [2, 4, 64, 16, 16, 2, 1, 16, 0, 0]
    assert lib.pdb_decode_attention(*dec, 7, None, 0, None) == 1
    assert _lib.last_error() == "use FP32 or FP16"
    assert lib.pdb_decode_attention(*dec, 1, None, 0, None) == 1
    assert _lib.last_error() == "null tensor pointer"
    pre = [None] * 6 + [2, 8, 4, 64, 16, 16, 2, 1]
    assert lib.pdb_prefill_attention(*pre, 0, None) == 1
    assert _lib.last_error() == "prefill attention takes FP16"
    assert lib.pdb_prefill_attention(*pre, 1, None) == 1
    assert _lib.last_error() == "null tensor pointer"
    for args in [(64, 9, 3, 64, 4096, 16, 7), (0, 9, 3, 64, 4096, 16, 1),
                 (64, 9, 0, 64, 4096, 16, 1), (64, 9, 2, 64, 4096, 16, 1)]:
        assert lib.pdb_decode_attention_supported(*args) == 0


@pytest.mark.skipif(torch.cuda.is_available(),
                    reason="uses made-up addresses: host-only checks, never a GPU")
@pytest.mark.parametrize("impl", [-1, _lib.IMPL_TMA_STATIC + 1])
def test_attention_unknown_kernel_selection(lib, impl):
    """An unknown kernel selector is rejected after the pointer checks, before
    any CUDA call (the addresses are never dereferenced)."""
    assert attn_impl(lib, [16] * 6, impl) == 1
    assert _lib.last_error() == "unknown kernel selection"


def test_prefill_ops_checks_without_device(pkg):
    """prefill_attention rejects CPU tensors before reaching the library."""
    q = torch.zeros(1, 4, 2, 64, dtype=torch.float16)
    kp = torch.zeros(2, 16, 1, 64, dtype=torch.float16)
    t = torch.zeros(1, 1, dtype=torch.int32)
    with pytest.raises(RuntimeError, match="CUDA"):
        pkg.prefill_attention(q, kp, kp, t, t[:, 0].contiguous())
