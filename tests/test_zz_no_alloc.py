"""pdb_paged_attention_noalloc: the decode attention entry point for callers
that cannot allocate device memory (an engine that owns the memory budget and
gives plugins no allocator, a loop that must not call cudaMalloc/cudaFree).

It must give the same result as pdb_paged_attention (same tolerance as every
parity test), call after call, although its scratch is one fixed array shared
by every call on the device. The inputs and outputs here are allocated by the
test, as a caller would; the entry point itself allocates nothing.

This file sorts last so that a run stopping at the first failure has run
every other test before it.
"""
from __future__ import annotations

import ctypes

import pytest
import torch

from conftest import import_module
from gpu_helpers import assert_parity

pytestmark = pytest.mark.gpu

W = import_module("workloads")
_lib = import_module("_lib")


def call_noalloc(q, k, v, tables, lengths, max_length, out):
    lib = _lib.load()
    B, H, D = q.shape
    N, bs, KVH, Dk = k.shape
    dtype = _lib.DTYPE_FLOAT16 if q.dtype == torch.float16 else _lib.DTYPE_FLOAT32
    stream = torch.cuda.current_stream(q.device).cuda_stream
    return lib.pdb_paged_attention_noalloc(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), tables.data_ptr(), lengths.data_ptr(),
        out.data_ptr(), B, H, D, N, bs, KVH, Dk, tables.size(1), int(max_length), dtype, stream)


WORKLOADS = {
    "llama3-8b fp16 batch 48": lambda: W.llama3_8b(batch=48, layers=1),
    "smollm2 fp16 batch 32": lambda: W.smollm_fp16(batch=32, layers=1),
    "smollm2 fp32 batch 4": lambda: W.smollm_cpu(),
}


@pytest.mark.parametrize("name", list(WORKLOADS))
def test_matches_workspace_entry_point_on_consecutive_calls(pkg, cuda, name):
    w = WORKLOADS[name]()
    t = W.materialize(w, cuda)
    args = (t.q[0], t.k_pools[0], t.v_pools[0], t.tables, t.lengths, w.max_length)
    expected = pkg.paged_attention(*args)
    for call in range(2):
        out = torch.full_like(t.q[0], float("nan"))
        rc = call_noalloc(*args, out)
        assert rc == 0, _lib.last_error()
        torch.cuda.synchronize()
        assert_parity(out, expected.cpu(), f"{name}, call {call + 1}")
    assert pkg.read_device_errors() == 0


def test_rejects_shapes_beyond_the_fixed_scratch(pkg, cuda):
    # 4096 sequences x 128 kv heads: the per-(sequence, kv head) arrival
    # counters alone fill the fixed array. Lengths are zero, so even a wrong
    # launch would read no pages.
    B, H, KVH, D, bs = 4096, 128, 128, 64, 16
    q = torch.zeros(B, H, D, dtype=torch.float16, device=cuda)
    k = torch.zeros(4, bs, KVH, D, dtype=torch.float16, device=cuda)
    tables = torch.zeros(B, 1, dtype=torch.int32, device=cuda)
    lengths = torch.zeros(B, dtype=torch.int32, device=cuda)
    out = torch.empty_like(q)
    rc = call_noalloc(q, k, k, tables, lengths, 16, out)
    torch.cuda.synchronize()
    assert rc == 2, f"status {rc}: {_lib.last_error()}"
    assert "fixed maximum" in _lib.last_error()
