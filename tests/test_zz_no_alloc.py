"""pdb_paged_attention_noalloc: the decode attention entry point for callers
that cannot allocate device memory (an engine that owns the memory budget and
gives plugins no allocator, a loop that must not call cudaMalloc/cudaFree).

It must give the same result as pdb_paged_attention (same tolerance as every
parity test), call after call, although its scratch is one fixed array shared
by every call on the device; and, like every kernel here, the reference's
result (the CPU oracle, and the golden outputs the reference's own code wrote).
The inputs and outputs here are allocated by the test, as a caller would; the
entry point itself allocates nothing.

This file sorts last so that a run stopping at the first failure has run
every other test before it.
"""
from __future__ import annotations

import ctypes

import pytest
import torch

from conftest import REPO, golden_module, import_module
from gpu_helpers import assert_matches_oracle, assert_parity

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
    # the largest shape the header quotes (Llama-3-8B at batch 256, ~1.3 MB)
    "llama3-8b fp16 batch 256": lambda: W.llama3_8b(batch=256, layers=1),
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
    assert_matches_oracle(out, t.q[0], w.tables, w.lengths, [t.k_pools[0], t.v_pools[0]],
                          w.block_size, f"{name} vs oracle")
    assert pkg.read_device_errors() == 0


def test_matches_reference_goldens(pkg, cuda):
    """The reference's own outputs on its kernel test case and on the edge
    cases (zero length, page-boundary lengths, MHA / GQA / MQA, several head
    dims and block sizes, FP32 and FP16). Shapes only the generic kernel
    handles are refused with a message; every other case must match."""
    gold = REPO / "tests" / "golden"
    cases = []
    for dtype, c in torch.load(gold / "reference_kernel_case.pt", weights_only=False).items():
        cases.append((f"kernel case {dtype}", c["q"], c["keys"], c["values"], c["tables"],
                      c["lengths"], c["max_length"], c["out"]))
    mg = golden_module()
    for e in torch.load(gold / "edge_cases.pt", weights_only=False):
        q, k, v, tables, lengths, max_len = mg.edge_case_inputs(e["spec"])
        cases.append((e["spec"]["name"], q, k, v, tables, lengths, max_len, e["out"]))
    accepted = 0
    for name, q, k, v, tables, lengths, max_len, ref in cases:
        dev = [x.to(cuda) for x in (q, k, v, tables, lengths)]
        for call in range(2):
            out = torch.full_like(dev[0], float("nan"))
            rc = call_noalloc(*dev, max_len, out)
            if rc != 0:
                assert rc == 1 and "generic kernel" in _lib.last_error(), (name, rc)
                break
            torch.cuda.synchronize()
            assert_parity(out, ref, f"{name}, call {call + 1}")
        else:
            accepted += 1
    assert accepted >= 15, accepted  # 15 of the 20 cases fit a stream-K kernel
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
