"""The reference's own CUDA kernel (cuda/paged_attention.cu, built from the
reference checkout into oracle/_ref/ by oracle/build_ref.py) as a second GPU
oracle: it must agree with the CPU oracle, and this library must agree with it."""
from __future__ import annotations

import pytest
import torch

from conftest import REPO, import_module
from gpu_helpers import assert_parity
from oracle import build_ref

pytestmark = pytest.mark.gpu
W = import_module("workloads")


@pytest.fixture(scope="module")
def ref_kernel():
    mod = build_ref.load_ref_module()
    if mod is None:
        pytest.skip("reference kernel was not built (no reference checkout at build time)")
    return mod


@pytest.mark.parametrize("dtype", ["float32", "float16"])
def test_reference_kernel_matches_golden(ref_kernel, cuda, dtype):
    c = torch.load(REPO / "tests" / "golden" / "reference_kernel_case.pt", weights_only=False)[dtype]
    out = ref_kernel.paged_attention(c["q"].to(cuda), c["keys"].to(cuda), c["values"].to(cuda),
                                     c["tables"].to(cuda), c["lengths"].to(cuda), c["max_length"])
    assert_parity(out, c["out"], "reference kernel vs golden")


@pytest.mark.parametrize("make", ["smollm_fp16", "llama3_8b"])
def test_matches_reference_kernel(pkg, ref_kernel, cuda, make):
    w = W.smollm_fp16(layers=1) if make == "smollm_fp16" else W.llama3_8b(batch=64, layers=1)
    t = W.materialize(w, cuda)
    args = (t.q[0], t.k_pools[0], t.v_pools[0], t.tables, t.lengths, w.max_length)
    ours = pkg.paged_attention(*args)
    theirs = ref_kernel.paged_attention(*args)
    assert_parity(ours, theirs.cpu(), f"{make}: ours vs reference kernel")
