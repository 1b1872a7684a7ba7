"""Pin the CPU oracle against golden vectors produced by the reference's code.

tests/golden/*.pt were written by tests/golden/make_golden.py, which calls the
reference's torch_paged_attention, PagedLlama.rope, slot writes and
PagedKV.attention (worker/llama.py, worker/engine.py). The oracle restates
those algorithms; here it must reproduce them bit for bit (same torch ops,
same dtype), and the inputs regenerated from seeds must match the digests.
"""
from __future__ import annotations

import math

import pytest
import torch

from conftest import REPO, golden_module, import_module
from gpu_helpers import prefill_fixture_layer
from oracle import kv_cache, paged_attention as opa, rope as orope, scalar

mg = golden_module()

GOLD = REPO / "tests" / "golden"
W = import_module("workloads")


def load(name):
    return torch.load(GOLD / name, weights_only=False)


@pytest.mark.parametrize("dtype", ["float32", "float16"])
def test_reference_kernel_case(dtype):
    c = load("reference_kernel_case.pt")[dtype]
    out = opa.paged_attention(c["q"], c["keys"], c["values"], c["tables"], c["lengths"],
                              c["max_length"])
    assert torch.equal(out, c["out"])


def test_edge_cases_inputs_and_outputs():
    cases = load("edge_cases.pt")
    assert len(cases) == len(mg.edge_case_specs())
    for case in cases:
        q, k, v, tables, lengths, max_len = mg.edge_case_inputs(case["spec"])
        assert [mg.digest(t) for t in (q, k, v, tables, lengths)] == case["digests"], case["spec"]
        out = opa.paged_attention(q, k, v, tables, lengths, max_len)
        assert torch.equal(out, case["out"]), case["spec"]["name"]
        assert torch.all(out[lengths == 0] == 0)


def test_rope_cases():
    for case in load("rope_cases.pt"):
        spec = case["spec"]
        q, k, pos = mg.rope_inputs(spec)
        assert [mg.digest(q), mg.digest(k)] == case["digests"]
        qo, ko = orope.rope(q, k, pos, orope.inv_freq(spec["theta"], spec["D"]))
        assert torch.equal(qo, case["q"]) and torch.equal(ko, case["k"])


def test_inv_freq_matches_workloads():
    for theta, D in ((1e5, 64), (5e5, 128)):
        assert torch.equal(orope.inv_freq(theta, D), W.inv_freq(theta, D))


def test_smollm_cpu_decode_step():
    g = load("smollm_cpu_decode.pt")
    w = W.smollm_cpu()
    t = W.materialize(w, "cpu")
    assert torch.equal(w.lengths, g["lengths"]) and torch.equal(w.tables, g["tables"])
    assert mg.digest(t.k_pools[0]) == g["input_digests"]["k_pool"]
    assert mg.digest(t.q[0]) == g["input_digests"]["q"]
    qr, kr = orope.rope(t.q[0].unsqueeze(1), t.k[0].unsqueeze(1), t.positions, t.inv_freq)
    kp, vp = t.k_pools[0].clone(), t.v_pools[0].clone()
    kv_cache.write_decode(kp, t.physical, t.offsets, kr[:, 0])
    kv_cache.write_decode(vp, t.physical, t.offsets, t.v[0])
    out = opa.paged_attention(qr[:, 0], kp, vp, t.tables, t.lengths, w.max_length)
    assert torch.equal(qr[:, 0], g["q_roped"]) and torch.equal(kr[:, 0], g["k_roped"])
    assert mg.digest(kp) == g["k_pool_digest"] and mg.digest(vp) == g["v_pool_digest"]
    assert torch.equal(out, g["out"])


def test_prefill_write():
    g = load("prefill.pt")
    pw = W.prefill_smollm()
    d = W.materialize_prefill(pw, "cpu")
    for key in ("q", "k", "v", "k_pool", "v_pool"):
        assert mg.digest(d[key]) == g["input_digests"][key], key
    qr, kr = orope.rope(d["q"], d["k"], d["positions"], d["inv_freq"])
    kp, vp = d["k_pool"].clone(), d["v_pool"].clone()
    kv_cache.write_prefill(kp, d["physical"], d["offsets"], kr, d["valid"])
    kv_cache.write_prefill(vp, d["physical"], d["offsets"], d["v"], d["valid"])
    assert mg.digest(qr) == g["q_roped_digest"] and mg.digest(kr) == g["k_roped_digest"]
    assert mg.digest(kp) == g["k_pool_digest"] and mg.digest(vp) == g["v_pool_digest"]


def test_scalar_known_answer():
    g = load("scalar_known_answer.pt")["scalar"]
    keys = [[None, None], [None, None]]
    vals = [[None, None], [None, None]]
    for i, (kk, vv) in enumerate(zip(g["keys"], g["values"])):
        blk, off = g["table"][i // g["block_size"]], i % g["block_size"]
        keys[blk][off], vals[blk][off] = kk, vv
    got = scalar.attention(g["q"], keys, vals, g["table"], 3, g["block_size"])
    for a, b in zip(got, g["out"]):
        assert math.isclose(a, b, rel_tol=1e-12, abs_tol=1e-12)
    # the same answer from the vectorised oracle in float64
    q = torch.tensor([g["q"]], dtype=torch.float64)[:, None, :]
    kt = torch.zeros(2, 2, 1, 2, dtype=torch.float64)
    vt = torch.zeros_like(kt)
    for i, (kk, vv) in enumerate(zip(g["keys"], g["values"])):
        blk, off = g["table"][i // 2], i % 2
        kt[blk, off, 0] = torch.tensor(kk)
        vt[blk, off, 0] = torch.tensor(vv)
    out = opa.paged_attention(q, kt, vt, torch.tensor([g["table"]], dtype=torch.int32),
                              torch.tensor([3], dtype=torch.int32), 3)
    assert torch.allclose(out[0, 0], torch.tensor(g["out"], dtype=torch.float64), atol=1e-12)


def test_oracle_close_to_float64():
    """The reference's FP32 path is within ~1e-6 of the exact answer on the
    SmolLM2 CPU workload; this bounds what an FP32 kernel can be held to."""
    g = load("smollm_cpu_decode.pt")
    w = W.smollm_cpu()
    t = W.materialize(w, "cpu")
    kp, vp = t.k_pools[0].clone(), t.v_pools[0].clone()
    kv_cache.write_decode(kp, t.physical, t.offsets, g["k_roped"])
    kv_cache.write_decode(vp, t.physical, t.offsets, t.v[0])
    exact = opa.paged_attention_fp64(g["q_roped"], kp, vp, t.tables, t.lengths)
    err = (g["out"].double() - exact).abs().max().item()
    assert err < 2e-6


def test_allocator_restatement():
    """TensorPagedKV behaviour: LIFO free list, whole-request reservation,
    release without clearing, metadata padding with block 0."""
    c = kv_cache.PagedKVCache(layers=1, kv_heads=1, head_dim=2, blocks=8, block_size=4)
    assert c.reserve("a", 9)          # 3 pages
    assert c.tables["a"] == [0, 1, 2]
    assert not c.reserve("b", 40)
    assert c.reserve("b", 4)
    c.lengths["a"], c.lengths["b"] = 9, 3
    phys, off = c.slots(["a", "b"], [[8], [2]])
    assert phys.tolist() == [2, 3] and off.tolist() == [0, 2]
    tables, lengths, max_len = c.metadata(["a", "b"])
    assert tables.tolist() == [[0, 1, 2], [3, 0, 0]] and lengths.tolist() == [9, 3] and max_len == 9
    c.keys[0, 3] = 5.0
    c.release("b")
    assert c.free[-1] == 3 and float(c.keys[0, 3].sum()) != 0.0   # not cleared
    with pytest.raises(ValueError):
        c.reserve("a", 1)


@pytest.mark.parametrize("dtype", ["float32", "float16"])
def test_prefill_attention_fixture(dtype):
    """The reference's PagedLlama.prefill attention (worker/llama.py:141-144)
    on a seeded tiny Llama: ragged prompts on fragmented, reused pages. The
    oracle's call in the inputs' dtype is the reference's bit for bit; its
    fp32 form (what the GPU kernels are held to) is within one FP16 ulp of
    the FP16 reference and equal to the FP32 one."""
    case = load("prefill_attention.pt")[dtype]
    assert case["dtype"] == dtype and case["spec"] == mg.PREFILL_ATTENTION
    for layer in range(len(case["layers"])):
        q, k, v, ctx, valid = prefill_fixture_layer(case, layer)
        native = opa.prefill_attention(q, k, v, native=True)
        assert native.dtype == q.dtype
        assert torch.equal(native[valid], ctx[valid]), f"layer {layer}"
        f32 = opa.prefill_attention(q, k, v)
        if dtype == "float32":
            assert torch.equal(f32[valid], ctx[valid])
        else:
            err = (f32[valid].half().float() - ctx[valid].float()).abs()
            assert err.max().item() <= 1e-3, f"layer {layer}: {err.max().item()}"


def test_prefill_attention_fixture_layout():
    """Pages of the fixture's prompts are fragmented and reused (the earlier
    requests' rows were released uncleared), and the prompts cross pages."""
    case = load("prefill_attention.pt")["float16"]
    lens = case["lengths"].tolist()
    bs = case["spec"]["block_size"]
    assert lens == list(case["spec"]["prompts"].values())
    assert any(n % bs for n in lens) and any(n % bs == 0 for n in lens) and 1 in lens
    used = [int(p) for b, n in enumerate(lens) for p in case["tables"][b, :(n + bs - 1) // bs]]
    assert len(set(used)) == len(used)
    assert any(b - a != 1 for a, b in zip(used, used[1:]))
