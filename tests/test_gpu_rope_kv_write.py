"""GPU parity of rope_kv_write (fused RoPE + paged KV-slot write).

Bars: rotated q/k within 2e-3 (FP16) / 1e-5 relative (FP32) of the
reference; written slots hold exactly the kernel's rotated k and the input v;
every other pool byte is unchanged (bit-exact)."""
from __future__ import annotations

import pytest
import torch

from conftest import REPO, golden_module, import_module
from gpu_helpers import assert_parity
from oracle import kv_cache, paged_attention as opa, rope as orope

pytestmark = pytest.mark.gpu

mg = golden_module()
W = import_module("workloads")


def gold(name):
    return torch.load(REPO / "tests" / "golden" / name, weights_only=False)


def exact_fraction(a, b):
    return (a.cpu() == b.cpu()).float().mean().item()


def test_rope_golden_positions(pkg, cuda):
    """Positions 0..8191 incl. page boundaries, both dtypes, three head dims."""
    for case in gold("rope_cases.pt"):
        spec = case["spec"]
        q, k, pos = mg.rope_inputs(spec)
        P = q.shape[1]
        v = torch.zeros_like(k)
        pool = torch.zeros(P, 1, k.shape[2], k.shape[3], dtype=q.dtype)
        phys = torch.arange(P, dtype=torch.int64)
        offs = torch.zeros(P, dtype=torch.int64)
        inv = W.inv_freq(spec["theta"], spec["D"]).to(cuda)
        qo, ko = pkg.rope_kv_write(q.to(cuda), k.to(cuda), v.to(cuda), pool.to(cuda),
                                   pool.clone().to(cuda), phys.to(cuda), offs.to(cuda),
                                   pos.to(cuda), inv)
        assert_parity(qo, case["q"], f"rope q {spec}")
        assert_parity(ko, case["k"], f"rope k {spec}")
        if q.dtype == torch.float16:
            assert exact_fraction(qo, case["q"]) > 0.999


def test_smollm_cpu_decode_step_matches_golden(pkg, cuda):
    """SmolLM2 FP32 decode step: rope_kv_write then paged_attention, against
    the reference's outputs; untouched pool bytes bit-exact."""
    g = gold("smollm_cpu_decode.pt")
    w = W.smollm_cpu()
    t = W.materialize(w, "cpu")
    kp, vp = t.k_pools[0].to(cuda), t.v_pools[0].to(cuda)
    qo, ko = pkg.rope_kv_write(t.q[0].to(cuda), t.k[0].to(cuda), t.v[0].to(cuda), kp, vp,
                               t.physical.to(cuda), t.offsets.to(cuda), t.positions.to(cuda),
                               t.inv_freq.to(cuda))
    out = pkg.paged_attention(qo, kp, vp, t.tables.to(cuda), t.lengths.to(cuda), w.max_length)
    assert_parity(qo, g["q_roped"], "q")
    assert_parity(ko, g["k_roped"], "k")
    assert_parity(out, g["out"], "attention")
    # pool: written slots == kernel's k / input v, everything else untouched
    exp_k, exp_v = t.k_pools[0].clone(), t.v_pools[0].clone()
    kv_cache.write_decode(exp_k, t.physical, t.offsets, ko.cpu())
    kv_cache.write_decode(exp_v, t.physical, t.offsets, t.v[0])
    assert torch.equal(kp.cpu(), exp_k) and torch.equal(vp.cpu(), exp_v)


@pytest.mark.parametrize("inplace", [False, True])
def test_decode_prologue_fp16(pkg, cuda, inplace):
    """SmolLM2 FP16 decode prologue (batch 64) against the oracle."""
    w = W.smollm_fp16(layers=1)
    t = W.materialize(w, cuda)
    k_before, v_before = t.k_pools[0].cpu(), t.v_pools[0].cpu()
    q_in, k_in, v_in = t.q[0].clone(), t.k[0].clone(), t.v[0].clone()
    qr, kr = orope.rope(q_in.cpu().unsqueeze(1), k_in.cpu().unsqueeze(1), w.positions(),
                        t.inv_freq.cpu(), exact_trig=True)
    qo, ko = pkg.rope_kv_write(t.q[0], t.k[0], t.v[0], t.k_pools[0], t.v_pools[0],
                               t.physical, t.offsets, t.positions, t.inv_freq, inplace=inplace)
    assert_parity(qo, qr[:, 0], "q")
    assert_parity(ko, kr[:, 0], "k")
    assert exact_fraction(qo, qr[:, 0]) > 0.999 and exact_fraction(ko, kr[:, 0]) > 0.999
    if inplace:
        assert qo.data_ptr() == t.q[0].data_ptr()
    else:
        assert torch.equal(t.q[0], q_in)
    exp_k, exp_v = k_before.clone(), v_before.clone()
    phys, off = w.slots()
    kv_cache.write_decode(exp_k, phys, off, ko.cpu())
    kv_cache.write_decode(exp_v, phys, off, v_in.cpu())
    assert torch.equal(t.k_pools[0].cpu(), exp_k)
    assert torch.equal(t.v_pools[0].cpu(), exp_v)


def test_prefill_write(pkg, cuda):
    """Prefill RoPE + KV write (16 prompts into a 4096-block pool): untouched
    blocks byte-for-byte, written slots equal the rotated k / input v."""
    g = gold("prefill.pt")
    pw = W.prefill_smollm()
    d = W.materialize_prefill(pw, "cpu")
    qr, kr = orope.rope(d["q"], d["k"], d["positions"], d["inv_freq"], exact_trig=True)
    dd = {k: v.to(cuda) for k, v in d.items()}
    qo, ko = pkg.rope_kv_write(dd["q"], dd["k"], dd["v"], dd["k_pool"], dd["v_pool"],
                               dd["physical"], dd["offsets"], dd["positions"], dd["inv_freq"],
                               valid=dd["valid"])
    assert_parity(qo, qr, "prefill q")
    assert_parity(ko, kr, "prefill k")
    exp_k, exp_v = d["k_pool"].clone(), d["v_pool"].clone()
    kv_cache.write_prefill(exp_k, d["physical"], d["offsets"], ko.cpu(), d["valid"])
    kv_cache.write_prefill(exp_v, d["physical"], d["offsets"], d["v"], d["valid"])
    assert torch.equal(dd["k_pool"].cpu(), exp_k)
    assert torch.equal(dd["v_pool"].cpu(), exp_v)
    touched = torch.zeros(pw.num_blocks, dtype=torch.bool)
    touched[d["physical"].unique()] = True
    assert torch.equal(dd["k_pool"].cpu()[~touched], d["k_pool"][~touched])
    # Against the reference's own pools (digests of tests/golden/prefill.pt).
    # v rows are copies: the v pool is byte-identical to the reference's.
    assert mg.digest(dd["v_pool"]) == g["v_pool_digest"]
    # The reference's k pool, restated on the CPU with its fp32 cos/sin
    # calls (the oracle's default path reproduces its digest).
    _, kr_ref = orope.rope(d["q"], d["k"], d["positions"], d["inv_freq"])
    ref_k = d["k_pool"].clone()
    kv_cache.write_prefill(ref_k, d["physical"], d["offsets"], kr_ref, d["valid"])
    assert mg.digest(ref_k) == g["k_pool_digest"]
    # The kernel's k pool equals the reference's wherever the reference's
    # fp32 cos/sin round to the correctly rounded FP16 values; where they do
    # not (a handful of angles, host dependent), it holds the correctly
    # rounded result instead.
    trig_differs = torch.zeros_like(ref_k, dtype=torch.bool)
    kv_cache.write_prefill(trig_differs, d["physical"], d["offsets"], kr_ref != kr, d["valid"])
    exact_k = d["k_pool"].clone()
    kv_cache.write_prefill(exact_k, d["physical"], d["offsets"], kr, d["valid"])
    got = dd["k_pool"].cpu()
    mismatch = got != ref_k
    unexplained = int((mismatch & ~trig_differs).sum())
    assert unexplained == 0, (f"{unexplained} k-pool elements differ from the reference "
                              f"where its cos/sin are correctly rounded")
    assert torch.equal(got[trig_differs], exact_k[trig_differs])
    assert int(trig_differs.sum()) <= 64, int(trig_differs.sum())
    assert pkg.read_device_errors() == 0


def test_prologue_then_attention_llama3(pkg, cuda):
    """Llama-3-8B shape, one layer, batch 256: prologue + attention on the GPU
    against the oracle pipeline for 8 sequences."""
    w = W.llama3_8b(layers=1)
    t = W.materialize(w, cuda)
    qo, ko = pkg.rope_kv_write(t.q[0], t.k[0], t.v[0], t.k_pools[0], t.v_pools[0],
                               t.physical, t.offsets, t.positions, t.inv_freq)
    out = pkg.paged_attention(qo, t.k_pools[0], t.v_pools[0], t.tables, t.lengths, w.max_length)
    qr, kr = orope.rope(t.q[0].cpu().unsqueeze(1), t.k[0].cpu().unsqueeze(1), w.positions(),
                        t.inv_freq.cpu(), exact_trig=True)
    assert_parity(qo, qr[:, 0], "q")
    assert_parity(ko, kr[:, 0], "k")
    from gpu_helpers import subset_pool
    pick = torch.argsort(w.lengths)[torch.tensor([0, 1, 64, 128, 200, 253, 254, 255])]
    tabs, (kp, vp) = subset_pool(w.tables[pick], w.lengths[pick], [t.k_pools[0], t.v_pools[0]],
                                 w.block_size)
    lens = w.lengths[pick]
    ref = opa.paged_attention(qo.cpu()[pick], kp, vp, tabs, lens, int(lens.max()))
    assert_parity(out.cpu()[pick], ref, "llama3 pipeline")


@pytest.mark.parametrize("dtype,D", [(torch.float16, 40), (torch.float32, 36), (torch.float16, 64)])
def test_rope_vector_and_scalar_paths(pkg, cuda, dtype, D):
    """head_dim*e a multiple of 32 bytes takes the vectorised kernel, other even
    head dims the scalar one; both match the oracle and write the same slots."""
    g = torch.Generator().manual_seed(D)
    B, H, KVH, N, bs = 5, 6, 2, 12, 8
    q = (torch.randn(B, 1, H, D, generator=g) * 2).to(dtype)
    k = (torch.randn(B, 1, KVH, D, generator=g) * 2).to(dtype)
    v = torch.randn(B, 1, KVH, D, generator=g).to(dtype)
    pos = torch.tensor([[0], [7], [8], [1000], [8191]], dtype=torch.int64)
    phys = torch.tensor([3, 0, 11, 5, 7], dtype=torch.int64)
    off = torch.tensor([0, 7, 3, 1, 6], dtype=torch.int64)
    inv = W.inv_freq(1e4, D)
    pool_k = torch.randn(N, bs, KVH, D, generator=g).to(dtype)
    pool_v = torch.randn(N, bs, KVH, D, generator=g).to(dtype)
    qr, kr = orope.rope(q, k, pos, inv, exact_trig=True)
    kd, vd = pool_k.to(cuda), pool_v.to(cuda)
    qo, ko = pkg.rope_kv_write(q.to(cuda), k.to(cuda), v.to(cuda), kd, vd, phys.to(cuda),
                               off.to(cuda), pos.to(cuda), inv.to(cuda))
    assert_parity(qo, qr, f"q D={D}")
    assert_parity(ko, kr, f"k D={D}")
    exp_k, exp_v = pool_k.clone(), pool_v.clone()
    kv_cache.write_decode(exp_k, phys, off, ko.cpu()[:, 0])
    kv_cache.write_decode(exp_v, phys, off, v[:, 0])
    assert torch.equal(kd.cpu(), exp_k) and torch.equal(vd.cpu(), exp_v)


@pytest.mark.parametrize("shape", [(21, 9, 3, 64), (24, 32, 8, 128)], ids=["smollm", "llama3"])
@pytest.mark.parametrize("shared_positions", [True, False])
def test_rope_many_short_rows(pkg, cuda, shared_positions, shape):
    """Many short rows: 21 sequences x 120 positions with SmolLM2 heads (more
    than 2048 rows of 72 16-byte work items: 8 rows per CTA, one warp per
    row), and 24 x 120 with Llama-3-8B heads (2 rows per CTA, four warps per
    row on named barriers, 1,440 CTAs: more than are resident at once). With
    positions shared across sequences (a prefill batch) and with sequences
    at different offsets, outputs match the oracle, the valid rows' slots
    hold the rotated k and the input v, and nothing else is written."""
    g = torch.Generator().manual_seed(31 if shared_positions else 32)
    B, H, KVH, D = shape
    S, N, bs = 120, 200, 16
    q = torch.randn(B, S, H, D, generator=g).half()
    k = torch.randn(B, S, KVH, D, generator=g).half()
    v = torch.randn(B, S, KVH, D, generator=g).half()
    pos = torch.arange(S)[None, :].expand(B, -1).clone()
    if not shared_positions:
        pos = pos + torch.randint(0, 3000, (B, 1), generator=g)
    lens = torch.randint(1, S + 1, (B,), generator=g)
    valid = torch.arange(S)[None, :] < lens[:, None]
    slots = torch.randperm(N * bs, generator=g)[: int(valid.sum())]
    phys, offs = slots // bs, slots % bs
    kp0 = torch.randn(N, bs, KVH, D, generator=g).half()
    vp0 = torch.randn(N, bs, KVH, D, generator=g).half()
    inv = W.inv_freq(1e5, D)
    kd, vd = kp0.to(cuda), vp0.to(cuda)
    qo, ko = pkg.rope_kv_write(q.to(cuda), k.to(cuda), v.to(cuda), kd, vd, phys.to(cuda),
                               offs.to(cuda), pos.to(cuda), inv.to(cuda), valid=valid.to(cuda))
    qr, kr = orope.rope(q, k, pos, inv, exact_trig=True)
    assert_parity(qo, qr, "q")
    assert_parity(ko, kr, "k")
    exp_k, exp_v = kp0.clone(), vp0.clone()
    kv_cache.write_prefill(exp_k, phys, offs, ko.cpu(), valid)
    kv_cache.write_prefill(exp_v, phys, offs, v, valid)
    assert torch.equal(kd.cpu(), exp_k) and torch.equal(vd.cpu(), exp_v)
    assert pkg.read_device_errors() == 0
