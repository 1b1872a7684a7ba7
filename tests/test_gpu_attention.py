"""GPU parity of paged_attention (both kernels) against the golden vectors and
the CPU oracle, on the reference's own test case, its edge cases, the
SmolLM2 and Llama-3-8B shaped workloads and random shapes."""
from __future__ import annotations

import math

import pytest
import torch

from conftest import REPO, golden_module, import_module
from gpu_helpers import assert_matches_oracle, assert_parity, subset_pool
from oracle import paged_attention as opa

pytestmark = pytest.mark.gpu

mg = golden_module()
W = import_module("workloads")
_lib = import_module("_lib")
IMPLS = [_lib.IMPL_AUTO, _lib.IMPL_FAST, _lib.IMPL_GENERIC, _lib.IMPL_SIMT, _lib.IMPL_MMA,
         _lib.IMPL_TMA_STATIC]
STREAMK = (_lib.IMPL_FAST, _lib.IMPL_SIMT, _lib.IMPL_MMA, _lib.IMPL_TMA_STATIC)


def gold(name):
    return torch.load(REPO / "tests" / "golden" / name, weights_only=False)


def run(pkg, q, k, v, tables, lengths, max_length, impl, dev):
    try:
        out = pkg.paged_attention(q.to(dev), k.to(dev), v.to(dev), tables.to(dev),
                                  lengths.to(dev), max_length, impl=impl)
    except RuntimeError as e:
        if impl in STREAMK and "fast kernel does not support" in str(e):
            pytest.skip("shape outside the stream-K kernel's instantiations")
        raise
    torch.cuda.synchronize()
    return out.cpu()


@pytest.mark.parametrize("impl", IMPLS)
@pytest.mark.parametrize("dtype", ["float32", "float16"])
def test_reference_kernel_case(pkg, cuda, dtype, impl):
    """tests/test_llama.py:123-134 of the reference: fragmented pages, lengths 1/17/35."""
    c = gold("reference_kernel_case.pt")[dtype]
    out = run(pkg, c["q"], c["keys"], c["values"], c["tables"], c["lengths"], c["max_length"],
              impl, cuda)
    assert_parity(out, c["out"], f"{dtype} impl={impl}")


@pytest.mark.parametrize("impl", IMPLS)
def test_edge_cases(pkg, cuda, impl):
    ran = 0
    for case in gold("edge_cases.pt"):
        q, k, v, tables, lengths, max_len = mg.edge_case_inputs(case["spec"])
        try:
            out = pkg.paged_attention(q.to(cuda), k.to(cuda), v.to(cuda), tables.to(cuda),
                                      lengths.to(cuda), max_len, impl=impl).cpu()
        except RuntimeError as e:
            if impl in STREAMK and "fast kernel does not support" in str(e):
                continue
            raise
        assert_parity(out, case["out"], case["spec"]["name"])
        assert torch.all(out[lengths == 0] == 0)
        ran += 1
    assert ran >= (4 if impl in (_lib.IMPL_MMA, _lib.IMPL_TMA_STATIC) else 8)


@pytest.mark.parametrize("impl", IMPLS)
@pytest.mark.parametrize("dtype", ["float32", "float16"])
def test_stale_pool_bytes_are_never_read(pkg, cuda, dtype, impl):
    """Every pool slot outside [0, len) of its sequence is NaN: the result must
    be bit-identical to the run on a clean pool (reads bounded by lengths)."""
    spec = [s for s in mg.edge_case_specs() if s["dtype"] == dtype][4]  # 32/8 heads, D 128
    q, k, v, tables, lengths, max_len = mg.edge_case_inputs(spec)
    clean = run(pkg, q, k, v, tables, lengths, max_len, impl, cuda)
    bs = k.shape[1]
    live = torch.zeros(k.shape[0], bs, dtype=torch.bool)
    for b, n in enumerate(lengths.tolist()):
        for t in range(n):
            live[tables[b, t // bs], t % bs] = True
    kn, vn = k.clone(), v.clone()
    kn[~live] = float("nan")
    vn[~live] = float("nan")
    poisoned = run(pkg, q, kn, vn, tables, lengths, max_len, impl, cuda)
    assert torch.equal(clean, poisoned)


@pytest.mark.parametrize("impl", [_lib.IMPL_FAST, _lib.IMPL_GENERIC, _lib.IMPL_SIMT, _lib.IMPL_MMA,
                                  _lib.IMPL_TMA_STATIC])
def test_repeated_calls_are_deterministic(pkg, cuda, impl):
    """Bit-identical results call after call (the dynamic tail changes which
    CTA runs a chunk, not the result)."""
    w = W.llama3_8b(batch=96, layers=1)
    t = W.materialize(w, cuda)
    outs = [pkg.paged_attention(t.q[0], t.k_pools[0], t.v_pools[0], t.tables, t.lengths,
                                w.max_length, impl=impl) for _ in range(5)]
    torch.cuda.synchronize()
    for o in outs[1:]:
        assert torch.equal(o, outs[0])


@pytest.mark.parametrize("impl", [_lib.IMPL_FAST, _lib.IMPL_TMA_STATIC, _lib.IMPL_MMA,
                                  _lib.IMPL_SIMT])
def test_cuda_graph_replays_match_eager(pkg, cuda, impl):
    """Calls captured once in a CUDA graph keep their call tags on every
    replay, so the arrival and tail-claim counters must be back at zero when
    a call ends. Two calls per graph share the stream's workspace; each replay
    with fresh queries matches eager calls bit for bit."""
    w = W.llama3_8b(batch=96, layers=2)
    t = W.materialize(w, cuda)
    q = t.q[0].clone()
    outs = [torch.empty_like(q) for _ in range(2)]
    s = torch.cuda.Stream()

    def call(i, out=None):
        return pkg.paged_attention(q, t.k_pools[i], t.v_pools[i], t.tables, t.lengths,
                                   w.max_length, out=out, impl=impl)

    with torch.cuda.stream(s):
        call(0, outs[0]), call(1, outs[1])  # workspace and kernel attributes set up
        s.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            call(0, outs[0])
            call(1, outs[1])
        gen = torch.Generator(device=cuda).manual_seed(3)
        for _ in range(3):
            q.copy_(torch.randn(q.shape, generator=gen, device=cuda).to(q.dtype))
            g.replay()
            eager = [call(0), call(1)]
            s.synchronize()
            for i in range(2):
                assert torch.equal(outs[i], eager[i]), f"replay differs from eager (layer {i})"
    del g
    assert pkg.read_device_errors() == 0


@pytest.mark.parametrize("layout", ["long_last", "long_first", "zeros_mixed"])
def test_tail_order_with_skewed_lengths(pkg, cuda, layout):
    """Batches whose long sequences sit at the end (index order would put
    them in the dynamically scheduled tail), at the start, or mixed with empty
    sequences: the tensor-core kernels agree with the generic kernel
    everywhere and with the CPU oracle on the long and the empty sequences."""
    g = torch.Generator().manual_seed(11)
    B, H, KVH, D, bs = 160, 32, 8, 128, 16
    lengths = torch.randint(64, 400, (B,), generator=g).to(torch.int32)
    if layout == "long_last":
        lengths[-6:] = torch.tensor([8192, 7000, 6100, 8000, 5000, 7777], dtype=torch.int32)
    elif layout == "long_first":
        lengths[:6] = torch.tensor([8192, 7000, 6100, 8000, 5000, 7777], dtype=torch.int32)
    else:
        lengths[::7] = 0
        lengths[3::11] = 6000
    need = (lengths.to(torch.int64) + bs - 1) // bs
    width = int(need.max())
    N = int(need.sum()) + 5
    perm = torch.randperm(N, generator=g)
    tables = torch.zeros(B, width, dtype=torch.int32)
    off = 0
    for b, n in enumerate(need.tolist()):
        tables[b, :n] = perm[off:off + n].to(torch.int32)
        off += n
    q = torch.randn(B, H, D, generator=g).half()
    k = torch.randn(N, bs, KVH, D, generator=g).half()
    v = torch.randn(N, bs, KVH, D, generator=g).half()
    args = (q.to(cuda), k.to(cuda), v.to(cuda), tables.to(cuda), lengths.to(cuda),
            int(lengths.max()))
    generic = pkg.paged_attention(*args, impl=_lib.IMPL_GENERIC).cpu()
    fast = pkg.paged_attention(*args, impl=_lib.IMPL_FAST).cpu()
    static = pkg.paged_attention(*args, impl=_lib.IMPL_TMA_STATIC).cpu()
    assert_parity(fast, generic, f"{layout}: dynamic vs generic")
    assert_parity(static, generic, f"{layout}: static vs generic")
    order = torch.argsort(lengths)
    pick = torch.cat([order[:4], order[-6:]]).unique()
    tabs, (kp, vp) = subset_pool(tables[pick], lengths[pick], [k, v], bs)
    lens = lengths[pick]
    ref = opa.paged_attention(q[pick], kp, vp, tabs, lens, int(lens.max()))
    assert_parity(fast[pick], ref, f"{layout}: dynamic vs oracle")
    assert pkg.read_device_errors() == 0


def test_smollm_fp16_layer(pkg, cuda):
    """SmolLM2 FP16 workload (batch 64, len U[128, 2048]), one layer vs the oracle."""
    w = W.smollm_fp16(layers=1)
    t = W.materialize(w, cuda)
    out = pkg.paged_attention(t.q[0], t.k_pools[0], t.v_pools[0], t.tables, t.lengths,
                              w.max_length)
    ref = opa.paged_attention(t.q[0].cpu(), t.k_pools[0].cpu(), t.v_pools[0].cpu(),
                              w.tables, w.lengths, w.max_length)
    assert_parity(out, ref, "smollm fp16")


def test_llama3_full_batch(pkg, cuda):
    """Llama-3-8B shape at the full batch of 256, one layer: the default
    kernel matches the CPU oracle on every one of the 256 sequences (checked
    in chunks of 32 sequences of similar length, each chunk's pages copied to
    the CPU and padded to the chunk's longest, as the reference pads to the
    batch's), and the four other kernels (TMA-fed static schedule, cp.async
    tensor-core and SIMT stream-K, generic split) agree with it."""
    w = W.llama3_8b(layers=1)
    t = W.materialize(w, cuda)
    args = (t.q[0], t.k_pools[0], t.v_pools[0], t.tables, t.lengths, w.max_length)
    fast = pkg.paged_attention(*args, impl=_lib.IMPL_FAST).cpu()
    checked = assert_matches_oracle(fast, t.q[0], w.tables, w.lengths,
                                    [t.k_pools[0], t.v_pools[0]], w.block_size, "llama3")
    assert checked == w.batch == 256
    for impl, name in ((_lib.IMPL_GENERIC, "generic split"),
                       (_lib.IMPL_TMA_STATIC, "tma tensor-core (static)"),
                       (_lib.IMPL_SIMT, "simt"), (_lib.IMPL_MMA, "cp.async tensor-core")):
        assert_parity(pkg.paged_attention(*args, impl=impl), fast, f"{name} vs default")


@pytest.mark.parametrize("seed", range(6))
def test_random_shapes(pkg, cuda, seed):
    g = torch.Generator().manual_seed(seed)
    dtype = [torch.float32, torch.float16][seed % 2]
    D = [32, 64, 128][seed % 3]
    KVH = [1, 2, 4][(seed // 2) % 3]
    G = [1, 2, 3, 4][seed % 4]
    H = KVH * G
    bs = [8, 16, 32][(seed // 3) % 3]
    B = int(torch.randint(1, 40, (1,), generator=g))
    lengths = torch.randint(0, 700, (B,), generator=g).to(torch.int32)
    lengths[0] = max(int(lengths[0]), 1)
    max_len = int(lengths.max())
    need = ((lengths.to(torch.int64) + bs - 1) // bs)
    N = int(need.sum()) + 3
    perm = torch.randperm(N, generator=g)
    width = math.ceil(max_len / bs)
    tables = torch.zeros(B, width, dtype=torch.int32)
    off = 0
    for b, n in enumerate(need.tolist()):
        tables[b, :n] = perm[off:off + n].to(torch.int32)
        off += n
    q = torch.randn(B, H, D, generator=g).to(dtype)
    k = torch.randn(N, bs, KVH, D, generator=g).to(dtype)
    v = torch.randn(N, bs, KVH, D, generator=g).to(dtype)
    ref = opa.paged_attention(q, k, v, tables, lengths, max_len)
    for impl in IMPLS:
        try:
            out = pkg.paged_attention(q.to(cuda), k.to(cuda), v.to(cuda), tables.to(cuda),
                                      lengths.to(cuda), max_len, impl=impl).cpu()
        except RuntimeError as e:
            assert impl in STREAMK and "fast kernel does not support" in str(e)
            continue
        assert_parity(out, ref, f"seed {seed} impl {impl}")


def test_no_device_errors_raised(pkg, cuda):
    assert pkg.read_device_errors() == 0


@pytest.mark.parametrize("shape", ["llama3", "smollm", "smollm_fp32", "llama3_fp32"])
def test_fused_decode_layer_equals_two_launches(pkg, cuda, shape):
    """decode_attention (RoPE + slot writes folded into the attention kernel)
    is bit-identical to rope_kv_write_decode + paged_attention: same output,
    same pool bytes everywhere; FP16 (tensor-core inner loop) and FP32 (SIMT
    inner loop), head_dim 64 and 128."""
    import dataclasses
    g = torch.Generator().manual_seed(17)
    if shape == "llama3":
        w = W.llama3_8b(batch=96, layers=1)
    elif shape == "llama3_fp32":
        w = dataclasses.replace(W.llama3_8b(batch=32, layers=1), dtype=torch.float32)
    elif shape == "smollm":
        w = W.smollm_fp16(batch=64, layers=1)
    else:
        w = W.smollm_fp32(batch=64, layers=1)
    B, H, KVH, D = w.batch, w.heads, w.kv_heads, w.head_dim
    t = W.materialize(w, cuda)
    q = torch.randn(B, H, D, generator=g).to(w.dtype).to(cuda)
    k = torch.randn(B, KVH, D, generator=g).to(w.dtype).to(cuda)
    v = torch.randn(B, KVH, D, generator=g).to(w.dtype).to(cuda)
    assert pkg.decode_attention_supported(q, t.k_pools[0])
    kp1, vp1 = t.k_pools[0].clone(), t.v_pools[0].clone()
    kp2, vp2 = t.k_pools[0].clone(), t.v_pools[0].clone()
    fused = pkg.decode_attention(q, k, v, kp1, vp1, t.tables, t.lengths, t.inv_freq,
                                 w.max_length)
    qr, _ = pkg.rope_kv_write_decode(q, k, v, kp2, vp2, t.tables, t.lengths, t.inv_freq)
    two = pkg.paged_attention(qr, kp2, vp2, t.tables, t.lengths, w.max_length)
    torch.cuda.synchronize()
    assert torch.equal(fused, two)
    assert torch.equal(kp1, kp2) and torch.equal(vp1, vp2)
    assert not torch.equal(kp1, t.k_pools[0])  # the new tokens were written
    assert pkg.read_device_errors() == 0


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_fused_decode_layer_reads_projection_slices(pkg, cuda, dtype):
    """q, k and v given as row slices of one fused q/k/v projection output
    (row stride (H + 2*KVH) * D) give the same output and pool bytes as
    contiguous copies, in FP16 and FP32 (whose slices stay 16-byte aligned:
    960-float rows, k and v at 576 and 768 floats)."""
    g = torch.Generator().manual_seed(19)
    if dtype == torch.float16:
        w = W.smollm_fp16(batch=48, layers=1)
    else:
        w = W.smollm_fp32(batch=48, layers=1)
    t = W.materialize(w, cuda)
    B, H, KVH, D = 48, 9, 3, 64
    qkv = torch.randn(B, (H + 2 * KVH) * D, generator=g).to(dtype).to(cuda)
    q = qkv[:, :H * D].view(B, H, D)
    k = qkv[:, H * D:(H + KVH) * D].view(B, KVH, D)
    v = qkv[:, (H + KVH) * D:].view(B, KVH, D)
    kp1, vp1 = t.k_pools[0].clone(), t.v_pools[0].clone()
    kp2, vp2 = t.k_pools[0].clone(), t.v_pools[0].clone()
    a = pkg.decode_attention(q, k, v, kp1, vp1, t.tables, t.lengths, t.inv_freq, w.max_length)
    b = pkg.decode_attention(q.contiguous(), k.contiguous(), v.contiguous(), kp2, vp2, t.tables,
                             t.lengths, t.inv_freq, w.max_length)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    assert torch.equal(kp1, kp2) and torch.equal(vp1, vp2)
    assert pkg.read_device_errors() == 0


@pytest.mark.parametrize("shape", ["llama3", "smollm", "smollm_fp32"])
def test_fused_decode_stable_metadata_is_identical(pkg, cuda, shape):
    """A decode step of 4 layers launched back to back with
    metadata_stable=True for layers 1..3 (plan and page lookups before the
    dependent-launch wait) gives the same outputs and pool bytes as the
    same step without it, eagerly and replayed from a CUDA graph; FP16 and
    FP32 (the SIMT inner loop)."""
    if shape == "llama3":
        w = W.llama3_8b(batch=40, layers=4)
    elif shape == "smollm":
        w = W.smollm_fp16(batch=64, layers=4)
    else:
        w = W.smollm_fp32(batch=64, layers=4)
    t = W.materialize(w, cuda)
    pools0 = [(kp.clone(), vp.clone()) for kp, vp in zip(t.k_pools, t.v_pools)]

    def step(stable, outs):
        for layer in range(w.layers):
            pkg.decode_attention(t.q[layer], t.k[layer], t.v[layer], t.k_pools[layer],
                                 t.v_pools[layer], t.tables, t.lengths, t.inv_freq,
                                 w.max_length, out=outs[layer],
                                 metadata_stable=stable and layer > 0,
                                 pools_stable=stable and layer > 0)

    def reset():  # on the current stream, then complete before the step's stream runs
        for (kp, vp), (k0, v0) in zip(zip(t.k_pools, t.v_pools), pools0):
            kp.copy_(k0)
            vp.copy_(v0)
        torch.cuda.synchronize()

    ref = [torch.empty_like(q) for q in t.q]
    got = [torch.empty_like(q) for q in t.q]
    s = torch.cuda.Stream(cuda)
    with torch.cuda.stream(s):
        step(False, ref)
    torch.cuda.synchronize()
    ref_pools = [(kp.clone(), vp.clone()) for kp, vp in zip(t.k_pools, t.v_pools)]
    reset()
    with torch.cuda.stream(s):
        step(True, got)
    torch.cuda.synchronize()
    for a, b in zip(got, ref):
        assert torch.equal(a, b)
    for (kp, vp), (kr, vr) in zip(zip(t.k_pools, t.v_pools), ref_pools):
        assert torch.equal(kp, kr) and torch.equal(vp, vr)
    # graph capture of the stable-metadata step, replayed
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        step(True, got)
    for _ in range(3):
        reset()
        for o in got:
            o.zero_()
        g.replay()
        torch.cuda.synchronize()
        for a, b in zip(got, ref):
            assert torch.equal(a, b)
        for (kp, vp), (kr, vr) in zip(zip(t.k_pools, t.v_pools), ref_pools):
            assert torch.equal(kp, kr) and torch.equal(vp, vr)
    assert pkg.read_device_errors() == 0


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
@pytest.mark.parametrize("H,KVH,D", [(9, 3, 64), (32, 8, 128)])
def test_fused_decode_boundary_lengths(pkg, cuda, dtype, H, KVH, D):
    """The fused decode layer at lengths on 16-token unit, page and 64-token
    tile boundaries (the new token is the first or the last row of its unit,
    page or tile), up to 8192, over fragmented tables: bit-identical to
    rope_kv_write_decode + paged_attention (outputs and every pool byte) and
    within the oracle's tolerance (FP32 1e-5 relative, FP16 2e-3)."""
    from oracle import rope as orope
    g = torch.Generator().manual_seed(29 + D)
    lengths_l = [1, 2, 15, 16, 17, 31, 32, 33, 63, 64, 65, 127, 128, 129, 255, 256, 257,
                 1000, 4096, 8192]
    B, bs, max_len = len(lengths_l), 16, 8192
    lengths = torch.tensor(lengths_l, dtype=torch.int32)
    pages = [(n + bs - 1) // bs for n in lengths_l]
    N = sum(pages) + 11
    perm = torch.randperm(N, generator=g)
    tables = torch.zeros(B, max(pages), dtype=torch.int32)
    off = 0
    for b, n in enumerate(pages):
        tables[b, :n] = perm[off:off + n].to(torch.int32)
        off += n
    kp = torch.randn(N, bs, KVH, D, generator=g).to(dtype)
    vp = torch.randn(N, bs, KVH, D, generator=g).to(dtype)
    q = torch.randn(B, H, D, generator=g).to(dtype)
    kn = torch.randn(B, KVH, D, generator=g).to(dtype)
    vn = torch.randn(B, KVH, D, generator=g).to(dtype)
    inv = orope.inv_freq(5e5 if D == 128 else 1e5, D)
    dq, dkn, dvn = q.to(cuda), kn.to(cuda), vn.to(cuda)
    dt, dl, dinv = tables.to(cuda), lengths.to(cuda), inv.to(cuda)
    kp1, vp1 = kp.to(cuda), vp.to(cuda)
    assert pkg.decode_attention_supported(dq, kp1)
    kp2, vp2 = kp.to(cuda), vp.to(cuda)
    fused = pkg.decode_attention(dq, dkn, dvn, kp1, vp1, dt, dl, dinv, max_len)
    qr_dev, _ = pkg.rope_kv_write_decode(dq, dkn, dvn, kp2, vp2, dt, dl, dinv)
    two = pkg.paged_attention(qr_dev, kp2, vp2, dt, dl, max_len)
    torch.cuda.synchronize()
    assert torch.equal(fused, two)
    assert torch.equal(kp1, kp2) and torch.equal(vp1, vp2)
    # against the oracle: rotate on the CPU, write the slots, attend
    pos = (lengths.to(torch.int64) - 1).unsqueeze(1)
    phys = tables.to(torch.int64).gather(1, pos // bs)[:, 0]
    offs = pos[:, 0] % bs
    qr, kr = orope.rope(q.unsqueeze(1), kn.unsqueeze(1), pos, inv, exact_trig=True)
    kc, vc = kp.clone(), vp.clone()
    kc[phys, offs] = kr[:, 0]
    vc[phys, offs] = vn
    assert_matches_oracle(fused, qr[:, 0], tables, lengths, (kc, vc), bs,
                          f"fused decode {dtype} D={D}")
    assert pkg.read_device_errors() == 0


def test_fused_decode_row_alignment(pkg, cuda):
    """q, k and v rows given as slices of wider rows. FP32 rotates 16-byte
    chunks, so its rows must be 16-byte aligned: a q row stride of H*D + 2
    floats, or a k starting 8 bytes into its buffer, is rejected with the
    library's message before anything is written. FP16 reads q in 4-byte
    pairs and takes the same q stride, with the packed call's result and
    pool bytes."""
    from oracle import rope as orope
    B, H, KVH, D, N, bs = 3, 6, 2, 64, 24, 16
    g = torch.Generator().manual_seed(41)
    tables = torch.tensor([[9, 2, 5], [1, 8, 4], [7, 0, 6]], dtype=torch.int32).to(cuda)
    lengths = torch.tensor([1, 17, 35], dtype=torch.int32).to(cuda)
    inv = orope.inv_freq(1e5, D).to(cuda)
    msg = "16-byte aligned q, k and v rows"
    for dtype in (torch.float32, torch.float16):
        kp = torch.randn(N, bs, KVH, D, generator=g).to(dtype).to(cuda)
        vp = torch.randn(N, bs, KVH, D, generator=g).to(dtype).to(cuda)
        wide = torch.randn(B, H * D + 2, generator=g).to(dtype).to(cuda)
        q_wide = wide.as_strided((B, H, D), (H * D + 2, D, 1))
        q = q_wide.contiguous()
        kn = torch.randn(B, KVH, D, generator=g).to(dtype).to(cuda)
        vn = torch.randn(B, KVH, D, generator=g).to(dtype).to(cuda)
        assert pkg.decode_attention_supported(q, kp)
        if dtype == torch.float32:
            kp0, vp0 = kp.clone(), vp.clone()
            with pytest.raises(RuntimeError, match=msg):
                pkg.decode_attention(q_wide, kn, vn, kp, vp, tables, lengths, inv, 35)
            kbuf = torch.randn(B * KVH * D + 2, generator=g).to(cuda)
            k_off = kbuf[2:].view(B, KVH, D)
            with pytest.raises(RuntimeError, match=msg):
                pkg.decode_attention(q, k_off, vn, kp, vp, tables, lengths, inv, 35)
            torch.cuda.synchronize()
            assert torch.equal(kp, kp0) and torch.equal(vp, vp0)
        else:
            kp2, vp2 = kp.clone(), vp.clone()
            a = pkg.decode_attention(q_wide, kn, vn, kp, vp, tables, lengths, inv, 35)
            b = pkg.decode_attention(q, kn, vn, kp2, vp2, tables, lengths, inv, 35)
            torch.cuda.synchronize()
            assert torch.equal(a, b)
            assert torch.equal(kp, kp2) and torch.equal(vp, vp2)
    assert pkg.read_device_errors() == 0
