"""GPU parity of prefill_attention (causal attention of a prompt batch with
K/V read from the paged pools) against the reference's prefill attention
(worker/llama.py:141-144, restated in oracle/paged_attention.py:
repeat_interleave + causal SDPA over the padded batch, fp32).

Both kernels are checked, pinned by `impl`: the tcgen05 kernel (TMA-staged
tiles, tcgen05.mma with TMEM accumulators; block_size % 16 == 0) and the
mma.sync kernel (cp.async tiles, any block size).

Bars: rows of real tokens within 2e-3 (FP16); rows at or beyond a prompt's
length exactly zero; pages placed in a fragmented pool through the tables."""
from __future__ import annotations

import pytest
import torch

from conftest import REPO, import_module
from gpu_helpers import assert_parity, prefill_fixture_layer, prefill_fixture_pools
from oracle import kv_cache
from oracle import paged_attention as opa

pytestmark = pytest.mark.gpu
W = import_module("workloads")


IMPLS = pytest.mark.parametrize("impl", ["tcgen05", "mma"])


@IMPLS
def test_prefill_attention_matches_reference_fixture(pkg, cuda, impl):
    """Both kernels against the reference's own output: the FP16 contexts
    that PagedLlama.prefill (worker/llama.py:141-144) computed on a seeded
    tiny Llama (tests/golden/prefill_attention.pt), fed the same rotated q and
    the same k/v rows, placed at the reference's slots in pools whose every
    other row is NaN. Every real token's row within 2e-3; padded rows zero."""
    case = torch.load(REPO / "tests" / "golden" / "prefill_attention.pt",
                      weights_only=False)["float16"]
    tables, lengths = case["tables"].to(cuda), case["lengths"].to(cuda)
    for layer in range(len(case["layers"])):
        q, _, _, ctx, valid = prefill_fixture_layer(case, layer)
        k_pool, v_pool = prefill_fixture_pools(case, layer)
        out = pkg.prefill_attention(q.to(cuda), k_pool.to(cuda), v_pool.to(cuda), tables,
                                    lengths, impl=_impl(pkg, impl)).cpu()
        assert_parity(out[valid], ctx[valid], f"reference prefill fixture, {impl}, layer {layer}")
        assert torch.equal(out[~valid], torch.zeros_like(out[~valid]))
    assert pkg.read_device_errors() == 0


def _impl(pkg, name):
    return {"tcgen05": pkg.PREFILL_TCGEN05, "mma": pkg.PREFILL_MMA}[name]


def make_case(lengths, H, KVH, D, bs=16, seed=0, width=None, extra_blocks=37, stale_nan=False):
    g = torch.Generator().manual_seed(seed)
    B = len(lengths)
    Wd = width or max(lengths)
    lens = torch.tensor(lengths, dtype=torch.int32)
    q = torch.randn(B, Wd, H, D, generator=g).half()
    k = torch.randn(B, Wd, KVH, D, generator=g).half()
    v = torch.randn(B, Wd, KVH, D, generator=g).half()
    pages = [(n + bs - 1) // bs for n in lengths]
    N = sum(pages) + extra_blocks
    perm = torch.randperm(N, generator=g)
    tables = torch.zeros(B, max(max(pages), 1), dtype=torch.int32)
    off = 0
    for b, n in enumerate(pages):
        tables[b, :n] = perm[off:off + n].to(torch.int32)
        off += n
    k_pool = (torch.randn(N, bs, KVH, D, generator=g) * 3).half()  # stale everywhere
    v_pool = (torch.randn(N, bs, KVH, D, generator=g) * 3).half()
    if stale_nan:  # rows no prompt owns are NaN: they must never reach an output
        k_pool.fill_(float("nan"))
        v_pool.fill_(float("nan"))
    valid = torch.arange(Wd)[None, :] < lens[:, None]
    phys, offs = [], []
    for b, n in enumerate(lengths):
        for t in range(n):
            phys.append(int(tables[b, t // bs]))
            offs.append(t % bs)
    phys, offs = torch.tensor(phys, dtype=torch.int64), torch.tensor(offs, dtype=torch.int64)
    kv_cache.write_prefill(k_pool, phys, offs, k, valid)
    kv_cache.write_prefill(v_pool, phys, offs, v, valid)
    return q, k, v, k_pool, v_pool, tables, lens, valid


def run(pkg, cuda, case, impl="tcgen05"):
    q, k, v, kp, vp, tables, lens, valid = case
    return pkg.prefill_attention(q.to(cuda), kp.to(cuda), vp.to(cuda), tables.to(cuda),
                                 lens.to(cuda), impl=_impl(pkg, impl)).cpu()


def check(out, case, what):
    q, k, v, kp, vp, tables, lens, valid = case
    ref = opa.prefill_attention(q, k, v)
    assert_parity(out[valid], ref[valid].half(), what)
    assert torch.equal(out[~valid], torch.zeros_like(out[~valid]))


@IMPLS
@pytest.mark.parametrize("H,KVH,D", [(9, 3, 64), (32, 8, 128), (4, 4, 64), (8, 1, 128)])
def test_prefill_attention_matches_reference(pkg, cuda, impl, H, KVH, D):
    lengths = [1, 63, 64, 65, 130, 200, 17, 128]
    case = make_case(lengths, H, KVH, D, seed=D + H)
    check(run(pkg, cuda, case, impl), case, f"prefill {impl} H={H} KVH={KVH} D={D}")
    assert pkg.read_device_errors() == 0


@IMPLS
def test_prefill_attention_cfg4_prompts(pkg, cuda, impl):
    """16 SmolLM2-shaped prompts, lengths U[64, 1024], padded to the longest."""
    g = torch.Generator().manual_seed(4)
    lengths = torch.randint(64, 1025, (16,), generator=g).tolist()
    case = make_case(lengths, 9, 3, 64, seed=44)
    check(run(pkg, cuda, case, impl), case, f"cfg4 prefill {impl}")


@IMPLS
@pytest.mark.parametrize("D", [64, 128])
def test_prefill_attention_ignores_nan_stale_rows(pkg, cuda, impl, D):
    """Every pool row no prompt wrote is NaN: partial 16-token units and the
    rest of each last page are staged but must not reach any output row."""
    lengths = [5, 129, 255, 0, 300, 16]
    case = make_case(lengths, 8, 2, D, seed=7 + D, width=320, stale_nan=True)
    out = run(pkg, cuda, case, impl)
    assert not torch.isnan(out).any()
    check(out, case, f"NaN-stale prefill {impl} D={D}")
    assert pkg.read_device_errors() == 0


@pytest.mark.parametrize("bs", [32, 64])
def test_prefill_attention_tcgen05_block_sizes(pkg, cuda, bs):
    lengths = [31, 32, 33, 257, 96, 1]
    case = make_case(lengths, 6, 2, 64, bs=bs, seed=bs)
    check(run(pkg, cuda, case, "tcgen05"), case, f"tcgen05 prefill bs={bs}")


def test_prefill_attention_block_size_8_takes_mma(pkg, cuda):
    """block_size 8 splits a 16-token unit over two pages: the default picks
    the mma.sync kernel, and pinning the tcgen05 kernel is refused."""
    lengths = [9, 40, 77]
    case = make_case(lengths, 4, 2, 64, bs=8, seed=8)
    q, k, v, kp, vp, tables, lens, valid = case
    out = pkg.prefill_attention(q.to(cuda), kp.to(cuda), vp.to(cuda), tables.to(cuda),
                                lens.to(cuda)).cpu()
    check(out, case, "bs=8 prefill (auto)")
    with pytest.raises(RuntimeError, match="block_size % 16"):
        run(pkg, cuda, case, "tcgen05")


def test_prefill_attention_kernels_agree(pkg, cuda):
    """The two kernels round P to FP16 alike: results within FP16 rounding."""
    lengths = [700, 513, 64, 1000]
    case = make_case(lengths, 9, 3, 64, seed=99)
    a = run(pkg, cuda, case, "tcgen05")
    b = run(pkg, cuda, case, "mma")
    torch.testing.assert_close(a, b, rtol=0, atol=2e-3)


def test_prefill_attention_rejects_unsupported_shapes(pkg, cuda):
    q = torch.zeros(2, 8, 4, 32, dtype=torch.float16, device=cuda)
    kp = torch.zeros(4, 16, 2, 32, dtype=torch.float16, device=cuda)
    t = torch.zeros(2, 1, dtype=torch.int32, device=cuda)
    with pytest.raises(RuntimeError, match="head_dim 64 and 128"):
        pkg.prefill_attention(q, kp, kp, t, t[:, 0].contiguous())
    with pytest.raises(RuntimeError, match="FP16"):
        pkg.prefill_attention(q.float(), kp.float(), kp.float(), t, t[:, 0].contiguous())


@pytest.mark.parametrize("B,seed", [(40, 5), (600, 6)])
def test_prefill_attention_tcgen05_many_prompts(pkg, cuda, B, seed):
    """More prompts than one warp ballot covers (40), and more than the
    kernel keeps in shared memory (600 > 512: lengths read from global
    memory); lengths include 0 and the full width, so every schedule phase
    (working tiles by level, padding tiles) is crossed by many CTAs."""
    g = torch.Generator().manual_seed(seed)
    hi = 300 if B == 40 else 70
    lengths = torch.randint(0, hi + 1, (B,), generator=g).tolist()
    lengths[0], lengths[-1] = 0, hi
    case = make_case(lengths, 4, 2, 64, seed=seed, width=hi, extra_blocks=5)
    check(run(pkg, cuda, case, "tcgen05"), case, f"tcgen05 prefill B={B}")
    assert pkg.read_device_errors() == 0


def test_prefill_attention_tcgen05_repeated_calls_and_graph(pkg, cuda):
    """The persistent kernel carries no state between launches: eager calls
    with different batches on one stream and replays of a captured call all
    match the oracle."""
    cases = [make_case([130, 7, 300], 6, 3, 64, seed=21),
             make_case([1000, 3], 6, 3, 64, seed=22)]
    for case in cases * 2:
        check(run(pkg, cuda, case, "tcgen05"), case, "eager")
    q, k, v, kp, vp, tables, lens, valid = cases[0]
    dq, dk, dvp = q.to(cuda), kp.to(cuda), vp.to(cuda)
    dt, dl = tables.to(cuda), lens.to(cuda)
    out = torch.empty_like(dq)
    s = torch.cuda.Stream(cuda)
    with torch.cuda.stream(s):
        pkg.prefill_attention(dq, dk, dvp, dt, dl, out=out)  # warm-up outside capture
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, stream=s):
            pkg.prefill_attention(dq, dk, dvp, dt, dl, out=out)
    for _ in range(3):
        out.zero_()
        gr.replay()
        torch.cuda.synchronize()
        check(out.cpu(), cases[0], "graph replay")
