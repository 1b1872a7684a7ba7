"""GPU parity of prefill_attention (causal attention of a prompt batch with
K/V read from the paged pools) against the reference's prefill attention
(worker/llama.py:141-144, restated in oracle/paged_attention.py:
repeat_interleave + causal SDPA over the padded batch, fp32).

Bars: rows of real tokens within 2e-3 (FP16); rows at or beyond a prompt's
length exactly zero; pages placed in a fragmented pool through the tables."""
from __future__ import annotations

import pytest
import torch

from conftest import import_module
from gpu_helpers import assert_parity
from oracle import kv_cache
from oracle import paged_attention as opa

pytestmark = pytest.mark.gpu
W = import_module("workloads")


def make_case(lengths, H, KVH, D, bs=16, seed=0, width=None, extra_blocks=37):
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


@pytest.mark.parametrize("H,KVH,D", [(9, 3, 64), (32, 8, 128), (4, 4, 64), (8, 1, 128)])
def test_prefill_attention_matches_reference(pkg, cuda, H, KVH, D):
    lengths = [1, 63, 64, 65, 130, 200, 17, 128]
    q, k, v, kp, vp, tables, lens, valid = make_case(lengths, H, KVH, D, seed=D + H)
    out = pkg.prefill_attention(q.to(cuda), kp.to(cuda), vp.to(cuda), tables.to(cuda),
                                lens.to(cuda)).cpu()
    ref = opa.prefill_attention(q, k, v)
    assert_parity(out[valid], ref[valid].half(), f"prefill H={H} KVH={KVH} D={D}")
    assert torch.equal(out[~valid], torch.zeros_like(out[~valid]))
    assert pkg.read_device_errors() == 0


def test_prefill_attention_cfg4_prompts(pkg, cuda):
    """16 SmolLM2-shaped prompts, lengths U[64, 1024], padded to the longest."""
    g = torch.Generator().manual_seed(4)
    lengths = torch.randint(64, 1025, (16,), generator=g).tolist()
    q, k, v, kp, vp, tables, lens, valid = make_case(lengths, 9, 3, 64, seed=44)
    out = pkg.prefill_attention(q.to(cuda), kp.to(cuda), vp.to(cuda), tables.to(cuda),
                                lens.to(cuda)).cpu()
    ref = opa.prefill_attention(q, k, v)
    assert_parity(out[valid], ref[valid].half(), "cfg4 prefill")
    assert torch.equal(out[~valid], torch.zeros_like(out[~valid]))


def test_prefill_attention_rejects_unsupported_shapes(pkg, cuda):
    q = torch.zeros(2, 8, 4, 32, dtype=torch.float16, device=cuda)
    kp = torch.zeros(4, 16, 2, 32, dtype=torch.float16, device=cuda)
    t = torch.zeros(2, 1, dtype=torch.int32, device=cuda)
    with pytest.raises(RuntimeError, match="head_dim 64 and 128"):
        pkg.prefill_attention(q, kp, kp, t, t[:, 0].contiguous())
    with pytest.raises(RuntimeError, match="FP16"):
        pkg.prefill_attention(q.float(), kp.float(), kp.float(), t, t[:, 0].contiguous())
