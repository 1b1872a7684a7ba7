"""Helpers shared by the -m gpu parity tests."""
from __future__ import annotations

import torch

# Parity bars: FP32 within 1e-5 relative (with a 1e-6 absolute floor for
# values that cancel to ~0); FP16 within 2e-3 absolute.
FP32_RTOL, FP32_ATOL = 1e-5, 1e-6
FP16_ATOL = 2e-3


def assert_parity(actual: torch.Tensor, expected: torch.Tensor, what: str = "") -> None:
    actual = actual.detach().cpu()
    expected = expected.detach().cpu()
    assert actual.dtype == expected.dtype, (actual.dtype, expected.dtype)
    if actual.dtype == torch.float32:
        torch.testing.assert_close(actual, expected, rtol=FP32_RTOL, atol=FP32_ATOL, msg=what or None)
    else:
        err = (actual.float() - expected.float()).abs()
        assert torch.isfinite(actual.float()).all(), what
        assert err.max().item() <= FP16_ATOL, f"{what}: max abs err {err.max().item():.3e}"


def subset_pool(tables, lengths, pools, block_size):
    """The used pages of some sequences, copied to the CPU with renumbered tables."""
    from conftest import import_module
    return import_module("workloads").compact_pages(tables, lengths, pools, block_size)


def assert_matches_oracle(out, q, tables, lengths, pools, block_size, what="", chunk=32):
    """Every sequence of a decode attention output against the CPU oracle
    (worker/llama.py:58-71 restated), in chunks of `chunk` sequences of
    similar length: each chunk's pages are copied to the CPU and padded to
    the chunk's longest (the reference pads to the batch's longest). Returns
    the number of sequences checked."""
    from oracle import paged_attention as opa
    out, q = out.detach().cpu(), q.detach().cpu()
    lengths = lengths.cpu()
    checked = 0
    for idx in torch.argsort(lengths).split(chunk):
        tabs, (kp, vp) = subset_pool(tables.cpu()[idx], lengths[idx], pools, block_size)
        lens = lengths[idx]
        ref = opa.paged_attention(q[idx], kp, vp, tabs, lens, max(int(lens.max()), 1))
        assert_parity(out[idx], ref, f"{what} (sequences {idx.tolist()[:4]}...)")
        checked += idx.numel()
    return checked


def prefill_fixture_layer(case: dict, layer: int):
    """One layer of tests/golden/prefill_attention.pt (the reference's
    PagedLlama.prefill, worker/llama.py:141-144) back in the padded layout its
    SDPA saw: q, k, v [B, W, heads, D] with zero padded rows, the reference's
    context [B, W, H, D] (zero padded rows), and the valid-row mask [B, W]."""
    lens = case["lengths"].tolist()
    B, width = len(lens), max(lens)
    valid = torch.arange(width)[None, :] < torch.tensor(lens)[:, None]
    L = case["layers"][layer]

    def pad(rows):
        out = torch.zeros((B, width) + tuple(rows.shape[1:]), dtype=rows.dtype)
        out[valid] = rows
        return out

    return pad(L["q"]), pad(L["k"]), pad(L["v"]), pad(L["context"]), valid


def prefill_fixture_pools(case: dict, layer: int, stale: float = float("nan")):
    """Paged pools [blocks, bs, KVH, D] holding the layer's prompt k/v rows at
    the slots the reference's tables give (token t of prompt b at page
    tables[b][t // bs], row t % bs); every other row holds `stale`."""
    spec = case["spec"]
    bs = spec["block_size"]
    L = case["layers"][layer]
    KVH, D = L["k"].shape[1], L["k"].shape[2]
    k_pool = torch.full((spec["blocks"], bs, KVH, D), stale, dtype=L["k"].dtype)
    v_pool = torch.full_like(k_pool, stale)
    row = 0
    for b, n in enumerate(case["lengths"].tolist()):
        for t in range(n):
            page = int(case["tables"][b, t // bs])
            k_pool[page, t % bs] = L["k"][row]
            v_pool[page, t % bs] = L["v"][row]
            row += 1
    return k_pool, v_pool
