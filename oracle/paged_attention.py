"""Oracle: paged GQA decode attention on the CPU (test infrastructure only).

Restates torch_paged_attention, worker/llama.py:58-71: every sequence's
pages are gathered to a dense [B, max_length, KVH, D] tensor through its
block table, the KV heads are repeated to the query heads, and masked
scaled-dot-product attention (default scale 1/sqrt(D)) is taken with the mask
position < length. The steps are kept alike on purpose: the oracle has to
reproduce the reference's rounding (same dtype, same SDPA kernel), and the
timed CPU baseline has to cost what the reference's CPU path costs.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F


def paged_attention(query: torch.Tensor, keys: torch.Tensor, values: torch.Tensor,
                    tables: torch.Tensor, lengths: torch.Tensor, max_length: int) -> torch.Tensor:
    """query [B, H, D]; keys/values [N, bs, KVH, D]; tables int [B, W];
    lengths int [B] -> [B, H, D] in query's dtype."""
    bs = keys.shape[1]
    pos = torch.arange(max_length, device=query.device)
    page_of = tables.to(torch.int64)[:, pos // bs]              # [B, max_len]
    slot_in_page = pos % bs                                      # [max_len]
    k = keys[page_of, slot_in_page].permute(0, 2, 1, 3)          # [B, KVH, max_len, D]
    v = values[page_of, slot_in_page].permute(0, 2, 1, 3)
    group = query.shape[1] // keys.shape[2]
    k = torch.repeat_interleave(k, group, dim=1)                 # [B, H, max_len, D]
    v = torch.repeat_interleave(v, group, dim=1)
    visible = pos.unsqueeze(0) < lengths.to(pos.device).unsqueeze(1)   # [B, max_len]
    out = F.scaled_dot_product_attention(query[:, :, None, :], k, v,
                                         attn_mask=visible[:, None, None, :])
    return out[:, :, 0, :]


def paged_attention_chunked(query, keys, values, tables, lengths, max_length, chunk: int):
    """Same result, `chunk` sequences at a time (bounds the gather's memory).

    The reference pads every sequence to the batch's max_length; so does each
    chunk here, so the work per sequence is the reference's.
    """
    outs = []
    for lo in range(0, query.shape[0], chunk):
        hi = lo + chunk
        outs.append(paged_attention(query[lo:hi], keys, values, tables[lo:hi], lengths[lo:hi],
                                    max_length))
    return torch.cat(outs)


def paged_attention_fp64(query, keys, values, tables, lengths) -> torch.Tensor:
    """Float64, per-sequence restatement of the same math (no padding), used
    to measure how far a result is from the exact answer."""
    B, H, D = query.shape
    bs, KVH = keys.shape[1], keys.shape[2]
    group = H // KVH
    out = torch.zeros(B, H, D, dtype=torch.float64)
    for b in range(B):
        n = int(lengths[b])
        if n == 0:
            continue
        t = torch.arange(n)
        pages = tables[b].to(torch.int64)[t // bs]
        k = keys[pages, t % bs].to(torch.float64)                # [n, KVH, D]
        v = values[pages, t % bs].to(torch.float64)
        for h in range(H):
            kh = k[:, h // group]
            s = (kh @ query[b, h].to(torch.float64)) / (D ** 0.5)
            p = torch.softmax(s, dim=0)
            out[b, h] = p @ v[:, h // group]
    return out


def prefill_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                      native: bool = False) -> torch.Tensor:
    """worker/llama.py:141-144: causal SDPA over the padded prompt batch,
    K/V repeated per query group. q [B, W, H, D], k/v [B, W, KVH, D];
    returns [B, W, H, D]. Computed in fp32 (the precision the reference's
    FP16 CUDA SDPA accumulates in), or with ``native`` in the inputs' dtype,
    which on the CPU is the reference's own call bit for bit."""
    groups = q.shape[2] // k.shape[2]
    qf, kf, vf = (q, k, v) if native else (q.float(), k.float(), v.float())
    ctx = F.scaled_dot_product_attention(
        qf.transpose(1, 2), kf.repeat_interleave(groups, dim=2).transpose(1, 2),
        vf.repeat_interleave(groups, dim=2).transpose(1, 2), is_causal=True)
    return ctx.transpose(1, 2)
