"""Oracle: scalar paged attention in pure Python (test infrastructure only).

Restates the readable spec PagedKV.attention, worker/engine.py:53-70:
scores q.k / sqrt(D) over the n stored tokens, max-subtracted exponentials,
weighted sum of values divided by the sum of weights; 0 for n == 0. Used only
on small cases (known answers, edge cases).
"""
from __future__ import annotations

import math


def attention(query, keys, values, table, length, block_size):
    """query [D]; keys/values indexable as [block][offset] -> [D] (one kv head)."""
    if length == 0:
        return [0.0] * len(query)
    scale = 1.0 / math.sqrt(len(query))
    scores, rows = [], []
    for i in range(length):
        block, offset = table[i // block_size], i % block_size
        key, value = keys[block][offset], values[block][offset]
        scores.append(sum(a * b for a, b in zip(query, key)) * scale)
        rows.append(value)
    top = max(scores)
    weights = [math.exp(s - top) for s in scores]
    total = sum(weights)
    return [sum(w * r[d] for w, r in zip(weights, rows)) / total for d in range(len(query))]
