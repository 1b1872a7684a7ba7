"""Oracle: rotate-half RoPE on the CPU (test infrastructure only).

Restates worker/llama.py:105-117:
  inv_freq = 1 / theta ** (arange(0, D, 2, fp32) / D)          (:105-106)
  ang      = positions.float()[..., None] * inv_freq, duplicated to D
  cos, sin = ang.cos(), ang.sin() cast to the model dtype, broadcast over heads
  out      = x * cos + rotate(x) * sin, rotate(x) = cat(-x[D/2:], x[:D/2])
Every elementwise op runs in the model dtype, as in the reference.
"""
from __future__ import annotations

import torch


def inv_freq(theta: float, head_dim: int) -> torch.Tensor:
    return 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim))


def _rotate(x: torch.Tensor) -> torch.Tensor:
    first, second = x.chunk(2, dim=-1)
    return torch.cat((-second, first), dim=-1)


def rope(q: torch.Tensor, k: torch.Tensor, positions: torch.Tensor, freqs: torch.Tensor):
    """q [B, S, H, D], k [B, S, KVH, D], positions int [B, S] -> rotated (q, k)."""
    f = positions.float()[..., None] * freqs
    ang = torch.cat((f, f), dim=-1)
    cos = ang.cos().to(q.dtype).unsqueeze(2)
    sin = ang.sin().to(q.dtype).unsqueeze(2)
    return q * cos + _rotate(q) * sin, k * cos + _rotate(k) * sin
