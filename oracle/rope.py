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


def rope(q: torch.Tensor, k: torch.Tensor, positions: torch.Tensor, freqs: torch.Tensor,
         exact_trig: bool = False):
    """q [B, S, H, D], k [B, S, KVH, D], positions int [B, S] -> rotated (q, k).

    The reference takes cos/sin of the FP32 angle in FP32, whose last bit
    depends on the math library that runs it (torch's CPU builds differ by
    host instruction set, and from its CUDA build), so a few FP16-rounded
    cos/sin values — and the outputs built from them — differ by one FP16 ulp
    between hosts. ``exact_trig=True`` takes them in float64 and rounds once to
    FP32 (the correctly rounded value of the same formula), which gives the
    same result on every host; the default keeps the reference's FP32 calls
    (the golden vectors were made with them).
    """
    f = positions.float()[..., None] * freqs
    ang = torch.cat((f, f), dim=-1)
    if exact_trig:
        c32, s32 = ang.double().cos().float(), ang.double().sin().float()
    else:
        c32, s32 = ang.cos(), ang.sin()
    cos = c32.to(q.dtype).unsqueeze(2)
    sin = s32.to(q.dtype).unsqueeze(2)
    return q * cos + _rotate(q) * sin, k * cos + _rotate(k) * sin
