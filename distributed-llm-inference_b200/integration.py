"""Swap-in points for the reference's worker/llama.py.

``cuda_paged_attention`` has the name and behaviour of the reference loader
(worker/llama.py:77-86): it makes q, tables and lengths contiguous and calls
the extension op. Because ``PagedLlama.decode`` looks the name up in its
module globals at call time (worker/llama.py:162), ``install(module)`` only
rebinds that global; nothing else in worker/llama.py or worker/batched.py
changes.
"""
from __future__ import annotations

from .ops import paged_attention


def cuda_paged_attention(query, keys, values, tables, lengths, max_length):
    """worker/llama.py:77-86 with the B200 op behind it (no JIT build)."""
    return paged_attention(query.contiguous(), keys, values, tables.contiguous(),
                           lengths.contiguous(), max_length)


def install(llama_module) -> None:
    """Point a ``worker.llama`` module's ``--attention cuda`` path at this library."""
    llama_module.cuda_paged_attention = cuda_paged_attention
