"""Swap-in points for the reference's worker/llama.py.

``cuda_paged_attention`` has the name and behaviour of the reference loader
(worker/llama.py:77-86): it makes q, tables and lengths contiguous and calls
the extension op. ``PagedLlama.decode`` looks that name up in its module
globals at call time (worker/llama.py:162), so rebinding it swaps the kernel
and nothing else.

``install(module)`` does that and, by default, also routes the ``decode`` and
``prefill`` methods of the module's ``PagedLlama`` class to
``llama_runner.b200_decode`` / ``b200_prefill`` for instances built with
``attention='cuda'``: the RoPE, the paged KV writes and the decode metadata
(slots, positions, tables, lengths; worker/llama.py:121-140, :152-172) then
run on the device as well, on the instance's own pools and allocator
(``DevicePagedKV.adopt`` shares its TensorPagedKV). Instances built with
``attention='torch'`` keep the module's own methods.
"""
from __future__ import annotations

from .llama_runner import b200_decode, b200_prefill
from .ops import paged_attention


def cuda_paged_attention(query, keys, values, tables, lengths, max_length):
    """worker/llama.py:77-86 with the B200 op behind it (no JIT build)."""
    return paged_attention(query.contiguous(), keys, values, tables.contiguous(),
                           lengths.contiguous(), max_length)


def install(llama_module, model_runner: bool = True) -> None:
    """Point a ``worker.llama`` module's ``--attention cuda`` path at this library."""
    llama_module.cuda_paged_attention = cuda_paged_attention
    cls = getattr(llama_module, "PagedLlama", None)
    if not model_runner or cls is None or getattr(cls, "_b200_installed", False):
        return
    own_decode, own_prefill = cls.decode, cls.prefill

    def decode(self, ids, tokens):
        if getattr(self, "attention", None) == "cuda":
            return b200_decode(self, ids, tokens)
        return own_decode(self, ids, tokens)

    def prefill(self, ids, token_lists):
        if getattr(self, "attention", None) == "cuda":
            return b200_prefill(self, ids, token_lists)
        return own_prefill(self, ids, token_lists)

    decode.__doc__, prefill.__doc__ = b200_decode.__doc__, b200_prefill.__doc__
    cls.decode, cls.prefill = decode, prefill
    cls._b200_own_methods = (own_decode, own_prefill)
    cls._b200_installed = True


def uninstall(llama_module) -> None:
    """Undo ``install`` on the module's PagedLlama class (the kernel name stays bound)."""
    cls = getattr(llama_module, "PagedLlama", None)
    if cls is not None and getattr(cls, "_b200_installed", False):
        cls.decode, cls.prefill = cls._b200_own_methods
        del cls._b200_own_methods
        cls._b200_installed = False
