"""Blackwell (sm_100a) paged-decode hot path of sri123vk/distributed-llm-inference.

Public ops (drop-in for the reference's decode path):
  paged_attention(q, k, v, tables, lengths, max_length)   cuda/binding.cpp:6-26
  rope_kv_write(q, k, v, k_pool, v_pool, physical, offsets, positions, inv_freq[, valid])
      worker/llama.py:108-117 + :171-172 (decode) / :139-140 (prefill)
  rope_kv_write_decode(q, k, v, k_pool, v_pool, tables, lengths, inv_freq, advance=...)
      the decode prologue with positions and slots derived on the device
      (worker/llama.py:40-55, :154-159, :168-172)
  decode_attention(q, k, v, k_pool, v_pool, tables, lengths, inv_freq, max_length)
      one decode layer (RoPE, slot writes, attention) in one launch
  prefill_attention(q, k_pool, v_pool, tables, lengths)
      causal prefill attention with K/V from the pools (worker/llama.py:141-144)
  DevicePagedKV              TensorPagedKV (worker/llama.py:13-55) + device-resident
                             decode tables/lengths
  PagedLlama                 worker/llama.py:89-177 on these ops (CUDA-graph decode ticks)
  cuda_paged_attention(...)  the reference loader's name (worker/llama.py:77-86)
  install(llama_module)      points a worker.llama module at these ops

The package directory name contains '-', so import it with
importlib.import_module("distributed-llm-inference_b200").
"""
from ._lib import IMPL_AUTO, IMPL_FAST, IMPL_GENERIC, IMPL_SIMT, IMPL_MMA, IMPL_TMA_STATIC, load as load_library  # noqa: F401
from ._lib import PREFILL_AUTO, PREFILL_MMA, PREFILL_TCGEN05  # noqa: F401
from .ops import (decode_attention, decode_attention_supported,  # noqa: F401
                  fast_grid_size, paged_attention, prefill_attention, read_device_errors,
                  rope_kv_write, rope_kv_write_decode)
from .paged_kv import DevicePagedKV  # noqa: F401
from .llama_runner import PagedLlama  # noqa: F401
from .integration import cuda_paged_attention, install, uninstall  # noqa: F401

__all__ = [
    "paged_attention", "decode_attention", "decode_attention_supported", "prefill_attention",
    "rope_kv_write", "rope_kv_write_decode",
    "DevicePagedKV", "PagedLlama",
    "cuda_paged_attention", "install", "uninstall",
    "read_device_errors", "fast_grid_size", "load_library",
    "IMPL_AUTO", "IMPL_FAST", "IMPL_GENERIC", "IMPL_SIMT", "IMPL_MMA", "IMPL_TMA_STATIC",
    "PREFILL_AUTO", "PREFILL_TCGEN05", "PREFILL_MMA",
]
