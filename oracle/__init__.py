"""CPU oracle for the paged-decode path — TEST INFRASTRUCTURE ONLY.

This package restates, on the CPU with PyTorch, the reference algorithms of
sri123vk/distributed-llm-inference that the CUDA library replaces:

  paged_attention.py  torch_paged_attention      worker/llama.py:58-71
  rope.py             PagedLlama.inv_freq / rope worker/llama.py:105-117
  kv_cache.py         TensorPagedKV (allocator, slots, metadata, slot writes)
                                                 worker/llama.py:13-55, :139-140, :171-172
  scalar.py           PagedKV.attention (scalar spec, pure Python loops)
                                                 worker/engine.py:53-70

Parity of the oracle itself is pinned against golden vectors produced by the
reference's own code (tests/golden/make_golden.py imports it from the
reference checkout and writes tests/golden/*.pt).

Only tests/, __graft_entry__.smoke() and the CPU-baseline / reference arm of
bench.py may import this package, and only as the checker or the timed CPU
baseline. The product path (the package's ops) never calls it.
"""
