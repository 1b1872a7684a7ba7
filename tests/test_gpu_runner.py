"""GPU parity of the device-metadata decode prologue and of the model runner.

* rope_kv_write_decode against the oracle (positions lengths[b] or
  lengths[b]-1, slots from the tables, lengths advanced in place); pool bytes
  outside the written slots unchanged; out-of-table rows skipped and flagged.
* llama_runner.PagedLlama (B200 ops, device metadata, CUDA-graph ticks) on a
  seeded random-init Llama through a serving scenario (prefill, decode,
  release, re-admission on reused pages): FP32 against the reference's own
  logits (tests/golden/llama_tiny_scenario.pt), FP16 against the oracle
  runner on the GPU; graph replays bit-identical to eager ticks; install()
  on a module shaped like worker/llama.py.

Logit bars: the runners differ only in the attention/RoPE kernels, so FP32
logits agree to 1e-5 of their largest magnitude (GEMM reduction order differs
between the CPU that made the golden logits and cuBLAS; measured 4e-7) and
FP16 logits to 5e-3 of it (FP16 rounding of activations compounds over the
layers; measured 8e-4).
"""
from __future__ import annotations

import types

import pytest
import torch

from conftest import REPO, import_module
from gpu_helpers import assert_parity
from oracle import kv_cache
from oracle import llama_model as LM
from oracle import rope as orope

pytestmark = pytest.mark.gpu

W = import_module("workloads")
R = import_module("llama_runner")


def gold():
    return torch.load(REPO / "tests" / "golden" / "llama_tiny_scenario.pt", weights_only=False)


def rel_err(a, b):
    return float((a.float() - b.float()).abs().max() / b.float().abs().max())


@pytest.mark.parametrize("dtype,D", [(torch.float16, 64), (torch.float16, 128),
                                     (torch.float32, 64), (torch.float16, 40)])
@pytest.mark.parametrize("advance", [True, False])
def test_rope_kv_write_decode(pkg, cuda, dtype, D, advance):
    g = torch.Generator().manual_seed(D + advance)
    B, H, KVH, N, bs, Wd = 37, 8, 2, 480, 16, 12
    lengths = torch.randint(1, Wd * bs - 1, (B,), generator=g).to(torch.int32)
    lengths[0], lengths[1] = 1, 15  # first token of a page / last slot of a page
    perm = torch.randperm(N, generator=g)[:B * Wd].view(B, Wd).to(torch.int32)
    q = torch.randn(B, H, D, generator=g).to(dtype)
    k = torch.randn(B, KVH, D, generator=g).to(dtype)
    v = torch.randn(B, KVH, D, generator=g).to(dtype)
    pk = torch.randn(N, bs, KVH, D, generator=g).to(dtype)
    pv = torch.randn(N, bs, KVH, D, generator=g).to(dtype)
    inv = W.inv_freq(1e5, D)
    pos = (lengths if advance else lengths - 1).to(torch.int64)
    phys = perm[torch.arange(B), (pos // bs)].to(torch.int64)
    off = pos % bs
    qr, kr = orope.rope(q.unsqueeze(1), k.unsqueeze(1), pos[:, None], inv, exact_trig=True)
    exp_k, exp_v = pk.clone(), pv.clone()
    kv_cache.write_decode(exp_k, phys, off, kr[:, 0])
    kv_cache.write_decode(exp_v, phys, off, v)
    dl, dk, dv = lengths.to(cuda), pk.to(cuda), pv.to(cuda)
    qo, ko = pkg.rope_kv_write_decode(q.to(cuda), k.to(cuda), v.to(cuda), dk, dv,
                                      perm.to(cuda), dl, inv.to(cuda), advance=advance)
    assert_parity(qo, qr[:, 0], "q")
    assert_parity(ko, kr[:, 0], "k")
    exp_k[phys, off] = ko.cpu()  # written slot holds exactly the kernel's k
    assert torch.equal(dk.cpu(), exp_k) and torch.equal(dv.cpu(), exp_v)
    assert torch.equal(dl.cpu(), lengths + 1 if advance else lengths)
    assert pkg.read_device_errors() == 0


def test_rope_kv_write_decode_rejects_rows_outside_the_table(pkg, cuda):
    """A row whose next position does not fit its table is skipped (no pool
    byte changes) and flagged; the other rows are written."""
    B, H, KVH, D, N, bs, Wd = 3, 4, 2, 64, 16, 16, 2
    lengths = torch.tensor([5, Wd * bs, 7], dtype=torch.int32)  # row 1: table full
    tables = torch.tensor([[3, 4], [5, 6], [7, 8]], dtype=torch.int32)
    q, k, v = (torch.randn(B, h, D).half() for h in (H, KVH, KVH))
    pk = torch.zeros(N, bs, KVH, D).half()
    pv = torch.zeros_like(pk)
    dk, dv, dl = pk.to(cuda), pv.to(cuda), lengths.to(cuda)
    pkg.read_device_errors()
    pkg.rope_kv_write_decode(q.to(cuda), k.to(cuda), v.to(cuda), dk, dv, tables.to(cuda), dl,
                             W.inv_freq(1e5, D).to(cuda), advance=True)
    assert pkg.read_device_errors() & 0x2
    touched = (dv.cpu() != 0).flatten(1).any(1)
    assert touched.nonzero().flatten().tolist() == [3, 7]  # rows 0 and 2 only
    assert torch.equal(dl.cpu(), lengths + 1)


def _fresh_runner(dtype, blocks, block_size, graphs=False, max_batch=8):
    g = gold()
    model = LM.seeded_model(LM.tiny_llama_config(), g["seed"], dtype=dtype, device="cuda")
    return R.PagedLlama(model, None, blocks=blocks, block_size=block_size, max_batch=max_batch,
                        max_tokens=1024, graphs=graphs)


def test_runner_fp32_matches_reference_logits(pkg, cuda):
    g = gold()
    runner = _fresh_runner(torch.float32, g["blocks"], g["block_size"])
    out = LM.run_scenario(runner, g["steps"])
    errs = [rel_err(a, b) for a, b in zip(out, g["logits"])]
    print("fp32 runner vs reference logits, max error / max |logit| per step:", errs)
    assert max(errs) < 1e-5
    assert pkg.read_device_errors() == 0


def test_runner_fp16_matches_oracle_runner_on_gpu(pkg, cuda):
    g = gold()
    runner = _fresh_runner(torch.float16, g["blocks"], g["block_size"])
    model = LM.seeded_model(LM.tiny_llama_config(), g["seed"], dtype=torch.float16,
                            device="cuda")
    oracle = LM.PagedLlamaOracle(model, blocks=g["blocks"], block_size=g["block_size"])
    out = LM.run_scenario(runner, g["steps"])
    ref = LM.run_scenario(oracle, g["steps"])
    errs = [rel_err(a, b) for a, b in zip(out, ref)]
    print("fp16 runner vs oracle runner, max error / max |logit| per step:", errs)
    assert max(errs) < 5e-3
    # the pools: same pages hold the same tokens (RoPE'd k within FP16 parity)
    assert_parity(runner.cache.keys, oracle.cache.keys, "k pools")
    assert_parity(runner.cache.values, oracle.cache.values, "v pools")
    assert pkg.read_device_errors() == 0


def test_graph_ticks_equal_eager_ticks(pkg, cuda):
    """Decode ticks replayed from a CUDA graph (captured once per batch size)
    give bit-identical logits and pools to eager ticks."""
    g = gold()
    eager = _fresh_runner(torch.float16, g["blocks"], g["block_size"])
    graphed = _fresh_runner(torch.float16, g["blocks"], g["block_size"], graphs=True)
    steps = LM.scenario(seed=9, decode_steps=6)
    a = LM.run_scenario(eager, steps)
    b = LM.run_scenario(graphed, steps)
    assert len(graphed._b200_graphs) == 1  # batch 3: one eager tick, then one graph replayed
    for x, y in zip(a, b):
        assert torch.equal(x, y)
    assert torch.equal(eager.cache.keys, graphed.cache.keys)
    assert torch.equal(eager.cache.values, graphed.cache.values)
    assert pkg.read_device_errors() == 0


def test_graphs_of_two_batch_sizes_keep_their_workspaces(pkg, cuda):
    """A tick graph captured at batch 1 keeps valid attention scratch after a
    batch-8 tick grows the stream's workspace (the graph addresses the buffer
    it was captured with; that buffer must not return to the allocator):
    later replays of the batch-1 graph match eager ticks bit for bit, and
    tensors allocated after the growth keep their contents."""
    eager = _fresh_runner(torch.float16, 64, 16)
    graphed = _fresh_runner(torch.float16, 64, 16, graphs=True)
    gen = torch.Generator().manual_seed(5)
    ids = [f"r{i}" for i in range(8)]
    prompts = [torch.randint(0, 512, (int(n),), generator=gen).tolist()
               for n in torch.randint(3, 60, (8,), generator=gen)]
    plan = [ids[:1]] * 3 + [ids] * 3 + [ids[:1]] * 3
    tokens = [torch.randint(0, 512, (len(b),), generator=gen).tolist() for b in plan]
    for run in (eager, graphed):
        for r in ids:
            assert run.cache.reserve(r, 100)
        run.prefill(ids, prompts)
    ws = import_module("ops")._ws_cache
    fill = []
    for step, (batch, toks) in enumerate(zip(plan, tokens)):
        if step == 6:  # the batch-8 ticks have grown the workspace: reuse freed memory now
            fill = [torch.full((1 << 18,), 1234567, dtype=torch.int32, device=cuda)
                    for _ in range(24)]
        a = eager.decode(batch, toks)
        b = graphed.decode(batch, toks)
        assert torch.equal(a, b), f"step {step}, batch {len(batch)}"
    assert sorted(graphed._b200_graphs) == [1, 8]
    assert all(bool((t == 1234567).all()) for t in fill)
    assert torch.equal(eager.cache.keys, graphed.cache.keys)
    assert len(ws) > 0
    assert pkg.read_device_errors() == 0


def test_install_on_a_llama_module(pkg, cuda):
    """install() routes PagedLlama.decode/prefill of a worker.llama-shaped
    module to the B200 methods for attention='cuda' instances (their own
    TensorPagedKV adopted), and leaves attention='torch' instances alone."""
    class PagedLlama(LM.PagedLlamaOracle):
        def __init__(self, model, blocks, block_size, attention):
            super().__init__(model, blocks, block_size)
            self.attention = attention

    mod = types.ModuleType("llama_like")
    mod.PagedLlama = PagedLlama
    g = gold()
    model = LM.seeded_model(LM.tiny_llama_config(), g["seed"], dtype=torch.float16,
                            device="cuda")
    plain = LM.PagedLlamaOracle(model, g["blocks"], g["block_size"])
    ref = LM.run_scenario(plain, g["steps"])
    pkg.install(mod)
    try:
        cuda_inst = mod.PagedLlama(model, g["blocks"], g["block_size"], "cuda")
        torch_inst = mod.PagedLlama(model, g["blocks"], g["block_size"], "torch")
        out = LM.run_scenario(cuda_inst, g["steps"])
        same = LM.run_scenario(torch_inst, g["steps"])
    finally:
        pkg.uninstall(mod)
    assert max(rel_err(a, b) for a, b in zip(out, ref)) < 5e-3
    for a, b in zip(same, ref):
        assert torch.equal(a, b)
    assert cuda_inst._b200_cache.keys is cuda_inst.cache.keys  # adopted, not copied
    assert pkg.read_device_errors() == 0
