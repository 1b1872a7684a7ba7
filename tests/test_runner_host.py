"""Host side of the model runner (CPU): the oracle PagedLlama against the
reference's own logits, DevicePagedKV against TensorPagedKV's bookkeeping,
the minimal-upload rule of DevicePagedKV.bind, and install() on the
reference module when its checkout is present."""
from __future__ import annotations

import random
import sys
from pathlib import Path

import pytest
import torch

from conftest import REPO, golden_module, import_module, import_pkg
from oracle import kv_cache
from oracle import llama_model as LM
from oracle.refroot import reference_root

P = import_module("paged_kv")
REF = reference_root() or Path("reference-checkout-not-found")


def gold():
    return torch.load(REPO / "tests" / "golden" / "llama_tiny_scenario.pt", weights_only=False)


def test_oracle_runner_matches_reference_logits():
    """worker/llama.py:89-177 restated: bit-identical logits and pools on the CPU."""
    g = gold()
    model = LM.seeded_model(LM.tiny_llama_config(), g["seed"])
    assert LM.weights_checksum(model) == g["weights_checksum"]
    runner = LM.PagedLlamaOracle(model, blocks=g["blocks"], block_size=g["block_size"])
    out = LM.run_scenario(runner, g["steps"])
    assert len(out) == len(g["logits"])
    for a, b in zip(out, g["logits"]):
        assert torch.equal(a, b)
    digest = golden_module().digest
    assert digest(runner.cache.keys) == g["k_pool_digest"]
    assert digest(runner.cache.values) == g["v_pool_digest"]


class _Cfg:
    num_hidden_layers, num_key_value_heads, head_dim = 2, 2, 8
    num_attention_heads, hidden_size = 4, 32


def test_device_paged_kv_bookkeeping_matches_tensor_paged_kv():
    """reserve / release / slots / metadata as TensorPagedKV (worker/llama.py:26-55)."""
    rng = random.Random(5)
    ours = P.DevicePagedKV(_Cfg, blocks=40, block_size=4, device="cpu", dtype=torch.float32,
                           max_batch=8, max_tokens=64)
    ref = kv_cache.PagedKVCache(2, 2, 8, blocks=40, block_size=4)
    live = []
    for step in range(200):
        op = rng.random()
        if op < 0.4 or not live:
            rid, n = f"r{step}", rng.randint(1, 60)
            assert ours.reserve(rid, n) == ref.reserve(rid, n)
            if rid in ref.tables:
                live.append(rid)
        elif op < 0.6:
            rid = live.pop(rng.randrange(len(live)))
            ours.release(rid)
            ref.release(rid)
        else:
            for rid in live:
                ref.lengths[rid] = ours.lengths[rid] = rng.randint(1, len(ref.tables[rid]) * 4)
            ids = rng.sample(live, min(len(live), 5))
            pos = [[rng.randrange(ref.lengths[i])] for i in ids]
            for a, b in zip(ours.slots(ids, pos), ref.slots(ids, pos)):
                assert torch.equal(a, b)
            for a, b in zip(ours.metadata(ids), ref.metadata(ids)):
                assert (a == b) if isinstance(a, int) else torch.equal(a, b)
        assert ours.free == ref.free and ours.tables == ref.tables
        assert ours.lengths == ref.lengths


def test_bind_uploads_only_changed_rows():
    """A steady batch uploads nothing; a joining or re-admitted request only its row."""
    kv = P.DevicePagedKV(_Cfg, blocks=64, block_size=4, device="cpu", dtype=torch.float32,
                         max_batch=4, max_tokens=32)
    for rid, n in (("a", 20), ("b", 8), ("c", 30)):
        assert kv.reserve(rid, n)
        kv.lengths[rid] = n // 2

    def check(ids):
        tabs, lens = kv.bind(ids)
        for i, rid in enumerate(ids):
            pages = kv.tables[rid]
            assert tabs[i, :len(pages)].tolist() == pages
            assert int(lens[i]) == kv.lengths[rid]
        return tabs, lens

    check(["a", "b", "c"])
    assert kv.uploaded_rows == 3
    for _ in range(3):  # decode steps: the device lengths advance in the prologue
        kv.bind(["a", "b", "c"])
        kv.advance(["a", "b", "c"])
        kv.dev_lengths[:3] += 1  # what rope_kv_write_decode(advance=True) does
    check(["a", "b", "c"])
    assert kv.uploaded_rows == 3
    kv.release("b")
    assert kv.reserve("d", 12)
    kv.lengths["d"] = 5
    check(["a", "d", "c"])
    assert kv.uploaded_rows == 4
    kv.release("d")  # same id again, new pages: must be uploaded although id/len match
    kv.free.reverse()
    assert kv.reserve("d", 12)
    kv.lengths["d"] = 5
    check(["a", "d", "c"])
    assert kv.uploaded_rows == 5
    check(["c", "a"])  # reorder: both rows move
    assert kv.uploaded_rows == 7


@pytest.mark.skipif(not (REF / "worker" / "llama.py").exists(),
                    reason="reference checkout not present")
def test_install_keeps_torch_instances_on_the_reference_path():
    """install() wraps worker.llama.PagedLlama's methods; attention='torch'
    instances still produce the reference's logits; uninstall() restores."""
    sys.dont_write_bytecode = True
    sys.path.insert(0, str(REF))
    try:
        import worker.llama as ref_llama
    finally:
        sys.path.remove(str(REF))
    pkg = import_pkg()
    own = ref_llama.PagedLlama.decode
    pkg.install(ref_llama)
    try:
        assert ref_llama.cuda_paged_attention is pkg.cuda_paged_attention
        assert ref_llama.PagedLlama.decode is not own
        g = gold()
        cfg = LM.tiny_llama_config()
        model = LM.seeded_model(cfg, g["seed"])
        cfg.rope_theta = LM.rope_theta(cfg)
        cfg.rope_scaling = None
        runner = ref_llama.PagedLlama(model, None, blocks=g["blocks"],
                                      block_size=g["block_size"], attention="torch")
        out = LM.run_scenario(runner, g["steps"])
        for a, b in zip(out, g["logits"]):
            assert torch.equal(a, b)
    finally:
        pkg.uninstall(ref_llama)
    assert ref_llama.PagedLlama.decode is own
