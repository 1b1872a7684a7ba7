"""Generate the golden fixtures of tests/golden/ from the REFERENCE's own code.

Run where the reference checkout (read-only) is available:

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py [/path/to/reference]

Without an argument the checkout is found by oracle/refroot.py
(PDB_REFERENCE_ROOT, else a ``reference`` directory beside this repository).

It imports worker.llama (torch_paged_attention, PagedLlama.rope) and
worker.engine (PagedKV) from the reference, feeds them the seeded inputs of
the package's workloads module (CPU generators, deterministic), and saves the
reference's outputs, plus SHA-256 digests of the inputs so that a drift of
the input generators is detected. The fixtures travel with the repository;
the reference itself does not.
"""
from __future__ import annotations

import hashlib
import importlib
import math
import sys
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO))
W = importlib.import_module("distributed-llm-inference_b200.workloads")


def digest(t: torch.Tensor) -> str:
    return hashlib.sha256(t.detach().contiguous().cpu().view(torch.uint8).numpy().tobytes()).hexdigest()


class _RopeHost:
    """Stand-in `self` for the unbound PagedLlama.rope (it only reads inv_freq)."""

    def __init__(self, inv_freq):
        self.inv_freq = inv_freq


def edge_case_specs():
    """Small decode cases covering the reference's edge cases: zero length,
    length 1, page-boundary lengths, non-power-of-two block sizes, MHA / GQA /
    MQA groupings, several head dims, fp32 and fp16."""
    specs = []
    shapes = [
        # (B, H, KVH, D, bs)
        (7, 4, 2, 32, 16),
        (7, 9, 3, 64, 16),
        (7, 8, 8, 64, 16),     # MHA
        (7, 8, 1, 64, 16),     # MQA, group 8
        (7, 32, 8, 128, 16),
        (7, 4, 4, 128, 8),
        (7, 6, 2, 40, 5),      # odd block size, head_dim not a multiple of 32
        (7, 2, 1, 256, 16),
        (7, 16, 2, 128, 16),   # group 8 at D=128
    ]
    for dtype in ("float32", "float16"):
        for i, (B, H, KVH, D, bs) in enumerate(shapes):
            lengths = [0, 1, bs - 1, bs, bs + 1, 2 * bs + 3, 70]
            specs.append(dict(name=f"{dtype}-{i}", dtype=dtype, B=B, H=H, KVH=KVH, D=D, bs=bs,
                              lengths=lengths, seed=1000 + i))
    return specs


def edge_case_inputs(spec):
    dtype = getattr(torch, spec["dtype"])
    g = torch.Generator().manual_seed(spec["seed"])
    lengths = torch.tensor(spec["lengths"], dtype=torch.int32)
    bs = spec["bs"]
    need = sum(math.ceil(n / bs) for n in spec["lengths"])
    blocks = need + 5
    max_len = max(spec["lengths"])
    width = math.ceil(max_len / bs)
    perm = torch.randperm(blocks, generator=g)
    tables = torch.zeros(spec["B"], width, dtype=torch.int32)
    off = 0
    for b, n in enumerate(spec["lengths"]):
        c = math.ceil(n / bs)
        tables[b, :c] = perm[off:off + c].to(torch.int32)
        off += c
    q = torch.randn(spec["B"], spec["H"], spec["D"], generator=g).to(dtype)
    k = torch.randn(blocks, bs, spec["KVH"], spec["D"], generator=g).to(dtype)
    v = torch.randn(blocks, bs, spec["KVH"], spec["D"], generator=g).to(dtype)
    return q, k, v, tables, lengths, max_len


def rope_specs():
    out = []
    for dtype in ("float32", "float16"):
        for D, theta in ((64, 1e5), (128, 5e5), (32, 1e4)):
            out.append(dict(dtype=dtype, D=D, theta=theta, H=3, KVH=1, seed=77 + D))
    return out


ROPE_POSITIONS = [0, 1, 2, 15, 16, 17, 127, 128, 1000, 1023, 2047, 4095, 4096, 6000, 8190, 8191]


def rope_inputs(spec):
    dtype = getattr(torch, spec["dtype"])
    g = torch.Generator().manual_seed(spec["seed"])
    P = len(ROPE_POSITIONS)
    q = (torch.randn(1, P, spec["H"], spec["D"], generator=g) * 3).to(dtype)
    k = (torch.randn(1, P, spec["KVH"], spec["D"], generator=g) * 3).to(dtype)
    pos = torch.tensor([ROPE_POSITIONS], dtype=torch.int64)
    return q, k, pos


PREFILL_ATTENTION = dict(
    model_seed=4321, token_seed=8, blocks=40, block_size=16,
    # earlier requests whose pages are released uncleared before the prompts
    # are admitted, so the prompts' pages are fragmented and hold stale rows
    warm={"w0": 50, "w1": 33, "w2": 90},
    # ragged prompts: partial pages, exact page multiples, a single token
    prompts={"p0": 37, "p1": 5, "p2": 64, "p3": 70, "p4": 16, "p5": 1},
)


def prefill_attention_config():
    """The tiny Llama of the runner fixtures (GQA 2, head_dim 64) with weights
    drawn at std 0.05, so that q, k and v come out near unit scale and the
    attention outputs are large enough for an absolute FP16 bar to mean
    something (at the default std 0.02 they would be ~1e-2)."""
    from oracle import llama_model as LM
    cfg = LM.tiny_llama_config()
    cfg.initializer_range = 0.05
    return cfg


def prefill_attention_capture(paged_llama_cls, dtype_name: str) -> dict:
    """Run the reference's PagedLlama.prefill on the spec above and record,
    per layer, what its attention consumed and produced: the rotated q (the
    output of its rope call), the k/v rows it wrote to the pool (read back
    from the cache through the slots), and the attention context (the input
    of o_proj). Only rows of real prompt tokens are kept; padded rows feed no
    real token's output."""
    from oracle import llama_model as LM
    spec = PREFILL_ATTENTION
    dtype = getattr(torch, dtype_name)
    cfg = prefill_attention_config()
    model = LM.seeded_model(cfg, seed=spec["model_seed"], dtype=dtype)
    cfg.rope_theta = LM.rope_theta(cfg)   # transformers-5 shim, as in section 7
    cfg.rope_scaling = None
    runner = paged_llama_cls(model, None, blocks=spec["blocks"],
                             block_size=spec["block_size"], attention="torch")
    g = torch.Generator().manual_seed(spec["token_seed"])

    def toks(n):
        return torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist()

    warm = spec["warm"]
    for rid, n in warm.items():
        assert runner.cache.reserve(rid, n)
    runner.prefill(list(warm), [toks(n) for n in warm.values()])
    for rid in ("w1", "w0", "w2"):
        runner.cache.release(rid)
    prompts = spec["prompts"]
    for rid, n in prompts.items():
        assert runner.cache.reserve(rid, n)
    ids = list(prompts)
    token_lists = [toks(n) for n in prompts.values()]

    layers = len(model.model.layers)
    qs, ctxs = [None] * layers, [None] * layers
    calls = []

    def rope_hook(q, k, positions):
        qo, ko = paged_llama_cls.rope(runner, q, k, positions)
        qs[len(calls)] = qo.clone()
        calls.append(1)
        return qo, ko

    runner.rope = rope_hook
    hooks = [layer.self_attn.o_proj.register_forward_pre_hook(
        lambda mod, args, i=i: ctxs.__setitem__(i, args[0].clone()))
        for i, layer in enumerate(model.model.layers)]
    try:
        runner.prefill(ids, token_lists)
    finally:
        for h in hooks:
            h.remove()
        del runner.rope
    tables, lengths, _ = runner.cache.metadata(ids)
    lens = list(prompts.values())
    width = max(lens)
    valid = torch.arange(width)[None, :] < torch.tensor(lens)[:, None]
    physical, offsets = runner.cache.slots(ids, [range(n) for n in lens])
    H, KVH, D = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
    out = dict(spec=spec, dtype=dtype_name, heads=H, kv_heads=KVH, head_dim=D,
               tables=tables, lengths=lengths, layers=[])
    for i in range(layers):
        out["layers"].append(dict(
            q=qs[i][valid],                                              # [T, H, D]
            k=runner.cache.keys[i][physical, offsets].clone(),           # [T, KVH, D]
            v=runner.cache.values[i][physical, offsets].clone(),
            context=ctxs[i].view(len(ids), width, H, D)[valid]))         # [T, H, D]
    return out


def main(ref_root: str) -> None:
    sys.path.insert(0, ref_root)
    from worker.llama import PagedLlama, torch_paged_attention
    from worker.engine import PagedKV

    torch.set_num_threads(4)
    fixtures = {}

    # 1. The reference's own kernel test case (tests/test_llama.py:123-134), on CPU.
    case = {}
    for dtype in (torch.float32, torch.float16):
        torch.manual_seed(11)
        q = torch.randn(3, 4, 32, dtype=dtype)
        keys = torch.randn(12, 16, 2, 32, dtype=dtype)
        values = torch.randn_like(keys)
        tables = torch.tensor([[9, 2, 5], [1, 8, 4], [7, 0, 6]], dtype=torch.int32)
        lengths = torch.tensor([1, 17, 35], dtype=torch.int32)
        out = torch_paged_attention(q, keys, values, tables, lengths, 35)
        case[str(dtype).split(".")[1]] = dict(q=q, keys=keys, values=values, tables=tables,
                                              lengths=lengths, max_length=35, out=out)
    torch.save(case, HERE / "reference_kernel_case.pt")

    # 2. Edge cases (outputs + input digests; inputs are regenerated from seeds).
    edges = []
    for spec in edge_case_specs():
        q, k, v, tables, lengths, max_len = edge_case_inputs(spec)
        out = torch_paged_attention(q, k, v, tables, lengths, max_len)
        edges.append(dict(spec=spec, out=out, digests=[digest(t) for t in (q, k, v, tables, lengths)]))
    torch.save(edges, HERE / "edge_cases.pt")

    # 3. RoPE at page-boundary and large positions, both dtypes.
    ropes = []
    for spec in rope_specs():
        q, k, pos = rope_inputs(spec)
        inv = W.inv_freq(spec["theta"], spec["D"])
        ref_inv = 1.0 / (spec["theta"] ** (torch.arange(0, spec["D"], 2, dtype=torch.float32) / spec["D"]))
        assert torch.equal(inv, ref_inv)
        qo, ko = PagedLlama.rope(_RopeHost(inv), q, k, pos)
        ropes.append(dict(spec=spec, q=qo, k=ko, digests=[digest(q), digest(k)]))
    torch.save(ropes, HERE / "rope_cases.pt")

    # 4. Decode step of the SmolLM2 CPU workload: rope -> slot write -> attention.
    w = W.smollm_cpu()
    t = W.materialize(w, "cpu")
    qn = t.q[0].unsqueeze(1)
    kn = t.k[0].unsqueeze(1)
    vn = t.v[0].unsqueeze(1)
    qr, kr = PagedLlama.rope(_RopeHost(t.inv_freq), qn, kn, t.positions)
    kp, vp = t.k_pools[0].clone(), t.v_pools[0].clone()
    kp[t.physical, t.offsets] = kr[:, 0]
    vp[t.physical, t.offsets] = vn[:, 0]
    out = torch_paged_attention(qr[:, 0], kp, vp, t.tables, t.lengths, w.max_length)
    fixtures_decode = dict(
        lengths=w.lengths, tables=w.tables, q_roped=qr[:, 0], k_roped=kr[:, 0], out=out,
        k_pool_digest=digest(kp), v_pool_digest=digest(vp),
        input_digests=dict(q=digest(t.q[0]), k=digest(t.k[0]), v=digest(t.v[0]),
                           k_pool=digest(t.k_pools[0]), v_pool=digest(t.v_pools[0])))
    torch.save(fixtures_decode, HERE / "smollm_cpu_decode.pt")

    # 5. Prefill RoPE + KV write (pool[slots] = k[valid]) of the prefill workload.
    pw = W.prefill_smollm()
    d = W.materialize_prefill(pw, "cpu")
    qr, kr = PagedLlama.rope(_RopeHost(d["inv_freq"]), d["q"], d["k"], d["positions"])
    kp, vp = d["k_pool"].clone(), d["v_pool"].clone()
    kp[d["physical"], d["offsets"]] = kr[d["valid"]]
    vp[d["physical"], d["offsets"]] = d["v"][d["valid"]]
    torch.save(dict(q_roped_digest=digest(qr), k_roped_digest=digest(kr),
                    k_pool_digest=digest(kp), v_pool_digest=digest(vp),
                    input_digests=dict(q=digest(d["q"]), k=digest(d["k"]), v=digest(d["v"]),
                                       k_pool=digest(d["k_pool"]), v_pool=digest(d["v_pool"]))),
               HERE / "prefill.pt")

    # 6. Dense-softmax known answer of the scalar spec (tests/test_engine.py:19-32).
    kv = PagedKV(blocks=2, block_size=2)
    kv.reserve("a", 3)
    keys = [[1., 0.], [0., 1.], [1., 1.]]
    vals = [[2., 0.], [0., 4.], [6., 8.]]
    for kk, vv in zip(keys, vals):
        kv.append("a", kk, vv)
    fixtures["scalar"] = dict(q=[1., 2.], keys=keys, values=vals, block_size=2,
                              table=kv.tables["a"], out=kv.attention("a", [1., 2.]))
    torch.save(fixtures, HERE / "scalar_known_answer.pt")

    # 7. The reference's own PagedLlama (worker/llama.py:89-177, torch attention)
    #    on a seeded random-init tiny Llama, driven through the serving
    #    scenario (prefill, decode, release, re-admit on reused pages), CPU FP32.
    #    transformers 5 moved rope_theta into rope_parameters and reports a
    #    default rope_scaling; the two-line shim restores the 4.x view the
    #    reference reads (worker/llama.py:94, :105).
    from oracle import llama_model as LM
    cfg = LM.tiny_llama_config()
    model = LM.seeded_model(cfg, seed=1234)
    cfg.rope_theta = LM.rope_theta(cfg)
    cfg.rope_scaling = None
    runner = PagedLlama(model, None, blocks=64, block_size=16, attention="torch")
    steps = LM.scenario(seed=7, vocab=cfg.vocab_size)
    logits = LM.run_scenario(runner, steps)
    torch.save(dict(seed=1234, blocks=64, block_size=16, steps=steps, logits=logits,
                    weights_checksum=LM.weights_checksum(model),
                    k_pool_digest=digest(runner.cache.keys),
                    v_pool_digest=digest(runner.cache.values)),
               HERE / "llama_tiny_scenario.pt")
    # 8. Prefill attention of the reference's own PagedLlama.prefill
    #    (worker/llama.py:141-144: causal SDPA over the padded prompt batch,
    #    K/V repeated per query group), FP32 and FP16, on the CPU.
    torch.save({dtype: prefill_attention_capture(PagedLlama, dtype)
                for dtype in ("float32", "float16")}, HERE / "prefill_attention.pt")
    print("wrote", sorted(p.name for p in HERE.glob("*.pt")))


if __name__ == "__main__":
    from oracle.refroot import reference_root
    root = sys.argv[1] if len(sys.argv) > 1 else reference_root()
    if root is None:
        sys.exit("reference checkout not found: pass its path or set PDB_REFERENCE_ROOT")
    main(str(root))
