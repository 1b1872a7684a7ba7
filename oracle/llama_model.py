"""Oracle: PagedLlama prefill and decode (test infrastructure only).

Restates the batched Llama runner of worker/llama.py:89-177 over the
oracle's paged cache (kv_cache.PagedKVCache = TensorPagedKV, :13-55), RoPE
(rope.rope = PagedLlama.rope, :108-117) and torch attention
(paged_attention.paged_attention = torch_paged_attention, :58-71). Hugging
Face supplies the model modules, as in the reference. Used by the tests as
the checker of the B200 runner (llama_runner.PagedLlama) on the same seeded
random-init model, on the CPU or — for FP16 and the larger shapes — on the
GPU with the same torch ops. Pinned to logits produced by the reference's own
PagedLlama (tests/golden/make_golden.py, "llama_tiny").
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from .kv_cache import PagedKVCache
from .paged_attention import paged_attention
from .rope import rope


def rope_theta(config) -> float:
    """config.rope_theta (transformers 4) or rope_parameters['rope_theta'] (5)."""
    theta = getattr(config, "rope_theta", None)
    if theta is None:
        theta = config.rope_parameters["rope_theta"]
    return float(theta)


class PagedLlamaOracle:
    """``attention`` plays the role of the reference's attention choice
    (worker/llama.py:162): the torch path by default, or any function with
    the paged_attention signature (e.g. the reference's own CUDA kernel)."""

    def __init__(self, model, blocks: int = 256, block_size: int = 16, attention=None):
        self.model = model.eval()
        self.attention_fn = attention or paged_attention
        self.config = model.config
        self.device = next(model.parameters()).device
        self.dtype = next(model.parameters()).dtype
        self.heads = self.config.num_attention_heads
        self.kv_heads = self.config.num_key_value_heads
        self.head_dim = getattr(self.config, "head_dim", None) or (
            self.config.hidden_size // self.heads)
        self.cache = PagedKVCache(self.config.num_hidden_layers, self.kv_heads, self.head_dim,
                                  blocks, block_size, self.device, self.dtype)
        # worker/llama.py:105-106, computed on the model's device
        self.inv_freq = 1.0 / (rope_theta(self.config) ** (
            torch.arange(0, self.head_dim, 2, device=self.device, dtype=torch.float32)
            / self.head_dim))

    @torch.inference_mode()
    def prefill(self, ids, token_lists):
        """worker/llama.py:119-149."""
        batch, width = len(ids), max(map(len, token_lists))
        tokens = torch.zeros((batch, width), device=self.device, dtype=torch.long)
        valid = torch.zeros((batch, width), device=self.device, dtype=torch.bool)
        for row, (request_id, sequence) in enumerate(zip(ids, token_lists)):
            tokens[row, :len(sequence)] = torch.tensor(sequence, device=self.device)
            valid[row, :len(sequence)] = True
            self.cache.lengths[request_id] = len(sequence)
        slots = self.cache.slots(ids, [range(len(s)) for s in token_lists])
        positions = torch.arange(width, device=self.device)[None, :].expand(batch, -1)
        x = self.model.model.embed_tokens(tokens)
        for index, layer in enumerate(self.model.model.layers):
            residual = x
            normalized = layer.input_layernorm(x)
            attn = layer.self_attn
            q = attn.q_proj(normalized).view(batch, width, self.heads, self.head_dim)
            k = attn.k_proj(normalized).view(batch, width, self.kv_heads, self.head_dim)
            v = attn.v_proj(normalized).view(batch, width, self.kv_heads, self.head_dim)
            q, k = rope(q, k, positions, self.inv_freq)
            self.cache.keys[index][slots] = k[valid]
            self.cache.values[index][slots] = v[valid]
            groups = self.heads // self.kv_heads
            context = F.scaled_dot_product_attention(
                q.transpose(1, 2), k.repeat_interleave(groups, dim=2).transpose(1, 2),
                v.repeat_interleave(groups, dim=2).transpose(1, 2), is_causal=True)
            x = residual + attn.o_proj(context.transpose(1, 2).reshape(batch, width, -1))
            x = x + layer.mlp(layer.post_attention_layernorm(x))
        last = torch.tensor([len(s) - 1 for s in token_lists], device=self.device)
        hidden = self.model.model.norm(x[torch.arange(batch, device=self.device), last])
        return self.model.lm_head(hidden).float()

    @torch.inference_mode()
    def decode(self, ids, tokens):
        """worker/llama.py:151-177 with the torch attention path."""
        batch = len(ids)
        positions_list = [self.cache.lengths[i] for i in ids]
        slots = self.cache.slots(ids, [[p] for p in positions_list])
        positions = torch.tensor(positions_list, device=self.device)[:, None]
        for request_id in ids:
            self.cache.lengths[request_id] += 1
        tables, lengths, max_length = self.cache.metadata(ids)
        token_tensor = torch.tensor(tokens, device=self.device, dtype=torch.long)[:, None]
        x = self.model.model.embed_tokens(token_tensor)
        for index, layer in enumerate(self.model.model.layers):
            residual = x
            normalized = layer.input_layernorm(x)
            attn = layer.self_attn
            q = attn.q_proj(normalized).view(batch, 1, self.heads, self.head_dim)
            k = attn.k_proj(normalized).view(batch, 1, self.kv_heads, self.head_dim)
            v = attn.v_proj(normalized).view(batch, 1, self.kv_heads, self.head_dim)
            q, k = rope(q, k, positions, self.inv_freq)
            self.cache.keys[index][slots] = k[:, 0]
            self.cache.values[index][slots] = v[:, 0]
            context = self.attention_fn(q[:, 0], self.cache.keys[index],
                                        self.cache.values[index], tables, lengths, max_length)
            x = residual + attn.o_proj(context.reshape(batch, 1, -1))
            x = x + layer.mlp(layer.post_attention_layernorm(x))
        return self.model.lm_head(self.model.model.norm(x[:, 0])).float()


def tiny_llama_config():
    """The small Llama used by the runner's parity tests (SmolLM2-like: tied
    embeddings, GQA 2, head_dim 64, theta 1e5)."""
    from transformers import LlamaConfig
    return LlamaConfig(vocab_size=512, hidden_size=256, intermediate_size=512,
                       num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
                       head_dim=64, max_position_embeddings=8192, rms_norm_eps=1e-5,
                       rope_theta=1e5, tie_word_embeddings=True)


def smollm2_135m_config():
    """SmolLM2-135M architecture (hidden 576, 30 layers, 9/3 heads, head_dim 64,
    MLP 1536, RMSNorm eps 1e-5, vocab 49152, theta 1e5, tied embeddings)."""
    from transformers import LlamaConfig
    return LlamaConfig(vocab_size=49152, hidden_size=576, intermediate_size=1536,
                       num_hidden_layers=30, num_attention_heads=9, num_key_value_heads=3,
                       head_dim=64, max_position_embeddings=8192, rms_norm_eps=1e-5,
                       rope_theta=1e5, tie_word_embeddings=True)


def seeded_model(config, seed: int, dtype=torch.float32, device="cpu"):
    """Random-init LlamaForCausalLM, identical for the same seed and versions
    (initialised on the CPU, then cast and moved)."""
    from transformers import LlamaForCausalLM
    torch.manual_seed(seed)
    model = LlamaForCausalLM(config).eval()
    for p in model.parameters():
        p.requires_grad_(False)
    return model.to(dtype=dtype, device=device)


def weights_checksum(model) -> float:
    return float(sum(p.detach().double().abs().sum() for p in model.parameters()))


# The scripted serving scenario of the runner tests: (op, payload) steps.
# Requests join by prefill, decode together, one leaves (its pages return to
# the free list uncleared) and another joins on reused pages. Decode tokens
# are drawn from the seed (not sampled from the logits), so runners whose
# logits differ in the last bits still see the same inputs.
def scenario(seed: int = 7, vocab: int = 512, decode_steps: int = 3):
    g = torch.Generator().manual_seed(seed)

    def toks(n):
        return torch.randint(0, vocab, (n,), generator=g).tolist()

    steps = [("reserve", {"a": 96, "b": 64, "c": 160}),
             ("prefill", {"a": toks(21), "b": toks(5), "c": toks(40)})]
    for _ in range(decode_steps):
        steps.append(("decode", {r: toks(1)[0] for r in ("a", "b", "c")}))
    steps.append(("release", ["b"]))
    steps.append(("reserve", {"d": 48}))
    steps.append(("prefill", {"d": toks(16)}))
    for _ in range(decode_steps):
        steps.append(("decode", {r: toks(1)[0] for r in ("a", "c", "d")}))
    return steps


def run_scenario(runner, steps):
    """Drive a PagedLlama-like runner through the scenario. Returns the
    logits of every prefill / decode step, on the CPU."""
    out = []
    for op, payload in steps:
        if op == "reserve":
            for rid, n in payload.items():
                assert runner.cache.reserve(rid, n)
        elif op == "release":
            for rid in payload:
                runner.cache.release(rid)
        elif op == "prefill":
            ids = list(payload)
            out.append(runner.prefill(ids, [payload[i] for i in ids]).cpu())
        else:
            ids = list(payload)
            out.append(runner.decode(ids, [payload[i] for i in ids]).cpu())
    return out
