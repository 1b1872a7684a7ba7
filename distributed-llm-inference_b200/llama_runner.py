"""Batched Llama decode on the B200 ops: worker/llama.py's PagedLlama, rebuilt.

``PagedLlama`` has the reference class's constructor, attributes and methods
(worker/llama.py:89-177): Hugging Face supplies the checkpoint and the layer
modules (norms, projections, MLP), this class runs prefill and decode with
the cache access on this library's kernels:

* decode (worker/llama.py:151-177): the batch's tables and lengths live on
  the GPU (``DevicePagedKV``); per layer one ``decode_attention`` launch (RoPE
  of q and k, k/v written to the new token's slot, attention) after the
  step's lengths are advanced once on the device — or, for shapes the fused
  kernel does not cover, ``rope_kv_write_decode`` (the first layer advancing
  the lengths) followed by ``paged_attention``. A step needs no host-side
  slot, position or metadata tensors, so with ``graphs=True`` the whole tick
  (embedding, every layer, final norm, LM head) is captured once per batch
  size as a CUDA graph and replayed; only the new token ids are copied in.
* prefill (worker/llama.py:119-149): RoPE and the paged KV writes of every
  prompt token in one ``rope_kv_write`` per layer (``valid`` mask), then the
  causal attention from the pools (``prefill_attention``: no padding, no
  repeated K/V) for FP16 with head_dim 64 or 128; other shapes use causal SDPA
  over the padded prompts as the reference does.

``b200_decode`` / ``b200_prefill`` are the same methods as plain functions, so
``integration.install`` can put them on the reference's own class.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from .ops import (decode_attention, decode_attention_supported, paged_attention,
                  prefill_attention, rope_kv_write, rope_kv_write_decode)
from .paged_kv import DevicePagedKV


def _rope_theta(config) -> float:
    theta = getattr(config, "rope_theta", None)
    if theta is None:  # transformers >= 5 keeps it in rope_parameters
        theta = config.rope_parameters["rope_theta"]
    return float(theta)


def _device_cache(runner) -> DevicePagedKV:
    cache = runner.cache
    if not isinstance(cache, DevicePagedKV):
        cache = getattr(runner, "_b200_cache", None)
        if cache is None or cache.keys is not runner.cache.keys:
            cache = DevicePagedKV.adopt(runner.cache)
            runner._b200_cache = cache
    return cache


def _side_stream(runner) -> torch.cuda.Stream:
    """The runner's capture stream; eager warm-up ticks run on it too, so the
    attention workspace (cached per stream) exists before capture."""
    s = runner.__dict__.get("_b200_stream")
    if s is None:
        s = runner._b200_stream = torch.cuda.Stream(runner.device)
    return s


class _TickGraph:
    """One captured decode tick for a fixed batch size. Capture records the
    launches without running them; ``run`` copies the token ids in and
    replays. max_length is the tables' capacity: reads are bounded by the
    device lengths, which the graph reads at replay time."""

    def __init__(self, runner, batch: int):
        dev = runner.device
        cache = _device_cache(runner)
        self.tokens = torch.zeros((batch, 1), dtype=torch.long, device=dev)
        tables, lengths = cache.dev_tables[:batch], cache.dev_lengths[:batch]
        stream = _side_stream(runner)
        stream.wait_stream(torch.cuda.current_stream(dev))
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=stream):
            self.logits = _tick(runner, cache, self.tokens, tables, lengths, cache.max_tokens)
        torch.cuda.current_stream(dev).wait_stream(stream)

    def run(self, tokens: torch.Tensor) -> torch.Tensor:
        self.tokens.copy_(tokens, non_blocking=True)
        self.graph.replay()
        return self.logits


def _fused_weights(layer):
    """The layer's q/k/v and gate/up projections as one weight each, so a
    decode tick runs one GEMM for q, k, v and one for gate, up. The modules'
    weights become views of them: the same values, no extra memory. Layers
    with projection biases keep their modules (returns None)."""
    cached = layer.__dict__.get("_b200_fused")
    if cached is not None:
        return cached or None
    attn, mlp = layer.self_attn, layer.mlp
    mods = (attn.q_proj, attn.k_proj, attn.v_proj, attn.o_proj, mlp.gate_proj, mlp.up_proj,
            mlp.down_proj)
    if any(getattr(m, "bias", None) is not None for m in mods):
        layer._b200_fused = False
        return None

    def fuse(group):
        w = torch.cat([m.weight.detach() for m in group], 0)
        off = 0
        for m in group:
            n = m.weight.shape[0]
            m.weight = torch.nn.Parameter(w[off:off + n], requires_grad=False)
            off += n
        return w

    with torch.no_grad():
        layer._b200_fused = (fuse((attn.q_proj, attn.k_proj, attn.v_proj)),
                             fuse((mlp.gate_proj, mlp.up_proj)))
    return layer._b200_fused


def _rms_norm(norm, x):
    """LlamaRMSNorm in one fused op (fp32 statistics, one rounding)."""
    eps = getattr(norm, "variance_epsilon", None) or getattr(norm, "eps", 1e-6)
    return F.rms_norm(x, (x.shape[-1],), norm.weight, eps)


def _tick(runner, cache, token_tensor, tables, lengths, max_length):
    """Embedding -> layers -> norm -> LM head for one decode token per sequence."""
    batch = token_tensor.size(0)
    x = runner.model.model.embed_tokens(token_tensor)
    fused = decode_attention_supported(
        torch.empty((batch, runner.heads, runner.head_dim), dtype=runner.dtype,
                    device="meta"), cache.keys[0])
    if fused:
        lengths.add_(1)  # the new token (PagedLlama.decode, worker/llama.py:157-158)
    H, KVH, D = runner.heads, runner.kv_heads, runner.head_dim
    for index, layer in enumerate(runner.model.model.layers):
        weights = _fused_weights(layer) if fused else None
        if weights is not None:
            # one GEMM for q/k/v (the attention reads its row slices), the
            # residual adds folded into the o and down GEMMs (addmm)
            wqkv, wgu = weights
            attn, mlp = layer.self_attn, layer.mlp
            x2 = x.view(batch, -1)
            qkv = F.linear(_rms_norm(layer.input_layernorm, x2), wqkv)
            q = qkv[:, :H * D].view(batch, H, D)
            k = qkv[:, H * D:(H + KVH) * D].view(batch, KVH, D)
            v = qkv[:, (H + KVH) * D:].view(batch, KVH, D)
            context = decode_attention(q, k, v, cache.keys[index], cache.values[index], tables,
                                       lengths, runner.inv_freq, max_length,
                                       metadata_stable=index > 0)
            x2 = torch.addmm(x2, context.view(batch, -1), attn.o_proj.weight.t())
            gu = F.linear(_rms_norm(layer.post_attention_layernorm, x2), wgu)
            inter = wgu.shape[0] // 2
            act = mlp.act_fn(gu[:, :inter]) * gu[:, inter:]
            x = torch.addmm(x2, act, mlp.down_proj.weight.t()).view(batch, 1, -1)
            continue
        residual = x
        normalized = layer.input_layernorm(x)
        attn = layer.self_attn
        q = attn.q_proj(normalized).view(batch, runner.heads, runner.head_dim)
        k = attn.k_proj(normalized).view(batch, runner.kv_heads, runner.head_dim)
        v = attn.v_proj(normalized).view(batch, runner.kv_heads, runner.head_dim)
        if fused:
            context = decode_attention(q, k, v, cache.keys[index], cache.values[index], tables,
                                       lengths, runner.inv_freq, max_length,
                                       metadata_stable=index > 0)
        else:
            q, k = rope_kv_write_decode(q, k, v, cache.keys[index], cache.values[index],
                                        tables, lengths, runner.inv_freq,
                                        advance=index == 0, inplace=True)
            context = paged_attention(q, cache.keys[index], cache.values[index], tables,
                                      lengths, max_length)
        x = residual + attn.o_proj(context.reshape(batch, 1, -1))
        x = x + layer.mlp(layer.post_attention_layernorm(x))
    return runner.model.lm_head(runner.model.model.norm(x[:, 0])).float()


@torch.inference_mode()
def b200_decode(self, ids, tokens):
    """PagedLlama.decode (worker/llama.py:151-177) on the fused decode ops.

    Same inputs, outputs and cache effects: the new token of each sequence is
    written at position lengths[id] (then lengths[id] += 1) and the logits of
    the next token are returned as float32 [batch, vocab]."""
    cache = _device_cache(self)
    batch = len(ids)
    tables, lengths = cache.bind(ids)
    max_length = cache.advance(ids)
    tok = torch.as_tensor(tokens, dtype=torch.long).view(batch, 1)
    if getattr(self, "graphs", False):
        graphs = self.__dict__.setdefault("_b200_graphs", {})
        g = graphs.get(batch)
        if g is None:
            # The first tick of a batch size runs eagerly on the capture
            # stream (kernel attributes and workspaces get set up), the next
            # one is captured and from then on replayed.
            cur, side = torch.cuda.current_stream(self.device), _side_stream(self)
            side.wait_stream(cur)
            with torch.cuda.stream(side):
                out = _tick(self, cache, tok.to(self.device), tables, lengths, cache.max_tokens)
            cur.wait_stream(side)
            graphs[batch] = "warm"
            return out
        if g == "warm":
            g = graphs[batch] = _TickGraph(self, batch)
        return g.run(tok.to(self.device, non_blocking=True)).clone()
    return _tick(self, cache, tok.to(self.device), tables, lengths, max_length)


@torch.inference_mode()
def b200_prefill(self, ids, token_lists):
    """PagedLlama.prefill (worker/llama.py:119-149) with RoPE and the paged KV
    writes of every prompt token fused into one launch per layer."""
    cache = _device_cache(self)
    batch, width = len(ids), max(map(len, token_lists))
    tokens = torch.zeros((batch, width), device=self.device, dtype=torch.long)
    valid = torch.zeros((batch, width), device=self.device, dtype=torch.bool)
    for row, (request_id, sequence) in enumerate(zip(ids, token_lists)):
        tokens[row, :len(sequence)] = torch.tensor(sequence, device=self.device)
        valid[row, :len(sequence)] = True
        cache.lengths[request_id] = len(sequence)
    physical, offsets = cache.slots(ids, [range(len(s)) for s in token_lists])
    positions = torch.arange(width, device=self.device)[None, :].expand(batch, -1).contiguous()
    x = self.model.model.embed_tokens(tokens)
    groups = self.heads // self.kv_heads
    paged = self.dtype == torch.float16 and self.head_dim in (64, 128)
    if paged:
        tables, lengths, _ = cache.metadata(ids)
    for index, layer in enumerate(self.model.model.layers):
        residual = x
        normalized = layer.input_layernorm(x)
        attn = layer.self_attn
        q = attn.q_proj(normalized).view(batch, width, self.heads, self.head_dim)
        k = attn.k_proj(normalized).view(batch, width, self.kv_heads, self.head_dim)
        v = attn.v_proj(normalized).view(batch, width, self.kv_heads, self.head_dim)
        q, k = rope_kv_write(q, k, v.contiguous(), cache.keys[index], cache.values[index],
                             physical, offsets, positions, self.inv_freq, valid=valid,
                             inplace=True)
        if paged:
            context = prefill_attention(q, cache.keys[index], cache.values[index], tables,
                                        lengths)
        else:
            context = F.scaled_dot_product_attention(
                q.transpose(1, 2), k.repeat_interleave(groups, dim=2).transpose(1, 2),
                v.repeat_interleave(groups, dim=2).transpose(1, 2),
                is_causal=True).transpose(1, 2)
        x = residual + attn.o_proj(context.reshape(batch, width, -1))
        x = x + layer.mlp(layer.post_attention_layernorm(x))
    last = torch.tensor([len(s) - 1 for s in token_lists], device=self.device)
    hidden = self.model.model.norm(x[torch.arange(batch, device=self.device), last])
    return self.model.lm_head(hidden).float()


class PagedLlama:
    """worker/llama.py:89-116 with a DevicePagedKV cache and the B200 methods."""

    def __init__(self, model, tokenizer=None, blocks=256, block_size=16, attention="cuda",
                 max_batch=256, max_tokens=8192, graphs=False):
        self.model = model.eval()
        self.tokenizer = tokenizer
        self.config = model.config
        if self.config.model_type != "llama":
            raise ValueError("Only Llama checkpoints with unscaled RoPE are supported")
        scaling = getattr(self.config, "rope_scaling", None)
        if scaling not in (None, {}) and (scaling.get("rope_type", "default") != "default"):
            raise ValueError("Only Llama checkpoints with unscaled RoPE are supported")
        self.device = next(model.parameters()).device
        self.dtype = next(model.parameters()).dtype
        if self.device.type != "cuda":
            raise ValueError("the B200 path requires an NVIDIA CUDA device")
        self.heads = self.config.num_attention_heads
        self.kv_heads = self.config.num_key_value_heads
        self.head_dim = getattr(self.config, "head_dim", None) or (
            self.config.hidden_size // self.heads)
        self.cache = DevicePagedKV(self.config, blocks, block_size, self.device, self.dtype,
                                   max_batch=max_batch, max_tokens=max_tokens)
        self.attention = attention
        self.graphs = graphs
        self.inv_freq = 1.0 / (_rope_theta(self.config) ** (
            torch.arange(0, self.head_dim, 2, device=self.device, dtype=torch.float32)
            / self.head_dim))

    decode = b200_decode
    prefill = b200_prefill
