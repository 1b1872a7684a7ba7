"""Reference-facing ops over the C ABI.

``paged_attention`` has the signature, argument meaning, checks, check order,
messages and error type (RuntimeError) of the reference extension op
``paged_attention`` (cuda/binding.cpp:6-26) as loaded by
``cuda_paged_attention`` (worker/llama.py:77-86). ``rope_kv_write`` fuses what
worker/llama.py does per layer before attention: ``PagedLlama.rope``
(worker/llama.py:108-117) and the paged KV-slot writes (decode :171-172,
prefill :139-140).

PyTorch is used only for device memory, the current stream and the workspace
allocation; all arithmetic runs in libpaged_decode_b200.so.
"""
from __future__ import annotations

import threading

import torch

from . import _lib

_DTYPES = {torch.float32: _lib.DTYPE_FLOAT32, torch.float16: _lib.DTYPE_FLOAT16}


def _check(cond: bool, msg: str) -> None:
    if not cond:
        raise RuntimeError(msg)


# --------------------------------------------------------------------------
# Workspace cache: one grow-only buffer per (device, stream, op). Calls on one
# stream are ordered, so calls of the same op can share it; the buffer never
# needs clearing (counters carry a per-call tag, so stale bytes count as zero).
# A CUDA graph captured with a call bakes in the buffer's address, and a
# graph does not keep the tensor alive: a buffer that a larger call replaces
# is therefore retired, never freed, so that graphs captured before the
# growth (e.g. a decode tick of a smaller batch) keep valid scratch memory.
# Buffers grow at least 2x at a time, so the retired ones together stay
# smaller than the live one.
# --------------------------------------------------------------------------
_ws_lock = threading.Lock()
_ws_cache: dict[tuple[int, int, str], torch.Tensor] = {}
_ws_retired: list[torch.Tensor] = []


def workspace(device: torch.device, stream: int, nbytes: int, tag: str) -> torch.Tensor | None:
    """Scratch for op `tag` on (device, stream); ops never share a buffer."""
    if nbytes == 0:
        return None
    key = (device.index, stream, tag)
    with _ws_lock:
        buf = _ws_cache.get(key)
        if buf is None or buf.numel() < nbytes:
            size = max(nbytes, 1 << 20)
            if buf is not None:
                size = max(size, 2 * buf.numel())
                _ws_retired.append(buf)
            buf = torch.zeros(size, dtype=torch.uint8, device=device)
            _ws_cache[key] = buf
        return buf


def _stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


class _DeviceGuard:
    """CUDAGuard(q.device()) of cuda/paged_attention.cu:62, cheap when already current."""

    __slots__ = ("idx", "prev")

    def __init__(self, device: torch.device):
        self.idx = device.index
        self.prev = None

    def __enter__(self):
        cur = torch.cuda.current_device()
        if cur != self.idx:
            self.prev = cur
            torch.cuda.set_device(self.idx)

    def __exit__(self, *exc):
        if self.prev is not None:
            torch.cuda.set_device(self.prev)


def _check_attention_inputs(q, k, v, tables, lengths, max_length) -> None:
    # cuda/binding.cpp:8-22, same order and messages.
    _check(q.is_cuda, "query must be on CUDA")
    for t in (q, k, v, tables, lengths):
        _check(t.device == q.device, "all tensors must be on the same GPU")
        _check(t.is_contiguous(), "all tensors must be contiguous")
    _check(q.dim() == 3 and k.dim() == 4 and k.shape == v.shape, "invalid Q/K/V shapes")
    _check(q.size(0) > 0 and q.size(1) > 0 and q.size(2) > 0 and q.size(2) <= 256,
           "invalid query shape")
    _check(k.size(0) > 0 and k.size(1) > 0 and k.size(2) > 0 and k.size(3) == q.size(2),
           "invalid cache shape")
    _check(q.size(1) % k.size(2) == 0, "query heads must be a multiple of KV heads")
    _check(q.dtype in _DTYPES, "use FP32 or FP16")
    _check(k.dtype == q.dtype and v.dtype == q.dtype, "dtype mismatch")
    _check(tables.dtype == torch.int32 and lengths.dtype == torch.int32, "metadata must be int32")
    _check(tables.dim() == 2 and tables.size(0) == q.size(0), "invalid block tables")
    _check(lengths.dim() == 1 and lengths.size(0) == q.size(0), "invalid lengths")
    _check(max_length > 0 and max_length <= 8192 and tables.size(1) * k.size(1) >= max_length,
           "invalid context bound")


def paged_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, tables: torch.Tensor,
                    lengths: torch.Tensor, max_length: int, *, out: torch.Tensor | None = None,
                    impl: int = _lib.IMPL_AUTO) -> torch.Tensor:
    """Paged GQA decode attention (drop-in for the reference ``paged_attention``).

    q [B, H, D]; k, v [blocks, block_size, KVH, D]; tables int32 [B, W];
    lengths int32 [B]; returns softmax(q K^T / sqrt(D)) V as [B, H, D] in q's
    dtype (zeros for zero-length rows). Asynchronous on the current stream.
    """
    _check_attention_inputs(q, k, v, tables, lengths, max_length)
    lib = _lib.load()
    if out is None:
        out = torch.empty_like(q)
    else:
        _check(out.shape == q.shape and out.dtype == q.dtype and out.is_contiguous()
               and out.device == q.device, "invalid output tensor")
    B, H, D = q.shape
    N, bs, KVH, Dk = k.shape
    dt = _DTYPES[q.dtype]
    with _DeviceGuard(q.device):
        stream = _stream_ptr(q.device)
        need = lib.pdb_paged_attention_workspace_size(B, H, KVH, D, int(max_length), dt)
        ws = workspace(q.device, stream, need, "attention")
        rc = lib.pdb_paged_attention_impl(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), tables.data_ptr(), lengths.data_ptr(),
            out.data_ptr(), B, H, D, N, bs, KVH, Dk, tables.size(1), int(max_length), dt,
            ws.data_ptr() if ws is not None else None, ws.numel() if ws is not None else 0,
            stream, int(impl))
    _lib.check(rc, "paged_attention")
    return out


def rope_kv_write(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, k_pool: torch.Tensor,
                  v_pool: torch.Tensor, physical: torch.Tensor, offsets: torch.Tensor,
                  positions: torch.Tensor, inv_freq: torch.Tensor,
                  valid: torch.Tensor | None = None, *, inplace: bool = False,
                  q_out: torch.Tensor | None = None, k_out: torch.Tensor | None = None):
    """RoPE on q and k, then k and v written to their paged KV slots.

    Shapes follow worker/llama.py: q [B, S, H, D], k and v [B, S, KVH, D]
    (S = 1 in decode; [B, H, D] is accepted as S = 1), positions int64
    broadcastable to [B, S], inv_freq fp32 [D/2], pools [blocks, bs, KVH, D].
    Slots: without ``valid`` row (b, s) writes slot b*S + s (decode,
    ``pool[physical, offsets] = k[:, 0]``); with ``valid`` (bool [B, S]) the
    j-th valid row in row-major order writes slot j (prefill,
    ``pool[slots] = k[valid]``). Returns the rotated (q, k): new tensors, or
    q/k themselves with ``inplace``, or the given ``q_out``/``k_out``.
    """
    _check(q.is_cuda, "query must be on CUDA")
    squeeze = q.dim() == 3
    if squeeze:
        q, k, v = q.unsqueeze(1), k.unsqueeze(1), v.unsqueeze(1)
    _check(q.dim() == 4 and k.dim() == 4 and k.shape == v.shape, "invalid Q/K/V shapes")
    _check(k_pool.dim() == 4 and k_pool.shape == v_pool.shape, "invalid cache shape")
    B, S, H, D = q.shape
    _check(k.size(0) == B and k.size(1) == S and k.size(3) == D, "invalid Q/K/V shapes")
    KVH = k.size(2)
    _check(k_pool.size(2) == KVH and k_pool.size(3) == D, "invalid cache shape")
    _check(q.dtype in _DTYPES, "use FP32 or FP16")
    for t in (k, v, k_pool, v_pool):
        _check(t.dtype == q.dtype, "dtype mismatch")
    for t in (q, k, v, k_pool, v_pool, physical, offsets, positions, inv_freq):
        _check(t.device == q.device, "all tensors must be on the same GPU")
    for t in (q, k, v, k_pool, v_pool, physical, offsets, inv_freq):
        _check(t.is_contiguous(), "all tensors must be contiguous")
    _check(physical.dtype == torch.int64 and offsets.dtype == torch.int64
           and positions.dtype == torch.int64, "slots and positions must be int64")
    _check(physical.dim() == 1 and physical.shape == offsets.shape, "invalid slots")
    _check(inv_freq.dtype == torch.float32 and inv_freq.numel() == D // 2, "invalid inv_freq")
    pos = positions
    if pos.dim() == 1:
        pos = pos.unsqueeze(1)
    _check(pos.dim() == 2 and pos.size(0) in (1, B) and pos.size(1) in (1, S),
           "positions must broadcast to [batch, seq]")
    sb = pos.stride(0) if pos.size(0) > 1 else 0
    ss = pos.stride(1) if pos.size(1) > 1 else 0
    if valid is not None:
        _check(valid.dtype == torch.bool and valid.shape == (B, S) and valid.is_contiguous()
               and valid.device == q.device, "valid must be a contiguous bool [batch, seq] mask")
    lib = _lib.load()
    if q_out is not None or k_out is not None:
        _check(q_out is not None and k_out is not None, "give both q_out and k_out")
        q_out = q_out.view(q.shape) if squeeze else q_out
        k_out = k_out.view(k.shape) if squeeze else k_out
        _check(q_out.shape == q.shape and k_out.shape == k.shape and q_out.dtype == q.dtype
               and k_out.dtype == q.dtype and q_out.is_contiguous() and k_out.is_contiguous()
               and q_out.device == q.device and k_out.device == q.device, "invalid outputs")
    else:
        q_out = q if inplace else torch.empty_like(q)
        k_out = k if inplace else torch.empty_like(k)
    with _DeviceGuard(q.device):
        stream = _stream_ptr(q.device)
        need = lib.pdb_rope_kv_write_workspace_size(B, S, 1 if valid is not None else 0)
        ws = workspace(q.device, stream, need, "rope")
        rc = lib.pdb_rope_kv_write(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), q_out.data_ptr(), k_out.data_ptr(),
            k_pool.data_ptr(), v_pool.data_ptr(), pos.data_ptr(), sb, ss, inv_freq.data_ptr(),
            physical.data_ptr(), offsets.data_ptr(), physical.numel(),
            valid.data_ptr() if valid is not None else None, B, S, H, KVH, D,
            k_pool.size(0), k_pool.size(1), _DTYPES[q.dtype],
            ws.data_ptr() if ws is not None else None, ws.numel() if ws is not None else 0,
            stream)
    _lib.check(rc, "rope_kv_write")
    if squeeze:
        return q_out.squeeze(1), k_out.squeeze(1)
    return q_out, k_out


def rope_kv_write_decode(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                         k_pool: torch.Tensor, v_pool: torch.Tensor, tables: torch.Tensor,
                         lengths: torch.Tensor, inv_freq: torch.Tensor, *,
                         advance: bool = False, inplace: bool = False,
                         q_out: torch.Tensor | None = None, k_out: torch.Tensor | None = None):
    """Decode prologue driven by device-resident metadata.

    The RoPE + KV-slot write of ``rope_kv_write`` for one new token per
    sequence, with each token's position and slot derived on the GPU from the
    batch's int32 block ``tables`` [B, W] and int32 ``lengths`` [B] instead of
    host-computed positions and slots (TensorPagedKV.slots/metadata and the
    bookkeeping of PagedLlama.decode, worker/llama.py:40-55, :154-159). With
    ``advance`` the position is ``lengths[b]`` and ``lengths`` is incremented
    in place (the first layer of a step); otherwise the position is
    ``lengths[b] - 1``. q [B, H, D] or [B, 1, H, D]; k, v [B, KVH, D] or
    [B, 1, KVH, D]. Returns the rotated (q, k) as ``rope_kv_write`` does.
    """
    _check(q.is_cuda, "query must be on CUDA")
    squeeze = q.dim() == 3
    if not squeeze:
        _check(q.dim() == 4 and q.size(1) == 1 and k.dim() == 4 and k.size(1) == 1,
               "decode takes one token per sequence")
        q, k, v = q.squeeze(1), k.squeeze(1), v.squeeze(1)
    _check(q.dim() == 3 and k.dim() == 3 and k.shape == v.shape, "invalid Q/K/V shapes")
    _check(k_pool.dim() == 4 and k_pool.shape == v_pool.shape, "invalid cache shape")
    B, H, D = q.shape
    KVH = k.size(1)
    _check(k.size(0) == B and k.size(2) == D, "invalid Q/K/V shapes")
    _check(k_pool.size(2) == KVH and k_pool.size(3) == D, "invalid cache shape")
    _check(q.dtype in _DTYPES, "use FP32 or FP16")
    for t in (k, v, k_pool, v_pool):
        _check(t.dtype == q.dtype, "dtype mismatch")
    for t in (q, k, v, k_pool, v_pool, tables, lengths, inv_freq):
        _check(t.device == q.device, "all tensors must be on the same GPU")
        _check(t.is_contiguous(), "all tensors must be contiguous")
    _check(tables.dtype == torch.int32 and lengths.dtype == torch.int32,
           "tables and lengths must be int32")
    _check(tables.dim() == 2 and tables.size(0) == B and tables.size(1) > 0,
           "tables must be [batch, width]")
    _check(lengths.dim() == 1 and lengths.size(0) == B, "lengths must be [batch]")
    _check(inv_freq.dtype == torch.float32 and inv_freq.numel() == D // 2, "invalid inv_freq")
    lib = _lib.load()
    if q_out is not None or k_out is not None:
        _check(q_out is not None and k_out is not None, "give both q_out and k_out")
        q_out, k_out = q_out.view(q.shape), k_out.view(k.shape)
        _check(q_out.dtype == q.dtype and k_out.dtype == q.dtype and q_out.is_contiguous()
               and k_out.is_contiguous() and q_out.device == q.device
               and k_out.device == q.device, "invalid outputs")
    else:
        q_out = q if inplace else torch.empty_like(q)
        k_out = k if inplace else torch.empty_like(k)
    with _DeviceGuard(q.device):
        rc = lib.pdb_rope_kv_write_decode(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), q_out.data_ptr(), k_out.data_ptr(),
            k_pool.data_ptr(), v_pool.data_ptr(), tables.data_ptr(), tables.size(1),
            lengths.data_ptr(), 1 if advance else 0, inv_freq.data_ptr(), B, H, KVH, D,
            k_pool.size(0), k_pool.size(1), _DTYPES[q.dtype], _stream_ptr(q.device))
    _lib.check(rc, "rope_kv_write_decode")
    return q_out, k_out


def decode_attention_supported(q: torch.Tensor, k_pool: torch.Tensor) -> bool:
    """Whether ``decode_attention`` covers this shape (FP16 or FP32, head_dim
    64/128, group <= 8 (FP32 head_dim 128: <= 4), block_size a multiple of
    16) on the current device."""
    if q.dim() != 3 or k_pool.dim() != 4 or q.dtype not in (torch.float16, torch.float32):
        return False
    B, H, D = q.shape  # q may be a meta tensor: only its shape and dtype are read
    N, bs, KVH, _ = k_pool.shape
    with _DeviceGuard(k_pool.device):
        return bool(_lib.load().pdb_decode_attention_supported(B, H, KVH, D, N, bs,
                                                               _DTYPES[q.dtype]))


def decode_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, k_pool: torch.Tensor,
                     v_pool: torch.Tensor, tables: torch.Tensor, lengths: torch.Tensor,
                     inv_freq: torch.Tensor, max_length: int, *,
                     out: torch.Tensor | None = None,
                     metadata_stable: bool = False,
                     pools_stable: bool = False) -> torch.Tensor:
    """One decode layer in one launch (worker/llama.py:168-174).

    ``rope_kv_write_decode(..., advance=False)`` followed by
    ``paged_attention``, fused: q [B, H, D] and the new token's k, v
    [B, KVH, D] un-rotated (none of them is modified; each may be a row
    slice of one fused q/k/v projection output), lengths already
    counting the new token (its position is lengths[b] - 1). The rotated k
    and v are written to the token's slot; returns the attention output
    [B, H, D], bit-identical to the two-launch path. FP16 and FP32 (see
    ``decode_attention_supported``; FP32 rows must be 16-byte aligned).

    ``metadata_stable=True`` promises that tables, lengths and inv_freq were
    not written by the previous kernel on the stream (every layer after the
    first of a decode step): the launch then plans its work and looks up
    pages while that kernel is still finishing. ``pools_stable=True``
    (requires ``metadata_stable``) adds that k_pool and v_pool were not
    written by it either — true when every layer of the step is one
    decode_attention launch — and lets the first K/V tiles load early too.
    Results are identical.
    """
    _check(metadata_stable or not pools_stable, "pools_stable requires metadata_stable")
    # q, k and v may be row slices of one fused projection output: heads packed
    # within a sequence (strides (row, D, 1)), any row stride between sequences
    _check(q.is_cuda and q.dim() == 3 and q.stride(2) == 1 and q.stride(1) == q.size(2)
           and q.stride(0) >= q.size(1) * q.size(2), "query heads must be packed in each row")
    qc = q if q.is_contiguous() else q.as_strided(q.shape, (q.size(1) * q.size(2), q.size(2), 1))
    _check_attention_inputs(qc, k_pool, v_pool, tables, lengths, max_length)
    B, H, D = q.shape
    N, bs, KVH, _ = k_pool.shape
    for t in (k, v):
        _check(t.shape == (B, KVH, D) and t.dtype == q.dtype and t.device == q.device
               and t.stride(2) == 1 and t.stride(1) == D and t.stride(0) >= KVH * D,
               "invalid new k/v")
    _check(k.stride(0) == v.stride(0), "k and v rows must have the same stride")
    _check(inv_freq.dtype == torch.float32 and inv_freq.numel() == D // 2
           and inv_freq.device == q.device and inv_freq.is_contiguous(), "invalid inv_freq")
    if out is None:
        out = torch.empty_like(q)
    else:
        _check(out.shape == q.shape and out.dtype == q.dtype and out.is_contiguous()
               and out.device == q.device, "invalid output tensor")
    lib = _lib.load()
    dt = _DTYPES[q.dtype]
    with _DeviceGuard(q.device):
        stream = _stream_ptr(q.device)
        need = lib.pdb_paged_attention_workspace_size(B, H, KVH, D, int(max_length), dt)
        ws = workspace(q.device, stream, need, "attention")
        rc = lib.pdb_decode_attention_ex(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), k_pool.data_ptr(), v_pool.data_ptr(),
            tables.data_ptr(), lengths.data_ptr(), inv_freq.data_ptr(), out.data_ptr(), B, H, D,
            N, bs, KVH, tables.size(1), int(max_length), q.stride(0), k.stride(0), dt,
            ws.data_ptr() if ws is not None else None, ws.numel() if ws is not None else 0,
            stream, (_lib.DECODE_STABLE_METADATA if metadata_stable else 0)
            | (_lib.DECODE_STABLE_POOLS if pools_stable else 0))
    _lib.check(rc, "decode_attention")
    return out


def prefill_attention(q: torch.Tensor, k_pool: torch.Tensor, v_pool: torch.Tensor,
                      tables: torch.Tensor, lengths: torch.Tensor, *,
                      out: torch.Tensor | None = None,
                      impl: int = _lib.PREFILL_AUTO) -> torch.Tensor:
    """Causal attention of a left-aligned prompt batch, K/V from the paged pools.

    The prefill attention of worker/llama.py:141-144 (causal SDPA over the
    padded batch with K/V repeated per query group) without the padding or
    the repeat: q [B, W, H, D] FP16 (head_dim 64 or 128), pools
    [blocks, bs, KVH, D] holding every prompt token's k/v (as rope_kv_write
    leaves them), tables int32 [B, pages], lengths int32 [B]. Returns
    [B, W, H, D]; rows at or beyond a prompt's length are zero. `impl` pins
    the kernel (PREFILL_TCGEN05: tcgen05.mma with TMEM accumulators, needs
    block_size % 16 == 0; PREFILL_MMA: mma.sync, any block size); the default
    takes the tcgen05 kernel whenever the block size allows.
    """
    _check(q.is_cuda, "query must be on CUDA")
    for t in (q, k_pool, v_pool, tables, lengths):
        _check(t.device == q.device, "all tensors must be on the same GPU")
        _check(t.is_contiguous(), "all tensors must be contiguous")
    _check(q.dim() == 4 and k_pool.dim() == 4 and k_pool.shape == v_pool.shape,
           "invalid Q/K/V shapes")
    B, Wd, H, D = q.shape
    N, bs, KVH, Dk = k_pool.shape
    _check(q.dtype == torch.float16 and k_pool.dtype == q.dtype and v_pool.dtype == q.dtype,
           "prefill attention takes FP16")
    _check(Dk == D and D in (64, 128), "prefill attention supports head_dim 64 and 128")
    _check(H % KVH == 0, "query heads must be a multiple of KV heads")
    _check(tables.dtype == torch.int32 and lengths.dtype == torch.int32, "metadata must be int32")
    _check(tables.dim() == 2 and tables.size(0) == B, "invalid block tables")
    _check(lengths.dim() == 1 and lengths.size(0) == B, "invalid lengths")
    if out is None:
        out = torch.empty_like(q)
    else:
        _check(out.shape == q.shape and out.dtype == q.dtype and out.is_contiguous()
               and out.device == q.device, "invalid output tensor")
    lib = _lib.load()
    with _DeviceGuard(q.device):
        rc = lib.pdb_prefill_attention_impl(
            q.data_ptr(), k_pool.data_ptr(), v_pool.data_ptr(), tables.data_ptr(),
            lengths.data_ptr(), out.data_ptr(), B, Wd, H, D, N, bs, KVH, tables.size(1),
            _lib.DTYPE_FLOAT16, _stream_ptr(q.device), int(impl))
    _lib.check(rc, "prefill_attention")
    return out


def read_device_errors(clear: bool = True) -> int:
    """Error bits raised by kernels on the current device (synchronises)."""
    import ctypes
    flags = ctypes.c_uint32(0)
    _lib.check(_lib.load().pdb_read_device_errors(ctypes.byref(flags), int(clear)),
               "read_device_errors")
    return int(flags.value)


def fast_grid_size(batch: int, heads: int, kv_heads: int, head_dim: int,
                   dtype: torch.dtype) -> int:
    """CTAs per launch of the fast kernel on the current device (0 = generic path)."""
    return int(_lib.load().pdb_fast_grid_size(batch, heads, kv_heads, head_dim, _DTYPES[dtype]))
