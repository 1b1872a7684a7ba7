/*
 * paged_decode_b200.h — C ABI of the sm_100a paged-decode library
 * (libpaged_decode_b200.so).
 *
 * The library replaces the decode hot path of
 * sri123vk/distributed-llm-inference:
 *   - the `paged_attention` torch extension op (cuda/binding.cpp:6-30,
 *     kernel cuda/paged_attention.cu:10-74), and
 *   - the per-token RoPE + paged KV-slot write that worker/llama.py performs
 *     in PyTorch (worker/llama.py:105-117 RoPE, :171-172 decode slot write,
 *     :138-140 prefill slot write).
 *
 * Conventions shared by every entry point:
 *   - Plain device pointers and sizes; no framework types. Tensors are dense,
 *     row-major ("contiguous") with the shapes given per argument.
 *   - `dtype` is a pdb_dtype_t. q, k, v, pools and outputs share it.
 *   - `stream` is a cudaStream_t (NULL = legacy default stream). All work is
 *     enqueued asynchronously on it; no entry point synchronises.
 *   - Return value is a pdb_status_t. On failure pdb_last_error() returns a
 *     message (thread-local) and nothing was enqueued. The argument checks and
 *     their messages are those of cuda/binding.cpp:8-22.
 *   - Inputs are borrowed; outputs and pools are written in place.
 *   - Device-side validation (table entries, lengths, slots) never faults: a
 *     bad entry is skipped and a bit is set in a per-device error word that
 *     pdb_read_device_errors() returns.
 */
#ifndef PAGED_DECODE_B200_H
#define PAGED_DECODE_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define PDB_API __attribute__((visibility("default")))
#else
#define PDB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  PDB_DTYPE_FLOAT32 = 0,
  PDB_DTYPE_FLOAT16 = 1
} pdb_dtype_t;

typedef enum {
  PDB_OK = 0,
  PDB_ERR_INVALID_ARGUMENT = 1, /* reference: TORCH_CHECK failure          */
  PDB_ERR_WORKSPACE = 2,        /* workspace missing, too small or misaligned */
  PDB_ERR_CUDA = 3              /* reference: C10_CUDA_KERNEL_LAUNCH_CHECK  */
} pdb_status_t;

/* Kernel selection for pdb_paged_attention_impl. */
typedef enum {
  PDB_IMPL_AUTO = 0,    /* stream-K kernel when the shape allows, else generic  */
  PDB_IMPL_FAST = 1,    /* stream-K, GQA-shared tiles: FP16 head_dim 64/128 on
                           tensor cores (TMA-fed with a dynamically claimed
                           tail when block_size % 16 == 0), SIMT otherwise     */
  PDB_IMPL_GENERIC = 2, /* any head_dim <= 256 / any alignment, split + combine */
  PDB_IMPL_SIMT = 3,    /* stream-K with the SIMT inner loop only               */
  PDB_IMPL_MMA = 4,     /* stream-K, tensor cores fed by cp.async (no TMA)      */
  PDB_IMPL_TMA_STATIC = 5 /* TMA-fed tensor cores, static schedule only       */
} pdb_impl_t;

/* Kernel selection for pdb_prefill_attention_impl. */
typedef enum {
  PDB_PREFILL_AUTO = 0,    /* tcgen05 kernel when block_size % 16 == 0, else mma.sync */
  PDB_PREFILL_TCGEN05 = 1, /* TMA-staged tiles, tcgen05.mma with TMEM accumulators   */
  PDB_PREFILL_MMA = 2      /* cp.async-staged tiles, mma.sync, any block size        */
} pdb_prefill_impl_t;

/* Bits of the per-device error word (pdb_read_device_errors). */
#define PDB_DEVERR_TABLE_ENTRY 0x1u  /* block-table entry outside [0, num_blocks) */
#define PDB_DEVERR_LENGTH 0x2u       /* length < 0 or > table_width*block_size   */
#define PDB_DEVERR_SLOT 0x4u         /* KV slot outside the pool                  */
#define PDB_DEVERR_VALID_COUNT 0x8u  /* valid-row count != number of slots        */
#define PDB_DEVERR_TIMEOUT 0x10u     /* a bounded wait on a shared-memory barrier
                                        expired (never expected; see kernel notes) */
#define PDB_DEVERR_ARRIVAL 0x20u     /* a piece could not register its arrival
                                        (never expected)                          */

/* Thread-local message of the last failed call ("" if none). */
PDB_API const char* pdb_last_error(void);

/* Library version string. */
PDB_API const char* pdb_version(void);

/*
 * Bytes of device workspace that pdb_paged_attention needs for this shape on
 * the current device (0 is a valid answer). It must be 256-byte aligned; its
 * contents do not matter (each call clears what it needs), so allocate it once
 * and reuse it. Calls that overlap on the GPU must not share one.
 */
PDB_API size_t pdb_paged_attention_workspace_size(int64_t batch, int64_t heads,
                                          int64_t kv_heads, int64_t head_dim,
                                          int64_t max_length, int dtype);

/*
 * Paged GQA decode attention.
 * Replaces: paged_attention(q, k, v, tables, lengths, max_length)
 *           cuda/binding.cpp:6-26 and cuda/paged_attention.cu:60-74.
 *   q       [batch, heads, head_dim]
 *   k_pool  [num_blocks, block_size, kv_heads, kv_head_dim]   (v_pool same)
 *   tables  int32 [batch, table_width]   physical block of page i of seq b
 *   lengths int32 [batch]                tokens to attend per sequence
 *   out     [batch, heads, head_dim]     softmax(q K^T / sqrt(head_dim)) V,
 *                                        0 for a zero-length sequence
 * Checks (messages of cuda/binding.cpp:12-22): batch, heads, head_dim > 0,
 * head_dim <= 256; num_blocks, block_size, kv_heads > 0 and
 * kv_head_dim == head_dim; heads % kv_heads == 0; dtype FP32/FP16;
 * 0 < max_length <= 8192 and table_width*block_size >= max_length.
 * The caller guarantees 0 <= lengths[b] <= max_length (cuda/binding.cpp:23-24).
 */
PDB_API int pdb_paged_attention(const void* q, const void* k_pool, const void* v_pool,
                        const int32_t* tables, const int32_t* lengths, void* out,
                        int64_t batch, int64_t heads, int64_t head_dim,
                        int64_t num_blocks, int64_t block_size, int64_t kv_heads,
                        int64_t kv_head_dim, int64_t table_width,
                        int64_t max_length, int dtype, void* workspace,
                        size_t workspace_bytes, void* stream);

/* Same as pdb_paged_attention with an explicit kernel choice (pdb_impl_t).
 * No reference counterpart: used by tests to pin each kernel separately. */
PDB_API int pdb_paged_attention_impl(const void* q, const void* k_pool,
                             const void* v_pool, const int32_t* tables,
                             const int32_t* lengths, void* out, int64_t batch,
                             int64_t heads, int64_t head_dim, int64_t num_blocks,
                             int64_t block_size, int64_t kv_heads,
                             int64_t kv_head_dim, int64_t table_width,
                             int64_t max_length, int dtype, void* workspace,
                             size_t workspace_bytes, void* stream, int impl);

/*
 * Paged GQA decode attention that allocates nothing and takes no workspace.
 * No counterpart in the reference (its extension allocates through PyTorch).
 * For callers that cannot allocate device memory or hand the library a
 * buffer: a plugin hosted by an engine that owns the whole device-memory
 * budget and gives plugins no allocator, or a loop that must not call
 * cudaMalloc/cudaFree (cudaFree synchronises the device). Same arguments,
 * checks and result as pdb_paged_attention, minus the workspace.
 *   - Scratch is a fixed 2 MiB array inside the library on each GPU that
 *     loads it (held until the process exits). Shapes whose scratch would
 *     exceed it, or that only the generic kernel handles, are rejected with
 *     PDB_ERR_WORKSPACE / PDB_ERR_INVALID_ARGUMENT and a message; for the
 *     Llama-3-8B shape at batch 256 the need is about 1.3 MB.
 *   - The first call on a device looks up that device's copy of the array
 *     (the device must be current); make that first call before any stream
 *     capture on the device. The address is kept for the life of the
 *     process: after cudaDeviceReset (or anything else that destroys the
 *     device's primary context) this entry point must not be called again
 *     in that process.
 *   - Every call on a device shares the one array: calls whose kernels can
 *     overlap on the GPU (different streams without ordering) race and give
 *     wrong results. Each call clears the part that must start at zero.
 *   - Allocates nothing: no cudaMalloc, cudaFree or allocating library call.
 */
PDB_API int pdb_paged_attention_noalloc(const void* q, const void* k_pool,
                                        const void* v_pool, const int32_t* tables,
                                        const int32_t* lengths, void* out,
                                        int64_t batch, int64_t heads, int64_t head_dim,
                                        int64_t num_blocks, int64_t block_size,
                                        int64_t kv_heads, int64_t kv_head_dim,
                                        int64_t table_width, int64_t max_length,
                                        int dtype, void* stream);

/*
 * Fused RoPE + paged KV-slot write (the prologue of one attention layer).
 * Replaces: PagedLlama.rope (worker/llama.py:108-117) followed by
 *           keys[layer][slots] = k ; values[layer][slots] = v
 *           (decode worker/llama.py:170-172, prefill :138-140).
 *   q, q_out   [rows, heads, head_dim]      (q_out may alias q)
 *   k, k_out   [rows, kv_heads, head_dim]   (k_out may alias k)
 *   v          [rows, kv_heads, head_dim]
 *   rows = batch * seq; row r is (r / seq, r % seq).
 *   positions  int64, position of row r = positions[(r/seq)*pos_stride_b +
 *              (r%seq)*pos_stride_s] (strides in elements; 0 broadcasts).
 *   inv_freq   fp32 [head_dim/2]   (worker/llama.py:105-106, computed by the
 *              caller so that both sides use identical frequencies)
 *   physical, offsets  int64 [num_slots]  slot j = (block, offset in block)
 *   valid      uint8 [rows] or NULL. NULL: row r writes slot r (decode,
 *              num_slots == rows). Otherwise the j-th valid row in row-major
 *              order writes slot j (the `pool[slots] = k[valid]` of prefill).
 *   k_pool, v_pool [num_blocks, block_size, kv_heads, head_dim]
 * Rounding follows the reference op by op: angles fp32, cos/sin rounded to
 * dtype, then x*cos and rotate(x)*sin each rounded to dtype, then their sum.
 */
PDB_API int pdb_rope_kv_write(const void* q, const void* k, const void* v, void* q_out,
                      void* k_out, void* k_pool, void* v_pool,
                      const int64_t* positions, int64_t pos_stride_b,
                      int64_t pos_stride_s, const float* inv_freq,
                      const int64_t* physical, const int64_t* offsets,
                      int64_t num_slots, const uint8_t* valid, int64_t batch,
                      int64_t seq, int64_t heads, int64_t kv_heads,
                      int64_t head_dim, int64_t num_blocks, int64_t block_size,
                      int dtype, void* workspace, size_t workspace_bytes,
                      void* stream);

/* Workspace bytes pdb_rope_kv_write needs (0 when valid is NULL). */
PDB_API size_t pdb_rope_kv_write_workspace_size(int64_t batch, int64_t seq,
                                        int has_valid);

/*
 * Decode prologue with the batch's metadata resident on the device: the
 * RoPE + KV-slot write of pdb_rope_kv_write for one new token per sequence,
 * its positions and slots derived on the device instead of computed on the
 * host and copied in every step.
 * Replaces: the host slot and position computation of a decode step
 *           (TensorPagedKV.slots / .metadata, worker/llama.py:40-55; the
 *           position, slot and length bookkeeping of PagedLlama.decode,
 *           worker/llama.py:154-159) together with its RoPE + slot writes
 *           (worker/llama.py:168-172).
 *   q, q_out [batch, heads, head_dim]; k, k_out, v [batch, kv_heads, head_dim]
 *   tables   int32 [batch, table_width], row b = sequence b's pages (padding
 *            beyond its pages is never read)
 *   lengths  int32 [batch], sequence b's cached tokens
 *   advance  nonzero: the new token's position is lengths[b] and the call
 *            sets lengths[b] += 1 (the first layer of a step, as
 *            PagedLlama.decode increments its lengths before attention);
 *            zero: the position is lengths[b] - 1 (later layers)
 * Sequence b's token goes to slot (tables[b][pos / block_size],
 * pos % block_size) of k_pool / v_pool. A length or position outside the
 * table, or a page outside the pool, skips the row's write and sets a
 * device error bit (pdb_read_device_errors). No workspace; capturable.
 */
PDB_API int pdb_rope_kv_write_decode(const void* q, const void* k, const void* v, void* q_out,
                                     void* k_out, void* k_pool, void* v_pool,
                                     const int32_t* tables, int64_t table_width,
                                     int32_t* lengths, int advance, const float* inv_freq,
                                     int64_t batch, int64_t heads, int64_t kv_heads,
                                     int64_t head_dim, int64_t num_blocks, int64_t block_size,
                                     int dtype, void* stream);

/*
 * Reads (and optionally clears) the error word of the current device.
 * Synchronises the device. No reference counterpart: the reference kernel
 * does not validate table entries or lengths on the device.
 */
PDB_API int pdb_read_device_errors(uint32_t* flags, int clear);

/*
 * Host-side copy of the fast kernel's work partition, for tests. No
 * reference counterpart. For each of `grid` CTAs writes into ranges[2*c] and
 * ranges[2*c+1] its [begin, end) in 16-token units over the sequence of
 * (sequence, kv_head) segments; returns the total unit count or -1.
 */
PDB_API int64_t pdb_debug_partition(const int32_t* lengths, int64_t batch,
                            int64_t kv_heads, int64_t grid, int64_t* ranges);

/*
 * One decode layer in one launch: the RoPE + KV-slot write of
 * pdb_rope_kv_write_decode (advance = 0) and the attention of
 * pdb_paged_attention, fused into the stream-K kernel (FP16: tensor-core inner
 * loop; FP32: fp32 SIMT inner loop, q / k_new / v_new rows 16-byte aligned).
 * Replaces: worker/llama.py:168-174 (rope, the two slot writes, attention)
 * for a decode step, given lengths that already count the new token.
 *   q            FP16 or FP32 [B, H, D], NOT rotated (the kernel rotates it at
 *                position lengths[b] - 1; q itself is not modified); sequence
 *                b's heads start at q + b * q_row_stride (elements; 0 = H * D,
 *                packed), e.g. a slice of a fused q/k/v projection's output
 *   k_new, v_new [B, KVH, D] of q's dtype, the new token's k (not rotated) and v,
 *                rows kv_row_stride elements apart (0 = KVH * D)
 *   k_pool, v_pool, tables, lengths, max_length, out, workspace: as for
 *                pdb_paged_attention; the new token's rotated k and its v
 *                are written to slot (tables[b][pos / bs], pos % bs),
 *                pos = lengths[b] - 1, exactly as pdb_rope_kv_write_decode
 *                writes them
 *   inv_freq     fp32 [D/2]
 * Results are bit-identical to pdb_rope_kv_write_decode followed by
 * pdb_paged_attention. Shapes the fused kernel does not cover return
 * PDB_ERR_INVALID_ARGUMENT (see pdb_decode_attention_supported); use the
 * two calls for them.
 */
PDB_API int pdb_decode_attention(const void* q, const void* k_new, const void* v_new,
                                 void* k_pool, void* v_pool, const int32_t* tables,
                                 const int32_t* lengths, const float* inv_freq, void* out,
                                 int64_t batch, int64_t heads, int64_t head_dim,
                                 int64_t num_blocks, int64_t block_size, int64_t kv_heads,
                                 int64_t table_width, int64_t max_length,
                                 int64_t q_row_stride, int64_t kv_row_stride, int dtype,
                                 void* workspace, size_t workspace_bytes, void* stream);

/* Flags of pdb_decode_attention_ex. */
#define PDB_DECODE_STABLE_METADATA 0x1u /* tables, lengths and inv_freq are not written by
                                           the previous kernel in the stream (every layer
                                           after the first of a decode step): the launch
                                           plans its work and looks up pages while that
                                           kernel finishes (programmatic dependent launch) */
#define PDB_DECODE_STABLE_POOLS 0x2u    /* with STABLE_METADATA: k_pool and v_pool are not
                                           written by the previous kernel either (every layer
                                           after the first of a step of one-launch layers,
                                           whose pools only their own launch writes): the
                                           first K/V tiles are loaded while it finishes too */

/* pdb_decode_attention with flags (0 = pdb_decode_attention). */
PDB_API int pdb_decode_attention_ex(const void* q, const void* k_new, const void* v_new,
                                    void* k_pool, void* v_pool, const int32_t* tables,
                                    const int32_t* lengths, const float* inv_freq, void* out,
                                    int64_t batch, int64_t heads, int64_t head_dim,
                                    int64_t num_blocks, int64_t block_size, int64_t kv_heads,
                                    int64_t table_width, int64_t max_length,
                                    int64_t q_row_stride, int64_t kv_row_stride, int dtype,
                                    void* workspace, size_t workspace_bytes, void* stream,
                                    unsigned flags);

/* 1 when pdb_decode_attention covers this shape on the current device, else 0. */
PDB_API int pdb_decode_attention_supported(int64_t batch, int64_t heads, int64_t kv_heads,
                                           int64_t head_dim, int64_t num_blocks,
                                           int64_t block_size, int dtype);

/*
 * Causal attention of a prefill batch, K/V read from the paged pools.
 * Replaces: the prefill attention of worker/llama.py:141-144,
 *   SDPA(q^T, repeat_interleave(k)^T, repeat_interleave(v)^T, is_causal=True)
 * over left-aligned padded prompts.
 *   q, out   FP16 [batch, width, heads, head_dim]   (head_dim 64 or 128)
 *   k_pool, v_pool FP16 [num_blocks, block_size, kv_heads, head_dim], holding
 *            every prompt token's (RoPE'd) k and v, as pdb_rope_kv_write leaves them
 *   tables   int32 [batch, table_width], prompt b's pages in order
 *   lengths  int32 [batch], prompt b's token count (<= width)
 * Query t < lengths[b] of prompt b attends to keys 0..t of prompt b; rows
 * t >= lengths[b] are written as zeros (no real row attends to them). Query
 * head h reads kv head h / (heads / kv_heads). Out-of-range lengths or pages
 * set device error bits (pdb_read_device_errors) and are clamped or skipped.
 * No workspace; capturable.
 */
PDB_API int pdb_prefill_attention(const void* q, const void* k_pool, const void* v_pool,
                                  const int32_t* tables, const int32_t* lengths, void* out,
                                  int64_t batch, int64_t width, int64_t heads, int64_t head_dim,
                                  int64_t num_blocks, int64_t block_size, int64_t kv_heads,
                                  int64_t table_width, int dtype, void* stream);

/* pdb_prefill_attention with the kernel pinned (pdb_prefill_impl_t); same
 * results within FP16 rounding. PDB_PREFILL_TCGEN05 needs block_size % 16 == 0
 * and num_blocks * block_size and batch * width under 2^31. */
PDB_API int pdb_prefill_attention_impl(const void* q, const void* k_pool, const void* v_pool,
                                       const int32_t* tables, const int32_t* lengths, void* out,
                                       int64_t batch, int64_t width, int64_t heads,
                                       int64_t head_dim, int64_t num_blocks, int64_t block_size,
                                       int64_t kv_heads, int64_t table_width, int dtype,
                                       void* stream, int impl);

/*
 * Host-side copy of the default FP16 kernel's worker partition, for tests.
 * No reference counterpart. For `units` 16-token units and `launched` CTAs,
 * writes per worker w: ranges[3w], ranges[3w+1] = its [begin, end) and
 * ranges[3w+2] = 0 (static range of CTA w) or 1 (dynamically claimed tail
 * chunk). Returns the number of static workers, or -1 (bad arguments or more
 * than max_workers workers).
 */
PDB_API int64_t pdb_debug_dyn_partition(int64_t units, int64_t launched, int64_t* ranges,
                                        int64_t max_workers);

/* CTAs the fast kernel launches per call on the current device for this
 * shape (0 when the fast kernel does not apply). No reference counterpart. */
PDB_API int64_t pdb_fast_grid_size(int64_t batch, int64_t heads, int64_t kv_heads,
                           int64_t head_dim, int dtype);

#ifdef __cplusplus
}
#endif

#endif /* PAGED_DECODE_B200_H */
