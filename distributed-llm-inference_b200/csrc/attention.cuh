// Paged GQA decode attention for sm_100a.
//
// Computes, for every sequence b and query head hq (kv head h = hq / G):
//   out[b, hq] = sum_t softmax_t(q[b,hq] . K[t] / sqrt(D)) * V[t],  t < len[b]
// where token t lives at pool[tables[b, t / bs], t % bs, h, :] and out is 0
// for len[b] == 0. This is the contract of attention_kernel in
// cuda/paged_attention.cu:10-58 and of torch_paged_attention in
// worker/llama.py:58-71.
//
// Kernels:
//  * attn_streamk_kernel<Math> — persistent stream-K decode, one launch per
//    call, with two inner loops ("Math" policies):
//      - MmaMath  (FP16, head_dim 64/128, group <= 8): tensor cores.
//        S^T = K Q^T with mma.sync.m16n8k16 (16 tokens x 8 query heads per
//        warp, fp32 accumulate), online softmax in fp32, P^T moved into the
//        B operand with movmatrix, O^T += V^T P^T with P split into two FP16
//        terms (hi + lo) so the weights keep ~22 bits. K/V tiles are staged by
//        cp.async into an XOR-swizzled layout that ldmatrix reads without
//        bank conflicts.
//      - SimtMath (FP32 and the remaining FP16 shapes): fp32 FMA; lanes split
//        a token row into 16-byte chunks, warp-shuffle reductions.
//    Shared by both:
//      - Work is flattened into 16-token units ordered by (sequence, kv head,
//        token). CTA c owns the contiguous unit range [c*U/grid, (c+1)*U/grid),
//        so every CTA streams the same number of K/V bytes whatever the
//        length distribution (no idle SMs at the tail of a lognormal batch).
//      - A CTA stages each K/V tile of one kv head into shared memory once
//        (cp.async, STAGES-deep ring) and all G query heads of the GQA group
//        read it there: K/V cross HBM exactly once.
//      - A (sequence, kv head) segment cut by a CTA boundary is a "piece":
//        its partial (m, l, o) goes to the workspace and the last CTA to
//        finish a piece of that segment (a tagged arrival counter, no
//        waiting) merges the pieces and writes the output.
//  * attn_generic_kernel + attn_combine_kernel — any head_dim <= 256, any
//    group size, any alignment: grid (splits, heads, batch), one query head
//    per CTA, plain loads, split partials merged by a second kernel.
#pragma once

#include <math.h>

#include "common.cuh"

namespace pdb {

struct AttnParams {
  const void* q;
  const void* k_pool;
  const void* v_pool;
  const int32_t* tables;
  const int32_t* lengths;
  void* out;
  int B, H, KVH, G, D;
  int64_t num_blocks;
  int block_size;
  int bs_shift;  // log2(block_size) if a power of two, else -1
  int table_width;
  int max_length;
  float scale_log2;  // log2(e) / sqrt(D)
  // workspace
  unsigned long long* counters;  // stream-K: [B*KVH] call tag << 16 | arrivals
  float* partials;               // stream-K: [2*grid][GP*(D+2)]; generic: [B*H*splits][D+2]
  unsigned long long call_tag;   // 48-bit salted tag of this call
  int splits;  // generic
  int chunk;   // generic: tokens per split
  // Decode prologue folded into attn_tma_dyn_kernel<M, true> (else unused):
  // q holds the un-rotated queries, rotated in the kernel at position
  // lengths[b] - 1; k_new / v_new [B, KVH, D] hold the new token's k (not yet
  // rotated) and v, which the kernel writes into the token's slot.
  const void* k_new;
  const void* v_new;
  const float* inv_freq;
  // Fused decode only: the caller guarantees that tables, lengths and
  // inv_freq (bit 0) and also the KV pools (bit 1) are not written by the
  // previous kernel in the stream (true for every layer after the first of a
  // fused decode step), so the launch may read them (plan, page lookups; K/V
  // tiles) before its programmatic-dependent-launch wait.
  int stable_meta;
  int64_t q_row;   // elements between consecutive sequences' q rows (H * D if packed)
  int64_t kv_row;  // fused: same for k_new / v_new (KVH * D if packed)
  // Dynamic TMA kernel: q (and, fused, k_new / v_new) rows and strides are
  // 16-byte aligned, so the producer warp may bulk-copy a piece's q rows and
  // new-token rows into shared memory along with its first tile.
  int bulk_q;
};

// Clamp a length read from device memory into [0, max_length].
__device__ __forceinline__ int checked_length(const int32_t* lengths, int b,
                                              int max_length) {
  int len = lengths[b];
  if (len < 0 || len > max_length) {
    raise_error(0x2u);
    len = len < 0 ? 0 : max_length;
  }
  return len;
}

// ---- tensor-core and shared-memory primitives --------------------------------
__device__ __forceinline__ void ldsm_x4(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3,
                                        const void* p) {
  const unsigned a = static_cast<unsigned>(__cvta_generic_to_shared(p));
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(a)
               : "memory");
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3,
                                          const void* p) {
  const unsigned a = static_cast<unsigned>(__cvta_generic_to_shared(p));
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(a)
               : "memory");
}
// D += A(16x16, row) * B(16x8, col), fp16 inputs, fp32 accumulators.
__device__ __forceinline__ void mma_16816(float* d, uint32_t a0, uint32_t a1, uint32_t a2,
                                          uint32_t a3, uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// Transpose an 8x8 fp16 matrix held as the standard m8n8 warp fragment.
__device__ __forceinline__ uint32_t movmatrix_t(uint32_t x) {
  uint32_t y;
  asm("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;\n" : "=r"(y) : "r"(x));
  return y;
}
__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

__device__ __forceinline__ unsigned long long cas_acq_rel(unsigned long long* p,
                                                          unsigned long long cmp,
                                                          unsigned long long val) {
  unsigned long long old;
  asm volatile("atom.acq_rel.gpu.global.cas.b64 %0, [%1], %2, %3;\n"
               : "=l"(old)
               : "l"(p), "l"(cmp), "l"(val)
               : "memory");
  return old;
}
__device__ __forceinline__ unsigned long long add_acq_rel(unsigned long long* p,
                                                          unsigned long long v) {
  unsigned long long old;
  asm volatile("atom.acq_rel.gpu.global.add.u64 %0, [%1], %2;\n"
               : "=l"(old)
               : "l"(p), "l"(v)
               : "memory");
  return old;
}
__device__ __forceinline__ void store_relaxed(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.gpu.global.b64 [%0], %1;\n" ::"l"(p), "l"(v) : "memory");
}

// Install this call's tag in a counter word of the form (tag << shift | count).
// A word carrying another tag (an earlier call, or the stale bytes of a fresh
// workspace) is replaced once by (tag << shift) with a compare-and-swap: the
// first thread to try wins and every other CAS fails by returning the
// installed word. Bounded: nothing else writes a stale word while a call runs.
__device__ __forceinline__ bool install_tag(unsigned long long* ctr, unsigned long long tag,
                                            int shift, int64_t bound) {
  const unsigned long long hi = tag << shift;
  unsigned long long cur = *reinterpret_cast<volatile unsigned long long*>(ctr);
  for (int64_t it = 0; (cur >> shift) != tag; ++it) {
    if (it > bound) {
      raise_error(0x20u);
      return false;
    }
    const unsigned long long prev = cas_acq_rel(ctr, cur, hi);
    cur = prev == cur ? hi : prev;
  }
  return true;
}

// Arrival of one piece on its segment's counter, a word (call tag << 16 |
// arrivals): the tag is installed if stale, then each piece adds one. Returns
// true for the arrival that completes `pieces`, which puts the count back to
// zero (tag kept), so a CUDA-graph replay of the same call — same tag — starts
// from zero; no other piece of the segment touches the word after it. acq_rel:
// the release orders this CTA's partial stores (made visible to this thread
// by the preceding barrier) before its arrival; the final arrival's acquire,
// through the chain of read-modify-writes, orders its reads of every other
// piece. One fetch-add per piece: the pieces of a segment that finish
// together do not serialise on a CAS loop.
__device__ __forceinline__ bool arrive_piece(unsigned long long* ctr, unsigned long long tag,
                                             unsigned pieces) {
  if (!install_tag(ctr, tag, 16, (int64_t)pieces + 64)) return false;
  const unsigned long long old = add_acq_rel(ctr, 1ull);
  const bool last = (unsigned)(old & 0xffffu) + 1u >= pieces;
  if (last) store_relaxed(ctr, tag << 16);
  return last;
}

// Arrival on a counter whose tag this thread installed earlier with
// install_tag (so no other tag can be in the word): one fetch-add, with the
// return value, reset and ordering of arrive_piece.
__device__ __forceinline__ bool arrive_installed(unsigned long long* ctr, unsigned long long tag,
                                                 unsigned pieces) {
  const unsigned long long old = add_acq_rel(ctr, 1ull);
  if ((old >> 16) != tag) {  // cannot happen after install_tag
    raise_error(0x20u);
    return false;
  }
  const bool last = (unsigned)(old & 0xffffu) + 1u >= pieces;
  if (last) store_relaxed(ctr, tag << 16);
  return last;
}

// Byte offset of 16-byte chunk `col` of token row `row` in a staged tile.
// SWZ: chunk positions are XOR-ed with (row & 7), so the 8 rows that one
// ldmatrix 8x8 load touches fall into 8 different bank groups.
template <int ROW_BYTES, bool SWZ>
__device__ __forceinline__ int tile_offset(int row, int col) {
  return row * ROW_BYTES + ((SWZ ? (col ^ (row & 7)) : col) << 4);
}

// ===========================================================================
// Work partition (identical in every CTA, recomputed from device lengths)
// ===========================================================================
struct Cursor {
  int b, h, nu;     // sequence, kv head, units per kv head of sequence b
  int64_t seg;      // first unit of segment (b, h)
  int64_t u;        // current unit
};

__device__ __forceinline__ void cursor_locate(Cursor& c, const int* P, int B,
                                              int KVH, int64_t u) {
  int lo = 0, hi = B - 1;  // largest b with P[b] <= u (then P[b+1] > u)
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (P[mid] <= u) lo = mid; else hi = mid - 1;
  }
  c.b = lo;
  c.nu = (P[lo + 1] - P[lo]) / KVH;
  const int64_t rel = u - P[lo];
  c.h = (int)(rel / c.nu);
  c.seg = P[lo] + (int64_t)c.h * c.nu;
  c.u = u;
}

template <int TILE_UNITS>
__device__ __forceinline__ int64_t cursor_tile_end(const Cursor& c, int64_t u_end) {
  int64_t e = c.u + TILE_UNITS;
  const int64_t s = c.seg + c.nu;
  e = e < s ? e : s;
  return e < u_end ? e : u_end;
}

__device__ __forceinline__ void cursor_advance(Cursor& c, int64_t te, int64_t u_end,
                                               const int* P, int KVH) {
  c.u = te;
  if (te == c.seg + c.nu && te < u_end) {
    if (++c.h == KVH) {
      c.h = 0;
      do { ++c.b; } while (P[c.b + 1] == P[c.b]);
      c.nu = (P[c.b + 1] - P[c.b]) / KVH;
      c.seg = P[c.b];
    } else {
      c.seg += c.nu;
    }
  }
}

// Valid tokens of the tile [c.u, te) of segment c.
__device__ __forceinline__ int tile_tokens(const Cursor& c, int64_t te, const int* Ls) {
  const int tok0 = (int)(c.u - c.seg) * kUnitTokens;
  const int rem = Ls[c.b] - tok0;
  const int span = (int)(te - c.u) * kUnitTokens;
  return span < rem ? span : rem;
}

// P[b] = KVH * sum_{b' < b} ceil(len_b' / 16) and the clamped lengths Ls.
// Returns the total unit count U. All threads of the CTA call it.
template <int NT>
__device__ int64_t plan_units(const AttnParams& p, int* P, int* Ls, int* misc) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) misc[0] = 0;
  __syncthreads();
  for (int base = 0; base < p.B; base += NT) {
    const int b = base + tid;
    int nu = 0;
    if (b < p.B) {
      const int len = checked_length(p.lengths, b, p.max_length);
      Ls[b] = len;
      nu = ((len + kUnitTokens - 1) / kUnitTokens) * p.KVH;
    }
    int incl = nu;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += t;
    }
    if (lane == 31) misc[4 + warp] = incl;
    __syncthreads();
    int woff = misc[0];
    for (int w = 0; w < warp; ++w) woff += misc[4 + w];
    if (b < p.B) P[b] = woff + incl - nu;
    __syncthreads();
    if (tid == NT - 1) misc[0] = woff + incl;
    __syncthreads();
  }
  if (tid == 0) P[p.B] = misc[0];
  __syncthreads();
  return P[p.B];
}

// Stage the K and V rows of tile [c.u, te) into shared memory (cp.async,
// zero-fill beyond the valid tokens). Table entries are range-checked before
// any address is formed; a bad entry raises PDB_DEVERR_TABLE_ENTRY and its
// rows are zero-filled.
template <typename T, int D, int TILE, int NT, bool SWZ>
__device__ __forceinline__ void load_tile(const AttnParams& p, const int* Ls, const Cursor& c,
                                          int64_t te, unsigned char* sk, unsigned char* sv) {
  constexpr int VEC = 16 / (int)sizeof(T), CH = D / VEC, ROW = D * (int)sizeof(T);
  static_assert(NT % CH == 0, "rows per pass");
  constexpr int RPP = NT / CH;  // rows per pass
  const T* kpool = static_cast<const T*>(p.k_pool);
  const T* vpool = static_cast<const T*>(p.v_pool);
  const int tok0 = (int)(c.u - c.seg) * kUnitTokens;
  const int ntok = tile_tokens(c, te, Ls);
  const int32_t* trow = p.tables + (int64_t)c.b * p.table_width;
  const int col = threadIdx.x % CH;
  int last_pi = -1, page = 0;
#pragma unroll
  for (int k = 0; k < TILE / RPP; ++k) {
    const int row = threadIdx.x / CH + k * RPP;
    bool ok = row < ntok;
    const T* ks = kpool;
    const T* vs = vpool;
    if (ok) {
      const int t = tok0 + row;
      int pi, off;
      if (p.bs_shift >= 0) {
        pi = t >> p.bs_shift;
        off = t & (p.block_size - 1);
      } else {
        pi = t / p.block_size;
        off = t - pi * p.block_size;
      }
      if (pi != last_pi) {
        page = __ldg(trow + pi);
        last_pi = pi;
      }
      if (page < 0 || (int64_t)page >= p.num_blocks) {
        raise_error(0x1u);
        ok = false;
      } else {
        const int64_t e = (((int64_t)page * p.block_size + off) * p.KVH + c.h) * D + col * VEC;
        ks = kpool + e;
        vs = vpool + e;
      }
    }
    const int o = tile_offset<ROW, SWZ>(row, col);
    cp_async16(sk + o, ks, ok);
    cp_async16(sv + o, vs, ok);
  }
}

// ===========================================================================
// Inner loop 1: tensor cores (FP16)
// ===========================================================================
// GQ: query heads of the group that are kept (4 or 8); the MMA N dimension
// always computes 8 columns, columns >= G see q = 0 and are never stored.
// Staged-tile layouts read by MmaMath:
//   kRowSwizzle  one D*2-byte row per token, 16-byte chunks XOR (row & 7)
//                (written by cp.async);
//   kTma128B     the tile split into D/64 column halves of 128-byte rows,
//                each [TILE rows x 128 B] with the TMA 128-byte swizzle
//                (chunk XOR (row & 7)); written by cp.async.bulk.tensor.
enum : int { kRowSwizzle = 0, kTma128B = 1 };

// SUB: 16-token blocks per warp per tile (TILE = 64 * SUB tokens). Two
// blocks per warp give the QK chains of one tile twice the independent work
// and share one max reduction and one rescale per tile, which pays where a
// 64-token tile carries few bytes (head_dim 64).
template <int D_, int GQ_, int STAGES_, int LAYOUT_ = kRowSwizzle, int SUB_ = 1>
struct MmaMath {
  using T = __half;
  static constexpr int D = D_, GP = GQ_, STAGES = STAGES_, LAYOUT = LAYOUT_, SUB = SUB_;
  static_assert(SUB_ == 1 || LAYOUT_ == kTma128B, "multi-block tiles are staged by TMA");
  static constexpr int NW = 4, NT = 128;
  static constexpr bool kSimt = false;   // tensor-core inner loop
  static constexpr int WT = 16 * SUB;    // tokens per warp per tile (SUB x MMA M)
  static constexpr int CHUNKS = D / 8;   // 16-byte chunks of a K/V row
  static constexpr int TILE = NW * WT;   // 64 * SUB tokens
  static constexpr int TILE_UNITS = TILE / kUnitTokens;
  static constexpr bool SWZ = true;
  static constexpr int KSTEPS = D / 16;  // QK k-steps == PV m-tiles
  static constexpr int ROW = D * 2;
  static constexpr int TILE_BYTES = TILE * ROW;
  static constexpr int STAGE_BYTES = 2 * TILE_BYTES;
  static constexpr int EXTRA_FLOATS = 0;
  static_assert(D % 64 == 0, "swizzle needs >= 8 chunks per row");
  static_assert(GQ_ == 4 || GQ_ == 8, "group");

  // Byte offset of 16-byte chunk `col` (0..D/8-1) of token row `row`.
  __device__ static __forceinline__ int offset(int row, int col) {
    if constexpr (LAYOUT == kTma128B) {
      return (col >> 3) * (TILE * 128) + row * 128 + (((col & 7) ^ (row & 7)) << 4);
    } else {
      return tile_offset<ROW, true>(row, col);
    }
  }

  struct State {
    uint32_t qb[KSTEPS][2];  // B fragments of Q^T (8 heads)
    float m[2], l[2];        // heads 2*tg, 2*tg+1
    float acc[KSTEPS][4];    // O^T fragments: dims x heads
  };

  __device__ static void begin_piece(State& s, const AttnParams& p, int b, int h) {
    const int lane = threadIdx.x & 31, g = lane >> 2, tg = lane & 3;
    const bool real = g < p.G;  // columns >= G are padding (q = 0)
    const __half* qrow = static_cast<const __half*>(p.q) +
                         ((int64_t)b * p.H + (int64_t)h * p.G + (real ? g : 0)) * D;
#pragma unroll
    for (int ks = 0; ks < KSTEPS; ++ks) {
      s.qb[ks][0] = real ? __ldg(reinterpret_cast<const unsigned*>(qrow + 16 * ks + 2 * tg)) : 0u;
      s.qb[ks][1] = real ? __ldg(reinterpret_cast<const unsigned*>(qrow + 16 * ks + 2 * tg + 8)) : 0u;
    }
    s.m[0] = s.m[1] = -INFINITY;
    s.l[0] = s.l[1] = 0.f;
#pragma unroll
    for (int i = 0; i < KSTEPS; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) s.acc[i][j] = 0.f;
  }

  // begin_piece with the group's G query rows (D halves each, consecutive)
  // at `qbase`, in global or shared memory.
  __device__ static void begin_piece_at(State& s, const __half* qbase, int G) {
    const int lane = threadIdx.x & 31, g = lane >> 2, tg = lane & 3;
    const bool real = g < G;  // columns >= G are padding (q = 0)
    const __half* qrow = qbase + (real ? g : 0) * D;
#pragma unroll
    for (int ks = 0; ks < KSTEPS; ++ks) {
      s.qb[ks][0] = real ? *reinterpret_cast<const unsigned*>(qrow + 16 * ks + 2 * tg) : 0u;
      s.qb[ks][1] = real ? *reinterpret_cast<const unsigned*>(qrow + 16 * ks + 2 * tg + 8) : 0u;
    }
    s.m[0] = s.m[1] = -INFINITY;
    s.l[0] = s.l[1] = 0.f;
#pragma unroll
    for (int i = 0; i < KSTEPS; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) s.acc[i][j] = 0.f;
  }

  __device__ static void compute_tile(State& s, const AttnParams& p, const unsigned char* sk,
                                      const unsigned char* sv, int ntok, float*) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r0 = warp * WT;
    if (r0 >= ntok) return;  // warp-uniform: no valid token in this warp's rows
    const int g = lane >> 2, mi = lane >> 3;

    // S^T[16 tokens x 8 heads] = K[16 x D] . Q^T[D x 8] per 16-token block;
    // two chains per block for ILP
    const float sc = p.scale_log2;
    float sA[SUB][2], sB[SUB][2];  // [block][token g, g+8]: heads 2tg, 2tg+1
#pragma unroll
    for (int sb = 0; sb < SUB; ++sb) {
      float c0[4] = {0.f, 0.f, 0.f, 0.f}, c1[4] = {0.f, 0.f, 0.f, 0.f};
      const int row = r0 + 16 * sb + ((mi & 1) << 3) + (lane & 7);
#pragma unroll
      for (int ks = 0; ks < KSTEPS; ++ks) {
        uint32_t a0, a1, a2, a3;
        ldsm_x4(a0, a1, a2, a3, sk + offset(row, 2 * ks + (mi >> 1)));
        mma_16816((ks & 1) ? c1 : c0, a0, a1, a2, a3, s.qb[ks][0], s.qb[ks][1]);
      }
      const int t = r0 + 16 * sb + g;
      const bool v0 = t < ntok, v1 = t + 8 < ntok;
      sA[sb][0] = v0 ? (c0[0] + c1[0]) * sc : -INFINITY;  // token g,   head 2tg
      sB[sb][0] = v0 ? (c0[1] + c1[1]) * sc : -INFINITY;  // token g,   head 2tg+1
      sA[sb][1] = v1 ? (c0[2] + c1[2]) * sc : -INFINITY;  // token g+8, head 2tg
      sB[sb][1] = v1 ? (c0[3] + c1[3]) * sc : -INFINITY;  // token g+8, head 2tg+1
    }

    float mA = -INFINITY, mB = -INFINITY;
#pragma unroll
    for (int sb = 0; sb < SUB; ++sb) {
      mA = fmaxf(mA, fmaxf(sA[sb][0], sA[sb][1]));
      mB = fmaxf(mB, fmaxf(sB[sb][0], sB[sb][1]));
    }
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
      mA = fmaxf(mA, __shfl_xor_sync(0xffffffffu, mA, o));
      mB = fmaxf(mB, __shfl_xor_sync(0xffffffffu, mB, o));
    }
    const float nA = fmaxf(s.m[0], mA), nB = fmaxf(s.m[1], mB);
    const bool grow = (nA > s.m[0]) || (nB > s.m[1]);
    if (__any_sync(0xffffffffu, grow)) {
      const float aA = (s.m[0] == -INFINITY) ? 0.f : exp2f(s.m[0] - nA);
      const float aB = (s.m[1] == -INFINITY) ? 0.f : exp2f(s.m[1] - nB);
      s.l[0] *= aA;
      s.l[1] *= aB;
#pragma unroll
      for (int i = 0; i < KSTEPS; ++i) {
        s.acc[i][0] *= aA; s.acc[i][1] *= aB;
        s.acc[i][2] *= aA; s.acc[i][3] *= aB;
      }
      s.m[0] = nA;
      s.m[1] = nB;
    }
    uint32_t bh0[SUB], bh1[SUB], bl0[SUB], bl1[SUB];
#pragma unroll
    for (int sb = 0; sb < SUB; ++sb) {
      const float pA0 = (sA[sb][0] == -INFINITY) ? 0.f : exp2f(sA[sb][0] - s.m[0]);
      const float pB0 = (sB[sb][0] == -INFINITY) ? 0.f : exp2f(sB[sb][0] - s.m[1]);
      const float pA1 = (sA[sb][1] == -INFINITY) ? 0.f : exp2f(sA[sb][1] - s.m[0]);
      const float pB1 = (sB[sb][1] == -INFINITY) ? 0.f : exp2f(sB[sb][1] - s.m[1]);
      s.l[0] += pA0 + pA1;
      s.l[1] += pB0 + pB1;
      // P^T as two FP16 B operands (hi + lo): the transposes of the C fragment.
      const uint32_t h0 = pack_half2(pA0, pB0), h1 = pack_half2(pA1, pB1);
      const float2 f0 = __half22float2(*reinterpret_cast<const __half2*>(&h0));
      const float2 f1 = __half22float2(*reinterpret_cast<const __half2*>(&h1));
      const uint32_t l0 = pack_half2(pA0 - f0.x, pB0 - f0.y),
                     l1 = pack_half2(pA1 - f1.x, pB1 - f1.y);
      bh0[sb] = movmatrix_t(h0);
      bh1[sb] = movmatrix_t(h1);
      bl0[sb] = movmatrix_t(l0);
      bl1[sb] = movmatrix_t(l1);
    }

    // O^T[D x 8] += V^T[D x 16 tokens] . P^T[16 x 8], block by block
    const int vrow = r0 + ((mi >> 1) << 3) + (lane & 7);
#pragma unroll
    for (int md = 0; md < KSTEPS; ++md) {
#pragma unroll
      for (int sb = 0; sb < SUB; ++sb) {
        uint32_t a0, a1, a2, a3;
        ldsm_x4_t(a0, a1, a2, a3, sv + offset(vrow + 16 * sb, 2 * md + (mi & 1)));
        mma_16816(s.acc[md], a0, a1, a2, a3, bh0[sb], bh1[sb]);
        mma_16816(s.acc[md], a0, a1, a2, a3, bl0[sb], bl1[sb]);
      }
    }
  }

  // Publish this warp's (m, l, O) for the heads < GQ into the merge area.
  __device__ static void store_state(State& s, float* ms, float* ls, float* accs) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, tg = lane & 3;
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
      s.l[0] += __shfl_xor_sync(0xffffffffu, s.l[0], o);
      s.l[1] += __shfl_xor_sync(0xffffffffu, s.l[1], o);
    }
    const int hA = 2 * tg, hB = 2 * tg + 1;
    if (hB < GP) {
      if (g == 0) {
        ms[warp * GP + hA] = s.m[0]; ms[warp * GP + hB] = s.m[1];
        ls[warp * GP + hA] = s.l[0]; ls[warp * GP + hB] = s.l[1];
      }
      float* oa = accs + (warp * GP + hA) * D;
      float* ob = accs + (warp * GP + hB) * D;
#pragma unroll
      for (int md = 0; md < KSTEPS; ++md) {
        oa[16 * md + g] = s.acc[md][0];
        ob[16 * md + g] = s.acc[md][1];
        oa[16 * md + g + 8] = s.acc[md][2];
        ob[16 * md + g + 8] = s.acc[md][3];
      }
    }
  }
};

// ===========================================================================
// Inner loop 2: SIMT fp32 FMA (FP32, and FP16 shapes outside MmaMath)
// ===========================================================================
template <typename T_, int D_, int GP_, int TPG_, int STAGES_, int LAYOUT_ = kRowSwizzle>
struct SimtMath {
  using T = T_;
  static constexpr int D = D_;
  // kRowSwizzle here: plain row-major stage tiles (cp.async); kTma128B: the
  // stage layout of the TMA kernels (128-byte column blocks, chunks XORed with
  // the row).
  static constexpr int LAYOUT = LAYOUT_;
  static constexpr int GP = GP_;          // group size padded to a power of 2
  static constexpr int TPG = TPG_;        // tokens per lane group per tile
  static constexpr int STAGES = STAGES_;  // cp.async ring depth
  static constexpr int E = sizeof(T);
  static constexpr int VEC = 16 / E;  // elements per 16-byte chunk
  static constexpr int CH = D / VEC;  // chunks per token row
  static constexpr int LPT = CH < 8 ? CH : 8;  // lanes per token (QK)
  static constexpr int CPL = CH / LPT;         // chunks per lane (QK)
  static constexpr int DL = CPL * VEC;         // dims per lane (QK)
  static constexpr int TPW = 32 / LPT;         // lane groups per warp
  static constexpr int NW = 4, NT = 128;
  static constexpr bool kSimt = true;       // fp32 FMA inner loop
  static constexpr int TW = TPW * TPG;      // tokens per warp per tile
  static constexpr int WT = TW;
  static constexpr int TILE = NW * TW;      // tokens per tile
  static constexpr int TILE_UNITS = TILE / kUnitTokens;
  static constexpr int DPL = D / 32;        // dims per lane (PV)
  static constexpr bool SWZ = false;
  static constexpr int ROW = D * E;
  static constexpr int TILE_BYTES = TILE * ROW;
  static constexpr int STAGE_BYTES = 2 * TILE_BYTES;
  static constexpr int EXTRA_FLOATS = NW * TW * GP;  // probability broadcast
  static_assert(TILE % kUnitTokens == 0, "tile must hold whole units");
  static_assert(D % 32 == 0 && CH % LPT == 0, "unsupported head_dim");
  static_assert(DPL * E <= 16, "PV lane width");
  static constexpr int CHUNKS = CH;  // 16-byte chunks of a K/V row
  static_assert(LAYOUT_ != kTma128B || (D * E) % 128 == 0, "whole 128-byte column blocks");

  // Byte offset of element d of token row `row` in a stage tile.
  __device__ static __forceinline__ int elem_offset(int row, int d) {
    if constexpr (LAYOUT == kTma128B) {
      const int chunk = d / VEC;
      return (chunk >> 3) * (TILE * 128) + row * 128 + (((chunk & 7) ^ (row & 7)) << 4) +
             (d % VEC) * E;
    } else {
      return (row * D + d) * E;
    }
  }
  // Byte offset of 16-byte chunk `col` of token row `row`.
  __device__ static __forceinline__ int offset(int row, int col) {
    return elem_offset(row, col * VEC);
  }

  struct State {
    float q[GP][DL];
    float m[GP], l[GP], acc[GP][DPL];
  };

  __device__ static void begin_piece(State& s, const AttnParams& p, int b, int h) {
    const int l8 = (threadIdx.x & 31) % LPT;
    const T* qb = static_cast<const T*>(p.q) + ((int64_t)b * p.H + (int64_t)h * p.G) * D;
#pragma unroll
    for (int g = 0; g < GP; ++g) {
#pragma unroll
      for (int c = 0; c < CPL; ++c) {
        if (g < p.G) {
          const uint4 raw = __ldg(reinterpret_cast<const uint4*>(qb + g * D + (l8 + LPT * c) * VEC));
          Chunk<T>::to_f(raw, &s.q[g][c * VEC]);
        } else {
#pragma unroll
          for (int e = 0; e < VEC; ++e) s.q[g][c * VEC + e] = 0.f;
        }
      }
      s.m[g] = -INFINITY;
      s.l[g] = 0.f;
#pragma unroll
      for (int d = 0; d < DPL; ++d) s.acc[g][d] = 0.f;
    }
  }

  // begin_piece with the group's G query rows (D elements each, consecutive)
  // at `qbase`, in global or shared memory.
  __device__ static void begin_piece_at(State& s, const T* qbase, int G) {
    const int l8 = (threadIdx.x & 31) % LPT;
#pragma unroll
    for (int g = 0; g < GP; ++g) {
#pragma unroll
      for (int c = 0; c < CPL; ++c) {
        if (g < G) {
          const uint4 raw = *reinterpret_cast<const uint4*>(qbase + g * D + (l8 + LPT * c) * VEC);
          Chunk<T>::to_f(raw, &s.q[g][c * VEC]);
        } else {
#pragma unroll
          for (int e = 0; e < VEC; ++e) s.q[g][c * VEC + e] = 0.f;
        }
      }
      s.m[g] = -INFINITY;
      s.l[g] = 0.f;
#pragma unroll
      for (int d = 0; d < DPL; ++d) s.acc[g][d] = 0.f;
    }
  }

  __device__ static void compute_tile(State& st, const AttnParams& p, const unsigned char* skb,
                                      const unsigned char* svb, int ntok, float* ps) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int grp = lane / LPT, l8 = lane % LPT;
    float s[GP][TPG];
#pragma unroll
    for (int r = 0; r < TPG; ++r) {
      const int row = warp * TW + r * TPW + grp;
      float part[GP];
#pragma unroll
      for (int g = 0; g < GP; ++g) part[g] = 0.f;
#pragma unroll
      for (int c = 0; c < CPL; ++c) {
        float kf[VEC];
        lds_to_f<T, VEC>(reinterpret_cast<const T*>(skb + offset(row, l8 + LPT * c)), kf);
#pragma unroll
        for (int g = 0; g < GP; ++g)
#pragma unroll
          for (int e = 0; e < VEC; ++e) part[g] = fmaf(st.q[g][c * VEC + e], kf[e], part[g]);
      }
#pragma unroll
      for (int o = 1; o < LPT; o <<= 1)
#pragma unroll
        for (int g = 0; g < GP; ++g) part[g] += __shfl_xor_sync(0xffffffffu, part[g], o);
#pragma unroll
      for (int g = 0; g < GP; ++g) s[g][r] = row < ntok ? part[g] * p.scale_log2 : -INFINITY;
    }

    // tile max, lazy rescale (m is warp-uniform)
#pragma unroll
    for (int g = 0; g < GP; ++g) {
      float mt = s[g][0];
#pragma unroll
      for (int r = 1; r < TPG; ++r) mt = fmaxf(mt, s[g][r]);
#pragma unroll
      for (int o = LPT; o < 32; o <<= 1) mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, o));
      const float mn = fmaxf(st.m[g], mt);
      if (mn > st.m[g]) {
        const float alpha = (st.m[g] == -INFINITY) ? 0.f : exp2f(st.m[g] - mn);
        st.l[g] *= alpha;
#pragma unroll
        for (int d = 0; d < DPL; ++d) st.acc[g][d] *= alpha;
        st.m[g] = mn;
      }
    }

    float* pw = ps + warp * TW * GP;
#pragma unroll
    for (int r = 0; r < TPG; ++r) {
      float pr[GP];
#pragma unroll
      for (int g = 0; g < GP; ++g) {
        pr[g] = (s[g][r] == -INFINITY) ? 0.f : exp2f(s[g][r] - st.m[g]);
        st.l[g] += pr[g];
      }
      if (l8 == 0) {
#pragma unroll
        for (int g = 0; g < GP; ++g) pw[(r * TPW + grp) * GP + g] = pr[g];
      }
    }
    __syncwarp();

    const int nrow = ntok - warp * TW;
#pragma unroll
    for (int i = 0; i < TW; ++i) {
      if (i < nrow) {
        float pv[GP];
#pragma unroll
        for (int g = 0; g < GP; ++g) pv[g] = pw[i * GP + g];
        float vf[DPL];
        lds_to_f<T, DPL>(reinterpret_cast<const T*>(svb + elem_offset(warp * TW + i, lane * DPL)),
                         vf);
#pragma unroll
        for (int g = 0; g < GP; ++g)
#pragma unroll
          for (int d = 0; d < DPL; ++d) st.acc[g][d] = fmaf(pv[g], vf[d], st.acc[g][d]);
      }
    }
    __syncwarp();
  }

  __device__ static void store_state(State& s, float* ms, float* ls, float* accs) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // l holds this lane group's share; sum over the groups of the warp.
#pragma unroll
    for (int g = 0; g < GP; ++g)
#pragma unroll
      for (int o = LPT; o < 32; o <<= 1) s.l[g] += __shfl_xor_sync(0xffffffffu, s.l[g], o);
    if (lane == 0) {
#pragma unroll
      for (int g = 0; g < GP; ++g) {
        ms[warp * GP + g] = s.m[g];
        ls[warp * GP + g] = s.l[g];
      }
    }
#pragma unroll
    for (int g = 0; g < GP; ++g)
#pragma unroll
      for (int d = 0; d < DPL; ++d) accs[(warp * GP + g) * D + lane * DPL + d] = s.acc[g][d];
  }
};

// ===========================================================================
// Stream-K driver
// ===========================================================================
template <class M>
struct StreamK {
  using T = typename M::T;
  static constexpr int D = M::D, GP = M::GP, NW = M::NW, NT = M::NT;
  static constexpr int SLOT_FLOATS = GP * (D + 2);
  static constexpr int MERGE_FLOATS = NW * GP * (D + 2);
  static size_t smem_bytes(int B) {
    return (size_t)M::STAGES * M::STAGE_BYTES + (size_t)(M::EXTRA_FLOATS + MERGE_FLOATS) * 4 +
           (size_t)(2 * B + 1 + 8) * 4;
  }
};

// Combine the partial slots of pieces w_first..w_last of one segment (the
// piece of w_first in `first_slot`, every later worker's in slot 2w) into the
// segment's G output rows, rescaling in base 2 piece by piece. Called by NTH
// threads, t in [0, NTH). When GP*D splits evenly, thread t owns the E
// consecutive elements [t*E, (t+1)*E) of one row and loads the entries (and
// the row's max and sum) of PU pieces at once — PU as large as the caller's
// register budget BUDGET (floats in flight per thread) allows, at most 8 —
// before combining them in piece order, so a merge costs about one L2 round
// trip per PU pieces. Per element the arithmetic and its order are those of a
// plain sequential loop over the pieces.
template <class T, int GP, int D, int NTH, int BUDGET>
__device__ __forceinline__ void merge_slots(const float* partials, T* outp, int G,
                                            int64_t w_first, int64_t w_last,
                                            int64_t first_slot, int t) {
  constexpr int SLOT_FLOATS = GP * (D + 2);
  constexpr int E = GP * D / NTH;
  constexpr int E_DIV = E > 0 ? E : 1;
  if constexpr (GP * D % NTH == 0 && E >= 1 && D % E_DIV == 0) {
    constexpr int PU0 = BUDGET / (E + 2);
    constexpr int PU = PU0 < 1 ? 1 : (PU0 > 8 ? 8 : PU0);  // pieces per batch of loads
    // 16-byte loads when every thread's run of E floats starts 16-byte aligned
    constexpr bool VEC = E % 4 == 0 && (SLOT_FLOATS * 4) % 16 == 0 && (2 * GP * 4) % 16 == 0 &&
                         (D * 4) % 16 == 0;
    const int g = t * E / D, d0 = t * E - g * D;
    float Mx = -INFINITY, Lx = 0.f, Ox[E];
#pragma unroll
    for (int e = 0; e < E; ++e) Ox[e] = 0.f;
    for (int64_t w0 = w_first; w0 <= w_last; w0 += PU) {
      float mc[PU], lc[PU], oc[PU][E];
#pragma unroll
      for (int u = 0; u < PU; ++u) {
        const int64_t w = w0 + u;
        if (w <= w_last) {
          const float* sl = partials + (size_t)(w == w_first ? first_slot : 2 * w) * SLOT_FLOATS;
          mc[u] = __ldcg(sl + g);
          lc[u] = __ldcg(sl + GP + g);
          const float* src = sl + 2 * GP + g * D + d0;
          if constexpr (VEC) {
#pragma unroll
            for (int e = 0; e < E; e += 4) {
              const float4 v = __ldcg(reinterpret_cast<const float4*>(src + e));
              oc[u][e] = v.x;
              oc[u][e + 1] = v.y;
              oc[u][e + 2] = v.z;
              oc[u][e + 3] = v.w;
            }
          } else {
#pragma unroll
            for (int e = 0; e < E; ++e) oc[u][e] = __ldcg(src + e);
          }
        }
      }
#pragma unroll
      for (int u = 0; u < PU; ++u) {
        if (w0 + u <= w_last) {
          const float Mn = fmaxf(Mx, mc[u]);
          const float a = (Mx == -INFINITY) ? 0.f : exp2f(Mx - Mn);
          const float b = (mc[u] == -INFINITY) ? 0.f : exp2f(mc[u] - Mn);
          Lx = fmaf(Lx, a, lc[u] * b);
#pragma unroll
          for (int e = 0; e < E; ++e) Ox[e] = fmaf(Ox[e], a, oc[u][e] * b);
          Mx = Mn;
        }
      }
    }
    if (g < G) {
#pragma unroll
      for (int e = 0; e < E; ++e) outp[g * D + d0 + e] = Elem<T>::from_f(Ox[e] / Lx);
    }
  } else {
    for (int idx = t; idx < GP * D; idx += NTH) {
      const int g = idx / D, d = idx - g * D;
      if (g >= G) continue;
      float M_ = -INFINITY, L = 0.f, O = 0.f;
#pragma unroll 4  // slot loads of consecutive pieces in flight together
      for (int64_t w = w_first; w <= w_last; ++w) {
        const float* sl = partials + (size_t)(w == w_first ? first_slot : 2 * w) * SLOT_FLOATS;
        const float mc = __ldcg(sl + g), lc = __ldcg(sl + GP + g);
        const float oc = __ldcg(sl + 2 * GP + g * D + d);
        const float Mn = fmaxf(M_, mc);
        const float a = (M_ == -INFINITY) ? 0.f : exp2f(M_ - Mn);
        const float b = (mc == -INFINITY) ? 0.f : exp2f(mc - Mn);
        L = fmaf(L, a, lc * b);
        O = fmaf(O, a, oc * b);
        M_ = Mn;
      }
      outp[g * D + d] = Elem<T>::from_f(O / L);
    }
  }
}

// Merge the NW warp states of a finished piece [piece_u0, ...) of segment
// (cc.b, cc.h) and write the output, or publish the piece's partial and, if
// this CTA is the last to finish a piece of the segment, combine all pieces.
// `sync` is a barrier over the threads that call this (all math warps).
// On entry the warp states are in ms/ls/accs and `sync` has been passed.
template <class M, class Sync>
__device__ __forceinline__ void finish_piece(const AttnParams& p, const Cursor& cc,
                                             int64_t piece_u0, int64_t u_beg, int64_t U,
                                             int64_t grid, bool seg_end, const float* ms,
                                             const float* ls, const float* accs, int* misc,
                                             Sync sync) {
  using T = typename M::T;
  constexpr int D = M::D, GP = M::GP, NW = M::NW, NT = M::NT;
  constexpr int SLOT_FLOATS = GP * (D + 2);
  const int tid = threadIdx.x;
  const bool whole = (piece_u0 == cc.seg) && seg_end;
  T* outp = static_cast<T*>(p.out) + ((int64_t)cc.b * p.H + (int64_t)cc.h * p.G) * D;
  float* slot = p.partials + (size_t)(2 * blockIdx.x + (piece_u0 == u_beg ? 0 : 1)) * SLOT_FLOATS;
  for (int idx = tid; idx < GP * D; idx += NT) {
    const int g = idx / D, d = idx - g * D;
    float M_ = -INFINITY;
#pragma unroll
    for (int w = 0; w < NW; ++w) M_ = fmaxf(M_, ms[w * GP + g]);
    float L = 0.f, O = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) {
      const float mw = ms[w * GP + g];
      const float f = (mw == -INFINITY) ? 0.f : exp2f(mw - M_);
      L = fmaf(ls[w * GP + g], f, L);
      O = fmaf(accs[(w * GP + g) * D + d], f, O);
    }
    if (whole) {
      if (g < p.G) outp[g * D + d] = Elem<T>::from_f(O / L);
    } else {
      slot[2 * GP + g * D + d] = O;
      if (d == 0) {
        slot[g] = M_;
        slot[GP + g] = L;
      }
    }
  }

  if (!whole) {
    sync();  // all partial stores of this CTA precede thread 0's release
    const int64_t S0 = cc.seg, S1 = cc.seg + cc.nu;
    const int64_t c0 = part_owner(S0, U, grid), c1 = part_owner(S1 - 1, U, grid);
    if (tid == 0)
      misc[1] = arrive_piece(p.counters + ((int64_t)cc.b * p.KVH + cc.h), p.call_tag,
                             (unsigned)(c1 - c0 + 1));
    sync();
    if (misc[1]) {
      // Only CTA c0 can hold its piece in slot 1 (it is the one CTA whose
      // range starts before the segment); every later CTA starts inside it.
      const int64_t first_slot = 2 * c0 + (part_begin(c0, U, grid) < S0 ? 1 : 0);
      merge_slots<T, GP, D, NT, 16>(p.partials, outp, p.G, c0, c1, first_slot, tid);
    }
  }
  sync();
}

template <class M>
__global__ void __launch_bounds__(M::NT)
attn_streamk_kernel(const AttnParams p) {
  using T = typename M::T;
  using SK = StreamK<M>;
  constexpr int D = M::D, GP = M::GP, STAGES = M::STAGES, NW = M::NW, NT = M::NT;
  constexpr int TILE = M::TILE;

  extern __shared__ __align__(128) unsigned char smem[];
  float* extra = reinterpret_cast<float*>(smem + (size_t)STAGES * M::STAGE_BYTES);
  float* ms = extra + M::EXTRA_FLOATS;  // [NW][GP]
  float* ls = ms + NW * GP;             // [NW][GP]
  float* accs = ls + NW * GP;           // [NW][GP][D]
  int* P = reinterpret_cast<int*>(accs + NW * GP * D);  // [B+1]
  int* Ls = P + p.B + 1;                                 // [B]
  int* misc = Ls + p.B;                                  // [8]
  const int tid = threadIdx.x;
  const int KVH = p.KVH;

  const int64_t U = plan_units<NT>(p, P, Ls, misc);

  // zero-length sequences produce zeros (cuda/paged_attention.cu:56)
  for (int b = blockIdx.x; b < p.B; b += gridDim.x) {
    if (Ls[b] == 0) {
      T* o = static_cast<T*>(p.out) + (int64_t)b * p.H * D;
      for (int i = tid; i < p.H * D; i += NT) o[i] = Elem<T>::from_f(0.f);
    }
  }

  // Effective grid: never more CTAs than units, so every working CTA owns at
  // least one unit and the CTAs covering a segment are exactly its pieces.
  const int64_t grid = part_grid(gridDim.x, U);
  if ((int64_t)blockIdx.x >= grid) return;
  const int64_t u_beg = part_begin(blockIdx.x, U, grid);
  const int64_t u_end = part_begin(blockIdx.x + 1, U, grid);
  if (u_beg >= u_end) return;

  unsigned char* stages = smem;
  auto stage_k = [&](int s) { return stages + (size_t)s * M::STAGE_BYTES; };

  Cursor lc;
  cursor_locate(lc, P, p.B, KVH, u_beg);
  Cursor cc = lc;
  bool l_done = false;
#pragma unroll 1
  for (int s = 0; s < STAGES - 1; ++s) {
    if (!l_done) {
      const int64_t te = cursor_tile_end<M::TILE_UNITS>(lc, u_end);
      load_tile<T, D, TILE, NT, M::SWZ>(p, Ls, lc, te, stage_k(s), stage_k(s) + M::TILE_BYTES);
      cursor_advance(lc, te, u_end, P, KVH);
      l_done = lc.u >= u_end;
    }
    cp_async_commit();
  }

  typename M::State st;
  bool piece_start = true;
  int64_t piece_u0 = u_beg;
  int stage = 0, lstage = STAGES - 1;

#pragma unroll 1
  while (true) {
    cp_async_wait<STAGES - 2>();
    __syncthreads();
    if (!l_done) {
      const int64_t te = cursor_tile_end<M::TILE_UNITS>(lc, u_end);
      load_tile<T, D, TILE, NT, M::SWZ>(p, Ls, lc, te, stage_k(lstage),
                                        stage_k(lstage) + M::TILE_BYTES);
      cursor_advance(lc, te, u_end, P, KVH);
      l_done = lc.u >= u_end;
    }
    cp_async_commit();
    lstage = (lstage + 1 == STAGES) ? 0 : lstage + 1;

    const int64_t cte = cursor_tile_end<M::TILE_UNITS>(cc, u_end);
    if (piece_start) {
      piece_u0 = cc.u;
      piece_start = false;
      M::begin_piece(st, p, cc.b, cc.h);
    }
    M::compute_tile(st, p, stage_k(stage), stage_k(stage) + M::TILE_BYTES,
                    tile_tokens(cc, cte, Ls), extra);

    const bool seg_end = (cte == cc.seg + cc.nu);
    if (seg_end || cte == u_end) {
      M::store_state(st, ms, ls, accs);
      __syncthreads();
      finish_piece<M>(p, cc, piece_u0, u_beg, U, grid, seg_end, ms, ls, accs, misc,
                      [] { __syncthreads(); });
      piece_start = true;
    }

    stage = (stage + 1 == STAGES) ? 0 : stage + 1;
    if (cte >= u_end) break;
    cursor_advance(cc, cte, u_end, P, KVH);
  }
  cp_async_wait<0>();
}

// ===========================================================================
// Generic kernel (fallback for shapes outside the stream-K instantiations)
// ===========================================================================
template <typename T>
__global__ void __launch_bounds__(128) attn_generic_kernel(const AttnParams p) {
  constexpr int NW = 4, MAXD = 8;  // head_dim <= 256
  __shared__ float qs[256];
  __shared__ float wm[NW], wl[NW];
  __shared__ float wacc[NW][256];
  const int split = blockIdx.x, hq = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int D = p.D, h = hq / p.G;
  const int len = checked_length(p.lengths, b, p.max_length);
  const int t0 = split * p.chunk;
  const int t1 = min(len, t0 + p.chunk);
  const T* qrow = static_cast<const T*>(p.q) + ((int64_t)b * p.H + hq) * D;
  for (int d = tid; d < D; d += 128) qs[d] = Elem<T>::to_f(qrow[d]);
  __syncthreads();

  const T* kpool = static_cast<const T*>(p.k_pool);
  const T* vpool = static_cast<const T*>(p.v_pool);
  const int32_t* trow = p.tables + (int64_t)b * p.table_width;
  float m = -INFINITY, l = 0.f, acc[MAXD];
#pragma unroll
  for (int i = 0; i < MAXD; ++i) acc[i] = 0.f;
  for (int t = t0 + warp; t < t1; t += NW) {
    const int pi = t / p.block_size, off = t - pi * p.block_size;
    const int page = trow[pi];
    if (page < 0 || (int64_t)page >= p.num_blocks) {
      if (lane == 0) raise_error(0x1u);
      continue;
    }
    const int64_t base = (((int64_t)page * p.block_size + off) * p.KVH + h) * D;
    float sc = 0.f;
    for (int d = lane; d < D; d += 32) sc = fmaf(qs[d], Elem<T>::to_f(kpool[base + d]), sc);
#pragma unroll
    for (int o = 16; o; o >>= 1) sc += __shfl_xor_sync(0xffffffffu, sc, o);
    sc *= p.scale_log2;
    const float mn = fmaxf(m, sc);
    const float alpha = (m == -INFINITY) ? 0.f : exp2f(m - mn);
    const float pr = exp2f(sc - mn);
    l = l * alpha + pr;
#pragma unroll
    for (int i = 0; i < MAXD; ++i) {
      const int d = lane + 32 * i;
      if (d < D) acc[i] = acc[i] * alpha + pr * Elem<T>::to_f(vpool[base + d]);
    }
    m = mn;
  }
  if (lane == 0) { wm[warp] = m; wl[warp] = l; }
#pragma unroll
  for (int i = 0; i < MAXD; ++i) {
    const int d = lane + 32 * i;
    if (d < D) wacc[warp][d] = acc[i];
  }
  __syncthreads();
  float M = -INFINITY;
  for (int w = 0; w < NW; ++w) M = fmaxf(M, wm[w]);
  float L = 0.f;
  for (int w = 0; w < NW; ++w) L += (wm[w] == -INFINITY) ? 0.f : wl[w] * exp2f(wm[w] - M);
  for (int d = tid; d < D; d += 128) {
    float O = 0.f;
    for (int w = 0; w < NW; ++w)
      O += (wm[w] == -INFINITY) ? 0.f : wacc[w][d] * exp2f(wm[w] - M);
    if (p.splits == 1) {
      T* o = static_cast<T*>(p.out) + ((int64_t)b * p.H + hq) * D;
      o[d] = Elem<T>::from_f(L > 0.f ? O / L : 0.f);
    } else {
      float* sl = p.partials + (((int64_t)b * p.H + hq) * p.splits + split) * (D + 2);
      sl[2 + d] = O;
      if (d == 0) { sl[0] = M; sl[1] = L; }
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(128) attn_combine_kernel(const AttnParams p) {
  const int hq = blockIdx.x, b = blockIdx.y, D = p.D;
  const float* base = p.partials + ((int64_t)b * p.H + hq) * p.splits * (D + 2);
  float M = -INFINITY;
  for (int s = 0; s < p.splits; ++s) M = fmaxf(M, base[s * (D + 2)]);
  float L = 0.f;
  for (int s = 0; s < p.splits; ++s) {
    const float ms = base[s * (D + 2)];
    if (ms != -INFINITY) L += base[s * (D + 2) + 1] * exp2f(ms - M);
  }
  T* o = static_cast<T*>(p.out) + ((int64_t)b * p.H + hq) * D;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float O = 0.f;
    for (int s = 0; s < p.splits; ++s) {
      const float ms = base[s * (D + 2)];
      if (ms != -INFINITY) O += base[s * (D + 2) + 2 + d] * exp2f(ms - M);
    }
    o[d] = Elem<T>::from_f(L > 0.f ? O / L : 0.f);
  }
}

}  // namespace pdb
