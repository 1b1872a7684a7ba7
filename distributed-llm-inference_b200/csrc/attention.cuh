// Paged GQA decode attention for sm_100a.
//
// Computes, for every sequence b and query head hq (kv head h = hq / G):
//   out[b, hq] = sum_t softmax_t(q[b,hq] . K[t] / sqrt(D)) * V[t],  t < len[b]
// where token t lives at pool[tables[b, t / bs], t % bs, h, :] and out is 0
// for len[b] == 0. This is the contract of attention_kernel in
// cuda/paged_attention.cu:10-58 and of torch_paged_attention in
// worker/llama.py:58-71.
//
// Two kernels:
//  * attn_fast_kernel — persistent, one work list per call.
//      - Work is flattened into 16-token units ordered by (sequence, kv head,
//        token). CTA c owns the contiguous unit range [c*U/grid, (c+1)*U/grid),
//        so every CTA streams the same number of K/V bytes whatever the
//        length distribution (no idle SMs at the tail of a lognormal batch).
//      - A CTA stages each K/V tile of one kv head into shared memory once
//        (cp.async, STAGES-deep ring) and all G query heads of the GQA group
//        read it there: K/V cross HBM exactly once.
//      - QK: lanes of a warp split a token row into 16-byte chunks
//        (conflict-free LDS.128), q lives in registers, scores are reduced
//        with warp shuffles. Online softmax in fp32 (base 2). PV: each lane
//        owns D/32 output dims; probabilities are broadcast through smem.
//      - A (sequence, kv head) segment cut by a CTA boundary is a "piece":
//        its partial (m, l, o) goes to the workspace and the last CTA to
//        finish a piece of that segment (epoch-tagged arrival counter, no
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
  unsigned long long* counters;  // fast: [B*KVH] epoch<<32 | arrivals
  float* partials;               // fast: [2*grid][GP*(D+2)]; generic: [B*H*splits][D+2]
  uint32_t epoch;
  int splits;  // generic
  int chunk;   // generic: tokens per split
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

// ===========================================================================
// Fast kernel
// ===========================================================================
template <typename T, int D_, int GP_, int TPG_, int STAGES_>
struct FastTraits {
  using Elem_t = T;
  static constexpr int D = D_;
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
  static constexpr int NW = 4;
  static constexpr int NT = NW * 32;
  static constexpr int TW = TPW * TPG;      // tokens per warp per tile
  static constexpr int TILE = NW * TW;      // tokens per tile
  static constexpr int TILE_UNITS = TILE / kUnitTokens;
  static constexpr int DPL = D / 32;        // dims per lane (PV)
  static constexpr int ROW = D * E;         // bytes per token row
  static constexpr int TILE_BYTES = TILE * ROW;
  static constexpr int STAGE_BYTES = 2 * TILE_BYTES;
  static constexpr int PS_FLOATS = NW * TW * GP;
  static constexpr int MERGE_FLOATS = NW * GP * (D + 2);
  static constexpr int SLOT_FLOATS = GP * (D + 2);
  static_assert(TILE % kUnitTokens == 0, "tile must hold whole units");
  static_assert(D % 32 == 0 && CH % LPT == 0, "unsupported head_dim");
  static_assert(DPL * E <= 16, "PV lane width");

  static size_t smem_bytes(int B) {
    return (size_t)STAGES * STAGE_BYTES + (size_t)(PS_FLOATS + MERGE_FLOATS) * 4 +
           (size_t)(2 * B + 1 + 8) * 4;
  }
};

// Position in the flattened unit stream of one CTA.
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

template <class Tr>
__global__ void __launch_bounds__(Tr::NT)
attn_fast_kernel(const AttnParams p) {
  using T = typename Tr::Elem_t;
  constexpr int D = Tr::D, GP = Tr::GP, TPG = Tr::TPG, STAGES = Tr::STAGES;
  constexpr int VEC = Tr::VEC, CH = Tr::CH, LPT = Tr::LPT, CPL = Tr::CPL;
  constexpr int DL = Tr::DL, TPW = Tr::TPW, NW = Tr::NW, NT = Tr::NT;
  constexpr int TW = Tr::TW, TILE = Tr::TILE, DPL = Tr::DPL;

  extern __shared__ __align__(128) unsigned char smem[];
  float* ps = reinterpret_cast<float*>(smem + (size_t)STAGES * Tr::STAGE_BYTES);
  float* ms = ps + Tr::PS_FLOATS;  // [NW][GP]
  float* ls = ms + NW * GP;        // [NW][GP]
  float* accs = ls + NW * GP;      // [NW][GP][D]
  int* P = reinterpret_cast<int*>(accs + NW * GP * D);  // [B+1]
  int* Ls = P + p.B + 1;                                 // [B]
  int* misc = Ls + p.B;                                  // [8]

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int B = p.B, KVH = p.KVH;
  const T* __restrict__ kpool = static_cast<const T*>(p.k_pool);
  const T* __restrict__ vpool = static_cast<const T*>(p.v_pool);

  // ---- plan: P[b] = KVH * sum_{b' < b} ceil(len_b' / 16) -------------------
  if (tid == 0) misc[0] = 0;
  __syncthreads();
  for (int base = 0; base < B; base += NT) {
    const int b = base + tid;
    int nu = 0;
    if (b < B) {
      const int len = checked_length(p.lengths, b, p.max_length);
      Ls[b] = len;
      nu = ((len + kUnitTokens - 1) / kUnitTokens) * KVH;
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
    if (b < B) P[b] = woff + incl - nu;
    __syncthreads();
    if (tid == NT - 1) misc[0] = woff + incl;
    __syncthreads();
  }
  if (tid == 0) P[B] = misc[0];
  __syncthreads();
  const int64_t U = P[B];

  // zero-length sequences produce zeros (cuda/paged_attention.cu:56)
  for (int b = blockIdx.x; b < B; b += gridDim.x) {
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
  const int grp = lane / LPT, l8 = lane % LPT;

  // ---- loader -----------------------------------------------------------
  auto load_tile = [&](const Cursor& c, int64_t te, int stage) {
    const int tok0 = (int)(c.u - c.seg) * kUnitTokens;
    const int rem = Ls[c.b] - tok0;
    const int span = (int)(te - c.u) * kUnitTokens;
    const int ntok = span < rem ? span : rem;
    const int32_t* trow = p.tables + (int64_t)c.b * p.table_width;
    unsigned char* sk = stages + (size_t)stage * Tr::STAGE_BYTES;
    unsigned char* sv = sk + Tr::TILE_BYTES;
#pragma unroll
    for (int i = tid; i < TILE * CH; i += NT) {
      const int row = i / CH, col = i % CH;
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
        const int page = __ldg(trow + pi);
        if (page < 0 || (int64_t)page >= p.num_blocks) {
          raise_error(0x1u);
          ok = false;
        } else {
          const int64_t e =
              (((int64_t)page * p.block_size + off) * KVH + c.h) * D + col * VEC;
          ks = kpool + e;
          vs = vpool + e;
        }
      }
      cp_async16(sk + row * Tr::ROW + col * 16, ks, ok);
      cp_async16(sv + row * Tr::ROW + col * 16, vs, ok);
    }
  };

  Cursor lc;
  cursor_locate(lc, P, B, KVH, u_beg);
  Cursor cc = lc;
  bool l_done = false;
#pragma unroll 1
  for (int s = 0; s < STAGES - 1; ++s) {
    if (!l_done) {
      const int64_t te = cursor_tile_end<Tr::TILE_UNITS>(lc, u_end);
      load_tile(lc, te, s);
      cursor_advance(lc, te, u_end, P, KVH);
      l_done = lc.u >= u_end;
    }
    cp_async_commit();
  }

  float q[GP][DL];
  float m[GP], l[GP], acc[GP][DPL];
  bool piece_start = true;
  int64_t piece_u0 = u_beg;
  int stage = 0, lstage = STAGES - 1;

#pragma unroll 1
  while (true) {
    cp_async_wait<STAGES - 2>();
    __syncthreads();
    if (!l_done) {
      const int64_t te = cursor_tile_end<Tr::TILE_UNITS>(lc, u_end);
      load_tile(lc, te, lstage);
      cursor_advance(lc, te, u_end, P, KVH);
      l_done = lc.u >= u_end;
    }
    cp_async_commit();
    lstage = (lstage + 1 == STAGES) ? 0 : lstage + 1;

    const int64_t cte = cursor_tile_end<Tr::TILE_UNITS>(cc, u_end);
    if (piece_start) {
      piece_u0 = cc.u;
      piece_start = false;
      const T* qb = static_cast<const T*>(p.q) + ((int64_t)cc.b * p.H + (int64_t)cc.h * p.G) * D;
#pragma unroll
      for (int g = 0; g < GP; ++g) {
#pragma unroll
        for (int c = 0; c < CPL; ++c) {
          if (g < p.G) {
            const uint4 raw = __ldg(reinterpret_cast<const uint4*>(qb + g * D + (l8 + LPT * c) * VEC));
            Chunk<T>::to_f(raw, &q[g][c * VEC]);
          } else {
#pragma unroll
            for (int e = 0; e < VEC; ++e) q[g][c * VEC + e] = 0.f;
          }
        }
        m[g] = -INFINITY;
        l[g] = 0.f;
#pragma unroll
        for (int d = 0; d < DPL; ++d) acc[g][d] = 0.f;
      }
    }

    // ---- compute one tile ------------------------------------------------
    {
      const int tok0 = (int)(cc.u - cc.seg) * kUnitTokens;
      const int rem = Ls[cc.b] - tok0;
      const int span = (int)(cte - cc.u) * kUnitTokens;
      const int ntok = span < rem ? span : rem;
      const T* sk = reinterpret_cast<const T*>(stages + (size_t)stage * Tr::STAGE_BYTES);
      const T* sv = reinterpret_cast<const T*>(stages + (size_t)stage * Tr::STAGE_BYTES + Tr::TILE_BYTES);

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
          lds_to_f<T, VEC>(sk + row * D + (l8 + LPT * c) * VEC, kf);
#pragma unroll
          for (int g = 0; g < GP; ++g)
#pragma unroll
            for (int e = 0; e < VEC; ++e) part[g] = fmaf(q[g][c * VEC + e], kf[e], part[g]);
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
        const float mn = fmaxf(m[g], mt);
        if (mn > m[g]) {
          const float alpha = (m[g] == -INFINITY) ? 0.f : exp2f(m[g] - mn);
          l[g] *= alpha;
#pragma unroll
          for (int d = 0; d < DPL; ++d) acc[g][d] *= alpha;
          m[g] = mn;
        }
      }

      float* pw = ps + warp * TW * GP;
#pragma unroll
      for (int r = 0; r < TPG; ++r) {
        float pr[GP];
#pragma unroll
        for (int g = 0; g < GP; ++g) {
          pr[g] = (s[g][r] == -INFINITY) ? 0.f : exp2f(s[g][r] - m[g]);
          l[g] += pr[g];
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
          lds_to_f<T, DPL>(sv + (warp * TW + i) * D + lane * DPL, vf);
#pragma unroll
          for (int g = 0; g < GP; ++g)
#pragma unroll
            for (int d = 0; d < DPL; ++d) acc[g][d] = fmaf(pv[g], vf[d], acc[g][d]);
        }
      }
      __syncwarp();
    }

    const bool seg_end = (cte == cc.seg + cc.nu);
    if (seg_end || cte == u_end) {
      // ---- finish the piece [piece_u0, cte) of segment (cc.b, cc.h) --------
      // l holds this lane group's share; sum over the groups of the warp.
#pragma unroll
      for (int g = 0; g < GP; ++g)
#pragma unroll
        for (int o = LPT; o < 32; o <<= 1) l[g] += __shfl_xor_sync(0xffffffffu, l[g], o);
      if (lane == 0) {
#pragma unroll
        for (int g = 0; g < GP; ++g) {
          ms[warp * GP + g] = m[g];
          ls[warp * GP + g] = l[g];
        }
      }
#pragma unroll
      for (int g = 0; g < GP; ++g)
#pragma unroll
        for (int d = 0; d < DPL; ++d) accs[(warp * GP + g) * D + lane * DPL + d] = acc[g][d];
      __syncthreads();

      const bool whole = (piece_u0 == cc.seg) && seg_end;
      T* outp = static_cast<T*>(p.out) + ((int64_t)cc.b * p.H + (int64_t)cc.h * p.G) * D;
      float* slot = p.partials +
                    (size_t)(2 * blockIdx.x + (piece_u0 == u_beg ? 0 : 1)) * Tr::SLOT_FLOATS;
      for (int idx = tid; idx < GP * D; idx += NT) {
        const int g = idx / D, d = idx - g * D;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < NW; ++w) M = fmaxf(M, ms[w * GP + g]);
        float L = 0.f, O = 0.f;
#pragma unroll
        for (int w = 0; w < NW; ++w) {
          const float mw = ms[w * GP + g];
          const float f = (mw == -INFINITY) ? 0.f : exp2f(mw - M);
          L = fmaf(ls[w * GP + g], f, L);
          O = fmaf(accs[(w * GP + g) * D + d], f, O);
        }
        if (whole) {
          if (g < p.G) outp[g * D + d] = Elem<T>::from_f(O / L);
        } else {
          slot[2 * GP + g * D + d] = O;
          if (d == 0) {
            slot[g] = M;
            slot[GP + g] = L;
          }
        }
      }

      if (!whole) {
        __threadfence();
        __syncthreads();
        const int64_t S0 = cc.seg, S1 = cc.seg + cc.nu;
        const int64_t c0 = part_owner(S0, U, grid), c1 = part_owner(S1 - 1, U, grid);
        unsigned long long* ctr = p.counters + ((int64_t)cc.b * KVH + cc.h);
        if (tid == 0) {
          const unsigned long long ep = (unsigned long long)p.epoch << 32;
          unsigned long long old = *reinterpret_cast<volatile unsigned long long*>(ctr);
          int last = 0;
          bool done = false;
          for (int it = 0; it < (1 << 20) && !done; ++it) {
            const unsigned cnt = ((old >> 32) == p.epoch) ? (unsigned)(old & 0xffffffffull) : 0u;
            const unsigned long long nw = ep | (unsigned long long)(cnt + 1u);
            const unsigned long long prev = atomicCAS(ctr, old, nw);
            if (prev == old) {
              done = true;
              last = ((int64_t)cnt + 1 == c1 - c0 + 1) ? 1 : 0;
            } else {
              old = prev;
            }
          }
          misc[1] = last;
        }
        __syncthreads();
        if (misc[1]) {
          __threadfence();
          for (int idx = tid; idx < GP * D; idx += NT) {
            const int g = idx / D, d = idx - g * D;
            if (g >= p.G) continue;
            float M = -INFINITY;
            for (int64_t c = c0; c <= c1; ++c) {
              const float* sl = p.partials +
                  (size_t)(2 * c + (part_begin(c, U, grid) >= S0 ? 0 : 1)) * Tr::SLOT_FLOATS;
              M = fmaxf(M, __ldcg(sl + g));
            }
            float L = 0.f, O = 0.f;
            for (int64_t c = c0; c <= c1; ++c) {
              const float* sl = p.partials +
                  (size_t)(2 * c + (part_begin(c, U, grid) >= S0 ? 0 : 1)) * Tr::SLOT_FLOATS;
              const float mc = __ldcg(sl + g);
              const float f = (mc == -INFINITY) ? 0.f : exp2f(mc - M);
              L = fmaf(__ldcg(sl + GP + g), f, L);
              O = fmaf(__ldcg(sl + 2 * GP + g * D + d), f, O);
            }
            outp[g * D + d] = Elem<T>::from_f(O / L);
          }
          if (tid == 0) atomicExch(ctr, (unsigned long long)p.epoch << 32);
        }
      }
      __syncthreads();
      piece_start = true;
    }

    stage = (stage + 1 == STAGES) ? 0 : stage + 1;
    if (cte >= u_end) break;
    cursor_advance(cc, cte, u_end, P, KVH);
  }
  cp_async_wait<0>();
}

// ===========================================================================
// Generic kernel (fallback for shapes outside the fast instantiations)
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
