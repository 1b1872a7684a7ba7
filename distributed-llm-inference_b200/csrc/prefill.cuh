// Paged causal prefill attention (sm_100a, FP16).
//
// Replaces the prefill attention of worker/llama.py:141-144:
//   SDPA(q^T, repeat_interleave(k)^T, repeat_interleave(v)^T, is_causal=True)
// over the padded prompt batch [B, W, H, D]. Prompts are left-aligned
// (row b holds len_b tokens at positions 0..len_b-1), so query t of prompt b
// attends to keys 0..t of the same prompt. Here K and V are read from the
// paged pools (the pages rope_kv_write has just filled, located through the
// prompt's block table), never from a padded or repeated copy; each query
// head reads its group's kv head directly.
//
// One CTA per (64-query tile, query head, prompt); 4 warps, 16 query rows
// each. Per 64-key tile (double-buffered with cp.async into XOR-swizzled
// shared memory): S = Q K^T on tensor cores (mma.sync m16n8k16, fp32
// accumulate), causal and length masks (only on the tiles that need them),
// online softmax in fp32 (base 2), then O += P V with P rounded to FP16 (the
// precision of the reference's own SDPA kernels). Rows at or beyond len_b are
// written as zeros: with
// left-aligned prompts and causal attention no real row attends to them and
// they feed only padded rows of later layers.
#pragma once

#include "attention.cuh"

namespace pdb {

struct PrefillParams {
  const __half* q;       // [B, W, H, D]
  const __half* k_pool;  // [N, bs, KVH, D]
  const __half* v_pool;
  const int32_t* tables;   // [B, table_width]
  const int32_t* lengths;  // [B]
  __half* out;             // [B, W, H, D]
  int B, W, H, KVH, G, table_width, block_size, bs_shift;
  int64_t num_blocks;
  float scale_log2;  // log2(e) / sqrt(D)
};

template <int D>
struct PrefillTile {
  static constexpr int NT = 128, BM = 64, BN = 64;
  static constexpr int ROW = D * 2;            // bytes per row
  static constexpr int TILE_BYTES = BM * ROW;  // one Q, K or V tile
  static constexpr int KSTEPS = D / 16;        // QK k-steps
  static constexpr int DT = D / 8;             // PV n-tiles of 8 dims
  static constexpr size_t SMEM = (size_t)TILE_BYTES * 5;  // Q + 2 stages x (K, V)
  static_assert(D % 64 == 0, "swizzle needs >= 8 chunks per row");
};

// Stage key rows [k0, k0 + 64) of prompt b, kv head hk (zero-filled at and
// beyond kend). Page numbers are range-checked before any address is formed.
template <int D>
__device__ __forceinline__ void prefill_load_kv(const PrefillParams& p, int b, int hk, int k0,
                                                int kend, unsigned char* sk, unsigned char* sv) {
  constexpr int CH = D / 8, ROW = D * 2, RPP = 128 / CH;
  const int32_t* trow = p.tables + (int64_t)b * p.table_width;
  const int col = threadIdx.x % CH;
#pragma unroll
  for (int k = 0; k < 64 / RPP; ++k) {
    const int row = threadIdx.x / CH + k * RPP;
    const int t = k0 + row;
    bool ok = t < kend;
    const __half* ks = p.k_pool;
    const __half* vs = p.v_pool;
    if (ok) {
      const int pi = p.bs_shift >= 0 ? (t >> p.bs_shift) : t / p.block_size;
      const int off = t - pi * p.block_size;
      const int page = pi < p.table_width ? __ldg(trow + pi) : -1;
      if (page < 0 || (int64_t)page >= p.num_blocks) {
        raise_error(0x1u);
        ok = false;
      } else {
        const int64_t e = (((int64_t)page * p.block_size + off) * p.KVH + hk) * D + col * 8;
        ks += e;
        vs += e;
      }
    }
    const int o = tile_offset<ROW, true>(row, col);
    cp_async16(sk + o, ks, ok);
    cp_async16(sv + o, vs, ok);
  }
}

template <int D>
__global__ void __launch_bounds__(128) prefill_attention_kernel(const PrefillParams p) {
  using PT = PrefillTile<D>;
  constexpr int KSTEPS = PT::KSTEPS, DT = PT::DT, ROW = PT::ROW, TB = PT::TILE_BYTES;
  constexpr int CH = D / 8, RPP = 128 / CH;
  extern __shared__ __align__(128) unsigned char smem[];
  unsigned char* sq = smem;
  auto stage = [&](int s) { return smem + TB + (size_t)s * 2 * TB; };  // K, then V

  const int b = blockIdx.z, hq = blockIdx.y;
  const int t0 = (int)(gridDim.x - 1 - blockIdx.x) * 64;  // the longest tiles start first
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, tg = lane & 3;
  grid_dependency_wait();
  launch_dependents();
  int n = p.lengths[b];
  if (n < 0 || n > p.W) {
    raise_error(0x2u);
    n = n < 0 ? 0 : p.W;
  }
  const int64_t row_stride = (int64_t)p.H * D;  // elements between consecutive tokens
  __half* obase = p.out + ((int64_t)b * p.W * p.H + hq) * D;
  if (t0 >= n) {  // a tile of padding rows only
    for (int i = tid; i < 64 * CH; i += 128) {
      const int row = i / CH, c = i - row * CH, t = t0 + row;
      if (t < p.W) *reinterpret_cast<uint4*>(obase + t * row_stride + c * 8) = make_uint4(0, 0, 0, 0);
    }
    return;
  }
  const int hk = hq / p.G;
  const __half* qbase = p.q + ((int64_t)b * p.W * p.H + hq) * D;
  {
    const int col = tid % CH;
#pragma unroll
    for (int k = 0; k < 64 / RPP; ++k) {
      const int row = tid / CH + k * RPP, t = t0 + row;
      const bool ok = t < n;
      cp_async16(sq + tile_offset<ROW, true>(row, col), ok ? qbase + t * row_stride + col * 8 : qbase,
                 ok);
    }
  }
  const int kend = n < t0 + 64 ? n : t0 + 64;  // keys [0, kend) can be seen by this tile
  const int nkt = (kend + 63) / 64;
  prefill_load_kv<D>(p, b, hk, 0, kend, stage(0), stage(0) + TB);
  cp_async_commit();

  uint32_t qa[KSTEPS][4];
  float o[DT][4];
#pragma unroll
  for (int i = 0; i < DT; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  const int qr0 = t0 + warp * 16 + g, qr1 = qr0 + 8;  // this lane's two query rows

  for (int j = 0; j < nkt; ++j) {
    if (j + 1 < nkt) prefill_load_kv<D>(p, b, hk, (j + 1) * 64, kend, stage((j + 1) & 1),
                                        stage((j + 1) & 1) + TB);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    if (j == 0) {
      const int row = warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
#pragma unroll
      for (int ks = 0; ks < KSTEPS; ++ks)
        ldsm_x4(qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3],
                sq + tile_offset<ROW, true>(row, 2 * ks + (lane >> 4)));
    }
    const unsigned char* sk = stage(j & 1);
    const unsigned char* sv = sk + TB;

    // S[16 rows x 64 keys] = Q K^T as 8 n-tiles of 8 keys
    float s[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < KSTEPS; ++ks) {
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t b0a, b1a, b0b, b1b;
        ldsm_x4(b0a, b1a, b0b, b1b,
                sk + tile_offset<ROW, true>(np * 16 + (lane & 7) + ((lane >> 4) << 3),
                                            2 * ks + ((lane >> 3) & 1)));
        mma_16816(s[2 * np], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], b0a, b1a);
        mma_16816(s[2 * np + 1], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], b0b, b1b);
      }
    }
    // scale; causal and length masks on the diagonal and the last key tile
    // only (every key of a tile wholly below the diagonal and inside the
    // prompt is visible to every row); row maxima
    const bool full = j * 64 + 64 <= t0 && j * 64 + 64 <= kend;
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      if (full) {
#pragma unroll
        for (int e = 0; e < 4; ++e) s[nt][e] *= p.scale_log2;
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int key = j * 64 + nt * 8 + 2 * tg + (e & 1);
          const int qr = e < 2 ? qr0 : qr1;
          const bool ok = key <= qr && key < kend;
          s[nt][e] = ok ? s[nt][e] * p.scale_log2 : -INFINITY;
        }
      }
      mx0 = fmaxf(mx0, fmaxf(s[nt][0], s[nt][1]));
      mx1 = fmaxf(mx1, fmaxf(s[nt][2], s[nt][3]));
    }
#pragma unroll
    for (int x = 1; x < 4; x <<= 1) {
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, x));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, x));
    }
    // Every row sees key 0 in the first tile and its own position in the
    // diagonal one, so the running maxima are finite from the first tile on.
    const float n0 = fmaxf(m0, mx0), n1 = fmaxf(m1, mx1);
    const float a0 = (m0 == -INFINITY) ? 0.f : exp2f(m0 - n0);
    const float a1 = (m1 == -INFINITY) ? 0.f : exp2f(m1 - n1);
    m0 = n0;
    m1 = n1;
    l0 *= a0;
    l1 *= a1;
#pragma unroll
    for (int i = 0; i < DT; ++i) {
      o[i][0] *= a0; o[i][1] *= a0;
      o[i][2] *= a1; o[i][3] *= a1;
    }
    // exp2(-inf - m) = 0 for masked keys (m is finite from the first tile on)
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      s[nt][0] = exp2f(s[nt][0] - m0);
      s[nt][1] = exp2f(s[nt][1] - m0);
      s[nt][2] = exp2f(s[nt][2] - m1);
      s[nt][3] = exp2f(s[nt][3] - m1);
      l0 += s[nt][0] + s[nt][1];
      l1 += s[nt][2] + s[nt][3];
    }
    // O[16 x D] += P[16 x 64] V[64 x D], P as the FP16 A operand:
    // (row g, keys 0-7), (row g+8, keys 0-7), (g, 8-15), (g+8, 8-15)
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const float* c0 = s[2 * kk];
      const float* c1 = s[2 * kk + 1];
      const uint32_t p0 = pack_half2(c0[0], c0[1]), p1 = pack_half2(c0[2], c0[3]);
      const uint32_t p2 = pack_half2(c1[0], c1[1]), p3 = pack_half2(c1[2], c1[3]);
#pragma unroll
      for (int dp = 0; dp < DT / 2; ++dp) {
        uint32_t b0x, b1x, b0y, b1y;
        ldsm_x4_t(b0x, b1x, b0y, b1y,
                  sv + tile_offset<ROW, true>(kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8,
                                              2 * dp + (lane >> 4)));
        mma_16816(o[2 * dp], p0, p1, p2, p3, b0x, b1x);
        mma_16816(o[2 * dp + 1], p0, p1, p2, p3, b0y, b1y);
      }
    }
    __syncthreads();  // the stage is refilled by the next iteration's loads
  }

#pragma unroll
  for (int x = 1; x < 4; x <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, x);
    l1 += __shfl_xor_sync(0xffffffffu, l1, x);
  }
  const float i0 = 1.f / l0, i1 = 1.f / l1;
#pragma unroll
  for (int dt = 0; dt < DT; ++dt) {
    const int d = dt * 8 + 2 * tg;
    if (qr0 < n)
      *reinterpret_cast<__half2*>(obase + qr0 * row_stride + d) =
          __floats2half2_rn(o[dt][0] * i0, o[dt][1] * i0);
    if (qr1 < n)
      *reinterpret_cast<__half2*>(obase + qr1 * row_stride + d) =
          __floats2half2_rn(o[dt][2] * i1, o[dt][3] * i1);
  }
  // padding rows of a partly filled tile
  for (int i = tid; i < 64 * CH; i += 128) {
    const int row = i / CH, c = i - row * CH, t = t0 + row;
    if (t >= n && t < p.W)
      *reinterpret_cast<uint4*>(obase + t * row_stride + c * 8) = make_uint4(0, 0, 0, 0);
  }
}

}  // namespace pdb
