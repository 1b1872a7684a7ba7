// Paged causal prefill attention on the 5th-generation tensor cores
// (tcgen05 + TMEM + TMA, sm_100a, FP16).
//
// Same contract as prefill_attention_kernel (prefill.cuh; worker/llama.py:
// 141-144): left-aligned prompts of the padded batch q [B, W, H, D], K/V read
// from the paged pools through each prompt's block table, query t of prompt b
// attends to keys 0..t, rows at or beyond len_b written as zeros.
//
// One CTA per (128-query tile, query head, prompt); tiles are dispatched
// longest first over the whole batch. Six warps with fixed roles:
//   * warp 4, producer: per 64-key tile, looks up the tile's four 16-token
//     units in the block table (one lane each, range-checked) and issues one
//     3-D TMA box per (unit, K|V, 64-column half) into a ring of STAGES
//     stages; the Q tile (128 x D) comes with the first tile. All boxes use
//     the 128-byte swizzle, which is the K-major SWIZZLE_128B operand layout
//     of tcgen05.mma. A stage is refilled once the MMA that read it is done.
//   * warp 5, MMA issuer (one lane): S_j = Q K_j^T into TMEM (fp32, 64
//     columns) as soon as K_j has landed and the softmax warps have read
//     S_{j-1}; then O += P_{j-1} V_{j-1} with P taken from TMEM (the A-from-
//     tensor-memory form) and V as an MN-major shared-memory operand. Each
//     group completes on an mbarrier through tcgen05.commit.
//   * warps 0-3, softmax (thread i owns query row i = TMEM lane i): load the
//     S row (tcgen05.ld), release S for the next QK^T, mask (causal, length),
//     exponentiate in base 2 against the row's running max, write P as FP16
//     into TMEM (tcgen05.st), and rescale the O row in TMEM when the row max
//     grew by more than 2^8 (lazy rescale: P <= 256 otherwise, exact after
//     the final division by the row sum). At the end: O / l to FP16, stored;
//     rows >= len_b stored as zeros.
// TMEM: 256 columns per CTA (O, S, P), allocated after the padding-tile exit
// and freed before the single exit; shared memory and registers keep a CTA
// pair per SM, which uses all 512 columns. Every mbarrier wait is bounded
// (~2^31 cycles) and raises PDB_DEVERR_TIMEOUT instead of hanging; a thread
// whose wait expired stops waiting, so a broken launch still ends.
#pragma once

#include <cuda.h>

#include "attention_tma.cuh"

namespace pdb {

// ---- tcgen05 / TMEM primitives ---------------------------------------------
__device__ __forceinline__ void tc_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(
                   smem_u32(dst)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
}
__device__ __forceinline__ void tc_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
}
// D[tmem] (+)= A[smem desc] * B[smem desc], kind::f16, one thread issues.
__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                       uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem desc], kind::f16: A is M lanes x K halves
// packed two per 32-bit column (K-major), one thread issues.
__device__ __forceinline__ void tc_mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on `bar` when every tcgen05.mma this thread issued so far completes.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(
                   smem_u32(bar))
               : "memory");
}
// 32 consecutive 32-bit columns of this thread's TMEM lane. The registers
// are valid only after tcgen05.wait::ld: call tc_wait_ld() and then
// tc_reg_fence32() on them before any use.
__device__ __forceinline__ void tc_ld32(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}
// Compiler-level fence: uses of r[] cannot move above the preceding
// (volatile) tcgen05.wait::ld.
__device__ __forceinline__ void tc_reg_fence32(uint32_t* r) {
  asm volatile(""
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]),
                 "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]),
                 "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]),
                 "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]),
                 "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]),
                 "+r"(r[30]), "+r"(r[31]));
}
__device__ __forceinline__ void tc_st32(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,"
      "%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};\n" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
// 2^x on the MUFU (PTX ex2.approx.ftz.f32; 2^-inf = 0).
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ void tc_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
}
__device__ __forceinline__ void tc_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory");
}

// Shared-memory matrix descriptor of a SWIZZLE_128B operand (1024-byte atoms
// of 8 rows x 128 bytes): start address, leading / stride byte offsets (16-byte
// units), descriptor version 1, layout type 2 = SWIZZLE_128B.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// Instruction descriptor, kind::f16: F16 A and B, F32 accumulator, M x N,
// A / B K-major (0) or MN-major (1).
__host__ __device__ constexpr uint32_t f16_idesc(int M, int N, int a_mn, int b_mn) {
  return (1u << 4) | ((uint32_t)a_mn << 15) | ((uint32_t)b_mn << 16) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

struct PrefillTcParams {
  const int32_t* tables;   // [B, table_width]
  const int32_t* lengths;  // [B]
  __half* out;             // [B, W, H, D]
  int B, W, H, KVH, G, table_width, block_size, bs_shift;
  int64_t num_blocks;
  float scale_log2;
};

template <int D>
struct PrefillTc {
  static constexpr int BM = 128;                 // query rows per CTA (TMEM lanes)
  static constexpr int BN = 64;                  // keys per tile
  static constexpr int STAGES = D == 64 ? 4 : 2;  // K/V ring
  static constexpr int HALVES = D / 64;          // 64-column (128-byte) blocks of a row
  static constexpr int UNITS = BN / 16;          // 16-token units per tile
  static constexpr int NT = 6 * 32;
  static constexpr int Q_BYTES = BM * D * 2;
  static constexpr int KV_TILE = BN * D * 2;     // one K or V tile
  static constexpr int STAGE_BYTES = 2 * KV_TILE;
  static constexpr uint32_t TMEM_COLS = 256;
  static constexpr uint32_t O_COL = 0, S_COL = 128, P_COL = 192;
  static_assert(D <= 128 && S_COL + BN <= P_COL && P_COL + BN / 2 <= TMEM_COLS, "TMEM columns");
  static constexpr int NBARS = 2 * STAGES + 4;
  static constexpr size_t SMEM = 1024 + Q_BYTES + (size_t)STAGES * STAGE_BYTES + NBARS * 8 + 16;
};

template <int D>
__global__ void __launch_bounds__(PrefillTc<D>::NT, 2)
prefill_tc_kernel(const PrefillTcParams p, const __grid_constant__ CUtensorMap qmap,
                  const __grid_constant__ CUtensorMap kmap,
                  const __grid_constant__ CUtensorMap vmap) {
  using PT = PrefillTc<D>;
  constexpr int BM = PT::BM, BN = PT::BN, HALVES = PT::HALVES, UNITS = PT::UNITS;
  constexpr int STAGES = PT::STAGES;
  constexpr int CH = D / 8;  // 16-byte chunks of an output row
  extern __shared__ unsigned char smem_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* sq = base;
  auto sk = [&](int s) { return base + PT::Q_BYTES + (size_t)s * PT::STAGE_BYTES; };
  auto sv = [&](int s) { return sk(s) + PT::KV_TILE; };
  uint64_t* bars = reinterpret_cast<uint64_t*>(base + PT::Q_BYTES + (size_t)STAGES * PT::STAGE_BYTES);
  uint64_t* full = bars;              // [STAGES] stage landed (TMA bytes; + Q with tile 0)
  uint64_t* empty = bars + STAGES;    // [STAGES] PV that read the stage done (commit)
  uint64_t* s_full = bars + 2 * STAGES;  // S_j in TMEM (commit)
  uint64_t* s_free = s_full + 1;         // softmax warps read S_j (4 arrivals)
  uint64_t* p_full = s_full + 2;         // P_j in TMEM, O rescaled, V zeroed (4 arrivals)
  uint64_t* pv_done = s_full + 3;        // PV_j done (commit)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + PT::NBARS);

  const int hq = blockIdx.x, b = blockIdx.y;
  const int t0 = (int)(gridDim.z - 1 - blockIdx.z) * BM;  // longest tiles first
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  grid_dependency_wait();
  launch_dependents();
  int n = p.lengths[b];
  if (n < 0 || n > p.W) {
    raise_error(0x2u);
    n = n < 0 ? 0 : p.W;
  }
  const int64_t row_stride = (int64_t)p.H * D;
  __half* obase = p.out + ((int64_t)b * p.W * p.H + hq) * D;
  if (t0 >= n) {  // padding rows only: no TMEM, no barriers
    for (int i = tid; i < BM * CH; i += PT::NT) {
      const int row = i / CH, c = i - row * CH, t = t0 + row;
      if (t < p.W)
        *reinterpret_cast<uint4*>(obase + t * row_stride + c * 8) = make_uint4(0, 0, 0, 0);
    }
    return;
  }
  const int hk = hq / p.G;
  const int kend = n < t0 + BM ? n : t0 + BM;  // keys [0, kend) are seen by this tile
  const int nkt = (kend + BN - 1) / BN;

  if (tid == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(s_free, 4);
    mbar_init(p_full, 4);
    mbar_init(pv_done, 1);
    fence_barrier_init();
  }
  if (warp == 0) {
    tc_alloc(tmem_slot, PT::TMEM_COLS);
    tc_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // After one expired wait (error bit raised) a thread stops waiting.
  bool live = true;
  auto wait = [&](uint64_t* bar, uint32_t parity) {
    if (live) live = mbar_wait(bar, parity);
  };

  if (warp == 4) {
    // ---- producer ---------------------------------------------------------
    for (int j = 0; j < nkt; ++j) {
      const int s = j % STAGES;
      if (j >= STAGES) wait(&empty[s], (uint32_t)(j / STAGES - 1) & 1u);
      const int k0 = j * BN;
      bool ok = false;
      int row0 = 0;
      if (lane < UNITS) {
        const int t = k0 + lane * 16;
        if (t < kend) {
          const int pi = p.bs_shift >= 0 ? (t >> p.bs_shift) : t / p.block_size;
          const int page =
              pi < p.table_width ? __ldg(p.tables + (int64_t)b * p.table_width + pi) : -1;
          if (page < 0 || (int64_t)page >= p.num_blocks) {
            raise_error(0x1u);
          } else {
            ok = true;
            row0 = page * p.block_size + (t - pi * p.block_size);
          }
        }
      }
      const unsigned okmask = __ballot_sync(0xffffffffu, ok);
      if (lane == 0) {
        uint32_t bytes = (uint32_t)__popc(okmask) * 2u * HALVES * 16u * 128u;
        if (j == 0) bytes += (uint32_t)PT::Q_BYTES;
        mbar_arrive_expect_tx(&full[s], bytes);
        if (j == 0) {
#pragma unroll
          for (int hf = 0; hf < HALVES; ++hf)
            tma_load_3d(sq + hf * (BM * 128), &qmap, hf * 64, hq, b * p.W + t0, &full[0]);
        }
      }
      __syncwarp();
      if (ok) {
#pragma unroll
        for (int hf = 0; hf < HALVES; ++hf) {
          const int dst = hf * (BN * 128) + lane * 16 * 128;
          tma_load_3d(sk(s) + dst, &kmap, hf * 64, hk, row0, &full[s]);
          tma_load_3d(sv(s) + dst, &vmap, hf * 64, hk, row0, &full[s]);
        }
      }
    }
    // Tail: every commit to an `empty` barrier has arrived before the CTA's
    // shared memory can be handed to the next CTA.
    for (int j = nkt > STAGES ? nkt - STAGES : 0; j < nkt; ++j)
      wait(&empty[j % STAGES], (uint32_t)(j / STAGES) & 1u);
  } else if (warp == 5) {
    // ---- MMA issuer (lane 0) ----------------------------------------------
    constexpr uint32_t IDESC_S = f16_idesc(BM, BN, 0, 0);  // Q, K both K-major
    constexpr uint32_t IDESC_O = f16_idesc(BM, D, 0, 1);   // P K-major (TMEM), V MN-major
    auto issue_pv = [&](int j) {
      const int s = j % STAGES;
      wait(p_full, (uint32_t)j & 1u);
      tc_fence_after();
#pragma unroll
      for (int kk = 0; kk < BN / 16; ++kk) {
        const uint64_t bd = sw128_desc(smem_u32(sv(s) + kk * 16 * 128), BN * 128, 1024);
        tc_mma_ts(tmem + PT::O_COL, tmem + PT::P_COL + kk * 8, bd, IDESC_O,
                  (j > 0 || kk > 0) ? 1u : 0u);
      }
      tc_commit(&empty[s]);
      tc_commit(pv_done);
    };
    for (int j = 0; j < nkt; ++j) {
      if (lane == 0) {
        const int s = j % STAGES;
        wait(&full[s], (uint32_t)(j / STAGES) & 1u);
        if (j > 0) wait(s_free, (uint32_t)(j - 1) & 1u);
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const int hf = kk >> 2, off = (kk & 3) * 32;
          const uint64_t ad = sw128_desc(smem_u32(sq + hf * (BM * 128) + off), 16, 1024);
          const uint64_t bd = sw128_desc(smem_u32(sk(s) + hf * (BN * 128) + off), 16, 1024);
          tc_mma(tmem + PT::S_COL, ad, bd, IDESC_S, kk > 0);
        }
        tc_commit(s_full);
        if (j > 0) issue_pv(j - 1);
      }
      __syncwarp();
    }
    if (lane == 0) issue_pv(nkt - 1);
    __syncwarp();
  } else {
    // ---- softmax warps: thread tid owns query row t0 + tid ------------------
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    const int qr = t0 + tid;
    const float c = p.scale_log2;
    float m_used = -INFINITY, l = 0.f;
    for (int j = 0; j < nkt; ++j) {
      wait(s_full, (uint32_t)j & 1u);
      tc_fence_after();
      uint32_t sraw[BN];
      tc_ld32(tmem + lane_base + PT::S_COL, sraw);
      tc_ld32(tmem + lane_base + PT::S_COL + 32, sraw + 32);
      tc_wait_ld();
      tc_reg_fence32(sraw);
      tc_reg_fence32(sraw + 32);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(s_free);  // S may be overwritten by the next QK^T
      float sc[BN];
#pragma unroll
      for (int i = 0; i < BN; ++i) sc[i] = __uint_as_float(sraw[i]);
      const int k0 = j * BN;
      if (k0 + BN > t0 || k0 + BN > kend) {  // diagonal or last tile: mask
        const int lim = qr + 1 < kend ? qr + 1 : kend;  // keys [0, lim) are visible
#pragma unroll
        for (int i = 0; i < BN; ++i)
          if (k0 + i >= lim) sc[i] = -INFINITY;
      }
      float mx = sc[0];
#pragma unroll
      for (int i = 1; i < BN; ++i) mx = fmaxf(mx, sc[i]);
      const float mt = mx * c;  // this tile's row max, log2 units
      float alpha = 1.f;
      if (mt > m_used + 8.f) {  // lazy rescale (always on the first tile)
        alpha = ex2(m_used - mt);
        m_used = mt;
      }
      uint32_t pk[BN / 2];
      float rs = 0.f;
#pragma unroll
      for (int i = 0; i < BN / 2; ++i) {
        const float a = ex2(fmaf(sc[2 * i], c, -m_used));
        const float bb = ex2(fmaf(sc[2 * i + 1], c, -m_used));
        rs += a + bb;
        pk[i] = pack_half2(a, bb);
      }
      l = l * alpha + rs;
      // V rows of keys >= kend in the last tile: zero them (stale pool bytes
      // must not meet a zero P; 0 * NaN would poison the row)
      const int vis = kend - k0;
      if (vis < BN) {
        const int s = j % STAGES;
        wait(&full[s], (uint32_t)(j / STAGES) & 1u);
        for (int i = tid; i < (BN - vis) * HALVES * 8; i += 128) {
          const int r = vis + i / (HALVES * 8), cc = i % (HALVES * 8);
          const int hf = cc >> 3, c8 = cc & 7;
          *reinterpret_cast<uint4*>(sv(s) + hf * (BN * 128) + r * 128 + ((c8 ^ (r & 7)) << 4)) =
              make_uint4(0, 0, 0, 0);
        }
        fence_proxy_async_smem();
      }
      // PV_{j-1} must be done before P and O are touched
      if (j > 0) {
        wait(pv_done, (uint32_t)(j - 1) & 1u);
        tc_fence_after();
        if (__any_sync(0xffffffffu, alpha != 1.f)) {
          uint32_t ov[32];
#pragma unroll
          for (int cc = 0; cc < D / 32; ++cc) {
            tc_ld32(tmem + lane_base + PT::O_COL + cc * 32, ov);
            tc_wait_ld();
            tc_reg_fence32(ov);
#pragma unroll
            for (int i = 0; i < 32; ++i) ov[i] = __float_as_uint(__uint_as_float(ov[i]) * alpha);
            tc_st32(tmem + lane_base + PT::O_COL + cc * 32, ov);
          }
        }
      }
      tc_st32(tmem + lane_base + PT::P_COL, pk);
      tc_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
    }
    // epilogue: O row / l
    wait(pv_done, (uint32_t)(nkt - 1) & 1u);
    tc_fence_after();
    const float inv = 1.f / l;
#pragma unroll
    for (int cc = 0; cc < D / 32; ++cc) {
      uint32_t ov[32];
      tc_ld32(tmem + lane_base + PT::O_COL + cc * 32, ov);
      tc_wait_ld();
      tc_reg_fence32(ov);
      if (qr < n) {
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          uint32_t w[4];
#pragma unroll
          for (int e = 0; e < 4; ++e)
            w[e] = pack_half2(__uint_as_float(ov[q4 * 8 + 2 * e]) * inv,
                              __uint_as_float(ov[q4 * 8 + 2 * e + 1]) * inv);
          *reinterpret_cast<uint4*>(obase + qr * row_stride + cc * 32 + q4 * 8) =
              make_uint4(w[0], w[1], w[2], w[3]);
        }
      } else if (qr < p.W) {
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4)
          *reinterpret_cast<uint4*>(obase + qr * row_stride + cc * 32 + q4 * 8) =
              make_uint4(0, 0, 0, 0);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tc_dealloc(tmem, PT::TMEM_COLS);
  }
}

}  // namespace pdb
