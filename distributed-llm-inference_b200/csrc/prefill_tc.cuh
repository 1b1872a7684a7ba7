// Paged causal prefill attention on the 5th-generation tensor cores
// (tcgen05 + TMEM + TMA, sm_100a, FP16).
//
// Same contract as prefill_attention_kernel (prefill.cuh; worker/llama.py:
// 141-144): left-aligned prompts of the padded batch q [B, W, H, D], K/V read
// from the paged pools through each prompt's block table, query t of prompt b
// attends to keys 0..t, rows at or beyond len_b written as zeros.
//
// Persistent: one CTA pair per SM; each CTA walks a list of items (a 128-row
// query tile of one query head of one prompt), dealt back and forth over the
// items ordered by cost. TMEM, barriers and the pipelines below carry over
// from item to item. Six warps with fixed roles:
//   * warp 4, producer: computes the CTA's items from the lengths (warp
//     ballots) and hands them to the other warps through a small queue of
//     records; per 64-key tile it looks up the tile's four 16-token units in
//     the block table (one lane each, range-checked) and issues one 3-D TMA
//     box per (unit, K|V, 64-column half) into a ring of STAGES stages. An
//     item's Q tile (128 x D; double-buffered for head_dim 64) rides on its
//     first tile's barrier. All boxes use the 128-byte swizzle, which is the
//     K-major SWIZZLE_128B operand layout of tcgen05.mma. A stage is refilled
//     once the MMA that read it is done.
//   * warp 5, MMA issuer (warp-uniform; one elected lane issues): S_g = Q K_g^T
//     into TMEM (fp32, 64 columns) as soon as K_g has landed and the softmax
//     warps have read S_{g-1}; then O += P_{g-1} V_{g-1} with P taken from
//     TMEM (the A-from-tensor-memory form) and V as an MN-major shared-memory
//     operand. Each group completes on an mbarrier through tcgen05.commit.
//   * warps 0-3, softmax (thread i owns query row t0 + i = TMEM lane i): load
//     the S row (tcgen05.ld), release S for the next QK^T, mask (causal,
//     length), exponentiate in base 2 against the row's running max, write P
//     as FP16 into one of two TMEM buffers (tcgen05.st; the PV of two tiles
//     back read it), and rescale the O row in TMEM when the row max grew by
//     more than 2^8 (lazy rescale: P <= 256 otherwise, exact after the final
//     division by the row sum). At an item's end: O / l to FP16, stored; rows
//     >= len_b stored as zeros (padding-only items are zeros throughout).
// TMEM: 256 columns per CTA (O, S, P), allocated once and freed before the
// single exit; shared memory and registers keep a CTA pair per SM, which uses
// all 512 columns. Every mbarrier wait is bounded (~2^31 cycles) and raises
// PDB_DEVERR_TIMEOUT instead of hanging; a thread whose wait expired stops
// waiting, so a broken launch still ends.
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
// Warp-collective forms: the whole (converged) warp executes them with
// warp-uniform operands and one elected lane issues, so the operands stay in
// uniform registers (a lane-divergent issue is markedly slower per group).
__device__ __forceinline__ void tc_mma_elect(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                             uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p, e;\n setp.ne.b32 p, %4, 0;\n elect.sync _|e, 0xffffffff;\n"
      " @e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void tc_mma_ts_elect(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                                uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p, e;\n setp.ne.b32 p, %4, 0;\n elect.sync _|e, 0xffffffff;\n"
      " @e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// The elected lane (the same lowest lane as in tc_mma_elect) commits.
__device__ __forceinline__ void tc_commit_elect(uint64_t* bar) {
  asm volatile(
      "{\n .reg .pred e;\n elect.sync _|e, 0xffffffff;\n"
      " @e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n}\n" ::"r"(
          smem_u32(bar))
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
// Adds `bytes` to the barrier's expected transaction count without arriving.
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;\n" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
// 2^x on the MUFU (PTX ex2.approx.ftz.f32; 2^-inf = 0).
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
  return y;
}
// Packed FP32 pairs (sm_100 f32x2 arithmetic: one instruction, two lanes).
__device__ __forceinline__ uint64_t f2(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};\n" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void f2_split(uint64_t v, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;\n" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;\n" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ uint64_t fadd2(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;\n" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;\n" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
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
  int TZ;                  // 128-row query tiles per prompt: ceil(W / 128)
  int64_t num_blocks;
  float scale_log2;
};

// One item of the persistent schedule: a 128-row query tile of one query
// head of one prompt.
struct PrefillItem {
  int b, hq, t0, n;  // prompt, query head, first row, prompt length (clamped)
  int kind;          // kItemWork, kItemPadding (rows >= n only) or kItemEnd
  int pad_[3];
};
constexpr int kItemWork = 0, kItemPadding = 1, kItemEnd = 2;

template <int D>
struct PrefillTc {
  static constexpr int BM = 128;                 // query rows per item (TMEM lanes)
  static constexpr int BN = 64;                  // keys per tile
  static constexpr int STAGES = D == 64 ? 4 : 2;  // K/V ring
  static constexpr int QBUF = D == 64 ? 2 : 1;   // Q tiles in flight
  static constexpr int IQ = 4;                   // item records in flight
  static constexpr int HALVES = D / 64;          // 64-column (128-byte) blocks of a row
  static constexpr int UNITS = BN / 16;          // 16-token units per tile
  static constexpr int NT = 6 * 32;
  static constexpr int Q_BYTES = BM * D * 2;
  static constexpr int KV_TILE = BN * D * 2;     // one K or V tile
  static constexpr int STAGE_BYTES = 2 * KV_TILE;
  static constexpr uint32_t TMEM_COLS = 256;
  // O (D fp32 columns), S (BN fp32), P double-buffered (BN halves = BN/2 columns each)
  static constexpr uint32_t O_COL = 0, S_COL = 128, P_COL = 192;
  static_assert(D <= 128 && S_COL + BN <= P_COL && P_COL + BN <= TMEM_COLS, "TMEM columns");
  static constexpr int NBARS = 2 * STAGES + QBUF + 6 + 2 * IQ;
  static constexpr int LCAP = 512;  // prompt lengths kept in shared memory (more: read from global)
  // Output staging: per softmax warp 32 rows x 32 columns of FP16 (2 KB).
  static constexpr int OUT_STAGE = 32 * 64;
  static constexpr size_t SMEM = 1024 + (size_t)QBUF * Q_BYTES + (size_t)STAGES * STAGE_BYTES +
                                 NBARS * 8 + 16 + IQ * sizeof(PrefillItem) + LCAP * 4 + 16 +
                                 4 * OUT_STAGE;
};

// Walks the global item order: first every working tile, level by level
// from the last 128-row tile of the longest prompts down to the first
// (levels are in decreasing cost: a tile at level z sees up to 128 (z + 1)
// keys), then every padding-only tile. Within a level: prompts in index
// order, query heads inner. Ranks are visited in increasing order, so the
// walk only moves forward. Executed by one whole warp (ballots over prompts).
struct PrefillWalk {
  int phase;        // 0 working tiles, 1 padding tiles
  int level;        // tile index z within a prompt (t0 = 128 z)
  long long start;  // rank of the first item of (phase, level)
  long long cnt;    // items of (phase, level)
};

// Prompt b's length, clamped to [0, W] (out-of-range lengths raise an error
// bit); `lens` caches the first LCAP clamped lengths in shared memory.
__device__ __forceinline__ int prefill_len_global(const PrefillTcParams& p, int b) {
  int n = __ldg(p.lengths + b);
  if (n < 0 || n > p.W) {
    raise_error(0x2u);
    n = n < 0 ? 0 : p.W;
  }
  return n;
}
template <int LCAP>
__device__ __forceinline__ int prefill_len(const PrefillTcParams& p, const int* lens, int b) {
  return b < LCAP ? lens[b] : prefill_len_global(p, b);
}
// Prompt b is in (phase, level) when its tile `level` has rows < n (phase 0)
// or none (phase 1).
template <int LCAP>
__device__ __forceinline__ bool prefill_in_level(const PrefillTcParams& p, const int* lens, int b,
                                                 int phase, int level) {
  const int tiles = (prefill_len<LCAP>(p, lens, b) + 127) >> 7;
  return phase == 0 ? tiles > level : tiles <= level;
}
template <int LCAP>
__device__ __forceinline__ long long prefill_level_items(const PrefillTcParams& p, const int* lens,
                                                         int phase, int level, int lane) {
  long long c = 0;
  for (int b0 = 0; b0 < p.B; b0 += 32) {
    const int b = b0 + lane;
    c += __popc(__ballot_sync(0xffffffffu,
                              b < p.B && prefill_in_level<LCAP>(p, lens, b, phase, level)));
  }
  return c * p.H;
}
// The j-th prompt (in index order) of (phase, level).
template <int LCAP>
__device__ __forceinline__ int prefill_level_prompt(const PrefillTcParams& p, const int* lens,
                                                    int phase, int level, long long j, int lane) {
  for (int b0 = 0; b0 < p.B; b0 += 32) {
    const int b = b0 + lane;
    const unsigned m = __ballot_sync(
        0xffffffffu, b < p.B && prefill_in_level<LCAP>(p, lens, b, phase, level));
    const int c = __popc(m);
    if (j < c) return b0 + (int)__fns(m, 0, (int)j + 1);
    j -= c;
  }
  return 0;  // unreachable for j < level count
}

// Persistent grid: CTA c processes the items of ranks k = r G + c (r even)
// or r G + G - 1 - c (r odd), r = 0, 1, ... (a back-and-forth deal over the
// cost-ordered list, which balances the CTAs without global state).
template <int D>
__global__ void __launch_bounds__(PrefillTc<D>::NT, 2)
prefill_tc_kernel(const PrefillTcParams p, const __grid_constant__ CUtensorMap qmap,
                  const __grid_constant__ CUtensorMap kmap,
                  const __grid_constant__ CUtensorMap vmap) {
  using PT = PrefillTc<D>;
  constexpr int BM = PT::BM, BN = PT::BN, HALVES = PT::HALVES, UNITS = PT::UNITS;
  constexpr int STAGES = PT::STAGES, QBUF = PT::QBUF, IQ = PT::IQ;
  constexpr int CH = D / 8;  // 16-byte chunks of an output row
  extern __shared__ unsigned char smem_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  auto sq = [&](int qb) { return base + (size_t)qb * PT::Q_BYTES; };
  auto sk = [&](int s) { return base + QBUF * PT::Q_BYTES + (size_t)s * PT::STAGE_BYTES; };
  auto sv = [&](int s) { return sk(s) + PT::KV_TILE; };
  uint64_t* bars = reinterpret_cast<uint64_t*>(base + QBUF * PT::Q_BYTES +
                                               (size_t)STAGES * PT::STAGE_BYTES);
  // Tiles are numbered g = 0, 1, ... over all items of this CTA; stage, P
  // buffer and every barrier phase below follow g (or the item count w).
  uint64_t* full = bars;              // [STAGES] stage landed (TMA bytes; + Q with an item's first tile)
  uint64_t* empty = bars + STAGES;    // [STAGES] PV that read the stage done (commit)
  uint64_t* q_free = bars + 2 * STAGES;  // [QBUF] last QK^T of item w done (commit)
  uint64_t* s_full = q_free + QBUF;      // S_g in TMEM (commit)
  uint64_t* s_free = s_full + 1;         // softmax warps read S_g (4 arrivals)
  // [2] P_g in TMEM buffer g & 1, O rescaled, V zeroed (4 arrivals on p_full[g & 1]).
  // One barrier per buffer: a warp may reach tile g + 1 before another warp
  // finished tile g, but not tile g + 2 (S_{g+2} is issued after PV_g).
  uint64_t* p_full = s_full + 2;
  uint64_t* pv_done = s_full + 4;        // [2] PV_g done (commit to pv_done[g & 1])
  uint64_t* item_full = s_full + 6;      // [IQ] item record written (1 arrival)
  uint64_t* item_empty = item_full + IQ;  // [IQ] record read by the MMA warp + 4 softmax warps
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + PT::NBARS);
  PrefillItem* items = reinterpret_cast<PrefillItem*>(tmem_slot + 4);
  int* lens = reinterpret_cast<int*>(items + IQ);  // [LCAP] clamped prompt lengths (producer)
  unsigned char* out_stage = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(lens + PT::LCAP) + 15) & ~uintptr_t(15));  // [4][OUT_STAGE]

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < QBUF; ++i) mbar_init(&q_free[i], 1);
    mbar_init(s_full, 1);
    mbar_init(s_free, 4);
    mbar_init(&p_full[0], 4);
    mbar_init(&p_full[1], 4);
    mbar_init(&pv_done[0], 1);
    mbar_init(&pv_done[1], 1);
    for (int i = 0; i < IQ; ++i) {
      mbar_init(&item_full[i], 1);
      mbar_init(&item_empty[i], 5);
    }
    fence_barrier_init();
  }
  // Every global access, and the TMEM allocation (a previous kernel still
  // running on this SM may hold TMEM), come after this wait.
  grid_dependency_wait();
  launch_dependents();
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
  // Item record q of the queue, read by a consumer warp (which then frees it).
  auto take_item = [&](int q) -> PrefillItem {
    wait(&item_full[q % IQ], (uint32_t)(q / IQ) & 1u);
    const PrefillItem it = items[q % IQ];
    __syncwarp();
    if (lane == 0) mbar_arrive(&item_empty[q % IQ]);
    return it;
  };

  if (warp == 4) {
    // ---- producer: schedule, block-table lookups, TMA -----------------------
    constexpr int LCAP = PT::LCAP;
    for (int b = lane; b < p.B && b < LCAP; b += 32) lens[b] = prefill_len_global(p, b);
    __syncwarp();
    const long long NI = (long long)p.H * p.B * p.TZ;
    const int G = (int)gridDim.x, c = (int)blockIdx.x;
    PrefillWalk wk{0, p.TZ - 1, 0, prefill_level_items<LCAP>(p, lens, 0, p.TZ - 1, lane)};
    int q = 0, w = 0;
    long long g = 0;
    for (long long r = 0;; ++r) {
      const long long k = r * G + ((r & 1) ? G - 1 - c : c);
      PrefillItem it{};
      if (k >= NI) {
        it.kind = kItemEnd;
      } else {
        while (k >= wk.start + wk.cnt) {
          wk.start += wk.cnt;
          if (wk.level > 0) {
            --wk.level;
          } else {
            ++wk.phase;
            wk.level = p.TZ - 1;
          }
          wk.cnt = prefill_level_items<LCAP>(p, lens, wk.phase, wk.level, lane);
        }
        const long long i = k - wk.start;
        it.b = prefill_level_prompt<LCAP>(p, lens, wk.phase, wk.level, i / p.H, lane);
        it.hq = (int)(i % p.H);
        it.t0 = wk.level * BM;
        it.n = prefill_len<LCAP>(p, lens, it.b);
        it.kind = wk.phase == 0 ? kItemWork : kItemPadding;
      }
      if (q >= IQ) wait(&item_empty[q % IQ], (uint32_t)(q / IQ - 1) & 1u);
      if (lane == 0) {
        items[q % IQ] = it;
        mbar_arrive(&item_full[q % IQ]);
      }
      ++q;
      __syncwarp();
      if (it.kind == kItemEnd) break;
      if (it.kind != kItemWork) continue;
      const int kend = it.n < it.t0 + BM ? it.n : it.t0 + BM;
      const int nkt = (kend + BN - 1) / BN;
      const int hk = it.hq / p.G;
      const int qb = w % QBUF;
      if (w >= QBUF) wait(&q_free[qb], (uint32_t)(w / QBUF - 1) & 1u);
      for (int j = 0; j < nkt; ++j, ++g) {
        const int s = (int)(g % STAGES);
        if (g >= STAGES) wait(&empty[s], (uint32_t)(g / STAGES - 1) & 1u);
        const int k0 = j * BN;
        bool ok = false;
        int row0 = 0;
        if (lane < UNITS) {
          const int t = k0 + lane * 16;
          if (t < kend) {
            const int pi = p.bs_shift >= 0 ? (t >> p.bs_shift) : t / p.block_size;
            const int page =
                pi < p.table_width ? __ldg(p.tables + (int64_t)it.b * p.table_width + pi) : -1;
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
          if (j == 0) {  // the item's Q tile lands on its first tile's barrier
            mbar_expect_tx(&full[s], (uint32_t)PT::Q_BYTES);
#pragma unroll
            for (int hf = 0; hf < HALVES; ++hf)
              tma_load_3d(sq(qb) + hf * (BM * 128), &qmap, hf * 64, it.hq, it.b * p.W + it.t0,
                          &full[s]);
          }
          mbar_arrive_expect_tx(&full[s], (uint32_t)__popc(okmask) * 2u * HALVES * 16u * 128u);
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
      ++w;
    }
    // Tail: every commit to an `empty` or `q_free` barrier has arrived before
    // the CTA's shared memory can be handed to another CTA.
    for (long long gg = g > STAGES ? g - STAGES : 0; gg < g; ++gg)
      wait(&empty[gg % STAGES], (uint32_t)(gg / STAGES) & 1u);
    for (int ww = w > QBUF ? w - QBUF : 0; ww < w; ++ww)
      wait(&q_free[ww % QBUF], (uint32_t)(ww / QBUF) & 1u);
  } else if (warp == 5) {
    // ---- MMA issuer: the whole warp runs the loop, one elected lane issues --
    constexpr uint32_t IDESC_S = f16_idesc(BM, BN, 0, 0);  // Q, K both K-major
    constexpr uint32_t IDESC_O = f16_idesc(BM, D, 0, 1);   // P K-major (TMEM), V MN-major
    // Descriptor start addresses advance in 16-byte units.
    const uint64_t q_desc = sw128_desc(smem_u32(sq(0)), 16, 1024);
    const uint64_t k_desc = sw128_desc(smem_u32(sk(0)), 16, 1024);
    const uint64_t v_desc = sw128_desc(smem_u32(sv(0)), BN * 128, 1024);
    constexpr uint64_t STAGE_STEP = PT::STAGE_BYTES >> 4, Q_STEP = PT::Q_BYTES >> 4;
    // PV of tile gg: O (+)= P_gg V_gg; `first` = the item's first tile.
    auto issue_pv = [&](long long gg, bool first) {
      const int s = (int)(gg % STAGES);
      const int pb = (int)(gg & 1);
      wait(&p_full[pb], (uint32_t)(gg >> 1) & 1u);
      __syncwarp();
      tc_fence_after();
#pragma unroll
      for (int kk = 0; kk < BN / 16; ++kk)
        tc_mma_ts_elect(tmem + PT::O_COL, tmem + PT::P_COL + pb * (BN / 2) + kk * 8,
                        v_desc + s * STAGE_STEP + kk * (16 * 128 >> 4), IDESC_O,
                        (!first || kk > 0) ? 1u : 0u);
      tc_commit_elect(&empty[s]);
      tc_commit_elect(&pv_done[pb]);
    };
    // Order per item: S_0, S_1, PV_0, S_2, PV_1, ..., S_last, PV_last-1, then
    // PV_last before the next record is taken: the item's epilogue never
    // waits on a later item (whose loads may wait on this item's records).
    long long g = 0;
    int w = 0;
    for (int q = 0;; ++q) {
      const PrefillItem it = take_item(q);
      if (it.kind == kItemEnd) break;
      if (it.kind != kItemWork) continue;
      const int kend = it.n < it.t0 + BM ? it.n : it.t0 + BM;
      const int nkt = (kend + BN - 1) / BN;
      const int qb = w % QBUF;
      for (int j = 0; j < nkt; ++j, ++g) {
        const int s = (int)(g % STAGES);
        wait(&full[s], (uint32_t)(g / STAGES) & 1u);
        if (g > 0) wait(s_free, (uint32_t)(g - 1) & 1u);
        __syncwarp();
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint64_t off = (uint64_t)((kk >> 2) * (BM * 128) + (kk & 3) * 32) >> 4;
          const uint64_t koff = (uint64_t)((kk >> 2) * (BN * 128) + (kk & 3) * 32) >> 4;
          tc_mma_elect(tmem + PT::S_COL, q_desc + qb * Q_STEP + off,
                       k_desc + s * STAGE_STEP + koff, IDESC_S, kk > 0 ? 1u : 0u);
        }
        tc_commit_elect(s_full);
        if (j == nkt - 1) tc_commit_elect(&q_free[qb]);
        if (j > 0) issue_pv(g - 1, j == 1);
      }
      issue_pv(g - 1, nkt == 1);
      ++w;
    }
    __syncwarp();
  } else {
    // ---- softmax warps: thread tid owns query row t0 + tid ------------------
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    const float c = p.scale_log2;
    long long g = 0;
    for (int q = 0;; ++q) {
      const PrefillItem it = take_item(q);
      if (it.kind == kItemEnd) break;
      const int qr = it.t0 + tid;
      if (it.kind != kItemWork) {  // rows >= n: zeros, whole rows per warp store
#pragma unroll
        for (int k = 0; k < CH; ++k) {  // this warp's 32 rows x CH 16-byte chunks
          const int qi = k * 32 + lane;
          const int row = it.t0 + warp * 32 + qi / CH;
          if (row < p.W)
            reinterpret_cast<uint4*>(p.out + (((int64_t)it.b * p.W + row) * p.H + it.hq) * D)
                [qi % CH] = make_uint4(0, 0, 0, 0);
        }
        continue;
      }
      const int n = it.n;
      const int kend = n < it.t0 + BM ? n : it.t0 + BM;  // keys [0, kend) are seen by this item
      const int nkt = (kend + BN - 1) / BN;
      float m_used = -INFINITY, l = 0.f;
      for (int j = 0; j < nkt; ++j, ++g) {
        wait(s_full, (uint32_t)g & 1u);
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
        if (k0 + BN > it.t0 || k0 + BN > kend) {  // diagonal or last tile: mask
          const int lim = qr + 1 < kend ? qr + 1 : kend;  // keys [0, lim) are visible
          if (k0 + BN > lim) {  // rows that see the whole tile skip the selects
#pragma unroll
            for (int i = 0; i < BN; ++i)
              if (k0 + i >= lim) sc[i] = -INFINITY;
          }
        }
        static_assert(BN == 64, "the max and exponent loops below are written for 64 keys");
        float mx8[8];  // independent chains of three-input max
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          mx8[i] = fmax3(sc[i], sc[i + 8], sc[i + 16]);
          mx8[i] = fmax3(mx8[i], sc[i + 24], sc[i + 32]);
          mx8[i] = fmax3(mx8[i], sc[i + 40], sc[i + 48]);
          mx8[i] = fmaxf(mx8[i], sc[i + 56]);
        }
        const float mx = fmax3(fmax3(mx8[0], mx8[1], mx8[2]), fmax3(mx8[3], mx8[4], mx8[5]),
                               fmaxf(mx8[6], mx8[7]));
        const float mt = mx * c;  // this tile's row max, log2 units
        float alpha = 1.f;
        if (mt > m_used + 8.f) {  // lazy rescale (always on the first tile)
          alpha = ex2(m_used - mt);
          m_used = mt;
        }
        uint32_t pk[BN / 2];
        const uint64_t c2 = f2(c, c), nm2 = f2(-m_used, -m_used);
        uint64_t acc[4] = {0ull, 0ull, 0ull, 0ull};  // row-sum pairs (0.f bits are 0)
#pragma unroll
        for (int i = 0; i < BN / 2; ++i) {
          float y0, y1;
          f2_split(ffma2(f2(sc[2 * i], sc[2 * i + 1]), c2, nm2), y0, y1);
          const float a = ex2(y0), bb = ex2(y1);
          acc[i & 3] = fadd2(acc[i & 3], f2(a, bb));
          pk[i] = pack_half2(a, bb);
        }
        float r8[8];
#pragma unroll
        for (int i = 0; i < 4; ++i) f2_split(acc[i], r8[2 * i], r8[2 * i + 1]);
        const float rs =
            ((r8[0] + r8[1]) + (r8[2] + r8[3])) + ((r8[4] + r8[5]) + (r8[6] + r8[7]));
        l = l * alpha + rs;
        // V rows of keys >= kend in the item's last tile: zero them (stale
        // pool bytes must not meet a zero P; 0 * NaN would poison the row)
        const int vis = kend - k0;
        if (vis < BN) {
          const int s = (int)(g % STAGES);
          wait(&full[s], (uint32_t)(g / STAGES) & 1u);
          for (int i = tid; i < (BN - vis) * HALVES * 8; i += 128) {
            const int r = vis + i / (HALVES * 8), cc = i % (HALVES * 8);
            const int hf = cc >> 3, c8 = cc & 7;
            *reinterpret_cast<uint4*>(sv(s) + hf * (BN * 128) + r * 128 + ((c8 ^ (r & 7)) << 4)) =
                make_uint4(0, 0, 0, 0);
          }
          fence_proxy_async_smem();
        }
        // P_g goes to buffer g & 1, last read by PV_{g-2} (possibly of the
        // previous item); an O rescale needs PV_{g-1} of this item.
        const bool rescale = j > 0 && __any_sync(0xffffffffu, alpha != 1.f);
        if (rescale)
          wait(&pv_done[(g - 1) & 1], (uint32_t)((g - 1) >> 1) & 1u);
        else if (g > 1)
          wait(&pv_done[g & 1], (uint32_t)((g - 2) >> 1) & 1u);
        tc_fence_after();
        if (rescale) {
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
        tc_st32(tmem + lane_base + PT::P_COL + (int)(g & 1) * (BN / 2), pk);
        tc_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[g & 1]);
      }
      // epilogue: O row / l (PV of the item's last tile, g - 1)
      wait(&pv_done[(g - 1) & 1], (uint32_t)((g - 1) >> 1) & 1u);
      tc_fence_after();
      const float inv = 1.f / l;
      // 32 columns at a time through this warp's staging buffer, so that
      // one store instruction writes 8 rows x 64 contiguous bytes instead of
      // 16 bytes of 32 rows (rows are H * D * 2 bytes apart). Row r's
      // 16-byte chunk ch sits at r * 64 + ((ch ^ ((r >> 1) & 3)) << 4): the
      // writes (a row per lane) and the reads (4 lanes per row) are both
      // free of bank conflicts.
      unsigned char* stg = out_stage + warp * PT::OUT_STAGE;
#pragma unroll
      for (int cc = 0; cc < D / 32; ++cc) {
        uint32_t ov[32];
        tc_ld32(tmem + lane_base + PT::O_COL + cc * 32, ov);
        tc_wait_ld();
        tc_reg_fence32(ov);
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          uint4 o = make_uint4(0, 0, 0, 0);  // rows >= n: zeros
          if (qr < n) {
            uint32_t wv[4];
#pragma unroll
            for (int e = 0; e < 4; ++e)
              wv[e] = pack_half2(__uint_as_float(ov[q4 * 8 + 2 * e]) * inv,
                                 __uint_as_float(ov[q4 * 8 + 2 * e + 1]) * inv);
            o = make_uint4(wv[0], wv[1], wv[2], wv[3]);
          }
          *reinterpret_cast<uint4*>(stg + lane * 64 + ((q4 ^ ((lane >> 1) & 3)) << 4)) = o;
        }
        __syncwarp();
#pragma unroll
        for (int k4 = 0; k4 < 4; ++k4) {
          const int r = k4 * 8 + (lane >> 2), ch = lane & 3;
          const int row = it.t0 + warp * 32 + r;  // rows >= W belong to no prompt: not written
          if (row < p.W) {
            const uint4 o = *reinterpret_cast<const uint4*>(stg + r * 64 + ((ch ^ ((r >> 1) & 3)) << 4));
            *reinterpret_cast<uint4*>(p.out + (((int64_t)it.b * p.W + row) * p.H + it.hq) * D +
                                      cc * 32 + ch * 8) = o;
          }
        }
        __syncwarp();  // the buffer is rewritten for the next 32 columns
      }
      // The O reads are complete (tcgen05.wait::ld) before this warp's next
      // p_full arrival, which is what lets the next item's first PV overwrite O.
      tc_fence_before();
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
