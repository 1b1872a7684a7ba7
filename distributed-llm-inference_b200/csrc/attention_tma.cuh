// Stream-K paged decode attention with a TMA producer warp (sm_100a, FP16).
//
// Same work partition, math (MmaMath, tensor cores) and piece combining as
// attn_streamk_kernel in attention.cuh; what changes is how K/V reach shared
// memory:
//   * warp 4 of each CTA is the producer. Per 64-token tile it looks up the
//     tile's 16-token units in the block table (one lane per unit) and issues
//     one 3-D cp.async.bulk.tensor box per (unit, K|V, 64-column half):
//     box {64 columns, 1 kv head, 16 rows} of the pool viewed as
//     [num_blocks*block_size rows, kv_heads, head_dim], 128-byte swizzle, so
//     ldmatrix reads the staged tile without bank conflicts. Completion is
//     counted in bytes on the stage's "full" mbarrier.
//   * warps 0-3 are consumers: wait on "full", run the tensor-core math,
//     release the stage on its "empty" mbarrier. They never compute an
//     address or wait on a table lookup, and the producer runs up to STAGES
//     tiles ahead.
// The boxes cover whole 16-token units, so rows past a sequence's length are
// staged too (stale pool rows); the consumer warp whose rows straddle the
// length zeroes those V rows before reading them, so stale bytes (even NaN)
// never reach the output, as in the reference where reads stop at len.
// Requires block_size % 16 == 0 (a unit never straddles two pages).
// Every mbarrier wait is bounded (~1 s); on expiry the waiting thread sets
// PDB_DEVERR_TIMEOUT and proceeds, so a kernel never hangs.
#pragma once

#include <cuda.h>

#include "attention.cuh"

namespace pdb {

constexpr unsigned kErrTimeout = 0x10u;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Wait for phase `parity` of `bar` to complete, for at most ~2^31 SM cycles
// (about a second). Returns false (and raises PDB_DEVERR_TIMEOUT) on expiry.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > (1ll << 31)) {
      raise_error(kErrTimeout);
      return false;
    }
  }
  return true;
}
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
}
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];\n" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}
// 1-D bulk copy global -> shared memory of this CTA (both addresses 16-byte
// aligned, `bytes` a multiple of 16), completion counted in bytes on `bar`.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n"
      ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes),
      "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void named_bar_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;\n" ::"r"(id), "r"(threads) : "memory");
}

template <class M>
struct TmaStreamK {
  static_assert(M::LAYOUT == kTma128B, "TMA kernel needs the 128-byte swizzle layout");
  static constexpr int D = M::D, GP = M::GP, NW = M::NW, STAGES = M::STAGES;
  static constexpr int NT = (NW + 1) * 32;         // + producer warp
  static constexpr int HALVES = D / 64;            // 64-column TMA boxes per row
  static constexpr int UNIT_BYTES = 2 * kUnitTokens * D * 2;  // K + V of one unit
  static constexpr int MERGE_FLOATS = NW * GP * (D + 2);
  static size_t smem_bytes(int B) {
    return 1024 /* alignment slack */ + (size_t)STAGES * M::STAGE_BYTES +
           (size_t)MERGE_FLOATS * 4 + (size_t)(2 * B + 1 + 16) * 4 + 2 * STAGES * 8 + 16;
  }
};

template <class M>
__global__ void __launch_bounds__(TmaStreamK<M>::NT)
attn_tma_kernel(const AttnParams p, const __grid_constant__ CUtensorMap kmap,
                const __grid_constant__ CUtensorMap vmap) {
  using T = typename M::T;
  using K = TmaStreamK<M>;
  constexpr int D = M::D, GP = M::GP, NW = M::NW, STAGES = M::STAGES, NT = K::NT;
  constexpr int TILE = M::TILE;

  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* ms = reinterpret_cast<float*>(smem + (size_t)STAGES * M::STAGE_BYTES);  // [NW][GP]
  float* ls = ms + NW * GP;
  float* accs = ls + NW * GP;                            // [NW][GP][D]
  int* P = reinterpret_cast<int*>(accs + NW * GP * D);   // [B+1]
  int* Ls = P + p.B + 1;                                 // [B]
  int* misc = Ls + p.B;                                  // [16]
  uint64_t* bars = reinterpret_cast<uint64_t*>(
      (reinterpret_cast<uintptr_t>(misc + 16) + 7) & ~uintptr_t(7));
  uint64_t* full = bars;            // [STAGES], 1 arrival + tx bytes
  uint64_t* empty = bars + STAGES;  // [STAGES], NW arrivals

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int KVH = p.KVH;

  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], NW);
    }
    fence_barrier_init();
  }
  launch_dependents();
  // Launch, shared-memory set-up and barrier init overlap the end of the
  // previous kernel in the stream; every global read or write comes after
  // this wait (the previous kernel may write q, the pools, lengths, tables).
  grid_dependency_wait();
  const int64_t U = plan_units<NT>(p, P, Ls, misc);  // ends with __syncthreads

  for (int b = blockIdx.x; b < p.B; b += gridDim.x) {
    if (Ls[b] == 0) {
      T* o = static_cast<T*>(p.out) + (int64_t)b * p.H * D;
      for (int i = tid; i < p.H * D; i += NT) o[i] = Elem<T>::from_f(0.f);
    }
  }

  const int64_t grid = part_grid(gridDim.x, U);
  if ((int64_t)blockIdx.x >= grid) return;
  const int64_t u_beg = part_begin(blockIdx.x, U, grid);
  const int64_t u_end = part_begin(blockIdx.x + 1, U, grid);
  if (u_beg >= u_end) return;
  auto stage_k = [&](int s) { return smem + (size_t)s * M::STAGE_BYTES; };

  if (warp == NW) {
    // ---------------- producer warp ----------------
    Cursor c;
    cursor_locate(c, P, p.B, KVH, u_beg);
    const int32_t* tables = p.tables;
    for (int k = 0;; ++k) {
      const int s = k % STAGES;
      const uint32_t use = (uint32_t)(k / STAGES);
      if (use > 0) mbar_wait(&empty[s], (use - 1) & 1);  // consumers released use-1
      const int64_t te = cursor_tile_end<M::TILE_UNITS>(c, u_end);
      const int nunits = (int)(te - c.u);
      const int tok0 = (int)(c.u - c.seg) * kUnitTokens;
      // lane i < nunits stages unit i of the tile
      bool ok = false;
      int row0 = 0;
      if (lane < nunits) {
        const int t = tok0 + lane * kUnitTokens;
        const int pi = p.bs_shift >= 0 ? (t >> p.bs_shift) : t / p.block_size;
        const int off = t - pi * p.block_size;
        const int page = __ldg(tables + (int64_t)c.b * p.table_width + pi);
        if (page < 0 || (int64_t)page >= p.num_blocks) {
          raise_error(0x1u);
        } else {
          ok = true;
          row0 = page * p.block_size + off;
        }
      }
      const unsigned okmask = __ballot_sync(0xffffffffu, ok);
      if (lane == 0) {
        fence_proxy_async_smem();
        mbar_arrive_expect_tx(&full[s], (uint32_t)__popc(okmask) * K::UNIT_BYTES);
      }
      __syncwarp();
      if (ok) {
        unsigned char* sk = stage_k(s);
        unsigned char* sv = sk + M::TILE_BYTES;
#pragma unroll
        for (int hf = 0; hf < K::HALVES; ++hf) {
          const int dst = hf * (TILE * 128) + lane * kUnitTokens * 128;
          tma_load_3d(sk + dst, &kmap, hf * 64, c.h, row0, &full[s]);
          tma_load_3d(sv + dst, &vmap, hf * 64, c.h, row0, &full[s]);
        }
      }
      cursor_advance(c, te, u_end, P, KVH);
      if (c.u >= u_end) break;
    }
    return;
  }

  // ---------------- consumer warps 0..NW-1 ----------------
  Cursor cc;
  cursor_locate(cc, P, p.B, KVH, u_beg);
  typename M::State st;
  bool piece_start = true;
  int64_t piece_u0 = u_beg;
  auto sync_math = [] { named_bar_sync(1, NW * 32); };
  for (int k = 0;; ++k) {
    const int s = k % STAGES;
    mbar_wait(&full[s], (uint32_t)(k / STAGES) & 1);
    const int64_t cte = cursor_tile_end<M::TILE_UNITS>(cc, u_end);
    const int ntok = tile_tokens(cc, cte, Ls);
    unsigned char* sk = stage_k(s);
    unsigned char* sv = sk + M::TILE_BYTES;
    // Zero this warp's V rows past the sequence end (stale pool rows of the
    // last unit, or rows of a previous tile when the tile is short).
    const int r0 = warp * M::WT;
    if (r0 < ntok && r0 + M::WT > ntok) {
      for (int i = lane; i < (r0 + M::WT - ntok) * (D / 8); i += 32) {
        const int row = ntok + i / (D / 8), col = i % (D / 8);
        *reinterpret_cast<uint4*>(sv + M::offset(row, col)) = make_uint4(0, 0, 0, 0);
      }
      fence_proxy_async_smem();  // generic writes before the next TMA into this stage
      __syncwarp();
    }
    if (piece_start) {
      piece_u0 = cc.u;
      piece_start = false;
      M::begin_piece(st, p, cc.b, cc.h);
    }
    M::compute_tile(st, p, sk, sv, ntok, nullptr);
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);

    const bool seg_end = (cte == cc.seg + cc.nu);
    if (seg_end || cte == u_end) {
      M::store_state(st, ms, ls, accs);
      sync_math();
      finish_piece<M>(p, cc, piece_u0, u_beg, U, grid, seg_end, ms, ls, accs, misc, sync_math);
      piece_start = true;
    }
    if (cte >= u_end) break;
    cursor_advance(cc, cte, u_end, P, KVH);
  }
}

}  // namespace pdb
