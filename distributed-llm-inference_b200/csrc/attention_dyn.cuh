// Stream-K paged decode attention with a TMA producer warp and a dynamic tail
// (sm_100a, FP16). Same math (MmaMath, tensor cores) and staging (3-D TMA
// boxes, 128-byte swizzle) as attn_tma_kernel; what changes is the
// schedule.
//
// CTAs that receive equal static shares do not finish together: measured on
// B200, the last tile of equal shares lands up to ~15 % apart. So the unit
// stream (16-token units ordered by sequence, kv head, token) is split into
//   * a static head, the first 15/16 of the units, in one contiguous range
//     per CTA (as in attn_tma_kernel), and
//   * a tail, the last 1/16, cut into at most kTailChunksPerCta chunks per CTA
//     of at least kMinChunkTiles 64-token tiles each, which CTAs claim one at
//     a time with a tagged atomic counter once their static range is done.
// Tail fraction and chunk size were chosen by measurement on B200 (Llama-3-8B
// shape, batch 32 to 256): smaller chunks or a larger tail cost more in piece
// finishes and merges than they gain in balance. A call whose static shares
// would be short (under kTailMinTiles tiles per CTA) has no tail: there a
// claimed chunk (a piece start, four tiles at the rate of one CTA, an
// arrival) finishes after the unclaimed CTAs, so the tail made the stragglers
// it was meant to absorb (Llama-3-8B shape at 32 sequences: 39.7 -> 36.3 us
// per launch without it; 64 sequences and up keep it).
// The unit stream lists first the sequences whose per-head segments are
// longer than two tail chunks, then the others (each group in index order),
// so the tail holds short segments that few chunk boundaries cut and the
// merges at the end of the kernel combine few pieces.
// Every range (a CTA's static range or a tail chunk) is a "worker" with a
// contiguous unit range. A (sequence, kv head) segment cut by worker
// boundaries is merged by the last of its pieces to arrive, exactly as in
// attn_tma_kernel, with two partial slots per worker — so the workspace stays
// bounded by the grid, not by the batch.
//
// The producer warp owns the schedule: it walks its workers, claims tail
// chunks ahead of time, issues the TMA boxes and writes a per-stage record
// (segment, token count, piece flags, merge information) that the four
// tensor-core warps read after the stage's "full" barrier; a final record
// marks the end. A piece that is not a whole segment costs the math warps
// only its partial-slot stores: they queue the piece's arrival for an
// epilogue warp and go on with the next tile, while the epilogue warp makes
// the arrival (a gpu-scope release and an L2 round trip) and, for the last
// piece of a segment, merges the segment's slots into its output rows. All
// mbarrier waits and the claim loop are bounded.
#pragma once

#include "attention_tma.cuh"
#include "rope_kv_write.cuh"

namespace pdb {

constexpr int kTailDen = 16;         // tail = U / kTailDen units
constexpr int kTailChunksPerCta = 4;  // target tail chunks per launched CTA
constexpr int kMinChunkTiles = 4;     // a tail chunk covers at least this many tiles
constexpr int kTailMinTiles = 24;     // no tail below this many tiles per launched CTA

// Worker layout of one call: static workers 0..gs-1 over [0, Us), tail
// workers gs..gs+K-1 over [Us, U).
// begin(w) for w in [0, gs + K] is non-decreasing, begin(0) = 0,
// begin(gs) = Us, begin(gs + K) = U; with U > 0, gs >= 1 and every worker
// owns at least one unit (tail chunks at least kMinChunkTiles tiles).
struct DynPlan {
  int64_t U, Us, Ut, gs, K;
  __host__ __device__ __forceinline__ int64_t begin(int64_t w) const {
    // w == gs (end of the static region) stays in the first branch, so no
    // division by K happens when there is no tail (K == 0).
    return w <= gs ? part_begin(w, Us, gs) : Us + part_begin(w - gs, Ut, K);
  }
  __host__ __device__ __forceinline__ int64_t owner(int64_t u) const {
    return u < Us ? part_owner(u, Us, gs) : gs + part_owner(u - Us, Ut, K);
  }
};

__host__ __device__ __forceinline__ DynPlan make_dyn_plan(int64_t U, int64_t launched,
                                                          int tile_units) {
  DynPlan pl;
  pl.U = U;
  int64_t Ut = (U >= (int64_t)kTailMinTiles * launched * tile_units) ? U / kTailDen : 0;
  int64_t K = launched * kTailChunksPerCta;
  const int64_t kmax = Ut / ((int64_t)kMinChunkTiles * tile_units);
  if (K > kmax) K = kmax;
  if (K <= 0) { K = 0; Ut = 0; }
  pl.Ut = Ut;
  pl.K = K;
  pl.Us = U - Ut;
  pl.gs = pl.Us > 0 ? part_grid(launched, pl.Us) : 0;
  return pl;
}

__host__ __device__ __forceinline__ unsigned long long claim_tag(unsigned long long tag48) {
  return tag48 & ((1ull << 44) - 1);  // 44 tag bits + 20 count bits per word
}

// Claim the next tail chunk from a counter word (call tag << 20 | claims):
// the epilogue warp installs the call's tag when the CTA starts, so a claim
// is normally one fetch-add (a claim that still finds another tag installs it
// and claims again); the CTAs that finish their static ranges together do not
// serialise on a CAS loop. With K > 0 every launched CTA claims until a claim comes back empty,
// so a call makes exactly K + launched claims (far below 2^20); the last one
// puts the count back to zero (tag kept), so a CUDA-graph replay of the same
// call starts from zero. Returns the chunk index, or K when none is left.
// Claims need no ordering: they only pick work; results are published by
// arrive_piece.
__device__ __forceinline__ int64_t claim_chunk(unsigned long long* ctr, unsigned long long tag48,
                                               int64_t K, int64_t launched) {
  const unsigned long long tag = claim_tag(tag48);
  unsigned long long old = atomicAdd(ctr, 1ull);
  if ((old >> 20) != tag) {  // the stale word absorbs the add; the install replaces it
    if (!install_tag(ctr, tag, 20, launched + 64)) return K;
    old = atomicAdd(ctr, 1ull);
  }
  const int64_t cnt = (int64_t)(old & 0xfffffull);
  if (cnt == K + launched - 1) store_relaxed(ctr, tag << 20);
  return cnt < K ? cnt : K;
}

// Unit stream of one call, written by stream position i: P[i] (first unit,
// P[B] = U), Ls[i] (clamped length) and ord[i] (sequence index). Sequences
// whose per-head unit count exceeds two tail chunks come first, the others
// after them, each group in index order; with no tail the order is the index
// order. Three block passes over the lengths: the unit total (which fixes the
// plan and the threshold), the long sequences' count and units, and a prefix
// scan placing every sequence; the lengths are read from global memory once,
// into Lidx (by sequence index). All NT threads call it; misc holds
// 3 + 3 * NT / 32 ints.
__device__ __forceinline__ void warp_scan3(int& a, int& b, int& c, int lane) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int ta = __shfl_up_sync(0xffffffffu, a, o);
    const int tb = __shfl_up_sync(0xffffffffu, b, o);
    const int tc = __shfl_up_sync(0xffffffffu, c, o);
    if (lane >= o) {
      a += ta;
      b += tb;
      c += tc;
    }
  }
}

template <int NT>
__device__ int64_t plan_dyn_stream(const AttnParams& p, int* P, int* Ls, int* ord, int* Lidx,
                                   int* misc, int64_t launched, int tile_units, DynPlan& pl) {
  constexpr int NWARP = NT / 32;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int B = p.B, KVH = p.KVH;
  auto units_of = [&](int len) { return (len + kUnitTokens - 1) / kUnitTokens; };
  // pass 1: unit total (lengths kept by index in Lidx)
  int part = 0;
  for (int b = tid; b < B; b += NT) {
    const int len = checked_length(p.lengths, b, p.max_length);
    Lidx[b] = len;
    part += units_of(len) * KVH;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
  if (lane == 0) misc[3 + warp] = part;
  __syncthreads();
  int U = 0;
#pragma unroll
  for (int w = 0; w < NWARP; ++w) U += misc[3 + w];
  __syncthreads();
  pl = make_dyn_plan(U, launched, tile_units);
  const int64_t thr64 = pl.K > 0 ? 2 * (pl.Ut / pl.K) : 0x7fffffff;
  const int thr = (int)(thr64 < 0x7fffffff ? thr64 : 0x7fffffff);
  // pass 2: long sequences' count and units
  int fc = 0, fu = 0;
  for (int b = tid; b < B; b += NT) {
    const int nu = units_of(Lidx[b]);
    if (nu > thr) {
      ++fc;
      fu += nu * KVH;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    fc += __shfl_xor_sync(0xffffffffu, fc, o);
    fu += __shfl_xor_sync(0xffffffffu, fu, o);
  }
  if (lane == 0) {
    misc[3 + warp] = fc;
    misc[3 + NWARP + warp] = fu;
  }
  __syncthreads();
  int FL = 0, NL = 0;
#pragma unroll
  for (int w = 0; w < NWARP; ++w) {
    FL += misc[3 + w];
    NL += misc[3 + NWARP + w];
  }
  __syncthreads();
  // pass 3: place every sequence
  int off_f = 0, off_fu = 0, off_a = 0;
  for (int base = 0; base < B; base += NT) {
    const int b = base + tid;
    int len = 0, nu = 0, f = 0;
    if (b < B) {
      len = Lidx[b];
      nu = units_of(len) * KVH;
      f = units_of(len) > thr ? 1 : 0;
    }
    int sf = f, sfu = f ? nu : 0, sa = nu;
    warp_scan3(sf, sfu, sa, lane);
    if (lane == 31) {
      misc[3 + warp] = sf;
      misc[3 + NWARP + warp] = sfu;
      misc[3 + 2 * NWARP + warp] = sa;
    }
    __syncthreads();
    int ef = off_f + sf - f, efu = off_fu + sfu - (f ? nu : 0), ea = off_a + sa - nu;
    int tf = 0, tfu = 0, ta = 0;
#pragma unroll
    for (int w = 0; w < NWARP; ++w) {
      const int a0 = misc[3 + w], a1 = misc[3 + NWARP + w], a2 = misc[3 + 2 * NWARP + w];
      if (w < warp) {
        ef += a0;
        efu += a1;
        ea += a2;
      }
      tf += a0;
      tfu += a1;
      ta += a2;
    }
    if (b < B) {
      const int pos = f ? ef : FL + (b - ef);
      P[pos] = f ? efu : NL + (ea - efu);
      Ls[pos] = len;
      ord[pos] = b;
    }
    off_f += tf;
    off_fu += tfu;
    off_a += ta;
    __syncthreads();
  }
  if (tid == 0) P[B] = U;
  __syncthreads();
  return U;
}

// What the producer tells the math warps about the tile in a stage.
struct TileRecord {
  int b, h;          // segment (sequence, kv head)
  int ntok;          // valid tokens in the tile
  int flags;         // kRecFirst | kRecLast | kRecWhole | kRecEnd
  int slot;          // partial slot of the piece (non-whole pieces)
  int pieces;        // pieces of the segment (arrival count)
  long long w_first; // first worker of the segment
  long long w_last;  // last worker of the segment
  int first_slot;    // slot of the segment's piece in w_first
  int len;           // tokens of sequence b (the fused prologue's position + 1)
  int slot_row;      // fused, kRecNewRow tiles: pool row of the new token (-1: none)
  int pad;
};
// kRecOpen: the piece that starts here will not be a whole segment.
// kRecNewTok (fused prologue): the piece that starts here contains the
// segment's last unit, i.e. the new token; kRecNewRow: this tile holds it.
constexpr int kRecFirst = 1, kRecLast = 2, kRecWhole = 4, kRecEnd = 8, kRecOpen = 16;
constexpr int kRecNewTok = 32, kRecNewRow = 64;
// kRecQPre: the piece that starts here has its q rows (and, with kRecNewTok,
// the new token's k and v rows) in the stage's prefetch slots.
constexpr int kRecQPre = 128;

// Work queued by the math warps for the epilogue warp: the tag install of a
// piece's counter when the piece starts, its arrival when it ends, the end.
struct PieceHandoff {
  long long w_first, w_last;  // workers of the segment
  int b, h;                   // segment
  int pieces;                 // arrival count of the segment
  int first_slot;             // slot of the segment's piece in w_first
  int kind;                   // kHandArrive | kHandInstall | kHandEnd
  int pad;
};
constexpr int kHandArrive = 0, kHandInstall = 1, kHandEnd = 2;
constexpr int kHandoffDepth = 8;
constexpr int kDynMisc = 32;  // ints of per-CTA scratch

// Fused decode prologue at the start of a piece (all math threads, tid <
// NW * 32), in place of MmaMath::begin_piece: the lane's q elements and — for
// the piece holding the new token — the token's k and v are read first (from
// the stage's prefetch slots, or from global memory, so their latency
// overlaps the piece's cos/sin table: FP16-rounded, as rope_kv_write computes
// them; inv_freq staged in shared memory); then q is rotated into the lane's
// Q^T fragment (rotate-half: element i < D/2 pairs with i + D/2) and the
// token's rotated k and its v go to `newrow`, from where the tile holding the
// token is patched and the pool slot written. Per-op FP16 rounding as in
// rope_kv_write. `qbase` points at the group's G query rows, `knew` / `vnew`
// at the token's k and v rows. `sync` is a barrier over the math threads.
// `cs_pos` is the position the table in `cs` was built for: consecutive
// pieces of one sequence (its kv heads are adjacent in the unit stream) share
// the position, and the table is reused (every math thread holds the same
// cs_pos, so all skip the build and its barrier together; the previous
// piece's reads of the table ended before its last tile's combine).
template <class M, class Sync>
__device__ __forceinline__ void fused_piece_start(typename M::State& st, const AttnParams& p,
                                                  const __half* qbase, const __half* knew,
                                                  const __half* vnew, int pos, bool new_tok,
                                                  const float* invf, float* cs, __half* newrow,
                                                  int& cs_pos, Sync sync) {
  constexpr int D = M::D, KS = M::KSTEPS, HALF = D / 2;
  static_assert(KS % 2 == 0, "lower and upper halves in whole k-steps");
  const int tid = threadIdx.x, lane = tid & 31, g = lane >> 2, tg = lane & 3;
  const bool real = g < p.G;  // columns >= G are padding (q = 0)
  const __half* qrow = qbase + (real ? g : 0) * D;
  __half2 qx1[KS / 2][2], qx2[KS / 2][2];
#pragma unroll
  for (int ks = 0; ks < KS / 2; ++ks)
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const int i = 16 * ks + 2 * tg + 8 * r;
      qx1[ks][r] = *reinterpret_cast<const __half2*>(qrow + i);
      qx2[ks][r] = *reinterpret_cast<const __half2*>(qrow + i + HALF);
    }
  __half k1 = __float2half_rn(0.f), k2 = k1, v1 = k1, v2 = k1;
  if (new_tok && tid < HALF) {
    k1 = knew[tid];
    k2 = knew[tid + HALF];
    v1 = vnew[tid];
    v2 = vnew[tid + HALF];
  }
  if (pos != cs_pos) {
    if (tid < HALF) {
      float c, s;
      rope_cos_sin<__half>(__fmul_rn((float)pos, invf[tid]), &c, &s);
      cs[tid] = __half2float(__float2half_rn(c));
      cs[HALF + tid] = __half2float(__float2half_rn(s));
    }
    cs_pos = pos;
    sync();
  }
  auto rot = [&](float x1, float x2, int i, __half* o1, __half* o2) {
    const float c = cs[i], sn = cs[HALF + i];
    const float a = __half2float(__float2half_rn(__fmul_rn(x1, c)));
    const float bb = __half2float(__float2half_rn(__fmul_rn(x2, sn)));
    const float d = __half2float(__float2half_rn(__fmul_rn(x2, c)));
    const float e = __half2float(__float2half_rn(__fmul_rn(x1, sn)));
    *o1 = __float2half_rn(__fsub_rn(a, bb));
    *o2 = __float2half_rn(__fadd_rn(d, e));
  };
#pragma unroll
  for (int ks = 0; ks < KS / 2; ++ks) {
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const int i = 16 * ks + 2 * tg + 8 * r;  // elements i, i + 1 (lower half)
      uint32_t lo = 0u, hi = 0u;
      if (real) {
        // the same rounding as rot(), two elements at a time: each product
        // and the sum rounded once to FP16 (no fma contraction)
        const __half2 c = __floats2half2_rn(cs[i], cs[i + 1]);
        const __half2 sn = __floats2half2_rn(cs[HALF + i], cs[HALF + i + 1]);
        const __half2 lo2 = __hsub2(__hmul2_rn(qx1[ks][r], c), __hmul2_rn(qx2[ks][r], sn));
        const __half2 hi2 = __hadd2(__hmul2_rn(qx2[ks][r], c), __hmul2_rn(qx1[ks][r], sn));
        lo = *reinterpret_cast<const uint32_t*>(&lo2);
        hi = *reinterpret_cast<const uint32_t*>(&hi2);
      }
      st.qb[ks][r] = lo;
      st.qb[ks + KS / 2][r] = hi;
    }
  }
  st.m[0] = st.m[1] = -INFINITY;
  st.l[0] = st.l[1] = 0.f;
#pragma unroll
  for (int i = 0; i < KS; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) st.acc[i][j] = 0.f;
  if (new_tok) {
    if (tid < HALF) {
      __half o1, o2;
      rot(__half2float(k1), __half2float(k2), tid, &o1, &o2);
      newrow[tid] = o1;
      newrow[tid + HALF] = o2;
      newrow[D + tid] = v1;
      newrow[D + tid + HALF] = v2;
    }
    sync();
  }
}

// The fused prologue's piece start for the SIMT inner loop (FP32): the
// cos/sin table of the piece's position (rebuilt only when the position
// changes), then the group's G query rows rotated into `rq` (shared memory;
// it may be the rows' own prefetch slot, each chunk pair is read and written
// by one thread) and, for the piece holding the new token, the token's
// rotated k and its v into `newrow`; then the SIMT state is loaded from `rq`.
// The rotation is rope_chunk_pair, the cos/sin rope_cos_sin of the position
// times inv_freq: the operations of the decode prologue kernel, so the fused
// layer equals rope_kv_write_decode + paged_attention bit for bit. q, k and v
// rows are read in 16-byte chunks (16-byte aligned rows).
template <class M, class Sync>
__device__ __forceinline__ void fused_piece_start_simt(
    typename M::State& st, const AttnParams& p, const typename M::T* qbase,
    const typename M::T* knew, const typename M::T* vnew, int pos, bool new_tok,
    const float* invf, float* cs, typename M::T* newrow, typename M::T* rq, int& cs_pos,
    Sync sync) {
  using T = typename M::T;
  constexpr int D = M::D, HALF = D / 2, VEC = 16 / (int)sizeof(T), HC = HALF / VEC;
  constexpr int NMT = M::NW * 32;  // math threads
  const int tid = threadIdx.x;
  if (pos != cs_pos) {
    for (int j = tid; j < HALF; j += NMT) {
      float c, s;
      rope_cos_sin<T>(__fmul_rn((float)pos, invf[j]), &c, &s);
      cs[j] = Elem<T>::to_f(Elem<T>::from_f(c));
      cs[HALF + j] = Elem<T>::to_f(Elem<T>::from_f(s));
    }
    cs_pos = pos;
    sync();
  }
  const int nq = p.G * HC, nk = new_tok ? HC : 0;
  for (int i = tid; i < nq + nk; i += NMT) {
    const bool isq = i < nq;
    const int ii = isq ? i : i - nq;
    const int g = ii / HC, c = ii - g * HC;
    uint4 o1, o2;
    rope_chunk_pair<T>(isq ? qbase + g * D : knew, c * VEC, HALF, cs, cs + HALF, o1, o2);
    store_chunk_pair<T>(isq ? rq + g * D : newrow, c * VEC, HALF, o1, o2);
  }
  if (new_tok) {
    for (int i = tid; i < D / VEC; i += NMT)
      reinterpret_cast<uint4*>(newrow + D)[i] = reinterpret_cast<const uint4*>(vnew)[i];
  }
  fence_proxy_async_smem();  // rq may be a prefetch slot the next bulk copy refills
  sync();
  M::begin_piece_at(st, rq, p.G);
}

template <class M>
struct DynStreamK {
  static_assert(M::LAYOUT == kTma128B, "dynamic kernel stages with TMA");
  using T = typename M::T;
  static constexpr int E = (int)sizeof(T);
  static constexpr int D = M::D, GP = M::GP, NW = M::NW, STAGES = M::STAGES;
  static constexpr int NT = (NW + 2) * 32;  // math warps, producer, epilogue
  static constexpr int BOX_COLS = 128 / E;  // elements of a 128-byte TMA box row
  static constexpr int HALVES = D / BOX_COLS;  // 128-byte column blocks of a row
  static constexpr int UNIT_BYTES = 2 * kUnitTokens * D * E;
  // Per-stage prefetch slots: a piece's q rows (G <= GP rows of D elements)
  // and the new token's k and v rows.
  static constexpr int QPRE_BYTES = GP * D * E;
  static constexpr int KVPRE_BYTES = 2 * D * E;
  // SIMT inner loops' probability broadcast (0 for the tensor-core loop)
  static constexpr int EXTRA_BYTES = M::EXTRA_FLOATS * 4;
  // At a piece end the warps' partial states (m, l, O per head) go through
  // the buffer of the stage just consumed.
  static_assert(NW * GP * (D + 2) * 4 <= M::STAGE_BYTES, "merge area fits in a stage");
  static size_t smem_bytes(int B) {
    return 1024 + (size_t)STAGES * (M::STAGE_BYTES + QPRE_BYTES + KVPRE_BYTES) + EXTRA_BYTES +
           (size_t)(4 * B + 1 + kDynMisc) * 4 + (2 * STAGES + 2 * kHandoffDepth) * 8 + 16 +
           (size_t)STAGES * sizeof(TileRecord) + kHandoffDepth * sizeof(PieceHandoff) +
           (size_t)D * 4 + (size_t)2 * D * E + (size_t)D / 2 * 4 +
           64;  // + fused prologue: cos/sin, new row, inv_freq (+ alignment)
  }
  // partial slots: two per worker (static workers + tail chunks)
  static int64_t slots(int64_t launched) { return 2 * launched * (1 + kTailChunksPerCta); }
};

// FUSE: the decode prologue (RoPE of q and of the new k, k/v slot writes) is
// folded in; see AttnParams::k_new.
template <class M, bool FUSE = false>
__global__ void __launch_bounds__(DynStreamK<M>::NT, 2)
attn_tma_dyn_kernel(const AttnParams p, const __grid_constant__ CUtensorMap kmap,
                    const __grid_constant__ CUtensorMap vmap) {
  using T = typename M::T;
  using K = DynStreamK<M>;
  constexpr int D = M::D, GP = M::GP, NW = M::NW, STAGES = M::STAGES, NT = K::NT;
  constexpr int TILE = M::TILE, TU = M::TILE_UNITS;
  constexpr int SLOT_FLOATS = GP * (D + 2);
  static_assert(!FUSE || M::CHUNKS <= 32, "one 16-byte chunk of the new token's row per lane");

  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* qpre = smem + (size_t)STAGES * M::STAGE_BYTES;  // [STAGES][QPRE_BYTES]
  unsigned char* kvpre = qpre + (size_t)STAGES * K::QPRE_BYTES;  // [STAGES][KVPRE_BYTES]
  float* extra = reinterpret_cast<float*>(kvpre + (size_t)STAGES * K::KVPRE_BYTES);
  int* P = reinterpret_cast<int*>(extra + M::EXTRA_FLOATS);  // by stream position
  int* Ls = P + p.B + 1;
  int* ord = Ls + p.B;
  int* Lidx = ord + p.B;  // lengths by sequence index (plan only)
  int* misc = Lidx + p.B;  // [kDynMisc]
  uint64_t* bars = reinterpret_cast<uint64_t*>(
      (reinterpret_cast<uintptr_t>(misc + kDynMisc) + 7) & ~uintptr_t(7));
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* hf_full = bars + 2 * STAGES;  // hand-off queue to the epilogue warp
  uint64_t* hf_empty = hf_full + kHandoffDepth;
  TileRecord* recs = reinterpret_cast<TileRecord*>(
      (reinterpret_cast<uintptr_t>(hf_empty + kHandoffDepth) + 15) & ~uintptr_t(15));
  PieceHandoff* hand = reinterpret_cast<PieceHandoff*>(recs + STAGES);
  // fused prologue buffers, each 16-byte aligned (newrow is read as uint4)
  auto align16 = [](const void* q) {
    return (reinterpret_cast<uintptr_t>(q) + 15) & ~uintptr_t(15);
  };
  float* cs_tab = reinterpret_cast<float*>(align16(hand + kHandoffDepth));  // [2][D/2]
  T* newrow = reinterpret_cast<T*>(align16(cs_tab + D));                    // k[D], v[D]
  float* invf = reinterpret_cast<float*>(align16(newrow + 2 * D));          // [D/2]

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int KVH = p.KVH;
  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], NW);
    }
    for (int j = 0; j < kHandoffDepth; ++j) {
      mbar_init(&hf_full[j], NW);
      mbar_init(&hf_empty[j], 1);
    }
    fence_barrier_init();
  }
  launch_dependents();
  // Every global access that may see the previous kernel's writes comes after
  // grid_dependency_wait(). With stable metadata (fused decode, layers after
  // the first of a step) the plan and the producer's page lookups read only
  // tables, lengths and inv_freq, so they run before it, overlapping the
  // previous launch's tail; with stable pools as well the producer's K/V
  // tiles are loaded before it too. Each role waits right before its first
  // access to anything else (q, new k/v, the output, the workspace counters;
  // the pools when they are not stable).
  const bool early = FUSE && (p.stable_meta & 1) != 0;
  const bool early_kv = early && (p.stable_meta & 2) != 0;  // K/V tiles too
  if (!early) grid_dependency_wait();
  if constexpr (FUSE) {
    for (int i = tid; i < D / 2; i += NT) invf[i] = __ldg(p.inv_freq + i);
  }
  static_assert(3 + 3 * (NT / 32) <= kDynMisc, "plan scratch");
  DynPlan pl;
  const int64_t U = plan_dyn_stream<NT>(p, P, Ls, ord, Lidx, misc, gridDim.x, TU, pl);
  if (early && warp != NW) grid_dependency_wait();  // math and epilogue warps
  if (warp < NW) {  // zero rows of empty sequences (the producer warp may not have waited)
    for (int i = blockIdx.x; i < p.B; i += gridDim.x) {
      if (Ls[i] == 0) {
        T* o = static_cast<T*>(p.out) + (int64_t)ord[i] * p.H * D;
        for (int j = tid; j < p.H * D; j += NW * 32) o[j] = Elem<T>::from_f(0.f);
      }
    }
  }
  if (U == 0) return;
  const bool has_static = (int64_t)blockIdx.x < pl.gs;
  if (!has_static && pl.K == 0) return;
  unsigned long long* claim_ctr = p.counters + (int64_t)p.B * KVH;  // one word after arrivals
  auto stage_k = [&](int s) { return smem + (size_t)s * M::STAGE_BYTES; };

  if (warp == NW) {
    // ---------------- producer warp: schedule + TMA ----------------
    int k = 0;  // tiles issued
    auto next_stage = [&](int& s) {
      s = k % STAGES;
      const uint32_t use = (uint32_t)(k / STAGES);
      if (use > 0) mbar_wait(&empty[s], (use - 1) & 1);
    };
    bool waited = !early;  // producer: wait before the first claim or TMA
    auto wait_prev = [&]() {
      if (!waited) {
        grid_dependency_wait();
        waited = true;
      }
    };
    // Tail chunks are claimed when the last tile of the current worker has
    // been issued, i.e. STAGES tiles before the math warps run out of work.
    auto claim = [&]() -> int64_t {
      wait_prev();
      int64_t c = pl.K;
      if (pl.K > 0 && lane == 0) c = claim_chunk(claim_ctr, p.call_tag, pl.K, gridDim.x);
      return __shfl_sync(0xffffffffu, c, 0);
    };
    int64_t w = has_static ? (int64_t)blockIdx.x : -1;
    if (w < 0) {
      const int64_t c0 = claim();
      w = c0 < pl.K ? pl.gs + c0 : -1;
    }
    while (w >= 0) {
      const int64_t wb = pl.begin(w), we = pl.begin(w + 1);
      Cursor c;
      cursor_locate(c, P, p.B, KVH, wb);
      bool piece_first = true;
      int64_t next_w = -1;
      while (true) {
        int s;
        next_stage(s);
        const int64_t te = cursor_tile_end<TU>(c, we);
        const int nunits = (int)(te - c.u);
        const int tok0 = (int)(c.u - c.seg) * kUnitTokens;
        const bool seg_end = te == c.seg + c.nu;
        const bool last = seg_end || te == we;
        const bool new_tok = FUSE && piece_first && c.seg + c.nu <= we;
        if (lane == 0) {
          TileRecord r{};
          r.b = ord[c.b];
          r.h = c.h;
          r.len = Ls[c.b];
          const int rem = Ls[c.b] - tok0;
          r.ntok = nunits * kUnitTokens < rem ? nunits * kUnitTokens : rem;
          r.flags = (piece_first ? kRecFirst : 0) | (last ? kRecLast : 0);
          if (piece_first && !(c.u == c.seg && c.seg + c.nu <= we)) r.flags |= kRecOpen;
          if (new_tok) r.flags |= kRecNewTok;
          if (FUSE && seg_end) r.flags |= kRecNewRow;
          if (last) {
            // The piece started at the worker's begin or at the segment's.
            const int64_t pstart = wb > c.seg ? wb : c.seg;
            if (seg_end && pstart == c.seg) {
              r.flags |= kRecWhole;
            } else {
              const int64_t S0 = c.seg, S1 = c.seg + c.nu;
              const int64_t w0 = pl.owner(S0), w1 = pl.owner(S1 - 1);
              r.slot = (int)(2 * w + (pstart == wb ? 0 : 1));
              r.pieces = (int)(w1 - w0 + 1);
              r.w_first = w0;
              r.w_last = w1;
              r.first_slot = (int)(2 * w0 + (pl.begin(w0) < S0 ? 1 : 0));
            }
          }
          recs[s] = r;
        }
        // page lookups: lane i < nunits stages unit i of the tile
        bool ok = false;
        int row0 = 0;
        if (lane < nunits) {
          const int t = tok0 + lane * kUnitTokens;
          const int pi = p.bs_shift >= 0 ? (t >> p.bs_shift) : t / p.block_size;
          const int off = t - pi * p.block_size;
          const int page = __ldg(p.tables + (int64_t)ord[c.b] * p.table_width + pi);
          if (page < 0 || (int64_t)page >= p.num_blocks) {
            raise_error(0x1u);
          } else {
            ok = true;
            row0 = page * p.block_size + off;
          }
        }
        const unsigned okmask = __ballot_sync(0xffffffffu, ok);
        if constexpr (FUSE) {
          if (seg_end) {  // the new token sits in this tile's last unit
            const int last = nunits - 1;
            const int lrow = __shfl_sync(0xffffffffu, row0, last);
            if (lane == 0)
              recs[s].slot_row = ((okmask >> last) & 1u)
                                     ? lrow + (Ls[c.b] - 1 - tok0 - last * kUnitTokens)
                                     : -1;
          }
        }
        // With stable pools the first STAGES tiles are issued before the
        // dependency wait; the producer would block on a stage release after
        // them anyway, so it waits there.
        if (!early_kv || k >= STAGES) wait_prev();
        // A piece's q rows (and the new token's k and v) ride on its first
        // tile's barrier, once the previous kernel (which may have written
        // them) is complete; before that, the math warps read them from
        // global memory themselves.
        const bool qp = p.bulk_q != 0 && waited && piece_first;
        const bool kvp = qp && new_tok;
        if (lane == 0) {
          const int qbytes = p.G * D * K::E;
          if (qp) recs[s].flags |= kRecQPre;
          fence_proxy_async_smem();
          mbar_arrive_expect_tx(&full[s], (uint32_t)__popc(okmask) * K::UNIT_BYTES +
                                              (qp ? qbytes : 0) + (kvp ? K::KVPRE_BYTES : 0));
          const int bq = ord[c.b];
          if (qp)
            bulk_load(qpre + (size_t)s * K::QPRE_BYTES,
                      static_cast<const T*>(p.q) + (int64_t)bq * p.q_row +
                          (int64_t)c.h * p.G * D,
                      (uint32_t)qbytes, &full[s]);
          if (kvp) {
            const int64_t kvo = (int64_t)bq * p.kv_row + (int64_t)c.h * D;
            unsigned char* dst = kvpre + (size_t)s * K::KVPRE_BYTES;
            bulk_load(dst, static_cast<const T*>(p.k_new) + kvo, D * K::E, &full[s]);
            bulk_load(dst + D * K::E, static_cast<const T*>(p.v_new) + kvo, D * K::E,
                      &full[s]);
          }
        }
        __syncwarp();
        if (ok) {
          unsigned char* sk = stage_k(s);
          unsigned char* sv = sk + M::TILE_BYTES;
#pragma unroll
          for (int hf = 0; hf < K::HALVES; ++hf) {
            const int dst = hf * (TILE * 128) + lane * kUnitTokens * 128;
            tma_load_3d(sk + dst, &kmap, hf * K::BOX_COLS, c.h, row0, &full[s]);
            tma_load_3d(sv + dst, &vmap, hf * K::BOX_COLS, c.h, row0, &full[s]);
          }
        }
        ++k;
        piece_first = last;  // a piece end makes the next tile a piece start
        if (te >= we) {
          const int64_t cn = claim();
          next_w = cn < pl.K ? pl.gs + cn : -1;
          break;
        }
        cursor_advance(c, te, we, P, KVH);
      }
      w = next_w;
    }
    // end record
    int s;
    next_stage(s);
    if (lane == 0) {
      TileRecord r{};
      r.flags = kRecEnd;
      recs[s] = r;
      mbar_arrive_expect_tx(&full[s], 0);
    }
    return;
  }

  if (warp == NW + 1) {
    // ---------------- epilogue warp: tag installs, arrivals, merges ----------
    if (lane == 0 && pl.K > 0) install_tag(claim_ctr, claim_tag(p.call_tag), 20, gridDim.x + 64);
    for (int hk = 0;; ++hk) {
      const int j = hk % kHandoffDepth;
      mbar_wait(&hf_full[j], (uint32_t)(hk / kHandoffDepth) & 1);
      const PieceHandoff r = hand[j];
      if (r.kind == kHandEnd) break;
      unsigned long long* ctr = p.counters + ((int64_t)r.b * KVH + r.h);
      if (r.kind == kHandInstall) {
        if (lane == 0) install_tag(ctr, p.call_tag, 16, (int64_t)gridDim.x * 8 + 64);
        __syncwarp();
        if (lane == 0) mbar_arrive(&hf_empty[j]);
        continue;
      }
      int last = 0;
      if (lane == 0) last = arrive_installed(ctr, p.call_tag, (unsigned)r.pieces);
      last = __shfl_sync(0xffffffffu, last, 0);
      __syncwarp();  // lane 0's acquire orders the other lanes' slot reads
      if (last) {
        T* outp = static_cast<T*>(p.out) + ((int64_t)r.b * p.H + (int64_t)r.h * p.G) * D;
        merge_slots<T, GP, D, 32, 48>(p.partials, outp, p.G, r.w_first, r.w_last, r.first_slot,
                                      lane);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&hf_empty[j]);
    }
    return;
  }

  // ---------------- math warps ----------------
  typename M::State st;
  int cs_pos = -1;  // position of the fused prologue's cos/sin table (none yet)
  auto sync_math = [] { named_bar_sync(1, NW * 32); };
  int hk = 0;  // pieces handed to the epilogue warp
  // Queue entry hk % depth: warp 0 waits until the epilogue warp has taken
  // the entry's previous use and writes it; each math warp's lane 0 arrives
  // after its warp's slot stores (release at CTA scope; the epilogue warp's
  // gpu-scope release in arrive_piece then covers them).
  auto hand_off = [&](const PieceHandoff& h) {
    const int j = hk % kHandoffDepth;
    if (warp == 0) {
      const uint32_t use = (uint32_t)(hk / kHandoffDepth);
      if (use > 0) mbar_wait(&hf_empty[j], (use - 1) & 1);
      if (lane == 0) hand[j] = h;
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&hf_full[j]);
    ++hk;
  };
  for (int k = 0;; ++k) {
    const int s = k % STAGES;
    mbar_wait(&full[s], (uint32_t)(k / STAGES) & 1);
    const TileRecord r = recs[s];
    if (r.flags & kRecEnd) break;
    unsigned char* sk = stage_k(s);
    unsigned char* sv = sk + M::TILE_BYTES;
    const int r0 = warp * M::WT;
    const bool pre = (r.flags & kRecQPre) != 0;
    const T* qbase =
        pre ? reinterpret_cast<const T*>(qpre + (size_t)s * K::QPRE_BYTES)
            : static_cast<const T*>(p.q) + (int64_t)r.b * p.q_row + (int64_t)r.h * p.G * D;
    if constexpr (FUSE) {
      if (r.flags & kRecFirst) {
        const T* kvs = reinterpret_cast<const T*>(kvpre + (size_t)s * K::KVPRE_BYTES);
        const int64_t kvo = (int64_t)r.b * p.kv_row + (int64_t)r.h * D;
        const T* kn = pre ? kvs : static_cast<const T*>(p.k_new) + kvo;
        const T* vn = pre ? kvs + D : static_cast<const T*>(p.v_new) + kvo;
        if constexpr (M::kSimt) {
          fused_piece_start_simt<M>(st, p, qbase, kn, vn, r.len - 1,
                                    (r.flags & kRecNewTok) != 0, invf, cs_tab, newrow,
                                    reinterpret_cast<T*>(qpre + (size_t)s * K::QPRE_BYTES),
                                    cs_pos, sync_math);
        } else {
          fused_piece_start<M>(st, p, qbase, kn, vn, r.len - 1, (r.flags & kRecNewTok) != 0,
                               invf, cs_tab, newrow, cs_pos, sync_math);
        }
      }
      // The new token's row of this tile: the TMA brought the slot's old
      // bytes; the owning warp writes the rotated k and the v in their place
      // and into the pool slot (for later steps; this launch never reads the
      // slot from global memory).
      const int nr = r.ntok - 1;
      if ((r.flags & kRecNewRow) && nr >= r0 && nr < r0 + M::WT) {
        if (lane < M::CHUNKS) {
          const uint4 kc = reinterpret_cast<const uint4*>(newrow)[lane];
          const uint4 vc = reinterpret_cast<const uint4*>(newrow + D)[lane];
          *reinterpret_cast<uint4*>(sk + M::offset(nr, lane)) = kc;
          *reinterpret_cast<uint4*>(sv + M::offset(nr, lane)) = vc;
          if (r.slot_row >= 0) {
            const int64_t base = ((int64_t)r.slot_row * KVH + r.h) * D;
            reinterpret_cast<uint4*>(static_cast<T*>(const_cast<void*>(p.k_pool)) +
                                     base)[lane] = kc;
            reinterpret_cast<uint4*>(static_cast<T*>(const_cast<void*>(p.v_pool)) +
                                     base)[lane] = vc;
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
      }
    }
    if (r0 < r.ntok && r0 + M::WT > r.ntok) {
      for (int i = lane; i < (r0 + M::WT - r.ntok) * M::CHUNKS; i += 32) {
        const int row = r.ntok + i / M::CHUNKS, col = i % M::CHUNKS;
        *reinterpret_cast<uint4*>(sv + M::offset(row, col)) = make_uint4(0, 0, 0, 0);
      }
      fence_proxy_async_smem();
      __syncwarp();
    }
    if ((r.flags & (kRecFirst | kRecOpen)) == (kRecFirst | kRecOpen))
      hand_off(PieceHandoff{0, 0, r.b, r.h, 0, 0, kHandInstall, 0});
    if (r.flags & kRecFirst) {
      if constexpr (!FUSE) M::begin_piece_at(st, qbase, p.G);  // fused: done above
    }
    M::compute_tile(st, p, sk, sv, r.ntok, extra);
    if (!(r.flags & kRecLast)) {
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
      continue;
    }
    // Piece end. Once every math warp is done with the tile, the stage's
    // buffer holds the warps' partial states (m, l, O per head) for the
    // combine; each warp releases the stage after its share of the combine
    // (the producer refills it only after all NW releases).
    sync_math();
    float* ms = reinterpret_cast<float*>(sk);
    float* ls = ms + NW * GP;
    float* accs = ls + NW * GP;
    M::store_state(st, ms, ls, accs);
    sync_math();
    {
      T* outp = static_cast<T*>(p.out) + ((int64_t)r.b * p.H + (int64_t)r.h * p.G) * D;
      const bool whole = r.flags & kRecWhole;
      const bool out8 = (reinterpret_cast<uintptr_t>(outp) & 7u) == 0;
      const bool out16 = (reinterpret_cast<uintptr_t>(outp) & 15u) == 0;
      float* slot = p.partials + (size_t)r.slot * SLOT_FLOATS;
      // four consecutive dims of one head per thread: the head's NW factors
      // once, then float4 reads of the warps' accumulators
      for (int i = tid; i < GP * D / 4; i += NW * 32) {
        const int g = (4 * i) / D, d = 4 * i - g * D;
        float mw[NW], M_ = -INFINITY;
#pragma unroll
        for (int ww = 0; ww < NW; ++ww) {
          mw[ww] = ms[ww * GP + g];
          M_ = fmaxf(M_, mw[ww]);
        }
        float L = 0.f;
        float4 O = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int ww = 0; ww < NW; ++ww) {
          const float f = (mw[ww] == -INFINITY) ? 0.f : exp2f(mw[ww] - M_);
          L = fmaf(ls[ww * GP + g], f, L);
          const float4 a = *reinterpret_cast<const float4*>(accs + (ww * GP + g) * D + d);
          O.x = fmaf(a.x, f, O.x);
          O.y = fmaf(a.y, f, O.y);
          O.z = fmaf(a.z, f, O.z);
          O.w = fmaf(a.w, f, O.w);
        }
        if (whole) {
          if (g < p.G) {
            T* o = outp + g * D + d;
            const T o0 = Elem<T>::from_f(O.x / L), o1 = Elem<T>::from_f(O.y / L);
            const T o2 = Elem<T>::from_f(O.z / L), o3 = Elem<T>::from_f(O.w / L);
            if constexpr (sizeof(T) == 2) {
              if (out8) {
                const __half2 lo = __halves2half2(o0, o1), hi = __halves2half2(o2, o3);
                uint2 v;
                v.x = *reinterpret_cast<const uint32_t*>(&lo);
                v.y = *reinterpret_cast<const uint32_t*>(&hi);
                *reinterpret_cast<uint2*>(o) = v;
              } else {
                o[0] = o0; o[1] = o1; o[2] = o2; o[3] = o3;
              }
            } else {
              if (out16) {
                *reinterpret_cast<float4*>(o) = make_float4(o0, o1, o2, o3);
              } else {
                o[0] = o0; o[1] = o1; o[2] = o2; o[3] = o3;
              }
            }
          }
        } else {
          // 16-byte stores when every slot and its O block start 16-byte
          // aligned (GP even); GP 1 (the SIMT inner loop's MHA case) stores
          // the four floats one by one
          constexpr bool kSlotVec = (GP * (D + 2) * 4) % 16 == 0 && (2 * GP * 4) % 16 == 0;
          float* so = slot + 2 * GP + g * D + d;
          if constexpr (kSlotVec) {
            *reinterpret_cast<float4*>(so) = O;
          } else {
            so[0] = O.x; so[1] = O.y; so[2] = O.z; so[3] = O.w;
          }
          if (d == 0) {
            slot[g] = M_;
            slot[GP + g] = L;
          }
        }
      }
      fence_proxy_async_smem();  // generic writes to the stage before TMA refills it
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
      if (!whole)
        hand_off(PieceHandoff{r.w_first, r.w_last, r.b, r.h, r.pieces, r.first_slot, kHandArrive,
                              0});
    }
  }
  hand_off(PieceHandoff{0, 0, 0, 0, 0, 0, kHandEnd, 0});
}

}  // namespace pdb
