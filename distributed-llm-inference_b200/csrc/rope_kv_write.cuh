// Fused RoPE + paged KV-slot write.
//
// Restates, as one kernel per layer, what worker/llama.py does per layer with
// ~12 ATen launches:
//   PagedLlama.rope            worker/llama.py:108-117
//   keys[layer][slots] = k     worker/llama.py:171 (decode), :139 (prefill)
//   values[layer][slots] = v   worker/llama.py:172 (decode), :140 (prefill)
//
// Rounding is reproduced op by op, so that outputs are bit-identical to the
// reference whenever cos/sin agree:
//   ang  = fp32(pos) * inv_freq[j]                  (fp32, round-to-nearest)
//   c, s = cos(ang), sin(ang)  rounded to fp32, then to the model dtype
//   a    = round(x[j] * c);  b = round(x[j + D/2] * s)      (model dtype)
//   out[j] = round(a - b);   out[j + D/2] = round(round(x[j+D/2]*c) + round(x[j]*s))
// For FP16 each product/sum is formed exactly in fp32 and rounded once to
// FP16 (an fp32 sum of two FP16 values rounds to the same FP16 value as an
// exact sum: 24 >= 2*11+2 bits). cos/sin: see rope_cos_sin.
#pragma once

#include "common.cuh"

namespace pdb {

// Exclusive scan of the valid mask: slot_of_row[r] = index of row r among the
// valid rows, or -1. One CTA; rows are processed in chunks of blockDim*ITEMS.
template <int THREADS, int ITEMS>
__global__ void __launch_bounds__(THREADS)
valid_scan_kernel(const uint8_t* __restrict__ valid, int64_t rows,
                  int64_t num_slots, int32_t* __restrict__ slot_of_row) {
  grid_dependency_wait();
  launch_dependents();
  __shared__ int warp_sums[THREADS / 32];
  __shared__ int carry_s;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) carry_s = 0;
  __syncthreads();
  for (int64_t base = 0; base < rows; base += (int64_t)THREADS * ITEMS) {
    int flags[ITEMS];
    int local = 0;
    const int64_t r_first = base + (int64_t)tid * ITEMS;
    if (ITEMS == 16 && r_first + 16 <= rows &&
        (reinterpret_cast<uintptr_t>(valid + r_first) & 15u) == 0) {  // one 16-byte load
      const uint4 w = *reinterpret_cast<const uint4*>(valid + r_first);
      const uint32_t wd[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int i = 0; i < ITEMS; ++i) {
        flags[i] = ((wd[(i / 4) & 3] >> (8 * (i % 4))) & 0xffu) ? 1 : 0;
        local += flags[i];
      }
    } else {
#pragma unroll
      for (int i = 0; i < ITEMS; ++i) {
        const int64_t r = r_first + i;
        flags[i] = (r < rows && valid[r]) ? 1 : 0;
        local += flags[i];
      }
    }
    // inclusive warp scan of per-thread counts
    int incl = local;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int t = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += t;
    }
    if (lane == 31) warp_sums[warp] = incl;
    __syncthreads();
    if (warp == 0) {
      int w = lane < THREADS / 32 ? warp_sums[lane] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        int t = __shfl_up_sync(0xffffffffu, w, o);
        if (lane >= o) w += t;
      }
      if (lane < THREADS / 32) warp_sums[lane] = w;  // inclusive
    }
    __syncthreads();
    const int carry = carry_s;
    int run = carry + (warp ? warp_sums[warp - 1] : 0) + incl - local;
    if (ITEMS % 4 == 0 && r_first + ITEMS <= rows &&
        (reinterpret_cast<uintptr_t>(slot_of_row + r_first) & 15u) == 0) {
      // 16-byte stores: a thread's results are consecutive, so scalar
      // stores would make every warp store instruction 32 partial sectors
#pragma unroll
      for (int i = 0; i < ITEMS; i += 4) {
        int4 o;
        o.x = flags[i] ? run : -1;
        run += flags[i];
        o.y = flags[i + 1] ? run : -1;
        run += flags[i + 1];
        o.z = flags[i + 2] ? run : -1;
        run += flags[i + 2];
        o.w = flags[i + 3] ? run : -1;
        run += flags[i + 3];
        *reinterpret_cast<int4*>(slot_of_row + r_first + i) = o;
      }
    } else {
#pragma unroll
      for (int i = 0; i < ITEMS; ++i) {
        const int64_t r = r_first + i;
        if (r < rows) slot_of_row[r] = flags[i] ? run : -1;
        run += flags[i];
      }
    }
    __syncthreads();
    if (tid == THREADS - 1) carry_s = run;
    __syncthreads();
  }
  if (tid == 0 && (int64_t)carry_s != num_slots) raise_error(0x8u);
}

struct RopeParams {
  const void* q;
  const void* k;
  const void* v;
  void* q_out;
  void* k_out;
  void* k_pool;
  void* v_pool;
  const int64_t* positions;
  int64_t pos_stride_b, pos_stride_s;
  const float* inv_freq;
  const int64_t* physical;
  const int64_t* offsets;
  const int32_t* slot_of_row;  // NULL: row r -> slot r
  int64_t num_slots;
  int64_t seq;
  int heads, kv_heads, dim;
  int64_t num_blocks;
  int block_size;
  int64_t num_rows;
  // Decode with device-resident metadata (tables != NULL, seq == 1): row b's
  // position and slot come from lengths[b] and its table row, see
  // resolve_row; positions / physical / offsets are unused.
  const int32_t* tables;
  int64_t table_width;
  int32_t* lengths;
  int advance;
  // Launched right after valid_scan_kernel (prefill with a valid mask): q, k,
  // v and positions were complete before the scan started, so the vectorised
  // kernel rotates q and k and stores q_out / k_out before its dependency
  // wait, and waits only before the slot writes, which need slot_of_row.
  int after_scan;
};

// Position of row r and the element offset of its pool slot (-1: no write).
// Given metadata: L = lengths[r]; the new token's position is L when the
// call advances the lengths (the first layer of a decode step, where
// lengths[r] then becomes L + 1, as PagedLlama.decode does with its host
// lengths, worker/llama.py:154-158), else L - 1 (later layers, lengths
// already count the token); its slot is (tables[r][pos / bs], pos % bs)
// (TensorPagedKV.slots, worker/llama.py:40-47). A length or position
// outside the table raises PDB_DEVERR_LENGTH, a page outside the pool
// PDB_DEVERR_TABLE_ENTRY; the row's write is then skipped.
// Without metadata: positions / physical / offsets / slot_of_row as given.
// Position of row r = (b, s) of the [batch, seq] input. Both entry points
// reject 2^31 rows or more, so b and s come from a 32-bit division.
__device__ __forceinline__ int64_t row_position(const RopeParams& p, int64_t r) {
  const uint32_t rr = (uint32_t)r, sq = (uint32_t)p.seq;
  const uint32_t bi = rr / sq, si = rr - bi * sq;
  return p.positions[(int64_t)bi * p.pos_stride_b + (int64_t)si * p.pos_stride_s];
}

// Slot of row r: its index among the valid rows (slot_of_row, -1 for a
// padding row), or r itself when every row is written.
__device__ __forceinline__ int64_t row_slot(const RopeParams& p, int64_t r) {
  return p.slot_of_row ? (int64_t)p.slot_of_row[r] : r;
}

// Element offset of the pool row at (physical block, offset), or -1 with
// PDB_DEVERR_SLOT raised when either lies outside the pool.
__device__ __forceinline__ long long slot_element_base(const RopeParams& p, int64_t phys,
                                                       int64_t off) {
  if (phys < 0 || phys >= p.num_blocks || off < 0 || off >= p.block_size) {
    raise_error(0x4u);
    return -1;
  }
  return (phys * p.block_size + off) * p.kv_heads * p.dim;
}

// Element offset of row r's pool slot (-1: no write). A slot beyond
// num_slots raises PDB_DEVERR_VALID_COUNT.
__device__ __forceinline__ long long resolve_slot(const RopeParams& p, int64_t r) {
  const int64_t slot = row_slot(p, r);
  if (slot < 0) return -1;
  if (slot >= p.num_slots) {
    raise_error(0x8u);
    return -1;
  }
  return slot_element_base(p, p.physical[slot], p.offsets[slot]);
}

__device__ __forceinline__ void resolve_row(const RopeParams& p, int64_t r, int64_t* pos_out,
                                            long long* base_out, int* len_out) {
  long long base = -1;
  int64_t pos = 0;
  if (p.tables) {
    const int L = p.lengths[r];
    *len_out = L;
    pos = p.advance ? (int64_t)L : (int64_t)L - 1;
    const int64_t cap = p.table_width * p.block_size;
    if (L < 0 || pos < 0 || pos >= cap) {
      raise_error(0x2u);
      pos = pos < 0 ? 0 : (pos >= cap ? cap - 1 : pos);
    } else {
      const int page = p.tables[r * p.table_width + pos / p.block_size];
      if (page < 0 || (int64_t)page >= p.num_blocks) {
        raise_error(0x1u);
      } else {
        base = ((int64_t)page * p.block_size + pos % p.block_size) * p.kv_heads * p.dim;
      }
    }
  } else {
    pos = row_position(p, r);
    base = resolve_slot(p, r);
  }
  *pos_out = pos;
  *base_out = base;
}

// cos and sin of an fp32 angle, as fp32 values destined for dtype T.
// sincosf is within 2 fp32 ulps. For FP16 the result is then rounded to 11
// bits; when either value lies within 2 ulps of an FP16 rounding boundary
// (rare) it is recomputed in double precision and rounded once to fp32, so
// the FP16 values equal those of correctly rounded fp32 cos/sin.
template <typename T>
__device__ __forceinline__ void rope_cos_sin(float ang, float* c, float* s) {
  sincosf(ang, s, c);
  if constexpr (sizeof(T) == 2) {
    auto near_boundary = [](float x) {
      const float d = fabsf(x) * 2.5e-7f + 1e-37f;
      return __float2half_rn(x - d) != __float2half_rn(x + d);
    };
    if (near_boundary(*c) || near_boundary(*s)) {
      *c = (float)cos((double)ang);
      *s = (float)sin((double)ang);
    }
  }
}

template <typename T>
__device__ __forceinline__ void rope_pair(const T* in, T* out, int j, int half,
                                          float c, float s) {
  // out[j]      = x[j]*c + (-x[j+half])*s
  // out[j+half] = x[j+half]*c + x[j]*s
  const float x1 = Elem<T>::to_f(in[j]);
  const float x2 = Elem<T>::to_f(in[j + half]);
  const T a = Elem<T>::from_f(__fmul_rn(x1, c));
  const T b = Elem<T>::from_f(__fmul_rn(x2, s));
  const T d = Elem<T>::from_f(__fmul_rn(x2, c));
  const T e = Elem<T>::from_f(__fmul_rn(x1, s));
  out[j] = Elem<T>::from_f(__fsub_rn(Elem<T>::to_f(a), Elem<T>::to_f(b)));
  out[j + half] = Elem<T>::from_f(__fadd_rn(Elem<T>::to_f(d), Elem<T>::to_f(e)));
}

// One CTA per row. cos/sin of the row's angles are computed once into shared
// memory (already rounded to the model dtype) and reused by all heads.
template <typename T>
__global__ void __launch_bounds__(128) rope_kv_write_kernel(RopeParams p) {
  grid_dependency_wait();
  launch_dependents();
  extern __shared__ float cs[];  // [2][dim/2]
  __shared__ long long row_pos, row_base;
  const int64_t r = blockIdx.x;
  const int half = p.dim >> 1;
  if (threadIdx.x == 0) {
    int64_t pos;
    long long base;
    int len = 0;
    resolve_row(p, r, &pos, &base, &len);
    row_pos = pos;
    row_base = base;
    if (p.tables && p.advance) p.lengths[r] = len + 1;  // only this thread reads it
  }
  __syncthreads();
  const float fpos = (float)row_pos;  // positions.float(): round-to-nearest
  for (int j = threadIdx.x; j < half; j += blockDim.x) {
    const float ang = __fmul_rn(fpos, p.inv_freq[j]);
    float c, s;
    rope_cos_sin<T>(ang, &c, &s);
    cs[j] = Elem<T>::to_f(Elem<T>::from_f(c));
    cs[half + j] = Elem<T>::to_f(Elem<T>::from_f(s));
  }
  __syncthreads();

  const long long base = row_base;  // destination slot of this row (or none)

  const T* q = static_cast<const T*>(p.q) + r * p.heads * p.dim;
  T* qo = static_cast<T*>(p.q_out) + r * p.heads * p.dim;
  const int qpairs = p.heads * half;
  for (int i = threadIdx.x; i < qpairs; i += blockDim.x) {
    const int h = i / half, j = i - h * half;
    rope_pair<T>(q + h * p.dim, qo + h * p.dim, j, half, cs[j], cs[half + j]);
  }

  const int64_t kv_row = r * p.kv_heads * p.dim;
  const T* k = static_cast<const T*>(p.k) + kv_row;
  T* ko = static_cast<T*>(p.k_out) + kv_row;
  const T* v = static_cast<const T*>(p.v) + kv_row;
  T* kslot = nullptr;
  T* vslot = nullptr;
  if (base >= 0) {
    kslot = static_cast<T*>(p.k_pool) + base;
    vslot = static_cast<T*>(p.v_pool) + base;
  }
  const int kpairs = p.kv_heads * half;
  for (int i = threadIdx.x; i < kpairs; i += blockDim.x) {
    const int h = i / half, j = i - h * half;
    T tmp[2];
    // rotate into registers first: k_out may alias k
    {
      const float c = cs[j], s = cs[half + j];
      const float x1 = Elem<T>::to_f(k[h * p.dim + j]);
      const float x2 = Elem<T>::to_f(k[h * p.dim + j + half]);
      const T a = Elem<T>::from_f(__fmul_rn(x1, c));
      const T b = Elem<T>::from_f(__fmul_rn(x2, s));
      const T d = Elem<T>::from_f(__fmul_rn(x2, c));
      const T e = Elem<T>::from_f(__fmul_rn(x1, s));
      tmp[0] = Elem<T>::from_f(__fsub_rn(Elem<T>::to_f(a), Elem<T>::to_f(b)));
      tmp[1] = Elem<T>::from_f(__fadd_rn(Elem<T>::to_f(d), Elem<T>::to_f(e)));
    }
    ko[h * p.dim + j] = tmp[0];
    ko[h * p.dim + j + half] = tmp[1];
    if (kslot) {
      kslot[h * p.dim + j] = tmp[0];
      kslot[h * p.dim + j + half] = tmp[1];
    }
  }
  if (vslot) {
    const int n = p.kv_heads * p.dim;
    for (int i = threadIdx.x; i < n; i += blockDim.x) vslot[i] = v[i];
  }
}

// Rotate the 16-byte chunk at element j0 of a row's first half and the
// matching chunk of its second half (rounding as rope_kv_write_kernel).
// FP16: packed half2 arithmetic. mul/add/sub.rn.f16x2 round the exact
// result once to FP16, which is what the per-op path does (the fp32 product
// of two FP16 values is exact, and an fp32 sum of two FP16 values rounds to
// the same FP16 value as the exact sum), so the results are bit-identical;
// the products must not be fused with the sum into one fma (one rounding),
// hence __hmul2_rn (measured: 0 of 4M random pairs differ; with contraction
// about 1 in 4 did).
// The rotated chunks are returned in o1 (first half) and o2 (second half).
template <typename T>
__device__ __forceinline__ void rope_chunk_pair(const T* in, int j0, int half, const float* cr,
                                                const float* sr, uint4& o1, uint4& o2);

template <>
__device__ __forceinline__ void rope_chunk_pair<__half>(const __half* in, int j0, int half,
                                                        const float* cr, const float* sr,
                                                        uint4& o1, uint4& o2) {
  const uint4 a = *reinterpret_cast<const uint4*>(in + j0);
  const uint4 b = *reinterpret_cast<const uint4*>(in + half + j0);
  const __half2* x1 = reinterpret_cast<const __half2*>(&a);
  const __half2* x2 = reinterpret_cast<const __half2*>(&b);
  __half2* t1 = reinterpret_cast<__half2*>(&o1);
  __half2* t2 = reinterpret_cast<__half2*>(&o2);
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    // cos/sin are FP16 values held as floats: the conversion is exact
    const __half2 c = __floats2half2_rn(cr[j0 + 2 * e], cr[j0 + 2 * e + 1]);
    const __half2 s = __floats2half2_rn(sr[j0 + 2 * e], sr[j0 + 2 * e + 1]);
    // __hmul2_rn: the products are never contracted into an fma with the sum
    t1[e] = __hsub2(__hmul2_rn(x1[e], c), __hmul2_rn(x2[e], s));
    t2[e] = __hadd2(__hmul2_rn(x2[e], c), __hmul2_rn(x1[e], s));
  }
}

template <>
__device__ __forceinline__ void rope_chunk_pair<float>(const float* in, int j0, int half,
                                                       const float* cr, const float* sr,
                                                       uint4& o1, uint4& o2) {
  float x1[4], x2[4];
  Chunk<float>::to_f(*reinterpret_cast<const uint4*>(in + j0), x1);
  Chunk<float>::to_f(*reinterpret_cast<const uint4*>(in + half + j0), x2);
  float* t1 = reinterpret_cast<float*>(&o1);
  float* t2 = reinterpret_cast<float*>(&o2);
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float cc = cr[j0 + e], ss = sr[j0 + e];
    t1[e] = __fsub_rn(__fmul_rn(x1[e], cc), __fmul_rn(x2[e], ss));
    t2[e] = __fadd_rn(__fmul_rn(x2[e], cc), __fmul_rn(x1[e], ss));
  }
}

template <typename T>
__device__ __forceinline__ void store_chunk_pair(T* out, int j0, int half, const uint4& o1,
                                                 const uint4& o2) {
  *reinterpret_cast<uint4*>(out + j0) = o1;
  *reinterpret_cast<uint4*>(out + half + j0) = o2;
}

// Vectorised variant: 16-byte loads and stores. Requires head_dim*e to be a
// multiple of 32 bytes (each half a whole number of 16-byte chunks) and
// 16-byte aligned q/k/v/outputs/pools. ROWS rows per CTA; per row, thread t
// owns chunk t of the row's (head, 16-byte column) grid and rotates the
// matching chunks of both halves. Rounding is identical to rope_kv_write_kernel.
template <typename T, int ROWS>
__global__ void __launch_bounds__(256) rope_kv_write_vec_kernel(RopeParams p) {
  if (!p.after_scan) grid_dependency_wait();  // inputs may come from the previous kernel
  launch_dependents();     // the attention kernel may start its set-up
  constexpr int VEC = 16 / (int)sizeof(T);
  extern __shared__ float cs[];  // [ROWS][2][dim/2]
  __shared__ long long slot_base[ROWS];
  __shared__ float row_fpos[ROWS];
  const int half = p.dim >> 1;
  const int hchunks = half / VEC;  // chunks per half-row of one head
  const int64_t r0 = (int64_t)blockIdx.x * ROWS;

  if (threadIdx.x < ROWS) {
    const int64_t r = r0 + threadIdx.x;
    long long base = -1;
    int64_t pos = 0;
    if (p.after_scan) {  // the slot is resolved after the dependency wait
      if (r < p.num_rows) pos = row_position(p, r);
    } else if (r < p.num_rows) {
      int len = 0;
      resolve_row(p, r, &pos, &base, &len);
      if (p.tables && p.advance) p.lengths[r] = len + 1;  // only this thread reads it
    }
    slot_base[threadIdx.x] = base;
    row_fpos[threadIdx.x] = (float)pos;  // positions.float(): round-to-nearest
  }
  __syncthreads();
  for (int i = threadIdx.x; i < ROWS * half; i += blockDim.x) {
    const int rr = i / half, j = i - rr * half;
    const int64_t r = r0 + rr;
    if (r >= p.num_rows) continue;
    const float fpos = row_fpos[rr];
    float c, s;
    rope_cos_sin<T>(__fmul_rn(fpos, p.inv_freq[j]), &c, &s);
    cs[(rr * 2) * half + j] = Elem<T>::to_f(Elem<T>::from_f(c));
    cs[(rr * 2 + 1) * half + j] = Elem<T>::to_f(Elem<T>::from_f(s));
  }
  __syncthreads();

  // Work items per row: q and k chunk pairs (one chunk of each half), then
  // the v row copied as 2*kchunks plain chunks.
  const int qchunks = p.heads * hchunks, kchunks = p.kv_heads * hchunks;
  if (p.after_scan) {
    // rotate q and k, store q_out / k_out; then, after the scan, the slots
    const int rot_row = qchunks + kchunks;
    for (int i = threadIdx.x; i < ROWS * rot_row; i += blockDim.x) {
      const int rr = i / rot_row, w = i - rr * rot_row;
      const int64_t r = r0 + rr;
      if (r >= p.num_rows) continue;
      const float* cr = cs + (rr * 2) * half;
      const float* sr = cr + half;
      const bool isq = w < qchunks;
      const int ww = isq ? w : w - qchunks;
      const int h = ww / hchunks, c = ww - h * hchunks;
      const int nh = isq ? p.heads : p.kv_heads;
      const T* in = static_cast<const T*>(isq ? p.q : p.k) + (r * nh + h) * p.dim;
      T* out = static_cast<T*>(isq ? p.q_out : p.k_out) + (r * nh + h) * p.dim;
      uint4 o1, o2;
      rope_chunk_pair<T>(in, c * VEC, half, cr, sr, o1, o2);
      store_chunk_pair<T>(out, c * VEC, half, o1, o2);
    }
    grid_dependency_wait();  // slot_of_row comes from the scan
    __syncthreads();         // every thread's k_out stores precede the slot copies
    if (threadIdx.x < ROWS) {
      const int64_t r = r0 + threadIdx.x;
      slot_base[threadIdx.x] = r < p.num_rows ? resolve_slot(p, r) : -1;
    }
    __syncthreads();
    // the rotated k row (from k_out) and the v row, each 2*kchunks chunks
    const int cp_row = 4 * kchunks;
    for (int i = threadIdx.x; i < ROWS * cp_row; i += blockDim.x) {
      const int rr = i / cp_row, w = i - rr * cp_row;
      const int64_t r = r0 + rr;
      if (r >= p.num_rows || slot_base[rr] < 0) continue;
      const bool isk = w < 2 * kchunks;
      const int c = isk ? w : w - 2 * kchunks;
      const T* src = static_cast<const T*>(isk ? p.k_out : p.v) + r * p.kv_heads * p.dim;
      T* dst = static_cast<T*>(isk ? p.k_pool : p.v_pool) + slot_base[rr];
      reinterpret_cast<uint4*>(dst)[c] = reinterpret_cast<const uint4*>(src)[c];
    }
    return;
  }
  const int per_row = qchunks + kchunks + 2 * kchunks;
  for (int i = threadIdx.x; i < ROWS * per_row; i += blockDim.x) {
    const int rr = i / per_row, w = i - rr * per_row;
    const int64_t r = r0 + rr;
    if (r >= p.num_rows) continue;
    const float* cr = cs + (rr * 2) * half;
    const float* sr = cr + half;
    if (w < qchunks + kchunks) {
      const bool isq = w < qchunks;
      const int ww = isq ? w : w - qchunks;
      const int h = ww / hchunks, c = ww - h * hchunks;
      const int nh = isq ? p.heads : p.kv_heads;
      const T* in = static_cast<const T*>(isq ? p.q : p.k) + (r * nh + h) * p.dim;
      T* out = static_cast<T*>(isq ? p.q_out : p.k_out) + (r * nh + h) * p.dim;
      const int j0 = c * VEC;
      uint4 o1, o2;
      rope_chunk_pair<T>(in, j0, half, cr, sr, o1, o2);
      store_chunk_pair<T>(out, j0, half, o1, o2);
      if (!isq && slot_base[rr] >= 0)
        store_chunk_pair<T>(static_cast<T*>(p.k_pool) + slot_base[rr] + h * p.dim, j0, half, o1,
                            o2);
    } else if (slot_base[rr] >= 0) {
      // v: copy the row's 2*kchunks 16-byte chunks to the slot unchanged
      const int c = w - qchunks - kchunks;  // 0 .. 2*kchunks-1 over the full row
      const T* vin = static_cast<const T*>(p.v) + r * p.kv_heads * p.dim;
      T* vs = static_cast<T*>(p.v_pool) + slot_base[rr];
      reinterpret_cast<uint4*>(vs)[c] = reinterpret_cast<const uint4*>(vin)[c];
    }
  }
}

// Prefill after the valid-mask scan, vectorised layouts: ROWS rows per CTA,
// each row owned by its own group of 8 / ROWS warps from start to end (one
// warp per row at 8 rows per CTA), so the phases of one row never wait for
// another row: the groups synchronise on their own named barrier (a warp
// barrier for single-warp groups), never on the whole CTA. A group stages its
// row's q, k and v into shared memory with cp.async at entry, so those loads
// are in flight while the row's position and cos/sin are computed; q and k
// are then rotated from shared memory and stored to q_out / k_out, the
// rotated k also back into shared memory. None of this needs the scan, so it
// runs before the dependency wait; after it, the row's slot is resolved and
// the rotated k and the v row are copied to it from shared memory.
// HQ, HK, DIM: the head counts and head_dim as compile-time constants for
// the common shapes (0: taken from p), which turns the index arithmetic's
// divisions into multiplications.
template <typename T, int ROWS, int HQ = 0, int HK = 0, int DIM = 0>
__global__ void __launch_bounds__(256) rope_prefill_vec_kernel(RopeParams p) {
  launch_dependents();
  constexpr int VEC = 16 / (int)sizeof(T);
  static_assert(ROWS >= 1 && 8 % ROWS == 0, "whole warp groups of the 256-thread CTA");
  constexpr int GT = 256 / ROWS;  // threads of a row's group
  extern __shared__ float cs[];   // [ROWS][2][dim/2], then the staged rows
  __shared__ long long slot_base[ROWS];
  __shared__ float row_fpos[ROWS];
  const int g = threadIdx.x / GT, gt = threadIdx.x % GT;
  auto group_sync = [&] {
    if constexpr (GT == 32) {
      __syncwarp();
    } else {
      asm volatile("bar.sync %0, %1;\n" ::"r"(1 + g), "r"(GT) : "memory");
    }
  };
  const int heads = HQ ? HQ : p.heads, kv_heads = HK ? HK : p.kv_heads;
  const int dim = DIM ? DIM : p.dim;
  const int half = dim >> 1, hchunks = half / VEC;
  const int qc = heads * dim / VEC, kc = kv_heads * dim / VEC;  // chunks per q / k row
  const int row_chunks = qc + 2 * kc;                                    // q, k, v
  uint4* stg = reinterpret_cast<uint4*>(cs + ROWS * dim) + (size_t)g * row_chunks;  // this row
  float* rcs = cs + g * dim;  // this row's cos [half], sin [half]
  const int64_t r = (int64_t)blockIdx.x * ROWS + g;
  if (r >= p.num_rows) return;  // the whole group: no barrier of it follows
  {
    const uint4* qs = static_cast<const uint4*>(p.q) + r * qc;
    const uint4* ks = static_cast<const uint4*>(p.k) + r * kc;
    const uint4* vs = static_cast<const uint4*>(p.v) + r * kc;
    for (int c = gt; c < qc; c += GT) cp_async16(stg + c, qs + c, true);
    for (int c = gt; c < kc; c += GT) {
      cp_async16(stg + qc + c, ks + c, true);
      cp_async16(stg + qc + kc + c, vs + c, true);
    }
  }
  cp_async_commit();
  if (gt == 0) row_fpos[g] = (float)row_position(p, r);  // positions.float(): round-to-nearest
  group_sync();
  for (int j = gt; j < half; j += GT) {
    float c, s;
    rope_cos_sin<T>(__fmul_rn(row_fpos[g], p.inv_freq[j]), &c, &s);
    rcs[j] = Elem<T>::to_f(Elem<T>::from_f(c));
    rcs[half + j] = Elem<T>::to_f(Elem<T>::from_f(s));
  }
  cp_async_wait<0>();
  group_sync();
  const int qpairs = heads * hchunks, rot_row = qpairs + kv_heads * hchunks;
  for (int w = gt; w < rot_row; w += GT) {
    const bool isq = w < qpairs;
    const int ww = isq ? w : w - qpairs;
    const int h = ww / hchunks, c = ww - h * hchunks;
    T* in = reinterpret_cast<T*>(stg + (isq ? 0 : qc)) + h * dim;
    T* out = isq ? static_cast<T*>(p.q_out) + (r * heads + h) * dim
                 : static_cast<T*>(p.k_out) + (r * kv_heads + h) * dim;
    uint4 o1, o2;
    rope_chunk_pair<T>(in, c * VEC, half, rcs, rcs + half, o1, o2);
    store_chunk_pair<T>(out, c * VEC, half, o1, o2);
    if (!isq) store_chunk_pair<T>(in, c * VEC, half, o1, o2);  // this thread's chunks only
  }
  grid_dependency_wait();  // slot_of_row comes from the scan
  if (gt == 0) slot_base[g] = resolve_slot(p, r);
  group_sync();  // the slot and the rotated k row in shared memory
  const long long base = slot_base[g];
  if (base < 0) return;
  for (int c = gt; c < 2 * kc; c += GT) {  // rotated k, then v
    const bool isk = c < kc;
    T* dst = static_cast<T*>(isk ? p.k_pool : p.v_pool) + base;
    reinterpret_cast<uint4*>(dst)[isk ? c : c - kc] = stg[qc + c];
  }
}

}  // namespace pdb
