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
// exact sum: 24 >= 2*11+2 bits). cos/sin are evaluated in double precision and
// rounded to fp32, i.e. correctly rounded.
#pragma once

#include "common.cuh"

namespace pdb {

// Exclusive scan of the valid mask: slot_of_row[r] = index of row r among the
// valid rows, or -1. One CTA; rows are processed in chunks of blockDim*ITEMS.
template <int THREADS, int ITEMS>
__global__ void __launch_bounds__(THREADS)
valid_scan_kernel(const uint8_t* __restrict__ valid, int64_t rows,
                  int64_t num_slots, int32_t* __restrict__ slot_of_row) {
  __shared__ int warp_sums[THREADS / 32];
  __shared__ int carry_s;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) carry_s = 0;
  __syncthreads();
  for (int64_t base = 0; base < rows; base += (int64_t)THREADS * ITEMS) {
    int flags[ITEMS];
    int local = 0;
#pragma unroll
    for (int i = 0; i < ITEMS; ++i) {
      const int64_t r = base + (int64_t)tid * ITEMS + i;
      flags[i] = (r < rows && valid[r]) ? 1 : 0;
      local += flags[i];
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
#pragma unroll
    for (int i = 0; i < ITEMS; ++i) {
      const int64_t r = base + (int64_t)tid * ITEMS + i;
      if (r < rows) slot_of_row[r] = flags[i] ? run : -1;
      run += flags[i];
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
};

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
  extern __shared__ float cs[];  // [2][dim/2]
  const int64_t r = blockIdx.x;
  const int half = p.dim >> 1;
  const int64_t bi = r / p.seq, si = r % p.seq;
  const int64_t pos = p.positions[bi * p.pos_stride_b + si * p.pos_stride_s];
  const float fpos = (float)pos;  // positions.float(): round-to-nearest
  for (int j = threadIdx.x; j < half; j += blockDim.x) {
    const float ang = __fmul_rn(fpos, p.inv_freq[j]);
    const double da = (double)ang;
    // correctly rounded fp32 cos/sin, then rounded to the model dtype
    cs[j] = Elem<T>::to_f(Elem<T>::from_f((float)cos(da)));
    cs[half + j] = Elem<T>::to_f(Elem<T>::from_f((float)sin(da)));
  }
  __syncthreads();

  // Destination slot of this row (or none).
  int64_t slot = p.slot_of_row ? (int64_t)p.slot_of_row[r] : r;
  int64_t phys = -1, off = 0;
  if (slot >= 0) {
    if (slot < p.num_slots) {
      phys = p.physical[slot];
      off = p.offsets[slot];
      if (phys < 0 || phys >= p.num_blocks || off < 0 || off >= p.block_size) {
        if (threadIdx.x == 0) raise_error(0x4u);
        phys = -1;
      }
    } else {
      if (threadIdx.x == 0) raise_error(0x8u);
    }
  }

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
  if (phys >= 0) {
    const int64_t base = (phys * p.block_size + off) * p.kv_heads * p.dim;
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

}  // namespace pdb
