// Shared device helpers for the paged-decode kernels (sm_100a).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace pdb {

// Per-device error word; bits are the PDB_DEVERR_* values of the C header.
// All kernels live in one translation unit, so a plain __device__ variable
// is visible to every kernel and to the host accessor.
__device__ unsigned int g_device_errors;

__device__ __forceinline__ void raise_error(unsigned bit) {
  atomicOr(&g_device_errors, bit);
}

// ---- programmatic dependent launch -----------------------------------------
// A kernel launched with programmatic stream serialization may start while
// the previous kernel in the stream is still running. It must call
// grid_dependency_wait() before it reads what that kernel writes or writes
// anything that kernel may touch; launch_dependents() lets the next kernel in
// the stream start its own independent set-up early. Both are no-ops for a
// kernel launched without the attribute.
__device__ __forceinline__ void grid_dependency_wait() {
  asm volatile("griddepcontrol.wait;\n" ::: "memory");
}
__device__ __forceinline__ void launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;\n" :::);
}

// ---- element conversion ---------------------------------------------------
template <typename T> struct Elem;
template <> struct Elem<float> {
  static __device__ __forceinline__ float to_f(float x) { return x; }
  static __device__ __forceinline__ float from_f(float x) { return x; }
};
template <> struct Elem<__half> {
  static __device__ __forceinline__ float to_f(__half x) { return __half2float(x); }
  static __device__ __forceinline__ __half from_f(float x) { return __float2half_rn(x); }
};

// Convert the 16-byte chunk `raw` holding 16/sizeof(T) elements to floats.
template <typename T> struct Chunk;
template <> struct Chunk<float> {
  static constexpr int N = 4;
  static __device__ __forceinline__ void to_f(const uint4& raw, float* f) {
    f[0] = __uint_as_float(raw.x); f[1] = __uint_as_float(raw.y);
    f[2] = __uint_as_float(raw.z); f[3] = __uint_as_float(raw.w);
  }
};
template <> struct Chunk<__half> {
  static constexpr int N = 8;
  static __device__ __forceinline__ void to_f(const uint4& raw, float* f) {
    const __half2* h = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 t = __half22float2(h[i]);
      f[2 * i] = t.x; f[2 * i + 1] = t.y;
    }
  }
};

// Load `n` consecutive elements (n*sizeof(T) in {2,4,8,16} bytes) from shared
// memory and convert to float.
template <typename T, int N>
__device__ __forceinline__ void lds_to_f(const T* p, float* f) {
  constexpr int BYTES = N * (int)sizeof(T);
  if constexpr (BYTES == 16) {
    uint4 r = *reinterpret_cast<const uint4*>(p);
    Chunk<T>::to_f(r, f);
  } else if constexpr (BYTES == 8) {
    uint2 r = *reinterpret_cast<const uint2*>(p);
    if constexpr (sizeof(T) == 2) {
      const __half2* h = reinterpret_cast<const __half2*>(&r);
      float2 a = __half22float2(h[0]), b = __half22float2(h[1]);
      f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y;
    } else {
      f[0] = __uint_as_float(r.x); f[1] = __uint_as_float(r.y);
    }
  } else if constexpr (BYTES == 4) {
    uint32_t r = *reinterpret_cast<const uint32_t*>(p);
    if constexpr (sizeof(T) == 2) {
      float2 a = __half22float2(*reinterpret_cast<const __half2*>(&r));
      f[0] = a.x; f[1] = a.y;
    } else {
      f[0] = __uint_as_float(r);
    }
  } else {
    static_assert(BYTES == 2, "unsupported width");
    f[0] = Elem<T>::to_f(*p);
  }
}

// ---- cp.async (16-byte, L2-only) -------------------------------------------
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc,
                                           bool valid) {
  const unsigned dst = static_cast<unsigned>(__cvta_generic_to_shared(smem_dst));
  const int src_bytes = valid ? 16 : 0;  // 0 => zero-fill, nothing is read
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst),
               "l"(gsrc), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;\n" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

// ---- work partition shared by host and device --------------------------------
// The fast kernel flattens the work of one call into "units" of 16 tokens,
// ordered by (sequence, kv_head, token). Sequence b contributes
// kv_heads * ceil(len_b / 16) units. CTA c < part_grid owns units
// [begin(c), begin(c+1)); CTAs beyond part_grid own nothing.
constexpr int kUnitTokens = 16;

// CTAs that take part: at most one per kMinUnitsPerCta units (a tiny batch is
// not shredded into many small pieces per segment) and at most `launched`;
// with begin(c) = c*total/grid every participating CTA owns >= 1 unit.
constexpr int64_t kMinUnitsPerCta = 16;
__host__ __device__ __forceinline__ int64_t part_grid(int64_t launched, int64_t total) {
  int64_t g = total / kMinUnitsPerCta;
  if (g < 1) g = 1;
  if (g > total) g = total;
  return launched < g ? launched : g;
}
__host__ __device__ __forceinline__ int64_t part_begin(int64_t c, int64_t total,
                                                       int64_t grid) {
  return (c * total) / grid;
}
// The CTA whose range contains unit u (largest c with begin(c) <= u).
__host__ __device__ __forceinline__ int64_t part_owner(int64_t u, int64_t total,
                                                       int64_t grid) {
  return ((u + 1) * grid + total - 1) / total - 1;
}

}  // namespace pdb
