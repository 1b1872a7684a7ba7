// C ABI of libpaged_decode_b200.so: argument checks, kernel selection,
// workspace layout and launches. Declarations: include/paged_decode_b200.h.
//
// All kernels are compiled in this one translation unit (the headers below),
// so the per-device error word is a single __device__ variable.
#include <atomic>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <map>
#include <type_traits>
#include <mutex>
#include <string>
#include <tuple>
#include <utility>

#include <cudaTypedefs.h>

#include "paged_decode_b200.h"
#include "attention.cuh"
#include "attention_tma.cuh"
#include "attention_dyn.cuh"
#include "rope_kv_write.cuh"
#include "prefill.cuh"
#include "prefill_tc.cuh"

namespace {

thread_local std::string g_last_error;

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

int cuda_fail(cudaError_t e, const char* where) {
  g_last_error = std::string(where) + ": " + cudaGetErrorString(e);
  return PDB_ERR_CUDA;
}

// ---- per-device facts -------------------------------------------------------
std::mutex g_mu;

int sm_count(int dev) {
  static std::map<int, int> cache;
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = cache.find(dev);
  if (it != cache.end()) return it->second;
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) n = 0;
  cache[dev] = n;
  return n;
}

// Occupancy (CTAs per SM) of `fn` with `smem` dynamic bytes on `dev`. The
// function's dynamic shared-memory limit is only ever raised (per device and
// function), so a launch with a smaller request never lowers the limit that
// an earlier, larger configuration relies on.
int ctas_per_sm(int dev, const void* fn, size_t smem, int threads) {
  static std::map<std::tuple<int, const void*, size_t>, int> cache;
  static std::map<std::pair<int, const void*>, size_t> limit;
  std::lock_guard<std::mutex> lk(g_mu);
  auto key = std::make_tuple(dev, fn, smem);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  size_t& cur = limit[std::make_pair(dev, fn)];
  if (smem > cur) {
    if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
        cudaSuccess) {
      cudaGetLastError();
      cache[key] = 0;
      return 0;
    }
    cur = smem;
  }
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, fn, threads, smem) != cudaSuccess) {
    cudaGetLastError();
    n = 0;
  }
  cache[key] = n;
  return n;
}


size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// 48-bit tag per call: a process salt plus a call counter, so that counter
// words left by other calls, processes or stale bytes do not match.
unsigned long long next_call_tag() {
  static std::atomic<unsigned long long> counter{0};
  static const unsigned long long salt = [] {
    unsigned long long x = (unsigned long long)std::chrono::high_resolution_clock::now()
                               .time_since_epoch().count();
    x ^= reinterpret_cast<uintptr_t>(&counter);
    x ^= x >> 33; x *= 0xff51afd7ed558ccdull; x ^= x >> 33;  // splitmix-style mixing
    return x;
  }();
  return (salt + 0x9e3779b97f4a7c15ull * (counter.fetch_add(1) + 1)) & ((1ull << 48) - 1);
}

// ---- stream-K kernel registry -----------------------------------------------
struct FastKernel {
  const void* fn;
  void (*launch)(const pdb::AttnParams&, int grid, size_t smem, cudaStream_t,
                 const CUtensorMap* kmap, const CUtensorMap* vmap);
  size_t (*smem)(int B);
  int gp;             // heads per kv head kept in partial slots
  int threads;        // CTA size
  bool tma;           // needs K/V tensor maps
  int slots_per_cta;  // partial slots per launched CTA
};

template <class M>
void launch_streamk(const pdb::AttnParams& p, int grid, size_t smem, cudaStream_t st,
                    const CUtensorMap*, const CUtensorMap*) {
  pdb::attn_streamk_kernel<M><<<grid, M::NT, smem, st>>>(p);
}

template <class M>
FastKernel make_fast() {
  return FastKernel{reinterpret_cast<const void*>(&pdb::attn_streamk_kernel<M>),
                    &launch_streamk<M>, &pdb::StreamK<M>::smem_bytes, M::GP, M::NT, false, 2};
}

// Launch with programmatic stream serialization: the kernel may begin while
// the previous kernel in the stream finishes (it waits on the device, with
// griddepcontrol, before touching that kernel's outputs).
template <typename... ExpT, typename... ActT>
cudaError_t launch_pdl(void (*kernel)(ExpT...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t st, ActT&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<ActT>(args)...);
}

template <class M>
void launch_tma(const pdb::AttnParams& p, int grid, size_t smem, cudaStream_t st,
                const CUtensorMap* kmap, const CUtensorMap* vmap) {
  launch_pdl(pdb::attn_tma_kernel<M>, dim3(grid), dim3(pdb::TmaStreamK<M>::NT), smem, st, p,
             *kmap, *vmap);
}

template <class M>
FastKernel make_tma() {
  return FastKernel{reinterpret_cast<const void*>(&pdb::attn_tma_kernel<M>), &launch_tma<M>,
                    &pdb::TmaStreamK<M>::smem_bytes, M::GP, pdb::TmaStreamK<M>::NT, true, 2};
}

template <class M>
void launch_dyn(const pdb::AttnParams& p, int grid, size_t smem, cudaStream_t st,
                const CUtensorMap* kmap, const CUtensorMap* vmap) {
  launch_pdl(pdb::attn_tma_dyn_kernel<M>, dim3(grid), dim3(pdb::DynStreamK<M>::NT), smem, st, p,
             *kmap, *vmap);
}

template <class M>
FastKernel make_dyn() {
  return FastKernel{reinterpret_cast<const void*>(&pdb::attn_tma_dyn_kernel<M>), &launch_dyn<M>,
                    &pdb::DynStreamK<M>::smem_bytes, M::GP, pdb::DynStreamK<M>::NT, true,
                    2 * (1 + pdb::kTailChunksPerCta)};
}

template <class M>
void launch_dyn_fused(const pdb::AttnParams& p, int grid, size_t smem, cudaStream_t st,
                      const CUtensorMap* kmap, const CUtensorMap* vmap) {
  launch_pdl(pdb::attn_tma_dyn_kernel<M, true>, dim3(grid), dim3(pdb::DynStreamK<M>::NT), smem,
             st, p, *kmap, *vmap);
}

template <class M>
FastKernel make_dyn_fused() {
  return FastKernel{reinterpret_cast<const void*>(&pdb::attn_tma_dyn_kernel<M, true>),
                    &launch_dyn_fused<M>, &pdb::DynStreamK<M>::smem_bytes, M::GP,
                    pdb::DynStreamK<M>::NT, true, 2 * (1 + pdb::kTailChunksPerCta)};
}

// cuTensorMapEncodeTiled from the driver (resolved once through the runtime,
// so the library needs no link-time dependency on libcuda).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess) {
      cudaGetLastError();
      ptr = nullptr;
    }
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }();
  return fn;
}

// Pool [N, bs, KVH, D] (FP16, or FP32 with esize 4) viewed as
// [N*bs rows, KVH, D]; box = one 16-token unit of one kv head, 128 bytes of
// columns (64 FP16 / 32 FP32 elements), 128-byte swizzle.
bool encode_pool_map(CUtensorMap* m, const void* pool, int64_t N, int64_t bs, int64_t KVH,
                     int64_t D, int esize = 2) {
  auto enc = tensor_map_encoder();
  if (!enc) return false;
  const cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)KVH, (cuuint64_t)(N * bs)};
  const cuuint64_t strides[2] = {(cuuint64_t)(D * esize), (cuuint64_t)(KVH * D * esize)};
  const cuuint32_t box[3] = {(cuuint32_t)(128 / esize), 1, (cuuint32_t)pdb::kUnitTokens};
  const cuuint32_t estr[3] = {1, 1, 1};
  return enc(m, esize == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
             const_cast<void*>(pool), dims, strides, box,
             estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Rows [R, heads, D] (FP16, e.g. a padded q batch [B, W, H, D] with R = B*W);
// box = `rows_box` rows of one head, 64 columns, 128-byte swizzle.
bool encode_rows_map(CUtensorMap* m, const void* base, int64_t R, int64_t heads, int64_t D,
                     int rows_box) {
  auto enc = tensor_map_encoder();
  if (!enc) return false;
  const cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)heads, (cuuint64_t)R};
  const cuuint64_t strides[2] = {(cuuint64_t)(D * 2), (cuuint64_t)(heads * D * 2)};
  const cuuint32_t box[3] = {64, 1, (cuuint32_t)rows_box};
  const cuuint32_t estr[3] = {1, 1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base), dims, strides, box,
             estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// SIMT inner loop: tile depth per (dtype, head_dim), ~16 KB (fp16) / 32 KB
// (fp32) per stage.
template <typename T, int D, int GP>
FastKernel simt_for() {
  if constexpr (sizeof(T) == 2) {
    if constexpr (D == 128) return make_fast<pdb::SimtMath<T, D, GP, 2, 4>>();
    else return make_fast<pdb::SimtMath<T, D, GP, 2, 6>>();
  } else {
    if constexpr (D == 128) return make_fast<pdb::SimtMath<T, D, GP, 2, 3>>();
    else if constexpr (D == 64) return make_fast<pdb::SimtMath<T, D, GP, 2, 4>>();
    else return make_fast<pdb::SimtMath<T, D, GP, 2, 6>>();
  }
}

template <typename T, int D>
bool pick_simt_gp(int G, FastKernel* out) {
  if (G <= 1) { *out = simt_for<T, D, 1>(); return true; }
  if (G <= 2) { *out = simt_for<T, D, 2>(); return true; }
  if (G <= 4) { *out = simt_for<T, D, 4>(); return true; }
  if constexpr (D <= 64) {
    if (G <= 8) { *out = simt_for<T, D, 8>(); return true; }
  }
  return false;
}

template <typename T>
bool pick_simt(int D, int G, FastKernel* out) {
  switch (D) {
    case 32: return pick_simt_gp<T, 32>(G, out);
    case 64: return pick_simt_gp<T, 64>(G, out);
    case 128: return pick_simt_gp<T, 128>(G, out);
    default: return false;
  }
}

// FP32: the SIMT inner loop in the TMA producer / dynamic-tail kernel
// (block_size % 16 == 0); 32 KB stages (64 tokens at head_dim 64, 32 at 128),
// three of them, so that two CTAs stay resident per SM. Measured at head_dim
// 64 (SmolLM2 shape, batch 64 / 256): 64-token tiles x 3 stages 0.445 / 0.629
// of the HBM peak, 32 x 6 0.407 / 0.529, 64 x 2 0.428 / 0.625.
template <int D, int GP>
FastKernel dyn_simt_f32() {
  if constexpr (D == 128) return make_dyn<pdb::SimtMath<float, D, GP, 2, 3, pdb::kTma128B>>();
  else return make_dyn<pdb::SimtMath<float, D, GP, 4, 3, pdb::kTma128B>>();
}
template <int D>
bool pick_dyn_f32_gp(int G, FastKernel* out) {
  if (G <= 1) { *out = dyn_simt_f32<D, 1>(); return true; }
  if (G <= 2) { *out = dyn_simt_f32<D, 2>(); return true; }
  if (G <= 4) { *out = dyn_simt_f32<D, 4>(); return true; }
  if constexpr (D <= 64) {
    if (G <= 8) { *out = dyn_simt_f32<D, 8>(); return true; }
  }
  return false;
}
// The same FP32 kernels with the decode prologue folded in (decode_attention).
template <int D, int GP>
FastKernel dyn_simt_f32_fused() {
  if constexpr (D == 128) return make_dyn_fused<pdb::SimtMath<float, D, GP, 2, 3, pdb::kTma128B>>();
  else return make_dyn_fused<pdb::SimtMath<float, D, GP, 4, 3, pdb::kTma128B>>();
}
template <int D>
bool pick_dyn_f32_fused_gp(int G, FastKernel* out) {
  if (G <= 1) { *out = dyn_simt_f32_fused<D, 1>(); return true; }
  if (G <= 2) { *out = dyn_simt_f32_fused<D, 2>(); return true; }
  if (G <= 4) { *out = dyn_simt_f32_fused<D, 4>(); return true; }
  if constexpr (D <= 64) {
    if (G <= 8) { *out = dyn_simt_f32_fused<D, 8>(); return true; }
  }
  return false;
}
bool pick_dyn_f32_fused(int D, int G, FastKernel* out) {
  switch (D) {
    case 64: return pick_dyn_f32_fused_gp<64>(G, out);
    case 128: return pick_dyn_f32_fused_gp<128>(G, out);
    default: return false;
  }
}

bool pick_dyn_f32(int D, int G, FastKernel* out) {
  switch (D) {
    case 64: return pick_dyn_f32_gp<64>(G, out);
    case 128: return pick_dyn_f32_gp<128>(G, out);
    default: return false;
  }
}

// Tensor-core inner loop, TMA producer warp and dynamic tail (FP16,
// block_size % 16 == 0). Stage depths keep two CTAs resident per SM.
bool pick_dyn_fused(int D, int G, FastKernel* out) {
  if (G > 8) return false;
  const bool g4 = G <= 4;
  if (D == 128) {
    *out = g4 ? make_dyn_fused<pdb::MmaMath<128, 4, 3, pdb::kTma128B>>()
              : make_dyn_fused<pdb::MmaMath<128, 8, 2, pdb::kTma128B>>();
    return true;
  }
  if (D == 64) {
    *out = g4 ? make_dyn_fused<pdb::MmaMath<64, 4, 3, pdb::kTma128B, 2>>()
              : make_dyn_fused<pdb::MmaMath<64, 8, 3, pdb::kTma128B, 2>>();
    return true;
  }
  return false;
}

bool pick_dyn(int D, int G, FastKernel* out) {
  if (G > 8) return false;
  const bool g4 = G <= 4;
  if (D == 128) {
    *out = g4 ? make_dyn<pdb::MmaMath<128, 4, 3, pdb::kTma128B>>()
              : make_dyn<pdb::MmaMath<128, 8, 2, pdb::kTma128B>>();
    return true;
  }
  if (D == 64) {
    *out = g4 ? make_dyn<pdb::MmaMath<64, 4, 3, pdb::kTma128B, 2>>()
              : make_dyn<pdb::MmaMath<64, 8, 3, pdb::kTma128B, 2>>();
    return true;
  }
  return false;
}

// Same with the static schedule only (two partial slots per CTA).
bool pick_tma(int D, int G, FastKernel* out) {
  if (G > 8) return false;
  const bool g4 = G <= 4;
  if (D == 128) {
    *out = g4 ? make_tma<pdb::MmaMath<128, 4, 3, pdb::kTma128B>>()
              : make_tma<pdb::MmaMath<128, 8, 2, pdb::kTma128B>>();
    return true;
  }
  if (D == 64) {
    *out = g4 ? make_tma<pdb::MmaMath<64, 4, 6, pdb::kTma128B>>()
              : make_tma<pdb::MmaMath<64, 8, 5, pdb::kTma128B>>();
    return true;
  }
  return false;
}

// Tensor-core inner loop (FP16): 64-token tiles (32 KB per stage at D 128).
bool pick_mma(int D, int G, FastKernel* out) {
  if (G > 8) return false;
  const bool g4 = G <= 4;
  if (D == 128) {
    *out = g4 ? make_fast<pdb::MmaMath<128, 4, 3>>() : make_fast<pdb::MmaMath<128, 8, 2>>();
    return true;
  }
  if (D == 64) {
    *out = g4 ? make_fast<pdb::MmaMath<64, 4, 4>>() : make_fast<pdb::MmaMath<64, 8, 4>>();
    return true;
  }
  return false;
}

constexpr int kFastMaxBatch = 4096;

bool streamk_shape_ok(int64_t B, int64_t KVH) {
  return B <= kFastMaxBatch && B * KVH * (8192 / pdb::kUnitTokens) < (int64_t(1) << 31);
}

// Kernel families a caller can pin (pdb_impl_t) below AUTO/FAST.
enum Family { kAny = 0, kSimtOnly = 1, kCpAsyncMma = 2, kStaticTma = 3 };

// The stream-K kernel for this shape: FP16 tensor cores fed by TMA when the
// pool allows (block_size % 16 == 0, rows addressable by 32-bit coordinates,
// driver encoder present), tensor cores fed by cp.async otherwise, the SIMT
// inner loop for FP32 and the remaining FP16 shapes. `bs`/`N` = 0 skips the
// TMA conditions (workspace sizing, where every candidate needs the same slots).
bool fast_applicable(int64_t B, int64_t H, int64_t KVH, int64_t D, int dtype, FastKernel* k,
                     int family = kAny, int64_t bs = 16, int64_t N = 1) {
  if (!streamk_shape_ok(B, KVH)) return false;
  const int G = (int)(H / KVH);
  const bool tma_ok = bs % pdb::kUnitTokens == 0 && N * bs < (int64_t(1) << 31) &&
                      tensor_map_encoder() != nullptr;
  if (dtype == PDB_DTYPE_FLOAT16) {
    if (family == kAny && tma_ok && pick_dyn((int)D, G, k)) return true;
    if (family == kStaticTma) return tma_ok && pick_tma((int)D, G, k);
    if (family != kSimtOnly && pick_mma((int)D, G, k)) return true;
    if (family == kCpAsyncMma) return false;
    return pick_simt<__half>((int)D, G, k);
  }
  if (family == kCpAsyncMma || family == kStaticTma) return false;
  if (family == kAny && tma_ok && pick_dyn_f32((int)D, G, k)) return true;
  return pick_simt<float>((int)D, G, k);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Grid of the fast kernel: one wave of resident CTAs, but never more CTAs
// than the upper bound on 16-token units.
int64_t fast_grid(int dev, const FastKernel& k, int64_t B, int64_t KVH, int64_t max_length) {
  const size_t smem = k.smem((int)B);
  const int occ = ctas_per_sm(dev, k.fn, smem, k.threads);
  const int sms = sm_count(dev);
  if (occ <= 0 || sms <= 0) return 0;
  int64_t grid = (int64_t)occ * sms;
  const int64_t units = B * KVH * ((max_length + pdb::kUnitTokens - 1) / pdb::kUnitTokens);
  if (grid > units) grid = units;
  return grid < 1 ? 1 : grid;
}

struct FastWs {
  size_t counters_off, partials_off, total;
};
// [arrival counters: B*KVH words + 1 tail-claim word][partial slots]
FastWs fast_ws_layout(int64_t B, int64_t KVH, int64_t D, const FastKernel& k, int64_t grid) {
  FastWs w;
  w.counters_off = 0;
  w.partials_off = align256((size_t)(B * KVH + 1) * sizeof(unsigned long long));
  w.total = w.partials_off +
            align256((size_t)(k.slots_per_cta * grid) * k.gp * (D + 2) * sizeof(float));
  return w;
}

int generic_splits(int64_t max_length) {
  int64_t s = (max_length + 511) / 512;
  if (s < 1) s = 1;
  if (s > 16) s = 16;
  return (int)s;
}
size_t generic_ws(int64_t B, int64_t H, int64_t D, int splits) {
  return splits > 1 ? align256((size_t)(B * H * splits) * (D + 2) * sizeof(float)) : 0;
}

int check_attention_args(int64_t B, int64_t H, int64_t D, int64_t N, int64_t bs, int64_t KVH,
                         int64_t Dk, int64_t W, int64_t max_length, int dtype) {
  // Messages and order of cuda/binding.cpp:14-22.
  if (!(B > 0 && H > 0 && D > 0 && D <= 256))
    return fail(PDB_ERR_INVALID_ARGUMENT, "invalid query shape");
  if (!(N > 0 && bs > 0 && KVH > 0 && Dk == D))
    return fail(PDB_ERR_INVALID_ARGUMENT, "invalid cache shape");
  if (H % KVH != 0)
    return fail(PDB_ERR_INVALID_ARGUMENT, "query heads must be a multiple of KV heads");
  if (dtype != PDB_DTYPE_FLOAT32 && dtype != PDB_DTYPE_FLOAT16)
    return fail(PDB_ERR_INVALID_ARGUMENT, "use FP32 or FP16");
  if (W < 0) return fail(PDB_ERR_INVALID_ARGUMENT, "invalid block tables");
  if (!(max_length > 0 && max_length <= 8192 && W * bs >= max_length))
    return fail(PDB_ERR_INVALID_ARGUMENT, "invalid context bound");
  if (B > INT32_MAX || H > INT32_MAX || N > INT64_MAX / (bs * KVH * D) ||
      W > INT32_MAX || bs > INT32_MAX)
    return fail(PDB_ERR_INVALID_ARGUMENT, "shape too large");
  return PDB_OK;
}

int current_device(int* dev) {
  cudaError_t e = cudaGetDevice(dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  return PDB_OK;
}

// ---- fixed scratch for callers that cannot allocate ------------------------
// Used only by pdb_paged_attention_noalloc. The array lives in this file, so
// every GPU that loads the library holds these bytes until the process exits.
constexpr size_t kNoAllocScratchBytes = size_t(2) << 20;  // 2 MiB
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of g_noalloc_scratch on device `dev` (which must be current).
// In host code the symbol is only a handle; the address comes from the
// runtime, once per device.
int noalloc_scratch(int dev, unsigned char** out) {
  static std::map<int, unsigned char*> cache;
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = cache.find(dev);
  if (it != cache.end()) {
    *out = it->second;
    return PDB_OK;
  }
  void* ptr = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(no-allocation scratch)");
  cache[dev] = static_cast<unsigned char*>(ptr);
  *out = static_cast<unsigned char*>(ptr);
  return PDB_OK;
}

// Launch the prologue over p.num_rows rows: the 16-byte vectorised kernel
// when each half head row is a whole number of 16-byte chunks and every
// row buffer is 16-byte aligned, else the scalar kernel.
int launch_rope(const pdb::RopeParams& p, int dtype, cudaStream_t st) {
  const int esize = dtype == PDB_DTYPE_FLOAT16 ? 2 : 4;
  const bool vec_ok = ((int64_t)p.dim * esize) % 32 == 0 && aligned16(p.q) && aligned16(p.k) &&
                      aligned16(p.v) && aligned16(p.q_out) && aligned16(p.k_out) &&
                      aligned16(p.k_pool) && aligned16(p.v_pool);
  if (vec_ok) {
    // 16-byte work items of one row (q and k chunk pairs, v chunks): with few
    // of them (small head counts) and many rows (prefill), 8 rows per CTA
    // keep the 256 threads busy and amortise each CTA's set-up.
    const int64_t per_row = (int64_t)(p.heads + 3 * p.kv_heads) * (p.dim / 2) * esize / 16;
    const bool wide = p.num_rows >= 2048 && per_row <= 128;
    auto go = [&](auto rows_tag) {
      constexpr int kRows = decltype(rows_tag)::value;
      const unsigned grid = (unsigned)((p.num_rows + kRows - 1) / kRows);
      const size_t smem = (size_t)kRows * p.dim * sizeof(float);
      // prefill after the scan: rows staged in shared memory (within the
      // default 48 KB of dynamic shared memory; larger rows take the kernel
      // that reads them from global memory)
      const size_t staged = smem + (size_t)kRows * (p.heads + 2 * p.kv_heads) * p.dim * esize;
      if (p.after_scan && staged <= 48 * 1024) {
        if (dtype == PDB_DTYPE_FLOAT16) {
          // compile-time shapes for the SmolLM2 and Llama-3-8B heads
          if (p.heads == 9 && p.kv_heads == 3 && p.dim == 64)
            launch_pdl(pdb::rope_prefill_vec_kernel<__half, kRows, 9, 3, 64>, dim3(grid),
                       dim3(256), staged, st, p);
          else if (p.heads == 32 && p.kv_heads == 8 && p.dim == 128)
            launch_pdl(pdb::rope_prefill_vec_kernel<__half, kRows, 32, 8, 128>, dim3(grid),
                       dim3(256), staged, st, p);
          else
            launch_pdl(pdb::rope_prefill_vec_kernel<__half, kRows>, dim3(grid), dim3(256),
                       staged, st, p);
        } else {
          launch_pdl(pdb::rope_prefill_vec_kernel<float, kRows>, dim3(grid), dim3(256), staged,
                     st, p);
        }
        return;
      }
      if (dtype == PDB_DTYPE_FLOAT16)
        launch_pdl(pdb::rope_kv_write_vec_kernel<__half, kRows>, dim3(grid), dim3(256), smem, st, p);
      else
        launch_pdl(pdb::rope_kv_write_vec_kernel<float, kRows>, dim3(grid), dim3(256), smem, st, p);
    };
    if (wide)
      go(std::integral_constant<int, 8>{});
    else
      go(std::integral_constant<int, 2>{});
  } else {
    const size_t smem = (size_t)p.dim * sizeof(float);
    if (dtype == PDB_DTYPE_FLOAT16)
      pdb::rope_kv_write_kernel<__half><<<(unsigned)p.num_rows, 128, smem, st>>>(p);
    else
      pdb::rope_kv_write_kernel<float><<<(unsigned)p.num_rows, 128, smem, st>>>(p);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "rope_kv_write launch");
  return PDB_OK;
}

}  // namespace

extern "C" {

const char* pdb_last_error(void) { return g_last_error.c_str(); }

const char* pdb_version(void) { return "paged_decode_b200 0.1 (sm_100a)"; }

size_t pdb_paged_attention_workspace_size(int64_t batch, int64_t heads, int64_t kv_heads,
                                          int64_t head_dim, int64_t max_length, int dtype) {
  if (batch <= 0 || heads <= 0 || kv_heads <= 0 || head_dim <= 0 || heads % kv_heads ||
      max_length <= 0)
    return 0;
  size_t need = generic_ws(batch, heads, head_dim, generic_splits(max_length));
  int dev = 0;
  if (!streamk_shape_ok(batch, kv_heads) || cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return need;
  }
  // The pool's block size is not known here, so cover every stream-K kernel
  // that a call of this shape may select.
  const int G = (int)(heads / kv_heads);
  FastKernel cand[4];
  int n = 0;
  if (dtype == PDB_DTYPE_FLOAT16) {
    if (tensor_map_encoder() && pick_dyn((int)head_dim, G, &cand[n])) ++n;
    if (tensor_map_encoder() && pick_tma((int)head_dim, G, &cand[n])) ++n;
    if (pick_mma((int)head_dim, G, &cand[n])) ++n;
    if (pick_simt<__half>((int)head_dim, G, &cand[n])) ++n;
  } else {
    if (tensor_map_encoder() && pick_dyn_f32((int)head_dim, G, &cand[n])) ++n;
    if (pick_simt<float>((int)head_dim, G, &cand[n])) ++n;
  }
  for (int i = 0; i < n; ++i) {
    const int64_t grid = fast_grid(dev, cand[i], batch, kv_heads, max_length);
    if (grid > 0) {
      const size_t f = fast_ws_layout(batch, kv_heads, head_dim, cand[i], grid).total;
      if (f > need) need = f;
    }
  }
  return need;
}

int64_t pdb_fast_grid_size(int64_t batch, int64_t heads, int64_t kv_heads, int64_t head_dim,
                           int dtype) {
  FastKernel k;
  int dev = 0;
  if (batch <= 0 || kv_heads <= 0 || heads % kv_heads) return 0;
  if (!fast_applicable(batch, heads, kv_heads, head_dim, dtype, &k)) return 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  return fast_grid(dev, k, batch, kv_heads, 8192);
}

int pdb_paged_attention_impl(const void* q, const void* k_pool, const void* v_pool,
                             const int32_t* tables, const int32_t* lengths, void* out,
                             int64_t B, int64_t H, int64_t D, int64_t N, int64_t bs,
                             int64_t KVH, int64_t Dk, int64_t W, int64_t max_length,
                             int dtype, void* workspace, size_t workspace_bytes, void* stream,
                             int impl) {
  int rc = check_attention_args(B, H, D, N, bs, KVH, Dk, W, max_length, dtype);
  if (rc) return rc;
  if (!q || !k_pool || !v_pool || !tables || !lengths || !out)
    return fail(PDB_ERR_INVALID_ARGUMENT, "null tensor pointer");
  if (impl < PDB_IMPL_AUTO || impl > PDB_IMPL_TMA_STATIC)
    return fail(PDB_ERR_INVALID_ARGUMENT, "unknown kernel selection");
  int dev = 0;
  if ((rc = current_device(&dev))) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);

  pdb::AttnParams p{};
  p.q = q; p.k_pool = k_pool; p.v_pool = v_pool;
  p.tables = tables; p.lengths = lengths; p.out = out;
  p.B = (int)B; p.H = (int)H; p.KVH = (int)KVH; p.G = (int)(H / KVH); p.D = (int)D;
  p.num_blocks = N; p.block_size = (int)bs;
  p.bs_shift = ((bs & (bs - 1)) == 0) ? __builtin_ctzll((unsigned long long)bs) : -1;
  p.table_width = (int)W;
  p.max_length = (int)max_length;
  p.scale_log2 = (float)(1.4426950408889634 / std::sqrt((double)D));

  if (workspace && (reinterpret_cast<uintptr_t>(workspace) & 255u))
    return fail(PDB_ERR_WORKSPACE, "workspace must be 256-byte aligned");

  FastKernel fk;
  const int family = impl == PDB_IMPL_SIMT         ? kSimtOnly
                     : impl == PDB_IMPL_MMA        ? kCpAsyncMma
                     : impl == PDB_IMPL_TMA_STATIC ? kStaticTma
                                                   : kAny;
  const bool fast_ok = fast_applicable(B, H, KVH, D, dtype, &fk, family, bs, N) &&
                       aligned16(q) && aligned16(k_pool) && aligned16(v_pool);
  if (impl != PDB_IMPL_AUTO && impl != PDB_IMPL_GENERIC && !fast_ok)
    return fail(PDB_ERR_INVALID_ARGUMENT, "fast kernel does not support this shape/alignment");

  if (fast_ok && impl != PDB_IMPL_GENERIC) {
    const int64_t grid = fast_grid(dev, fk, B, KVH, max_length);
    if (grid <= 0) return fail(PDB_ERR_CUDA, "fast kernel cannot be resident on this device");
    const FastWs ws = fast_ws_layout(B, KVH, D, fk, grid);
    if (!workspace || workspace_bytes < ws.total)
      return fail(PDB_ERR_WORKSPACE, "workspace too small: need " + std::to_string(ws.total) +
                                         " bytes");
    unsigned char* wb = static_cast<unsigned char*>(workspace);
    p.counters = reinterpret_cast<unsigned long long*>(wb + ws.counters_off);
    p.partials = reinterpret_cast<float*>(wb + ws.partials_off);
    p.call_tag = next_call_tag();
    p.q_row = H * D;
    p.bulk_q = aligned16(q) && (H * D) % 8 == 0;
    CUtensorMap kmap, vmap;
    const int esize = dtype == PDB_DTYPE_FLOAT32 ? 4 : 2;
    if (fk.tma && !(encode_pool_map(&kmap, k_pool, N, bs, KVH, D, esize) &&
                    encode_pool_map(&vmap, v_pool, N, bs, KVH, D, esize)))
      return fail(PDB_ERR_CUDA, "cuTensorMapEncodeTiled failed for the KV pools");
    fk.launch(p, (int)grid, fk.smem((int)B), st, &kmap, &vmap);
  } else {
    const int splits = generic_splits(max_length);
    const size_t need = generic_ws(B, H, D, splits);
    if (need && (!workspace || workspace_bytes < need))
      return fail(PDB_ERR_WORKSPACE, "workspace too small: need " + std::to_string(need) +
                                         " bytes");
    p.splits = splits;
    p.chunk = (int)((max_length + splits - 1) / splits);
    p.partials = static_cast<float*>(workspace);
    dim3 grid(splits, (unsigned)H, (unsigned)B);
    if (dtype == PDB_DTYPE_FLOAT16) {
      pdb::attn_generic_kernel<__half><<<grid, 128, 0, st>>>(p);
      if (splits > 1) pdb::attn_combine_kernel<__half><<<dim3((unsigned)H, (unsigned)B), 128, 0, st>>>(p);
    } else {
      pdb::attn_generic_kernel<float><<<grid, 128, 0, st>>>(p);
      if (splits > 1) pdb::attn_combine_kernel<float><<<dim3((unsigned)H, (unsigned)B), 128, 0, st>>>(p);
    }
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "paged_attention launch");
  return PDB_OK;
}

int pdb_paged_attention_noalloc(const void* q, const void* k_pool, const void* v_pool,
                                const int32_t* tables, const int32_t* lengths, void* out,
                                int64_t B, int64_t H, int64_t D, int64_t N, int64_t bs,
                                int64_t KVH, int64_t Dk, int64_t W, int64_t max_length,
                                int dtype, void* stream) {
  int rc = check_attention_args(B, H, D, N, bs, KVH, Dk, W, max_length, dtype);
  if (rc) return rc;
  if (!q || !k_pool || !v_pool || !tables || !lengths || !out)
    return fail(PDB_ERR_INVALID_ARGUMENT, "null tensor pointer");
  int dev = 0;
  if ((rc = current_device(&dev))) return rc;
  FastKernel fk;
  const bool fits = fast_applicable(B, H, KVH, D, dtype, &fk, kStaticTma, bs, N) ||
                    fast_applicable(B, H, KVH, D, dtype, &fk, kCpAsyncMma, bs, N) ||
                    fast_applicable(B, H, KVH, D, dtype, &fk, kSimtOnly, bs, N);
  if (!(fits && aligned16(q) && aligned16(k_pool) && aligned16(v_pool)))
    return fail(PDB_ERR_INVALID_ARGUMENT,
                "pdb_paged_attention_noalloc: shape or alignment needs the generic kernel; "
                "use pdb_paged_attention with a workspace");
  const int64_t grid = fast_grid(dev, fk, B, KVH, max_length);
  if (grid <= 0) return fail(PDB_ERR_CUDA, "fast kernel cannot be resident on this device");
  const FastWs ws = fast_ws_layout(B, KVH, D, fk, grid);
  if (ws.total > kNoAllocScratchBytes)
    return fail(PDB_ERR_WORKSPACE,
                "pdb_paged_attention_noalloc: this shape needs " + std::to_string(ws.total) +
                    " bytes of scratch, above the fixed maximum of " +
                    std::to_string(kNoAllocScratchBytes) + " bytes");
  unsigned char* scratch = nullptr;
  if ((rc = noalloc_scratch(dev, &scratch))) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);

  pdb::AttnParams p{};
  p.q = q; p.k_pool = k_pool; p.v_pool = v_pool;
  p.tables = tables; p.lengths = lengths; p.out = out;
  p.B = (int)B; p.H = (int)H; p.KVH = (int)KVH; p.G = (int)(H / KVH); p.D = (int)D;
  p.num_blocks = N; p.block_size = (int)bs;
  p.bs_shift = ((bs & (bs - 1)) == 0) ? __builtin_ctzll((unsigned long long)bs) : -1;
  p.table_width = (int)W;
  p.max_length = (int)max_length;
  p.scale_log2 = (float)(1.4426950408889634 / std::sqrt((double)D));
  p.counters = reinterpret_cast<unsigned long long*>(scratch + ws.counters_off);
  p.partials = reinterpret_cast<float*>(scratch + ws.partials_off);
  p.call_tag = next_call_tag();
  // The shared array keeps the previous call's bytes: the arrival counters
  // must read zero for this call (stream-ordered clear, nothing allocated).
  cudaError_t e = cudaMemsetAsync(p.counters, 0, (size_t)(B * KVH) * sizeof(unsigned long long), st);
  if (e != cudaSuccess) return cuda_fail(e, "clear no-allocation scratch");
  CUtensorMap kmap, vmap;
  if (fk.tma && !(encode_pool_map(&kmap, k_pool, N, bs, KVH, D) &&
                  encode_pool_map(&vmap, v_pool, N, bs, KVH, D)))
    return fail(PDB_ERR_CUDA, "cuTensorMapEncodeTiled failed for the KV pools");
  fk.launch(p, (int)grid, fk.smem((int)B), st, &kmap, &vmap);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "paged_attention_noalloc launch");
  return PDB_OK;
}

int pdb_paged_attention(const void* q, const void* k_pool, const void* v_pool,
                        const int32_t* tables, const int32_t* lengths, void* out, int64_t B,
                        int64_t H, int64_t D, int64_t N, int64_t bs, int64_t KVH, int64_t Dk,
                        int64_t W, int64_t max_length, int dtype, void* workspace,
                        size_t workspace_bytes, void* stream) {
  return pdb_paged_attention_impl(q, k_pool, v_pool, tables, lengths, out, B, H, D, N, bs, KVH,
                                  Dk, W, max_length, dtype, workspace, workspace_bytes, stream,
                                  PDB_IMPL_AUTO);
}

size_t pdb_rope_kv_write_workspace_size(int64_t batch, int64_t seq, int has_valid) {
  if (!has_valid || batch <= 0 || seq <= 0) return 0;
  return align256((size_t)(batch * seq) * sizeof(int32_t));
}

int pdb_rope_kv_write(const void* q, const void* k, const void* v, void* q_out, void* k_out,
                      void* k_pool, void* v_pool, const int64_t* positions,
                      int64_t pos_stride_b, int64_t pos_stride_s, const float* inv_freq,
                      const int64_t* physical, const int64_t* offsets, int64_t num_slots,
                      const uint8_t* valid, int64_t batch, int64_t seq, int64_t heads,
                      int64_t kv_heads, int64_t head_dim, int64_t num_blocks,
                      int64_t block_size, int dtype, void* workspace, size_t workspace_bytes,
                      void* stream) {
  if (!(batch > 0 && seq > 0 && heads > 0 && kv_heads > 0 && head_dim > 0))
    return fail(PDB_ERR_INVALID_ARGUMENT, "invalid q/k/v shapes");
  if (head_dim % 2)
    return fail(PDB_ERR_INVALID_ARGUMENT, "head_dim must be even for rotate-half RoPE");
  if (!(num_blocks > 0 && block_size > 0))
    return fail(PDB_ERR_INVALID_ARGUMENT, "invalid cache shape");
  if (dtype != PDB_DTYPE_FLOAT32 && dtype != PDB_DTYPE_FLOAT16)
    return fail(PDB_ERR_INVALID_ARGUMENT, "use FP32 or FP16");
  const int64_t rows = batch * seq;
  if (num_slots < 0 || (!valid && num_slots != rows))
    return fail(PDB_ERR_INVALID_ARGUMENT, "number of slots must match the rows written");
  if (rows > INT32_MAX || heads * head_dim > INT32_MAX || kv_heads * head_dim > INT32_MAX)
    return fail(PDB_ERR_INVALID_ARGUMENT, "shape too large");
  if (!q || !k || !v || !q_out || !k_out || !k_pool || !v_pool || !positions || !inv_freq ||
      (num_slots > 0 && (!physical || !offsets)))
    return fail(PDB_ERR_INVALID_ARGUMENT, "null tensor pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);

  const int32_t* slot_of_row = nullptr;
  if (valid) {
    const size_t need = pdb_rope_kv_write_workspace_size(batch, seq, 1);
    if (!workspace || workspace_bytes < need)
      return fail(PDB_ERR_WORKSPACE, "workspace too small: need " + std::to_string(need) +
                                         " bytes");
    int32_t* sor = static_cast<int32_t*>(workspace);
    // Programmatic launch: the scan becomes resident while the previous
    // kernel drains and waits for it (griddepcontrol.wait) before it reads
    // the mask or overwrites slot_of_row, which that kernel may still read.
    const cudaError_t le =
        launch_pdl(pdb::valid_scan_kernel<1024, 16>, dim3(1), dim3(1024), 0, st, valid, rows,
                   num_slots, sor);
    if (le != cudaSuccess) return cuda_fail(le, "valid_scan launch");
    slot_of_row = sor;
  }
  pdb::RopeParams p{};
  p.q = q; p.k = k; p.v = v; p.q_out = q_out; p.k_out = k_out;
  p.k_pool = k_pool; p.v_pool = v_pool;
  p.positions = positions; p.pos_stride_b = pos_stride_b; p.pos_stride_s = pos_stride_s;
  p.inv_freq = inv_freq; p.physical = physical; p.offsets = offsets;
  p.slot_of_row = slot_of_row; p.num_slots = num_slots; p.seq = seq;
  p.heads = (int)heads; p.kv_heads = (int)kv_heads; p.dim = (int)head_dim;
  p.num_blocks = num_blocks; p.block_size = (int)block_size;
  p.num_rows = rows;
  p.after_scan = valid ? 1 : 0;
  return launch_rope(p, dtype, st);
}

int pdb_rope_kv_write_decode(const void* q, const void* k, const void* v, void* q_out,
                             void* k_out, void* k_pool, void* v_pool, const int32_t* tables,
                             int64_t table_width, int32_t* lengths, int advance,
                             const float* inv_freq, int64_t batch, int64_t heads,
                             int64_t kv_heads, int64_t head_dim, int64_t num_blocks,
                             int64_t block_size, int dtype, void* stream) {
  if (!(batch > 0 && heads > 0 && kv_heads > 0 && head_dim > 0))
    return fail(PDB_ERR_INVALID_ARGUMENT, "invalid q/k/v shapes");
  if (head_dim % 2)
    return fail(PDB_ERR_INVALID_ARGUMENT, "head_dim must be even for rotate-half RoPE");
  if (!(num_blocks > 0 && block_size > 0))
    return fail(PDB_ERR_INVALID_ARGUMENT, "invalid cache shape");
  if (table_width <= 0) return fail(PDB_ERR_INVALID_ARGUMENT, "invalid table width");
  if (dtype != PDB_DTYPE_FLOAT32 && dtype != PDB_DTYPE_FLOAT16)
    return fail(PDB_ERR_INVALID_ARGUMENT, "use FP32 or FP16");
  if (batch > INT32_MAX || heads * head_dim > INT32_MAX || kv_heads * head_dim > INT32_MAX ||
      table_width * block_size > INT32_MAX)
    return fail(PDB_ERR_INVALID_ARGUMENT, "shape too large");
  if (!q || !k || !v || !q_out || !k_out || !k_pool || !v_pool || !tables || !lengths ||
      !inv_freq)
    return fail(PDB_ERR_INVALID_ARGUMENT, "null tensor pointer");
  pdb::RopeParams p{};
  p.q = q; p.k = k; p.v = v; p.q_out = q_out; p.k_out = k_out;
  p.k_pool = k_pool; p.v_pool = v_pool;
  p.inv_freq = inv_freq;
  p.seq = 1;
  p.heads = (int)heads; p.kv_heads = (int)kv_heads; p.dim = (int)head_dim;
  p.num_blocks = num_blocks; p.block_size = (int)block_size;
  p.num_rows = batch;
  p.tables = tables; p.table_width = table_width; p.lengths = lengths;
  p.advance = advance ? 1 : 0;
  return launch_rope(p, dtype, static_cast<cudaStream_t>(stream));
}

int pdb_read_device_errors(uint32_t* flags, int clear) {
  if (!flags) return fail(PDB_ERR_INVALID_ARGUMENT, "null output pointer");
  unsigned v = 0;
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceSynchronize");
  e = cudaMemcpyFromSymbol(&v, pdb::g_device_errors, sizeof(v));
  if (e != cudaSuccess) return cuda_fail(e, "read error word");
  if (clear) {
    const unsigned zero = 0;
    e = cudaMemcpyToSymbol(pdb::g_device_errors, &zero, sizeof(zero));
    if (e != cudaSuccess) return cuda_fail(e, "clear error word");
  }
  *flags = v;
  return PDB_OK;
}

int pdb_decode_attention_supported(int64_t batch, int64_t heads, int64_t kv_heads,
                                   int64_t head_dim, int64_t num_blocks, int64_t block_size,
                                   int dtype) {
  FastKernel fk;
  if ((dtype != PDB_DTYPE_FLOAT16 && dtype != PDB_DTYPE_FLOAT32) || batch <= 0 ||
      kv_heads <= 0 || heads % kv_heads)
    return 0;
  const bool tma_ok = block_size % pdb::kUnitTokens == 0 &&
                      num_blocks * block_size < (int64_t(1) << 31) &&
                      tensor_map_encoder() != nullptr;
  const int G = (int)(heads / kv_heads);
  return streamk_shape_ok(batch, kv_heads) && tma_ok &&
         (dtype == PDB_DTYPE_FLOAT16 ? pick_dyn_fused((int)head_dim, G, &fk)
                                     : pick_dyn_f32_fused((int)head_dim, G, &fk));
}

int pdb_decode_attention(const void* q, const void* k_new, const void* v_new, void* k_pool,
                         void* v_pool, const int32_t* tables, const int32_t* lengths,
                         const float* inv_freq, void* out, int64_t B, int64_t H, int64_t D,
                         int64_t N, int64_t bs, int64_t KVH, int64_t W, int64_t max_length,
                         int64_t q_row_stride, int64_t kv_row_stride, int dtype,
                         void* workspace, size_t workspace_bytes, void* stream) {
  return pdb_decode_attention_ex(q, k_new, v_new, k_pool, v_pool, tables, lengths, inv_freq, out,
                                 B, H, D, N, bs, KVH, W, max_length, q_row_stride, kv_row_stride,
                                 dtype, workspace, workspace_bytes, stream, 0u);
}

int pdb_decode_attention_ex(const void* q, const void* k_new, const void* v_new, void* k_pool,
                            void* v_pool, const int32_t* tables, const int32_t* lengths,
                            const float* inv_freq, void* out, int64_t B, int64_t H, int64_t D,
                            int64_t N, int64_t bs, int64_t KVH, int64_t W, int64_t max_length,
                            int64_t q_row_stride, int64_t kv_row_stride, int dtype,
                            void* workspace, size_t workspace_bytes, void* stream,
                            unsigned flags) {
  if (flags & ~(unsigned)(PDB_DECODE_STABLE_METADATA | PDB_DECODE_STABLE_POOLS))
    return fail(PDB_ERR_INVALID_ARGUMENT, "unknown decode attention flags");
  if ((flags & PDB_DECODE_STABLE_POOLS) && !(flags & PDB_DECODE_STABLE_METADATA))
    return fail(PDB_ERR_INVALID_ARGUMENT,
                "PDB_DECODE_STABLE_POOLS requires PDB_DECODE_STABLE_METADATA");
  int rc = check_attention_args(B, H, D, N, bs, KVH, D, W, max_length, dtype);
  if (rc) return rc;
  if (!q || !k_new || !v_new || !k_pool || !v_pool || !tables || !lengths || !inv_freq || !out)
    return fail(PDB_ERR_INVALID_ARGUMENT, "null tensor pointer");
  if (!pdb_decode_attention_supported(B, H, KVH, D, N, bs, dtype) || !aligned16(k_pool) ||
      !aligned16(v_pool) || (reinterpret_cast<uintptr_t>(q) & 3u))
    return fail(PDB_ERR_INVALID_ARGUMENT,
                "fused decode attention does not support this shape/alignment");
  const int64_t q_row = q_row_stride ? q_row_stride : H * D;
  const int64_t kv_row = kv_row_stride ? kv_row_stride : KVH * D;
  if (q_row < H * D || kv_row < KVH * D || (q_row & 1))
    return fail(PDB_ERR_INVALID_ARGUMENT, "invalid row strides");
  const int esize = dtype == PDB_DTYPE_FLOAT16 ? 2 : 4;
  const int per16 = 16 / esize;  // elements per 16-byte chunk
  // FP32 rotates q, k and v in 16-byte chunks: rows 16-byte aligned
  if (dtype == PDB_DTYPE_FLOAT32 && !(aligned16(q) && aligned16(k_new) && aligned16(v_new) &&
                                      q_row % per16 == 0 && kv_row % per16 == 0))
    return fail(PDB_ERR_INVALID_ARGUMENT,
                "fused FP32 decode attention needs 16-byte aligned q, k and v rows");
  if (workspace && (reinterpret_cast<uintptr_t>(workspace) & 255u))
    return fail(PDB_ERR_WORKSPACE, "workspace must be 256-byte aligned");
  int dev = 0;
  if ((rc = current_device(&dev))) return rc;
  FastKernel fk;
  if (dtype == PDB_DTYPE_FLOAT16)
    pick_dyn_fused((int)D, (int)(H / KVH), &fk);
  else
    pick_dyn_f32_fused((int)D, (int)(H / KVH), &fk);
  const int64_t grid = fast_grid(dev, fk, B, KVH, max_length);
  if (grid <= 0) return fail(PDB_ERR_CUDA, "fast kernel cannot be resident on this device");
  const FastWs ws = fast_ws_layout(B, KVH, D, fk, grid);
  if (!workspace || workspace_bytes < ws.total)
    return fail(PDB_ERR_WORKSPACE, "workspace too small: need " + std::to_string(ws.total) +
                                       " bytes");
  pdb::AttnParams p{};
  p.q = q; p.k_pool = k_pool; p.v_pool = v_pool;
  p.tables = tables; p.lengths = lengths; p.out = out;
  p.B = (int)B; p.H = (int)H; p.KVH = (int)KVH; p.G = (int)(H / KVH); p.D = (int)D;
  p.num_blocks = N; p.block_size = (int)bs;
  p.bs_shift = ((bs & (bs - 1)) == 0) ? __builtin_ctzll((unsigned long long)bs) : -1;
  p.table_width = (int)W;
  p.max_length = (int)max_length;
  p.scale_log2 = (float)(1.4426950408889634 / std::sqrt((double)D));
  unsigned char* wb = static_cast<unsigned char*>(workspace);
  p.counters = reinterpret_cast<unsigned long long*>(wb + ws.counters_off);
  p.partials = reinterpret_cast<float*>(wb + ws.partials_off);
  p.call_tag = next_call_tag();
  p.k_new = k_new;
  p.v_new = v_new;
  p.inv_freq = inv_freq;
  p.stable_meta = ((flags & PDB_DECODE_STABLE_METADATA) ? 1 : 0) |
                  ((flags & PDB_DECODE_STABLE_POOLS) ? 2 : 0);
  p.q_row = q_row;
  p.kv_row = kv_row;
  p.bulk_q = aligned16(q) && q_row % per16 == 0 && aligned16(k_new) && aligned16(v_new) &&
             kv_row % per16 == 0;
  CUtensorMap kmap, vmap;
  if (!(encode_pool_map(&kmap, k_pool, N, bs, KVH, D, esize) &&
        encode_pool_map(&vmap, v_pool, N, bs, KVH, D, esize)))
    return fail(PDB_ERR_CUDA, "cuTensorMapEncodeTiled failed for the KV pools");
  fk.launch(p, (int)grid, fk.smem((int)B), static_cast<cudaStream_t>(stream), &kmap, &vmap);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "decode attention launch");
  return PDB_OK;
}

int pdb_prefill_attention_impl(const void* q, const void* k_pool, const void* v_pool,
                               const int32_t* tables, const int32_t* lengths, void* out,
                               int64_t batch, int64_t width, int64_t heads, int64_t head_dim,
                               int64_t num_blocks, int64_t block_size, int64_t kv_heads,
                               int64_t table_width, int dtype, void* stream, int impl) {
  if (impl < PDB_PREFILL_AUTO || impl > PDB_PREFILL_MMA)
    return fail(PDB_ERR_INVALID_ARGUMENT, "unknown prefill kernel");
  if (dtype != PDB_DTYPE_FLOAT16)
    return fail(PDB_ERR_INVALID_ARGUMENT, "prefill attention takes FP16");
  if (!(batch > 0 && width > 0 && heads > 0 && kv_heads > 0))
    return fail(PDB_ERR_INVALID_ARGUMENT, "invalid q shape");
  if (head_dim != 64 && head_dim != 128)
    return fail(PDB_ERR_INVALID_ARGUMENT, "prefill attention supports head_dim 64 and 128");
  if (heads % kv_heads) return fail(PDB_ERR_INVALID_ARGUMENT, "query heads must be a multiple of KV heads");
  if (!(num_blocks > 0 && block_size > 0 && table_width > 0))
    return fail(PDB_ERR_INVALID_ARGUMENT, "invalid cache shape");
  if (batch > 65535 || heads > 65535 || width > (int64_t)64 * 65535 || width > INT32_MAX / 2)
    return fail(PDB_ERR_INVALID_ARGUMENT, "shape too large");
  if (!q || !k_pool || !v_pool || !tables || !lengths || !out)
    return fail(PDB_ERR_INVALID_ARGUMENT, "null tensor pointer");
  if (!aligned16(q) || !aligned16(k_pool) || !aligned16(v_pool) || !aligned16(out))
    return fail(PDB_ERR_INVALID_ARGUMENT, "tensors must be 16-byte aligned");
  // The tensor-core kernel stages whole 16-token units of a page by TMA;
  // pool rows and q rows are addressed as int32 TMA coordinates.
  const bool tc_ok = block_size % pdb::kUnitTokens == 0 && num_blocks * block_size <= INT32_MAX &&
                     batch * width <= INT32_MAX;
  if (impl == PDB_PREFILL_TCGEN05 && !tc_ok)
    return fail(PDB_ERR_INVALID_ARGUMENT,
                block_size % pdb::kUnitTokens
                    ? "the tcgen05 prefill kernel needs block_size % 16 == 0"
                    : "the tcgen05 prefill kernel needs under 2^31 pool rows and query rows");
  const bool use_tc = impl == PDB_PREFILL_TCGEN05 || (impl == PDB_PREFILL_AUTO && tc_ok);
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int G = (int)(heads / kv_heads);
  const int bs_shift = ((block_size & (block_size - 1)) == 0)
                           ? __builtin_ctzll((unsigned long long)block_size) : -1;
  const float scale_log2 = (float)(1.4426950408889634 / std::sqrt((double)head_dim));
  if (use_tc) {
    pdb::PrefillTcParams p{};
    p.tables = tables;
    p.lengths = lengths;
    p.out = static_cast<__half*>(out);
    p.B = (int)batch; p.W = (int)width; p.H = (int)heads; p.KVH = (int)kv_heads; p.G = G;
    p.table_width = (int)table_width;
    p.block_size = (int)block_size;
    p.bs_shift = bs_shift;
    p.num_blocks = num_blocks;
    p.scale_log2 = scale_log2;
    p.TZ = (int)((width + pdb::PrefillTc<64>::BM - 1) / pdb::PrefillTc<64>::BM);
    CUtensorMap qmap, kmap, vmap;
    if (!(encode_rows_map(&qmap, q, batch * width, heads, head_dim, pdb::PrefillTc<64>::BM) &&
          encode_pool_map(&kmap, k_pool, num_blocks, block_size, kv_heads, head_dim) &&
          encode_pool_map(&vmap, v_pool, num_blocks, block_size, kv_heads, head_dim)))
      return fail(PDB_ERR_CUDA, "cuTensorMapEncodeTiled failed for q or the KV pools");
    const void* fn = head_dim == 64 ? reinterpret_cast<const void*>(&pdb::prefill_tc_kernel<64>)
                                    : reinterpret_cast<const void*>(&pdb::prefill_tc_kernel<128>);
    const size_t smem = head_dim == 64 ? pdb::PrefillTc<64>::SMEM : pdb::PrefillTc<128>::SMEM;
    // Two CTAs per SM need the largest shared-memory carveout, which the
    // driver does not pick by itself (a per-function preference).
    static bool carveout_set[2] = {false, false};
    if (!carveout_set[head_dim == 128]) {
      if (cudaFuncSetAttribute(fn, cudaFuncAttributePreferredSharedMemoryCarveout,
                               (int)cudaSharedmemCarveoutMaxShared) != cudaSuccess)
        cudaGetLastError();
      carveout_set[head_dim == 128] = true;
    }
    // Each resident CTA holds 256 TMEM columns: at most two fit an SM's 512.
    constexpr int NT = pdb::PrefillTc<64>::NT;
    static_assert(NT == pdb::PrefillTc<128>::NT, "one block size");
    if (ctas_per_sm(dev, fn, smem, NT) <= 0)
      return fail(PDB_ERR_CUDA, "tcgen05 prefill kernel cannot be resident");
    // Persistent grid of two CTAs per SM, or one CTA per item if fewer. Two
    // fit by registers (128 x 192 threads each), shared memory (with the
    // largest carveout) and TMEM (256 columns each); the runtime's occupancy
    // query answers 1 for tcgen05 kernels. CTAs never wait on one another, so
    // a grid larger than what is resident is still correct.
    const int64_t items = heads * batch * p.TZ;
    const int64_t slots = 2 * (int64_t)sm_count(dev);
    const dim3 grid((unsigned)(items < slots ? items : slots));
    if (head_dim == 64)
      e = launch_pdl(pdb::prefill_tc_kernel<64>, grid, dim3(NT), smem, st, p, qmap, kmap, vmap);
    else
      e = launch_pdl(pdb::prefill_tc_kernel<128>, grid, dim3(NT), smem, st, p, qmap, kmap, vmap);
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "prefill attention launch");
    return PDB_OK;
  }
  pdb::PrefillParams p{};
  p.q = static_cast<const __half*>(q);
  p.k_pool = static_cast<const __half*>(k_pool);
  p.v_pool = static_cast<const __half*>(v_pool);
  p.tables = tables;
  p.lengths = lengths;
  p.out = static_cast<__half*>(out);
  p.B = (int)batch; p.W = (int)width; p.H = (int)heads; p.KVH = (int)kv_heads; p.G = G;
  p.table_width = (int)table_width;
  p.block_size = (int)block_size;
  p.bs_shift = bs_shift;
  p.num_blocks = num_blocks;
  p.scale_log2 = scale_log2;
  const void* fn = head_dim == 64 ? reinterpret_cast<const void*>(&pdb::prefill_attention_kernel<64>)
                                  : reinterpret_cast<const void*>(&pdb::prefill_attention_kernel<128>);
  const size_t smem = head_dim == 64 ? pdb::PrefillTile<64>::SMEM : pdb::PrefillTile<128>::SMEM;
  if (ctas_per_sm(dev, fn, smem, 128) <= 0)
    return fail(PDB_ERR_CUDA, "prefill attention kernel cannot be resident");
  const dim3 grid((unsigned)((width + 63) / 64), (unsigned)heads, (unsigned)batch);
  if (head_dim == 64)
    launch_pdl(pdb::prefill_attention_kernel<64>, grid, dim3(128), smem, st, p);
  else
    launch_pdl(pdb::prefill_attention_kernel<128>, grid, dim3(128), smem, st, p);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "prefill attention launch");
  return PDB_OK;
}

int pdb_prefill_attention(const void* q, const void* k_pool, const void* v_pool,
                          const int32_t* tables, const int32_t* lengths, void* out,
                          int64_t batch, int64_t width, int64_t heads, int64_t head_dim,
                          int64_t num_blocks, int64_t block_size, int64_t kv_heads,
                          int64_t table_width, int dtype, void* stream) {
  return pdb_prefill_attention_impl(q, k_pool, v_pool, tables, lengths, out, batch, width, heads,
                                    head_dim, num_blocks, block_size, kv_heads, table_width, dtype,
                                    stream, PDB_PREFILL_AUTO);
}

int64_t pdb_debug_dyn_partition(int64_t units, int64_t launched, int64_t* ranges,
                                int64_t max_workers) {
  if (units <= 0 || launched <= 0 || !ranges) return -1;
  const pdb::DynPlan pl = pdb::make_dyn_plan(units, launched, 4);
  const int64_t nw = pl.gs + pl.K;
  if (nw > max_workers) return -1;
  for (int64_t w = 0; w < nw; ++w) {
    ranges[3 * w] = pl.begin(w);
    ranges[3 * w + 1] = pl.begin(w + 1);
    ranges[3 * w + 2] = w < pl.gs ? 0 : 1;
  }
  return pl.gs;
}

int64_t pdb_debug_partition(const int32_t* lengths, int64_t batch, int64_t kv_heads,
                            int64_t grid, int64_t* ranges) {
  if (!lengths || !ranges || batch <= 0 || kv_heads <= 0 || grid <= 0) return -1;
  int64_t U = 0;
  for (int64_t b = 0; b < batch; ++b) {
    const int64_t len = lengths[b] < 0 ? 0 : lengths[b];
    U += kv_heads * ((len + pdb::kUnitTokens - 1) / pdb::kUnitTokens);
  }
  const int64_t g = pdb::part_grid(grid, U);
  for (int64_t c = 0; c < grid; ++c) {
    ranges[2 * c] = c < g ? pdb::part_begin(c, U, g) : U;
    ranges[2 * c + 1] = c < g ? pdb::part_begin(c + 1, U, g) : U;
  }
  return U;
}

}  // extern "C"
