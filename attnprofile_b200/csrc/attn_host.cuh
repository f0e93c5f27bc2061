// Host side of the attention forward: tensor-map construction (cached),
// launch configuration and the C++ host entry attn<BM, BN>(...).
//
// Replaces the reference launchers runAttnWS2StageBaselineKernel /
// runAttnWS2StageSmemPKernel / runAttnWSForNSmemPKernel
// (tuning/attn_test.cu:1583-1663) and the tensor-map helper create_tensor_map
// (tuning/utils.cuh:33-69).  Differences that matter to callers:
//   * the stream is an argument (the reference always used the default stream);
//   * tensor maps are cached per (pointer, shape, box) instead of re-encoded
//     on every call (the reference encodes four per call);
//   * errors are returned as codes instead of exit(1)/assert;
//   * Q/O may have SQO >= S rows per head and K/V SKV >= S rows per head (the
//     reference's padded layout); rows >= S are never read (TMA fills zeros)
//     nor written (TMA clips the store).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <cstring>
#include <mutex>
#include <unordered_map>

#if __has_include("attnprof.h")
#include "attnprof.h"
#else
#include "../../include/attnprof.h"  // builds without -I include (the tuning-harness driver)
#endif
#include "attn_kernel.cuh"

namespace attnprof {

constexpr int kSmemLimit = 232448;  // opt-in dynamic shared memory per CTA on sm_100

template <typename T, int D, int BN, int NQ>
constexpr int auto_stages(int cap = 8) {
  int best = 0;
  for (int s = 2; s <= cap; ++s) {
    if (AttnConfig<T, D, BN, NQ, 2>::OFF_KV + s * (BN * D * 2) + 256 + 1024 + 16 <= kSmemLimit)
      best = s;
  }
  return best;
}

struct LaunchOpts {
  unsigned long long timeout_ns = 2000000000ull;  // bounded-wait limit: 2 s
  int fault_mode = 0;
  unsigned long long* prof = nullptr;
  int prof_cta = 0;
};

// ---------------------------------------------------------------------------
// Driver entry point for cuTensorMapEncodeTiled (no link-time libcuda).
// ---------------------------------------------------------------------------
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_tiled_fn() {
  static EncodeTiledFn fn = []() -> EncodeTiledFn {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault,
                                         &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}

struct MapKey {
  uintptr_t ptr;
  int dtype, D, S, BH, box_rows;
  long long rows;
  bool operator==(const MapKey& o) const {
    return ptr == o.ptr && dtype == o.dtype && D == o.D && S == o.S && BH == o.BH &&
           box_rows == o.box_rows && rows == o.rows;
  }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    size_t h = std::hash<uintptr_t>()(k.ptr);
    auto mix = [&](long long v) { h ^= std::hash<long long>()(v) + 0x9e3779b97f4a7c15ull + (h << 6) + (h >> 2); };
    mix(k.dtype); mix(k.D); mix(k.S); mix(k.BH); mix(k.box_rows); mix(k.rows);
    return h;
  }
};

// 3-D map over a [B*H][rows][D] tensor: dims {D, S, B*H}; the row pitch is D
// elements and the head pitch `rows` rows, so rows >= S padding is skipped.
// Box {64, box_rows, 1} with 128-byte swizzle: one 64-column block per copy.
inline int get_tensor_map(CUtensorMap* out, const void* ptr, int dtype, int D, int S, int BH,
                          long long rows, int box_rows) {
  static std::mutex mu;
  static std::unordered_map<MapKey, CUtensorMap, MapKeyHash> cache;
  const MapKey key{reinterpret_cast<uintptr_t>(ptr), dtype, D, S, BH, box_rows, rows};
  {
    std::lock_guard<std::mutex> g(mu);
    auto it = cache.find(key);
    if (it != cache.end()) {
      *out = it->second;
      return ATTN_OK;
    }
  }
  EncodeTiledFn enc = encode_tiled_fn();
  if (enc == nullptr) return ATTN_ERR_CUDA;
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(S),
                              static_cast<cuuint64_t>(BH)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(D) * 2,
                                 static_cast<cuuint64_t>(rows) * D * 2};
  const cuuint32_t box[3] = {64u, static_cast<cuuint32_t>(box_rows), 1u};
  const cuuint32_t estr[3] = {1u, 1u, 1u};
  CUtensorMap m;
  const CUresult r = enc(&m, dtype == ATTN_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                      : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                         3, const_cast<void*>(ptr), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return ATTN_ERR_TENSOR_MAP;
  {
    std::lock_guard<std::mutex> g(mu);
    if (cache.size() > 4096) cache.clear();
    cache.emplace(key, m);
  }
  *out = m;
  return ATTN_OK;
}

// Per-device status word written by the kernel's bounded waits.
int* device_status_ptr();

template <typename T, int D, int BN, int NQ, int STAGES, bool PROFILE>
int launch_attn(const void* Q, const void* K, const void* V, void* O, int B, int H, int S,
                long long q_rows, long long kv_rows, cudaStream_t stream, const LaunchOpts& o) {
  using C = AttnConfig<T, D, BN, NQ, STAGES>;
  static_assert(C::SMEM_BYTES <= kSmemLimit, "shared memory over the sm_100 per-CTA limit");
  const int dtype = std::is_same<T, __half>::value ? ATTN_DTYPE_F16 : ATTN_DTYPE_BF16;
  const long long BH = static_cast<long long>(B) * H;
  if (BH > 65535) return ATTN_ERR_INVALID_ARG;  // grid.y limit
  CUtensorMap mq, mk, mv, mo;
  int rc;
  if ((rc = get_tensor_map(&mq, Q, dtype, D, S, static_cast<int>(BH), q_rows, C::QROWS))) return rc;
  if ((rc = get_tensor_map(&mk, K, dtype, D, S, static_cast<int>(BH), kv_rows, BN))) return rc;
  if ((rc = get_tensor_map(&mv, V, dtype, D, S, static_cast<int>(BH), kv_rows, BN))) return rc;
  if ((rc = get_tensor_map(&mo, O, dtype, D, S, static_cast<int>(BH), q_rows, C::QROWS))) return rc;

  auto kern = attn_fwd_kernel<T, D, BN, NQ, STAGES, PROFILE>;
  static bool attr_done[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return ATTN_ERR_CUDA;
  if (dev < 64 && !attr_done[dev]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES) !=
        cudaSuccess)
      return ATTN_ERR_RESOURCE;
    attr_done[dev] = true;
  }
  AttnParams p;
  p.S = S;
  p.num_kv_tiles = (S + BN - 1) / BN;
  p.scale_log2 = static_cast<float>(1.4426950408889634 / std::sqrt(static_cast<double>(D)));
  p.status = device_status_ptr();
  if (p.status == nullptr) return ATTN_ERR_CUDA;
  p.timeout_ns = o.timeout_ns;
  p.fault_mode = o.fault_mode;
  p.prof = o.prof;
  p.prof_cta = o.prof_cta;
  const dim3 grid((S + C::BM - 1) / C::BM, static_cast<unsigned>(BH), 1);
  kern<<<grid, C::NUM_THREADS, C::SMEM_BYTES, stream>>>(mq, mk, mv, mo, p);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return ATTN_ERR_CUDA;
  return ATTN_OK;
}

}  // namespace attnprof
