// Run-time (BM, BN) -> compile-time kernel variant dispatch.
//
// Plays the role of the reference's compile-time dispatcher
// runAttn<..., KERNEL_IDX, ...> (tuning/attn_test.cu:1665-1691): BM = 128
// maps to one 128-row Q tile per CTA (NQ = 1), BM = 256 to two ping-ponged
// Q tiles (NQ = 2).  The K/V ring depth is the deepest that fits the 227 KB
// shared-memory limit (at most 8 slots).
#pragma once

#include "attn_host.cuh"

namespace attnprof {

struct VariantInfo {
  int num_threads, smem_bytes, tmem_cols, stages;
};

template <typename T, int D, int BN, int NQ, bool PAIR = false>
inline VariantInfo variant_info() {
  constexpr int ST = auto_stages<T, D, BN, NQ, PAIR>();
  using C = AttnConfig<T, D, BN, NQ, ST, PAIR>;
  return VariantInfo{C::NUM_THREADS, C::SMEM_BYTES, C::TMEM_ALLOC, ST};
}

// BM = 512 (D = 128, BN = 128): a CTA pair of two 256-row CTAs sharing every
// K/V tile through cta_group::2 MMAs (AttnConfig::PAIR).
constexpr int kPairBM = 512;

#define ATTNPROF_FOR_EACH_TILE(X) \
  X(128, 32)                      \
  X(128, 64)                      \
  X(128, 96)                      \
  X(128, 128)                     \
  X(128, 256)                     \
  X(256, 32)                      \
  X(256, 64)                      \
  X(256, 96)                      \
  X(256, 128)

template <typename T, int D, bool PROFILE>
int dispatch_attn(int BM, int BN, const void* Q, const void* K, const void* V, void* O, int B,
                  int H, int S, long long q_rows, long long kv_rows, cudaStream_t stream,
                  const LaunchOpts& o) {
#define ATTNPROF_CASE(BM_, BN_)                                                              \
  if (BM == BM_ && BN == BN_)                                                                \
    return launch_attn<T, D, BN_, BM_ / 128, auto_stages<T, D, BN_, BM_ / 128>(), PROFILE>( \
        Q, K, V, O, B, H, S, q_rows, kv_rows, stream, o);
  ATTNPROF_FOR_EACH_TILE(ATTNPROF_CASE)
#undef ATTNPROF_CASE
  if constexpr (D == 128) {
    if (BM == kPairBM && BN == 128)
      return launch_attn<T, D, 128, 2, auto_stages<T, D, 128, 2, true>(), PROFILE, true>(
          Q, K, V, O, B, H, S, q_rows, kv_rows, stream, o);
  }
  return ATTN_ERR_UNSUPPORTED;
}

template <typename T, int D>
int query_variant(int BM, int BN, VariantInfo* out) {
#define ATTNPROF_QCASE(BM_, BN_)                         \
  if (BM == BM_ && BN == BN_) {                          \
    *out = variant_info<T, D, BN_, BM_ / 128>();         \
    return ATTN_OK;                                      \
  }
  ATTNPROF_FOR_EACH_TILE(ATTNPROF_QCASE)
#undef ATTNPROF_QCASE
  if constexpr (D == 128) {
    if (BM == kPairBM && BN == 128) {
      *out = variant_info<T, D, 128, 2, true>();
      return ATTN_OK;
    }
  }
  return ATTN_ERR_UNSUPPORTED;
}

#define ATTNPROF_DECLARE(T, D, P)                                                              \
  extern template int dispatch_attn<T, D, P>(int, int, const void*, const void*, const void*, \
                                             void*, int, int, int, long long, long long,       \
                                             cudaStream_t, const LaunchOpts&);
#define ATTNPROF_INSTANTIATE(T, D, P)                                                   \
  template int dispatch_attn<T, D, P>(int, int, const void*, const void*, const void*, \
                                      void*, int, int, int, long long, long long,       \
                                      cudaStream_t, const LaunchOpts&);

}  // namespace attnprof
