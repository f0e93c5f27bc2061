/*
 * attnprof.hpp -- C++ host template over the C ABI (attnprof.h).
 *
 *   template <int BM, int BN, typename T>
 *   int attnprof::attn(const T* Q, const T* K, const T* V, T* O,
 *                      int B, int H, int S, int D, cudaStream_t stream);
 *
 * The tile is a compile-time choice, as in the reference's
 * runAttn<B,H,S,D,BM,BN,...> (tuning/attn_test.cu:1665-1691); the shape is a
 * run-time argument.  T is __half or __nv_bfloat16 (the dtype code is
 * deduced).  Tiles that are not built fail to compile; D that is not built
 * returns ATTN_ERR_UNSUPPORTED at run time.  Asynchronous on `stream`;
 * returns 0 or a negative ATTN_ERR_* code (attn_error_string()).  Contiguous
 * [B, H, S, D] tensors; attn_padded() takes the reference's padded rows.
 *
 * Header only: it forwards to the exported attn_fwd / attn_fwd_padded, so a
 * C++ caller links libattnprof.so exactly like a C caller.
 */
#ifndef ATTNPROF_HPP
#define ATTNPROF_HPP

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <type_traits>

#include "attnprof.h"

namespace attnprof {

// (BM, BN) pairs built into the library; BM = 512 is the CTA pair (D = 128).
template <int BM, int BN>
struct tile_is_built
    : std::integral_constant<bool, ((BM == 128 || BM == 256) &&
                                    (BN == 32 || BN == 64 || BN == 96 || BN == 128 ||
                                     (BN == 256 && BM == 128))) ||
                                       (BM == 512 && BN == 128)> {};

template <typename T>
struct dtype_code;
template <>
struct dtype_code<__half> : std::integral_constant<int, ATTN_DTYPE_F16> {};
template <>
struct dtype_code<__nv_bfloat16> : std::integral_constant<int, ATTN_DTYPE_BF16> {};

template <int BM, int BN, typename T>
inline int attn(const T* Q, const T* K, const T* V, T* O, int B, int H, int S, int D,
                cudaStream_t stream = nullptr) {
  static_assert(tile_is_built<BM, BN>::value, "this (BM, BN) tile is not built");
  return attn_fwd(Q, K, V, O, B, H, S, D, dtype_code<T>::value, BM, BN,
                  static_cast<void*>(stream));
}

// Q/O with SQO >= S rows per head, K/V with SKV >= S (the reference's padded
// allocation, tuning/utils.cuh:86-87); rows >= S are neither read nor written.
template <int BM, int BN, typename T>
inline int attn_padded(const T* Q, const T* K, const T* V, T* O, int B, int H, int S, int D,
                       int SQO, int SKV, cudaStream_t stream = nullptr) {
  static_assert(tile_is_built<BM, BN>::value, "this (BM, BN) tile is not built");
  return attn_fwd_padded(Q, K, V, O, B, H, S, D, SQO, SKV, dtype_code<T>::value, BM, BN,
                         static_cast<void*>(stream));
}

}  // namespace attnprof

#endif /* ATTNPROF_HPP */
