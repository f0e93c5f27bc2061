// runAttn<...> of the B200 engine with the reference's template parameter
// list (tuning/attn_test.cu:1665-1691), usable as an AttnRunner
// (tuning/utils.cuh:71) by the reference's benchmark_attn and verify_attn.
//
// Knob mapping onto the B200 kernel:
//   BM              128 -> one 128-row Q tile per CTA, 256 -> two ping-ponged
//   BN              keys per KV tile (multiple of 32, <= 256; the kernel
//                   static_asserts TMEM/shared-memory fit, so a config that
//                   cannot run fails to compile and the harness records it)
//   NUM_SMEM        accepted (>= 1); the K/V ring has the depth the library
//                   ships for this tile (auto_stages: the deepest ring of at
//                   most 8 slots that fits shared memory), so a harness sweep
//                   times the configuration attn_fwd runs.  (The reference's
//                   NUM_SMEM stages each of K and V; here K and V share one
//                   ring, and a shallower ring never measured faster.)
//   KERNEL_IDX      1, 2 or 3 accepted (validated); the Hopper variants differ
//                   only in where P lives, and here P always lives in TMEM
//   P_SMEM_K_TILES, PRODUCER_REG_DEALLOC, CONSUMER_REG_ALLOC, NUM_THREADS
//                   Hopper register/smem-split knobs: accepted and ignored
//                   (the register split is fixed per variant)
// Buffers use the reference's padded layout (Q/O [B,H,SQO,D], K/V
// [B,H,SKV,D], SQO = ceil(S/BM)*BM, SKV = ceil(S/BN)*BN); rows >= S are
// neither read nor written.  Launches go to the default stream, as the
// reference's did; a failed launch prints the error and exits, as the
// reference's cudaCheck does (tuning/tools.cuh:14-21).
#pragma once

#include <cstdio>
#include <cstdlib>

#include "../csrc/attn_host.cuh"

typedef __half fp16;
using AttnRunner = void (*)(fp16*, fp16*, fp16*, fp16*);

namespace attnprof {
__device__ int g_harness_status;
int* device_status_ptr() {
  static int* p = nullptr;
  if (p == nullptr) {
    void* a = nullptr;
    if (cudaGetSymbolAddress(&a, g_harness_status) != cudaSuccess) return nullptr;
    p = static_cast<int*>(a);
  }
  return p;
}
}  // namespace attnprof

template <int B, int H, int S, int D, int BM, int BN, int NUM_SMEM,
          uint32_t PRODUCER_REG_DEALLOC, uint32_t CONSUMER_REG_ALLOC, int P_SMEM_K_TILES,
          int KERNEL_IDX, int NUM_THREADS = 384>
void runAttn(fp16* Q, fp16* K, fp16* V, fp16* O) {
  static_assert(KERNEL_IDX >= 1 && KERNEL_IDX <= 3, "KERNEL_IDX must be 1, 2 or 3");
  static_assert(BM == 128 || BM == 256, "BM must be 128 or 256 on B200");
  static_assert(NUM_SMEM >= 1, "NUM_SMEM must be >= 1");
  constexpr int NQ = BM / 128;
  constexpr int SQO = ((S + BM - 1) / BM) * BM;
  constexpr int SKV = ((S + BN - 1) / BN) * BN;
  constexpr int STAGES = attnprof::auto_stages<__half, D, BN, NQ>();
  static_assert(STAGES >= 2, "K/V tile does not fit shared memory");
  attnprof::LaunchOpts opts;
  const int rc = attnprof::launch_attn<__half, D, BN, NQ, STAGES, false>(
      Q, K, V, O, B, H, S, SQO, SKV, nullptr, opts);
  if (rc != 0) {
    std::fprintf(stderr, "[attn] launch failed: %s (%d)\n", "see include/attnprof.h", rc);
    std::exit(1);
  }
}
