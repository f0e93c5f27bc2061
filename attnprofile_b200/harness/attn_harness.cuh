// Runtime of the tuning-harness driver (attn_test.cu next to this file).
//
// Gives the reference's tuning harness (tuning/benchmark_run_attn.py) what it
// expects from tuning/attn_test.cu: a runAttn<...> template with the same
// parameter list (tuning/attn_test.cu:1665-1691), used through an AttnRunner
// function pointer (tuning/utils.cuh:71), and benchmark_attn<B,H,S,D,BM,BN>
// with the reference's timing contract (60 warm-up + 250 timed launches
// between two CUDA events, tuning/utils.cuh:246-302) and its output line
// "B, H, S, D, BM, BN, avg_ms, tflops" (tuning/utils.cuh:296), which the
// harness parses (benchmark_run_attn.py:318-336).
//
// Knob mapping onto the B200 kernel:
//   BM              128 -> one 128-row Q tile per CTA, 256 -> two ping-ponged
//   BN              keys per KV tile (multiple of 32, <= 256; the kernel
//                   static_asserts TMEM/shared-memory fit, so a config that
//                   cannot run fails to compile and the harness records it)
//   NUM_SMEM        K/V ring slots = 2 * NUM_SMEM (the reference had NUM_SMEM
//                   slots each for K and V), at least 2, capped by the 227 KB
//                   shared-memory limit
//   KERNEL_IDX      1, 2 or 3 accepted (validated); the Hopper variants differ
//                   only in where P lives, and here P always lives in TMEM
//   P_SMEM_K_TILES, PRODUCER_REG_DEALLOC, CONSUMER_REG_ALLOC, NUM_THREADS
//                   Hopper register/smem-split knobs: accepted and ignored
//                   (the register split is fixed per variant)
// Buffers use the reference's padded layout (Q/O [B,H,SQO,D], K/V
// [B,H,SKV,D], SQO = ceil(S/BM)*BM, SKV = ceil(S/BN)*BN); rows >= S are not
// read.  Inputs are seeded N(0,1) (the reference times all-zero inputs).
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

// Seeded approximately-normal fill (sum of four uniforms from a 32-bit hash,
// rescaled to unit variance); rows >= valid_rows of each head are zeroed.
__global__ void harness_fill(__half* x, long long rows_per_head, long long valid_rows, int D,
                             long long heads, unsigned seed) {
  const long long n = rows_per_head * D * heads;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const long long row = (i / D) % rows_per_head;
    float v = 0.f;
    if (row < valid_rows) {
      unsigned h = static_cast<unsigned>(i) * 2654435761u ^ seed;
      float acc = 0.f;
      for (int k = 0; k < 4; ++k) {
        h ^= h >> 16; h *= 0x7feb352du; h ^= h >> 15; h *= 0x846ca68bu; h ^= h >> 16;
        acc += (h >> 8) * (1.0f / 16777216.0f);
      }
      v = (acc - 2.0f) * 1.7320508f;  // variance of 4 uniforms is 1/3
    }
    x[i] = __float2half_rn(v);
  }
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
  constexpr int FIT = attnprof::auto_stages<__half, D, BN, NQ>(16);
  static_assert(FIT >= 2, "K/V tile does not fit shared memory");
  constexpr int WANT = 2 * NUM_SMEM < 2 ? 2 : 2 * NUM_SMEM;
  constexpr int STAGES = WANT < FIT ? WANT : FIT;
  attnprof::LaunchOpts opts;
  const int rc = attnprof::launch_attn<__half, D, BN, NQ, STAGES, false>(
      Q, K, V, O, B, H, S, SQO, SKV, nullptr, opts);
  if (rc != 0) {
    std::fprintf(stderr, "[attn] launch failed: %s (%d)\n", "see include/attnprof.h", rc);
    std::exit(1);
  }
}

#define HARNESS_CHECK(x)                                                              \
  do {                                                                                \
    cudaError_t e_ = (x);                                                             \
    if (e_ != cudaSuccess) {                                                          \
      std::fprintf(stderr, "[CUDA ERROR] %s:%d: %s\n", __FILE__, __LINE__,           \
                   cudaGetErrorString(e_));                                           \
      std::exit(1);                                                                   \
    }                                                                                 \
  } while (0)

template <int B, int H, int S, int D, int BM, int BN>
void benchmark_attn(AttnRunner kernel) {
  constexpr int SQO = ((S + BM - 1) / BM) * BM;
  constexpr int SKV = ((S + BN - 1) / BN) * BN;
  const size_t qo = static_cast<size_t>(B) * H * SQO * D, kv = static_cast<size_t>(B) * H * SKV * D;
  fp16 *dQ, *dK, *dV, *dO;
  HARNESS_CHECK(cudaMalloc(&dQ, qo * 2));
  HARNESS_CHECK(cudaMalloc(&dK, kv * 2));
  HARNESS_CHECK(cudaMalloc(&dV, kv * 2));
  HARNESS_CHECK(cudaMalloc(&dO, qo * 2));
  attnprof::harness_fill<<<1184, 256>>>(dQ, SQO, S, D, (long long)B * H, 1u);
  attnprof::harness_fill<<<1184, 256>>>(dK, SKV, S, D, (long long)B * H, 2u);
  attnprof::harness_fill<<<1184, 256>>>(dV, SKV, S, D, (long long)B * H, 3u);
  HARNESS_CHECK(cudaMemset(dO, 0, qo * 2));
  for (int i = 0; i < 60; ++i) kernel(dQ, dK, dV, dO);
  HARNESS_CHECK(cudaDeviceSynchronize());
  cudaEvent_t a, b;
  HARNESS_CHECK(cudaEventCreate(&a));
  HARNESS_CHECK(cudaEventCreate(&b));
  HARNESS_CHECK(cudaEventRecord(a));
  for (int i = 0; i < 250; ++i) kernel(dQ, dK, dV, dO);
  HARNESS_CHECK(cudaEventRecord(b));
  HARNESS_CHECK(cudaEventSynchronize(b));
  float ms = 0.f;
  HARNESS_CHECK(cudaEventElapsedTime(&ms, a, b));
  int status = 0;
  HARNESS_CHECK(cudaMemcpyFromSymbol(&status, attnprof::g_harness_status, sizeof(int)));
  if (status != 0) {
    std::fprintf(stderr, "[attn] device timeout status 0x%x\n", status);
    std::exit(1);
  }
  const double avg_ms = static_cast<double>(ms) / 250;
  const double flops = 4.0 * B * H * static_cast<double>(S) * S * D;
  std::printf("%d, %d, %d, %d, %d, %d, %.6f, %.3f\n", B, H, S, D, BM, BN, avg_ms,
              flops / (avg_ms * 1e-3) / 1e12);
  cudaFree(dQ);
  cudaFree(dK);
  cudaFree(dV);
  cudaFree(dO);
}
