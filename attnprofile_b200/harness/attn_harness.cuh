// Runtime of the tuning-harness driver (attn_test.cu next to this file).
//
// Gives the reference's tuning harness (tuning/benchmark_run_attn.py) what it
// expects from tuning/attn_test.cu: a runAttn<...> template with the same
// parameter list (attn_runner.cuh), used through an AttnRunner function
// pointer (tuning/utils.cuh:71), and benchmark_attn<B,H,S,D,BM,BN> with the
// reference's timing contract (60 warm-up + 250 timed launches between two
// CUDA events, tuning/utils.cuh:246-302) and its output line
// "B, H, S, D, BM, BN, avg_ms, tflops" (tuning/utils.cuh:296), which the
// harness parses (benchmark_run_attn.py:318-336).  Inputs are seeded N(0,1)
// (the reference times all-zero inputs).
#pragma once

#include <cstdio>
#include <cstdlib>

#include "attn_runner.cuh"

namespace attnprof {
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
