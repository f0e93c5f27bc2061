// A C++ caller of the engine through include/attnprof.hpp (the host template
// over the C ABI).  Mode "host": calls that need no GPU (argument checks,
// dtype deduction).  Mode "gpu": one forward per dtype with V constant per
// head; every O row must equal that head's V value.  Exit code 0 on success.
#include <cstdio>
#include <cstring>
#include <vector>

#include "attnprof.hpp"

static int host_checks() {
  const __half* nq = nullptr;
  __half* no = nullptr;
  // null pointers are rejected before any device work, the empty problem is a no-op
  if (attnprof::attn<256, 128>(nq, nq, nq, no, 1, 1, 128, 128) != ATTN_ERR_INVALID_ARG) return 1;
  if (attnprof::attn<256, 128>(nq, nq, nq, no, 0, 1, 128, 128) != ATTN_OK) return 2;
  const __nv_bfloat16* bq = nullptr;
  __nv_bfloat16* bo = nullptr;
  if (attnprof::attn_padded<128, 64>(bq, bq, bq, bo, 1, 1, 64, 128, 32, 64) != ATTN_ERR_INVALID_ARG)
    return 3;
  static_assert(attnprof::tile_is_built<512, 128>::value, "");
  static_assert(!attnprof::tile_is_built<256, 256>::value, "");
  static_assert(attnprof::dtype_code<__nv_bfloat16>::value == ATTN_DTYPE_BF16, "");
  return 0;
}

template <typename T>
static int gpu_check(float (*to_f)(T), T (*from_f)(float)) {
  const int B = 1, H = 3, S = 777, D = 128;
  const size_t n = static_cast<size_t>(B) * H * S * D;
  std::vector<T> hq(n), hk(n), hv(n), ho(n);
  unsigned x = 12345u;
  for (size_t i = 0; i < n; ++i) {
    x = x * 1664525u + 1013904223u;
    hq[i] = from_f(static_cast<float>(x >> 9) / 8388608.0f - 1.0f);
    x = x * 1664525u + 1013904223u;
    hk[i] = from_f(static_cast<float>(x >> 9) / 8388608.0f - 1.0f);
    hv[i] = from_f(0.25f * static_cast<float>(i / (static_cast<size_t>(S) * D) + 1));
  }
  T *dq, *dk, *dv, *dO;
  if (cudaMalloc(&dq, n * sizeof(T)) || cudaMalloc(&dk, n * sizeof(T)) ||
      cudaMalloc(&dv, n * sizeof(T)) || cudaMalloc(&dO, n * sizeof(T)))
    return 20;
  cudaStream_t st;
  cudaStreamCreate(&st);
  cudaMemcpy(dq, hq.data(), n * sizeof(T), cudaMemcpyHostToDevice);
  cudaMemcpy(dk, hk.data(), n * sizeof(T), cudaMemcpyHostToDevice);
  cudaMemcpy(dv, hv.data(), n * sizeof(T), cudaMemcpyHostToDevice);
  const int rc = attnprof::attn<256, 128>(dq, dk, dv, dO, B, H, S, D, st);
  if (rc != ATTN_OK) {
    std::fprintf(stderr, "attn: %s\n", attn_error_string(rc));
    return 21;
  }
  if (cudaStreamSynchronize(st) != cudaSuccess) return 22;
  if (attn_get_status(0, 1, nullptr) != ATTN_OK) return 23;
  cudaMemcpy(ho.data(), dO, n * sizeof(T), cudaMemcpyDeviceToHost);
  for (int h = 0; h < H; ++h) {
    const float want = 0.25f * static_cast<float>(h + 1);
    for (size_t i = static_cast<size_t>(h) * S * D; i < static_cast<size_t>(h + 1) * S * D; ++i) {
      const float got = to_f(ho[i]);
      if (got - want > 2e-3f || want - got > 2e-3f) {
        std::fprintf(stderr, "head %d element %zu: %f != %f\n", h, i, got, want);
        return 24;
      }
    }
  }
  cudaFree(dq);
  cudaFree(dk);
  cudaFree(dv);
  cudaFree(dO);
  cudaStreamDestroy(st);
  return 0;
}

int main(int argc, char** argv) {
  int rc = host_checks();
  if (rc) {
    std::fprintf(stderr, "host check %d failed\n", rc);
    return rc;
  }
  if (argc > 1 && std::strcmp(argv[1], "gpu") == 0) {
    rc = gpu_check<__half>([](__half v) { return __half2float(v); },
                           [](float f) { return __float2half_rn(f); });
    if (!rc)
      rc = gpu_check<__nv_bfloat16>([](__nv_bfloat16 v) { return __bfloat162float(v); },
                                    [](float f) { return __float2bfloat16_rn(f); });
    if (rc) {
      std::fprintf(stderr, "gpu check %d failed\n", rc);
      return rc;
    }
  }
  std::printf("ok\n");
  return 0;
}
