/* A plain C99 caller of the engine's C ABI (include/attnprof.h), the way a
 * foreign-function binding would use it.  Mode "host": calls that need no
 * GPU (error strings, partition rule, split planner, argument checks).  Mode
 * "gpu": one attention forward with V constant per head on device buffers
 * from the CUDA runtime; softmax rows sum to one, so every O row must equal
 * that head's V value.  Exit code 0 on success. */
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "attnprof.h"

static int host_checks(void) {
  int b, e, k;
  long long whole, ctas;
  if (attn_version() < 100) return 1;
  if (strlen(attn_error_string(ATTN_ERR_INVALID_ARG)) == 0) return 2;
  if (attn_shard_range(10, 3, 1, &b, &e) != ATTN_OK || b != 3 || e != 6) return 3;
  if (attn_plan_split(64, 128, 148, 0, &k, &whole, &ctas) != ATTN_OK || k != 2 || ctas != 128)
    return 4;
  /* null pointers are rejected before any device work */
  if (attn_fwd(NULL, NULL, NULL, NULL, 1, 1, 128, 128, ATTN_DTYPE_F16, 256, 128, NULL) !=
      ATTN_ERR_INVALID_ARG)
    return 5;
  /* the empty problem is a no-op */
  if (attn_fwd(NULL, NULL, NULL, NULL, 0, 1, 128, 128, ATTN_DTYPE_F16, 256, 128, NULL) != ATTN_OK)
    return 6;
  return 0;
}

#ifdef WITH_CUDA
#include <stdint.h>

#include <cuda_runtime.h>

/* f16 <-> f32 for normal values (the test data), round to nearest even */
static uint16_t to_half(float f) {
  union { float f; uint32_t u; } v;
  uint32_t sign, mant, lsb;
  int exp;
  v.f = f;
  sign = (v.u >> 16) & 0x8000u;
  exp = (int)((v.u >> 23) & 0xffu) - 127 + 15;
  mant = v.u & 0x7fffffu;
  if (exp <= 0) return (uint16_t)sign; /* tiny: flush */
  lsb = (mant >> 13) & 1u;
  mant += 0xfffu + lsb;
  if (mant & 0x800000u) {
    mant = 0;
    ++exp;
  }
  return (uint16_t)(sign | ((uint32_t)exp << 10) | (mant >> 13));
}
static float from_half(uint16_t h) {
  union { float f; uint32_t u; } v;
  const uint32_t exp = (h >> 10) & 0x1fu, mant = h & 0x3ffu;
  v.u = ((uint32_t)(h & 0x8000u) << 16) | (exp ? ((exp - 15 + 127) << 23) | (mant << 13) : 0u);
  return v.f;
}

static int gpu_check(void) {
  const int B = 1, H = 3, S = 777, D = 128;
  const size_t n = (size_t)B * H * S * D;
  uint16_t *hq = malloc(n * 2), *hk = malloc(n * 2), *hv = malloc(n * 2), *ho = malloc(n * 2);
  void *dq, *dk, *dv, *dO;
  size_t i;
  int rc, h;
  unsigned int x = 12345u;
  for (i = 0; i < n; ++i) {
    x = x * 1664525u + 1013904223u;
    hq[i] = to_half(((float)(x >> 9) / 8388608.0f) - 1.0f);
    x = x * 1664525u + 1013904223u;
    hk[i] = to_half(((float)(x >> 9) / 8388608.0f) - 1.0f);
    hv[i] = to_half(0.25f * (float)(i / ((size_t)S * D) + 1)); /* constant per head */
  }
  if (cudaMalloc(&dq, n * 2) || cudaMalloc(&dk, n * 2) || cudaMalloc(&dv, n * 2) ||
      cudaMalloc(&dO, n * 2))
    return 20;
  cudaMemcpy(dq, hq, n * 2, cudaMemcpyHostToDevice);
  cudaMemcpy(dk, hk, n * 2, cudaMemcpyHostToDevice);
  cudaMemcpy(dv, hv, n * 2, cudaMemcpyHostToDevice);
  rc = attn_fwd(dq, dk, dv, dO, B, H, S, D, ATTN_DTYPE_F16, 256, 128, NULL);
  if (rc != ATTN_OK) {
    fprintf(stderr, "attn_fwd: %s\n", attn_error_string(rc));
    return 21;
  }
  if (cudaDeviceSynchronize() != cudaSuccess) return 22;
  if (attn_get_status(0, 1, NULL) != ATTN_OK) return 23;
  cudaMemcpy(ho, dO, n * 2, cudaMemcpyDeviceToHost);
  for (h = 0; h < H; ++h) {
    const float want = 0.25f * (float)(h + 1);
    for (i = (size_t)h * S * D; i < (size_t)(h + 1) * S * D; ++i) {
      const float got = from_half(ho[i]);
      if (got - want > 2e-3f || want - got > 2e-3f) {
        fprintf(stderr, "head %d element %zu: %f != %f\n", h, i, got, want);
        return 24;
      }
    }
  }
  cudaFree(dq);
  cudaFree(dk);
  cudaFree(dv);
  cudaFree(dO);
  free(hq);
  free(hk);
  free(hv);
  free(ho);
  return 0;
}
#endif

int main(int argc, char** argv) {
  int rc = host_checks();
  if (rc) {
    fprintf(stderr, "host check %d failed\n", rc);
    return rc;
  }
#ifdef WITH_CUDA
  if (argc > 1 && strcmp(argv[1], "gpu") == 0) {
    rc = gpu_check();
    if (rc) fprintf(stderr, "gpu check %d failed\n", rc);
    return rc;
  }
#endif
  (void)argc;
  (void)argv;
  printf("ok\n");
  return 0;
}
