// ref_shim.cu -- runs the reference's own host-side attention oracle
// (verify_attn, tuning/utils.cuh:73-244) on a machine without a GPU.
//
// TEST INFRASTRUCTURE ONLY (builds oracle/_ref/ref_attn, never shipped).
//
// The reference's utils.cuh is compiled from where it lies (include path
// points at the reference's tuning/ directory; nothing is copied).  Its CUDA
// runtime calls are redirected at link time (-Wl,--wrap=...) to the host
// stand-ins below, so "device" buffers are host memory.  verify_attn then
//   1. draws Q, K ~ U(-0.5, 0.5), V ~ U(-1, 1) from std::mt19937(42)
//      (tuning/utils.cuh:95-118),
//   2. calls our runner with the "device" pointers -- the runner saves the
//      inputs and leaves O at zero,
//   3. computes its CPU reference output hORef (tuning/utils.cuh:139-198).
// hORef is a local std::vector; the global operator new/delete (ref_hooks.cpp) note the
// fifth allocation made inside verify_attn (hQ, hK, hV, hO, hORef -- the order
// of tuning/utils.cuh:89-90) and copy its bytes out when it is freed.
//
// Modes:
//   ref_attn golden <outdir>          write golden_<tag>.bin for each fixture
//   ref_attn time <cfg> <threads>     run verify_attn on `threads` host threads
//                                     at once (cfg: c1 | c2head | c3head) and
//                                     print one JSON line with the wall time
#include "utils.cuh"

#include <atomic>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <new>
#include <string>
#include <thread>
#include <vector>

// ---------------------------------------------------------------------------
// CUDA runtime stand-ins (host memory)
// ---------------------------------------------------------------------------
extern "C" {
cudaError_t __wrap_cudaGetDevice(int* d) {
  *d = 0;
  return cudaSuccess;
}
cudaError_t __wrap_cudaGetDeviceProperties_v2(cudaDeviceProp* p, int) {
  std::memset(p, 0, sizeof(*p));
  p->major = 9;  // the reference's guard wants SM90+ (tuning/utils.cuh:80-83)
  p->minor = 0;
  return cudaSuccess;
}
cudaError_t __wrap_cudaMalloc(void** p, size_t n) {
  *p = std::malloc(n ? n : 1);
  return *p ? cudaSuccess : cudaErrorMemoryAllocation;
}
cudaError_t __wrap_cudaFree(void* p) {
  std::free(p);
  return cudaSuccess;
}
cudaError_t __wrap_cudaMemcpy(void* dst, const void* src, size_t n, cudaMemcpyKind) {
  std::memcpy(dst, src, n);
  return cudaSuccess;
}
cudaError_t __wrap_cudaMemset(void* dst, int v, size_t n) {
  std::memset(dst, v, n);
  return cudaSuccess;
}
cudaError_t __wrap_cudaGetLastError(void) { return cudaSuccess; }
cudaError_t __wrap_cudaDeviceSynchronize(void) { return cudaSuccess; }
}

// Capture of verify_attn's hORef buffer: the global operator new/delete live
// in ref_hooks.cpp (host-only translation unit).
extern "C" void ref_capture_arm(size_t oref_bytes);
extern "C" int ref_capture_take(void* out, size_t nbytes);

// ---------------------------------------------------------------------------
// Runner passed to verify_attn: saves the inputs, leaves O = 0.
// ---------------------------------------------------------------------------
static std::vector<unsigned char> g_q, g_k, g_v;
static size_t g_qo_bytes = 0, g_kv_bytes = 0;

static void capture_runner(fp16* Q, fp16* K, fp16* V, fp16*) {
  g_q.assign(reinterpret_cast<unsigned char*>(Q), reinterpret_cast<unsigned char*>(Q) + g_qo_bytes);
  g_k.assign(reinterpret_cast<unsigned char*>(K), reinterpret_cast<unsigned char*>(K) + g_kv_bytes);
  g_v.assign(reinterpret_cast<unsigned char*>(V), reinterpret_cast<unsigned char*>(V) + g_kv_bytes);
}

static void noop_runner(fp16*, fp16*, fp16*, fp16*) {}

template <int B, int H, int S, int D, int BM, int BN>
static int golden(const std::string& outdir, const char* tag) {
  constexpr int SQO = ((S + BM - 1) / BM) * BM;
  constexpr int SKV = ((S + BN - 1) / BN) * BN;
  g_qo_bytes = static_cast<size_t>(B) * H * SQO * D * 2;
  g_kv_bytes = static_cast<size_t>(B) * H * SKV * D * 2;
  std::vector<unsigned char> oref(g_qo_bytes);
  ref_capture_arm(g_qo_bytes);
  verify_attn<B, H, S, D, BM, BN>(capture_runner);
  if (ref_capture_take(oref.data(), oref.size()) != 0 || g_q.size() != g_qo_bytes) {
    std::fprintf(stderr, "capture failed for %s\n", tag);
    return 1;
  }
  const std::string path = outdir + "/golden_" + tag + ".bin";
  FILE* f = std::fopen(path.c_str(), "wb");
  if (!f) return 1;
  const int hdr[8] = {B, H, S, D, BM, BN, SQO, SKV};
  std::fwrite(hdr, sizeof(int), 8, f);
  std::fwrite(g_q.data(), 1, g_q.size(), f);
  std::fwrite(g_k.data(), 1, g_k.size(), f);
  std::fwrite(g_v.data(), 1, g_v.size(), f);
  std::fwrite(oref.data(), 1, oref.size(), f);
  std::fclose(f);
  std::printf("wrote %s\n", path.c_str());
  return 0;
}

template <int B, int H, int S, int D, int BM, int BN>
static int timed(int threads, const char* cfg) {
  std::vector<std::thread> pool;
  // verify_attn prints two lines per call; silence them for the timing run.
  std::fflush(stdout);
  FILE* devnull = std::freopen("/dev/null", "w", stdout);
  (void)devnull;
  const auto t0 = std::chrono::steady_clock::now();
  for (int i = 0; i < threads; ++i)
    pool.emplace_back([] { verify_attn<B, H, S, D, BM, BN>(noop_runner); });
  for (auto& t : pool) t.join();
  const auto t1 = std::chrono::steady_clock::now();
  const double sec = std::chrono::duration<double>(t1 - t0).count();
  FILE* out = std::fopen("/dev/stderr", "w");
  const double flops = 4.0 * B * H * static_cast<double>(S) * S * D * threads;
  std::fprintf(out,
               "{\"cfg\": \"%s\", \"threads\": %d, \"heads\": %d, \"seconds\": %.6f, "
               "\"flops\": %.6e, \"tflops\": %.9f}\n",
               cfg, threads, B * H * threads, sec, flops, flops / sec / 1e12);
  std::fclose(out);
  return 0;
}

int main(int argc, char** argv) {
  if (argc >= 3 && std::strcmp(argv[1], "golden") == 0) {
    const std::string out = argv[2];
    int rc = 0;
    rc |= golden<1, 1, 256, 128, 128, 64>(out, "b1h1s256d128bn64");
    rc |= golden<1, 2, 200, 64, 128, 64>(out, "b1h2s200d64bn64");
    rc |= golden<2, 1, 96, 128, 128, 32>(out, "b2h1s96d128bn32");
    rc |= golden<1, 1, 512, 128, 128, 128>(out, "b1h1s512d128bn128");
    return rc;
  }
  if (argc >= 4 && std::strcmp(argv[1], "time") == 0) {
    const int threads = std::atoi(argv[3]);
    if (threads <= 0) return 2;
    if (std::strcmp(argv[2], "c1") == 0) return timed<1, 1, 512, 128, 128, 128>(threads, "c1");
    if (std::strcmp(argv[2], "c2head") == 0)
      return timed<1, 1, 4096, 128, 128, 128>(threads, "c2head");
    if (std::strcmp(argv[2], "c3head") == 0)
      return timed<1, 1, 4096, 64, 128, 128>(threads, "c3head");
    return 2;
  }
  std::fprintf(stderr, "usage: %s golden <outdir> | time <c1|c2head|c3head> <threads>\n", argv[0]);
  return 2;
}
