// attn_fwd_noalloc: attention forward that allocates no GPU memory.
//
// Who needs it: callers that are not allowed to call cudaMalloc (or a pool
// allocation) at the moment they launch attention.  A serving process that
// reserved its whole GPU memory budget when it started hands its kernels
// pre-sized buffers and keeps every other byte for its own use; a custom
// allocator, or code called back from inside one, must not re-enter the CUDA
// allocator; a latency-bound loop cannot take the device-wide stall that
// cudaMalloc / cudaFree can bring.  attn_fwd takes the scratch of a key-split
// launch (partial O, row statistics, merge counters) from a stream-ordered
// pool; this entry point takes it from one fixed array in this file instead,
// so a launch here never allocates.
//
// The price is a fixed footprint.  The array is a __device__ variable of
// this library, so it is part of the library's module on every GPU the
// module is loaded on: with lazy module loading (the CUDA default) from the
// first attn_fwd_noalloc call on that GPU, with CUDA_MODULE_LOADING=EAGER
// from the moment the process creates its context there, whether or not
// attn_fwd_noalloc is ever called.  It stays until the process exits.
#include <cuda_runtime.h>

#include <mutex>

#include "attn_host.cuh"

namespace attnprof {
int run_in_workspace(const void* Q, const void* K, const void* V, void* O, int B, int H, int S,
                     int D, int dtype, int BM, int BN, cudaStream_t st, int split_mode, void* ws,
                     size_t ws_bytes, SplitPlan* plan, bool plan_only);
int current_split_mode();
}  // namespace attnprof

namespace {

constexpr size_t kScratchBytes = ATTN_NOALLOC_SCRATCH_BYTES;
static_assert(kScratchBytes % 256 == 0, "scratch size must keep 256-byte alignment");

// One array per GPU (each device's copy of this module has its own).  In host
// code this name stands for the symbol, not for device memory: a kernel given
// &g_noalloc_scratch from host code would read host-side storage.  Its device
// address comes from cudaGetSymbolAddress, looked up below per device.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_scratch_addr[kMaxDevices] = {};

// Device address of the current device's scratch array.  Looked up once per
// device, on the first call made with that device current (that lookup is
// the only set-up; every later call on the device reuses the address).
int scratch_of_current_device(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return ATTN_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr)
      return ATTN_ERR_CUDA;
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return ATTN_OK;
}

}  // namespace

extern "C" int attn_fwd_noalloc(const void* Q, const void* K, const void* V, void* O, int B,
                                int H, int S, int D, int dtype, int BM, int BN, void* stream) {
  using namespace attnprof;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  // One reading of the split mode for both the size check and the launch, so
  // an attn_set_split from another thread cannot make them disagree.
  const int mode = current_split_mode();
  // The plan first: a launch whose scratch would not fit is refused before
  // anything is launched.
  SplitPlan plan;
  int rc = run_in_workspace(Q, K, V, O, B, H, S, D, dtype, BM, BN, st, mode, nullptr, 0, &plan,
                            true);
  if (rc != ATTN_OK || B == 0 || H == 0 || S == 0) return rc;
  if (plan.ws_bytes > kScratchBytes) return ATTN_ERR_SCRATCH_LIMIT;
  // Every call on a device resolves the array's address, whether or not this
  // plan splits, so the first call on a device always does the lookup.
  void* scratch = nullptr;
  if ((rc = scratch_of_current_device(&scratch)) != ATTN_OK) return rc;
  // With a workspace given and no pool allowed, the launch uses the array as
  // is (a plan that outgrew it returns ATTN_ERR_SCRATCH_LIMIT) and zeroes its
  // merge counters on `st` (cudaMemsetAsync) before the kernel; partial
  // results left by an earlier call are overwritten before they are read.
  return run_in_workspace(Q, K, V, O, B, H, S, D, dtype, BM, BN, st, mode, scratch, kScratchBytes,
                          nullptr, false);
}
