// attn_fwd_noalloc: attention forward that allocates no GPU memory.
//
// Who needs it: callers that cannot call cudaMalloc at the point where they
// launch attention -- a CUDA graph under stream capture, a serving process
// that reserved its whole memory budget up front, code running inside an
// allocator hook.  attn_fwd takes the scratch of a key-split launch (partial
// O, row statistics, merge counters) from a stream-ordered pool; this entry
// point takes it from one fixed array below instead, so a launch here never
// allocates.  The price is a fixed footprint: every GPU on which this entry
// point runs holds kScratchBytes until the process exits.
#include <cuda_runtime.h>

#include <mutex>

#include "attn_host.cuh"

namespace attnprof {
int run_in_workspace(const void* Q, const void* K, const void* V, void* O, int B, int H, int S,
                     int D, int dtype, int BM, int BN, cudaStream_t st, void* ws,
                     size_t ws_bytes, SplitPlan* plan, bool plan_only);
}  // namespace attnprof

namespace {

constexpr size_t kScratchBytes = ATTN_NOALLOC_SCRATCH_BYTES;
static_assert(kScratchBytes % 256 == 0, "scratch size must keep 256-byte alignment");

// One array per GPU (each device's copy of this module has its own).  In host
// code this name stands for the symbol, not for device memory: its device
// address comes from cudaGetSymbolAddress, looked up below per device.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_scratch_addr[kMaxDevices] = {};

// Device address of the current device's scratch array.  Looked up once per
// device, on the first call made with that device current.
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
  // The plan first: a launch whose scratch would not fit is refused before
  // anything is launched.
  SplitPlan plan;
  int rc = run_in_workspace(Q, K, V, O, B, H, S, D, dtype, BM, BN, st, nullptr, 0, &plan, true);
  if (rc != ATTN_OK || B == 0 || H == 0 || S == 0) return rc;
  if (plan.ws_bytes > kScratchBytes) return ATTN_ERR_SCRATCH_LIMIT;
  void* scratch = nullptr;
  if (plan.ws_bytes > 0 && (rc = scratch_of_current_device(&scratch)) != ATTN_OK) return rc;
  // With a workspace given, the launch uses it as is and zeroes its merge
  // counters on `st` (cudaMemsetAsync) before the kernel; partial results
  // left by an earlier call are overwritten before they are read.
  return run_in_workspace(Q, K, V, O, B, H, S, D, dtype, BM, BN, st, scratch, kScratchBytes,
                          nullptr, false);
}
