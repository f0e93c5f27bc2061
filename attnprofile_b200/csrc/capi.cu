// extern "C" entry points declared in include/attnprof.h.
#include <cuda_runtime.h>

#include <atomic>
#include <climits>
#include <mutex>
#include <vector>

#include "dispatch.cuh"

namespace attnprof {

ATTNPROF_DECLARE(__half, 64, false)
ATTNPROF_DECLARE(__half, 128, false)
ATTNPROF_DECLARE(__nv_bfloat16, 64, false)
ATTNPROF_DECLARE(__nv_bfloat16, 128, false)
ATTNPROF_DECLARE(__half, 64, true)
ATTNPROF_DECLARE(__half, 128, true)
ATTNPROF_DECLARE(__nv_bfloat16, 64, true)
ATTNPROF_DECLARE(__nv_bfloat16, 128, true)

// One status word per device (each device's module holds its own copy).
__device__ int g_attn_status;

namespace {
std::atomic<unsigned long long> g_timeout_ns{2000000000ull};
std::atomic<int> g_fault_mode{0};
std::atomic<int> g_split_mode{0};
std::atomic<int> g_schedule_mode{0};
std::atomic<int> g_corr_mode{0};
constexpr int kMaxDev = 64;
std::mutex g_status_mu;
int* g_status_ptr[kMaxDev] = {};
}  // namespace

int* device_status_ptr() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDev) return nullptr;
  std::lock_guard<std::mutex> g(g_status_mu);
  if (g_status_ptr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_attn_status) != cudaSuccess) return nullptr;
    g_status_ptr[dev] = static_cast<int*>(p);
  }
  return g_status_ptr[dev];
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

static int validate(const void* Q, const void* K, const void* V, const void* O, int B, int H,
                    int S, int D, long long SQO, long long SKV, int dtype) {
  if (B < 0 || H < 0 || S < 0) return ATTN_ERR_INVALID_ARG;
  if (dtype != ATTN_DTYPE_F16 && dtype != ATTN_DTYPE_BF16) return ATTN_ERR_UNSUPPORTED;
  if (D != 64 && D != 128) return ATTN_ERR_UNSUPPORTED;
  if (B == 0 || H == 0 || S == 0) return ATTN_OK;  // empty problem: nothing to do
  if (!Q || !K || !V || !O) return ATTN_ERR_INVALID_ARG;
  if (SQO < S || SKV < S) return ATTN_ERR_INVALID_ARG;
  if (static_cast<long long>(B) * H > INT_MAX) return ATTN_ERR_INVALID_ARG;
  if (!aligned16(Q) || !aligned16(K) || !aligned16(V) || !aligned16(O)) return ATTN_ERR_MISALIGNED;
  return 1;  // proceed
}

static int dispatch(const void* Q, const void* K, const void* V, void* O, int B, int H, int S,
                    int D, long long SQO, long long SKV, int dtype, int BM, int BN, cudaStream_t st,
                    const LaunchOpts& o);

static int run(const void* Q, const void* K, const void* V, void* O, int B, int H, int S, int D,
               long long SQO, long long SKV, int dtype, int BM, int BN, cudaStream_t st,
               unsigned long long* prof, int prof_cta) {
  const int v = validate(Q, K, V, O, B, H, S, D, SQO, SKV, dtype);
  if (v <= 0) return v;
  LaunchOpts o;
  o.timeout_ns = g_timeout_ns.load();
  o.fault_mode = g_fault_mode.load();
  o.prof = prof;
  o.prof_cta = prof_cta;
  o.split = g_split_mode.load();
  o.schedule = g_schedule_mode.load();
  o.corr = g_corr_mode.load() != 0;
  return dispatch(Q, K, V, O, B, H, S, D, SQO, SKV, dtype, BM, BN, st, o);
}

static int dispatch(const void* Q, const void* K, const void* V, void* O, int B, int H, int S,
                    int D, long long SQO, long long SKV, int dtype, int BM, int BN, cudaStream_t st,
                    const LaunchOpts& o) {
  const bool pf = o.prof != nullptr;
  if (dtype == ATTN_DTYPE_F16) {
    if (D == 64)
      return pf ? dispatch_attn<__half, 64, true>(BM, BN, Q, K, V, O, B, H, S, SQO, SKV, st, o)
                : dispatch_attn<__half, 64, false>(BM, BN, Q, K, V, O, B, H, S, SQO, SKV, st, o);
    return pf ? dispatch_attn<__half, 128, true>(BM, BN, Q, K, V, O, B, H, S, SQO, SKV, st, o)
              : dispatch_attn<__half, 128, false>(BM, BN, Q, K, V, O, B, H, S, SQO, SKV, st, o);
  }
  if (D == 64)
    return pf ? dispatch_attn<__nv_bfloat16, 64, true>(BM, BN, Q, K, V, O, B, H, S, SQO, SKV, st, o)
              : dispatch_attn<__nv_bfloat16, 64, false>(BM, BN, Q, K, V, O, B, H, S, SQO, SKV, st, o);
  return pf ? dispatch_attn<__nv_bfloat16, 128, true>(BM, BN, Q, K, V, O, B, H, S, SQO, SKV, st, o)
            : dispatch_attn<__nv_bfloat16, 128, false>(BM, BN, Q, K, V, O, B, H, S, SQO, SKV, st, o);
}

// The key-split mode attn_set_split last stored.
int current_split_mode() { return g_split_mode.load(); }

// Launch with a caller-provided workspace and per-call tensor maps (no
// device or host allocation, never the stream-ordered pool: a plan that
// needs more than ws_bytes returns ATTN_ERR_SCRATCH_LIMIT); split_mode as
// for attn_set_split, the other settings as for attn_fwd.  When plan_only is
// set, only *plan is filled.  Used by attn_fwd_noalloc.
int run_in_workspace(const void* Q, const void* K, const void* V, void* O, int B, int H, int S,
                     int D, int dtype, int BM, int BN, cudaStream_t st, int split_mode, void* ws,
                     size_t ws_bytes, SplitPlan* plan, bool plan_only) {
  const int v = validate(Q, K, V, O, B, H, S, D, S, S, dtype);
  if (v <= 0) return v;
  LaunchOpts o;
  o.timeout_ns = g_timeout_ns.load();
  o.fault_mode = g_fault_mode.load();
  o.split = split_mode;
  o.schedule = g_schedule_mode.load();
  o.corr = g_corr_mode.load() != 0;
  o.workspace = ws;
  o.workspace_bytes = ws_bytes;
  o.no_pool = true;
  o.plan_out = plan;
  o.plan_only = plan_only;
  o.cache_maps = false;
  return dispatch(Q, K, V, O, B, H, S, D, S, S, dtype, BM, BN, st, o);
}

}  // namespace attnprof

using namespace attnprof;

extern "C" {

int attn_fwd(const void* Q, const void* K, const void* V, void* O, int B, int H, int S, int D,
             int dtype, int BM, int BN, void* stream) {
  return run(Q, K, V, O, B, H, S, D, S, S, dtype, BM, BN, static_cast<cudaStream_t>(stream),
             nullptr, 0);
}

int attn_fwd_padded(const void* Q, const void* K, const void* V, void* O, int B, int H, int S,
                    int D, int SQO, int SKV, int dtype, int BM, int BN, void* stream) {
  return run(Q, K, V, O, B, H, S, D, SQO, SKV, dtype, BM, BN, static_cast<cudaStream_t>(stream),
             nullptr, 0);
}

int attn_fwd_profiled(const void* Q, const void* K, const void* V, void* O, int B, int H, int S,
                      int D, int dtype, int BM, int BN, void* stream,
                      unsigned long long* dev_profile_buf, int profile_cta) {
  if (dev_profile_buf == nullptr || profile_cta < 0) return ATTN_ERR_INVALID_ARG;
  return run(Q, K, V, O, B, H, S, D, S, S, dtype, BM, BN, static_cast<cudaStream_t>(stream),
             dev_profile_buf, profile_cta);
}

int attn_profile_layout(int* phases, int* slots) {
  if (phases) *phases = kProfPhases;
  if (slots) *slots = kProfSlots;
  return ATTN_OK;
}

int attn_shard_range(int units, int n_dev, int g, int* begin, int* end) {
  if (units < 0 || n_dev <= 0 || g < 0 || g >= n_dev || !begin || !end) return ATTN_ERR_SHARD;
  *begin = static_cast<int>(static_cast<long long>(units) * g / n_dev);
  *end = static_cast<int>(static_cast<long long>(units) * (g + 1) / n_dev);
  return ATTN_OK;
}

int attn_fwd_sharded(int n_dev, const int* devices, const void* const* Q, const void* const* K,
                     const void* const* V, void* const* O, int B, int H, int S, int D, int dtype,
                     int BM, int BN, float* ms_per_device) {
  if (n_dev <= 0 || n_dev > 64 || !devices || !Q || !K || !V || !O) return ATTN_ERR_SHARD;
  if (B < 0 || H < 0 || S < 0) return ATTN_ERR_INVALID_ARG;
  int prev = 0;
  if (cudaGetDevice(&prev) != cudaSuccess) return ATTN_ERR_CUDA;
  const int units = B * H;
  struct Slot {
    cudaStream_t st = nullptr;
    cudaEvent_t a = nullptr, b = nullptr;
    int rc = ATTN_OK;
    bool launched = false;
  };
  static std::mutex mu;
  static cudaStream_t streams[64] = {};
  std::vector<Slot> slot(n_dev);
  int rc = ATTN_OK;
  for (int g = 0; g < n_dev; ++g) {
    int u0, u1;
    attn_shard_range(units, n_dev, g, &u0, &u1);
    if (cudaSetDevice(devices[g]) != cudaSuccess) { rc = ATTN_ERR_CUDA; break; }
    {
      std::lock_guard<std::mutex> lk(mu);
      const int d = devices[g];
      if (d < 0 || d >= 64) { rc = ATTN_ERR_SHARD; break; }
      if (streams[d] == nullptr &&
          cudaStreamCreateWithFlags(&streams[d], cudaStreamNonBlocking) != cudaSuccess) {
        rc = ATTN_ERR_CUDA;
        break;
      }
      slot[g].st = streams[d];
    }
    if (u1 == u0) continue;
    if (cudaEventCreate(&slot[g].a) != cudaSuccess || cudaEventCreate(&slot[g].b) != cudaSuccess) {
      rc = ATTN_ERR_CUDA;
      break;
    }
    cudaEventRecord(slot[g].a, slot[g].st);
    slot[g].rc = run(Q[g], K[g], V[g], O[g], 1, u1 - u0, S, D, S, S, dtype, BM, BN, slot[g].st,
                     nullptr, 0);
    cudaEventRecord(slot[g].b, slot[g].st);
    slot[g].launched = true;
    if (slot[g].rc != ATTN_OK) { rc = slot[g].rc; }
  }
  // Join every device that got work, also after an error on another one.
  for (int g = 0; g < n_dev; ++g) {
    if (!slot[g].launched) {
      if (ms_per_device) ms_per_device[g] = 0.f;
      continue;
    }
    cudaSetDevice(devices[g]);
    if (cudaEventSynchronize(slot[g].b) != cudaSuccess && rc == ATTN_OK) rc = ATTN_ERR_CUDA;
    float ms = 0.f;
    cudaEventElapsedTime(&ms, slot[g].a, slot[g].b);
    if (ms_per_device) ms_per_device[g] = ms;
    const int st = attn_get_status(devices[g], 0, nullptr);
    if (st != ATTN_OK && rc == ATTN_OK) rc = st;
    cudaEventDestroy(slot[g].a);
    cudaEventDestroy(slot[g].b);
  }
  cudaSetDevice(prev);
  return rc;
}

int attn_get_status(int device, int reset, int* site) {
  int prev = 0;
  if (cudaGetDevice(&prev) != cudaSuccess) return ATTN_ERR_CUDA;
  if (cudaSetDevice(device) != cudaSuccess) return ATTN_ERR_CUDA;
  int rc = ATTN_OK;
  int v = 0;
  if (cudaDeviceSynchronize() != cudaSuccess ||
      cudaMemcpyFromSymbol(&v, g_attn_status, sizeof(int)) != cudaSuccess) {
    rc = ATTN_ERR_CUDA;
  } else {
    if (site) *site = v;
    if (v != 0) rc = ATTN_ERR_DEVICE_TIMEOUT;
    if (reset) {
      const int z = 0;
      if (cudaMemcpyToSymbol(g_attn_status, &z, sizeof(int)) != cudaSuccess) rc = ATTN_ERR_CUDA;
    }
  }
  cudaSetDevice(prev);
  return rc;
}

void attn_set_timeout_ns(unsigned long long ns) { g_timeout_ns.store(ns ? ns : 1ull); }

int attn_query_config(int D, int BM, int BN, int dtype, int* num_threads, int* smem_bytes,
                      int* tmem_cols, int* stages) {
  if (dtype != ATTN_DTYPE_F16 && dtype != ATTN_DTYPE_BF16) return ATTN_ERR_UNSUPPORTED;
  VariantInfo vi{};
  int rc;
  if (dtype == ATTN_DTYPE_F16)
    rc = D == 64 ? query_variant<__half, 64>(BM, BN, &vi)
                 : D == 128 ? query_variant<__half, 128>(BM, BN, &vi) : ATTN_ERR_UNSUPPORTED;
  else
    rc = D == 64 ? query_variant<__nv_bfloat16, 64>(BM, BN, &vi)
                 : D == 128 ? query_variant<__nv_bfloat16, 128>(BM, BN, &vi)
                            : ATTN_ERR_UNSUPPORTED;
  if (rc != ATTN_OK) return rc;
  if (num_threads) *num_threads = vi.num_threads;
  if (smem_bytes) *smem_bytes = vi.smem_bytes;
  if (tmem_cols) *tmem_cols = vi.tmem_cols;
  if (stages) *stages = vi.stages;
  return ATTN_OK;
}

const char* attn_error_string(int code) {
  switch (code) {
    case ATTN_OK: return "ok";
    case ATTN_ERR_INVALID_ARG: return "invalid argument";
    case ATTN_ERR_UNSUPPORTED: return "unsupported dtype / head dim / tile combination";
    case ATTN_ERR_MISALIGNED: return "tensor base address not 16-byte aligned";
    case ATTN_ERR_CUDA: return "CUDA runtime error";
    case ATTN_ERR_TENSOR_MAP: return "TMA tensor map encoding failed";
    case ATTN_ERR_DEVICE_TIMEOUT: return "bounded in-kernel wait expired (device timeout)";
    case ATTN_ERR_RESOURCE: return "shared memory or tensor memory request over the limit";
    case ATTN_ERR_SHARD: return "invalid multi-GPU partition";
    case ATTN_ERR_SCRATCH_LIMIT:
      return "problem needs more scratch than the fixed no-allocation buffer holds "
             "(ATTN_NOALLOC_SCRATCH_BYTES); use attn_fwd";
    default: return "unknown error";
  }
}

int attn_set_split(int mode) {
  if (mode < 0 || mode > kMaxSplit) return ATTN_ERR_INVALID_ARG;
  g_split_mode.store(mode);
  return ATTN_OK;
}

int attn_set_schedule(int mode) {
  if (mode < 0 || mode > 2) return ATTN_ERR_INVALID_ARG;
  g_schedule_mode.store(mode);
  return ATTN_OK;
}

int attn_set_correction(int mode) {
  if (mode < 0 || mode > 1) return ATTN_ERR_INVALID_ARG;
  g_corr_mode.store(mode);
  return ATTN_OK;
}

int attn_plan_schedule(long long units, int num_kv_tiles, long long slots, int* persistent,
                       long long* ctas, int* pieces, double* persistent_cost_out,
                       double* classic_cost_out) {
  if (units <= 0 || num_kv_tiles <= 0 || slots <= 0) return ATTN_ERR_INVALID_ARG;
  const SplitPlan cl = plan_split(units, num_kv_tiles, slots, 0);
  const SplitPlan pp = plan_persistent(units, num_kv_tiles, slots);
  const double cp = persistent_cost(units, num_kv_tiles, pp.ctas);
  const double cc = classic_cost(cl, num_kv_tiles, slots);
  if (persistent) *persistent = 0;  // the automatic mode runs the classic plan
  if (ctas) *ctas = pp.ctas;
  if (pieces) *pieces = pp.split;
  if (persistent_cost_out) *persistent_cost_out = cp;
  if (classic_cost_out) *classic_cost_out = cc;
  return ATTN_OK;
}

int attn_plan_split(long long units, int num_kv_tiles, long long slots, int mode, int* split,
                    long long* whole_units, long long* ctas) {
  if (units < 0 || num_kv_tiles < 0 || slots <= 0 || mode < 0 || mode > kMaxSplit)
    return ATTN_ERR_INVALID_ARG;
  const SplitPlan pl = plan_split(units, num_kv_tiles, slots, mode);
  if (split) *split = pl.split;
  if (whole_units) *whole_units = pl.whole;
  if (ctas) *ctas = pl.ctas;
  return ATTN_OK;
}

int attn_query_split(int B, int H, int S, int D, int dtype, int BM, int BN, int* split,
                     long long* whole_units, long long* ctas, unsigned long long* workspace_bytes) {
  if (B < 0 || H < 0 || S < 0) return ATTN_ERR_INVALID_ARG;
  if (dtype != ATTN_DTYPE_F16 && dtype != ATTN_DTYPE_BF16) return ATTN_ERR_UNSUPPORTED;
  if (D != 64 && D != 128) return ATTN_ERR_UNSUPPORTED;
  SplitPlan pl;
  LaunchOpts o;
  o.split = g_split_mode.load();
  o.schedule = g_schedule_mode.load();
  o.corr = g_corr_mode.load() != 0;
  o.plan_out = &pl;
  o.plan_only = true;
  const int rc = dispatch(nullptr, nullptr, nullptr, nullptr, B, H, S, D, S, S, dtype, BM, BN,
                          nullptr, o);
  if (rc != ATTN_OK) return rc;
  if (split) *split = pl.split;
  if (whole_units) *whole_units = pl.whole;
  if (ctas) *ctas = pl.ctas;
  if (workspace_bytes) *workspace_bytes = pl.ws_bytes;
  return ATTN_OK;
}

int attn_debug_fault(int mode) {
  if (mode != 0 && mode != 1) return ATTN_ERR_INVALID_ARG;
  g_fault_mode.store(mode);
  return ATTN_OK;
}

int attn_version(void) { return 100; }

}  // extern "C"
