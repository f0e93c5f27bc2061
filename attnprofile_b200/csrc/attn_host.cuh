// Host side of the attention forward: tensor-map construction (cached),
// launch configuration and the C++ host entry attn<BM, BN>(...).
//
// Replaces the reference launchers runAttnWS2StageBaselineKernel /
// runAttnWS2StageSmemPKernel / runAttnWSForNSmemPKernel
// (tuning/attn_test.cu:1583-1663) and the tensor-map helper create_tensor_map
// (tuning/utils.cuh:33-69).  Differences that matter to callers:
//   * the stream is an argument (the reference always used the default stream);
//   * tensor maps are cached per (pointer, shape, box) instead of re-encoded
//     on every call (the reference encodes four per call);
//   * errors are returned as codes instead of exit(1)/assert;
//   * Q/O may have SQO >= S rows per head and K/V SKV >= S rows per head (the
//     reference's padded layout); rows >= S are never read (TMA fills zeros)
//     nor written (TMA clips the store).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <climits>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <mutex>
#include <unordered_map>

#if __has_include("attnprof.h")
#include "attnprof.h"
#else
#include "../../include/attnprof.h"  // builds without -I include (the tuning-harness driver)
#endif
#include "attn_kernel.cuh"

namespace attnprof {

constexpr int kSmemLimit = 232448;  // opt-in dynamic shared memory per CTA on sm_100

// Deepest K/V ring (at most `cap` slots) that fits the shared memory of one
// CTA, or of each of two CTAs on an SM for the variants built for two
// (AttnConfig::MIN_CTAS_PER_SM; the SM has 233472 bytes, 1 KB of which each
// CTA reserves).
template <typename T, int D, int BN, int NQ, bool PAIR = false>
constexpr int auto_stages(int cap = PAIR ? 12 : 8) {
  using C2 = AttnConfig<T, D, BN, NQ, 2, PAIR>;
  const int limit = C2::MIN_CTAS_PER_SM == 2 ? 233472 / 2 - 1024 : kSmemLimit;
  int best = 0;
  for (int s = 2; s <= cap; ++s) {
    const int bars = ((C2::NUM_BARS + 2 * (s - 2)) * 8 + 15) / 16 * 16;
    if (C2::OFF_KV + s * C2::KV_TILE_BYTES + C2::STAGE_BYTES + (bars > 256 ? bars : 256) +
            1024 + 32 <= limit)
      best = s;
  }
  return best;
}

// How the units (BM query rows of one (batch, head)) of one launch are laid
// out over CTAs: `whole` units run over all key tiles, the other
// units - whole are each split into `split` key ranges.
struct SplitPlan {
  int split = 1;
  long long units = 0, whole = 0, ctas = 0;
  size_t ws_bytes = 0;           // workspace for the split units (0: none)
  size_t off_ml = 0, off_cnt = 0, cnt_bytes = 0;
  // Persistent schedule: `ctas` resident CTAs, rr_rounds whole units each
  // round-robin, then total_steps tail steps (from step tail_base) shared
  // evenly; split = the most pieces any unit is cut into.
  bool persistent = false;
  long long rr_rounds = 0, tail_base = 0, total_steps = 0;
};

struct LaunchOpts {
  unsigned long long timeout_ns = 2000000000ull;  // bounded-wait limit: 2 s
  int fault_mode = 0;
  unsigned long long* prof = nullptr;
  int prof_cta = 0;
  int split = 0;                 // 0: automatic, 1: never split, k >= 2: split k ways
  int schedule = 0;              // 0: automatic, 1: classic only, 2: persistent where built
  bool corr = false;             // correction-warpgroup kernel where built (whole units)
  void* workspace = nullptr;     // caller-provided workspace (else stream-ordered pool)
  size_t workspace_bytes = 0;
  bool no_pool = false;          // never fall back to the pool: a split plan needs `workspace`
  SplitPlan* plan_out = nullptr; // receives the plan
  bool plan_only = false;        // compute the plan, launch nothing
  bool cache_maps = true;        // false: encode tensor maps per call, no host allocation
};

// Chooses the key split of the last, partially filled wave of units.  A
// wave of `slots` CTAs (SMs x resident CTAs per SM) runs one unit each; when
// units % slots leaves a partial wave, those units can instead run as k key
// ranges each (more, shorter CTAs), with the last range of each unit merging
// the k partial results.  Cost model in KV-tile periods, fitted to B200
// measurements (1x{1,2,4,6,16}x{1024..16384}x128, BM 256, BN 128): a whole
// unit costs n_kv + 2; a part ceil(n_kv / k) + 4 + k (its prologue and
// epilogue, the partial-O write and count-in, and the merge of k partials by
// the last part, which grows with k); a split launch adds 3 (workspace
// allocation and counter reset).  The split is taken when it saves at least
// 5 %.  It pays for few, long units (1x2x8192: 1.6x faster), not for a second
// wave of many (1x16x4096 stays unsplit).  mode: 0 automatic, 1 never,
// k >= 2 forced (when units % slots == 0, the last full wave is split).
inline SplitPlan plan_split(long long units, int n_kv, long long slots, int mode) {
  SplitPlan pl;
  pl.units = pl.whole = pl.ctas = units;
  if (mode == 1 || units <= 0 || n_kv < 2 || slots <= 0) return pl;
  const long long full = units / slots, rem = units % slots;
  const int kmax = std::min(kMaxSplit, n_kv);
  if (mode >= 2) {
    const long long nsplit = rem ? rem : std::min(units, slots);
    pl.split = std::min(mode, kmax);
    pl.whole = units - nsplit;
    pl.ctas = pl.whole + nsplit * pl.split;
    return pl;
  }
  if (rem == 0) return pl;
  double best = 0.95 * static_cast<double>(full + 1) * (n_kv + 2);
  for (int k = 2; k <= kmax; ++k) {
    const long long waves = (rem * k + slots - 1) / slots;
    const double c = static_cast<double>(full) * (n_kv + 2) +
                     static_cast<double>(waves) * ((n_kv + k - 1) / k + 4 + k) + 3.0;
    if (c < best) {
      best = c;
      pl.split = k;
    }
  }
  if (pl.split > 1) {
    pl.whole = full * slots;
    pl.ctas = pl.whole + rem * pl.split;
  }
  return pl;
}

// Persistent schedule (variants with AttnConfig::PERSIST_OK) on `grid`
// resident CTAs: with R = units / grid and r = units % grid, every CTA first
// runs R' whole units round-robin (R' = R when r = 0, else R - 1, at least 0),
// then an equal share of the remaining units' steps (the tail: the last
// r + grid units, or all of them when R = 0), so each share spans at least a
// unit whenever the units outnumber the CTAs.  Cost model in key-tile periods
// of one CTA: its steps, plus a fixed 2 (its first Q load and pipeline fill,
// its last epilogue), plus 0.5 per item boundary (the next item's first S is
// computed under the epilogue), plus, when its tail share starts or ends
// inside a unit, 1 (partial write) and 1.5 + 0.5 per further piece (merge).
// The grid size with the lowest cost wins; the classic plan (plan_split) is
// costed by its own model, and the persistent schedule is taken when it is
// no slower.
inline long long rr_rounds_of(long long units, long long grid) {
  const long long R = units / grid, r = units % grid;
  return r == 0 ? R : (R > 0 ? R - 1 : 0);
}

inline double persistent_cost(long long units, int n_kv, long long grid) {
  const long long rr = rr_rounds_of(units, grid);
  const long long Tt = (units - rr * grid) * n_kv;  // tail steps
  const long long share = (Tt + grid - 1) / grid;
  const long long items = rr + (share + n_kv - 1) / n_kv + 1;
  double c = static_cast<double>(rr * n_kv + share) + 2.0 + 0.5 * static_cast<double>(items - 1);
  if (Tt % grid != 0 || (Tt / grid) % n_kv != 0) {
    const long long pieces = std::min<long long>((n_kv + share - 1) / share + 1, 64);
    c += 1.0 + 1.5 + 0.5 * static_cast<double>(pieces - 1);
  }
  return c;
}

inline double classic_cost(const SplitPlan& pl, int n_kv, long long slots) {
  const long long nsplit = pl.units - pl.whole;
  const long long full_waves = (pl.whole + slots - 1) / slots;
  double c = static_cast<double>(full_waves) * (n_kv + 2);
  if (pl.split > 1 && nsplit > 0) {
    const long long waves = (nsplit * pl.split + slots - 1) / slots;
    c = static_cast<double>(pl.whole / slots) * (n_kv + 2) +
        static_cast<double>(waves) * ((n_kv + pl.split - 1) / pl.split + 4 + pl.split) + 3.0;
  }
  return c;
}

// The persistent plan for `units` units of n_kv key tiles on `slots`
// resident CTAs: the grid size with the lowest modelled cost (grid <= the
// tail's steps).
inline SplitPlan plan_persistent(long long units, int n_kv, long long slots) {
  SplitPlan pl;
  pl.persistent = true;
  pl.units = units;
  const long long gmax = std::min<long long>(slots, units * n_kv);
  long long best_g = gmax;
  double best = persistent_cost(units, n_kv, gmax);
  for (long long g = gmax - 1; g >= 1 && g >= gmax / 2; --g) {
    const double c = persistent_cost(units, n_kv, g);
    if (c < best - 1e-9) {
      best = c;
      best_g = g;
    }
  }
  pl.ctas = best_g;
  pl.rr_rounds = rr_rounds_of(units, best_g);
  pl.tail_base = pl.rr_rounds * best_g * n_kv;
  pl.total_steps = (units - pl.rr_rounds * best_g) * n_kv;  // tail steps
  // Units cut between CTAs, and the most pieces any of them has.
  long long cut_units = 0;
  int most = 1;
  const long long Tt = pl.total_steps;
  const int g = static_cast<int>(best_g);
  for (long long u0 = -1, c = 1; c < best_g; ++c) {
    const long long b = pl.tail_base + c * Tt / best_g;
    if (b % n_kv == 0) continue;
    const long long u = b / n_kv;
    if (u != u0) {
      ++cut_units;
      u0 = u;
      const long long first = step_owner(u * n_kv - pl.tail_base, Tt, g);
      const long long last = step_owner((u + 1) * n_kv - 1 - pl.tail_base, Tt, g);
      most = std::max<int>(most, static_cast<int>(last - first + 1));
    }
  }
  pl.split = most;
  pl.whole = units - cut_units;
  return pl;
}

// Workspace of a persistent plan with cut units: one partial block (BM x D
// f32) and one (max, sum) row block per CTA, one counter per (CTA, Q tile).
inline void plan_workspace_persistent(SplitPlan* pl, int BM, int D, int NQ) {
  auto up = [](size_t x) { return (x + 255) & ~static_cast<size_t>(255); };
  if (pl->split <= 1) return;
  const size_t g = static_cast<size_t>(pl->ctas);
  pl->off_ml = up(g * BM * D * sizeof(float));
  pl->off_cnt = pl->off_ml + up(g * BM * sizeof(float2));
  pl->cnt_bytes = g * NQ * sizeof(int);
  pl->ws_bytes = pl->off_cnt + up(pl->cnt_bytes);
}

// Workspace of a plan: partial O (pt_bytes per element), (max, sum) per row,
// one counter per (split unit, 128-row Q tile).  Each part 256-byte aligned.
inline void plan_workspace(SplitPlan* pl, int BM, int D, int NQ, size_t pt_bytes) {
  auto up = [](size_t x) { return (x + 255) & ~static_cast<size_t>(255); };
  if (pl->split <= 1) return;
  const size_t nsplit = static_cast<size_t>(pl->units - pl->whole);
  const size_t rows = nsplit * pl->split * BM;
  pl->off_ml = up(rows * D * pt_bytes);
  pl->off_cnt = pl->off_ml + up(rows * sizeof(float2));
  pl->cnt_bytes = nsplit * NQ * sizeof(int);
  pl->ws_bytes = pl->off_cnt + up(pl->cnt_bytes);
}

// Stream-ordered workspace from a per-device pool that keeps its memory
// (release threshold at the maximum), so steady-state calls map no pages.
inline int workspace_acquire(size_t bytes, cudaStream_t st, void** out) {
  static std::mutex mu;
  static cudaMemPool_t pools[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return ATTN_ERR_CUDA;
  cudaMemPool_t pool;
  {
    std::lock_guard<std::mutex> g(mu);
    if (pools[dev] == nullptr) {
      cudaMemPoolProps props{};
      props.allocType = cudaMemAllocationTypePinned;
      props.location.type = cudaMemLocationTypeDevice;
      props.location.id = dev;
      if (cudaMemPoolCreate(&pools[dev], &props) != cudaSuccess) {
        pools[dev] = nullptr;
        return ATTN_ERR_CUDA;
      }
      unsigned long long keep = ULLONG_MAX;
      cudaMemPoolSetAttribute(pools[dev], cudaMemPoolAttrReleaseThreshold, &keep);
    }
    pool = pools[dev];
  }
  if (cudaMallocFromPoolAsync(out, bytes, pool, st) != cudaSuccess) return ATTN_ERR_RESOURCE;
  return ATTN_OK;
}

// ---------------------------------------------------------------------------
// Driver entry point for cuTensorMapEncodeTiled (no link-time libcuda).
// ---------------------------------------------------------------------------
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_tiled_fn() {
  static EncodeTiledFn fn = []() -> EncodeTiledFn {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault,
                                         &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}

struct MapKey {
  uintptr_t ptr;
  int dtype, D, S, BH, box_rows;
  long long rows;
  bool operator==(const MapKey& o) const {
    return ptr == o.ptr && dtype == o.dtype && D == o.D && S == o.S && BH == o.BH &&
           box_rows == o.box_rows && rows == o.rows;
  }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    size_t h = std::hash<uintptr_t>()(k.ptr);
    auto mix = [&](long long v) { h ^= std::hash<long long>()(v) + 0x9e3779b97f4a7c15ull + (h << 6) + (h >> 2); };
    mix(k.dtype); mix(k.D); mix(k.S); mix(k.BH); mix(k.box_rows); mix(k.rows);
    return h;
  }
};

// 3-D map over a [B*H][rows][D] tensor: dims {D, S, B*H}; the row pitch is D
// elements and the head pitch `rows` rows, so rows >= S padding is skipped.
// Box {64, box_rows, 1} with 128-byte swizzle: one 64-column block per copy.
// use_cache = false encodes the map without touching the cache (no host
// allocation).
inline int get_tensor_map(CUtensorMap* out, const void* ptr, int dtype, int D, int S, int BH,
                          long long rows, int box_rows, bool use_cache = true) {
  static std::mutex mu;
  static std::unordered_map<MapKey, CUtensorMap, MapKeyHash> cache;
  const MapKey key{reinterpret_cast<uintptr_t>(ptr), dtype, D, S, BH, box_rows, rows};
  if (use_cache) {
    std::lock_guard<std::mutex> g(mu);
    auto it = cache.find(key);
    if (it != cache.end()) {
      *out = it->second;
      return ATTN_OK;
    }
  }
  EncodeTiledFn enc = encode_tiled_fn();
  if (enc == nullptr) return ATTN_ERR_CUDA;
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(S),
                              static_cast<cuuint64_t>(BH)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(D) * 2,
                                 static_cast<cuuint64_t>(rows) * D * 2};
  const cuuint32_t box[3] = {64u, static_cast<cuuint32_t>(box_rows), 1u};
  const cuuint32_t estr[3] = {1u, 1u, 1u};
  CUtensorMap m;
  const CUresult r = enc(&m, dtype == ATTN_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                      : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                         3, const_cast<void*>(ptr), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return ATTN_ERR_TENSOR_MAP;
  if (use_cache) {
    std::lock_guard<std::mutex> g(mu);
    if (cache.size() > 4096) cache.clear();
    cache.emplace(key, m);
  }
  *out = m;
  return ATTN_OK;
}

// Per-device status word written by the kernel's bounded waits.
int* device_status_ptr();

template <typename T, int D, int BN, int NQ, int STAGES, bool PROFILE, bool PAIR = false>
int launch_attn(const void* Q, const void* K, const void* V, void* O, int B, int H, int S,
                long long q_rows, long long kv_rows, cudaStream_t stream, const LaunchOpts& o) {
  using C = AttnConfig<T, D, BN, NQ, STAGES, PAIR>;
  static_assert(C::SMEM_BYTES <= kSmemLimit, "shared memory over the sm_100 per-CTA limit");
  const int dtype = std::is_same<T, __half>::value ? ATTN_DTYPE_F16 : ATTN_DTYPE_BF16;
  const long long BH = static_cast<long long>(B) * H;
  if (BH > INT_MAX) return ATTN_ERR_INVALID_ARG;  // the grid is 1-D over work tiles

  auto kern = attn_fwd_kernel<T, D, BN, NQ, STAGES, PROFILE, PAIR>;
  // The persistent schedule's kernel (the classic one again where the
  // variant has no persistent schedule).
  auto kern_p = attn_fwd_kernel<T, D, BN, NQ, STAGES, PROFILE, PAIR, C::PERSIST_OK>;
  // The classic schedule with a correction warpgroup (the classic kernel
  // again where the variant has none).
  constexpr bool kCorr = C::CORR_OK;
  using CC = AttnConfig<T, D, BN, NQ, STAGES, PAIR, kCorr>;
  static_assert(CC::SMEM_BYTES <= kSmemLimit, "shared memory over the sm_100 per-CTA limit");
  auto kern_c = attn_fwd_kernel<T, D, BN, NQ, STAGES, PROFILE, PAIR, false, kCorr>;
  const bool corr = kCorr && o.corr;
  // Eight-warp variants (AttnConfig::W8) store whole units only; their
  // four-warp kernel runs the launches whose plan splits units along the keys.
  using C4 = AttnConfig<T, D, BN, NQ, STAGES, PAIR, false, C::W8>;
  static_assert(C4::SMEM_BYTES <= kSmemLimit, "shared memory over the sm_100 per-CTA limit");
  auto kern_4 = attn_fwd_kernel<T, D, BN, NQ, STAGES, PROFILE, PAIR, false, false, C::W8>;
  // CTA pairs run as clusters of two consecutive CTAs.
  cudaLaunchAttribute cluster_attr{};
  cluster_attr.id = cudaLaunchAttributeClusterDimension;
  cluster_attr.val.clusterDim.x = C::CTAS;
  cluster_attr.val.clusterDim.y = 1;
  cluster_attr.val.clusterDim.z = 1;
  auto launch_cfg = [&](unsigned grid) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(C::NUM_THREADS);
    cfg.dynamicSmemBytes = C::SMEM_BYTES;
    cfg.stream = stream;
    cfg.attrs = &cluster_attr;
    cfg.numAttrs = 1;
    return cfg;
  };
  // Per-device set-up of this variant (shared-memory attribute, resident CTAs
  // per wave), once per device; thread-safe.
  static std::mutex init_mu;
  static std::atomic<int> slots_of[64];  // 0 until the device is set up
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) return ATTN_ERR_CUDA;
  int slots = dev < 64 ? slots_of[dev].load(std::memory_order_acquire) : 0;
  if (slots == 0) {
    std::lock_guard<std::mutex> g(init_mu);
    slots = dev < 64 ? slots_of[dev].load(std::memory_order_relaxed) : 0;
    if (slots == 0) {
      if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES) !=
              cudaSuccess ||
          cudaFuncSetAttribute(kern_p, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               C::SMEM_BYTES) != cudaSuccess ||
          cudaFuncSetAttribute(kern_c, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               CC::SMEM_BYTES) != cudaSuccess ||
          cudaFuncSetAttribute(kern_4, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               C4::SMEM_BYTES) != cudaSuccess)
        return ATTN_ERR_RESOURCE;
      int sms = 0, occ = 0;
      if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
          cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, C::NUM_THREADS,
                                                        C::SMEM_BYTES) != cudaSuccess)
        return ATTN_ERR_CUDA;
      if (occ < 1) return ATTN_ERR_RESOURCE;
      slots = sms * occ;
      if constexpr (PAIR) {
        // Resident pairs (both CTAs of a cluster on one GPC at once).
        int clusters = 0;
        const cudaLaunchConfig_t cfg = launch_cfg(static_cast<unsigned>(2 * sms));
        if (cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg) != cudaSuccess)
          return ATTN_ERR_CUDA;
        if (clusters < 1) return ATTN_ERR_RESOURCE;
        slots = clusters * C::CTAS;
      }
      if (dev < 64) slots_of[dev].store(slots, std::memory_order_release);
    }
  }
  // Units: BM rows of one (batch, head) per CTA, or 2 * BM per CTA pair (one
  // unit per cluster; pairs take no key split).
  const long long qt = (S + C::BM * C::CTAS - 1) / (C::BM * C::CTAS);
  const int n_kv = (S + BN - 1) / BN;
  // (The correction-warpgroup kernel stores whole units only: no key split.
  // An eight-warp variant whose plan splits runs its four-warp kernel.)
  SplitPlan plan = plan_split(BH * qt, n_kv, slots / C::CTAS, (PAIR || corr) ? 1 : o.split);
  const bool four = C::W8 && plan.split > 1;
  plan_workspace(&plan, C::BM, D, NQ, sizeof(float));
  // Persistent schedule: only when asked for (attn_set_schedule(2)), where
  // the variant has it and the split mode is automatic.  The automatic mode
  // runs the classic plan: on a B200 the persistent schedule measured within
  // -3 .. +2 % of it on the benchmark shapes and slower on few long units
  // (its per-CTA partial writes, merges and item boundaries cost about what
  // the classic grid's last wave leaves idle).  (A CTA's steps are counted
  // in 32 bits.)
  if (C::PERSIST_OK && !corr && o.split == 0 && o.schedule == 2 && BH * qt > 0 &&
      BH * qt * n_kv / slots < (1ll << 29)) {
    SplitPlan pp = plan_persistent(BH * qt, n_kv, slots);
    plan_workspace_persistent(&pp, C::BM, D, NQ);
    plan = pp;
  }
  if (o.plan_out) *o.plan_out = plan;
  if (o.plan_only) return ATTN_OK;
  if (plan.ctas * C::CTAS > INT_MAX || qt > INT_MAX) return ATTN_ERR_INVALID_ARG;

  CUtensorMap mq, mk, mv, mo;
  int rc;
  const int bhi = static_cast<int>(BH);
  if ((rc = get_tensor_map(&mq, Q, dtype, D, S, bhi, q_rows, C::QROWS, o.cache_maps))) return rc;
  if ((rc = get_tensor_map(&mk, K, dtype, D, S, bhi, kv_rows, C::K_ROWS, o.cache_maps))) return rc;
  if ((rc = get_tensor_map(&mv, V, dtype, D, S, bhi, kv_rows, BN, o.cache_maps))) return rc;
  if ((rc = get_tensor_map(&mo, O, dtype, D, S, bhi, q_rows, C::QROWS, o.cache_maps))) return rc;

  AttnParams p;
  p.S = S;
  p.num_kv_tiles = n_kv;
  p.qt_per_bh = static_cast<int>(qt);
  p.num_whole = static_cast<int>(plan.whole);
  p.split = plan.split;
  p.ws_o = nullptr;
  p.ws_ml = nullptr;
  p.ws_cnt = nullptr;
  p.scale_log2 = static_cast<float>(1.4426950408889634 / std::sqrt(static_cast<double>(D)));
  p.status = device_status_ptr();
  if (p.status == nullptr) return ATTN_ERR_CUDA;
  p.timeout_ns = o.timeout_ns;
  p.fault_mode = o.fault_mode;
  p.prof = o.prof;
  p.prof_cta = o.prof_cta;
  p.grid = static_cast<int>(plan.ctas);
  p.tail_steps = plan.total_steps;
  if (plan.persistent) p.num_whole = static_cast<int>(plan.rr_rounds);
  p.o_ptr = O;
  p.o_head_elems = q_rows * D;

  uint8_t* ws = nullptr;
  bool pooled = false;
  if (plan.split > 1) {  // classic key split, or units cut between persistent CTAs
    if (o.no_pool && (o.workspace == nullptr || o.workspace_bytes < plan.ws_bytes))
      return ATTN_ERR_SCRATCH_LIMIT;
    if (o.workspace != nullptr) {
      if (o.workspace_bytes < plan.ws_bytes) return ATTN_ERR_RESOURCE;
      ws = static_cast<uint8_t*>(o.workspace);
    } else {
      void* w = nullptr;
      if ((rc = workspace_acquire(plan.ws_bytes, stream, &w))) return rc;
      ws = static_cast<uint8_t*>(w);
      pooled = true;
    }
    p.ws_o = reinterpret_cast<float4*>(ws);
    p.ws_ml = reinterpret_cast<float2*>(ws + plan.off_ml);
    p.ws_cnt = reinterpret_cast<int*>(ws + plan.off_cnt);
    if (cudaMemsetAsync(p.ws_cnt, 0, plan.cnt_bytes, stream) != cudaSuccess) rc = ATTN_ERR_CUDA;
  }
  if (rc == ATTN_OK && plan.persistent) {
    // Cooperative launch: every CTA of the grid is resident at once, which
    // the merge of a unit cut between CTAs relies on (its merging CTA waits,
    // bounded, for pieces that other CTAs compute first).
    cudaLaunchAttribute coop{};
    coop.id = cudaLaunchAttributeCooperative;
    coop.val.cooperative = 1;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(static_cast<unsigned>(plan.ctas));
    cfg.blockDim = dim3(C::NUM_THREADS);
    cfg.dynamicSmemBytes = C::SMEM_BYTES;
    cfg.stream = stream;
    cfg.attrs = &coop;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, kern_p, mq, mk, mv, mo, p) != cudaSuccess) rc = ATTN_ERR_CUDA;
  } else if (rc == ATTN_OK) {
    if constexpr (PAIR) {
      const cudaLaunchConfig_t cfg = launch_cfg(static_cast<unsigned>(plan.ctas * C::CTAS));
      if (cudaLaunchKernelEx(&cfg, kern, mq, mk, mv, mo, p) != cudaSuccess) rc = ATTN_ERR_CUDA;
    } else if (corr) {
      kern_c<<<static_cast<unsigned>(plan.ctas), CC::NUM_THREADS, CC::SMEM_BYTES, stream>>>(
          mq, mk, mv, mo, p);
      if (cudaGetLastError() != cudaSuccess) rc = ATTN_ERR_CUDA;
    } else if (four) {
      kern_4<<<static_cast<unsigned>(plan.ctas), C4::NUM_THREADS, C4::SMEM_BYTES, stream>>>(
          mq, mk, mv, mo, p);
      if (cudaGetLastError() != cudaSuccess) rc = ATTN_ERR_CUDA;
    } else {
      kern<<<static_cast<unsigned>(plan.ctas), C::NUM_THREADS, C::SMEM_BYTES, stream>>>(mq, mk,
                                                                                       mv, mo, p);
      if (cudaGetLastError() != cudaSuccess) rc = ATTN_ERR_CUDA;
    }
  }
  if (pooled && cudaFreeAsync(ws, stream) != cudaSuccess && rc == ATTN_OK) rc = ATTN_ERR_CUDA;
  return rc;
}

}  // namespace attnprof
