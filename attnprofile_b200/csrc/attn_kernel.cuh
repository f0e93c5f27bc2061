// Non-causal attention forward O = softmax(Q K^T / sqrt(D)) V for sm_100a.
//
// Computes what the reference's warp-specialised Hopper kernels compute
// (tuning/attn_test.cu:50-523 attnWS2StageBaselineKernel, :526-1055,
// :1058-1580), with the reference's tail semantics (key columns >= S masked
// before the softmax, tuning/attn_test.cu:152-170), built on Blackwell units:
//
//   * one TMA producer warp loads the Q tile(s) once and streams K and V tiles
//     through a STAGES-deep ring of 128B-swizzled shared-memory slots guarded
//     by full/empty mbarriers (with one S buffer per tile, one empty commit
//     per step frees both the V_j and the K_{j+1} slot);
//   * one MMA warp (a single elected lane; one per Q tile when S is
//     double-buffered in a two-tile CTA) issues tcgen05.mma:
//       S_i = Q_i K_j^T    (A, B from shared memory, D in TMEM, f32)
//       O_i += P_i V_j     (A = P read from TMEM, B = V from shared memory)
//     and signals completion with tcgen05.commit onto mbarriers;
//   * NQ softmax warpgroups (one per 128-row Q tile; thread t owns row t, which
//     is TMEM lane t) read S with tcgen05.ld, run the online softmax in fp32
//     with exp2 on the MUFU unit, write P (f16/bf16) back into TMEM over the S
//     columns, and rescale O in TMEM only when the running row max grew by
//     more than RESCALE_THRESHOLD (log2 units) -- the lazy correction step;
//   * the same warpgroups finish the tile: O / rowsum, convert, stage in the
//     (now free) Q shared-memory slot with the TMA 128B swizzle, TMA store.
//
// BM = 128 * NQ rows of Q per CTA (a unit), or one key range of a unit when
// the launch splits its last wave along the keys (WorkTile; the parts' partial
// results are merged by the part that finishes last).  With NQ = 2 and one S
// buffer per Q tile the two softmax warpgroups ping-pong: while one runs exp2
// on its S tile the tensor core runs the other tile's P V and next Q K^T.  The
// S accumulator is double-buffered in TMEM whenever it fits
// (NQ * (2 * BN + D) <= 512 columns) so Q K_{j+1}^T overlaps the softmax of
// tile j; two-tile CTAs then issue each tile's MMAs from its own warp.
//
// CTA pairs (AttnConfig::PAIR, BM = 512 on the host): a cluster of two
// two-tile CTAs whose tile i shares one cta_group::2 MMA of M = 256; each CTA
// loads half of every K and V tile, the even CTA issues the MMAs and fans
// its commits out to both, a relay thread in the odd CTA forwards the
// landing of its loads to the even CTA's barriers.
//
// Every wait is bounded (see wait_bar): on expiry the kernel records an error
// code in a device status word, raises a CTA-local abort flag so the other
// roles stop waiting, drains its own outstanding tensor-core work and returns
// (a pair's two CTAs then meet at the final cluster barrier).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cstdint>

#include "ptx.cuh"

namespace attnprof {

// Status codes written by the kernel (the first error wins).  The host maps
// them to ATTNPROF_ERR_DEVICE_TIMEOUT.
enum : int {
  kSiteQ = 1,
  kSiteKvFull = 2,
  kSiteKvEmpty = 3,
  kSiteSFull = 4,
  kSitePReady = 5,
  kSiteODone = 6,
  kSiteDrain = 7,
  kSiteQFree = 8,
  kSiteMerge = 9,
  kSiteStage = 10,
  kSiteCorr = 11,
  kDeviceTimeoutBase = 0x7100,
};

// Phase profiler layout (one designated CTA): [phase][slot][begin,end] u64
// clock64 stamps, the first kProfSlots KV iterations.  The phases are those of
// the reference's profiler (attn.cu:5-22): LoadQ, LoadK, LoadV, GEMM-QK,
// SOFTMAX, GEMM-PV.
// Four more phases split SOFTMAX of the profiled warp into its steps: the S
// load from TMEM, the row max (and lazy-rescale decision), the exponentials
// with the P stores issued, and the wait for the P stores to land.
// The last phase, Epilogue, is stamped once per CTA by the same warp, its
// slots holding steps instead of iterations: 0 the whole epilogue (loop exit
// to the O store issued, or to the exit of a part that does not merge),
// 1 the wait for the last P V, 2 the partial-O write of a split part,
// 3 its count-in, 4 the merge (split) or the O normalisation into shared
// memory (whole unit), 5 the TMA store issue.
// Three trace phases relate the Q tiles of a two-tile CTA: 11 SOFTMAX of
// tile 1 (its S observed -> its last P part signalled), 12 and 13 the MMA
// issuer's window for tile 0 / tile 1 (first P part observed -> the tile's
// next S issued, or its last P V committed); 14 the first P part signalled
// by tile 0 (begin) and by tile 1 (end); 15 the MMA issuer's wait for V_j
// (wait entered -> V_j observed landed); 16 its wait for K_{j+1}.
constexpr int kProfPhases = 17;
constexpr int kProfSlots = 32;
enum : int {
  kPhLoadQ = 0, kPhLoadK = 1, kPhLoadV = 2, kPhQK = 3, kPhSoftmax = 4, kPhPV = 5,
  kPhSmLoadS = 6, kPhSmMax = 7, kPhSmExp = 8, kPhSmStoreP = 9, kPhEpilogue = 10,
  kPhSoftmaxT1 = 11, kPhMmaT0 = 12, kPhMmaT1 = 13, kPhPFirst = 14, kPhVWait = 15, kPhKWait = 16
};
enum : int {
  kEpAll = 0, kEpWaitO = 1, kEpPartial = 2, kEpCount = 3, kEpMerge = 4, kEpStore = 5
};

struct AttnParams {
  int S;                       // logical sequence length (rows of Q and of K/V per head)
  int num_kv_tiles;            // ceil(S / BN)
  // Work decomposition (1-D grid).  Unit u = bh * qt_per_bh + q tile (BM rows
  // of one (batch, head)).  CTAs [0, num_whole) run units 0 .. num_whole-1
  // over all KV tiles; each remaining unit is split into `split` key ranges
  // (1 < split <= kMaxSplit, split <= num_kv_tiles), one CTA each, merged by
  // whichever of them finishes last.  No split: num_whole = all units.
  int qt_per_bh;
  int num_whole;               // persistent schedule: round-robin rounds of whole units
  int split;
  float4* ws_o;                // [split units][split][D / 4][BM] (float4 columns of partial O)
  float2* ws_ml;               // [split units][split][BM]: (row max in raw score units, row sum)
  int* ws_cnt;                 // [split units][NQ]: parts finished; zero between launches
  float scale_log2;            // log2(e) / sqrt(D)
  int* status;                 // device status word (0 = ok)
  unsigned long long timeout_ns;
  int fault_mode;              // 0 normal; 1 = producer never loads K/V (test of bounded waits)
  unsigned long long* prof;    // PROFILE builds: stamp buffer, may be null
  int prof_cta;                // linear CTA index to profile
  // Persistent schedule (the kernel's PERSIST variant): the grid is `grid`
  // CTAs that are all resident at once.  CTA c first runs the whole units
  // c, c + grid, ... (num_whole of them, "rounds"), then the tail: steps
  // [base + c * tail_steps / grid, base + (c + 1) * tail_steps / grid),
  // base = num_whole * grid * num_kv_tiles, of the sequence of (unit, key
  // tile) steps, unit-major (ItemCursor).  Its workspace: ws_o / ws_ml hold
  // one partial block per CTA, ws_cnt one counter per (CTA, Q tile).  O is
  // stored from registers straight to o_ptr.  (The parameter block keeps
  // its size: the classic kernels' register allocation is sensitive to it.)
  int grid;
  long long tail_steps;
  void* o_ptr;
  long long o_head_elems;      // elements from one (batch, head) block of O to the next
};

constexpr int kMaxSplit = 4;

// What one CTA computes: BM query rows of one (batch, head) against key tiles
// [kv_lo, kv_lo + n); part < 0 for a whole unit, else its slot in the workspace.
// For CTA pairs a unit is the 2 * BM rows of one pair; `rank` is the CTA's
// place in its pair (its rows start BM * rank into the unit), 0 otherwise.
struct WorkTile {
  int bh, q_row0, kv_lo, n, part, rank;
  long long slot;  // (split unit index) * split + part, for partial units
};

// ---------------------------------------------------------------------------
// Persistent schedule: items of a CTA
// ---------------------------------------------------------------------------
// The steps of a launch are (unit u, key tile k), numbered u * num_kv_tiles
// + k.  CTA c of G first runs the whole units c, c + G, ..., c + (R - 1) G
// (R = rr_rounds; the units running at any one time are neighbours, so the
// K/V of their heads stay in L2), then its share of the tail -- the steps of
// the remaining units, T_t of them from step tail_base -- namely
// [tail_base + floor(c T_t / G), tail_base + floor((c + 1) T_t / G)).  The
// host makes the tail at least G units long, so each share spans a unit or
// more and a unit is cut at most once.  A share cut at unit boundaries gives
// the CTA's tail items; a unit cut between two CTAs is finished by the piece
// holding its first key tile (kMerger), the last item of its CTA c0; the
// other piece (kWriter) is the first tail item of CTA c0 + 1, which writes
// its partial result into that CTA's workspace slot and counts in on c0's
// counter.  (The code allows any number of pieces: writers are the first
// tail items of CTAs c0 + 1 .. c1.)
enum : int { kWhole = 0, kMerger = 1, kWriter = 2 };

struct Item {
  int bh, q_row0, kv_lo, n, role;
  int peer;  // kMerger: last CTA holding a piece of the unit; kWriter: the merging CTA
};

// The CTA whose tail share holds tail step x (counted from tail_base): the
// largest c with floor(c T / G) <= x.
__host__ __device__ __forceinline__ int step_owner(long long x, long long T, int G) {
  return static_cast<int>(((x + 1) * G - 1) / T);
}

__device__ __forceinline__ long long tail_base_of(const AttnParams& p) {
  return static_cast<long long>(p.num_whole) * p.grid * p.num_kv_tiles;
}

struct ItemCursor {
  int cta, rr, rr_end;
  long long cur, end;
  __device__ __forceinline__ void init(int c, const AttnParams& p) {
    cta = c;
    rr = 0;
    rr_end = p.num_whole;
    const long long base = tail_base_of(p);
    cur = base + static_cast<long long>(c) * p.tail_steps / p.grid;
    end = base + static_cast<long long>(c + 1) * p.tail_steps / p.grid;
  }
  __device__ __forceinline__ bool next(Item& it, const AttnParams& p, int BM) {
    if (rr < rr_end) {
      const long long u = static_cast<long long>(rr) * p.grid + cta;
      it.bh = static_cast<int>(u / p.qt_per_bh);
      it.q_row0 = static_cast<int>(u % p.qt_per_bh) * BM;
      it.kv_lo = 0;
      it.n = p.num_kv_tiles;
      it.role = kWhole;
      it.peer = -1;
      ++rr;
      return true;
    }
    if (cur >= end) return false;
    const long long nkv = p.num_kv_tiles;
    const long long u = cur / nkv;
    const long long lo = cur - u * nkv;
    const long long hi = lo + (end - cur) < nkv ? lo + (end - cur) : nkv;
    it.bh = static_cast<int>(u / p.qt_per_bh);
    it.q_row0 = static_cast<int>(u % p.qt_per_bh) * BM;
    it.kv_lo = static_cast<int>(lo);
    it.n = static_cast<int>(hi - lo);
    if (lo == 0 && hi == nkv) {
      it.role = kWhole;
      it.peer = -1;
    } else if (lo == 0) {
      it.role = kMerger;
      it.peer = step_owner((u + 1) * nkv - 1 - tail_base_of(p), p.tail_steps, p.grid);
    } else {
      it.role = kWriter;
      it.peer = step_owner(u * nkv - tail_base_of(p), p.tail_steps, p.grid);
    }
    cur += it.n;
    return true;
  }
};

__device__ __forceinline__ WorkTile work_tile_of(int cta, int BM, int ctas, int rank,
                                                 const AttnParams& p) {
  WorkTile t;
  int u;
  cta /= ctas;
  if (cta < p.num_whole) {
    u = cta;
    t.part = -1;
    t.kv_lo = 0;
    t.n = p.num_kv_tiles;
    t.slot = 0;
  } else {
    const int r = cta - p.num_whole;
    u = p.num_whole + r / p.split;
    t.part = r % p.split;
    t.kv_lo = static_cast<int>(static_cast<long long>(t.part) * p.num_kv_tiles / p.split);
    t.n = static_cast<int>(static_cast<long long>(t.part + 1) * p.num_kv_tiles / p.split) - t.kv_lo;
    t.slot = static_cast<long long>(r);
  }
  t.bh = u / p.qt_per_bh;
  t.q_row0 = (u % p.qt_per_bh) * BM * ctas + rank * BM;
  t.rank = rank;
  return t;
}

template <typename T>
__device__ __forceinline__ uint32_t pack2(float lo, float hi);
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Partial O of a split unit in the workspace: f32 (a 16-bit partial adds a
// second rounding of the output's own size; one f16 ulp is 3.9e-3 for |O| in
// [4, 8), above the 2e-3 parity bound), as float4 columns (float4 number
// (col / 4) * BM + row of the unit's block), so the 32 lanes of a warp (32
// consecutive rows) touch 512 contiguous bytes per access.  Stores are plain
// (they stay in L2 for the merging CTA); the merge loads them with
// ld.global.cg (L2, past L1), since other CTAs wrote them.

// Of every 8 (column-pair) exponentials in a softmax chunk, kPolyPairsOf8
// run as the FMA-pipe polynomial (ptx::exp2_poly_pair) and the rest on the
// MUFU unit, so the two pipes share the B*H*S^2 exponentials.  -1 (default):
// per variant (AttnConfig::POLY8); 0..8 forces that share for every variant.
#ifndef ATTNPROF_POLY_PAIRS_OF_8
#define ATTNPROF_POLY_PAIRS_OF_8 -1
#endif
constexpr int kPolyPairsOf8 = ATTNPROF_POLY_PAIRS_OF_8;

// Where the first published part of P ends, in quarters of the key tile: P V
// starts on those keys while the softmax computes the rest, and only the
// rest's P V (with the next S) follows the last part.  -1 (default): 3 at
// BN = 128 (C2: 1068 -> 1082 TFLOP/s against 2), 2 elsewhere.
#ifndef ATTNPROF_PSPLIT_QUARTERS
#define ATTNPROF_PSPLIT_QUARTERS -1
#endif
constexpr int kPsplitQuarters = ATTNPROF_PSPLIT_QUARTERS;

// 1 (default): with one S buffer per Q tile, no per-step O_DONE commit (see
// AttnConfig::ODONE_PER_STEP); 0 commits it every step as two-buffer tiles do.
#ifndef ATTNPROF_LEAN_COMMITS
#define ATTNPROF_LEAN_COMMITS 1
#endif
constexpr bool kLeanCommits = ATTNPROF_LEAN_COMMITS != 0;
// 1 (default): the double-buffered D = 64 tiles run eight softmax warps per Q
// tile, 16 rows each (AttnConfig::W8); 0: four, 32 rows each.
#ifndef ATTNPROF_W8
#define ATTNPROF_W8 1
#endif
constexpr bool kW8 = ATTNPROF_W8 != 0;
// 1: also the D = 128 two-buffer tiles (256 x 64, 256 x 32); 0 (default).
#ifndef ATTNPROF_W8_D128
#define ATTNPROF_W8_D128 0
#endif
constexpr bool kW8D128 = ATTNPROF_W8_D128 != 0;
// 1: also the D = 64 tile with one S buffer per Q tile (256 x 128); 0 (default).
#ifndef ATTNPROF_W8_ONE
#define ATTNPROF_W8_ONE 0
#endif
constexpr bool kW8One = ATTNPROF_W8_ONE != 0;
// 1 (default): one FULL wait per step for V_j and K_{j+1} (AttnConfig::KV_JOINT_FULL).
#ifndef ATTNPROF_JOINT_FULL
#define ATTNPROF_JOINT_FULL 1
#endif
constexpr bool kJointFull = ATTNPROF_JOINT_FULL != 0;


// PAIR: the CTA is one of a cluster pair that shares every K/V tile through
// cta_group::2 MMAs of M = 256 (tile i of the even CTA on rows 0-127, tile i
// of the odd CTA on rows 128-255).  Each CTA loads half of every K tile (BN/2
// keys) and half of every V tile (D/2 columns), so the per-SM shared-memory
// traffic of the B operands, the TMA writes and the L2 reads halve and the
// same ring holds twice as many key tiles.  The even CTA issues all MMAs.
template <typename T, int D_, int BN_, int NQ_, int STAGES_, bool PAIR_ = false, bool CORR_ = false,
          bool FOUR_ = false>
struct AttnConfig {
  static constexpr int D = D_;
  static constexpr int BN = BN_;
  static constexpr int NQ = NQ_;
  static constexpr int STAGES = STAGES_;
  static constexpr bool PAIR = PAIR_;
  // CORR: a correction warpgroup owns the lazy rescale of both tiles' O in
  // tensor memory, the final 1 / rowsum normalisation and the TMA store of O;
  // the softmax warpgroups hand it each step's rescale factors and, after
  // their last step, the row sums.  Built for two-tile CTAs without pairs.
  static constexpr bool CORR = CORR_;
  static constexpr int CTAS = PAIR ? 2 : 1;  // CTAs that share one MMA
  static constexpr bool kBF16 = sizeof(T) == 2 && !std::is_same<T, __half>::value;

  static_assert(D == 64 || D == 128, "head dim must be 64 or 128");
  static_assert(BN % 32 == 0 && BN >= 32 && BN <= 256, "BN must be a multiple of 32 in [32, 256]");
  static_assert(NQ == 1 || NQ == 2, "NQ must be 1 or 2");
  static_assert(STAGES >= 2, "need at least two K/V slots");
  static_assert(!PAIR || (D == 128 && BN == 128 && NQ == 2),
                "CTA pairs are built for D = 128, BN = 128, two Q tiles per CTA");
  static_assert(!CORR || (NQ == 2 && !PAIR), "the correction warpgroup serves two-tile CTAs");

  static constexpr int QROWS = 128;  // rows per Q tile = MMA M = TMEM lanes
  static constexpr int BM = QROWS * NQ;
  static constexpr int DBLK = D / 64;  // 64-element (128 B) column blocks per row

  // TMEM columns (32-bit each).  S_i (and P_i over it) then O_i.
  static constexpr int NSBUF = (NQ * (2 * BN + D) <= 512) ? 2 : 1;
  static constexpr int TMEM_S_COLS = NQ * NSBUF * BN;
  static constexpr int TMEM_O_COL = TMEM_S_COLS;
  static constexpr int TMEM_USED = TMEM_S_COLS + NQ * D;
  static_assert(TMEM_USED <= 512, "tile does not fit in tensor memory");
  static constexpr int TMEM_ALLOC = TMEM_USED <= 32    ? 32
                                    : TMEM_USED <= 64  ? 64
                                    : TMEM_USED <= 128 ? 128
                                    : TMEM_USED <= 256 ? 256
                                                       : 512;

  // Shared memory (offsets from a 1024-byte aligned base).
  static constexpr int Q_TILE_BYTES = QROWS * D * 2;
  static constexpr int Q_BLK_BYTES = QROWS * 128;
  // One ring slot: a K or a V tile (this CTA's half of it for pairs).  K
  // slots hold BN / CTAS keys as DBLK 64-column blocks of K_BLK_BYTES; V slots
  // hold all BN keys of D / CTAS columns, 64-column blocks V_BLK_BYTES apart.
  static constexpr int KV_TILE_BYTES = BN * D * 2 / CTAS;
  static constexpr int K_ROWS = BN / CTAS;
  static constexpr int K_BLK_BYTES = K_ROWS * 128;
  static constexpr int V_BLK_BYTES = BN * 128;
  static constexpr int V_DBLK = DBLK / CTAS;
  static constexpr int KV_BLK_BYTES = BN * 128;
  // Variants that can run the persistent schedule: two Q tiles with one S
  // buffer each (the next item's first S follows the last P V like any other
  // S) and no CTA pair.  (One-tile CTAs with one S buffer, BN = 256, would
  // spill registers in it.)
  // (W8_ONE: the D = 64 one-buffer tile that runs eight softmax warps.)
  static constexpr bool W8_ONE =
      kW8 && kW8One && !FOUR_ && NQ == 2 && NSBUF == 1 && !PAIR && !CORR && D == 64 && BN <= 128;
  static constexpr bool PERSIST_OK = NSBUF == 1 && !PAIR && NQ == 2 && !CORR && !W8_ONE;
  // Variants that also have the correction-warpgroup kernel (the tiles of
  // the benchmark configurations).
  static constexpr bool CORR_OK = NQ == 2 && !PAIR && (BN == 128 || (D == 64 && BN == 96));
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_KV = OFF_Q + NQ * Q_TILE_BYTES;
  // Those variants also hold one Q tile's worth of O staging (128B-swizzled,
  // the TMA store's layout), which the two Q tiles' epilogues take turns on
  // in the persistent schedule, where the Q slots already hold the next
  // item's Q.  (It costs the ring a slot: 4 instead of 5 at 256 x 128, D =
  // 128, which measured the same.)
  static constexpr int STAGE_BYTES = PERSIST_OK ? Q_TILE_BYTES : 0;
  static constexpr int OFF_STAGE = OFF_KV + STAGES * KV_TILE_BYTES;
  // CORR: per Q tile and S buffer, each row's rescale factor of the step in
  // that buffer ([NQ][NSBUF][QROWS] floats), then per Q tile each row's sum
  // ([NQ][QROWS], after the last step).
  static constexpr int CORR_ALPHA_FLOATS = NQ * NSBUF * QROWS;
  static constexpr int CORR_BYTES = CORR ? (CORR_ALPHA_FLOATS + NQ * QROWS) * 4 : 0;
  static constexpr int OFF_CORR = OFF_STAGE + STAGE_BYTES;
  static constexpr int OFF_BAR = OFF_CORR + CORR_BYTES;

  static constexpr int BAR_Q = 0;
  static constexpr int BAR_KV_FULL = BAR_Q + NQ;
  static constexpr int BAR_KV_EMPTY = BAR_KV_FULL + STAGES;
  static constexpr int BAR_S_FULL = BAR_KV_EMPTY + STAGES;  // [NQ][NSBUF]
  // P is published in PHALVES parts so P V can start on the first keys while
  // the softmax computes the rest: with >= 2 chunks of 32 columns, part 0 is
  // the first PSPLIT_CHUNKS chunks (P V K-steps [0, 2 * PSPLIT_CHUNKS)).
  // Variants that double-buffer S at D = 64 keep both softmax warpgroups on
  // the exponentials back to back, where the MUFU unit is the bound: there
  // part of the exponentials go to the FMA pipe (POLY8) and P is published in
  // one piece (C3 at 256 x 96: 631 -> 664 TFLOP/s).  At D = 128 neither helps.
  static constexpr bool EXP_BOUND = NQ == 2 && D == 64 && NQ * (2 * BN + D) <= 512;
  // W8: those tiles give each Q tile eight softmax warps of 16 rows (the
  // 16-lane tensor-memory forms), so that four softmax warps share each SM
  // sub-partition and its exponential unit instead of two: their softmax
  // step is bound by the exponentials and by each warp's own instruction
  // stream.  (At D = 128 the single issuer's chain makes a step's latency
  // matter, and eight warps per tile measured slower there.)  Whole units
  // only: such launches take no key split.
  // FOUR_: the four-warp kernel of such a tile, which the host runs when
  // its plan splits units along the keys.
  static constexpr bool W8 =
      (kW8 && !FOUR_ && NQ == 2 && NSBUF == 2 && !PAIR && !CORR && (D == 64 || kW8D128)) ||
      W8_ONE;
  static constexpr int PHALVES = (BN >= 64 && !EXP_BOUND && !(W8 && NSBUF == 2)) ? 2 : 1;

  static constexpr int PSPLIT_QUARTERS = kPsplitQuarters >= 0 ? kPsplitQuarters
                                                              : (BN == 128 ? 3 : 2);
  static constexpr int PSPLIT_CHUNKS =
      (BN / 32) * PSPLIT_QUARTERS / 4 >= 1 ? (BN / 32) * PSPLIT_QUARTERS / 4 : 1;
  static constexpr int BAR_P_READY = BAR_S_FULL + NQ * NSBUF;      // [NQ][NSBUF][PHALVES]
  static constexpr int BAR_O_DONE = BAR_P_READY + NQ * NSBUF * PHALVES;  // every P V of tile i
  // Is O_DONE committed after every step?  With one S buffer per tile,
  // S_i(j+1) is issued behind P_i(j) V_j by the same thread, and a commit
  // covers every earlier MMA of its thread: the S_FULL that the softmax
  // waits for before step j+1 already says that P_i(j) V_j is complete, so a
  // rescale of O needs no O_DONE, and the commit (~50-120 cycles of the
  // issuing thread, which is short of slack) is left out.  Two S buffers
  // issue S_i(j+1) one step earlier, so they keep it.  (The profiler's
  // observer then reads each P V's completion from that S_FULL.)
  static constexpr bool ODONE_PER_STEP = NSBUF == 2 || !kLeanCommits;
  // Ring releases.  With one S buffer the ring items are K_0, then V_j,
  // K_{j+1} for each step j, and V_j and K_{j+1} are both free once step j's
  // MMAs (P V_j of every tile, then S(j+1)) complete, so one commit, on
  // K_{j+1}'s EMPTY barrier, releases both, and V slots get none.  K_m is
  // item 2m, in slot 2m mod STAGES; the K items that share a slot recur every
  // K_SLOT_PERIOD of them, so K_m's commit completes phase m / K_SLOT_PERIOD
  // of that barrier.  The producer reloading slot t mod STAGES (item t >=
  // STAGES) waits for the commit of K_m with m = (t - STAGES + 1) / 2: the
  // previous occupant of the slot is K_m itself or V_{m-1}.
  static constexpr bool V_RELEASE_WITH_K = kLeanCommits && NSBUF == 1;
  // Joint landing (single CTAs): V_j and K_{j+1} complete on V_j's FULL
  // barrier (armed for both tiles' bytes), so the MMA issuer makes one wait
  // per step instead of two -- its waits cost it ~100 cycles each and it is
  // on the per-tile chain.  K_{j+1}'s own FULL barrier still gets one plain
  // arrival from the producer, so every slot's barrier advances one phase per
  // item and the phase parities stay (t / STAGES) & 1.
  //
  // Pairs too: the odd CTA's loads land on its own barriers, which the relay
  // forwards to the even CTA's; under the joint landing the relay forwards
  // K_{j+1}'s slot before V_j's (see relay_role).
  static constexpr bool KV_JOINT_FULL = kJointFull && V_RELEASE_WITH_K;
  static constexpr int K_SLOT_PERIOD = STAGES % 2 == 0 ? STAGES / 2 : STAGES;
  static constexpr int BAR_O_FINAL = BAR_O_DONE + NQ;            // the last P V of tile i
  static constexpr int BAR_DRAIN = BAR_O_FINAL + NQ;
  // Persistent schedule: the last S of an item has read Q tile i, so the
  // next item's Q tile i may be loaded over it (one phase per item).
  static constexpr int BAR_Q_FREE = BAR_DRAIN + 1;
  // CORR: tile i's softmax warps arrive on BAR_CORR + i * NSBUF + (j mod
  // NSBUF) at step j (the step's rescale factors are in shared memory), and
  // on BAR_CORR_END + i after the last step (the row sums are).  Each S
  // buffer has its own request barrier and factors: with two buffers the
  // softmax may post step j + 1 (its S was issued before P V of step j)
  // while the correction warps still serve step j, but not step j + 2 (its S
  // follows P V of step j, which waits for them).  The end gets a barrier of
  // its own: the last step's request and the end's follow each other with
  // nothing in between that waits for the correction warps.
  static constexpr int BAR_CORR = BAR_Q_FREE + NQ;
  static constexpr int BAR_CORR_END = BAR_CORR + NQ * NSBUF;
  static constexpr int NUM_BARS = BAR_CORR + (CORR ? NQ * NSBUF + NQ : 0);

  // Misc words: TMEM base (0), abort flag (4), the split merge's last-part
  // flags (8, 12), the O staging lock (16).
  static constexpr int OFF_MISC = OFF_BAR + ((NUM_BARS * 8 + 15) / 16) * 16;
  static constexpr int SMEM_USED = OFF_MISC + 32;
  static constexpr int SMEM_BYTES = SMEM_USED + 1024;  // slack for manual 1024 B alignment

  // Warp roles.
  static constexpr int WARPS_PER_TILE = W8 ? 8 : 4;
  static constexpr int NUM_SOFTMAX_WARPS = WARPS_PER_TILE * NQ;
  static constexpr int LOAD_WARP = NUM_SOFTMAX_WARPS;
  static constexpr int MMA_WARP = NUM_SOFTMAX_WARPS + 1;
  static constexpr int OBSERVER_WARP = NUM_SOFTMAX_WARPS + 2;  // profiler only
  // MMA issuers.  With one S buffer per Q tile (NSBUF = 1) a single thread
  // issues both tiles' MMAs in turn, which keeps the two softmax steps taking
  // turns (each tile's next S waits for its own P V anyway).  With S double
  // buffered (NQ = 2, BN <= 64 at D = 128) S_i(j+1) is ready before the
  // softmax of S_i(j) ends, and an in-order issuer would make tile 0 wait for
  // tile 1's P: one issuer per Q tile (MMA_WARP for tile 0, MMA_WARP2 for
  // tile 1) lets both softmax warpgroups run back to back (C2 at 256 x 64:
  // 742 -> 1030 TFLOP/s).  Each K/V slot is then released by NUM_ISSUERS
  // commits.
  static constexpr int NUM_ISSUERS = (NQ == 2 && NSBUF == 2) ? 2 : 1;
  static constexpr int MMA_WARP2 = NUM_SOFTMAX_WARPS + 3;
  // CORR: the correction warpgroup is the last four warps; warp w of it
  // serves TMEM lanes 32 (w % 4) .. 32 (w % 4) + 31, the rows of softmax warp
  // w % 4 of each tile.
  static constexpr int CORR_WARP0 = NUM_SOFTMAX_WARPS + 4;
  static constexpr int NUM_THREADS = 32 * (NUM_SOFTMAX_WARPS + 4 + (CORR ? 4 : 0));
  // One 128-row Q tile with narrow key tiles fits two CTAs per SM (shared
  // and tensor memory); the register budget is capped to keep that possible.
  static constexpr int MIN_CTAS_PER_SM = (NQ == 1 && BN <= 64) ? 2 : 1;
  // Register split for NQ = 2: 384 threads launched at 168 registers each
  // (64512): softmax warpgroups 2 x 128 x 192 + producer/MMA warpgroup
  // 128 x 120.  CORR: 512 threads launched at 128 (65536): softmax
  // 2 x 128 x 192 + producer/MMA 128 x 72 + correction 128 x 56 (the MMA
  // issuer spills below 72).
  static constexpr int LAUNCH_REGS = (65536 / NUM_THREADS) & ~7;
  // W8: 640 threads launched at 96 (61440): softmax 16 x 32 x 104 + the
  // producer/MMA warpgroup 128 x 64.
  static constexpr uint32_t REG_SOFTMAX = W8 ? 104 : 192;
  static constexpr uint32_t REG_OTHER = W8 ? 64 : (CORR ? 72 : 120);
  static constexpr uint32_t REG_CORR = 56;
  static_assert(NQ != 2 || NUM_SOFTMAX_WARPS * 32 * REG_SOFTMAX + 128 * REG_OTHER +
                                   (CORR ? 128 * REG_CORR : 0) <=
                               NUM_THREADS * LAUNCH_REGS,
                "register split exceeds the launch allocation");

  // Polynomial share: 2 of 8 pairs on the four-warp EXP_BOUND tiles, 1 of 8
  // with eight warps per tile (C3: 709-711 TFLOP/s against 693-695 at 2 and
  // 696 at 0), none elsewhere.
  static constexpr int POLY8 =
      kPolyPairsOf8 >= 0 ? kPolyPairsOf8 : (W8 ? (D == 64 ? 1 : 0) : (EXP_BOUND ? 2 : 0));
  static constexpr int MMA_M = 128 * CTAS;
  static constexpr uint32_t IDESC_S = ptx::idesc_f16(MMA_M, BN, kBF16, false);
  static constexpr uint32_t IDESC_PV = ptx::idesc_f16(MMA_M, D, kBF16, true);
  // Arrivals per P part: one per softmax warp of the tile, of both CTAs for
  // pairs.
  static constexpr int P_ARRIVALS = WARPS_PER_TILE * CTAS;
  // The first P part of a step also waits for the correction warps (O is
  // rescaled, when it had to be, before P V adds to it).
  static constexpr int P0_ARRIVALS = P_ARRIVALS + (CORR ? 4 : 0);
};

// Lazy-rescale threshold in log2 units: O and the row sum are rescaled only
// when the running max of a row grows by more than this; otherwise P is
// computed against the stale max, so P <= 2^8 which f16, bf16 and the f32
// accumulators all hold exactly enough.
constexpr float RESCALE_THRESHOLD = 8.0f;


// Which column pairs of a 32-column chunk take the polynomial: spread evenly
// (e.g. 4 of 8 -> every other pair) so both pipes stay busy.
template <int POLY8>
__host__ __device__ constexpr bool poly_pair(int e) {
  return POLY8 > 0 && ((e % 8) * POLY8) % 8 + POLY8 > 7;
}

// Row maximum of N register values with independent partial maxima (short
// dependency chains; max is exact, so the order does not change the result).
template <int N>
__device__ __forceinline__ float row_max(const uint32_t* r, float init) {
  static_assert(N % 8 == 0, "");
  float a[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) a[k] = __uint_as_float(r[k]);
  int c = 8;
#pragma unroll
  for (; c + 16 <= N; c += 16) {
#pragma unroll
    for (int k = 0; k < 8; ++k)
      a[k] = ptx::fmax3(a[k], __uint_as_float(r[c + k]), __uint_as_float(r[c + 8 + k]));
  }
  if (c < N) {
#pragma unroll
    for (int k = 0; k < 8; ++k) a[k] = fmaxf(a[k], __uint_as_float(r[c + k]));
  }
  const float b0 = ptx::fmax3(a[0], a[1], a[2]);
  const float b1 = ptx::fmax3(a[3], a[4], a[5]);
  const float b2 = ptx::fmax3(a[6], a[7], init);
  return ptx::fmax3(b0, b1, b2);
}

struct WaitCtx {
  volatile int* abort;  // CTA-local abort flag in shared memory
  int* status;
  unsigned long long timeout_ns;
};

static __device__ __forceinline__ bool wait_bar_slow(uint32_t bar, uint32_t parity, const WaitCtx& w,
                                           int site) {
  const unsigned long long t0 = ptx::globaltimer_ns();
  for (uint32_t it = 1;; ++it) {
    if (ptx::mbar_try_wait(bar, parity)) return true;
    if ((it & 31u) == 0) {
      if (*w.abort) return false;
      if (ptx::globaltimer_ns() - t0 > w.timeout_ns) {
        *w.abort = 1;
        if (w.status) atomicCAS(w.status, 0, kDeviceTimeoutBase + site);
        return false;
      }
    }
  }
}

// Bounded wait for the completion of the mbarrier phase with parity `parity`.
// Also for the barriers that the peer CTA of a pair arrives on: the waits
// keep the default (CTA-scope) acquire, like the arrivals; an acquire at
// cluster scope on every poll made the pair kernel 27 % slower on B200.
__device__ __forceinline__ bool wait_bar(uint32_t bar, uint32_t parity, const WaitCtx& w,
                                         int site) {
  if (ptx::mbar_try_wait(bar, parity)) return true;
  return wait_bar_slow(bar, parity, w, site);
}

template <bool PROFILE>
struct Prof {
  unsigned long long* buf;
  __device__ __forceinline__ void stamp(int phase, int slot, int which) const {
    if constexpr (PROFILE) {
      if (buf != nullptr && slot < kProfSlots)
        buf[(phase * kProfSlots + slot) * 2 + which] = clock64();
    }
  }
};

// ----------------------------------------------------------------------------
// Producer: Q once, then the K/V sequence
//   K_0 .. K_{NSBUF-1}, then for each j: V_j, K_{j+NSBUF}
// which is exactly the order in which the MMA warp consumes ring slots.
// ----------------------------------------------------------------------------
template <class C, bool PROFILE>
__device__ void load_role(const CUtensorMap* tmQ, const CUtensorMap* tmK, const CUtensorMap* tmV,
                          uint32_t sbase, const WorkTile& wt, const AttnParams& p,
                          const WaitCtx& w, const Prof<PROFILE>& prof) {
  auto bar = [&](int i) { return sbase + C::OFF_BAR + 8u * i; };
  const int n = wt.n;
  const int q_row0 = wt.q_row0, bh = wt.bh;
  const uint64_t pol_kv = ptx::l2_policy_evict_last();
  const uint64_t pol_q = ptx::l2_policy_evict_first();

  prof.stamp(kPhLoadQ, 0, 0);
#pragma unroll
  for (int i = 0; i < C::NQ; ++i) {
    ptx::mbar_arrive_expect_tx(bar(C::BAR_Q + i), C::Q_TILE_BYTES);
#pragma unroll
    for (int d = 0; d < C::DBLK; ++d)
      ptx::tma_load_3d_hint(sbase + C::OFF_Q + i * C::Q_TILE_BYTES + d * C::Q_BLK_BYTES, tmQ,
                            bar(C::BAR_Q + i), d * 64, q_row0 + i * C::QROWS, bh, pol_q);
  }
  if (p.fault_mode == 1) return;  // test hook: K/V never arrive; consumers time out

  int t = 0;          // ring item counter
  int last_issued[C::STAGES];
#pragma unroll
  for (int s = 0; s < C::STAGES; ++s) last_issued[s] = -1;
  bool ok = true;

  // joint: this V item's FULL barrier also takes the next K item's bytes
  // (KV_JOINT_FULL); k_bar: the barrier a K item's load completes on (-1: its own).
  auto produce = [&](bool is_k, int j, bool joint = false, int k_bar = -1) {
    const int s = t % C::STAGES;
    if (t >= C::STAGES) {
      uint32_t eb, par;
      if constexpr (C::V_RELEASE_WITH_K) {
        const int m = (t - C::STAGES + 1) / 2;  // the K item whose commit frees slot s
        eb = bar(C::BAR_KV_EMPTY + (2 * m) % C::STAGES);
        par = static_cast<uint32_t>(m / C::K_SLOT_PERIOD) & 1u;
      } else {
        eb = bar(C::BAR_KV_EMPTY + s);
        par = static_cast<uint32_t>(t / C::STAGES - 1) & 1u;
      }
      if (!wait_bar(eb, par, w, kSiteKvEmpty)) {
        ok = false;
        return;
      }
    }
    prof.stamp(is_k ? kPhLoadK : kPhLoadV, j, 0);
    uint32_t full = bar(C::BAR_KV_FULL + s);
    if (k_bar >= 0) {
      ptx::mbar_arrive(full);  // keeps this slot's phase count; the bytes go to k_bar
      full = bar(C::BAR_KV_FULL + k_bar);
    } else {
      ptx::mbar_arrive_expect_tx(full, joint ? 2 * C::KV_TILE_BYTES : C::KV_TILE_BYTES);
    }
    const uint32_t dst = sbase + C::OFF_KV + s * C::KV_TILE_BYTES;
    const int key0 = (wt.kv_lo + j) * C::BN;
    if (is_k) {
      // K: keys [key0 + rank * K_ROWS, + K_ROWS), all D columns.
#pragma unroll
      for (int d = 0; d < C::DBLK; ++d)
        ptx::tma_load_3d_hint(dst + d * C::K_BLK_BYTES, tmK, full, d * 64,
                              key0 + wt.rank * C::K_ROWS, bh, pol_kv);
    } else {
      // V: all BN keys, column blocks [rank * V_DBLK, + V_DBLK).
#pragma unroll
      for (int d = 0; d < C::V_DBLK; ++d)
        ptx::tma_load_3d_hint(dst + d * C::V_BLK_BYTES, tmV, full,
                              (wt.rank * C::V_DBLK + d) * 64, key0, bh, pol_kv);
    }
    last_issued[s] = t;
    ++t;
  };

  for (int jj = 0; jj < C::NSBUF && jj < n && ok; ++jj) produce(true, jj);
  for (int j = 0; j < n && ok; ++j) {
    const bool joint = C::KV_JOINT_FULL && j + C::NSBUF < n;
    const int sv = t % C::STAGES;
    produce(false, j, joint);
    if (ok && j + C::NSBUF < n) produce(true, j + C::NSBUF, false, joint ? sv : -1);
  }
  if (!ok) {
    // Do not leave this CTA with bulk copies in flight: wait (bounded) for the
    // most recent load issued into every slot to land.  Under the joint
    // landing a K item's bytes complete V_j's barrier (slot sv), not its own,
    // whose phase the plain arrival completed at once; that K load was issued
    // right after V_j into sv's phase, so the wait on slot sv below covers it
    // (slot sv cannot have been reloaded since: a reload first waits for the
    // commit that releases both V_j and K_{j+1}).
#pragma unroll
    for (int s = 0; s < C::STAGES; ++s) {
      if (last_issued[s] < 0) continue;
      const int r = last_issued[s] / C::STAGES;
      const unsigned long long t0 = ptx::globaltimer_ns();
      while (!ptx::mbar_try_wait(bar(C::BAR_KV_FULL + s), r & 1)) {
        if (ptx::globaltimer_ns() - t0 > w.timeout_ns) break;
      }
    }
  }
}

// ----------------------------------------------------------------------------
// MMA issuer (single thread)
// ----------------------------------------------------------------------------
template <class C, bool PROFILE>
__device__ void mma_role(uint32_t tmem, uint32_t sbase, const WorkTile& wt, const AttnParams& p,
                         const WaitCtx& w, const Prof<PROFILE>& prof, int i0, int i1) {
  // Issues the MMAs of Q tiles [i0, i1) of this CTA (for a CTA pair: of both
  // CTAs, from the even one).
  constexpr int G = C::CTAS;
  auto bar = [&](int i) { return sbase + C::OFF_BAR + 8u * i; };
  // Completion signals that the softmax / producer warps wait on: in both
  // CTAs of a pair.
  auto signal = [&](uint32_t b) {
    if constexpr (C::PAIR)
      ptx::mma_commit_pair(b);
    else
      ptx::mma_commit(b);
  };
  const int n = wt.n;
  bool ok = true;

  for (int i = i0; i < i1 && ok; ++i) ok = wait_bar(bar(C::BAR_Q + i), 0, w, kSiteQ);
  if (ok && i0 == 0) prof.stamp(kPhLoadQ, 0, 1);

  int t = 0;
  // Wait for ring item t (K_j when is_k, else V_j) to land in its slot.
  auto ring_wait = [&](int& stage, bool is_k, int j) -> bool {
    stage = t % C::STAGES;
    const bool r =
        wait_bar(bar(C::BAR_KV_FULL + stage), (t / C::STAGES) & 1, w, kSiteKvFull);
    ++t;
    if (r) {
      if (i0 == 0) prof.stamp(is_k ? kPhLoadK : kPhLoadV, j, 1);
      ptx::tc_fence_after();
    }
    return r;
  };

  // Descriptors are built once; per MMA only byte offsets >> 4 are added to
  // the start-address field (bits 0-13; no carry out of it because every
  // operand lies below 256 KB of shared memory).  Per-k-step offsets are
  // compile-time constants, the slot offset is added once per GEMM.
  constexpr int KSTEPS_S = C::D / 16;
  uint64_t qd0[C::NQ];
#pragma unroll
  for (int i = 0; i < C::NQ; ++i)
    qd0[i] = ptx::smem_desc_sw128(sbase + C::OFF_Q + i * C::Q_TILE_BYTES, 16, 1024);
  const uint64_t kd0 = ptx::smem_desc_sw128(sbase + C::OFF_KV, 16, 1024);
  const uint64_t vd0 = ptx::smem_desc_sw128(sbase + C::OFF_KV, C::V_BLK_BYTES, 1024);
  auto slot_off = [](int stage) -> uint32_t {
    return static_cast<uint32_t>((stage * C::KV_TILE_BYTES) >> 4);
  };

  // S_i(j) = Q_i K_j^T : D/16 MMAs of 128 x BN x 16.  K-step kk reads 16
  // elements (32 B) of every 128 B row of 64-column block kk / 4.
  auto issue_s = [&](int i, int j, int stage) {
    const uint32_t d_tmem = tmem + (i * C::NSBUF + j % C::NSBUF) * C::BN;
    const uint64_t kd = ptx::desc_add(kd0, slot_off(stage));
#pragma unroll
    for (int kk = 0; kk < KSTEPS_S; ++kk) {
      const uint32_t qo = static_cast<uint32_t>(((kk >> 2) * C::Q_BLK_BYTES + (kk & 3) * 32) >> 4);
      const uint32_t ko = static_cast<uint32_t>(((kk >> 2) * C::K_BLK_BYTES + (kk & 3) * 32) >> 4);
      ptx::mma_ss<G>(d_tmem, ptx::desc_add(qd0[i], qo), ptx::desc_add(kd, ko), C::IDESC_S,
                     kk > 0 ? 1u : 0u);
    }
  };
  // O_i += P_i(j) V_j : BN/16 MMAs of 128 x D x 16, A = P from TMEM; K-step
  // kk reads 16 rows (keys) = two 1024 B atoms of V.
  auto issue_pv = [&](int i, int j, int stage, int k0, int k1) {
    const uint32_t p_tmem = tmem + (i * C::NSBUF + j % C::NSBUF) * C::BN;
    const uint32_t o_tmem = tmem + C::TMEM_O_COL + i * C::D;
    const uint64_t vd = ptx::desc_add(vd0, slot_off(stage));
#pragma unroll
    for (int kk = k0; kk < k1; ++kk)
      ptx::mma_ts<G>(o_tmem, p_tmem + kk * 8, ptx::desc_add(vd, static_cast<uint32_t>(kk * 2048 >> 4)),
                     C::IDESC_PV, (j > 0 || kk > 0) ? 1u : 0u);
  };

  // Prologue: S for the first NSBUF KV tiles.
  for (int jj = 0; jj < C::NSBUF && jj < n && ok; ++jj) {
    int sk;
    if (!(ok = ring_wait(sk, true, jj))) break;
    for (int i = i0; i < i1; ++i) {
      if (i == 0) prof.stamp(kPhQK, jj, 0);
      issue_s(i, jj, sk);
      signal(bar(C::BAR_S_FULL + i * C::NSBUF + jj % C::NSBUF));
    }
    signal(bar(C::BAR_KV_EMPTY + sk));
  }

  for (int j = 0; j < n && ok; ++j) {
    int sv;
    if (i0 == 0) prof.stamp(kPhVWait, j, 0);
    if (!(ok = ring_wait(sv, false, j))) break;
    if (i0 == 0) prof.stamp(kPhVWait, j, 1);
    // K_{j+1} landed with V_j: its load ends here for the profiler.
    if (C::KV_JOINT_FULL && i0 == 0 && j + 1 < n) prof.stamp(kPhLoadK, j + 1, 1);
    const int jn = j + C::NSBUF;
    int sk = -1;
    for (int i = i0; i < i1 && ok; ++i) {
      const int pb = C::BAR_P_READY + (i * C::NSBUF + j % C::NSBUF) * C::PHALVES;
      constexpr int KSTEPS = C::BN / 16;
#pragma unroll
      for (int h = 0; h < C::PHALVES; ++h) {
        // K_{j+NSBUF} is normally resident long before the last P part: its
        // wait sits here, off the path from that P part to the next S.
        if (h == C::PHALVES - 1 && jn < n && sk < 0) {
          if constexpr (C::KV_JOINT_FULL) {
            sk = t % C::STAGES;  // landed with V_j (waited for above)
            ++t;
          } else {
            if (i0 == 0) prof.stamp(kPhKWait, j, 0);
            if (!(ok = ring_wait(sk, true, jn))) break;
            if (i0 == 0) prof.stamp(kPhKWait, j, 1);
          }
        }
        if (!(ok = wait_bar(bar(pb + h), (j / C::NSBUF) & 1, w, kSitePReady))) break;
        ptx::tc_fence_after();
        if (h == 0) {
          if (i == 0) prof.stamp(kPhPV, j, 0);
          prof.stamp(kPhMmaT0 + i, j, 0);
        }
        constexpr int KSPLIT = C::PHALVES == 2 ? 2 * C::PSPLIT_CHUNKS : KSTEPS;
        issue_pv(i, j, sv, h == 0 ? 0 : KSPLIT, h == 0 ? KSPLIT : KSTEPS);
      }
      if (!ok) break;
      // The tile's next S follows its last P V MMAs directly; the O commits
      // come after it (O_DONE then also covers that S, which every waiter on
      // O_DONE has already seen complete).  S_FULL covers this step's P V.
      if (jn < n) {
        if (i == 0) prof.stamp(kPhQK, jn, 0);
        issue_s(i, jn, sk);
        signal(bar(C::BAR_S_FULL + i * C::NSBUF + jn % C::NSBUF));
      }
      if (C::ODONE_PER_STEP) signal(bar(C::BAR_O_DONE + i));
      if (j == n - 1) signal(bar(C::BAR_O_FINAL + i));
      prof.stamp(kPhMmaT0 + i, j, 1);
    }
    if (!ok) break;
    if constexpr (!C::V_RELEASE_WITH_K) signal(bar(C::BAR_KV_EMPTY + sv));
    if (sk >= 0) signal(bar(C::BAR_KV_EMPTY + sk));  // with V_RELEASE_WITH_K: V_j's slot too
  }

  // Drain: every MMA this thread issued has completed before TMEM is freed.
  ptx::mma_commit<G>(bar(C::BAR_DRAIN));
  const unsigned long long t0 = ptx::globaltimer_ns();
  while (!ptx::mbar_try_wait(bar(C::BAR_DRAIN), 0)) {
    if (ptx::globaltimer_ns() - t0 > w.timeout_ns) {
      if (w.status) atomicCAS(w.status, 0, kDeviceTimeoutBase + kSiteDrain);
      break;
    }
  }
}

// ----------------------------------------------------------------------------
// Relay (odd CTA of a pair, one thread): the even CTA's MMAs read this CTA's
// Q and K/V halves, so each landing of a load here (observed on this CTA's own
// barrier, which the TMA completes) is passed on as an arrival on the even
// CTA's barrier of the same slot; there the MMA issuer waits for both halves
// (two arrivals).  Items in the producer's order: Q tiles, K_0, then V_j,
// K_{j+1}.  A failed wait ends the relay; the even CTA then times out too.
// ----------------------------------------------------------------------------
template <class C>
__device__ void relay_role(uint32_t sbase, const WorkTile& wt, const WaitCtx& w) {
  auto bar = [&](int i) { return sbase + C::OFF_BAR + 8u * i; };
  // Waits with a suspend hint: the relay thread sleeps inside try_wait until
  // the load lands instead of taking issue slots from the softmax warps of its
  // SM sub-partition.
  auto wait = [&](uint32_t b, uint32_t parity, int site) {
    const unsigned long long t0 = ptx::globaltimer_ns();
    while (!ptx::mbar_try_wait_sleep(b, parity, 20000u)) {
      if (*w.abort) return false;
      if (ptx::globaltimer_ns() - t0 > w.timeout_ns) {
        *w.abort = 1;
        if (w.status) atomicCAS(w.status, 0, kDeviceTimeoutBase + site);
        return false;
      }
    }
    return true;
  };
  for (int i = 0; i < C::NQ; ++i) {
    if (!wait(bar(C::BAR_Q + i), 0, kSiteQ)) return;
    ptx::mbar_arrive_cluster(ptx::mapa_shared(bar(C::BAR_Q + i), 0));
  }
  auto wait_item = [&](int t) {
    return wait(bar(C::BAR_KV_FULL + t % C::STAGES), (t / C::STAGES) & 1, kSiteKvFull);
  };
  auto forward = [&](int t) {
    ptx::mbar_arrive_cluster(ptx::mapa_shared(bar(C::BAR_KV_FULL + t % C::STAGES), 0));
  };
  if constexpr (C::KV_JOINT_FULL) {
    // Items K_0, then V_j (t = 2j + 1) and K_{j+1} (t = 2j + 2).  V_j's
    // barrier here completes only after K_{j+1}'s loads land (they were
    // issued after K's plain arrival), so once it has, K's phase is complete
    // too, and neither can move on before the even CTA's issuer sees V_j
    // forwarded.  K's slot is forwarded first: the even CTA's K barrier then
    // completes this phase before its producer, which waits for the commit
    // that follows V_j, can arrive for the slot's next item.
    static_assert(C::NSBUF == 1, "the joint landing interleaves one K per V");
    if (!wait_item(0)) return;
    forward(0);
    for (int j = 0; j < wt.n; ++j) {
      const int tv = 2 * j + 1;
      if (!wait_item(tv)) return;
      if (j + 1 < wt.n) {
        if (!wait_item(tv + 1)) return;
        forward(tv + 1);
      }
      forward(tv);
    }
  } else {
    const int items = 2 * wt.n;
    for (int t = 0; t < items; ++t) {
      if (!wait_item(t)) return;
      forward(t);
    }
  }
}

// ----------------------------------------------------------------------------
// Softmax warpgroup for Q tile qi (128 threads; thread row = TMEM lane)
// ----------------------------------------------------------------------------
// The KV steps of one item of Q tile qi: key tiles kv_lo .. kv_lo + n - 1,
// which are steps J0 .. J0 + n - 1 of this CTA's sequence (the phases of the
// S and P barriers follow the CTA's step count).  Leaves the row's running
// max (raw score units) and running sum in m_run / l_run; false if a wait
// failed (the warp then stops early).
template <typename T, class C, bool PROFILE>
__device__ __forceinline__ bool softmax_steps(int qi, uint32_t tmem, uint32_t sbase,
                                              const AttnParams& p, const WaitCtx& w,
                                              const Prof<PROFILE>& prof, int kv_lo, int n,
                                              int J0, int rank, float& m_run,
                                              float& l_run) {
  auto bar = [&](int i) { return sbase + C::OFF_BAR + 8u * i; };
  const int wi = (threadIdx.x / 32) & 3;  // warp within the warpgroup = TMEM lane quarter
  const int lane = threadIdx.x & 31;
  const uint32_t lane_base = tmem + (static_cast<uint32_t>(wi * 32) << 16);
  const uint32_t o_col = C::TMEM_O_COL + qi * C::D;
  const float sl2 = p.scale_log2;
  const bool rec = PROFILE && qi == 0 && wi == 0 && lane == 0;
  const bool rec1 = PROFILE && qi == 1 && wi == 0 && lane == 0;
  // P parts are signalled to the MMA issuer, in the even CTA of a pair.
  auto p_arrive = [&](uint32_t b) {
    if constexpr (C::PAIR) {
      if (rank != 0) {
        ptx::mbar_arrive_cluster(ptx::mapa_shared(b, 0));
        return;
      }
    }
    ptx::mbar_arrive(b);
  };

  m_run = -INFINITY;  // running max (raw score units)
  l_run = 0.f;        // running row sum of P (relative to m_run)
  bool ok = true;

  for (int j = 0; j < n; ++j) {
    const int g = J0 + j;  // this CTA's step: barrier phases
    const int sl = g < kProfSlots ? g : kProfSlots;  // profiler slot
    const int buf = g % C::NSBUF;
    const uint32_t s_col = (qi * C::NSBUF + buf) * C::BN;
    ok = __all_sync(0xffffffffu,
                    wait_bar(bar(C::BAR_S_FULL + qi * C::NSBUF + buf), static_cast<uint32_t>((g / C::NSBUF) & 1), w,
                             kSiteSFull));
    if (!ok) break;
    ptx::tc_fence_after();
    if (rec) {
      prof.stamp(kPhQK, sl, 1);
      prof.stamp(kPhSoftmax, sl, 0);
      prof.stamp(kPhSmLoadS, sl, 0);
    }
    if (rec1) prof.stamp(kPhSoftmaxT1, sl, 0);

    const int lim = p.S - (kv_lo + j) * C::BN;  // valid key columns in this tile
    const int pbar = C::BAR_P_READY + (qi * C::NSBUF + buf) * C::PHALVES;
    float mx = -INFINITY;
    constexpr int KEEP = C::BN <= 128;
    constexpr int NCH = C::BN / 32;
    uint32_t sreg[KEEP ? C::BN : 32];

    if constexpr (KEEP) {
#pragma unroll
      for (int c = 0; c < NCH; ++c) {
        uint32_t(&r)[32] = *reinterpret_cast<uint32_t(*)[32]>(&sreg[c * 32]);
        ptx::tmem_ld32(lane_base + s_col + c * 32, r);
      }
      ptx::tmem_wait_ld();
      ptx::reg_fence(sreg);
      if (rec) {
        prof.stamp(kPhSmLoadS, sl, 1);
        prof.stamp(kPhSmMax, sl, 0);
      }
      if (lim < C::BN) {
#pragma unroll
        for (int c = 0; c < C::BN; ++c)
          if (c >= lim) sreg[c] = __float_as_uint(-INFINITY);
      }
      mx = row_max<C::BN>(sreg, mx);
    } else {
#pragma unroll 1
      for (int c = 0; c < NCH; ++c) {
        ptx::tmem_ld32(lane_base + s_col + c * 32, sreg);
        ptx::tmem_wait_ld();
        ptx::reg_fence(sreg);
        if (lim < C::BN) {
#pragma unroll
          for (int e = 0; e < 32; ++e)
            if (c * 32 + e >= lim) sreg[e] = __float_as_uint(-INFINITY);
        }
        mx = row_max<32>(sreg, mx);
      }
    }

    // Lazy rescale decision.
    float alpha = 1.f;
    bool resc = false;
    if (j == 0) {
      m_run = mx;
    } else if ((mx - m_run) * sl2 > RESCALE_THRESHOLD) {
      alpha = ptx::ex2_approx((m_run - mx) * sl2);
      m_run = mx;
      resc = true;
    }
    if constexpr (C::CORR) {
      // Hand this step's factor to the correction warpgroup, which rescales
      // O where a row of this warp needs it before it lets P V add to O.
      ptx::st_shared_f32(
          sbase + C::OFF_CORR + 4u * ((qi * C::NSBUF + buf) * C::QROWS + wi * 32 + lane), alpha);
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(bar(C::BAR_CORR + qi * C::NSBUF + buf));
    } else if (__any_sync(0xffffffffu, resc)) {
      // O holds the sum through PV(j-1); wait for that MMA, then scale in
      // place.  With one S buffer the S_FULL observed above already covers it.
      if constexpr (C::ODONE_PER_STEP) {
        ok = __all_sync(0xffffffffu,
                        wait_bar(bar(C::BAR_O_DONE + qi), static_cast<uint32_t>((g - 1) & 1), w, kSiteODone));
        if (!ok) break;
        ptx::tc_fence_after();
      }
#pragma unroll 1
      for (int c = 0; c < C::D / 32; ++c) {
        uint32_t o[32];
        ptx::tmem_ld32(lane_base + o_col + c * 32, o);
        ptx::tmem_wait_ld();
        ptx::reg_fence(o);
#pragma unroll
        for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
        ptx::tmem_st32(lane_base + o_col + c * 32, o);
      }
    }

    if (rec) {
      prof.stamp(kPhSmMax, sl, 1);
      prof.stamp(kPhSmExp, sl, 0);
    }
    // P = exp2(s * scale_log2 - m * scale_log2), packed to T pairs over S.
    const float neg = -m_run * sl2;
    const uint64_t sl2x2 = ptx::f2_pack(sl2, sl2);
    const uint64_t negx2 = ptx::f2_pack(neg, neg);
    const float poly_a = sl2 * (1.0f / 134.0f), poly_b = (neg + 126.0f) * (1.0f / 134.0f);
    uint64_t part[2] = {0ull, 0ull};  // packed partial row sums (4 short FADD chains)
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      if constexpr (!KEEP) {
        ptx::tmem_ld32(lane_base + s_col + c * 32, sreg);
        ptx::tmem_wait_ld();
        ptx::reg_fence(sreg);
        if (lim < C::BN) {
#pragma unroll
          for (int e = 0; e < 32; ++e)
            if (c * 32 + e >= lim) sreg[e] = __float_as_uint(-INFINITY);
        }
      }
      uint32_t pk[16];
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        const int c0 = (KEEP ? c * 32 : 0) + 2 * e;
        float p0, p1;
        if (poly_pair<C::POLY8>(e)) {
          ptx::exp2_poly_pair(__uint_as_float(sreg[c0]), __uint_as_float(sreg[c0 + 1]), poly_a,
                              poly_b, p0, p1);
        } else {
          // x = s * scale_log2 - m * scale_log2 for two columns in one f32x2 FMA
          const uint64_t x2 = ptx::f2_fma(
              ptx::f2_pack(__uint_as_float(sreg[c0]), __uint_as_float(sreg[c0 + 1])), sl2x2, negx2);
          float x0, x1;
          ptx::f2_unpack(x2, x0, x1);
          p0 = ptx::ex2_approx(x0);
          p1 = ptx::ex2_approx(x1);
        }
        part[e & 1] = ptx::f2_add(part[e & 1], ptx::f2_pack(p0, p1));
        pk[e] = pack2<T>(p0, p1);
      }
      ptx::tmem_st16(lane_base + s_col + c * 16, pk);
      if (C::PHALVES == 2 && c == C::PSPLIT_CHUNKS - 1) {
        // First half of P is in TMEM: let the MMA warp start P V on it.
        ptx::tmem_wait_st();
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) p_arrive(bar(pbar));
        if (rec) prof.stamp(kPhPFirst, sl, 0);
        if (rec1) prof.stamp(kPhPFirst, sl, 1);
      }
    }
    float sa, sb, sc_, sd;
    ptx::f2_unpack(part[0], sa, sb);
    ptx::f2_unpack(part[1], sc_, sd);
    const float sum = (sa + sb) + (sc_ + sd);
    if (rec) {
      prof.stamp(kPhSmExp, sl, 1);
      prof.stamp(kPhSmStoreP, sl, 0);
    }
    ptx::tmem_wait_st();
    if (rec) prof.stamp(kPhSmStoreP, sl, 1);
    ptx::tc_fence_before();
    __syncwarp();
    if (lane == 0) p_arrive(bar(pbar + C::PHALVES - 1));
    if (rec) prof.stamp(kPhSoftmax, sl, 1);
    if (rec1) prof.stamp(kPhSoftmaxT1, sl, 1);
    l_run = l_run * alpha + sum;
  }
  return ok;
}

// The classic schedule: one work tile per CTA, the softmax steps of it, then
// its epilogue (TMA store of O through the Q tile's shared memory, or the
// partial write / merge of a key split).
template <typename T, class C, bool PROFILE>
__device__ void softmax_role(int qi, uint32_t tmem, uint32_t sbase, uint8_t* sgen,
                             const CUtensorMap* tmO, const WorkTile& wt, const AttnParams& p,
                             const WaitCtx& w, const Prof<PROFILE>& prof) {
  const int q_row0 = wt.q_row0, bh = wt.bh;
  auto bar = [&](int i) { return sbase + C::OFF_BAR + 8u * i; };
  const int wi = (threadIdx.x / 32) & 3;  // warp within the warpgroup = TMEM lane quarter
  const int lane = threadIdx.x & 31;
  const int row = wi * 32 + lane;
  const uint32_t lane_base = tmem + (static_cast<uint32_t>(wi * 32) << 16);
  const uint32_t o_col = C::TMEM_O_COL + qi * C::D;
  const float sl2 = p.scale_log2;
  const bool rec = PROFILE && qi == 0 && wi == 0 && lane == 0;

  float m_run, l_run;
  bool ok = softmax_steps<T, C, PROFILE>(qi, tmem, sbase, p, w, prof, wt.kv_lo, wt.n, 0, wt.rank,
                                         m_run, l_run);
  if constexpr (C::CORR) {
    // The correction warpgroup normalises and stores O: hand it the row sums
    // (after a failed wait the abort flag releases it instead).
    if (ok) {
      ptx::st_shared_f32(sbase + C::OFF_CORR + 4u * (C::CORR_ALPHA_FLOATS + qi * C::QROWS + row),
                         l_run);
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(bar(C::BAR_CORR_END + qi));
    }
    return;
  }

  // Epilogue: wait for the last P V, normalise, stage in the Q slot, TMA store.
  // Every warp of the group reaches both named barriers, also after a failed
  // wait, so no warp can be left behind at a barrier; the abort flag (set by
  // any timed-out wait before it returns) decides uniformly whether to store.
  if (rec) prof.stamp(kPhEpilogue, kEpAll, 0);
  ptx::named_bar_sync(1 + qi, 128);
  bool go = ok && (*w.abort == 0);
  if (rec) prof.stamp(kPhEpilogue, kEpWaitO, 0);
  if (go) go = wait_bar(bar(C::BAR_O_FINAL + qi), 0, w, kSiteODone);
  go = __all_sync(0xffffffffu, go);
  if (rec) prof.stamp(kPhEpilogue, kEpWaitO, 1);
  const uint32_t stage_s = sbase + C::OFF_Q + qi * C::Q_TILE_BYTES;
  uint8_t* stage_g = sgen + C::OFF_Q + qi * C::Q_TILE_BYTES;
  // Writes 16 output values (columns 16b .. 16b+15) of this thread's row
  // into the 128B-swizzled staging tile (layout of the TMA box {64, QROWS}).
  auto stage16 = [&](int b, const float* v) {
    const int dblk = (b * 16) / 64;
    const int chunk0 = ((b * 16) % 64) / 8;  // first 16-byte chunk of these 16 columns
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      uint4 u;
      u.x = pack2<T>(v[8 * q + 0], v[8 * q + 1]);
      u.y = pack2<T>(v[8 * q + 2], v[8 * q + 3]);
      u.z = pack2<T>(v[8 * q + 4], v[8 * q + 5]);
      u.w = pack2<T>(v[8 * q + 6], v[8 * q + 7]);
      const int chunk = (chunk0 + q) ^ (row & 7);
      *reinterpret_cast<uint4*>(stage_g + dblk * C::Q_BLK_BYTES + row * 128 + chunk * 16) = u;
    }
  };
  auto stage32 = [&](int c, const float (&v)[32]) {
    stage16(2 * c, v);
    stage16(2 * c + 1, v + 16);
  };
  // This thread's row of O, normalised by its own row sum, 32 columns at a time.
  auto own32 = [&](int c, float inv, float (&v)[32]) {
    uint32_t o[32];
    ptx::tmem_ld32(lane_base + o_col + c * 32, o);
    ptx::tmem_wait_ld();
    ptx::reg_fence(o);
#pragma unroll
    for (int e = 0; e < 32; ++e) v[e] = __uint_as_float(o[e]) * inv;
  };

  if (wt.part >= 0) {
    // One key range of a split unit.  Every part writes its normalised O rows
    // and (row max, row sum) to the workspace, then counts itself in; the part
    // that arrives last merges all of them and stores O like a whole unit.
    // The merge adds the parts in a fixed order and recomputes its own rows
    // exactly as written, so the output does not depend on which part is last.
    const int rrow = qi * C::QROWS + row;  // row within the unit
    const long long slot0 = wt.slot - wt.part;
    // float4 column 0 of this row in the partial block of slot s
    auto col0 = [&](long long s) { return p.ws_o + s * (C::BM * C::D / 4) + rrow; };
    if (rec) prof.stamp(kPhEpilogue, kEpPartial, 0);
    if (go) {
      ptx::tc_fence_after();
      const float inv = 1.f / l_run;
      float4* dst = col0(wt.slot);
#pragma unroll 1
      for (int b = 0; b < C::D / 16; ++b) {
        uint32_t o[16];
        ptx::tmem_ld16(lane_base + o_col + b * 16, o);
        ptx::tmem_wait_ld();
        ptx::reg_fence(o);
#pragma unroll
        for (int t = 0; t < 4; ++t)
          dst[(b * 4 + t) * C::BM] =
              make_float4(__uint_as_float(o[4 * t + 0]) * inv, __uint_as_float(o[4 * t + 1]) * inv,
                          __uint_as_float(o[4 * t + 2]) * inv, __uint_as_float(o[4 * t + 3]) * inv);
      }
      p.ws_ml[wt.slot * C::BM + rrow] = make_float2(m_run, l_run);
      __threadfence();
    }
    if (rec) {
      prof.stamp(kPhEpilogue, kEpPartial, 1);
      prof.stamp(kPhEpilogue, kEpCount, 0);
    }
    volatile int* last_flag = reinterpret_cast<volatile int*>(sgen + C::OFF_MISC + 8) + qi;
    ptx::named_bar_sync(1 + qi, 128);
    if (row == 0) {
      int last = 0;
      if (*w.abort == 0) {
        int* cnt = p.ws_cnt + (slot0 / p.split) * C::NQ + qi;
        last = atomicAdd(cnt, 1) == p.split - 1;
        if (last) {
          __threadfence();
          *cnt = 0;  // ready for the next launch
        }
      }
      *last_flag = last;
    }
    ptx::named_bar_sync(1 + qi, 128);
    if (rec) prof.stamp(kPhEpilogue, kEpCount, 1);
    if (*last_flag == 0) {  // uniform over the warpgroup
      if (rec) prof.stamp(kPhEpilogue, kEpAll, 1);
      return;
    }
    if (rec) prof.stamp(kPhEpilogue, kEpMerge, 0);

    float wgt[kMaxSplit], mq[kMaxSplit];
    float mmax = -INFINITY;
#pragma unroll
    for (int q = 0; q < kMaxSplit; ++q) {
      if (q < p.split) {
        const float2 ml = q == wt.part ? make_float2(m_run, l_run)
                                       : __ldcg(p.ws_ml + (slot0 + q) * C::BM + rrow);
        mq[q] = ml.x;
        wgt[q] = ml.y;
        mmax = fmaxf(mmax, ml.x);
      }
    }
    float tot = 0.f;
#pragma unroll
    for (int q = 0; q < kMaxSplit; ++q) {
      if (q < p.split) {
        wgt[q] *= ptx::ex2_approx((mq[q] - mmax) * sl2);
        tot += wgt[q];
      }
    }
    const float inv_tot = 1.f / tot;
    const float inv_own = 1.f / l_run;
    // 16 columns at a time: the loads of every other part are issued before
    // any of them is used, so their L2 latencies overlap.
#pragma unroll 1
    for (int b = 0; b < C::D / 16; ++b) {
      float4 rv[kMaxSplit][4];
#pragma unroll
      for (int q = 0; q < kMaxSplit; ++q) {
        if (q < p.split && q != wt.part) {
          const float4* src = col0(slot0 + q) + (b * 4) * C::BM;
#pragma unroll
          for (int t = 0; t < 4; ++t) rv[q][t] = __ldcg(src + t * C::BM);
        }
      }
      uint32_t o[16];  // this part's own values, recomputed exactly as written
      ptx::tmem_ld16(lane_base + o_col + b * 16, o);
      ptx::tmem_wait_ld();
      ptx::reg_fence(o);
      float acc[16];
#pragma unroll
      for (int e = 0; e < 16; ++e) acc[e] = 0.f;
#pragma unroll
      for (int q = 0; q < kMaxSplit; ++q) {
        if (q < p.split) {
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            const float4 v =
                q == wt.part
                    ? make_float4(__uint_as_float(o[4 * t + 0]) * inv_own, __uint_as_float(o[4 * t + 1]) * inv_own,
                                  __uint_as_float(o[4 * t + 2]) * inv_own, __uint_as_float(o[4 * t + 3]) * inv_own)
                    : rv[q][t];
            acc[4 * t + 0] = fmaf(wgt[q], v.x, acc[4 * t + 0]);
            acc[4 * t + 1] = fmaf(wgt[q], v.y, acc[4 * t + 1]);
            acc[4 * t + 2] = fmaf(wgt[q], v.z, acc[4 * t + 2]);
            acc[4 * t + 3] = fmaf(wgt[q], v.w, acc[4 * t + 3]);
          }
        }
      }
#pragma unroll
      for (int e = 0; e < 16; ++e) acc[e] *= inv_tot;
      stage16(b, acc);
    }
    ptx::fence_proxy_async_smem();
    if (rec) prof.stamp(kPhEpilogue, kEpMerge, 1);
  } else if (go) {
    if (rec) prof.stamp(kPhEpilogue, kEpMerge, 0);
    ptx::tc_fence_after();
    const float inv = 1.f / l_run;
#pragma unroll 1
    for (int c = 0; c < C::D / 32; ++c) {
      float v[32];
      own32(c, inv, v);
      stage32(c, v);
    }
    ptx::fence_proxy_async_smem();
    if (rec) prof.stamp(kPhEpilogue, kEpMerge, 1);
  }
  if (rec) prof.stamp(kPhEpilogue, kEpStore, 0);
  ptx::named_bar_sync(1 + qi, 128);
  if (wi == 0 && lane == 0 && *w.abort == 0) {
#pragma unroll
    for (int d = 0; d < C::DBLK; ++d)
      ptx::tma_store_3d(tmO, stage_s + d * C::Q_BLK_BYTES, d * 64, q_row0 + qi * C::QROWS, bh);
    ptx::tma_store_commit();
    if (rec) {
      prof.stamp(kPhEpilogue, kEpStore, 1);
      prof.stamp(kPhEpilogue, kEpAll, 1);
    }
    ptx::tma_store_wait_read0();
  }
}

// Eight softmax warps per Q tile (AttnConfig::W8; two S buffers, P in one
// part, whole units).  Warp w of tile i serves TMEM lanes 32 (w % 4) +
// 16 ((w / 4) % 2) .. + 15 through the 16-lane forms: thread t holds rows
// r = 16-lane base + t / 4 and r + 8, and per 8-key block the two keys
// 2 (t % 4), 2 (t % 4) + 1 of each.  The four threads of a row combine its
// maximum by two shuffles; its sum stays a per-thread partial (rescaled by
// the same factors) until the epilogue adds the four.  The arithmetic per
// element is the four-warp step's: same argument FMA, exponential and
// rounding of P; the row max is the same value; the row sum is added up in
// another order.
template <int NB>
__device__ __forceinline__ void tmem_ld_rows16(uint32_t taddr, uint32_t (&r)[4 * NB]) {
  static_assert(NB % 4 == 0, "8-column blocks in multiples of 4");
#pragma unroll
  for (int k = 0; k + 8 <= NB; k += 8)
    ptx::tmem_ld16x256b_x8(taddr + 8 * k, *reinterpret_cast<uint32_t(*)[32]>(&r[4 * k]));
  if constexpr (NB % 8 == 4)
    ptx::tmem_ld16x256b_x4(taddr + 8 * (NB - 4), *reinterpret_cast<uint32_t(*)[16]>(&r[4 * (NB - 4)]));
}

// P of 8-key blocks [K0, K1) of NB: packed columns 4 K0 .. 4 K1 - 1, two
// registers per 4 columns.
template <int K0, int K1, int NB>
__device__ __forceinline__ void tmem_st_p16(uint32_t taddr, const uint32_t (&pk)[2 * NB]) {
  static_assert((K1 - K0) % 4 == 0, "8-key blocks in multiples of 4");
#pragma unroll
  for (int k = K0; k + 8 <= K1; k += 8)
    ptx::tmem_st16x128b_x8(taddr + 4 * k, *reinterpret_cast<const uint32_t(*)[16]>(&pk[2 * k]));
  if constexpr ((K1 - K0) % 8 == 4)
    ptx::tmem_st16x128b_x4(taddr + 4 * (K1 - 4),
                           *reinterpret_cast<const uint32_t(*)[8]>(&pk[2 * (K1 - 4)]));
}

template <typename T, class C, bool PROFILE>
__device__ void softmax_role16(int qi, uint32_t tmem, uint32_t sbase, uint8_t* sgen,
                               const CUtensorMap* tmO, const WorkTile& wt, const AttnParams& p,
                               const WaitCtx& w, const Prof<PROFILE>& prof) {
  static_assert(!C::PAIR && (C::NSBUF == 1 || C::PHALVES == 1), "W8 tiles");
  static_assert(C::BN % 32 == 0 && C::D % 64 == 0, "");
  constexpr int NB = C::BN / 8;  // 8-key blocks of S
  constexpr int NO = C::D / 8;   // 8-column blocks of O
  auto bar = [&](int i) { return sbase + C::OFF_BAR + 8u * i; };
  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  const int row0 = 32 * (warp & 3) + 16 * ((warp >> 2) & 1);  // first TMEM lane of this warp
  const int rA = row0 + lane / 4, rB = rA + 8;                 // this thread's rows
  const int kc = 2 * (lane & 3);                               // its first key of each block
  const uint32_t lane_base = tmem + (static_cast<uint32_t>(row0) << 16);
  const uint32_t o_col = C::TMEM_O_COL + qi * C::D;
  const float sl2 = p.scale_log2;
  const bool lead = row0 == 0 && lane == 0;
  const bool rec = PROFILE && qi == 0 && lead;
  const bool rec1 = PROFILE && qi == 1 && lead;
  const uint64_t sl2x2 = ptx::f2_pack(sl2, sl2);

  float mA = -INFINITY, mB = -INFINITY;  // running maxima of rows rA, rB
  float lA = 0.f, lB = 0.f;              // this thread's partial row sums
  bool ok = true;
  for (int j = 0; j < wt.n; ++j) {
    const int sl = j < kProfSlots ? j : kProfSlots;
    const int buf = j % C::NSBUF;
    const uint32_t s_col = (qi * C::NSBUF + buf) * C::BN;
    ok = __all_sync(0xffffffffu, wait_bar(bar(C::BAR_S_FULL + qi * C::NSBUF + buf),
                                          static_cast<uint32_t>((j / C::NSBUF) & 1), w, kSiteSFull));
    if (!ok) break;
    ptx::tc_fence_after();
    if (rec) {
      prof.stamp(kPhQK, sl, 1);
      prof.stamp(kPhSoftmax, sl, 0);
      prof.stamp(kPhSmLoadS, sl, 0);
    }
    if (rec1) prof.stamp(kPhSoftmaxT1, sl, 0);
    uint32_t sr[4 * NB];
    tmem_ld_rows16<NB>(lane_base + s_col, sr);
    ptx::tmem_wait_ld();
    ptx::reg_fence(sr);
    if (rec) {
      prof.stamp(kPhSmLoadS, sl, 1);
      prof.stamp(kPhSmMax, sl, 0);
    }
    const int lim = p.S - (wt.kv_lo + j) * C::BN;  // valid keys in this tile
    if (lim < C::BN) {
#pragma unroll
      for (int k = 0; k < NB; ++k)
#pragma unroll
        for (int e = 0; e < 4; ++e)
          if (8 * k + kc + (e & 1) >= lim) sr[4 * k + e] = __float_as_uint(-INFINITY);
    }
    float xa[2] = {-INFINITY, -INFINITY}, xb[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int k = 0; k < NB; ++k) {
      xa[k & 1] = ptx::fmax3(xa[k & 1], __uint_as_float(sr[4 * k]), __uint_as_float(sr[4 * k + 1]));
      xb[k & 1] = ptx::fmax3(xb[k & 1], __uint_as_float(sr[4 * k + 2]), __uint_as_float(sr[4 * k + 3]));
    }
    float xA = fmaxf(xa[0], xa[1]), xB = fmaxf(xb[0], xb[1]);
    xA = fmaxf(xA, __shfl_xor_sync(0xffffffffu, xA, 1));
    xB = fmaxf(xB, __shfl_xor_sync(0xffffffffu, xB, 1));
    xA = fmaxf(xA, __shfl_xor_sync(0xffffffffu, xA, 2));
    xB = fmaxf(xB, __shfl_xor_sync(0xffffffffu, xB, 2));

    // Lazy rescale per row, as in the four-warp step.
    float aA = 1.f, aB = 1.f;
    bool resc = false;
    if (j == 0) {
      mA = xA;
      mB = xB;
    } else {
      if ((xA - mA) * sl2 > RESCALE_THRESHOLD) {
        aA = ptx::ex2_approx((mA - xA) * sl2);
        mA = xA;
        resc = true;
      }
      if ((xB - mB) * sl2 > RESCALE_THRESHOLD) {
        aB = ptx::ex2_approx((mB - xB) * sl2);
        mB = xB;
        resc = true;
      }
    }
    if (__any_sync(0xffffffffu, resc)) {
      // O holds the sum through P V of step j - 1: with two S buffers wait
      // for its O_DONE; with one, the S_FULL seen above already covers it.
      if constexpr (C::ODONE_PER_STEP) {
        ok = __all_sync(0xffffffffu, wait_bar(bar(C::BAR_O_DONE + qi),
                                              static_cast<uint32_t>((j - 1) & 1), w, kSiteODone));
        if (!ok) break;
      }
      ptx::tc_fence_after();
#pragma unroll 1
      for (int c0 = 0; c0 < NO; c0 += 8) {  // 64 columns of O at a time
        uint32_t o[32];
        ptx::tmem_ld16x256b_x8(lane_base + o_col + 8 * c0, o);
        ptx::tmem_wait_ld();
        ptx::reg_fence(o);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          o[4 * k] = __float_as_uint(__uint_as_float(o[4 * k]) * aA);
          o[4 * k + 1] = __float_as_uint(__uint_as_float(o[4 * k + 1]) * aA);
          o[4 * k + 2] = __float_as_uint(__uint_as_float(o[4 * k + 2]) * aB);
          o[4 * k + 3] = __float_as_uint(__uint_as_float(o[4 * k + 3]) * aB);
        }
        ptx::tmem_st16x256b_x8(lane_base + o_col + 8 * c0, o);
      }
    }
    if (rec) {
      prof.stamp(kPhSmMax, sl, 1);
      prof.stamp(kPhSmExp, sl, 0);
    }

    // P = exp2(s * scale_log2 - m * scale_log2), rounded to T, over S.
    const float negA = -mA * sl2, negB = -mB * sl2;
    const uint64_t negA2 = ptx::f2_pack(negA, negA), negB2 = ptx::f2_pack(negB, negB);
    const float poly_a = sl2 * (1.0f / 134.0f);
    const float poly_bA = (negA + 126.0f) * (1.0f / 134.0f);
    const float poly_bB = (negB + 126.0f) * (1.0f / 134.0f);
    uint64_t sumA2 = 0ull, sumB2 = 0ull;
    uint32_t pk[2 * NB];
    // With P in two parts, the first (blocks [0, KB)) is published as soon
    // as it is in tensor memory.
    constexpr int KB = C::PHALVES == 2 ? 4 * C::PSPLIT_CHUNKS : NB;
    const int pbar = C::BAR_P_READY + (qi * C::NSBUF + buf) * C::PHALVES;
#pragma unroll
    for (int k = 0; k < NB; ++k) {
      if (C::PHALVES == 2 && k == KB) {
        tmem_st_p16<0, (C::PHALVES == 2 ? KB : 0), NB>(lane_base + s_col, pk);
        ptx::tmem_wait_st();
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(bar(pbar));
        if (rec) prof.stamp(kPhPFirst, sl, 0);
        if (rec1) prof.stamp(kPhPFirst, sl, 1);
      }
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const float s0 = __uint_as_float(sr[4 * k + 2 * r]), s1 = __uint_as_float(sr[4 * k + 2 * r + 1]);
        float p0, p1;
        if (poly_pair<C::POLY8>((2 * k + r) % 16)) {
          ptx::exp2_poly_pair(s0, s1, poly_a, r ? poly_bB : poly_bA, p0, p1);
        } else {
          const uint64_t x2 = ptx::f2_fma(ptx::f2_pack(s0, s1), sl2x2, r ? negB2 : negA2);
          float x0, x1;
          ptx::f2_unpack(x2, x0, x1);
          p0 = ptx::ex2_approx(x0);
          p1 = ptx::ex2_approx(x1);
        }
        if (r)
          sumB2 = ptx::f2_add(sumB2, ptx::f2_pack(p0, p1));
        else
          sumA2 = ptx::f2_add(sumA2, ptx::f2_pack(p0, p1));
        pk[2 * k + r] = pack2<T>(p0, p1);
      }
    }
    tmem_st_p16<(C::PHALVES == 2 ? KB : 0), NB, NB>(lane_base + s_col, pk);
    float s0, s1, s2, s3;
    ptx::f2_unpack(sumA2, s0, s1);
    ptx::f2_unpack(sumB2, s2, s3);
    if (rec) {
      prof.stamp(kPhSmExp, sl, 1);
      prof.stamp(kPhSmStoreP, sl, 0);
    }
    ptx::tmem_wait_st();
    if (rec) prof.stamp(kPhSmStoreP, sl, 1);
    ptx::tc_fence_before();
    __syncwarp();
    if (lane == 0) ptx::mbar_arrive(bar(pbar + C::PHALVES - 1));
    if (rec) prof.stamp(kPhSoftmax, sl, 1);
    if (rec1) prof.stamp(kPhSoftmaxT1, sl, 1);
    lA = lA * aA + (s0 + s1);
    lB = lB * aB + (s2 + s3);
  }

  // Epilogue: the row sums, then O / rowsum into the Q slot and a TMA store.
  lA += __shfl_xor_sync(0xffffffffu, lA, 1);
  lB += __shfl_xor_sync(0xffffffffu, lB, 1);
  lA += __shfl_xor_sync(0xffffffffu, lA, 2);
  lB += __shfl_xor_sync(0xffffffffu, lB, 2);
  constexpr uint32_t kTileThreads = 32 * C::WARPS_PER_TILE;
  if (rec) prof.stamp(kPhEpilogue, kEpAll, 0);
  ptx::named_bar_sync(1 + qi, kTileThreads);
  bool go = ok && (*w.abort == 0);
  if (go) go = wait_bar(bar(C::BAR_O_FINAL + qi), 0, w, kSiteODone);
  go = __all_sync(0xffffffffu, go);
  const uint32_t stage_s = sbase + C::OFF_Q + qi * C::Q_TILE_BYTES;
  uint8_t* stage_g = sgen + C::OFF_Q + qi * C::Q_TILE_BYTES;
  if (go) {
    ptx::tc_fence_after();
    const float invA = 1.f / lA, invB = 1.f / lB;
    // Columns 8k + kc, + 1 of rows rA and rB: one 4-byte value each in the
    // 128B-swizzled staging tile (the TMA box {64, QROWS}); 64 columns (one
    // 128 B block of every row) at a time.
#pragma unroll 1
    for (int c0 = 0; c0 < NO; c0 += 8) {
      uint32_t o[32];
      ptx::tmem_ld16x256b_x8(lane_base + o_col + 8 * c0, o);
      ptx::tmem_wait_ld();
      ptx::reg_fence(o);
      const int dblk = c0 / 8;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const uint32_t va =
            pack2<T>(__uint_as_float(o[4 * k]) * invA, __uint_as_float(o[4 * k + 1]) * invA);
        const uint32_t vb =
            pack2<T>(__uint_as_float(o[4 * k + 2]) * invB, __uint_as_float(o[4 * k + 3]) * invB);
        *reinterpret_cast<uint32_t*>(stage_g + dblk * C::Q_BLK_BYTES + rA * 128 +
                                     ((k ^ (rA & 7)) * 16) + 2 * kc) = va;
        *reinterpret_cast<uint32_t*>(stage_g + dblk * C::Q_BLK_BYTES + rB * 128 +
                                     ((k ^ (rB & 7)) * 16) + 2 * kc) = vb;
      }
    }
    ptx::fence_proxy_async_smem();
  }
  ptx::named_bar_sync(1 + qi, kTileThreads);
  if (lead && *w.abort == 0) {
#pragma unroll
    for (int d = 0; d < C::DBLK; ++d)
      ptx::tma_store_3d(tmO, stage_s + d * C::Q_BLK_BYTES, d * 64, wt.q_row0 + qi * C::QROWS, wt.bh);
    ptx::tma_store_commit();
    if (rec) prof.stamp(kPhEpilogue, kEpAll, 1);
    ptx::tma_store_wait_read0();
  }
}

// Correction warpgroup (AttnConfig::CORR; classic schedule, whole units).
// Warp w serves rows 32 (w % 4) .. 32 (w % 4) + 31 of both Q tiles.
//   Steps: for each step, tile 0 then tile 1, it takes the tile's rescale
//   factors (BAR_CORR), rescales the rows of O that need it once P V of the
//   previous step is complete, and adds its arrival to the first P part of
//   the step, so the MMA warp issues P V only onto a rescaled O.  A step with
//   no rescale costs it one wait and one arrival, off the softmax warps'
//   path (the request comes after the row max, the first P part about a
//   thousand cycles later).
//   Epilogue: for each tile, the row sums (BAR_CORR_END) and the last P V
//   (BAR_O_FINAL), then O / rowsum into the tile's Q slot (free once the
//   last S has read it) in the TMA store's 128B-swizzled layout, and the TMA
//   store.  Tile 0's runs while tile 1's last step does.
// Every wait is bounded; after a failed one the abort flag releases the
// other roles, and every correction warp still reaches each named barrier.
template <typename T, class C>
__device__ void correction_role(uint32_t tmem, uint32_t sbase, uint8_t* sgen,
                                const CUtensorMap* tmO, const WorkTile& wt, const WaitCtx& w) {
  auto bar = [&](int i) { return sbase + C::OFF_BAR + 8u * i; };
  const int wi = (threadIdx.x / 32) & 3;  // TMEM lane quarter
  const int lane = threadIdx.x & 31;
  const int row = wi * 32 + lane;
  const uint32_t lane_base = tmem + (static_cast<uint32_t>(wi * 32) << 16);
  constexpr uint32_t kBarEpi = 3;  // named barrier of the correction warpgroup

  // Step j of tile qi: rescale the rows of this warp that need it, then
  // count in on the step's first P part.
  auto step = [&](int qi, int j) -> bool {
    const int buf = j % C::NSBUF;
    const float alpha =
        ptx::ld_shared_f32(sbase + C::OFF_CORR + 4u * ((qi * C::NSBUF + buf) * C::QROWS + row));
    if (__any_sync(0xffffffffu, alpha != 1.f)) {
      // O holds the sum through P V of step j - 1 (j >= 1: the first step
      // sets the max and never rescales).  With one S buffer S_i(j), whose
      // completion the softmax has seen, was issued behind that P V by the
      // same thread and committed after it; otherwise O_DONE says so.
      bool done;
      if constexpr (C::ODONE_PER_STEP) {
        done = wait_bar(bar(C::BAR_O_DONE + qi), static_cast<uint32_t>((j - 1) & 1), w, kSiteODone);
      } else {
        done = wait_bar(bar(C::BAR_S_FULL + qi * C::NSBUF + buf),
                        static_cast<uint32_t>((j / C::NSBUF) & 1), w, kSiteSFull);
      }
      if (!__all_sync(0xffffffffu, done)) return false;
      ptx::tc_fence_after();
      const uint32_t o_col = C::TMEM_O_COL + qi * C::D;
#pragma unroll 1
      for (int c = 0; c < C::D / 32; ++c) {
        uint32_t o[32];
        ptx::tmem_ld32(lane_base + o_col + c * 32, o);
        ptx::tmem_wait_ld();
        ptx::reg_fence(o);
#pragma unroll
        for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
        ptx::tmem_st32(lane_base + o_col + c * 32, o);
      }
      ptx::tmem_wait_st();
    }
    ptx::tc_fence_before();
    __syncwarp();
    if (lane == 0) ptx::mbar_arrive(bar(C::BAR_P_READY + (qi * C::NSBUF + buf) * C::PHALVES));
    return true;
  };

  // Requests are served in step order, tile 0 then tile 1, with a bounded
  // wait on the one expected next.  With one MMA issuer that is the order in
  // which they come (S_0(j) completes before S_1(j)); with two, a tile that
  // runs ahead waits at its first P part for the other's request of the same
  // step.  (Serving whichever comes first by polling both barriers in turn
  // measured far slower: a thread suspended in try_wait on one barrier woke
  // up to ~2000 cycles after the other's request, which delayed P V.)  No
  // request barrier runs two phases ahead (the request of step j + NSBUF
  // needs the S that follows P V of step j).
  bool ok = true;
#pragma unroll 1
  for (int j = 0; j < wt.n && ok; ++j) {
    const uint32_t par = static_cast<uint32_t>((j / C::NSBUF) & 1);
#pragma unroll 1
    for (int qi = 0; qi < C::NQ && ok; ++qi) {
      ok = __all_sync(0xffffffffu,
                      wait_bar(bar(C::BAR_CORR + qi * C::NSBUF + j % C::NSBUF), par, w, kSiteCorr));
      if (ok) ok = step(qi, j);
    }
  }

#pragma unroll 1
  for (int qi = 0; qi < C::NQ; ++qi) {
    bool go = ok && *w.abort == 0;
    if (go) go = wait_bar(bar(C::BAR_CORR_END + qi), 0, w, kSiteCorr);
    if (go) go = wait_bar(bar(C::BAR_O_FINAL + qi), 0, w, kSiteODone);
    go = __all_sync(0xffffffffu, go);
    const uint32_t stage_s = sbase + C::OFF_Q + qi * C::Q_TILE_BYTES;
    if (go) {
      ptx::tc_fence_after();
      const float inv =
          1.f / ptx::ld_shared_f32(sbase + C::OFF_CORR +
                                   4u * (C::CORR_ALPHA_FLOATS + qi * C::QROWS + row));
      uint8_t* stage_g = sgen + C::OFF_Q + qi * C::Q_TILE_BYTES;
      const uint32_t o_col = C::TMEM_O_COL + qi * C::D;
#pragma unroll 1
      for (int c = 0; c < C::D / 32; ++c) {
        uint32_t o[32];
        ptx::tmem_ld32(lane_base + o_col + c * 32, o);
        ptx::tmem_wait_ld();
        ptx::reg_fence(o);
        // Columns 32c .. 32c + 31: four 16-byte chunks of 8 values each, in
        // 64-column block (32c) / 64, chunk ((32c) % 64) / 8 + q, swizzled by
        // the row (the layout of the TMA box {64, QROWS}).
        const int dblk = (c * 32) / 64;
        const int chunk0 = ((c * 32) % 64) / 8;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint4 u;
          u.x = pack2<T>(__uint_as_float(o[8 * q + 0]) * inv, __uint_as_float(o[8 * q + 1]) * inv);
          u.y = pack2<T>(__uint_as_float(o[8 * q + 2]) * inv, __uint_as_float(o[8 * q + 3]) * inv);
          u.z = pack2<T>(__uint_as_float(o[8 * q + 4]) * inv, __uint_as_float(o[8 * q + 5]) * inv);
          u.w = pack2<T>(__uint_as_float(o[8 * q + 6]) * inv, __uint_as_float(o[8 * q + 7]) * inv);
          const int chunk = (chunk0 + q) ^ (row & 7);
          *reinterpret_cast<uint4*>(stage_g + dblk * C::Q_BLK_BYTES + row * 128 + chunk * 16) = u;
        }
      }
      ptx::fence_proxy_async_smem();
    }
    ptx::named_bar_sync(kBarEpi, 128);
    if (wi == 0 && lane == 0 && *w.abort == 0) {
#pragma unroll
      for (int d = 0; d < C::DBLK; ++d)
        ptx::tma_store_3d(tmO, stage_s + d * C::Q_BLK_BYTES, d * 64, wt.q_row0 + qi * C::QROWS,
                          wt.bh);
      ptx::tma_store_commit();
    }
  }
  if (wi == 0 && lane == 0) ptx::tma_store_wait_read0();
}

// Profiler observer: stamps the completion of each P V of Q tile 0.  It only
// watches; a missed phase costs a stamp, never an error status.  It waits
// with a suspend hint so it does not take issue slots from the softmax warps
// of its SM sub-partition (a polling observer slowed them visibly).  Where
// O_DONE is not committed every step (one S buffer), the completion of
// P_0(j) V_j is that of S_0(j+1), committed right behind it by the same
// thread, and the last step's is O_FINAL; the profiled kernel thus commits
// exactly what the production kernel does.
template <class C>
__device__ void observer_role(uint32_t sbase, int n, const WaitCtx& w, const Prof<true>& prof) {
  if (!C::ODONE_PER_STEP && n > 1) {
    // Step past S_0(0), the first completion of S_FULL (a parity-1 wait on a
    // fresh barrier would return at once), so that the k-th wait below is
    // for the (k+1)-th completion.
    const uint32_t bar = sbase + C::OFF_BAR + 8u * (C::BAR_S_FULL + 0);
    const unsigned long long t0 = ptx::globaltimer_ns();
    while (!ptx::mbar_try_wait_sleep(bar, 0, 100000u)) {
      if (*w.abort || ptx::globaltimer_ns() - t0 > w.timeout_ns) return;
    }
  }
  for (int j = 0; j < n; ++j) {
    uint32_t b, parity;
    if (C::ODONE_PER_STEP) {
      b = C::BAR_O_DONE + 0;
      parity = j & 1;
    } else if (j + 1 < n) {
      b = C::BAR_S_FULL + 0;  // tile 0, the only S buffer
      parity = (j + 1) & 1;
    } else {
      b = C::BAR_O_FINAL + 0;
      parity = 0;
    }
    const uint32_t bar = sbase + C::OFF_BAR + 8u * b;
    const unsigned long long t0 = ptx::globaltimer_ns();
    while (!ptx::mbar_try_wait_sleep(bar, parity, 100000u)) {
      if (*w.abort || ptx::globaltimer_ns() - t0 > w.timeout_ns) return;
    }
    prof.stamp(kPhPV, j, 1);
  }
}

// ============================================================================
// Persistent schedule (the PERSIST kernel variant): every CTA runs its step range
// as a series of items (ItemCursor), all three roles walking the same items.
// The K/V ring, the S and P barriers run on the CTA's step count J, so a new
// item's first S follows the previous item's last P V like any other S; the
// Q, O_FINAL and Q_FREE barriers complete one phase per item.  The next
// item's Q tiles are loaded as soon as the current item's last S has read
// them (Q_FREE), so its first S is computed while the softmax warps finish
// the current item; O goes from registers straight to global memory.
// ============================================================================

// Producer: Q of the first item, K_0, then per step V_J and K_{J+1}; at an
// item's last step the next item's Q tiles (after Q_FREE) and its K_0.
template <class C, bool PROFILE>
__device__ void load_role_persistent(const CUtensorMap* tmQ, const CUtensorMap* tmK,
                                     const CUtensorMap* tmV, uint32_t sbase, const AttnParams& p,
                                     const WaitCtx& w, const Prof<PROFILE>& prof) {
  auto bar = [&](int i) { return sbase + C::OFF_BAR + 8u * i; };
  const uint64_t pol_kv = ptx::l2_policy_evict_last();
  const uint64_t pol_q = ptx::l2_policy_evict_first();
  ItemCursor cur;
  cur.init(blockIdx.x, p);
  Item it, nx;
  if (!cur.next(it, p, C::BM)) return;
  bool has_nx = cur.next(nx, p, C::BM);

  int q_item = 0;  // the item whose Q load is the latest issued
  auto load_q = [&](const Item& x) {
#pragma unroll
    for (int i = 0; i < C::NQ; ++i) {
      ptx::mbar_arrive_expect_tx(bar(C::BAR_Q + i), C::Q_TILE_BYTES);
#pragma unroll
      for (int d = 0; d < C::DBLK; ++d)
        ptx::tma_load_3d_hint(sbase + C::OFF_Q + i * C::Q_TILE_BYTES + d * C::Q_BLK_BYTES, tmQ,
                              bar(C::BAR_Q + i), d * 64, x.q_row0 + i * C::QROWS, x.bh, pol_q);
    }
  };
  prof.stamp(kPhLoadQ, 0, 0);
  load_q(it);
  if (p.fault_mode == 1) return;  // test hook: K/V never arrive; consumers time out

  int t = 0;  // ring item counter: K_J is item 2J, V_J item 2J + 1
  int last_issued[C::STAGES];
#pragma unroll
  for (int s = 0; s < C::STAGES; ++s) last_issued[s] = -1;
  bool ok = true;

  // k_bar >= 0: the K load completes on that slot's FULL barrier (armed by
  // the V item just before it for both tiles' bytes); its own gets a plain
  // arrival to keep its phase count.
  auto produce = [&](bool is_k, const Item& x, int j, int J, bool joint, int k_bar) {
    const int s = t % C::STAGES;
    if (t >= C::STAGES) {
      uint32_t eb, par;
      if constexpr (C::V_RELEASE_WITH_K) {
        const int m = (t - C::STAGES + 1) / 2;  // the K item whose commit frees slot s
        eb = bar(C::BAR_KV_EMPTY + (2 * m) % C::STAGES);
        par = static_cast<uint32_t>(m / C::K_SLOT_PERIOD) & 1u;
      } else {
        eb = bar(C::BAR_KV_EMPTY + s);
        par = static_cast<uint32_t>(t / C::STAGES - 1) & 1u;
      }
      if (!wait_bar(eb, par, w, kSiteKvEmpty)) {
        ok = false;
        return;
      }
    }
    prof.stamp(is_k ? kPhLoadK : kPhLoadV, J < kProfSlots ? J : kProfSlots, 0);
    uint32_t full = bar(C::BAR_KV_FULL + s);
    if (k_bar >= 0) {
      ptx::mbar_arrive(full);
      full = bar(C::BAR_KV_FULL + k_bar);
    } else {
      ptx::mbar_arrive_expect_tx(full, joint ? 2 * C::KV_TILE_BYTES : C::KV_TILE_BYTES);
    }
    const uint32_t dst = sbase + C::OFF_KV + s * C::KV_TILE_BYTES;
    const int key0 = (x.kv_lo + j) * C::BN;
    if (is_k) {
#pragma unroll
      for (int d = 0; d < C::DBLK; ++d)
        ptx::tma_load_3d_hint(dst + d * C::K_BLK_BYTES, tmK, full, d * 64, key0, x.bh, pol_kv);
    } else {
#pragma unroll
      for (int d = 0; d < C::DBLK; ++d)
        ptx::tma_load_3d_hint(dst + d * C::V_BLK_BYTES, tmV, full, d * 64, key0, x.bh, pol_kv);
    }
    last_issued[s] = t;
    ++t;
  };

  produce(true, it, 0, 0, false, -1);
  int J = 0;
  int item = 0;
  while (ok) {
    // The next item's Q tiles go to L2 a few steps ahead, so that their load
    // into shared memory (which has to wait for Q_FREE) is short.
    const int pf = it.n > 3 ? it.n - 3 : 0;
    for (int j = 0; j < it.n && ok; ++j, ++J) {
      const bool last = j == it.n - 1;
      if (j == pf && has_nx) {
#pragma unroll
        for (int i = 0; i < C::NQ; ++i)
#pragma unroll
          for (int d = 0; d < C::DBLK; ++d)
            ptx::tma_prefetch_l2_3d(tmQ, d * 64, nx.q_row0 + i * C::QROWS, nx.bh);
      }
      // V_J and K_{J+1} land together only inside an item; at an item's end
      // the next item's K_0 has its own barrier.
      const bool joint = C::KV_JOINT_FULL && !last;
      const int sv = t % C::STAGES;
      produce(false, it, j, J, joint, -1);
      if (!ok) break;
      if (!last) {
        produce(true, it, j + 1, J + 1, false, joint ? sv : -1);
      } else if (has_nx) {
        // The next item's K_0 first (it needs only a free slot), then its Q
        // tiles once this item's last S has read the current ones.
        produce(true, nx, 0, J + 1, false, -1);
        if (!ok) break;
#pragma unroll
        for (int i = 0; i < C::NQ; ++i)
          if (ok && !wait_bar(bar(C::BAR_Q_FREE + i), static_cast<uint32_t>(item & 1), w,
                              kSiteQFree))
            ok = false;
        if (!ok) break;
        load_q(nx);
        q_item = item + 1;
      }
    }
    if (!ok || !has_nx) break;
    it = nx;
    ++item;
    has_nx = cur.next(nx, p, C::BM);
  }
  if (!ok) {
    // Leave no bulk copy in flight: wait (bounded) for the latest load into
    // every slot (a K load of a joint landing completes with the V load of
    // the slot just before it, whose wait covers it) and for the latest Q
    // loads.
    const unsigned long long t0 = ptx::globaltimer_ns();
#pragma unroll
    for (int s = 0; s < C::STAGES; ++s) {
      if (last_issued[s] < 0) continue;
      const uint32_t r = static_cast<uint32_t>(last_issued[s] / C::STAGES) & 1u;
      while (!ptx::mbar_try_wait(bar(C::BAR_KV_FULL + s), r)) {
        if (ptx::globaltimer_ns() - t0 > w.timeout_ns) break;
      }
    }
#pragma unroll
    for (int i = 0; i < C::NQ; ++i) {
      while (!ptx::mbar_try_wait(bar(C::BAR_Q + i), static_cast<uint32_t>(q_item & 1))) {
        if (ptx::globaltimer_ns() - t0 > w.timeout_ns) break;
      }
    }
  }
}

// MMA issuer (single thread) over the CTA's items.
template <class C, bool PROFILE>
__device__ void mma_role_persistent(uint32_t tmem, uint32_t sbase, const AttnParams& p,
                                    const WaitCtx& w, const Prof<PROFILE>& prof) {
  auto bar = [&](int i) { return sbase + C::OFF_BAR + 8u * i; };
  auto signal = [&](uint32_t b) { ptx::mma_commit(b); };
  ItemCursor cur;
  cur.init(blockIdx.x, p);
  Item it, nx;
  if (!cur.next(it, p, C::BM)) return;
  bool has_nx = cur.next(nx, p, C::BM);
  bool ok = true;

  // Ring position of the next item: slot and phase parity, advanced
  // incrementally (no division on the issuing thread, which sits on the
  // per-tile chain).
  int rs = 0;
  uint32_t rph = 0;
  auto ring_advance = [&]() {
    if (++rs == C::STAGES) {
      rs = 0;
      rph ^= 1u;
    }
  };
  auto ring_wait = [&](int& stage) -> bool {
    stage = rs;
    const bool r = wait_bar(bar(C::BAR_KV_FULL + stage), rph, w, kSiteKvFull);
    ring_advance();
    if (r) ptx::tc_fence_after();
    return r;
  };

  constexpr int KSTEPS_S = C::D / 16;
  uint64_t qd0[C::NQ];
#pragma unroll
  for (int i = 0; i < C::NQ; ++i)
    qd0[i] = ptx::smem_desc_sw128(sbase + C::OFF_Q + i * C::Q_TILE_BYTES, 16, 1024);
  const uint64_t kd0 = ptx::smem_desc_sw128(sbase + C::OFF_KV, 16, 1024);
  const uint64_t vd0 = ptx::smem_desc_sw128(sbase + C::OFF_KV, C::V_BLK_BYTES, 1024);
  auto slot_off = [](int stage) -> uint32_t {
    return static_cast<uint32_t>((stage * C::KV_TILE_BYTES) >> 4);
  };
  auto issue_s = [&](int i, int stage) {
    const uint32_t d_tmem = tmem + i * C::BN;
    const uint64_t kd = ptx::desc_add(kd0, slot_off(stage));
#pragma unroll
    for (int kk = 0; kk < KSTEPS_S; ++kk) {
      const uint32_t qo = static_cast<uint32_t>(((kk >> 2) * C::Q_BLK_BYTES + (kk & 3) * 32) >> 4);
      const uint32_t ko = static_cast<uint32_t>(((kk >> 2) * C::K_BLK_BYTES + (kk & 3) * 32) >> 4);
      ptx::mma_ss<1>(d_tmem, ptx::desc_add(qd0[i], qo), ptx::desc_add(kd, ko), C::IDESC_S,
                     kk > 0 ? 1u : 0u);
    }
  };
  auto issue_pv = [&](int i, int stage, int k0, int k1, bool first) {
    const uint32_t p_tmem = tmem + i * C::BN;
    const uint32_t o_tmem = tmem + C::TMEM_O_COL + i * C::D;
    const uint64_t vd = ptx::desc_add(vd0, slot_off(stage));
#pragma unroll
    for (int kk = k0; kk < k1; ++kk)
      ptx::mma_ts<1>(o_tmem, p_tmem + kk * 8, ptx::desc_add(vd, static_cast<uint32_t>(kk * 2048 >> 4)),
                     C::IDESC_PV, (!first || kk > 0) ? 1u : 0u);
  };

  // The first item: its Q tiles, K_0 and the S of its first step.
#pragma unroll
  for (int i = 0; i < C::NQ; ++i)
    if (ok) ok = wait_bar(bar(C::BAR_Q + i), 0, w, kSiteQ);
  if (ok) {
    ptx::tc_fence_after();
    prof.stamp(kPhLoadQ, 0, 1);
    int sk;
    if ((ok = ring_wait(sk))) {
      prof.stamp(kPhLoadK, 0, 1);
#pragma unroll
      for (int i = 0; i < C::NQ; ++i) {
        if (i == 0) prof.stamp(kPhQK, 0, 0);
        issue_s(i, sk);
        signal(bar(C::BAR_S_FULL + i));
      }
      signal(bar(C::BAR_KV_EMPTY + sk));
    }
  }

  constexpr int KSTEPS = C::BN / 16;
  constexpr int KSPLIT = C::PHALVES == 2 ? 2 * C::PSPLIT_CHUNKS : KSTEPS;
  int J = 0;
  int item = 0;
  while (ok) {
    const int n = it.n;
    // Steps 0 .. n - 2: as in the classic issuer (K_{J+1} of the same item,
    // which landed with V_J under the joint landing).
    for (int j = 0; j < n - 1 && ok; ++j, ++J) {
      const int sl = J < kProfSlots ? J : kProfSlots;
      int sv;
      prof.stamp(kPhVWait, sl, 0);
      if (!(ok = ring_wait(sv))) break;
      prof.stamp(kPhVWait, sl, 1);
      prof.stamp(kPhLoadV, sl, 1);
      int sk = -1;
#pragma unroll
      for (int i = 0; i < C::NQ; ++i) {
        const int pb = C::BAR_P_READY + i * C::PHALVES;
#pragma unroll
        for (int h = 0; h < C::PHALVES; ++h) {
          if (h == C::PHALVES - 1 && sk < 0) {
            if constexpr (C::KV_JOINT_FULL) {
              sk = rs;
              ring_advance();
            } else if (!(ok = ring_wait(sk))) {
              break;
            }
            if (J + 1 < kProfSlots) prof.stamp(kPhLoadK, J + 1, 1);
          }
          if (!(ok = wait_bar(bar(pb + h), static_cast<uint32_t>(J) & 1u, w, kSitePReady))) break;
          ptx::tc_fence_after();
          if (h == 0) {
            if (i == 0) prof.stamp(kPhPV, sl, 0);
            prof.stamp(kPhMmaT0 + i, sl, 0);
          }
          issue_pv(i, sv, h == 0 ? 0 : KSPLIT, h == 0 ? KSPLIT : KSTEPS, j == 0);
        }
        if (!ok) break;
        if (i == 0 && J + 1 < kProfSlots) prof.stamp(kPhQK, J + 1, 0);
        issue_s(i, sk);
        signal(bar(C::BAR_S_FULL + i));
        if (C::ODONE_PER_STEP) signal(bar(C::BAR_O_DONE + i));
        prof.stamp(kPhMmaT0 + i, sl, 1);
      }
      if (!ok) break;
      if constexpr (!C::V_RELEASE_WITH_K) signal(bar(C::BAR_KV_EMPTY + sv));
      signal(bar(C::BAR_KV_EMPTY + sk));  // with V_RELEASE_WITH_K: V_J's slot too
    }
    if (!ok) break;

    // The item's last step.  Every S of the item has been issued: Q_FREE
    // lets the producer load the next item's Q tiles.  Each tile's last P V
    // and O_FINAL come before anything of the next item, whose K_0 and Q
    // tiles are waited for only by the next S.
    {
      const int sl = J < kProfSlots ? J : kProfSlots;
#pragma unroll
      for (int i = 0; i < C::NQ; ++i) signal(bar(C::BAR_Q_FREE + i));
      int sv;
      prof.stamp(kPhVWait, sl, 0);
      if (!(ok = ring_wait(sv))) break;
      prof.stamp(kPhVWait, sl, 1);
      prof.stamp(kPhLoadV, sl, 1);
      int sk = -1;
#pragma unroll
      for (int i = 0; i < C::NQ; ++i) {
        const int pb = C::BAR_P_READY + i * C::PHALVES;
#pragma unroll
        for (int h = 0; h < C::PHALVES; ++h) {
          if (!(ok = wait_bar(bar(pb + h), static_cast<uint32_t>(J) & 1u, w, kSitePReady))) break;
          ptx::tc_fence_after();
          if (h == 0) {
            if (i == 0) prof.stamp(kPhPV, sl, 0);
            prof.stamp(kPhMmaT0 + i, sl, 0);
          }
          issue_pv(i, sv, h == 0 ? 0 : KSPLIT, h == 0 ? KSPLIT : KSTEPS, n == 1);
        }
        if (!ok) break;
        signal(bar(C::BAR_O_FINAL + i));
        if (has_nx) {
          if (sk < 0) {
            if (!(ok = ring_wait(sk))) break;  // the next item's K_0
            if (J + 1 < kProfSlots) prof.stamp(kPhLoadK, J + 1, 1);
          }
          if (!(ok = wait_bar(bar(C::BAR_Q + i), static_cast<uint32_t>(item + 1) & 1u, w,
                              kSiteQ)))
            break;
          ptx::tc_fence_after();
          if (i == 0 && J + 1 < kProfSlots) prof.stamp(kPhQK, J + 1, 0);
          issue_s(i, sk);
          signal(bar(C::BAR_S_FULL + i));
        }
        if (C::ODONE_PER_STEP) signal(bar(C::BAR_O_DONE + i));
        prof.stamp(kPhMmaT0 + i, sl, 1);
      }
      if (!ok) break;
      if constexpr (!C::V_RELEASE_WITH_K) signal(bar(C::BAR_KV_EMPTY + sv));
      if (sk >= 0) signal(bar(C::BAR_KV_EMPTY + sk));
      ++J;
    }
    if (!has_nx) break;
    it = nx;
    ++item;
    has_nx = cur.next(nx, p, C::BM);
  }

  // Drain: every MMA this thread issued has completed before TMEM is freed.
  ptx::mma_commit<1>(bar(C::BAR_DRAIN));
  const unsigned long long t0 = ptx::globaltimer_ns();
  while (!ptx::mbar_try_wait(bar(C::BAR_DRAIN), 0)) {
    if (ptx::globaltimer_ns() - t0 > w.timeout_ns) {
      if (w.status) atomicCAS(w.status, 0, kDeviceTimeoutBase + kSiteDrain);
      break;
    }
  }
}

// Softmax warpgroup of Q tile qi over the CTA's items, with each item's
// epilogue: a whole unit normalises O into the CTA's O staging buffer and
// stores it with TMA; a kWriter piece writes its normalised partial O and
// (row max, row sum) into its CTA's workspace slot and counts in on the
// merging CTA's counter; the kMerger piece waits for its unit's writers,
// adds their partials to its own in key order and stores O as a whole unit
// does.  The two Q tiles take turns on the staging buffer (a lock in shared
// memory, held from the first write into the buffer until the TMA store
// has read it).  Every decision that guards a named barrier is taken by all
// 128 threads together (named_bar_and).
template <typename T, class C, bool PROFILE>
__device__ void softmax_role_persistent(int qi, uint32_t tmem, uint32_t sbase, uint8_t* sgen,
                                        const CUtensorMap* tmO, const AttnParams& p,
                                        const WaitCtx& w, const Prof<PROFILE>& prof) {
  auto bar = [&](int i) { return sbase + C::OFF_BAR + 8u * i; };
  const int wi = (threadIdx.x / 32) & 3;
  const int lane = threadIdx.x & 31;
  const int row = wi * 32 + lane;
  const int rrow = qi * C::QROWS + row;  // row within the unit
  const uint32_t lane_base = tmem + (static_cast<uint32_t>(wi * 32) << 16);
  const uint32_t o_col = C::TMEM_O_COL + qi * C::D;
  const float sl2 = p.scale_log2;
  const bool rec = PROFILE && qi == 0 && wi == 0 && lane == 0;
  const uint32_t nbar = 1 + qi;
  constexpr int BLK = C::BM * C::D / 4;  // float4 per workspace slot
  int* stage_lock = reinterpret_cast<int*>(sgen + C::OFF_MISC + 16);
  uint8_t* stage_g = sgen + C::OFF_STAGE;
  const uint32_t stage_s = sbase + C::OFF_STAGE;

  // Writes 16 values (columns 16b .. 16b + 15 of this thread's row) into the
  // 128B-swizzled staging tile (the layout of the TMA box {64, 128}).
  auto stage16 = [&](int b, const float* v) {
    const int dblk = (b * 16) / 64;
    const int chunk0 = ((b * 16) % 64) / 8;
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      uint4 u;
      u.x = pack2<T>(v[8 * q + 0], v[8 * q + 1]);
      u.y = pack2<T>(v[8 * q + 2], v[8 * q + 3]);
      u.z = pack2<T>(v[8 * q + 4], v[8 * q + 5]);
      u.w = pack2<T>(v[8 * q + 6], v[8 * q + 7]);
      const int chunk = (chunk0 + q) ^ (row & 7);
      *reinterpret_cast<uint4*>(stage_g + dblk * C::Q_BLK_BYTES + row * 128 + chunk * 16) = u;
    }
  };
  // One thread takes the staging lock (bounded wait).
  auto take_stage = [&]() -> bool {
    const unsigned long long t0 = ptx::globaltimer_ns();
    while (atomicCAS(stage_lock, 0, 1) != 0) {
      if (*w.abort) return false;
      if (ptx::globaltimer_ns() - t0 > w.timeout_ns) {
        *w.abort = 1;
        if (w.status) atomicCAS(w.status, 0, kDeviceTimeoutBase + kSiteStage);
        return false;
      }
    }
    return true;
  };
  // After the staging writes: one thread stores the tile with TMA (rows >= S
  // are clipped by the tensor map), waits until the TMA has read the buffer
  // and releases the lock; the others go on at once.
  auto store_staged = [&](const Item& x, bool last_rec) {
    ptx::fence_proxy_async_smem();
    ptx::named_bar_sync(nbar, 128);
    if (row == 0) {
      if (last_rec) prof.stamp(kPhEpilogue, kEpStore, 0);
#pragma unroll
      for (int d = 0; d < C::DBLK; ++d)
        ptx::tma_store_3d(tmO, stage_s + d * C::Q_BLK_BYTES, d * 64, x.q_row0 + qi * C::QROWS, x.bh);
      ptx::tma_store_commit();
      ptx::tma_store_wait_read0();
      atomicExch(stage_lock, 0);
      if (last_rec) prof.stamp(kPhEpilogue, kEpStore, 1);
    }
  };

  ItemCursor cur;
  cur.init(blockIdx.x, p);
  Item it;
  int J = 0;
  int item = 0;
  bool go = true;
  while (go && cur.next(it, p, C::BM)) {
    float m_run, l_run;
    const bool ok = softmax_steps<T, C, PROFILE>(qi, tmem, sbase, p, w, prof, it.kv_lo, it.n, J,
                                                 0, m_run, l_run);
    J += it.n;
    const bool rec0 = rec && item == 0;
    if (rec0) prof.stamp(kPhEpilogue, kEpAll, 0);
    go = ptx::named_bar_and(nbar, 128, ok && *w.abort == 0);
    if (!go) break;
    if (rec0) prof.stamp(kPhEpilogue, kEpWaitO, 0);
    bool fin = wait_bar(bar(C::BAR_O_FINAL + qi), static_cast<uint32_t>(item & 1), w, kSiteODone);
    go = ptx::named_bar_and(nbar, 128, fin);
    if (rec0) prof.stamp(kPhEpilogue, kEpWaitO, 1);
    if (!go) break;
    ptx::tc_fence_after();

    if (it.role == kWriter) {
      if (rec0) prof.stamp(kPhEpilogue, kEpPartial, 0);
      // Normalised partial O as float4 columns of this CTA's slot: the 32
      // lanes of a warp (32 consecutive rows) write 512 contiguous bytes.
      const float inv = 1.f / l_run;
      float4* dst = p.ws_o + static_cast<long long>(blockIdx.x) * BLK + rrow;
#pragma unroll 1
      for (int c = 0; c < C::D / 32; c += 2) {
        uint32_t o[64];
        ptx::tmem_ld32(lane_base + o_col + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&o[0]));
        ptx::tmem_ld32(lane_base + o_col + c * 32 + 32, *reinterpret_cast<uint32_t(*)[32]>(&o[32]));
        ptx::tmem_wait_ld();
        ptx::reg_fence(o);
#pragma unroll
        for (int t4 = 0; t4 < 16; ++t4)
          dst[(c * 8 + t4) * C::BM] = make_float4(
              __uint_as_float(o[4 * t4 + 0]) * inv, __uint_as_float(o[4 * t4 + 1]) * inv,
              __uint_as_float(o[4 * t4 + 2]) * inv, __uint_as_float(o[4 * t4 + 3]) * inv);
      }
      p.ws_ml[static_cast<long long>(blockIdx.x) * C::BM + rrow] = make_float2(m_run, l_run);
      // Every thread counts itself in with release semantics: its own
      // partial is visible to the merger before its increment is.
      ptx::red_release_gpu_add(p.ws_cnt + it.peer * C::NQ + qi, 1);
      if (rec0) prof.stamp(kPhEpilogue, kEpPartial, 1);
    } else {
      const bool merge = it.role == kMerger;
      const int nw = merge ? it.peer - static_cast<int>(blockIdx.x) : 0;  // writers: next nw CTAs
      int* cnt = p.ws_cnt + static_cast<int>(blockIdx.x) * C::NQ + qi;
      if (rec0) prof.stamp(kPhEpilogue, kEpCount, 0);
      bool ready = true;
      if (row == 0) {
        // The writers' 128 threads each count in once.
        if (merge) {
          const unsigned long long t0 = ptx::globaltimer_ns();
          while (ptx::ld_acquire_gpu(cnt) < nw * 128) {
            if (*w.abort) {
              ready = false;
              break;
            }
            if (ptx::globaltimer_ns() - t0 > w.timeout_ns) {
              *w.abort = 1;
              if (w.status) atomicCAS(w.status, 0, kDeviceTimeoutBase + kSiteMerge);
              ready = false;
              break;
            }
          }
        }
        if (ready) ready = take_stage();
      }
      go = ptx::named_bar_and(nbar, 128, ready);
      if (rec0) prof.stamp(kPhEpilogue, kEpCount, 1);
      if (!go) break;
      if (rec0) prof.stamp(kPhEpilogue, kEpMerge, 0);
      if (merge) {
        if (row == 0) *cnt = 0;  // ready for the next launch (only this CTA reads it)
        // Weights of the pieces in key order (own piece first), as the
        // classic merge computes them: w_q = l_q 2^((m_q - m) scale), m
        // their max.
        float mmax = m_run;
#pragma unroll 1
        for (int q = 1; q <= nw; ++q)
          mmax = fmaxf(mmax, __ldcg(p.ws_ml + static_cast<long long>(blockIdx.x + q) * C::BM + rrow).x);
        const float w_own = l_run * ptx::ex2_approx((m_run - mmax) * sl2);
        float tot = w_own;
#pragma unroll 1
        for (int q = 1; q <= nw; ++q) {
          const float2 ml = __ldcg(p.ws_ml + static_cast<long long>(blockIdx.x + q) * C::BM + rrow);
          tot += ml.y * ptx::ex2_approx((ml.x - mmax) * sl2);
        }
        const float inv_tot = 1.f / tot;
        const float inv_own = 1.f / l_run;
#pragma unroll 1
        for (int b = 0; b < C::D / 16; ++b) {
          uint32_t o[16];
          ptx::tmem_ld16(lane_base + o_col + b * 16, o);
          ptx::tmem_wait_ld();
          ptx::reg_fence(o);
          float acc[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) acc[e] = w_own * (__uint_as_float(o[e]) * inv_own);
#pragma unroll 1
          for (int q = 1; q <= nw; ++q) {
            const long long sq = static_cast<long long>(blockIdx.x + q);
            const float2 ml = __ldcg(p.ws_ml + sq * C::BM + rrow);
            const float wq = ml.y * ptx::ex2_approx((ml.x - mmax) * sl2);
            const float4* src = p.ws_o + sq * BLK + rrow + (b * 4) * C::BM;
            float4 v[4];
#pragma unroll
            for (int t4 = 0; t4 < 4; ++t4) v[t4] = __ldcg(src + t4 * C::BM);
#pragma unroll
            for (int t4 = 0; t4 < 4; ++t4) {
              acc[4 * t4 + 0] = fmaf(wq, v[t4].x, acc[4 * t4 + 0]);
              acc[4 * t4 + 1] = fmaf(wq, v[t4].y, acc[4 * t4 + 1]);
              acc[4 * t4 + 2] = fmaf(wq, v[t4].z, acc[4 * t4 + 2]);
              acc[4 * t4 + 3] = fmaf(wq, v[t4].w, acc[4 * t4 + 3]);
            }
          }
#pragma unroll
          for (int e = 0; e < 16; ++e) acc[e] *= inv_tot;
          stage16(b, acc);
        }
      } else {
        const float inv = 1.f / l_run;
#pragma unroll 1
        for (int c = 0; c < C::D / 32; ++c) {
          uint32_t o[32];
          ptx::tmem_ld32(lane_base + o_col + c * 32, o);
          ptx::tmem_wait_ld();
          ptx::reg_fence(o);
          float v[32];
#pragma unroll
          for (int e = 0; e < 32; ++e) v[e] = __uint_as_float(o[e]) * inv;
          stage16(2 * c, v);
          stage16(2 * c + 1, v + 16);
        }
      }
      if (rec0) prof.stamp(kPhEpilogue, kEpMerge, 1);
      store_staged(it, rec0);
    }
    if (rec0) prof.stamp(kPhEpilogue, kEpAll, 1);
    ++item;
  }
}

// PERSIST: the persistent schedule (AttnParams::grid and following), compiled as a
// kernel of its own for the variants that have it (AttnConfig::PERSIST_OK),
// so that its softmax loop and the classic one are allocated registers
// separately.  CORR: the classic schedule with a correction warpgroup
// (AttnConfig::CORR), whole units only.  FOUR: four softmax warps per Q tile
// where the variant would run eight (AttnConfig::W8), for split plans.
template <typename T, int D, int BN, int NQ, int STAGES, bool PROFILE, bool PAIR = false,
          bool PERSIST = false, bool CORR = false, bool FOUR = false>
__global__ void __launch_bounds__(AttnConfig<T, D, BN, NQ, STAGES, PAIR, CORR, FOUR>::NUM_THREADS,
                                  AttnConfig<T, D, BN, NQ, STAGES, PAIR, CORR, FOUR>::MIN_CTAS_PER_SM)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tmQ,
                    const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV,
                    const __grid_constant__ CUtensorMap tmO, const AttnParams p) {
// The body uses sm_100a-only instructions (tcgen05, setmaxnreg): it is
// compiled for the arch-specific target only.  A build that also emits
// generic compute_100 PTX (nvcc -arch=sm_100a does) gets an empty kernel there,
// which a B200 never runs because the sm_100a binary matches it.
#if defined(__CUDA_ARCH_FEAT_SM100_ALL) || !defined(__CUDA_ARCH__)
  using C = AttnConfig<T, D, BN, NQ, STAGES, PAIR, CORR, FOUR>;
  static_assert(!(CORR && PERSIST), "the correction warpgroup runs the classic schedule");
  constexpr int G = C::CTAS;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_s = ptx::smem_u32(smem_raw);
  const uint32_t sbase = (raw_s + 1023u) & ~1023u;
  uint8_t* sgen = smem_raw + (sbase - raw_s);
  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  // A pair is a cluster of two consecutive CTAs; every shared-memory offset
  // below is the same in both (same kernel, same dynamic shared memory).
  const int rank = PAIR ? static_cast<int>(ptx::cluster_ctarank()) : 0;
  const WorkTile wt = work_tile_of(blockIdx.x, C::BM, G, rank, p);

  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sgen + C::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sgen + C::OFF_MISC + 4);

  if (threadIdx.x == 0) {
    auto bar = [&](int i) { return sbase + C::OFF_BAR + 8u * i; };
    // Load barriers of the even CTA of a pair also take the relay's arrival
    // for the peer's half.
    const uint32_t loads = (PAIR && rank == 0) ? 2u : 1u;
    for (int i = 0; i < C::NQ; ++i) ptx::mbar_init(bar(C::BAR_Q + i), loads);
    for (int s = 0; s < C::STAGES; ++s) {
      ptx::mbar_init(bar(C::BAR_KV_FULL + s), loads);
      ptx::mbar_init(bar(C::BAR_KV_EMPTY + s), C::NUM_ISSUERS);
    }
    for (int i = 0; i < C::NQ * C::NSBUF; ++i) ptx::mbar_init(bar(C::BAR_S_FULL + i), 1);
    for (int i = 0; i < C::NQ * C::NSBUF * C::PHALVES; ++i)
      ptx::mbar_init(bar(C::BAR_P_READY + i), i % C::PHALVES == 0 ? C::P0_ARRIVALS : C::P_ARRIVALS);
    if constexpr (C::CORR) {
      for (int i = 0; i < C::NQ * C::NSBUF + C::NQ; ++i)
        ptx::mbar_init(bar(C::BAR_CORR + i), C::WARPS_PER_TILE);
    }
    for (int i = 0; i < C::NQ; ++i) {
      ptx::mbar_init(bar(C::BAR_O_DONE + i), 1);
      ptx::mbar_init(bar(C::BAR_O_FINAL + i), 1);
      ptx::mbar_init(bar(C::BAR_Q_FREE + i), 1);
    }
    ptx::mbar_init(bar(C::BAR_DRAIN), C::NUM_ISSUERS);
    *abort_flag = 0;
    *reinterpret_cast<volatile int*>(sgen + C::OFF_MISC + 16) = 0;  // O staging lock
    ptx::fence_mbar_init();
  }
  if (warp == C::LOAD_WARP && lane == 0) {
    ptx::tma_prefetch_desc(&tmQ);
    ptx::tma_prefetch_desc(&tmK);
    ptx::tma_prefetch_desc(&tmV);
    ptx::tma_prefetch_desc(&tmO);
  }
  if (warp == C::MMA_WARP) {
    ptx::tmem_alloc<G>(ptx::smem_u32(tmem_slot), C::TMEM_ALLOC);
    ptx::tmem_relinquish<G>();
  }
  ptx::tc_fence_before();
  __syncthreads();
  // Pairs: the peer's barriers are initialised before anything arrives on them.
  if constexpr (PAIR) ptx::cluster_sync();
  ptx::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  const WaitCtx w{abort_flag, p.status, p.timeout_ns};
  Prof<PROFILE> prof{(PROFILE && static_cast<int>(blockIdx.x) == p.prof_cta) ? p.prof : nullptr};

  if constexpr (PERSIST) {
    static_assert(C::PERSIST_OK, "the persistent schedule needs one S buffer per Q tile, no pair");
    {
      if (warp < C::NUM_SOFTMAX_WARPS) {
        if constexpr (C::NQ == 2) ptx::setmaxnreg_inc<C::REG_SOFTMAX>();
        softmax_role_persistent<T, C, PROFILE>(warp / 4, tmem, sbase, sgen, &tmO, p, w, prof);
      } else {
        if constexpr (C::NQ == 2) ptx::setmaxnreg_dec<C::REG_OTHER>();
        if (warp == C::LOAD_WARP) {
          if (lane == 0) load_role_persistent<C, PROFILE>(&tmQ, &tmK, &tmV, sbase, p, w, prof);
        } else if (warp == C::MMA_WARP) {
          if (lane == 0) mma_role_persistent<C, PROFILE>(tmem, sbase, p, w, prof);
        } else if (warp == C::OBSERVER_WARP) {
          if constexpr (PROFILE) {
            // Stamps the completions of the first P Vs of tile 0 (the CTA's
            // first item; its O_FINAL ends the watch).
            if (lane == 0 && prof.buf != nullptr) {
              ItemCursor c0;
              c0.init(blockIdx.x, p);
              Item first;
              if (c0.next(first, p, C::BM))
                observer_role<C>(sbase, first.n < kProfSlots ? first.n : kProfSlots, w, prof);
            }
          }
        }
        __syncwarp();
      }
    }
  } else if (warp < C::NUM_SOFTMAX_WARPS) {
    if constexpr (C::NQ == 2) ptx::setmaxnreg_inc<C::REG_SOFTMAX>();
    if constexpr (C::W8)
      softmax_role16<T, C, PROFILE>(warp / C::WARPS_PER_TILE, tmem, sbase, sgen, &tmO, wt, p, w,
                                    prof);
    else
      softmax_role<T, C, PROFILE>(warp / 4, tmem, sbase, sgen, &tmO, wt, p, w, prof);
  } else if (C::CORR && warp >= C::CORR_WARP0) {
    if constexpr (C::CORR) {
      ptx::setmaxnreg_dec<C::REG_CORR>();
      correction_role<T, C>(tmem, sbase, sgen, &tmO, wt, w);
    }
  } else {
    if constexpr (C::NQ == 2) ptx::setmaxnreg_dec<C::REG_OTHER>();
    if (warp == C::LOAD_WARP) {
      if (lane == 0) load_role<C, PROFILE>(&tmQ, &tmK, &tmV, sbase, wt, p, w, prof);
    } else if (warp == C::MMA_WARP) {
      if (PAIR && rank != 0) {
        if (lane == 0) relay_role<C>(sbase, wt, w);
      } else if (lane == 0) {
        mma_role<C, PROFILE>(tmem, sbase, wt, p, w, prof, 0, C::NUM_ISSUERS == 2 ? 1 : C::NQ);
      }
    } else if (C::NUM_ISSUERS == 2 && warp == C::MMA_WARP2) {
      if (lane == 0 && (!PAIR || rank == 0)) mma_role<C, PROFILE>(tmem, sbase, wt, p, w, prof, 1, 2);
    } else if (warp == C::OBSERVER_WARP) {
      if constexpr (PROFILE) {
        if (lane == 0 && prof.buf != nullptr) observer_role<C>(sbase, wt.n, w, prof);
      }
    }
    __syncwarp();
  }

  ptx::tc_fence_before();
  __syncthreads();
  // Pairs: neither CTA frees its tensor memory or exits while the even CTA's
  // MMAs or the peer's arrivals may still reach it.
  if constexpr (PAIR) ptx::cluster_sync();
  if (warp == C::MMA_WARP) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc<G>(tmem, C::TMEM_ALLOC);
  }
#endif
}

}  // namespace attnprof
