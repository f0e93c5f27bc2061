/*
 * attnprof.h -- C ABI of the B200 (sm_100a) attention forward engine.
 *
 * Non-causal attention O = softmax(Q K^T / sqrt(D)) V over tensors laid out
 * row-major as [B, H, rows, D] (rows = S unless stated), f16 or bf16 in and
 * out, fp32 accumulation.  All pointers are device pointers of the current
 * CUDA device unless stated.  Calls are asynchronous on the given stream
 * (NULL = legacy default stream) unless stated; the functions never
 * synchronise except where the comment says so.
 *
 * The reference (Xiebaokang/AttnProfile) exposes this path only as C++
 * templates compiled per configuration:
 *   runAttn<B,H,S,D,BM,BN,NUM_SMEM,PRODUCER_REG_DEALLOC,CONSUMER_REG_ALLOC,
 *           P_SMEM_K_TILES,KERNEL_IDX,NUM_THREADS>(fp16* Q, fp16* K,
 *           fp16* V, fp16* O)                      tuning/attn_test.cu:1665-1691
 * passed around as AttnRunner = void(*)(fp16*,fp16*,fp16*,fp16*)
 *                                                 tuning/utils.cuh:71
 * The entry points below are what a foreign-function binding of that path
 * binds: shape and tile at run time, an explicit stream, and error codes in
 * place of the reference's cudaCheck -> exit(1) (tuning/tools.cuh:14-21).
 */
#ifndef ATTNPROF_H
#define ATTNPROF_H

#ifdef __cplusplus
extern "C" {
#endif

#define ATTN_DTYPE_F16 0
#define ATTN_DTYPE_BF16 1

/* Return codes (0 = success, negative = error). */
#define ATTN_OK 0
#define ATTN_ERR_INVALID_ARG -1    /* null pointer, non-positive size, rows < S, ... */
#define ATTN_ERR_UNSUPPORTED -2    /* (dtype, D, BM, BN) combination not built      */
#define ATTN_ERR_MISALIGNED -3     /* a tensor base is not 16-byte aligned          */
#define ATTN_ERR_CUDA -4           /* CUDA runtime error (no device, launch error)  */
#define ATTN_ERR_TENSOR_MAP -5     /* cuTensorMapEncodeTiled rejected the layout    */
#define ATTN_ERR_DEVICE_TIMEOUT -6 /* a bounded in-kernel wait expired              */
#define ATTN_ERR_RESOURCE -7       /* shared memory / TMEM request over the limit   */
#define ATTN_ERR_SHARD -8          /* multi-GPU partition error                     */
#define ATTN_ERR_SCRATCH_LIMIT -9  /* attn_fwd_noalloc: scratch over its fixed size  */

/*
 * attn_fwd -- one attention forward over contiguous [B, H, S, D] tensors.
 * BM in {128, 256} query rows per CTA; BN in {32, 64, 96, 128, 256} keys per
 * KV tile (BM = 256 with BN = 256 does not fit tensor memory: UNSUPPORTED).
 * D in {64, 128}.  BM = 512 with BN = 128 at D = 128: a cluster of two
 * 256-row CTAs sharing each K/V tile through cta_group::2 MMAs (no key
 * split).  Asynchronous; returns launch errors only
 * (device-side timeouts are reported by attn_get_status).
 * Replaces: runAttn<...>(Q, K, V, O)            tuning/attn_test.cu:1665-1691
 *           (BM, BN as run-time values instead of template parameters).
 */
int attn_fwd(const void* Q, const void* K, const void* V, void* O, int B, int H, int S, int D,
             int dtype, int BM, int BN, void* stream);

/*
 * attn_fwd_padded -- the reference's padded layout: Q and O are
 * [B, H, SQO, D], K and V are [B, H, SKV, D], with SQO >= S and SKV >= S
 * (the reference allocates SQO = ceil(S/BM)*BM, SKV = ceil(S/BN)*BN,
 * tuning/attn_test.cu:1590-1595, tuning/utils.cuh:86-87).  Rows >= S are
 * neither read nor written.
 * Replaces: runAttnWS2StageBaselineKernel / ...SmemP... / ...ForNSmemP...
 *           launchers                         tuning/attn_test.cu:1583-1663
 */
int attn_fwd_padded(const void* Q, const void* K, const void* V, void* O, int B, int H, int S,
                    int D, int SQO, int SKV, int dtype, int BM, int BN, void* stream);

/*
 * attn_fwd_profiled -- attn_fwd with the per-phase cycle profiler compiled in
 * (f16 and bf16).  CTA number profile_cta (CTAs are numbered in launch
 * order; CTA 0 runs the first BM query rows of head 0 over all keys) writes
 * clock64 begin/end stamps for the phases LoadQ, LoadK, LoadV, GEMM-QK,
 * SOFTMAX, GEMM-PV (then the SOFTMAX steps S-load, max, exp, P-store) of its
 * first 32 KV iterations, and for its epilogue (phase 10; slots 0-5: the
 * whole epilogue, the wait for the last P V, partial-O write and count-in of
 * a split part, merge or O normalisation, O store issue), and trace phases
 * relating the two Q tiles of BM = 256 (11 SOFTMAX of the second Q tile,
 * 12 / 13 the MMA issuer's window per Q tile: first P part observed -> next S
 * issued, 14 first P part signalled by tile 0 / tile 1, 15 / 16 the issuer's
 * waits for V_j / K_{j+1}) into dev_profile_buf, laid out as u64 [17][32][2]
 * (see attn_profile_layout).
 * The caller zeroes the buffer before the launch; unstamped slots stay 0.
 * Replaces: the clock64 profiler of attn.cu (ProfileResult attn.cu:5-22,
 *           stamps attn.cu:133-444, run_one_case attn.cu:1400-1494).
 */
int attn_fwd_profiled(const void* Q, const void* K, const void* V, void* O, int B, int H, int S,
                      int D, int dtype, int BM, int BN, void* stream,
                      unsigned long long* dev_profile_buf, int profile_cta);

/* Profile buffer geometry: *phases = 17, *slots = 32 (u64 pairs). */
int attn_profile_layout(int* phases, int* slots);

/*
 * attn_fwd_sharded -- (batch, head) sharding over n_dev GPUs of this process,
 * no collective.  Units u = b*H + h are split as [g*U/n, (g+1)*U/n) for
 * GPU g (see attn_shard_range); Q[g], K[g], V[g], O[g] are device pointers on
 * devices[g] holding that GPU's units contiguously ([units_g, S, D]).
 * Launches on every device, then synchronises them all (this call blocks).
 * ms_per_device (optional, host array of n_dev) receives each device's
 * kernel time in milliseconds from CUDA events.
 * No counterpart in the reference (single-GPU only); this is the (b,h)
 * partition the benchmark configurations C4/C5 run on 1/2/4/8 GPUs.
 */
int attn_fwd_sharded(int n_dev, const int* devices, const void* const* Q, const void* const* K,
                     const void* const* V, void* const* O, int B, int H, int S, int D, int dtype,
                     int BM, int BN, float* ms_per_device);

/* The partition rule used by attn_fwd_sharded: units [*begin, *end) of GPU g. */
int attn_shard_range(int units, int n_dev, int g, int* begin, int* end);

/*
 * attn_get_status -- synchronise `device` and read the device status word
 * that bounded in-kernel waits set on expiry.  Returns ATTN_OK or
 * ATTN_ERR_DEVICE_TIMEOUT (*site, if non-NULL, receives the raw code);
 * reset != 0 clears the word.  Blocking.
 * Replaces: the reference's unbounded mbarrier spin (tuning/tools.cuh:870-885),
 * which has no error path.
 */
int attn_get_status(int device, int reset, int* site);

/* Bounded-wait limit for kernels launched after this call (default 2 s). */
void attn_set_timeout_ns(unsigned long long ns);

/*
 * attn_query_config -- launch geometry of a (D, BM, BN, dtype) variant:
 * threads per CTA, dynamic shared memory bytes, TMEM columns allocated and
 * K/V ring depth.  Returns ATTN_ERR_UNSUPPORTED for combinations not built.
 * The D = 64 tiles with two S buffers per Q tile (BM = 256, BN <= 96) report
 * their eight-warp kernel (640 threads); their launches that split units
 * along the keys, and the correction-warpgroup kernel (512), use other
 * thread counts with the same shared memory layout.
 * Replaces: the reference's resource model (tuning/solver.py:14-95), which
 * the tuning harness uses to filter configurations.
 */
int attn_query_config(int D, int BM, int BN, int dtype, int* num_threads, int* smem_bytes,
                      int* tmem_cols, int* stages);

/*
 * Key split of the last wave.  A launch has U = B*H*ceil(S/BM) units (BM
 * query rows of one head); a B200 runs one unit per SM at a time, so when U
 * is not a multiple of the SM count the last wave leaves SMs idle (1x16x4096
 * at BM=256: 256 units on 148 SMs).  Each unit of that last wave can instead
 * run as k CTAs over disjoint key ranges; every part writes its normalised
 * partial O and (row max, row sum) to a stream-ordered workspace, and the
 * part that finishes last merges them (fixed order: the result does not
 * depend on arrival order).  Default: automatic (a cost model picks k).
 *
 * attn_set_split -- mode 0 automatic, 1 never split, 2..4 force k-way splits
 *   of the last wave (of the last full wave when U is a multiple of the slot
 *   count) for kernels launched after this call.
 * attn_plan_split -- the planner alone (host only, no GPU): U units,
 *   num_kv_tiles = ceil(S/BN), `slots` resident CTAs per wave.
 * attn_query_split -- the plan and workspace size for a problem on the
 *   current device (needs a GPU).
 * No counterpart in the reference, whose grid is one CTA per unit
 * (tuning/attn_test.cu:1583-1663).
 */
int attn_set_split(int mode);

/*
 * Schedule of the launch (two-tile variants with one S buffer per tile:
 * BM = 256 with BN = 96 or 128 at D = 128, BN = 128 at D = 64).
 *   classic     one CTA per unit of BM query rows (or per key range of a
 *               unit of the last wave, attn_set_split); a grid of units.
 *   persistent  one resident CTA per SM slot, each running an equal share of
 *               the launch's (unit, key tile) steps in order, crossing unit
 *               boundaries: the next unit's Q and first S overlap the
 *               current unit's end, and no wave is left partly empty.  A
 *               unit cut between two CTAs is finished by the CTA holding its
 *               first key tile, which adds the other pieces' partial results
 *               (written by the next CTAs first) in key order.  Launched
 *               cooperatively (all CTAs resident at once).
 * attn_set_schedule -- mode 0 automatic, 1 classic, 2 persistent whenever
 *   the variant has it (and the split mode is automatic).  The automatic
 *   mode runs the classic schedule: on a B200 the persistent one measured
 *   within -3 .. +2 % of it on the benchmark shapes and slower on shapes of
 *   few long units, so it is opt-in.
 * attn_plan_schedule -- the host planner alone (no GPU): for U units of
 *   num_kv_tiles key tiles on `slots` resident CTAs, whether the automatic
 *   mode picks the persistent schedule (it does not), the persistent grid,
 *   the most pieces a unit is cut into, and both schedules' modelled costs
 *   (in key-tile periods of one CTA).
 * No counterpart in the reference, whose grid is one CTA per unit
 * (tuning/attn_test.cu:1583-1663).
 */
int attn_set_schedule(int mode);

/*
 * attn_set_correction -- mode 1 runs launches made after this call with a
 * correction warpgroup where the variant has one (BM = 256 with BN = 128,
 * and BM = 256, BN = 96 at D = 64): a fourth warpgroup owns the lazy
 * rescale of O in tensor memory (the softmax warps hand it each step's
 * factors; it lets P V add to O only after rescaling), the final division by
 * the row sums and the TMA store of O.  Such launches take the classic
 * schedule without key split.  Mode 0 (default): the softmax warpgroups do
 * that work themselves.  Same results either way.
 * No counterpart in the reference, which rescales O eagerly inside its
 * softmax consumer (tuning/attn_test.cu:305-321).
 */
int attn_set_correction(int mode);
int attn_plan_schedule(long long units, int num_kv_tiles, long long slots, int* persistent,
                       long long* ctas, int* pieces, double* persistent_cost,
                       double* classic_cost);
int attn_plan_split(long long units, int num_kv_tiles, long long slots, int mode, int* split,
                    long long* whole_units, long long* ctas);
int attn_query_split(int B, int H, int S, int D, int dtype, int BM, int BN, int* split,
                     long long* whole_units, long long* ctas, unsigned long long* workspace_bytes);

/*
 * attn_fwd_noalloc -- attn_fwd for callers that must not allocate GPU
 * memory when they launch: a serving process that reserved its whole memory
 * budget at start-up and hands its kernels pre-sized buffers, a custom
 * allocator (or code it calls back) that must not re-enter the CUDA
 * allocator, a latency-bound loop that cannot take the device-wide stall of
 * cudaMalloc / cudaFree.  Arguments and results are those of attn_fwd.  When
 * the launch's plan splits units along the keys (attn_set_split /
 * attn_query_split) it needs scratch for the partial results; attn_fwd takes
 * that from a stream-ordered pool, this entry point from a fixed array of
 * ATTN_NOALLOC_SCRATCH_BYTES (32 MiB) inside the library.  It calls no
 * cudaMalloc / cudaFree / pool allocation, and encodes its tensor maps per
 * call instead of caching them.
 *   - Footprint: the array belongs to the library's device module, so each
 *     GPU holds the 32 MiB from the moment that module is loaded there --
 *     with lazy module loading (the CUDA default) at the first
 *     attn_fwd_noalloc call on the GPU, with CUDA_MODULE_LOADING=EAGER when
 *     the process creates its context on the GPU, even if this entry point
 *     is never called -- until the process exits.
 *   - A plan needing more scratch returns ATTN_ERR_SCRATCH_LIMIT and launches
 *     nothing (attn_fwd runs any size).
 *   - Set-up: the first call on each device (any shape) looks up the array's
 *     device address (cudaGetSymbolAddress) with that device current; make
 *     that first call before any stream capture.
 *   - All calls share the one array, which keeps the last call's contents.
 *     Calls that may overlap on the GPU (different streams, or different
 *     host threads) race on it; order them on one stream.  Each call clears
 *     the counters it needs at zero before its kernel.
 * No counterpart in the reference: its launchers allocate nothing beyond
 * the caller's tensors (tuning/attn_test.cu:1583-1663) and have no key split.
 */
#define ATTN_NOALLOC_SCRATCH_BYTES (32u << 20)
int attn_fwd_noalloc(const void* Q, const void* K, const void* V, void* O, int B, int H, int S,
                     int D, int dtype, int BM, int BN, void* stream);

/* Human-readable text for a return code.  Never NULL. */
const char* attn_error_string(int code);

/*
 * attn_debug_fault -- test hook for the failure path: mode 1 makes the next
 * launches' producer warp load Q but never K/V, so every consumer's bounded
 * wait expires and the kernel returns with ATTN_ERR_DEVICE_TIMEOUT in the
 * status word (no fault, no trap, no hang).  mode 0 restores normal runs.
 */
int attn_debug_fault(int mode);

/* ABI version (major*100 + minor). */
int attn_version(void);

#ifdef __cplusplus
}
#endif

#endif /* ATTNPROF_H */
