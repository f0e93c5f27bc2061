"""B200 resource model for the tuning harness's BM/BN sweep.

Same interface as the reference's tuning/solver.py (solve / solve_reuse,
tuning/solver.py:376-411, and the keys its callers read: BM, BN, NumSmem,
NumSmemP, RepeatN, SmemSize, RegSize, EstimatedRegsPerThread), so
tuning/benchmark_run_attn.py picks it up unchanged through
`from solver import solve` when this directory comes first on sys.path.

The constraints are those of the sm_100a kernel (attnprofile_b200/csrc/
attn_kernel.cuh, AttnConfig) instead of the Hopper wgmma/register model of the
reference (tuning/solver.py:14-132):

  * BM in {128, 256}: one or two 128-row Q tiles per CTA (MMA M = 128);
    RepeatN = BM / 128 (KernelIdx 1/2 -> 128, 3 -> 256, as the harness's
    get_configs expects, tuning/benchmark_run_attn.py:76-84);
  * BN a multiple of 32 in [32, 256] (32-column softmax chunks, TMA box <= 256);
  * tensor memory: NQ * NSBUF * BN + NQ * HD <= 512 columns, NSBUF = 2 when
    one Q tile and the doubled S buffer fit, else 1;
  * shared memory: Q tiles + STAGES K/V slots + barriers + alignment slack
    <= SmemLimit, with STAGES the ring depth the library ships for the tile
    (lib_stages, the mirror of auto_stages in csrc/attn_host.cuh: the deepest
    ring of at most 8 slots that fits; NumSmem does not change it, as in the
    driver's runAttn);
  * registers are not modelled (fixed split per variant): every register
    field is reported as 240 so the harness keeps one consumer-register
    setting, and each solution says so with "RegsModelled": False.
"""
from __future__ import annotations

TMEM_COLS = 512
MMA_M_B200 = 128


def tmem_columns(BM: int, BN: int, HD: int) -> int:
    nq = BM // MMA_M_B200
    nsbuf = 2 if nq * (2 * BN + HD) <= TMEM_COLS else 1
    return nq * nsbuf * BN + nq * HD


def smem_bytes(BM: int, BN: int, HD: int, stages: int) -> int:
    """Dynamic shared memory of the kernel variant (mirrors AttnConfig)."""
    nq = BM // MMA_M_B200
    nsbuf = 2 if nq * (2 * BN + HD) <= TMEM_COLS else 1
    exp_bound = nq == 2 and HD == 64 and nq * (2 * BN + HD) <= TMEM_COLS
    phalves = 2 if (BN >= 64 and not exp_bound) else 1
    stage = 128 * HD * 2 if (nq == 2 and nsbuf == 1) else 0  # O staging (persistent tiles)
    off_bar = nq * 128 * HD * 2 + stages * BN * HD * 2 + stage
    num_bars = nq + 2 * stages + nq * nsbuf + nq * nsbuf * phalves + 2 * nq + 1 + nq
    off_misc = off_bar + ((num_bars * 8 + 15) // 16) * 16
    return off_misc + 32 + 1024


def lib_stages(BM: int, BN: int, HD: int, cap: int = 8) -> int:
    """K/V ring depth of the library's variant (mirrors auto_stages in
    csrc/attn_host.cuh): the deepest ring of at most `cap` slots that fits one
    CTA's shared memory, or half the SM's for the variants built for two CTAs
    per SM (one Q tile, BN <= 64).  0 if not even two slots fit."""
    nq = BM // MMA_M_B200
    limit = 233472 // 2 - 1024 if (nq == 1 and BN <= 64) else 232_448
    nsbuf = 2 if nq * (2 * BN + HD) <= TMEM_COLS else 1
    exp_bound = nq == 2 and HD == 64 and nq * (2 * BN + HD) <= TMEM_COLS
    phalves = 2 if (BN >= 64 and not exp_bound) else 1
    bars2 = nq + 2 * 2 + nq * nsbuf + nq * nsbuf * phalves + 2 * nq + 1 + nq
    off_kv = nq * 128 * HD * 2
    stage = 128 * HD * 2 if (nq == 2 and nsbuf == 1) else 0
    best = 0
    for s in range(2, cap + 1):
        bars = ((bars2 + 2 * (s - 2)) * 8 + 15) // 16 * 16
        if off_kv + s * BN * HD * 2 + stage + max(bars, 256) + 1024 + 32 <= limit:
            best = s
    return best


def _solve(HD=64, NumSmem=2, MMA_M=64, MMA_K=16, NumConsumer=2, ElementWidth=2,
           SmemLimit=232_448, KernelIdx=2, ConsumerRegLimit=240):
    if HD not in (64, 128) or ElementWidth != 2:
        return []
    bms = [256] if KernelIdx == 3 else [128]
    solutions = []
    for BM in bms:
        for BN in range(32, 257, 32):
            if tmem_columns(BM, BN, HD) > TMEM_COLS:
                continue
            stages = lib_stages(BM, BN, HD)
            if stages < 2:
                continue
            size = smem_bytes(BM, BN, HD, stages)
            if size > SmemLimit:
                continue
            regs = 240
            solutions.append({
                "BM": BM,
                "BN": BN,
                "NumSmem": NumSmem,
                # P lives in tensor memory on B200; the harness only needs 0
                # for kernel 1 and a nonzero multiple of 4 for kernels 2/3.
                "NumSmemP": 0 if KernelIdx == 1 else 4,
                "RepeatN": BM // MMA_M_B200,
                "SmemSize": size,
                "RegSize": regs * (BM // MMA_M_B200) * 128 * 4,
                "TmemCols": tmem_columns(BM, BN, HD),
                "EstimatedRegsPerThread": regs,
                "ConservativeRegsPerThread": regs,
                "CombinedRegs": regs,
                "QKStageRegs": regs,
                "PVStageRegs": regs,
                "RegsModelled": False,
                "Stages": stages,
            })
    return solutions


def solve(HD: int = 64, NumSmem: int = 2, MMA_M: int = 64, MMA_K: int = 16,
          NumConsumer: int = 2, ElementWidth: int = 2, SmemLimit: int = 232_448,
          KernelIdx: int = 2, ConsumerRegLimit: int = 240):
    """Feasible (BM, BN) tiles of the B200 kernel for head dim HD."""
    return _solve(HD, NumSmem, MMA_M, MMA_K, NumConsumer, ElementWidth, SmemLimit, KernelIdx,
                  ConsumerRegLimit)


def solve_reuse(HD: int = 64, NumSmem: int = 2, MMA_M: int = 64, MMA_K: int = 16,
                NumConsumer: int = 2, ElementWidth: int = 2, SmemLimit: int = 232_448,
                KernelIdx: int = 2, ConsumerRegLimit: int = 240):
    """Same as solve(): the B200 model has no separate register-reuse variant."""
    return solve(HD, NumSmem, MMA_M, MMA_K, NumConsumer, ElementWidth, SmemLimit, KernelIdx,
                 ConsumerRegLimit)


if __name__ == "__main__":
    for hd in (64, 128):
        for k in (1, 3):
            for s in solve(HD=hd, NumSmem=2, KernelIdx=k):
                print(hd, k, s["BM"], s["BN"], s["SmemSize"], s["TmemCols"])
