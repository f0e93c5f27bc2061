"""Per-phase cycle profiler (post-processing on the host).

Rebuilds the reference's clock64 phase profiler (attn.cu:3-38 ProfileResult /
Profile, stamps attn.cu:133-444, host averaging and table printing in
run_one_case attn.cu:1400-1494) on the phases of the B200 pipeline.  One CTA
of the profiler-enabled kernel variant (attn_fwd_profiled) writes clock64
begin/end stamps per KV iteration (first 32 iterations, one slot each):

  LoadQ    producer issues the Q TMA            -> MMA warp sees Q landed
  LoadK    producer issues K_j (slot free)      -> MMA warp sees K_j landed (in
           single one-buffer CTAs K_j lands with V_{j-1}, on one barrier, so
           this is the V_{j-1} wait and the K-wait trace phase stays empty)
  LoadV    producer issues V_j (slot free)      -> MMA warp sees V_j landed
  GEMM-QK  MMA warp issues S_0 = Q_0 K_j^T       -> softmax warp sees S_0 complete
  SOFTMAX  softmax warp sees S_0                 -> P_0 written to TMEM and signalled
  GEMM-PV  MMA warp issues O_0 += P_0 V_j        -> observer warp sees it (and the
           next S_0, committed with it) complete

(Tile 0 of the CTA; all stamps come from one SM's clock.)  SOFTMAX is also
split into its steps: S-ld (tcgen05.ld of S and its wait), max (row max and
the lazy-rescale decision), exp (exponentials, P stores issued) and P-st (wait
for the P stores to land).  Unlike the
reference's synchronous profiled kernel, the phases here overlap: a load or
GEMM phase includes the time its consumer took to look.  `period` is the
mean distance between consecutive SOFTMAX starts, i.e. cycles per KV
iteration of the whole pipeline.

    python -m attnprofile_b200.profiler [--s 4096] [--d 128] [--h 16]
           [--tiles 256x128,128x128,...] [--runs 20]
prints one markdown row per tile in the reference's table format
(the reference project's README.md:11-19:
| BM | BN | LoadQ | LoadK | LoadV | GEMM-QK | SOFTMAX | GEMM-PV |).
"""
from __future__ import annotations

import argparse

PHASES = ["LoadQ", "LoadK", "LoadV", "GEMM-QK", "SOFTMAX", "GEMM-PV"]
# Steps of SOFTMAX (same warp): S tcgen05.ld + wait, row max + rescale
# decision, exponentials with the P tcgen05.st issued, wait for the P stores.
SUBPHASES = ["S-ld", "max", "exp", "P-st"]
ALL_PHASES = PHASES + SUBPHASES
# The epilogue phase (index 10) is stamped once per CTA; its slots are steps:
# the whole epilogue, the wait for the last P V, the partial-O write and the
# count-in of a split part, the merge (split) or O normalisation (whole), and
# the TMA store issue.
EPILOGUE_STEPS = ["epilogue", "ep-waitO", "ep-partial", "ep-count", "ep-merge", "ep-store"]
# Trace phases (11-13) relating the two Q tiles of a BM = 256 CTA: SOFTMAX of
# tile 1, and the MMA issuer's window per tile (first P part observed -> the
# tile's next S issued).
TRACE_PHASES = ["SOFTMAX-t1", "MMA-t0", "MMA-t1", "P-first", "V-wait", "K-wait"]
TRACE_BASE = len(ALL_PHASES) + 1


def summarize(stamps_list) -> dict:
    """Mean cycles per phase over recorded slots and runs.

    stamps_list: iterable of int64 arrays [phases, 32, 2] (begin, end); 0 = unset."""
    import numpy as np
    sums = {p: [] for p in ALL_PHASES}
    periods = []
    for st in stamps_list:
        a = np.asarray(st, dtype=np.int64)
        for k, name in enumerate(ALL_PHASES[: a.shape[0]]):
            b, e = a[k, :, 0], a[k, :, 1]
            ok = (b != 0) & (e != 0) & (e >= b)
            if name == "LoadQ":
                ok[1:] = False
            sums[name].extend((e[ok] - b[ok]).tolist())
        sb = a[PHASES.index("SOFTMAX"), :, 0]
        sb = sb[sb != 0]
        if sb.size > 2:
            periods.extend(np.diff(sb[1:]).tolist())  # skip the first (pipeline fill)
    out = {p: (float(np.mean(v)) if v else float("nan")) for p, v in sums.items()}
    out["period"] = float(np.mean(periods)) if periods else float("nan")
    ep = {n: [] for n in EPILOGUE_STEPS}
    for st in stamps_list:
        a = np.asarray(st, dtype=np.int64)
        if a.shape[0] <= len(ALL_PHASES):
            continue
        for k, n in enumerate(EPILOGUE_STEPS):
            b, e = a[len(ALL_PHASES), k]
            if b != 0 and e != 0 and e >= b:
                ep[n].append(int(e - b))
    for n, v in ep.items():
        out[n] = float(np.mean(v)) if v else float("nan")
    tr = {n: [] for n in TRACE_PHASES}
    for st in stamps_list:
        a = np.asarray(st, dtype=np.int64)
        for k, n in enumerate(TRACE_PHASES):
            if a.shape[0] <= TRACE_BASE + k:
                continue
            b, e = a[TRACE_BASE + k, :, 0], a[TRACE_BASE + k, :, 1]
            ok = (b != 0) & (e != 0) & (e >= b)
            tr[n].extend((e[ok] - b[ok]).tolist())
    for n, v in tr.items():
        out[n] = float(np.mean(v)) if v else float("nan")
    return out


def timeline(st, first: int = 8, count: int = 4) -> str:
    """Event times of KV iterations [first, first + count) of one profiled CTA,
    in cycles from the start of tile 0's SOFTMAX of iteration `first`:
    each tile's SOFTMAX (S observed -> last P part signalled), the MMA
    issuer's window per tile, and tile 0's P V completion as observed."""
    import numpy as np
    a = np.asarray(st, dtype=np.int64)
    sm0 = PHASES.index("SOFTMAX")
    pv0 = PHASES.index("GEMM-PV")
    t0 = a[sm0, first, 0]
    ex = len(PHASES) + SUBPHASES.index("exp")
    qk = PHASES.index("GEMM-QK")
    rows = ["| j | tile | SOFTMAX | exp step | first P part | MMA window (P seen -> next S "
            "issued) | V_j wait | K_j+1 wait | S_j+1 issue | P V issue | P V done |",
            "|---|---|---|---|---|---|---|---|---|---|---|"]
    rel = lambda v: "-" if v == 0 else f"{int(v - t0)}"
    tr = lambda k, j, w: a[TRACE_BASE + k, j, w] if a.shape[0] > TRACE_BASE + k else 0
    for j in range(first, min(first + count, a.shape[1])):
        rows.append(f"| {j} | 0 | {rel(a[sm0, j, 0])} .. {rel(a[sm0, j, 1])} | "
                    f"{rel(a[ex, j, 0])} .. {rel(a[ex, j, 1])} | {rel(tr(3, j, 0))} | "
                    f"{rel(tr(1, j, 0))} .. {rel(tr(1, j, 1))} | "
                    f"{rel(tr(4, j, 0))} .. {rel(tr(4, j, 1))} | "
                    f"{rel(tr(5, j, 0))} .. {rel(tr(5, j, 1))} | "
                    f"{rel(a[qk, j + 1, 0]) if j + 1 < a.shape[1] else '-'} | "
                    f"{rel(a[pv0, j, 0])} | {rel(a[pv0, j, 1])} |")
        if tr(0, j, 0) != 0:
            rows.append(f"| {j} | 1 | {rel(tr(0, j, 0))} .. {rel(tr(0, j, 1))} | | "
                        f"{rel(tr(3, j, 1))} | {rel(tr(2, j, 0))} .. {rel(tr(2, j, 1))} | | | | | |")
    return "\n".join(rows)


def run(B=1, H=16, S=4096, D=128, BM=256, BN=128, dtype="f16", runs=20, cta=None, seed=0,
        raw=False):
    import torch
    import attnprofile_b200 as ap
    dt = torch.float16 if dtype == "f16" else torch.bfloat16
    g = torch.Generator(device="cuda").manual_seed(seed)
    Q, K, V = (torch.randn(B, H, S, D, generator=g, device="cuda").to(dt) for _ in range(3))
    n_qt = (S + BM - 1) // BM
    # a CTA from the middle of the grid (the persistent schedule's grid is
    # one CTA per resident slot, not one per unit)
    ctas = ap.query_split(B, H, S, D, BM=BM, BN=BN, dtype=0 if dtype == "f16" else 1)["ctas"]
    cta = min(n_qt * B * H, ctas) // 2 if cta is None else cta
    for _ in range(3):
        ap.attn(Q, K, V, BM=BM, BN=BN)
    stamps = []
    for _ in range(runs):
        _, st = ap.attn_profiled(Q, K, V, BM=BM, BN=BN, cta=cta)
        stamps.append(st.numpy())
    torch.cuda.synchronize()
    rc, site = ap.get_status(torch.cuda.current_device())
    if rc != 0:
        raise RuntimeError(f"device status {site:#x}")
    return stamps if raw else summarize(stamps)


def step_starts(st) -> str:
    """Cycles between consecutive SOFTMAX starts of tile 0, per step of the
    profiled CTA (its first 32 steps, across its items): a long gap marks an
    item boundary of the persistent schedule."""
    import numpy as np
    a = np.asarray(st, dtype=np.int64)
    sb = a[PHASES.index("SOFTMAX"), :, 0]
    rows = ["| step | SOFTMAX start | since previous |", "|---|---|---|"]
    for j in range(sb.shape[0]):
        if sb[j] == 0:
            continue
        d = "-" if j == 0 or sb[j - 1] == 0 else f"{int(sb[j] - sb[j - 1])}"
        rows.append(f"| {j} | {int(sb[j] - sb[0])} | {d} |")
    return "\n".join(rows)


def table_header(epilogue: bool = False) -> str:
    cols = ["BM", "BN"] + PHASES + ["period"] + SUBPHASES + TRACE_PHASES
    if epilogue:
        cols += EPILOGUE_STEPS
    return "| " + " | ".join(cols) + " |\n|" + "---|" * len(cols)


def table_row(BM, BN, r, epilogue: bool = False) -> str:
    names = PHASES + ["period"] + SUBPHASES + TRACE_PHASES + (EPILOGUE_STEPS if epilogue else [])
    vals = [f"{r[p]:.0f}" for p in names]
    return f"| {BM} | {BN} | " + " | ".join(vals) + " |"


def main(argv=None):
    ap_ = argparse.ArgumentParser()
    ap_.add_argument("--b", type=int, default=1)
    ap_.add_argument("--h", type=int, default=16)
    ap_.add_argument("--s", type=int, default=4096)
    ap_.add_argument("--d", type=int, default=128)
    ap_.add_argument("--dtype", default="f16")
    ap_.add_argument("--tiles", default="256x128,128x128,256x64,128x64,128x256,256x32,128x32")
    ap_.add_argument("--runs", type=int, default=20)
    ap_.add_argument("--timeline", type=int, default=0, metavar="N",
                     help="also print N iterations (from 8) of one run's event timeline per tile")
    ap_.add_argument("--schedule", type=int, default=0, choices=[0, 1, 2],
                     help="attn_set_schedule mode (0 automatic, 1 classic, 2 persistent)")
    ap_.add_argument("--correction", type=int, default=0, choices=[0, 1],
                     help="attn_set_correction mode (1: correction warpgroup where built)")
    ap_.add_argument("--cta", type=int, default=None, help="CTA to profile (default: middle)")
    ap_.add_argument("--steps", action="store_true",
                     help="also print the per-step SOFTMAX starts of one run (item boundaries)")
    ap_.add_argument("--epilogue", action="store_true",
                     help="add the epilogue steps (of the CTA's first item) to the table")
    a = ap_.parse_args(argv)
    import attnprofile_b200 as ap
    ap.set_schedule(a.schedule)
    ap.set_correction(a.correction)
    print(f"B={a.b} H={a.h} S={a.s} D={a.d} {a.dtype}: cycles (clock64) per phase, "
          f"mean over KV iterations 0-31 and {a.runs} runs")
    print(table_header(a.epilogue))
    for t in a.tiles.split(","):
        bm, bn = (int(x) for x in t.split("x"))
        st = run(a.b, a.h, a.s, a.d, bm, bn, a.dtype, a.runs, cta=a.cta, raw=True)
        print(table_row(bm, bn, summarize(st), a.epilogue), flush=True)
        if a.steps:
            print(f"\n{bm}x{bn} per-step SOFTMAX starts (cycles, last run):\n"
                  + step_starts(st[-1]) + "\n", flush=True)
        if a.timeline:
            print(f"\n{bm}x{bn} timeline (cycles, last run):\n" + timeline(st[-1], 8, a.timeline)
                  + "\n", flush=True)


if __name__ == "__main__":
    main()
