"""Nsight Compute sweep of the attention kernel over shapes and (BM, BN) tiles.

The B200 counterpart of the reference's run_attn_ws_sweep.py
(run_attn_ws_sweep.py:12-16 metrics, :157-209 loop and CSV): for every
(B, H, S, D) x (BM, BN) it runs one small child process through the C ABI,
first without ncu (it must exit 0), then under

    ncu --metrics <METRICS> --clock-control none -k regex:attn_fwd_kernel -s 2 -c 1

and appends one CSV row: the reference's fields (B, H, S, D, time [ms],
tflops, tc_utilization [% of peak sustained active]) plus BM, BN and the
sm_100 counters that explain the kernel's bound (exponential unit, issue
slots, DRAM bytes, tensor-core shared-memory reads).  The tiles need no
recompilation: the C ABI dispatches them at run time.

    python -m attnprofile_b200.ncu_sweep --seq-lens 4096 --head-dims 64,128 \\
        --tiles 256x128,256x64,128x128 --out profiles/ncu_sweep.csv
    python -m attnprofile_b200.ncu_sweep --shapes 1x32x8192x128:bf16,1x8x32768x128 \\
        --tiles 256x128 --out shards.csv        # explicit shapes, f16 unless :bf16

Run it on one GPU; every capture is one launch of a small problem (a few
passes of ~0.1 ms kernels).
"""
from __future__ import annotations

import argparse
import csv
import io
import itertools
import math
import os
import subprocess
import sys
from pathlib import Path

METRICS = {
    "gpu__time_duration.sum": "time",
    "sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_active": "tc_utilization",
    "sm__inst_executed_pipe_xu.avg.pct_of_peak_sustained_active": "xu_utilization",
    "smsp__issue_active.avg.pct_of_peak_sustained_active": "issue_active",
    "dram__bytes_read.sum": "dram_read_bytes",
    "dram__bytes_write.sum": "dram_write_bytes",
    "l1tex__data_pipe_tc_wavefronts_mem_shared.sum.pct_of_peak_sustained_elapsed": "tc_smem_pct",
}
CSV_FIELDS = ["B", "H", "S", "D", "dtype", "BM", "BN", "time", "tflops", "tc_utilization",
              "xu_utilization", "issue_active", "dram_read_bytes", "dram_write_bytes",
              "tc_smem_pct"]
UNIT_SCALE = {"ns": 1e-6, "nsecond": 1e-6, "us": 1e-3, "usecond": 1e-3, "ms": 1.0, "msecond": 1.0,
              "s": 1e3, "second": 1e3, "byte": 1.0, "kbyte": 1e3, "mbyte": 1e6, "gbyte": 1e9, "%": 1.0}


def child(B: int, H: int, S: int, D: int, BM: int, BN: int, bf16: int = 0) -> int:
    """Three launches (two warm-up, the third captured) of one tile."""
    import torch

    import attnprofile_b200 as ap
    g = torch.Generator(device="cuda").manual_seed(B * 1000 + H * 10 + D)
    dt = torch.bfloat16 if bf16 else torch.float16
    Q, K, V = (torch.randn(B, H, S, D, generator=g, device="cuda").to(dt) for _ in range(3))
    O = torch.empty_like(Q)
    for _ in range(3):
        ap.attn(Q, K, V, O, BM=BM, BN=BN)
    torch.cuda.synchronize()
    rc, site = ap.get_status(torch.cuda.current_device())
    return 0 if rc == 0 else 1


def parse_ncu_csv(text: str) -> dict:
    """Metric name -> value in the CSV field's base unit (ms for time, bytes, %)."""
    rows = list(csv.reader(io.StringIO(text[text.find('"ID"'):] if '"ID"' in text else text)))
    if not rows:
        return {}
    hdr = rows[0]
    idx = {k: hdr.index(k) for k in ("Metric Name", "Metric Unit", "Metric Value") if k in hdr}
    out = {}
    for r in rows[1:]:
        if len(r) != len(hdr):
            continue
        name = r[idx["Metric Name"]]
        if name not in METRICS:
            continue
        unit = r[idx["Metric Unit"]].strip().lower()
        try:
            val = float(r[idx["Metric Value"]].replace(",", ""))
        except ValueError:
            val = math.nan
        out[METRICS[name]] = val * UNIT_SCALE.get(unit, 1.0)
    return out


def profile(ncu: str, shape, tile, timeout: float) -> dict | None:
    B, H, S, D = shape[:4]
    dtype = shape[4] if len(shape) > 4 else "f16"
    BM, BN = tile
    cmd = [sys.executable, "-m", "attnprofile_b200.ncu_sweep", "--child",
           *map(str, (B, H, S, D, BM, BN, 1 if dtype == "bf16" else 0))]
    env = dict(os.environ)
    plain = subprocess.run(cmd, capture_output=True, text=True, timeout=timeout, env=env)
    if plain.returncode != 0:
        return None  # not run under ncu: the plain run must succeed first
    prof = subprocess.run([ncu, "--metrics", ",".join(METRICS), "--clock-control", "none",
                           "-k", "regex:attn_fwd_kernel", "-s", "2", "-c", "1", "--csv", *cmd],
                          capture_output=True, text=True, timeout=timeout, env=env)
    if prof.returncode != 0:
        return None
    m = parse_ncu_csv(prof.stdout)
    if "time" not in m:
        return None
    row = {"B": B, "H": H, "S": S, "D": D, "dtype": dtype, "BM": BM, "BN": BN}
    row.update({k: m.get(k, math.nan) for k in CSV_FIELDS if k in METRICS.values()})
    row["tflops"] = 4.0 * B * H * S * S * D / (m["time"] * 1e-3) / 1e12
    return row


def ints(v: str):
    return [int(x) for x in v.replace(" ", ",").split(",") if x.strip()]


def parse_shapes(v: str):
    """'1x32x8192x128:bf16,1x8x32768x128' -> [(1, 32, 8192, 128, 'bf16'), (1, 8, 32768, 128, 'f16')]."""
    out = []
    for item in v.split(","):
        if not item.strip():
            continue
        dims, _, dt = item.strip().partition(":")
        B, H, S, D = (int(x) for x in dims.split("x"))
        if (dt or "f16") not in ("f16", "bf16"):
            raise ValueError(f"dtype must be f16 or bf16, got {dt!r}")
        out.append((B, H, S, D, dt or "f16"))
    return out


def main(argv=None) -> int:
    ap_ = argparse.ArgumentParser()
    ap_.add_argument("--child", nargs=7, type=int, metavar=("B", "H", "S", "D", "BM", "BN", "BF16"))
    ap_.add_argument("--shapes", default=None,
                     help="explicit shapes BxHxSxD[:bf16],... (instead of the product of the lists)")
    ap_.add_argument("--batch-sizes", default="1")
    ap_.add_argument("--num-heads", default="16")
    ap_.add_argument("--seq-lens", default="4096")
    ap_.add_argument("--head-dims", default="128")
    ap_.add_argument("--tiles", default="256x128,256x96,256x64,256x32,128x128,128x64,128x256")
    ap_.add_argument("--out", default="ncu_sweep.csv")
    ap_.add_argument("--ncu", default="ncu")
    ap_.add_argument("--timeout", type=float, default=300.0)
    a = ap_.parse_args(argv)
    if a.child:
        return child(*a.child)
    tiles = [tuple(int(x) for x in t.split("x")) for t in a.tiles.split(",")]
    if a.shapes:
        shapes = parse_shapes(a.shapes)
    else:
        shapes = list(itertools.product(ints(a.batch_sizes), ints(a.num_heads), ints(a.seq_lens),
                                        ints(a.head_dims)))
    out = Path(a.out)
    with out.open("w", newline="") as f:
        csv.DictWriter(f, fieldnames=CSV_FIELDS).writeheader()
    for shape in shapes:
        for tile in tiles:
            row = profile(a.ncu, shape, tile, a.timeout)
            if row is None:
                print(f"{shape} {tile}: not profiled (plain run or ncu failed)", flush=True)
                continue
            with out.open("a", newline="") as f:
                csv.DictWriter(f, fieldnames=CSV_FIELDS).writerow(
                    {k: (f"{v:.4g}" if isinstance(v, float) else v) for k, v in row.items()})
            print(", ".join(f"{k}={row[k]:.4g}" if isinstance(row[k], float) else f"{k}={row[k]}"
                            for k in CSV_FIELDS), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
