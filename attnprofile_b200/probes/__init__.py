"""Phase-isolation probes (phase_probes.cu): the TMA K/V stream, the MMA
issue sequence and the softmax step of one KV iteration, each run alone on
every SM, to read the kernel's per-phase profile against.

    python -m attnprofile_b200.probes [tma|mma|softmax|all]

build() compiles the probe binary in-tree for sm_100a; run() builds it if
needed and returns its report (one line per probe).
"""
from __future__ import annotations

import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
SRC = HERE / "phase_probes.cu"
BIN = HERE / "phase_probes"
DEPS = [SRC, HERE.parent / "csrc" / "ptx.cuh", HERE.parent / "csrc" / "attn_kernel.cuh"]


def build(force: bool = False) -> Path:
    if not force and BIN.exists() and BIN.stat().st_mtime >= max(p.stat().st_mtime for p in DEPS):
        return BIN
    cmd = ["nvcc", "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17", "-lineinfo",
           "-I", str(HERE.parent.parent / "include"), "-o", str(BIN), str(SRC)]
    subprocess.run(cmd, check=True)
    return BIN


def run(which: str = "all", timeout: float = 300.0) -> str:
    build()
    out = subprocess.run([str(BIN), which], capture_output=True, text=True, timeout=timeout)
    if out.returncode != 0:
        raise RuntimeError(f"phase_probes {which} failed ({out.returncode}): {out.stdout}{out.stderr}")
    return out.stdout


def main(argv=None) -> int:
    argv = sys.argv[1:] if argv is None else argv
    print(run(argv[0] if argv else "all"), end="")
    return 0
