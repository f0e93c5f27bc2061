"""Regenerate the golden fixtures from the reference's own CPU oracle.

Runs oracle/_ref/ref_attn (the reference's verify_attn, tuning/utils.cuh:73-244,
compiled from the reference sources by oracle/Makefile with host stand-ins for
the CUDA runtime) and stores, per fixture, the inputs it drew from
std::mt19937(42) and the output hORef it computed, with the reference's
padding rows removed:

    q, k, v, o_ref : uint16 bit patterns of fp16, shape [B, H, S, D]
    meta           : int32 [B, H, S, D, BM, BN]   (BN = the oracle's key tile)

Usage:  python tests/golden/gen_golden.py      (needs the reference checkout)
"""
from __future__ import annotations

import subprocess
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent


def main() -> int:
    subprocess.run(["make", "-s", "-C", str(ROOT / "oracle")], check=True)
    exe = ROOT / "oracle" / "_ref" / "ref_attn"
    if not exe.exists():
        print("oracle/_ref/ref_attn missing (reference sources absent?)", file=sys.stderr)
        return 1
    with tempfile.TemporaryDirectory() as td:
        subprocess.run([str(exe), "golden", td], check=True)
        for f in sorted(Path(td).glob("golden_*.bin")):
            raw = f.read_bytes()
            hdr = np.frombuffer(raw[:32], dtype=np.int32)
            B, H, S, D, BM, BN, SQO, SKV = (int(x) for x in hdr)
            off = 32
            def take(rows):
                nonlocal off
                n = B * H * rows * D
                a = np.frombuffer(raw[off:off + 2 * n], dtype=np.uint16).reshape(B, H, rows, D)
                off += 2 * n
                return a
            q, k, v, o = take(SQO), take(SKV), take(SKV), take(SQO)
            assert off == len(raw)
            name = f.stem.replace("golden_", "")
            np.savez_compressed(HERE / f"{name}.npz", q=q[:, :, :S], k=k[:, :, :S],
                                v=v[:, :, :S], o_ref=o[:, :, :S],
                                meta=np.array([B, H, S, D, BM, BN], dtype=np.int32))
            print("wrote", HERE / f"{name}.npz")
    return 0


if __name__ == "__main__":
    sys.exit(main())
