"""The reference's own correctness entry on the B200 engine.

oracle/_ref/verify_runner is the reference's verify_attn<B,H,S,D,BM,BN>
(tuning/utils.cuh:73-244), compiled from the reference's sources where they
lie (oracle/Makefile), with our runAttn<...> (attnprofile_b200/harness/
attn_runner.cuh) as its AttnRunner.  verify_attn draws its own mt19937(42)
inputs, runs the kernel, computes its CPU output and prints its max-abs
difference and its count of elements over its own 5e-2 tolerance; here the
difference must be within the north-star bound (2e-3) and the count zero.

The binary is built where the reference checkout is (build()); a GPU box
without it uses the prebuilt file, and the test skips when there is none.
"""
import re
import subprocess
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parent.parent
EXE = ROOT / "oracle" / "_ref" / "verify_runner"
MAX_ABS = 2e-3
LINE = re.compile(r"max_abs_diff=([0-9.eE+-]+) .* mismatches\(abs>[0-9.]+\)=(\d+)/(\d+)")


@pytest.mark.parametrize("case", [0, 1, 2, 3, 4, 5])
def test_reference_verify_attn_accepts_our_runner(case):
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    if not EXE.exists():
        pytest.skip("oracle/_ref/verify_runner not built (needs the reference checkout)")
    r = subprocess.run([str(EXE), str(case)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    assert "Need SM90+" not in r.stdout
    m = [LINE.search(ln) for ln in r.stdout.splitlines()]
    m = [x for x in m if x]
    assert len(m) == 1, r.stdout
    diff, mism, total = float(m[0].group(1)), int(m[0].group(2)), int(m[0].group(3))
    assert total > 0 and mism == 0
    assert diff <= MAX_ABS, r.stdout
