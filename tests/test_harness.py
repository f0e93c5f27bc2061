"""The reference's tuning harness drives the B200 engine unchanged.

CPU part: the B200 solver agrees with the library's own launch geometry; when
the reference checkout is present, its benchmark_run_attn.py (imported from
where it lies, with our harness directory first on sys.path so its
`from solver import solve` finds the B200 solver) generates configs, rewrites
the constexpr lines of our attn_test.cu, and compiles it with its own nvcc
command line (`-arch=sm_100a -lcuda -Xptxas=-v`), without a ptxas
performance-loss rejection.  GPU part: the compiled driver runs and prints
the reference's 8-field result line.
"""
import importlib
import os
import re
import shutil
import subprocess
import sys
from argparse import Namespace
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
HARNESS = ROOT / "attnprofile_b200" / "harness"
# The reference checkout: $ATTNPROF_REF, else a `reference` directory beside
# this repository; the tests that need it skip when it is absent.
REF_TUNING = Path(os.environ.get("ATTNPROF_REF") or (ROOT.parent / "reference")) / "tuning"


def _solver():
    sys.path.insert(0, str(HARNESS))
    try:
        import solver
        importlib.reload(solver)
        return solver
    finally:
        sys.path.remove(str(HARNESS))


def test_solver_matches_library_geometry(engine):
    solver = _solver()
    for D in (64, 128):
        for BM, BN in engine.SUPPORTED_TILES:
            q = engine.query_config(D, BM, BN, 0)
            assert solver.lib_stages(BM, BN, D) == q["stages"]
            assert solver.smem_bytes(BM, BN, D, q["stages"]) == q["smem_bytes"]
            assert solver.tmem_columns(BM, BN, D) <= q["tmem_cols"]


def test_pair_tile_geometry(engine):
    """BM = 512 (CTA pairs, D = 128 only): each CTA holds two Q tiles and
    half-size K/V slots, so the ring is at least twice as deep as at BM = 256
    (whose CTA also holds the persistent schedule's O staging)."""
    for BM, BN in engine.PAIR_TILES:
        q = engine.query_config(128, BM, BN, 0)
        single = engine.query_config(128, 256, BN, 0)
        assert q["num_threads"] == single["num_threads"] and q["tmem_cols"] == 512
        assert q["stages"] >= 2 * single["stages"] and q["smem_bytes"] <= 232448
        with pytest.raises(engine.AttnError):
            engine.query_config(64, BM, BN, 0)


def test_solver_keys_and_constraints():
    solver = _solver()
    for k in (1, 2, 3):
        sols = solver.solve(HD=128, NumSmem=2, KernelIdx=k)
        assert sols
        for s in sols:
            assert s["BN"] % 32 == 0 and s["SmemSize"] <= 232448 and s["TmemCols"] <= 512
            assert s["RegsModelled"] is False and s["Stages"] == solver.lib_stages(
                s["BM"], s["BN"], 128)
            assert (s["RepeatN"] == 1) == (k != 3)
            assert (s["NumSmemP"] == 0) == (k == 1)
        # the ring depth is the library's whatever NumSmem says (runAttn ignores it)
        assert [x["SmemSize"] for x in solver.solve(HD=128, NumSmem=1, KernelIdx=k)] == \
            [x["SmemSize"] for x in sols]
    # BM = 256 with BN = 256 at D = 128 needs 768 TMEM columns: never proposed
    assert all(s["BN"] <= 128 for s in solver.solve(HD=128, NumSmem=1, KernelIdx=3))


def test_driver_constexpr_lines_are_unique():
    text = (HARNESS / "attn_test.cu").read_text()
    for name in ("BM", "BN", "B", "H", "S", "D", "NUM_SMEM", "P_SMEM_K_TILES", "KERNEL_IDX",
                 "NUM_THREADS"):
        assert len(re.findall(rf"constexpr\s+int\s+{name}\s*=\s*[^;]+;", text)) == 1, name
    for name in ("PRODUCER_REG_DEALLOC", "CONSUMER_REG_ALLOC"):
        assert len(re.findall(rf"constexpr\s+uint32_t\s+{name}\s*=\s*[^;]+;", text)) == 1


def _reference_harness():
    if not (REF_TUNING / "benchmark_run_attn.py").exists():
        pytest.skip("reference checkout not present")
    sys.path.insert(0, str(HARNESS))
    sys.path.insert(1, str(REF_TUNING))
    try:
        sys.modules.pop("solver", None)
        sys.modules.pop("benchmark_run_attn", None)
        mod = importlib.import_module("benchmark_run_attn")
    finally:
        sys.path.remove(str(HARNESS))
        sys.path.remove(str(REF_TUNING))
    return mod


def test_reference_harness_generates_b200_configs():
    h = _reference_harness()
    for k in (1, 3):
        cfgs = h.get_configs(1, 16, 4096, 128, kernel_idx=k, bn_min=32)
        assert cfgs, k
        assert all(c["BN"] % 32 == 0 for c in cfgs)
        assert {c["BM"] for c in cfgs} == ({128} if k == 1 else {256})


def test_reference_harness_compiles_our_driver(tmp_path):
    h = _reference_harness()
    build = HARNESS / "build" / "pytest"
    if build.exists():
        shutil.rmtree(build)
    build.mkdir(parents=True)
    src = HARNESS / "attn_test.cu"
    args = Namespace(nvcc=shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc", arch="sm_100a",
                     device=None, force_generate=True, force_compile=True)
    for k, bm, bn in ((1, 128, 128), (3, 256, 64)):
        params = {"B": 1, "H": 16, "S": 4096, "D": 128, "BM": bm, "BN": bn, "NUM_SMEM": 2,
                  "PRODUCER_REG_DEALLOC": 24, "CONSUMER_REG_ALLOC": 240, "P_SMEM_K_TILES": 4,
                  "KERNEL_IDX": k, "NUM_THREADS": 384}
        h.validate_params(params)
        gen = h.make_source(src, build, params, force=True)
        _, exe = h.config_paths(build, params)
        h.compile_config(args, src, gen, exe)  # raises on error or ptxas perf-loss warning
        assert exe.exists()
    line = "1, 16, 4096, 128, 256, 128, 0.125000, 1099.512"
    m = h.parse_benchmark_output("noise\n" + line)
    assert m["BM"] == 256 and abs(m["tflops"] - 1099.512) < 1e-9


@pytest.mark.gpu
def test_driver_runs_and_prints_result_line(tmp_path):
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    build = HARNESS / "build" / "pytest_gpu"
    build.mkdir(parents=True, exist_ok=True)
    src = (HARNESS / "attn_test.cu").read_text()
    gen = build / "attn_test_gpu.cu"
    gen.write_text(src)
    exe = build / "attn_test_gpu"
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    r = subprocess.run([nvcc, "-std=c++17", "-arch=sm_100a", "-O3", str(gen), "-o", str(exe),
                        "-lcuda", "-Xptxas=-v"], cwd=HARNESS, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-2000:]
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stderr
    last = [ln for ln in out.stdout.splitlines() if len(ln.split(",")) == 8][-1]
    parts = [p.strip() for p in last.split(",")]
    assert parts[:6] == ["1", "16", "4096", "128", "256", "128"]
    assert float(parts[7]) > 100.0
