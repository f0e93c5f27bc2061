"""The reference's tuning loop over the B200 engine, split between a machine
that has the reference checkout (and nvcc) and a B200 box that has neither
the checkout nor a network.

The loop is the reference's own benchmark_get_configs
(tuning/benchmark_run_attn.py:339-441): get_configs -> validate_params ->
make_source -> compile_config -> run_config -> parse_benchmark_output ->
ranking -> top-k JSON.  Every step runs as the reference wrote it, imported
from the checkout with this directory first on sys.path (so its
`from solver import solve` takes the B200 solver), except run_config, the
step that executes a compiled driver on a GPU:

  prepare  (checkout + nvcc, no GPU)  get_configs, then make_source and
           compile_config for each configuration into --build-dir (the
           reference's functions, several compiles at once); writes
           manifest.json beside the binaries.
  run      (B200, no checkout)        executes every binary of the manifest
           the way run_config does (no arguments, cwd = the source's
           directory, stdout captured) and writes outputs.json.
  collect  (checkout, no GPU)         runs the reference's
           benchmark_get_configs with force_compile off, so compile_config
           takes its cache path for the binaries built above, and with
           run_config answering from outputs.json; the reference's code then
           parses, ranks and writes its top-k JSON.

    python -m attnprofile_b200.harness.remote_sweep prepare --kernel-idx 1 --bn-min 128
    python -m attnprofile_b200.harness.remote_sweep run
    python -m attnprofile_b200.harness.remote_sweep collect --kernel-idx 1 --bn-min 128 \\
        --output profiles/top10_k1_b1_h16_s4096_d128_bnmin128.json

The reference checkout is $ATTNPROF_REF, else a `reference` directory beside
this repository.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import importlib
import json
import os
import shutil
import subprocess
import sys
from argparse import Namespace
from pathlib import Path

HARNESS = Path(__file__).resolve().parent
ROOT = HARNESS.parent.parent
SOURCE = HARNESS / "attn_test.cu"
DEFAULT_BUILD = HARNESS / "build" / "sweep"


def reference_tuning() -> Path:
    return Path(os.environ.get("ATTNPROF_REF") or (ROOT.parent / "reference")) / "tuning"


def reference_harness():
    """The reference's benchmark_run_attn module, imported from the checkout,
    with the B200 solver first on sys.path."""
    tuning = reference_tuning()
    if not (tuning / "benchmark_run_attn.py").exists():
        raise SystemExit(f"reference checkout not found at {tuning.parent} (set ATTNPROF_REF)")
    sys.path.insert(0, str(HARNESS))
    sys.path.insert(1, str(tuning))
    try:
        sys.modules.pop("solver", None)
        sys.modules.pop("benchmark_run_attn", None)
        return importlib.import_module("benchmark_run_attn")
    finally:
        sys.path.remove(str(HARNESS))
        sys.path.remove(str(tuning))


def _nvcc() -> str:
    return shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"


def prepare(a) -> None:
    h = reference_harness()
    build = Path(a.build_dir).resolve()
    build.mkdir(parents=True, exist_ok=True)
    configs = h.get_configs(a.B, a.H, a.S, a.D, kernel_idx=a.kernel_idx, bn_min=a.bn_min)
    args = Namespace(nvcc=_nvcc(), arch="sm_100a", device=None, force_generate=True,
                     force_compile=True)
    jobs = []
    for params in configs:
        h.validate_params(params)
        gen = h.make_source(SOURCE, build, params, force=True)
        _, exe = h.config_paths(build, params)
        jobs.append((params, gen, exe))

    def compile_one(job):
        params, gen, exe = job
        try:
            h.compile_config(args, SOURCE, gen, exe)
            return None
        except Exception as e:  # noqa: BLE001 -- recorded, as the reference's loop does
            return f"{h.config_tag(params)}: {e}"

    with cf.ThreadPoolExecutor(a.jobs) as ex:
        errors = [e for e in ex.map(compile_one, jobs) if e]
    manifest = {"source": str(SOURCE), "configs": [
        {"params": p, "exe": str(exe.relative_to(ROOT))} for p, _, exe in jobs if exe.exists()],
        "compile_errors": errors}
    (build / "manifest.json").write_text(json.dumps(manifest, indent=1))
    print(f"{len(manifest['configs'])} binaries, {len(errors)} compile errors -> {build}")


def run(a) -> None:
    build = Path(a.build_dir).resolve()
    manifest = json.loads((build / "manifest.json").read_text())
    outputs = {}
    for c in manifest["configs"]:
        exe = ROOT / c["exe"]
        # as run_config: the binary with no arguments, cwd = the source's directory
        r = subprocess.run([str(exe)], cwd=SOURCE.parent, capture_output=True, text=True,
                           timeout=a.timeout)
        outputs[c["exe"]] = {"returncode": r.returncode, "stdout": r.stdout.strip(),
                             "stderr": r.stderr.strip()}
        last = r.stdout.strip().splitlines()[-1:] or [""]
        print(f"{Path(c['exe']).name}: rc={r.returncode} {last[0]}", flush=True)
    (build / "outputs.json").write_text(json.dumps(outputs, indent=1))


def collect(a) -> None:
    h = reference_harness()
    build = Path(a.build_dir).resolve()
    outputs = json.loads((build / "outputs.json").read_text())

    def run_config_from_record(args, source_path, exe):
        rec = outputs[str(Path(exe).resolve().relative_to(ROOT))]
        if rec["returncode"] != 0:
            raise subprocess.CalledProcessError(rec["returncode"], [str(exe)], rec["stdout"],
                                                rec["stderr"])
        return rec["stdout"]

    h.run_config = run_config_from_record
    out = Path(a.output).resolve() if a.output else None
    h.benchmark_get_configs(a.B, a.H, a.S, a.D, kernel_idx=a.kernel_idx, bn_min=a.bn_min,
                            rank=a.rank, source=SOURCE, build_dir=build, nvcc=_nvcc(),
                            arch="sm_100a", force_generate=False, force_compile=False,
                            output_path=out)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("step", choices=["prepare", "run", "collect"])
    ap.add_argument("--build-dir", default=str(DEFAULT_BUILD))
    ap.add_argument("--kernel-idx", type=int, default=1)
    ap.add_argument("--bn-min", type=int, default=128)
    ap.add_argument("--rank", type=int, default=10)
    ap.add_argument("-B", type=int, default=1)
    ap.add_argument("-H", type=int, default=16)
    ap.add_argument("-S", type=int, default=4096)
    ap.add_argument("-D", type=int, default=128)
    ap.add_argument("--jobs", type=int, default=os.cpu_count() or 4)
    ap.add_argument("--timeout", type=float, default=300.0)
    ap.add_argument("--output", default=None)
    a = ap.parse_args(argv)
    {"prepare": prepare, "run": run, "collect": collect}[a.step](a)
    return 0


if __name__ == "__main__":
    sys.exit(main())
