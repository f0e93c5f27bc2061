"""Build of the sm_100a engine library (attnprofile_b200/libattnprof.so).

Every translation unit under csrc/ is compiled with
    nvcc -gencode arch=compute_100a,code=sm_100a -O3 -lineinfo -Xcompiler -fPIC
in parallel, and linked into one shared library with the CUDA runtime linked
statically, so loading the library needs no GPU driver (a CPU-only machine can
load it and list its symbols; calls then return ATTN_ERR_CUDA).
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
ROOT = PKG.parent
BUILD_DIR = ROOT / "_build"
LIB_PATH = PKG / "libattnprof.so"
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _deps() -> list[Path]:
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + [ROOT / "include" / "attnprof.h"]


def up_to_date() -> bool:
    if not LIB_PATH.exists():
        return False
    t = LIB_PATH.stat().st_mtime
    return all(p.stat().st_mtime <= t for p in _deps())


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile csrc/*.cu for sm_100a and link libattnprof.so (in-tree)."""
    if not force and up_to_date():
        return LIB_PATH
    BUILD_DIR.mkdir(exist_ok=True)
    cc = nvcc()

    def compile_one(src: Path) -> Path:
        obj = BUILD_DIR / (src.stem + ".o")
        cmd = [cc, *NVCC_FLAGS, *ARCH_FLAGS, "-I", str(ROOT / "include"), "-c", str(src), "-o",
               str(obj)]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")
        if verbose:
            print(r.stdout + r.stderr)
        return obj

    workers = max(1, min(len(_sources()), os.cpu_count() or 1))
    with cf.ThreadPoolExecutor(workers) as ex:
        objs = list(ex.map(compile_one, _sources()))
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [cc, "-shared", *ARCH_FLAGS, "-o", str(tmp), *map(str, objs), "-lpthread"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    import sys
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
