"""The C ABI from plain C: tests/c_abi/caller.c compiled as C99 against
include/attnprof.h and linked to libattnprof.so (the binding a foreign
caller of this path would use).  Host checks run everywhere; the GPU check
runs one attention forward on device buffers from the CUDA runtime."""
import os
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
SRC = ROOT / "tests" / "c_abi" / "caller.c"
CUDA = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))


def _build(engine, tmp_path, with_cuda: bool) -> Path:
    out = tmp_path / ("caller_gpu" if with_cuda else "caller")
    lib = Path(engine.LIB_PATH)
    cmd = ["gcc", "-std=c99", "-Wall", "-Wextra", "-Werror", "-O1", "-I", str(ROOT / "include"),
           str(SRC), "-o", str(out), "-L", str(lib.parent), "-lattnprof",
           f"-Wl,-rpath,{lib.parent}"]
    if with_cuda:
        cmd[1:1] = ["-DWITH_CUDA", "-I", str(CUDA / "include")]
        cmd += ["-L", str(CUDA / "lib64"), "-lcudart", f"-Wl,-rpath,{CUDA / 'lib64'}"]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    return out


@pytest.mark.skipif(shutil.which("gcc") is None, reason="no C compiler")
def test_c_caller_host_checks(engine, tmp_path):
    exe = _build(engine, tmp_path, with_cuda=False)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0, r.stderr
    assert r.stdout.strip() == "ok"


@pytest.mark.gpu
def test_c_caller_runs_attention_on_gpu(engine, tmp_path):
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    exe = _build(engine, tmp_path, with_cuda=True)
    r = subprocess.run([str(exe), "gpu"], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
