"""The C++ host template include/attnprof.hpp: tests/cxx_abi/caller.cpp is
compiled with g++ against it and linked to libattnprof.so.  The host checks
run everywhere (argument checks through the template, dtype deduction, the
compile-time tile check); the GPU check runs one f16 and one bf16 forward on
device buffers from the CUDA runtime."""
import os
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
SRC = ROOT / "tests" / "cxx_abi" / "caller.cpp"
CUDA = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))


def _build(engine, tmp_path, extra=()) -> Path:
    out = tmp_path / "caller_cxx"
    lib = Path(engine.LIB_PATH)
    cmd = ["g++", "-std=c++17", "-Wall", "-Wextra", "-Werror", "-O1", *extra,
           "-I", str(ROOT / "include"), "-I", str(CUDA / "include"), str(SRC), "-o", str(out),
           "-L", str(lib.parent), "-lattnprof", f"-Wl,-rpath,{lib.parent}",
           "-L", str(CUDA / "lib64"), "-lcudart", f"-Wl,-rpath,{CUDA / 'lib64'}"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return out


@pytest.mark.skipif(shutil.which("g++") is None, reason="no C++ compiler")
def test_cxx_caller_host_checks(engine, tmp_path):
    exe = _build(engine, tmp_path)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0, r.stderr
    assert r.stdout.strip() == "ok"


@pytest.mark.skipif(shutil.which("g++") is None, reason="no C++ compiler")
def test_cxx_template_rejects_unbuilt_tile_at_compile_time(tmp_path):
    src = tmp_path / "bad.cpp"
    src.write_text('#include "attnprof.hpp"\n'
                   "int f(const __half* q, __half* o) {\n"
                   "  return attnprof::attn<256, 256>(q, q, q, o, 1, 1, 1, 128);\n}\n")
    r = subprocess.run(["g++", "-std=c++17", "-fsyntax-only", "-I", str(ROOT / "include"),
                        "-I", str(CUDA / "include"), str(src)], capture_output=True, text=True)
    assert r.returncode != 0 and "not built" in r.stderr


@pytest.mark.gpu
def test_cxx_caller_runs_attention_on_gpu(engine, tmp_path):
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    exe = _build(engine, tmp_path)
    r = subprocess.run([str(exe), "gpu"], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    assert r.stdout.strip() == "ok"
