"""C-ABI library: loads without a GPU, exports every declared symbol, and
validates arguments on the host (no kernel is launched here)."""
import ctypes
import re
from pathlib import Path

import pytest

HEADER = Path(__file__).resolve().parent.parent / "include" / "attnprof.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(attn_\w+)\s*\(", text)))


def test_header_declares_the_boundary():
    names = declared_functions()
    for must in ("attn_fwd", "attn_fwd_padded", "attn_fwd_profiled", "attn_fwd_sharded",
                 "attn_error_string", "attn_get_status", "attn_query_config"):
        assert must in names


def test_library_exports_every_declared_symbol(engine):
    L = engine.lib()
    missing = [n for n in declared_functions() if not hasattr(L, n)]
    assert not missing, missing


def test_library_has_no_libcuda_link_dependency(engine):
    import subprocess
    out = subprocess.run(["ldd", str(engine.LIB_PATH)], capture_output=True, text=True).stdout
    assert "libcuda.so" not in out


def test_error_strings(engine):
    L = engine.lib()
    for code in list(engine.ERR.values()) + [-99]:
        s = L.attn_error_string(code)
        assert s and len(s) > 1


@pytest.mark.parametrize("units,n", [(16, 1), (16, 3), (256, 8), (64, 8), (5, 8), (0, 4)])
def test_shard_range_partitions_units(engine, units, n):
    spans = [engine.shard_range(units, n, g) for g in range(n)]
    assert spans[0][0] == 0 and spans[-1][1] == units
    for (a0, a1), (b0, b1) in zip(spans, spans[1:]):
        assert a1 == b0
    sizes = [e - b for b, e in spans]
    assert max(sizes) - min(sizes) <= 1


def test_shard_range_rejects_bad_rank(engine):
    b, e = ctypes.c_int(), ctypes.c_int()
    assert engine.lib().attn_shard_range(16, 4, 4, ctypes.byref(b), ctypes.byref(e)) == -8


@pytest.mark.parametrize("bm,bn", [(128, 32), (128, 64), (128, 96), (128, 128), (128, 256),
                                   (256, 32), (256, 64), (256, 96), (256, 128)])
@pytest.mark.parametrize("d", [64, 128])
def test_query_config_fits_b200(engine, bm, bn, d):
    for dt in (0, 1):
        c = engine.query_config(d, bm, bn, dt)
        assert c["smem_bytes"] <= 232448
        assert c["tmem_cols"] in (32, 64, 128, 256, 512)
        assert c["stages"] >= 2
        # Softmax warps per Q tile: four of 32 rows, or eight of 16 rows on
        # the two-tile D = 64 variants that hold two S buffers per tile.
        two_s = bm == 256 and 2 * (2 * bn + d) <= 512
        per_tile = 8 if d == 64 and two_s else 4
        assert c["num_threads"] == 32 * (per_tile * (bm // 128) + 4)


@pytest.mark.parametrize("d,bm,bn", [(128, 256, 256), (96, 128, 128), (128, 64, 128),
                                     (128, 128, 48)])
def test_query_config_rejects_unbuilt(engine, d, bm, bn):
    vals = [ctypes.c_int() for _ in range(4)]
    rc = engine.lib().attn_query_config(d, bm, bn, 0, *[ctypes.byref(v) for v in vals])
    assert rc == engine.ERR["UNSUPPORTED"]


def test_host_validation_without_gpu(engine):
    L = engine.lib()
    good = 0x10000
    # empty problem: nothing to do, success
    assert L.attn_fwd(good, good, good, good, 0, 16, 4096, 128, 0, 128, 128, None) == 0
    assert L.attn_fwd(good, good, good, good, 1, 1, 0, 128, 0, 128, 128, None) == 0
    # bad arguments
    assert L.attn_fwd(good, good, good, good, 1, 1, -1, 128, 0, 128, 128, None) == -1
    assert L.attn_fwd(None, good, good, good, 1, 1, 16, 128, 0, 128, 128, None) == -1
    assert L.attn_fwd(good + 2, good, good, good, 1, 1, 16, 128, 0, 128, 128, None) == -3
    assert L.attn_fwd(good, good, good, good, 1, 1, 16, 96, 0, 128, 128, None) == -2
    assert L.attn_fwd(good, good, good, good, 1, 1, 16, 128, 7, 128, 128, None) == -2
    # B*H beyond a 32-bit count (the grid is 1-D over work tiles, no 65535 limit)
    assert L.attn_fwd(good, good, good, good, 65536, 65536, 16, 128, 0, 128, 128, None) == -1
    # padded rows fewer than S
    assert L.attn_fwd_padded(good, good, good, good, 1, 1, 64, 128, 32, 64, 0, 128, 128,
                             None) == -1
    # profiled call needs a buffer
    assert L.attn_fwd_profiled(good, good, good, good, 1, 1, 64, 128, 0, 128, 128, None,
                               None, 0) == -1


def test_no_cpu_fallback_without_gpu(engine):
    """With no usable GPU a valid call fails loudly; it never computes on the host."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("GPU present")
    good = 0x10000
    rc = engine.lib().attn_fwd(good, good, good, good, 1, 1, 64, 128, 0, 128, 128, None)
    assert rc == engine.ERR["CUDA"]


def test_plan_split_cost_model(engine):
    # Few long units leave most SMs idle: 1x1x16384 at BM=256, BN=128 has
    # 64 units of 128 key tiles; two key ranges each fill 128 SMs.
    assert engine.plan_split(64, 128, 148) == {"split": 2, "whole": 0, "ctas": 128}
    # 1x6x8192: 192 units of 64 tiles; the 44 of the second wave run as 3 ranges.
    assert engine.plan_split(192, 64, 148) == {"split": 3, "whole": 148, "ctas": 148 + 44 * 3}
    # A second wave of many units (1x16x4096: 256 units of 32 tiles) does not
    # pay for the partial-O write and merge: unsplit.
    assert engine.plan_split(256, 32, 148)["split"] == 1
    # Short units do not either (1x16x1024: 64 units of 8 tiles).
    assert engine.plan_split(64, 8, 148)["split"] == 1
    # Units that fill whole waves (8x32x8192 and 1x64x32768 at BM=256 give
    # 8192 units; 8192 % 148 = 52, a short tail of a long run) stay unsplit.
    assert engine.plan_split(8192, 64, 148)["split"] == 1
    assert engine.plan_split(296, 32, 148)["split"] == 1     # exactly two waves


@pytest.mark.parametrize("units,n_kv,slots", [(256, 32, 148), (17, 8, 16), (3, 2, 148),
                                              (1000, 5, 148), (148, 64, 148), (0, 8, 148)])
@pytest.mark.parametrize("mode", [0, 1, 2, 3, 4])
def test_plan_split_invariants(engine, units, n_kv, slots, mode):
    p = engine.plan_split(units, n_kv, slots, mode)
    k = p["split"]
    assert 1 <= k <= min(4, max(n_kv, 1))
    assert 0 <= p["whole"] <= units
    assert p["ctas"] == p["whole"] + (units - p["whole"]) * k
    if mode == 1 or units == 0:
        assert k == 1 and p["whole"] == units
    if k > 1:
        assert k <= n_kv                 # every key range holds at least one tile
    if mode >= 2 and units and n_kv >= 2:
        assert k == min(mode, n_kv)      # forced split
    if k == 1:
        assert p["whole"] == units


def test_plan_split_rejects_bad_arguments(engine):
    L = engine.lib()
    k, w, c = ctypes.c_int(), ctypes.c_longlong(), ctypes.c_longlong()
    args = (ctypes.byref(k), ctypes.byref(w), ctypes.byref(c))
    assert L.attn_plan_split(10, 4, 0, 0, *args) == engine.ERR["INVALID_ARG"]
    assert L.attn_plan_split(10, 4, 148, 5, *args) == engine.ERR["INVALID_ARG"]
    assert L.attn_plan_split(-1, 4, 148, 0, *args) == engine.ERR["INVALID_ARG"]
    assert L.attn_set_split(5) == engine.ERR["INVALID_ARG"]
    assert L.attn_set_split(-1) == engine.ERR["INVALID_ARG"]
    assert L.attn_set_split(0) == 0


def test_work_distribution_setters_reject_bad_modes(engine):
    """attn_set_schedule takes 0..2 and attn_set_correction 0..1; both leave
    the previous mode in place on a bad one (checked by setting the default
    back).  Host-only calls: no GPU needed."""
    L = engine.lib()
    for bad in (-1, 3, 100):
        assert L.attn_set_schedule(bad) == engine.ERR["INVALID_ARG"]
    for bad in (-1, 2, 7):
        assert L.attn_set_correction(bad) == engine.ERR["INVALID_ARG"]
    for ok in (1, 0):
        assert L.attn_set_correction(ok) == 0
    for ok in (2, 1, 0):
        assert L.attn_set_schedule(ok) == 0
    with pytest.raises(engine.AttnError):
        engine.set_correction(5)
