"""attn_fwd_noalloc: the entry point for callers that must not allocate GPU
memory when they launch (a server that reserved its whole memory budget at
start-up, a custom allocator or its callbacks, a loop that cannot take a
cudaMalloc stall).  Its scratch for key-split launches is one fixed array in
the library instead of a pool allocation.

Checked through the C ABI:
  * two calls in a row on shapes whose automatic plan splits units (so the
    fixed scratch is used, and reused by the second call) against attn_fwd,
    within the parity tolerance of every other test (max-abs 2e-3, mean-abs
    2e-4), and the second call's output against the CPU oracle on sampled
    rows of every (batch, head) unit;
  * a first call on a shape that does not split, then one that does: the
    scratch address is looked up by whichever call comes first;
  * a plan whose scratch exceeds the fixed size is refused with
    ATTN_ERR_SCRATCH_LIMIT without touching the output.
This file sorts last so that a failure here stops a `-x` run only after all
other tests.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-3
MEAN_ABS = 2e-4
SCRATCH_BYTES = 32 << 20  # ATTN_NOALLOC_SCRATCH_BYTES in include/attnprof.h


def _torch():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


def _bind(engine):
    L = engine.lib()
    vp, i = ctypes.c_void_p, ctypes.c_int
    L.attn_fwd_noalloc.argtypes = [vp, vp, vp, vp, i, i, i, i, i, i, i, vp]
    L.attn_fwd_noalloc.restype = ctypes.c_int
    return L


def _call(L, fn, Q, K, V, O, BM, BN):
    torch = _torch()
    B, H, S, D = Q.shape
    dt = 0 if Q.dtype == torch.float16 else 1
    stream = torch.cuda.current_stream().cuda_stream
    return getattr(L, fn)(Q.data_ptr(), K.data_ptr(), V.data_ptr(), O.data_ptr(), B, H, S, D, dt,
                          BM, BN, stream)


def _inputs(B, H, S, D, dt, seed):
    torch = _torch()
    g = torch.Generator(device="cuda").manual_seed(seed)
    return tuple(torch.randn(B, H, S, D, generator=g, device="cuda").to(dt) for _ in range(3))


def _check_oracle_rows(oracle_mod, Q, K, V, O, BN, rows_per_unit=8, seed=0):
    """O against the CPU oracle (tuning/utils.cuh:139-198) on sampled rows."""
    torch = _torch()
    B, H, S, D = Q.shape
    dt = 0 if Q.dtype == torch.float16 else 1
    rng = np.random.default_rng(seed)
    rows = []
    for u in range(B * H):
        rows += list(u * S + rng.choice(S, size=rows_per_unit, replace=False))
    rows = np.array(sorted(rows), dtype=np.int64)
    u16 = lambda t: t.view(torch.int16).cpu().numpy().view(np.uint16)
    ref = oracle_mod.attention_rows(u16(Q), u16(K), u16(V), rows, bn_tile=BN, dtype=dt)
    got = u16(O).reshape(-1, D)[rows]
    d = np.abs(oracle_mod.to_f32(got, dt) - oracle_mod.to_f32(ref, dt))
    assert d.max() <= MAX_ABS and d.mean() <= MEAN_ABS, (float(d.max()), float(d.mean()))


@pytest.mark.parametrize("B,H,S,dtype", [(1, 2, 8192, "f16"), (1, 6, 8192, "bf16")])
def test_noalloc_matches_attn_fwd_twice(engine, oracle_mod, B, H, S, dtype):
    torch = _torch()
    L = _bind(engine)
    engine.set_split(0)
    dt = torch.float16 if dtype == "f16" else torch.bfloat16
    BM, BN, D = 256, 128, 128
    plan = engine.query_split(B, H, S, D, BM=BM, BN=BN, dtype=0 if dtype == "f16" else 1)
    if torch.cuda.get_device_properties(0).multi_processor_count == 148:
        assert plan["split"] > 1, plan          # the fixed scratch is in use
    assert plan["workspace_bytes"] <= SCRATCH_BYTES
    Q, K, V = _inputs(B, H, S, D, dt, B * 100 + H)
    ref = torch.empty_like(Q)
    assert _call(L, "attn_fwd", Q, K, V, ref, BM, BN) == 0
    for _ in range(2):
        O = torch.full_like(Q, float("nan"))
        assert _call(L, "attn_fwd_noalloc", Q, K, V, O, BM, BN) == 0
        torch.cuda.synchronize()
        rc, site = engine.get_status(0)
        assert rc == 0, hex(site)
        d = (O.float() - ref.float()).abs()
        assert torch.isfinite(O.float()).all()
        assert d.max().item() <= MAX_ABS and d.mean().item() <= MEAN_ABS
    _check_oracle_rows(oracle_mod, Q, K, V, O, BN, seed=H)


def test_noalloc_on_an_eight_warp_tile_with_a_split_plan(engine, oracle_mod):
    """1 x 2 x 8192 at D = 64 on 256 x 96: the tile runs eight softmax warps
    for whole units, and this plan splits, so the launch runs the tile's
    four-warp kernel with its partials in the fixed scratch.  Equal to
    attn_fwd, and to the oracle on sampled rows."""
    torch = _torch()
    L = _bind(engine)
    engine.set_split(0)
    B, H, S, D, BM, BN = 1, 2, 8192, 64, 256, 96
    plan = engine.query_split(B, H, S, D, BM=BM, BN=BN)
    if torch.cuda.get_device_properties(0).multi_processor_count == 148:
        assert plan["split"] > 1, plan
    assert plan["workspace_bytes"] <= SCRATCH_BYTES
    Q, K, V = _inputs(B, H, S, D, torch.float16, 64)
    ref = torch.empty_like(Q)
    assert _call(L, "attn_fwd", Q, K, V, ref, BM, BN) == 0
    O = torch.full_like(Q, float("nan"))
    assert _call(L, "attn_fwd_noalloc", Q, K, V, O, BM, BN) == 0
    torch.cuda.synchronize()
    rc, site = engine.get_status(0)
    assert rc == 0, hex(site)
    assert torch.equal(O, ref)
    _check_oracle_rows(oracle_mod, Q, K, V, O, BN)


def test_noalloc_unsplit_call_then_split_call(engine):
    """The first call on the device needs no scratch (one whole wave), the
    next one splits: both run, and the second matches attn_fwd."""
    torch = _torch()
    L = _bind(engine)
    engine.set_split(0)
    BM, BN = 256, 128
    small = _inputs(1, 1, 256, 128, torch.float16, 5)
    assert engine.query_split(1, 1, 256, 128)["split"] == 1
    O = torch.empty_like(small[0])
    assert _call(L, "attn_fwd_noalloc", *small, O, BM, BN) == 0
    Q, K, V = _inputs(1, 2, 8192, 128, torch.float16, 6)
    ref, O2 = torch.empty_like(Q), torch.full_like(Q, float("nan"))
    assert _call(L, "attn_fwd", Q, K, V, ref, BM, BN) == 0
    assert _call(L, "attn_fwd_noalloc", Q, K, V, O2, BM, BN) == 0
    torch.cuda.synchronize()
    assert engine.get_status(0)[0] == 0
    d = (O2.float() - ref.float()).abs()
    assert d.max().item() <= MAX_ABS and d.mean().item() <= MEAN_ABS


def test_noalloc_refuses_scratch_over_its_size(engine):
    """A forced 4-way split of 1x16x4096 needs about 57 MB of partial results,
    more than the fixed 32 MiB: refused, nothing launched."""
    torch = _torch()
    L = _bind(engine)
    Q, K, V = (torch.randn(1, 16, 4096, 128, device="cuda").half() for _ in range(3))
    O = torch.full_like(Q, 3.0)
    try:
        engine.set_split(4)
        if engine.query_split(1, 16, 4096, 128)["workspace_bytes"] <= SCRATCH_BYTES:
            pytest.skip("this GPU's plan fits the scratch")
        assert _call(L, "attn_fwd_noalloc", Q, K, V, O, 256, 128) == engine.ERR["SCRATCH_LIMIT"]
    finally:
        engine.set_split(0)
    torch.cuda.synchronize()
    assert torch.all(O == 3.0)
    # the same call within the limit (no split) runs
    assert _call(L, "attn_fwd_noalloc", Q, K, V, O, 256, 128) == 0
    torch.cuda.synchronize()
    assert engine.get_status(0)[0] == 0
    assert torch.isfinite(O.float()).all()
