"""The per-phase cycle profiler (attn_fwd_profiled, attnprofile_b200.profiler):
the profiled variant computes the same O as attn_fwd, and the stamps have the
layout and ordering the host summary relies on.

The reference's profiler (attn.cu:5-22, stamps attn.cu:133-444) records
clock64 begin/end per phase and KV iteration for one CTA; here the phases are
LoadQ, LoadK, LoadV, GEMM-QK, SOFTMAX, GEMM-PV, the four SOFTMAX steps, and an
Epilogue phase whose slots are steps.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _torch():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


def _inputs(B, H, S, D, seed=0):
    torch = _torch()
    g = torch.Generator(device="cuda").manual_seed(seed)
    return [torch.randn(B, H, S, D, generator=g, device="cuda").half() for _ in range(3)]


@pytest.mark.parametrize("BM,BN", [(256, 128), (128, 64), (128, 256), (512, 128)])
def test_profiled_variant_matches_attn(engine, BM, BN):
    torch = _torch()
    Q, K, V = _inputs(1, 4, 2048, 128, seed=BM + BN)
    engine.set_split(1)
    try:
        ref = engine.attn(Q, K, V, BM=BM, BN=BN)
        O, st = engine.attn_profiled(Q, K, V, BM=BM, BN=BN, cta=1)
    finally:
        engine.set_split(0)
    torch.cuda.synchronize()
    assert engine.get_status(0)[0] == 0
    assert torch.equal(O, ref)
    phases, slots = engine.profile_layout()
    assert tuple(st.shape) == (phases, slots, 2) == (17, 32, 2)


def test_stamps_are_ordered(engine):
    from attnprofile_b200 import profiler
    torch = _torch()
    Q, K, V = _inputs(1, 16, 4096, 128, seed=3)
    engine.set_split(1)
    try:
        _, st = engine.attn_profiled(Q, K, V, BM=256, BN=128, cta=100)
    finally:
        engine.set_split(0)
    torch.cuda.synchronize()
    a = st.numpy().astype(np.int64)
    n_kv = 4096 // 128
    names = profiler.ALL_PHASES
    for k, name in enumerate(names):
        b, e = a[k, :, 0], a[k, :, 1]
        rec = (b != 0) & (e != 0)
        if name == "LoadQ":
            assert rec[0]
            continue
        assert rec[:n_kv].all(), name          # every KV iteration stamped (32 slots)
        assert (e[rec] >= b[rec]).all(), name  # end after begin
    soft = a[names.index("SOFTMAX"), :, 0]
    assert (np.diff(soft[:n_kv]) > 0).all()    # iterations in order
    # GEMM-QK of a tile completes before its softmax starts; the softmax of a
    # tile publishes P before that tile's P V completes.
    qk_end = a[names.index("GEMM-QK"), :n_kv, 1]
    sm_begin = a[names.index("SOFTMAX"), :n_kv, 0]
    assert (qk_end <= sm_begin).all()
    # Epilogue: whole step and the wait for the last P V and the O store issue
    ep = a[len(names)]
    for step in (profiler.EPILOGUE_STEPS.index(s) for s in ("epilogue", "ep-waitO", "ep-store")):
        assert ep[step, 0] != 0 and ep[step, 1] >= ep[step, 0]
    assert ep[0, 0] >= a[names.index("SOFTMAX"), n_kv - 1, 1]
    r = profiler.summarize([a])
    assert 0 < r["period"] < 1e6 and r["epilogue"] > 0


def test_split_part_stamps_its_epilogue_steps(engine):
    """A CTA that runs one key range of a split unit stamps the partial-O
    write and the count-in."""
    from attnprofile_b200 import profiler
    torch = _torch()
    Q, K, V = _inputs(1, 2, 2048, 128, seed=4)
    engine.set_split(2)
    try:
        _, st = engine.attn_profiled(Q, K, V, BM=256, BN=128, cta=0)
        O = engine.attn(Q, K, V, BM=256, BN=128)
    finally:
        engine.set_split(0)
    torch.cuda.synchronize()
    assert engine.get_status(0)[0] == 0
    ep = st.numpy().astype(np.int64)[len(profiler.ALL_PHASES)]
    for name in ("ep-partial", "ep-count"):
        i = profiler.EPILOGUE_STEPS.index(name)
        assert ep[i, 0] != 0 and ep[i, 1] >= ep[i, 0], name
    assert torch.isfinite(O.float()).all()
