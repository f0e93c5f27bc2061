"""attn_fwd_noalloc: the entry point for callers that must not allocate GPU
memory (a CUDA graph under capture, a process that reserved its memory budget
up front).  Its scratch for key-split launches is one fixed array in the
library instead of a pool allocation.

Checked through the C ABI: two calls in a row on shapes whose automatic plan
splits units (so the fixed scratch is used, and reused by the second call)
against attn_fwd, within the parity tolerance of every other test (max-abs
2e-3, mean-abs 2e-4); and a plan whose scratch exceeds the fixed size is
refused with ATTN_ERR_SCRATCH_LIMIT without touching the output.  This file
sorts last so that a failure here stops a `-x` run only after all other tests.
"""
import ctypes

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


@pytest.mark.parametrize("B,H,S,dtype", [(1, 2, 8192, "f16"), (1, 6, 8192, "bf16")])
def test_noalloc_matches_attn_fwd_twice(engine, B, H, S, dtype):
    torch = _torch()
    L = _bind(engine)
    engine.set_split(0)
    dt = torch.float16 if dtype == "f16" else torch.bfloat16
    BM, BN, D = 256, 128, 128
    plan = engine.query_split(B, H, S, D, BM=BM, BN=BN, dtype=0 if dtype == "f16" else 1)
    if torch.cuda.get_device_properties(0).multi_processor_count == 148:
        assert plan["split"] > 1, plan          # the fixed scratch is in use
    assert plan["workspace_bytes"] <= SCRATCH_BYTES
    g = torch.Generator(device="cuda").manual_seed(B * 100 + H)
    Q, K, V = (torch.randn(B, H, S, D, generator=g, device="cuda").to(dt) for _ in range(3))
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
