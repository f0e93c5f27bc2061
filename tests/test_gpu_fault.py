"""Failure path on the GPU without a GPU fault.

attn_debug_fault(1) makes the producer warp load Q but never K/V -- a flag that
nothing sets.  Every consumer's bounded mbarrier wait then expires after the
configured limit, the kernel records a timeout code in the device status word,
drains its own tensor-core work, frees TMEM and returns.  The context stays
usable: the next normal launch must succeed and be correct.
"""
import pytest

pytestmark = pytest.mark.gpu


def test_bounded_wait_reports_timeout_and_context_survives(engine):
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    g = torch.Generator(device="cuda").manual_seed(0)
    Q, K, V = (torch.randn(1, 2, 512, 128, generator=g, device="cuda").half() for _ in range(3))
    engine.get_status(0, reset=True)
    engine.set_timeout_ns(50_000_000)  # 50 ms
    try:
        engine.debug_fault(1)
        for bm in (128, 256):
            engine.attn(Q, K, V, BM=bm, BN=128)
            rc, site = engine.get_status(0, reset=True)
            assert rc == engine.ERR["DEVICE_TIMEOUT"], (rc, hex(site))
            assert site & 0xFF00 == 0x7100
    finally:
        engine.debug_fault(0)
        engine.set_timeout_ns(2_000_000_000)
    O = engine.attn(Q, K, V, BM=256, BN=128)
    torch.cuda.synchronize()
    assert engine.get_status(0)[0] == 0
    ref = torch.softmax((Q.float() @ K.float().transpose(-1, -2)) / 128 ** 0.5, -1) @ V.float()
    assert (O.float() - ref).abs().max().item() < 2e-3
