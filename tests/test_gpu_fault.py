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
        # one MMA issuer (NSBUF = 1), one issuer per Q tile (256 x 64, 256 x 32),
        # a key-split launch whose parts never count in, and CTA pairs (the
        # odd CTA's relay and the even CTA's issuer both time out; the two
        # meet at the cluster barrier before freeing tensor memory)
        for bm, bn, split in ((128, 128, 0), (256, 128, 0), (256, 64, 0), (256, 32, 0),
                              (256, 128, 2), (512, 128, 0)):
            engine.set_split(split)
            engine.attn(Q, K, V, BM=bm, BN=bn)
            rc, site = engine.get_status(0, reset=True)
            assert rc == engine.ERR["DEVICE_TIMEOUT"], (bm, bn, split, rc, hex(site))
            assert site & 0xFF00 == 0x7100
    finally:
        engine.debug_fault(0)
        engine.set_split(0)
        engine.set_timeout_ns(2_000_000_000)
    ref = torch.softmax((Q.float() @ K.float().transpose(-1, -2)) / 128 ** 0.5, -1) @ V.float()
    for bm, bn, split in ((256, 128, 0), (256, 64, 0), (256, 128, 2), (512, 128, 0)):
        engine.set_split(split)
        try:
            O = engine.attn(Q, K, V, BM=bm, BN=bn)
            torch.cuda.synchronize()
        finally:
            engine.set_split(0)
        assert engine.get_status(0)[0] == 0
        assert (O.float() - ref).abs().max().item() < 2e-3, (bm, bn, split)
