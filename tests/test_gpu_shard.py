"""attn_fwd_sharded on the GPUs of one process: (batch, head) partition, join,
and error propagation from one failed shard (injected on the host: a
misaligned pointer the library rejects before launching)."""
import ctypes

import pytest

pytestmark = pytest.mark.gpu


def _setup():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    n = torch.cuda.device_count()
    return torch, ([0, 1] if n >= 2 else [0, 0])


@pytest.mark.parametrize("BM", [256, 512])
def test_sharded_matches_single_call(engine, BM):
    torch, devices = _setup()
    B, H, S, D = 2, 4, 512, 128
    g = torch.Generator().manual_seed(5)
    Q, K, V = (torch.randn(B, H, S, D, generator=g).half() for _ in range(3))
    ref = engine.attn(Q.cuda(0), K.cuda(0), V.cuda(0), BM=BM).cpu()
    U = B * H
    shards = [engine.shard_range(U, len(devices), r) for r in range(len(devices))]
    flat = lambda t: t.reshape(1, U, S, D)
    Qs = [flat(Q)[:, a:b].contiguous().cuda(d) for (a, b), d in zip(shards, devices)]
    Ks = [flat(K)[:, a:b].contiguous().cuda(d) for (a, b), d in zip(shards, devices)]
    Vs = [flat(V)[:, a:b].contiguous().cuda(d) for (a, b), d in zip(shards, devices)]
    Os = [torch.empty_like(q) for q in Qs]
    ms = engine.attn_sharded(Qs, Ks, Vs, Os, devices, B=B, H=H, BM=BM)
    assert len(ms) == len(devices) and all(m > 0 for m in ms)
    got = torch.cat([o.cpu() for o in Os], dim=1).reshape(B, H, S, D)
    assert torch.equal(got, ref)


def test_failed_shard_propagates_and_others_join(engine):
    torch, devices = _setup()
    B, H, S, D = 1, 4, 256, 128
    U = B * H
    shards = [engine.shard_range(U, len(devices), r) for r in range(len(devices))]
    mk = lambda n, d: torch.randn(1, n, S, D, device=f"cuda:{d}").half()
    Qs = [mk(b - a, d) for (a, b), d in zip(shards, devices)]
    Ks = [mk(b - a, d) for (a, b), d in zip(shards, devices)]
    Vs = [mk(b - a, d) for (a, b), d in zip(shards, devices)]
    Os = [torch.zeros_like(q) for q in Qs]
    n = len(devices)
    vp = ctypes.c_void_p
    ptrs = lambda ts, bad=None: (vp * n)(*[vp(t.data_ptr() + (2 if i == bad else 0))
                                          for i, t in enumerate(ts)])
    rc = engine.lib().attn_fwd_sharded(n, (ctypes.c_int * n)(*devices), ptrs(Qs, bad=1),
                                       ptrs(Ks), ptrs(Vs), ptrs(Os), B, H, S, D, 0, 256, 128,
                                       None)
    assert rc == engine.ERR["MISALIGNED"]
    torch.cuda.synchronize()
    # shard 0 ran to completion and is correct; the rejected shard left O untouched
    ref0 = engine.attn(Qs[0], Ks[0], Vs[0])
    torch.cuda.synchronize()
    assert torch.equal(Os[0], ref0)
    assert torch.count_nonzero(Os[1]).item() == 0
