"""The persistent schedule (attn_set_schedule; two-tile variants with one S
buffer per tile) against the CPU oracle, on the GPU, through the C ABI.

Forced on (mode 2) for shapes that cut units between CTAs in every way the
planner produces -- one cut per CTA (1x16x4096), many pieces per unit
(1x2x8192: a unit spread over four CTAs), items of one key tile, ragged key
tails, D = 64, bf16, the padded layout -- and compared with the oracle
(tuning/utils.cuh:139-198) within the north-star bounds (max-abs 2e-3,
mean-abs 2e-4; bf16 with the counted one-ulp exception of
test_gpu_attn.compare).  Also: repeated launches are bit-identical (the
merge order is fixed), the classic and the persistent schedule agree, the
padding rows of O are never written, and the bounded waits of the persistent
roles report a timeout and leave the context usable.
"""
import numpy as np
import pytest

from tests.test_gpu_attn import MEAN_ABS, _torch, code, compare, make_inputs, to_u16

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _restore(engine):
    yield
    engine.set_schedule(0)
    engine.set_split(0)


def run(engine, q, k, v, BM, BN, schedule):
    torch = _torch()
    engine.set_schedule(schedule)
    Q, K, V = (x.cuda() for x in (q, k, v))
    O = engine.attn(Q, K, V, BM=BM, BN=BN)
    torch.cuda.synchronize()
    rc, site = engine.get_status(0)
    assert rc == 0, f"device status {site:#x}"
    return O.cpu()


SHAPES = [
    # B, H, S, D, dtype, BM, BN
    (1, 2, 512, 128, "f16", 256, 128),
    (1, 3, 1000, 128, "f16", 256, 128),
    (3, 7, 129, 128, "f16", 256, 128),
    (1, 2, 2048, 128, "bf16", 256, 128),
    (2, 5, 333, 64, "f16", 256, 128),
    (1, 4, 1536, 64, "bf16", 256, 128),
    (1, 2, 1000, 128, "f16", 256, 96),
    (1, 1, 4096, 128, "f16", 256, 96),
]


@pytest.mark.parametrize("B,H,S,D,dt,BM,BN", SHAPES)
def test_persistent_parity(engine, oracle_mod, B, H, S, D, dt, BM, BN):
    torch = _torch()
    dtype = torch.float16 if dt == "f16" else torch.bfloat16
    q, k, v = make_inputs(B, H, S, D, dtype, seed=S + H + D)
    plan = engine.query_split(B, H, S, D, BM=BM, BN=BN, dtype=code(dtype))
    out = run(engine, q, k, v, BM, BN, 2)
    ref = oracle_mod.attention(to_u16(q), to_u16(k), to_u16(v), bn_tile=BN, dtype=code(dtype))
    mx, mean = compare(oracle_mod, to_u16(out), ref, code(dtype))
    assert mx <= 1.0 and mean <= MEAN_ABS, (plan, mx, mean)


@pytest.mark.parametrize("B,H,S", [(1, 16, 4096), (1, 2, 8192), (1, 1, 16384)])
def test_persistent_parity_cut_units_sampled(engine, oracle_mod, B, H, S):
    """Shapes whose units are cut between CTAs (the plan has pieces > 1):
    every (batch, head) checked on 64 sampled rows, which include the rows of
    every 128-row Q tile of the cut units' first and last key ranges."""
    torch = _torch()
    engine.set_schedule(2)
    plan = engine.query_split(B, H, S, 128)
    if torch.cuda.get_device_properties(0).multi_processor_count == 148:
        assert plan["split"] > 1, plan
    g = torch.Generator(device="cuda").manual_seed(S + H)
    Q, K, V = (torch.randn(B, H, S, 128, generator=g, device="cuda").half() for _ in range(3))
    O = engine.attn(Q, K, V, BM=256, BN=128)
    torch.cuda.synchronize()
    assert engine.get_status(0)[0] == 0
    rng = np.random.default_rng(S)
    rows = np.unique(np.concatenate([u * S + rng.choice(S, 64, replace=False)
                                     for u in range(B * H)]).astype(np.int64))
    u16 = lambda t: t.view(torch.int16).cpu().numpy().view(np.uint16)
    ref = oracle_mod.attention_rows(u16(Q), u16(K), u16(V), rows, bn_tile=128)
    got = u16(O).reshape(-1, 128)[rows]
    mx, mean = compare(oracle_mod, got, ref, 0)
    assert mx <= 1.0 and mean <= MEAN_ABS, (plan, mx, mean)


def test_persistent_repeats_bit_identical_and_matches_classic(engine):
    torch = _torch()
    q, k, v = make_inputs(1, 16, 4096, 128, torch.float16, seed=77)
    a = run(engine, q, k, v, 256, 128, 2)
    b = run(engine, q, k, v, 256, 128, 2)
    c = run(engine, q, k, v, 256, 128, 1)
    assert torch.equal(a, b)
    d = (a.float() - c.float()).abs()
    assert d.max().item() <= 2e-3 and d.mean().item() <= MEAN_ABS / 10


def test_persistent_padded_layout_writes_only_valid_rows(engine, oracle_mod):
    torch = _torch()
    engine.set_schedule(2)
    B, H, S, D, BN = 1, 3, 700, 128, 128
    SQO, SKV = 768, 768
    q, k, v = make_inputs(B, H, S, D, torch.float16, seed=8)
    Qp = torch.full((B, H, SQO, D), float("nan"), dtype=torch.float16)
    Kp, Vp = Qp.clone(), Qp.clone()
    Qp[:, :, :S], Kp[:, :, :S], Vp[:, :, :S] = q, k, v
    Op = torch.full((B, H, SQO, D), 7.0, dtype=torch.float16).cuda()
    engine.attn_padded(Qp.cuda(), Kp.cuda(), Vp.cuda(), Op, S, BM=256, BN=BN)
    torch.cuda.synchronize()
    assert engine.get_status(0)[0] == 0
    O = Op.cpu()
    assert torch.all(O[:, :, S:] == 7.0), "padding rows of O were written"
    ref = oracle_mod.attention(to_u16(q), to_u16(k), to_u16(v), bn_tile=BN)
    mx, mean = compare(oracle_mod, to_u16(O[:, :, :S]), ref, 0)
    assert mx <= 1.0 and mean <= MEAN_ABS


def test_persistent_bounded_waits_time_out_and_context_survives(engine):
    """attn_debug_fault(1): the producer loads the first item's Q and never
    K/V, so every role's bounded wait expires (no fault, no hang); the next
    normal launch is correct.  Run on a shape whose CTAs hold several items
    and cut units, so the merger's bounded wait for its writers is reached
    too when the writers time out first."""
    torch = _torch()
    engine.set_schedule(2)
    g = torch.Generator(device="cuda").manual_seed(1)
    Q, K, V = (torch.randn(1, 16, 4096, 128, generator=g, device="cuda").half() for _ in range(3))
    engine.get_status(0, reset=True)
    engine.set_timeout_ns(50_000_000)
    try:
        engine.debug_fault(1)
        engine.attn(Q, K, V, BM=256, BN=128)
        rc, site = engine.get_status(0, reset=True)
        assert rc == engine.ERR["DEVICE_TIMEOUT"] and site & 0xFF00 == 0x7100, (rc, hex(site))
    finally:
        engine.debug_fault(0)
        engine.set_timeout_ns(2_000_000_000)
    O = engine.attn(Q, K, V, BM=256, BN=128)
    torch.cuda.synchronize()
    assert engine.get_status(0)[0] == 0
    ref = torch.softmax((Q[0, :2].float() @ K[0, :2].float().transpose(-1, -2)) / 128 ** 0.5,
                        -1) @ V[0, :2].float()
    assert (O[0, :2].float() - ref).abs().max().item() < 2e-3
