"""Key-split of the last wave (attn_set_split / attn_query_split): parity of
every split count against the CPU oracle, bit-identical repeats, and the plan
chosen for the benchmark shapes.

A split unit runs as k CTAs over disjoint key ranges; each writes its
normalised partial O and (row max, row sum) to the workspace and the last to
finish merges them in a fixed order.  Same tolerance as every parity test:
max-abs 2e-3, mean-abs 2e-4 (bf16: one ulp of the reference value where that
is larger, as in test_gpu_attn.py).
"""
import numpy as np
import pytest

from tests.test_gpu_attn import MEAN_ABS, _torch, code, compare, make_inputs, to_u16

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _restore_split(engine):
    # These tests are about the classic schedule's key split; the persistent
    # schedule (tests/test_gpu_persistent.py) has its own plan.
    engine.set_schedule(1)
    yield
    engine.set_split(0)
    engine.set_schedule(0)


def run_mode(engine, q, k, v, BM, BN, mode):
    torch = _torch()
    engine.set_split(mode)
    Q, K, V = (x.cuda() for x in (q, k, v))
    O = engine.attn(Q, K, V, BM=BM, BN=BN)
    torch.cuda.synchronize()
    rc, site = engine.get_status(0)
    assert rc == 0, f"device status {site:#x}"
    return O.cpu()


@pytest.mark.parametrize("mode", [1, 2, 3, 4])
@pytest.mark.parametrize("BM,BN", [(256, 128), (128, 64), (128, 256), (256, 32)])
@pytest.mark.parametrize("S", [1000, 2048])
def test_split_parity_f16(engine, oracle_mod, mode, BM, BN, S):
    torch = _torch()
    q, k, v = make_inputs(1, 3, S, 128, torch.float16, seed=S + mode)
    out = run_mode(engine, q, k, v, BM, BN, mode)
    ref = oracle_mod.attention(to_u16(q), to_u16(k), to_u16(v), bn_tile=BN)
    mx, mean = compare(oracle_mod, to_u16(out), ref, 0)
    assert mx <= 1.0 and mean <= MEAN_ABS, (mx, mean)


@pytest.mark.parametrize("mode", [2, 3, 4])
@pytest.mark.parametrize("D", [64, 128])
def test_split_parity_bf16(engine, oracle_mod, mode, D):
    """D = 128 on 256 x 64 (two S buffers), D = 64 on 256 x 128 (one): the
    D = 64 two-buffer tiles run eight softmax warps and take no key split."""
    torch = _torch()
    BN = 64 if D == 128 else 128
    q, k, v = make_inputs(2, 2, 1500, D, torch.bfloat16, seed=D + mode)
    out = run_mode(engine, q, k, v, 256, BN, mode)
    plan = engine.query_split(2, 2, 1500, D, BM=256, BN=BN, dtype=1)  # under the forced mode
    assert plan["split"] > 1, plan
    ref = oracle_mod.attention(to_u16(q), to_u16(k), to_u16(v), bn_tile=BN, dtype=1)
    mx, mean = compare(oracle_mod, to_u16(out), ref, 1)
    assert mx <= 1.0 and mean <= MEAN_ABS, (mx, mean)


@pytest.mark.parametrize("mode", [0, 2, 4])
@pytest.mark.parametrize("BN", [96, 64])
def test_split_on_eight_warp_tiles(engine, oracle_mod, mode, BN):
    """The D = 64 two-buffer tiles run eight softmax warps per Q tile for
    whole units; a launch whose plan splits units along the keys (forced, or
    automatic on few long units: 1 x 2 x 4096 is 32 units for 148 SMs) runs
    the tile's four-warp kernel with the split, against the oracle."""
    torch = _torch()
    q, k, v = make_inputs(1, 2, 4096, 64, torch.float16, seed=mode + BN)
    out = run_mode(engine, q, k, v, 256, BN, mode)
    plan = engine.query_split(1, 2, 4096, 64, BM=256, BN=BN)  # under the same mode
    if torch.cuda.get_device_properties(0).multi_processor_count == 148:
        assert plan["split"] > 1, plan
    ref = oracle_mod.attention(to_u16(q), to_u16(k), to_u16(v), bn_tile=BN)
    mx, mean = compare(oracle_mod, to_u16(out), ref, 0)
    assert mx <= 1.0 and mean <= MEAN_ABS, (mx, mean)


def test_split_counts_above_the_tile_count_are_clamped(engine, oracle_mod):
    """S = 200 at BN = 128 has two key tiles: a forced 4-way split runs 2 ranges."""
    torch = _torch()
    q, k, v = make_inputs(1, 2, 200, 128, torch.float16, seed=3)
    out = run_mode(engine, q, k, v, 128, 128, 4)
    ref = oracle_mod.attention(to_u16(q), to_u16(k), to_u16(v), bn_tile=128)
    mx, mean = compare(oracle_mod, to_u16(out), ref, 0)
    assert mx <= 1.0 and mean <= MEAN_ABS, (mx, mean)


def test_split_repeats_bit_identical(engine):
    """The merge adds the parts in key order whichever part finishes last."""
    torch = _torch()
    q, k, v = make_inputs(1, 8, 4096, 128, torch.float16, seed=4)
    outs = [run_mode(engine, q, k, v, 256, 128, 4) for _ in range(4)]
    for o in outs[1:]:
        assert torch.equal(outs[0], o)


def test_split_agrees_with_unsplit_at_c2(engine):
    """1x16x4096x128: second wave split four ways against no split."""
    torch = _torch()
    g = torch.Generator(device="cuda").manual_seed(7)
    Q, K, V = (torch.randn(1, 16, 4096, 128, generator=g, device="cuda").half()
               for _ in range(3))
    outs = []
    for mode in (4, 1):
        engine.set_split(mode)
        outs.append(engine.attn(Q, K, V, BM=256, BN=128).float())
    torch.cuda.synchronize()
    assert engine.get_status(0)[0] == 0
    d = (outs[0] - outs[1]).abs()
    assert d.max().item() <= 2e-3 and d.mean().item() <= MEAN_ABS


def test_automatic_split_of_few_long_units(engine, oracle_mod):
    """1x2x8192 (64 units of 64 key tiles on a 148-SM B200): the automatic
    plan splits every unit in two; checked on a sample of rows against the
    oracle."""
    torch = _torch()
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    p = engine.query_split(1, 2, 8192, 128, BM=256, BN=128)
    if sms >= 128:
        assert p["split"] == 2 and p["whole"] == 0
    q, k, v = make_inputs(1, 2, 8192, 128, torch.float16, seed=8)
    out = run_mode(engine, q, k, v, 256, 128, 0)
    rows = np.sort(np.random.default_rng(8).choice(2 * 8192, size=96, replace=False))
    ref = oracle_mod.attention_rows(to_u16(q), to_u16(k), to_u16(v), rows, bn_tile=128)
    got = to_u16(out).reshape(-1, 128)[rows]
    mx, mean = compare(oracle_mod, got, ref, 0)
    assert mx <= 1.0 and mean <= MEAN_ABS, (mx, mean)


def test_plan_for_benchmark_shapes(engine):
    torch = _torch()
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    p = engine.query_split(1, 16, 4096, 128, BM=256, BN=128)
    units = 16 * 16
    assert p["whole"] + (units - p["whole"]) * p["split"] == p["ctas"]
    if sms == 148:
        assert p["split"] == 1 and p["workspace_bytes"] == 0
    assert engine.query_split(8, 32, 8192, 128, BM=256, BN=128, dtype=1)["split"] == 1
    engine.set_split(4)
    p = engine.query_split(1, 16, 4096, 128)
    if sms == 148:
        assert p["split"] == 4 and p["whole"] == 148
        # partial O in f32 (256 rows x 128) + (max, sum) per row, per part
        assert p["workspace_bytes"] >= 108 * 4 * 256 * (128 * 4 + 8)
    engine.set_split(1)
    assert engine.query_split(1, 1, 16384, 128)["split"] == 1


def test_split_padded_layout_writes_only_valid_rows(engine, oracle_mod):
    """attn_fwd_padded with a forced split: the merging part's TMA store goes
    through the padded map, rows >= S stay untouched."""
    torch = _torch()
    B, H, S, D, BM, BN = 1, 2, 300, 128, 256, 128
    SQO, SKV = 512, 384
    q, k, v = make_inputs(B, H, S, D, torch.float16, seed=15)
    Qp = torch.full((B, H, SQO, D), float("nan"), dtype=torch.float16)
    Kp = torch.full((B, H, SKV, D), float("nan"), dtype=torch.float16)
    Vp = torch.full((B, H, SKV, D), float("nan"), dtype=torch.float16)
    Qp[:, :, :S], Kp[:, :, :S], Vp[:, :, :S] = q, k, v
    Op = torch.full((B, H, SQO, D), 7.0, dtype=torch.float16).cuda()
    engine.set_split(3)
    try:
        engine.attn_padded(Qp.cuda(), Kp.cuda(), Vp.cuda(), Op, S, BM=BM, BN=BN)
        torch.cuda.synchronize()
    finally:
        engine.set_split(0)
    assert engine.get_status(0)[0] == 0
    O = Op.cpu()
    assert torch.all(O[:, :, S:] == 7.0), "padding rows of O were written"
    ref = oracle_mod.attention(to_u16(q), to_u16(k), to_u16(v), bn_tile=BN)
    mx, mean = compare(oracle_mod, to_u16(O[:, :, :S]), ref, 0)
    assert mx <= 1.0 and mean <= MEAN_ABS, (mx, mean)
