"""The CPU oracle against the reference's own outputs (no GPU).

tests/golden/*.npz hold inputs drawn by the reference's verify_attn
(std::mt19937(42), tuning/utils.cuh:95-118) and the output hORef that the
reference's host attention (tuning/utils.cuh:139-198) computed for them; see
tests/golden/gen_golden.py.  The restatement in oracle/attn_oracle.c must
reproduce them bit for bit.
"""
from pathlib import Path

import numpy as np
import pytest

GOLDEN = sorted((Path(__file__).parent / "golden").glob("*.npz"))


def test_golden_fixtures_present():
    assert len(GOLDEN) >= 4


@pytest.mark.parametrize("path", GOLDEN, ids=lambda p: p.stem)
def test_oracle_bit_exact_vs_reference(oracle_mod, path):
    z = np.load(path)
    B, H, S, D, BM, BN = (int(x) for x in z["meta"])
    out = oracle_mod.attention(z["q"], z["k"], z["v"], bn_tile=BN, nthreads=2)
    assert out.shape == (B, H, S, D)
    assert np.array_equal(out, z["o_ref"])


@pytest.mark.parametrize("path", GOLDEN, ids=lambda p: p.stem)
def test_oracle_single_thread_equals_threaded(oracle_mod, path):
    z = np.load(path)
    BN = int(z["meta"][5])
    a = oracle_mod.attention(z["q"], z["k"], z["v"], bn_tile=BN, nthreads=1)
    b = oracle_mod.attention(z["q"], z["k"], z["v"], bn_tile=BN, nthreads=4)
    assert np.array_equal(a, b)


def test_oracle_rows_match_full(oracle_mod):
    z = np.load(next(p for p in GOLDEN if p.stem.startswith("b1h2")))
    B, H, S, D, BM, BN = (int(x) for x in z["meta"])
    full = oracle_mod.attention(z["q"], z["k"], z["v"], bn_tile=BN)
    rows = np.array([0, 1, S - 1, S, B * H * S - 1], dtype=np.int64)
    sel = oracle_mod.attention_rows(z["q"], z["k"], z["v"], rows, bn_tile=BN)
    flat = full.reshape(-1, D)
    assert np.array_equal(sel, flat[rows])


def test_planted_mistake_is_caught(oracle_mod):
    """A checker that cannot fail proves nothing: a one-ulp change to one key
    element must change the oracle's output (and so fail the golden match)."""
    z = np.load(GOLDEN[0])
    BN = int(z["meta"][5])
    k = z["k"].copy()
    k[0, 0, 3, 5] ^= 1  # flip the lowest mantissa bit
    out = oracle_mod.attention(z["q"], k, z["v"], bn_tile=BN)
    assert not np.array_equal(out, z["o_ref"])


def test_tile_width_matters_to_the_bit(oracle_mod):
    """The key tile of the online softmax is part of the reference's rounding
    (P is rounded per tile against the running max): another tile width must
    not reproduce the golden bits exactly, while staying within 1e-3."""
    z = np.load(GOLDEN[0])
    BN = int(z["meta"][5])
    other = oracle_mod.attention(z["q"], z["k"], z["v"], bn_tile=BN * 2)
    assert not np.array_equal(other, z["o_ref"])
    a = oracle_mod.to_f32(other, 0)
    b = oracle_mod.to_f32(z["o_ref"], 0)
    assert np.abs(a - b).max() < 1e-3


def test_f16_conversion_exhaustive(oracle_mod):
    """fp32 -> fp16 RNE of the oracle equals numpy's on all fp16 values, their
    midpoints and a random sample of fp32 bit patterns."""
    L = oracle_mod.lib()
    h = np.arange(0, 1 << 16, dtype=np.uint32).astype(np.uint16)
    f = h.view(np.float16).astype(np.float32)
    finite = np.isfinite(f)
    back = np.array([L.oracle_f16_to_f32(int(x)) for x in h[finite][::7]], dtype=np.float32)
    assert np.array_equal(back, f[finite][::7])
    rng = np.random.default_rng(1)
    bits = rng.integers(0, 1 << 32, size=20000, dtype=np.uint64).astype(np.uint32)
    vals = bits.view(np.float32)
    vals = vals[np.isfinite(vals)]
    ours = np.array([L.oracle_f32_to_f16(float(v)) for v in vals], dtype=np.uint16)
    with np.errstate(over="ignore"):
        ref = vals.astype(np.float16).view(np.uint16)
    assert np.array_equal(ours, ref)


def test_bf16_conversion_matches_numpy_rne(oracle_mod):
    L = oracle_mod.lib()
    rng = np.random.default_rng(2)
    vals = rng.standard_normal(5000).astype(np.float32) * 10
    ours = np.array([L.oracle_f32_to_bf16(float(v)) for v in vals], dtype=np.uint16)
    ref = oracle_mod.from_f32(vals, 1)
    assert np.array_equal(ours, ref)
