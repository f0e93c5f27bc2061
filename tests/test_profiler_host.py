"""Host-side post-processing of the phase profiler (no GPU): the per-phase
means, the iteration period, the trace phases of the second Q tile and the
MMA issuer, and the per-iteration timeline view, on synthetic clock64
stamps laid out like the kernel's buffer."""
import numpy as np

from attnprofile_b200 import profiler

PHASES = 17  # attn_profile_layout(): phases
SLOTS = 32


def synthetic(period=1000, n=12):
    """Stamps of a steady pipeline: SOFTMAX of tile 0 every `period` cycles,
    tile 1 offset by half a period, the issuer's windows and waits after them."""
    a = np.zeros((PHASES, SLOTS, 2), dtype=np.int64)
    sm = profiler.PHASES.index("SOFTMAX")
    pv = profiler.PHASES.index("GEMM-PV")
    exp = len(profiler.PHASES) + profiler.SUBPHASES.index("exp")
    base = profiler.TRACE_BASE
    for j in range(n):
        t = 10_000 + j * period
        a[sm, j] = (t, t + 600)
        a[exp, j] = (t + 100, t + 550)
        a[pv, j] = (t + 500, t + 900)
        a[base + 0, j] = (t + period // 2, t + period // 2 + 600)  # SOFTMAX-t1
        a[base + 1, j] = (t + 450, t + 800)                        # MMA-t0
        a[base + 2, j] = (t + 950, t + 1300)                       # MMA-t1
        a[base + 3, j] = (t + 300, t + period // 2 + 300)          # P-first t0 / t1
        a[base + 4, j] = (t + 400, t + 420)                        # V-wait
        a[base + 5, j] = (t + 700, t + 710)                        # K-wait
    return a


def test_summary_reports_period_and_trace_phases():
    r = profiler.summarize([synthetic(period=1000)])
    assert r["period"] == 1000
    assert r["SOFTMAX"] == 600 and r["exp"] == 450
    assert r["SOFTMAX-t1"] == 600
    assert r["MMA-t0"] == 350 and r["MMA-t1"] == 350
    assert r["P-first"] == 500  # tile 1's first P part half a period after tile 0's
    assert r["V-wait"] == 20 and r["K-wait"] == 10


def test_unstamped_slots_are_ignored():
    a = synthetic(n=4)
    a[:, 6] = 0  # a hole: iteration 6 never stamped
    r = profiler.summarize([a])
    assert np.isfinite(r["SOFTMAX"]) and r["SOFTMAX"] == 600


def test_timeline_is_relative_to_tile0_softmax():
    text = profiler.timeline(synthetic(period=1000), first=2, count=2)
    rows = [line for line in text.splitlines() if line.startswith("| 2 ") or line.startswith("| 3 ")]
    assert len(rows) == 4  # two iterations, both tiles
    t0, t1 = rows[0], rows[1]
    assert t0.startswith("| 2 | 0 | 0 .. 600 | 100 .. 550 | 300 |")
    assert t1.startswith("| 2 | 1 | 500 .. 1100 |")
    assert rows[2].startswith("| 3 | 0 | 1000 .. 1600 |")


def test_timeline_of_a_single_tile_cta_has_no_tile1_rows():
    a = synthetic(n=4)
    a[profiler.TRACE_BASE] = 0  # no second Q tile
    text = profiler.timeline(a, first=1, count=2)
    assert "| 1 | 1 |" not in text and "| 1 | 0 |" in text
