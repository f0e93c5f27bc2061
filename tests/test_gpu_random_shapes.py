"""Seeded random problems against the CPU oracle (tuning/utils.cuh:139-198),
through the C ABI on the GPU.

Each case draws (B, H, S), the head dimension, the dtype, a built tile
(BM x BN, CTA pairs included), the key-split mode, the schedule and the
correction-warpgroup mode, and the input scale, from a fixed seed, so the
set is the same on every run and covers combinations the targeted tests do
not list one by one: ragged S against every tile width, splits on one-,
two- and eight-warp tiles, the persistent and correction kernels on odd
shapes.  Bounds as everywhere: max-abs 2e-3, mean-abs 2e-4, bf16 with the
counted one-ulp exception of test_gpu_attn.compare.

One regime is held to another bound: bf16 with sharp attention (Q and K
scaled by 2, so logits of standard deviation ~4).  There the kernel's lazy
rescale rounds each row's dominant P relative to a stale maximum (P up to
2^8, not exactly representable), while the reference rounds it relative to
the exact maximum (P = 1, exact), so the two differ by up to about two bf16
ulps of O where |V| is near 1.  Those cases are compared with an exact fp64
attention instead: the kernel's error must stay within 2.5 times the
reference algorithm's own error (max) and 1.5 times it (mean).  Measured on
a B200 on these inputs: kernel 6.2-8.4e-3 max and 3.3-3.9e-4 mean, reference
3.9-4.1e-3 and 2.9-3.2e-4.
"""
import numpy as np
import pytest

from tests.test_gpu_attn import MEAN_ABS, _torch, code, compare, make_inputs, to_u16

pytestmark = pytest.mark.gpu

TILES = {64: [(128, 32), (128, 64), (128, 96), (128, 128), (128, 256), (256, 32), (256, 64),
              (256, 96), (256, 128)],
         128: [(128, 32), (128, 64), (128, 96), (128, 128), (128, 256), (256, 32), (256, 64),
               (256, 96), (256, 128), (512, 128)]}
N_CASES = 48


def draw(i):
    rng = np.random.default_rng(1000 + i)
    D = int(rng.choice([64, 128]))
    BM, BN = TILES[D][int(rng.integers(len(TILES[D])))]
    B = int(rng.integers(1, 3))
    H = int(rng.integers(1, 4))
    S = int(rng.integers(1, 1600))
    dt = str(rng.choice(["f16", "bf16"]))
    split = int(rng.choice([0, 0, 1, 2, 3, 4]))
    schedule = int(rng.choice([0, 0, 2]))
    corr = int(rng.choice([0, 0, 0, 1]))
    sigma = float(rng.choice([0.5, 1.0, 2.0]))
    return dict(B=B, H=H, S=S, D=D, BM=BM, BN=BN, dt=dt, split=split, schedule=schedule,
                corr=corr, sigma=sigma)


@pytest.fixture(autouse=True)
def _restore(engine):
    yield
    engine.set_split(0)
    engine.set_schedule(0)
    engine.set_correction(0)


@pytest.mark.parametrize("i", range(N_CASES))
def test_random_problem(engine, oracle_mod, i):
    c = draw(i)
    torch = _torch()
    dtype = torch.float16 if c["dt"] == "f16" else torch.bfloat16
    q, k, v = make_inputs(c["B"], c["H"], c["S"], c["D"], dtype, seed=2000 + i)
    if c["sigma"] != 1.0:
        q, k = ((x.float() * c["sigma"]).to(dtype) for x in (q, k))
    if c["sigma"] > 1.0:
        # Sharper attention puts O close to single rows of V: V is halved so
        # that |O| stays below 4, where one f16 ulp is still under 2e-3.
        v = (v.float() * 0.5).to(dtype)
    engine.set_split(c["split"])
    engine.set_schedule(c["schedule"])
    engine.set_correction(c["corr"])
    Q, K, V = (x.cuda() for x in (q, k, v))
    O = engine.attn(Q, K, V, BM=c["BM"], BN=c["BN"])
    torch.cuda.synchronize()
    rc, site = engine.get_status(0)
    assert rc == 0, (c, hex(site))
    ref = oracle_mod.attention(to_u16(q), to_u16(k), to_u16(v), bn_tile=c["BN"],
                               dtype=code(dtype))
    if c["dt"] == "bf16" and c["sigma"] > 1.0:
        qd, kd, vd = (x.double() for x in (q, k, v))
        exact = (torch.softmax(qd @ kd.transpose(-1, -2) / c["D"] ** 0.5, -1) @ vd).numpy()
        got = O.float().cpu().numpy().astype(np.float64)
        r = oracle_mod.to_f32(ref, 1).reshape(got.shape).astype(np.float64)
        e_k, e_r = np.abs(got - exact), np.abs(r - exact)
        assert e_k.max() <= 2.5 * e_r.max() and e_k.mean() <= 1.5 * e_r.mean(), (
            c, float(e_k.max()), float(e_r.max()), float(e_k.mean()), float(e_r.mean()))
        return
    mx, mean = compare(oracle_mod, to_u16(O.cpu()), ref, code(dtype))
    assert mx <= 1.0 and mean <= MEAN_ABS, (c, mx, mean)
