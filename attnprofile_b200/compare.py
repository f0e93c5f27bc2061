"""Comparison point: the same attention forward through attention kernels
installed on the box (torch SDPA backends -- cuDNN, flash, memory-efficient --,
flashinfer's single-prefill kernels, flash_attn 2.8), timed with CUDA events
next to attnprofile_b200.attn on the same inputs.  Library code is only timed
here, never used by the engine.  Prints TFLOP/s (4*B*H*S^2*D / t) and each
library's max |difference| to this engine's output.

    python -m attnprofile_b200.compare c2,c3,c5s,c4s
"""
from __future__ import annotations

import sys
import time

# BASELINE configurations; c4s / c5s are the per-GPU shards of C4 / C5 at 4 GPUs.
SHAPES = {
    "c2": (1, 16, 4096, 128, "f16"),
    "c3": (1, 16, 4096, 64, "f16"),
    "c4s": (2, 32, 8192, 128, "bf16"),
    "c5s": (1, 16, 32768, 128, "f16"),
}


def _time(fn, n: int) -> float:
    """Best of three runs of n calls, ms per call (CUDA events)."""
    import torch
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    best = float("inf")
    for _ in range(3):
        a.record()
        for _ in range(n):
            fn()
        b.record()
        torch.cuda.synchronize()
        best = min(best, a.elapsed_time(b) / n)
    return best


def compare(name: str) -> dict:
    import torch
    import torch.nn.functional as F
    from torch.nn.attention import SDPBackend, sdpa_kernel

    import attnprofile_b200 as ap

    B, H, S, D, dt = SHAPES[name]
    dtype = torch.float16 if dt == "f16" else torch.bfloat16
    q, k, v = (torch.randn(B, H, S, D, device="cuda").to(dtype) for _ in range(3))
    n = 20 if S <= 4096 else 3
    ref = ap.attn(q, k, v)
    maxdiff = lambda o: (o.float() - ref.float()).abs().max().item()
    out = {"attnprofile_b200": (_time(lambda: ap.attn(q, k, v), n), 0.0)}

    for be in (SDPBackend.CUDNN_ATTENTION, SDPBackend.FLASH_ATTENTION,
               SDPBackend.EFFICIENT_ATTENTION):
        try:
            with sdpa_kernel([be]):
                err = maxdiff(F.scaled_dot_product_attention(q, k, v))
                out[f"torch sdpa {be.name.lower()}"] = (
                    _time(lambda: F.scaled_dot_product_attention(q, k, v), n), err)
        except Exception as e:  # backend not available for this device / shape
            out[f"torch sdpa {be.name.lower()}"] = str(e).splitlines()[0][:100]

    if B == 1:
        try:
            import flashinfer
            qn = q[0].transpose(0, 1).contiguous()  # [S, H, D]
            kk, vv = k[0].contiguous(), v[0].contiguous()  # [H, S, D]
            run = lambda: flashinfer.single_prefill_with_kv_cache(qn, kk, vv, causal=False,
                                                                  kv_layout="HND", backend="fa2")
            t0 = time.time()
            err = (run().transpose(0, 1).float() - ref[0].float()).abs().max().item()
            out[f"flashinfer fa2 (JIT {time.time() - t0:.0f} s)"] = (_time(run, n), err)
        except Exception as e:
            out["flashinfer fa2"] = str(e).splitlines()[0][:100]

    try:
        from flash_attn import flash_attn_func
        qt, kt, vt = (x.transpose(1, 2).contiguous() for x in (q, k, v))  # [B, S, H, D]
        err = maxdiff(flash_attn_func(qt, kt, vt).transpose(1, 2))
        out["flash_attn 2.8"] = (_time(lambda: flash_attn_func(qt, kt, vt), n), err)
    except Exception as e:
        out["flash_attn 2.8"] = str(e).splitlines()[0][:100]

    flop = 4 * B * H * S * S * D
    return {k_: (v_ if isinstance(v_, str) else (v_[0], flop / v_[0] / 1e9, v_[1]))
            for k_, v_ in out.items()}


def main(names) -> None:
    for name in names:
        for impl, r in compare(name).items():
            if isinstance(r, str):
                print(f"{name:4s} {impl:36s} n/a: {r}", flush=True)
            else:
                print(f"{name:4s} {impl:36s} {r[0] * 1e3:9.1f} us {r[1]:8.1f} TFLOP/s "
                      f"max|diff| {r[2]:.1e}", flush=True)


if __name__ == "__main__":
    main(sys.argv[1].split(",") if len(sys.argv) > 1 else list(SHAPES))
