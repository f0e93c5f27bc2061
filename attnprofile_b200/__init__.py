"""attnprofile_b200 -- B200 (sm_100a) attention forward engine.

Python face of the C ABI in include/attnprof.h (libattnprof.so, built in-tree
from attnprofile_b200/csrc).  Tensors are torch CUDA tensors laid out
[B, H, S, D] (f16 or bf16); the work runs on the current CUDA stream.

There is no CPU or PyTorch fallback: if the CUDA library is missing or the
device cannot run it, every call raises.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

from ._build import LIB_PATH, build  # noqa: F401

__all__ = [
    "AttnError", "attn", "attn_padded", "attn_profiled", "query_config", "get_status",
    "set_timeout_ns", "debug_fault", "lib", "build", "ERR", "SUPPORTED_TILES", "PAIR_TILES",
    "attn_sharded",
    "shard_range", "set_split", "set_schedule", "plan_split", "plan_schedule", "query_split",
    "set_correction",
]

ERR = {
    "OK": 0, "INVALID_ARG": -1, "UNSUPPORTED": -2, "MISALIGNED": -3, "CUDA": -4,
    "TENSOR_MAP": -5, "DEVICE_TIMEOUT": -6, "RESOURCE": -7, "SHARD": -8, "SCRATCH_LIMIT": -9,
}
DTYPE_F16 = 0
DTYPE_BF16 = 1
SUPPORTED_TILES = [(128, 32), (128, 64), (128, 96), (128, 128), (128, 256), (256, 32), (256, 64),
                   (256, 96), (256, 128)]
# D = 128 only: a cluster of two 256-row CTAs sharing every K/V tile through
# cta_group::2 (2-SM) tensor-core MMAs.
PAIR_TILES = [(512, 128)]

_lib = None


class AttnError(RuntimeError):
    def __init__(self, code: int, what: str = ""):
        self.code = code
        msg = lib().attn_error_string(code).decode()
        super().__init__(f"{what}: {msg} (code {code})" if what else f"{msg} (code {code})")


def lib() -> ctypes.CDLL:
    """Load libattnprof.so (raises if it has not been built).  ATTNPROF_LIB may
    name another build of the same library (e.g. one compiled with other
    tuning macros)."""
    global _lib
    if _lib is None:
        import os
        path = Path(os.environ.get("ATTNPROF_LIB", str(LIB_PATH)))
        if not path.exists():
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python -m attnprofile_b200._build` "
                "(there is no CPU fallback)")
        L = ctypes.CDLL(str(path))
        vp, i, u64p = ctypes.c_void_p, ctypes.c_int, ctypes.POINTER(ctypes.c_ulonglong)
        L.attn_fwd.argtypes = [vp, vp, vp, vp, i, i, i, i, i, i, i, vp]
        L.attn_fwd_padded.argtypes = [vp, vp, vp, vp, i, i, i, i, i, i, i, i, i, vp]
        L.attn_fwd_profiled.argtypes = [vp, vp, vp, vp, i, i, i, i, i, i, i, vp, u64p, i]
        L.attn_fwd_sharded.argtypes = [i, ctypes.POINTER(i), ctypes.POINTER(vp),
                                       ctypes.POINTER(vp), ctypes.POINTER(vp), ctypes.POINTER(vp),
                                       i, i, i, i, i, i, i, ctypes.POINTER(ctypes.c_float)]
        L.attn_shard_range.argtypes = [i, i, i, ctypes.POINTER(i), ctypes.POINTER(i)]
        L.attn_get_status.argtypes = [i, i, ctypes.POINTER(i)]
        L.attn_set_timeout_ns.argtypes = [ctypes.c_ulonglong]
        L.attn_set_timeout_ns.restype = None
        L.attn_query_config.argtypes = [i, i, i, i] + [ctypes.POINTER(i)] * 4
        L.attn_profile_layout.argtypes = [ctypes.POINTER(i), ctypes.POINTER(i)]
        L.attn_error_string.argtypes = [i]
        L.attn_error_string.restype = ctypes.c_char_p
        L.attn_debug_fault.argtypes = [i]
        ll, llp = ctypes.c_longlong, ctypes.POINTER(ctypes.c_longlong)
        L.attn_set_split.argtypes = [i]
        L.attn_set_schedule.argtypes = [i]
        L.attn_set_correction.argtypes = [i]
        L.attn_plan_schedule.argtypes = [ll, i, ll, ctypes.POINTER(i), llp, ctypes.POINTER(i),
                                         ctypes.POINTER(ctypes.c_double),
                                         ctypes.POINTER(ctypes.c_double)]
        L.attn_plan_split.argtypes = [ll, i, ll, i, ctypes.POINTER(i), llp, llp]
        L.attn_query_split.argtypes = [i, i, i, i, i, i, i, ctypes.POINTER(i), llp, llp, u64p]
        for name in ("attn_fwd", "attn_fwd_padded", "attn_fwd_profiled", "attn_fwd_sharded",
                     "attn_shard_range", "attn_get_status", "attn_query_config",
                     "attn_profile_layout", "attn_debug_fault", "attn_version",
                     "attn_set_split", "attn_plan_split", "attn_query_split",
                     "attn_set_schedule", "attn_plan_schedule", "attn_set_correction"):
            getattr(L, name).restype = ctypes.c_int
        _lib = L
    return _lib


def _check(rc: int, what: str) -> None:
    if rc != 0:
        raise AttnError(rc, what)


def _dtype_code(t) -> int:
    import torch
    if t.dtype == torch.float16:
        return DTYPE_F16
    if t.dtype == torch.bfloat16:
        return DTYPE_BF16
    raise TypeError(f"unsupported dtype {t.dtype} (float16 or bfloat16)")


def _stream_ptr(stream) -> int:
    import torch
    s = torch.cuda.current_stream() if stream is None else stream
    return int(s.cuda_stream)


def _check_tensors(Q, K, V, O):
    for name, t in (("Q", Q), ("K", K), ("V", V), ("O", O)):
        if not t.is_cuda:
            raise ValueError(f"{name} must be a CUDA tensor")
        if t.dim() != 4 or not t.is_contiguous():
            raise ValueError(f"{name} must be a contiguous [B, H, rows, D] tensor")
        if t.dtype != Q.dtype:
            raise TypeError("Q, K, V, O must share one dtype")


def attn(Q, K, V, O=None, *, BM: int = 256, BN: int = 128, stream=None):
    """O = softmax(Q K^T / sqrt(D)) V for contiguous [B, H, S, D] tensors.

    Asynchronous on `stream` (default: current stream).  Returns O."""
    import torch
    if O is None:
        O = torch.empty_like(Q)
    _check_tensors(Q, K, V, O)
    B, H, S, D = Q.shape
    if K.shape != Q.shape or V.shape != Q.shape or O.shape != Q.shape:
        raise ValueError("Q, K, V, O must have the same [B, H, S, D] shape")
    rc = lib().attn_fwd(Q.data_ptr(), K.data_ptr(), V.data_ptr(), O.data_ptr(), B, H, S, D,
                        _dtype_code(Q), BM, BN, _stream_ptr(stream))
    _check(rc, "attn_fwd")
    return O


def attn_padded(Q, K, V, O, S: int, *, BM: int = 256, BN: int = 128, stream=None):
    """The reference's padded layout: Q/O [B, H, SQO, D], K/V [B, H, SKV, D],
    SQO, SKV >= S.  Rows >= S are neither read nor written."""
    _check_tensors(Q, K, V, O)
    B, H, SQO, D = Q.shape
    SKV = K.shape[2]
    rc = lib().attn_fwd_padded(Q.data_ptr(), K.data_ptr(), V.data_ptr(), O.data_ptr(), B, H, S,
                               D, SQO, SKV, _dtype_code(Q), BM, BN, _stream_ptr(stream))
    _check(rc, "attn_fwd_padded")
    return O


def profile_layout() -> tuple[int, int]:
    p, s = ctypes.c_int(), ctypes.c_int()
    lib().attn_profile_layout(ctypes.byref(p), ctypes.byref(s))
    return p.value, s.value


def attn_profiled(Q, K, V, O=None, *, BM: int = 256, BN: int = 128, cta: int = 0, stream=None):
    """One launch of the profiler-enabled variant; returns (O, stamps) where
    stamps is an int64 CPU tensor [phases, 32 slots, 2] of clock64 values
    (0 = not recorded; geometry from profile_layout()).  Phases: LoadQ, LoadK,
    LoadV, GEMM-QK, SOFTMAX, GEMM-PV, then the SOFTMAX steps S-ld, max, exp,
    P-st (slots = KV iterations), then Epilogue (slots = steps,
    profiler.EPILOGUE_STEPS), then the trace phases (profiler.TRACE_PHASES)."""
    import torch
    if O is None:
        O = torch.empty_like(Q)
    _check_tensors(Q, K, V, O)
    B, H, S, D = Q.shape
    phases, slots = profile_layout()
    buf = torch.zeros(phases * slots * 2, dtype=torch.int64, device=Q.device)
    rc = lib().attn_fwd_profiled(
        Q.data_ptr(), K.data_ptr(), V.data_ptr(), O.data_ptr(), B, H, S, D, _dtype_code(Q), BM,
        BN, _stream_ptr(stream), ctypes.cast(buf.data_ptr(), ctypes.POINTER(ctypes.c_ulonglong)),
        cta)
    _check(rc, "attn_fwd_profiled")
    return O, buf.view(phases, slots, 2).cpu()


def query_config(D: int, BM: int, BN: int, dtype: int = DTYPE_F16) -> dict:
    """Launch geometry of one variant: threads, smem bytes, TMEM columns, ring depth."""
    vals = [ctypes.c_int() for _ in range(4)]
    rc = lib().attn_query_config(D, BM, BN, dtype, *[ctypes.byref(v) for v in vals])
    _check(rc, "attn_query_config")
    return dict(zip(("num_threads", "smem_bytes", "tmem_cols", "stages"), (v.value for v in vals)))


def get_status(device: int = 0, reset: bool = True) -> tuple[int, int]:
    """Synchronise `device`; return (rc, raw site code) of the bounded-wait status word."""
    site = ctypes.c_int(0)
    rc = lib().attn_get_status(device, 1 if reset else 0, ctypes.byref(site))
    return rc, site.value


def set_timeout_ns(ns: int) -> None:
    lib().attn_set_timeout_ns(int(ns))


def debug_fault(mode: int) -> None:
    _check(lib().attn_debug_fault(mode), "attn_debug_fault")


def attn_sharded(Qs, Ks, Vs, Os, devices, *, B: int, H: int, BM: int = 256, BN: int = 128):
    """(batch, head)-sharded attention over several GPUs of this process.

    Qs[g] etc. hold GPU g's units contiguously ([1, units_g, S, D] on
    devices[g]; units_g from shard_range(B*H, len(devices), g)).  Launches on
    every device, joins them all, and raises AttnError with the first error.
    Returns the per-device kernel times in ms."""
    n = len(devices)
    S, D = Qs[0].shape[2], Qs[0].shape[3]
    vp = ctypes.c_void_p
    arr = lambda ts: (vp * n)(*[vp(t.data_ptr()) for t in ts])
    devs = (ctypes.c_int * n)(*devices)
    ms = (ctypes.c_float * n)()
    rc = lib().attn_fwd_sharded(n, devs, arr(Qs), arr(Ks), arr(Vs), arr(Os), B, H, S, D,
                                _dtype_code(Qs[0]), BM, BN, ms)
    _check(rc, "attn_fwd_sharded")
    return list(ms)


def set_split(mode: int) -> None:
    """Key split of the last wave for later launches: 0 automatic (default),
    1 never, 2..4 force that many key ranges per unit of the last wave."""
    _check(lib().attn_set_split(int(mode)), "attn_set_split")


def set_schedule(mode: int) -> None:
    """Schedule of later launches: 0 automatic (default; runs the classic
    schedule), 1 classic (one CTA per unit), 2 persistent wherever the tile
    has it (one resident CTA per SM slot sharing the launch's (unit, key
    tile) steps)."""
    _check(lib().attn_set_schedule(int(mode)), "attn_set_schedule")


def set_correction(mode: int) -> None:
    """1: later launches run with a correction warpgroup where the tile has
    one (BM 256 with BN 128, and 256 x 96 at D = 64), which owns the lazy O
    rescale, the final normalisation and the TMA store of O (classic
    schedule, no key split); 0 (default): the softmax warpgroups do that."""
    _check(lib().attn_set_correction(int(mode)), "attn_set_correction")


def plan_schedule(units: int, num_kv_tiles: int, slots: int) -> dict:
    """The host planner alone (no GPU): whether the automatic mode picks the
    persistent schedule (it does not), the persistent grid and the most
    pieces a unit is cut into, with both schedules' modelled costs."""
    pers, ctas, pieces = ctypes.c_int(), ctypes.c_longlong(), ctypes.c_int()
    cp, cc = ctypes.c_double(), ctypes.c_double()
    _check(lib().attn_plan_schedule(units, num_kv_tiles, slots, ctypes.byref(pers),
                                    ctypes.byref(ctas), ctypes.byref(pieces), ctypes.byref(cp),
                                    ctypes.byref(cc)), "attn_plan_schedule")
    return {"persistent": bool(pers.value), "ctas": ctas.value, "pieces": pieces.value,
            "persistent_cost": cp.value, "classic_cost": cc.value}


def plan_split(units: int, num_kv_tiles: int, slots: int, mode: int = 0) -> dict:
    """The host planner alone (no GPU): how `units` (B*H*ceil(S/BM)) units
    with `num_kv_tiles` key tiles each run on `slots` resident CTAs."""
    k, whole, ctas = ctypes.c_int(), ctypes.c_longlong(), ctypes.c_longlong()
    _check(lib().attn_plan_split(units, num_kv_tiles, slots, mode, ctypes.byref(k),
                                 ctypes.byref(whole), ctypes.byref(ctas)), "attn_plan_split")
    return {"split": k.value, "whole": whole.value, "ctas": ctas.value}


def query_split(B: int, H: int, S: int, D: int, *, BM: int = 256, BN: int = 128,
                dtype: int = DTYPE_F16) -> dict:
    """The plan a launch of this shape uses on the current device, with its
    workspace size in bytes (needs a GPU)."""
    k, whole, ctas = ctypes.c_int(), ctypes.c_longlong(), ctypes.c_longlong()
    ws = ctypes.c_ulonglong()
    _check(lib().attn_query_split(B, H, S, D, dtype, BM, BN, ctypes.byref(k), ctypes.byref(whole),
                                  ctypes.byref(ctas), ctypes.byref(ws)), "attn_query_split")
    return {"split": k.value, "whole": whole.value, "ctas": ctas.value,
            "workspace_bytes": ws.value}


def shard_range(units: int, n_dev: int, g: int) -> tuple[int, int]:
    """Units [begin, end) owned by GPU g under the (batch, head) partition."""
    b, e = ctypes.c_int(), ctypes.c_int()
    _check(lib().attn_shard_range(units, n_dev, g, ctypes.byref(b), ctypes.byref(e)),
           "attn_shard_range")
    return b.value, e.value
