import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 GPU")


def gpu_available() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def engine():
    """The built engine package (builds libattnprof.so in-tree if stale)."""
    import attnprofile_b200 as ap
    ap.build()
    return ap


@pytest.fixture(scope="session")
def oracle_mod():
    from oracle import oracle
    oracle.build()
    return oracle


def pytest_terminal_summary(terminalreporter):
    """Reports how often the bf16 one-ulp exception of the parity checks was
    used (tests/test_gpu_attn.py::compare) in this session."""
    # The module can be loaded under two names (as collected, and as
    # imported by tests/test_gpu_split.py): add both counts up.
    mods = {id(m): m for m in (sys.modules.get("test_gpu_attn"),
                               sys.modules.get("tests.test_gpu_attn")) if m is not None}
    parts = [m.ULP_EXCEPTIONS for m in mods.values() if hasattr(m, "ULP_EXCEPTIONS")]
    if not parts:
        return
    stats = {k: sum(p[k] for p in parts) for k in ("compared", "bf16_compared", "exceptions")}
    stats.update({k: max(p[k] for p in parts) for k in ("max_excess", "worst_share")})
    if stats["compared"]:
        terminalreporter.write_line(
            "parity: {compared} elements compared ({bf16_compared} bf16); {exceptions} passed "
            "only through the bf16 one-ulp exception (largest |diff| {max_excess:.3g}, largest "
            "share in one comparison {worst_share:.2e})".format(**stats))
