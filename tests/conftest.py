import os
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def _cuda_available() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if _cuda_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def cuda_lib():
    """Built C-ABI library (built on first use)."""
    from vlcache_b200 import build as _build
    _build.build()
    from vlcache_b200._lib import lib
    return lib()


# ---------------------------------------------------------------- error margins
# Attention tests record their measured error against the tolerance here; the table is
# printed at the end of every session (also under -q), so the margins are on record.
_MARGINS: list[tuple[str, str, float, float, float, float]] = []


def record_margin(test: str, what: str, max_abs: float, mean_abs: float, tol_max: float = 2e-2,
                  tol_mean: float = 2e-3) -> None:
    _MARGINS.append((test, what, float(max_abs), float(mean_abs), tol_max, tol_mean))


@pytest.fixture
def margins(request):
    """``margins(what, max_abs, mean_abs)`` records an error measurement of this test."""
    def rec(what, max_abs, mean_abs, tol_max=2e-2, tol_mean=2e-3):
        record_margin(request.node.name, what, max_abs, mean_abs, tol_max, tol_mean)
    return rec


def pytest_terminal_summary(terminalreporter, exitstatus, config):
    if not _MARGINS:
        return
    tr = terminalreporter
    tr.section("attention error margins (max-abs / mean-abs vs tolerance)")
    for test, what, mx, mean, tmx, tmean in _MARGINS:
        tr.write_line(f"{test:<60s} {what:<34s} max {mx:.3e} ({mx / tmx:5.1%} of {tmx:g})  "
                      f"mean {mean:.3e} ({mean / tmean:5.1%} of {tmean:g})")
