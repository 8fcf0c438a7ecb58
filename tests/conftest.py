"""Shared pytest setup: markers, import paths and golden-fixture access."""
from __future__ import annotations

import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
PKG_ROOT = REPO / "ss-grpo_b200"
GOLDEN = REPO / "tests" / "golden"
for p in (str(REPO), str(PKG_ROOT)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def golden_dir() -> Path:
    return GOLDEN


def cuda_available() -> bool:
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:  # pragma: no cover
        return False


def compare_stats(res: dict, want: dict, skip=("timing_sample_count",)):
    """Every deterministic statistic of the reference's generate result dict:
    counts exactly, rates within float rounding, histograms by key (JSON
    fixtures keep integer keys as strings)."""
    import math

    for k, v in want.items():
        if k in skip:
            continue
        assert k in res, k
        got = res[k]
        if isinstance(v, dict):
            assert {str(a): b for a, b in got.items()} == {str(a): b for a, b in v.items()}, (k, got, v)
        elif isinstance(v, float):
            assert math.isclose(got, v, rel_tol=1e-12, abs_tol=1e-12), (k, got, v)
        else:
            assert got == v, (k, got, v)
