"""Shared fixtures. GPU tests carry @pytest.mark.gpu and call the CUDA library
through its C ABI (rabbit_b200.capi); CPU tests cover the oracle, the golden
fixtures, host logic and the ABI surface."""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

# Stated numeric contract for fp32 outputs (expert and layer outputs).
RTOL = 1e-4
ATOL = 1e-5


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200) device")


@pytest.fixture(scope="session")
def oracle():
    from oracle.oracle import Oracle

    return Oracle()


@pytest.fixture(scope="session")
def reference():
    from oracle.oracle import Reference, REF_SO, build_reference

    if not REF_SO.exists() and build_reference() is None:
        pytest.skip("reference C (oracle/_ref) not built and sources unavailable")
    return Reference()


@pytest.fixture(scope="session")
def rc():
    """The CUDA library; on a GPU box this must load (no fallback)."""
    from rabbit_b200 import capi

    capi.lib()
    return capi


def near_tie(scores: np.ndarray, k: int, rel: float = 1e-6) -> bool:
    """True if the top-k selection or its order could flip on last-ulp changes."""
    s = np.sort(np.asarray(scores, np.float64))[::-1]
    scale = max(np.abs(s).max(), 1e-30)
    m = min(k + 1, s.size)
    gaps = np.diff(s[:m])
    return bool(gaps.size and np.abs(gaps).min() < rel * scale)


def router_scores(oracle, h, rms, w_router):
    xn = oracle.rmsnorm(h, rms)
    return oracle.gemv_f32(w_router, xn)
