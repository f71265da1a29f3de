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


def oracle_kw(*, H, E, k, I, S, records, expert_size, rms_ffn, w_router, quant=4):
    """Keyword arguments of Oracle.moe_step for one layer's records."""
    return dict(H=H, E=E, top_k=k, inter=I, n_shared=S, quant=quant, n_records=E + S,
                expert_size=expert_size, records=records, rms_ffn=rms_ffn, w_router=w_router)


def check_tokens(oracle, h, got_h, got_ids, got_w, kw, min_checked, ref=None):
    """Per token: top-k ids identical and routing weights, the MoE delta and
    h_out within RTOL / ATOL of the oracle's moe_step on that token alone;
    tokens whose router scores hold a near-tie are skipped. `ref` may hold
    the oracle outputs already computed, as [(h_out, ids, w)] per token."""
    checked = 0
    for t in range(h.shape[0]):
        ref_h, ref_ids, ref_w = ref[t] if ref is not None else oracle.moe_step(h[t], **kw)
        if near_tie(router_scores(oracle, h[t], kw["rms_ffn"], kw["w_router"]), len(ref_ids)):
            continue
        if got_ids is not None:
            np.testing.assert_array_equal(got_ids[t], ref_ids, err_msg=f"token {t}: ids")
            np.testing.assert_allclose(got_w[t], ref_w, rtol=RTOL, atol=ATOL,
                                       err_msg=f"token {t}: weights")
        np.testing.assert_allclose(got_h[t] - h[t], ref_h - h[t], rtol=RTOL, atol=ATOL,
                                   err_msg=f"token {t}: MoE delta")
        np.testing.assert_allclose(got_h[t], ref_h, rtol=RTOL, atol=ATOL,
                                   err_msg=f"token {t}: h_out")
        checked += 1
    assert checked >= min_checked, f"only {checked} tokens free of near-ties"


def oracle_many(oracle, h, kw, workers=None):
    """The oracle's moe_step for every row of h, run on host threads (the C
    oracle releases the GIL), for layers too large to check token by token on
    one core."""
    import os
    from concurrent.futures import ThreadPoolExecutor

    n = workers or max(1, min(h.shape[0], os.cpu_count() or 1))
    with ThreadPoolExecutor(n) as ex:
        return list(ex.map(lambda t: oracle.moe_step(h[t], **kw), range(h.shape[0])))


def dequant_g32(blob, rows, cols):
    """fl(q * scale) of a group-32 int4 blob as float32 [rows, cols]
    (quant.c:123-142)."""
    n = rows * cols
    ng = n // 32
    sc = blob[4:4 + 4 * ng].view(np.float32)
    nib = blob[4 + 4 * ng:4 + 4 * ng + n // 2]
    q = np.empty(n, np.int8)
    q[0::2] = (nib & 15).astype(np.int8) - 8
    q[1::2] = (nib >> 4).astype(np.int8) - 8
    return (q.astype(np.float32).reshape(ng, 32) * sc[:, None]).reshape(rows, cols)


def exact_moe_layer(oracle, h, kw, ref):
    """float64 evaluation of moe_step for every row of h over the same
    quantised weights and the oracle's routing (ref[t] = (h_out, ids, w)):
    the value the fp32 computations approximate. Group-32 int4 records, no
    shared-expert padding assumptions beyond the record layout."""
    H, I, E = kw["H"], kw["inter"], kw["E"]
    size, recs = kw["expert_size"], kw["records"]
    nb = 4 + 4 * (H * I // 32) + H * I // 2
    T = h.shape[0]
    xn = np.stack([oracle.rmsnorm(h[t], kw["rms_ffn"]) for t in range(T)]).astype(np.float64)
    out = h.astype(np.float64).copy()
    users = {}
    for t in range(T):
        for j, e in enumerate(ref[t][1]):
            users.setdefault(int(e), []).append((t, float(ref[t][2][j])))
    for s in range(kw["n_shared"]):
        users[E + s] = [(t, 1.0) for t in range(T)]
    for e, lst in users.items():
        rec = recs[e * size:(e + 1) * size]
        ts = np.array([t for t, _ in lst])
        x = xn[ts].T
        g = dequant_g32(rec[:nb], I, H) @ x
        u = dequant_g32(rec[nb:2 * nb], I, H) @ x
        mid = (g / (1.0 + np.exp(-g))) * u
        d = dequant_g32(rec[2 * nb:3 * nb], H, I) @ mid
        for i, (t, wt) in enumerate(lst):
            out[t] += wt * d[:, i]
    return out


def check_tokens_long(oracle, h, got_h, got_ids, got_w, kw, ref, exact, min_checked):
    """check_tokens for layers whose rows sum so many terms that the oracle's
    own serial fp32 rounding is of the order of ATOL: per element the bar is
    ATOL + RTOL |oracle| + |oracle - exact|, exact the float64 value of the
    same quantised layer (the reference may be off by that much itself)."""
    checked = 0
    for t in range(h.shape[0]):
        ref_h, ref_ids, ref_w = ref[t]
        if near_tie(router_scores(oracle, h[t], kw["rms_ffn"], kw["w_router"]), len(ref_ids)):
            continue
        np.testing.assert_array_equal(got_ids[t], ref_ids, err_msg=f"token {t}: ids")
        np.testing.assert_allclose(got_w[t], ref_w, rtol=RTOL, atol=ATOL,
                                   err_msg=f"token {t}: weights")
        own = np.abs(ref_h.astype(np.float64) - exact[t])
        bar = ATOL + RTOL * np.abs(ref_h) + own
        dev = np.abs(got_h[t].astype(np.float64) - ref_h)
        bad = np.flatnonzero(dev > bar)
        assert bad.size == 0, (f"token {t}: {bad.size} elements off, e.g. [{bad[0]}] got "
                               f"{got_h[t][bad[0]]} oracle {ref_h[bad[0]]} exact {exact[t][bad[0]]}")
        checked += 1
    assert checked >= min_checked, f"only {checked} tokens free of near-ties"
