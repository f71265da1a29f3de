"""Pin the oracle (plain-C restatement) to the reference.

1. Against the committed golden fixtures (made by the reference's own C):
   bit-identical outputs for every case.
2. Against the reference's known-answer test (tests/test_quant.c:43-65):
   nbytes formula and the group-int4 round-trip error bound.
3. Against the live reference library (oracle/_ref, when built here) on fresh
   seeded inputs, including ragged shapes and edge cases.
"""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from rabbit_b200 import synth

GOLD = Path(__file__).resolve().parent / "golden"


def _load(name):
    return np.load(GOLD / f"{name}.npz")


def _same(a, b):
    a, b = np.asarray(a), np.asarray(b)
    assert a.shape == b.shape
    if a.dtype.kind == "f":
        np.testing.assert_array_equal(a.view(np.uint32), b.view(np.uint32))
    else:
        np.testing.assert_array_equal(a, b)


def test_golden_gemv_and_dequant(oracle):
    g = _load("gemv")
    for i in range(int(g["gemv_count"])):
        r, c, gs = (int(v) for v in g[f"gemv{i}_shape"])
        y = oracle.gemv_int4_grouped(g[f"gemv{i}_blob"], g[f"gemv{i}_x"], r, c)
        _same(y, g[f"gemv{i}_y"])
        if f"gemv{i}_deq" in g:
            _same(oracle.dequant_int4_grouped(g[f"gemv{i}_blob"], r * c), g[f"gemv{i}_deq"])
        else:  # invalid group size: zeros, and dequant rejects the blob
            assert not g[f"gemv{i}_y"].any()
            with pytest.raises(ValueError):
                oracle.dequant_int4_grouped(g[f"gemv{i}_blob"], r * c)


def test_golden_pack(oracle):
    g = _load("pack")
    for i in range(2):
        _same(oracle.pack_int4_grouped(g[f"pack{i}_src"], 32), g[f"pack{i}_blob"])


def test_reference_known_answer_group_roundtrip(oracle):
    """tests/test_quant.c:43-65: n=100, sin(i*0.17)*3, group 32."""
    src = (np.sin(np.arange(100, dtype=np.float32) * np.float32(0.17)) * np.float32(3))
    blob = oracle.pack_int4_grouped(src.astype(np.float32), 32)
    assert blob.size == oracle.int4_grouped_nbytes(100, 32) == 4 + 4 * 4 + 50
    back = oracle.dequant_int4_grouped(blob, 100)
    assert np.abs(back - src).max() < 0.6


def test_golden_topk(oracle):
    g = _load("topk")
    for i in range(int(g["topk_count"])):
        ids, w = oracle.select_top_k(g[f"topk{i}_scores"], int(g[f"topk{i}_k"]))
        _same(ids, g[f"topk{i}_ids"])
        _same(w, g[f"topk{i}_w"])
    # the tie case: equal scores keep ascending ids
    np.testing.assert_array_equal(g["topk3_ids"], [1, 2, 4])
    # NaN never enters; -inf scores never beat the -1e30 seed
    assert 0 not in g["topk4_ids"] and 3 not in g["topk4_ids"]
    np.testing.assert_array_equal(g["topk5_ids"], [-1, -1])


def test_golden_swiglu(oracle):
    g = _load("swiglu")
    for i in range(int(g["swiglu_count"])):
        q, H, I, size = (int(v) for v in g[f"swiglu{i}_meta"])
        w = 0.375 if i < 3 else 1.0
        d = oracle.expert_swiglu(g[f"swiglu{i}_rec"], size, q, g[f"swiglu{i}_xn"], H, I, w,
                                 g[f"swiglu{i}_delta0"])
        _same(d, g[f"swiglu{i}_delta"])
    assert not g["swiglu3_delta"].any()  # too-small record adds nothing


def test_golden_moe(oracle):
    g = _load("moe")
    for i in range(int(g["moe_count"])):
        H, E, k, I, S, q, size = (int(v) for v in g[f"moe{i}_meta"])
        h_out, ids, w = oracle.moe_step(g[f"moe{i}_h"], H=H, E=E, top_k=k, inter=I, n_shared=S,
                                        quant=q, n_records=E + S, expert_size=size,
                                        records=g[f"moe{i}_recs"], rms_ffn=g[f"moe{i}_rms"],
                                        w_router=g[f"moe{i}_router"])
        _same(h_out, g[f"moe{i}_hout"])


def test_golden_attention_rope_logits(oracle):
    g = _load("attn")
    H, nh, nkv, hd, T = (int(v) for v in g["attn_meta"])
    w = {k: g["attn_" + k] for k in ("rms_attn", "w_q", "w_k", "w_v", "w_o")}
    kv_k = np.zeros((8, nkv * hd), np.float32)
    kv_v = np.zeros((8, nkv * hd), np.float32)
    n = 0
    for pos in range(T):
        h2, n = oracle.attention_step(g["attn_h"][pos], kv_k, kv_v, n, pos, n_heads=nh,
                                      n_kv_heads=nkv, head_dim=hd, **w)
        _same(h2, g["attn_hout"][pos])
    _same(oracle.logits(g["logits_lm"], g["logits_h"]), g["logits_y"])
    for j, p in enumerate((0, 1, 7, 200)):
        _same(oracle.apply_rope_head(g["rope_x"], p), g["rope_y"][j])


# ---------------------------------------------------------------- live ----

@pytest.mark.parametrize("shape", [(1, 1), (2, 31), (3, 33), (17, 64), (40, 4096), (256, 1408),
                                   (5, 1000)])
def test_live_gemv_matches_reference(oracle, reference, shape):
    r, c = shape
    rng = np.random.default_rng(r * 1000 + c)
    for gs in (32, 64, 3):
        blob = synth.int4_blob(rng, r, c, gs)
        x = rng.standard_normal(c).astype(np.float32)
        _same(oracle.gemv_int4_grouped(blob, x, r, c), reference.gemv_int4_grouped(blob, x, r, c))
        _same(oracle.dequant_int4_grouped(blob, r * c), reference.dequant_int4_grouped(blob, r * c))


def test_live_topk_matches_reference(oracle, reference):
    rng = np.random.default_rng(7)
    for _ in range(200):
        E = int(rng.integers(1, 80))
        k = int(rng.integers(1, min(E, 8) + 1))
        s = rng.standard_normal(E).astype(np.float32)
        if rng.random() < 0.3:  # inject ties
            s[rng.integers(0, E, 3)] = s[0]
        a, b = oracle.select_top_k(s, k), reference.select_top_k(s, k)
        _same(a[0], b[0])
        _same(a[1], b[1])


@pytest.mark.parametrize("spec", [(256, 8, 2, 512, 0), (256, 16, 6, 192, 2), (128, 64, 8, 64, 0)])
def test_live_moe_matches_reference(oracle, reference, spec):
    H, E, k, I, S = spec
    recs, size, w_router, rms = synth.moe_layer(H + E, H, E, I, S)
    rng = np.random.default_rng(5)
    for _ in range(3):
        h = rng.standard_normal(H).astype(np.float32)
        kw = dict(H=H, E=E, top_k=k, inter=I, n_shared=S, quant=4, n_records=E + S,
                  expert_size=size, records=recs, rms_ffn=rms, w_router=w_router)
        _same(oracle.moe_step(h, **kw)[0], reference.moe_step(h, **kw))


def test_golden_legacy_expert(oracle):
    """moe.c:119-224: the oracle's legacy per-tensor expert equals the
    reference's on every committed case, bit for bit."""
    g = _load("legacy")
    for i in range(int(g["legacy_count"])):
        q, H, ed = (int(v) for v in g[f"legacy{i}_meta"])
        got = oracle.legacy_apply_expert(g[f"legacy{i}_rec"], q, g[f"legacy{i}_h"], ed,
                                         float(g[f"legacy{i}_w"]))
        _same(got, g[f"legacy{i}_hout"])


def test_live_legacy_expert_matches_reference(oracle, reference):
    from legacy_cases import legacy_cases

    for name, q, H, ed, rec, h, w in legacy_cases():
        _same(oracle.legacy_apply_expert(rec, q, h, ed, w),
              reference.legacy_apply_expert(rec, q, h, ed, w))
