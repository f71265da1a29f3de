"""Generate the golden fixtures in this directory from the reference's own C.

    make -C oracle ref            # builds oracle/_ref/libref.so from the reference sources
    python tests/golden/make_golden.py [name ...]   # all files, or only those named

The reference publishes no int4 golden vectors (its tests/test_quant.c only
bounds round-trip error), so these fixtures pin the reference's behaviour by
running its compiled routines (rabbit_gemv_int4_grouped, rabbit_dequant_
int4_grouped, rabbit_pack_int4_grouped, and forward_v2.c's select_top_k,
expert_swiglu, moe_step, attention_step, logits_from_hidden; moe.c's legacy
apply_expert) on small seeded
inputs. Every array is stored with its inputs, so the oracle and the CUDA
path can be checked against them on machines without the reference.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))

from oracle.oracle import Reference  # noqa: E402
from rabbit_b200 import synth  # noqa: E402


def gemv_cases(ref: Reference, out: dict) -> None:
    rng = np.random.default_rng(100)
    shapes = [(1, 1, 32), (1, 32, 32), (3, 17, 32), (5, 33, 32), (7, 100, 32), (64, 64, 32),
              (96, 128, 32), (130, 256, 32), (33, 96, 64), (12, 40, 16), (9, 31, 7),
              (4, 64, 0), (4, 64, 5000)]
    for i, (r, c, gs) in enumerate(shapes):
        g = gs if 0 < gs <= 4096 else 32
        blob = synth.int4_blob(rng, r, c, g)
        if gs == 0 or gs > 4096:  # invalid header: the reference writes zeros
            blob[:4] = np.frombuffer(np.uint32(gs).tobytes(), np.uint8)
        x = rng.standard_normal(c).astype(np.float32)
        out[f"gemv{i}_shape"] = np.array([r, c, gs], np.int64)
        out[f"gemv{i}_blob"] = blob
        out[f"gemv{i}_x"] = x
        out[f"gemv{i}_y"] = ref.gemv_int4_grouped(blob, x, r, c)
        if 0 < gs <= 4096:
            out[f"gemv{i}_deq"] = ref.dequant_int4_grouped(blob, r * c)
    out["gemv_count"] = np.array(len(shapes))


def pack_cases(ref: Reference, out: dict) -> None:
    # the reference's own known-answer input (tests/test_quant.c:43-65)
    src = (np.sin(np.arange(100, dtype=np.float32) * np.float32(0.17)) * np.float32(3)).astype(
        np.float32)
    out["pack0_src"] = src
    out["pack0_blob"] = ref.pack_int4_grouped(src, 32)
    rng = np.random.default_rng(101)
    src = (0.05 * rng.standard_normal(333)).astype(np.float32)
    out["pack1_src"] = src
    out["pack1_blob"] = ref.pack_int4_grouped(src, 32)


def topk_cases(ref: Reference, out: dict) -> None:
    rng = np.random.default_rng(102)
    cases = [
        (rng.standard_normal(8).astype(np.float32), 2),
        (rng.standard_normal(64).astype(np.float32), 8),
        (rng.standard_normal(64).astype(np.float32), 6),
        (np.array([1, 3, 3, 2, 3, 0], np.float32), 3),           # ties: lower id first
        (np.array([np.nan, 1, 2, np.nan, 0.5], np.float32), 2),  # NaN never selected
        (np.array([-np.inf, -np.inf, -np.inf], np.float32), 2),  # nothing beats -1e30
        (np.array([0.25, -1.0, 0.75, 0.5], np.float32), 4),      # k == E
        (np.full(16, 0.5, np.float32), 8),
    ]
    for i, (s, k) in enumerate(cases):
        ids, w = ref.select_top_k(s, k)
        out[f"topk{i}_scores"] = s
        out[f"topk{i}_k"] = np.array(k)
        out[f"topk{i}_ids"] = ids
        out[f"topk{i}_w"] = w
    out["topk_count"] = np.array(len(cases))


def swiglu_cases(ref: Reference, out: dict) -> None:
    rng = np.random.default_rng(103)
    H, I = 64, 96
    recs = {
        4: synth.expert_record(rng, H, I),
        0: synth.f32_expert_record(rng, H, I),
        8: synth.int8_expert_record(rng, H, I),
    }
    for i, (q, rec) in enumerate(recs.items()):
        xn = rng.standard_normal(H).astype(np.float32)
        delta0 = (0.1 * rng.standard_normal(H)).astype(np.float32)
        out[f"swiglu{i}_meta"] = np.array([q, H, I, rec.size], np.int64)
        out[f"swiglu{i}_rec"] = rec
        out[f"swiglu{i}_xn"] = xn
        out[f"swiglu{i}_delta0"] = delta0
        out[f"swiglu{i}_delta"] = ref.expert_swiglu(rec, rec.size, q, xn, H, I, 0.375, delta0)
    # record too small: the reference adds nothing
    rec = recs[4][:-1].copy()
    xn = rng.standard_normal(H).astype(np.float32)
    out["swiglu3_meta"] = np.array([4, H, I, rec.size], np.int64)
    out["swiglu3_rec"] = rec
    out["swiglu3_xn"] = xn
    out["swiglu3_delta0"] = np.zeros(H, np.float32)
    out["swiglu3_delta"] = ref.expert_swiglu(rec, rec.size, 4, xn, H, I, 1.0)
    out["swiglu_count"] = np.array(4)


def moe_cases(ref: Reference, out: dict) -> None:
    specs = [  # H, E, top_k, I, S, quant, seed, pad
        (64, 4, 2, 128, 0, 4, 110, 0),
        (64, 4, 2, 128, 2, 4, 111, 12),
        (128, 16, 4, 64, 1, 4, 112, 0),
        (64, 8, 0, 96, 0, 4, 113, 0),   # top_k 0 -> 2 (forward_v2.c:113)
        (96, 6, 3, 64, 0, 0, 114, 0),
        (96, 6, 3, 64, 0, 8, 115, 0),
        (64, 4, 9, 64, 0, 4, 116, 0),   # top_k clamps to E
    ]
    for i, (H, E, k, I, S, q, seed, pad) in enumerate(specs):
        rng = np.random.default_rng(seed)
        if q == 4:
            size = synth.expert_record_size(H, I) + pad
            recs = np.concatenate([synth.expert_record(rng, H, I, size) for _ in range(E + S)])
        elif q == 0:
            one = [synth.f32_expert_record(rng, H, I) for _ in range(E + S)]
            size = one[0].size
            recs = np.concatenate(one)
        else:
            one = [synth.int8_expert_record(rng, H, I) for _ in range(E + S)]
            size = one[0].size
            recs = np.concatenate(one)
        w_router = rng.normal(0, 0.02, (E, H)).astype(np.float32)
        rms = (1.0 + 0.01 * rng.standard_normal(H)).astype(np.float32)
        h = rng.standard_normal(H).astype(np.float32)
        h_out = ref.moe_step(h, H=H, E=E, top_k=k, inter=I, n_shared=S, quant=q,
                             n_records=E + S, expert_size=size, records=recs, rms_ffn=rms,
                             w_router=w_router)
        out[f"moe{i}_meta"] = np.array([H, E, k, I, S, q, size], np.int64)
        out[f"moe{i}_recs"] = recs
        out[f"moe{i}_router"] = w_router
        out[f"moe{i}_rms"] = rms
        out[f"moe{i}_h"] = h
        out[f"moe{i}_hout"] = h_out
    out["moe_count"] = np.array(len(specs))


def attn_cases(ref: Reference, out: dict) -> None:
    rng = np.random.default_rng(120)
    H, nh, nkv, hd, T = 64, 4, 2, 16, 5
    w = {
        "rms_attn": (1 + 0.01 * rng.standard_normal(H)).astype(np.float32),
        "w_q": (0.02 * rng.standard_normal((nh * hd, H))).astype(np.float32),
        "w_k": (0.02 * rng.standard_normal((nkv * hd, H))).astype(np.float32),
        "w_v": (0.02 * rng.standard_normal((nkv * hd, H))).astype(np.float32),
        "w_o": (0.02 * rng.standard_normal((H, nh * hd))).astype(np.float32),
    }
    kv_k = np.zeros((8, nkv * hd), np.float32)
    kv_v = np.zeros((8, nkv * hd), np.float32)
    kv_len = 0
    hs, outs = [], []
    for pos in range(T):
        h = rng.standard_normal(H).astype(np.float32)
        h2, kv_len = ref.attention_step(h, kv_k, kv_v, kv_len, pos, n_heads=nh, n_kv_heads=nkv,
                                        head_dim=hd, **w)
        hs.append(h)
        outs.append(h2)
    for k, v in w.items():
        out["attn_" + k] = v
    out["attn_meta"] = np.array([H, nh, nkv, hd, T], np.int64)
    out["attn_h"] = np.stack(hs)
    out["attn_hout"] = np.stack(outs)
    lm = (0.02 * rng.standard_normal((H, 40))).astype(np.float32)
    out["logits_lm"] = lm
    out["logits_h"] = outs[-1]
    out["logits_y"] = ref.logits(lm, outs[-1])
    x = rng.standard_normal(16).astype(np.float32)
    out["rope_x"] = x
    out["rope_y"] = np.stack([ref.apply_rope_head(x, p) for p in (0, 1, 7, 200)])


def legacy_cases(ref: Reference, out: dict) -> None:
    """moe.c:119-224 (apply_expert) on the cases of tests/legacy_cases.py."""
    sys.path.insert(0, str(HERE.parent))
    from legacy_cases import legacy_cases as cases

    for i, (name, q, H, ed, rec, h, w) in enumerate(cases()):
        out[f"legacy{i}_meta"] = np.array([q, H, ed], np.int64)
        out[f"legacy{i}_rec"] = rec
        out[f"legacy{i}_h"] = h
        out[f"legacy{i}_w"] = np.array(w, np.float32)
        out[f"legacy{i}_hout"] = ref.legacy_apply_expert(rec, q, h, ed, float(w))
    out["legacy_count"] = np.array(i + 1)


def main() -> None:
    ref = Reference()
    only = set(sys.argv[1:])  # e.g. `legacy`: write only those files
    for name, fn in [("gemv", gemv_cases), ("pack", pack_cases), ("topk", topk_cases),
                     ("swiglu", swiglu_cases), ("moe", moe_cases), ("attn", attn_cases),
                     ("legacy", legacy_cases)]:
        if only and name not in only:
            continue
        out: dict = {}
        fn(ref, out)
        np.savez_compressed(HERE / f"{name}.npz", **out)
        print(f"wrote {name}.npz ({(HERE / f'{name}.npz').stat().st_size} bytes)")


if __name__ == "__main__":
    main()
