"""Seeded cases for the legacy per-tensor expert (src/moe.c:119-224,
apply_expert): every branch it takes -- the three-matrix SwiGLU in int4 and
int8 (quant 0 reads as int8), the expert_dim default and clamp, stored scales
that are not positive finite numbers, int4 rows of an odd width, and the
square-matrix and raw-byte fallbacks for records too small for three
matrices. Used by tests/golden/make_golden.py (run on the reference's own C),
the oracle pins and the GPU tests."""
from __future__ import annotations

import numpy as np


def _swiglu_record(rng, quant, H, inter, scales, pad=0):
    mat = H * inter
    parts = []
    for s in scales:
        parts.append(np.frombuffer(np.float32(s).tobytes(), np.uint8))
        n = (mat + 1) // 2 if quant == 4 else mat
        parts.append(rng.integers(0, 256, n, dtype=np.uint8))
    parts.append(np.zeros(pad, np.uint8))
    return np.concatenate(parts)


def _square_record(rng, quant, H, scale, extra=0):
    n = H * ((H + 1) // 2) if quant == 4 else H * H
    return np.concatenate([np.frombuffer(np.float32(scale).tobytes(), np.uint8),
                           rng.integers(0, 256, n + extra, dtype=np.uint8)])


def legacy_cases():
    """[(name, quant, H, expert_dim, record, hidden, weight)]"""
    rng = np.random.default_rng(31)
    out = []

    def add(name, quant, H, expert_dim, rec, weight):
        out.append((name, quant, H, expert_dim, rec,
                    rng.standard_normal(H).astype(np.float32), np.float32(weight)))

    add("int4_swiglu", 4, 64, 128, _swiglu_record(rng, 4, 64, 128, (0.02, 0.025, 0.02)), 0.7)
    add("int4_swiglu_wide", 4, 128, 256,
        _swiglu_record(rng, 4, 128, 256, (0.01, 0.01, 0.012)), 1.0)
    add("int8_swiglu_default_inter", 8, 48, 0,
        _swiglu_record(rng, 8, 48, 96, (0.002, 0.003, 0.002)), 0.45)
    # odd widths: int4 rows of (in + 1) / 2 bytes read past each matrix's
    # (mat + 1) / 2 payload; the padding keeps the last rows inside the record
    add("int4_odd_padded", 4, 33, 65, _swiglu_record(rng, 4, 33, 65, (0.03, 0.02, 0.03), 64), 0.9)
    add("bad_scales", 8, 32, 64,
        _swiglu_record(rng, 8, 32, 64, (-1.0, float("nan"), float("inf"))), 0.01)
    add("int8_inter_clamped", 8, 16, 100, _swiglu_record(rng, 8, 16, 32, (0.004, 0.004, 0.004)),
        0.5)
    add("quant0_as_int8", 0, 32, 64, _swiglu_record(rng, 0, 32, 64, (0.003, 0.003, 0.003)), 0.6)
    add("int4_square_fallback", 4, 40, 0, _square_record(rng, 4, 40, 0.05, 7), 0.8)
    add("int8_square_fallback", 8, 24, 0, _square_record(rng, 8, 24, 0.01), 0.8)
    rec = rng.integers(0, 256, 20 * 20, dtype=np.uint8)  # payload < H*H <= size: bytes from 0
    add("int8_unscaled_square", 8, 20, 0, rec, 0.3)
    add("raw_bytes", 8, 64, 0, rng.integers(0, 256, 40, dtype=np.uint8), 0.25)
    add("int4_too_small", 4, 64, 0, rng.integers(0, 256, 100, dtype=np.uint8), 1.0)
    return out
