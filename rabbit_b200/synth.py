"""Seeded synthetic inputs in the .rabbit expert format.

Group-32 int4 matrix blob (quant.c:66-75, docs/file-format.md:57-67):
    u32 group_size | f32 scales[ceil(n/gs)] | u8 packed[(n+1)/2]
element i: nibble = byte[i/2] >> 4 if i odd else byte[i/2] & 0xF, q = nibble - 8,
value = q * scales[i / gs], i the flat row-major index.

Expert record (forward_v2.c:315-332): gate [I,H] | up [I,H] | down [H,I], padded
to a uniform expert_size.

Distributions follow the workload definitions: q uniform on [-8, 7] (uniform
random bytes give two independent uniform nibbles), scales |N(0, 0.02)| / 7,
activations N(0, 1), router weights N(0, 0.02), norm weights 1.
"""
from __future__ import annotations

import numpy as np


def int4_nbytes(n: int, group_size: int = 32) -> int:
    """quant.c:190-195"""
    if n <= 0:
        return 0
    return 4 + 4 * ((n + group_size - 1) // group_size) + (n + 1) // 2


def int4_blob(rng: np.random.Generator, rows: int, cols: int, group_size: int = 32,
              scale_sigma: float = 0.02) -> np.ndarray:
    """One random group-scaled int4 matrix blob (uint8 array)."""
    n = rows * cols
    ng = (n + group_size - 1) // group_size
    nb = (n + 1) // 2
    out = np.empty(4 + 4 * ng + nb, np.uint8)
    out[:4] = np.frombuffer(np.uint32(group_size).tobytes(), np.uint8)
    sc = (np.abs(rng.normal(0.0, scale_sigma, ng)) / 7.0).astype(np.float32)
    out[4:4 + 4 * ng] = sc.view(np.uint8)
    out[4 + 4 * ng:] = rng.integers(0, 256, nb, dtype=np.uint8)
    if n % 2:  # the unused high nibble of the last byte: the packer writes q=0 (nibble 8)
        out[-1] = (out[-1] & 0x0F) | 0x80
    return out


def expert_record(rng: np.random.Generator, H: int, inter: int, expert_size: int | None = None,
                  group_size: int = 32) -> np.ndarray:
    """gate | up | down int4 blobs, zero padded to expert_size."""
    parts = [int4_blob(rng, inter, H, group_size), int4_blob(rng, inter, H, group_size),
             int4_blob(rng, H, inter, group_size)]
    rec = np.concatenate(parts)
    if expert_size is not None:
        if expert_size < rec.size:
            raise ValueError("expert_size smaller than the record")
        rec = np.concatenate([rec, np.zeros(expert_size - rec.size, np.uint8)])
    return rec


def expert_record_size(H: int, inter: int) -> int:
    return 2 * int4_nbytes(H * inter) + int4_nbytes(H * inter)


def moe_layer(seed: int, H: int, E: int, inter: int, n_shared: int = 0, pad: int = 0):
    """Records (E routed + S shared), router [E,H], rms_ffn [H] for one layer."""
    rng = np.random.default_rng(seed)
    size = expert_record_size(H, inter) + pad
    recs = np.concatenate([expert_record(rng, H, inter, size) for _ in range(E + n_shared)])
    w_router = rng.normal(0.0, 0.02, (E, H)).astype(np.float32)
    rms_ffn = np.ones(H, np.float32)
    return recs, size, w_router, rms_ffn


def f32_expert_record(rng: np.random.Generator, H: int, inter: int, sigma: float = 0.02):
    """quant 0 record: raw fp32 gate | up | down."""
    return (sigma * rng.standard_normal(3 * H * inter)).astype(np.float32).view(np.uint8)


def int8_expert_record(rng: np.random.Generator, H: int, inter: int):
    """quant 8 record: per matrix f32 scale + int8 payload."""
    parts = []
    for _ in range(3):
        parts.append(np.frombuffer(np.float32(abs(rng.normal(0, 0.02)) / 127 + 1e-4).tobytes(),
                                   np.uint8))
        parts.append(rng.integers(-128, 128, H * inter, dtype=np.int8).view(np.uint8))
    return np.concatenate(parts)
