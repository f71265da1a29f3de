"""Pre-tiled expert records (RABBIT_CUDA_QUANT_INT4_TILED): the converter-side
re-layout, rabbit_cuda_tile_records, runs on the host without a GPU.

Bar (CPU): the tiled record holds exactly the scale and nibble bytes of the
record's three group-32 blobs (gate, up, down: forward_v2.c:314-332), moved,
with zeros elsewhere -- so the byte sums agree -- followed by a trailer naming
the tile plan; tiling is deterministic; other formats are refused. On the GPU
(tests/test_pretiled_gpu.py) a pool of tiled records decodes bit-identically
to a pool that tiles the same records at upload.
"""
from __future__ import annotations

import numpy as np
import pytest

from rabbit_b200 import synth

SHAPE = dict(hidden=256, n_experts=8, top_k=2, inter=128, n_shared=1)


def records(seed=7):
    recs, size, _, _ = synth.moe_layer(seed, SHAPE["hidden"], SHAPE["n_experts"],
                                        SHAPE["inter"], SHAPE["n_shared"])
    return recs, size


def test_tiled_records_hold_the_same_bytes(rc):
    recs, size = records()
    tiled, tsize = rc.tile_records(recs, size, **SHAPE)
    n = recs.size // size
    assert tiled.size == n * tsize and tsize % 256 == 0
    nb = synth.int4_nbytes(SHAPE["hidden"] * SHAPE["inter"])
    for r in range(n):
        rec = recs[r * size:(r + 1) * size]
        out = tiled[r * tsize:(r + 1) * tsize]
        body, trailer = out[:tsize - 256], out[tsize - 256:]
        payload = sum(int(rec[m * nb + 4:(m + 1) * nb].astype(np.int64).sum()) for m in range(3))
        assert int(body.astype(np.int64).sum()) == payload, f"record {r}"
        assert bytes(trailer[:8]) == b"RB2TILE1"
        assert int(np.count_nonzero(body)) <= 3 * (nb - 4)
    again, _ = rc.tile_records(recs, size, **SHAPE)
    np.testing.assert_array_equal(again, tiled)


def test_tile_records_refuses_other_formats(rc):
    recs, size = records()
    bad = recs.copy()
    bad[size:size + 4] = np.frombuffer(np.uint32(16).tobytes(), np.uint8)  # record 1: group 16
    with pytest.raises(rc.RabbitCudaError, match="group size"):
        rc.tile_records(bad, size, **SHAPE)
    with pytest.raises(rc.RabbitCudaError):
        rc.tile_records(recs, size, **SHAPE, sm_count=0)


@pytest.mark.parametrize("shape", [
    dict(hidden=128, n_experts=8, top_k=2, inter=2048, n_shared=0),   # W2 in two column chunks
    dict(hidden=2048, n_experts=64, top_k=6, inter=1408, n_shared=2),  # DeepSeek-MoE-16B shape
    dict(hidden=256, n_experts=16, top_k=3, inter=96, n_shared=2),     # inter not a multiple of 128
])
def test_tiled_bytes_match_for_other_shapes(rc, shape):
    H, I = shape["hidden"], shape["inter"]
    recs, size, _, _ = synth.moe_layer(3, H, 2, I, 0)  # two records of this shape
    tiled, tsize = rc.tile_records(recs, size, **shape)
    nb = synth.int4_nbytes(H * I)
    for r in range(2):
        rec = recs[r * size:(r + 1) * size]
        body = tiled[r * tsize:(r + 1) * tsize - 256]
        payload = sum(int(rec[m * nb + 4:(m + 1) * nb].astype(np.int64).sum()) for m in range(3))
        assert int(body.astype(np.int64).sum()) == payload
        assert bytes(tiled[(r + 1) * tsize - 256:(r + 1) * tsize - 248]) == b"RB2TILE1"
