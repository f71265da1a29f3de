"""GPU: a windowed pool (rabbit_cuda_moe_create_window) -- HBM blocks for
fewer layers than the model has, filled on demand and reassigned least
recently used first -- against a pool that holds every layer.

Bar: every layer decodes and prefills bit-identically to the full pool
whenever it holds a block; a layer whose block was taken back reports "not
uploaded" instead of reading another layer's experts; uploads from the host
map and from the model file both fill blocks.
"""
from __future__ import annotations

import numpy as np
import pytest

from rabbit_b200 import synth

pytestmark = pytest.mark.gpu

H, E, K, I, S, L = 256, 8, 2, 128, 1, 4


def model():
    layers = [synth.moe_layer(40 + l, H, E, I, S) for l in range(L)]
    table = np.concatenate([m[0] for m in layers])
    kw = dict(expert_size=layers[0][1], n_layers=L, hidden=H, n_experts=E, top_k=K, inter=I,
              n_shared=S, quant=4, rms_ffn=[m[3] for m in layers],
              w_router=[m[2] for m in layers])
    return table, kw


def same(pool, ref, layer, h):
    for t in range(h.shape[0]):
        a, ia, wa = ref.decode(layer, h[t])
        b, ib, wb = pool.decode(layer, h[t])
        np.testing.assert_array_equal(b, a)
        np.testing.assert_array_equal(ib, ia)
        np.testing.assert_array_equal(wb, wa)


def test_window_of_two_layers_over_four(rc, tmp_path):
    table, kw = model()
    ref = rc.MoePool(records=table, **kw)
    pool = rc.MoePool(records=table, window=2, **kw)
    h = np.random.default_rng(8).standard_normal((3, H)).astype(np.float32)
    assert pool.stats()["pool_bytes"] * 2 <= ref.stats()["pool_bytes"] + 4096
    with pytest.raises(rc.RabbitCudaError, match="not uploaded"):
        pool.decode(0, h[0])
    pool.upload(0, 2)
    same(pool, ref, 0, h)
    same(pool, ref, 1, h)
    pool.upload(2, 3)             # takes layer 0's block, the least recently used
    same(pool, ref, 2, h)
    same(pool, ref, 1, h)
    with pytest.raises(rc.RabbitCudaError, match="not uploaded"):
        pool.decode(0, h[0])
    pool.upload(3, 4)             # takes layer 2's block (layer 1 was used last)
    with pytest.raises(rc.RabbitCudaError, match="not uploaded"):
        pool.decode(2, h[0])
    same(pool, ref, 3, h)
    a, _, _ = ref.prefill(3, h)
    b, _, _ = pool.prefill(3, h)
    np.testing.assert_array_equal(b, a)
    with pytest.raises(rc.RabbitCudaError, match="window"):
        pool.upload(0, 3)         # more layers than blocks
    # a layer back from the model file
    path = tmp_path / "model.rabbit"
    with open(path, "wb") as f:
        f.write(bytes(1000))
        f.write(table.tobytes())
    pool.upload_file(path, 1000, 0, 1)
    same(pool, ref, 0, h)
    ref.free()
    pool.free()


def test_window_refusals(rc):
    table, kw = model()
    size = kw["expert_size"]
    shared = dict(kw, experts_per_layer=E + S)
    with pytest.raises(rc.RabbitCudaError, match="shared by every layer"):
        rc.MoePool(records=table[:(E + S) * size], experts_shared=True, window=2, **shared)
    pool = rc.MoePool(records=table, window=2, **kw)
    with pytest.raises(rc.RabbitCudaError, match="on demand"):
        pool.fill_synthetic(1)
    pool.free()
