"""GPU: a windowed pool (rabbit_cuda_moe_create_window) -- HBM blocks for
fewer layers than the model has, filled on demand and reassigned least
recently used first -- against a pool that holds every layer.

Bar: every layer decodes and prefills bit-identically to the full pool
whenever it holds a block, and within rtol 1e-4 / atol 1e-5 of the oracle's
moe_step (ids identical); a layer whose block was taken back reports "not
uploaded" instead of reading another layer's experts; uploads from the host
map and from the model file both fill blocks.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import check_tokens, oracle_kw
from rabbit_b200 import synth

pytestmark = pytest.mark.gpu

H, E, K, I, S, L = 256, 8, 2, 128, 1, 4


def model():
    layers = [synth.moe_layer(40 + l, H, E, I, S) for l in range(L)]
    table = np.concatenate([m[0] for m in layers])
    kw = dict(expert_size=layers[0][1], n_layers=L, hidden=H, n_experts=E, top_k=K, inter=I,
              n_shared=S, quant=4, rms_ffn=[m[3] for m in layers],
              w_router=[m[2] for m in layers])
    okw = [oracle_kw(H=H, E=E, k=K, I=I, S=S, records=m[0], expert_size=m[1], rms_ffn=m[3],
                     w_router=m[2]) for m in layers]
    return table, kw, okw


def same(pool, ref, layer, h, oracle=None, okw=None):
    outs = []
    for t in range(h.shape[0]):
        a, ia, wa = ref.decode(layer, h[t])
        b, ib, wb = pool.decode(layer, h[t])
        np.testing.assert_array_equal(b, a)
        np.testing.assert_array_equal(ib, ia)
        np.testing.assert_array_equal(wb, wa)
        outs.append((b, ib, wb))
    if oracle is not None:
        check_tokens(oracle, h, np.stack([o[0] for o in outs]), np.stack([o[1] for o in outs]),
                     np.stack([o[2] for o in outs]), okw[layer], min_checked=2)


def test_window_of_two_layers_over_four(rc, oracle, tmp_path):
    table, kw, okw = model()
    ref = rc.MoePool(records=table, **kw)
    pool = rc.MoePool(records=table, window=2, **kw)
    h = np.random.default_rng(8).standard_normal((3, H)).astype(np.float32)
    assert pool.stats()["pool_bytes"] * 2 <= ref.stats()["pool_bytes"] + 4096
    with pytest.raises(rc.RabbitCudaError, match="not uploaded"):
        pool.decode(0, h[0])
    pool.upload(0, 2)
    same(pool, ref, 0, h, oracle, okw)
    same(pool, ref, 1, h, oracle, okw)
    pool.upload(2, 3)             # takes layer 0's block, the least recently used
    same(pool, ref, 2, h, oracle, okw)
    same(pool, ref, 1, h, oracle, okw)
    with pytest.raises(rc.RabbitCudaError, match="not uploaded"):
        pool.decode(0, h[0])
    pool.upload(3, 4)             # takes layer 2's block (layer 1 was used last)
    with pytest.raises(rc.RabbitCudaError, match="not uploaded"):
        pool.decode(2, h[0])
    same(pool, ref, 3, h, oracle, okw)
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
    same(pool, ref, 0, h, oracle, okw)
    ref.free()
    pool.free()


def test_window_refusals(rc):
    table, kw, _ = model()
    size = kw["expert_size"]
    shared = dict(kw, experts_per_layer=E + S)
    with pytest.raises(rc.RabbitCudaError, match="shared by every layer"):
        rc.MoePool(records=table[:(E + S) * size], experts_shared=True, window=2, **shared)
    pool = rc.MoePool(records=table, window=2, **kw)
    with pytest.raises(rc.RabbitCudaError, match="on demand"):
        pool.fill_synthetic(1)
    pool.free()
