"""GPU: expert records staged straight from a model file
(rabbit_cuda_moe_upload_file, the pread path of memory.c:255-279) against the
same records staged from a host map.

A file laid out like a .rabbit model -- a header and dense block of
arbitrary size, then the expert table -- is read with the expert table's
offset passed explicitly (the reference never sets expert_file_offset,
model.c:236-348). Bar: the pool then decodes bit-identically to a pool
uploaded from the in-memory records (same bytes, same kernels), and every
read failure comes back as a status, never a fault: missing file, a file
that ends inside a record, a group size the pool was not planned for.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import check_tokens, oracle_kw
from rabbit_b200 import synth

pytestmark = pytest.mark.gpu

# name: H, E, k, I, S, quant
SHAPES = {
    "group32_tiled": (256, 8, 2, 128, 1, 4),
    "fp32_verbatim": (64, 4, 2, 32, 0, 0),
}
HEAD = 264 + 4099  # header + an odd-sized dense block: record 0 is not 4 KB aligned


def model(name, seed, n_layers=2):
    H, E, k, I, S, quant = SHAPES[name]
    recs, size, router, rms = synth.moe_layer(seed, H, E, I, S)
    if quant == 0:
        rng = np.random.default_rng(seed)
        recs = np.concatenate([synth.f32_expert_record(rng, H, I) for _ in range(E + S)])
        size = recs.size // (E + S)
    # layer l's records differ: layer 1 reverses the expert order
    per = recs.reshape(E + S, size)
    layers = [per.reshape(-1), np.ascontiguousarray(per[::-1]).reshape(-1)][:n_layers]
    table = np.concatenate(layers)
    kw = dict(expert_size=size, n_layers=n_layers, hidden=H, n_experts=E, top_k=k, inter=I,
              n_shared=S, quant=quant, rms_ffn=[rms] * n_layers, w_router=[router] * n_layers)
    okw = [oracle_kw(H=H, E=E, k=k, I=I, S=S, records=layer, expert_size=size, rms_ffn=rms,
                     w_router=router, quant=quant) for layer in layers]
    return table, kw, okw


def write_model(path, table, tail=0):
    head = np.random.default_rng(1).integers(0, 256, HEAD, dtype=np.uint8)
    with open(path, "wb") as f:
        f.write(head.tobytes())
        f.write(table[:table.size - tail].tobytes())


@pytest.mark.parametrize("name", list(SHAPES))
def test_file_pool_decodes_like_the_mapped_pool(rc, oracle, tmp_path, name):
    table, kw, okw = model(name, seed=31)
    path = tmp_path / "model.rabbit"
    write_model(path, table)
    ref = rc.MoePool(records=table, **kw)
    pool = rc.MoePool(records=None, **kw)
    pool.upload_file(path, HEAD, 0, 1)  # layer by layer, as an engine would
    pool.upload_file(path, HEAD, 1, 2)
    pool.upload_file(path, HEAD, 0, 2)  # resident records are skipped
    pool.sync()
    st = pool.stats()
    assert st["resident_records"] == table.size // kw["expert_size"]
    assert st["uploads"] == st["resident_records"]
    h = np.random.default_rng(3).standard_normal((4, kw["hidden"])).astype(np.float32)
    for layer in range(kw["n_layers"]):
        outs = []
        for t in range(h.shape[0]):
            a, ia, wa = ref.decode(layer, h[t])
            b, ib, wb = pool.decode(layer, h[t])
            np.testing.assert_array_equal(b, a)
            np.testing.assert_array_equal(ib, ia)
            np.testing.assert_array_equal(wb, wa)
            outs.append((b, ib, wb))
        check_tokens(oracle, h, np.stack([o[0] for o in outs]), np.stack([o[1] for o in outs]),
                     np.stack([o[2] for o in outs]), okw[layer], min_checked=3)
        pf, pids, pw = pool.prefill(layer, h)
        check_tokens(oracle, h, pf, pids, pw, okw[layer], min_checked=3)
    ref.free()
    pool.free()


def test_file_read_failures_are_statuses(rc, tmp_path):
    table, kw, _ = model("group32_tiled", seed=5)
    size = kw["expert_size"]
    pool = rc.MoePool(records=None, **kw)
    with pytest.raises(rc.RabbitCudaError, match="cannot open"):
        pool.upload_file(tmp_path / "missing.rabbit", HEAD, 0, 2)
    short = tmp_path / "short.rabbit"
    write_model(short, table, tail=size // 2)  # the last record is cut in half
    with pytest.raises(rc.RabbitCudaError, match="ends inside record"):
        pool.upload_file(short, HEAD, 0, 2)
    assert pool.stats()["resident_records"] < table.size // size
    bad = table.copy()
    bad[3 * size:3 * size + 4] = np.frombuffer(np.uint32(64).tobytes(), np.uint8)  # group 64
    badf = tmp_path / "bad.rabbit"
    write_model(badf, bad)
    pool2 = rc.MoePool(records=None, **kw)
    with pytest.raises(rc.RabbitCudaError, match="group size"):
        pool2.upload_file(badf, HEAD, 0, 2)
    with pytest.raises(rc.RabbitCudaError, match="layer range"):
        pool2.upload_file(badf, HEAD, 1, 3)
    pool.free()
    pool2.free()
