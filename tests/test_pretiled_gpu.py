"""GPU: a pool of pre-tiled records (RABBIT_CUDA_QUANT_INT4_TILED, written by
rabbit_cuda_tile_records for this GPU's SM count) against a pool that tiles
the same group-32 records at upload. Bar: bit-identical decode and prefill
outputs, from a host map and from the model file; records tiled for another
plan are refused with a status; the pre-tiled pool's outputs are also held to
the oracle's moe_step (rtol 1e-4 / atol 1e-5, ids identical).
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import check_tokens, oracle_kw
from rabbit_b200 import synth

pytestmark = pytest.mark.gpu

H, E, K, I, S = 256, 8, 2, 128, 1


def sm_count():
    import torch

    return torch.cuda.get_device_properties(0).multi_processor_count


def pools(rc, recs, size, router, rms, tiled, tsize, **extra):
    kw = dict(n_layers=1, hidden=H, n_experts=E, top_k=K, inter=I, n_shared=S,
              rms_ffn=[rms], w_router=[router])
    ref = rc.MoePool(records=recs, expert_size=size, quant=4, **kw)
    pre = rc.MoePool(records=tiled, expert_size=tsize, quant=rc.QUANT_INT4_TILED, **kw, **extra)
    return ref, pre


def test_pretiled_pool_matches_tiling_at_upload(rc, oracle, tmp_path):
    recs, size, router, rms = synth.moe_layer(11, H, E, I, S)
    tiled, tsize = rc.tile_records(recs, size, hidden=H, n_experts=E, top_k=K, inter=I,
                                   n_shared=S, sm_count=sm_count())
    ref, pre = pools(rc, recs, size, router, rms, tiled, tsize)
    h = np.random.default_rng(2).standard_normal((6, H)).astype(np.float32)
    for t in range(h.shape[0]):
        a, ia, wa = ref.decode(0, h[t])
        b, ib, wb = pre.decode(0, h[t])
        np.testing.assert_array_equal(b, a)
        np.testing.assert_array_equal(ib, ia)
        np.testing.assert_array_equal(wb, wa)
    pa, _, _ = ref.prefill(0, h)
    pb, pids, pw = pre.prefill(0, h)
    np.testing.assert_array_equal(pb, pa)
    okw = oracle_kw(H=H, E=E, k=K, I=I, S=S, records=recs, expert_size=size, rms_ffn=rms,
                    w_router=router)
    check_tokens(oracle, h, pb, pids, pw, okw, min_checked=5)
    dec = [pre.decode(0, h[t]) for t in range(h.shape[0])]
    check_tokens(oracle, h, np.stack([d[0] for d in dec]), np.stack([d[1] for d in dec]),
                 np.stack([d[2] for d in dec]), okw, min_checked=5)
    # the same tiled records straight from a file, after a 300-byte header
    path = tmp_path / "tiled.rabbit"
    with open(path, "wb") as f:
        f.write(bytes(300))
        f.write(tiled.tobytes())
    filed = rc.MoePool(records=None, expert_size=tsize, quant=rc.QUANT_INT4_TILED, n_layers=1,
                       hidden=H, n_experts=E, top_k=K, inter=I, n_shared=S, rms_ffn=[rms],
                       w_router=[router])
    filed.upload_file(path, 300, 0, 1)
    filed.sync()
    c, _, _ = filed.decode(0, h[0])
    a, _, _ = ref.decode(0, h[0])
    np.testing.assert_array_equal(c, a)
    for p in (ref, pre, filed):
        p.free()


def test_pretiled_records_for_another_plan_are_refused(rc):
    recs, size, router, rms = synth.moe_layer(12, H, E, I, S)
    tiled, tsize = rc.tile_records(recs, size, hidden=H, n_experts=E, top_k=K, inter=I,
                                   n_shared=S, sm_count=sm_count())
    kw = dict(n_layers=1, hidden=H, n_experts=E, top_k=K, inter=I, n_shared=S,
              rms_ffn=[rms], w_router=[router], quant=rc.QUANT_INT4_TILED)
    with pytest.raises(rc.RabbitCudaError, match="tile plan"):  # record size of another plan
        rc.MoePool(records=np.zeros((E + S) * (tsize + 256), np.uint8), expert_size=tsize + 256,
                   **kw)
    bad = tiled.copy()
    bad[3 * tsize - 256:3 * tsize - 248] = np.frombuffer(b"NOTTILED", np.uint8)  # record 2
    with pytest.raises(rc.RabbitCudaError, match="not tiled for this pool"):
        rc.MoePool(records=bad, expert_size=tsize, **kw)
