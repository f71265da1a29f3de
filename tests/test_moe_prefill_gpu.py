"""GPU parity: the multi-token MoE path (rabbit_cuda_moe_prefill[_dev]) --
T tokens through one layer's MoE block at once -- against the oracle's
moe_step (forward_v2.c:362-402) run on each token alone.

Bar: per token, top-k expert ids identical (tokens whose router scores hold a
near-tie -- adjacent top-k+1 scores within 1e-6 of the largest -- excluded),
routing weights, the MoE delta and h_out within rtol 1e-4 / atol 1e-5.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import ATOL, RTOL, check_tokens, check_tokens_long, exact_moe_layer, oracle_many
from rabbit_b200 import synth

pytestmark = pytest.mark.gpu

SHAPES = {
    # name: H, E, k, I, S
    "small_top4": (256, 16, 4, 128, 0),
    "shared_experts": (256, 16, 3, 96, 2),
    "w2_two_chunks": (128, 8, 2, 2048, 0),
    "mixtral_like": (512, 8, 2, 1024, 0),
    # hidden 6144: gate/up tiles of 4 rows, two of them per work item
    "wide_hidden": (6144, 8, 2, 128, 0),
}


def make_pool(rc, H, E, k, I, S, seed, n_layers=1, quant=4):
    recs, size, router, rms = synth.moe_layer(seed, H, E, I, S)
    if quant == 0:
        rng = np.random.default_rng(seed)
        recs = np.concatenate([synth.f32_expert_record(rng, H, I) for _ in range(E + S)])
        size = recs.size // (E + S)
    pool = rc.MoePool(records=np.concatenate([recs] * n_layers), expert_size=size,
                      n_layers=n_layers, hidden=H, n_experts=E, top_k=k, inter=I, n_shared=S,
                      quant=quant, rms_ffn=[rms] * n_layers, w_router=[router] * n_layers)
    kw = dict(H=H, E=E, top_k=k, inter=I, n_shared=S, quant=quant, n_records=E + S,
              expert_size=size, records=recs, rms_ffn=rms, w_router=router)
    return pool, kw


@pytest.mark.parametrize("name", list(SHAPES))
@pytest.mark.parametrize("T", [1, 5, 33])
def test_prefill_matches_oracle_per_token(rc, oracle, name, T):
    H, E, k, I, S = SHAPES[name]
    pool, kw = make_pool(rc, H, E, k, I, S, seed=sum(map(ord, name)) + T)
    h = np.random.default_rng(T).standard_normal((T, H)).astype(np.float32)
    got_h, ids, w = pool.prefill(0, h)
    check_tokens(oracle, h, got_h, ids, w, kw, min_checked=max(1, T - 2))
    pool.free()


def test_prefill_many_tokens_per_expert_and_decode_agree(rc, oracle):
    """64 tokens over 8 experts top-2: ~16 tokens per expert, more than one
    staged chunk of 8; the prefill equals the per-token decode on the GPU."""
    H, E, k, I, S = 256, 8, 2, 256, 1
    pool, kw = make_pool(rc, H, E, k, I, S, seed=77)
    h = np.random.default_rng(5).standard_normal((64, H)).astype(np.float32)
    got_h, ids, w = pool.prefill(0, h)
    check_tokens(oracle, h, got_h, ids, w, kw, min_checked=60)
    for t in range(0, 64, 9):
        dh, dids, dw = pool.decode(0, h[t])
        np.testing.assert_allclose(got_h[t], dh, rtol=RTOL, atol=ATOL)
        np.testing.assert_array_equal(ids[t], dids)
    pool.free()


@pytest.mark.parametrize("T", [8, 32])
def test_prefill_deepseek_shaped_layer(rc, oracle, T):
    """hidden 2048, 64 routed experts top-6 + 2 shared, inter 1408 (W2 in two
    column chunks of 704 inputs); T = 32 is the DeepSeek-MoE-16B-shaped
    prefill chunk, where the two shared experts see every token (two work
    units each)."""
    H, E, k, I, S = 2048, 64, 6, 1408, 2
    pool, kw = make_pool(rc, H, E, k, I, S, seed=4)
    h = np.random.default_rng(4 + T).standard_normal((T, H)).astype(np.float32)
    got_h, ids, w = pool.prefill(0, h)
    check_tokens(oracle, h, got_h, ids, w, kw, min_checked=T - 2,
                 ref=oracle_many(oracle, h, kw))
    pool.free()


def test_prefill_mixtral_8x22b_shaped_layer_and_expert_parallel_shares(rc, oracle):
    """One Mixtral-8x22B-shaped layer (hidden 6144, 8 experts top-2, inter
    16384: W2 in 16 column chunks of 1024 inputs) with a batch of 64 decode
    tokens through the multi-token path, then the same layer split
    expert-parallel over 2, 4 and 8 ranks, emulated as pools on this GPU
    (rank r holds experts e = r mod G): the whole layer and each sum of
    shares against the oracle's moe_step per token. Rows of W2 sum 16384
    products, and the oracle's serial fp32 sum is itself up to ~2e-5 from the
    exact value there, so each element may also differ by the oracle's own
    deviation from the float64 value of the same quantised layer."""
    H, E, k, I, S, T = 6144, 8, 2, 16384, 0, 64
    recs, size, router, rms = synth.moe_layer(5, H, E, I, S)
    kw = dict(H=H, E=E, top_k=k, inter=I, n_shared=S, quant=4, n_records=E + S,
              expert_size=size, records=recs, rms_ffn=rms, w_router=router)
    h = np.random.default_rng(55).standard_normal((T, H)).astype(np.float32)
    ref = oracle_many(oracle, h, kw)
    exact = exact_moe_layer(oracle, h, kw, ref)
    pool = rc.MoePool(records=recs, expert_size=size, n_layers=1, hidden=H, n_experts=E,
                      top_k=k, inter=I, n_shared=S, quant=4, rms_ffn=[rms], w_router=[router])
    got_h, ids, w = pool.prefill(0, h)
    pool.free()
    check_tokens_long(oracle, h, got_h, ids, w, kw, ref, exact, min_checked=T - 2)
    rec_of = lambda e: recs[e * size:(e + 1) * size]  # noqa: E731
    for G in (2, 4, 8):
        total = np.zeros_like(h)
        for r in range(G):
            share = rc.MoePool(records=np.concatenate([rec_of(e) for e in range(r, E, G)]),
                               expert_size=size, n_layers=1, hidden=H, n_experts=E, top_k=k,
                               inter=I, n_shared=S, quant=4, rms_ffn=[rms], w_router=[router],
                               experts_per_layer=E // G)
            share.set_expert_parallel(r, G)
            out, sids, _ = share.prefill(0, h)
            np.testing.assert_array_equal(sids, ids)
            total += out
            share.free()
        check_tokens_long(oracle, h, total, ids, w, kw, ref, exact, min_checked=T - 2)


def test_prefill_dev_in_place_and_second_layer(rc, oracle):
    import torch

    H, E, k, I, S = 256, 16, 4, 128, 0
    recs, size, router, rms = synth.moe_layer(9, H, E, I, S)
    router2 = np.ascontiguousarray(router[::-1])
    pool = rc.MoePool(records=np.concatenate([recs, recs]), expert_size=size, n_layers=2,
                      hidden=H, n_experts=E, top_k=k, inter=I, n_shared=S, quant=4,
                      rms_ffn=[rms, rms], w_router=[router, router2])
    h = np.random.default_rng(11).standard_normal((12, H)).astype(np.float32)
    d = torch.from_numpy(h).cuda()
    stream = torch.cuda.current_stream().cuda_stream
    pool.prefill_dev(1, d.data_ptr(), d.data_ptr(), 12, 0, 0, stream)  # h_out aliases h_in
    pool.check(stream)
    kw = dict(H=H, E=E, top_k=k, inter=I, n_shared=S, quant=4, n_records=E + S,
              expert_size=size, records=recs, rms_ffn=rms, w_router=router2)
    check_tokens(oracle, h, d.cpu().numpy(), None, None, kw, min_checked=10)
    pool.free()


def test_prefill_fp32_experts_run_per_token(rc, oracle):
    """Records outside the group-32 layout take the per-token decode."""
    H, E, k, I, S = 64, 4, 2, 32, 0
    pool, kw = make_pool(rc, H, E, k, I, S, seed=3, quant=0)
    h = np.random.default_rng(2).standard_normal((6, H)).astype(np.float32)
    got_h, ids, w = pool.prefill(0, h)
    check_tokens(oracle, h, got_h, ids, w, kw, min_checked=5)
    pool.free()


def test_prefill_rejects_bad_arguments(rc):
    H, E, k, I, S = 64, 4, 2, 64, 0
    pool, _ = make_pool(rc, H, E, k, I, S, seed=1)
    h = np.zeros((1, H), np.float32)
    with pytest.raises(rc.RabbitCudaError, match="n_tokens"):
        rc.check(rc.lib().rabbit_cuda_moe_prefill(pool.handle, 0, h.ctypes.data, h.ctypes.data,
                                                  0, None, None))
    with pytest.raises(rc.RabbitCudaError, match="n_tokens"):
        rc.check(rc.lib().rabbit_cuda_moe_prefill(pool.handle, 0, h.ctypes.data, h.ctypes.data,
                                                  257, None, None))
    with pytest.raises(rc.RabbitCudaError, match="out of range"):
        pool.prefill(3, h)
    pool.free()


@pytest.mark.parametrize("G", [2, 4])
def test_expert_parallel_shares_sum_to_the_layer(rc, oracle, G):
    """G pools, each holding the routed experts e = r (mod G) of one layer (as
    local records e / G) plus the shared experts, with
    rabbit_cuda_moe_set_expert_parallel(r, G): the sum of their outputs is
    the layer output (what an all-reduce over G ranks computes)."""
    H, E, k, I, S = 256, 8, 2, 256, 1
    recs, size, router, rms = synth.moe_layer(21, H, E, I, S)
    rec_of = lambda e: recs[e * size:(e + 1) * size]  # noqa: E731
    h = np.random.default_rng(6).standard_normal((40, H)).astype(np.float32)
    total = np.zeros_like(h)
    for r in range(G):
        mine = [rec_of(e) for e in range(r, E, G)] + [rec_of(E + s) for s in range(S)]
        pool = rc.MoePool(records=np.concatenate(mine), expert_size=size, n_layers=1, hidden=H,
                          n_experts=E, top_k=k, inter=I, n_shared=S, quant=4, rms_ffn=[rms],
                          w_router=[router], experts_per_layer=E // G + S)
        pool.set_expert_parallel(r, G)
        out, ids, w = pool.prefill(0, h)
        total += out
        if r == 0:
            all_ids, all_w = ids, w
        else:
            np.testing.assert_array_equal(ids, all_ids)  # routing is computed in full everywhere
        with pytest.raises(rc.RabbitCudaError, match="expert-parallel"):
            pool.decode(0, h[0])
        pool.free()
    kw = dict(H=H, E=E, top_k=k, inter=I, n_shared=S, quant=4, n_records=E + S, expert_size=size,
              records=recs, rms_ffn=rms, w_router=router)
    check_tokens(oracle, h, total, all_ids, all_w, kw, min_checked=36)


def test_expert_parallel_rejects_bad_shares(rc):
    H, E, k, I, S = 64, 8, 2, 64, 0
    pool, _ = make_pool(rc, H, E, k, I, S, seed=2)
    with pytest.raises(rc.RabbitCudaError):
        pool.set_expert_parallel(0, 3)  # 8 experts do not split over 3 ranks
    with pytest.raises(rc.RabbitCudaError):
        pool.set_expert_parallel(0, 2)  # this pool holds all 8 experts per layer
    with pytest.raises(rc.RabbitCudaError):
        pool.set_expert_parallel(2, 2)
    pool.set_expert_parallel(0, 1)
    pool.free()
