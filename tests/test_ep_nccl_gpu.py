"""GPU (two or more devices): the library's own expert-parallel exchange
(rabbit_cuda_ep_* over NCCL, rabbit_cuda_moe_set_ep). Two processes, one GPU
each; rank r's pool holds the routed experts e = r (mod 2) of each layer plus
the shared ones.

  * all-to-all: each rank passes its own tokens; the outputs must equal, bit
    for bit, what one pool holding the whole layer gives for those tokens
    (same pairs, same combine order), and the oracle's moe_step
    (forward_v2.c:362-402) within rtol 1e-4 / atol 1e-5;
  * all-reduce: both ranks pass the same tokens and must both get the layer
    output (oracle within rtol 1e-4 / atol 1e-5; the two ranks' outputs equal);
  * the per-call timing counts the calls and puts the exchange inside them.

Skipped with fewer than two GPUs."""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

G = 2
SHAPES = {
    # H, E, k, I, S, tokens per rank
    "small": (512, 8, 2, 1024, 1, 12),
    "deepseek": (2048, 64, 6, 1408, 2, 16),
}


def _gpus() -> int:
    try:
        import torch

        return torch.cuda.device_count()
    except Exception:
        return 0


def _layer(shape):
    from rabbit_b200 import synth

    H, E, k, I, S, _ = SHAPES[shape]
    return synth.moe_layer(23, H, E, I, S)


def _tokens(shape):
    H, _, _, _, _, T = SHAPES[shape]
    return np.random.default_rng(5).standard_normal((G * T, H)).astype(np.float32)


def _share(recs, size, E, S, rank):
    mine = [recs[e * size:(e + 1) * size] for e in range(rank, E, G)]
    mine += [recs[(E + s) * size:(E + s + 1) * size] for s in range(S)]
    return np.concatenate(mine)


def _worker(rank, shape, q_id, q_out):
    from rabbit_b200 import capi

    try:
        H, E, k, I, S, T = SHAPES[shape]
        capi.check(capi.lib().rabbit_cuda_set_device(rank))
        if rank == 0:
            uid = capi.ep_unique_id()
            for _ in range(G - 1):
                q_id.put(uid)
        else:
            uid = q_id.get(timeout=120)
        ep = capi.Ep(uid, rank, G, rank)
        recs, size, router, rms = _layer(shape)
        pool = capi.MoePool(records=_share(recs, size, E, S, rank), expert_size=size,
                            n_layers=1, hidden=H, n_experts=E, top_k=k, inter=I, n_shared=S,
                            quant=4, rms_ffn=[rms], w_router=[router],
                            experts_per_layer=E // G + S, device=rank)
        h = _tokens(shape)
        res = {"rank": rank}
        ep.set_timing(True)
        pool.set_ep(ep, capi.EP_ALLTOALL)
        mine = h[rank * T:(rank + 1) * T]
        res["a2a"] = pool.prefill(0, mine)
        res["a2a_again"] = pool.prefill(0, mine)[0]
        pool.set_ep(ep, capi.EP_ALLREDUCE)
        res["ar"] = pool.prefill(0, h)
        res["stats"] = ep.stats()
        pool.set_ep(None)
        if rank == 0:  # the whole layer in one pool, for the bit-exact comparison
            full = capi.MoePool(records=recs, expert_size=size, n_layers=1, hidden=H,
                                n_experts=E, top_k=k, inter=I, n_shared=S, quant=4,
                                rms_ffn=[rms], w_router=[router], device=rank)
            res["single"] = full.prefill(0, h)
            full.free()
        pool.free()
        ep.free()
        q_out.put(res)
    except Exception as e:  # reported to the test, which fails on it
        q_out.put({"rank": rank, "error": repr(e)})


@pytest.mark.parametrize("shape", list(SHAPES))
def test_library_exchange_all_to_all_and_all_reduce(oracle, shape):
    if _gpus() < G:
        pytest.skip(f"needs {G} GPUs")
    import multiprocessing as mp

    from conftest import check_tokens, oracle_kw

    ctx = mp.get_context("spawn")
    q_id, q_out = ctx.Queue(), ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, shape, q_id, q_out)) for r in range(G)]
    for p in procs:
        p.start()
    got = {}
    for _ in range(G):
        r = q_out.get(timeout=600)
        got[r["rank"]] = r
    for p in procs:
        p.join(timeout=120)
    for r in range(G):
        assert "error" not in got[r], got[r].get("error")
    for p in procs:
        assert p.exitcode == 0

    H, E, k, I, S, T = SHAPES[shape]
    h = _tokens(shape)
    single_h, single_ids, single_w = got[0]["single"]
    for r in range(G):
        out, ids, w = got[r]["a2a"]
        sl = slice(r * T, (r + 1) * T)
        np.testing.assert_array_equal(ids, single_ids[sl])
        np.testing.assert_array_equal(w, single_w[sl])
        np.testing.assert_array_equal(out, single_h[sl], err_msg=f"rank {r}: all-to-all")
        np.testing.assert_array_equal(got[r]["a2a_again"], out)
    np.testing.assert_array_equal(got[0]["ar"][0], got[1]["ar"][0])
    np.testing.assert_array_equal(got[0]["ar"][1], single_ids)

    recs, size, router, rms = _layer(shape)
    kw = oracle_kw(H=H, E=E, k=k, I=I, S=S, records=recs, expert_size=size, rms_ffn=rms,
                   w_router=router)
    a2a = np.concatenate([got[r]["a2a"][0] for r in range(G)])
    check_tokens(oracle, h, a2a, single_ids, single_w, kw, min_checked=G * T - 3)
    check_tokens(oracle, h, got[0]["ar"][0], got[0]["ar"][1], got[0]["ar"][2], kw,
                 min_checked=G * T - 3)
    for r in range(G):
        st = got[r]["stats"]
        assert st["calls"] == 3
        assert 0.0 < st["exchange_ms"] < st["total_ms"]
