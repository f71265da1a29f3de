"""GPU: the expert-parallel multi-token path of the CUDA pool over two gloo
ranks. Each rank is a process with its own pool on cuda:0 holding the routed
experts e = r (mod 2) of the layer (as local records e / 2) plus, on rank 0,
the shared expert, set up with rabbit_cuda_moe_set_expert_parallel(r, 2); each
prefills the same tokens through the host-buffer entry point and the two
outputs are summed by a gloo all-reduce of host tensors. Bar: the sum equals
the oracle's moe_step (forward_v2.c:362-402) per token within rtol 1e-4 /
atol 1e-5, and both ranks report the full routing."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

H, E, K, I, S, T, G = 512, 8, 2, 1024, 1, 24, 2


def _layer():
    from rabbit_b200 import synth

    return synth.moe_layer(17, H, E, I, S)


def _tokens():
    return np.random.default_rng(2).standard_normal((T, H)).astype(np.float32)


def _worker(rank, port, q):
    import torch
    import torch.distributed as dist

    from rabbit_b200 import capi

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=G)
    try:
        recs, size, router, rms = _layer()
        mine = [recs[e * size:(e + 1) * size] for e in range(rank, E, G)]
        mine += [recs[(E + s) * size:(E + s + 1) * size] for s in range(S)]
        pool = capi.MoePool(records=np.concatenate(mine), expert_size=size, n_layers=1,
                            hidden=H, n_experts=E, top_k=K, inter=I, n_shared=S, quant=4,
                            rms_ffn=[rms], w_router=[router], experts_per_layer=E // G + S)
        pool.set_expert_parallel(rank, G)
        out, ids, w = pool.prefill(0, _tokens())
        pool.free()
        part = torch.from_numpy(out)
        dist.all_reduce(part, op=dist.ReduceOp.SUM)
        if rank == 0:
            q.put((part.numpy(), ids, w))
        else:
            q.put(("ids", ids))
    finally:
        dist.destroy_process_group()


def test_cuda_pool_shares_over_gloo_sum_to_the_layer(oracle):
    import multiprocessing as mp

    from conftest import check_tokens, oracle_kw

    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(G)]
    for p in procs:
        p.start()
    got = [q.get(timeout=300) for _ in range(G)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    total, ids, w = next(g for g in got if not isinstance(g[0], str))
    other = next(g for g in got if isinstance(g[0], str))
    np.testing.assert_array_equal(other[1], ids)
    recs, size, router, rms = _layer()
    kw = oracle_kw(H=H, E=E, k=K, I=I, S=S, records=recs, expert_size=size, rms_ffn=rms,
                   w_router=router)
    check_tokens(oracle, _tokens(), total, ids, w, kw, min_checked=T - 2)
