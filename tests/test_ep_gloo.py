"""CPU: the expert-parallel decomposition of one MoE layer over two gloo
ranks, with the oracle as the arithmetic. Rank r applies the routed experts
e = r (mod 2) of every token (and rank 0 the residual and the shared experts);
an all-reduce (sum) of the two shares equals moe_step (forward_v2.c:362-402)
on the whole layer. This is the host-side contract
rabbit_cuda_moe_set_expert_parallel gives its callers."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

from conftest import ATOL, RTOL

H, E, K, I, S, T, G = 64, 8, 2, 64, 1, 6, 2


def _layer():
    from rabbit_b200 import synth

    return synth.moe_layer(5, H, E, I, S)


def _share(rank, h):
    """This rank's share of the layer for tokens h [T, H], by the oracle."""
    from oracle.oracle import Oracle

    orc = Oracle()
    recs, size, router, rms = _layer()
    out = np.zeros_like(h) if rank else h.copy()
    for t in range(h.shape[0]):
        xn = orc.rmsnorm(h[t], rms)
        ids, w = orc.select_top_k(orc.gemv_f32(router, xn), K)
        delta = np.zeros(H, np.float32)
        for i in range(K):
            if ids[i] >= 0 and ids[i] % G == rank:
                e = ids[i]
                delta = orc.expert_swiglu(recs[e * size:(e + 1) * size], size, 4, xn, H, I,
                                          w[i], delta)
        if rank == 0:
            for s in range(S):
                e = E + s
                delta = orc.expert_swiglu(recs[e * size:(e + 1) * size], size, 4, xn, H, I, 1.0,
                                          delta)
        out[t] += delta
    return out


def _worker(rank, port, q):
    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=G)
    h = np.random.default_rng(1).standard_normal((T, H)).astype(np.float32)
    part = torch.from_numpy(_share(rank, h))
    dist.all_reduce(part, op=dist.ReduceOp.SUM)
    if rank == 0:
        q.put(part.numpy())
    dist.destroy_process_group()


def test_expert_parallel_all_reduce_equals_moe_step():
    import multiprocessing as mp

    from oracle.oracle import Oracle

    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(G)]
    for p in procs:
        p.start()
    got = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    orc = Oracle()
    recs, size, router, rms = _layer()
    h = np.random.default_rng(1).standard_normal((T, H)).astype(np.float32)
    for t in range(T):
        want, _, _ = orc.moe_step(h[t], H=H, E=E, top_k=K, inter=I, n_shared=S, quant=4,
                                  n_records=E + S, expert_size=size, records=recs, rms_ffn=rms,
                                  w_router=router)
        np.testing.assert_allclose(got[t], want, rtol=RTOL, atol=ATOL, err_msg=f"token {t}")
