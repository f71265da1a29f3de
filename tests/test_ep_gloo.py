"""CPU: the expert-parallel decompositions of one MoE layer over gloo ranks,
with the oracle as the arithmetic, in the library's two exchange forms.
All-reduce: rank r applies the routed experts e = r (mod 2) of every token
(and rank 0 the residual and the shared experts); an all-reduce (sum) of the
two shares equals moe_step (forward_v2.c:362-402) on the whole layer.
All-to-all: each rank's own tokens go to the experts' owners and come back
(below), bit-identical to moe_step. These are the host-side contracts
rabbit_cuda_moe_set_expert_parallel and rabbit_cuda_moe_set_ep give their
callers."""
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


# ------------------------------------------------------------ all-to-all ----
# The library's other exchange (rabbit_cuda_moe_set_ep with
# RABBIT_CUDA_EP_ALLTOALL), restated on the oracle: each rank owns its own
# tokens and routes them; for every peer it fills a list of fixed capacity
# cap = T * max(1, min(k, E / N)) rows with the pairs whose expert that peer
# holds (e mod N), in token-major, slot-minor order, each row {token, slot,
# local record e / N, 1} and the token's normalised row, unused rows zero.
# The peer runs its experts on the rows it received and returns each pair's
# unweighted expert output at the row it came in; the sender then adds
# w_i * output_i in slot order, local or returned, then the shared experts,
# which is moe_step's own arithmetic (forward_v2.c:362-402): the result is
# bit-identical to moe_step on the whole layer.
T_OWN = 5


def _exchange(dist, torch, peers, send):
    """send[qi] goes to peer peers[qi]; returns what each peer sent here."""
    recv = [torch.zeros_like(torch.from_numpy(s)) for s in send]
    reqs = []
    for qi, q in enumerate(peers):
        reqs.append(dist.irecv(recv[qi], src=q))
    for qi, q in enumerate(peers):
        reqs.append(dist.isend(torch.from_numpy(np.ascontiguousarray(send[qi])), dst=q))
    for r in reqs:
        r.wait()
    return [r.numpy() for r in recv]


def _a2a_worker(rank, world, port, q):
    import torch
    import torch.distributed as dist

    from oracle.oracle import Oracle

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    orc = Oracle()
    recs, size, router, rms = _layer()

    def rec(e):
        return recs[e * size:(e + 1) * size]

    h = np.random.default_rng(100 + rank).standard_normal((T_OWN, H)).astype(np.float32)
    xn = np.stack([orc.rmsnorm(h[t], rms) for t in range(T_OWN)])
    routed = [orc.select_top_k(orc.gemv_f32(router, xn[t]), K) for t in range(T_OWN)]
    cap = T_OWN * max(1, min(K, E // world))
    peers = [p for p in range(world) if p != rank]
    meta = np.zeros((len(peers), cap, 4), np.int32)
    rows = np.zeros((len(peers), cap, H), np.float32)
    pos = np.full((T_OWN, K), -1, np.int64)
    count = [0] * len(peers)
    for t, (ids, _) in enumerate(routed):
        for i in range(K):
            e = int(ids[i])
            if e < 0 or e % world == rank:
                continue
            qi = peers.index(e % world)
            c = count[qi]
            assert c < cap, "a peer's list overflows its capacity"
            meta[qi, c] = (t, i, e // world, 1)
            rows[qi, c] = xn[t]
            pos[t, i] = c
            count[qi] += 1
    got_meta = _exchange(dist, torch, peers, list(meta))
    got_rows = _exchange(dist, torch, peers, list(rows))
    ret = np.zeros((len(peers), cap, H), np.float32)
    for qi in range(len(peers)):
        prev = (-1, -1)
        for r in range(cap):
            t, i, local, used = (int(v) for v in got_meta[qi][r])
            if not used:
                assert not got_meta[qi][r:].any(), "used rows come first"
                break
            assert (t, i) > prev, "a list is in token-major, slot-minor order"
            prev = (t, i)
            e = local * world + rank
            ret[qi, r] = orc.expert_swiglu(rec(e), size, 4, got_rows[qi][r], H, I, 1.0)
    back = _exchange(dist, torch, peers, list(ret))
    out = np.empty_like(h)
    for t, (ids, w) in enumerate(routed):
        delta = np.zeros(H, np.float32)
        for i in range(K):
            e = int(ids[i])
            if e < 0:
                continue
            if e % world == rank:
                delta = orc.expert_swiglu(rec(e), size, 4, xn[t], H, I, w[i], delta)
            else:
                dj = back[peers.index(e % world)][pos[t, i]]
                delta = delta + np.float32(w[i]) * dj
        for s in range(S):
            delta = orc.expert_swiglu(rec(E + s), size, 4, xn[t], H, I, 1.0, delta)
        out[t] = h[t] + delta
    q.put((rank, h, out, sum(count)))
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_expert_parallel_all_to_all_equals_moe_step(world):
    import multiprocessing as mp

    from oracle.oracle import Oracle

    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_a2a_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert sum(r[3] for r in results) > 0, "no pair crossed ranks"
    orc = Oracle()
    recs, size, router, rms = _layer()
    for rank, h, out, _ in results:
        for t in range(T_OWN):
            want, _, _ = orc.moe_step(h[t], H=H, E=E, top_k=K, inter=I, n_shared=S, quant=4,
                                      n_records=E + S, expert_size=size, records=recs,
                                      rms_ffn=rms, w_router=router)
            np.testing.assert_array_equal(out[t], want, err_msg=f"rank {rank} token {t}")
