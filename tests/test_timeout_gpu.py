"""GPU: the bounded-wait failure path of the fused MoE decode, run for real.

A test hook (rabbit_cuda_moe_debug_withhold_score) keeps every CTA from
publishing one router score for the next decode, so every CTA's bounded
wait for that score runs out -- a flag that nothing sets; no copy is in
flight at that point of the kernel, and no GPU fault is involved. Bar: the
launch ends, rabbit_cuda_moe_check reports RABBIT_CUDA_ERR_TIMEOUT (and
clears the error word), and the next decodes on the same pool -- device and
host buffers -- match the oracle's moe_step (forward_v2.c:362-402) within
rtol 1e-4 / atol 1e-5 with the same expert ids.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import check_tokens, oracle_kw
from rabbit_b200 import synth

pytestmark = pytest.mark.gpu

# a 64 x 2048 router (512 KB) is split over the CTAs, which publish the scores
H, E, K, I, S = 2048, 64, 8, 256, 0


def test_a_wait_that_runs_out_is_a_status_and_the_pool_recovers(rc, oracle):
    import torch

    recs, size, router, rms = synth.moe_layer(23, H, E, I, S)
    pool = rc.MoePool(records=recs, expert_size=size, n_layers=1, hidden=H, n_experts=E,
                      top_k=K, inter=I, n_shared=S, quant=4, rms_ffn=[rms], w_router=[router])
    okw = oracle_kw(H=H, E=E, k=K, I=I, S=S, records=recs, expert_size=size, rms_ffn=rms,
                    w_router=router)
    h = np.random.default_rng(8).standard_normal((3, H)).astype(np.float32)
    stream = torch.cuda.current_stream().cuda_stream
    d_h = torch.from_numpy(h[0]).cuda()
    out = torch.full_like(d_h, float("nan"))
    lib = rc.lib()
    try:
        rc.check(lib.rabbit_cuda_set_wait_limit_us(20000))  # 20 ms
        rc.check(lib.rabbit_cuda_moe_debug_withhold_score(pool.handle, 5))
        pool.decode_dev(0, d_h.data_ptr(), out.data_ptr(), 0, 0, stream)
        with pytest.raises(rc.RabbitCudaError) as ei:
            pool.check(stream)
        assert ei.value.status == rc.ERR_TIMEOUT, ei.value
        pool.check(stream)  # the error word was cleared
    finally:
        rc.check(lib.rabbit_cuda_set_wait_limit_ms(2000))
    # the next decodes on the same pool are right
    got = []
    for t in range(h.shape[0]):
        o = torch.empty_like(d_h)
        ids = torch.zeros(K, dtype=torch.int32, device="cuda")
        w = torch.zeros(K, dtype=torch.float32, device="cuda")
        x = torch.from_numpy(h[t]).cuda()
        pool.decode_dev(0, x.data_ptr(), o.data_ptr(), ids.data_ptr(), w.data_ptr(), stream)
        pool.check(stream)
        got.append((o.cpu().numpy(), ids.cpu().numpy(), w.cpu().numpy()))
    check_tokens(oracle, h, np.stack([g[0] for g in got]), np.stack([g[1] for g in got]),
                 np.stack([g[2] for g in got]), okw, min_checked=2)
    hd, hids, hw = pool.decode(0, h[1])
    check_tokens(oracle, h[1:2], hd[None], hids[None], hw[None], okw, min_checked=1)
    pool.free()


def test_withhold_hook_refuses_pools_that_publish_no_scores(rc):
    recs, size, router, rms = synth.moe_layer(3, 256, 8, 64, 0)
    pool = rc.MoePool(records=recs, expert_size=size, n_layers=1, hidden=256, n_experts=8,
                      top_k=2, inter=64, n_shared=0, quant=4, rms_ffn=[rms], w_router=[router])
    assert rc.lib().rabbit_cuda_moe_debug_withhold_score(pool.handle, 1) == rc.ERR_UNSUPPORTED
    pool.free()
