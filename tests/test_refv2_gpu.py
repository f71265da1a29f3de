"""GPU parity: the device-resident ref-v2 decode context (rabbit_cuda_refv2,
the RabbitRefV2Ctx of src/rabbit.h:160-167) against the oracle's per-token
loop of rabbit_ref_v2_forward (forward_v2.c:457-484): h = embed[id % V]; per
layer attention_step (forward_v2.c:171-246) then moe_step
(forward_v2.c:362-402); final rmsnorm; logits = lm_head^T h.

Bar: logits and the final-normed hidden within rtol 1e-4 / atol 1e-5 after
every token, the argmax identical whenever the oracle's top two logits are
apart by more than 1e-4 of the largest |logit|. Sequences run past max_ctx,
where the KV cache stops growing (forward_v2.c:198-202), and past 32 cached
positions, where the shared-memory attention splits a head's positions over
several CTAs. A token whose
router scores hold a near-tie in any layer (adjacent top-k+1 scores within
1e-5 of the largest) ends the comparison of that sequence: after it the two
sides may route differently, legitimately.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import ATOL, RTOL, near_tie, router_scores
from rabbit_b200 import synth

pytestmark = pytest.mark.gpu

CONFIGS = {
    # name: L, H, V, nh, nkv, hd, E, k, I, S, max_ctx
    "gqa": (2, 128, 1000, 4, 2, 32, 8, 2, 64, 0, 8),
    "wide_q_shared_odd_vocab": (2, 128, 997, 6, 3, 40, 4, 2, 96, 1, 6),
    "mha_one_layer": (1, 64, 512, 2, 2, 32, 4, 1, 64, 0, 4),
    # windows past 32 positions: head_dim 32 (registers, one CTA per head)
    # and head_dim 40 (shared memory, positions split over CTAs and merged)
    "long_window": (2, 128, 1000, 4, 2, 32, 8, 2, 64, 0, 80),
    "long_window_split": (1, 128, 1000, 4, 2, 40, 8, 2, 64, 0, 72),
    # the OLMoE-1B-7B shape of the full-decode workload (hidden 2048, 16 heads
    # of 128: the register attention with 4 values per lane, 64 experts top-8,
    # inter 1024) with 2 layers and a 4096-id vocabulary so the oracle stays
    # fast; the window passes 32 cached positions
    "olmoe_dims": (2, 2048, 4096, 16, 16, 128, 64, 8, 1024, 0, 48),
}

# Standard deviations of the dense weights: (embed, lm_head, norm spread,
# w_q, w_k, w_v, w_o). The OLMoE-shaped model uses the workload's N(0, 0.02).
SIGMAS = {"olmoe_dims": (1.0, 0.02, 0.1, 0.02, 0.02, 0.02, 0.02)}
DEFAULT_SIGMAS = (1.0, 0.05, 0.1, 0.15, 0.15, 0.1, 0.1)


class Model:
    """Dense + MoE weights of a small ref-v2 model and the oracle loop."""

    def __init__(self, name, seed):
        L, H, V, nh, nkv, hd, E, k, I, S, max_ctx = CONFIGS[name]
        self.L, self.H, self.V, self.nh, self.nkv, self.hd = L, H, V, nh, nkv, hd
        self.E, self.k, self.I, self.S, self.max_ctx = E, k, I, S, max_ctx
        rng = np.random.default_rng(seed)
        qd, kvd = nh * hd, nkv * hd
        f = lambda *s, sg: (rng.standard_normal(s) * sg).astype(np.float32)  # noqa: E731
        s_emb, s_lm, s_nrm, s_q, s_k, s_v, s_o = SIGMAS.get(name, DEFAULT_SIGMAS)
        self.w = {
            "embed": f(V, H, sg=s_emb),
            "lm_head": f(H, V, sg=s_lm),
            "final_norm": (1.0 + f(H, sg=s_nrm)),
            "rms_attn": [1.0 + f(H, sg=s_nrm) for _ in range(L)],
            "w_q": [f(qd, H, sg=s_q) for _ in range(L)],
            "w_k": [f(kvd, H, sg=s_k) for _ in range(L)],
            "w_v": [f(kvd, H, sg=s_v) for _ in range(L)],
            "w_o": [f(H, qd, sg=s_o) for _ in range(L)],
        }
        self.moe = [synth.moe_layer(seed * 31 + l, H, E, I, S) for l in range(L)]
        self.size = self.moe[0][1]

    def pool(self, rc):
        return rc.MoePool(records=np.concatenate([m[0] for m in self.moe]),
                          expert_size=self.size, n_layers=self.L, hidden=self.H,
                          n_experts=self.E, top_k=self.k, inter=self.I, n_shared=self.S, quant=4,
                          rms_ffn=[m[3] for m in self.moe], w_router=[m[2] for m in self.moe])

    def ctx(self, rc, pool):
        return rc.RefV2(pool, vocab=self.V, n_heads=self.nh, n_kv_heads=self.nkv,
                        head_dim=self.hd, max_ctx=self.max_ctx, weights=self.w)

    # -- oracle ---------------------------------------------------------------
    def reset(self):
        kvd = self.nkv * self.hd
        self.kc = [np.zeros((self.max_ctx, kvd), np.float32) for _ in range(self.L)]
        self.vc = [np.zeros((self.max_ctx, kvd), np.float32) for _ in range(self.L)]
        self.kv_len = [0] * self.L
        self.pos = 0

    def step(self, oracle, tid):
        """One token; returns (logits, hidden, tie) -- tie: a near-tie in the
        router scores of some layer."""
        # C semantics (forward_v2.c:459-461): id % V truncates toward zero,
        # a negative result selects row 0
        t = tid % self.V if tid >= 0 else 0
        h = self.w["embed"][t].copy()
        tie = False
        for l in range(self.L):
            h, self.kv_len[l] = oracle.attention_step(
                h, self.kc[l], self.vc[l], self.kv_len[l], self.pos, n_heads=self.nh,
                n_kv_heads=self.nkv, head_dim=self.hd,
                **{n: self.w[n][l] for n in ("rms_attn", "w_q", "w_k", "w_v", "w_o")})
            recs, size, router, rms = self.moe[l]
            tie |= near_tie(router_scores(oracle, h, rms, router), self.k, rel=1e-5)
            h, _, _ = oracle.moe_step(h, H=self.H, E=self.E, top_k=self.k, inter=self.I,
                                      n_shared=self.S, quant=4, n_records=self.E + self.S,
                                      expert_size=size, records=recs, rms_ffn=rms,
                                      w_router=router)
        self.pos += 1
        hidden = oracle.rmsnorm(h, self.w["final_norm"])
        return oracle.logits(self.w["lm_head"], hidden), hidden, tie


def clear_argmax(logits) -> bool:
    s = np.sort(logits.astype(np.float64))[::-1]
    return s[0] - s[1] > 1e-4 * max(abs(s[0]), 1e-30)


def check(got_logits, got_hidden, got_am, ref_logits, ref_hidden, what):
    np.testing.assert_allclose(got_logits, ref_logits, rtol=RTOL, atol=ATOL,
                               err_msg=f"{what}: logits")
    np.testing.assert_allclose(got_hidden, ref_hidden, rtol=RTOL, atol=ATOL,
                               err_msg=f"{what}: hidden")
    if clear_argmax(ref_logits):
        assert got_am == int(np.argmax(ref_logits)), what


@pytest.mark.parametrize("name", list(CONFIGS))
def test_steps_match_oracle_past_max_ctx(rc, oracle, name):
    m = Model(name, seed=sum(map(ord, name)))
    pool = m.pool(rc)
    ctx = m.ctx(rc, pool)
    rng = np.random.default_rng(5)
    ids = rng.integers(-3, 2 * m.V, size=m.max_ctx + 5)  # negatives and ids >= V too
    m.reset()
    compared = 0
    for i, tid in enumerate(ids):
        ref_logits, ref_hidden, tie = m.step(oracle, int(tid))
        logits, hidden, am = ctx.step(int(tid))
        assert ctx.position == i + 1
        if tie:
            break
        check(logits, hidden, am, ref_logits, ref_hidden, f"{name} token {i}")
        compared += 1
    assert compared >= m.max_ctx, f"only {compared} tokens compared (router near-ties)"
    ctx.free()
    pool.free()


@pytest.mark.parametrize("name", ["gqa", "wide_q_shared_odd_vocab"])
def test_prefill_reset_and_greedy_generate(rc, oracle, name):
    m = Model(name, seed=sum(map(ord, name)) + 1)
    pool = m.pool(rc)
    ctx = m.ctx(rc, pool)
    prompt = np.random.default_rng(9).integers(0, m.V, size=5)

    # prefill == the oracle's tokens one by one; only the last outputs return
    m.reset()
    for tid in prompt:
        ref_logits, ref_hidden, tie = m.step(oracle, int(tid))
        if tie:
            pytest.skip("router near-tie in the prompt for this seed")
    logits, hidden, am = ctx.prefill(prompt)
    assert ctx.position == len(prompt)
    check(logits, hidden, am, ref_logits, ref_hidden, "prefill")

    # greedy continuation chained on the device vs. the oracle's argmax chain
    n_new = m.max_ctx + 3
    got = ctx.generate(n_new)
    assert ctx.position == len(prompt) + n_new
    last = int(np.argmax(ref_logits))
    assert clear_argmax(ref_logits), "pick another seed: unclear first argmax"
    for i in range(n_new):
        ref_logits, _, tie = m.step(oracle, last)
        if tie or not clear_argmax(ref_logits):
            break
        last = int(np.argmax(ref_logits))
        assert got[i] == last, f"generated token {i}: {got[:i + 1]} vs oracle {last}"

    # reset: the same prompt again gives the same outputs
    ctx.reset()
    assert ctx.position == 0
    logits2, hidden2, am2 = ctx.prefill(prompt)
    np.testing.assert_array_equal(logits2, logits)
    np.testing.assert_array_equal(hidden2, hidden)
    assert am2 == am
    ctx.free()
    pool.free()


def test_generate_needs_a_step_and_bounds(rc):
    m = Model("mha_one_layer", seed=3)
    pool = m.pool(rc)
    ctx = m.ctx(rc, pool)
    with pytest.raises(rc.RabbitCudaError, match="no step"):
        ctx.generate(2)
    ctx.step(1)
    with pytest.raises(rc.RabbitCudaError):
        ctx.generate(0)
    with pytest.raises(rc.RabbitCudaError):
        ctx.generate(4097)
    out = ctx.generate(3)
    assert ((out >= 0) & (out < m.V)).all()
    ctx.free()
    pool.free()


def test_create_rejects_mismatched_shapes(rc):
    m = Model("gqa", seed=4)
    pool = m.pool(rc)
    for kw in ({"n_heads": 3, "n_kv_heads": 2, "head_dim": 32},   # nh not a multiple of nkv
               {"n_heads": 4, "n_kv_heads": 2, "head_dim": 31},   # odd head_dim
               {"n_heads": 4, "n_kv_heads": 2, "head_dim": 32, "max_ctx": 257}):
        with pytest.raises(rc.RabbitCudaError):
            rc.RefV2(pool, vocab=m.V, weights=m.w, **kw)
    pool.free()


def test_olmoe_shape_synthetic_decode_is_finite_and_repeatable(rc):
    """The OLMoE-shaped model (16 layers, hidden 2048, 16 heads of 128,
    64 experts top-8, inter 1024, vocab 50304) with device-filled weights:
    a short prompt and a greedy continuation give finite logits, and the same
    prompt after reset gives the same logits."""
    L, H, E, k, I, V = 16, 2048, 64, 8, 1024, 50304
    pool = rc.MoePool(records=None, expert_size=synth.expert_record_size(H, I), n_layers=L,
                      hidden=H, n_experts=E, top_k=k, inter=I, quant=4,
                      rms_ffn=[np.ones(H, np.float32)] * L,
                      w_router=[np.random.default_rng(l).standard_normal((E, H)).astype(
                          np.float32) * 0.02 for l in range(L)])
    pool.fill_synthetic(7)
    ctx = rc.RefV2(pool, vocab=V, n_heads=16, n_kv_heads=16, head_dim=128, max_ctx=256)
    ctx.fill_synthetic(11, 0.02)
    prompt = [1, 50, 2000, 50303, 7]
    logits, hidden, am = ctx.prefill(prompt)
    assert np.isfinite(logits).all() and np.isfinite(hidden).all()
    assert am == int(np.argmax(logits))
    out = ctx.generate(8)
    assert ((out >= 0) & (out < V)).all()
    ctx.reset()
    logits2, _, am2 = ctx.prefill(prompt)
    np.testing.assert_allclose(logits2, logits, rtol=1e-6, atol=1e-7)
    ctx.free()
    pool.free()
