#!/usr/bin/env python3
"""Benchmark of the routed-expert hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl rabbit|reference]

Workload (the MoE-layer decode configuration): Mixtral-shaped MoE blocks,
hidden 4096, expert FFN 14336 SwiGLU, 8 experts top-2, group-32 int4 experts,
fp32 router N(0, 0.02), batch 1. A step is one decode token through the MoE
blocks of 32 distinct layers (28.2 GB of resident experts, far larger than the
126 MB L2), h chained layer to layer: 32 launches of the fused decode kernel
(rmsnorm + router + top-2 + gate/up + SiLU + down + combine).

metric: algorithmic bytes streamed per second (GB/s): per token-layer the
router (E*H*4 B) plus, for each selected expert, 2*B(I*H) + B(H*I) with
B(n) = 4 + 4*ceil(n/32) + n/2 -- 220,332,056 B. tokens/s is reported beside it.

N > 1: one process per GPU (torchrun); each rank decodes its own token stream
through its own resident copy (data-parallel decode replicas, no collective
on the data path), so per-GPU work is fixed: "scaling": "weak".

--impl reference times the reference's own C (oracle/_ref, built from the
reference sources) on the host cores, on the same workload and metric.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

H, I, E, TOPK = 4096, 14336, 8, 2
LAYERS = 32  # distinct layers per step (--layers)
SEED = 1
METRIC = "MoE decode int4 expert GB/s (Mixtral-shaped layer, batch 1)"
WORKLOAD = "Mixtral-shaped MoE layer decode x {} distinct layers per step"


def measured_peak():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except Exception:
            pass
    return 6650.0, "fallback"


def profile_traffic():
    """Per-launch DRAM traffic of the decode kernel from the committed ncu summary."""
    p = ROOT / "profiles" / "traffic.json"
    if p.exists():
        try:
            return json.loads(p.read_text()).get("k_moe_decode_g32_bytes_per_launch")
        except Exception:
            return None
    return None


# ------------------------------------------------------------ clocks -------
class ClockSampler:
    """nvidia-smi clocks + throttle reasons for one GPU while the timed region runs."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id: str | None):
        self.gpu_id = gpu_id
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        cmd = ["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
               "-lms", "50"]
        if self.gpu_id:
            cmd += ["-i", self.gpu_id]
        try:
            self.proc = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL,
                                         text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
        except OSError:
            self.proc = None
        time.sleep(0.3)

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.1)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self._t.join(timeout=2)
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        loaded = [s for s in sm if mx and s > 0.5 * max(mx)] or sm
        return {"sm_mhz": statistics.median(loaded) if loaded else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------------ CPU side -----
def host_layer(seed: int = SEED):
    """One Mixtral-shaped layer on the host (8 int4 experts, router, norm)."""
    from rabbit_b200 import synth

    return synth.moe_layer(seed, H, E, I, 0)


def layer_bytes() -> int:
    from rabbit_b200 import synth

    return 4 * E * H + TOPK * (3 * synth.int4_nbytes(H * I))


def time_cpu_moe(checker, layer, tokens: int, threads: int) -> tuple[float, int]:
    """Run `tokens` moe_step calls per thread; returns (seconds, token-layers)."""
    from concurrent.futures import ThreadPoolExecutor

    recs, size, router, rms = layer
    kw = dict(H=H, E=E, top_k=TOPK, inter=I, n_shared=0, quant=4, n_records=E,
              expert_size=size, records=recs, rms_ffn=rms, w_router=router)
    rng = np.random.default_rng(99)
    hs = [rng.standard_normal(H).astype(np.float32) for _ in range(threads)]

    def work(t):
        h = hs[t]
        for _ in range(tokens):
            out = checker.moe_step(h, **kw)
            h = out[0] if isinstance(out, tuple) else out
        return h

    t0 = time.perf_counter()
    if threads == 1:
        work(0)
    else:
        with ThreadPoolExecutor(threads) as ex:  # ctypes drops the GIL during the C call
            list(ex.map(work, range(threads)))
    return time.perf_counter() - t0, tokens * threads


def cpu_checker():
    """(checker, kind): the reference's own C when built, else the oracle port."""
    from oracle.oracle import REF_SO, Oracle, Reference

    if REF_SO.exists():
        return Reference(), "reference"
    return Oracle(), "port"


def cpu_baseline_single(layer) -> dict:
    chk, kind = cpu_checker()
    secs, n = time_cpu_moe(chk, layer, tokens=8, threads=1)
    gbs = layer_bytes() * n / secs / 1e9
    return {"value": round(gbs, 4), "unit": "GB/s", "cores": 1, "kind": kind,
            "sample": f"{n} Mixtral-shaped token-layers (moe_step, 1 thread), {secs:.1f} s"}


# ------------------------------------------------------------ GEMV ---------
GEMV_ROWS = GEMV_COLS = 4096  # the single int4 grouped GEMV (quant.c:152-188)
HOST_AHEAD_CYCLES = 20_000_000  # ~10 ms of device sleep before a timed launch chain


def gemv_item(capi, synth, stream, peak: float, copies: int = 16, iters: int = 200) -> dict:
    """The batch-1 group-32 int4 GEMV W[4096, 4096] x fp32 x, resident matrices
    in the tiled layout, `copies` distinct ones in rotation (168 MB > L2),
    back to back on `stream`, timed with CUDA events."""
    import torch

    rng = np.random.default_rng(0)
    mats = [capi.Matrix(synth.int4_blob(rng, GEMV_ROWS, GEMV_COLS), GEMV_ROWS, GEMV_COLS)
            for _ in range(copies)]
    x = torch.from_numpy(rng.standard_normal(GEMV_COLS).astype(np.float32)).cuda()
    y = torch.empty(GEMV_ROWS, device="cuda")
    s = stream.cuda_stream
    for m in mats:
        m.gemv_dev(x.data_ptr(), y.data_ptr(), s)
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # One dependent GEMV lasts about as long as the host's own cost of one
    # call through ctypes, so a slow or busy host would set the pace. A
    # device-side sleep queued first lets the host enqueue every launch
    # before the first timed one starts: the events then time the device
    # chain alone (ev0 is recorded after the sleep).
    with torch.cuda.stream(stream):
        torch.cuda._sleep(HOST_AHEAD_CYCLES)
    ev0.record(stream)
    for i in range(iters):
        mats[i % copies].gemv_dev(x.data_ptr(), y.data_ptr(), s)
    ev1.record(stream)
    torch.cuda.synchronize()
    sec = ev0.elapsed_time(ev1) / 1e3 / iters
    nbytes = synth.int4_nbytes(GEMV_ROWS * GEMV_COLS) + 4 * (GEMV_ROWS + GEMV_COLS)
    gbs = nbytes / sec / 1e9
    # the same matrices as one launch of `copies` independent GEMVs sharing x
    # (rabbit_cuda_matrix_gemv_batch_dev); each launch streams all of them
    ys = [torch.empty(GEMV_ROWS, device="cuda") for _ in range(copies)]
    xp, yp = [x.data_ptr()] * copies, [t.data_ptr() for t in ys]
    for _ in range(3):
        capi.gemv_batch_dev(mats, xp, yp, s)
    torch.cuda.synchronize()
    biters = max(1, iters // copies)
    with torch.cuda.stream(stream):
        torch.cuda._sleep(HOST_AHEAD_CYCLES)
    ev0.record(stream)
    for _ in range(biters):
        capi.gemv_batch_dev(mats, xp, yp, s)
    ev1.record(stream)
    torch.cuda.synchronize()
    bsec = ev0.elapsed_time(ev1) / 1e3 / (biters * copies)
    bgbs = nbytes / bsec / 1e9
    for m in mats:
        m.free()
    return {"metric": "int4 expert GEMV GB/s (4096x4096, batch 1)", "value": round(gbs, 1),
            "unit": "GB/s", "us_per_gemv": round(sec * 1e6, 3), "bytes_per_gemv": nbytes,
            "frac_of_hbm_peak": round(gbs / peak, 4), "launches": iters,
            "l2": f"{copies} distinct matrices in rotation ({copies * nbytes / 1e6:.0f} MB)",
            "kernel": "k_gemv_g32", "mode": "one GEMV per launch, each after the previous "
                                            "(all launches enqueued before the first runs)",
            "batched": {"value": round(bgbs, 1), "unit": "GB/s",
                        "us_per_gemv": round(bsec * 1e6, 3),
                        "frac_of_hbm_peak": round(bgbs / peak, 4),
                        "mode": f"{copies} independent GEMVs (shared x) per launch, "
                                "rabbit_cuda_matrix_gemv_batch_dev", "launches": biters}}


# ------------------------------------------------------------ full decode --
# The OLMoE-shaped full decode (ref-v2 model, random init): 16 layers, hidden
# 2048, 16 heads x 128 (no GQA), RoPE, 64 experts top-8 with SwiGLU FFN 1024
# int4 group-32, fp32 dense weights N(0, 0.02)-scaled, KV window 256, vocab
# 50304; a random 16-id prompt, then 128 greedy tokens.
OL = dict(L=16, H=2048, nh=16, nkv=16, hd=128, E=64, k=8, I=1024, V=50304, ctx=256)
OL_PROMPT, OL_NEW = 16, 128


def olmoe_dense_bytes(kv_len: int, layers: int | None = None) -> int:
    """Algorithmic bytes of one token's dense part at KV length kv_len (after
    the append): per layer rms_attn + W_q/W_k/W_v/W_o + the K/V rows read and
    the row written; the embedding row, final norm and lm_head once."""
    L, H, V = layers or OL["L"], OL["H"], OL["V"]
    qd, kvd = OL["nh"] * OL["hd"], OL["nkv"] * OL["hd"]
    per_layer = H + qd * H + 2 * kvd * H + H * qd + 2 * kvd * (kv_len + 1)
    return 4 * (L * per_layer + 2 * H + H * V)


def olmoe_cpu_sample(seconds: float = 6.0) -> dict:
    """The reference's own C (or the oracle port) on one host thread: one
    layer's attention_step + moe_step at KV length ~ the run's middle, repeated
    for about `seconds`, and one lm_head pass; a token = 16 layers + lm_head."""
    from rabbit_b200 import synth

    chk, kind = cpu_checker()
    L, H, V, E, k, I = OL["L"], OL["H"], OL["V"], OL["E"], OL["k"], OL["I"]
    nh, nkv, hd = OL["nh"], OL["nkv"], OL["hd"]
    rng = np.random.default_rng(SEED + 11)
    f = lambda *sh: (rng.standard_normal(sh, dtype=np.float32) * 0.02)  # noqa: E731
    w = dict(rms_attn=np.ones(H, np.float32), w_q=f(nh * hd, H), w_k=f(nkv * hd, H),
             w_v=f(nkv * hd, H), w_o=f(H, nh * hd))
    recs, size, router, rms = synth.moe_layer(SEED + 12, H, E, I)
    kv_len = OL_PROMPT + OL_NEW // 2
    kc = np.zeros((OL["ctx"], nkv * hd), np.float32)
    vc = np.zeros_like(kc)
    kc[:kv_len] = rng.standard_normal((kv_len, nkv * hd), dtype=np.float32)
    vc[:kv_len] = rng.standard_normal((kv_len, nkv * hd), dtype=np.float32)
    h = rng.standard_normal(H, dtype=np.float32)
    n, t_layer = 0, 0.0
    while t_layer < seconds or n < 2:
        t0 = time.perf_counter()
        h, _ = chk.attention_step(h, kc, vc, kv_len, kv_len, n_heads=nh, n_kv_heads=nkv,
                                  head_dim=hd, **w)
        out = chk.moe_step(h, H=H, E=E, top_k=k, inter=I, n_shared=0, quant=4, n_records=E,
                           expert_size=size, records=recs, rms_ffn=rms, w_router=router)
        h = out[0] if isinstance(out, tuple) else out
        t_layer += time.perf_counter() - t0
        n += 1
    lm = f(H, V)
    t0 = time.perf_counter()
    chk.logits(lm, chk.rmsnorm(h, np.ones(H, np.float32)))
    t_lm = time.perf_counter() - t0
    per_token = L * t_layer / n + t_lm
    steps = sum(OL_PROMPT + t for t in range(OL_NEW))  # forward passes of its greedy loop
    return {"value": round(1.0 / per_token, 4), "unit": "tokens/s", "cores": 1, "kind": kind,
            "sample": f"{n} layer steps (attention_step + moe_step, KV length {kv_len}) + 1 "
                      f"lm_head pass on one thread, {t_layer + t_lm:.1f} s; a token = "
                      f"{L} layers + lm_head",
            "greedy_tokens_per_s": round(OL_NEW / (per_token * steps), 6),
            "greedy_note": ("rabbit_ref_v2_greedy re-runs the whole prefix for every new token "
                            f"({steps} token passes for {OL_NEW} tokens after a {OL_PROMPT}-id "
                            "prompt)")}


def full_decode_item(capi, synth, peak: float, runs: int = 3, cpu: bool = True,
                     layers: int | None = None, n_new: int = OL_NEW,
                     n_prompt: int = OL_PROMPT) -> dict:
    """Device-resident full decode through rabbit_cuda_refv2: prefill a random
    prompt, then generate 128 tokens chained on the device; device time from
    CUDA events around the generate call's kernels, e2e from the host call.
    layers / n_new / n_prompt below the workload's: profiling cases."""
    L, H, V, E, k, I = layers or OL["L"], OL["H"], OL["V"], OL["E"], OL["k"], OL["I"]
    rng = np.random.default_rng(SEED + 5)
    routers = [rng.normal(0, 0.02, (E, H)).astype(np.float32) for _ in range(L)]
    pool = capi.MoePool(records=None, expert_size=synth.expert_record_size(H, I), n_layers=L,
                        hidden=H, n_experts=E, top_k=k, inter=I, quant=4,
                        rms_ffn=[np.ones(H, np.float32)] * L, w_router=routers)
    pool.fill_synthetic(SEED * 1000 + 77)
    ctx = capi.RefV2(pool, vocab=V, n_heads=OL["nh"], n_kv_heads=OL["nkv"],
                     head_dim=OL["hd"], max_ctx=OL["ctx"])
    ctx.fill_synthetic(SEED * 1000 + 78, 0.02)
    prompt = rng.integers(0, V, n_prompt)
    dev, wall = [], []
    for r in range(runs + 1):  # the first run warms up
        ctx.reset()
        ctx.prefill(prompt, want_logits=False, want_hidden=False)
        t0 = time.perf_counter()
        out = ctx.generate(n_new)
        t = time.perf_counter() - t0
        if r:
            dev.append(ctx.device_ms / 1e3)
            wall.append(t)
    assert ((out >= 0) & (out < V)).all()
    moe_bytes = pool.decode_bytes * L
    gen_bytes = (sum(olmoe_dense_bytes(n_prompt + i, L) for i in range(n_new))
                 + n_new * moe_bytes)
    dsec, wsec = statistics.median(dev), statistics.median(wall)
    achieved = gen_bytes / dsec / 1e9
    item = {
        "metric": "full decode tokens/s (OLMoE-shaped, batch 1)",
        "value": round(n_new / dsec, 2), "unit": "tokens/s",
        "ms_per_token": round(1e3 * dsec / n_new, 4),
        "config": {"workload": (f"OLMoE-shaped ref-v2 decode: {L} layers, hidden {H}, "
                                f"{OL['nh']}x{OL['hd']} heads, {E} experts top-{k}, inter {I}, "
                                f"vocab {V}, KV window {OL['ctx']}; {n_prompt}-id random "
                                f"prompt, {n_new} greedy tokens"),
                   "l2": "inputs larger than L2 (1.5 GB fp32 dense + 0.46 GB experts per token)",
                   "runs": runs},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                     "unit": "GB/s", "frac": round(achieved / peak, 4),
                     "bytes_per_token": round(gen_bytes / n_new),
                     "moe_bytes_per_token": moe_bytes,
                     "what": "every weight byte a token needs read once, over the whole chain"},
        "e2e": {"value": round(n_new / wsec, 2), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 4 * n_new,
                "api": "rabbit_cuda_refv2_generate (host output ids)"},
        "gpu_launches_per_token": 4 * L + 2,
    }
    ctx.free()
    pool.free()
    if cpu:
        item["cpu_baseline"] = olmoe_cpu_sample()
    return item


# ------------------------------------------------------------ prefill chunk --
# The DeepSeek-MoE-16B-shaped prefill chunk (MoE blocks): 28 layers, hidden
# 2048, 64 routed experts top-6 + 2 shared, expert FFN 1408 SwiGLU int4
# group-32, a 32-token chunk of random hidden states, layer to layer.
def dense_share(L: int, H: int, q_dim: int, kv_dim: int, V: int, T: int, moe_ms: float,
                runs: int = 3) -> dict:
    """The dense part of a full step beside an MoE-block line: every layer's
    Q, K, V and O projections for T tokens plus the lm_head, fp32 (TF32 off),
    as torch matmuls (cuBLAS) over seeded weights resident in HBM. Context for
    the MoE line, not this library's work: the attention core over the KV
    window, the norms and the embedding are left out."""
    import torch

    tf32 = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        g = torch.Generator(device="cuda").manual_seed(SEED)
        mats = []
        for _ in range(L):
            mats.append([torch.randn(o, i, device="cuda", generator=g) * 0.02
                         for o, i in ((q_dim, H), (kv_dim, H), (kv_dim, H), (H, q_dim))])
        lm = torch.randn(V, H, device="cuda", generator=g) * 0.02
        x = torch.randn(T, H, device="cuda", generator=g)

        def step():
            h = x
            for wq, wk, wv, wo in mats:
                q = h @ wq.t()
                h.matmul(wk.t())
                h.matmul(wv.t())
                h = h + q @ wo.t()
            return h @ lm.t()

        for _ in range(2):
            step()
        torch.cuda.synchronize()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record()
        for _ in range(runs):
            step()
        ev1.record()
        torch.cuda.synchronize()
        ms = ev0.elapsed_time(ev1) / runs
        nbytes = 4 * (L * (q_dim * H * 2 + kv_dim * H * 2) + V * H)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = tf32
        del mats
        torch.cuda.empty_cache()
    return {"what": (f"Q/K/V/O projections of every layer and the lm_head for {T} tokens, "
                     f"fp32, torch matmul (cuBLAS) on seeded resident weights; attention core, "
                     f"norms and embedding not included"),
            "dense_bytes": nbytes, "dense_ms": round(ms, 3), "moe_ms": round(moe_ms, 3),
            "dense_share": round(ms / (ms + moe_ms), 3),
            "full_step_tokens_per_s": round(T / ((ms + moe_ms) / 1e3), 1)}


DS = dict(L=28, H=2048, E=64, k=6, S=2, I=1408)
DS_T = 32


def prefill_item(capi, synth, peak: float, runs: int = 5, cpu: bool = True,
                 layers: int | None = None) -> dict:
    """rabbit_cuda_moe_prefill_dev over the 28 layers' MoE blocks for one
    32-token chunk; bytes = the router plus every distinct expert the chunk
    touches in each layer (counted from this chunk's routing)."""
    import torch

    L, H, E, k, S, I = layers or DS["L"], DS["H"], DS["E"], DS["k"], DS["S"], DS["I"]
    rng = np.random.default_rng(SEED + 4)
    routers = [rng.normal(0, 0.02, (E, H)).astype(np.float32) for _ in range(L)]
    size = synth.expert_record_size(H, I)
    pool = capi.MoePool(records=None, expert_size=size, n_layers=L, hidden=H, n_experts=E,
                        top_k=k, inter=I, n_shared=S, quant=4,
                        rms_ffn=[np.ones(H, np.float32)] * L, w_router=routers)
    pool.fill_synthetic(SEED * 1000 + 4)
    stream = torch.cuda.current_stream()
    s = stream.cuda_stream
    # each layer gets its own seeded N(0, 1) chunk (chained layers of random
    # weights crowd the tokens onto a few experts)
    hin = torch.from_numpy(rng.standard_normal((L, DS_T, H)).astype(np.float32)).cuda()
    hout = torch.empty_like(hin)
    ids = torch.zeros((L, DS_T, k), dtype=torch.int32, device="cuda")
    wts = torch.zeros((L, DS_T, k), dtype=torch.float32, device="cuda")

    def chunk(with_ids: bool):
        for layer in range(L):
            pool.prefill_dev(layer, hin[layer].data_ptr(), hout[layer].data_ptr(), DS_T,
                             ids[layer].data_ptr() if with_ids else 0,
                             wts[layer].data_ptr() if with_ids else 0, s)

    chunk(True)
    pool.check(s)
    routed = ids.cpu().numpy()
    distinct = [len(np.unique(routed[l])) for l in range(L)]
    expert_bytes = 2 * synth.int4_nbytes(H * I) + synth.int4_nbytes(H * I)
    chunk_bytes = sum(E * H * 4 + (d + S) * expert_bytes for d in distinct)
    for _ in range(2):
        chunk(False)
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(runs):
        chunk(False)
    ev1.record(stream)
    torch.cuda.synchronize()
    pool.check(s)
    sec = ev0.elapsed_time(ev1) / 1e3 / runs
    achieved = chunk_bytes / sec / 1e9
    # end to end through the host-buffer entry point (H2D of the chunk, D2H of
    # the layer outputs and routing, every layer)
    hh = rng.standard_normal((DS_T, H)).astype(np.float32)
    pool.prefill(0, hh)
    t0 = time.perf_counter()
    x = hh
    for layer in range(L):
        x = pool.prefill(layer, x)[0]
    e2e = time.perf_counter() - t0
    item = {
        "metric": "MoE prefill chunk tokens/s (DeepSeek-MoE-16B-shaped, 32 tokens)",
        "value": round(DS_T / sec, 1), "unit": "tokens/s",
        "ms_per_chunk": round(sec * 1e3, 4),
        "config": {"workload": (f"DeepSeek-MoE-16B-shaped MoE blocks: {L} layers, hidden {H}, "
                                f"{E} routed experts top-{k} + {S} shared, inter {I}, "
                                f"{DS_T}-token chunk; each layer's chunk seeded N(0, 1)"),
                   "distinct_experts_per_layer": round(float(np.mean(distinct)), 2),
                   "l2": f"inputs larger than L2 ({pool.stats()['pool_bytes'] / 1e9:.1f} GB of experts)",
                   "note": "MoE blocks only (the routed-expert hot path); the chunk's attention "
                           "is not in this line"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "bytes_per_chunk": chunk_bytes},
        "e2e": {"value": round(DS_T / e2e, 1), "unit": "tokens/s",
                "h2d_bytes_per_step": L * DS_T * H * 4,
                "d2h_bytes_per_step": L * DS_T * (H * 4 + 2 * k * 4),
                "api": "rabbit_cuda_moe_prefill (host buffers)"},
        "gpu_launches_per_chunk": 7 * L,
    }
    pool.free()
    # the chunk's dense projections beside it (DeepSeek-MoE-16B: 16 heads x 128,
    # vocab 102400)
    item["dense"] = dense_share(L, H, 2048, 2048, 102400, DS_T, sec * 1e3)
    if cpu:
        chk, kind = cpu_checker()
        recs, size2, router, rms = synth.moe_layer(SEED + 14, H, E, I, S)
        kw = dict(H=H, E=E, top_k=k, inter=I, n_shared=S, quant=4, n_records=E + S,
                  expert_size=size2, records=recs, rms_ffn=rms, w_router=router)
        n, t_cpu = 0, 0.0
        hs = rng.standard_normal((8, H)).astype(np.float32)
        while t_cpu < 4.0 or n < 2:
            t0 = time.perf_counter()
            chk.moe_step(hs[n % 8], **kw)
            t_cpu += time.perf_counter() - t0
            n += 1
        per_token_layer = t_cpu / n
        item["cpu_baseline"] = {
            "value": round(1.0 / (per_token_layer * L), 4), "unit": "tokens/s", "cores": 1,
            "kind": kind,
            "sample": f"{n} DeepSeek-shaped token-layers (moe_step, 1 thread), {t_cpu:.1f} s; "
                      f"a token = {L} layers"}
    return item


# ------------------------------------------------------------ EP decode ------
# Mixtral-8x22B-shaped decode, expert-parallel: 56 layers, hidden 6144, expert
# FFN 16384, 8 experts top-2, int4 group-32 (84.5 GB of experts); a batch of
# 64 decode tokens per step. Rank r of N holds experts e = r (mod N) of every
# layer. The exchange is the library's own (rabbit_cuda_ep_* over NCCL,
# rabbit_cuda_moe_set_ep), inside each rabbit_cuda_moe_prefill_dev call:
#   all-to-all  each rank owns 64 / N of the tokens, routes them, sends the
#               pairs routed to other ranks' experts there (grouped
#               ncclSend / ncclRecv) and combines the rows that come back;
#   all-reduce  every rank routes all 64 tokens, applies its experts, and the
#               shares are summed (ncclAllReduce).
XL = dict(L=56, H=6144, E=8, k=2, I=16384)
XL_T = 64


def ep_item(capi, synth, peak: float, rank: int, world: int, dist, steps: int = 3,
            layers: int | None = None) -> dict:
    import torch

    L, H, E, k, I = layers or XL["L"], XL["H"], XL["E"], XL["k"], XL["I"]
    if E % world or XL_T % world:
        return {"unavailable": f"{E} experts / {XL_T} tokens do not split over {world} ranks"}
    rng = np.random.default_rng(SEED + 5)  # the same routers and tokens on every rank
    routers = [rng.normal(0, 0.02, (E, H)).astype(np.float32) for _ in range(L)]
    size = synth.expert_record_size(H, I)
    dev = torch.cuda.current_device()
    pool = capi.MoePool(records=None, expert_size=size, n_layers=L, hidden=H, n_experts=E,
                        top_k=k, inter=I, quant=4, rms_ffn=[np.ones(H, np.float32)] * L,
                        w_router=routers, experts_per_layer=E // world, device=dev)
    pool.fill_synthetic(SEED * 1000 + 5 + rank)
    ep = None
    if world > 1:
        box = [capi.ep_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(box, src=0)
        ep = capi.Ep(box[0], rank, world, dev)
    stream = torch.cuda.current_stream()
    s = stream.cuda_stream
    # each layer gets its own seeded N(0, 1) batch: chained layers of random
    # weights pull every token onto the same two experts, which real traffic
    # does not do
    hin = torch.from_numpy(rng.standard_normal((L, XL_T, H)).astype(np.float32)).cuda()
    expert_bytes = 3 * synth.int4_nbytes(H * I)

    def measure(mode: int) -> dict:
        a2a = mode == capi.EP_ALLTOALL
        Tm = XL_T // world if a2a else XL_T
        src = hin[:, rank * Tm:(rank + 1) * Tm].contiguous() if a2a else hin
        h = torch.empty((L, Tm, H), dtype=torch.float32, device="cuda")
        ids = torch.zeros((L, Tm, k), dtype=torch.int32, device="cuda")
        wts = torch.zeros((L, Tm, k), dtype=torch.float32, device="cuda")
        if ep:
            pool.set_ep(ep, mode)

        def step(with_ids: bool = False):
            for layer in range(L):
                pool.prefill_dev(layer, src[layer].data_ptr(), h[layer].data_ptr(), Tm,
                                 ids[layer].data_ptr() if with_ids else 0,
                                 wts[layer].data_ptr() if with_ids else 0, s)

        step(True)
        pool.check(s)
        if a2a and world > 1:  # every rank's routing, for the bytes the step reads
            parts = [torch.empty_like(ids) for _ in range(world)]
            dist.all_gather(parts, ids)
            routed = torch.cat(parts, dim=1).cpu().numpy()
        else:
            routed = ids.cpu().numpy()
        distinct = [len(np.unique(routed[l])) for l in range(L)]
        step_bytes = sum(E * H * 4 + d * expert_bytes for d in distinct)  # whole job
        for _ in range(2):
            step()
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record(stream)
        for _ in range(steps):
            step()
        ev1.record(stream)
        torch.cuda.synchronize()
        pool.check(s)
        ms = ev0.elapsed_time(ev1)
        if dist:
            t = torch.tensor([ms], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        sec = ms / 1e3 / steps
        out = {"tokens_per_s": round(XL_T / sec, 1), "ms_per_step": round(sec * 1e3, 3),
               "distinct_experts_per_layer": round(float(np.mean(distinct)), 2),
               "achieved_per_gpu": round(step_bytes / world / sec / 1e9, 1),
               "bytes_per_step_whole_job": step_bytes}
        if ep:  # one more step with per-call events: kernels vs exchange, per rank
            ep.set_timing(True)
            ep.stats(reset=True)
            step()
            st = ep.stats(reset=True)
            ep.set_timing(False)
            mine = [st["total_ms"] / max(1, st["calls"]), st["exchange_ms"] / max(1, st["calls"])]
            allr = [None] * world
            dist.all_gather_object(allr, mine)
            out["per_layer_ms_by_rank"] = [
                {"rank": r, "layer_ms": round(v[0], 4), "exchange_ms": round(v[1], 4),
                 "kernels_ms": round(v[0] - v[1], 4)} for r, v in enumerate(allr)]
        return out

    if world > 1:
        res = {"all_to_all": measure(capi.EP_ALLTOALL), "all_reduce": measure(capi.EP_ALLREDUCE)}
        # the line's value is the faster of the two exchanges the library offers
        best_mode = max(res, key=lambda m: res[m]["tokens_per_s"])
        best = res[best_mode]
        pool.set_ep(None)
    else:
        res = {"single_gpu": measure(0)}
        best_mode = "single_gpu"
        best = res["single_gpu"]
    pool.free()
    if ep:
        ep.free()
    sec = best["ms_per_step"] / 1e3
    # the step's dense projections, which every rank runs for its own 64 / N
    # tokens (attention data-parallel over the ranks, as in the all-to-all
    # mode; Mixtral-8x22B: 48 heads x 128, 8 KV heads, vocab 32768)
    dense = dense_share(L, H, 6144, 1024, 32768, XL_T // world if world > 1 else XL_T,
                        best["ms_per_step"])
    return {
        "metric": "EP MoE decode tokens/s (Mixtral-8x22B-shaped, batch 64)",
        "value": best["tokens_per_s"], "unit": "tokens/s", "n_gpus": world,
        "ms_per_step": best["ms_per_step"], "steps": steps,
        "config": {"workload": (f"Mixtral-8x22B-shaped MoE blocks: {L} layers, hidden {H}, "
                                f"inter {I}, {E} experts top-{k}, batch {XL_T} decode tokens, "
                                f"expert-parallel over {world} GPU(s); the exchange is the "
                                f"library's own (NCCL all-to-all dispatch / combine, or an "
                                f"all-reduce of the shares) inside rabbit_cuda_moe_prefill_dev, "
                                f"both measured, the value the faster; each layer's batch "
                                f"seeded N(0, 1)"),
                   "value_mode": best_mode,
                   "experts_per_gpu_per_layer": E // world,
                   "expert_bytes_per_gpu_gb": round(L * (E // world) * size / 1e9, 1),
                   "note": "MoE blocks only (the routed-expert hot path); the attention and "
                           "dense fp32 projections of the step are not in this line"},
        "modes": res,
        "dense": dense,
        # this library's kernels per step (NCCL's own not counted): route,
        # bucket, two B-row images, two GEMMs, combine per layer, plus the
        # all-to-all pack and return
        "gpu_launches_per_step": {"single_gpu": 7 * L} if world == 1 else
                                 {"all_to_all": 9 * L, "all_reduce": 7 * L},
        "roofline": {"bound": "hbm", "achieved_per_gpu": best["achieved_per_gpu"],
                     "peak": peak, "unit": "GB/s",
                     "frac": round(best["achieved_per_gpu"] / peak, 4),
                     "bytes_per_step_whole_job": best["bytes_per_step_whole_job"]},
        "scaling": "strong",
    }


# ------------------------------------------------------------ arms ---------
def run_reference(args) -> None:
    """--impl reference: the reference's C on all host cores."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    chk, kind = cpu_checker()
    threads = os.cpu_count() or 1
    layer = host_layer()
    # one step = each thread runs one full moe_step token-layer (~1 s on one core)
    for _ in range(args.warmup):
        time_cpu_moe(chk, layer, 1, threads)
    steps = args.steps
    budget_steps = max(1, int(150 / 1.5))  # keep the whole run within a few minutes
    timed = min(steps, budget_steps)
    secs, n = time_cpu_moe(chk, layer, timed, threads)
    gbs = layer_bytes() * n / secs / 1e9
    ms = secs * 1000 / timed
    line = {
        "impl": "reference", "metric": METRIC, "value": round(gbs, 4), "unit": "GB/s",
        "n_gpus": args.gpus, "steps": timed, "warmup": args.warmup,
        "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "u4 weights, f32 math", "data": "synthetic",
        "config": {"workload": "Mixtral-shaped MoE layer decode (reference C moe_step)",
                   "hidden": H, "inter": I, "experts": E, "top_k": TOPK,
                   "threads": threads},
        "cpu_baseline": {"value": round(gbs, 4), "unit": "GB/s", "cores": threads, "kind": kind,
                         "sample": f"{n} token-layers ({threads} threads x {timed} steps)"},
        "e2e": {"value": round(gbs, 4), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "tokens_per_s": round(n / secs / LAYERS, 6),
    }
    if timed != steps:
        line["note"] = f"{timed} of {steps} requested steps timed to bound the CPU run"
    print(json.dumps(line), flush=True)


def run_rabbit(args) -> None:
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE {world}")
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    from rabbit_b200 import capi, synth

    if args.ep_only:  # the expert-parallel decode item alone
        item = ep_item(capi, synth, measured_peak()[0], rank, world, dist, layers=args.ep_layers)
        if rank == 0:
            print(json.dumps({"ep_decode": item}), flush=True)
        if dist:
            dist.destroy_process_group()
        return
    if args.prefill_only:  # the DeepSeek-shaped prefill chunk item alone (profiling)
        if rank == 0:
            item = prefill_item(capi, synth, measured_peak()[0], cpu=not args.no_cpu_baseline,
                                layers=args.prefill_layers)
            print(json.dumps({"prefill": item}), flush=True)
        if dist:
            dist.destroy_process_group()
        return
    if args.full_decode_only:  # the OLMoE-shaped full decode item alone (profiling)
        if rank == 0:
            item = full_decode_item(capi, synth, measured_peak()[0], cpu=not args.no_cpu_baseline,
                                    layers=args.fd_layers, n_new=args.fd_new,
                                    n_prompt=args.fd_prompt)
            print(json.dumps({"full_decode": item}), flush=True)
        if dist:
            dist.destroy_process_group()
        return
    L = args.layers

    capi.check(capi.lib().rabbit_cuda_set_device(local))
    rng = np.random.default_rng(SEED + rank)
    routers = [rng.normal(0, 0.02, (E, H)).astype(np.float32) for _ in range(L)]
    norms = [np.ones(H, np.float32) for _ in range(L)]
    size = synth.expert_record_size(H, I)
    pool = capi.MoePool(records=None, expert_size=size, n_layers=L, hidden=H, n_experts=E,
                        top_k=TOPK, inter=I, quant=4, rms_ffn=norms, w_router=routers,
                        device=local)
    pool.fill_synthetic(SEED * 1000 + rank)
    per_layer = pool.decode_bytes
    step_bytes = per_layer * L

    stream = torch.cuda.current_stream()
    s = stream.cuda_stream
    h0 = torch.from_numpy(rng.standard_normal(H).astype(np.float32)).cuda()
    bufs = [h0.clone(), torch.empty_like(h0)]
    ids = torch.zeros(8, dtype=torch.int32, device="cuda")
    wts = torch.zeros(8, dtype=torch.float32, device="cuda")

    def step():
        for layer in range(L):
            a, b = bufs[layer & 1], bufs[(layer + 1) & 1]
            pool.decode_dev(layer, a.data_ptr(), b.data_ptr(), ids.data_ptr(), wts.data_ptr(), s)

    for _ in range(args.warmup):
        step()
    pool.check(s)
    torch.cuda.synchronize()

    props = torch.cuda.get_device_properties(local)
    clocks = ClockSampler("GPU-" + str(props.uuid))
    clocks.start()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(args.steps):
        step()
    ev1.record(stream)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    clk = clocks.stop()
    pool.check(s)
    ms = ev0.elapsed_time(ev1)
    if dist:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    secs = ms / 1000.0
    value = world * step_bytes * args.steps / secs / 1e9
    launches = args.steps * L
    kernel_s = secs / launches
    achieved = per_layer / kernel_s / 1e9
    peak, peak_kind = measured_peak()

    # end to end through the host-buffer C ABI, h updated in place in a host
    # array as an engine's token loop does (per layer: h from host memory into
    # HBM, h_out and the routing back into host memory, one synchronisation)
    h_host = rng.standard_normal(H).astype(np.float32)
    e2e_steps = max(1, min(args.steps, 50))
    for _ in range(2):
        for layer in range(L):
            pool.decode_into(layer, h_host, h_host)
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        for layer in range(L):
            pool.decode_into(layer, h_host, h_host)
    e2e_s = time.perf_counter() - t0
    if dist:
        t = torch.tensor([e2e_s], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    e2e_value = world * step_bytes * e2e_steps / e2e_s / 1e9

    pool_stats = pool.stats()
    pool.free()  # the items below need the room (the EP item holds 84.5 GB at N = 1)
    ep = None
    if not args.no_ep:
        ep = ep_item(capi, synth, measured_peak()[0], rank, world, dist, layers=args.ep_layers)
    gemv = None if args.no_gemv else gemv_item(capi, synth, stream, measured_peak()[0])
    prefill = None
    if world == 1 and not args.no_prefill:
        prefill = prefill_item(capi, synth, measured_peak()[0], cpu=not args.no_cpu_baseline)
    full = None
    if world == 1 and not args.no_full_decode:
        full = full_decode_item(capi, synth, measured_peak()[0], cpu=not args.no_cpu_baseline)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline_single(host_layer())

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "u4 weights, f32 math", "data": "synthetic",
            "config": {"workload": WORKLOAD.format(L), "hidden": H, "inter": I, "experts": E,
                       "top_k": TOPK, "layers_per_step": L, "batch": 1,
                       "expert_bytes_resident_gb": round(pool_stats["pool_bytes"] / 1e9, 2),
                       "l2": (f"inputs larger than L2 ({L} distinct layers, "
                              f"{pool_stats['pool_bytes'] / 1e9:.1f} GB of experts)"),
                       "parallelism": f"dp{world} decode replicas" if world > 1 else "single"},
            "tokens_per_s": round(world * args.steps / secs, 2),
            "us_per_token_layer": round(1e6 * secs / launches, 3),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                         "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "traffic": profile_traffic(), "peak_kind": peak_kind,
                         "kernel": "k_moe_decode_g32",
                         "bytes_per_launch": per_layer},
            "e2e": {"value": round(e2e_value, 2), "unit": "GB/s",
                    "h2d_bytes_per_step": L * H * 4,
                    # one copy per layer: h_out, ids[8], weights[8], error word
                    "d2h_bytes_per_step": L * (H * 4 + 80),
                    "steps": e2e_steps, "api": "rabbit_cuda_moe_decode (host buffers)"},
            "gpu_launches": launches,
            "gemv": gemv,
            "full_decode": full,
            "prefill": prefill,
            "ep_decode": ep,
            "clocks": clk,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    if dist:
        dist.destroy_process_group()


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["rabbit", "reference"], default="rabbit")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--layers", type=int, default=LAYERS,
                    help="distinct layers per step (small values: profiling cases)")
    ap.add_argument("--no-gemv", action="store_true", help="skip the GEMV line item")
    ap.add_argument("--no-full-decode", action="store_true",
                    help="skip the OLMoE-shaped full decode line item")
    ap.add_argument("--no-prefill", action="store_true",
                    help="skip the DeepSeek-shaped prefill chunk line item")
    ap.add_argument("--prefill-only", action="store_true",
                    help="run only the prefill chunk item (profiling cases)")
    ap.add_argument("--prefill-layers", type=int, default=None, help="prefill chunk: layers")
    ap.add_argument("--no-ep", action="store_true", help="skip the expert-parallel decode item")
    ap.add_argument("--ep-only", action="store_true",
                    help="run only the expert-parallel decode item (profiling cases)")
    ap.add_argument("--ep-layers", type=int, default=None, help="EP decode: layers")
    ap.add_argument("--full-decode-only", action="store_true",
                    help="run only the full decode item (profiling cases)")
    ap.add_argument("--fd-layers", type=int, default=None, help="full decode: layers")
    ap.add_argument("--fd-new", type=int, default=OL_NEW, help="full decode: generated tokens")
    ap.add_argument("--fd-prompt", type=int, default=OL_PROMPT, help="full decode: prompt ids")
    args = ap.parse_args(argv)
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_rabbit(args)
    return 0


if __name__ == "__main__":
    sys.exit(main())
