"""Seeded ref-v2 model files in the .rabbit format (src/rabbit.h:28-56,
src/model.c:236-348): a 264-byte header, the fp32 dense block in the order
parse_weights reads it (src/forward_v2.c:106-169), then the expert table
(per layer E routed + S shared group-32 int4 records, src/forward_v2.c:
280-332). Test helper; sizes stay small."""
from __future__ import annotations

import struct
from pathlib import Path

import numpy as np


def write_refv2_model(path: Path, seed: int, *, L: int, H: int, V: int, n_heads: int,
                      n_kv: int, head_dim: int, E: int, k: int, I: int, S: int = 0,
                      sigma: float = 0.05) -> dict:
    from rabbit_b200 import synth

    rng = np.random.default_rng(seed)
    q_dim, kv_dim = n_heads * head_dim, n_kv * head_dim
    parts = [rng.standard_normal((V, H)).astype(np.float32),          # embed
             (rng.standard_normal((H, V)) * sigma).astype(np.float32),  # lm_head
             np.ones(H, np.float32)]                                   # final_norm
    for _ in range(L):
        parts += [np.ones(H, np.float32), np.ones(H, np.float32),      # rms_attn, rms_ffn
                  (rng.standard_normal((q_dim, H)) * sigma).astype(np.float32),
                  (rng.standard_normal((kv_dim, H)) * sigma).astype(np.float32),
                  (rng.standard_normal((kv_dim, H)) * sigma).astype(np.float32),
                  (rng.standard_normal((H, q_dim)) * sigma).astype(np.float32),
                  (rng.standard_normal((E, H)) * 0.02).astype(np.float32)]  # router
    dense = np.concatenate([p.ravel() for p in parts]).tobytes()
    size = synth.expert_record_size(H, I)
    experts = np.concatenate([synth.expert_record(rng, H, I, size) for _ in range(L * (E + S))])
    reserved = struct.pack("<4I", n_heads, n_kv, head_dim, S) + bytes(112)
    hdr = (b"RABBIT01" + struct.pack("<II", 1, 264)
           + struct.pack("<6I", L, H, V, E, k, I)
           + struct.pack("<3Q", len(dense), size, experts.size)
           + struct.pack("<II", 0, 4)
           + b"refv2-test".ljust(64, b"\0") + reserved)
    assert len(hdr) == 264
    Path(path).write_bytes(hdr + dense + experts.tobytes())
    return dict(L=L, H=H, V=V, E=E, k=k, I=I, S=S, expert_size=size)
