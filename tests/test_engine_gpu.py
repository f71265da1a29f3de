"""GPU: the drop-in boundary exercised by the reference engine itself. The
engine is built twice from its own sources by oracle/engine/Makefile (where
the reference checkout is present; the binaries travel in oracle/_ref/engine):
`rabbit` as it is, `rabbit_cuda` with moe_step and rabbit_ref_v2_greedy
hooked into librabbit_cuda.so (oracle/engine/rabbit_cuda_engine.c).

`probe-v2` (src/main.c:119-175) prints the greedy ids of a prompt on a seeded
int4 ref-v2 model file. The bar: the same ids from
  * the unmodified engine (every block on the CPU),
  * rabbit_cuda (moe_step -> rabbit_cuda_moe_decode per layer and token),
  * rabbit_cuda with RABBIT_CUDA_CTX=1 (RabbitRefV2Ctx -> rabbit_cuda_refv2_*:
    one prefill and a greedy continuation on the device),
  * rabbit_cuda with RABBIT_CUDA_OFF=1 (the hooks step aside)."""
from __future__ import annotations

import os
import re
import subprocess
from pathlib import Path

import pytest

from rabbit_file import write_refv2_model

pytestmark = pytest.mark.gpu

ENGINE = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "engine"
PROMPT = "hello there"
N_NEW = 12
MODELS = {
    # GQA, a shared expert, two layers
    "gqa_shared": dict(L=2, H=256, V=512, n_heads=4, n_kv=2, head_dim=64, E=8, k=2, I=512, S=1),
    # OLMoE-like head_dim 128, eight experts of top-4
    "hd128": dict(L=2, H=512, V=1024, n_heads=4, n_kv=4, head_dim=128, E=8, k=4, I=256, S=0),
}


def _probe(binary: str, model: Path, env_extra: dict) -> list[int]:
    env = dict(os.environ)
    env.pop("RABBIT_CUDA_CTX", None)
    env.pop("RABBIT_CUDA_OFF", None)
    env.update(env_extra)
    r = subprocess.run([str(ENGINE / binary), "probe-v2", "--model", str(model), "--prompt",
                        PROMPT, "--tokens", str(N_NEW)], capture_output=True, text=True,
                       env=env, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    m = re.search(r"PROBE_V2 prompt=.* n=(\d+) ids=([\d,]+)", r.stdout)
    assert m, r.stdout[-2000:]
    ids = [int(x) for x in m.group(2).split(",")]
    assert len(ids) == int(m.group(1))
    return ids


@pytest.mark.parametrize("name", list(MODELS))
def test_probe_v2_greedy_ids_through_the_shim(tmp_path, name):
    for b in ("rabbit", "rabbit_cuda"):
        if not (ENGINE / b).exists():
            pytest.skip(f"{ENGINE / b} not built (make -C oracle/engine REF_SRC=...)")
    model = tmp_path / f"{name}.rabbit"
    write_refv2_model(model, seed=sum(map(ord, name)), **MODELS[name])
    ref = _probe("rabbit", model, {})
    assert len(ref) > N_NEW
    assert _probe("rabbit_cuda", model, {"RABBIT_CUDA_OFF": "1"}) == ref
    assert _probe("rabbit_cuda", model, {}) == ref, "moe_step through rabbit_cuda_moe_decode"
    assert _probe("rabbit_cuda", model, {"RABBIT_CUDA_CTX": "1"}) == ref, \
        "greedy through the RabbitRefV2Ctx shim"
