"""GPU: rabbit_cuda_moe_decode_dev_noalloc (scratch in the library's fixed
device array) against rabbit_cuda_moe_decode_dev (scratch owned by the pool)
on the same pool and tokens, through the C ABI.

Two no-alloc calls run back to back after the reference calls, so the second
one starts from whatever the first left in the shared array. Bar: layer
outputs, routing weights within rtol 1e-4 / atol 1e-5, expert ids identical.
This file is collected last on purpose: it must pass both in a fresh process
(the first call on the device sets the array up) and after the other tests.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import ATOL, RTOL
from rabbit_b200 import synth

pytestmark = pytest.mark.gpu

SHAPES = {
    # name: H, E, k, I, S
    "mixtral": (4096, 8, 2, 14336, 0),
    "olmoe": (2048, 64, 8, 1024, 0),
    "tiny_shared": (64, 4, 2, 128, 2),
}


def _pool(rc, H, E, k, I, S, seed, n_layers=2):
    recs, size, router, rms = synth.moe_layer(seed, H, E, I, S)
    # the same records for every layer, different routers per layer
    routers = [router, np.ascontiguousarray(router[::-1])][:n_layers]
    return rc.MoePool(records=np.concatenate([recs] * n_layers), expert_size=size,
                      n_layers=n_layers, hidden=H, n_experts=E, top_k=k, inter=I, n_shared=S,
                      quant=4, rms_ffn=[rms] * n_layers, w_router=routers)


@pytest.mark.parametrize("name", list(SHAPES))
def test_noalloc_matches_decode_dev(rc, name):
    import torch

    H, E, k, I, S = SHAPES[name]
    pool = _pool(rc, H, E, k, I, S, seed=sum(map(ord, name)) + 7)
    dev = torch.device("cuda:0")
    stream = torch.cuda.current_stream().cuda_stream
    rng = np.random.default_rng(3)
    tokens = [torch.from_numpy(rng.standard_normal(H).astype(np.float32)).to(dev)
              for _ in range(2)]
    layers = [0, 1]

    want = []
    for layer, h in zip(layers, tokens):
        out = torch.empty_like(h)
        ids = torch.full((k,), -7, dtype=torch.int32, device=dev)
        w = torch.zeros(k, dtype=torch.float32, device=dev)
        pool.decode_dev(layer, h.data_ptr(), out.data_ptr(), ids.data_ptr(), w.data_ptr(), stream)
        pool.check(stream)
        want.append((out.cpu().numpy(), ids.cpu().numpy(), w.cpu().numpy()))

    # two calls in a row; the second passes no id/weight buffers
    got = []
    outs = [torch.full_like(h, float("nan")) for h in tokens]
    ids0 = torch.full((k,), -7, dtype=torch.int32, device=dev)
    w0 = torch.zeros(k, dtype=torch.float32, device=dev)
    pool.decode_dev_noalloc(layers[0], tokens[0].data_ptr(), outs[0].data_ptr(), ids0.data_ptr(),
                            w0.data_ptr(), stream)
    pool.decode_dev_noalloc(layers[1], tokens[1].data_ptr(), outs[1].data_ptr(), 0, 0, stream)
    pool.check(stream)
    got.append((outs[0].cpu().numpy(), ids0.cpu().numpy(), w0.cpu().numpy()))
    got.append((outs[1].cpu().numpy(), None, None))

    for i, ((o_ref, i_ref, w_ref), (o, ids, w)) in enumerate(zip(want, got)):
        np.testing.assert_allclose(o, o_ref, rtol=RTOL, atol=ATOL, err_msg=f"call {i}: h_out")
        np.testing.assert_allclose(o - tokens[i].cpu().numpy(), o_ref - tokens[i].cpu().numpy(),
                                   rtol=RTOL, atol=ATOL, err_msg=f"call {i}: MoE delta")
        if ids is not None:
            np.testing.assert_array_equal(ids, i_ref, err_msg=f"call {i}: expert ids")
            np.testing.assert_allclose(w, w_ref, rtol=RTOL, atol=ATOL, err_msg=f"call {i}: weights")
    pool.free()


def test_noalloc_rejects_scratch_over_limit(rc):
    """The SwiGLU activations alone, (k + S) * I tagged values of 8 bytes each
    (24 * 16384 * 8 = 3 MiB), exceed the 2 MiB array: a clear error, nothing
    launched; the pool still decodes through decode_dev."""
    import torch

    H, E, k, I, S = 64, 8, 8, 16384, 16
    pool = _pool(rc, H, E, k, I, S, seed=11, n_layers=1)
    h = torch.randn(H, device="cuda:0")
    out = torch.empty_like(h)
    stream = torch.cuda.current_stream().cuda_stream
    with pytest.raises(rc.RabbitCudaError, match="limit"):
        pool.decode_dev_noalloc(0, h.data_ptr(), out.data_ptr(), 0, 0, stream)
    pool.decode_dev(0, h.data_ptr(), out.data_ptr(), 0, 0, stream)
    pool.check(stream)
    assert torch.isfinite(out).all()
    pool.free()


def test_noalloc_refuses_a_capturing_stream(rc):
    """Each call tags the values its CTAs share with a number picked when the
    call is issued; a graph replay would reuse it, so calls on a stream that
    is being captured are refused before anything is recorded, and the pool
    decodes normally afterwards."""
    import torch

    H, E, k, I, S = SHAPES["tiny_shared"]
    pool = _pool(rc, H, E, k, I, S, seed=5, n_layers=1)
    h = torch.randn(H, device="cuda:0")
    out = torch.empty_like(h)
    side = torch.cuda.Stream()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        with pytest.raises(rc.RabbitCudaError, match="captured"):
            pool.decode_dev_noalloc(0, h.data_ptr(), out.data_ptr(), 0, 0, side.cuda_stream)
        with pytest.raises(rc.RabbitCudaError, match="captured"):
            pool.decode_dev(0, h.data_ptr(), out.data_ptr(), 0, 0, side.cuda_stream)
    del graph
    stream = torch.cuda.current_stream().cuda_stream
    want = torch.empty_like(h)
    pool.decode_dev(0, h.data_ptr(), want.data_ptr(), 0, 0, stream)
    pool.decode_dev_noalloc(0, h.data_ptr(), out.data_ptr(), 0, 0, stream)
    pool.check(stream)
    np.testing.assert_allclose(out.cpu().numpy(), want.cpu().numpy(), rtol=RTOL, atol=ATOL)
    pool.free()
