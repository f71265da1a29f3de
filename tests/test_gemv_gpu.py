"""GPU parity: group-32 int4 dequant and GEMV against the oracle.

Bar: dequant bit-identical (integer nibble unpack, one fp32 multiply);
GEMV y within rtol 1e-4 / atol 1e-5 of the oracle's serial fp32 sum.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

import numpy as np
import pytest

from conftest import ATOL, RTOL
from rabbit_b200 import synth

pytestmark = pytest.mark.gpu
GOLD = Path(__file__).resolve().parent / "golden"


class Dev:
    """Minimal device buffers through the CUDA runtime torch already loads."""

    def __init__(self):
        import torch

        self.torch = torch
        assert torch.cuda.is_available(), "GPU test on a host without CUDA"

    def put(self, a: np.ndarray):
        t = self.torch.from_numpy(np.ascontiguousarray(a)).cuda()
        return t

    def empty(self, n, dtype):
        return self.torch.empty(n, dtype=dtype, device="cuda")

    @property
    def stream(self) -> int:
        """torch's current stream, so library kernels follow torch's copies."""
        return self.torch.cuda.current_stream().cuda_stream


@pytest.fixture(scope="module")
def dev():
    return Dev()


def test_dequant_bit_exact_golden(rc, dev):
    g = np.load(GOLD / "gemv.npz")
    for i in range(int(g["gemv_count"])):
        if f"gemv{i}_deq" not in g:
            continue
        r, c, _ = (int(v) for v in g[f"gemv{i}_shape"])
        blob = dev.put(g[f"gemv{i}_blob"])
        out = dev.empty(r * c, dev.torch.float32)
        rc.check(rc.lib().rabbit_cuda_dequant_int4_grouped_dev(blob.data_ptr(), out.data_ptr(),
                                                               r * c, dev.stream))
        dev.torch.cuda.synchronize()
        np.testing.assert_array_equal(out.cpu().numpy().view(np.uint32),
                                      g[f"gemv{i}_deq"].view(np.uint32))


@pytest.mark.parametrize("n", [1, 17, 4097, 1 << 20])
def test_dequant_bit_exact_unaligned(rc, dev, oracle, n):
    rng = np.random.default_rng(n)
    blob = synth.int4_blob(rng, 1, n)
    padded = np.concatenate([np.zeros(3, np.uint8), blob])  # device blob at offset 3
    d = dev.put(padded)
    out = dev.empty(n, dev.torch.float32)
    rc.check(rc.lib().rabbit_cuda_dequant_int4_grouped_dev(d.data_ptr() + 3, out.data_ptr(), n,
                                                           dev.stream))
    dev.torch.cuda.synchronize()
    np.testing.assert_array_equal(out.cpu().numpy().view(np.uint32),
                                  oracle.dequant_int4_grouped(blob, n).view(np.uint32))


def test_dequant_rejects_bad_group(rc, dev):
    blob = dev.put(np.zeros(64, np.uint8))
    out = dev.empty(16, dev.torch.float32)
    assert rc.lib().rabbit_cuda_dequant_int4_grouped_dev(blob.data_ptr(), out.data_ptr(), 16,
                                                         dev.stream) == rc.ERR_FORMAT


def test_gemv_golden_host_buffers(rc):
    g = np.load(GOLD / "gemv.npz")
    for i in range(int(g["gemv_count"])):
        r, c, gs = (int(v) for v in g[f"gemv{i}_shape"])
        y = rc.gemv_int4_grouped(g[f"gemv{i}_blob"], g[f"gemv{i}_x"], r, c)
        np.testing.assert_allclose(y, g[f"gemv{i}_y"], rtol=RTOL, atol=ATOL,
                                   err_msg=f"case {i} shape {r}x{c} gs {gs}")


SHAPES = [(1, 32), (3, 64), (4, 4096), (27, 4096), (4096, 4096), (14336, 4096), (4096, 14336),
          (1024, 2048), (2048, 1024), (1408, 2048), (2048, 1408), (6144, 16384), (5, 100),
          (7, 33)]


@pytest.mark.parametrize("shape", SHAPES, ids=[f"{r}x{c}" for r, c in SHAPES])
def test_matrix_gemv_vs_oracle(rc, oracle, shape):
    r, c = shape
    rng = np.random.default_rng(r * 7 + c)
    blob = synth.int4_blob(rng, r, c)
    m = rc.Matrix(blob, r, c)
    for trial in range(2):
        x = rng.standard_normal(c).astype(np.float32)
        y = m.gemv(x)
        ref = oracle.gemv_int4_grouped(blob, x, r, c)
        np.testing.assert_allclose(y, ref, rtol=RTOL, atol=ATOL)
    assert m.nbytes == synth.int4_nbytes(r * c) + 4 * (r + c)
    m.free()


def test_stateless_gemv_fast_and_flat_agree(rc, oracle):
    rng = np.random.default_rng(11)
    for r, c, gs in [(512, 4096, 32), (300, 96, 32), (64, 100, 32), (48, 256, 64)]:
        blob = synth.int4_blob(rng, r, c, gs)
        x = rng.standard_normal(c).astype(np.float32)
        np.testing.assert_allclose(rc.gemv_int4_grouped(blob, x, r, c),
                                   oracle.gemv_int4_grouped(blob, x, r, c), rtol=RTOL, atol=ATOL)


def test_gemv_dev_raw_blob_any_alignment(rc, dev, oracle):
    rng = np.random.default_rng(12)
    r, c = 37, 96
    blob = synth.int4_blob(rng, r, c)
    x = rng.standard_normal(c).astype(np.float32)
    d = dev.put(np.concatenate([np.zeros(1, np.uint8), blob]))
    dx = dev.put(x)
    dy = dev.empty(r, dev.torch.float32)
    rc.check(rc.lib().rabbit_cuda_gemv_int4_grouped_dev(d.data_ptr() + 1, dx.data_ptr(),
                                                        dy.data_ptr(), r, c, dev.stream))
    dev.torch.cuda.synchronize()
    np.testing.assert_allclose(dy.cpu().numpy(), oracle.gemv_int4_grouped(blob, x, r, c),
                               rtol=RTOL, atol=ATOL)


def test_matrix_gemv_dev_linearity_full_size(rc, dev):
    """4096x4096 on device buffers: W(a x + b z) = a Wx + b Wz (size-independent check)."""
    rng = np.random.default_rng(13)
    r = c = 4096
    m = rc.Matrix(synth.int4_blob(rng, r, c), r, c)
    x = rng.standard_normal(c).astype(np.float32)
    z = rng.standard_normal(c).astype(np.float32)
    outs = []
    for v in (x, z, 2.0 * x + 0.5 * z):
        dx = dev.put(v.astype(np.float32))
        dy = dev.empty(r, dev.torch.float32)
        m.gemv_dev(dx.data_ptr(), dy.data_ptr(), dev.stream)
        dev.torch.cuda.synchronize()
        outs.append(dy.cpu().numpy().astype(np.float64))
    np.testing.assert_allclose(outs[2], 2.0 * outs[0] + 0.5 * outs[1], rtol=1e-4, atol=1e-4)


def test_wait_limit_setting(rc):
    assert rc.lib().rabbit_cuda_set_wait_limit_ms(500) == rc.OK
    assert rc.lib().rabbit_cuda_set_wait_limit_ms(2000) == rc.OK


@pytest.mark.parametrize("shape,n,shared", [((300, 4096), 5, False), ((300, 4096), 5, True),
                                            ((64, 14336), 3, False), ((96, 160), 32, True)],
                         ids=["300x4096-n5", "300x4096-n5-shared-x", "64x14336-n3", "96x160-n32"])
def test_matrix_gemv_batch_vs_oracle(rc, dev, oracle, shape, n, shared):
    """n GEMVs in one launch (ragged row counts, long rows, the 32-matrix maximum,
    shared and distinct inputs) against the oracle, twice in a row."""
    r, c = shape
    rng = np.random.default_rng(r + c + n)
    blobs = [synth.int4_blob(rng, r, c) for _ in range(n)]
    mats = [rc.Matrix(b, r, c) for b in blobs]
    for _ in range(2):
        xs = [rng.standard_normal(c).astype(np.float32) for _ in range(1 if shared else n)]
        dxs = [dev.put(x) for x in xs]
        dys = [dev.empty(r, dev.torch.float32) for _ in range(n)]
        rc.gemv_batch_dev(mats, [dxs[0 if shared else i].data_ptr() for i in range(n)],
                          [d.data_ptr() for d in dys], dev.stream)
        dev.torch.cuda.synchronize()
        for i in range(n):
            ref = oracle.gemv_int4_grouped(blobs[i], xs[0 if shared else i], r, c)
            np.testing.assert_allclose(dys[i].cpu().numpy(), ref, rtol=RTOL, atol=ATOL,
                                       err_msg=f"matrix {i}")
    for m in mats:
        m.free()


def test_matrix_gemv_batch_rejects_bad_batches(rc, dev):
    rng = np.random.default_rng(5)
    a = rc.Matrix(synth.int4_blob(rng, 64, 256), 64, 256)
    b = rc.Matrix(synth.int4_blob(rng, 32, 256), 32, 256)
    dx = dev.put(rng.standard_normal(256).astype(np.float32))
    dy = dev.empty(64, dev.torch.float32)
    with pytest.raises(rc.RabbitCudaError, match="differs"):
        rc.gemv_batch_dev([a, b], [dx.data_ptr()] * 2, [dy.data_ptr()] * 2, dev.stream)
    with pytest.raises(rc.RabbitCudaError, match="1..32"):
        rc.gemv_batch_dev([a] * 33, [dx.data_ptr()] * 33, [dy.data_ptr()] * 33, dev.stream)
    a.free()
    b.free()
