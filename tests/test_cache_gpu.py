"""GPU: the HBM-backed expert cache (rabbit_cuda_cache_*) against the
reference's own expert cache (rabbit_cache_*, src/memory.c:12-193, compiled
into oracle/_ref) driven by the same seeded sequence of get / put / pin
calls. Bar: every call returns NULL / -1 exactly when the reference's does,
every record a non-NULL get or put returns holds the bytes the caller put
there (read back from HBM), and the stats_ex counters (hits, misses, inserts,
evictions, bytes copied, slots, pinned slots) are identical after every call.
Edge cases as the reference handles them: n_slots <= 0 (4 slots), more than
64 slots (64), put before the record size is set, every slot pinned.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


class RefCache:
    """ctypes view of the reference's cache in oracle/_ref/libref.so."""

    def __init__(self, lib, n_slots):
        self.lib = lib
        lib.rabbit_cache_create.restype = C.c_void_p
        lib.rabbit_cache_create.argtypes = [C.c_int]
        lib.rabbit_cache_free.argtypes = [C.c_void_p]
        lib.rabbit_cache_set_expert_size.argtypes = [C.c_void_p, C.c_size_t]
        lib.rabbit_cache_get.restype = C.c_void_p
        lib.rabbit_cache_get.argtypes = [C.c_void_p, C.c_int]
        lib.rabbit_cache_put.restype = C.c_void_p
        lib.rabbit_cache_put.argtypes = [C.c_void_p, C.c_int, C.c_void_p]
        lib.rabbit_cache_pin.restype = C.c_int
        lib.rabbit_cache_pin.argtypes = [C.c_void_p, C.c_int, C.c_void_p]
        lib.rabbit_cache_stats_ex.argtypes = [C.c_void_p] + [C.POINTER(C.c_uint64)] * 5 + [
            C.POINTER(C.c_int)] * 2
        self.h = lib.rabbit_cache_create(n_slots)

    def set_expert_size(self, n):
        self.lib.rabbit_cache_set_expert_size(self.h, n)

    def get(self, i):
        return self.lib.rabbit_cache_get(self.h, i) or 0

    def put(self, i, rec):
        return self.lib.rabbit_cache_put(self.h, i, None if rec is None else rec.ctypes.data) or 0

    def pin(self, i, rec=None):
        return self.lib.rabbit_cache_pin(self.h, i, None if rec is None else rec.ctypes.data)

    def stats_ex(self):
        v = [C.c_uint64() for _ in range(5)]
        n = [C.c_int(), C.c_int()]
        self.lib.rabbit_cache_stats_ex(self.h, *[C.byref(x) for x in v], *[C.byref(x) for x in n])
        return tuple(x.value for x in v) + (n[0].value, n[1].value)

    def free(self):
        self.lib.rabbit_cache_free(self.h)


def read_back(addr, size):
    """The bytes at a device address (cuda-python's runtime binding)."""
    from cuda.bindings import runtime as rt

    out = np.empty(size, np.uint8)
    (err,) = rt.cudaMemcpy(out.ctypes.data, addr, size, rt.cudaMemcpyKind.cudaMemcpyDeviceToHost)
    assert err == rt.cudaError_t.cudaSuccess, err
    return out


@pytest.mark.parametrize("n_slots", [6, 1, 0, 80])
def test_cache_follows_the_reference(rc, reference, n_slots):
    size = 4096 + 48  # not a multiple of 256: the slots are padded, the records are not
    rng = np.random.default_rng(11 + n_slots)
    recs = {i: rng.integers(0, 256, size, dtype=np.uint8) for i in range(24)}
    ref = RefCache(reference.lib, n_slots)
    hbm = rc.Cache(n_slots)
    # put before the size is known: NULL on both sides
    assert hbm.put(3, recs[3]) == 0 and ref.put(3, recs[3]) == 0
    ref.set_expert_size(size)
    hbm.set_expert_size(size)
    assert hbm.stats_ex() == ref.stats_ex()
    for step in range(400):
        op = rng.choice(["get", "put", "pin", "pin_null"], p=[0.45, 0.35, 0.1, 0.1])
        i = int(rng.integers(-1, 24)) if op == "get" else int(rng.integers(0, 24))
        if op == "get":
            # id -1 matches an empty slot (expert_id -1) and counts a hit, in
            # the reference as here
            a, b = ref.get(i), hbm.get(i)
            assert (a == 0) == (b == 0), (step, op, i)
            if b and i >= 0:
                np.testing.assert_array_equal(read_back(b, size), recs[i], err_msg=f"step {step}")
        elif op == "put":
            a, b = ref.put(i, recs[i]), hbm.put(i, recs[i])
            assert (a == 0) == (b == 0), (step, op, i)
            if b:
                assert b % 256 == 0
                np.testing.assert_array_equal(read_back(b, size), recs[i], err_msg=f"step {step}")
        elif op == "pin":
            assert hbm.pin(i, recs[i]) == ref.pin(i, recs[i]), (step, op, i)
        else:
            assert hbm.pin(i) == ref.pin(i), (step, op, i)
        assert hbm.stats_ex() == ref.stats_ex(), (step, op, i)
    # every slot pinned: further records find no victim on either side
    for i in range(24):
        assert hbm.pin(i, recs[i]) == ref.pin(i, recs[i])
    for i in range(24):
        assert (hbm.put(100 + i, recs[i]) == 0) == (ref.put(100 + i, recs[i]) == 0)
    assert hbm.stats_ex() == ref.stats_ex()
    hbm.free()
    ref.free()


def test_pool_counters_follow_the_cache_semantics(rc):
    """rabbit_cuda_moe_stats_ex on a windowed pool: uploads are inserts,
    reassigned blocks count evictions, calls on layers not resident count
    misses, kernel calls count hits."""
    from rabbit_b200 import synth

    H, E, K, I, S, L = 128, 4, 2, 64, 0, 3
    layers = [synth.moe_layer(70 + l, H, E, I, S) for l in range(L)]
    kw = dict(expert_size=layers[0][1], n_layers=L, hidden=H, n_experts=E, top_k=K, inter=I,
              n_shared=S, quant=4, rms_ffn=[m[3] for m in layers], w_router=[m[2] for m in layers])
    pool = rc.MoePool(records=np.concatenate([m[0] for m in layers]), window=2, **kw)
    h = np.random.default_rng(1).standard_normal(H).astype(np.float32)
    st = pool.stats_ex()
    assert (st["inserts"], st["evictions"], st["misses"], st["n_slots"], st["n_pinned"]) == (
        0, 0, 0, 2 * E, 0)
    with pytest.raises(rc.RabbitCudaError):
        pool.decode(0, h)
    pool.upload(0, 2)
    pool.decode(0, h)
    pool.decode(1, h)
    pool.upload(2, 3)  # takes layer 0's block: its E records are evicted
    st = pool.stats_ex()
    assert st["misses"] == 1 and st["inserts"] == 3 * E and st["evictions"] == E
    assert st["hits"] == 2 and st["bytes_copied"] > 0
    pool.free()
    full = rc.MoePool(records=np.concatenate([m[0] for m in layers]), **kw)
    assert full.stats_ex()["n_pinned"] == L * E
    full.free()
