"""ctypes binding of include/rabbit_cuda.h (librabbit_cuda.so, built in-tree).

There is no CPU fallback: `lib()` raises if the shared library is missing or
cannot be loaded, and every wrapper raises RabbitCudaError on a non-zero
status, carrying rabbit_cuda_last_error().
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

import numpy as np

SO = Path(__file__).resolve().parent / "librabbit_cuda.so"

OK, ERR_IO, ERR_MEM, ERR_FORMAT, ERR_UNSUPPORTED, ERR_ARGS, ERR_DEVICE, ERR_TIMEOUT = range(8)
STATUS_NAMES = ["OK", "IO", "MEM", "FORMAT", "UNSUPPORTED", "ARGS", "DEVICE", "TIMEOUT"]


class RabbitCudaError(RuntimeError):
    def __init__(self, status: int, msg: str):
        name = STATUS_NAMES[status] if 0 <= status < len(STATUS_NAMES) else str(status)
        super().__init__(f"rabbit_cuda status {name}: {msg}")
        self.status = status


class MoeDesc(C.Structure):
    """rabbit_cuda_moe_desc"""
    _fields_ = [("n_layers", C.c_int), ("hidden", C.c_int), ("n_experts", C.c_int),
                ("experts_per_token", C.c_int), ("inter", C.c_int), ("n_shared", C.c_int),
                ("expert_quant", C.c_int), ("expert_size", C.c_uint64),
                ("n_records", C.c_int), ("experts_per_layer", C.c_int),
                ("experts_shared", C.c_int), ("expert_map", C.c_void_p),
                ("rms_ffn", C.POINTER(C.c_void_p)), ("w_router", C.POINTER(C.c_void_p))]


class DenseDesc(C.Structure):
    """rabbit_cuda_dense_desc"""
    _fields_ = [("n_layers", C.c_int), ("hidden", C.c_int), ("vocab", C.c_int),
                ("n_heads", C.c_int), ("n_kv_heads", C.c_int), ("head_dim", C.c_int),
                ("max_ctx", C.c_int), ("embed", C.c_void_p), ("lm_head", C.c_void_p),
                ("final_norm", C.c_void_p), ("rms_attn", C.POINTER(C.c_void_p)),
                ("w_q", C.POINTER(C.c_void_p)), ("w_k", C.POINTER(C.c_void_p)),
                ("w_v", C.POINTER(C.c_void_p)), ("w_o", C.POINTER(C.c_void_p))]


_P = C.c_void_p
_I = C.c_int
# name -> (restype, argtypes)
SIGNATURES = {
    "rabbit_cuda_version": (C.c_char_p, []),
    "rabbit_cuda_last_error": (C.c_char_p, []),
    "rabbit_cuda_device_count": (_I, [C.POINTER(_I)]),
    "rabbit_cuda_set_device": (_I, [_I]),
    "rabbit_cuda_set_wait_limit_ms": (_I, [_I]),
    "rabbit_cuda_set_wait_limit_us": (_I, [_I]),
    "rabbit_cuda_gemv_int4_grouped": (_I, [_P, _P, _P, _I, _I]),
    "rabbit_cuda_dequant_int4_grouped_dev": (_I, [_P, _P, _I, _P]),
    "rabbit_cuda_gemv_int4_grouped_dev": (_I, [_P, _P, _P, _I, _I, _P]),
    "rabbit_cuda_matrix_upload": (_I, [_P, _I, _I, C.POINTER(_P)]),
    "rabbit_cuda_matrix_free": (_I, [_P]),
    "rabbit_cuda_matrix_gemv_dev": (_I, [_P, _P, _P, _P]),
    "rabbit_cuda_matrix_gemv_batch_dev": (_I, [_P, _I, _P, _P, _P]),
    "rabbit_cuda_matrix_gemv": (_I, [_P, _P, _P]),
    "rabbit_cuda_matrix_bytes": (C.c_uint64, [_P]),
    "rabbit_cuda_moe_create": (_I, [C.POINTER(MoeDesc), _I, C.POINTER(_P)]),
    "rabbit_cuda_moe_upload": (_I, [_P, _I, _I]),
    "rabbit_cuda_moe_upload_file": (_I, [_P, C.c_char_p, C.c_uint64, _I, _I]),
    "rabbit_cuda_tile_records": (_I, [_P, _I, _P, _I, _P, C.POINTER(C.c_uint64)]),
    "rabbit_cuda_moe_create_window": (_I, [_P, _I, _I, _P]),
    "rabbit_cuda_moe_sync": (_I, [_P]),
    "rabbit_cuda_moe_fill_synthetic": (_I, [_P, C.c_uint64, C.c_float]),
    "rabbit_cuda_moe_free": (_I, [_P]),
    "rabbit_cuda_moe_decode": (_I, [_P, _I, _P, _P, _P, _P, C.POINTER(_I)]),
    "rabbit_cuda_moe_decode_dev": (_I, [_P, _I, _P, _P, _P, _P, _P]),
    "rabbit_cuda_moe_decode_dev_noalloc": (_I, [_P, _I, _P, _P, _P, _P, _P]),
    "rabbit_cuda_moe_check": (_I, [_P, _P]),
    "rabbit_cuda_moe_debug_withhold_score": (_I, [_P, _I]),
    "rabbit_cuda_moe_stats": (_I, [_P, C.POINTER(C.c_uint64), C.POINTER(C.c_uint64),
                                   C.POINTER(C.c_uint64), C.POINTER(_I),
                                   C.POINTER(C.c_uint64)]),
    "rabbit_cuda_moe_stats_ex": (_I, [_P, C.POINTER(C.c_uint64), C.POINTER(C.c_uint64),
                                      C.POINTER(C.c_uint64), C.POINTER(C.c_uint64),
                                      C.POINTER(C.c_uint64), C.POINTER(_I), C.POINTER(_I)]),
    "rabbit_cuda_moe_decode_bytes": (C.c_uint64, [_P]),
    "rabbit_cuda_cache_create": (_P, [_I]),
    "rabbit_cuda_cache_free": (None, [_P]),
    "rabbit_cuda_cache_set_expert_size": (None, [_P, C.c_size_t]),
    "rabbit_cuda_cache_get": (_P, [_P, _I]),
    "rabbit_cuda_cache_put": (_P, [_P, _I, _P]),
    "rabbit_cuda_cache_pin": (_I, [_P, _I, _P]),
    "rabbit_cuda_cache_stats": (None, [_P, C.POINTER(C.c_uint64), C.POINTER(C.c_uint64),
                                       C.POINTER(C.c_uint64)]),
    "rabbit_cuda_cache_stats_ex": (None, [_P, C.POINTER(C.c_uint64), C.POINTER(C.c_uint64),
                                          C.POINTER(C.c_uint64), C.POINTER(C.c_uint64),
                                          C.POINTER(C.c_uint64), C.POINTER(_I), C.POINTER(_I)]),
    "rabbit_cuda_moe_prefill_dev": (_I, [_P, _I, _P, _P, _I, _P, _P, _P]),
    "rabbit_cuda_moe_prefill": (_I, [_P, _I, _P, _P, _I, _P, _P]),
    "rabbit_cuda_moe_set_expert_parallel": (_I, [_P, _I, _I]),
    "rabbit_cuda_ep_unique_id": (_I, [_P]),
    "rabbit_cuda_ep_create": (_P, [_P, _I, _I, _I]),
    "rabbit_cuda_ep_free": (None, [_P]),
    "rabbit_cuda_ep_abort": (_I, [_P]),
    "rabbit_cuda_ep_set_timing": (_I, [_P, _I]),
    "rabbit_cuda_ep_stats": (_I, [_P, C.POINTER(C.c_uint64), C.POINTER(C.c_double),
                                  C.POINTER(C.c_double), _I]),
    "rabbit_cuda_moe_set_ep": (_I, [_P, _P, _I]),
    "rabbit_cuda_legacy_apply_expert": (_I, [_P, C.c_uint64, _I, _I, _I, _P, C.c_float]),
    "rabbit_cuda_legacy_apply_expert_dev": (_I, [_P, C.c_uint64, _I, _I, _I, _P, C.c_float,
                                                 _P]),
    "rabbit_cuda_refv2_create": (_I, [C.POINTER(DenseDesc), _P, C.POINTER(_P)]),
    "rabbit_cuda_refv2_fill_synthetic": (_I, [_P, C.c_uint64, C.c_float]),
    "rabbit_cuda_refv2_free": (_I, [_P]),
    "rabbit_cuda_refv2_reset": (_I, [_P]),
    "rabbit_cuda_refv2_step": (_I, [_P, _I, _P, _P, C.POINTER(_I)]),
    "rabbit_cuda_refv2_prefill": (_I, [_P, _P, _I, _P, _P, C.POINTER(_I)]),
    "rabbit_cuda_refv2_generate": (_I, [_P, _I, _P]),
    "rabbit_cuda_refv2_position": (_I, [_P]),
    "rabbit_cuda_refv2_device_ms": (_I, [_P, C.POINTER(C.c_float)]),
}

_LIB: C.CDLL | None = None


def lib() -> C.CDLL:
    """Load librabbit_cuda.so once. Raises if it is missing (no fallback)."""
    global _LIB
    if _LIB is None:
        if not SO.exists():
            raise RuntimeError(f"{SO} is not built; run `python -m rabbit_b200.build`")
        so = C.CDLL(str(SO))
        for name, (res, args) in SIGNATURES.items():
            f = getattr(so, name)
            f.restype = res
            f.argtypes = args
        _LIB = so
    return _LIB


def check(status: int) -> None:
    if status != OK:
        raise RabbitCudaError(status, lib().rabbit_cuda_last_error().decode(errors="replace"))


def device_count() -> int:
    n = C.c_int(0)
    check(lib().rabbit_cuda_device_count(C.byref(n)))
    return n.value


def _ptr(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


def gemv_int4_grouped(blob: np.ndarray, x: np.ndarray, out_dim: int, in_dim: int) -> np.ndarray:
    """Host-buffer drop-in for rabbit_gemv_int4_grouped."""
    blob = np.ascontiguousarray(blob, np.uint8)
    x = np.ascontiguousarray(x, np.float32)
    y = np.full(max(out_dim, 1), np.nan, np.float32)
    check(lib().rabbit_cuda_gemv_int4_grouped(_ptr(blob), _ptr(x), _ptr(y), out_dim, in_dim))
    return y[:out_dim]


class Matrix:
    """A resident group-32 int4 matrix (rabbit_cuda_matrix)."""

    def __init__(self, blob: np.ndarray, out_dim: int, in_dim: int):
        blob = np.ascontiguousarray(blob, np.uint8)
        h = C.c_void_p()
        check(lib().rabbit_cuda_matrix_upload(_ptr(blob), out_dim, in_dim, C.byref(h)))
        self.handle = h
        self.out_dim, self.in_dim = out_dim, in_dim

    def gemv(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        y = np.zeros(self.out_dim, np.float32)
        check(lib().rabbit_cuda_matrix_gemv(self.handle, _ptr(x), _ptr(y)))
        return y

    def gemv_dev(self, d_x: int, d_y: int, stream: int = 0) -> None:
        check(lib().rabbit_cuda_matrix_gemv_dev(self.handle, d_x, d_y, stream or None))

    @property
    def nbytes(self) -> int:
        return int(lib().rabbit_cuda_matrix_bytes(self.handle))

    def free(self) -> None:
        if self.handle:
            check(lib().rabbit_cuda_matrix_free(self.handle))
            self.handle = C.c_void_p()

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def gemv_batch_dev(mats, d_xs, d_ys, stream: int = 0) -> None:
    """d_ys[i] = mats[i] @ d_xs[i] in one launch (rabbit_cuda_matrix_gemv_batch_dev);
    device pointers as ints, one shape for all matrices."""
    n = len(mats)
    hs = (C.c_void_p * n)(*[m.handle.value for m in mats])
    xs = (C.c_void_p * n)(*d_xs)
    ys = (C.c_void_p * n)(*d_ys)
    check(lib().rabbit_cuda_matrix_gemv_batch_dev(hs, n, xs, ys, stream or None))


QUANT_INT4_TILED = 36  # RABBIT_CUDA_QUANT_INT4_TILED


def tile_records(records: np.ndarray, expert_size: int, *, hidden: int, n_experts: int,
                 top_k: int, inter: int, n_shared: int = 0, sm_count: int = 148):
    """Group-32 int4 records re-laid into the pool's tiled layout for a GPU
    with sm_count SMs, each with its plan trailer (rabbit_cuda_tile_records;
    host only). Returns (tiled records as one uint8 array, bytes per record)."""
    records = np.ascontiguousarray(records, np.uint8)
    n = records.size // expert_size
    d = MoeDesc(1, hidden, n_experts, top_k, inter, n_shared, 4, expert_size, n, n_experts + n_shared,
                0, None, None, None)
    size = C.c_uint64()
    check(lib().rabbit_cuda_tile_records(C.byref(d), sm_count, None, 0, None, C.byref(size)))
    out = np.empty(n * size.value, np.uint8)
    check(lib().rabbit_cuda_tile_records(C.byref(d), sm_count, _ptr(records), n, _ptr(out),
                                         C.byref(size)))
    return out, size.value


class MoePool:
    """HBM-resident expert pool + MoE decode (rabbit_cuda_moe)."""

    def __init__(self, *, records: np.ndarray, expert_size: int, n_layers: int, hidden: int,
                 n_experts: int, top_k: int, inter: int, n_shared: int = 0, quant: int = 4,
                 experts_per_layer: int | None = None, experts_shared: bool = False,
                 rms_ffn, w_router, device: int = 0, upload: bool = True,
                 window: int | None = None):
        """window: HBM blocks for that many layers (rabbit_cuda_moe_create_window);
        layers are then uploaded on demand and nothing is uploaded here."""
        if records is None:  # device-filled (fill_synthetic) or file-backed (upload_file) pool
            self._records = None
            n_records = n_layers * (experts_per_layer or (n_experts + n_shared))
            upload = False
        else:
            self._records = np.ascontiguousarray(records, np.uint8)
            n_records = self._records.size // expert_size
        self._rms = [np.ascontiguousarray(r, np.float32) for r in rms_ffn]
        self._router = [np.ascontiguousarray(r, np.float32) for r in w_router]
        rms_arr = (C.c_void_p * n_layers)(*[r.ctypes.data for r in self._rms])
        rt_arr = (C.c_void_p * n_layers)(*[r.ctypes.data for r in self._router])
        self._keep = (rms_arr, rt_arr)
        d = MoeDesc(n_layers, hidden, n_experts, top_k, inter, n_shared, quant, expert_size,
                    n_records, experts_per_layer or (n_experts + n_shared),
                    1 if experts_shared else 0,
                    None if self._records is None else self._records.ctypes.data,
                    C.cast(rms_arr, C.POINTER(C.c_void_p)), C.cast(rt_arr, C.POINTER(C.c_void_p)))
        h = C.c_void_p()
        if window:
            check(lib().rabbit_cuda_moe_create_window(C.byref(d), device, window, C.byref(h)))
            upload = False
        else:
            check(lib().rabbit_cuda_moe_create(C.byref(d), device, C.byref(h)))
        self.handle = h
        self._decode = lib().rabbit_cuda_moe_decode
        self.hidden, self.n_layers = hidden, n_layers
        self.k = min(top_k if top_k > 0 else 2, n_experts, 8)
        if upload:
            self.upload(0, n_layers)
            self.sync()

    def upload(self, lb: int, le: int) -> None:
        check(lib().rabbit_cuda_moe_upload(self.handle, lb, le))

    def upload_file(self, path, expert_offset: int, lb: int, le: int) -> None:
        """Records of layers [lb, le) read from `path`, record 0 at byte
        `expert_offset` (rabbit_cuda_moe_upload_file); queued, see sync()."""
        check(lib().rabbit_cuda_moe_upload_file(self.handle, str(path).encode(), expert_offset,
                                                lb, le))

    def sync(self) -> None:
        check(lib().rabbit_cuda_moe_sync(self.handle))

    def fill_synthetic(self, seed: int, sigma: float = 0.02) -> None:
        check(lib().rabbit_cuda_moe_fill_synthetic(self.handle, seed, sigma))

    def decode(self, layer: int, h: np.ndarray):
        """Host buffers. Returns (h_out, ids[k], weights[k])."""
        h = np.ascontiguousarray(h, np.float32)
        out = np.zeros_like(h)
        ids = np.zeros(8, np.int32)
        w = np.zeros(8, np.float32)
        k = C.c_int(0)
        check(lib().rabbit_cuda_moe_decode(self.handle, layer, _ptr(h), _ptr(out), _ptr(ids),
                                           _ptr(w), C.byref(k)))
        return out, ids[:k.value].copy(), w[:k.value].copy()

    def decode_into(self, layer: int, h: np.ndarray, out: np.ndarray) -> None:
        """decode on caller-owned host buffers (C-contiguous float32 [H]; out may
        be h), allocating nothing per call: the form an engine's token loop uses."""
        check(self._decode(self.handle, layer, h.ctypes.data, out.ctypes.data, None, None, None))

    def decode_dev(self, layer: int, d_h_in: int, d_h_out: int, d_ids: int = 0,
                   d_w: int = 0, stream: int = 0) -> None:
        check(lib().rabbit_cuda_moe_decode_dev(self.handle, layer, d_h_in, d_h_out,
                                               d_ids or None, d_w or None, stream or None))

    def decode_dev_noalloc(self, layer: int, d_h_in: int, d_h_out: int, d_ids: int = 0,
                           d_w: int = 0, stream: int = 0) -> None:
        """decode_dev with the library's fixed scratch array instead of the
        pool's; allocates nothing (one call at a time per device)."""
        check(lib().rabbit_cuda_moe_decode_dev_noalloc(self.handle, layer, d_h_in, d_h_out,
                                                       d_ids or None, d_w or None,
                                                       stream or None))

    def prefill(self, layer: int, h: np.ndarray):
        """Host buffers, h [T, H]. Returns (h_out [T, H], ids [T, k], weights [T, k])."""
        h = np.ascontiguousarray(h, np.float32)
        T = h.shape[0]
        out = np.zeros_like(h)
        ids = np.zeros((T, self.k), np.int32)
        w = np.zeros((T, self.k), np.float32)
        check(lib().rabbit_cuda_moe_prefill(self.handle, layer, _ptr(h), _ptr(out), T, _ptr(ids),
                                            _ptr(w)))
        return out, ids, w

    def set_expert_parallel(self, rank: int, size: int) -> None:
        """This pool holds rank `rank`'s experts (e % size == rank) of `size`."""
        check(lib().rabbit_cuda_moe_set_expert_parallel(self.handle, rank, size))

    def set_ep(self, ep: "Ep | None", mode: int = 0) -> None:
        """Exchange the pool's expert-parallel share through `ep` in `mode`
        (EP_ALLREDUCE / EP_ALLTOALL) inside every prefill call; None: none."""
        check(lib().rabbit_cuda_moe_set_ep(self.handle, ep.handle if ep else None, mode))

    def prefill_dev(self, layer: int, d_h_in: int, d_h_out: int, n_tokens: int, d_ids: int = 0,
                    d_w: int = 0, stream: int = 0) -> None:
        check(lib().rabbit_cuda_moe_prefill_dev(self.handle, layer, d_h_in, d_h_out, n_tokens,
                                                d_ids or None, d_w or None, stream or None))

    def check(self, stream: int = 0) -> None:
        check(lib().rabbit_cuda_moe_check(self.handle, stream or None))

    def stats(self) -> dict:
        a, b, c, e = C.c_uint64(), C.c_uint64(), C.c_uint64(), C.c_uint64()
        r = C.c_int()
        check(lib().rabbit_cuda_moe_stats(self.handle, C.byref(a), C.byref(b), C.byref(c),
                                          C.byref(r), C.byref(e)))
        return {"hbm_hits": a.value, "uploads": b.value, "h2d_bytes": c.value,
                "resident_records": r.value, "pool_bytes": e.value}

    def stats_ex(self) -> dict:
        """The rabbit_cache_stats_ex counters of the pool."""
        v = [C.c_uint64() for _ in range(5)]
        n = [C.c_int(), C.c_int()]
        check(lib().rabbit_cuda_moe_stats_ex(self.handle, *[C.byref(x) for x in v],
                                             *[C.byref(x) for x in n]))
        keys = ("hits", "misses", "inserts", "evictions", "bytes_copied")
        return {**{k: x.value for k, x in zip(keys, v)}, "n_slots": n[0].value,
                "n_pinned": n[1].value}

    @property
    def decode_bytes(self) -> int:
        return int(lib().rabbit_cuda_moe_decode_bytes(self.handle))

    def free(self) -> None:
        if self.handle:
            check(lib().rabbit_cuda_moe_free(self.handle))
            self.handle = C.c_void_p()

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class RefV2:
    """Device-resident incremental ref-v2 decode (rabbit_cuda_refv2): dense
    weights + KV cache in HBM, the MoE blocks from `pool` (which must outlive
    this object).

    weights=None leaves the dense weights for fill_synthetic(); otherwise a
    dict with embed [V, H], lm_head [H, V], final_norm [H] and per-layer lists
    rms_attn, w_q, w_k, w_v, w_o (row-major, as the .rabbit dense block).
    """

    def __init__(self, pool: MoePool, *, vocab: int, n_heads: int, n_kv_heads: int,
                 head_dim: int, max_ctx: int = 256, weights: dict | None = None):
        L, H = pool.n_layers, pool.hidden
        self.pool, self.vocab, self.hidden = pool, vocab, H
        null = C.POINTER(C.c_void_p)()
        if weights is None:
            d = DenseDesc(L, H, vocab, n_heads, n_kv_heads, head_dim, max_ctx, None, None, None,
                          null, null, null, null, null)
            keep = ()
        else:
            f32 = lambda a: np.ascontiguousarray(a, np.float32)  # noqa: E731
            glob = [f32(weights[n]) for n in ("embed", "lm_head", "final_norm")]
            per = {n: [f32(a) for a in weights[n]] for n in ("rms_attn", "w_q", "w_k", "w_v",
                                                              "w_o")}
            arrs = {n: (C.c_void_p * L)(*[a.ctypes.data for a in per[n]]) for n in per}
            keep = (glob, per, arrs)
            d = DenseDesc(L, H, vocab, n_heads, n_kv_heads, head_dim, max_ctx,
                          *[a.ctypes.data for a in glob],
                          *[C.cast(arrs[n], C.POINTER(C.c_void_p)) for n in ("rms_attn", "w_q",
                                                                              "w_k", "w_v",
                                                                              "w_o")])
        h = C.c_void_p()
        check(lib().rabbit_cuda_refv2_create(C.byref(d), pool.handle, C.byref(h)))
        del keep  # the weights are on the device now
        self.handle = h

    def fill_synthetic(self, seed: int, sigma: float = 0.02) -> None:
        check(lib().rabbit_cuda_refv2_fill_synthetic(self.handle, seed, sigma))

    def reset(self) -> None:
        check(lib().rabbit_cuda_refv2_reset(self.handle))

    @property
    def position(self) -> int:
        return int(lib().rabbit_cuda_refv2_position(self.handle))

    def prefill(self, ids, want_logits: bool = True, want_hidden: bool = True):
        """Returns (logits[V] or None, hidden[H] or None, argmax)."""
        ids = np.ascontiguousarray(ids, np.int32)
        logits = np.full(self.vocab, np.nan, np.float32) if want_logits else None
        hidden = np.full(self.hidden, np.nan, np.float32) if want_hidden else None
        am = C.c_int(-1)
        check(lib().rabbit_cuda_refv2_prefill(
            self.handle, ids.ctypes.data, ids.size, None if logits is None else _ptr(logits),
            None if hidden is None else _ptr(hidden), C.byref(am)))
        return logits, hidden, am.value

    def step(self, token_id: int, want_logits: bool = True, want_hidden: bool = True):
        return self.prefill([token_id], want_logits, want_hidden)

    @property
    def device_ms(self) -> float:
        """Device time of the kernels of the latest prefill/step/generate (ms)."""
        ms = C.c_float()
        check(lib().rabbit_cuda_refv2_device_ms(self.handle, C.byref(ms)))
        return ms.value

    def generate(self, n_new: int) -> np.ndarray:
        out = np.full(n_new, -1, np.int32)
        check(lib().rabbit_cuda_refv2_generate(self.handle, n_new, _ptr(out)))
        return out

    def free(self) -> None:
        if self.handle:
            check(lib().rabbit_cuda_refv2_free(self.handle))
            self.handle = C.c_void_p()

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def legacy_apply_expert(record: np.ndarray, quant: int, hidden: np.ndarray, expert_dim: int,
                        weight: float) -> np.ndarray:
    """src/moe.c:119-224 on the GPU: hidden + the legacy per-tensor expert's
    output (host arrays; returns a new array)."""
    record = np.ascontiguousarray(record, np.uint8)
    h = np.ascontiguousarray(hidden, np.float32).copy()
    check(lib().rabbit_cuda_legacy_apply_expert(_ptr(record), record.size, quant, h.size,
                                                expert_dim, _ptr(h), float(weight)))
    return h


EP_ID_BYTES = 128
EP_ALLREDUCE = 1
EP_ALLTOALL = 2


def ep_unique_id() -> bytes:
    """A new communicator id for Ep (made by one rank, handed to the others)."""
    buf = C.create_string_buffer(EP_ID_BYTES)
    check(lib().rabbit_cuda_ep_unique_id(buf))
    return buf.raw


class Ep:
    """The library's expert-parallel exchange (rabbit_cuda_ep_*): an NCCL
    communicator joined collectively by every rank."""

    def __init__(self, uid: bytes, rank: int, size: int, device: int):
        assert len(uid) == EP_ID_BYTES
        buf = C.create_string_buffer(uid, EP_ID_BYTES)
        self.handle = lib().rabbit_cuda_ep_create(buf, rank, size, device)
        if not self.handle:
            raise RabbitCudaError(ERR_DEVICE, lib().rabbit_cuda_last_error().decode())
        self.rank, self.size, self.device = rank, size, device

    def set_timing(self, on: bool) -> None:
        check(lib().rabbit_cuda_ep_set_timing(self.handle, 1 if on else 0))

    def stats(self, reset: bool = False) -> dict:
        n, t, x = C.c_uint64(), C.c_double(), C.c_double()
        check(lib().rabbit_cuda_ep_stats(self.handle, C.byref(n), C.byref(t), C.byref(x),
                                         1 if reset else 0))
        return {"calls": n.value, "total_ms": t.value, "exchange_ms": x.value}

    def abort(self) -> None:
        check(lib().rabbit_cuda_ep_abort(self.handle))

    def free(self) -> None:
        if self.handle:
            lib().rabbit_cuda_ep_free(self.handle)
            self.handle = None


class Cache:
    """The reference's expert cache API (rabbit_cache_*, src/rabbit.h:123-134)
    with HBM slots: get / put / pin return device addresses (0 for NULL)."""

    def __init__(self, n_slots: int):
        self.handle = lib().rabbit_cuda_cache_create(n_slots)
        if not self.handle:
            raise RabbitCudaError(ERR_DEVICE, lib().rabbit_cuda_last_error().decode())

    def set_expert_size(self, size: int) -> None:
        lib().rabbit_cuda_cache_set_expert_size(self.handle, size)

    def get(self, expert_id: int) -> int:
        return lib().rabbit_cuda_cache_get(self.handle, expert_id) or 0

    def put(self, expert_id: int, record) -> int:
        src = None if record is None else _ptr(record)
        return lib().rabbit_cuda_cache_put(self.handle, expert_id, src) or 0

    def pin(self, expert_id: int, record=None) -> int:
        src = None if record is None else _ptr(record)
        return int(lib().rabbit_cuda_cache_pin(self.handle, expert_id, src))

    def stats_ex(self) -> tuple:
        v = [C.c_uint64() for _ in range(5)]
        n = [C.c_int(), C.c_int()]
        lib().rabbit_cuda_cache_stats_ex(self.handle, *[C.byref(x) for x in v],
                                         *[C.byref(x) for x in n])
        return tuple(x.value for x in v) + (n[0].value, n[1].value)

    def free(self) -> None:
        if self.handle:
            lib().rabbit_cuda_cache_free(self.handle)
            self.handle = None
