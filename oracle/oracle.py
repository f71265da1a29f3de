"""ctypes front end for the CPU checkers (test infrastructure only).

`Oracle()` wraps liborc.so, the plain-C restatement of the reference's hot-path
arithmetic (rabbit_oracle.c). `Reference()` wraps _ref/libref.so, the
reference engine's own C compiled from its sources by oracle/Makefile. Both
expose the same methods so tests can pin one against the other.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this module, and only as the checker or the timed CPU baseline.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORC_SO = HERE / "liborc.so"
REF_SO = HERE / "_ref" / "libref.so"

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")


def build_oracle() -> Path:
    """Compile liborc.so (gcc) if it is missing."""
    if not ORC_SO.exists():
        subprocess.check_call(["make", "-s", "-C", str(HERE), "oracle"])
    return ORC_SO


def build_reference(ref_src: str | None = None) -> Path | None:
    """Compile _ref/libref.so from the reference sources (`ref_src`, else the
    RABBIT_REF_SRC environment variable: the reference checkout's src/). Returns
    None when the library is not built and no sources are given."""
    if REF_SO.exists():
        return REF_SO
    src = ref_src or os.environ.get("RABBIT_REF_SRC")
    if not src or not Path(src, "quant.c").exists():
        return None
    subprocess.check_call(["make", "-s", "-C", str(HERE), "ref", f"REF_SRC={src}"])
    return REF_SO


def build_engine(ref_src: str | None = None) -> Path | None:
    """Build the reference engine twice from its sources (engine/Makefile):
    _ref/engine/rabbit as it is and _ref/engine/rabbit_cuda with moe_step and
    rabbit_ref_v2_greedy hooked into librabbit_cuda.so (build that first).
    None when no sources are given."""
    src = ref_src or os.environ.get("RABBIT_REF_SRC")
    if not src or not Path(src, "forward_v2.c").exists():
        return None
    subprocess.check_call(["make", "-s", "-C", str(HERE / "engine"), f"REF_SRC={src}"])
    return HERE / "_ref" / "engine"


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


class _Checker:
    """Shared numpy-level API over either shared object."""

    prefix = ""

    def __init__(self, lib: C.CDLL, prefix: str, quant_prefix: str):
        self.lib = lib
        p, q = prefix, quant_prefix
        self._nbytes = getattr(lib, q + "int4_grouped_nbytes")
        self._nbytes.argtypes = [C.c_int, C.c_int]
        self._nbytes.restype = C.c_int
        self._pack = getattr(lib, q + "pack_int4_grouped")
        self._pack.argtypes = [_f32p, C.c_int, C.c_int, _u8p, C.c_int]
        self._pack.restype = C.c_int
        self._deq = getattr(lib, q + "dequant_int4_grouped")
        self._deq.argtypes = [_u8p, _f32p, C.c_int]
        self._deq.restype = C.c_int
        self._gemv = getattr(lib, q + "gemv_int4_grouped")
        self._gemv.argtypes = [_u8p, _f32p, _f32p, C.c_int, C.c_int]
        self._gemv.restype = None
        self._rms = getattr(lib, p + "rmsnorm")
        self._rms.argtypes = [_f32p, _f32p, _f32p, C.c_int]
        self._gemvf = getattr(lib, p + "gemv_f32")
        self._gemvf.argtypes = [_f32p, _f32p, _f32p, C.c_int, C.c_int]
        self._topk = getattr(lib, p + "select_top_k")
        self._topk.argtypes = [_f32p, C.c_int, C.c_int, _i32p, _f32p]
        self._rope = getattr(lib, p + "apply_rope_head")
        self._rope.argtypes = [_f32p, C.c_int, C.c_int]
        self._swiglu = getattr(lib, p + "expert_swiglu")
        self._logits = getattr(lib, p + "logits")
        self._logits.argtypes = [_f32p, _f32p, _f32p, C.c_int, C.c_int]
        self._legacy = getattr(lib, p + "legacy_apply_expert")
        self._legacy.argtypes = [_u8p, C.c_size_t, C.c_int, C.c_int, C.c_int, _f32p, C.c_float]
        self._legacy.restype = None

    # -- quant ---------------------------------------------------------------
    def int4_grouped_nbytes(self, n: int, group_size: int = 32) -> int:
        return int(self._nbytes(n, group_size))

    def pack_int4_grouped(self, src, group_size: int = 32) -> np.ndarray:
        src = _c(src, np.float32).ravel()
        cap = self.int4_grouped_nbytes(src.size, group_size)
        out = np.zeros(max(cap, 1), np.uint8)
        n = self._pack(src, src.size, group_size, out, cap)
        if n < 0:
            raise ValueError("pack failed")
        return out[:n]

    def dequant_int4_grouped(self, blob, n: int) -> np.ndarray:
        out = np.zeros(max(n, 1), np.float32)
        rc = self._deq(_c(blob, np.uint8), out, n)
        if rc != 0:
            raise ValueError("dequant rejected the blob")
        return out[:n]

    def gemv_int4_grouped(self, blob, x, out_dim: int, in_dim: int) -> np.ndarray:
        y = np.full(max(out_dim, 1), np.nan, np.float32)
        self._gemv(_c(blob, np.uint8), _c(x, np.float32), y, out_dim, in_dim)
        return y[:out_dim]

    # -- fp32 pieces ---------------------------------------------------------
    def rmsnorm(self, x, w) -> np.ndarray:
        x = _c(x, np.float32)
        out = np.zeros_like(x)
        self._rms(x, _c(w, np.float32), out, x.size)
        return out

    def gemv_f32(self, W, x) -> np.ndarray:
        W = _c(W, np.float32)
        y = np.zeros(W.shape[0], np.float32)
        self._gemvf(W, _c(x, np.float32), y, W.shape[0], W.shape[1])
        return y

    def select_top_k(self, scores, k: int):
        scores = _c(scores, np.float32)
        ids = np.zeros(k, np.int32)
        w = np.zeros(k, np.float32)
        self._topk(scores, scores.size, k, ids, w)
        return ids, w

    def apply_rope_head(self, x, pos: int) -> np.ndarray:
        x = _c(x, np.float32).copy()
        self._rope(x, x.size, pos)
        return x

    def legacy_apply_expert(self, record, quant: int, hidden, expert_dim: int,
                            weight: float) -> np.ndarray:
        """moe.c:119-224: hidden + the legacy per-tensor expert's output."""
        record = _c(record, np.uint8)
        h = _c(hidden, np.float32).copy()
        self._legacy(record, record.size, quant, h.size, expert_dim, h, float(weight))
        return h

    def logits(self, lm_head, h) -> np.ndarray:
        lm_head = _c(lm_head, np.float32)
        H, V = lm_head.shape
        out = np.zeros(V, np.float32)
        self._logits(lm_head, _c(h, np.float32), out, H, V)
        return out


class Oracle(_Checker):
    """The plain-C restatement (liborc.so)."""

    def __init__(self):
        lib = C.CDLL(str(build_oracle()))
        super().__init__(lib, "orc_", "orc_")
        self._swiglu.argtypes = [_u8p, C.c_size_t, C.c_int, _f32p, _f32p, C.c_int, C.c_int,
                                 C.c_float]
        self._swiglu.restype = C.c_int
        self._moe = lib.orc_moe_step
        self._moe.argtypes = [C.c_void_p, _f32p, _i32p, _f32p]
        self._moe.restype = C.c_int
        self._attn = lib.orc_attention_step
        self._attn.argtypes = [C.c_void_p, _f32p, C.c_void_p, C.c_int]

    def expert_swiglu(self, record, expert_size, quant, xn, H, inter, weight, delta=None):
        delta = np.zeros(H, np.float32) if delta is None else _c(delta, np.float32).copy()
        self._swiglu(_c(record, np.uint8), expert_size, quant, _c(xn, np.float32), delta, H,
                     inter, float(weight))
        return delta

    def moe_step(self, h, *, H, E, top_k, inter, n_shared, quant, n_records, expert_size,
                 records, rms_ffn, w_router):
        """Returns (h_out, ids[k], weights[k])."""
        records = _c(records, np.uint8)
        rms_ffn = _c(rms_ffn, np.float32)
        w_router = _c(w_router, np.float32)
        desc = _OrcMoeLayer(H, E, top_k, inter, n_shared, quant, n_records, expert_size,
                            records.ctypes.data, rms_ffn.ctypes.data, w_router.ctypes.data)
        h = _c(h, np.float32).copy()
        ids = np.full(8, -1, np.int32)
        w = np.zeros(8, np.float32)
        k = self._moe(C.byref(desc), h, ids, w)
        return h, ids[:k].copy(), w[:k].copy()

    def attention_step(self, h, kv_k, kv_v, kv_len, pos, *, n_heads, n_kv_heads, head_dim,
                       rms_attn, w_q, w_k, w_v, w_o):
        """kv_k/kv_v are [max_len, kv_dim] float32 arrays updated in place.
        Returns (h_out, new_kv_len)."""
        arrs = [_c(a, np.float32) for a in (rms_attn, w_q, w_k, w_v, w_o)]
        desc = _OrcAttnLayer(h.size, n_heads, n_kv_heads, head_dim,
                             *[a.ctypes.data for a in arrs])
        kv = _OrcKV(kv_k.ctypes.data, kv_v.ctypes.data, kv_len, kv_k.shape[0])
        h = _c(h, np.float32).copy()
        self._attn(C.byref(desc), h, C.byref(kv), pos)
        return h, kv.len


class Reference(_Checker):
    """The reference engine's own C (oracle/_ref/libref.so)."""

    def __init__(self, path: Path | None = None):
        so = path or build_reference()
        if so is None or not Path(so).exists():
            raise FileNotFoundError("oracle/_ref/libref.so is not built")
        lib = C.CDLL(str(so))
        super().__init__(lib, "ref_", "rabbit_")
        self._swiglu.argtypes = [_u8p, C.c_size_t, C.c_int, _f32p, _f32p, C.c_int, C.c_int,
                                 C.c_float]
        self._swiglu.restype = None
        self._moe = lib.ref_moe_step
        self._moe.argtypes = [C.c_int] * 7 + [C.c_size_t, _u8p, _f32p, _f32p, _f32p]
        self._moe.restype = None
        self._attn = lib.ref_attention_step
        self._attn.argtypes = [C.c_int] * 4 + [_f32p] * 5 + [_f32p, C.c_void_p, C.c_void_p,
                                                               C.POINTER(C.c_int), C.c_int,
                                                               C.c_int]

    def expert_swiglu(self, record, expert_size, quant, xn, H, inter, weight, delta=None):
        delta = np.zeros(H, np.float32) if delta is None else _c(delta, np.float32).copy()
        self._swiglu(_c(record, np.uint8), expert_size, quant, _c(xn, np.float32), delta, H,
                     inter, float(weight))
        return delta

    def moe_step(self, h, *, H, E, top_k, inter, n_shared, quant, n_records, expert_size,
                 records, rms_ffn, w_router):
        """Returns h_out (the reference's moe_step does not report its routing)."""
        h = _c(h, np.float32).copy()
        self._moe(H, E, top_k, inter, n_shared, quant, n_records, expert_size,
                  _c(records, np.uint8), _c(rms_ffn, np.float32), _c(w_router, np.float32), h)
        return h

    def attention_step(self, h, kv_k, kv_v, kv_len, pos, *, n_heads, n_kv_heads, head_dim,
                       rms_attn, w_q, w_k, w_v, w_o):
        h = _c(h, np.float32).copy()
        ln = C.c_int(kv_len)
        self._attn(h.size, n_heads, n_kv_heads, head_dim, *[_c(a, np.float32) for a in
                                                            (rms_attn, w_q, w_k, w_v, w_o)],
                   h, kv_k.ctypes.data, kv_v.ctypes.data, C.byref(ln), kv_k.shape[0], pos)
        return h, ln.value


class _OrcMoeLayer(C.Structure):
    _fields_ = [("hidden", C.c_int), ("n_experts", C.c_int), ("experts_per_token", C.c_int),
                ("inter", C.c_int), ("n_shared", C.c_int), ("quant", C.c_int),
                ("n_records", C.c_int), ("expert_size", C.c_size_t), ("records", C.c_void_p),
                ("rms_ffn", C.c_void_p), ("w_router", C.c_void_p)]


class _OrcAttnLayer(C.Structure):
    _fields_ = [("hidden", C.c_int), ("n_heads", C.c_int), ("n_kv_heads", C.c_int),
                ("head_dim", C.c_int), ("rms_attn", C.c_void_p), ("w_q", C.c_void_p),
                ("w_k", C.c_void_p), ("w_v", C.c_void_p), ("w_o", C.c_void_p)]


class _OrcKV(C.Structure):
    _fields_ = [("k", C.c_void_p), ("v", C.c_void_p), ("len", C.c_int), ("max_len", C.c_int)]
