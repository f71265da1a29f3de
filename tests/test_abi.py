"""The C ABI library: builds, loads, exports every symbol include/rabbit_cuda.h
declares, and rejects bad arguments on the host (no GPU needed)."""
from __future__ import annotations

import ctypes as C
import re
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "rabbit_cuda.h"


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(rabbit_cuda_\w+)\s*\(", text)))


def test_header_declares_the_boundary():
    names = declared_functions()
    for must in ("rabbit_cuda_gemv_int4_grouped", "rabbit_cuda_moe_decode",
                 "rabbit_cuda_moe_create", "rabbit_cuda_dequant_int4_grouped_dev"):
        assert must in names


def test_library_exports_every_declared_symbol(rc):
    so = rc.lib()
    missing = [n for n in declared_functions() if not hasattr(so, n)]
    assert not missing, missing
    assert set(declared_functions()) == set(rc.SIGNATURES), "capi.SIGNATURES out of date"


def test_version_and_device_count(rc):
    assert rc.lib().rabbit_cuda_version().decode().startswith("rabbit-b200")
    assert rc.device_count() >= 0


def test_null_arguments_are_rejected_on_host(rc):
    so = rc.lib()
    assert so.rabbit_cuda_gemv_int4_grouped(None, None, None, 4, 4) == rc.ERR_ARGS
    assert b"NULL" in so.rabbit_cuda_last_error()
    x = np.zeros(4, np.float32)
    assert so.rabbit_cuda_gemv_int4_grouped(x.ctypes.data, x.ctypes.data, x.ctypes.data, 0,
                                            4) == rc.ERR_ARGS
    assert so.rabbit_cuda_moe_create(None, 0, None) == rc.ERR_ARGS
    assert so.rabbit_cuda_set_wait_limit_ms(0) == rc.ERR_ARGS
    h = C.c_void_p()
    assert so.rabbit_cuda_matrix_upload(None, 4, 4, C.byref(h)) == rc.ERR_ARGS
    assert so.rabbit_cuda_moe_decode(None, 0, None, None, None, None, None) == rc.ERR_ARGS


def test_invalid_group_size_writes_zeros_without_device(rc):
    """quant.c:158-161: a bad header zeroes y before any device work."""
    blob = np.zeros(4 + 4 + 8, np.uint8)  # group_size 0
    x = np.ones(16, np.float32)
    y = np.full(1, 7.0, np.float32)
    assert rc.lib().rabbit_cuda_gemv_int4_grouped(blob.ctypes.data, x.ctypes.data,
                                                  y.ctypes.data, 1, 16) == rc.OK
    assert y[0] == 0.0


def test_moe_desc_layout_matches_header(rc):
    """The ctypes mirror of rabbit_cuda_moe_desc has the C field order."""
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    body = re.search(r"typedef struct \{(.*?)\} rabbit_cuda_moe_desc;", text, re.S).group(1)
    fields = re.findall(r"(\w+)\s*;", body)
    assert fields == [f for f, _ in rc.MoeDesc._fields_]


def test_cache_api_without_a_device_follows_null_conventions(rc):
    """The cache keeps the reference's conventions for a NULL cache
    (src/memory.c:68-92): stats read as zeros, get / put return NULL, pin -1;
    creating one on a host without a GPU returns NULL with the reason set."""
    so = rc.lib()
    v = [C.c_uint64(7) for _ in range(5)]
    n = [C.c_int(7), C.c_int(7)]
    so.rabbit_cuda_cache_stats_ex(None, *[C.byref(x) for x in v], *[C.byref(x) for x in n])
    assert [x.value for x in v] == [0] * 5 and [x.value for x in n] == [0, 0]
    assert not so.rabbit_cuda_cache_get(None, 1)
    assert not so.rabbit_cuda_cache_put(None, 1, None)
    assert so.rabbit_cuda_cache_pin(None, 1, None) == -1
    so.rabbit_cuda_cache_free(None)
    if rc.device_count() == 0:
        assert not so.rabbit_cuda_cache_create(4)
        assert so.rabbit_cuda_last_error()
