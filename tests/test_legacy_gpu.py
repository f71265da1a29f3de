"""GPU: the legacy per-tensor expert (src/moe.c:119-224, apply_expert)
through rabbit_cuda_legacy_apply_expert[_dev], against the oracle (pinned to
the reference's own apply_expert bit for bit by test_oracle_pin.py) on every
case of legacy_cases.py -- int4 / int8 / quant-0 SwiGLU, the expert_dim default
and clamp, invalid scales, odd int4 row widths, and the square and raw-byte
fallbacks. Bar: rtol 1e-4 / atol 1e-5 on hidden and on the expert's output."""
from __future__ import annotations

import numpy as np
import pytest

from legacy_cases import legacy_cases

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-4, 1e-5
CASES = legacy_cases()


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_legacy_expert_matches_oracle(oracle, case):
    from rabbit_b200 import capi

    name, q, H, ed, rec, h, w = case
    ref = oracle.legacy_apply_expert(rec, q, h, ed, w)
    got = capi.legacy_apply_expert(rec, q, h, ed, w)
    np.testing.assert_allclose(got - h, ref - h, rtol=RTOL, atol=ATOL, err_msg=name)
    np.testing.assert_allclose(got, ref, rtol=RTOL, atol=ATOL, err_msg=name)


def test_legacy_expert_on_device_buffers_and_cached_records(oracle):
    """The _dev entry point on a record held in an HBM cache slot
    (rabbit_cuda_cache_put returns its device address)."""
    import torch

    from rabbit_b200 import capi

    name, q, H, ed, rec, h, w = CASES[1]
    cache = capi.Cache(4)
    cache.set_expert_size(rec.size)
    slot = cache.put(3, rec)
    assert slot and cache.get(3) == slot
    d_h = torch.from_numpy(h.copy()).cuda()
    s = torch.cuda.current_stream()
    capi.check(capi.lib().rabbit_cuda_legacy_apply_expert_dev(slot, rec.size, q, H, ed,
                                                              d_h.data_ptr(), float(w),
                                                              s.cuda_stream))
    torch.cuda.synchronize()
    ref = oracle.legacy_apply_expert(rec, q, h, ed, w)
    np.testing.assert_allclose(d_h.cpu().numpy(), ref, rtol=RTOL, atol=ATOL)
    cache.free()


def test_legacy_odd_rows_past_the_record_are_refused():
    """Odd-width int4 rows that would read past the record's end (the
    reference reads beyond its buffer there) are refused, not read."""
    from rabbit_b200 import capi

    H, inter = 33, 65
    mat = H * inter
    rec = np.zeros(3 * (4 + (mat + 1) // 2), np.uint8)  # no padding
    with pytest.raises(capi.RabbitCudaError, match="past the record"):
        capi.legacy_apply_expert(rec, 4, np.ones(H, np.float32), inter, 1.0)
