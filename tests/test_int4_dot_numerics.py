"""The integer arithmetic of the group-32 int4 dot products, restated in numpy
and checked against exact int64 sums at the extremes of its ranges (no GPU).

Both kernel families quantise a group's 32 activations to
X = rint(x * 2^(22-e)) with 2^e > max|x| (so |X| <= 2^22) and split X into
8-bit planes:
  * decode (rb_device.cuh make_xplanes / dot32): bytes 0 and 1 of X unsigned,
    byte 2 signed; dp4a sums S_p = sum nib * B_p over the unsigned nibbles, and
    sum q X = S0 + 256 S1 + 65536 S2 - 8 sum X formed in 32-bit wrap-around
    arithmetic;
  * tensor cores (rb_moe_tc.cu k_tc_images / readout): signed digits
    D0, D1 in [-128, 127], D2 in [-64, 64]; A = 16 q; the MMA's plane sums
    S_p = sum 16 q D_p, and sum q X = S0 / 16 + 16 S1 + 4096 S2 in int32.
Both rely on |sum q X| <= 32 * 8 * 2^22 = 2^30; these tests pin that bound and
the exactness of both combinations, including the worst cases."""
from __future__ import annotations

import numpy as np
import pytest

I32_MIN, I32_MAX = -(2**31), 2**31 - 1


def exponent_of(amax: np.ndarray) -> np.ndarray:
    """e with 2^e > amax, from the float's exponent field, clamped at -100
    (the kernels' rule)."""
    bits = np.asarray(amax, dtype=np.float32).view(np.uint32)
    e = ((bits >> 23) & 0xFF).astype(np.int64) - 126
    return np.maximum(e, -100)


def quantise(x: np.ndarray) -> np.ndarray:
    """X = rint(x * 2^(22-e)) per group (rows of x), as int64."""
    amax = np.abs(x).max(axis=1)
    e = exponent_of(amax.astype(np.float32))
    scale = np.ldexp(np.float32(1.0), (22 - e)).astype(np.float32)
    return np.rint(x.astype(np.float32) * scale[:, None]).astype(np.int64)


def decode_combine(nib: np.ndarray, X: np.ndarray) -> np.ndarray:
    """dot32: unsigned byte planes, dp4a sums, 32-bit wrap-around combine."""
    Xu = X.astype(np.int64) & 0xFFFFFFFF
    b0 = Xu & 0xFF
    b1 = (Xu >> 8) & 0xFF
    b2 = X >> 16  # byte 2 read as a signed int8
    assert np.all((b2 >= -64) & (b2 <= 64))
    n = nib.astype(np.int64)
    s0 = (n * b0).sum(axis=1)
    s1 = (n * b1).sum(axis=1)
    s2 = (n * b2).sum(axis=1)
    # each dp4a sum fits int32 by itself
    for s in (s0, s1, s2):
        assert np.all((s >= I32_MIN) & (s <= I32_MAX))
    m8sum = -8 * X.sum(axis=1)
    assert np.all(np.abs(m8sum) <= 2**30)
    t = (s0.astype(np.uint64) + (s1.astype(np.uint64) << 8) +
         ((s2 & 0xFFFFFFFF).astype(np.uint64) << 16) +
         (m8sum & 0xFFFFFFFF).astype(np.uint64)) & 0xFFFFFFFF
    return t.astype(np.uint32).view(np.int32).astype(np.int64)


def tc_digits(X: np.ndarray):
    d0 = ((X + 128) & 255) - 128
    x1 = (X - d0) >> 8
    d1 = ((x1 + 128) & 255) - 128
    d2 = (x1 - d1) >> 8
    return d0, d1, d2


def tc_combine(nib: np.ndarray, X: np.ndarray) -> np.ndarray:
    """Readout: plane sums of A = 16 q against signed digits, then
    S0 / 16 + 16 S1 + 4096 S2 with every intermediate inside int32."""
    d0, d1, d2 = tc_digits(X)
    assert np.all((d0 >= -128) & (d0 <= 127) & (d1 >= -128) & (d1 <= 127))
    assert np.all((d2 >= -64) & (d2 <= 64))
    assert np.array_equal(d0 + 256 * d1 + 65536 * d2, X)
    A = 16 * (nib.astype(np.int64) - 8)
    S = [(A * d).sum(axis=1) for d in (d0, d1, d2)]
    for s in S:
        assert np.all(np.abs(s) <= 2**19)
        assert np.all(s % 16 == 0)
    part = (S[0] >> 4) + 16 * S[1]
    assert np.all((part >= I32_MIN) & (part <= I32_MAX))
    t = part + 4096 * S[2]
    assert np.all((t >= I32_MIN) & (t <= I32_MAX))
    return t


def exact(nib: np.ndarray, X: np.ndarray) -> np.ndarray:
    return ((nib.astype(np.int64) - 8) * X).sum(axis=1)


def extreme_cases():
    """(nibbles, X) rows that push every bound: |X| = 2^22 everywhere with all
    weights at -8 or at 7, alternating signs, and mixed extremes."""
    rows_n, rows_x = [], []
    top = 2**22
    for nv in (0, 15, 8, 7):
        for xv in (top, -top, top - 1, -(top - 1)):
            rows_n.append(np.full(32, nv))
            rows_x.append(np.full(32, xv))
    alt = np.array([top if i % 2 else -top for i in range(32)])
    rows_n.append(np.array([0 if i % 2 else 15 for i in range(32)]))
    rows_x.append(alt)
    rows_n.append(np.array([15 if i % 2 else 0 for i in range(32)]))
    rows_x.append(alt)
    return np.array(rows_n), np.array(rows_x, dtype=np.int64)


def test_quantised_range_and_error():
    rng = np.random.default_rng(7)
    x = rng.standard_normal((4096, 32)).astype(np.float32)
    x[::7] *= np.float32(1e-30)   # tiny groups hit the exponent clamp
    x[1::7] *= np.float32(1e30)
    # a group whose maximum is exactly a power of two
    x[2] = 0.5
    x[2, 3] = 1.0
    X = quantise(x)
    assert np.all(np.abs(X) <= 2**22)
    amax = np.abs(x).max(axis=1)
    e = exponent_of(amax)
    assert np.all(np.ldexp(1.0, e) > amax)
    # error <= 2^(e-23) per element
    back = X * np.ldexp(1.0, e - 22)[:, None]
    err = np.abs(back - x.astype(np.float64))
    assert np.all(err <= np.ldexp(1.0, e - 23)[:, None] * (1 + 1e-12))


@pytest.mark.parametrize("combine", [decode_combine, tc_combine])
def test_combination_is_exact_at_the_extremes(combine):
    nib, X = extreme_cases()
    want = exact(nib, X)
    assert np.all(np.abs(want) <= 2**30)
    assert np.array_equal(combine(nib, X), want)


@pytest.mark.parametrize("combine", [decode_combine, tc_combine])
def test_combination_is_exact_on_random_groups(combine):
    rng = np.random.default_rng(11)
    nib = rng.integers(0, 16, size=(20000, 32))
    x = rng.standard_normal((20000, 32)).astype(np.float32)
    x[::3] = np.where(rng.random((len(x[::3]), 32)) < 0.5, 1.0, -1.0) * rng.random(
        (len(x[::3]), 32)).astype(np.float32) ** 8
    X = quantise(x)
    assert np.array_equal(combine(nib, X), exact(nib, X))


def test_one_rounding_per_group():
    """The combined integer converts to fp32 with one rounding: within half
    an ulp of the exact value."""
    nib, X = extreme_cases()
    t = tc_combine(nib, X)
    f = t.astype(np.float32).astype(np.float64)
    ulp = np.spacing(np.abs(t).astype(np.float32)).astype(np.float64)
    assert np.all(np.abs(f - t) <= ulp / 2)
