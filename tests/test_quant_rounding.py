"""The quantiser's division-free fast path gives rint(v / s) bit for bit.

The CUDA quantiser (quant_code in ouroboros_b200/csrc/hadamard.cuh) computes
t = v * rcp(s) with two correctly rounded fp32 operations and uses rint(t)
unless t is within 2^-14 of a half-integer, where it falls back to the IEEE
division. This restates that decision in numpy float32 (IEEE round to nearest
even, like the device intrinsics) and checks it against the correctly rounded
quotient on random tokens and on values built to sit next to rounding ties.
"""
import numpy as np

THRESH = np.float32(0.5) - np.float32(2.0 ** -14)


def fast_codes(v, s):
    v = v.astype(np.float32)
    s = np.float32(s)
    with np.errstate(over="ignore", invalid="ignore"):
        rs = np.float32(1.0) / s
        t = (v * rs).astype(np.float32)
    r = np.rint(t)
    with np.errstate(invalid="ignore"):
        slow = ~(np.abs((t - r).astype(np.float32)) < THRESH)
    if slow.any():
        r[slow] = np.rint((v[slow] / s).astype(np.float32))
    return np.clip(r, -127, 127).astype(np.int32), int(slow.sum())


def exact_codes(v, s):
    q = np.rint((v.astype(np.float32) / np.float32(s)).astype(np.float32))
    return np.clip(q, -127, 127).astype(np.int32)


def token_scale(x):
    return np.float32(np.max(np.abs(x))) / np.float32(127.0)


def test_fast_path_random_tokens():
    rng = np.random.default_rng(5)
    for scale in (1e-30, 1e-6, 1.0, 3.7, 1e5, 1e30):
        x = (rng.standard_normal((64, 4096)) * scale).astype(np.float32)
        x[:, ::97] *= 20.0
        for row in x:
            s = token_scale(row)
            got, _ = fast_codes(row, s)
            assert np.array_equal(got, exact_codes(row, s))


def test_fast_path_near_ties():
    rng = np.random.default_rng(6)
    s = np.float32(0.0123)
    # values whose quotient is within a few ulp of n + 0.5: the fallback cases
    n = rng.integers(-127, 127, 200000).astype(np.float32)
    base = ((n + np.float32(0.5)) * s).astype(np.float32)
    ulps = rng.integers(-8, 9, base.size).astype(np.int32)
    toward = np.where(ulps >= 0, np.float32(np.inf), np.float32(-np.inf))
    v = np.nextafter(base, toward).astype(np.float32)
    v = np.where(ulps == 0, base, v)
    for k in range(2, 9):
        v2 = np.where(np.abs(ulps) >= k, np.nextafter(v, toward), v)
        v = v2.astype(np.float32)
    got, nslow = fast_codes(v, s)
    assert np.array_equal(got, exact_codes(v, s))
    assert nslow > 0  # the fallback was exercised


def test_zero_and_subnormal_scales():
    v = np.array([0.0, 1e-45, -1e-45, 3e-45], np.float32)
    for s in (np.float32(1e-45), np.float32(1e-40), np.float32(0.0)):
        if s == 0:
            continue  # s == 0 returns 0 before any arithmetic
        got, _ = fast_codes(v, s)
        assert np.array_equal(got, exact_codes(v, s))
