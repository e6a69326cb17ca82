"""The int8 row quantizers' fast path, restated in float32 numpy: the code of
v at scale s is rn_even(v / s); the kernels form t = RN(v * RN(1 / s)), round
it to the nearest integer (ties to even) and fall back to the division only
when t lies within 1e-4 of a half-integer. Here every rounding step is the
same IEEE float32 step the device takes, over millions of bf16 values and
scales, ties and near-ties included: the fast path must give the division
rule's codes everywhere (the device itself is checked against the oracle in
tests/test_gpu_gemm.py)."""
import numpy as np


def _bf16(a):
    b = np.asarray(a, np.float32).view(np.uint32).astype(np.uint64)
    return (((b + 0x7FFF + ((b >> 16) & 1)) >> 16) << 16).astype(np.uint32).view(np.float32)


def _codes_div(v, s):
    return np.clip(np.rint((v / s).astype(np.float32)), -127, 127).astype(np.int32)


def _codes_fast(v, s):
    r = (np.float32(1.0) / s).astype(np.float32)
    t = (v * r).astype(np.float32)
    k = np.rint(t).astype(np.int32)          # numpy rounds half to even, as the device add does
    d = (t - np.rint(t)).astype(np.float32)
    near = np.abs(np.abs(d) - np.float32(0.5)) < np.float32(1e-4)
    sb = np.broadcast_to(np.asarray(s, np.float32), v.shape)
    k[near] = _codes_div(v[near], sb[near])
    return np.clip(k, -127, 127)


def test_random_rows():
    rng = np.random.default_rng(0)
    for scale in (1e-3, 0.02, 1.0, 37.0):
        x = _bf16(rng.normal(0, scale, (256, 4096)))
        amax = np.abs(x).max(axis=1, keepdims=True)
        s = (amax / np.float32(127.0)).astype(np.float32)
        assert np.array_equal(_codes_fast(x, s), _codes_div(x, s))


def test_ties_and_near_ties():
    rng = np.random.default_rng(1)
    for amax in (127.0, 63.5, 100.0, 3.3, 0.015):
        a = _bf16(np.float32(amax))
        s = np.float32(a / np.float32(127.0))
        k = rng.integers(-126, 126, 200000).astype(np.float32)
        v = _bf16(((k + np.float32(0.5)) * s).astype(np.float32))
        for d in (0, 1, -1):
            bits = (v.view(np.uint32) >> 16).astype(np.int64) + d
            w = np.clip((bits.astype(np.uint32) << 16).view(np.float32), -a, a)
            assert np.array_equal(_codes_fast(w, s), _codes_div(w, s))
