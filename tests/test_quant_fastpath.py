"""The int8 quantizers' fast path, restated in numpy: the code of v at scale
s is rn_even(v / s) clamped to +-127; the kernels round the exact product
p = v * RN(1 / s) to the nearest integer k (ties to even; one fma with
1.5 * 2^23), form d = p - k rounded once to float32 (a second fma), and fall
back to the clamped division for a group of 8 holding a value with
|d| > 0.4999, or for every value when the scale is subnormal (1 / s > 2^126).
p is exact in float64 (24 x 24 significant bits), so np.rint(p) and
float32(p - k) are the fma results. Over millions of bf16 values and scales,
ties and near-ties included, the fast path must give the division rule's codes
everywhere (the device itself is checked against the oracle in
tests/test_gpu_gemm.py)."""
import numpy as np


def _bf16(a):
    b = np.asarray(a, np.float32).view(np.uint32).astype(np.uint64)
    return (((b + 0x7FFF + ((b >> 16) & 1)) >> 16) << 16).astype(np.uint32).view(np.float32)


def _codes_div(v, s):
    with np.errstate(divide="ignore", invalid="ignore"):
        t = np.where(s > 0, (v / s).astype(np.float32), np.float32(0.0))
    return np.clip(np.rint(t), -127, 127).astype(np.int32)


def _codes_fast(v, s):
    v = np.asarray(v, np.float32)
    sb = np.broadcast_to(np.asarray(s, np.float32), v.shape)
    with np.errstate(divide="ignore", over="ignore", invalid="ignore"):
        r = np.where(sb > 0, np.float32(1.0) / sb, np.float32(0.0)).astype(np.float32)
        p = v.astype(np.float64) * r.astype(np.float64)
        k = np.rint(p)
        d = (p - k).astype(np.float32)
    tie = (np.abs(d) > np.float32(0.4999)) | (r > np.float32(2.0 ** 126))
    g = tie.reshape(v.shape[:-1] + (-1, 8)).any(axis=-1)      # whole groups of 8
    tie = np.repeat(g, 8, axis=-1).reshape(v.shape)
    codes = np.zeros(v.shape, np.int32)
    codes[~tie] = k[~tie].astype(np.int32)
    codes[tie] = _codes_div(v[tie], sb[tie])
    return codes


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


def test_tiny_and_zero_scales():
    """amax around 127 * 2^-126, where the scale turns subnormal, and below,
    down to bf16 subnormals, plus an all-zero row."""
    rng = np.random.default_rng(2)
    rows = []
    for amax in (1.6e-36, 1.5e-36, 1.4e-36, 1e-37, 1e-38, 3e-39, 1e-40, 0.0):
        v = _bf16(rng.uniform(-1, 1, 4096).astype(np.float32) * np.float32(amax))
        if amax:
            v[7] = _bf16(np.float32(amax))
        rows.append(v)
    x = np.stack(rows)
    amax = np.abs(x).max(axis=1, keepdims=True)
    s = (amax / np.float32(127.0)).astype(np.float32)
    assert np.array_equal(_codes_fast(x, s), _codes_div(x, s))
