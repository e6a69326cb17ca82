"""Affine packs as the reference's fixture writes them
(tests/u15-m5-test.cc:263-310 quantize_w8, widened to 4-bit codes and F16
scale storage) and their exact host dequantization: test helpers."""
import numpy as np


def bf16_bits(x):
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def from_bf16_bits(b):
    return (b.astype(np.uint32) << 16).view(np.float32)


def rnd_bf16(x):
    return from_bf16_bits(bf16_bits(x))


def quantize(w, group=64, bits=8, scale_dtype="BF16"):
    """w [N][K] f32 -> (codes u32 [N][K*bits/32], scales, biases [N][K/group]
    as stored (uint16 bf16 bits or float16), the values the kernel sees)."""
    N, K = w.shape
    levels = (1 << bits) - 1
    g = w.reshape(N, K // group, group)
    lo, hi = g.min(-1), g.max(-1)
    s_raw = ((hi - lo) / np.float32(levels)).astype(np.float32)
    if scale_dtype == "BF16":
        s_st, b_st = bf16_bits(s_raw), bf16_bits(lo)
        s = from_bf16_bits(s_st)
        b = from_bf16_bits(b_st)
    else:   # F16 storage; the kernel reads it rounded to bf16
        s_st, b_st = s_raw.astype(np.float16), lo.astype(np.float16)
        s = rnd_bf16(s_st.astype(np.float32))
        b = rnd_bf16(b_st.astype(np.float32))
    with np.errstate(divide="ignore", invalid="ignore"):
        c = np.where(s[..., None] > 0, np.rint((g - b[..., None]) / s[..., None]), 0)
    c = np.clip(c, 0, levels).astype(np.uint32).reshape(N, K)
    per = 32 // bits
    cw = c.reshape(N, K // per, per)
    codes = np.zeros((N, K // per), np.uint32)
    for k in range(per):
        codes |= cw[:, :, k] << np.uint32(k * bits)
    return codes, s_st, b_st, c


def dequant(c, s_st, b_st, group, scale_dtype="BF16"):
    """The kernel's values: bf16(bf16(s) * code + bf16(b)), product and sum in f32."""
    if scale_dtype == "BF16":
        s, b = from_bf16_bits(s_st), from_bf16_bits(b_st)
    else:
        s, b = rnd_bf16(s_st.astype(np.float32)), rnd_bf16(b_st.astype(np.float32))
    N, K = c.shape
    s = np.repeat(s, group, axis=1)
    b = np.repeat(b, group, axis=1)
    prod = (s * c.astype(np.float32)).astype(np.float32)
    return rnd_bf16((prod + b).astype(np.float32))
