"""Helpers shared by the GPU parity tests: bf16 rounding on the host, seeded
inputs, torch <-> numpy moves and the comparison metrics."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")


def bf16_round(a):
    """Round-to-nearest-even to bf16, returned as float32 (what the device holds)."""
    a = np.ascontiguousarray(a, np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    r = ((u >> 16) & 1) + 0x7FFF
    return (((u + r) >> 16) << 16).astype(np.uint32).view(np.float32)


def randn(shape, seed, std=1.0, mean=0.0):
    return (np.random.default_rng(seed).normal(mean, std, shape)).astype(np.float32)


def dev_bf16(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to("cuda").to(torch.bfloat16)


def dev_f32(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to("cuda")


def dev_i32(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.int32)).to("cuda")


def host(t):
    return t.float().cpu().numpy() if t.dtype == torch.bfloat16 else t.cpu().numpy()


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    den = np.sqrt((b * b).sum())
    return np.sqrt(((a - b) ** 2).sum()) / den if den > 0 else np.sqrt(((a - b) ** 2).sum())


def max_rel(a, b):
    """max |a - b| / max |b|: the north star's per-layer bar is stated on it."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return np.abs(a - b).max() / max(np.abs(b).max(), 1e-30)
