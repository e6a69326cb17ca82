"""TEST INFRASTRUCTURE ONLY: ctypes access to the CPU checkers.

Two libraries are bound here, both built by ``oracle/Makefile``:

* ``liboracle.so`` -- our C restatement of the reference's CPU algorithm
  (``u15_oracle.c``), the checker every GPU parity test compares against;
* ``_ref/libu15ref.so`` -- the reference's own ``src/u15-ref.cc`` compiled
  unchanged (plus ``ref_shim.cc``), used to generate the golden fixtures that
  pin the restatement. It exists only where the reference tree does.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg may import this module, and only as the checker.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libu15ref.so")

BIDIR, CAUSAL, BLOCK_CAUSAL = 0, 1, 2

_f32p = C.POINTER(C.c_float)
_i32p = C.POINTER(C.c_int)
_i8p = C.POINTER(C.c_int8)


def build(ref: bool = False) -> None:
    """Build the restatement (and, if asked and present, the reference: the
    checkout named by U15_REFERENCE_DIR, else a `reference` directory beside
    the repository)."""
    target = ["oracle"]
    if ref:
        d = os.environ.get("U15_REFERENCE_DIR") or os.path.join(
            os.path.dirname(os.path.dirname(HERE)), "reference")
        target = ["all", f"REF={d}"]
    subprocess.run(["make", "-s", "-C", HERE] + target, check=True)


def _fp(a):
    return a.ctypes.data_as(_f32p) if a is not None else None


def _ip(a):
    return a.ctypes.data_as(_i32p) if a is not None else None


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


class _Expert(C.Structure):
    _fields_ = [(n, _f32p) for n in (
        "input_layernorm", "post_attention_layernorm", "q_proj", "k_proj",
        "v_proj", "o_proj", "q_norm", "k_norm", "q_norm_hw", "k_norm_hw",
        "gate_proj", "up_proj", "down_proj")]


class _Dims(C.Structure):
    _fields_ = [("hidden", C.c_long), ("heads", C.c_long),
                ("kv_heads", C.c_long), ("head_dim", C.c_long),
                ("inter", C.c_long), ("eps", C.c_double),
                ("theta_t", C.c_double), ("theta_hw", C.c_double)]


EXPERT_KEYS = [n for n, _ in _Expert._fields_]

_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(ORACLE_SO):
            build()
        L = C.CDLL(ORACLE_SO)
        L.orc_rms_norm.argtypes = [_f32p, _f32p, C.c_float, C.c_long, C.c_long, _f32p]
        L.orc_linear.argtypes = [_f32p, _f32p, _f32p, C.c_long, C.c_long, C.c_long, _f32p]
        L.orc_swiglu.argtypes = [_f32p, _f32p, _f32p, C.c_long]
        L.orc_rope_tables.argtypes = [_i32p, _i32p, _i32p, C.c_long, C.c_int, C.c_int,
                                      C.c_int, C.c_double, C.c_double, C.c_int, _f32p, _f32p]
        L.orc_split_qk_norm.argtypes = [_f32p, _f32p, _f32p, C.c_long, C.c_long, C.c_long,
                                        C.c_float]
        L.orc_split_rope.argtypes = [_f32p, _f32p, _f32p, C.c_long, C.c_long, C.c_long,
                                     C.c_int, C.c_int]
        L.orc_attention.argtypes = [_f32p, _f32p, _f32p] + [C.c_long] * 6 + [
            C.c_int, C.c_long, _i32p, _f32p]
        L.orc_mot_layer.argtypes = [_f32p, C.c_long, C.c_int, _i32p, _i32p,
                                    C.POINTER(_Expert), C.POINTER(_Dims), _i32p, _i32p,
                                    _i32p, C.c_long, _f32p, _f32p, C.c_int, _i32p, _f32p,
                                    _f32p, _f32p]
        L.orc_mot_layer_ex.argtypes = [_f32p, C.c_long, C.c_int, _i32p, _i32p,
                                       C.POINTER(_Expert), C.POINTER(_Dims), _i32p, _i32p,
                                       _i32p, C.c_long, _f32p, _f32p, C.c_int, _i32p, C.c_int,
                                       _f32p, _f32p, _f32p]
        L.orc_quant_rows_i8.argtypes = [_f32p, C.c_long, C.c_long, _i8p, _f32p]
        L.orc_gemm_i8.argtypes = [_i8p, _i8p, C.c_long, C.c_long, C.c_long, _i32p]
        L.orc_dequant_i8.argtypes = [_i32p, _f32p, _f32p, C.c_long, C.c_long, _f32p]
        L.orc_sage_attention.argtypes = [_f32p, _f32p, _f32p] + [C.c_long] * 8 + [_f32p]
        L.orc_time_schedule.argtypes = [C.c_int, C.c_double, _f32p]
        L.orc_init_noise.argtypes = [C.c_uint64, C.c_double, _f32p, C.c_long]
        L.orc_mt19937_64_nth.argtypes = [C.c_uint64, C.c_long]
        L.orc_mt19937_64_nth.restype = C.c_uint64
        L.orc_init_noise_scale.argtypes = [C.c_int, C.c_int, C.c_double, C.c_double, C.c_int]
        L.orc_init_noise_scale.restype = C.c_double
        L.orc_velocity.argtypes = [_f32p, _f32p, C.c_long, C.c_double, _f32p]
        L.orc_optimized_scale.argtypes = [_f32p, _f32p, C.c_long]
        L.orc_optimized_scale.restype = C.c_double
        L.orc_cfg.argtypes = [_f32p, _f32p, _f32p, C.c_long, C.c_long, C.c_int, C.c_int,
                              C.c_double, C.c_double, C.c_int, _f32p]
        L.orc_euler.argtypes = [_f32p, _f32p, C.c_long, C.c_double]
        L.orc_patchify_cf.argtypes = [_f32p, C.c_int, C.c_int, C.c_int, C.c_int, _f32p]
        L.orc_gelu_erf.argtypes = [_f32p, C.c_long]
        L.orc_vision_embed.argtypes = [_f32p] * 5 + [C.c_int] * 6 + [C.c_double, _f32p]
        L.orc_conv_decoder_hwc.argtypes = [_f32p] * 5 + [C.c_int] * 4 + [_f32p]
        L.orc_timestep_row.argtypes = [C.c_double, C.c_double, C.c_int, C.c_int] + [_f32p] * 9
        _lib = L
    return _lib


# ---------------------------------------------------------------------------
# restatement wrappers (numpy in, numpy out)
# ---------------------------------------------------------------------------

def rms_norm(x, w, eps=1e-6):
    x = _f32(x); w = _f32(w)
    out = np.empty_like(x)
    rows, dim = x.reshape(-1, x.shape[-1]).shape
    lib().orc_rms_norm(_fp(x), _fp(w), eps, rows, dim, _fp(out))
    return out


def linear(x, w, b=None):
    x = _f32(x); w = _f32(w)
    b = _f32(b) if b is not None else None
    rows = x.shape[0]
    out = np.empty((rows, w.shape[0]), np.float32)
    lib().orc_linear(_fp(x), _fp(w), _fp(b), rows, x.shape[1], w.shape[0], _fp(out))
    return out


def swiglu(g, u):
    g = _f32(g); u = _f32(u)
    y = np.empty_like(g)
    lib().orc_swiglu(_fp(g), _fp(u), _fp(y), g.size)
    return y


def rope_tables(pos_t, pos_h, pos_w, head_dim=128, theta_t=5e6, theta_hw=1e4,
                inv_freq_f32=False):
    pt, ph, pw = (np.ascontiguousarray(p, np.int32) for p in (pos_t, pos_h, pos_w))
    T = pt.size
    c = np.empty((T, head_dim), np.float32)
    s = np.empty((T, head_dim), np.float32)
    lib().orc_rope_tables(_ip(pt), _ip(ph), _ip(pw), T, head_dim, head_dim // 2,
                          head_dim // 4, theta_t, theta_hw, int(inv_freq_f32),
                          _fp(c), _fp(s))
    return c, s


def split_qk_norm(x, w_t, w_hw, heads, eps=1e-6):
    """Token-major [T][heads*hd]; returns a new array."""
    x = _f32(x).copy()
    T = x.shape[0]
    hd = x.shape[1] // heads
    lib().orc_split_qk_norm(_fp(x), _fp(_f32(w_t)), _fp(_f32(w_hw)), heads, T, hd, eps)
    return x


def split_rope(x, cos, sin, heads):
    x = _f32(x).copy()
    T = x.shape[0]
    hd = x.shape[1] // heads
    lib().orc_split_rope(_fp(x), _fp(_f32(cos)), _fp(_f32(sin)), heads, T, hd,
                         hd // 2, hd // 4)
    return x


def attention(q, k, v, tk=None, mode=BIDIR, q_offset=0, t_index=None):
    """q [hq][tq][d]; k/v [hkv][cap][d] (cap >= tk); out [tq][hq*d]."""
    q = _f32(q); k = _f32(k); v = _f32(v)
    hq, tq, d = q.shape
    hkv, cap, _ = k.shape
    tk = cap if tk is None else tk
    ti = np.ascontiguousarray(t_index, np.int32) if t_index is not None else None
    out = np.empty((tq, hq * d), np.float32)
    lib().orc_attention(_fp(q), _fp(k), _fp(v), hq, hkv, tq, tk, d, cap, mode,
                        q_offset, _ip(ti), _fp(out))
    return out


def sage_attention(q, k, v, tk=None, bq=64, bk=64):
    q = _f32(q); k = _f32(k); v = _f32(v)
    hq, tq, d = q.shape
    hkv, cap, _ = k.shape
    tk = cap if tk is None else tk
    out = np.empty((tq, hq * d), np.float32)
    lib().orc_sage_attention(_fp(q), _fp(k), _fp(v), hq, hkv, tq, tk, d, cap, bq, bk,
                             _fp(out))
    return out


def mot_layer(x, segments, experts, dims, pos_t, pos_h, pos_w, k_prefix=None,
              v_prefix=None, mode=BIDIR, t_index=None, int8=False, sage=False,
              bf16_buffers=False):
    """The joint MoT layer. segments: list of (start, end, expert_id).
    int8: every projection under the W8A8 rule; sage: the bidirectional
    attention as Sage int8 QK (64-row / 32-key blocks); bf16_buffers: the
    activations rounded to bf16 wherever the reference's layer stores them.
    experts: list of two dicts keyed by EXPERT_KEYS (fp32 arrays).
    dims: dict(hidden, heads, kv_heads, head_dim, inter, eps, theta_t, theta_hw).
    Returns (out [T][H], k_new [hkv][T][hd], v_new [hkv][T][hd])."""
    x = _f32(x)
    T = x.shape[0]
    keep = []
    E = (_Expert * len(experts))()
    for i, e in enumerate(experts):
        for n in EXPERT_KEYS:
            a = _f32(e[n]); keep.append(a)
            setattr(E[i], n, _fp(a))
    D = _Dims(dims["hidden"], dims["heads"], dims["kv_heads"], dims["head_dim"],
              dims["inter"], dims.get("eps", 1e-6), dims.get("theta_t", 5e6),
              dims.get("theta_hw", 1e4))
    off = np.array([s[0] for s in segments] + [segments[-1][1]], np.int32)
    ex = np.array([s[2] for s in segments], np.int32)
    pt, ph, pw = (np.ascontiguousarray(p, np.int32) for p in (pos_t, pos_h, pos_w))
    npre = 0 if k_prefix is None else k_prefix.shape[1]
    kp = _f32(k_prefix) if k_prefix is not None else None
    vp = _f32(v_prefix) if v_prefix is not None else None
    ti = np.ascontiguousarray(t_index, np.int32) if t_index is not None else None
    out = np.empty_like(x)
    hkv, hd = dims["kv_heads"], dims["head_dim"]
    kn = np.empty((hkv, T, hd), np.float32)
    vn = np.empty((hkv, T, hd), np.float32)
    flags = (1 if int8 else 0) | (2 if sage else 0) | (4 if bf16_buffers else 0)
    lib().orc_mot_layer_ex(_fp(x), T, len(segments), _ip(off), _ip(ex), E, C.byref(D),
                           _ip(pt), _ip(ph), _ip(pw), npre, _fp(kp), _fp(vp), mode,
                           _ip(ti), flags, _fp(out), _fp(kn), _fp(vn))
    return out, kn, vn


def quant_rows_i8(x):
    x = _f32(x)
    rows, cols = x.shape
    q = np.empty((rows, cols), np.int8)
    s = np.empty(rows, np.float32)
    lib().orc_quant_rows_i8(_fp(x), rows, cols, q.ctypes.data_as(_i8p), _fp(s))
    return q, s


def gemm_i8(a, w):
    a = np.ascontiguousarray(a, np.int8); w = np.ascontiguousarray(w, np.int8)
    M, K = a.shape
    N = w.shape[0]
    acc = np.empty((M, N), np.int32)
    lib().orc_gemm_i8(a.ctypes.data_as(_i8p), w.ctypes.data_as(_i8p), M, K, N, _ip(acc))
    return acc


def dequant_i8(acc, s_tok, s_ch):
    acc = np.ascontiguousarray(acc, np.int32)
    M, N = acc.shape
    y = np.empty((M, N), np.float32)
    lib().orc_dequant_i8(_ip(acc), _fp(_f32(s_tok)), _fp(_f32(s_ch)), M, N, _fp(y))
    return y


def init_noise(seed, noise_scale, n):
    """The render's start image, flat channel-last (src/u15-generator.cc:413-417)."""
    out = np.empty(n, np.float32)
    lib().orc_init_noise(seed, noise_scale, _fp(out), n)
    return out


def mt19937_64_nth(seed, nth):
    return int(lib().orc_mt19937_64_nth(seed, nth))


NOISE_CONSTANT, NOISE_RESOLUTION, NOISE_DYNAMIC_SQRT = 0, 1, 2


def init_noise_scale(image_tokens, mode=NOISE_RESOLUTION, noise_scale=1.0, max_value=16.0,
                     base=64):
    return float(lib().orc_init_noise_scale(image_tokens, mode, noise_scale, max_value, base))


def time_schedule(n, shift):
    out = np.empty(n + 1, np.float32)
    lib().orc_time_schedule(n, shift, _fp(out))
    return out


CFG_NONE, CFG_IMG, CFG_UNC, CFG_BOTH = 0, 1, 2, 3
NORM_NONE, NORM_GLOBAL, NORM_CHANNEL, NORM_ZERO_STAR = 0, 1, 2, 3


def velocity(x_pred, img, denom):
    x_pred = _f32(x_pred); img = _f32(img)
    v = np.empty_like(img)
    lib().orc_velocity(_fp(x_pred), _fp(img), img.size, denom, _fp(v))
    return v


def optimized_scale(pos, neg):
    pos = _f32(pos); neg = _f32(neg)
    return lib().orc_optimized_scale(_fp(pos), _fp(neg), pos.size)


def cfg(v_cond, v_unc, v_img, form, norm, cfg_scale, icfg, step):
    """[H][W][3] velocities -> combined velocity (src/u15-generator.cc:596-693)."""
    vc = _f32(v_cond)
    H, W, _ = vc.shape
    vu = _f32(v_unc) if v_unc is not None else vc
    vi = _f32(v_img) if v_img is not None else vc
    out = np.empty_like(vc)
    lib().orc_cfg(_fp(vc), _fp(vu), _fp(vi), H, W, form, norm, cfg_scale, icfg, step, _fp(out))
    return out


def euler(img, v, dt):
    img = _f32(img).copy()
    lib().orc_euler(_fp(img), _fp(_f32(v)), img.size, dt)
    return img


# ---------------------------------------------------------------------------
# the reference's own CPU code (fixture generation and pinning only)
# ---- the image path ---------------------------------------------------------
# Weight dicts use the checkpoint's names and layouts: patch_w [C][3p^2],
# patch_b [C], dense_w [LLM][C m^2], dense_b [LLM]; conv1_w [hid][in/4][3][3],
# conv1_b, conv2_w [192][hid/4][3][3], conv2_b; tstep_w0 [H][dim], tstep_b0,
# tstep_w2 [H][H], tstep_b2 (and nscale_* the same, optional).

def patchify_cf(img_hwc, p=16):
    H, W, c = img_hwc.shape
    img = _f32(img_hwc)
    out = np.empty(((H // p) * (W // p), c * p * p), np.float32)
    lib().orc_patchify_cf(_fp(img), c, H, W, p, _fp(out))
    return out


def gelu_erf(x):
    y = _f32(x).copy()
    lib().orc_gelu_erf(_fp(y), y.size)
    return y


def vision_embed(px, w, gh, gw, p=16, merge=2, theta=1e4):
    pw, pb, dw, db = (_f32(w[k]) for k in ("patch_w", "patch_b", "dense_w", "dense_b"))
    C_, LLM = pw.shape[0], dw.shape[0]
    out = np.empty(((gh // merge) * (gw // merge), LLM), np.float32)
    lib().orc_vision_embed(_fp(_f32(px)), _fp(pw), _fp(pb), _fp(dw), _fp(db), gh, gw, p, C_,
                           LLM, merge, theta, _fp(out))
    return out


def conv_decoder_hwc(x, w, th, tw):
    """x [th*tw][in_ch] (a [th][tw][in_ch] map) -> [32 th][32 tw][3]."""
    c1w, c1b, c2w, c2b = (_f32(w[k]) for k in ("conv1_w", "conv1_b", "conv2_w", "conv2_b"))
    in_ch, hid = x.shape[-1], c1w.shape[0]
    out = np.empty((32 * th, 32 * tw, 3), np.float32)
    lib().orc_conv_decoder_hwc(_fp(_f32(x)), _fp(c1w), _fp(c1b), _fp(c2w), _fp(c2b), in_ch, th,
                               tw, hid, _fp(out))
    return out


def timestep_row(t, ratio, w):
    w0, b0, w2, b2 = (_f32(w[k]) for k in ("tstep_w0", "tstep_b0", "tstep_w2", "tstep_b2"))
    H, dim = w0.shape
    ns = [w.get(k) for k in ("nscale_w0", "nscale_b0", "nscale_w2", "nscale_b2")]
    ns = [_f32(a) if a is not None else None for a in ns]
    out = np.empty(H, np.float32)
    lib().orc_timestep_row(t, ratio, dim, H, _fp(w0), _fp(b0), _fp(w2), _fp(b2),
                           *(_fp(a) for a in ns), _fp(out))
    return out


def thw_indexes(ids, img_id, img_ctx_id, grids):
    """Prompt::thw_indexes (src/u15-prompt.cc:349-386), restated loop by loop."""
    n = len(ids)
    t, h, w = np.zeros(n, np.int32), np.zeros(n, np.int32), np.zeros(n, np.int32)
    cum = 0
    for i in range(n):
        shift = 1 if (i > 0 and ids[i - 1] == img_id) else 0
        cum += shift + (0 if ids[i] == img_ctx_id else 1)
        t[i] = cum - 1
    img, seen = 0, 0
    for i in range(n):
        if ids[i] != img_ctx_id:
            continue
        while img < len(grids) and seen >= (grids[img][0] // 2) * (grids[img][1] // 2):
            img, seen = img + 1, 0
        if img >= len(grids):
            break
        tw = grids[img][1] // 2
        h[i], w[i] = seen // tw, seen % tw
        seen += 1
    return t, h, w


# ---------------------------------------------------------------------------

_ref = None


def ref_available() -> bool:
    return os.path.exists(REF_SO)


def ref():
    """The reference's u15::ref through oracle/ref_shim.cc."""
    global _ref
    if _ref is None:
        L = C.CDLL(REF_SO)
        L.refx_rms_norm.argtypes = [_f32p, _f32p, C.c_float, C.c_long, C.c_long, _f32p]
        L.refx_linear.argtypes = [_f32p, _f32p, _f32p, C.c_long, C.c_long, C.c_long, _f32p]
        L.refx_rope_inv_freq.argtypes = [C.c_int, C.c_double, _f32p]
        L.refx_split_rope_project.argtypes = [
            _f32p, _f32p, _f32p, _f32p, _i32p, _i32p, _i32p, C.c_long, C.c_long, C.c_int,
            C.c_int, C.c_double, C.c_double, C.c_double, _f32p]
        L.refx_attention.argtypes = [_f32p, _f32p, _f32p, _f32p] + [C.c_long] * 5 + [_f32p]
        L.refx_block_causal_mask.argtypes = [_i32p, C.c_long, _f32p]
        L.refx_decoder_layer.argtypes = [
            _f32p, C.POINTER(_f32p)] + [C.c_long] * 5 + [C.c_double] * 3 + [
            _i32p, _i32p, _i32p, _f32p, C.c_long, _f32p]
        L.refx_time_schedule.argtypes = [C.c_int, C.c_double, _f32p]
        L.refx_optimized_scale.argtypes = [_f32p, _f32p, C.c_long]
        L.refx_optimized_scale.restype = C.c_double
        L.refx_vision_embed.argtypes = [_f32p] * 5 + [C.c_int] * 6 + [C.c_double, _f32p]
        L.refx_conv_decoder.argtypes = [_f32p] * 5 + [C.c_int] * 4 + [_f32p]
        L.refx_patchify_channel_first_hwc.argtypes = [_f32p] + [C.c_int] * 4 + [_f32p]
        L.refx_timestep_sinusoid.argtypes = [C.c_double, C.c_int, C.c_double, _f32p]
        L.refx_gelu_erf.argtypes = [_f32p, C.c_long]
        _ref = L
    return _ref
