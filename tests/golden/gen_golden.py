"""Generate the golden fixtures that pin the CPU restatement (oracle/).

Run in a checkout that has the reference tree: it calls the reference's own
CPU implementation (src/u15-ref.cc, compiled unchanged by oracle/Makefile
into oracle/_ref/libu15ref.so) on seeded inputs and stores inputs and outputs
as .npz files beside this script. The fixtures are committed; the tests read
them and never need the reference at run time.

    make -C oracle all && python tests/golden/gen_golden.py

Dimensions: the reference's own golden-test geometry (hidden 64, 4 query /
2 kv heads of 32, intermediate 128; tests/u15-ref-test.cc:82-83 in the
reference), plus a full-head-width case (head_dim 128, positions out to the
4416-token cache) where the theta=5e6 ladder's precision matters.
"""
from __future__ import annotations

import ctypes as C
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", ".."))
from oracle import oracle as O  # noqa: E402

f32p = C.POINTER(C.c_float)
i32p = C.POINTER(C.c_int)


def fp(a):
    return a.ctypes.data_as(f32p) if a is not None else None


def ip(a):
    return a.ctypes.data_as(i32p)


def layer_weights(rng, hid, nh, kv, hd, inter):
    """One expert-layer in the reference's LayerWeights order. Projections
    N(0, 0.02) as BASELINE states; norm gains N(1, 0.2) so that a skipped
    gain is visible (tests/u15-kernels-test.cc:136-144 in the reference)."""
    g = lambda *s: rng.normal(0.0, 0.02, s).astype(np.float32)  # noqa: E731
    n = lambda *s: rng.normal(1.0, 0.2, s).astype(np.float32)  # noqa: E731
    return {
        "input_layernorm": n(hid), "post_attention_layernorm": n(hid),
        "q_proj": g(nh * hd, hid), "k_proj": g(kv * hd, hid),
        "v_proj": g(kv * hd, hid), "o_proj": g(hid, nh * hd),
        "q_norm": n(hd // 2), "k_norm": n(hd // 2),
        "q_norm_hw": n(hd // 2), "k_norm_hw": n(hd // 2),
        "gate_proj": g(inter, hid), "up_proj": g(inter, hid),
        "down_proj": g(hid, inter),
    }


def ref_decoder_layer(x, w, dims, pt, ph, pw, mask):
    R = O.ref()
    arr = (f32p * 13)(*[fp(w[k]) for k in O.EXPERT_KEYS])
    out = np.empty_like(x)
    R.refx_decoder_layer(fp(x), arr, dims["hidden"], dims["heads"], dims["kv_heads"],
                         dims["head_dim"], dims["inter"], 1e-6, 5e6, 1e4, ip(pt), ip(ph),
                         ip(pw), fp(mask), x.shape[0], fp(out))
    return out


def ref_split_rope_project(x, wp, wn, wnh, pt, ph, pw, heads, hd):
    R = O.ref()
    T, hid = x.shape
    out = np.empty((heads, T, hd), np.float32)
    R.refx_split_rope_project(fp(x), fp(wp), fp(wn), fp(wnh), ip(pt), ip(ph), ip(pw), T,
                              hid, heads, hd, 5e6, 1e4, 1e-6, fp(out))
    return out


def ref_attention(q, k, v, mask):
    R = O.ref()
    hq, tq, d = q.shape
    hkv, tk, _ = k.shape
    out = np.empty((tq, hq * d), np.float32)
    R.refx_attention(fp(q), fp(k), fp(v), fp(mask), hq, hkv, tq, tk, d, fp(out))
    return out


def ref_block_causal_mask(t):
    R = O.ref()
    m = np.empty((t.size, t.size), np.float32)
    R.refx_block_causal_mask(ip(t), t.size, fp(m))
    return m


def main():
    if not O.ref_available():
        raise SystemExit("build the reference first: make -C oracle all")
    R = O.ref()
    rng = np.random.default_rng(20261201)
    fx = {}

    # ---- primitives -----------------------------------------------------
    x = rng.normal(0, 1, (7, 64)).astype(np.float32)
    w = rng.normal(1, 0.2, 64).astype(np.float32)
    y = np.empty_like(x)
    R.refx_rms_norm(fp(x), fp(w), 1e-6, 7, 64, fp(y))
    fx.update({"rms.x": x, "rms.w": w, "rms.y": y})

    W = rng.normal(0, 0.02, (48, 64)).astype(np.float32)
    b = rng.normal(0, 0.1, 48).astype(np.float32)
    y = np.empty((7, 48), np.float32)
    R.refx_linear(fp(x), fp(W), fp(b), 7, 64, 48, fp(y))
    fx.update({"lin.w": W, "lin.b": b, "lin.y": y})

    for dim, th, key in ((16, 5e6, "t"), (8, 1e4, "hw"), (64, 5e6, "t128"),
                         (32, 1e4, "hw128")):
        f = np.empty(dim // 2, np.float32)
        R.refx_rope_inv_freq(dim, th, fp(f))
        fx["inv_freq." + key] = f

    # ---- split rope projection, toy (hd 32) and full width (hd 128) -----
    for tag, (T, hid, heads, hd, tmax) in {
            "toy": (12, 64, 4, 32, 12), "hd128": (24, 128, 4, 128, 4416)}.items():
        xs = rng.normal(0, 1, (T, hid)).astype(np.float32)
        wp = rng.normal(0, 0.02, (heads * hd, hid)).astype(np.float32)
        wn = rng.normal(1, 0.2, hd // 2).astype(np.float32)
        wnh = rng.normal(1, 0.2, hd // 2).astype(np.float32)
        pt = np.sort(rng.integers(0, tmax, T)).astype(np.int32)
        ph = rng.integers(0, 64, T).astype(np.int32)
        pw = rng.integers(0, 64, T).astype(np.int32)
        out = ref_split_rope_project(xs, wp, wn, wnh, pt, ph, pw, heads, hd)
        fx.update({f"srp.{tag}.x": xs, f"srp.{tag}.w": wp, f"srp.{tag}.wn": wn,
                   f"srp.{tag}.wnh": wnh, f"srp.{tag}.pt": pt, f"srp.{tag}.ph": ph,
                   f"srp.{tag}.pw": pw, f"srp.{tag}.out": out})

    # ---- attention: GQA unmasked, causal and block-causal ---------------
    hq, hkv, T, d = 4, 2, 11, 32
    q = rng.normal(0, 1, (hq, T, d)).astype(np.float32)
    k = rng.normal(0, 1, (hkv, T, d)).astype(np.float32)
    v = rng.normal(0, 1, (hkv, T, d)).astype(np.float32)
    tidx = np.array([0, 1, 2, 3, 3, 3, 3, 3, 3, 4, 5], np.int32)  # kernels-test:612
    causal_t = np.arange(T, dtype=np.int32)
    fx.update({"att.q": q, "att.k": k, "att.v": v, "att.t_block": tidx,
               "att.bidir": ref_attention(q, k, v, None),
               "att.mask_causal": ref_block_causal_mask(causal_t),
               "att.mask_block": ref_block_causal_mask(tidx)})
    fx["att.causal"] = ref_attention(q, k, v, fx["att.mask_causal"])
    fx["att.block"] = ref_attention(q, k, v, fx["att.mask_block"])

    # ---- decoder layer, both experts (tests/u15-layer0-test.cc geometry) --
    dims = dict(hidden=64, heads=4, kv_heads=2, head_dim=32, inter=128)
    for e in ("und", "gen"):
        wts = layer_weights(rng, 64, 4, 2, 32, 128)
        for kname, arr in wts.items():
            fx[f"dl.{e}.{kname}"] = arr
    # und: causal over 9 text tokens (distinct t, h = w = 0)
    xu = rng.normal(0, 1, (9, 64)).astype(np.float32)
    pt = np.arange(9, dtype=np.int32)
    z = np.zeros(9, np.int32)
    wu = {k2: fx[f"dl.und.{k2}"] for k2 in O.EXPERT_KEYS}
    fx.update({"dl.und.x": xu, "dl.und.pt": pt, "dl.und.ph": z, "dl.und.pw": z,
               "dl.und.out": ref_decoder_layer(xu, wu, dims, pt, z, z,
                                               ref_block_causal_mask(pt))})
    # gen: bidirectional over a 2x3 image block at one t
    xg = rng.normal(0, 1, (6, 64)).astype(np.float32)
    pt = np.full(6, 9, np.int32)
    ph = np.array([0, 0, 0, 1, 1, 1], np.int32)
    pw = np.array([0, 1, 2, 0, 1, 2], np.int32)
    wg = {k2: fx[f"dl.gen.{k2}"] for k2 in O.EXPERT_KEYS}
    fx.update({"dl.gen.x": xg, "dl.gen.pt": pt, "dl.gen.ph": ph, "dl.gen.pw": pw,
               "dl.gen.out": ref_decoder_layer(xg, wg, dims, pt, ph, pw, None)})
    # the same 15 tokens as ONE sequence through each expert, bidirectional:
    # pins the joint layer's attention composition (oracle/u15_oracle.c)
    xj = np.concatenate([xu, xg])
    pj = [np.concatenate([np.arange(9), np.full(6, 9)]).astype(np.int32),
          np.concatenate([z, ph]).astype(np.int32),
          np.concatenate([z, pw]).astype(np.int32)]
    fx.update({"dl.joint.x": xj, "dl.joint.pt": pj[0], "dl.joint.ph": pj[1],
               "dl.joint.pw": pj[2],
               "dl.joint.out_und": ref_decoder_layer(xj, wu, dims, *pj, None),
               "dl.joint.out_gen": ref_decoder_layer(xj, wg, dims, *pj, None)})

    # ---- the image path (src/u15-ref.cc vision_embed, conv_decoder) ------
    img = rng.uniform(-1, 1, (32, 48, 3)).astype(np.float32)     # [H][W][3]
    pc = np.empty((6, 3 * 16 * 16), np.float32)
    R.refx_patchify_channel_first_hwc(fp(img), 3, 32, 48, 16, fp(pc))
    fx.update({"img.hwc": img, "img.patch_cf": pc})
    g = np.linspace(-6, 6, 97).astype(np.float32)
    gy = g.copy()
    R.refx_gelu_erf(fp(gy), gy.size)
    fx.update({"gelu.x": g, "gelu.y": gy})
    gh, gw, Cv, LLM = 4, 6, 32, 48
    ve = {"px": rng.normal(0, 1, (gh * gw, 768)).astype(np.float32),
          "patch_w": rng.normal(0, 0.03, (Cv, 768)).astype(np.float32),
          "patch_b": rng.normal(0, 0.1, Cv).astype(np.float32),
          "dense_w": rng.normal(0, 0.05, (LLM, Cv * 4)).astype(np.float32),
          "dense_b": rng.normal(0, 0.1, LLM).astype(np.float32)}
    vo = np.empty(((gh // 2) * (gw // 2), LLM), np.float32)
    R.refx_vision_embed(fp(ve["px"]), fp(ve["patch_w"]), fp(ve["patch_b"]), fp(ve["dense_w"]),
                        fp(ve["dense_b"]), gh, gw, 16, Cv, LLM, 2, 1e4, fp(vo))
    fx.update({f"ve.{k}": v for k, v in ve.items()})
    fx["ve.out"] = vo
    in_ch, th, tw, hid = 64, 2, 3, 32
    cd = {"x_chw": rng.normal(0, 1, (in_ch, th, tw)).astype(np.float32),
          "conv1_w": rng.normal(0, 0.05, (hid, in_ch // 4, 3, 3)).astype(np.float32),
          "conv1_b": rng.normal(0, 0.1, hid).astype(np.float32),
          "conv2_w": rng.normal(0, 0.05, (192, hid // 4, 3, 3)).astype(np.float32),
          "conv2_b": rng.normal(0, 0.1, 192).astype(np.float32)}
    co = np.empty((3, 32 * th, 32 * tw), np.float32)
    R.refx_conv_decoder(fp(cd["x_chw"]), fp(cd["conv1_w"]), fp(cd["conv1_b"]),
                        fp(cd["conv2_w"]), fp(cd["conv2_b"]), in_ch, th, tw, hid, fp(co))
    fx.update({f"cd.{k}": v for k, v in cd.items()})
    fx["cd.out_chw"] = co
    sn = np.empty(256, np.float32)
    R.refx_timestep_sinusoid(0.37, 256, 10000.0, fp(sn))
    fx["tsin.t037.d256"] = sn

    # ---- sampling ---------------------------------------------------------
    ts = np.empty(21, np.float32)
    R.refx_time_schedule(20, 3.0, fp(ts))
    fx["sched.n20.shift3"] = ts

    path = os.path.join(HERE, "ref_goldens.npz")
    np.savez_compressed(path, **fx)
    print(f"wrote {path}: {len(fx)} arrays, {os.path.getsize(path)} bytes")


if __name__ == "__main__":
    main()
