"""Checkpoint binding on the GPU: the affine-pack dequantization bit for bit
against its host restatement, and a whole synthetic checkpoint in the
reference's tensor naming (src/u15-weights.cc:361-430, 534-578) -- some
matrices w8g64 / w4g32 packed, others bf16 or f32 -- loaded through
u15b200.checkpoint into a model and an image path that must equal the same
weights bound directly."""
import numpy as np
import pytest

from ckpt_util import bf16_bits, dequant, from_bf16_bits, quantize
from gpu_util import bf16_round, dev_bf16, dev_f32, dev_i32, host, randn, torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("bits,group,sdt", [(8, 64, "BF16"), (8, 32, "F16"), (4, 64, "F16"),
                                            (4, 32, "BF16")])
def test_dequant_affine_bit_exact(bits, group, sdt):
    import u15b200
    from u15b200 import _lib as L
    rng = np.random.default_rng(bits * 100 + group)
    N, K = 96, 512
    w = rng.normal(0, 0.02, (N, K)).astype(np.float32)
    codes, s, b, c = quantize(w, group, bits, sdt)
    tod = lambda a: torch.from_numpy(a.view(np.int16) if a.dtype == np.uint16 else a).cuda()  # noqa
    cd, sd, bd = tod(codes.view(np.int32)), tod(s), tod(b)
    out = torch.empty(N, K, dtype=torch.bfloat16, device="cuda")
    dt = L.DT_BF16 if sdt == "BF16" else L.DT_F16
    L.check(u15b200.lib().u15c_dequant_affine(None, cd.data_ptr(), sd.data_ptr(), bd.data_ptr(),
                                              dt, N, K, bits, group, out.data_ptr()))
    torch.cuda.synchronize()
    assert np.array_equal(host(out), dequant(c, s, b, group, sdt))


def test_dequant_refuses_unclosed_packs():
    import u15b200
    from u15b200 import _lib as L
    z = torch.zeros(64, dtype=torch.int32, device="cuda")
    out = torch.empty(4, 64, dtype=torch.bfloat16, device="cuda")
    for bits, group in ((2, 64), (8, 16), (8, 48)):
        rc = u15b200.lib().u15c_dequant_affine(None, z.data_ptr(), z.data_ptr(), z.data_ptr(),
                                               L.DT_F16, 4, 64, bits, group, out.data_ptr())
        assert rc == L.EINVAL


SMALL = dict(n_layers=2, hidden=512, heads=4, kv_heads=1, head_dim=128, inter=1024, n_experts=2)
IMG_CFG = dict(vision_hidden=64, llm_hidden=512, patch=16, merge=2, head_hidden=64, freq_dim=256,
               noise_scale_embedding=1, vision_theta=1e4)


def synthetic_checkpoint(path):
    """(file, direct): the checkpoint and, per tensor, the exact f32 values
    the device must end up with."""
    from u15b200.checkpoint import IMAGE_NAMES, layer_names, write_safetensors
    rng = np.random.default_rng(31)
    H, I, QD, KD = 512, 1024, 512, 128
    shapes = {"input_layernorm": (H,), "post_attention_layernorm": (H,), "q_proj": (QD, H),
              "k_proj": (KD, H), "v_proj": (KD, H), "o_proj": (H, QD), "q_norm": (64,),
              "k_norm": (64,), "q_norm_hw": (64,), "k_norm_hw": (64,), "gate_proj": (I, H),
              "up_proj": (I, H), "down_proj": (H, I)}
    packs = {("q_proj", 0): (8, 64, "F16"), ("gate_proj", 0): (8, 64, "F16"),
             ("down_proj", 1): (8, 64, "F16"), ("o_proj", 1): (4, 32, "BF16")}
    t, direct = {}, {}
    for li in range(2):
        for e in range(2):
            names = layer_names(li, e)
            for k, shp in shapes.items():
                is_norm = len(shp) == 1
                w = (rng.normal(1, 0.2, shp) if is_norm else rng.normal(0, 0.02, shp)).astype(
                    np.float32)
                if (k, e) in packs and li == 1:
                    bits, group, sdt = packs[(k, e)]
                    codes, s, b, c = quantize(w, group, bits, sdt)
                    base = names[k]
                    t[base + ".weight"] = codes
                    t[base + ".scales"] = ("BF16", s) if sdt == "BF16" else s
                    t[base + ".biases"] = ("BF16", b) if sdt == "BF16" else b
                    direct[(li, e, k)] = dequant(c, s, b, group, sdt)
                elif (li + e) % 2 == 0:
                    key = names[k] if is_norm else names[k] + ".weight"
                    t[key] = w
                    direct[(li, e, k)] = w
                else:
                    key = names[k] if is_norm else names[k] + ".weight"
                    t[key] = ("BF16", bf16_bits(w))
                    direct[(li, e, k)] = from_bf16_bits(bf16_bits(w))
    for k, e in (("language_model.model.norm.weight", 0),
                 ("language_model.model.norm_mot_gen.weight", 1)):
        v = rng.normal(1, 0.1, H).astype(np.float32)
        t[k] = v
        direct[("final", e)] = v
    emb = rng.normal(0, 1, (300, H)).astype(np.float32)
    t["language_model.model.embed_tokens.weight"] = ("BF16", bf16_bits(emb))
    direct["embed"] = from_bf16_bits(bf16_bits(emb))
    C, L, hid, D = 64, 512, 64, 256
    ishapes = {"patch_w": (C, 3, 16, 16), "patch_b": (C,), "dense_w": (L, C, 2, 2),
               "dense_b": (L,), "conv1_w": (hid, L // 4, 3, 3), "conv1_b": (hid,),
               "conv2_w": (192, hid // 4, 3, 3), "conv2_b": (192,), "tstep_w0": (L, D),
               "tstep_b0": (L,), "tstep_w2": (L, L), "tstep_b2": (L,), "nscale_w0": (L, D),
               "nscale_b0": (L,), "nscale_w2": (L, L), "nscale_b2": (L,)}
    for (k, e), name in IMAGE_NAMES.items():
        w = rng.normal(0, 0.05, ishapes[k]).astype(np.float32)
        if k.startswith("conv"):   # the pixel head ships bf16
            t[name] = ("BF16", bf16_bits(w))
            w = from_bf16_bits(bf16_bits(w))
        else:
            t[name] = w
        direct[("img", k, e)] = w
    f = str(path / "model-00001-of-00001.safetensors")
    write_safetensors(f, t)
    return f, direct


def test_load_synthetic_checkpoint(tmp_path):
    import u15b200
    from u15b200.checkpoint import SafeTensors, bind_image, bind_model
    f, direct = synthetic_checkpoint(tmp_path)
    st = SafeTensors(str(tmp_path))
    ml = u15b200.Model(**SMALL)
    table = bind_model(ml, st)
    il = u15b200.ImagePath(**IMG_CFG)
    bind_image(il, st)
    md = u15b200.Model(**SMALL)
    for key, v in direct.items():
        if isinstance(key, str) or key[0] in ("final", "img"):
            continue
        md.bind(key[0], key[1], key[2], np.ascontiguousarray(v))
    md.bind(0, 0, "final_norm", direct[("final", 0)])
    md.bind(0, 1, "final_norm", direct[("final", 1)])
    idd = u15b200.ImagePath(**IMG_CFG)
    for key, v in direct.items():
        if not isinstance(key, str) and key[0] == "img":
            idd.bind(key[1], np.ascontiguousarray(v.reshape(v.shape[0], -1)) if v.ndim > 1
                     else v, expert=key[2])
    torch.cuda.synchronize()
    assert np.array_equal(host(table), direct["embed"])
    # the same layer pass through both models
    T = 96
    x = bf16_round(randn((T, 512), 32))
    pos = [dev_i32(np.arange(T) % 7), dev_i32(np.arange(T) // 12), dev_i32(np.arange(T) % 12)]
    segs = [(0, 32, 0), (32, T, 1)]
    outs = []
    for m in (ml, md):
        kv = m.make_cache(T)
        xd = dev_bf16(x)
        m.forward(xd, kv, 0, T, *pos, segments=segs)
        m.final_norm(xd, 1)
        torch.cuda.synchronize()
        outs.append(host(xd))
    assert np.array_equal(outs[0], outs[1])
    # and the image path: embed, timestep row, decode
    img = randn((64, 64, 3), 33)
    res = []
    for im in (il, idd):
        px = im.patchify(dev_f32(img))
        e = im.embed(px, 4, 4, gen=True)
        r = im.timestep_row(0.4, 0.3)
        d = im.decode(dev_bf16(bf16_round(randn((4, 512), 34))), 2, 2)
        torch.cuda.synchronize()
        res.append((host(e), host(r), host(d)))
    for a, b in zip(*res):
        assert np.array_equal(a, b)
