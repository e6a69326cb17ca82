"""The denoise step on the GPU against the CPU restatement of
Generator::generate's step body (src/u15-generator.cc:582-705): velocity,
the four CFG forms with the three renorms, the Euler update, the pixel
packing, and a short end-to-end loop (three CFG branches, prefills into
paged caches, two flow-matching steps) through a small model."""
import numpy as np
import pytest

from gpu_util import bf16_round, dev_bf16, dev_f32, dev_i32, host, randn, rel_l2, torch
from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lib():
    import u15b200
    u15b200.CudaOps(0)
    return u15b200.lib()


def _p(t):
    import ctypes as C
    return None if t is None else C.c_void_p(t.data_ptr())


def _st():
    import ctypes as C
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def test_velocity_and_euler_exact(lib):
    H, W = 64, 96
    xp, img, v = (randn((H, W, 3), s) for s in (1, 2, 3))
    n = H * W * 3
    out = torch.empty(H, W, 3, device="cuda")
    # keep every device input referenced while the library uses its pointer
    xp_d, img_d, v_d = dev_f32(xp), dev_f32(img), dev_f32(v)
    assert lib.u15c_velocity(_st(), _p(xp_d), _p(img_d), _p(out), n, 0.37) == 0
    assert np.array_equal(host(out), O.velocity(xp, img, 0.37))
    d = dev_f32(img)
    assert lib.u15c_euler(_st(), _p(d), _p(v_d), n, -0.061) == 0
    assert np.array_equal(host(d), O.euler(img, v, -0.061))


FORMS = [(O.CFG_IMG, O.NORM_NONE), (O.CFG_UNC, O.NORM_NONE), (O.CFG_BOTH, O.NORM_NONE),
         (O.CFG_UNC, O.NORM_ZERO_STAR), (O.CFG_UNC, O.NORM_GLOBAL), (O.CFG_BOTH, O.NORM_GLOBAL),
         (O.CFG_IMG, O.NORM_CHANNEL), (O.CFG_BOTH, O.NORM_CHANNEL), (O.CFG_NONE, O.NORM_NONE)]


@pytest.mark.parametrize("form,norm", FORMS)
@pytest.mark.parametrize("step", [0, 3])
def test_cfg_forms(lib, form, norm, step):
    H, W = 64, 96
    vc, vu, vi = randn((H, W, 3), 4), randn((H, W, 3), 5), randn((H, W, 3), 6)
    ws = torch.empty(lib.u15c_cfg_workspace_bytes(), dtype=torch.uint8, device="cuda")
    out = torch.empty(H, W, 3, device="cuda")
    vc_d, vu_d, vi_d = dev_f32(vc), dev_f32(vu), dev_f32(vi)
    rc = lib.u15c_cfg_combine(_st(), _p(vc_d), _p(vu_d), _p(vi_d), _p(out),
                              H, W, form, norm, 4.0, 1.5, step, _p(ws))
    assert rc == 0
    ref = O.cfg(vc, vu, vi, form, norm, 4.0, 1.5, step)
    got = host(out)
    if norm in (O.NORM_NONE,):
        assert np.array_equal(got, ref)            # elementwise fp64: identical
    else:
        # fp64 reductions in another order: equal to ~1 ulp
        assert np.abs(got - ref).max() <= 2e-6 * max(np.abs(ref).max(), 1e-30)


def test_pixel_packing(lib):
    H, W = 64, 96
    img = bf16_round(randn((H, W, 3), 7))
    rows = torch.empty((H // 32) * (W // 32), 3072, dtype=torch.bfloat16, device="cuda")
    img_d = dev_f32(img)
    assert lib.u15c_patchify(_st(), _p(img_d), _p(rows), H, W) == 0
    ref = img.reshape(H // 32, 32, W // 32, 32, 3).transpose(0, 2, 1, 3, 4).reshape(-1, 3072)
    assert np.array_equal(host(rows), ref)
    back = torch.empty(H, W, 3, device="cuda")
    assert lib.u15c_unpatchify(_st(), _p(rows), _p(back), H, W) == 0
    assert np.array_equal(host(back), img)


def test_short_denoise_three_branches():
    """An edit-style run: cond + image-conditional + unconditional branches
    (img_cfg != 1 and != cfg), block-causal prefill for the branches with a
    reference image, two steps, against the loop restated on the CPU."""
    import u15b200
    from u15b200 import _lib as L
    from u15b200.generator import Branch, Generator, LinearImagePath, time_schedule
    from test_gpu_layer import SMALL, build, dims_of

    cfg = dict(SMALL)
    m, Wts = build(cfg, 300)
    hidden = cfg["hidden"]
    H = W = 128
    th, tw = H // 32, W // 32
    Ltok = th * tw
    rng = np.random.default_rng(8)

    def prefix(n_text, n_img):
        n = n_text + n_img
        x = bf16_round(rng.normal(0, 1, (n, hidden)).astype(np.float32))
        if n_img:
            t = np.concatenate([np.arange(n_text), np.full(n_img, n_text)]).astype(np.int32)
            gh = int(np.sqrt(n_img))
            h = np.concatenate([np.zeros(n_text), np.arange(n_img) // gh]).astype(np.int32)
            w = np.concatenate([np.zeros(n_text), np.arange(n_img) % gh]).astype(np.int32)
        else:
            t = np.arange(n).astype(np.int32)
            h = w = np.zeros(n, np.int32)
        return x, t, h, w

    specs = [("cond", prefix(10, 16), True), ("img_cond", prefix(3, 16), True),
             ("uncond", prefix(5, 0), False)]
    branches = [Branch(name, dev_bf16(x), t, h, w, block_causal=bc)
                for name, (x, t, h, w), bc in specs]
    image = LinearImagePath(hidden, seed=3)
    gen = Generator(m, image)
    noise = randn((H, W, 3), 9)
    steps, shift, cfgs, icfg, t_eps = 2, 3.0, 4.0, 1.5, 0.05
    img = gen.generate(branches, H, W, steps=steps, shift=shift, cfg=cfgs, icfg=icfg,
                       form=L.CFG_BOTH, i_img=1, i_unc=2, t_eps=t_eps,
                       init_noise=torch.from_numpy(noise))
    torch.cuda.synchronize()

    # ---- the same loop on the CPU ----
    D = dims_of(cfg)
    w_in, w_out = host(image.w_in), host(image.w_out)
    kv = []
    for _, (x, t, h, w), bc in specs:
        n = x.shape[0]
        mode = O.BLOCK_CAUSAL if bc else O.CAUSAL
        ti = t if bc else None
        ks, vs = [], []
        cur = x
        for li in range(cfg["n_layers"]):
            cur, kn, vn = O.mot_layer(cur, [(0, n, 0)], Wts[li], D, t, h, w, mode=mode,
                                      t_index=ti)
            ks.append(kn)
            vs.append(vn)
        kv.append((ks, vs, int(t.max()) + 1, n))
    ts = time_schedule(steps, shift)
    z = noise.copy()
    for step in range(steps):
        t, tn = ts[step], ts[step + 1]
        rows = bf16_round(z.reshape(th, 32, tw, 32, 3).transpose(0, 2, 1, 3, 4).reshape(-1, 3072))
        emb = bf16_round(O.linear(rows, w_in))
        emb = bf16_round(emb + host(image.timestep_row(t))[None])
        vel = []
        for ks, vs, tpos, npre in kv:
            pt = np.full(Ltok, tpos, np.int32)
            ph = (np.arange(Ltok) // tw).astype(np.int32)
            pw = (np.arange(Ltok) % tw).astype(np.int32)
            hcur = emb
            for li in range(cfg["n_layers"]):
                hcur, _, _ = O.mot_layer(hcur, [(0, Ltok, 1)], Wts[li], D, pt, ph, pw,
                                         k_prefix=ks[li], v_prefix=vs[li])
            hn = O.rms_norm(hcur, np.ones(hidden, np.float32))
            xo = bf16_round(O.linear(hn, w_out))
            xp = xo.reshape(th, tw, 32, 32, 3).transpose(0, 2, 1, 3, 4).reshape(H, W, 3)
            vel.append(O.velocity(xp, z, max(1 - t, t_eps)))
        comb = O.cfg(vel[0], vel[2], vel[1], O.CFG_BOTH, O.NORM_NONE, cfgs, icfg, step)
        z = O.euler(z, comb, tn - t)
    got = host(img)
    assert rel_l2(got - noise, z - noise) < 5e-2
    assert np.isfinite(got).all()
    assert isinstance(m, u15b200.Model)


def test_denoise_with_device_image_path():
    """Two steps of the loop with the device image path (patch embedder,
    timestep + noise-scale row, pixel head) against the same steps restated on
    the CPU from the pinned restatements (vision_embed, conv_decoder,
    timestep_row)."""
    import u15b200
    from u15b200 import _lib as L
    from u15b200.generator import Branch, DeviceImagePath, Generator, time_schedule
    from test_gpu_image import make
    from test_gpu_layer import SMALL, build, dims_of

    cfg = dict(SMALL)
    m, Wts = build(cfg, 400)
    hidden = cfg["hidden"]
    icfg = dict(vision_hidden=64, llm_hidden=hidden, patch=16, merge=2, head_hidden=64,
                freq_dim=256, noise_scale_embedding=1, vision_theta=1e4)
    im, Wv, Hw = make(icfg, 12)
    H = W = 128
    th, tw = H // 32, W // 32
    Ltok = th * tw
    rng = np.random.default_rng(13)
    n_text = 10
    px0 = bf16_round(rng.normal(0, 1, (n_text, hidden)).astype(np.float32))
    t_pre = np.arange(n_text).astype(np.int32)
    z0 = np.zeros(n_text, np.int32)
    branches = [Branch("cond", dev_bf16(px0), t_pre, z0, z0)]
    gen = Generator(m, DeviceImagePath(im))
    noise = randn((H, W, 3), 14)
    steps, shift, t_eps, nscale = 2, 3.0, 0.05, 4.0
    img = gen.generate(branches, H, W, steps=steps, shift=shift, form=L.CFG_NONE, t_eps=t_eps,
                       init_noise=torch.from_numpy(noise), noise_scale=nscale)
    torch.cuda.synchronize()

    # ---- the same loop on the CPU ----
    D = dims_of(cfg)
    ks, vs = [], []
    cur = px0
    for li in range(cfg["n_layers"]):
        cur, kn, vn = O.mot_layer(cur, [(0, n_text, 0)], Wts[li], D, t_pre, z0, z0,
                                  mode=O.CAUSAL)
        ks.append(kn)
        vs.append(vn)
    ts = time_schedule(steps, shift)
    z = noise.copy()
    ratio = nscale / 16.0
    for step in range(steps):
        t, tn = ts[step], ts[step + 1]
        px = bf16_round(O.patchify_cf(z, 16))
        emb = bf16_round(O.vision_embed(px, Wv[1], H // 16, W // 16))
        emb = bf16_round(emb + bf16_round(O.timestep_row(t, ratio, Hw))[None])
        pt = np.full(Ltok, n_text, np.int32)
        ph = (np.arange(Ltok) // tw).astype(np.int32)
        pw = (np.arange(Ltok) % tw).astype(np.int32)
        hcur = emb
        for li in range(cfg["n_layers"]):
            hcur, _, _ = O.mot_layer(hcur, [(0, Ltok, 1)], Wts[li], D, pt, ph, pw,
                                     k_prefix=ks[li], v_prefix=vs[li])
        hn = bf16_round(O.rms_norm(hcur, np.ones(hidden, np.float32)))
        xp = O.conv_decoder_hwc(hn, Hw, th, tw)
        z = O.euler(z, O.velocity(xp, z, max(1 - t, t_eps)), tn - t)
    got = host(img)
    assert np.isfinite(got).all()
    assert rel_l2(got - noise, z - noise) < 5e-2
    assert isinstance(im, u15b200.ImagePath)


def test_start_image_is_the_reference_draw(tmp_path):
    """The generator's start image on the device: the reference's seeded draw
    (std::mt19937_64 + std::normal_distribution<float>) scaled by
    GenConfig::init_noise_scale of the image's token count, bit for bit
    against the CPU checker; the init_noise file is taken as is, and one of
    the wrong size is refused (src/u15-generator.cc:400-412)."""
    import u15b200
    from u15b200.generator import Generator
    H, W = 256, 192
    L_tok = (H // 32) * (W // 32)
    scale = Generator.noise_scale(L_tok)
    assert scale == O.init_noise_scale(L_tok)
    img = Generator.initial_image(H, W, 1234, scale)
    want = O.init_noise(1234, scale, H * W * 3).reshape(H, W, 3)
    got = host(img)
    assert img.is_cuda and np.array_equal(got.view(np.uint32), want.view(np.uint32))
    # injected noise, raw f32 channel-last
    noise = randn((H, W, 3), 99)
    f = tmp_path / "noise.f32"
    noise.tofile(f)
    assert np.array_equal(host(Generator.initial_image(H, W, 0, scale, init_noise_path=str(f))),
                          noise)
    noise[:-1].tofile(f)
    with pytest.raises(u15b200.U15Error, match="wrong size"):
        Generator.initial_image(H, W, 0, scale, init_noise_path=str(f))
    with pytest.raises(u15b200.U15Error, match="cannot read"):
        Generator.initial_image(H, W, 0, scale, init_noise_path=str(tmp_path / "absent"))
