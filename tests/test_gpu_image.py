"""The image path (ImagePath: patch embedder, pixel head, timestep embedding)
on the GPU against the CPU restatement, which is pinned to the reference's
own vision_embed / conv_decoder (tests/test_oracle_golden.py).

Inputs and weights are bf16-rounded once on the host; both sides start from
the same values. The device keeps bf16 activations between the steps (as the
reference's device path does), so the bars are those of the reference's
image test: 2e-2 rel-L2 for the embedder and the pixel head
(tests/u15-image-test.cc:196, 263); the timestep row is f32 math on bf16
weights, 1e-4.
"""
import numpy as np
import pytest

from gpu_util import bf16_round, dev_bf16, dev_f32, host, randn, rel_l2, torch
from oracle import oracle as O

pytestmark = pytest.mark.gpu

SMALL = dict(vision_hidden=64, llm_hidden=256, patch=16, merge=2, head_hidden=64, freq_dim=256,
             noise_scale_embedding=1, vision_theta=1e4)


def make(cfg, seed):
    import u15b200
    im = u15b200.ImagePath(**cfg)
    rng = np.random.default_rng(seed)
    C, L, hid, D = cfg["vision_hidden"], cfg["llm_hidden"], cfg["head_hidden"], cfg["freq_dim"]
    p, m = cfg["patch"], cfg["merge"]
    g = lambda s, *sh: bf16_round(rng.normal(0, s, sh).astype(np.float32))  # noqa: E731
    W = [{"patch_w": g(0.03, C, 3 * p * p), "patch_b": g(0.1, C),
          "dense_w": g(0.05, L, C * m * m), "dense_b": g(0.1, L)} for _ in range(2)]
    H = {"conv1_w": g(0.03, hid, L // 4, 3, 3), "conv1_b": g(0.1, hid),
         "conv2_w": g(0.05, 192, hid // 4, 3, 3), "conv2_b": g(0.1, 192),
         "tstep_w0": g(0.05, L, D), "tstep_b0": g(0.1, L), "tstep_w2": g(0.02, L, L),
         "tstep_b2": g(0.1, L), "nscale_w0": g(0.05, L, D), "nscale_b0": g(0.1, L),
         "nscale_w2": g(0.02, L, L), "nscale_b2": g(0.1, L)}
    for e in range(2):
        for k, v in W[e].items():
            im.bind(k, v, expert=e)
    for k, v in H.items():
        im.bind(k, v)
    torch.cuda.synchronize()
    return im, W, H


@pytest.fixture(scope="module")
def small():
    return make(SMALL, 1)


def test_patchify_matches_restatement(small):
    im, _, _ = small
    img = randn((64, 96, 3), 2)
    px = im.patchify(dev_f32(img))
    assert np.array_equal(host(px), bf16_round(O.patchify_cf(img, 16)))


@pytest.mark.parametrize("gh,gw", [(8, 12), (4, 4), (2, 14)])
def test_embed_small(small, gh, gw):
    im, W, _ = small
    px = bf16_round(randn((gh * gw, 768), 3))
    for gen in (0, 1):
        out = im.embed(dev_bf16(px), gh, gw, gen=bool(gen))
        torch.cuda.synchronize()
        ref = O.vision_embed(px, W[gen], gh, gw)
        assert rel_l2(host(out), ref) < 2e-2
    # negative control: the other twin's weights
    assert rel_l2(host(out), O.vision_embed(px, W[0], gh, gw)) > 1e-1


def test_decode_small(small):
    im, _, Hw = small
    th, tw = 4, 6
    x = bf16_round(randn((th * tw, SMALL["llm_hidden"]), 4))
    out = im.decode(dev_bf16(x), th, tw)
    torch.cuda.synchronize()
    ref = O.conv_decoder_hwc(x, Hw, th, tw)
    assert out.shape == (32 * th, 32 * tw, 3)
    assert rel_l2(host(out), ref) < 2e-2
    # negative control: the transposed token grid
    xt = x.reshape(th, tw, -1).transpose(1, 0, 2).reshape(th * tw, -1)
    assert rel_l2(host(out), O.conv_decoder_hwc(xt, Hw, th, tw)) > 1e-1


def test_timestep_row_and_add(small):
    im, _, Hw = small
    for t, ratio in ((0.37, 0.25), (0.95, 1.0)):
        row = im.timestep_row(t, ratio)
        torch.cuda.synchronize()
        assert rel_l2(host(row), O.timestep_row(t, ratio, Hw)) < 1e-4
    x = bf16_round(randn((10, SMALL["llm_hidden"]), 5))
    xd = dev_bf16(x)
    im.add_timestep(xd, 0.95, 1.0)
    torch.cuda.synchronize()
    want = bf16_round(x + bf16_round(host(row))[None])
    assert np.array_equal(host(xd), want)


def test_to_u8_planar(small):
    im, _, _ = small
    px = np.linspace(-1.5, 1.5, 8 * 6 * 3).astype(np.float32).reshape(8, 6, 3)
    u8 = host(im.to_u8_planar(dev_f32(px)))
    want = (np.clip(px * 0.5 + 0.5, 0, 1) * 255 + 0.5).astype(np.uint8).transpose(2, 0, 1)
    assert np.array_equal(u8, want)


def test_full_width_embed_and_decode():
    """The model's widths (1024-wide patches, 4096 hidden, 1024-wide head) on a
    small grid: every GEMM of the path at its real K and N."""
    import u15b200
    im, W, Hw = make(u15b200.FULL_IMAGE, 7)
    gh = gw = 8
    px = bf16_round(randn((gh * gw, 768), 8))
    out = im.embed(dev_bf16(px), gh, gw, gen=True)
    torch.cuda.synchronize()
    assert rel_l2(host(out), O.vision_embed(px, W[1], gh, gw)) < 2e-2
    th = tw = 2
    x = bf16_round(randn((th * tw, 4096), 9))
    dec = im.decode(dev_bf16(x), th, tw)
    torch.cuda.synchronize()
    assert rel_l2(host(dec), O.conv_decoder_hwc(x, Hw, th, tw)) < 2e-2
    row = im.timestep_row(0.5, 0.5)
    torch.cuda.synchronize()
    assert rel_l2(host(row), O.timestep_row(0.5, 0.5, Hw)) < 1e-4
    im.close()


def test_pair_kernel_sizes(small):
    """Grids large enough that every GEMM runs on the CTA-pair kernel (M > 128),
    conv2's N = 192 as a partial 256-column tile."""
    im, W, Hw = small
    gh = gw = 32
    px = bf16_round(randn((gh * gw, 768), 10))
    out = im.embed(dev_bf16(px), gh, gw, gen=False)
    th = tw = 8
    x = bf16_round(randn((th * tw, SMALL["llm_hidden"]), 11))
    dec = im.decode(dev_bf16(x), th, tw)
    torch.cuda.synchronize()
    assert rel_l2(host(out), O.vision_embed(px, W[0], gh, gw)) < 2e-2
    assert rel_l2(host(dec), O.conv_decoder_hwc(x, Hw, th, tw)) < 2e-2
