"""The prefill from token ids on the GPU (src/u15-generator.cc:308-392): the
embed_tokens gather, the reference image's understanding-twin patch
embedding spliced over its <IMG_CONTEXT> run, the (t, h, w) triple, and the
block-causal prefill into the paged cache, against the CPU restatement."""
import numpy as np
import pytest

from gpu_util import bf16_round, dev_f32, host, randn, rel_l2, torch
from oracle import oracle as O

pytestmark = pytest.mark.gpu

IMG, CTX, END = 290, 291, 292


def test_prefill_from_ids_with_reference_image():
    import u15b200
    from u15b200.generator import DeviceImagePath, Generator, branch_from_ids
    from test_gpu_image import make
    from test_gpu_layer import SMALL, build, dims_of

    cfg = dict(SMALL)
    m, Wts = build(cfg, 500)
    hidden = cfg["hidden"]
    im, _, _ = make(dict(vision_hidden=64, llm_hidden=hidden, patch=16, merge=2, head_hidden=64,
                         freq_dim=256, noise_scale_embedding=1, vision_theta=1e4), 21)
    table = bf16_round(randn((300, hidden), 22))
    table_d = torch.from_numpy(table).cuda().to(torch.bfloat16)
    img = randn((64, 96, 3), 23)          # grid 4 x 6 -> 2 x 3 = 6 tokens
    ids = [100, 101, 102, IMG] + [CTX] * 6 + [END, 103, 104]
    b = branch_from_ids("edit_cond", ids, table_d, img_id=IMG, img_ctx_id=CTX,
                        images=[dev_f32(img)], image_path=im)
    torch.cuda.synchronize()
    x = host(b.prefix)
    ids_a = np.array(ids)
    ctx = ids_a == CTX
    assert np.array_equal(x[~ctx], table[ids_a[~ctx]])
    emb = host(im.embed(im.patchify(dev_f32(img)), 4, 6, gen=False))
    assert np.array_equal(x[ctx], emb)
    t, h, w = O.thw_indexes(ids, IMG, CTX, [(4, 6)])
    assert np.array_equal(b.t, t) and np.array_equal(b.h, h) and np.array_equal(b.w, w)
    assert b.block_causal

    # the block-causal prefill: layer 0's K in the cache vs the restatement
    gen = Generator(m, DeviceImagePath(im))
    gen._geom = (2, 2)
    gen.prefill(b, 4)
    torch.cuda.synchronize()
    _, kn, vn = O.mot_layer(x, [(0, len(ids), 0)], Wts[0], dims_of(cfg), t, h, w,
                            mode=O.BLOCK_CAUSAL, t_index=t)
    assert rel_l2(host(b.kv.read(0, False, len(ids))), kn) < 1e-2
    assert rel_l2(host(b.kv.read(0, True, len(ids))), vn) < 1e-2
    # and the generated image's tokens sit at max(t) + 1
    assert int(host(b.pos[0])[0]) == int(t.max()) + 1
    assert isinstance(im, u15b200.ImagePath)


def test_embed_tokens_bad_id_reports():
    import u15b200
    from u15b200 import _lib as L
    ops = u15b200.CudaOps(0)
    table = torch.ones(10, 64, dtype=torch.bfloat16, device="cuda")
    ids = torch.tensor([1, 12, 3], dtype=torch.int32, device="cuda")
    out = torch.full((3, 64), 7.0, dtype=torch.bfloat16, device="cuda")
    L.check(u15b200.lib().u15c_embed_tokens(None, table.data_ptr(), 10, 64, ids.data_ptr(), 3,
                                            out.data_ptr()))
    with pytest.raises(u15b200.U15Error):
        ops.sync()
    o = host(out)
    assert (o[0] == 1).all() and (o[1] == 0).all() and (o[2] == 1).all()


def test_c4_prefill_through_the_model():
    """BASELINE config 4's image-conditional prefill through the backbone: 64
    text tokens around two reference images of 1024 tokens (2116 tokens, t, h,
    w from u15c_thw_indexes) in one block-causal pass of both layers of a
    small-width model over the paged cache (a permuted page table), against
    the CPU restatement layer by layer: the output and each layer's K / V."""
    import ctypes as C
    from u15b200 import _lib as L
    from test_gpu_attention import c4_prefill_ids
    from test_gpu_layer import SMALL, build, check_layer, dims_of

    ids, IMG, CTX, grids = c4_prefill_ids()
    T = ids.size
    t, h, w = (np.zeros(T, np.int32) for _ in range(3))
    g = np.ascontiguousarray(np.array(grids, np.int32).reshape(-1))
    vp = lambda a: C.c_void_p(a.ctypes.data)  # noqa: E731
    assert L.lib().u15c_thw_indexes(vp(ids), T, IMG, CTX, vp(g), 2, vp(t), vp(h), vp(w)) == 0
    m, Wts = build(SMALL, 600)
    x = bf16_round(randn((T, SMALL["hidden"]), 601))
    kv = m.make_cache(T)
    kv.set_page_table(np.random.default_rng(602).permutation((T + 63) // 64).astype(np.int32))
    xd = torch.from_numpy(x).cuda().to(torch.bfloat16)
    pos = [torch.from_numpy(a).cuda() for a in (t, h, w)]
    m.forward(xd, kv, 0, T, *pos, segments=[(0, T, 0)], attn=L.ATTN_BLOCK_CAUSAL,
              t_index=torch.from_numpy(t).cuda())
    torch.cuda.synchronize()
    ref = x
    for li in range(SMALL["n_layers"]):
        cur = host(xd) if li == SMALL["n_layers"] - 1 else None
        ref_in = ref
        ref, kn, vn = O.mot_layer(ref_in, [(0, T, 0)], Wts[li], dims_of(SMALL), t, h, w,
                                  mode=O.BLOCK_CAUSAL, t_index=t)
        assert rel_l2(host(kv.read(li, False, T)), kn) < 1e-2, li
        assert rel_l2(host(kv.read(li, True, T)), vn) < 1e-2, li
    check_layer(cur, x, ref, bar=5e-2, delta_bar=5e-2)
