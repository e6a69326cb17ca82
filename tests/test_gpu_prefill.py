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
