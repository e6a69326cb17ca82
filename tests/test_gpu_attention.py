"""GPU parity of the flash attention against the CPU restatement.

Geometry from the reference's steel test (tests/u15-kernels-test.cc:737-828:
hq 8 / hkv 2 at head_dim 128, tq 48, tk 67, cache capacity 88 > tk) and its
negative controls (GQA factor 1 must differ, plain causal must differ from
block-causal, the kv stride is the capacity), plus the BASELINE attention
shape (4096 queries over a 320-token prefix + 4096) on sampled heads, the
paged cache with a permuted page table, and the Sage int8-QK path against its
own restatement (the reference's Sage tiles: 64 query rows and 32 keys per
scale) and against exact attention. The tcgen05 kernel's masked rules are
held to the same bar, up to the BASELINE block-causal prefill (64 text
tokens + 2 reference images of 1024 tokens, t from thw_indexes).
"""
import numpy as np
import pytest

from gpu_util import bf16_round, dev_bf16, dev_i32, host, randn, rel_l2, torch
from oracle import oracle as O

pytestmark = pytest.mark.gpu
BAR = 4e-3


@pytest.fixture(scope="module")
def ops():
    import u15b200
    return u15b200.CudaOps(0)


def qkv(hq, hkv, tq, cap, seed, k_mean=0.0):
    q = bf16_round(randn((hq, tq, 128), seed))
    k = bf16_round(randn((hkv, cap, 128), seed + 1, 1.0, k_mean))
    v = bf16_round(randn((hkv, cap, 128), seed + 2))
    return q, k, v


def run(ops, q, k, v, tk, mode=0, q_offset=0, t_index=None, sage=False, page_table=None):
    hq, tq, _ = q.shape
    hkv, cap, _ = k.shape
    out = torch.empty(tq, hq * 128, dtype=torch.bfloat16, device="cuda")
    ws = ops.sage_workspace(hq, hkv, tq, tk) if sage else None
    if page_table is None:
        ops.attention(dev_bf16(q), dev_bf16(k), dev_bf16(v), out, hq, hkv, tq, tk, cap=cap,
                      mode=mode, q_offset=q_offset,
                      t_index=dev_i32(t_index) if t_index is not None else None, sage_ws=ws)
    else:
        kp, vp = to_pages(k, page_table), to_pages(v, page_table)
        ops.attention(dev_bf16(q), dev_bf16(kp), dev_bf16(vp), out, hq, hkv, tq, tk,
                      page_table=dev_i32(page_table), mode=mode, q_offset=q_offset,
                      t_index=dev_i32(t_index) if t_index is not None else None, sage_ws=ws)
    ops.sync()
    return host(out)


def to_pages(kc, table):
    """[hkv][cap][128] -> pool [pages][hkv][64][128] under a logical->physical table."""
    hkv, cap, _ = kc.shape
    n = len(table)
    pool = np.zeros((n, hkv, 64, 128), np.float32)
    for lp in range(n):
        seg = kc[:, lp * 64:(lp + 1) * 64]
        pool[table[lp], :, :seg.shape[1]] = seg
    return pool


def test_steel_geometry_bidirectional(ops):
    q, k, v = qkv(8, 2, 48, 88, 1)
    got = run(ops, q, k, v, 67)
    ref = O.attention(q, k, v, tk=67)
    assert rel_l2(got, ref) < BAR
    # negative control: GQA factor 1 (query head h reads kv head h % 2)
    wrong = O.attention(q, np.concatenate([k] * 4)[:8], np.concatenate([v] * 4)[:8], tk=67)
    assert rel_l2(got, wrong) > 1e-2
    # negative control: the stride is the capacity, not the key length
    packed_k = np.ascontiguousarray(k[:, :67])
    assert rel_l2(run(ops, q, packed_k, np.ascontiguousarray(v[:, :67]), 67), ref) < BAR


def test_causal_with_offset(ops):
    q, k, v = qkv(4, 1, 40, 100, 4)
    got = run(ops, q, k, v, 90, mode=1, q_offset=50)
    ref = O.attention(q, k, v, tk=90, mode=O.CAUSAL, q_offset=50)
    assert rel_l2(got, ref) < BAR


def test_block_causal(ops):
    # the reference's t pattern, extended: a text run, an image block sharing
    # one t, more text (tests/u15-kernels-test.cc:612)
    t = np.array([0, 1, 2] + [3] * 70 + [4, 5, 6], np.int32)
    T = t.size
    q, k, v = qkv(8, 2, T, T + 4, 7)
    got = run(ops, q, k, v, T, mode=2, t_index=t)
    ref = O.attention(q, k, v, tk=T, mode=O.BLOCK_CAUSAL, t_index=t)
    assert rel_l2(got, ref) < BAR
    causal = O.attention(q, k, v, tk=T, mode=O.CAUSAL)
    assert rel_l2(got, causal) > 1e-2


def test_paged_permuted(ops):
    q, k, v = qkv(32, 8, 100, 320, 9)
    table = np.array([3, 0, 4, 1, 2], np.int32)   # 5 pages of 64
    got = run(ops, q, k, v, 300, page_table=table)
    ref = O.attention(q, k, v, tk=300)
    assert rel_l2(got, ref) < BAR


def test_baseline_shape_sampled_heads(ops):
    """4096 generation queries over [320 prefix || 4096], GQA 32/8."""
    tq, tk = 4096, 4416
    torch.manual_seed(11)
    qd = torch.randn(32, tq, 128, device="cuda").to(torch.bfloat16)
    kd = torch.randn(8, tk, 128, device="cuda").to(torch.bfloat16)
    vd = torch.randn(8, tk, 128, device="cuda").to(torch.bfloat16)
    out = torch.empty(tq, 32 * 128, dtype=torch.bfloat16, device="cuda")
    ops.attention(qd, kd, vd, out, 32, 8, tq, tk, cap=tk)
    ops.sync()
    rows = np.sort(np.random.default_rng(12).choice(tq, 48, replace=False))
    for h in (0, 13, 31):
        hk = h // 4
        q = host(qd[h:h + 1, torch.from_numpy(rows).cuda()])
        ref = O.attention(q, host(kd[hk:hk + 1]), host(vd[hk:hk + 1]))
        got = host(out[torch.from_numpy(rows).cuda(), h * 128:(h + 1) * 128])
        assert rel_l2(got, ref) < BAR


def test_sage_matches_restatement(ops):
    q, k, v = qkv(8, 2, 130, 200, 13, k_mean=0.7)
    got = run(ops, q, k, v, 170, sage=True)
    sage_ref = O.sage_attention(q, k, v, tk=170, bq=64, bk=32)
    exact = O.attention(q, k, v, tk=170)
    assert rel_l2(got, sage_ref) < 1e-2
    assert rel_l2(got, exact) < 3e-2


def test_sage_refuses_masked(ops):
    import u15b200
    q, k, v = qkv(4, 1, 16, 64, 14)
    with pytest.raises(u15b200.U15Error):
        run(ops, q, k, v, 64, mode=1, sage=True)


# ---------------------------------------------------------------------------
# the tcgen05 kernel over the model's paged layout (V pages transposed)
# ---------------------------------------------------------------------------
def to_model_pages(k, v, table):
    """[hkv][cap][128] K and V -> K pool [P][hkv][64][128] and transposed V pool
    [P][hkv][128][64] under a logical->physical page table."""
    hkv, cap, _ = k.shape
    n = len(table)
    kp = np.zeros((n, hkv, 64, 128), np.float32)
    vp = np.zeros((n, hkv, 128, 64), np.float32)
    for lp in range(n):
        ks = k[:, lp * 64:(lp + 1) * 64]
        vs = v[:, lp * 64:(lp + 1) * 64]
        kp[table[lp], :, :ks.shape[1]] = ks
        vp[table[lp], :, :, :vs.shape[1]] = vs.transpose(0, 2, 1)
    return kp, vp


def run_paged(ops, q, k, v, tk, table=None, mode=0, q_offset=0, t_index=None, sage=False):
    hq, tq, _ = q.shape
    hkv, cap, _ = k.shape
    n = (cap + 63) // 64
    table = np.arange(n, dtype=np.int32) if table is None else np.asarray(table, np.int32)
    kp, vp = to_model_pages(k, v, table)
    out = torch.empty(tq, hq * 128, dtype=torch.bfloat16, device="cuda")
    ws = ops.sage_workspace(hq, hkv, tq, tk) if sage else None
    ops.attention_paged(dev_bf16(q), dev_bf16(kp), dev_bf16(vp), out, hq, hkv, tq, tk,
                        page_table=dev_i32(table), mode=mode, q_offset=q_offset,
                        t_index=dev_i32(t_index) if t_index is not None else None, sage_ws=ws)
    ops.sync()
    return host(out)


@pytest.mark.parametrize("hq,hkv,tq,cap,tk", [(8, 2, 48, 88, 67), (4, 1, 300, 320, 320),
                                              (32, 8, 257, 200, 130), (8, 8, 512, 640, 577)])
def test_tc_bidirectional(ops, hq, hkv, tq, cap, tk):
    q, k, v = qkv(hq, hkv, tq, cap, 21)
    got = run_paged(ops, q, k, v, tk)
    assert rel_l2(got, O.attention(q, k, v, tk=tk)) < BAR


def test_tc_permuted_pages_and_gqa_control(ops):
    q, k, v = qkv(32, 8, 260, 320, 22)
    got = run_paged(ops, q, k, v, 300, table=[4, 2, 0, 3, 1])
    ref = O.attention(q, k, v, tk=300)
    assert rel_l2(got, ref) < BAR
    wrong = O.attention(q, np.repeat(k, 4, axis=0)[np.arange(32) % 8 * 4],
                        np.repeat(v, 4, axis=0)[np.arange(32) % 8 * 4], tk=300)
    assert rel_l2(got, wrong) > 1e-2


def test_tc_baseline_shape_sampled(ops):
    tq, tk = 4096, 4416
    q, k, v = qkv(32, 8, tq, tk, 23)
    got = run_paged(ops, q, k, v, tk)
    rows = np.sort(np.random.default_rng(24).choice(tq, 40, replace=False))
    for h in (0, 9, 31):
        hk = h // 4
        ref = O.attention(q[h:h + 1, rows], k[hk:hk + 1], v[hk:hk + 1])
        assert rel_l2(got[rows, h * 128:(h + 1) * 128], ref) < BAR


def test_tc_sage(ops):
    q, k, v = qkv(8, 2, 300, 256, 25, k_mean=0.7)
    got = run_paged(ops, q, k, v, 230, sage=True)
    assert rel_l2(got, O.sage_attention(q, k, v, tk=230, bq=64, bk=32)) < 1e-2
    assert rel_l2(got, O.attention(q, k, v, tk=230)) < 3e-2


def test_paged_masked_rules_transposed_v(ops):
    q, k, v = qkv(8, 2, 40, 128, 26)
    got = run_paged(ops, q, k, v, 100, table=[1, 0], mode=1, q_offset=60)
    assert rel_l2(got, O.attention(q, k, v, tk=100, mode=O.CAUSAL, q_offset=60)) < BAR
    t = np.array([0, 1] + [2] * 50 + [3, 4], np.int32)
    q2, k2, v2 = qkv(8, 2, t.size, 64, 27)
    got = run_paged(ops, q2, k2, v2, t.size, mode=2, t_index=t)
    assert rel_l2(got, O.attention(q2, k2, v2, tk=t.size, mode=O.BLOCK_CAUSAL, t_index=t)) < BAR


# ---------------------------------------------------------------------------
# the tcgen05 kernel's prefill rules (causal, block-causal)
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("hq,hkv,tq,cap,tk,off", [(8, 2, 48, 88, 67, 19), (4, 1, 300, 640, 600, 300),
                                                  (32, 8, 257, 320, 257, 0),
                                                  (8, 8, 640, 768, 700, 60)])
def test_tc_causal(ops, hq, hkv, tq, cap, tk, off):
    q, k, v = qkv(hq, hkv, tq, cap, 31)
    got = run_paged(ops, q, k, v, tk, mode=1, q_offset=off)
    ref = O.attention(q, k, v, tk=tk, mode=O.CAUSAL, q_offset=off)
    assert rel_l2(got, ref) < BAR
    # negative control: the bidirectional rule over the same keys differs
    assert rel_l2(got, O.attention(q, k, v, tk=tk)) > 1e-2


def test_tc_block_causal_reference_pattern(ops):
    # the reference kernel test's t pattern (tests/u15-kernels-test.cc:612),
    # stretched so an image run crosses 128-key blocks and query tiles
    t = np.array([0, 1, 2] + [3] * 300 + [4, 5, 6] + [7] * 40 + [8], np.int32)
    T = t.size
    q, k, v = qkv(8, 2, T, T + 20, 32)
    got = run_paged(ops, q, k, v, T, table=np.random.default_rng(3).permutation((T + 83) // 64),
                    mode=2, t_index=t)
    ref = O.attention(q, k, v, tk=T, mode=O.BLOCK_CAUSAL, t_index=t)
    assert rel_l2(got, ref) < BAR
    assert rel_l2(got, O.attention(q, k, v, tk=T, mode=O.CAUSAL)) > 1e-2


def test_tc_block_causal_offset_and_unsorted_t(ops):
    # queries after a prefix (q_offset), and a t vector that is not sorted:
    # rows see later keys wherever their t matches
    rng = np.random.default_rng(5)
    T, off = 520, 200
    t = rng.integers(0, 6, T).astype(np.int32)
    q, k, v = qkv(4, 2, T - off, T, 33)
    got = run_paged(ops, q, k, v, T, mode=2, q_offset=off, t_index=t)
    ref = O.attention(q, k, v, tk=T, mode=O.BLOCK_CAUSAL, q_offset=off, t_index=t)
    assert rel_l2(got, ref) < BAR


def c4_prefill_ids():
    """BASELINE config 4's prefill: 64 text tokens around two reference
    images of 1024 tokens each (a 64 x 64 patch grid, merge 2), with their
    <img> / </img> markers."""
    IMG, CTX, END = 151665, 151667, 151666
    text = list(range(1000, 1064))
    ids = (text[:32] + [IMG] + [CTX] * 1024 + [END] + text[32:48] + [IMG] + [CTX] * 1024 +
           [END] + text[48:])
    return np.array(ids, np.int32), IMG, CTX, [(64, 64), (64, 64)]


def test_tc_block_causal_c4_prefill(ops):
    """The whole C4 prefill (2116 tokens, GQA 32/8) through the tcgen05
    kernel, t from u15c_thw_indexes; sampled heads and rows against the CPU
    restatement, and the causal rule as the negative control."""
    import ctypes as C
    from u15b200 import _lib as L
    ids, IMG, CTX, grids = c4_prefill_ids()
    T = ids.size
    t, hh, ww = (np.zeros(T, np.int32) for _ in range(3))
    g = np.ascontiguousarray(np.array(grids, np.int32).reshape(-1))
    vp = lambda a: C.c_void_p(a.ctypes.data)  # noqa: E731
    assert L.lib().u15c_thw_indexes(vp(ids), T, IMG, CTX, vp(g), 2, vp(t), vp(hh), vp(ww)) == 0
    assert np.array_equal(t, O.thw_indexes(ids, IMG, CTX, grids)[0])
    q, k, v = qkv(32, 8, T, T, 34)
    got = run_paged(ops, q, k, v, T, mode=2, t_index=t)
    rng = np.random.default_rng(35)
    # rows in the text, inside each image (early, middle, last) and after it
    rows = np.unique(np.concatenate([rng.choice(T, 40, replace=False), [0, 31, 32, 33, 600, 1057,
                                     1058, 1075, 2000, 2114, T - 1]]))
    for h in (0, 17, 31):
        hk = h // 4
        ref = np.concatenate([O.attention(q[h:h + 1, r:r + 1], k[hk:hk + 1], v[hk:hk + 1], tk=T,
                                          mode=O.BLOCK_CAUSAL, q_offset=int(r), t_index=t)
                              for r in rows])
        cau = np.concatenate([O.attention(q[h:h + 1, r:r + 1], k[hk:hk + 1], v[hk:hk + 1], tk=T,
                                          mode=O.CAUSAL, q_offset=int(r)) for r in rows])
        mine = got[rows, h * 128:(h + 1) * 128]
        assert rel_l2(mine, ref) < BAR, h
        assert rel_l2(mine, cau) > 1e-2, h


def test_tc_masked_matches_mma_sync_kernel(ops):
    """The tcgen05 and mma.sync kernels on one cache (the op-level contiguous
    layout for the latter): the same rule, the same answer within the bar."""
    t = np.array([0] * 10 + [1] * 200 + list(range(2, 60)) + [60] * 130, np.int32)
    T = t.size
    q, k, v = qkv(16, 4, T, T, 36)
    for mode, kw in ((1, {}), (2, {"t_index": t})):
        a = run_paged(ops, q, k, v, T, mode=mode, **kw)
        b = run(ops, q, k, v, T, mode=mode, **kw)
        assert rel_l2(a, b) < BAR


@pytest.mark.parametrize("mode", [0, 1, 2], ids=["bidirectional", "causal", "block_causal"])
def test_tc_forms_agree(ops, mode, monkeypatch):
    """The tcgen05 kernel's forms, chosen per launch by the A/B switches (the
    softmax layout, one or two MMA issuers, who releases the K/V stages),
    give the same answer: bit for bit where only the hand-off differs, and
    within 1e-3 of each other where the softmax sums a row in another order;
    each form within the attention bar of the CPU restatement."""
    t = np.array([0] * 40 + [1] * 300 + list(range(2, 150)) + [150] * 160, np.int32)
    T = t.size
    q, k, v = qkv(8, 2, T - 130, T, 37)
    kw = {"mode": mode, "q_offset": 130 if mode else 0}
    if mode == 2:
        kw["t_index"] = t
    forms = [{}, {"U15_ATTN_RELEASE": "0"}, {"U15_ATTN_KS": "0", "U15_ATTN_ISSUERS": "1"},
             {"U15_ATTN_KS": "1", "U15_ATTN_ISSUERS": "2"}, {"U15_ATTN_KS": "1", "U15_ATTN_ISSUERS": "1"},
             {"U15_ATTN_TILES": "1"}]
    keys = ("U15_ATTN_RELEASE", "U15_ATTN_KS", "U15_ATTN_ISSUERS", "U15_ATTN_TILES")
    outs = []
    for f in forms:
        for key in keys:
            monkeypatch.delenv(key, raising=False)
        for key, val in f.items():
            monkeypatch.setenv(key, val)
        outs.append(run_paged(ops, q, k, v, T, **kw))
    for key in keys:
        monkeypatch.delenv(key, raising=False)
    ref = O.attention(q, k, v, tk=T, mode={0: O.BIDIR, 1: O.CAUSAL, 2: O.BLOCK_CAUSAL}[mode],
                      q_offset=kw["q_offset"], t_index=kw.get("t_index"))
    for i, o in enumerate(outs):
        assert rel_l2(o, ref) < BAR, (mode, forms[i])
        assert rel_l2(o, outs[0]) < 1e-3, (mode, forms[i])
    # the release form and the issuer's commits differ only in the hand-off;
    # the one-tile kernel runs the key-split softmax's arithmetic in the same
    # order as the two-tile key-split form
    if mode == 0:
        assert np.array_equal(outs[0], outs[1])
        assert np.array_equal(outs[5], outs[4])


@pytest.mark.parametrize("hq,hkv,tq,cap,tk", [(8, 2, 48, 88, 67), (4, 1, 300, 320, 320),
                                              (32, 8, 257, 200, 130), (8, 8, 512, 640, 577),
                                              (8, 2, 130, 1100, 1025)])
def test_tc_one_tile_kernel(ops, monkeypatch, hq, hkv, tq, cap, tk):
    """The bidirectional pass with one 128-row tile a CTA (U15_ATTN_TILES=1,
    two or three S buffers in TMEM): bf16 and Sage against the CPU
    restatements, ragged query and key counts, one to nine key blocks; the
    two buffer counts run the same arithmetic in the same order."""
    q, k, v = qkv(hq, hkv, tq, cap, 23)
    monkeypatch.setenv("U15_ATTN_TILES", "1")
    outs = []
    for sbuf in ("2", "3"):
        monkeypatch.setenv("U15_ATTN_SBUF", sbuf)
        got = run_paged(ops, q, k, v, tk)
        assert rel_l2(got, O.attention(q, k, v, tk=tk)) < BAR
        got8 = run_paged(ops, q, k, v, tk, sage=True)
        assert rel_l2(got8, O.sage_attention(q, k, v, tk=tk, bq=64, bk=32)) < 1e-2
        outs.append((got, got8))
    assert np.array_equal(outs[0][0], outs[1][0]) and np.array_equal(outs[0][1], outs[1][1])


def test_tc_last_round_split(ops, monkeypatch):
    """The bidirectional pass hands a part-empty last round of two-tile units
    to a second launch of the one-tile kernel (here 160 units on 148 SMs:
    the last 12 units, heads 29-31, as 24 one-tile CTAs). bf16 and Sage:
    within 1e-3 of the single launch (the tail rows sum their softmax in
    the key-split order) and within the bars of the CPU restatements on
    heads from both launches."""
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    hq, hkv, tk = 32, 8, 600
    tq = 256 * ((sms + 12 + hq - 1) // hq)   # just over one round of units
    units = tq // 256 * hq
    assert units % sms and 2 * (units % sms) <= sms
    q, k, v = qkv(hq, hkv, tq, tk, 29)
    for sage in (False, True):
        monkeypatch.setenv("U15_ATTN_SPLIT", "0")
        one = run_paged(ops, q, k, v, tk, sage=sage)
        monkeypatch.delenv("U15_ATTN_SPLIT")
        got = run_paged(ops, q, k, v, tk, sage=sage)
        assert rel_l2(got, one) < 1e-3
        for h in (0, hq - 2, hq - 1):
            hk = h // (hq // hkv)
            if sage:
                ref = O.sage_attention(q[h:h + 1], k[hk:hk + 1], v[hk:hk + 1], tk=tk, bq=64, bk=32)
                assert rel_l2(got[:, h * 128:(h + 1) * 128], ref) < 1e-2
            else:
                ref = O.attention(q[h:h + 1], k[hk:hk + 1], v[hk:hk + 1], tk=tk)
                assert rel_l2(got[:, h * 128:(h + 1) * 128], ref) < BAR
