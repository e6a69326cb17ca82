"""GPU parity of the tcgen05 projection GEMMs.

bf16: the CPU restatement's double-accumulated product of the same
bf16-rounded inputs, bar kBf16Bar = 4e-3 rel-L2 (tests/u15-kernels-test.cc:55
in the reference). Full BASELINE shapes (M = 4096 routed 512 und / 3584 gen,
the four projections) are checked on a seeded sample of rows: the GPU
computes every row, the oracle the sampled ones.

int8 (BASELINE's W8A8 config): quantised inputs equal bit for bit, the int32
accumulators equal the exact integer product bit for bit, the dequantised
bf16 output within one bf16 rounding of the restatement.
"""
import numpy as np
import pytest

from gpu_util import bf16_round, dev_bf16, host, randn, rel_l2, torch
from oracle import oracle as O

pytestmark = pytest.mark.gpu
BAR = 4e-3
EPI_STORE, EPI_RESIDUAL, EPI_SWIGLU = 0, 1, 2


@pytest.fixture(scope="module")
def ops():
    import u15b200
    return u15b200.CudaOps(0)


def sample_rows(M, n, seed):
    if M <= n:
        return np.arange(M)
    return np.sort(np.random.default_rng(seed).choice(M, n, replace=False))


@pytest.mark.parametrize("M,K,N", [(128, 64, 256), (1, 64, 8), (200, 136, 48), (333, 4096, 1024),
                                   (130, 12288, 512), (300, 1160, 520)])
def test_linear_bf16(ops, M, K, N):
    x = bf16_round(randn((M, K), 1))
    w = bf16_round(randn((N, K), 2, 0.02))
    y = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    ops.linear(dev_bf16(x), dev_bf16(w), None, y, M, K, N)
    ops.sync()
    assert rel_l2(host(y), O.linear(x, w)) < BAR


def test_linear_bias(ops):
    M, K, N = 100, 256, 300
    x = bf16_round(randn((M, K), 3))
    w = bf16_round(randn((N, K), 4, 0.02))
    b = bf16_round(randn(N, 5, 0.5))
    y = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    ops.linear(dev_bf16(x), dev_bf16(w), dev_bf16(b), y, M, K, N)
    assert rel_l2(host(y), O.linear(x, w, b)) < BAR


def routed_ref(x, w, segs, rows):
    out = []
    for r in rows:
        e = [s[2] for s in segs if s[0] <= r < s[1]][0]
        out.append(O.linear(x[r:r + 1], w[e])[0])
    return np.stack(out)


@pytest.mark.parametrize("segs", [[(0, 64, 0), (64, 256, 1)],
                                  [(0, 100, 1), (100, 101, 0), (101, 300, 1)],
                                  [(0, 300, 0)]])
def test_mot_routing(ops, segs):
    M, K, N = segs[-1][1], 512, 768
    x = bf16_round(randn((M, K), 6))
    w = bf16_round(randn((2, N, K), 7, 0.02))
    y = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    ops.mot_linear(dev_bf16(x), dev_bf16(w), segs, y, M, K, N)
    rows = np.arange(M)
    assert rel_l2(host(y), routed_ref(x, w, segs, rows)) < BAR
    if len(segs) > 1:   # negative control: the experts differ
        assert rel_l2(host(y), O.linear(x, w[segs[0][2]])) > 1e-2


def test_mot_routing_many_rows(ops):
    """A routed pass of 60000 rows over five segments (the row units come from
    the segment table, so M has no cap), checked on rows around every segment
    boundary and the last row against the CPU restatement; blocks of the
    CTA-pair kernel straddle three of the boundaries; every row against
    torch's product of the same bf16 operands."""
    M, K, N = 60000, 256, 256
    segs = [(0, 7000, 0), (7000, 7001, 1), (7001, 30000, 0), (30000, 41000, 1), (41000, M, 0)]
    torch.manual_seed(16)
    xd = torch.randn(M, K, device="cuda").to(torch.bfloat16)
    wd = (torch.randn(2, N, K, device="cuda") * 0.02).to(torch.bfloat16)
    y = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    ops.mot_linear(xd, wd, segs, y, M, K, N)
    ops.sync()
    rows = np.unique(np.concatenate([[b + d for b in (0, 7000, 7001, 30000, 41000) for d in
                                      (-2, -1, 0, 1, 2)], [M - 1]]))
    rows = rows[(rows >= 0) & (rows < M)]
    want = np.stack([O.linear(host(xd[r:r + 1]), host(wd[[s[2] for s in segs if s[0] <= r < s[1]][0]]))[0]
                     for r in rows])
    assert rel_l2(host(y[torch.from_numpy(rows).cuda()]), want) < BAR
    full = torch.empty_like(y, dtype=torch.float32)
    for lo, hi, e in segs:
        full[lo:hi] = xd[lo:hi].float() @ wd[e].float().t()
    assert ((y.float() - full).norm() / full.norm()).item() < BAR


def test_residual_epilogue_in_place(ops):
    M, K, N = 256, 1024, 512
    x = bf16_round(randn((M, K), 8))
    w = bf16_round(randn((2, N, K), 9, 0.02))
    r = bf16_round(randn((M, N), 10))
    segs = [(0, 64, 0), (64, M, 1)]
    rd = dev_bf16(r)
    ops.mot_linear(dev_bf16(x), dev_bf16(w), segs, rd, M, K, N, epilogue=EPI_RESIDUAL, resid=rd)
    ref = r + routed_ref(x, w, segs, np.arange(M))
    assert rel_l2(host(rd), ref) < BAR


def interleave_gate_up(g, u):
    """[gate_j | up_j] 128-row blocks, the SwiGLU epilogue's bound layout."""
    I, K = g.shape
    out = np.empty((2 * I, K), np.float32)
    for j in range(I // 128):
        out[256 * j:256 * j + 128] = g[128 * j:128 * j + 128]
        out[256 * j + 128:256 * j + 256] = u[128 * j:128 * j + 128]
    return out


def test_swiglu_epilogue(ops):
    M, K, I = 200, 512, 384
    x = bf16_round(randn((M, K), 11))
    g = bf16_round(randn((I, K), 12, 0.05))
    u = bf16_round(randn((I, K), 13, 0.05))
    w = interleave_gate_up(g, u)[None]
    y = torch.empty(M, I, dtype=torch.bfloat16, device="cuda")
    ops.mot_linear(dev_bf16(x), dev_bf16(w), None, y, M, K, 2 * I, epilogue=EPI_SWIGLU)
    ref = O.swiglu(O.linear(x, g), O.linear(x, u))
    assert rel_l2(host(y), ref) < BAR


# the four projections at M = 4096, routed 512 / 3584
SHAPES = {"qkv": (4096, 6144), "o": (4096, 4096), "gate_up": (4096, 24576),
          "down": (12288, 4096)}


@pytest.mark.parametrize("name", list(SHAPES))
def test_baseline_shapes_routed(ops, name):
    K, N = SHAPES[name]
    M = 4096
    segs = [(0, 512, 0), (512, 4096, 1)]
    torch.manual_seed(17)
    xd = torch.randn(M, K, device="cuda").to(torch.bfloat16)
    wd = (torch.randn(2, N, K, device="cuda") * 0.02).to(torch.bfloat16)
    y = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    ops.mot_linear(xd, wd, segs, y, M, K, N)
    ops.sync()
    rows = sample_rows(M, 24, 18)
    rows = np.union1d(rows, [0, 511, 512, 4095])
    x = host(xd[torch.from_numpy(rows).cuda()])
    got = host(y[torch.from_numpy(rows).cuda()])
    ref = np.stack([O.linear(x[i:i + 1], host(wd[0 if r < 512 else 1]))[0]
                    for i, r in enumerate(rows)])
    assert rel_l2(got, ref) < BAR


# ---------------------------------------------------------------- W8A8
def quantised(ops, x):
    rows, cols = x.shape
    q = torch.empty(rows, cols, dtype=torch.int8, device="cuda")
    s = torch.empty(rows, dtype=torch.float32, device="cuda")
    ops.quant_rows_i8(dev_bf16(x), q, s, rows, cols)
    return q, s


def _bf16_step(v, d):
    """v (bf16-representable f32) moved d bf16 steps (toward +inf for d > 0
    on positive values)."""
    b = (v.view(np.uint32) >> 16).astype(np.int64) + d
    return (b.astype(np.uint32) << 16).view(np.float32)


@pytest.mark.parametrize("cols", [4096, 12288, 16384])
def test_quant_rows_ties_bit_exact(ops, cols):
    """Quotients at and one bf16 step either side of half-integers, for scales
    that are exact (amax 127, 63.5) and inexact (amax 100, 3.3): the device's
    reciprocal path must reproduce the division rule's codes, ties to even
    included. Column counts cover the 16- and 48-per-thread register forms and
    the two-pass form."""
    rng = np.random.default_rng(5)
    rows = []
    for amax in (127.0, 63.5, 100.0, 3.3):
        a = bf16_round(np.array([amax], np.float32))[0]
        sc = np.float32(a) / np.float32(127.0)
        for d in (0, 1, -1):
            k = rng.integers(-126, 126, cols).astype(np.float32)
            v = bf16_round(((k + np.float32(0.5)) * sc).astype(np.float32))
            if d:
                v = _bf16_step(v, d)
            v = np.clip(v, -a, a)
            v[0] = a
            rows.append(v)
    x = np.stack(rows).astype(np.float32)
    q, s = quantised(ops, x)
    rq, rs = O.quant_rows_i8(x)
    assert np.array_equal(host(s), rs)
    assert np.array_equal(host(q), rq)


@pytest.mark.parametrize("cols", [4096, 12288, 16384])
def test_quant_rows_tiny_scales_bit_exact(ops, cols):
    """Rows whose scale is subnormal (amax below 127 * 2^-126, down to bf16
    subnormals), rows at that edge, and an all-zero row: the device takes the
    clamped division for the subnormal scales and must match the oracle."""
    rng = np.random.default_rng(6)
    rows = []
    for amax in (1.6e-36, 1.5e-36, 1.4e-36, 1e-37, 1e-38, 3e-39, 1e-40, 0.0, 1.0):
        v = bf16_round(rng.uniform(-1, 1, cols).astype(np.float32) * np.float32(amax))
        if amax:
            v[7] = bf16_round(np.array([amax], np.float32))[0]
        rows.append(v)
    x = np.stack(rows).astype(np.float32)
    q, s = quantised(ops, x)
    rq, rs = O.quant_rows_i8(x)
    assert np.array_equal(host(s), rs)
    assert np.array_equal(host(q), rq)


@pytest.mark.parametrize("M,K,N", [(128, 128, 256), (77, 4096, 1000), (256, 12288, 512),
                                   (200, 384, 256), (300, 1104, 520)])
def test_linear_i8_bit_exact(ops, M, K, N):
    x = bf16_round(randn((M, K), 20))
    w = bf16_round(randn((N, K), 21, 0.02))
    xq, xs = quantised(ops, x)
    wq, ws = quantised(ops, w)
    rxq, rxs = O.quant_rows_i8(x)
    rwq, rws = O.quant_rows_i8(w)
    assert np.array_equal(host(xq), rxq) and np.array_equal(host(wq), rwq)
    y = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    acc = torch.empty(M, N, dtype=torch.int32, device="cuda")
    ops.linear_i8(xq, xs, wq, ws, y, M, K, N, acc_dump=acc)
    ops.sync()
    racc = O.gemm_i8(rxq, rwq)
    assert np.array_equal(host(acc), racc)          # int32 accumulators: bit-exact
    ry = bf16_round(O.dequant_i8(racc, rxs, rws))
    assert rel_l2(host(y), ry) < 2e-3
    # and the W8A8 product stays close to the bf16 one
    assert rel_l2(host(y), O.linear(x, w)) < 3e-2


def test_mot_linear_i8_routed_full_k(ops):
    M, K, N = 640, 4096, 1536
    segs = [(0, 512, 0), (512, 640, 1)]
    x = bf16_round(randn((M, K), 22))
    w = bf16_round(randn((2, N, K), 23, 0.02))
    xq, xs = quantised(ops, x)
    wq, ws = quantised(ops, w.reshape(2 * N, K))
    y = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    acc = torch.empty(M, N, dtype=torch.int32, device="cuda")
    ops.mot_linear_i8(xq, xs, wq.view(2, N, K), ws.view(2, N), segs, y, M, K, N, acc_dump=acc)
    ops.sync()
    rxq, _ = O.quant_rows_i8(x)
    rwq, _ = O.quant_rows_i8(w.reshape(2 * N, K))
    rwq = rwq.reshape(2, N, K)
    ref = np.concatenate([O.gemm_i8(rxq[a:b], rwq[e]) for a, b, e in segs])
    assert np.array_equal(host(acc), ref)


# ------------------------------------------------- split-tail schedule
# Tile counts whose last round of the persistent schedule leaves at least
# half of the B200's 74 SM pairs idle: those tiles run as half-width tiles
# (each CTA stages 64 weight rows). Every row and column is checked.
SPLIT_SEGS = [(0, 512, 0), (512, 2560, 1)]


def test_split_tail_routed_bf16(ops):
    M, K, N = 2560, 512, 2304   # 10 row blocks x 9 column blocks = 90 tiles
    x = bf16_round(randn((M, K), 30))
    w = bf16_round(randn((2, N, K), 31, 0.02))
    y = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    ops.mot_linear(dev_bf16(x), dev_bf16(w), SPLIT_SEGS, y, M, K, N)
    ops.sync()
    ref = np.concatenate([O.linear(x[a:b], w[e]) for a, b, e in SPLIT_SEGS])
    assert rel_l2(host(y), ref) < BAR
    # the tail's columns on their own (the last 34 tiles' column blocks)
    assert rel_l2(host(y)[:, 1792:], ref[:, 1792:]) < BAR


def test_split_tail_swiglu(ops):
    M, K, I = 2560, 256, 1152   # gate+up 2304 rows: 90 tiles
    x = bf16_round(randn((M, K), 32))
    g = bf16_round(randn((I, K), 33, 0.05))
    u = bf16_round(randn((I, K), 34, 0.05))
    w = interleave_gate_up(g, u)[None]
    y = torch.empty(M, I, dtype=torch.bfloat16, device="cuda")
    ops.mot_linear(dev_bf16(x), dev_bf16(w), None, y, M, K, 2 * I, epilogue=EPI_SWIGLU)
    ops.sync()
    ref = O.swiglu(O.linear(x, g), O.linear(x, u))
    assert rel_l2(host(y), ref) < BAR
    assert rel_l2(host(y)[:, 896:], ref[:, 896:]) < BAR


def test_split_tail_residual_i8_bit_exact(ops):
    M, K, N = 2560, 256, 2304
    x = bf16_round(randn((M, K), 35))
    w = bf16_round(randn((2, N, K), 36, 0.02))
    r = bf16_round(randn((M, N), 37))
    xq, xs = quantised(ops, x)
    wq, ws = quantised(ops, w.reshape(2 * N, K))
    rd = dev_bf16(r)
    acc = torch.empty(M, N, dtype=torch.int32, device="cuda")
    ops.mot_linear_i8(xq, xs, wq.view(2, N, K), ws.view(2, N), SPLIT_SEGS, rd, M, K, N,
                      epilogue=EPI_RESIDUAL, resid=rd, acc_dump=acc)
    ops.sync()
    rxq, rxs = O.quant_rows_i8(x)
    rwq, rws = O.quant_rows_i8(w.reshape(2 * N, K))
    rwq, rws = rwq.reshape(2, N, K), rws.reshape(2, N)
    racc = np.concatenate([O.gemm_i8(rxq[a:b], rwq[e]) for a, b, e in SPLIT_SEGS])
    assert np.array_equal(host(acc), racc)
    deq = np.concatenate([O.dequant_i8(racc[a:b], rxs[a:b], rws[e]) for a, b, e in SPLIT_SEGS])
    ref = bf16_round(r + bf16_round(deq))
    assert rel_l2(host(rd), ref) < 2e-3


def test_single_segment_unbounded_rows(ops):
    """One routing segment has implicit row units: M far beyond the routed
    table's 200 units (the pixel head's conv2 at 2048^2 px: M = 65536,
    N = 192 as one partial column tile, bias)."""
    M, K, N = 65536, 144, 192
    torch.manual_seed(40)
    xd = torch.randn(M, K, device="cuda").to(torch.bfloat16)
    wd = (torch.randn(N, K, device="cuda") * 0.05).to(torch.bfloat16)
    bd = (torch.randn(N, device="cuda") * 0.1).to(torch.bfloat16)
    y = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    ops.linear(xd, wd, bd, y, M, K, N)
    ops.sync()
    rows = np.union1d(sample_rows(M, 40, 41), [0, 255, 256, 51199, 51200, M - 1])
    idx = torch.from_numpy(rows).cuda()
    got = host(y[idx])
    ref = O.linear(host(xd[idx]), host(wd), host(bd))
    assert rel_l2(got, ref) < BAR


@pytest.mark.parametrize("int8", [False, True], ids=["bf16", "i8"])
@pytest.mark.parametrize("K", [1160, 4096], ids=["odd-kblocks", "even-kblocks"])
def test_pair_stage_forms_agree(ops, monkeypatch, int8, K):
    """The CTA-pair GEMM stages one, two or three k-blocks per pipeline stage
    (U15_GEMM_KPS, read per launch); an odd k-block count leaves a last stage
    part full. Every form sums the same products in the same order, so the
    routed outputs are bit-identical, and the default form matches the
    oracle."""
    M, N = 640, 768
    segs = [(0, 192, 0), (192, M, 1)]
    g = torch.Generator(device="cuda").manual_seed(41)
    if int8:
        K -= K % 16   # int8 rows: 16-byte TMA strides
        xq = torch.randint(-127, 128, (M, K), dtype=torch.int8, device="cuda", generator=g)
        xs = torch.rand(M, device="cuda", generator=g) * 0.01 + 0.01
        wq = torch.randint(-127, 128, (2, N, K), dtype=torch.int8, device="cuda", generator=g)
        ws = torch.rand(2, N, device="cuda", generator=g) * 0.001 + 0.001
    else:
        x = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
        w = (torch.randn(2, N, K, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    outs = {}
    for kps in ("1", "2", "3"):
        monkeypatch.setenv("U15_GEMM_KPS", kps)
        y = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device="cuda")
        if int8:
            acc = torch.empty(M, N, dtype=torch.int32, device="cuda")
            ops.mot_linear_i8(xq, xs, wq, ws, segs, y, M, K, N, acc_dump=acc)
            outs[kps] = (y, acc)
        else:
            ops.mot_linear(x, w, segs, y, M, K, N)
            outs[kps] = (y,)
        ops.sync()
    for kps in ("1", "3"):
        for a, b in zip(outs["2"], outs[kps]):
            assert torch.equal(a, b), kps
    if int8:
        racc = np.concatenate([O.gemm_i8(host(xq)[lo:hi], host(wq)[e]) for lo, hi, e in segs])
        assert np.array_equal(host(outs["2"][1]), racc)
    else:
        xh, wh = host(x), host(w)
        ref = np.concatenate([O.linear(xh[lo:hi], wh[e]) for lo, hi, e in segs])
        assert rel_l2(host(outs["2"][0]), ref) < BAR
