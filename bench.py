"""Benchmark: one SenseNova-U1.5 MoT layer at 4096 tokens on B200.

Workload (BASELINE configs 2 and 4 in one layer): 4096 tokens routed 512 to
the understanding expert and 3584 to the _mot_gen expert (the MoT projection
GEMMs: QKV 4096x6144, O 4096x4096, gate+up 4096x24576, down 12288x4096),
joint bidirectional attention of the 4096 queries over a frozen 320-token
prefix plus themselves (4416 keys, GQA 32/8 x 128) through the paged KV
cache. Random-init weights N(0, 0.02) (no checkpoint), synthetic inputs
N(0, 1), all seeded. A step = one layer forward; steps rotate over 4 layers
with distinct weights (772 MB per layer, far above the 126 MB L2), so every
step streams its weights from HBM.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Under torchrun each rank runs an independent replica (a CFG branch or seed
of its own); no collective is on the data path, value = whole-job
effective ms per layer (max-over-ranks time / layers done by all ranks).
--impl reference times the reference's own CPU implementation (u15-ref,
compiled from the reference sources into oracle/_ref) on the host cores.
"""
from __future__ import annotations

import argparse
import csv
import io
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "vpipe-sensenova-u1.5_b200")
for _p in (ROOT, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "ms/MoT layer @4096 tok (bf16)"
UNIT = "ms"
M_TOK, N_UND, N_PRE = 4096, 512, 320
H, NH, KV, HD, I = 4096, 32, 8, 128, 12288
TK = N_PRE + M_TOK
GEMMS = {"qkv": (H, (NH + 2 * KV) * HD), "o": (NH * HD, H), "gate_up": (H, 2 * I),
         "down": (I, H)}
PROJ_FLOP = sum(2.0 * M_TOK * k * n for k, n in GEMMS.values())      # 1.5806e12
ATTN_FLOP = 4.0 * NH * M_TOK * TK * HD                                  # 2.964e11
LAYER_FLOP = PROJ_FLOP + ATTN_FLOP
PUBLISHED_MS = 148.0   # the published figure: Apple M5, bf16 (README.md:112-114 of the reference)
WORKLOAD = ("MoT layer @4096 tok: 512 und + 3584 gen routed, frozen 320-token prefix, "
            "bidirectional GQA 32/8x128 over 4416 keys (paged KV)")


LONG_WINDOW_S = 2.5   # the sustained window's default length (--sustained-s)


def bench_config(world):
    """The workload both arms report (the reference arm times the same layer
    on the host cores)."""
    return {"workload": WORKLOAD, "global_batch": M_TOK * world, "seq_len": TK,
            "parallelism": f"replicas x{world}" if world > 1 else "single",
            "l2": "inputs larger than L2: 4 layers x 772 MB of weights rotated per step"}


def int8_reference_rate():
    """Dense int8 tensor rate measured here (no int8 figure is in
    MEASURED_PEAKS.json): torch._int_mm (cuBLASLt) at 8192^3, best of 10,
    CUDA events; TOP/s (2 ops per multiply-add)."""
    import torch
    try:
        n = 8192
        a = torch.randint(-127, 128, (n, n), device="cuda", dtype=torch.int8)
        b = torch.randint(-127, 128, (n, n), device="cuda", dtype=torch.int8).t()
        for _ in range(3):
            torch._int_mm(a, b)
        best = min(ev_time(lambda: torch._int_mm(a, b), 1) for _ in range(10))
        del a, b
        return {"tops": 2.0 * n ** 3 / best / 1e9, "ms": best,
                "how": "torch._int_mm (cuBLASLt) int8 x int8 -> int32 at 8192^3, best of 10, "
                       "measured by this bench"}
    except Exception as e:   # an int8 library GEMM this torch build lacks
        return {"tops": None, "error": str(e)[:120]}


def i8_roofline(kern, peak):
    """The routed gate+up W8A8 GEMM against the measured int8 rate."""
    g = kern.get("i8_gate_up")
    if not g or not peak or not peak.get("tops"):
        return None
    return {"bound": "tensor (int8)", "kernel": "gemm_tc<i8> (gate_up, routed, SwiGLU epilogue)",
            "achieved": g["tflops"], "peak": peak["tops"], "unit": "TOP/s",
            "frac": g["tflops"] / peak["tops"], "peak_kind": peak["how"]}


def c4_prefill():
    """BASELINE config 4's block-causal prefill: 64 text tokens around two
    reference images of 1024 tokens each (+ <img> / </img> markers), t from
    the reference's thw_indexes rule (u15c_thw_indexes)."""
    import ctypes as C
    from u15b200 import _lib as L
    IMG, CTX, END = 151665, 151667, 151666
    text = list(range(1000, 1064))
    ids = np.array(text[:32] + [IMG] + [CTX] * 1024 + [END] + text[32:48] + [IMG] +
                   [CTX] * 1024 + [END] + text[48:], np.int32)
    T = ids.size
    t, h, w = (np.zeros(T, np.int32) for _ in range(3))
    g = np.array([64, 64, 64, 64], np.int32)
    vp = lambda a: C.c_void_p(a.ctypes.data)  # noqa: E731
    if L.lib().u15c_thw_indexes(vp(ids), T, IMG, CTX, vp(g), 2, vp(t), vp(h), vp(w)) != 0:
        raise RuntimeError(L.last_error())
    return t


def prefill_bench(ops, steps):
    """The C4 prefill attention (2116 tokens, GQA 32/8 x 128) over a paged
    cache: block-causal on the tcgen05 kernel, the causal rule over the same
    tokens, and the block-causal rule on the mma.sync kernel (the reference's
    contiguous layout). TFLOP/s count only the visible (query, key) pairs."""
    import torch
    t = c4_prefill()
    T = t.size
    vis = (np.arange(T)[None, :] <= np.arange(T)[:, None]) | (t[None, :] == t[:, None])
    pairs_bc = int(vis.sum())
    pairs_c = T * (T + 1) // 2
    g = torch.Generator(device="cuda").manual_seed(5)
    npg = (T + 63) // 64
    q = torch.randn(NH, T, HD, device="cuda", generator=g).bfloat16()
    kp = torch.randn(npg, KV, 64, HD, device="cuda", generator=g).bfloat16()
    vp = torch.randn(npg, KV, HD, 64, device="cuda", generator=g).bfloat16()
    kc = torch.randn(KV, T, HD, device="cuda", generator=g).bfloat16()
    vc = torch.randn(KV, T, HD, device="cuda", generator=g).bfloat16()
    table = torch.arange(npg, dtype=torch.int32, device="cuda")
    td = torch.from_numpy(t).cuda()
    o = torch.empty(T, NH * HD, device="cuda").bfloat16()
    runs = {
        "block_causal": (lambda: ops.attention_paged(q, kp, vp, o, NH, KV, T, T, page_table=table,
                                                     mode=2, t_index=td), pairs_bc),
        "causal": (lambda: ops.attention_paged(q, kp, vp, o, NH, KV, T, T, page_table=table,
                                               mode=1), pairs_c),
        "block_causal_mma_sync": (lambda: ops.attention(q, kc, vc, o, NH, KV, T, T, cap=T, mode=2,
                                                        t_index=td), pairs_bc),
    }
    out = {"tokens": T, "config": "64 text + 2 x (1024 image tokens + 2 markers), GQA 32/8 x 128,"
                                  " t from thw_indexes; FLOPs = 4 x 128 x heads x visible pairs",
           "visible_pairs_block_causal": pairs_bc, "visible_pairs_causal": pairs_c}
    for name, (fn, pairs) in runs.items():
        for _ in range(3):
            fn()
        ms = ev_time(fn, steps)
        out[name] = {"ms": ms, "tflops": 4.0 * HD * NH * pairs / ms / 1e9}
    out["kernel"] = "attn_tc_kernel<MODE 2> (tcgen05, paged KV, masked key blocks skipped)"
    return out


def profile_case(case, steps):
    """A small workload of one kind of kernel for ncu captures (the kernels
    the bench times, on the bench's inputs); returns the mean ms of a step."""
    import torch
    import u15b200
    ops = u15b200.CudaOps(0)
    g = torch.Generator(device="cuda").manual_seed(5)
    if case == "prefill":
        t = c4_prefill()
        T = t.size
        npg = (T + 63) // 64
        q = torch.randn(NH, T, HD, device="cuda", generator=g).bfloat16()
        kp = torch.randn(npg, KV, 64, HD, device="cuda", generator=g).bfloat16()
        vp = torch.randn(npg, KV, HD, 64, device="cuda", generator=g).bfloat16()
        table = torch.arange(npg, dtype=torch.int32, device="cuda")
        td = torch.from_numpy(t).cuda()
        o = torch.empty(T, NH * HD, device="cuda").bfloat16()
        fn = lambda: ops.attention_paged(q, kp, vp, o, NH, KV, T, T, page_table=table, mode=2,  # noqa
                                         t_index=td)
    elif case == "attention":
        npg = (TK + 63) // 64
        q = torch.randn(NH, M_TOK, HD, device="cuda", generator=g).bfloat16()
        kp = torch.randn(npg, KV, 64, HD, device="cuda", generator=g).bfloat16()
        vp = torch.randn(npg, KV, HD, 64, device="cuda", generator=g).bfloat16()
        table = torch.arange(npg, dtype=torch.int32, device="cuda")
        o = torch.empty(M_TOK, NH * HD, device="cuda").bfloat16()
        ws = ops.sage_workspace(NH, KV, M_TOK, TK)
        state = {"i": 0}

        def fn():   # bf16 and Sage launches alternate
            ops.attention_paged(q, kp, vp, o, NH, KV, M_TOK, TK, page_table=table,
                                sage_ws=ws if state["i"] % 2 else None)
            state["i"] += 1
    else:
        m = u15b200.Model(int8=True, n_layers=1)
        m.bind_random(seed=1234, std=0.02, norm_mean=1.0, norm_std=0.2)
        m.finalize()
        kv = m.make_cache(TK)
        for v in (False, True):
            kv.write(0, v, torch.randn(KV, N_PRE, HD, device="cuda", generator=g).bfloat16())
        pos = [torch.from_numpy(p).cuda() for p in positions()]
        x = torch.randn(M_TOK, H, device="cuda", generator=g).bfloat16()
        segs = [(0, N_UND, 0), (N_UND, M_TOK, 1)]
        state = {"i": 0}

        def fn():   # bf16 and W8A8 layers alternate
            m.layer_forward(0, x, kv, N_PRE, TK, *pos, segments=segs, int8=state["i"] % 2 == 1)
            state["i"] += 1
    fn()
    torch.cuda.synchronize()
    return ev_time(fn, steps)


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p["hbm_gbs"], p["bf16_tflops"], "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


def sustained_bf16_peak():
    """cuBLAS bf16 held for seconds under the 1 kW power cap (TFLOP/s)."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["bf16_tflops_sustained"])
    except Exception:
        return 1400.0


def positions():
    pt = np.concatenate([N_PRE + np.arange(N_UND), np.full(M_TOK - N_UND, N_PRE + N_UND)])
    gh, gw = 56, 64
    ph = np.concatenate([np.zeros(N_UND), np.repeat(np.arange(gh), gw)])
    pw = np.concatenate([np.zeros(N_UND), np.tile(np.arange(gw), gh)])
    return [a.astype(np.int32) for a in (pt, ph, pw)]


class Clocks:
    """nvidia-smi sampled every 200 ms while the bench runs; samples carry
    the host time, so the clock seen inside one timed window can be read
    back (window())."""
    Q = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, dev):
        self.dev = dev
        self.p = None

    def __enter__(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv",
                                       "-lms", "200", "-i", str(self.dev)],
                                      stdout=subprocess.PIPE, stderr=subprocess.DEVNULL,
                                      text=True)
        except Exception:
            self.p = None
        return self

    def __exit__(self, *a):
        self.out = ""
        if self.p is not None:
            self.p.terminate()
            try:
                self.out, _ = self.p.communicate(timeout=5)
            except Exception:
                self.p.kill()

    def _rows(self):
        import datetime
        out = []
        for r in list(csv.reader(io.StringIO(getattr(self, "out", "") or "")))[1:]:
            if len(r) < 10:
                continue
            try:
                ts = datetime.datetime.strptime(r[0].strip(), "%Y/%m/%d %H:%M:%S.%f").timestamp()
                out.append((ts, float(r[2].split()[0]), float(r[3].split()[0]),
                            float(r[4].split()[0]), r[6:10]))
            except (ValueError, IndexError):
                continue
        return out

    def summary(self):
        """Median SM clock over samples under load (power above 40% of the
        peak seen), the max clock, and every throttle reason seen active."""
        rows = self._rows()
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        for r in rows:
            for n, v in zip(names, r[4]):
                if "Active" in v and "Not" not in v:
                    reasons.add(n)
        pw = [r[3] for r in rows]
        load = [r[1] for r in rows if r[3] > 0.4 * max(pw)]
        return {"sm_mhz": float(np.median(load)) if load else None, "sm_max_mhz": rows[-1][2],
                "reasons": sorted(reasons), "samples": len(rows), "samples_under_load": len(load),
                "window": "whole bench (model set-up, warm-up, every timed loop)"}

    def window(self, t0, t1):
        """Median SM clock and mean power of the samples taken in [t0, t1]
        (host time)."""
        w = [r for r in self._rows() if t0 <= r[0] <= t1]
        if not w:
            return {"sm_mhz": None, "power_w": None, "samples": 0}
        return {"sm_mhz": float(np.median([r[1] for r in w])),
                "power_w": float(np.mean([r[3] for r in w])), "samples": len(w)}


def ev_time(fn, n, stream=None):
    """Average ms of fn() over n runs, CUDA events on the current stream."""
    import torch
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    s.record()
    for _ in range(n):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / n


# ---------------------------------------------------------------------------
# CPU baseline: the reference's own u15-ref (or the restatement) row-sharded
# ---------------------------------------------------------------------------
class CpuLayer:
    """ms per MoT layer @4096 tok from a bounded sample of rows: ref::linear
    over the seven projections and ref::attention for the sampled queries,
    rows sharded over threads (rows are independent, results identical)."""

    def __init__(self, threads, rows):
        import ctypes as C
        from oracle import oracle as O
        self.C = C
        if O.ref_available():
            self.kind, L = "reference", O.ref()
            self.lin, self.att = L.refx_linear, L.refx_attention
        else:
            self.kind, L = "port", O.lib()
            self.lin = L.orc_linear
            self.att = None
            self.O = O
        self.threads, self.rows = threads, rows
        rng = np.random.default_rng(0)
        f = lambda *s: (rng.standard_normal(s, dtype=np.float32) * 0.02)  # noqa: E731
        self.W = {"q": f(NH * HD, H), "k": f(KV * HD, H), "v": f(KV * HD, H), "o": f(H, NH * HD),
                  "gate": f(I, H), "up": f(I, H), "down": f(H, I)}
        self.x = rng.standard_normal((rows, max(H, I)), dtype=np.float32)
        self.q = rng.standard_normal((NH, rows, HD), dtype=np.float32)
        self.k = rng.standard_normal((KV, TK, HD), dtype=np.float32)
        self.v = rng.standard_normal((KV, TK, HD), dtype=np.float32)

    def _shard(self, fn):
        n = self.rows
        parts = [(i * n // self.threads, (i + 1) * n // self.threads) for i in range(self.threads)]
        ts = [threading.Thread(target=fn, args=p) for p in parts if p[1] > p[0]]
        for t in ts:
            t.start()
        for t in ts:
            t.join()

    def step(self):
        C = self.C
        fp = lambda a: a.ctypes.data_as(C.POINTER(C.c_float))  # noqa: E731
        t0 = time.perf_counter()
        for name, w in self.W.items():
            kin = w.shape[1]

            def run(a, b, w=w, kin=kin):
                xs = np.ascontiguousarray(self.x[a:b, :kin])
                out = np.empty((b - a, w.shape[0]), np.float32)
                self.lin(fp(xs), fp(w), None, b - a, kin, w.shape[0], fp(out))
            self._shard(run)

        def att(a, b):
            qs = np.ascontiguousarray(self.q[:, a:b])
            out = np.empty((b - a, NH * HD), np.float32)
            if self.att is not None:
                self.att(fp(qs), fp(self.k), fp(self.v), None, NH, KV, b - a, TK, HD, fp(out))
            else:
                self.O.lib().orc_attention(fp(qs), fp(self.k), fp(self.v), NH, KV, b - a, TK,
                                           HD, TK, 0, 0, None, fp(out))
        self._shard(att)
        self.last_sample_ms = (time.perf_counter() - t0) * 1e3
        return self.last_sample_ms * (M_TOK / self.rows)   # extrapolated ms per layer

    def describe(self):
        return (f"{self.rows} of 4096 token rows through all seven projections and "
                f"attention over {TK} keys, extrapolated x{M_TOK // self.rows}; "
                f"u15::ref::linear/attention row-sharded over {self.threads} threads")


def run_reference(args, rank, world):
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    cpu = CpuLayer(threads, rows=max(32, 2 * threads))
    for _ in range(args.warmup):
        cpu.step()
    vals, raw = [], []
    for _ in range(args.steps):
        vals.append(cpu.step())
        raw.append(cpu.last_sample_ms)
    v = float(np.median(vals))
    # a step is the bounded sample (its measured time); value extrapolates it
    # to the whole 4096-token layer
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": float(np.median(raw)),
            "extrapolation": f"x{M_TOK // cpu.rows} (sampled rows -> 4096)",
            "higher_is_better": False, "scaling": "weak", "vs_baseline": v / PUBLISHED_MS,
            "dtype": "f32", "data": "synthetic",
            "config": bench_config(world),
            "cpu_baseline": {"value": v, "unit": UNIT, "cores": threads, "kind": cpu.kind,
                             "sample": cpu.describe()},
            "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def run_ours(args, rank, world, local):
    import torch
    import u15b200

    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    clk = Clocks(local).__enter__()
    n_layers = args.layers
    m = u15b200.Model(int8=True, n_layers=n_layers)
    m.bind_random(seed=1234 + rank, std=0.02, norm_mean=1.0, norm_std=0.2)
    m.finalize()
    kv = m.make_cache(TK)
    g = torch.Generator(device="cuda").manual_seed(99 + rank)
    for li in range(n_layers):
        kv.write(li, False, torch.randn(KV, N_PRE, HD, device="cuda", generator=g).bfloat16())
        kv.write(li, True, torch.randn(KV, N_PRE, HD, device="cuda", generator=g).bfloat16())
    pos = [torch.from_numpy(p).cuda() for p in positions()]
    segs = [(0, N_UND, 0), (N_UND, M_TOK, 1)]
    x0 = torch.randn(M_TOK, H, device="cuda", generator=g).bfloat16()
    x = x0.clone()
    state = {"i": 0}

    def step(int8=False, sage=False):
        li = state["i"] % n_layers
        state["i"] += 1
        m.layer_forward(li, x, kv, N_PRE, TK, *pos, segments=segs, int8=int8, sage=sage)

    ops = u15b200.CudaOps(local)
    for _ in range(args.warmup):
        step()
    ops.sync()
    x.copy_(x0)

    # ---- timed region: K layer steps, bf16 ----
    def timed(fn, k, tail=None):
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(k):
            fn()
        if tail is not None:
            tail()
        e.record()
        torch.cuda.synchronize()
        ms = s.elapsed_time(e)
        if dist is not None:
            t = torch.tensor([ms], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
            dist.barrier()
        return ms

    win = {}
    t0 = time.time()
    total_ms = timed(step, args.steps)
    win["burst"] = (t0, time.time())
    ops.sync()
    ms_step = total_ms / args.steps
    value = ms_step / world
    # rope tables, norm, QKV, qkv_post, attention, O, norm, gate+up, down; the
    # attention takes a second launch when its last round of 256-row units is
    # at most half full (the library's rule, U15_ATTN_SPLIT=0 turns it off)
    sms = torch.cuda.get_device_properties(local).multi_processor_count
    units = (M_TOK // 256) * NH
    split = (os.environ.get("U15_ATTN_SPLIT", "1") != "0" and M_TOK % 256 == 0 and
             units > sms and 0 < units % sms <= sms // 2)
    launches_per_layer = 9 + int(split)


    # ---- W8A8 and Sage variants (same loop, same rules) ----
    for _ in range(args.warmup):
        step(int8=True)
    x.copy_(x0)
    ms_i8 = timed(lambda: step(int8=True), args.steps) / args.steps
    for _ in range(args.warmup):
        step(int8=True, sage=True)
    x.copy_(x0)
    ms_i8_sage = timed(lambda: step(int8=True, sage=True), args.steps) / args.steps
    ops.sync()

    # ---- e2e through the C ABI with host buffers (H2D + layer + D2H) ----
    xh = x0.cpu().pin_memory()
    oh = torch.empty_like(xh).pin_memory()

    def e2e_step():
        li = state["i"] % n_layers
        state["i"] += 1
        m.layer_forward_host(li, xh, oh, kv, N_PRE, TK, *pos, segments=segs)
    for _ in range(args.warmup):
        e2e_step()
    ms_e2e_sync = timed(e2e_step, args.steps) / args.steps

    # The serving loop's form: the same call enqueued back to back through
    # u15c_layer_forward_host_async (two device staging buffers in turn, the
    # uploads and downloads on their own streams). Every step still uploads
    # its 32 MB input from pinned host memory and downloads its 32 MB result
    # inside the timed region; the downloads are drained into the timed
    # stream before the closing event.
    ohs = [oh, torch.empty_like(xh).pin_memory()]

    def e2e_async_step():
        li = state["i"] % n_layers
        state["i"] += 1
        m.layer_forward_host_async(li, xh, ohs[state["i"] % 2], kv, N_PRE, TK, *pos,
                                   segments=segs)
    for _ in range(args.warmup):
        e2e_async_step()
    m.host_drain()
    ops.sync()
    ms_e2e = timed(e2e_async_step, args.steps, tail=m.host_drain) / args.steps

    # ---- per-kernel timing on the launching stream (dominant: gate_up) ----
    hbm, bf16_peak, peak_kind = peaks()
    kern = {}
    i8_peak = None
    prefill = None
    if rank == 0:
        i8_peak = int8_reference_rate()
        prefill = prefill_bench(ops, max(5, args.steps))
        xa = torch.randn(M_TOK, I, device="cuda").bfloat16()
        for name, (K, N) in GEMMS.items():
            w = (torch.randn(2, N, K, device="cuda") * 0.02).bfloat16()
            epi = {"gate_up": 2, "o": 1, "down": 1}.get(name, 0)
            y = torch.empty(M_TOK, N // 2 if epi == 2 else N, device="cuda").bfloat16()
            xin = xa[:, :K].contiguous()
            fn = lambda: ops.mot_linear(xin, w, segs, y, M_TOK, K, N, epilogue=epi,  # noqa
                                        resid=y if epi == 1 else None)
            for _ in range(3):
                fn()
            t = ev_time(fn, max(5, args.steps))
            kern[name] = {"ms": t, "tflops": 2.0 * M_TOK * K * N / t / 1e9}
            del w, y, xin
        # the W8A8 projections (int8 x int8 -> int32, dequant epilogue)
        xq = torch.randint(-127, 128, (M_TOK, I), device="cuda", dtype=torch.int8)
        st_ = torch.rand(M_TOK, device="cuda") * 0.01
        for name, (K, N) in GEMMS.items():
            wq = torch.randint(-127, 128, (2, N, K), device="cuda", dtype=torch.int8)
            sc = torch.rand(2, N, device="cuda") * 0.001
            epi = {"gate_up": 2, "o": 1, "down": 1}.get(name, 0)
            y = torch.zeros(M_TOK, N // 2 if epi == 2 else N, device="cuda").bfloat16()
            xin = xq[:, :K].contiguous()
            fn = lambda: ops.mot_linear_i8(xin, st_, wq, sc, segs, y, M_TOK, K, N,  # noqa
                                           epilogue=epi, resid=y if epi == 1 else None)
            for _ in range(3):
                fn()
            t = ev_time(fn, max(5, args.steps))
            kern["i8_" + name] = {"ms": t, "tflops": 2.0 * M_TOK * K * N / t / 1e9,
                                  "unit": "TOP/s"}
            del wq, y, xin
        q = torch.randn(NH, M_TOK, HD, device="cuda").bfloat16()
        npg = (TK + 63) // 64
        kp = torch.randn(npg, KV, 64, HD, device="cuda").bfloat16()
        vp = torch.randn(npg, KV, HD, 64, device="cuda").bfloat16()
        table = torch.arange(npg, dtype=torch.int32, device="cuda")
        o = torch.empty(M_TOK, NH * HD, device="cuda").bfloat16()
        fn = lambda: ops.attention_paged(q, kp, vp, o, NH, KV, M_TOK, TK,  # noqa: E731
                                         page_table=table)
        fn()
        t = ev_time(fn, max(5, args.steps))
        kern["attention"] = {"ms": t, "tflops": ATTN_FLOP / t / 1e9,
                             "kernel": "attn_tc_kernel (tcgen05, paged KV)"}
        ws = ops.sage_workspace(NH, KV, M_TOK, TK)
        fn = lambda: ops.attention_paged(q, kp, vp, o, NH, KV, M_TOK, TK,  # noqa: E731
                                         page_table=table, sage_ws=ws)
        fn()
        t = ev_time(fn, max(5, args.steps))
        kern["attention_sage"] = {"ms": t, "tflops": ATTN_FLOP / t / 1e9,
                                  "kernel": "Sage prologue + attn_tc_kernel<int8 QK>"}
        kc = torch.randn(KV, TK, HD, device="cuda").bfloat16()
        vc = torch.randn(KV, TK, HD, device="cuda").bfloat16()
        fn = lambda: ops.attention(q, kc, vc, o, NH, KV, M_TOK, TK, cap=TK)  # noqa: E731
        fn()
        t = ev_time(fn, max(5, args.steps))
        kern["attention_mma_sync_reference_layout"] = {"ms": t, "tflops": ATTN_FLOP / t / 1e9}
        torch.cuda.empty_cache()

    # ---- the bf16 layer loop held for seconds: the clock a render settles at ----
    # (the burst windows above are tens of ms each; a denoise step streams 126
    # layers). Last of the layer measurements, so its heat reaches none of them.
    n_long = max(args.steps, int(np.ceil(args.sustained_s * 1e3 / ms_step)))
    x.copy_(x0)
    t0 = time.time()
    ms_long = timed(step, n_long) / n_long
    win["sustained"] = (t0, time.time())
    x.copy_(x0)

    # ---- one render over all ranks: tensor parallelism (N > 1) ----
    tp = None
    if world > 1:
        del m, kv
        torch.cuda.empty_cache()
        tp = tp_bench(args, rank, world, dist, timed, pos, segs, x0)
        tp["speedup_vs_one_gpu"] = ms_step / tp["ms_per_layer_fused"]

    # ---- the image path of one branch (rank 0) ----
    img_line = image_bench(max(5, min(args.steps, 20))) if rank == 0 else None

    # ---- denoise steps/s (BASELINE config 5 geometry), one replica per rank ----
    den = None
    if args.denoise_steps > 0:
        if world == 1:
            del m, kv
        torch.cuda.empty_cache()
        # the one-image tensor-parallel denoise uses the row-parallel reduction
        # the layer measurement above found faster at this rank count
        nccl_faster = tp is not None and (tp["ms_per_layer_nccl"] < tp["ms_per_layer_fused"] or
                                          os.environ.get("U15_TP_NCCL") == "1")
        den = denoise_bench(args, rank, world, dist, tp_nccl=nccl_faster)
    clk.__exit__(None, None, None)

    # ---- CPU baseline (rank 0, N=1 only): bounded sample, ~10-30 s ----
    cpu_line = None
    if rank == 0 and world == 1 and not args.no_cpu:
        threads = os.cpu_count() or 1
        cpu = CpuLayer(threads, rows=max(32, 2 * threads))
        cpu.step()
        vals = [cpu.step() for _ in range(3)]
        cpu_line = {"value": float(np.median(vals)), "unit": UNIT, "cores": threads,
                    "kind": cpu.kind, "sample": cpu.describe() + "; median of 3"}

    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    gu = kern.get("gate_up", {})
    traffic = None
    tf = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(tf):
        try:
            traffic = json.load(open(tf)).get("gemm_gate_up_bytes_per_launch")
        except Exception:
            traffic = None
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": False,
        "scaling": "weak", "vs_baseline": value / PUBLISHED_MS, "dtype": "bf16",
        "data": "synthetic",
        "config": bench_config(world),
        "tflops_per_gpu": LAYER_FLOP / ms_step / 1e9,
        "i8": {"ms_per_layer": ms_i8 / world, "ms_per_step": ms_i8,
               "sage_ms_per_step": ms_i8_sage,
               "roofline": i8_roofline(kern, i8_peak)},
        "sustained": {"ms_per_layer": ms_long / world, "ms_per_step": ms_long, "steps": n_long,
                      "seconds": n_long * ms_long / 1e3,
                      "tflops": LAYER_FLOP / ms_long / 1e9,
                      "frac_of_sustained_bf16_peak": LAYER_FLOP / ms_long / 1e9 /
                      sustained_bf16_peak(),
                      "clock": clk.window(*win["sustained"]),
                      "note": "the burst line's loop held for >= %.1f s (same layers, same "
                              "inputs); frac against the sustained (power-capped) cuBLAS bf16 "
                              "rate in MEASURED_PEAKS.json" % args.sustained_s},
        "prefill": prefill,
        "e2e": {"value": ms_e2e / world, "unit": UNIT,
                "h2d_bytes_per_step": M_TOK * H * 2, "d2h_bytes_per_step": M_TOK * H * 2,
                "api": "u15c_layer_forward_host_async, calls back to back, drained at the end",
                "sync_value": ms_e2e_sync / world,
                "sync_api": "u15c_layer_forward_host (returns after its download)"},
        "gpu_launches": launches_per_layer * args.steps,
        "roofline": {"bound": "tensor", "kernel": "gemm_tc (gate_up, routed, SwiGLU epilogue)",
                     "achieved": gu.get("tflops"), "peak": bf16_peak, "unit": "TFLOP/s",
                     "frac": (gu.get("tflops") or 0) / bf16_peak, "traffic": traffic,
                     "peak_kind": f"{peak_kind} burst bf16",
                     "frac_sustained": (gu.get("tflops") or 0) / sustained_bf16_peak()},
        "kernels": kern,
        "tensor_parallel": tp,
        "denoise": den,
        "image_path": img_line,
        "clocks": clk.summary(),
        "cpu_baseline": cpu_line,
    }
    print(json.dumps(line), flush=True)


def tp_bench(args, rank, world, dist, timed, pos, segs, x0):
    """The same layer workload as ONE render split over all ranks (tensor
    parallelism: q/k/v heads, KV cache and gate/up by rank; o_proj and
    down_proj row-parallel). Two forms of the row-parallel reduction: the
    fused GEMM + reduction over NVLink peer memory (the product) and the
    GEMM followed by NCCL all_reduce (the baseline). ms per layer is the
    max over ranks of CUDA-event time."""
    import torch
    import u15b200
    out = {"ranks": world, "workload": "the layer above, one copy split over all ranks"}
    for form in ("nccl", "fused"):
        m = u15b200.Model(int8=True, n_layers=args.layers, tp_rank=rank, tp_size=world)
        m.bind_random(seed=4321, std=0.02, norm_mean=1.0, norm_std=0.2)
        m.finalize()
        if form == "fused":
            m.tp_connect(None, M_TOK)
        else:
            m.set_allreduce(None, M_TOK)
        kv = m.make_cache(TK)
        g = torch.Generator(device="cuda").manual_seed(7 + rank)
        for li in range(args.layers):
            for v in (False, True):
                kv.write(li, v, torch.randn(KV // world, N_PRE, HD, device="cuda",
                                            generator=g).bfloat16())
        x = x0.clone()
        state = {"i": 0}

        def step(int8=False):
            li = state["i"] % args.layers
            state["i"] += 1
            m.layer_forward(li, x, kv, N_PRE, TK, *pos, segments=segs, int8=int8)

        for int8 in (False, True):
            for _ in range(args.warmup):
                step(int8)
            torch.cuda.synchronize()
            x.copy_(x0)
            ms = timed(lambda: step(int8), args.steps) / args.steps
            out[f"ms_per_layer_{form}" + ("_i8" if int8 else "")] = ms
        torch.cuda.synchronize()
        if form == "fused":
            m.tp_disconnect(None)
        del kv
        m.close()
        del m
        torch.cuda.empty_cache()
    return out


IMG_FLOP = {"patch": 2.0 * 16384 * 1024 * 768, "dense": 2.0 * 4096 * 4096 * 4096,
            "conv1": 2.0 * 16384 * 1024 * 9216, "conv2": 2.0 * 65536 * 192 * 2304}


def image_bench(steps):
    """The device image path of one CFG branch at the denoise geometry
    (2048 x 2048 px, 4096 tokens): patchify + patch embedder (patch GEMM,
    GELU / 2-D RoPE / merge, dense GEMM) and the pixel head (PS(2), im2col,
    conv1 GEMM, GELU + PS(2), im2col, conv2 GEMM, PS(8)). Seeded random
    weights and inputs; CUDA events, inputs resident."""
    import torch
    import u15b200
    im = u15b200.ImagePath()
    im.bind_random(seed=3)
    g = torch.Generator(device="cuda").manual_seed(11)
    img = torch.randn(2048, 2048, 3, device="cuda", generator=g)
    h = torch.randn(4096, 4096, device="cuda", generator=g).bfloat16()
    emb = torch.empty(4096, 4096, device="cuda", dtype=torch.bfloat16)
    dec = torch.empty(2048, 2048, 3, device="cuda", dtype=torch.float32)

    def embed():
        im.embed(im.patchify(img), 128, 128, gen=True, out=emb)

    def decode():
        im.decode(h, 64, 64, out=dec)
    for _ in range(3):
        embed()
        decode()
    t_e = ev_time(embed, steps)
    t_d = ev_time(decode, steps)
    im.close()
    fe = IMG_FLOP["patch"] + IMG_FLOP["dense"]
    fd = IMG_FLOP["conv1"] + IMG_FLOP["conv2"]
    return {"embed_ms": t_e, "decode_ms": t_d, "embed_tflops": fe / t_e / 1e9,
            "decode_tflops": fd / t_d / 1e9,
            "config": "one branch at 2048x2048 px / 4096 tokens; embed = patchify + patch "
                      "embedder (25.8 + 137.4 GFLOP), decode = pixel head (309.2 + 58.0 GFLOP)"}


def denoise_bench(args, rank, world, dist, tp_nccl=False):
    """Denoise steps/s at BASELINE config 5's geometry: 42 layers (random
    N(0, 0.02) weights, both experts), 4096 generation tokens (64x64 token
    grid, 2048x2048 px), three CFG forwards per step -- text-conditional
    (320-token prefix), image-conditional (8 text + one 1024-token reference
    image, block-causal prefill) and unconditional (13 tokens) -- shift 3.0,
    cfg 4.0, img_cfg 1.5. The image path is the device ImagePath (patch
    embedder, timestep + noise-scale row, pixel head) with seeded weights.

    Four placements (N > 1; at N = 1 only the first):
      replicas    every rank runs its own seed: job steps/s = N / max-over-ranks s/step
      branches    ONE image, its three CFG branches placed round-robin over the
                  ranks, one velocity all-gather per step (NCCL)
      tensor_par  ONE image, every branch on all ranks, the model split by
                  tensor parallelism (fused row-parallel reduction over NVLink)
      hybrid      ONE image, its branches over tensor-parallel groups of ranks
                  (plan_groups; at 6 and 8 ranks three two-rank groups), run
                  where the plan differs from the two above
    """
    import torch
    import u15b200
    from u15b200 import _lib as L
    from u15b200.generator import Branch, Generator, plan_groups

    def specs_on(seed):
        g = torch.Generator(device="cuda").manual_seed(seed)

        def pre(n_text, n_img):
            n = n_text + n_img
            x = torch.randn(n, H, device="cuda", generator=g).bfloat16()
            t = np.concatenate([np.arange(n_text), np.full(n_img, n_text)]).astype(np.int32)
            h = np.concatenate([np.zeros(n_text), np.arange(n_img) // 32]).astype(np.int32)
            w = np.concatenate([np.zeros(n_text), np.arange(n_img) % 32]).astype(np.int32)
            return x, t, h, w
        specs = [("cond", pre(320, 0), False), ("img_cond", pre(8, 1024), True),
                 ("uncond", pre(13, 0), False)]
        return [Branch(nm, x, t, h, w, block_causal=bc) for nm, (x, t, h, w), bc in specs]

    def run(gen, branches, seed, int8=False, sage=False):
        evs = []

        def cb(step, img):
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            evs.append(e)
        if dist is not None:
            dist.barrier()
        gen.generate(branches, 2048, 2048, steps=1 + args.denoise_steps, shift=3.0, cfg=4.0,
                     icfg=1.5, form=L.CFG_BOTH, i_img=1, i_unc=2, seed=seed, step_callback=cb,
                     int8=int8, sage=sage)
        torch.cuda.synchronize()
        sps = evs[0].elapsed_time(evs[-1]) / 1e3 / args.denoise_steps
        if dist is not None:
            t = torch.tensor([sps], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            sps = float(t.item())
        return sps

    # bf16 weights and their per-channel int8 twin (BASELINE config 4 times both)
    m = u15b200.Model(int8=True, n_layers=42)
    m.bind_random(seed=77, std=0.02, norm_mean=1.0, norm_std=0.2)
    for e in range(2):
        m.bind(0, e, "final_norm", torch.ones(H, device="cuda"))
    m.finalize()
    s_rep = run(Generator(m), specs_on(5 + rank), rank)
    s_rep8 = run(Generator(m), specs_on(5 + rank), rank, int8=True)
    # the W8A8 twin with Sage int8 QK on the bidirectional denoise passes
    s_rep8s = run(Generator(m), specs_on(5 + rank), rank, int8=True, sage=True)
    out = {"steps_per_s": world / s_rep, "s_per_step_per_replica": s_rep,
           "steps_per_s_i8": world / s_rep8, "s_per_step_per_replica_i8": s_rep8,
           "steps_per_s_i8_sage": world / s_rep8s, "s_per_step_per_replica_i8_sage": s_rep8s,
           "timed_steps": args.denoise_steps, "warmup_steps": 1,
           "config": "42 layers, 4096 gen tokens (BASELINE '1024^2' = 64x64 tokens = 2048^2 px),"
                     " 3 CFG forwards/step (prefix 320 / 8+1024 img block-causal / 13),"
                     " device image path (patch embedder, timestep + noise-scale row,"
                     " pixel head; seeded weights), replicas x%d" % world,
           "layers_per_step": 3 * 42}
    if world > 1:
        # one image, branches over the ranks (same weights and inputs everywhere)
        s_br = run(Generator(m, group=dist.group.WORLD), specs_on(5), 0)
        out["one_image_branch_placement"] = {"steps_per_s": 1.0 / s_br, "s_per_step": s_br,
                                             "branches_per_rank": -(-3 // world)}
        del m
        torch.cuda.empty_cache()
        # one image, tensor parallelism over all ranks
        mt = u15b200.Model(n_layers=42, tp_rank=rank, tp_size=world)
        mt.bind_random(seed=77, std=0.02, norm_mean=1.0, norm_std=0.2)
        for e in range(2):
            mt.bind(0, e, "final_norm", torch.ones(H, device="cuda"))
        if tp_nccl:
            mt.set_allreduce(None, 3 * M_TOK)
        else:
            mt.tp_connect(None, 3 * M_TOK)
        s_tp = run(Generator(mt), specs_on(5), 0)
        out["one_image_tensor_parallel"] = {
            "steps_per_s": 1.0 / s_tp, "s_per_step": s_tp, "tp": world,
            "reduction": "NCCL all-reduce" if tp_nccl else "fused, peer memory"}
        torch.cuda.synchronize()
        if not tp_nccl:
            mt.tp_disconnect(None)
        mt.close()
        del mt
        torch.cuda.empty_cache()
        # one image, hybrid: the branches over tensor-parallel groups of ranks
        # (plan_groups), where that differs from both placements above
        plan = plan_groups(3, world)
        sizes = [len(g.ranks) for g in plan]
        if max(sizes) > 1 and not (len(plan) == 1 and sizes[0] == world):
            subs = [dist.new_group(g.ranks) for g in plan]   # every rank, same order
            mine = [i for i, g in enumerate(plan) if rank in g.ranks]
            mh = None
            if mine:
                g, sub = plan[mine[0]], subs[mine[0]]
                mh = u15b200.Model(n_layers=42, tp_rank=g.ranks.index(rank),
                                   tp_size=len(g.ranks))
                mh.bind_random(seed=77, std=0.02, norm_mean=1.0, norm_std=0.2)
                for e in range(2):
                    mh.bind(0, e, "final_norm", torch.ones(H, device="cuda"))
                if len(g.ranks) > 1:
                    mh.tp_connect(sub, 3 * M_TOK)
            s_hy = run(Generator(mh, group=dist.group.WORLD, groups=plan), specs_on(5), 0)
            out["one_image_hybrid"] = {
                "steps_per_s": 1.0 / s_hy, "s_per_step": s_hy,
                "groups": [{"ranks": g.ranks, "branches": g.branches} for g in plan],
                "reduction": "fused, peer memory, within each group"}
            torch.cuda.synchronize()
            if mh is not None:
                if len(plan[mine[0]].ranks) > 1:
                    mh.tp_disconnect(subs[mine[0]])
                mh.close()
            dist.barrier()
    else:
        del m
    torch.cuda.empty_cache()
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--layers", type=int, default=4)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--denoise-steps", type=int, default=3,
                    help="timed denoise steps after one warm-up step (0: skip)")
    ap.add_argument("--image-only", action="store_true",
                    help="time only the image path of one branch (a small case for profiling)")
    ap.add_argument("--sustained-s", type=float, default=LONG_WINDOW_S,
                    help="length of the sustained layer window (0: --steps layers only)")
    ap.add_argument("--case", choices=["prefill", "attention", "layer"],
                    help="one small workload for a profiler, then exit: the C4 prefill "
                         "attention (block-causal, tcgen05), the bidirectional attention at "
                         "4096 x 4416 (bf16 then Sage), or --steps bf16 + W8A8 layers")
    args = ap.parse_args()
    if args.image_only:
        import torch
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", 0)))
        print(json.dumps({"image_path": image_bench(max(1, args.steps))}))
        return
    if args.case:
        import torch
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", 0)))
        print(json.dumps({"case": args.case, "ms": profile_case(args.case, max(1, args.steps))}))
        return
    args.warmup = max(args.warmup, 3)
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    if args.impl == "reference":
        run_reference(args, rank, world)
    else:
        run_ours(args, rank, world, local)


if __name__ == "__main__":
    main()
