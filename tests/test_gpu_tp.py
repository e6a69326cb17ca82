"""Tensor parallelism (one render over two GPUs): q/k/v heads, the KV cache
and gate/up split column-wise, o_proj and down_proj row-wise with an
all-reduce of the f32 partial products (NCCL through torch.distributed).
Two spawned ranks bind the same full weights; their outputs must be equal,
match the CPU restatement of the layer (same bars as the one-GPU layer
tests) and match a one-GPU model on the same weights. Both forms of the
row-parallel reduction are checked: the all-reduce hook (NCCL) and the
fused GEMM + reduction over peer memory."""
import os
import socket
from datetime import timedelta

import numpy as np
import pytest

from gpu_util import bf16_round, dev_bf16, dev_i32, host, randn, rel_l2, torch

pytestmark = pytest.mark.gpu

TPCFG = dict(n_layers=2, hidden=512, heads=4, kv_heads=2, head_dim=128, inter=1024,
             n_experts=2)
N_UND, GH, GW = 32, 8, 12


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _inputs():
    from test_gpu_layer import grid_positions
    T = N_UND + GH * GW
    segs = [(0, N_UND, 0), (N_UND, T, 1)]
    pos = grid_positions(N_UND, GH, GW, N_UND)
    x = bf16_round(randn((T, TPCFG["hidden"]), 41))
    return T, segs, pos, x


def _bind(m, cfg, seed):
    from test_gpu_layer import expert_weights
    W = [[expert_weights(cfg, seed + 100 * li + e) for e in range(cfg["n_experts"])]
         for li in range(cfg["n_layers"])]
    for li in range(cfg["n_layers"]):
        for e in range(cfg["n_experts"]):
            m.bind_expert_layer(li, e, W[li][e])
    for e in range(cfg["n_experts"]):
        m.bind(0, e, "final_norm", np.ones(cfg["hidden"], np.float32))
    m.finalize()
    return W


def _tp_worker(rank, world, port, q, fused=False):
    import torch.distributed as dist
    import u15b200
    torch.cuda.set_device(rank)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        T, segs, pos, x = _inputs()
        m = u15b200.Model(tp_rank=rank, tp_size=world, **TPCFG)
        _bind(m, TPCFG, 1)
        if fused:
            m.tp_connect(None, T)
        else:
            m.set_allreduce(None, T)
        pd = [dev_i32(p) for p in pos]
        kv = m.make_cache(T)
        xd = dev_bf16(x)
        m.layer_forward(0, xd, kv, 0, T, *pd, segments=segs)
        torch.cuda.synchronize()
        layer_out, k0 = host(xd), host(kv.read(0, False, T))
        xd2 = dev_bf16(x)
        kv2 = m.make_cache(T)
        m.forward(xd2, kv2, 0, T, *pd, segments=segs)
        torch.cuda.synchronize()
        q.put((rank, layer_out, k0, host(xd2)))
        if fused:
            m.tp_disconnect(None)
        dist.barrier()
        m.close()
    finally:
        dist.destroy_process_group()


def _run_ranks(fused):
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_tp_worker, args=(r, 2, port, q, fused)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=300) for _ in procs], key=lambda r: r[0])
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    return res


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two visible GPUs")
@pytest.mark.parametrize("fused", [False, True], ids=["nccl_hook", "fused_peer"])
def test_tp2_layer_and_stack(fused):
    import u15b200
    from oracle import oracle as O
    from test_gpu_layer import check_layer, dims_of
    (_, l0, k0, f0), (_, l1, k1, f1) = _run_ranks(fused)
    # the all-reduce hands every rank the same sums: replicas stay identical
    assert np.array_equal(l0, l1) and np.array_equal(f0, f1)
    T, segs, pos, x = _inputs()
    # one-GPU model on the same weights, for the layer and the stack
    m = u15b200.Model(**TPCFG)
    W = _bind(m, TPCFG, 1)
    pd = [dev_i32(p) for p in pos]
    kv = m.make_cache(T)
    xd = dev_bf16(x)
    m.forward(xd, kv, 0, T, *pd, segments=segs)
    torch.cuda.synchronize()
    assert rel_l2(f0, host(xd)) < 1e-2
    # layer 0 against the CPU restatement; rank r holds kv head r
    ref, kn, _ = O.mot_layer(x, segs, W[0], dims_of(TPCFG), *pos)
    check_layer(l0, x, ref)
    assert rel_l2(np.concatenate([k0, k1]), kn) < 1e-2
    assert rel_l2(k0, kn[:1]) < 1e-2 and rel_l2(k0, kn[1:]) > 1e-1   # negative control
