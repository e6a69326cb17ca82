"""Tensor parallelism (one render over two or four GPUs): q/k/v heads, the
KV cache and gate/up split column-wise, o_proj and down_proj row-wise with an
all-reduce of the f32 partial products (NCCL through torch.distributed).
Spawned ranks bind the same full weights; their outputs must be equal,
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
# four ranks: one kv head, two q heads and 512 of the MLP's columns per rank;
# hidden 1024 gives every rank one 256-column block of the fused reduction
TPCFG4 = dict(n_layers=2, hidden=1024, heads=8, kv_heads=4, head_dim=128, inter=2048,
              n_experts=2)
CFGS = {2: TPCFG, 4: TPCFG4}
N_UND, GH, GW = 32, 8, 12


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _inputs(cfg):
    from test_gpu_layer import grid_positions
    T = N_UND + GH * GW
    segs = [(0, N_UND, 0), (N_UND, T, 1)]
    pos = grid_positions(N_UND, GH, GW, N_UND)
    x = bf16_round(randn((T, cfg["hidden"]), 41))
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
        cfg = CFGS[world]
        T, segs, pos, x = _inputs(cfg)
        m = u15b200.Model(tp_rank=rank, tp_size=world, **cfg)
        _bind(m, cfg, 1)
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


def _run_ranks(fused, world):
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_tp_worker, args=(r, world, port, q, fused))
             for r in range(world)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=300) for _ in procs], key=lambda r: r[0])
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    return res


@pytest.mark.parametrize("world", [2, 4])
@pytest.mark.parametrize("fused", [False, True], ids=["nccl_hook", "fused_peer"])
def test_tp_layer_and_stack(fused, world):
    import u15b200
    from oracle import oracle as O
    from test_gpu_layer import check_layer, dims_of
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} visible GPUs")
    cfg = CFGS[world]
    res = _run_ranks(fused, world)
    l0, f0 = res[0][1], res[0][3]
    # the reduction hands every rank the same sums: replicas stay identical
    for _, lr, _, fr in res[1:]:
        assert np.array_equal(l0, lr) and np.array_equal(f0, fr)
    T, segs, pos, x = _inputs(cfg)
    # one-GPU model on the same weights, for the layer and the stack
    m = u15b200.Model(**cfg)
    W = _bind(m, cfg, 1)
    pd = [dev_i32(p) for p in pos]
    kv = m.make_cache(T)
    xd = dev_bf16(x)
    m.forward(xd, kv, 0, T, *pd, segments=segs)
    torch.cuda.synchronize()
    assert rel_l2(f0, host(xd)) < 1e-2
    # layer 0 against the CPU restatement; rank r holds kv heads
    # [r * kv / world, (r + 1) * kv / world)
    ref, kn, _ = O.mot_layer(x, segs, W[0], dims_of(cfg), *pos)
    check_layer(l0, x, ref)
    ks = [r[2] for r in res]
    assert rel_l2(np.concatenate(ks), kn) < 1e-2
    per = cfg["kv_heads"] // world
    assert rel_l2(ks[0], kn[:per]) < 1e-2 and rel_l2(ks[0], kn[per:2 * per]) > 1e-1   # negative control
