"""The CFG-branch placement and the per-step velocity exchange across ranks
(the denoise loop's one collective), on CPU with the gloo backend and two
and four ranks. No GPU: the exchange is host logic over torch.distributed."""
import os
import socket

import pytest

torch = pytest.importorskip("torch")


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, n_branch, numel, q):
    import torch.distributed as dist
    from u15b200.generator import exchange_velocities, placement
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        owner = placement(n_branch, world)
        local = {b: torch.full((numel,), float(10 * b + 1)) for b in range(n_branch)
                 if owner[b] == rank}
        out = exchange_velocities(local, n_branch, numel, None, device=torch.device("cpu"))
        q.put((rank, [float(v[0]) for v in out], [float(v[-1]) for v in out]))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,n_branch", [(2, 1), (2, 2), (2, 3), (4, 3)])
def test_velocity_exchange(world, n_branch):
    """Every rank ends with every branch's velocity; at 4 ranks and 3 branches
    one rank owns none and contributes only padding."""
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, n_branch, 37, q))
             for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    want = [float(10 * b + 1) for b in range(n_branch)]
    for rank, first, last in res:
        assert first == want and last == want, (rank, first)


def test_branch_plan_matches_reference_rules():
    from u15b200 import _lib as L
    from u15b200.generator import branch_plan, placement
    # t2i with cfg: cond + uncond, unconditional baseline
    assert branch_plan(False, 4.0, 1.0) == (["cond", "uncond"], -1, 1, L.CFG_UNC)
    # edit, img_cfg == 1: image-conditioned baseline
    assert branch_plan(True, 4.0, 1.0) == (["cond", "img_cond"], 1, -1, L.CFG_IMG)
    # edit, cfg == img_cfg != 1: one axis, unconditional baseline
    assert branch_plan(True, 2.0, 2.0) == (["cond", "uncond"], -1, 1, L.CFG_UNC)
    # edit, both axes
    assert branch_plan(True, 4.0, 1.5) == (["cond", "img_cond", "uncond"], 1, 2, L.CFG_BOTH)
    # no guidance
    assert branch_plan(False, 1.0, 1.0) == (["cond"], -1, -1, L.CFG_NONE)
    assert placement(3, 2) == [0, 1, 0]
