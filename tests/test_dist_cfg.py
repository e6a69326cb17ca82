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


def _worker(rank, world, port, n_branch, numel, q, groups=None):
    import torch.distributed as dist
    from u15b200.generator import exchange_velocities, owners_of, placement
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        owner = placement(n_branch, world) if groups is None else owners_of(groups, n_branch)
        local = {b: torch.full((numel,), float(10 * b + 1)) for b in range(n_branch)
                 if owner[b] == rank}
        out = exchange_velocities(local, n_branch, numel, None, device=torch.device("cpu"),
                                  owner=owner)
        q.put((rank, [float(v[0]) for v in out], [float(v[-1]) for v in out]))
    finally:
        dist.destroy_process_group()


def _groups(world, n_branch, kind):
    from u15b200.generator import Group, plan_groups
    if kind == "plan":
        return plan_groups(n_branch, world)
    if kind == "pairs":   # two two-rank groups, the first running two branches
        return [Group([0, 1], [0, 1]), Group([2, 3], [2])]
    return None


@pytest.mark.parametrize("world,n_branch,kind", [(2, 1, None), (2, 2, None), (2, 3, None),
                                                 (4, 3, None), (4, 3, "pairs"),
                                                 (2, 3, "plan")])
def test_velocity_exchange(world, n_branch, kind):
    """Every rank ends with every branch's velocity; at 4 ranks and 3 branches
    one rank owns none and contributes only padding; with tensor-parallel
    groups each group's first rank speaks for its branches."""
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    groups = _groups(world, n_branch, kind)
    procs = [ctx.Process(target=_worker, args=(r, world, port, n_branch, 37, q, groups))
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


def test_plan_groups():
    """One image's CFG branches over the ranks: branch placement up to as many
    ranks as branches, tensor-parallel groups beyond (the sizes the model
    splits into), the step time of the cost model minimal."""
    from u15b200.generator import TP_SPEEDUP, owners_of, plan_groups
    shapes = {w: [(g.ranks, g.branches) for g in plan_groups(3, w)] for w in range(1, 9)}
    assert shapes[1] == [([0], [0, 1, 2])]
    assert shapes[3] == [([0], [0]), ([1], [1]), ([2], [2])]
    assert shapes[4] == shapes[3]            # a fourth rank cannot shorten the step
    assert shapes[6] == [([0, 1], [0]), ([2, 3], [1]), ([4, 5], [2])]
    assert shapes[8] == shapes[6]
    for w in range(1, 9):
        g = plan_groups(3, w)
        assert sorted(b for x in g for b in x.branches) == [0, 1, 2]
        ranks = [r for x in g for r in x.ranks]
        assert len(set(ranks)) == len(ranks) and max(ranks) < w
        assert all(len(x.ranks) in TP_SPEEDUP for x in g)
    assert owners_of(plan_groups(3, 6), 3) == [0, 2, 4]
    # a heavier branch gets the larger group
    g = plan_groups(2, 6, weights=[2.0, 1.2])
    assert [len(x.ranks) for x in g] == [4, 2]
