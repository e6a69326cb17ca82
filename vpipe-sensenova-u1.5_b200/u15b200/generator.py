"""The denoise loop: Generator::generate (src/u15-generator.cc:151-717 of the
reference) over libu15c.

Per generation: the CFG branches the reference would build
(src/u15-generator.cc:174-276) -- conditional, image-conditional when
editing with img_cfg != 1, unconditional when needed -- each with its own
prefix prefilled into its own paged KV cache by the und expert (causal, or
block-causal when the prefix holds a reference image), then seeded noise and
the shifted flow-matching schedule. Per step: embed the current image, add
the timestep row, run the 42-layer gen-expert pass of every branch against
its frozen prefix (bidirectional), final norm + pixel head, then on the
device v = (x_pred - z) / max(1 - t, t_eps), the CFG form and renorm, and
the Euler update (u15c_velocity / u15c_cfg_combine / u15c_euler).

The image half of each step is the reference's ImagePath on the device
(`DeviceImagePath` over u15b200.ImagePath: patch embedder, pixel head,
timestep + noise-scale row); `LinearImagePath` is a lighter stand-in (one
linear map each way per 32x32 token) that tests use when they restate the
whole loop on the CPU.

Across ranks (torch.distributed), branches are placed round-robin; after
each step's forwards every rank all-gathers the velocities (the loop's one
exchange) and applies CFG and Euler redundantly, so every rank holds the
same image with no broadcast.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field

import numpy as np
import torch

from . import _lib as L
from ._lib import U15Error, check, lib
from .ops import CudaOps, _p, _stream

PIX = 32   # pixels per LLM token side (src/u15-config.h:23-28)


def time_schedule(num_steps: int, shift: float) -> list[float]:
    """src/u15-ref.cc:722-733: sigma = 1 - i/n, shifted, t = 1 - sigma (f32)."""
    out = []
    for i in range(num_steps + 1):
        sigma = 1.0 - i / num_steps
        sigma = shift * sigma / (1.0 + (shift - 1.0) * sigma)
        out.append(float(np.float32(1.0 - sigma)))
    return out


def image_positions(t: int, th: int, tw: int):
    """src/u15-generator.cc:62-73: every image token at t, h = row, w = column."""
    n = th * tw
    return (np.full(n, t, np.int32), (np.arange(n) // tw).astype(np.int32),
            (np.arange(n) % tw).astype(np.int32))


def branch_plan(editing: bool, cfg: float, icfg: float):
    """Which branches run (src/u15-generator.cc:174-186, 243-276): returns
    (names, i_img, i_unc, form)."""
    icfg = icfg if editing else 1.0
    needs_cfg = not (cfg == 1.0 and icfg == 1.0)
    needs_img = editing and needs_cfg and (icfg == 1.0 or cfg != icfg)
    needs_unc = needs_cfg and (not editing or icfg != 1.0)
    names = ["cond"] + (["img_cond"] if needs_img else []) + (["uncond"] if needs_unc else [])
    i_img = 1 if needs_img else -1
    i_unc = (2 if needs_img else 1) if needs_unc else -1
    if i_img >= 0 and i_unc < 0:
        form = L.CFG_IMG
    elif i_img < 0 and i_unc >= 0:
        form = L.CFG_UNC
    elif i_img >= 0 and i_unc >= 0:
        form = L.CFG_BOTH
    else:
        form = L.CFG_NONE
    return names, i_img, i_unc, form


def placement(n_branch: int, world: int) -> list[int]:
    """Rank that runs each branch: round-robin."""
    return [b % world for b in range(n_branch)]


# Per-layer speed-up of a tensor-parallel group of 1, 2, 4 and 8 GPUs over one
# GPU on the 4096-token layer (the bench's `tensor_parallel` section, fused
# reduction): the cost model of plan_groups.
TP_SPEEDUP = {1: 1.0, 2: 1.58, 4: 1.79, 8: 1.38}


@dataclass
class Group:
    ranks: list           # consecutive global ranks; tensor-parallel over them when > 1
    branches: list        # branch indices this group runs (through forward_many)


def plan_groups(n_branch: int, world: int, speedup: dict = None,
                weights: list = None) -> list:
    """Place ONE image's CFG branches over `world` ranks: disjoint groups of
    consecutive ranks (1, 2, 4 or 8 of them, the tensor-parallel sizes the
    model splits into), each running a run of consecutive branches, every
    rank in at most one group. The plan minimises the step time
    max_g(sum of its branches' weights / speedup[size]); ties go to fewer
    ranks. world <= n_branch gives branch placement (groups of one rank);
    e.g. 3 branches: 4 ranks keep 1 + 1 + 1, 6 and 8 ranks run three
    two-rank groups."""
    sp = TP_SPEEDUP if speedup is None else speedup
    w = [1.0] * n_branch if weights is None else list(weights)
    sizes = sorted(k for k in sp if k <= world)
    best = None

    def rec(b0, used, acc):
        nonlocal best
        if b0 == n_branch:
            t = max(x[2] for x in acc)
            key = (round(t, 9), used)
            if best is None or key < best[0]:
                best = (key, list(acc))
            return
        for b1 in range(b0 + 1, n_branch + 1):
            load = sum(w[b0:b1])
            for sz in sizes:
                if used + sz > world:
                    continue
                acc.append((list(range(b0, b1)), sz, load / sp[sz]))
                rec(b1, used + sz, acc)
                acc.pop()

    rec(0, 0, [])
    groups, r0 = [], 0
    for br, sz, _ in best[1]:
        groups.append(Group(list(range(r0, r0 + sz)), br))
        r0 += sz
    return groups


def owners_of(groups: list, n_branch: int) -> list:
    """The rank that contributes each branch's velocity: its group's first."""
    own = [0] * n_branch
    for g in groups:
        for b in g.branches:
            own[b] = g.ranks[0]
    return own


def exchange_velocities(local: dict, n_branch: int, numel: int, group=None, device=None,
                        owner: list = None):
    """All-gather per-branch velocities so every rank holds all of them.

    `local` maps branch index -> flat f32 tensor of `numel` elements for the
    branches this rank contributes; `owner[b]` is the rank that contributes
    branch b (default: round-robin placement). Each rank sends as many slots
    as the busiest owner (unused slots zero); returns a list of n_branch
    tensors."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    own = placement(n_branch, world) if owner is None else list(owner)
    per = max(1, max(own.count(r) for r in range(world)))
    dev = device if device is not None else next(iter(local.values())).device
    send = torch.zeros(per, numel, dtype=torch.float32, device=dev)
    mine = [b for b in range(n_branch) if own[b] == rank]
    for i, b in enumerate(mine):
        send[i].copy_(local[b].reshape(-1))
    recv = torch.empty(world * per, numel, dtype=torch.float32, device=dev)
    dist.all_gather_into_tensor(recv, send, group=group)
    out = [None] * n_branch
    for r in range(world):
        owned = [b for b in range(n_branch) if own[b] == r]
        for i, b in enumerate(owned):
            out[b] = recv[r * per + i]
    return out


class LinearImagePath:
    """Stand-in for the reference's ImagePath: token rows of 32x32x3 pixels
    (channel-last) -> hidden by one linear map, hidden -> pixels by another,
    plus a timestep row from the cos-first sinusoid through a fixed linear
    map (src/u15-ref.cc:735-753 for the sinusoid). Seeded weights."""

    def __init__(self, hidden: int, seed: int = 0, device="cuda"):
        g = torch.Generator(device="cpu").manual_seed(seed)
        d = PIX * PIX * 3
        self.hidden = hidden
        self.w_in = (torch.randn(hidden, d, generator=g) / d ** 0.5).to(device, torch.bfloat16)
        self.w_out = (torch.randn(d, hidden, generator=g) / hidden ** 0.5).to(device,
                                                                             torch.bfloat16)
        self.w_t = (torch.randn(hidden, 256, generator=g) * 0.05).numpy()

    @staticmethod
    def sinusoid(t: float, dim: int = 256, max_period: float = 10000.0):
        half = dim // 2
        freqs = np.exp(-np.log(max_period) * np.arange(half) / half)
        a = t * freqs
        return np.concatenate([np.cos(a), np.sin(a)]).astype(np.float32)

    def timestep_row(self, t: float) -> torch.Tensor:
        row = self.w_t @ self.sinusoid(t * 1000.0)
        return torch.from_numpy(row.astype(np.float32)).to("cuda", torch.bfloat16)

    def embed(self, img: torch.Tensor, H: int, W: int, out: torch.Tensor, rows: torch.Tensor):
        check(lib().u15c_patchify(_stream(), _p(img), _p(rows), H, W))
        n = (H // PIX) * (W // PIX)
        check(lib().u15c_linear_bf16(_stream(), _p(rows), _p(self.w_in), None, _p(out), n,
                                     PIX * PIX * 3, self.hidden))

    def decode(self, h: torch.Tensor, H: int, W: int, x_pred: torch.Tensor):
        n = (H // PIX) * (W // PIX)
        rows = self._rows(n)
        check(lib().u15c_linear_bf16(_stream(), _p(h), _p(self.w_out), None, _p(rows), n,
                                     self.hidden, PIX * PIX * 3))
        check(lib().u15c_unpatchify(_stream(), _p(rows), _p(x_pred), H, W))

    def _rows(self, n):
        if getattr(self, "_rowbuf", None) is None or self._rowbuf.shape[0] < n:
            self._rowbuf = torch.empty(n, PIX * PIX * 3, device="cuda", dtype=torch.bfloat16)
        return self._rowbuf[:n]

    def embed_step(self, img, H: int, W: int, emb, t: float, noise_ratio: float):
        """embed the current image and add the timestep row (the stand-in
        ignores the noise-scale ratio)"""
        n = (H // PIX) * (W // PIX)
        self.embed(img, H, W, emb, self._rows(n))
        check(lib().u15c_add_row(_stream(), _p(emb), _p(self.timestep_row(t)), n, self.hidden))


class DeviceImagePath:
    """The reference's ImagePath on the device (u15b200.ImagePath): per step
    patchify (channel-first, patch 16), the generation twin of the patch
    embedder, the timestep + noise-scale row added to every token
    (src/u15-generator.cc:477-499), and the pixel head after the final norm
    (src/u15-generator.cc:554-568)."""

    def __init__(self, image):
        self.im = image

    def embed_step(self, img, H: int, W: int, emb, t: float, noise_ratio: float):
        p = self.im.cfg["patch"]
        px = self.im.patchify(img)
        self.im.embed(px, H // p, W // p, gen=True, out=emb)
        self.im.add_timestep(emb, t, noise_ratio)

    def decode(self, h, H: int, W: int, x_pred):
        self.im.decode(h, H // PIX, W // PIX, out=x_pred)


@dataclass
class Branch:
    name: str
    prefix: torch.Tensor                      # [n][hidden] bf16 prefix embeddings
    t: np.ndarray                             # prefix positions
    h: np.ndarray
    w: np.ndarray
    block_causal: bool = False
    kv: object = None
    pos: list = field(default_factory=list)   # device image positions (t, h, w)
    v: torch.Tensor = None


def branch_from_ids(name: str, ids, embed_table: torch.Tensor, *, img_id: int = 151665,
                    img_ctx_id: int = 151667, images=(), image_path=None):
    """A prefix from token ids (src/u15-generator.cc:308-392): the
    embed_tokens rows of the ids, each reference image's patch embedding --
    the UNDERSTANDING twin, src/u15-generator.cc:231-238 -- spliced over its
    <IMG_CONTEXT> run, and the (t, h, w) triple of Prompt::thw_indexes.
    `images`: [H][W][3] f32 device tensors in model space; block-causal
    prefill when there are any."""
    ids = np.ascontiguousarray(np.asarray(ids, np.int32))
    n = len(ids)
    vocab, hidden = embed_table.shape
    x = torch.empty(n, hidden, dtype=torch.bfloat16, device="cuda")
    ids_dev = torch.from_numpy(ids).cuda()
    check(lib().u15c_embed_tokens(_stream(), _p(embed_table), vocab, hidden, _p(ids_dev), n,
                                  _p(x)))
    grids = []
    if images:
        if image_path is None:
            raise ValueError("reference images need the image path (its understanding twin)")
        im = image_path.im if hasattr(image_path, "im") else image_path
        p = im.cfg["patch"]
        embeds, tokens = [], []
        for img in images:
            gh, gw = img.shape[0] // p, img.shape[1] // p
            grids.append((gh, gw))
            e = im.embed(im.patchify(img), gh, gw, gen=False)
            embeds.append(e)
            tokens.append(e.shape[0])
        ptrs = (C.c_void_p * len(embeds))(*[e.data_ptr() for e in embeds])
        toks = (C.c_int * len(tokens))(*tokens)
        check(lib().u15c_splice_image_rows(_stream(), _p(x), hidden,
                                           C.c_void_p(ids.ctypes.data), n, img_ctx_id, ptrs,
                                           toks, len(embeds)))
        torch.cuda.current_stream().synchronize()   # the embeddings may go out of scope
    t, h, w = (np.zeros(n, np.int32) for _ in range(3))
    g = np.ascontiguousarray(np.array(grids, np.int32).reshape(-1))
    vp = lambda a: C.c_void_p(a.ctypes.data)  # noqa: E731
    check(lib().u15c_thw_indexes(vp(ids), n, img_id, img_ctx_id, vp(g) if grids else None,
                                 len(grids), vp(t), vp(h), vp(w)))
    return Branch(name, x, t, h, w, block_causal=bool(images))


class Generator:
    """Generator::generate over a u15b200.Model (both experts bound)."""

    def __init__(self, model, image_path=None, device: int | None = None, group=None,
                 image_seed: int = 0, groups: list = None):
        """group: the ranks that share ONE image (torch.distributed group,
        None for a single process). groups: how that image's branches sit on
        those ranks (plan_groups); None places the branches round-robin, one
        rank each. A rank of a multi-rank group passes that group's
        tensor-parallel model as `model`."""
        self.m = model
        self.groups = groups
        # the model's device is the caller's current one (one process per GPU)
        self.ops = CudaOps(torch.cuda.current_device() if device is None else device)
        # a rank that runs no branch of the plan holds no model (it still
        # takes part in each step's velocity exchange)
        self.hidden = model.cfg["hidden"] if model is not None else 4096
        if image_path is None:
            # no checkpoint here: the device image path with seeded weights
            from .image import ImagePath
            im = ImagePath(llm_hidden=self.hidden)
            im.bind_random(image_seed, 0.02)
            image_path = DeviceImagePath(im)
        self.image = image_path
        self.group = group

    def prefill(self, b: Branch, ltok: int):
        """Prefill one branch's prefix into its own cache with the und expert
        (src/u15-generator.cc:308-392): causal, or block-causal when the
        prefix holds a reference image."""
        n = b.prefix.shape[0]
        b.kv = self.m.make_cache(n + ltok)
        x = b.prefix.clone()
        pos = [torch.from_numpy(a).cuda() for a in (b.t, b.h, b.w)]
        t_index = None
        attn = L_CAUSAL
        if b.block_causal:
            ti = np.concatenate([b.t, np.zeros(ltok, np.int32)]).astype(np.int32)
            t_index = torch.from_numpy(ti).cuda()
            attn = L_BLOCK
        self.m.forward(x, b.kv, 0, n, *pos, segments=[(0, n, L.EXPERT_UND)], attn=attn,
                       t_index=t_index)
        th_tw = self._geom
        b.pos = [torch.from_numpy(a).cuda() for a in image_positions(int(b.t.max()) + 1, *th_tw)]

    @staticmethod
    def noise_scale(image_tokens: int, mode: int = L.NOISE_RESOLUTION, scale: float = 1.0,
                    max_value: float = 16.0, base: int = 64) -> float:
        """GenConfig::init_noise_scale (src/u15-config.cc:106-122), the
        reference's defaults: sqrt(L / 64), capped at 16."""
        out = C.c_double()
        check(lib().u15c_init_noise_scale(image_tokens, mode, scale, max_value, base,
                                          C.byref(out)))
        return out.value

    @staticmethod
    def initial_image(H: int, W: int, seed: int, noise_scale: float, init_noise=None,
                      init_noise_path: str = None) -> torch.Tensor:
        """The start image on the device (src/u15-generator.cc:394-417): the
        injected noise (a tensor, or a file of H*W*3 raw f32 values,
        channel-last), or the seeded draw of u15c_init_noise."""
        n = H * W * 3
        if init_noise_path:
            try:
                with open(init_noise_path, "rb") as f:
                    raw = f.read(n * 4 + 1)
            except OSError as e:
                raise U15Error(L.EINVAL, f"cannot read init_noise {init_noise_path}") from e
            if len(raw) < n * 4:
                raise U15Error(L.EINVAL, f"init_noise is the wrong size: want {n} f32")
            host = np.frombuffer(raw[:n * 4], np.float32).copy()
        elif init_noise is not None:
            return init_noise.clone().reshape(H, W, 3).float().cuda()
        else:
            host = np.empty(n, np.float32)
            check(lib().u15c_init_noise(seed, noise_scale, C.c_void_p(host.ctypes.data), n))
        return torch.from_numpy(host).reshape(H, W, 3).cuda()

    def generate(self, branches: list, H: int, W: int, steps: int = 20, shift: float = 3.0,
                 cfg: float = 4.0, icfg: float = 1.0, cfg_norm: int = L.NORM_NONE,
                 t_eps: float = 0.05, seed: int = 0, noise_scale: float = None,
                 form: int = None, i_img: int = -1, i_unc: int = -1,
                 cfg_interval=(0.0, 1.0), int8: bool = False, sage: bool = False,
                 init_noise: torch.Tensor = None, init_noise_path: str = None,
                 step_callback=None, noise_scale_max: float = 16.0):
        """Run the loop; returns the final [H][W][3] f32 image (device).
        `branches` are already ordered cond, [img_cond], [uncond]. The start
        image is the reference's seeded draw scaled by the resolution's noise
        scale (noise_scale None: GenConfig::init_noise_scale of the image's
        token count), or the injected init_noise / init_noise_path."""
        th, tw = H // PIX, W // PIX
        Ltok = th * tw
        self._geom = (th, tw)
        dist = None
        world, rank = 1, 0
        if self.group is not None:
            import torch.distributed as dist
            world, rank = dist.get_world_size(self.group), dist.get_rank(self.group)
        nb = len(branches)
        if self.groups is not None:
            covered = sorted(b for g in self.groups for b in g.branches)
            ranks = [r for g in self.groups for r in g.ranks]
            if covered != list(range(nb)) or len(set(ranks)) != len(ranks) or \
                    any(r >= world for r in ranks):
                raise ValueError("groups must cover every branch once on distinct ranks")
            owner = owners_of(self.groups, nb)
            runs = [any(rank in g.ranks and bi in g.branches for g in self.groups)
                    for bi in range(nb)]
        else:
            owner = placement(nb, world)
            runs = [owner[bi] == rank for bi in range(nb)]
        for bi, b in enumerate(branches):
            if runs[bi]:
                self.prefill(b, Ltok)
        if form is None:
            form = {(-1, -1): L.CFG_NONE}.get((i_img, i_unc), L.CFG_NONE)
        n = H * W * 3
        if noise_scale is None:
            noise_scale = self.noise_scale(Ltok, max_value=noise_scale_max)
        img = self.initial_image(H, W, seed, noise_scale, init_noise, init_noise_path)
        ts = time_schedule(steps, shift)
        emb = torch.empty(Ltok, self.hidden, device="cuda", dtype=torch.bfloat16)
        # the noise-scale embedder sees the scale as a ratio of its maximum
        # (src/u15-generator.cc:465-466)
        ns_ratio = noise_scale / max(1e-9, noise_scale_max)
        # one hidden state per branch this rank runs, contiguous, so the
        # branches go through the stack together (u15c_forward_many)
        mine = [bi for bi in range(nb) if runs[bi]]
        hstate = torch.empty(max(len(mine), 1), Ltok, self.hidden, device="cuda",
                             dtype=torch.bfloat16)
        x_pred = torch.empty(H, W, 3, device="cuda", dtype=torch.float32)
        combined = torch.empty_like(x_pred)
        ws = torch.empty(lib().u15c_cfg_workspace_bytes(), dtype=torch.uint8, device="cuda")
        for b in branches:
            b.v = torch.zeros(H, W, 3, device="cuda", dtype=torch.float32)
        for step in range(steps):
            t, t_next = ts[step], ts[step + 1]
            self.image.embed_step(img, H, W, emb, t, ns_ratio)
            denom = max(1.0 - t, t_eps)
            lo, hi = cfg_interval
            use_cfg = (lo < t < hi) or lo == 0.0
            guided = form != L.CFG_NONE and use_cfg
            n_branch = len(branches) if guided else 1
            local = {}
            run = [bi for bi in mine if bi < n_branch]
            if run:
                for i in range(len(run)):
                    hstate[i].copy_(emb)
                slots = []
                for bi in run:
                    b = branches[bi]
                    npre = b.prefix.shape[0]
                    slots.append({"kv": b.kv, "kv_off": npre, "kv_len": npre + Ltok,
                                  "pos": b.pos})
                self.m.forward_many(hstate[:len(run)], Ltok, slots, expert=L.EXPERT_GEN,
                                    int8=int8, sage=sage)
                for i, bi in enumerate(run):
                    b = branches[bi]
                    self.m.final_norm(hstate[i], L.EXPERT_GEN)
                    self.image.decode(hstate[i], H, W, x_pred)
                    check(lib().u15c_velocity(_stream(), _p(x_pred), _p(img), _p(b.v), n,
                                              denom))
                    if owner[bi] == rank:   # a group's first rank speaks for it
                        local[bi] = b.v
            if world > 1:
                vs = exchange_velocities(local, n_branch, n, self.group, device=img.device,
                                         owner=owner[:n_branch])
                vs = [v.reshape(H, W, 3) for v in vs]
            else:
                vs = [branches[bi].v for bi in range(n_branch)]
            if guided:
                vu = vs[i_unc] if i_unc >= 0 else None
                vi = vs[i_img] if i_img >= 0 else None
                check(lib().u15c_cfg_combine(_stream(), _p(vs[0]), _p(vu), _p(vi),
                                             _p(combined), H, W, form, cfg_norm, cfg, icfg, step,
                                             _p(ws)))
                v = combined
            else:
                v = vs[0]
            check(lib().u15c_euler(_stream(), _p(img), _p(v), n, t_next - t))
            if step_callback is not None:
                step_callback(step, img)
        return img


L_CAUSAL = L.ATTN_CAUSAL
L_BLOCK = L.ATTN_BLOCK_CAUSAL
