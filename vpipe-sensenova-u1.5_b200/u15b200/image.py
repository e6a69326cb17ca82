"""The image path over libu15c's C ABI: the Python face of ImagePath
(src/u15-image.h of the reference) -- patch embedder in, pixel head out,
timestep + noise-scale embedding. Channel-last throughout."""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from . import _lib as L
from ._lib import check, lib
from .ops import _p, _stream

FULL_IMAGE = dict(vision_hidden=1024, llm_hidden=4096, patch=16, merge=2, head_hidden=1024,
                  freq_dim=256, noise_scale_embedding=1, vision_theta=1e4)


class ImagePath:
    def __init__(self, **cfg):
        c = dict(FULL_IMAGE)
        c.update(cfg)
        self.cfg = c
        self._cfg = L.ImageConfig(**c)
        h = C.c_void_p()
        check(lib().u15c_image_create(C.byref(self._cfg), C.byref(h)))
        self.h = h

    def close(self):
        if self.h:
            lib().u15c_image_destroy(self.h)
            self.h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def bind(self, name: str, array, expert: int = 0) -> None:
        """One checkpoint tensor (host numpy f32/f16 or CUDA f32/f16/bf16);
        patch/dense tensors take expert 0 (understanding) or 1 (generation)."""
        tid = L.IMAGE_TENSORS.index(name)
        if isinstance(array, np.ndarray):
            a = np.ascontiguousarray(array)
            dt = {np.dtype(np.float32): L.DT_F32, np.dtype(np.float16): L.DT_F16}[a.dtype]
            check(lib().u15c_image_bind(self.h, _stream(), tid, expert,
                                        C.c_void_p(a.ctypes.data), dt, 1))
            torch.cuda.current_stream().synchronize()
        else:
            a = array.contiguous()
            dt = {torch.float32: L.DT_F32, torch.float16: L.DT_F16,
                  torch.bfloat16: L.DT_BF16}[a.dtype]
            check(lib().u15c_image_bind(self.h, _stream(), tid, expert, _p(a), dt, 0))

    def bind_random(self, seed: int, std: float = 0.02) -> None:
        check(lib().u15c_image_bind_random(self.h, _stream(), seed, std))

    def patchify(self, img_hwc: torch.Tensor) -> torch.Tensor:
        """[H][W][3] f32 -> [(H/p)(W/p)][3p^2] bf16 (channel-first patches)."""
        H, W, _ = img_hwc.shape
        p = self.cfg["patch"]
        px = torch.empty((H // p) * (W // p), 3 * p * p, dtype=torch.bfloat16, device="cuda")
        check(lib().u15c_image_patchify(_stream(), _p(img_hwc), _p(px), H, W, p))
        return px

    def embed(self, px, grid_h: int, grid_w: int, gen: bool = True, out=None) -> torch.Tensor:
        m = self.cfg["merge"]
        if out is None:
            out = torch.empty((grid_h // m) * (grid_w // m), self.cfg["llm_hidden"],
                              dtype=torch.bfloat16, device="cuda")
        check(lib().u15c_image_embed(self.h, _stream(), _p(px), grid_h, grid_w, int(gen),
                                     _p(out)))
        return out

    def timestep_row(self, t: float, noise_ratio: float) -> torch.Tensor:
        out = torch.empty(self.cfg["llm_hidden"], dtype=torch.float32, device="cuda")
        check(lib().u15c_image_timestep_row(self.h, _stream(), t, noise_ratio, _p(out)))
        return out

    def add_timestep(self, x, t: float, noise_ratio: float) -> None:
        check(lib().u15c_image_add_timestep(self.h, _stream(), _p(x), x.shape[0], t,
                                            noise_ratio))

    def decode(self, hidden, th: int, tw: int, out=None) -> torch.Tensor:
        if out is None:
            out = torch.empty(32 * th, 32 * tw, 3, dtype=torch.float32, device="cuda")
        check(lib().u15c_image_decode(self.h, _stream(), _p(hidden), th, tw, _p(out)))
        return out

    def to_u8_planar(self, px) -> torch.Tensor:
        H, W, _ = px.shape
        out = torch.empty(3, H, W, dtype=torch.uint8, device="cuda")
        check(lib().u15c_image_to_u8_planar(_stream(), _p(px), _p(out), H, W))
        return out
