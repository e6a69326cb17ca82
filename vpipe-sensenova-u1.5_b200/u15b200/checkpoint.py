"""Binding a released checkpoint: safetensors files -> the device layout
(U15Weights::load, src/u15-weights.cc:341-511 of the reference).

Tensor names are the reference's (src/u15-weights.cc:361-430, 534-578):
the MoT split is the same thirteen tensors per layer, bare for the
understanding expert and with `_mot_gen` for the generation expert (on the
tensor for attention, on the module for the MLP and layer norms). A matrix
with a `.scales` sibling is an affine pack (u32 codes + per-group scales and
biases); its bits and group are derived from the column counts against the
known input width K, and a shape that does not close is refused
(bind_matrix_, src/u15-weights.cc:248-325). Packs are dequantized on the
device (u15c_dequant_affine) into the bound bf16 layout; a model created with
int8 twins then requantizes them per output channel in `finalize()`.
"""
from __future__ import annotations

import ctypes as C
import glob
import json
import os
import struct

import numpy as np
import torch

from . import _lib as L
from ._lib import check, lib
from .ops import _p, _stream

# safetensors dtype -> (numpy storage dtype, bytes per element)
_DT = {"F32": (np.float32, 4), "F16": (np.float16, 2), "BF16": (np.uint16, 2),
       "U32": (np.uint32, 4), "I32": (np.int32, 4), "U8": (np.uint8, 1), "I8": (np.int8, 1),
       "I64": (np.int64, 8), "F64": (np.float64, 8)}


class SafeTensors:
    """Every tensor of a .safetensors file or of a directory of them, memory
    mapped: an 8-byte little-endian header length, the JSON header
    (dtype, shape, data_offsets per name), the data."""

    def __init__(self, path: str):
        files = [path] if os.path.isfile(path) else sorted(
            glob.glob(os.path.join(path, "*.safetensors")))
        if not files:
            raise FileNotFoundError(f"no .safetensors under {path}")
        self.index = {}
        for f in files:
            with open(f, "rb") as fh:
                n = struct.unpack("<Q", fh.read(8))[0]
                header = json.loads(fh.read(n))
            mm = np.memmap(f, dtype=np.uint8, mode="r")
            for name, info in header.items():
                if name == "__metadata__":
                    continue
                a, b = info["data_offsets"]
                self.index[name] = (mm, 8 + n + a, 8 + n + b, info["dtype"],
                                    tuple(info["shape"]))

    def __contains__(self, name):
        return name in self.index

    def dtype(self, name):
        return self.index[name][3]

    def shape(self, name):
        return self.index[name][4]

    def array(self, name) -> np.ndarray:
        """The stored values (BF16 as its uint16 bit patterns)."""
        mm, a, b, dt, shape = self.index[name]
        np_dt, es = _DT[dt]
        if b - a != int(np.prod(shape, dtype=np.int64)) * es:
            raise ValueError(f"'{name}': {b - a} bytes for shape {shape} of {dt}")
        return np.asarray(mm[a:b]).view(np_dt).reshape(shape)

    def to_device(self, name) -> torch.Tensor:
        """CUDA tensor: f32 / f16 as stored, BF16 as torch.bfloat16, integers as stored."""
        a = np.ascontiguousarray(self.array(name))
        t = torch.from_numpy(a.view(np.int16) if self.dtype(name) == "BF16" else a)
        t = t.cuda()
        return t.view(torch.bfloat16) if self.dtype(name) == "BF16" else t


def write_safetensors(path: str, tensors: dict) -> None:
    """Write tensors (numpy arrays; a ("BF16", uint16 array) pair for bf16)
    as one .safetensors file: fixtures and tools."""
    back = {np.dtype(v[0]): k for k, v in _DT.items() if k != "BF16"}
    header, blobs, off = {}, [], 0
    for name, v in tensors.items():
        dt, a = (v if isinstance(v, tuple) else (back[np.asarray(v).dtype], v))
        a = np.ascontiguousarray(a)
        raw = a.tobytes()
        header[name] = {"dtype": dt, "shape": list(a.shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    h = json.dumps(header).encode()
    h += b" " * (-len(h) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def _scalar_dtype(dt: str) -> int:
    return {"F32": L.DT_F32, "F16": L.DT_F16, "BF16": L.DT_BF16}[dt]


def pack_shape(K: int, scale_cols: int, code_cols: int):
    """(bits, group) of an affine pack from its column counts against the
    input width K, or None when they do not close (src/u15-weights.cc:270-283)."""
    g = K // scale_cols if scale_cols > 0 else 0
    b = code_cols * 32 // K if K > 0 else 0
    if g not in (32, 64) or b not in (4, 8) or scale_cols * g != K or code_cols * 32 != K * b:
        return None
    return b, g


def matrix_to_device(st: SafeTensors, base: str, K: int) -> torch.Tensor:
    """`base`.weight as a device tensor, or the affine pack under `base`
    dequantized on the device to bf16 [N][K]."""
    if base + ".scales" in st and base + ".weight" in st:
        sc, cd = st.shape(base + ".scales"), st.shape(base + ".weight")
        shp = pack_shape(K, sc[1], cd[1]) if len(sc) == 2 and len(cd) == 2 else None
        if shp is None:
            raise ValueError(f"'{base}' looks quantized but its shapes do not close: K={K}, "
                             f"scales cols={sc[-1]}, codes cols={cd[-1]}")
        bits, group = shp
        N = cd[0]
        codes = st.to_device(base + ".weight")
        scales = st.to_device(base + ".scales")
        biases = st.to_device(base + ".biases")
        out = torch.empty(N, K, dtype=torch.bfloat16, device="cuda")
        check(lib().u15c_dequant_affine(_stream(), _p(codes), _p(scales), _p(biases),
                                        _scalar_dtype(st.dtype(base + ".scales")), N, K, bits,
                                        group, _p(out)))
        torch.cuda.current_stream().synchronize()   # the staged pack goes out of scope
        return out
    return st.to_device(base + ".weight")


def layer_names(i: int, expert: int) -> dict:
    """Our tensor name -> the checkpoint's (for matrices: the base, without
    .weight / .scales), src/u15-weights.cc:534-578."""
    p = f"language_model.model.layers.{i}."
    s = ("", "_mot_gen")[expert]
    a = p + "self_attn."
    return {"input_layernorm": p + f"input_layernorm{s}.weight",
            "post_attention_layernorm": p + f"post_attention_layernorm{s}.weight",
            "q_proj": a + f"q_proj{s}", "k_proj": a + f"k_proj{s}", "v_proj": a + f"v_proj{s}",
            "o_proj": a + f"o_proj{s}", "q_norm": a + f"q_norm{s}.weight",
            "k_norm": a + f"k_norm{s}.weight", "q_norm_hw": a + f"q_norm_hw{s}.weight",
            "k_norm_hw": a + f"k_norm_hw{s}.weight", "gate_proj": p + f"mlp{s}.gate_proj",
            "up_proj": p + f"mlp{s}.up_proj", "down_proj": p + f"mlp{s}.down_proj"}


MATRICES = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")


def bind_model(model, st: SafeTensors, n_layers: int | None = None) -> torch.Tensor:
    """Bind every layer (both experts) and the two final norms of `model`
    from `st`; returns the token-embedding table (bf16, device)."""
    c = model.cfg
    H, I, QD = c["hidden"], c["inter"], c["heads"] * c["head_dim"]
    K_of = {"q_proj": H, "k_proj": H, "v_proj": H, "o_proj": QD, "gate_proj": H, "up_proj": H,
            "down_proj": I}
    n = c["n_layers"] if n_layers is None else n_layers
    for i in range(n):
        for e in range(2):
            for ours, theirs in layer_names(i, e).items():
                if ours in MATRICES:
                    model.bind(i, e, ours, matrix_to_device(st, theirs, K_of[ours]))
                else:
                    if theirs not in st:
                        raise KeyError(f"layer {i}: missing '{theirs}'")
                    model.bind(i, e, ours, st.to_device(theirs))
    model.bind(0, 0, "final_norm", st.to_device("language_model.model.norm.weight"))
    model.bind(0, 1, "final_norm", st.to_device("language_model.model.norm_mot_gen.weight"))
    torch.cuda.current_stream().synchronize()
    emb = st.to_device("language_model.model.embed_tokens.weight")
    return emb if emb.dtype == torch.bfloat16 else emb.to(torch.bfloat16)


IMAGE_NAMES = {
    ("patch_w", 0): "vision_model.embeddings.patch_embedding.weight",
    ("patch_b", 0): "vision_model.embeddings.patch_embedding.bias",
    ("dense_w", 0): "vision_model.embeddings.dense_embedding.weight",
    ("dense_b", 0): "vision_model.embeddings.dense_embedding.bias",
    ("patch_w", 1): "fm_modules.vision_model_mot_gen.embeddings.patch_embedding.weight",
    ("patch_b", 1): "fm_modules.vision_model_mot_gen.embeddings.patch_embedding.bias",
    ("dense_w", 1): "fm_modules.vision_model_mot_gen.embeddings.dense_embedding.weight",
    ("dense_b", 1): "fm_modules.vision_model_mot_gen.embeddings.dense_embedding.bias",
    ("conv1_w", 0): "fm_modules.fm_head.conv1.weight",
    ("conv1_b", 0): "fm_modules.fm_head.conv1.bias",
    ("conv2_w", 0): "fm_modules.fm_head.conv2.weight",
    ("conv2_b", 0): "fm_modules.fm_head.conv2.bias",
    ("tstep_w0", 0): "fm_modules.timestep_embedder.mlp.0.weight",
    ("tstep_b0", 0): "fm_modules.timestep_embedder.mlp.0.bias",
    ("tstep_w2", 0): "fm_modules.timestep_embedder.mlp.2.weight",
    ("tstep_b2", 0): "fm_modules.timestep_embedder.mlp.2.bias",
    ("nscale_w0", 0): "fm_modules.noise_scale_embedder.mlp.0.weight",
    ("nscale_b0", 0): "fm_modules.noise_scale_embedder.mlp.0.bias",
    ("nscale_w2", 0): "fm_modules.noise_scale_embedder.mlp.2.weight",
    ("nscale_b2", 0): "fm_modules.noise_scale_embedder.mlp.2.bias",
}


def bind_image(image_path, st: SafeTensors) -> None:
    """Bind the patch embedders (both twins), the pixel head and the two
    scalar embedders (src/u15-weights.cc:372-420) into an ImagePath."""
    for (ours, expert), theirs in IMAGE_NAMES.items():
        if ours.startswith("nscale") and not image_path.cfg["noise_scale_embedding"]:
            continue
        if theirs not in st:
            raise KeyError(f"missing image-path tensor '{theirs}'")
        image_path.bind(ours, st.to_device(theirs), expert=expert)
    torch.cuda.current_stream().synchronize()
