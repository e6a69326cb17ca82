"""Load libu15c.so (built in-tree by ../build.py) and declare its C ABI.

There is no fallback: if the library is missing or does not load, every
caller gets an exception naming the file. The argument lists below follow
include/u15c.h one to one.
"""
from __future__ import annotations

import ctypes as C
import os
import re

PKG = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ROOT = os.path.dirname(PKG)
LIB_PATH = os.path.join(PKG, "lib", "libu15c.so")
HEADER = os.path.join(ROOT, "include", "u15c.h")

OK, EINVAL, ECUDA, ENOMEM, EDEVICE, ESTOPPED = 0, 1, 2, 3, 4, 5
EPI_STORE, EPI_RESIDUAL, EPI_SWIGLU, EPI_STORE_F32 = 0, 1, 2, 3
TP_BLOB_BYTES = 128
ATTN_BIDIRECTIONAL, ATTN_CAUSAL, ATTN_BLOCK_CAUSAL = 0, 1, 2
EXPERT_UND, EXPERT_GEN = 0, 1
MODEL_INT8 = 1
FWD_INT8, FWD_SAGE = 1, 2
DT_F32, DT_F16, DT_BF16 = 0, 1, 2
CFG_NONE, CFG_IMG, CFG_UNC, CFG_BOTH = 0, 1, 2, 3
NORM_NONE, NORM_GLOBAL, NORM_CHANNEL, NORM_ZERO_STAR = 0, 1, 2, 3
NOISE_CONSTANT, NOISE_RESOLUTION, NOISE_DYNAMIC_SQRT = 0, 1, 2
TENSORS = ["input_layernorm", "post_attention_layernorm", "q_proj", "k_proj", "v_proj",
           "o_proj", "q_norm", "k_norm", "q_norm_hw", "k_norm_hw", "gate_proj", "up_proj",
           "down_proj", "final_norm"]


class U15Error(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"u15c error {code}: {msg}")
        self.code = code


class Config(C.Structure):
    _fields_ = [("n_layers", C.c_int), ("hidden", C.c_int), ("heads", C.c_int),
                ("kv_heads", C.c_int), ("head_dim", C.c_int), ("inter", C.c_int),
                ("n_experts", C.c_int), ("eps", C.c_double), ("theta_t", C.c_double),
                ("theta_hw", C.c_double)]


vp, ip, i32p = C.c_void_p, C.c_int, C.POINTER(C.c_int)


class ImageConfig(C.Structure):
    _fields_ = [("vision_hidden", C.c_int), ("llm_hidden", C.c_int), ("patch", C.c_int),
                ("merge", C.c_int), ("head_hidden", C.c_int), ("freq_dim", C.c_int),
                ("noise_scale_embedding", C.c_int), ("vision_theta", C.c_double)]


IMAGE_TENSORS = ["patch_w", "patch_b", "dense_w", "dense_b", "conv1_w", "conv1_b", "conv2_w",
                 "conv2_b", "tstep_w0", "tstep_b0", "tstep_w2", "tstep_b2", "nscale_w0",
                 "nscale_b0", "nscale_w2", "nscale_b2"]


class Slot(C.Structure):
    _fields_ = [("kv", C.c_void_p), ("kv_off", C.c_int), ("kv_len", C.c_int),
                ("pos_t", C.c_void_p), ("pos_h", C.c_void_p), ("pos_w", C.c_void_p),
                ("t_index", C.c_void_p)]
STOP_FN = C.CFUNCTYPE(C.c_int, C.c_void_p)
ALLREDUCE_FN = C.CFUNCTYPE(C.c_int, C.c_void_p, C.c_long, C.c_void_p)

SIGNATURES = {
    "u15c_last_error": (C.c_char_p, []),
    "u15c_version": (C.c_char_p, []),
    "u15c_init": (ip, [ip, C.c_uint]),
    "u15c_device_status": (ip, [ip, C.POINTER(C.c_uint)]),
    "u15c_sync": (ip, [vp]),
    "u15c_set_wait_limit": (ip, [ip, C.c_ulonglong]),
    "u15c_init_noise": (ip, [C.c_uint64, C.c_double, vp, C.c_long]),
    "u15c_init_noise_scale": (ip, [ip, ip, C.c_double, C.c_double, ip,
                                   C.POINTER(C.c_double)]),
    "u15c_wait_counter": (ip, [vp, vp, C.c_ulonglong]),
    "u15c_linear_bf16": (ip, [vp, vp, vp, vp, vp, ip, ip, ip]),
    "u15c_mot_linear_bf16": (ip, [vp, vp, vp, ip, i32p, i32p, ip, ip, vp, vp, vp, ip, ip, ip]),
    "u15c_quant_rows_i8": (ip, [vp, vp, vp, vp, ip, ip]),
    "u15c_linear_i8": (ip, [vp, vp, vp, vp, vp, vp, vp, vp, ip, ip, ip]),
    "u15c_mot_linear_i8": (ip, [vp, vp, vp, vp, vp, ip, i32p, i32p, ip, ip, vp, vp, vp, ip,
                                ip, ip]),
    "u15c_rms_norm": (ip, [vp, vp, vp, vp, ip, ip, C.c_float]),
    "u15c_mot_rms_norm": (ip, [vp, vp, vp, ip, i32p, i32p, ip, vp, ip, ip, C.c_float]),
    "u15c_mot_rms_norm_quant_i8": (ip, [vp, vp, vp, ip, i32p, i32p, ip, vp, vp, ip, ip,
                                        C.c_float]),
    "u15c_split_qk_norm": (ip, [vp, vp, vp, vp, ip, ip, ip, C.c_float]),
    "u15c_split_rope": (ip, [vp, vp, vp, vp, ip, ip, ip, ip, ip]),
    "u15c_build_rope_tables": (ip, [vp, vp, vp, vp, ip, ip, ip, ip, C.c_double, C.c_double,
                                    vp, vp]),
    "u15c_qkv_post": (ip, [vp, vp, vp, ip, i32p, i32p, ip, vp, vp, vp, vp, vp, vp, ip, ip, ip,
                           ip, ip, C.c_float]),
    "u15c_transpose_thd": (ip, [vp, vp, vp, ip, ip, ip]),
    "u15c_transpose_htd": (ip, [vp, vp, vp, ip, ip, ip]),
    "u15c_transpose_into_cache": (ip, [vp, vp, vp, ip, ip, ip, ip, ip]),
    "u15c_kv_append": (ip, [vp, vp, vp, vp, ip, ip, ip]),
    "u15c_swiglu": (ip, [vp, vp, vp, vp, ip, ip]),
    "u15c_add": (ip, [vp, vp, vp, C.c_long]),
    "u15c_add_row": (ip, [vp, vp, vp, ip, ip]),
    "u15c_silu": (ip, [vp, vp, C.c_long]),
    "u15c_sage_workspace_bytes": (C.c_size_t, [ip, ip, ip, ip]),
    "u15c_attention": (ip, [vp, vp, vp, vp, vp, ip, vp, ip, ip, ip, ip, ip, ip, ip, vp, vp]),
    "u15c_attention_paged": (ip, [vp, vp, vp, vp, vp, ip, vp, ip, ip, ip, ip, ip, ip, ip, vp,
                                  vp]),
    "u15c_attention_sage_static": (ip, [vp, vp, vp, vp, vp, ip, vp, ip, ip, ip, ip, ip]),
    "u15c_sdpa": (ip, [vp, vp, vp, vp, vp, ip, ip, ip, ip, ip, ip, ip, ip]),
    "u15c_sdpa_steel": (ip, [vp, vp, vp, vp, vp, ip, ip, ip, ip, ip, ip, vp]),
    "u15c_sdpa_block_causal": (ip, [vp, vp, vp, vp, vp, vp, ip, ip, ip, ip, ip, ip, ip]),
    "u15c_velocity": (ip, [vp, vp, vp, vp, C.c_long, C.c_double]),
    "u15c_cfg_workspace_bytes": (C.c_size_t, []),
    "u15c_cfg_combine": (ip, [vp, vp, vp, vp, vp, ip, ip, ip, ip, C.c_double, C.c_double, ip,
                              vp]),
    "u15c_euler": (ip, [vp, vp, vp, C.c_long, C.c_double]),
    "u15c_patchify": (ip, [vp, vp, vp, ip, ip]),
    "u15c_embed_tokens": (ip, [vp, vp, ip, ip, vp, ip, vp]),
    "u15c_dequant_affine": (ip, [vp, vp, vp, vp, ip, ip, ip, ip, ip, vp]),
    "u15c_thw_indexes": (ip, [vp, ip, ip, ip, vp, ip, vp, vp, vp]),
    "u15c_splice_image_rows": (ip, [vp, vp, ip, vp, ip, ip, C.POINTER(vp), i32p, ip]),
    "u15c_image_create": (ip, [C.POINTER(ImageConfig), C.POINTER(vp)]),
    "u15c_image_destroy": (None, [vp]),
    "u15c_image_bind": (ip, [vp, vp, ip, ip, vp, ip, ip]),
    "u15c_image_bind_random": (ip, [vp, vp, C.c_uint64, C.c_float]),
    "u15c_image_patchify": (ip, [vp, vp, vp, ip, ip, ip]),
    "u15c_image_embed": (ip, [vp, vp, vp, ip, ip, ip, vp]),
    "u15c_image_timestep_row": (ip, [vp, vp, C.c_double, C.c_double, vp]),
    "u15c_image_add_timestep": (ip, [vp, vp, vp, ip, C.c_double, C.c_double]),
    "u15c_image_decode": (ip, [vp, vp, vp, ip, ip, vp]),
    "u15c_image_to_u8_planar": (ip, [vp, vp, vp, ip, ip]),
    "u15c_unpatchify": (ip, [vp, vp, vp, ip, ip]),
    "u15c_model_create": (ip, [C.POINTER(Config), C.c_uint, C.POINTER(vp)]),
    "u15c_model_destroy": (None, [vp]),
    "u15c_model_create_tp": (ip, [C.POINTER(Config), C.c_uint, ip, ip, C.POINTER(vp)]),
    "u15c_model_tp": (ip, [vp, i32p, i32p]),
    "u15c_model_set_sage_dense_layers": (ip, [vp, ip]),
    "u15c_model_set_allreduce": (ip, [vp, ALLREDUCE_FN, vp, vp, C.c_long]),
    "u15c_model_tp_export": (ip, [vp, ip, vp]),
    "u15c_model_tp_import": (ip, [vp, vp]),
    "u15c_model_tp_disconnect": (ip, [vp]),
    "u15c_model_bind": (ip, [vp, vp, ip, ip, ip, vp, ip, ip]),
    "u15c_model_bind_random": (ip, [vp, vp, C.c_uint64, C.c_float, C.c_float, C.c_float]),
    "u15c_model_finalize": (ip, [vp, vp]),
    "u15c_model_weight_bytes": (C.c_size_t, [vp]),
    "u15c_model_scratch_bytes": (C.c_size_t, [vp, ip]),
    "u15c_model_kv_bytes": (C.c_size_t, [vp, ip]),
    "u15c_kv_create": (ip, [vp, ip, C.POINTER(vp)]),
    "u15c_kv_destroy": (None, [vp]),
    "u15c_kv_capacity": (ip, [vp]),
    "u15c_kv_set_page_table": (ip, [vp, i32p, ip]),
    "u15c_kv_pages": (ip, [vp, ip, C.POINTER(vp), C.POINTER(vp), C.POINTER(vp),
                           C.POINTER(C.c_int)]),
    "u15c_kv_read": (ip, [vp, vp, ip, ip, vp, ip]),
    "u15c_kv_write": (ip, [vp, vp, ip, ip, vp, ip]),
    "u15c_layer_forward": (ip, [vp, vp, ip, vp, ip, i32p, i32p, ip, vp, ip, ip, vp, vp, vp, ip,
                                vp, C.c_uint]),
    "u15c_forward": (ip, [vp, vp, vp, ip, i32p, i32p, ip, vp, ip, ip, vp, vp, vp, ip, vp,
                          C.c_uint, STOP_FN, vp]),
    "u15c_forward_many": (ip, [vp, vp, vp, ip, C.POINTER(Slot), ip, ip, ip, C.c_uint, STOP_FN,
                               vp]),
    "u15c_final_norm": (ip, [vp, vp, vp, ip, ip]),
    "u15c_layer_forward_host": (ip, [vp, vp, ip, vp, vp, ip, i32p, i32p, ip, vp, ip, ip, vp, vp,
                                     vp, ip, vp, C.c_uint]),
    "u15c_layer_forward_host_async": (ip, [vp, vp, ip, vp, vp, ip, i32p, i32p, ip, vp, ip, ip, vp,
                                           vp, vp, ip, vp, C.c_uint]),
    "u15c_layer_host_drain": (ip, [vp, vp]),
}

_lib = None


def header_symbols() -> list[str]:
    """Every function include/u15c.h declares."""
    txt = open(HEADER).read()
    return re.findall(r"^\s*(?:int|void|size_t|const char\*)\s+(u15c_\w+)\(", txt, re.M)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise U15Error(ECUDA, f"{LIB_PATH} is missing: run vpipe-sensenova-u1.5_b200/build.py")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def check(rc: int) -> None:
    if rc != OK:
        raise U15Error(rc, lib().u15c_last_error().decode())


def last_error() -> str:
    return lib().u15c_last_error().decode()
