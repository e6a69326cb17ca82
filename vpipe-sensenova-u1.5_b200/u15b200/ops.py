"""CudaOps: the reference's MetalOps operator vocabulary
(src/u15-metal-ops.h:59-403 of the reference) over libu15c's C ABI.

Method names, argument meaning and order follow MetalOps; where MetalOps
takes an encoder, these take the current torch CUDA stream; buffers are
torch CUDA tensors (bf16 unless named otherwise) standing in for
SharedBuffers. Errors raise U15Error (the reference returns bool + err).
torch supplies device memory and streams only; every computation runs in
libu15c's kernels.
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib as L
from ._lib import check, lib


def _p(t):
    return None if t is None else C.c_void_p(t.data_ptr())


def _stream():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def segments_arrays(segments, rows):
    """[(start, end, expert), ...] -> (off int[n+1], expert int[n], n)."""
    if not segments:
        segments = [(0, rows, 0)]
    n = len(segments)
    off = (C.c_int * (n + 1))(*([s[0] for s in segments] + [segments[-1][1]]))
    ex = (C.c_int * n)(*[s[2] for s in segments])
    return off, ex, n


def _bf16(t):
    if t.dtype != torch.bfloat16 or not t.is_cuda or not t.is_contiguous():
        raise L.U15Error(L.EINVAL, "expected a contiguous CUDA bf16 tensor")
    return t


class CudaOps:
    """MetalOps mirror. One instance per device; stateless apart from that."""

    def __init__(self, device: int = 0):
        self.device = device
        check(lib().u15c_init(device, 0))

    # ---- GEMMs -------------------------------------------------------
    def linear(self, x, w, bias, y, M, K, N):
        check(lib().u15c_linear_bf16(_stream(), _p(_bf16(x)), _p(_bf16(w)), _p(bias), _p(y),
                                     M, K, N))

    def mot_linear(self, x, w_stack, segments, y, M, K, N, epilogue=L.EPI_STORE, bias=None,
                   resid=None):
        off, ex, n = segments_arrays(segments, M)
        check(lib().u15c_mot_linear_bf16(_stream(), _p(x), _p(w_stack), w_stack.shape[0], off,
                                         ex, n, epilogue, _p(bias), _p(resid), _p(y), M, K, N))

    def quant_rows_i8(self, x, q, scale, rows, cols):
        check(lib().u15c_quant_rows_i8(_stream(), _p(x), _p(q), _p(scale), rows, cols))

    def linear_i8(self, xq, s_tok, wq, s_ch, y, M, K, N, bias=None, acc_dump=None):
        check(lib().u15c_linear_i8(_stream(), _p(xq), _p(s_tok), _p(wq), _p(s_ch), _p(bias),
                                   _p(y), _p(acc_dump), M, K, N))

    def mot_linear_i8(self, xq, s_tok, wq_stack, s_ch_stack, segments, y, M, K, N,
                      epilogue=L.EPI_STORE, resid=None, acc_dump=None):
        off, ex, n = segments_arrays(segments, M)
        check(lib().u15c_mot_linear_i8(_stream(), _p(xq), _p(s_tok), _p(wq_stack),
                                       _p(s_ch_stack), wq_stack.shape[0], off, ex, n, epilogue,
                                       _p(resid), _p(y), _p(acc_dump), M, K, N))

    # ---- norms, rope, layout -----------------------------------------
    def rms_norm(self, x, w, y, rows, dim, eps):
        check(lib().u15c_rms_norm(_stream(), _p(x), _p(w), _p(y), rows, dim, eps))

    def mot_rms_norm(self, x, w_stack, segments, y, rows, dim, eps):
        off, ex, n = segments_arrays(segments, rows)
        check(lib().u15c_mot_rms_norm(_stream(), _p(x), _p(w_stack), w_stack.shape[0], off, ex,
                                      n, _p(y), rows, dim, eps))

    def mot_rms_norm_quant_i8(self, x, w_stack, segments, q, scale, rows, dim, eps):
        off, ex, n = segments_arrays(segments, rows)
        check(lib().u15c_mot_rms_norm_quant_i8(_stream(), _p(x), _p(w_stack), w_stack.shape[0],
                                               off, ex, n, _p(q), _p(scale), rows, dim, eps))

    def split_qk_norm(self, x, w_t, w_hw, heads, tokens, head_dim, eps):
        check(lib().u15c_split_qk_norm(_stream(), _p(x), _p(w_t), _p(w_hw), heads, tokens,
                                       head_dim, eps))

    def split_rope(self, x, cos, sin, heads, tokens, head_dim, d_t, d_h):
        check(lib().u15c_split_rope(_stream(), _p(x), _p(cos), _p(sin), heads, tokens,
                                    head_dim, d_t, d_h))

    def build_rope_tables(self, pos_t, pos_h, pos_w, head_dim=128, d_t=64, d_h=32,
                          theta_t=5e6, theta_hw=1e4):
        """Returns (cos, sin) f32 [T][head_dim]; positions are int32 CUDA tensors."""
        T = pos_t.numel()
        c = torch.empty(T, head_dim, dtype=torch.float32, device=pos_t.device)
        s = torch.empty_like(c)
        check(lib().u15c_build_rope_tables(_stream(), _p(pos_t), _p(pos_h), _p(pos_w), T,
                                           head_dim, d_t, d_h, theta_t, theta_hw, _p(c), _p(s)))
        return c, s

    def qkv_post(self, qkv, norms_stack, segments, cos, sin, q_out, k_cache, v_cache,
                 page_table, cap, heads, kv_heads, T, kv_off, eps):
        off, ex, n = segments_arrays(segments, T)
        check(lib().u15c_qkv_post(_stream(), _p(qkv), _p(norms_stack), norms_stack.shape[0],
                                  off, ex, n, _p(cos), _p(sin), _p(q_out), _p(k_cache),
                                  _p(v_cache), _p(page_table), cap, heads, kv_heads, T, kv_off,
                                  eps))

    def transpose_thd(self, x, out, T, H, D):
        check(lib().u15c_transpose_thd(_stream(), _p(x), _p(out), T, H, D))

    def transpose_htd(self, x, out, T, H, D):
        check(lib().u15c_transpose_htd(_stream(), _p(x), _p(out), T, H, D))

    def transpose_into_cache(self, x, cache, T, H, D, cap, offset):
        check(lib().u15c_transpose_into_cache(_stream(), _p(x), _p(cache), T, H, D, cap,
                                              offset))

    def kv_append(self, x, pages, page_table, T, H, offset):
        check(lib().u15c_kv_append(_stream(), _p(x), _p(pages), _p(page_table), T, H, offset))

    # ---- elementwise -------------------------------------------------
    def swiglu(self, gate, up, y, rows, inter):
        check(lib().u15c_swiglu(_stream(), _p(gate), _p(up), _p(y), rows, inter))

    def add(self, dst, src, n):
        check(lib().u15c_add(_stream(), _p(dst), _p(src), n))

    def add_row(self, dst, row, rows, dim):
        check(lib().u15c_add_row(_stream(), _p(dst), _p(row), rows, dim))

    def silu(self, x, n):
        check(lib().u15c_silu(_stream(), _p(x), n))

    # ---- attention ---------------------------------------------------
    def sage_workspace(self, hq, hkv, tq, tk, device="cuda"):
        n = lib().u15c_sage_workspace_bytes(hq, hkv, tq, tk)
        return torch.empty(n, dtype=torch.uint8, device=device)

    def attention(self, q, k, v, out, hq, hkv, tq, tk, cap=0, page_table=None,
                  mode=L.ATTN_BIDIRECTIONAL, q_offset=0, t_index=None, sage_ws=None):
        check(lib().u15c_attention(_stream(), _p(q), _p(k), _p(v), _p(page_table), cap, _p(out),
                                   hq, hkv, tq, tk, 128, mode, q_offset, _p(t_index),
                                   _p(sage_ws)))

    def attention_paged(self, q, k_pages, vt_pages, out, hq, hkv, tq, tk, page_table=None,
                        n_pages=None, mode=L.ATTN_BIDIRECTIONAL, q_offset=0, t_index=None,
                        sage_ws=None):
        """The model's cache layout: K pages [P][hkv][64][128], V pages transposed
        [P][hkv][128][64]; bidirectional runs the tcgen05 kernel."""
        n_pages = k_pages.shape[0] if n_pages is None else n_pages
        check(lib().u15c_attention_paged(_stream(), _p(q), _p(k_pages), _p(vt_pages),
                                         _p(page_table), n_pages, _p(out), hq, hkv, tq, tk, 128,
                                         mode, q_offset, _p(t_index), _p(sage_ws)))

    def sdpa(self, q, k, v, out, hq, hkv, tq, tk, d, cap, causal, q_offset=0):
        check(lib().u15c_sdpa(_stream(), _p(q), _p(k), _p(v), _p(out), hq, hkv, tq, tk, d, cap,
                              int(causal), q_offset))

    def sdpa_steel(self, q, k, v, out, hq, hkv, tq, tk, d, cap, sage_ws=None):
        check(lib().u15c_sdpa_steel(_stream(), _p(q), _p(k), _p(v), _p(out), hq, hkv, tq, tk, d,
                                    cap, _p(sage_ws)))

    def sdpa_block_causal(self, q, k, v, out, t_index, hq, hkv, tq, tk, d, cap, q_offset):
        check(lib().u15c_sdpa_block_causal(_stream(), _p(q), _p(k), _p(v), _p(out),
                                           _p(t_index), hq, hkv, tq, tk, d, cap, q_offset))

    # ---- status ------------------------------------------------------
    def sync(self):
        check(lib().u15c_sync(_stream()))

    def device_status(self) -> int:
        code = C.c_uint(0)
        check(lib().u15c_device_status(self.device, C.byref(code)))
        return code.value
