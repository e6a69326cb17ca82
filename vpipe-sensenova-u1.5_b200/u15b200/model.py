"""Model, KV cache and backbone handles over libu15c's C ABI: the Python
face of U15Weights (bind), KvCache and U15Backbone (src/u15-weights.h,
src/u15-backbone.h of the reference)."""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from . import _lib as L
from ._lib import check, lib
from .ops import _p, _stream, segments_arrays

FULL = dict(n_layers=42, hidden=4096, heads=32, kv_heads=8, head_dim=128, inter=12288,
            n_experts=2, eps=1e-6, theta_t=5e6, theta_hw=1e4)


class Model:
    """U15Weights + U15Backbone for one device, or this rank's share of a
    tensor-parallel model (tp_size > 1: bind full tensors, then install the
    all-reduce with set_allreduce before the first pass)."""

    def __init__(self, int8: bool = False, tp_rank: int = 0, tp_size: int = 1, **cfg):
        c = dict(FULL)
        c.update(cfg)
        self.cfg = c
        self._cfg = L.Config(**c)
        h = C.c_void_p()
        check(lib().u15c_model_create_tp(C.byref(self._cfg), L.MODEL_INT8 if int8 else 0,
                                         tp_rank, tp_size, C.byref(h)))
        self.h = h
        self.int8 = int8
        self.tp_rank, self.tp_size = tp_rank, tp_size
        self._ar_cb = None
        self._part = None

    def set_allreduce(self, group, max_tokens: int) -> None:
        """Sum the row-parallel partial products over `group` with
        torch.distributed.all_reduce (NCCL on GPUs), on the stream of the pass."""
        import torch.distributed as dist
        self._part = torch.empty(max_tokens * self.cfg["hidden"], dtype=torch.float32,
                                 device="cuda")
        part = self._part

        def _ar(_ctx, count, _stream):
            try:
                dist.all_reduce(part[:count], group=group)
                return 0
            except Exception:   # reported to the caller as the pass's error
                return 1

        self._ar_cb = L.ALLREDUCE_FN(_ar)
        check(lib().u15c_model_set_allreduce(self.h, self._ar_cb, None, _p(part), part.numel()))

    def tp_connect(self, group, max_tokens: int) -> None:
        """The fused form: o_proj / down_proj and their all-reduce in one kernel
        over NVLink peer memory. Exchanges the ranks' peer-region handles over
        `group` (an all-gather of small host blobs)."""
        import torch.distributed as dist
        blob = (C.c_char * L.TP_BLOB_BYTES)()
        check(lib().u15c_model_tp_export(self.h, max_tokens, blob))
        blobs = [None] * self.tp_size
        dist.all_gather_object(blobs, bytes(blob), group=group)
        arr = (C.c_char * (L.TP_BLOB_BYTES * self.tp_size)).from_buffer_copy(b"".join(blobs))
        check(lib().u15c_model_tp_import(self.h, arr))

    def tp_disconnect(self, group) -> None:
        """Unmap the peers' regions, then meet the other ranks: after this
        every rank may destroy its model."""
        import torch.distributed as dist
        check(lib().u15c_model_tp_disconnect(self.h))
        dist.barrier(group=group)

    def close(self):
        if self.h:
            lib().u15c_model_destroy(self.h)
            self.h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ---- bind (U15Weights::load) --------------------------------------
    def bind(self, layer: int, expert: int, name: str, array) -> None:
        """Bind one tensor from a host numpy array (f32/f16) or a CUDA tensor
        (f32/f16/bf16)."""
        tid = L.TENSORS.index(name)
        if isinstance(array, np.ndarray):
            a = np.ascontiguousarray(array)
            dt = {np.dtype(np.float32): L.DT_F32, np.dtype(np.float16): L.DT_F16}[a.dtype]
            check(lib().u15c_model_bind(self.h, _stream(), layer, expert, tid,
                                        C.c_void_p(a.ctypes.data), dt, 1))
            torch.cuda.current_stream().synchronize()
        else:
            a = array.contiguous()
            dt = {torch.float32: L.DT_F32, torch.float16: L.DT_F16,
                  torch.bfloat16: L.DT_BF16}[a.dtype]
            check(lib().u15c_model_bind(self.h, _stream(), layer, expert, tid, _p(a), dt, 0))

    def bind_expert_layer(self, layer: int, expert: int, weights: dict) -> None:
        for k, v in weights.items():
            self.bind(layer, expert, k, v)

    def bind_random(self, seed: int, std: float = 0.02, norm_mean: float = 1.0,
                    norm_std: float = 0.0) -> None:
        check(lib().u15c_model_bind_random(self.h, _stream(), seed, std, norm_mean, norm_std))

    def finalize(self) -> None:
        check(lib().u15c_model_finalize(self.h, _stream()))

    def set_sage_dense_layers(self, n: int) -> None:
        """Sage's `dense_layers`: with sage=True, layers [0, n) keep the bf16
        attention (src/u15-metal-ops.cc:852-855)."""
        check(lib().u15c_model_set_sage_dense_layers(self.h, n))

    def weight_bytes(self) -> int:
        return lib().u15c_model_weight_bytes(self.h)

    def scratch_bytes(self, n: int) -> int:
        return lib().u15c_model_scratch_bytes(self.h, n)

    def kv_bytes(self, capacity: int) -> int:
        return lib().u15c_model_kv_bytes(self.h, capacity)

    def make_cache(self, capacity: int) -> "KvCache":
        return KvCache(self, capacity)

    # ---- backbone -----------------------------------------------------
    def layer_forward(self, layer, x, kv, kv_off, kv_len, pos_t, pos_h, pos_w, segments=None,
                      attn=L.ATTN_BIDIRECTIONAL, t_index=None, int8=False, sage=False):
        n = x.shape[0]
        off, ex, ns = segments_arrays(segments, n)
        flags = (L.FWD_INT8 if int8 else 0) | (L.FWD_SAGE if sage else 0)
        check(lib().u15c_layer_forward(self.h, _stream(), layer, _p(x), n, off, ex, ns, kv.h,
                                       kv_off, kv_len, _p(pos_t), _p(pos_h), _p(pos_w), attn,
                                       _p(t_index), flags))

    def forward(self, x, kv, kv_off, kv_len, pos_t, pos_h, pos_w, segments=None,
                attn=L.ATTN_BIDIRECTIONAL, t_index=None, int8=False, sage=False, stop=None):
        n = x.shape[0]
        off, ex, ns = segments_arrays(segments, n)
        flags = (L.FWD_INT8 if int8 else 0) | (L.FWD_SAGE if sage else 0)
        cb = L.STOP_FN(lambda _ctx: int(bool(stop()))) if stop is not None else L.STOP_FN()
        check(lib().u15c_forward(self.h, _stream(), _p(x), n, off, ex, ns, kv.h, kv_off, kv_len,
                                 _p(pos_t), _p(pos_h), _p(pos_w), attn, _p(t_index), flags, cb,
                                 None))

    def forward_many(self, x, n, slots, expert=L.EXPERT_GEN, attn=L.ATTN_BIDIRECTIONAL,
                     int8=False, sage=False, stop=None):
        """x [len(slots) * n][hidden]; slots: list of dicts with kv, kv_off, kv_len,
        pos (t, h, w device int32 tensors) and optional t_index."""
        arr = (L.Slot * len(slots))()
        for i, s in enumerate(slots):
            pt, ph, pw = s["pos"]
            arr[i] = L.Slot(s["kv"].h, s["kv_off"], s["kv_len"], pt.data_ptr(), ph.data_ptr(),
                            pw.data_ptr(), s["t_index"].data_ptr() if s.get("t_index") is not None
                            else None)
        flags = (L.FWD_INT8 if int8 else 0) | (L.FWD_SAGE if sage else 0)
        cb = L.STOP_FN(lambda _ctx: int(bool(stop()))) if stop is not None else L.STOP_FN()
        check(lib().u15c_forward_many(self.h, _stream(), _p(x), n, arr, len(slots), expert, attn,
                                      flags, cb, None))

    def final_norm(self, x, expert):
        check(lib().u15c_final_norm(self.h, _stream(), _p(x), x.shape[0], expert))

    def layer_forward_host(self, layer, x_host, out_host, kv, kv_off, kv_len, pos_t, pos_h,
                           pos_w, segments=None, attn=L.ATTN_BIDIRECTIONAL, t_index=None,
                           int8=False, sage=False):
        n = x_host.shape[0]
        off, ex, ns = segments_arrays(segments, n)
        flags = (L.FWD_INT8 if int8 else 0) | (L.FWD_SAGE if sage else 0)
        check(lib().u15c_layer_forward_host(self.h, _stream(), layer, _p(x_host), _p(out_host),
                                            n, off, ex, ns, kv.h, kv_off, kv_len, _p(pos_t),
                                            _p(pos_h), _p(pos_w), attn, _p(t_index), flags))

    def layer_forward_host_async(self, layer, x_host, out_host, kv, kv_off, kv_len, pos_t, pos_h,
                                 pos_w, segments=None, attn=L.ATTN_BIDIRECTIONAL, t_index=None,
                                 int8=False, sage=False):
        """Enqueue the layer through pinned host buffers without waiting
        (u15c_layer_forward_host_async): x_host must stay unchanged and
        out_host unread until host_drain() and a stream synchronisation."""
        n = x_host.shape[0]
        off, ex, ns = segments_arrays(segments, n)
        flags = (L.FWD_INT8 if int8 else 0) | (L.FWD_SAGE if sage else 0)
        check(lib().u15c_layer_forward_host_async(self.h, _stream(), layer, _p(x_host),
                                                  _p(out_host), n, off, ex, ns, kv.h, kv_off,
                                                  kv_len, _p(pos_t), _p(pos_h), _p(pos_w), attn,
                                                  _p(t_index), flags))

    def host_drain(self):
        """Make the current stream wait for every download the async host
        path has enqueued (u15c_layer_host_drain)."""
        check(lib().u15c_layer_host_drain(self.h, _stream()))


class KvCache:
    """Paged bf16 KV cache for every layer of one branch."""

    def __init__(self, model: Model, capacity: int):
        self.model = model
        h = C.c_void_p()
        check(lib().u15c_kv_create(model.h, capacity, C.byref(h)))
        self.h = h
        self.capacity = capacity
        self.pages = (capacity + 63) // 64

    def close(self):
        if self.h:
            lib().u15c_kv_destroy(self.h)
            self.h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_page_table(self, pages):
        arr = (C.c_int * len(pages))(*[int(p) for p in pages])
        check(lib().u15c_kv_set_page_table(self.h, arr, len(pages)))

    def read(self, layer: int, v: bool, n: int) -> torch.Tensor:
        hkv = self.model.cfg["kv_heads"] // self.model.tp_size   # this rank's kv heads
        out = torch.empty(hkv, n, 128, dtype=torch.bfloat16, device="cuda")
        check(lib().u15c_kv_read(self.h, _stream(), layer, int(v), _p(out), n))
        return out

    def write(self, layer: int, v: bool, data: torch.Tensor) -> None:
        d = data.contiguous()
        check(lib().u15c_kv_write(self.h, _stream(), layer, int(v), _p(d), d.shape[1]))
