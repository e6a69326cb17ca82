// The model half of the C ABI: the bound weight layout (U15Weights' bind
// step), the paged KV cache (KvCache) and the backbone layer/stack
// (U15Backbone::layer_step_ / forward), src/u15-weights.*, u15-backbone.*
// in the reference.
//
// Bound layout, per layer, experts stacked on the outer axis:
//   qkv   [E][(NH + 2*KV) * HD][H]   q rows, then k rows, then v rows
//   o     [E][H][NH * HD]
//   gu    [E][2 * I][H]              128-row blocks [gate_j | up_j] for the
//                                    SwiGLU epilogue
//   down  [E][H][I]
//   ln_in, ln_post [E][H]; norms [E][4][64] = q_norm, q_norm_hw, k_norm, k_norm_hw
//   (INT8) the same four matrices as per-output-channel int8 plus f32 scales
// The GEMM's TMA maps tile these row-major buffers into 128-byte-swizzled
// shared-memory tiles; no further repacking pays at these shapes.
//
// Paged KV cache: per layer a K and a V pool [pages][KV][64][128] bf16,
// one logical->physical page table shared by all layers.
#include "u15_capi_internal.h"
#include "u15_common.cuh"

#include <algorithm>
#include <cstring>
#include <vector>

using u15::fail;
using u15::cuda_fail;
using u15::DeviceScope;

namespace {

using bf16 = __nv_bfloat16;

struct LayerW {
  bf16* qkv = nullptr;
  bf16* o = nullptr;
  bf16* gu = nullptr;
  bf16* down = nullptr;
  bf16* ln_in = nullptr;
  bf16* ln_post = nullptr;
  bf16* norms = nullptr;
  int8_t* qkv8 = nullptr;
  int8_t* o8 = nullptr;
  int8_t* gu8 = nullptr;
  int8_t* down8 = nullptr;
  float* qkv_s = nullptr;
  float* o_s = nullptr;
  float* gu_s = nullptr;
  float* down_s = nullptr;
};

// ---------------------------------------------------------------------
// kernels: dtype conversion into the bound layout, seeded init
// ---------------------------------------------------------------------
__device__ __forceinline__ float src_value(const void* src, int dtype, long i)
{
  if (dtype == U15C_DT_F32) return static_cast<const float*>(src)[i];
  if (dtype == U15C_DT_F16) return __half2float(static_cast<const __half*>(src)[i]);
  return __bfloat162float(static_cast<const bf16*>(src)[i]);
}

// Element (r, c) of the [rows][cols] destination comes from source element
// (src_r0 + r, src_c0 + c) of a row-major source with src_ld columns: the
// whole tensor, or (tensor parallelism) this rank's rows or columns of it.
// dst row for r: r, or (interleave >= 0) the gate/up block layout
// (r/128)*256 + interleave*128 + r%128.
__global__ void bind_kernel(const void* src, int dtype, long rows, long cols, long src_ld,
                            long src_r0, long src_c0, bf16* dst, int interleave)
{
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * cols) return;
  const long r = i / cols, c = i % cols;
  long dr = r;
  if (interleave >= 0) dr = (r / 128) * 256 + interleave * 128 + r % 128;
  dst[dr * cols + c] =
      __float2bfloat16_rn(src_value(src, dtype, (src_r0 + r) * src_ld + src_c0 + c));
}

// x = bf16(x + bf16(sum)): the residual epilogue's rounding points, applied
// after the ranks' f32 partial products were summed.
__global__ void resid_add_f32_kernel(bf16* x, const float* sum, long n)
{
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float proj = __bfloat162float(__float2bfloat16_rn(sum[i]));
  x[i] = __float2bfloat16_rn(__bfloat162float(x[i]) + proj);
}

__device__ __forceinline__ uint64_t splitmix(uint64_t x)
{
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

// N(mean, std) by Box-Muller on a counter hash (seed, stream, index).
__global__ void randn_kernel(bf16* dst, long n, uint64_t seed, uint64_t stream, float mean,
                             float std)
{
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const uint64_t h = splitmix(seed ^ splitmix(stream * 0x100000001B3ull + (uint64_t)i));
  const float u1 = ((float)(h >> 40) + 1.0f) * (1.0f / 16777217.0f);
  const float u2 = (float)((h >> 16) & 0xFFFFFF) * (1.0f / 16777216.0f);
  const float z = sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
  dst[i] = __float2bfloat16_rn(mean + std * z);
}

inline unsigned nblk(long n, int t) { return (unsigned)((n + t - 1) / t); }

}  // namespace

struct u15c_model {
  // cfg: this rank's share (heads, kv_heads and inter divided by tp_size);
  // full: the model as the caller described it (bind reads full tensors)
  u15c_config cfg{};
  u15c_config full{};
  int tp_rank = 0, tp_size = 1;
  // tensor parallelism: the caller's all-reduce of part[0 : count) (f32 sum
  // over the ranks, in place, ordered on the stream)
  u15c_allreduce_fn ar_fn = nullptr;
  void* ar_ctx = nullptr;
  float* part = nullptr;
  long part_elems = 0;
  // tensor parallelism fused over peer memory (u15c_model_tp_export/import):
  // this rank's region [inbox | x | arrive | done], the peers' mappings of
  // theirs, and the done count every rank reaches after each fused product
  void* tp_mem = nullptr;
  int tp_rows = 0;
  void* tp_peer[u15::kMaxTp] = {};
  u15::TpPeers tpp;
  bool tp_fused = false;
  unsigned long long tp_done_target = 0;
  unsigned flags = 0;
  int device = 0;
  // layers [0, sage_dense_layers) keep the bf16 attention under U15C_FWD_SAGE
  int sage_dense_layers = 0;
  std::vector<LayerW> layers;
  bf16* final_norm = nullptr;   // [E][H]
  size_t weight_bytes = 0;
  std::vector<void*> allocs;

  // grow-only activation arena (U15Backbone::ensure_scratch_)
  int scratch_n = 0;
  int scratch_tk = 0;
  bf16* xn = nullptr;
  bf16* qkv = nullptr;
  bf16* qh = nullptr;
  bf16* attn = nullptr;
  bf16* h = nullptr;
  float* rcos = nullptr;
  float* rsin = nullptr;
  int8_t* x8 = nullptr;
  float* s_tok = nullptr;
  void* sage_ws = nullptr;
  size_t sage_ws_bytes = 0;
  bf16* io = nullptr;   // layer_forward_host staging
  // layer_forward_host's copy stream and its chunk events (made on first use)
  cudaStream_t copy_st = nullptr;
  cudaEvent_t copy_ev[2 * 4 + 1] = {};
  // layer_forward_host_async: two staging buffers used in turn, an upload and
  // a download stream (so one call's upload overlaps the previous call's
  // download), per staging buffer its upload-landed, layer-done and
  // download-done events (the last: the buffer is free again); made on first
  // use, grow-only
  bf16* hio[2] = {};
  int hio_n = 0;
  int hio_next = 0;
  bool hio_used[2] = {};
  cudaStream_t up_st = nullptr, down_st = nullptr;
  cudaEvent_t hio_in[2][1] = {}, hio_out[2][1] = {}, hio_free[2] = {};
  // forward_many's branch attentions run on these beside the model's stream
  // (made on first use), so one branch's last part-empty round of CTAs is
  // filled by the next branch's
  static constexpr int kSideStreams = 3;
  cudaStream_t side_st[kSideStreams] = {};
  cudaEvent_t side_ev[kSideStreams + 1] = {};   // [i]: side i done; [last]: inputs ready
  // a Sage workspace per side stream, so that Sage slots can run side by side
  // (grown on first use to the largest slot's size)
  void* side_sage[kSideStreams] = {};
  size_t side_sage_bytes = 0;
  std::vector<void*> scratch_allocs;

  int qkv_n() const { return (cfg.heads + 2 * cfg.kv_heads) * cfg.head_dim; }
  int qd() const { return cfg.heads * cfg.head_dim; }

  template <class T>
  int alloc(T** p, size_t bytes, std::vector<void*>& list)
  {
    const cudaError_t e = cudaMalloc(reinterpret_cast<void**>(p), bytes);
    if (e != cudaSuccess) return fail(U15C_ENOMEM, "out of device memory (" +
                                                       std::to_string(bytes >> 20) + " MB)");
    list.push_back(*p);
    return U15C_OK;
  }

  void free_side_sage()
  {
    for (void*& p : side_sage) {
      if (p) cudaFree(p);
      p = nullptr;
    }
    side_sage_bytes = 0;
  }

  int ensure_side_sage(size_t bytes)
  {
    if (bytes <= side_sage_bytes) return U15C_OK;
    free_side_sage();
    for (void*& p : side_sage)
      if (cudaMalloc(&p, bytes) != cudaSuccess) {
        free_side_sage();
        return fail(U15C_ENOMEM, "out of device memory (Sage side workspaces, " +
                                     std::to_string(bytes >> 20) + " MB each)");
      }
    side_sage_bytes = bytes;
    return U15C_OK;
  }

  void free_scratch()
  {
    for (void* p : scratch_allocs) cudaFree(p);
    scratch_allocs.clear();
    scratch_n = 0;
    scratch_tk = 0;
    sage_ws = nullptr;
    sage_ws_bytes = 0;
    free_side_sage();
  }

  int ensure_scratch(int n, int tk)
  {
    if (n <= scratch_n && tk <= scratch_tk) return U15C_OK;
    free_scratch();
    n = std::max(n, 1);
    tk = std::max(tk, n);
    const size_t H = cfg.hidden, I = cfg.inter;
    const size_t maxk = std::max({H, I, (size_t)qd()});
    int rc = 0;
    rc |= alloc(&xn, n * H * 2, scratch_allocs);
    rc |= alloc(&qkv, (size_t)n * qkv_n() * 2, scratch_allocs);
    rc |= alloc(&qh, (size_t)n * qd() * 2, scratch_allocs);
    rc |= alloc(&attn, (size_t)n * qd() * 2, scratch_allocs);
    rc |= alloc(&h, n * I * 2, scratch_allocs);
    rc |= alloc(&rcos, (size_t)n * 128 * 4, scratch_allocs);
    rc |= alloc(&rsin, (size_t)n * 128 * 4, scratch_allocs);
    rc |= alloc(&x8, n * maxk, scratch_allocs);
    rc |= alloc(&s_tok, (size_t)n * 4, scratch_allocs);
    rc |= alloc(&io, n * H * 2, scratch_allocs);
    sage_ws_bytes = u15::sage_bytes(cfg.heads, cfg.kv_heads, n, tk);
    rc |= alloc(reinterpret_cast<uint8_t**>(&sage_ws), sage_ws_bytes, scratch_allocs);
    if (rc) {
      free_scratch();
      return U15C_ENOMEM;
    }
    scratch_n = n;
    scratch_tk = tk;
    return U15C_OK;
  }

  // the async host path's staging and streams (grow-only; a regrowth waits
  // for the copies in flight)
  int ensure_host_staging(int n)
  {
    if (up_st == nullptr) {
      if (cudaStreamCreateWithFlags(&up_st, cudaStreamNonBlocking) != cudaSuccess ||
          cudaStreamCreateWithFlags(&down_st, cudaStreamNonBlocking) != cudaSuccess)
        return fail(U15C_ECUDA, "layer_forward_host_async: copy streams");
      for (int b = 0; b < 2; ++b) {
        if (cudaEventCreateWithFlags(&hio_in[b][0], cudaEventDisableTiming) != cudaSuccess ||
            cudaEventCreateWithFlags(&hio_out[b][0], cudaEventDisableTiming) != cudaSuccess)
          return fail(U15C_ECUDA, "layer_forward_host_async: copy events");
        if (cudaEventCreateWithFlags(&hio_free[b], cudaEventDisableTiming) != cudaSuccess)
          return fail(U15C_ECUDA, "layer_forward_host_async: copy events");
      }
    }
    if (n <= hio_n) return U15C_OK;
    cudaStreamSynchronize(up_st);
    cudaStreamSynchronize(down_st);
    for (bf16*& b : hio) {
      if (b) cudaFree(b);
      b = nullptr;
    }
    hio_n = 0;
    for (bf16*& b : hio)
      if (cudaMalloc(reinterpret_cast<void**>(&b), (size_t)n * cfg.hidden * 2) != cudaSuccess) {
        for (bf16*& c : hio) {
          if (c) cudaFree(c);
          c = nullptr;
        }
        return fail(U15C_ENOMEM, "out of device memory (host-path staging)");
      }
    hio_n = n;
    return U15C_OK;
  }

  ~u15c_model()
  {
    if (up_st) cudaStreamSynchronize(up_st);
    if (down_st) cudaStreamSynchronize(down_st);
    for (int b = 0; b < 2; ++b) {
      if (hio_in[b][0]) cudaEventDestroy(hio_in[b][0]);
      if (hio_out[b][0]) cudaEventDestroy(hio_out[b][0]);
      if (hio_free[b]) cudaEventDestroy(hio_free[b]);
      if (hio[b]) cudaFree(hio[b]);
    }
    if (up_st) cudaStreamDestroy(up_st);
    if (down_st) cudaStreamDestroy(down_st);
    for (cudaEvent_t e : copy_ev)
      if (e) cudaEventDestroy(e);
    if (copy_st) cudaStreamDestroy(copy_st);
    for (cudaEvent_t e : side_ev)
      if (e) cudaEventDestroy(e);
    for (cudaStream_t s : side_st)
      if (s) cudaStreamDestroy(s);
    free_scratch();
    for (int q = 0; q < u15::kMaxTp; ++q)
      if (tp_peer[q] != nullptr && tp_peer[q] != tp_mem) cudaIpcCloseMemHandle(tp_peer[q]);
    if (tp_mem != nullptr) cudaFree(tp_mem);
    for (void* p : allocs) cudaFree(p);
  }
};

struct u15c_kv {
  u15c_model* m = nullptr;
  int capacity = 0;
  int pages = 0;
  long layer_elems = 0;   // elements of one layer's K (or V) pool
  bf16* k = nullptr;      // [layers][pages][KV][64][128]
  bf16* v = nullptr;
  int32_t* table = nullptr;   // [pages]

  u15::KvView view(int layer) const
  {
    u15::KvView kv;
    kv.k = k + (long)layer * layer_elems;
    kv.v = v + (long)layer * layer_elems;
    kv.page_table = table;
    kv.page_stride = (long)m->cfg.kv_heads * u15::kPageTokens * 128;
    kv.head_stride = (long)u15::kPageTokens * 128;
    kv.v_t = true;
    return kv;
  }
  ~u15c_kv()
  {
    cudaFree(k);
    cudaFree(v);
    cudaFree(table);
  }
};

namespace {

int check_cfg(const u15c_config& c)
{
  if (c.n_layers <= 0 || c.hidden <= 0 || c.heads <= 0 || c.kv_heads <= 0 || c.inter <= 0 ||
      c.n_experts <= 0 || c.n_experts > 8)
    return fail(U15C_EINVAL, "model config: sizes must be positive (experts <= 8)");
  if (c.head_dim != 128) return fail(U15C_EINVAL, "model config: head_dim must be 128");
  if (c.heads % c.kv_heads) return fail(U15C_EINVAL, "model config: heads % kv_heads != 0");
  if (c.hidden % 64 || c.inter % 128)
    return fail(U15C_EINVAL, "model config: hidden % 64 and inter % 128 must be 0");
  return U15C_OK;
}

// One branch's share of a layer pass: its rows [row0, row0 + n) of the
// activations, its cache and attention rule. (U15Backbone::PassSlot,
// src/u15-backbone.h:112-124.)
struct SlotRun {
  int row0 = 0, n = 0;
  u15c_kv* kv = nullptr;
  int kv_off = 0, kv_len = 0, attn = 0;
  const int32_t* t_index = nullptr;
};

// Restrict a row-segment map to rows [r0, r0 + n), renumbered from 0.
u15::SegInfo slice_seg(const u15::SegInfo& g, int r0, int n)
{
  u15::SegInfo s;
  s.nseg = 0;
  for (int i = 0; i < g.nseg; ++i) {
    const int lo = std::max(g.off[i], r0), hi = std::min(g.off[i + 1], r0 + n);
    if (lo >= hi) continue;
    s.off[s.nseg] = lo - r0;
    s.expert[s.nseg] = g.expert[i];
    ++s.nseg;
    s.off[s.nseg] = hi - r0;
  }
  if (s.nseg == 0) {
    s.nseg = 1;
    s.off[0] = 0;
    s.off[1] = n;
    s.expert[0] = g.expert[0];
  }
  return s;
}

// One layer over every slot (U15Backbone::layer_step_, src/u15-backbone.cc:
// 173-257). The row-wise steps -- both norms and all four projection GEMMs --
// run once over all M rows of all slots; the QKV post-processing (into each
// slot's own cache) and the attention (over each slot's own keys) run per
// slot. rcos/rsin already hold the tables for all M rows.
// The parts of a layer pass. The row-wise parts (the norm + QKV before the
// attention, o_proj through down_proj after it) can run on a range of rows,
// which is how u15c_layer_forward_host overlaps its host copies with them.
enum LayerPart { kPartPre = 1, kPartAttn = 2, kPartPost = 4, kPartAll = 7 };

int layer_impl(u15c_model* m, cudaStream_t st, int li, bf16* x_all, int M,
               const u15::SegInfo& seg_all, const int* seg_off_all, const int* seg_expert_all,
               int nseg_all, const std::vector<SlotRun>& slots, unsigned flags,
               int parts = kPartAll, int r0 = 0, int rn = -1)
{
  const u15c_config& c = m->cfg;
  const LayerW& L = m->layers[li];
  const int E = c.n_experts, H = c.hidden, I = c.inter;
  const bool i8 = (flags & U15C_FWD_INT8) != 0;
  // the Sage tier leaves a prefix of the stack on the bf16 attention
  // (sdpa_steel's `sage_layer >= dense_layers`, src/u15-metal-ops.cc:852-855)
  if (li < m->sage_dense_layers) flags &= ~U15C_FWD_SAGE;
  if (i8 && L.qkv8 == nullptr)
    return fail(U15C_EINVAL, "W8A8 requested but the model has no int8 twins "
                             "(create with U15C_MODEL_INT8 and call u15c_model_finalize)");
  int rc;
  // the row range of the row-wise parts, its segments renumbered from 0
  const bool whole = r0 == 0 && (rn < 0 || rn == M);
  const int Mr = whole ? M : rn;
  const u15::SegInfo seg = whole ? seg_all : slice_seg(seg_all, r0, Mr);
  int roff[u15::kMaxSeg + 1], rex[u15::kMaxSeg];
  for (int i = 0; i <= seg.nseg; ++i) roff[i] = seg.off[i];
  for (int i = 0; i < seg.nseg; ++i) rex[i] = seg.expert[i];
  const int* seg_off = whole ? seg_off_all : roff;
  const int* seg_expert = whole ? seg_expert_all : rex;
  const int nseg = whole ? nseg_all : seg.nseg;
  bf16* x = x_all + (long)r0 * H;
  // prequant: the activation was already quantised into x8/s_tok (by the
  // fused RMSNorm + quantisation), so the int8 path skips its own pass.
  auto gemm = [&](const void* in, int K, const bf16* w, const int8_t* w8, const float* ws, int N,
                  int epi, void* y, bool prequant = false, int* out_tiles = nullptr) -> int {
    u15::GemmArgs a;
    a.n_experts = E;
    a.M = Mr;
    a.K = K;
    a.N = N;
    a.seg_off = seg_off;
    a.seg_expert = seg_expert;
    a.nseg = nseg;
    a.epilogue = epi;
    a.y = y;
    a.resid = epi == u15::kEpiResid ? x : nullptr;
    if (epi == u15::kEpiTpReduce) {
      a.tp = &m->tpp;
      a.out_tiles = out_tiles;
    }
    if (i8) {
      if (!prequant && u15::launch_quant_rows(in, m->x8, m->s_tok, Mr, K, st))
        return fail(U15C_ECUDA, "quant_rows launch failed");
      a.int8 = true;
      a.x = m->x8;
      a.w = w8;
      a.s_tok = m->s_tok;
      a.s_ch = ws;
    } else {
      a.x = in;
      a.w = w;
    }
    return u15::run_gemm(a, st);
  };
  // o_proj / down_proj + residual. One device: the GEMM's residual
  // epilogue. Tensor parallelism (row-parallel split, this rank holds K/tp of
  // the inner dimension): f32 partial products, the caller's all-reduce sums
  // them across the ranks, then x = bf16(x + bf16(sum)).
  auto row_parallel = [&](const void* in, int K, const bf16* w, const int8_t* w8,
                          const float* ws) -> int {
    if (m->tp_size == 1) return gemm(in, K, w, w8, ws, H, u15::kEpiResid, x);
    if (m->tp_fused) {
      // one kernel: partial products to their owners over NVLink, the
      // owners' sums + residual into every rank's x, then wait for all of x
      int tiles = 0;
      int r = gemm(in, K, w, w8, ws, H, u15::kEpiTpReduce, nullptr, false, &tiles);
      if (r) return r;
      m->tp_done_target += 2ull * (unsigned long long)tiles;
      u15::DevState* d = u15::dev();
      if (u15::launch_tp_wait(m->tpp.done[m->tp_rank], m->tp_done_target, d ? d->err : nullptr,
                              st))
        return fail(U15C_ECUDA, "tensor-parallel wait launch failed");
      return U15C_OK;
    }
    const long n = (long)Mr * H;
    if (m->ar_fn == nullptr || m->part == nullptr || m->part_elems < n)
      return fail(U15C_EINVAL, "tensor-parallel model: no all-reduce installed, or its "
                               "buffer holds fewer than tokens x hidden floats "
                               "(u15c_model_set_allreduce)");
    int r = gemm(in, K, w, w8, ws, H, u15::kEpiStoreF32, m->part);
    if (r) return r;
    if (m->ar_fn(m->ar_ctx, n, static_cast<u15c_stream>(st)) != 0)
      return fail(U15C_ECUDA, "tensor-parallel all-reduce failed");
    resid_add_f32_kernel<<<nblk(n, 256), 256, 0, st>>>(x, m->part, n);
    return cudaGetLastError() == cudaSuccess ? U15C_OK
                                             : fail(U15C_ECUDA, "residual add launch failed");
  };
  // the layer norms: bf16 out, or (W8A8 with hidden <= 4096) fused with the
  // activation quantisation
  const bool fuse_q = i8 && H <= 4096;
  auto norm = [&](const bf16* w) -> int {
    const int r = fuse_q ? u15::launch_rms_norm_quant(x, w, m->x8, m->s_tok, Mr, H, (float)c.eps,
                                                      seg, st)
                         : u15::launch_rms_norm(x, w, m->xn, Mr, H, (float)c.eps, seg, st);
    return r ? fail(U15C_ECUDA, "rms_norm launch failed") : U15C_OK;
  };

  // ---- attention half (src/u15-backbone.cc:191-235) ----
  if (parts & kPartPre) {
    if ((rc = norm(L.ln_in))) return rc;
    if ((rc = gemm(m->xn, H, L.qkv, L.qkv8, L.qkv_s, m->qkv_n(), u15::kEpiStore,
                   m->qkv + (long)r0 * m->qkv_n(), fuse_q)))
      return rc;
  }
  if (parts & kPartAttn) {
    // q / K / V of every slot first; then the attentions. Two or more
    // bidirectional slots run their attentions on side streams beside `st`
    // (forked after the qkv_post kernels, joined before o_proj), so the
    // GPU schedules their CTAs as one pool; with Sage each side stream has
    // its own workspace.
    int n_par = 0;
    size_t side_sage_need = 0;
    for (const SlotRun& sl : slots)
      if (sl.attn == U15C_ATTN_BIDIRECTIONAL) {
        ++n_par;
        if (flags & U15C_FWD_SAGE)
          side_sage_need = std::max(side_sage_need,
                                    u15::sage_bytes(c.heads, c.kv_heads, sl.n, sl.kv_len));
      }
    const bool fork = n_par >= 2 && n_par <= u15c_model::kSideStreams;
    if (fork && side_sage_need && (rc = m->ensure_side_sage(side_sage_need))) return rc;
    if (fork && m->side_st[0] == nullptr) {
      for (cudaStream_t& s : m->side_st)
        if (cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking) != cudaSuccess)
          return fail(U15C_ECUDA, "forward: attention side streams");
      for (cudaEvent_t& e : m->side_ev)
        if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess)
          return fail(U15C_ECUDA, "forward: attention side events");
    }
    for (const SlotRun& sl : slots) {
      const u15::SegInfo sseg = slice_seg(seg_all, sl.row0, sl.n);
      if (u15::launch_qkv_post(m->qkv + (long)sl.row0 * m->qkv_n(), L.norms,
                               m->rcos + (long)sl.row0 * 128, m->rsin + (long)sl.row0 * 128,
                               m->qh + (long)sl.row0 * m->qd(), sl.kv->view(li), sl.n, c.heads,
                               c.kv_heads, sl.kv_off, (float)c.eps, sseg, st))
        return fail(U15C_ECUDA, "qkv_post launch failed");
    }
    if (fork) cudaEventRecord(m->side_ev[u15c_model::kSideStreams], st);
    int k_side = 0;
    for (const SlotRun& sl : slots) {
      const u15::KvView view = sl.kv->view(li);
      bf16* qh = m->qh + (long)sl.row0 * m->qd();
      bf16* out = m->attn + (long)sl.row0 * m->qd();
      const bool sage = (flags & U15C_FWD_SAGE) != 0 && sl.attn == U15C_ATTN_BIDIRECTIONAL;
      if (sl.attn == U15C_ATTN_BIDIRECTIONAL) {
        cudaStream_t as = st;
        if (fork) {
          as = m->side_st[k_side];
          cudaStreamWaitEvent(as, m->side_ev[u15c_model::kSideStreams], 0);
        }
        void* ws = !sage ? nullptr : fork ? m->side_sage[k_side] : m->sage_ws;
        rc = u15::run_attention_tc(as, qh, view, sl.kv->pages, out, c.heads, c.kv_heads, sl.n,
                                   sl.kv_len, U15C_ATTN_BIDIRECTIONAL, 0, nullptr, ws);
        if (!rc && fork) {
          cudaEventRecord(m->side_ev[k_side], as);
          cudaStreamWaitEvent(st, m->side_ev[k_side], 0);
          ++k_side;
        }
      } else {
        // the prefill rules: the queries sit at kv_off among the keys
        rc = u15::run_attention_tc(st, qh, view, sl.kv->pages, out, c.heads, c.kv_heads, sl.n,
                                   sl.kv_len, sl.attn, sl.kv_off, sl.t_index, nullptr);
      }
      if (rc) return rc;
    }
  }
  if (!(parts & kPartPost)) return U15C_OK;
  if ((rc = row_parallel(m->attn + (long)r0 * m->qd(), m->qd(), L.o, L.o8, L.o_s))) return rc;

  // ---- MLP half (src/u15-backbone.cc:246-256) ----
  if ((rc = norm(L.ln_post))) return rc;
  if ((rc = gemm(m->xn, H, L.gu, L.gu8, L.gu_s, 2 * I, u15::kEpiSwiglu, m->h, fuse_q))) return rc;
  if ((rc = row_parallel(m->h, I, L.down, L.down8, L.down_s))) return rc;
  return U15C_OK;
}

// Fused tensor parallelism runs a pass on this rank's residual stream in
// the peer region (the owners of the row-parallel products store their
// results there on every rank): copy the caller's activations in before the
// layers and out after them.
struct TpStream {
  u15c_model* m;
  void* user;
  long bytes;
  cudaStream_t st;
  bf16* x = nullptr;
  int enter(int M)
  {
    x = static_cast<bf16*>(user);
    if (!m->tp_fused) return U15C_OK;
    if (M > m->tp_rows)
      return fail(U15C_EINVAL, "tensor-parallel pass of " + std::to_string(M) +
                                   " tokens exceeds the peer buffers (" +
                                   std::to_string(m->tp_rows) + ")");
    x = static_cast<bf16*>(m->tpp.x[m->tp_rank]);
    const cudaError_t e = cudaMemcpyAsync(x, user, bytes, cudaMemcpyDeviceToDevice, st);
    return e == cudaSuccess ? U15C_OK : cuda_fail(e, "tensor-parallel pass: copy in");
  }
  int leave(int rc)
  {
    if (rc != U15C_OK || !m->tp_fused) return rc;
    const cudaError_t e = cudaMemcpyAsync(user, x, bytes, cudaMemcpyDeviceToDevice, st);
    return e == cudaSuccess ? U15C_OK : cuda_fail(e, "tensor-parallel pass: copy out");
  }
};

int validate_pass(u15c_model* m, int n, u15c_kv* kv, int kv_off, int kv_len, int attn,
                  const int32_t* pos_t, const int32_t* pos_h, const int32_t* pos_w,
                  const int32_t* t_index)
{
  if (m == nullptr || kv == nullptr) return fail(U15C_EINVAL, "no model or KV cache");
  if (kv->m != m) return fail(U15C_EINVAL, "the KV cache belongs to another model");
  if (n <= 0) return fail(U15C_EINVAL, "token count must be positive");
  if (kv_off < 0 || kv_off + n > kv->capacity)
    return fail(U15C_EINVAL, "KV cache too small: need " + std::to_string(kv_off + n) +
                                 ", capacity " + std::to_string(kv->capacity));
  if (kv_len < kv_off + n || kv_len > kv->capacity)
    return fail(U15C_EINVAL, "kv_len is shorter than the tokens just written");
  if (pos_t == nullptr || pos_h == nullptr || pos_w == nullptr)
    return fail(U15C_EINVAL, "position arrays are required");
  if (attn < 0 || attn > 2) return fail(U15C_EINVAL, "unknown attention rule");
  if (attn == U15C_ATTN_BLOCK_CAUSAL && t_index == nullptr)
    return fail(U15C_EINVAL, "Attn::BlockCausal needs the t-index vector");
  return U15C_OK;
}

}  // namespace

extern "C" {

int u15c_model_create(const u15c_config* cfg, unsigned flags, u15c_model** out)
{
  return u15c_model_create_tp(cfg, flags, 0, 1, out);
}

int u15c_model_create_tp(const u15c_config* full, unsigned flags, int tp_rank, int tp_size,
                         u15c_model** out)
{
  if (full == nullptr || out == nullptr) return fail(U15C_EINVAL, "null argument");
  *out = nullptr;
  int rc = check_cfg(*full);
  if (rc) return rc;
  if (tp_size < 1 || tp_size > 8 || (tp_size & (tp_size - 1)) || tp_rank < 0 ||
      tp_rank >= tp_size)
    return fail(U15C_EINVAL, "tensor parallelism: tp_size must be 1, 2, 4 or 8 and "
                             "0 <= tp_rank < tp_size");
  if (full->heads % tp_size || full->kv_heads % tp_size || full->inter % (128 * tp_size))
    return fail(U15C_EINVAL, "tensor parallelism: heads and kv_heads must divide by tp_size "
                             "and inter by 128 * tp_size");
  if (u15::dev() == nullptr) return U15C_ECUDA;
  auto* m = new u15c_model();
  m->full = *full;
  m->cfg = *full;
  m->cfg.heads /= tp_size;
  m->cfg.kv_heads /= tp_size;
  m->cfg.inter /= tp_size;
  m->tp_rank = tp_rank;
  m->tp_size = tp_size;
  m->flags = flags;
  const u15c_config* cfg = &m->cfg;
  cudaGetDevice(&m->device);
  const size_t E = cfg->n_experts, H = cfg->hidden, I = cfg->inter;
  const size_t QKV = (size_t)m->qkv_n(), QD = (size_t)m->qd();
  m->layers.resize(cfg->n_layers);
  for (auto& L : m->layers) {
    rc |= m->alloc(&L.qkv, E * QKV * H * 2, m->allocs);
    rc |= m->alloc(&L.o, E * H * QD * 2, m->allocs);
    rc |= m->alloc(&L.gu, E * 2 * I * H * 2, m->allocs);
    rc |= m->alloc(&L.down, E * H * I * 2, m->allocs);
    rc |= m->alloc(&L.ln_in, E * H * 2, m->allocs);
    rc |= m->alloc(&L.ln_post, E * H * 2, m->allocs);
    rc |= m->alloc(&L.norms, E * 256 * 2, m->allocs);
    m->weight_bytes += E * (QKV * H + H * QD + 2 * I * H + H * I + 2 * H + 256) * 2;
    if (flags & U15C_MODEL_INT8) {
      rc |= m->alloc(&L.qkv8, E * QKV * H, m->allocs);
      rc |= m->alloc(&L.o8, E * H * QD, m->allocs);
      rc |= m->alloc(&L.gu8, E * 2 * I * H, m->allocs);
      rc |= m->alloc(&L.down8, E * H * I, m->allocs);
      rc |= m->alloc(&L.qkv_s, E * QKV * 4, m->allocs);
      rc |= m->alloc(&L.o_s, E * H * 4, m->allocs);
      rc |= m->alloc(&L.gu_s, E * 2 * I * 4, m->allocs);
      rc |= m->alloc(&L.down_s, E * H * 4, m->allocs);
      m->weight_bytes += E * (QKV * H + H * QD + 2 * I * H + H * I) + E * (QKV + 2 * H + 2 * I) * 4;
    }
    if (rc) break;
  }
  if (!rc) rc |= m->alloc(&m->final_norm, E * H * 2, m->allocs);
  if (rc) {
    delete m;
    return U15C_ENOMEM;
  }
  *out = m;
  return U15C_OK;
}

int u15c_model_set_allreduce(u15c_model* m, u15c_allreduce_fn fn, void* ctx, float* buf,
                             long buf_elems)
{
  if (m == nullptr) return fail(U15C_EINVAL, "null model");
  if (fn != nullptr && (buf == nullptr || buf_elems <= 0))
    return fail(U15C_EINVAL, "set_allreduce: the partial-sum buffer is required");
  m->ar_fn = fn;
  m->ar_ctx = ctx;
  m->part = fn ? buf : nullptr;
  m->part_elems = fn ? buf_elems : 0;
  return U15C_OK;
}

int u15c_model_set_sage_dense_layers(u15c_model* m, int n)
{
  if (m == nullptr) return fail(U15C_EINVAL, "null model");
  if (n < 0) return fail(U15C_EINVAL, "sage_dense_layers must be non-negative");
  m->sage_dense_layers = n;
  return U15C_OK;
}

int u15c_model_tp(const u15c_model* m, int* tp_rank, int* tp_size)
{
  if (m == nullptr) return fail(U15C_EINVAL, "null model");
  if (tp_rank) *tp_rank = m->tp_rank;
  if (tp_size) *tp_size = m->tp_size;
  return U15C_OK;
}

namespace {
// the peer region of one rank: [inbox: P planes of bf16 tile slots | x bf16
// rows x H | arrive u64 [tiles][2] | done u64], sections 256-byte aligned.
// A pass of `rows` tokens has at most rows/256 + 8 row units (one more per
// segment boundary) and H/256 column blocks, P-th of them owned here; a
// slot holds one 256 x 256 tile of partials (2 CTAs x 8 chunks x 128 x 32).
struct TpLayout {
  size_t inbox, x, arrive, done, total;
  long plane;   // elements
  TpLayout(long rows, long H, int P)
  {
    auto up = [](size_t v) { return (v + 255) & ~size_t(255); };
    const long units = (rows + 255) / 256 + u15::kMaxSeg;
    const long tiles = units * (H / 256);
    plane = units * (H / 256 / P) * 2 * 8 * 4096;
    inbox = 0;
    x = up(inbox + (size_t)plane * P * 2);
    arrive = up(x + (size_t)rows * H * 2);
    done = up(arrive + (size_t)tiles * 2 * 8);
    total = up(done + 8);
  }
};
struct TpBlob {   // U15C_TP_BLOB_BYTES: what one rank hands its peers
  cudaIpcMemHandle_t handle;   // 64 bytes
  unsigned char uuid[16];
  int rows, rank, size, hidden;
  unsigned char pad[128 - 64 - 16 - 16];
};
static_assert(sizeof(TpBlob) == U15C_TP_BLOB_BYTES, "tp blob size");
}  // namespace

int u15c_model_tp_export(u15c_model* m, int max_tokens, void* blob)
{
  if (m == nullptr || blob == nullptr || max_tokens <= 0)
    return fail(U15C_EINVAL, "tp_export: bad argument");
  if (m->tp_size < 2) return fail(U15C_EINVAL, "tp_export: the model is not tensor-parallel");
  if (m->cfg.hidden % (256 * m->tp_size))
    return fail(U15C_EINVAL, "tp_export: hidden must be a multiple of 256 x tp_size");
  if (m->tp_mem != nullptr) return fail(U15C_EINVAL, "tp_export: already exported");
  DeviceScope ds(m->device);
  const TpLayout lay(max_tokens, m->cfg.hidden, m->tp_size);
  cudaError_t e = cudaMalloc(&m->tp_mem, lay.total);
  if (e != cudaSuccess) {
    m->tp_mem = nullptr;
    return fail(U15C_ENOMEM, "tp_export: peer region allocation failed");
  }
  e = cudaMemset(m->tp_mem, 0, lay.total);
  TpBlob b{};
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&b.handle, m->tp_mem);
  cudaDeviceProp prop{};
  if (e == cudaSuccess) e = cudaGetDeviceProperties(&prop, m->device);
  if (e != cudaSuccess) {
    cudaFree(m->tp_mem);
    m->tp_mem = nullptr;
    return cuda_fail(e, "tp_export");
  }
  std::memcpy(b.uuid, prop.uuid.bytes, 16);
  b.rows = max_tokens;
  b.rank = m->tp_rank;
  b.size = m->tp_size;
  b.hidden = m->cfg.hidden;
  std::memcpy(blob, &b, sizeof b);
  m->tp_rows = max_tokens;
  return U15C_OK;
}

int u15c_model_tp_import(u15c_model* m, const void* blobs)
{
  if (m == nullptr || blobs == nullptr) return fail(U15C_EINVAL, "tp_import: bad argument");
  if (m->tp_mem == nullptr) return fail(U15C_EINVAL, "tp_import: call u15c_model_tp_export first");
  if (m->tp_fused) return fail(U15C_EINVAL, "tp_import: already connected");
  const int P = m->tp_size;
  std::vector<TpBlob> b(P);
  std::memcpy(b.data(), blobs, sizeof(TpBlob) * P);
  for (int q = 0; q < P; ++q) {
    if (b[q].rank != q || b[q].size != P || b[q].rows != m->tp_rows || b[q].hidden != m->cfg.hidden)
      return fail(U15C_EINVAL, "tp_import: the ranks' blobs disagree (order by rank; same "
                               "max_tokens and model on every rank)");
    for (int r = 0; r < q; ++r)
      if (std::memcmp(b[q].uuid, b[r].uuid, 16) == 0)
        return fail(U15C_EINVAL, "tp_import: two ranks share one GPU; the fused ranks wait on "
                                 "each other inside their kernels and need a GPU each");
  }
  DeviceScope ds(m->device);
  for (int q = 0; q < P; ++q) {
    if (q == m->tp_rank) {
      m->tp_peer[q] = m->tp_mem;
      continue;
    }
    void* ptr = nullptr;
    const cudaError_t e =
        cudaIpcOpenMemHandle(&ptr, b[q].handle, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      for (int r = 0; r < q; ++r)
        if (r != m->tp_rank && m->tp_peer[r]) cudaIpcCloseMemHandle(m->tp_peer[r]);
      for (int r = 0; r < P; ++r) m->tp_peer[r] = nullptr;
      return cuda_fail(e, "tp_import: opening a peer's region");
    }
    m->tp_peer[q] = ptr;
  }
  const TpLayout lay(m->tp_rows, m->cfg.hidden, P);
  m->tpp.plane = lay.plane;
  m->tpp.rank = m->tp_rank;
  m->tpp.size = P;
  m->tpp.rows = m->tp_rows;
  for (int q = 0; q < P; ++q) {
    char* base = static_cast<char*>(m->tp_peer[q]);
    m->tpp.inbox[q] = reinterpret_cast<__nv_bfloat16*>(base + lay.inbox);
    m->tpp.x[q] = base + lay.x;
    m->tpp.arrive[q] = reinterpret_cast<unsigned long long*>(base + lay.arrive);
    m->tpp.done[q] = reinterpret_cast<unsigned long long*>(base + lay.done);
  }
  m->tp_done_target = 0;
  m->tp_fused = true;
  return U15C_OK;
}

int u15c_model_tp_disconnect(u15c_model* m)
{
  if (m == nullptr) return fail(U15C_EINVAL, "null model");
  DeviceScope ds(m->device);
  cudaError_t e = cudaDeviceSynchronize();   // no kernel of ours still touches a peer
  for (int q = 0; q < u15::kMaxTp; ++q) {
    if (m->tp_peer[q] != nullptr && m->tp_peer[q] != m->tp_mem) {
      const cudaError_t c = cudaIpcCloseMemHandle(m->tp_peer[q]);
      if (e == cudaSuccess) e = c;
    }
    m->tp_peer[q] = nullptr;
  }
  m->tpp = u15::TpPeers{};
  m->tp_fused = false;
  return e == cudaSuccess ? U15C_OK : cuda_fail(e, "tp_disconnect");
}

void u15c_model_destroy(u15c_model* m)
{
  if (m == nullptr) return;
  DeviceScope ds(m->device);
  delete m;
}

int u15c_model_bind(u15c_model* m, u15c_stream stream, int layer, int expert, int tensor,
                    const void* src, int dtype, int src_on_host)
{
  if (m == nullptr || src == nullptr) return fail(U15C_EINVAL, "null argument");
  DeviceScope ds(m->device);
  const u15c_config& c = m->cfg;
  if (expert < 0 || expert >= c.n_experts) return fail(U15C_EINVAL, "expert out of range");
  if (tensor != U15C_T_FINAL_NORM && (layer < 0 || layer >= c.n_layers))
    return fail(U15C_EINVAL, "layer out of range");
  if (dtype < 0 || dtype > 2) return fail(U15C_EINVAL, "unknown source dtype");
  const long H = c.hidden, I = c.inter, QD = m->qd(), KD = (long)c.kv_heads * c.head_dim;
  // the source is always the full tensor; with tensor parallelism this rank
  // binds its q/k/v heads and gate/up rows (column-parallel) and its columns
  // of o and down (row-parallel)
  const long r = m->tp_rank;
  const long QDf = (long)m->full.heads * c.head_dim, If = m->full.inter;
  LayerW* L = tensor == U15C_T_FINAL_NORM ? nullptr : &m->layers[layer];
  bf16* dst = nullptr;
  long rows = 0, cols = 0, src_rows = 0, src_ld = 0, r0 = 0, c0 = 0;
  int inter = -1;
  auto whole = [&](long n) { rows = 1; cols = n; src_rows = 1; src_ld = n; };
  switch (tensor) {
    case U15C_T_INPUT_LN: dst = L->ln_in + expert * H; whole(H); break;
    case U15C_T_POST_LN: dst = L->ln_post + expert * H; whole(H); break;
    case U15C_T_Q:
      dst = L->qkv + (long)expert * m->qkv_n() * H;
      rows = QD; cols = H; src_rows = QDf; src_ld = H; r0 = r * QD;
      break;
    case U15C_T_K:
    case U15C_T_V:
      dst = L->qkv + ((long)expert * m->qkv_n() + QD + (tensor == U15C_T_V ? KD : 0)) * H;
      rows = KD; cols = H; src_rows = KD * m->tp_size; src_ld = H; r0 = r * KD;
      break;
    case U15C_T_O:
      dst = L->o + (long)expert * H * QD;
      rows = H; cols = QD; src_rows = H; src_ld = QDf; c0 = r * QD;
      break;
    case U15C_T_Q_NORM: dst = L->norms + expert * 256 + 0; whole(64); break;
    case U15C_T_Q_NORM_HW: dst = L->norms + expert * 256 + 64; whole(64); break;
    case U15C_T_K_NORM: dst = L->norms + expert * 256 + 128; whole(64); break;
    case U15C_T_K_NORM_HW: dst = L->norms + expert * 256 + 192; whole(64); break;
    case U15C_T_GATE:
    case U15C_T_UP:
      dst = L->gu + (long)expert * 2 * I * H;
      rows = I; cols = H; src_rows = If; src_ld = H; r0 = r * I;
      inter = tensor == U15C_T_GATE ? 0 : 1;
      break;
    case U15C_T_DOWN:
      dst = L->down + (long)expert * H * I;
      rows = H; cols = I; src_rows = H; src_ld = If; c0 = r * I;
      break;
    case U15C_T_FINAL_NORM: dst = m->final_norm + expert * H; whole(H); break;
    default: return fail(U15C_EINVAL, "unknown tensor id");
  }
  const size_t es = dtype == U15C_DT_F32 ? 4 : 2;
  const size_t bytes = (size_t)src_rows * src_ld * es;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const void* dsrc = src;
  void* staging = nullptr;
  if (src_on_host) {
    cudaError_t e = cudaMalloc(&staging, bytes);
    if (e != cudaSuccess) return fail(U15C_ENOMEM, "bind: staging allocation failed");
    e = cudaMemcpyAsync(staging, src, bytes, cudaMemcpyHostToDevice, st);
    if (e != cudaSuccess) {
      cudaFree(staging);
      return cuda_fail(e, "bind: upload");
    }
    dsrc = staging;
  }
  bind_kernel<<<nblk(rows * cols, 256), 256, 0, st>>>(dsrc, dtype, rows, cols, src_ld, r0, c0,
                                                       dst, inter);
  cudaError_t e = cudaGetLastError();
  if (staging != nullptr) {
    cudaStreamSynchronize(st);
    cudaFree(staging);
  }
  return e == cudaSuccess ? U15C_OK : cuda_fail(e, "bind kernel");
}

int u15c_model_bind_random(u15c_model* m, u15c_stream stream, uint64_t seed, float std,
                           float norm_mean, float norm_std)
{
  if (m == nullptr) return fail(U15C_EINVAL, "null model");
  DeviceScope ds(m->device);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const u15c_config& c = m->cfg;
  const long E = c.n_experts, H = c.hidden, I = c.inter, QD = m->qd(), QKV = m->qkv_n();
  uint64_t sid = 0;
  auto fill = [&](bf16* p, long n, float mean, float sd) {
    randn_kernel<<<nblk(n, 256), 256, 0, st>>>(p, n, seed, ++sid, mean, sd);
  };
  for (auto& L : m->layers) {
    fill(L.qkv, E * QKV * H, 0.0f, std);
    fill(L.o, E * H * QD, 0.0f, std);
    fill(L.gu, E * 2 * I * H, 0.0f, std);
    fill(L.down, E * H * I, 0.0f, std);
    fill(L.ln_in, E * H, norm_mean, norm_std);
    fill(L.ln_post, E * H, norm_mean, norm_std);
    fill(L.norms, E * 256, norm_mean, norm_std);
  }
  fill(m->final_norm, E * H, norm_mean, norm_std);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? U15C_OK : cuda_fail(e, "random init");
}

int u15c_model_finalize(u15c_model* m, u15c_stream stream)
{
  if (m == nullptr) return fail(U15C_EINVAL, "null model");
  if (!(m->flags & U15C_MODEL_INT8)) return U15C_OK;
  DeviceScope ds(m->device);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const u15c_config& c = m->cfg;
  const int E = c.n_experts, H = c.hidden, I = c.inter, QD = m->qd(), QKV = m->qkv_n();
  for (auto& L : m->layers) {
    int rc = 0;
    rc |= u15::launch_quant_rows(L.qkv, L.qkv8, L.qkv_s, E * QKV, H, st);
    rc |= u15::launch_quant_rows(L.o, L.o8, L.o_s, E * H, QD, st);
    rc |= u15::launch_quant_rows(L.gu, L.gu8, L.gu_s, E * 2 * I, H, st);
    rc |= u15::launch_quant_rows(L.down, L.down8, L.down_s, E * H, I, st);
    if (rc) return fail(U15C_ECUDA, "finalize: quantisation launch failed");
  }
  return U15C_OK;
}

size_t u15c_model_weight_bytes(const u15c_model* m) { return m ? m->weight_bytes : 0; }

size_t u15c_model_scratch_bytes(const u15c_model* m, int n)
{
  if (m == nullptr || n <= 0) return 0;
  const size_t H = m->cfg.hidden, I = m->cfg.inter, QD = m->qd(), QKV = m->qkv_n();
  const size_t maxk = std::max({H, I, QD});
  return (size_t)n * (2 * (H + QKV + 2 * QD + I + H) + 8 * 128 + maxk + 4);
}

size_t u15c_model_kv_bytes(const u15c_model* m, int capacity)
{
  if (m == nullptr || capacity <= 0) return 0;
  const size_t pages = (size_t)(capacity + u15::kPageTokens - 1) / u15::kPageTokens;
  return pages * u15::kPageTokens * (size_t)m->cfg.kv_heads * 128 * 2 * 2 *
         (size_t)m->cfg.n_layers;
}

int u15c_kv_create(u15c_model* m, int capacity, u15c_kv** out)
{
  if (m == nullptr || out == nullptr) return fail(U15C_EINVAL, "null argument");
  *out = nullptr;
  if (capacity <= 0) return fail(U15C_EINVAL, "capacity must be positive");
  DeviceScope ds(m->device);
  auto* kv = new u15c_kv();
  kv->m = m;
  kv->capacity = capacity;
  kv->pages = (capacity + u15::kPageTokens - 1) / u15::kPageTokens;
  kv->layer_elems = (long)kv->pages * m->cfg.kv_heads * u15::kPageTokens * 128;
  const size_t bytes = (size_t)kv->layer_elems * m->cfg.n_layers * 2;
  if (cudaMalloc(&kv->k, bytes) != cudaSuccess || cudaMalloc(&kv->v, bytes) != cudaSuccess ||
      cudaMalloc(&kv->table, (size_t)kv->pages * 4) != cudaSuccess) {
    delete kv;
    return fail(U15C_ENOMEM, "out of memory allocating the KV cache (" +
                                 std::to_string(2 * bytes >> 20) + " MB)");
  }
  cudaMemset(kv->k, 0, bytes);
  cudaMemset(kv->v, 0, bytes);
  std::vector<int32_t> ident(kv->pages);
  for (int i = 0; i < kv->pages; ++i) ident[i] = i;
  cudaMemcpy(kv->table, ident.data(), ident.size() * 4, cudaMemcpyHostToDevice);
  *out = kv;
  return U15C_OK;
}

void u15c_kv_destroy(u15c_kv* kv)
{
  if (kv == nullptr) return;
  DeviceScope ds(kv->m->device);
  delete kv;
}

int u15c_kv_capacity(const u15c_kv* kv) { return kv ? kv->capacity : 0; }

int u15c_kv_set_page_table(u15c_kv* kv, const int32_t* pages_host, int n)
{
  if (kv == nullptr || pages_host == nullptr || n != kv->pages)
    return fail(U15C_EINVAL, "page table must have exactly one entry per page");
  std::vector<char> seen(n, 0);
  for (int i = 0; i < n; ++i) {
    if (pages_host[i] < 0 || pages_host[i] >= n || seen[pages_host[i]])
      return fail(U15C_EINVAL, "page table must be a permutation of the cache's pages");
    seen[pages_host[i]] = 1;
  }
  const cudaError_t e = cudaMemcpy(kv->table, pages_host, (size_t)n * 4, cudaMemcpyHostToDevice);
  return e == cudaSuccess ? U15C_OK : cuda_fail(e, "set_page_table");
}

int u15c_kv_read(u15c_kv* kv, u15c_stream stream, int layer, int which_v, void* out, int n)
{
  if (kv == nullptr || out == nullptr || n <= 0 || n > kv->capacity || layer < 0 ||
      layer >= kv->m->cfg.n_layers)
    return fail(U15C_EINVAL, "kv_read: bad argument");
  DeviceScope ds(kv->m->device);
  if (u15::launch_kv_copy(out, kv->view(layer), which_v != 0, false, n, kv->m->cfg.kv_heads,
                          static_cast<cudaStream_t>(stream)))
    return fail(U15C_ECUDA, "kv_read: launch failed");
  return U15C_OK;
}

int u15c_kv_write(u15c_kv* kv, u15c_stream stream, int layer, int which_v, const void* in, int n)
{
  if (kv == nullptr || in == nullptr || n <= 0 || n > kv->capacity || layer < 0 ||
      layer >= kv->m->cfg.n_layers)
    return fail(U15C_EINVAL, "kv_write: bad argument");
  DeviceScope ds(kv->m->device);
  if (u15::launch_kv_copy(const_cast<void*>(in), kv->view(layer), which_v != 0, true, n,
                          kv->m->cfg.kv_heads, static_cast<cudaStream_t>(stream)))
    return fail(U15C_ECUDA, "kv_write: launch failed");
  return U15C_OK;
}

int u15c_kv_pages(u15c_kv* kv, int layer, void** k_pages, void** vt_pages,
                  const int32_t** page_table, int* n_pages)
{
  if (kv == nullptr || layer < 0 || layer >= kv->m->cfg.n_layers)
    return fail(U15C_EINVAL, "kv_pages: bad argument");
  const u15::KvView v = kv->view(layer);
  if (k_pages) *k_pages = v.k;
  if (vt_pages) *vt_pages = v.v;
  if (page_table) *page_table = kv->table;
  if (n_pages) *n_pages = kv->pages;
  return U15C_OK;
}

int u15c_layer_forward(u15c_model* m, u15c_stream stream, int layer, void* x, int n,
                       const int* seg_off, const int* seg_expert, int nseg, u15c_kv* kv,
                       int kv_off, int kv_len, const int32_t* pos_t, const int32_t* pos_h,
                       const int32_t* pos_w, int attn, const int32_t* t_index, unsigned flags)
{
  int rc = validate_pass(m, n, kv, kv_off, kv_len, attn, pos_t, pos_h, pos_w, t_index);
  if (rc) return rc;
  if (layer < 0 || layer >= m->cfg.n_layers) return fail(U15C_EINVAL, "layer out of range");
  if (x == nullptr) return fail(U15C_EINVAL, "null activations");
  DeviceScope ds(m->device);
  u15::SegInfo seg;
  std::string err;
  if (!u15::fill_seg(&seg, seg_off, seg_expert, nseg, n, m->cfg.n_experts, &err))
    return fail(U15C_EINVAL, err);
  if ((rc = m->ensure_scratch(n, kv_len))) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (u15::launch_rope_tables(pos_t, pos_h, pos_w, n, 64, 32, m->cfg.theta_t, m->cfg.theta_hw,
                              m->rcos, m->rsin, st))
    return fail(U15C_ECUDA, "rope tables launch failed");
  SlotRun sl;
  sl.n = n;
  sl.kv = kv;
  sl.kv_off = kv_off;
  sl.kv_len = kv_len;
  sl.attn = attn;
  sl.t_index = t_index;
  TpStream tx{m, x, (long)n * m->cfg.hidden * 2, st};
  if ((rc = tx.enter(n))) return rc;
  return tx.leave(
      layer_impl(m, st, layer, tx.x, n, seg, seg_off, seg_expert, nseg, {sl}, flags));
}

int u15c_forward(u15c_model* m, u15c_stream stream, void* x, int n, const int* seg_off,
                 const int* seg_expert, int nseg, u15c_kv* kv, int kv_off, int kv_len,
                 const int32_t* pos_t, const int32_t* pos_h, const int32_t* pos_w, int attn,
                 const int32_t* t_index, unsigned flags, int (*stop)(void*), void* stop_ctx)
{
  int rc = validate_pass(m, n, kv, kv_off, kv_len, attn, pos_t, pos_h, pos_w, t_index);
  if (rc) return rc;
  if (x == nullptr) return fail(U15C_EINVAL, "null activations");
  DeviceScope ds(m->device);
  u15::SegInfo seg;
  std::string err;
  if (!u15::fill_seg(&seg, seg_off, seg_expert, nseg, n, m->cfg.n_experts, &err))
    return fail(U15C_EINVAL, err);
  if ((rc = m->ensure_scratch(n, kv_len))) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // The rope tables depend on the positions only: built once per pass
  // (src/u15-backbone.cc:340-367), not per layer.
  if (u15::launch_rope_tables(pos_t, pos_h, pos_w, n, 64, 32, m->cfg.theta_t, m->cfg.theta_hw,
                              m->rcos, m->rsin, st))
    return fail(U15C_ECUDA, "rope tables launch failed");
  TpStream tx{m, x, (long)n * m->cfg.hidden * 2, st};
  if ((rc = tx.enter(n))) return rc;
  for (int li = 0; li < m->cfg.n_layers; ++li) {
    // with tensor parallelism the stop callback must answer alike on every
    // rank (the ranks meet in every layer)
    if (stop != nullptr && stop(stop_ctx) != 0) return fail(U15C_ESTOPPED, "stopped");
    SlotRun sl;
    sl.n = n;
    sl.kv = kv;
    sl.kv_off = kv_off;
    sl.kv_len = kv_len;
    sl.attn = attn;
    sl.t_index = t_index;
    if ((rc = layer_impl(m, st, li, tx.x, n, seg, seg_off, seg_expert, nseg, {sl}, flags)))
      return rc;
  }
  return tx.leave(U15C_OK);
}

int u15c_forward_many(u15c_model* m, u15c_stream stream, void* x, int n, const u15c_slot* slots,
                      int nslots, int expert, int attn, unsigned flags, int (*stop)(void*),
                      void* stop_ctx)
{
  if (m == nullptr || x == nullptr || slots == nullptr || nslots <= 0)
    return fail(U15C_EINVAL, "forward_many: no branches to run");
  if (expert < 0 || expert >= m->cfg.n_experts) return fail(U15C_EINVAL, "expert out of range");
  DeviceScope ds(m->device);
  int rc;
  int max_kv = 0;
  for (int i = 0; i < nslots; ++i) {
    const u15c_slot& s = slots[i];
    if ((rc = validate_pass(m, n, s.kv, s.kv_off, s.kv_len, attn, s.pos_t, s.pos_h, s.pos_w,
                            s.t_index)))
      return rc;
    max_kv = std::max(max_kv, s.kv_len);
  }
  const int M = n * nslots;
  if ((rc = m->ensure_scratch(M, max_kv))) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  std::vector<SlotRun> runs(nslots);
  for (int i = 0; i < nslots; ++i) {
    const u15c_slot& s = slots[i];
    if (u15::launch_rope_tables(s.pos_t, s.pos_h, s.pos_w, n, 64, 32, m->cfg.theta_t,
                                m->cfg.theta_hw, m->rcos + (long)i * n * 128,
                                m->rsin + (long)i * n * 128, st))
      return fail(U15C_ECUDA, "rope tables launch failed");
    runs[i].row0 = i * n;
    runs[i].n = n;
    runs[i].kv = s.kv;
    runs[i].kv_off = s.kv_off;
    runs[i].kv_len = s.kv_len;
    runs[i].attn = attn;
    runs[i].t_index = s.t_index;
  }
  u15::SegInfo seg;
  seg.nseg = 1;
  seg.off[0] = 0;
  seg.off[1] = M;
  seg.expert[0] = expert;
  const int off[2] = {0, M}, ex[1] = {expert};
  TpStream tx{m, x, (long)M * m->cfg.hidden * 2, st};
  if ((rc = tx.enter(M))) return rc;
  for (int li = 0; li < m->cfg.n_layers; ++li) {
    if (stop != nullptr && stop(stop_ctx) != 0) return fail(U15C_ESTOPPED, "stopped");
    if ((rc = layer_impl(m, st, li, tx.x, M, seg, off, ex, 1, runs, flags))) return rc;
  }
  return tx.leave(U15C_OK);
}

int u15c_final_norm(u15c_model* m, u15c_stream stream, void* x, int n, int expert)
{
  if (m == nullptr || x == nullptr || expert < 0 || expert >= m->cfg.n_experts)
    return fail(U15C_EINVAL, "final_norm: bad argument");
  DeviceScope ds(m->device);
  u15::SegInfo seg;
  seg.nseg = 1;
  seg.off[0] = 0;
  seg.off[1] = n;
  seg.expert[0] = 0;
  const bf16* w = m->final_norm + (long)expert * m->cfg.hidden;
  if (u15::launch_rms_norm(x, w, x, n, m->cfg.hidden, (float)m->cfg.eps, seg,
                           static_cast<cudaStream_t>(stream)))
    return fail(U15C_ECUDA, "final_norm launch failed");
  return U15C_OK;
}

int u15c_layer_forward_host(u15c_model* m, u15c_stream stream, int layer, const void* x_host,
                            void* out_host, int n, const int* seg_off, const int* seg_expert,
                            int nseg, u15c_kv* kv, int kv_off, int kv_len, const int32_t* pos_t,
                            const int32_t* pos_h, const int32_t* pos_w, int attn,
                            const int32_t* t_index, unsigned flags)
{
  if (m == nullptr || x_host == nullptr || out_host == nullptr)
    return fail(U15C_EINVAL, "layer_forward_host: null argument");
  DeviceScope ds(m->device);
  int rc = m->ensure_scratch(n, kv_len);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int H = m->cfg.hidden;
  const size_t bytes = (size_t)n * H * 2;
  // Pipelined: the upload in 4 row chunks on a copy stream, each chunk's
  // norm + QKV as soon as it lands; attention over all rows; o_proj through
  // down_proj per chunk, each chunk's download while the next one runs. The
  // host buffers should be pinned for the copies to overlap. Small passes
  // and tensor-parallel models take the plain upload -> layer -> download.
  constexpr int kChunks = 4;
  if (n >= 1024 && m->tp_size == 1) {
    if ((rc = validate_pass(m, n, kv, kv_off, kv_len, attn, pos_t, pos_h, pos_w, t_index)))
      return rc;
    if (layer < 0 || layer >= m->cfg.n_layers) return fail(U15C_EINVAL, "layer out of range");
    u15::SegInfo seg;
    std::string err;
    if (!u15::fill_seg(&seg, seg_off, seg_expert, nseg, n, m->cfg.n_experts, &err))
      return fail(U15C_EINVAL, err);
    if (m->copy_st == nullptr) {
      if (cudaStreamCreateWithFlags(&m->copy_st, cudaStreamNonBlocking) != cudaSuccess)
        return fail(U15C_ECUDA, "layer_forward_host: copy stream");
      for (cudaEvent_t& e : m->copy_ev)
        if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess)
          return fail(U15C_ECUDA, "layer_forward_host: copy events");
    }
    cudaStream_t cs = m->copy_st;
    const int rows = ((n + kChunks - 1) / kChunks + 255) / 256 * 256;   // whole 256-row blocks
    const char* hin = static_cast<const char*>(x_host);
    char* hout = static_cast<char*>(out_host);
    cudaEvent_t* in_ev = m->copy_ev;
    cudaEvent_t* out_ev = m->copy_ev + kChunks;
    // the copy stream starts after what the caller already queued on `st`
    cudaEventRecord(m->copy_ev[2 * kChunks], st);
    cudaStreamWaitEvent(cs, m->copy_ev[2 * kChunks], 0);
    for (int k = 0, r0 = 0; r0 < n; ++k, r0 += rows) {
      const size_t off = (size_t)r0 * H * 2, len = (size_t)std::min(rows, n - r0) * H * 2;
      cudaError_t e = cudaMemcpyAsync(reinterpret_cast<char*>(m->io) + off, hin + off, len,
                                      cudaMemcpyHostToDevice, cs);
      if (e != cudaSuccess) return cuda_fail(e, "layer_forward_host: upload");
      cudaEventRecord(in_ev[k], cs);
    }
    if (u15::launch_rope_tables(pos_t, pos_h, pos_w, n, 64, 32, m->cfg.theta_t, m->cfg.theta_hw,
                                m->rcos, m->rsin, st))
      return fail(U15C_ECUDA, "rope tables launch failed");
    SlotRun sl;
    sl.n = n;
    sl.kv = kv;
    sl.kv_off = kv_off;
    sl.kv_len = kv_len;
    sl.attn = attn;
    sl.t_index = t_index;
    const std::vector<SlotRun> slots{sl};
    for (int k = 0, r0 = 0; r0 < n; ++k, r0 += rows) {
      cudaStreamWaitEvent(st, in_ev[k], 0);
      if ((rc = layer_impl(m, st, layer, m->io, n, seg, seg_off, seg_expert, nseg, slots, flags,
                           kPartPre, r0, std::min(rows, n - r0))))
        return rc;
    }
    if ((rc = layer_impl(m, st, layer, m->io, n, seg, seg_off, seg_expert, nseg, slots, flags,
                         kPartAttn)))
      return rc;
    for (int k = 0, r0 = 0; r0 < n; ++k, r0 += rows) {
      const int rk = std::min(rows, n - r0);
      if ((rc = layer_impl(m, st, layer, m->io, n, seg, seg_off, seg_expert, nseg, slots, flags,
                           kPartPost, r0, rk)))
        return rc;
      cudaEventRecord(out_ev[k], st);
      cudaStreamWaitEvent(cs, out_ev[k], 0);
      const size_t off = (size_t)r0 * H * 2;
      cudaError_t e = cudaMemcpyAsync(hout + off, reinterpret_cast<char*>(m->io) + off,
                                      (size_t)rk * H * 2, cudaMemcpyDeviceToHost, cs);
      if (e != cudaSuccess) return cuda_fail(e, "layer_forward_host: download");
    }
    cudaEventRecord(m->copy_ev[2 * kChunks], cs);
    cudaStreamWaitEvent(st, m->copy_ev[2 * kChunks], 0);
    return u15c_sync(stream);
  }
  cudaError_t e = cudaMemcpyAsync(m->io, x_host, bytes, cudaMemcpyHostToDevice, st);
  if (e != cudaSuccess) return cuda_fail(e, "layer_forward_host: upload");
  rc = u15c_layer_forward(m, stream, layer, m->io, n, seg_off, seg_expert, nseg, kv, kv_off,
                          kv_len, pos_t, pos_h, pos_w, attn, t_index, flags);
  if (rc) return rc;
  e = cudaMemcpyAsync(out_host, m->io, bytes, cudaMemcpyDeviceToHost, st);
  if (e != cudaSuccess) return cuda_fail(e, "layer_forward_host: download");
  return u15c_sync(stream);
}

int u15c_layer_forward_host_async(u15c_model* m, u15c_stream stream, int layer,
                                  const void* x_host, void* out_host, int n, const int* seg_off,
                                  const int* seg_expert, int nseg, u15c_kv* kv, int kv_off,
                                  int kv_len, const int32_t* pos_t, const int32_t* pos_h,
                                  const int32_t* pos_w, int attn, const int32_t* t_index,
                                  unsigned flags)
{
  if (m == nullptr || x_host == nullptr || out_host == nullptr)
    return fail(U15C_EINVAL, "layer_forward_host_async: null argument");
  DeviceScope ds(m->device);
  if (m->tp_size != 1)
    return fail(U15C_EINVAL, "layer_forward_host_async: tensor-parallel models take the "
                             "synchronous u15c_layer_forward_host");
  int rc = validate_pass(m, n, kv, kv_off, kv_len, attn, pos_t, pos_h, pos_w, t_index);
  if (rc) return rc;
  if (layer < 0 || layer >= m->cfg.n_layers) return fail(U15C_EINVAL, "layer out of range");
  u15::SegInfo seg;
  std::string err;
  if (!u15::fill_seg(&seg, seg_off, seg_expert, nseg, n, m->cfg.n_experts, &err))
    return fail(U15C_EINVAL, err);
  if ((rc = m->ensure_scratch(n, kv_len)) || (rc = m->ensure_host_staging(n))) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t bytes = (size_t)n * m->cfg.hidden * 2;
  const int b = m->hio_next;
  m->hio_next ^= 1;
  bf16* io = m->hio[b];
  // The staging buffer is free once the call two back (the last one that
  // used it) has downloaded its result. Back to back, call k + 1's upload
  // runs during call k's layer and call k's download during call k + 1's, so
  // the pass is not cut into row chunks (whole-pass GEMMs), unlike the
  // synchronous form, which can only overlap copies within its own call.
  if (m->hio_used[b]) cudaStreamWaitEvent(m->up_st, m->hio_free[b], 0);
  m->hio_used[b] = true;
  cudaError_t e = cudaMemcpyAsync(io, x_host, bytes, cudaMemcpyHostToDevice, m->up_st);
  if (e != cudaSuccess) return cuda_fail(e, "layer_forward_host_async: upload");
  cudaEventRecord(m->hio_in[b][0], m->up_st);
  cudaStreamWaitEvent(st, m->hio_in[b][0], 0);
  if (u15::launch_rope_tables(pos_t, pos_h, pos_w, n, 64, 32, m->cfg.theta_t, m->cfg.theta_hw,
                              m->rcos, m->rsin, st))
    return fail(U15C_ECUDA, "rope tables launch failed");
  SlotRun sl;
  sl.n = n;
  sl.kv = kv;
  sl.kv_off = kv_off;
  sl.kv_len = kv_len;
  sl.attn = attn;
  sl.t_index = t_index;
  const std::vector<SlotRun> slots{sl};
  if ((rc = layer_impl(m, st, layer, io, n, seg, seg_off, seg_expert, nseg, slots, flags)))
    return rc;
  cudaEventRecord(m->hio_out[b][0], st);
  cudaStreamWaitEvent(m->down_st, m->hio_out[b][0], 0);
  e = cudaMemcpyAsync(out_host, io, bytes, cudaMemcpyDeviceToHost, m->down_st);
  if (e != cudaSuccess) return cuda_fail(e, "layer_forward_host_async: download");
  cudaEventRecord(m->hio_free[b], m->down_st);
  e = cudaGetLastError();
  return e == cudaSuccess ? U15C_OK : cuda_fail(e, "layer_forward_host_async");
}

int u15c_layer_host_drain(u15c_model* m, u15c_stream stream)
{
  if (m == nullptr) return fail(U15C_EINVAL, "layer_host_drain: null model");
  DeviceScope ds(m->device);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  for (int b = 0; b < 2; ++b)
    if (m->hio_used[b]) cudaStreamWaitEvent(st, m->hio_free[b], 0);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? U15C_OK : cuda_fail(e, "layer_host_drain");
}

}  // extern "C"
