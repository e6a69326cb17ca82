// Internal launcher interface between the C ABI (u15_capi.cu) and the
// kernel files. Not installed; the public surface is include/u15c.h.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <string>
#include <utility>

#include <cuda_bf16.h>

namespace u15 {

// Launch the layer's tensor-core kernels with programmatic dependent launch
// (U15_PDL=0 turns it off; read per launch, for A/B checks).
bool pdl_enabled();

// The layer's row kernels are launched with programmatic stream
// serialisation (unless U15_PDL=0): their CTAs may be placed while the
// previous kernel drains, and each waits (griddepcontrol.wait) before it
// touches global memory.
template <class... KArgs, class... Args>
cudaError_t launch_pdl(void (*k)(KArgs...), dim3 grid, dim3 block, cudaStream_t st,
                       Args&&... args)
{
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, k, std::forward<Args>(args)...);
}

// Kernel attributes are per device: a process that drives several GPUs
// (or that switches its current device between calls) must set a kernel's
// dynamic shared-memory limit on each of them. `done` holds one bit per
// device; the attribute is set the first time a launch meets a device.
template <class Kernel>
inline bool smem_attr_once(Kernel kern, int bytes, std::atomic<uint64_t>& done)
{
  int d = 0;
  if (cudaGetDevice(&d) != cudaSuccess) return false;
  const uint64_t bit = 1ull << (d & 63);
  if (done.load(std::memory_order_acquire) & bit) return true;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) !=
      cudaSuccess)
    return false;
  done.fetch_or(bit, std::memory_order_release);
  return true;
}

enum Epilogue {
  kEpiStore = 0,
  kEpiResid = 1,
  kEpiSwiglu = 2,
  kEpiStoreF32 = 3,
  kEpiTpReduce = 4,   // row-parallel product summed over tensor-parallel ranks (TpPeers)
};

// Tensor-parallel peers for the fused row-parallel GEMM (kEpiTpReduce).
// Column block nb (256 columns) of the [M][N] product is owned by rank
// nb % size; tile (unit u, nb) is the owner's slot u * (N / 256 / size) +
// nb / size. Every rank stores its partial of a tile, rounded to bf16, into
// the owner's inbox plane [rank], chunk-major (32 columns x 128 rows of one
// CTA contiguous, so a warp writes 256 contiguous bytes per store), and
// counts it on the owner's arrive[tile][cta]; the owner sums the planes in
// f32, adds the residual x, rounds as the residual epilogue does, stores the
// bf16 result into every rank's x and counts it on every rank's done.
constexpr int kMaxTp = 8;
struct TpPeers {
  int rank = 0, size = 1;
  long rows = 0;                              // rows of x (the largest pass)
  long plane = 0;                             // elements of one inbox plane
  __nv_bfloat16* inbox[kMaxTp] = {};          // owner q: [size planes][slot][cta 2][chunk 8][128][32] bf16
  void* x[kMaxTp] = {};                       // rank q: residual stream [rows][N] bf16
  unsigned long long* arrive[kMaxTp] = {};    // owner q: [tiles][2] (reset by the owner)
  unsigned long long* done[kMaxTp] = {};      // rank q: cumulative count of finished tile halves
};

// Token segments routed to experts: rows [off[i], off[i+1]) use expert[i].
constexpr int kMaxSeg = 8;
struct SegInfo {
  int nseg = 1;
  int off[kMaxSeg + 1] = {0};
  int expert[kMaxSeg] = {0};
};

struct GemmArgs {
  bool int8 = false;
  const void* x = nullptr;       // [M][K] bf16 or int8
  const void* w = nullptr;       // [n_experts][N][K] bf16 or int8
  int n_experts = 1;
  int M = 0, N = 0, K = 0;
  const int* seg_off = nullptr;  // host, nseg + 1 entries (null: one segment, expert 0)
  const int* seg_expert = nullptr;
  int nseg = 0;
  int epilogue = kEpiStore;
  void* y = nullptr;             // bf16 [M][ldy]
  long ldy = 0;                  // 0: N (SwiGLU: N / 2)
  const void* resid = nullptr;   // bf16 [M][ldr]
  long ldr = 0;
  const void* bias = nullptr;    // bf16 [n_experts][N]
  const float* s_tok = nullptr;  // int8
  const float* s_ch = nullptr;   // int8 [n_experts][N]
  int32_t* acc_dump = nullptr;   // int8 debug [M][N]
  unsigned* dev_err = nullptr;
  int num_sms = 148;
  const TpPeers* tp = nullptr;   // kEpiTpReduce
  int* out_tiles = nullptr;      // kEpiTpReduce: tiles of the launch (done counts 2 per tile)
};

int gemm_tc(const GemmArgs& a, cudaStream_t st, std::string* err);
// One thread waits (bounded) until *done >= target with acquire semantics at
// system scope, so the stream's later kernels see the peers' stores.
int launch_tp_wait(const unsigned long long* done, unsigned long long target, unsigned* err,
                   cudaStream_t st);

// Paged or contiguous K/V addressing shared by the attention and KV kernels.
// Token j of kv head h lives at
//   base + page(j >> 6) * page_stride + h * head_stride + (j & 63) * 128
// with page(i) = page_table ? page_table[i] : i. The reference's contiguous
// cache [hkv][cap][128] is page_stride = 64*128, head_stride = cap*128; the
// paged pool [page][hkv][64][128] is page_stride = hkv*64*128,
// head_stride = 64*128.
struct KvView {
  void* k = nullptr;
  void* v = nullptr;
  const int32_t* page_table = nullptr;   // device; null = identity
  long page_stride = 0;                  // elements
  long head_stride = 0;                  // elements
  // V pages stored transposed, [128 dims][64 tokens] per (page, head): token j,
  // dim d of head h at v + page * page_stride + h * head_stride + d * 64 + (j & 63).
  // The model's cache uses this form (the P.V operand of the tcgen05
  // attention); the op-level reference layouts do not.
  bool v_t = false;
};
constexpr int kPageTokens = 64;
constexpr int kHeadDim = 128;

struct AttnArgs {
  const void* q = nullptr;      // [hq][tq][128] bf16 (head-major, tq rows per head)
  KvView kv;
  void* out = nullptr;          // [tq][hq*128] bf16 (token-major)
  int hq = 0, hkv = 0, tq = 0, tk = 0;
  int mode = 0;                 // 0 bidirectional, 1 causal, 2 block-causal
  int q_offset = 0;
  const int32_t* t_index = nullptr;   // device [tk], block-causal
  // Sage int8 QK (bidirectional only): prepared by sage_prepare()
  const int8_t* q8 = nullptr;   // [hq][tq][128]
  const int8_t* k8 = nullptr;   // [hkv][tk_pad][128]
  const float* sq = nullptr;    // [hq][ceil(tq/64)]
  const float* sk = nullptr;    // [hkv][2 * ceil(tk/64)]: one per 32-key block
  unsigned* dev_err = nullptr;
};

int attention(const AttnArgs& a, cudaStream_t st, std::string* err);

// The tcgen05 attention (u15_attn_tc.cu) over the paged cache: K pages
// [n_pages][hkv][64][128], V pages transposed [n_pages][hkv][128][64]; the
// bidirectional rule (bf16 or Sage int8 QK) and the causal / block-causal
// prefill rules (bf16).
struct TcAttnArgs {
  const void* q = nullptr;          // [hq][tq][128] bf16
  const void* k_pages = nullptr;
  const void* vt_pages = nullptr;
  const int32_t* page_table = nullptr;   // device, null = identity
  int n_pages = 0;                  // pages in the pool (tensor-map extent)
  void* out = nullptr;              // [tq][hq*128] bf16
  int hq = 0, hkv = 0, tq = 0, tk = 0;
  int mode = 0;                     // 0 bidirectional, 1 causal, 2 block-causal
  int q_offset = 0;                 // the queries' first position among the keys
  const int32_t* t_index = nullptr; // block-causal: device [tk], 16-byte aligned
  // Sage int8 QK (from sage_prepare): q8 [hq][tq][128], k8 [hkv][npg*64][128]
  const int8_t* q8 = nullptr;
  const int8_t* k8 = nullptr;
  const float* sq = nullptr;
  const float* sk = nullptr;
  unsigned* dev_err = nullptr;
};
int attention_tc(const TcAttnArgs& a, cudaStream_t st, std::string* err);
// Whether the tcgen05 kernel serves this rule (block-causal: a 16-byte
// aligned t-index vector and at most 32768 keys); the callers route the
// rest to the mma.sync kernel.
bool attention_tc_serves(int mode, int tk, const int32_t* t_index);

// A cached 2-D TMA map over a row-major [rows][cols] tensor (elsize 2 = bf16,
// 1 = int8): box of 128 bytes x box_rows, 128-byte swizzle, zero fill.
int make_tma_2d(CUtensorMap* out, const void* ptr, uint64_t rows, uint64_t cols,
                uint32_t box_rows, int elsize, std::string* err);

// Sage prologue: K smoothing (mean over tk keys per kv head and channel),
// int8 quantisation of Q per 64-row block and of the smoothed K per 32-key
// block (the reference's bq = 64, bk = 32).
int sage_prepare(const void* q, const KvView& kv, int hq, int hkv, int tq, int tk, int8_t* q8,
                 int8_t* k8, float* sq, float* sk, float* kmean, cudaStream_t st,
                 std::string* err);

// bandwidth kernels (u15_elem.cu); all bf16 unless stated
int launch_rms_norm(const void* x, const void* w, void* y, int rows, int dim, float eps,
                    const SegInfo& seg, cudaStream_t st);
// RMSNorm + per-token int8 quantisation of the (bf16-rounded) output; dim <= 4096.
int launch_rms_norm_quant(const void* x, const void* w, int8_t* q, float* s, int rows, int dim,
                          float eps, const SegInfo& seg, cudaStream_t st);
int launch_split_qk_norm(void* x, const void* w_t, const void* w_hw, int heads, int tokens,
                         float eps, cudaStream_t st);
int launch_split_rope(void* x, const float* c, const float* s, int heads, int tokens,
                      cudaStream_t st);
int launch_rope_tables(const int32_t* pt, const int32_t* ph, const int32_t* pw, int tokens,
                       int d_t, int d_h, double theta_t, double theta_hw, float* c, float* s,
                       cudaStream_t st);
int launch_qkv_post(const void* qkv, const void* norms, const float* c, const float* s,
                    void* q_out, const KvView& kv, int T, int nh, int nkv, int kv_off, float eps,
                    const SegInfo& seg, cudaStream_t st);
int launch_transpose(const void* in, void* out, int T, int H, int D, bool to_head_major,
                     cudaStream_t st);
int launch_kv_append(const void* in, void* cache, const int32_t* page_table, long page_stride,
                     long head_stride, int T, int H, int off, cudaStream_t st);
int launch_swiglu(const void* g, const void* u, void* y, long n, cudaStream_t st);
int launch_add(void* d, const void* s, long n, cudaStream_t st);
int launch_add_row(void* d, const void* r, long rows, int dim, cudaStream_t st);
int launch_silu(void* x, long n, cudaStream_t st);
int launch_quant_rows(const void* x, int8_t* q, float* s, int rows, int cols, cudaStream_t st);
// Copy tokens [0, n) of one K or V cache view to/from a contiguous
// [hkv][n][128] buffer (prefix seeding and diagnostics).
int launch_kv_copy(void* contig, const KvView& kv, bool is_v, bool to_cache, int n, int hkv,
                   cudaStream_t st);

}  // namespace u15
