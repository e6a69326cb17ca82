// Bandwidth-bound kernels of the MoT layer: each reads and writes its
// tensors once with 16-byte vector accesses, coalesced across a warp, and
// reduces with warp shuffles. Grids are sized from the row count; every
// kernel is HBM-bound and is reported in GB/s against the copy peak.
//
// Rounding points follow the reference's bf16 buffers: every op reads
// bf16, computes in f32 and writes bf16 once, as the Metal kernels do
// (src/u15-kernels.metal in the reference).
#include "u15_common.cuh"
#include "u15_kernels.h"

#include <utility>

#include <algorithm>

namespace u15 {

namespace {

__device__ __forceinline__ float warp_sum(float v)
{
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v)
{
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ int expert_of(int row, const SegInfo& s)
{
  int e = s.expert[0];
#pragma unroll 1
  for (int i = 1; i < s.nseg; ++i)
    if (row >= s.off[i]) e = s.expert[i];
  return e;
}

__device__ __forceinline__ void load8(const __nv_bfloat16* p, float (&v)[8])
{
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  float2 a = unpack_bf2(u.x), b = unpack_bf2(u.y), c = unpack_bf2(u.z), d = unpack_bf2(u.w);
  v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y; v[4] = c.x; v[5] = c.y; v[6] = d.x; v[7] = d.y;
}
__device__ __forceinline__ void store8(__nv_bfloat16* p, const float (&v)[8])
{
  uint4 u;
  u.x = pack_bf2(v[0], v[1]);
  u.y = pack_bf2(v[2], v[3]);
  u.z = pack_bf2(v[4], v[5]);
  u.w = pack_bf2(v[6], v[7]);
  *reinterpret_cast<uint4*>(p) = u;
}

// ---------------------------------------------------------------------
// RMSNorm, one CTA per row, gains chosen per expert segment.
// y = bf16(x * rsqrt(mean(x^2) + eps) * w_e)
// ---------------------------------------------------------------------
// CTA of the per-row kernels. 128 threads (32 values each, reductions over 4
// warps) against 256: the fused RMSNorm + quantisation 21.2 -> 19.1 us and the
// 4096-wide quantizer 14.8 -> 12.9 us at 4096 rows, RMSNorm alone 13.0 -> 12.8.
constexpr int kRmsThreads = 128;
constexpr int kRmsPer = 4096 / kRmsThreads;    // values a thread keeps (rows up to 4096 wide)
static_assert(kRmsPer % 8 == 0, "a thread keeps whole 16-byte runs");

__device__ __forceinline__ void unpack8(const uint4& u, float (&v)[8])
{
  float2 a = unpack_bf2(u.x), b = unpack_bf2(u.y), c = unpack_bf2(u.z), d = unpack_bf2(u.w);
  v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y; v[4] = c.x; v[5] = c.y; v[6] = d.x; v[7] = d.y;
}

// Block-wide sum / max over NT threads with one barrier. red[] holds NT / 32
// floats and is still being read when the call returns, so a second
// reduction in the same CTA takes its own red[].
template <int NT>
__device__ __forceinline__ float block_sum(float v, float* red)
{
  v = warp_sum(v);
  if (lane_id() == 0) red[warp_id()] = v;
  __syncthreads();
  float t = 0.0f;
#pragma unroll
  for (int i = 0; i < NT / 32; ++i) t += red[i];
  return t;
}
template <int NT>
__device__ __forceinline__ float block_max(float v, float* red)
{
  v = warp_max(v);
  if (lane_id() == 0) red[warp_id()] = v;
  __syncthreads();
  float t = 0.0f;
#pragma unroll
  for (int i = 0; i < NT / 32; ++i) t = fmaxf(t, red[i]);
  return t;
}

// One CTA per row; thread i holds columns 8 (i + NT k) .. + 8, k < kRmsPer / 8,
// the row and its gains packed as bf16 in registers between the reduction and
// the output. The sum of squares is one fma chain per thread in column order,
// the same in rms_norm_quant_kernel, so the two kernels norm a row to the same
// bits. One warp per row (8 rows a CTA, shuffle-only reductions) measured 30 %
// slower.
__global__ void __launch_bounds__(kRmsThreads)
    rms_norm_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w,
                    __nv_bfloat16* __restrict__ y, int rows, int dim, float eps, SegInfo seg)
{
  griddep_launch();   // the next (tensor-core) kernel may start its set-up
  griddep_wait();     // launched early (PDL): the previous kernel's writes first
  const int row = blockIdx.x;
  if (row >= rows) return;
  const __nv_bfloat16* xr = x + (long)row * dim;
  const __nv_bfloat16* wr = w + (long)expert_of(row, seg) * dim;
  __nv_bfloat16* yr = y + (long)row * dim;
  __shared__ float red[kRmsThreads / 32];
  if (dim <= kRmsThreads * kRmsPer) {
    constexpr int kW = kRmsPer / 8;
    uint4 xv[kW];
    float acc = 0.0f;
#pragma unroll
    for (int k = 0; k < kW; ++k) {
      const int c = (k * kRmsThreads + threadIdx.x) * 8;
      xv[k] = make_uint4(0, 0, 0, 0);
      if (c < dim) xv[k] = *reinterpret_cast<const uint4*>(xr + c);
      float t[8];
      unpack8(xv[k], t);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc = __fmaf_rn(t[i], t[i], acc);
    }
    const float inv = rsqrtf(block_sum<kRmsThreads>(acc, red) / (float)dim + eps);
    // the gains are read in this pass (L1-resident: every row of an expert
    // reads the same ones), which keeps 16 registers a thread free
#pragma unroll
    for (int k = 0; k < kW; ++k) {
      const int c = (k * kRmsThreads + threadIdx.x) * 8;
      if (c >= dim) continue;
      float t[8], u[8];
      unpack8(xv[k], t);
      unpack8(__ldg(reinterpret_cast<const uint4*>(wr + c)), u);
#pragma unroll
      for (int i = 0; i < 8; ++i) t[i] = t[i] * inv * u[i];
      store8(yr + c, t);
    }
    return;
  }
  float acc = 0.0f;
  for (int c = threadIdx.x * 8; c < dim; c += kRmsThreads * 8) {
    float v[8];
    load8(xr + c, v);
#pragma unroll
    for (int i = 0; i < 8; ++i) acc = __fmaf_rn(v[i], v[i], acc);
  }
  const float inv = rsqrtf(block_sum<kRmsThreads>(acc, red) / (float)dim + eps);
  for (int c = threadIdx.x * 8; c < dim; c += kRmsThreads * 8) {
    float v[8], g[8];
    load8(xr + c, v);
    load8(wr + c, g);
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = v[i] * inv * g[i];
    store8(yr + c, v);
  }
}

// RMSNorm fused with the symmetric per-token int8 quantisation of its output
// (the W8A8 path's activation half): the normed row is rounded to bf16 in
// registers (the value the unfused path would store), its absmax reduced
// over the CTA, and the codes written directly: q = rn_even(y / (amax/127)).
// Codes are bit-identical to rms_norm followed by quant_rows. dim <= 4096.
__global__ void __launch_bounds__(kRmsThreads)
    rms_norm_quant_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w,
                          int8_t* __restrict__ q, float* __restrict__ scale, int rows, int dim,
                          float eps, SegInfo seg)
{
  griddep_launch();   // the next (tensor-core) kernel may start its set-up
  griddep_wait();     // launched early (PDL): the previous kernel's writes first
  const int row = blockIdx.x;
  if (row >= rows) return;
  const __nv_bfloat16* xr = x + (long)row * dim;
  const __nv_bfloat16* wr = w + (long)expert_of(row, seg) * dim;
  __shared__ float red_sum[kRmsThreads / 32], red_max[kRmsThreads / 32];
  constexpr int kW = kRmsPer / 8;
  uint4 xv[kW];
  float acc = 0.0f;
#pragma unroll
  for (int k = 0; k < kW; ++k) {
    const int c = (k * kRmsThreads + threadIdx.x) * 8;
    xv[k] = make_uint4(0, 0, 0, 0);
    if (c < dim) xv[k] = *reinterpret_cast<const uint4*>(xr + c);
    float t[8];
    unpack8(xv[k], t);
#pragma unroll
    for (int i = 0; i < 8; ++i) acc = __fmaf_rn(t[i], t[i], acc);
  }
  const float inv = rsqrtf(block_sum<kRmsThreads>(acc, red_sum) / (float)dim + eps);
  // The normed row rounded to bf16 (the value the unfused path stores), kept
  // packed. Rounding to bf16 is monotone, so the absmax of the rounded row is
  // the rounded absmax of the f32 row. The gains are read here, not kept from
  // the first pass: every row of an expert reads the same 8 KB (L1-resident),
  // and 16 fewer registers a thread fit more rows in flight per SM.
  float m = 0.0f;
#pragma unroll
  for (int k = 0; k < kW; ++k) {
    const int c = (k * kRmsThreads + threadIdx.x) * 8;
    const uint4 g = c < dim ? __ldg(reinterpret_cast<const uint4*>(wr + c)) : make_uint4(0, 0, 0, 0);
    float t[8], u[8];
    unpack8(xv[k], t);
    unpack8(g, u);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      t[i] = t[i] * inv * u[i];
      m = fmaxf(m, fabsf(t[i]));
    }
    xv[k] = make_uint4(pack_bf2(t[0], t[1]), pack_bf2(t[2], t[3]), pack_bf2(t[4], t[5]),
                       pack_bf2(t[6], t[7]));
  }
  const float s = __fdiv_rn(bfround(block_max<kRmsThreads>(m, red_max)), 127.0f);
  const float r = quant_recip(s);
  if (threadIdx.x == 0) scale[row] = s;
#pragma unroll
  for (int k = 0; k < kW; ++k) {
    const int c = (k * kRmsThreads + threadIdx.x) * 8;
    if (c >= dim) continue;
    float t[8];
    unpack8(xv[k], t);
    *reinterpret_cast<uint2*>(q + (long)row * dim + c) = quant8(t, s, r);
  }
}

// ---------------------------------------------------------------------
// Split q/k RMSNorm (src/u15-kernels.metal:50-87): one warp per
// (token, head) row of 128, lanes 0-15 own the t half [0,64) and lanes
// 16-31 the hw half [64,128), 4 elements each; two 16-lane reductions.
// ---------------------------------------------------------------------
__device__ __forceinline__ float half_sum(float v)
{
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__global__ void split_qk_norm_kernel(__nv_bfloat16* __restrict__ x,
                                     const __nv_bfloat16* __restrict__ w_t,
                                     const __nv_bfloat16* __restrict__ w_hw, long nrows,
                                     float eps)
{
  const long row = (long)blockIdx.x * (blockDim.x / 32) + warp_id();
  if (row >= nrows) return;
  const int l = lane_id();
  __nv_bfloat16* r = x + row * 128 + l * 4;
  const uint2 u = *reinterpret_cast<const uint2*>(r);
  const float2 a = unpack_bf2(u.x), b = unpack_bf2(u.y);
  float v[4] = {a.x, a.y, b.x, b.y};
  float ss = v[0] * v[0] + v[1] * v[1] + v[2] * v[2] + v[3] * v[3];
  ss = half_sum(ss);
  const float inv = rsqrtf(ss / 64.0f + eps);
  const __nv_bfloat16* g = (l < 16 ? w_t : w_hw) + (l & 15) * 4;
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] = v[i] * inv * bf2f(g[i]);
  uint2 o;
  o.x = pack_bf2(v[0], v[1]);
  o.y = pack_bf2(v[2], v[3]);
  *reinterpret_cast<uint2*>(r) = o;
}

// ---------------------------------------------------------------------
// Split-3 RoPE (src/u15-kernels.metal:118-157), same warp-per-row layout:
// pairs (i, i+32) of the t range sit 8 lanes apart, pairs (64+i, 80+i)
// and (96+i, 112+i) of h and w sit 4 lanes apart, so each lane fetches its
// partner's values with one shuffle. Tables are [T][128] f32, doubled, so
// both members of a pair read the same angle at their own column.
// ---------------------------------------------------------------------
__device__ __forceinline__ void rope4(float (&v)[4], const float* cs, const float* sn, int l)
{
  const int m = l < 16 ? 8 : 4;
  const bool first = l < 16 ? (l < 8) : ((l & 7) < 4);
  float p[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) p[i] = __shfl_xor_sync(0xffffffffu, v[i], m);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float c = cs[i], s = sn[i];
    v[i] = first ? (v[i] * c - p[i] * s) : (v[i] * c + p[i] * s);
  }
}

__global__ void split_rope_kernel(__nv_bfloat16* __restrict__ x, const float* __restrict__ cosf_,
                                  const float* __restrict__ sinf_, long nrows, int heads)
{
  const long row = (long)blockIdx.x * (blockDim.x / 32) + warp_id();
  if (row >= nrows) return;
  const int l = lane_id();
  const long t = row / heads;
  __nv_bfloat16* r = x + row * 128 + l * 4;
  const uint2 u = *reinterpret_cast<const uint2*>(r);
  const float2 a = unpack_bf2(u.x), b = unpack_bf2(u.y);
  float v[4] = {a.x, a.y, b.x, b.y};
  const float4 c4 = *reinterpret_cast<const float4*>(cosf_ + t * 128 + l * 4);
  const float4 s4 = *reinterpret_cast<const float4*>(sinf_ + t * 128 + l * 4);
  const float cs[4] = {c4.x, c4.y, c4.z, c4.w}, sn[4] = {s4.x, s4.y, s4.z, s4.w};
  rope4(v, cs, sn, l);
  uint2 o;
  o.x = pack_bf2(v[0], v[1]);
  o.y = pack_bf2(v[2], v[3]);
  *reinterpret_cast<uint2*>(r) = o;
}

// ---------------------------------------------------------------------
// RoPE tables on the device, angles in fp64 (src/u15-metal-ops.cc:547-605).
// A block covers kRopeTok tokens x 128 columns; the 128 inverse frequencies
// (column c in range [off, off + width)) are formed once per block.
// ---------------------------------------------------------------------
constexpr int kRopeTok = 16;

__global__ void rope_tables_kernel(const int32_t* __restrict__ pt, const int32_t* __restrict__ ph,
                                   const int32_t* __restrict__ pw, int tokens, int d_t, int d_h,
                                   double theta_t, double theta_hw, float* __restrict__ cos_out,
                                   float* __restrict__ sin_out)
{
  griddep_launch();
  griddep_wait();
  __shared__ double inv_s[128];
  if (threadIdx.x < 128) {
    const int c = threadIdx.x;
    int off, width;
    double theta;
    if (c < d_t) { off = 0; width = d_t; theta = theta_t; }
    else if (c < d_t + d_h) { off = d_t; width = d_h; theta = theta_hw; }
    else { off = d_t + d_h; width = d_h; theta = theta_hw; }
    const int i = (c - off) % (width / 2);
    inv_s[c] = 1.0 / pow(theta, (double)(2 * i) / (double)width);
  }
  __syncthreads();
  const int c = threadIdx.x & 127;
  const int32_t* pos = c < d_t ? pt : (c < d_t + d_h ? ph : pw);
  const double inv = inv_s[c];
  for (int r = threadIdx.x >> 7; r < kRopeTok; r += blockDim.x >> 7) {
    const int t = blockIdx.x * kRopeTok + r;
    if (t >= tokens) break;
    const double ang = (double)pos[t] * inv;
    const long idx = (long)t * 128 + c;
    cos_out[idx] = (float)cos(ang);
    sin_out[idx] = (float)sin(ang);
  }
}

// The same tables when the sections are even and fill the 128 columns
// (d_t + 2 d_h = 128): column c and c + width / 2 of a section share their
// frequency, so a thread forms one angle of the 64 distinct ones per token,
// takes its sine and cosine together and writes both columns.
__global__ void rope_tables_pair_kernel(const int32_t* __restrict__ pt,
                                        const int32_t* __restrict__ ph,
                                        const int32_t* __restrict__ pw, int tokens, int d_t,
                                        int d_h, double theta_t, double theta_hw,
                                        float* __restrict__ cos_out, float* __restrict__ sin_out)
{
  griddep_launch();
  griddep_wait();
  __shared__ double inv_s[64];
  __shared__ int col_s[64], half_s[64], sec_s[64];
  if (threadIdx.x < 64) {
    const int u = threadIdx.x, ht = d_t / 2, hh = d_h / 2;
    int off, width, i, sec;
    double theta;
    if (u < ht) { off = 0; width = d_t; i = u; theta = theta_t; sec = 0; }
    else if (u < ht + hh) { off = d_t; width = d_h; i = u - ht; theta = theta_hw; sec = 1; }
    else { off = d_t + d_h; width = d_h; i = u - ht - hh; theta = theta_hw; sec = 2; }
    inv_s[u] = 1.0 / pow(theta, (double)(2 * i) / (double)width);
    col_s[u] = off + i;
    half_s[u] = width / 2;
    sec_s[u] = sec;
  }
  __syncthreads();
  const int u = threadIdx.x & 63;
  const int32_t* pos = sec_s[u] == 0 ? pt : (sec_s[u] == 1 ? ph : pw);
  const double inv = inv_s[u];
  const int c0 = col_s[u], c1 = c0 + half_s[u];
  for (int r = threadIdx.x >> 6; r < kRopeTok; r += blockDim.x >> 6) {
    const int t = blockIdx.x * kRopeTok + r;
    if (t >= tokens) break;
    const double ang = (double)pos[t] * inv;
    double sv, cv;
    sincos(ang, &sv, &cv);
    const long row = (long)t * 128;
    cos_out[row + c0] = (float)cv;
    cos_out[row + c1] = (float)cv;
    sin_out[row + c0] = (float)sv;
    sin_out[row + c1] = (float)sv;
  }
}

// ---------------------------------------------------------------------
// Fused QKV post-processing of the token-major GEMM output
// qkv [T][(NH + 2*KV) * 128], per (token, head) row:
//   q heads: split norm (q_norm, q_norm_hw of the row's expert) -> bf16 ->
//            split rope -> bf16 -> q_out [NH][T][128]      (transpose_thd)
//   k heads: the same with k_norm / k_norm_hw -> K cache @ kv_off (append)
//   v heads: copied -> V cache @ kv_off                    (append)
// The reference runs these as split_qk_norm, split_rope, transpose_thd and
// transpose_into_cache (src/u15-backbone.cc:199-214); the bf16 rounding
// after the norm and after the rope is kept.
// norms: [E][4][64] bf16 = q_t, q_hw, k_t, k_hw per expert.
// ---------------------------------------------------------------------
constexpr int kQkvWarps = 8;
constexpr int kQkvTok = 4;       // tokens per token block (two warps a token)
constexpr int kQkvBatch = 4;     // rows a warp loads before it computes
constexpr int kVtPad = 130;      // bf16 per staged V row: 65 words, odd, so the
                                 // column reads of the transpose spread over banks

// One launch, two kinds of block.
// Blocks [0, ntb): four tokens each, two warps a token. Warp w takes token
// w / 2 of the block and its heads w % 2, w % 2 + 2, ... of the q and k heads
// (and, for a cache with untransposed V, the v heads); the token's cos / sin
// columns are loaded once per warp and serve all of them. (One token per
// block spent a quarter of the kernel launching and retiring blocks.)
// Blocks [ntb, ntb + nwin * nkv): one (64-token page window, v head) of a cache
// whose V pages are transposed: the window's V rows are staged in shared
// memory and written as [128 dims][64 tokens] rows, 16 bytes a thread.
// Tokens of a window outside [0, T) (the frozen prefix, past the block) are
// never written.
__global__ void __launch_bounds__(kQkvWarps * 32)
    qkv_post_kernel(const __nv_bfloat16* __restrict__ qkv, const __nv_bfloat16* __restrict__ norms,
                    const float* __restrict__ cosf_, const float* __restrict__ sinf_,
                    __nv_bfloat16* __restrict__ q_out, KvView kv, int T, int nh, int nkv,
                    int kv_off, float eps, SegInfo seg)
{
  griddep_launch();   // the next (tensor-core) kernel may start its set-up
  griddep_wait();     // launched early (PDL): the previous kernel's writes first
  const int heads = nh + 2 * nkv;
  const int l = lane_id(), w = warp_id();
  const int ntb = (T + kQkvTok - 1) / kQkvTok;
  if ((int)blockIdx.x < ntb) {
    constexpr int kWpt = kQkvWarps / kQkvTok;   // warps per token
    const int t = (int)blockIdx.x * kQkvTok + w / kWpt;
    if (t >= T) return;
    const int e = expert_of(t, seg);
    const int nrow = nh + nkv + (kv.v_t ? 0 : nkv);
    const float4 c4 = *reinterpret_cast<const float4*>(cosf_ + (long)t * 128 + l * 4);
    const float4 s4 = *reinterpret_cast<const float4*>(sinf_ + (long)t * 128 + l * 4);
    const float cs[4] = {c4.x, c4.y, c4.z, c4.w}, sn[4] = {s4.x, s4.y, s4.z, s4.w};
    const int j = kv_off + t;
    const long page = kv.page_table ? kv.page_table[j >> 6] : (j >> 6);
    const long kv_row = page * kv.page_stride + (long)(j & 63) * 128 + l * 4;
    const __nv_bfloat16* src = qkv + (long)t * heads * 128 + l * 4;
    const int g = (l < 16 ? 0 : 64) + (l & 15) * 4;
    for (int h0 = w % kWpt; h0 < nrow; h0 += kWpt * kQkvBatch) {
      uint2 u[kQkvBatch];
#pragma unroll
      for (int i = 0; i < kQkvBatch; ++i) {
        const int h = h0 + i * kWpt;
        if (h < nrow) u[i] = *reinterpret_cast<const uint2*>(src + (long)h * 128);
      }
#pragma unroll
      for (int i = 0; i < kQkvBatch; ++i) {
        const int h = h0 + i * kWpt;   // warp-uniform
        if (h >= nrow) break;
        const float2 a = unpack_bf2(u[i].x), b = unpack_bf2(u[i].y);
        float v[4] = {a.x, a.y, b.x, b.y};
        __nv_bfloat16* dst;
        if (h < nh + nkv) {
          const uint2 wn = *reinterpret_cast<const uint2*>(norms + (long)e * 256 +
                                                           (h < nh ? 0 : 128) + g);
          const float2 w0 = unpack_bf2(wn.x), w1 = unpack_bf2(wn.y);
          const float wv[4] = {w0.x, w0.y, w1.x, w1.y};
          float ss = v[0] * v[0] + v[1] * v[1] + v[2] * v[2] + v[3] * v[3];
          ss = half_sum(ss);
          const float inv = rsqrtf(ss / 64.0f + eps);
#pragma unroll
          for (int k = 0; k < 4; ++k) v[k] = bfround(v[k] * inv * wv[k]);
          rope4(v, cs, sn, l);
          dst = h < nh ? q_out + ((long)h * T + t) * 128 + l * 4
                       : reinterpret_cast<__nv_bfloat16*>(kv.k) + kv_row +
                             (long)(h - nh) * kv.head_stride;
        } else {
          dst = reinterpret_cast<__nv_bfloat16*>(kv.v) + kv_row +
                (long)(h - nh - nkv) * kv.head_stride;
        }
        uint2 o;
        o.x = pack_bf2(v[0], v[1]);
        o.y = pack_bf2(v[2], v[3]);
        *reinterpret_cast<uint2*>(dst) = o;
      }
    }
    return;
  }
  // ---- transposed V: one (window, v head)
  __shared__ uint32_t tile[64 * kVtPad / 2];
  const int vb = (int)blockIdx.x - ntb;
  const int win = vb / nkv, hv = vb % nkv;
  const int jw = (kv_off & ~63) + win * 64;       // first cache token of the window
  const int t_lo = max(0, kv_off - jw), t_hi = min(64, kv_off + T - jw);   // valid [t_lo, t_hi)
  // stage: 64 rows x 16 chunks of 8 dims, 4 per thread
#pragma unroll
  for (int it = 0; it < 4; ++it) {
    const int item = threadIdx.x + it * kQkvWarps * 32;
    const int r = item >> 4, q = item & 15;
    if (r >= t_lo && r < t_hi) {
      const int t = jw + r - kv_off;
      const uint4 x = *reinterpret_cast<const uint4*>(
          qkv + ((long)t * heads + nh + nkv + hv) * 128 + q * 8);
      uint32_t* d = tile + r * (kVtPad / 2) + q * 4;
      d[0] = x.x;
      d[1] = x.y;
      d[2] = x.z;
      d[3] = x.w;
    }
  }
  __syncthreads();
  const long page = kv.page_table ? kv.page_table[jw >> 6] : (jw >> 6);
  __nv_bfloat16* base = reinterpret_cast<__nv_bfloat16*>(kv.v) + page * kv.page_stride +
                        (long)hv * kv.head_stride;
  const unsigned short* tb = reinterpret_cast<const unsigned short*>(tile);
  // write: 128 dim rows x 8 chunks of 8 tokens, 4 per thread; eight lanes
  // fill one 128-byte dim row
#pragma unroll
  for (int it = 0; it < 4; ++it) {
    const int item = threadIdx.x + it * kQkvWarps * 32;
    const int c = item & 7, d = item >> 3;
    unsigned short x[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) x[k] = tb[(8 * c + k) * kVtPad + d];
    __nv_bfloat16* dst = base + (long)d * 64 + 8 * c;
    if (8 * c >= t_lo && 8 * c + 8 <= t_hi) {
      uint4 o;
      o.x = x[0] | ((uint32_t)x[1] << 16);
      o.y = x[2] | ((uint32_t)x[3] << 16);
      o.z = x[4] | ((uint32_t)x[5] << 16);
      o.w = x[6] | ((uint32_t)x[7] << 16);
      *reinterpret_cast<uint4*>(dst) = o;
    } else {
#pragma unroll
      for (int k = 0; k < 8; ++k)
        if (8 * c + k >= t_lo && 8 * c + k < t_hi)
          reinterpret_cast<unsigned short*>(dst)[k] = x[k];
    }
  }
}

// ---------------------------------------------------------------------
// Layout moves (src/u15-kernels.metal:544-600), 16 bytes per thread.
// ---------------------------------------------------------------------
// [T][H*D] -> [H][T][D]
__global__ void transpose_thd_kernel(const __nv_bfloat16* __restrict__ in,
                                     __nv_bfloat16* __restrict__ out, int T, int H, int D)
{
  const long idx = (long)blockIdx.x * blockDim.x + threadIdx.x;   // 8-element chunk
  const int cpr = D / 8;
  if (idx >= (long)T * H * cpr) return;
  const int c = (int)(idx % cpr);
  const long th = idx / cpr;
  const int h = (int)(th % H);
  const long t = th / H;
  const uint4 v = *reinterpret_cast<const uint4*>(in + (t * H + h) * D + c * 8);
  *reinterpret_cast<uint4*>(out + ((long)h * T + t) * D + c * 8) = v;
}
// [H][T][D] -> [T][H*D]
__global__ void transpose_htd_kernel(const __nv_bfloat16* __restrict__ in,
                                     __nv_bfloat16* __restrict__ out, int T, int H, int D)
{
  const long idx = (long)blockIdx.x * blockDim.x + threadIdx.x;
  const int cpr = D / 8;
  if (idx >= (long)T * H * cpr) return;
  const int c = (int)(idx % cpr);
  const long th = idx / cpr;
  const int h = (int)(th % H);
  const long t = th / H;
  const uint4 v = *reinterpret_cast<const uint4*>(in + ((long)h * T + t) * D + c * 8);
  *reinterpret_cast<uint4*>(out + (t * H + h) * D + c * 8) = v;
}
// [T][H*128] -> KV view (paged or contiguous) at token offset `off`.
__global__ void kv_append_kernel(const __nv_bfloat16* __restrict__ in, void* cache,
                                 const int32_t* __restrict__ page_table, long page_stride,
                                 long head_stride, int T, int H, int off)
{
  const long idx = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long)T * H * 16) return;
  const int c = (int)(idx % 16);
  const long th = idx / 16;
  const int h = (int)(th % H);
  const int t = (int)(th / H);
  const int j = off + t;
  const long page = page_table ? page_table[j >> 6] : (j >> 6);
  const uint4 v = *reinterpret_cast<const uint4*>(in + ((long)t * H + h) * 128 + c * 8);
  *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(cache) + page * page_stride +
                            h * head_stride + (long)(j & 63) * 128 + c * 8) = v;
}

// Contiguous [hkv][n][128] <-> cache view, one thread per 8 elements.
__global__ void kv_copy_kernel(__nv_bfloat16* contig, KvView kv, bool is_v, bool to_cache, int n,
                               int hkv)
{
  const long idx = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long)hkv * n * 16) return;
  const int c = (int)(idx % 16);
  const long ht = idx / 16;
  const int t = (int)(ht % n), h = (int)(ht / n);
  const long page = kv.page_table ? kv.page_table[t >> 6] : (t >> 6);
  __nv_bfloat16* base = reinterpret_cast<__nv_bfloat16*>(is_v ? kv.v : kv.k) +
                        page * kv.page_stride + (long)h * kv.head_stride;
  __nv_bfloat16* lin = contig + ((long)h * n + t) * 128 + c * 8;
  if (is_v && kv.v_t) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      __nv_bfloat16* e = base + (long)(c * 8 + i) * 64 + (t & 63);
      if (to_cache) *e = lin[i];
      else lin[i] = *e;
    }
  } else {
    uint4* e = reinterpret_cast<uint4*>(base + (long)(t & 63) * 128 + c * 8);
    if (to_cache) *e = *reinterpret_cast<const uint4*>(lin);
    else *reinterpret_cast<uint4*>(lin) = *e;
  }
}

// ---------------------------------------------------------------------
// Elementwise
// ---------------------------------------------------------------------
__global__ void swiglu_kernel(const __nv_bfloat16* __restrict__ g, const __nv_bfloat16* __restrict__ u,
                              __nv_bfloat16* __restrict__ y, long n8)
{
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n8) return;
  float a[8], b[8];
  load8(g + i * 8, a);
  load8(u + i * 8, b);
#pragma unroll
  for (int k = 0; k < 8; ++k) a[k] = (a[k] / (1.0f + expf(-a[k]))) * b[k];
  store8(y + i * 8, a);
}
__global__ void add_kernel(__nv_bfloat16* __restrict__ d, const __nv_bfloat16* __restrict__ s,
                           long n8)
{
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n8) return;
  float a[8], b[8];
  load8(d + i * 8, a);
  load8(s + i * 8, b);
#pragma unroll
  for (int k = 0; k < 8; ++k) a[k] += b[k];
  store8(d + i * 8, a);
}
__global__ void add_row_kernel(__nv_bfloat16* __restrict__ d, const __nv_bfloat16* __restrict__ r,
                               long rows, int dim8)
{
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * dim8) return;
  float a[8], b[8];
  load8(d + i * 8, a);
  load8(r + (i % dim8) * 8, b);
#pragma unroll
  for (int k = 0; k < 8; ++k) a[k] += b[k];
  store8(d + i * 8, a);
}
__global__ void silu_kernel(__nv_bfloat16* __restrict__ x, long n8)
{
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n8) return;
  float a[8];
  load8(x + i * 8, a);
#pragma unroll
  for (int k = 0; k < 8; ++k) a[k] = a[k] / (1.0f + expf(-a[k]));
  store8(x + i * 8, a);
}

// ---------------------------------------------------------------------
// Symmetric per-row int8 quantisation, one CTA per row:
//   s = absmax / 127 (IEEE fp32 division), q = rn_even(x / s), clamp +-127
// Every step is a single correctly-rounded fp32 operation, so the codes
// equal the CPU restatement's bit for bit.
// ---------------------------------------------------------------------
// One CTA of NT threads per row: absmax, s = amax / 127, codes. PER > 0:
// rows up to NT x PER columns stay in registers (packed) between the two
// passes (NT = kRmsThreads for the rows up to 4096 wide, 256 x 48 for the
// 12288-wide ones); PER = 0 reads the row twice.
template <int NT, int PER>
__global__ void __launch_bounds__(NT)
    quant_rows_kernel(const __nv_bfloat16* __restrict__ x, int8_t* __restrict__ q,
                      float* __restrict__ scale, int cols)
{
  griddep_launch();   // the next (tensor-core) kernel may start its set-up
  griddep_wait();     // launched early (PDL): the previous kernel's writes first
  constexpr int kQuantPer = PER > 0 ? PER : 8;
  const long row = blockIdx.x;
  const __nv_bfloat16* xr = x + row * cols;
  __shared__ float red[NT / 32];
  if (PER > 0) {
    // the row stays packed; its absmax is taken on bf16 pairs (exact)
    uint4 raw[kQuantPer / 8];
    __nv_bfloat162 m2 = __float2bfloat162_rn(0.0f);
#pragma unroll
    for (int k = 0; k < kQuantPer / 8; ++k) {
      const int c = (k * NT + threadIdx.x) * 8;
      raw[k] = make_uint4(0, 0, 0, 0);
      if (c < cols) raw[k] = *reinterpret_cast<const uint4*>(xr + c);
      const uint32_t w4[4] = {raw[k].x, raw[k].y, raw[k].z, raw[k].w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
        m2 = __hmax2(m2, __habs2(*reinterpret_cast<const __nv_bfloat162*>(&w4[i])));
    }
    const float2 mf = __bfloat1622float2(m2);
    const float s = __fdiv_rn(block_max<NT>(fmaxf(mf.x, mf.y), red), 127.0f);
    const float r = quant_recip(s);
    if (threadIdx.x == 0) scale[row] = s;
#pragma unroll
    for (int k = 0; k < kQuantPer / 8; ++k) {
      const int c = (k * NT + threadIdx.x) * 8;
      if (c >= cols) continue;
      float t[8];
      unpack8(raw[k], t);
      *reinterpret_cast<uint2*>(q + row * cols + c) = quant8(t, s, r);
    }
    return;
  }
  float m = 0.0f;
  for (int c = threadIdx.x * 8; c < cols; c += NT * 8) {
    float v[8];
    load8(xr + c, v);
#pragma unroll
    for (int i = 0; i < 8; ++i) m = fmaxf(m, fabsf(v[i]));
  }
  const float s = __fdiv_rn(block_max<NT>(m, red), 127.0f);
  const float r = quant_recip(s);
  if (threadIdx.x == 0) scale[row] = s;
  for (int c = threadIdx.x * 8; c < cols; c += NT * 8) {
    float v[8];
    load8(xr + c, v);
    *reinterpret_cast<uint2*>(q + row * cols + c) = quant8(v, s, r);
  }
}

inline unsigned blocks_for(long n, int threads) { return (unsigned)((n + threads - 1) / threads); }

}  // namespace

// ---------------------------------------------------------------------
// launchers
// ---------------------------------------------------------------------

int launch_rms_norm(const void* x, const void* w, void* y, int rows, int dim, float eps,
                    const SegInfo& seg, cudaStream_t st)
{
  if (rows <= 0) return 0;
  const cudaError_t e = launch_pdl(rms_norm_kernel, dim3(rows), dim3(kRmsThreads), st,
                                   static_cast<const __nv_bfloat16*>(x),
                                   static_cast<const __nv_bfloat16*>(w),
                                   static_cast<__nv_bfloat16*>(y), rows, dim, eps, seg);
  return e == cudaSuccess ? 0 : 2;
}

int launch_rms_norm_quant(const void* x, const void* w, int8_t* q, float* s, int rows, int dim,
                          float eps, const SegInfo& seg, cudaStream_t st)
{
  if (rows <= 0) return 0;
  if (dim > kRmsThreads * kRmsPer || dim % 8) return 1;
  const cudaError_t e = launch_pdl(rms_norm_quant_kernel, dim3(rows), dim3(kRmsThreads), st,
                                   static_cast<const __nv_bfloat16*>(x),
                                   static_cast<const __nv_bfloat16*>(w), q, s, rows, dim, eps,
                                   seg);
  return e == cudaSuccess ? 0 : 2;
}

int launch_split_qk_norm(void* x, const void* w_t, const void* w_hw, int heads, int tokens,
                         float eps, cudaStream_t st)
{
  const long rows = (long)heads * tokens;
  if (rows <= 0) return 0;
  split_qk_norm_kernel<<<blocks_for(rows, 8), 256, 0, st>>>(
      static_cast<__nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(w_t),
      static_cast<const __nv_bfloat16*>(w_hw), rows, eps);
  return cudaGetLastError() == cudaSuccess ? 0 : 2;
}

int launch_split_rope(void* x, const float* c, const float* s, int heads, int tokens,
                      cudaStream_t st)
{
  const long rows = (long)heads * tokens;
  if (rows <= 0) return 0;
  split_rope_kernel<<<blocks_for(rows, 8), 256, 0, st>>>(static_cast<__nv_bfloat16*>(x), c, s,
                                                          rows, heads);
  return cudaGetLastError() == cudaSuccess ? 0 : 2;
}

int launch_rope_tables(const int32_t* pt, const int32_t* ph, const int32_t* pw, int tokens,
                       int d_t, int d_h, double theta_t, double theta_hw, float* c, float* s,
                       cudaStream_t st)
{
  if (tokens <= 0) return 0;
  const unsigned blocks = (unsigned)((tokens + kRopeTok - 1) / kRopeTok);
  const cudaError_t e =
      d_t > 0 && d_h >= 0 && d_t % 2 == 0 && d_h % 2 == 0 && d_t + 2 * d_h == 128
          ? launch_pdl(rope_tables_pair_kernel, dim3(blocks), dim3(256), st, pt, ph, pw, tokens,
                       d_t, d_h, theta_t, theta_hw, c, s)
          : launch_pdl(rope_tables_kernel, dim3(blocks), dim3(256), st, pt, ph, pw, tokens, d_t,
                       d_h, theta_t, theta_hw, c, s);
  return e == cudaSuccess ? 0 : 2;
}

int launch_qkv_post(const void* qkv, const void* norms, const float* c, const float* s,
                    void* q_out, const KvView& kv, int T, int nh, int nkv, int kv_off, float eps,
                    const SegInfo& seg, cudaStream_t st)
{
  if (T <= 0 || nh + 2 * nkv <= 0) return 0;
  // transposed-V windows: the 64-token pages the block [kv_off, kv_off + T) touches
  const long nwin = kv.v_t ? ((kv_off & 63) + T + 63) / 64 : 0;
  const long ntb = (T + kQkvTok - 1) / kQkvTok;
  const cudaError_t e = launch_pdl(
      qkv_post_kernel, dim3((unsigned)(ntb + nwin * nkv)), dim3(kQkvWarps * 32), st,
      static_cast<const __nv_bfloat16*>(qkv), static_cast<const __nv_bfloat16*>(norms), c, s,
      static_cast<__nv_bfloat16*>(q_out), kv, T, nh, nkv, kv_off, eps, seg);
  return e == cudaSuccess ? 0 : 2;
}

int launch_transpose(const void* in, void* out, int T, int H, int D, bool to_head_major,
                     cudaStream_t st)
{
  const long n = (long)T * H * (D / 8);
  if (n <= 0) return 0;
  if (to_head_major)
    transpose_thd_kernel<<<blocks_for(n, 256), 256, 0, st>>>(
        static_cast<const __nv_bfloat16*>(in), static_cast<__nv_bfloat16*>(out), T, H, D);
  else
    transpose_htd_kernel<<<blocks_for(n, 256), 256, 0, st>>>(
        static_cast<const __nv_bfloat16*>(in), static_cast<__nv_bfloat16*>(out), T, H, D);
  return cudaGetLastError() == cudaSuccess ? 0 : 2;
}

int launch_kv_append(const void* in, void* cache, const int32_t* page_table, long page_stride,
                     long head_stride, int T, int H, int off, cudaStream_t st)
{
  const long n = (long)T * H * 16;
  if (n <= 0) return 0;
  kv_append_kernel<<<blocks_for(n, 256), 256, 0, st>>>(static_cast<const __nv_bfloat16*>(in),
                                                        cache, page_table, page_stride,
                                                        head_stride, T, H, off);
  return cudaGetLastError() == cudaSuccess ? 0 : 2;
}

int launch_kv_copy(void* contig, const KvView& kv, bool is_v, bool to_cache, int n, int hkv,
                   cudaStream_t st)
{
  const long m = (long)hkv * n * 16;
  if (m <= 0) return 0;
  kv_copy_kernel<<<blocks_for(m, 256), 256, 0, st>>>(static_cast<__nv_bfloat16*>(contig), kv,
                                                      is_v, to_cache, n, hkv);
  return cudaGetLastError() == cudaSuccess ? 0 : 2;
}

int launch_swiglu(const void* g, const void* u, void* y, long n, cudaStream_t st)
{
  if (n <= 0) return 0;
  swiglu_kernel<<<blocks_for(n / 8, 256), 256, 0, st>>>(static_cast<const __nv_bfloat16*>(g),
                                                         static_cast<const __nv_bfloat16*>(u),
                                                         static_cast<__nv_bfloat16*>(y), n / 8);
  return cudaGetLastError() == cudaSuccess ? 0 : 2;
}

int launch_add(void* d, const void* s, long n, cudaStream_t st)
{
  if (n <= 0) return 0;
  add_kernel<<<blocks_for(n / 8, 256), 256, 0, st>>>(static_cast<__nv_bfloat16*>(d),
                                                      static_cast<const __nv_bfloat16*>(s), n / 8);
  return cudaGetLastError() == cudaSuccess ? 0 : 2;
}

int launch_add_row(void* d, const void* r, long rows, int dim, cudaStream_t st)
{
  if (rows <= 0) return 0;
  add_row_kernel<<<blocks_for(rows * (dim / 8), 256), 256, 0, st>>>(
      static_cast<__nv_bfloat16*>(d), static_cast<const __nv_bfloat16*>(r), rows, dim / 8);
  return cudaGetLastError() == cudaSuccess ? 0 : 2;
}

int launch_silu(void* x, long n, cudaStream_t st)
{
  if (n <= 0) return 0;
  silu_kernel<<<blocks_for(n / 8, 256), 256, 0, st>>>(static_cast<__nv_bfloat16*>(x), n / 8);
  return cudaGetLastError() == cudaSuccess ? 0 : 2;
}

int launch_quant_rows(const void* x, int8_t* q, float* s, int rows, int cols, cudaStream_t st)
{
  if (rows <= 0) return 0;
  const __nv_bfloat16* xb = static_cast<const __nv_bfloat16*>(x);
  cudaError_t e;
  if (cols <= kRmsThreads * kRmsPer)
    e = launch_pdl(quant_rows_kernel<kRmsThreads, kRmsPer>, dim3(rows), dim3(kRmsThreads), st,
                   xb, q, s, cols);
  else if (cols <= 256 * 48)
    e = launch_pdl(quant_rows_kernel<256, 48>, dim3(rows), dim3(256), st, xb, q, s, cols);
  else
    e = launch_pdl(quant_rows_kernel<256, 0>, dim3(rows), dim3(256), st, xb, q, s, cols);
  return e == cudaSuccess ? 0 : 2;
}

}  // namespace u15
