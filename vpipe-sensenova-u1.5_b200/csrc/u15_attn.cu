// Flash attention for the MoT layer, head_dim 128, GQA.
//
//   out[i][h*128 + :] = softmax_j(q_h[i] . k_{h/G}[j] / sqrt(128) + mask) v_{h/G}[j]
//
// q head-major [hq][tq][128] (what the QKV epilogue writes), K/V read from
// a paged or contiguous cache through KvView (the reference reads its
// contiguous [hkv][cap][128] cache with cap as the head stride,
// src/u15-metal-ops.cc:687-787), out token-major [tq][hq*128] -- the
// reference's transpose_htd is folded into the store.
//
// One CTA serves the G query heads of one kv-head group for R = 128/G query
// rows (128 rows total, 8 warps x 16), so each K/V tile is read once for
// all G heads. K/V tiles are 64 keys (one cache page), double-buffered with
// cp.async; S = QK^T and O += PV on mma.sync m16n8k16 (bf16) with online
// softmax in registers. Masks are evaluated per element from the rule:
//   0 bidirectional   every key j < tk                (denoise)
//   1 causal          j <= q_offset + i               (text prefill)
//   2 block-causal    t[j] == t[q_offset+i] or j <= q_offset + i   (edit prefill)
// The causal form skips KV tiles past the CTA's last query.
//
// The Sage variant (bidirectional only) computes QK^T with mma.sync
// m16n8k32 s8 x s8 -> s32 from int8 Q and smoothed int8 K prepared by
// sage_prepare(), with one scale per 64-row Q block and per 32-key K
// block (the reference's Sage tiles, bq 64 / bk 32); P.V stays bf16.
#include "u15_common.cuh"
#include "u15_kernels.h"

#include <algorithm>
#include <cmath>

namespace u15 {

namespace {

constexpr int kRows = 128;      // query rows per CTA (all heads of the group)
constexpr int kKeys = 64;       // keys per tile (= one cache page)
constexpr int kThreads = 256;

struct AttnP {
  const __nv_bfloat16* q;
  KvView kv;
  __nv_bfloat16* out;
  int hq, hkv, tq, tk, mode, q_offset, G, R;
  const int32_t* t_index;
  float scale_log2;
  const int8_t* q8;
  const int8_t* k8;
  const float* sq;
  const float* sk;
  int nqb, nkb;
  long k8_stride;   // rows per kv head in k8
};

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid)
{
  const int n = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3)
{
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                          uint32_t& r3)
{
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma_bf16_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0,
                                               uint32_t b1)
{
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma_s8_16832(int (&c)[4], const uint32_t (&a)[4], uint32_t b0,
                                             uint32_t b1)
{
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Swizzled shared-memory offsets: 16-byte chunk c of row r is stored at
// chunk (c ^ (r & 7)), so the 8 rows an ldmatrix reads hit 8 bank groups.
__device__ __forceinline__ uint32_t swz256(int r, int c) { return r * 256 + ((c ^ (r & 7)) << 4); }
__device__ __forceinline__ uint32_t swz128(int r, int c) { return r * 128 + ((c ^ (r & 7)) << 4); }

__device__ __forceinline__ const __nv_bfloat16* kv_row(const KvView& kv, const void* base, int h,
                                                       int j)
{
  const long page = kv.page_table ? (long)kv.page_table[j >> 6] : (long)(j >> 6);
  return reinterpret_cast<const __nv_bfloat16*>(base) + page * kv.page_stride +
         (long)h * kv.head_stride + (long)(j & 63) * 128;
}

template <bool SAGE, bool VT>
__global__ void __launch_bounds__(kThreads, 2) attn_kernel(const __grid_constant__ AttnP p)
{
  extern __shared__ __align__(128) uint8_t sm[];
  // bf16: Q 32 KB | K 2 x 16 KB | V 2 x 16 KB.  Sage: Q8 16 KB | K8 2 x 8 KB | V 2 x 16 KB
  constexpr int kQBytes = SAGE ? kRows * 128 : kRows * 256;
  constexpr int kKBytes = SAGE ? kKeys * 128 : kKeys * 256;
  constexpr int kVBytes = kKeys * 256;
  uint8_t* sQ = sm;
  uint8_t* sK = sm + kQBytes;
  uint8_t* sV = sK + 2 * kKBytes;
  const uint32_t aQ = smem_u32(sQ), aK = smem_u32(sK), aV = smem_u32(sV);

  const int hk = blockIdx.y;
  const int q0 = blockIdx.x * p.R;
  const int tid = threadIdx.x, w = tid >> 5, l = tid & 31;

  // ---- Q tile: row r -> head hk*G + r/R, query q0 + r%R ----
  if constexpr (SAGE) {
    for (int i = tid; i < kRows * 8; i += kThreads) {
      const int r = i >> 3, c = i & 7;
      const int h = hk * p.G + r / p.R, qi = q0 + r % p.R;
      const bool ok = qi < p.tq;
      const int8_t* src = p.q8 + ((long)h * p.tq + (ok ? qi : 0)) * 128 + c * 16;
      cp_async16(aQ + swz128(r, c), src, ok);
    }
  } else {
    for (int i = tid; i < kRows * 16; i += kThreads) {
      const int r = i >> 4, c = i & 15;
      const int h = hk * p.G + r / p.R, qi = q0 + r % p.R;
      const bool ok = qi < p.tq;
      const __nv_bfloat16* src = p.q + ((long)h * p.tq + (ok ? qi : 0)) * 128 + c * 8;
      cp_async16(aQ + swz256(r, c), src, ok);
    }
  }

  // ---- which KV tiles this CTA needs ----
  int n_tiles = (p.tk + kKeys - 1) / kKeys;
  if (p.mode == 1) {
    const int last_q = p.q_offset + min(q0 + p.R, p.tq) - 1;
    n_tiles = min(n_tiles, last_q / kKeys + 1);
  }

  auto load_kv = [&](int tile, int buf) {
    const int j0 = tile * kKeys;
    if constexpr (SAGE) {
      for (int i = tid; i < kKeys * 8; i += kThreads) {
        const int r = i >> 3, c = i & 7;
        const int j = j0 + r;
        const bool ok = j < p.tk;
        const int8_t* src = p.k8 + ((long)hk * p.k8_stride + (ok ? j : 0)) * 128 + c * 16;
        cp_async16(aK + buf * kKBytes + swz128(r, c), src, ok);
      }
    } else {
      for (int i = tid; i < kKeys * 16; i += kThreads) {
        const int r = i >> 4, c = i & 15;
        const int j = j0 + r;
        const bool ok = j < p.tk;
        const __nv_bfloat16* src = kv_row(p.kv, p.kv.k, hk, ok ? j : 0) + c * 8;
        cp_async16(aK + buf * kKBytes + swz256(r, c), src, ok);
      }
    }
    if constexpr (VT) {
      // transposed page: 128 dim rows of 64 keys (8 chunks), one page per tile
      const long page = p.kv.page_table ? (long)p.kv.page_table[j0 >> 6] : (long)(j0 >> 6);
      const __nv_bfloat16* vb = reinterpret_cast<const __nv_bfloat16*>(p.kv.v) +
                                page * p.kv.page_stride + (long)hk * p.kv.head_stride;
      for (int i = tid; i < 128 * 8; i += kThreads) {
        const int r = i >> 3, c = i & 7;
        cp_async16(aV + buf * kVBytes + swz128(r, c), vb + (long)r * 64 + c * 8,
                   j0 + c * 8 < p.tk);
      }
    } else {
      for (int i = tid; i < kKeys * 16; i += kThreads) {
        const int r = i >> 4, c = i & 15;
        const int j = j0 + r;
        const bool ok = j < p.tk;
        const __nv_bfloat16* src = kv_row(p.kv, p.kv.v, hk, ok ? j : 0) + c * 8;
        cp_async16(aV + buf * kVBytes + swz256(r, c), src, ok);
      }
    }
  };

  if (n_tiles > 0) load_kv(0, 0);
  cp_async_commit();

  // per-thread rows: r0 = w*16 + l/4, r1 = r0 + 8
  const int r0 = w * 16 + (l >> 2), r1 = r0 + 8;
  const int h0 = hk * p.G + r0 / p.R, h1 = hk * p.G + r1 / p.R;
  const int qi0 = q0 + r0 % p.R, qi1 = q0 + r1 % p.R;
  const int qp0 = p.q_offset + qi0, qp1 = p.q_offset + qi1;
  int tq0 = 0, tq1 = 0;
  if (p.mode == 2) {
    tq0 = qi0 < p.tq ? p.t_index[qp0] : 0;
    tq1 = qi1 < p.tq ? p.t_index[qp1] : 0;
  }
  float sq0 = 1.0f, sq1 = 1.0f;
  if constexpr (SAGE) {
    sq0 = qi0 < p.tq ? p.sq[(long)h0 * p.nqb + qi0 / 64] : 0.0f;
    sq1 = qi1 < p.tq ? p.sq[(long)h1 * p.nqb + qi1 / 64] : 0.0f;
  }

  float o[16][4];
#pragma unroll
  for (int d = 0; d < 16; ++d) o[d][0] = o[d][1] = o[d][2] = o[d][3] = 0.0f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.0f, l1 = 0.0f;

  for (int t = 0; t < n_tiles; ++t) {
    cp_async_wait_all();
    __syncthreads();
    if (t + 1 < n_tiles) load_kv(t + 1, (t + 1) & 1);
    cp_async_commit();
    const int buf = t & 1;
    const int j0 = t * kKeys;

    // ---- S = Q K^T, 16 rows x 64 keys per warp ----
    float s[8][4];
    if constexpr (SAGE) {
      int si[8][4];
#pragma unroll
      for (int n = 0; n < 8; ++n) si[n][0] = si[n][1] = si[n][2] = si[n][3] = 0;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        uint32_t a[4];
        const int ar = w * 16 + (l & 7) + ((l >> 3) & 1) * 8;
        ldsm_x4(aQ + swz128(ar, 2 * kk + (l >> 4)), a[0], a[1], a[2], a[3]);
#pragma unroll
        for (int np = 0; np < 4; ++np) {
          uint32_t b0, b1, b2, b3;
          const int br = np * 16 + (l & 7) + (l >> 4) * 8;
          ldsm_x4(aK + buf * kKBytes + swz128(br, 2 * kk + ((l >> 3) & 1)), b0, b1, b2, b3);
          mma_s8_16832(si[2 * np], a, b0, b1);
          mma_s8_16832(si[2 * np + 1], a, b2, b3);
        }
      }
      // keys [0, 32) and [32, 64) of the tile are two K blocks (columns n * 8 + ..)
      const float ska = p.sk[(long)hk * p.nkb + 2 * t] * p.scale_log2;
      const float skb = p.sk[(long)hk * p.nkb + 2 * t + 1] * p.scale_log2;
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        const float skv = n < 4 ? ska : skb;
        const float f0 = sq0 * skv, f1 = sq1 * skv;
        s[n][0] = (float)si[n][0] * f0;
        s[n][1] = (float)si[n][1] * f0;
        s[n][2] = (float)si[n][2] * f1;
        s[n][3] = (float)si[n][3] * f1;
      }
    } else {
#pragma unroll
      for (int n = 0; n < 8; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.0f;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        uint32_t a[4];
        const int ar = w * 16 + (l & 7) + ((l >> 3) & 1) * 8;
        ldsm_x4(aQ + swz256(ar, 2 * kk + (l >> 4)), a[0], a[1], a[2], a[3]);
#pragma unroll
        for (int np = 0; np < 4; ++np) {
          uint32_t b0, b1, b2, b3;
          const int br = np * 16 + (l & 7) + (l >> 4) * 8;
          ldsm_x4(aK + buf * kKBytes + swz256(br, 2 * kk + ((l >> 3) & 1)), b0, b1, b2, b3);
          mma_bf16_16816(s[2 * np], a, b0, b1);
          mma_bf16_16816(s[2 * np + 1], a, b2, b3);
        }
      }
#pragma unroll
      for (int n = 0; n < 8; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) s[n][e] *= p.scale_log2;
    }

    // ---- mask ----
    const bool tail = j0 + kKeys > p.tk;
    if (tail || p.mode != 0) {
#pragma unroll
      for (int n = 0; n < 8; ++n) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int j = j0 + n * 8 + (l & 3) * 2 + (e & 1);
          const int qp = e < 2 ? qp0 : qp1;
          bool ok = j < p.tk;
          if (p.mode == 1) ok = ok && (j <= qp);
          else if (p.mode == 2) ok = ok && ((j <= qp) || (p.t_index[j] == (e < 2 ? tq0 : tq1)));
          if (!ok) s[n][e] = -INFINITY;
        }
      }
    }

    // ---- online softmax (base 2) ----
    float mx0 = m0, mx1 = m1;
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      mx0 = fmaxf(mx0, fmaxf(s[n][0], s[n][1]));
      mx1 = fmaxf(mx1, fmaxf(s[n][2], s[n][3]));
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float use0 = mx0 == -INFINITY ? 0.0f : mx0;
    const float use1 = mx1 == -INFINITY ? 0.0f : mx1;
    const float c0 = exp2f(m0 - use0), c1 = exp2f(m1 - use1);   // exp2(-inf) = 0
    m0 = mx0;
    m1 = mx1;
    l0 *= c0;
    l1 *= c1;
#pragma unroll
    for (int d = 0; d < 16; ++d) {
      o[d][0] *= c0; o[d][1] *= c0;
      o[d][2] *= c1; o[d][3] *= c1;
    }
    uint32_t pa[4][4];   // P as the A operand of 4 k-steps of 16 keys
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      const float p0 = exp2f(s[n][0] - use0), p1 = exp2f(s[n][1] - use0);
      const float p2 = exp2f(s[n][2] - use1), p3 = exp2f(s[n][3] - use1);
      l0 += p0 + p1;
      l1 += p2 + p3;
      const int kk = n >> 1, hi = n & 1;
      pa[kk][hi * 2 + 0] = pack_bf2(p0, p1);
      pa[kk][hi * 2 + 1] = pack_bf2(p2, p3);
    }

    // ---- O += P V ----
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const uint32_t a[4] = {pa[kk][0], pa[kk][1], pa[kk][2], pa[kk][3]};
#pragma unroll
      for (int dp = 0; dp < 8; ++dp) {
        uint32_t b0, b1, b2, b3;
        if constexpr (VT) {
          const int vr = dp * 16 + (l & 7) + (l >> 4) * 8;
          ldsm_x4(aV + buf * kVBytes + swz128(vr, 2 * kk + ((l >> 3) & 1)), b0, b1, b2, b3);
        } else {
          const int vr = kk * 16 + (l & 7) + ((l >> 3) & 1) * 8;
          ldsm_x4_t(aV + buf * kVBytes + swz256(vr, 2 * dp + (l >> 4)), b0, b1, b2, b3);
        }
        mma_bf16_16816(o[2 * dp], a, b0, b1);
        mma_bf16_16816(o[2 * dp + 1], a, b2, b3);
      }
    }
  }
  cp_async_wait_all();

  // ---- normalise and store token-major through shared memory ----
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const float inv0 = l0 > 0.0f ? 1.0f / l0 : 0.0f, inv1 = l1 > 0.0f ? 1.0f / l1 : 0.0f;
  __syncthreads();
  uint8_t* sO = SAGE ? sV : sQ;   // 32 KB of bf16 staging
  const uint32_t aO = smem_u32(sO);
#pragma unroll
  for (int d = 0; d < 16; ++d) {
    const int col = d * 8 + (l & 3) * 2;
    const uint32_t v0 = pack_bf2(o[d][0] * inv0, o[d][1] * inv0);
    const uint32_t v1 = pack_bf2(o[d][2] * inv1, o[d][3] * inv1);
    *reinterpret_cast<uint32_t*>(sO + swz256(r0, col >> 3) + (col & 7) * 2) = v0;
    *reinterpret_cast<uint32_t*>(sO + swz256(r1, col >> 3) + (col & 7) * 2) = v1;
  }
  (void)aO;
  __syncthreads();
  for (int i = tid; i < kRows * 16; i += kThreads) {
    const int r = i >> 4, c = i & 15;
    const int h = hk * p.G + r / p.R, qi = q0 + r % p.R;
    if (qi >= p.tq) continue;
    const uint4 v = *reinterpret_cast<const uint4*>(sO + swz256(r, c));
    *reinterpret_cast<uint4*>(p.out + (long)qi * p.hq * 128 + (long)h * 128 + c * 8) = v;
  }
}

// ---------------------------------------------------------------------
// Sage prologue
// ---------------------------------------------------------------------
// Two launches, both with programmatic dependent launch. The first runs,
// side by side, the Q blocks (four 64-row blocks of one head per CTA, each
// block: absmax, s = amax / 127, int8 codes) and the K-mean partials (one
// 64-key page of one kv head per CTA: the page's channel sums; these CTAs
// follow the Q CTAs, pages of every kv head packed with no empty CTA). The
// second runs the K blocks: each CTA forms kmean[c] = sum of the page
// partials / tk (each warp sums every eighth page, four channels a lane,
// the eight warp sums added in warp order), smooths its page's 64 keys by
// it and quantizes them like Q as two 32-key blocks, one scale each (the
// reference's key block, bk = 32, src/u15-metal-ops.cc:702). Rows stay in
// registers between the absmax and the codes: 16-byte loads, 8-byte stores.
constexpr int kSageThreads = 256;
constexpr int kSageQBlocks = 2;   // 64-row Q blocks per CTA

__device__ __forceinline__ void unpack8_bf(const uint4 u, float (&v)[8])
{
  const float2 a = unpack_bf2(u.x), b = unpack_bf2(u.y), c = unpack_bf2(u.z), d = unpack_bf2(u.w);
  v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y; v[4] = c.x; v[5] = c.y; v[6] = d.x; v[7] = d.y;
}

__device__ __forceinline__ void load8_bf(const __nv_bfloat16* p, float (&v)[8])
{
  unpack8_bf(*reinterpret_cast<const uint4*>(p), v);
}

__device__ __forceinline__ float block_absmax(float m, float* red)
{
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (lane_id() == 0) red[warp_id()] = m;
  __syncthreads();
  float amax = 0.0f;
#pragma unroll
  for (int i = 0; i < kSageThreads / 32; ++i) amax = fmaxf(amax, red[i]);
  return amax;
}

// codes of v[4][8] (rows r0 + 16 i, columns 8 c8 ..) with scale s
__device__ __forceinline__ void store_codes(const float (&v)[4][8], float s, bool (&valid)[4],
                                            int8_t* out, long row0, int c8)
{
  const float r = quant_recip(s);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if (!valid[i]) continue;
    *reinterpret_cast<uint2*>(out + (row0 + 16 * i) * 128 + c8 * 8) = quant8(v[i], s, r);
  }
}

__global__ void __launch_bounds__(kSageThreads)
    sage_q_kernel(const __nv_bfloat16* q, KvView kv, int hq, int hkv, int tq, int tk, int nqb,
                  int npg, int8_t* q8, float* sq, float* kpart)
{
  griddep_wait();
  griddep_launch();
  const int tid = threadIdx.x;
  const int nqc = (nqb + kSageQBlocks - 1) / kSageQBlocks;   // Q CTAs a head
  if ((int)blockIdx.x >= nqc) {
    // K-mean partial of one page: thread (key slot kr, 8-channel group c8)
    // sums keys kr, kr + 16, kr + 32, kr + 48 of the page with 16-byte loads,
    // then the 16 key slots of each channel are added in slot order
    const int f = ((int)blockIdx.x - nqc) * hq + (int)blockIdx.y;
    if (f >= hkv * npg) return;
    const int hk = f / npg, pg = f % npg;
    const int c8 = tid & 15, kr = tid >> 4;
    float acc[8] = {};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int j = pg * 64 + kr + 16 * i;
      if (j < tk) {
        float v[8];
        load8_bf(kv_row(kv, kv.k, hk, j) + c8 * 8, v);
#pragma unroll
        for (int k = 0; k < 8; ++k) acc[k] += v[k];
      }
    }
    __shared__ float part[16][129];
#pragma unroll
    for (int k = 0; k < 8; ++k) part[kr][c8 * 8 + k] = acc[k];
    __syncthreads();
    if (tid < 128) {
      float t = 0.0f;
#pragma unroll
      for (int r = 0; r < 16; ++r) t += part[r][tid];
      kpart[((long)hk * npg + pg) * 128 + tid] = t;
    }
    return;
  }
  // Q: blocks b0 .. b0 + 3 of head h; thread (row slot rr, 8-column group
  // c8) holds rows 64 b + rr + 16 i of each block, all 16 loads in flight
  const int h = blockIdx.y, b0 = (int)blockIdx.x * kSageQBlocks;
  const int c8 = tid & 15, rr = tid >> 4;
  const __nv_bfloat16* qh = q + (long)h * tq * 128;
  uint4 raw[kSageQBlocks][4];
  float m[kSageQBlocks];
#pragma unroll
  for (int g = 0; g < kSageQBlocks; ++g) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = (b0 + g) * 64 + rr + 16 * i;
      raw[g][i] = r < tq ? *reinterpret_cast<const uint4*>(qh + (long)r * 128 + c8 * 8)
                         : make_uint4(0u, 0u, 0u, 0u);
    }
  }
#pragma unroll
  for (int g = 0; g < kSageQBlocks; ++g) {
    m[g] = 0.0f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float v[8];
      unpack8_bf(raw[g][i], v);
#pragma unroll
      for (int k = 0; k < 8; ++k) m[g] = fmaxf(m[g], fabsf(v[k]));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m[g] = fmaxf(m[g], __shfl_xor_sync(0xffffffffu, m[g], o));
  }
  __shared__ float red[kSageQBlocks][kSageThreads / 32];
  if (lane_id() == 0) {
#pragma unroll
    for (int g = 0; g < kSageQBlocks; ++g) red[g][warp_id()] = m[g];
  }
  __syncthreads();
#pragma unroll
  for (int g = 0; g < kSageQBlocks; ++g) {
    const int b = b0 + g;
    if (b >= nqb) break;
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < kSageThreads / 32; ++i) amax = fmaxf(amax, red[g][i]);
    const float sc = __fdiv_rn(amax, 127.0f);
    if (tid == 0) sq[(long)h * nqb + b] = sc;
    const float rc = quant_recip(sc);
    int8_t* out = q8 + (long)h * tq * 128;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = b * 64 + rr + 16 * i;
      if (r >= tq) continue;
      float v[8];
      unpack8_bf(raw[g][i], v);
      *reinterpret_cast<uint2*>(out + (long)r * 128 + c8 * 8) = quant8(v, sc, rc);
    }
  }
}

__global__ void __launch_bounds__(kSageThreads)
    sage_k_kernel(KvView kv, int tk, int npg, const float* kpart, int8_t* k8, float* sk,
                  long k8_stride)
{
  griddep_wait();
  griddep_launch();
  __shared__ float red[2][kSageThreads / 32];
  __shared__ float km[128];
  const int pg = blockIdx.x, hk = blockIdx.y, tid = threadIdx.x;
  {
    // kmean over the pages: warp w sums pages w, w + 8, ... in page order
    // (lane l: channels 4 l .. 4 l + 3, four pages' loads in flight), then
    // the eight warp sums are added in warp order
    __shared__ float4 wsum[kSageThreads / 32][32];
    const int wp = (int)warp_id();
    const float4* kp = reinterpret_cast<const float4*>(kpart + (long)hk * npg * 128) + lane_id();
    float4 a = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    int i = wp;
    for (; i + 24 < npg; i += 32) {
      float4 t[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) t[u] = kp[(long)(i + 8 * u) * 32];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        a.x += t[u].x; a.y += t[u].y; a.z += t[u].z; a.w += t[u].w;
      }
    }
    for (; i < npg; i += 8) {
      const float4 t = kp[(long)i * 32];
      a.x += t.x; a.y += t.y; a.z += t.z; a.w += t.w;
    }
    wsum[wp][lane_id()] = a;
    __syncthreads();
    if (tid < 128) {
      const float* ws = reinterpret_cast<const float*>(&wsum[0][0]);
      float t = 0.0f;
#pragma unroll
      for (int u = 0; u < kSageThreads / 32; ++u) t += ws[u * 128 + tid];
      km[tid] = t / (float)tk;
    }
  }
  __syncthreads();
  // rows r0 + 16 i: i = 0, 1 are the page's first 32-key block, i = 2, 3 its second
  const int c8 = tid & 15, r0 = pg * 64 + (tid >> 4);
  float v[4][8];
  float m[2] = {0.0f, 0.0f};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = r0 + 16 * i;
    if (r < tk) {   // every row of the page is written; rows past tk as zeros
      load8_bf(kv_row(kv, kv.k, hk, r) + c8 * 8, v[i]);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        v[i][k] -= km[c8 * 8 + k];
        m[i >> 1] = fmaxf(m[i >> 1], fabsf(v[i][k]));
      }
    } else {
#pragma unroll
      for (int k = 0; k < 8; ++k) v[i][k] = 0.0f;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    m[0] = fmaxf(m[0], __shfl_xor_sync(0xffffffffu, m[0], o));
    m[1] = fmaxf(m[1], __shfl_xor_sync(0xffffffffu, m[1], o));
  }
  if (lane_id() == 0) {
    red[0][warp_id()] = m[0];
    red[1][warp_id()] = m[1];
  }
  __syncthreads();
  float amax[2] = {0.0f, 0.0f};
#pragma unroll
  for (int i = 0; i < kSageThreads / 32; ++i) {
    amax[0] = fmaxf(amax[0], red[0][i]);
    amax[1] = fmaxf(amax[1], red[1][i]);
  }
  const float s[2] = {__fdiv_rn(amax[0], 127.0f), __fdiv_rn(amax[1], 127.0f)};
  if (tid < 2) sk[(long)hk * 2 * npg + 2 * pg + tid] = s[tid];
  const float rc[2] = {quant_recip(s[0]), quant_recip(s[1])};
  int8_t* out = k8 + (long)hk * k8_stride * 128;
#pragma unroll
  for (int i = 0; i < 4; ++i)
    *reinterpret_cast<uint2*>(out + (long)(r0 + 16 * i) * 128 + c8 * 8) =
        quant8(v[i], s[i >> 1], rc[i >> 1]);
}

}  // namespace

int attention(const AttnArgs& a, cudaStream_t st, std::string* err)
{
  if (a.hq <= 0 || a.hkv <= 0 || a.hq % a.hkv != 0) {
    *err = "attention: hq must be a positive multiple of hkv";
    return 1;
  }
  const int G = a.hq / a.hkv;
  if (G > 8 || (kRows % G) != 0) {
    *err = "attention: GQA group size must divide 128 and be at most 8";
    return 1;
  }
  if (a.tq <= 0 || a.tk <= 0) return 0;
  if (a.mode == 2 && a.t_index == nullptr) {
    *err = "attention: block-causal needs the t-index vector";
    return 1;
  }
  const bool sage = a.q8 != nullptr;
  if (sage && a.mode != 0) {
    *err = "attention: the int8-QK path serves the bidirectional pass only";
    return 1;
  }
  AttnP p{};
  p.q = static_cast<const __nv_bfloat16*>(a.q);
  p.kv = a.kv;
  p.out = static_cast<__nv_bfloat16*>(a.out);
  p.hq = a.hq;
  p.hkv = a.hkv;
  p.tq = a.tq;
  p.tk = a.tk;
  p.mode = a.mode;
  p.q_offset = a.q_offset;
  p.G = G;
  p.R = kRows / G;
  p.t_index = a.t_index;
  p.scale_log2 = (float)(1.4426950408889634 / std::sqrt(128.0));
  p.q8 = a.q8;
  p.k8 = a.k8;
  p.sq = a.sq;
  p.sk = a.sk;
  p.nqb = (a.tq + 63) / 64;
  p.nkb = 2 * ((a.tk + 63) / 64);   // 32-key K blocks, two per page
  p.k8_stride = (long)p.nkb * 32;
  const dim3 grid((a.tq + p.R - 1) / p.R, a.hkv);
  const int smem = sage ? (kRows * 128 + 2 * kKeys * 128 + 2 * kKeys * 256)
                        : (kRows * 256 + 2 * kKeys * 256 + 2 * kKeys * 256);
  static std::atomic<uint64_t> attr_done[4];
  auto launch = [&](auto kern, int which) {
    if (smem_attr_once(kern, smem, attr_done[which])) kern<<<grid, kThreads, smem, st>>>(p);
  };
  if (sage)
    a.kv.v_t ? launch(attn_kernel<true, true>, 3) : launch(attn_kernel<true, false>, 2);
  else
    a.kv.v_t ? launch(attn_kernel<false, true>, 1) : launch(attn_kernel<false, false>, 0);
  if (cudaGetLastError() != cudaSuccess) {
    *err = "attention: kernel launch failed";
    return 2;
  }
  return 0;
}

int sage_prepare(const void* q, const KvView& kv, int hq, int hkv, int tq, int tk, int8_t* q8,
                 int8_t* k8, float* sq, float* sk, float* kmean, cudaStream_t st,
                 std::string* err)
{
  if (hq <= 0 || hkv <= 0 || hq % hkv != 0) {
    *err = "sage_prepare: hq must be a positive multiple of hkv";
    return 1;
  }
  if (tq <= 0 || tk <= 0) return 0;
  const int nqb = (tq + 63) / 64, npg = (tk + 63) / 64;
  // kmean holds the per-page partial sums [hkv][npg][128]; sk two 32-key
  // block scales per page [hkv][2 * npg]
  // Q CTAs, then the K-mean page CTAs packed over the grid's hq rows
  const int nqc = (nqb + kSageQBlocks - 1) / kSageQBlocks;
  const int nkc = (hkv * npg + hq - 1) / hq;
  cudaError_t e = launch_pdl(sage_q_kernel, dim3(nqc + nkc, hq), dim3(kSageThreads), st,
                             static_cast<const __nv_bfloat16*>(q), kv, hq, hkv, tq, tk, nqb,
                             npg, q8, sq, kmean);
  if (e == cudaSuccess)
    e = launch_pdl(sage_k_kernel, dim3(npg, hkv), dim3(kSageThreads), st, kv, tk, npg,
                   static_cast<const float*>(kmean), k8, sk, (long)npg * 64);
  if (e != cudaSuccess || cudaGetLastError() != cudaSuccess) {
    *err = "sage_prepare: kernel launch failed";
    return 2;
  }
  return 0;
}

}  // namespace u15
