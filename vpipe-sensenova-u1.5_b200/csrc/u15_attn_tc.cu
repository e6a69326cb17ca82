// Flash attention on sm_100a tensor cores (tcgen05 + TMEM + TMA): the
// denoise pass's bidirectional attention (src/u15-metal-ops.cc:835-882 in
// the reference: q head-major, every key of [prefix || block]) and the
// prefill's masked rules (src/u15-metal-ops.cc:648-677, 884-908;
// src/u15-kernels.metal:186-252), over the paged cache.
//
// One CTA = 256 query rows of one head as two 128-row tiles sharing every
// K/V block it loads; keys in blocks of 128 (two 64-token pages of the
// paged cache). One query row per softmax thread, P kept in TMEM (written
// over its own S, read by the P.V MMA as the A operand), and the two tiles
// in ping-pong: while the softmax warps of one tile work, the tensor core
// runs the other tile's P.V and next S.
//
//   warp 0      TMA producer: Q once; per block j two K pages (four
//               [64 keys][64 dims] boxes) and two transposed V pages
//               ([128 dims][64 keys] each) into a 2-stage ring
//   warp 1      MMA issuer, per block j and tile t (in this order):
//                 wait P_t(j);  O_t += P_t(j) V_j   (A from TMEM)
//                 S_t(j+1) = Q_t K_{j+1}^T          (overwrites P_t(j); the
//                                                     MMAs run in issue order)
//                 commit -> s_full[t]
//               so s_full[t] completing means S_t(j+1) is ready AND every
//               earlier P.V of the tile has finished: the softmax may
//               rescale O_t and overwrite the S columns with P without
//               another wait.
//               (with the key-split softmax: warp 1 + t issues tile t's
//               MMAs alone, the same sequence)
//   warps 2-3   idle (they complete the first warpgroup; warp 2 is tile 1's
//               issuer in the key-split form)
//   warps 4-11  softmax, four warps per tile, one row per thread: the whole
//               128-score row in registers, base-2 online softmax with lazy
//               rescale (O is rescaled only when a row max grows by more
//               than 2^8), P as bf16 pairs into TMEM, final O / l to global
//               token-major [tq][hq*128]. The block-causal rule takes the
//               key-split form instead: the eight warps serve both tiles in
//               turn, two warps per lane quadrant, lanes l and l + 16 holding
//               keys [0, 64) and [64, 128) of one row (TMEM shape 16x32bx2),
//               which halves the per-thread mask tests and exponentials of
//               that rule (0.118 -> 0.103 ms at BASELINE config 4's prefill;
//               0.317 -> 0.325 ms bidirectional, so that pass keeps the
//               one-row form)
// TMEM (512 columns): tile t at t*256: S_t / P_t [0,128) | O_t [128,256).
//
// The exponentials stay on the MUFU unit: moving a quarter or half of them
// to the FMA pipe (a fitted polynomial on the fraction plus an exponent-field
// add) measured 4 % and 12 % slower on B200 -- the softmax is bound by its
// dependency latency, not by the MUFU's throughput -- so the row max and
// row sum are split into independent chains instead.
//
// The Sage variant (int8 QK, SageAttention) feeds S from int8 Q and smoothed
// int8 K (kind::i8, s32 accumulators) and scales the scores by the per-64-row
// Q block and per-32-key K block scales (the reference's bq 64 / bk 32, so a
// 128-key block carries four K scales, one per 32-column chunk of a score
// row); P.V stays bf16.
//
// Masked rules (MODE 1 causal: key j visible to query row i iff
// j <= q_offset + i; MODE 2 block-causal: iff j <= q_offset + i or
// t[j] == t[q_offset + i], t the caller's int32 t-index vector). Each tile
// runs only the key blocks up to its last visible one (n_t blocks; the
// CTA's producer loads max(n_0, n_1)), and per (tile, block) a uniform test
// says whether every pair is visible -- the block lies wholly at or below
// the tile's first row, or (block-causal) the tile's rows and the block's
// keys all carry one t value -- in which case the softmax runs as in the
// bidirectional pass; only the other blocks test the rule per element. For
// the block-causal rule a prologue forms each key block's t range
// (min, max) in shared memory and each tile's last block: a block can hold
// a key visible to row i only if it starts at or below i or its t range
// holds t[i].
//
// K/V come from the paged cache: K page [64 tokens][128] and V page
// transposed [128 dims][64 tokens], per kv head, page index from the page
// table. Every wait is bounded (u15_common.cuh).
#include "u15_common.cuh"
#include "u15_kernels.h"

#include <algorithm>
#include <climits>
#include <cmath>
#include <cstdlib>

namespace u15 {

namespace {

constexpr int kTile = 128;
constexpr int kBlk = 128;                       // keys per block: two pages
constexpr int kStages = 2;
// Three warpgroups: WG0 = producer, MMA issuer and two idle warps; WG1 and
// WG2 = the softmax of tile 0 and tile 1. Launched at 168 registers a thread
// (the most 12 warps fit: three warps share each quarter of the register
// file), WG0 then gives registers back (setmaxnreg.dec to 72) and the
// softmax warpgroups take them (setmaxnreg.inc to 216) so a whole 128-score
// row stays in registers: 128 x 72 + 256 x 216 = 384 x 168, the launch's
// total, which the increase may not exceed.
constexpr int kThreads = 384;
constexpr int kRegsLow = 72, kRegsHigh = 216;
constexpr int kQBytes = 2 * kTile * 256;        // bf16 Q, 2 tiles; int8 uses half
constexpr int kKBytes = kBlk * 256;             // [2 dims blocks][128 keys][128 B]
constexpr int kVBytes = 128 * kBlk * 2;         // [2 key blocks][128 dims][128 B]
// block-causal: per key block the t range (min, max); tk <= kMaxBlk * 128
constexpr int kMaxBlk = 256;
// the exponential form a launch takes unless U15_ATTN_EXP says otherwise
constexpr int kDefaultExp = 0;

constexpr int kSmem = kQBytes + kStages * (kKBytes + kVBytes) + 1024 + 256 + 2 * kMaxBlk * 4 + 64;

struct TcAttnP {
  int hq, hkv, tq, tk, G;
  int q_offset;
  const int32_t* t_index;   // block-causal: [tk], 16-byte aligned
  float scale_log2;
  const int32_t* page_table;
  __nv_bfloat16* out;
  const float* sq;   // Sage: [hq][nqb]
  const float* sk;   // Sage: [hkv][nkb], one scale per 32-key block
  int nqb, nkb;
  long k8_stride;    // Sage: rows per kv head in the int8 K copy
  unsigned* err;
  int issuers;       // MMA issuing warps: 1 (warp 1, both tiles) or 2 (warp 1 + t, tile t)
  int release;       // 1: the softmax warps release K/V stages (bidirectional, one issuer)
  int unit_base;     // bidirectional: the first unit (two-tile: 256-row block of a head;
                     // one-tile: 128-row block) of this launch's 1-D grid
};

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32])
{
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// max(a, b, c) in one instruction (the three-input max.f32 of sm_100)
__device__ __forceinline__ float fmax3(float a, float b, float c)
{
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// 2^x on the MUFU unit (PTX ex2.approx.ftz.f32; relative error ~2^-22,
// far below the bf16 rounding P receives).
__device__ __forceinline__ float ex2(float x)
{
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16])
{
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15])
      : "memory");
}

// 64 32-bit columns per thread in the 16x32bx2 shape: threads 0-15 read
// lanes taddr.lane + (0..15) at columns [c, c + 64), threads 16-31 the same
// lanes at [c + OFF, c + OFF + 64)
template <int OFF>
__device__ __forceinline__ void tmem_ld_pair64(uint32_t taddr, uint32_t (&r)[64])
{
  asm volatile(
      "tcgen05.ld.sync.aligned.16x32bx2.x64.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32,%33,%34,%35,"
      "%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,"
      "%58,%59,%60,%61,%62,%63}, [%64], %65;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]), "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]), "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]), "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]), "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
      : "r"(taddr), "n"(OFF)
      : "memory");
}

// the store of the same shape: threads 0-15 write columns [c, c + 16),
// threads 16-31 [c + OFF, c + OFF + 16) of the same 16 lanes
template <int OFF>
__device__ __forceinline__ void tmem_st_pair16(uint32_t taddr, const uint32_t (&r)[16])
{
  asm volatile(
      "tcgen05.st.sync.aligned.16x32bx2.x16.b32 [%0], %17, {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,"
      "%12,%13,%14,%15,%16};"
      :: "r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "n"(OFF)
      : "memory");
}

// 32 32-bit columns per thread in the 16x32bx2 shape: threads 0-15 read
// lanes taddr.lane + (0..15) at columns [c, c + 32), threads 16-31 the same
// lanes at [c + OFF, c + OFF + 32)
template <int OFF>
__device__ __forceinline__ void tmem_ld_pair32(uint32_t taddr, uint32_t (&r)[32])
{
  asm volatile(
      "tcgen05.ld.sync.aligned.16x32bx2.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32], %33;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr), "n"(OFF)
      : "memory");
}

// the store of the same shape: threads 0-15 write columns [c, c + 32),
// threads 16-31 [c + OFF, c + OFF + 32) of the same 16 lanes
template <int OFF>
__device__ __forceinline__ void tmem_st_pair32(uint32_t taddr, const uint32_t (&r)[32])
{
  asm volatile(
      "tcgen05.st.sync.aligned.16x32bx2.x32.b32 [%0], %33, {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,"
      "%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
      :: "r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31]), "n"(OFF)
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem desc]^T, kind::f16: A is M=128 lanes x K
// bf16 packed two per 32-bit column.
__device__ __forceinline__ void mma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc,
                                            uint32_t idesc, uint32_t accumulate)
{
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 2^x for x <= 2^7 on the FMA pipe: x = n + f with n = rint(x) taken from
// the low mantissa bits of x + 1.5 * 2^23, f in [-0.5, 0.5]; 2^f by a degree-3
// polynomial fitted to minimise the relative error on that interval (max
// relative error 7.5e-5, below the bf16 rounding P receives); 2^n added to
// the exponent field. Inputs below -125 are clamped there (2^-125, a
// normal float) so the exponent never underflows; masked scores (-inf) give
// 2^-125 instead of 0, which no bf16 output can show.
__device__ __forceinline__ float ex2_fma(float x)
{
  x = fmaxf(x, -125.0f);
  const float t = x + 12582912.0f;
  const float f = x - (t - 12582912.0f);
  float q = fmaf(0.05517132207751274f, f, 0.24261054396629333f);
  q = fmaf(q, f, 0.6932609677314758f);
  q = fmaf(q, f, 0.9999281167984009f);
  return __int_as_float(__float_as_int(q) + (__float_as_int(t) << 23));
}

// Per-tile key-block schedule of the masked rules, shared by every warp
// (see the file comment): n[t] blocks for tile t, and for block-causal the
// tile's t range and each key block's t range.
struct MaskPlan {
  int n[2];
  int tlo[2], thi[2];
};

// The softmax in the key-split layout. Warp w of 4..11 serves rows
// 32 * (w & 3) + 16 * ((w - 4) >> 2) + (0..15) of BOTH tiles, the tiles in
// turn (tile 0 of block j, tile 1 of block j, tile 0 of block j + 1, ...);
// it reads them through the 16x32bx2 TMEM shape, so lane l < 16 holds keys
// [0, 64) of its row and lane l + 16 keys [64, 128) of the same row. Two
// warps share each lane quadrant: every warp exponentiates 64 scores a row
// instead of 128, and the two keep the SM sub-partition's MUFU busy where a
// single warp issuing 128 dependent-chain exponentials could not. The row
// max takes one shuffle between the two lanes of a row; the row sum stays
// split until the end. P lands where the one-row-per-thread layout puts it
// (key k of the block at bf16 column k of the tile's S columns), so the
// MMA issuer is unchanged.
template <bool SAGE, int EXPM, int MODE>
__device__ __forceinline__ void softmax_key_split(const TcAttnP& p, const MaskPlan* plan,
                                                  const int* blk_tlo, const int* blk_thi,
                                                  uint32_t tmem, uint32_t s_full, uint32_t p_full,
                                                  int h, int hk, int q0, int n_t0, int n_t1)
{
  const int w = (int)warp_id();
  const int q4 = w & 3, hf = (w - 4) >> 2;
  const int kh = (int)lane_id() >> 4;   // key half of the block this lane holds
  const int kb0 = 64 * kh;
  const int row = q4 * 32 + hf * 16 + ((int)lane_id() & 15);
  const uint32_t lane_off = (uint32_t)(q4 * 32 + hf * 16) << 16;
  const int nt[2] = {n_t0, n_t1};
  const int n = max(n_t0, n_t1);
  float m_ref[2] = {-INFINITY, -INFINITY}, l[2] = {0.0f, 0.0f};
  float sqv[2] = {1.0f, 1.0f};
  int qi[2], gi[2], g_first[2], ti[2] = {0, 0};
  bool t_uniform[2] = {false, false};
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    qi[t] = q0 + t * kTile + row;
    gi[t] = p.q_offset + qi[t];
    g_first[t] = p.q_offset + q0 + t * kTile;
    if constexpr (SAGE) sqv[t] = (qi[t] < p.tq) ? p.sq[(long)h * p.nqb + qi[t] / 64] : 0.0f;
    if constexpr (MODE == 2) {
      ti[t] = qi[t] < p.tq ? p.t_index[gi[t]] : 0;
      t_uniform[t] = plan->tlo[t] == plan->thi[t];
    }
  }
  const int kb_last = (p.tk - 1) >> 5;
  bool ok = true;
  for (int j = 0; j < n && ok; ++j) {
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      if (j >= nt[t]) continue;
      // warp-uniform: the TMEM loads and stores below are warp-collective
      if (!__all_sync(0xffffffffu, mbar_wait(s_full + 8 * t, j & 1, p.err, kDevWaitAccFull))) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t tS = tmem + t * 256 + lane_off;
      const uint32_t tO = tS + 128;
      uint32_t r[64];
      tmem_ld_pair64<64>(tS, r);
      tmem_ld_wait();
      // base-2 scale of this lane's two 32-key chunks (Sage: the Q block's and
      // the chunk's K block's scales; never zero, so -inf stays -inf)
      float f[2];
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        f[c] = p.scale_log2;
        if constexpr (SAGE)
          f[c] = fmaxf(f[c] * sqv[t] * p.sk[(long)hk * p.nkb + min(4 * j + 2 * kh + c, kb_last)],
                       1e-30f);
      }
      float s[64];
#pragma unroll
      for (int i = 0; i < 64; ++i) {
        if constexpr (SAGE) s[i] = __int_as_float((int)r[i] + 0x4B400000) - 12582912.0f;
        else s[i] = __uint_as_float(r[i]);
      }
      const int j0 = j * kBlk;
      const int kmax = p.tk - j0;
      if constexpr (MODE == 0) {
        if (kmax < kBlk) {
#pragma unroll
          for (int i = 0; i < 64; ++i)
            if (kb0 + i >= kmax) s[i] = -INFINITY;
        }
      } else {
        bool full = kmax >= kBlk && j0 + kBlk - 1 <= g_first[t];
        if constexpr (MODE == 2)
          full = full || (kmax >= kBlk && t_uniform[t] && blk_tlo[j] == blk_thi[j] &&
                          blk_tlo[j] == plan->tlo[t]);
        if (!full) {
          if constexpr (MODE == 1) {
            const int lim = min(kmax - 1, gi[t] - j0);   // visible keys [0, lim] of the block
#pragma unroll
            for (int i = 0; i < 64; ++i)
              if (kb0 + i > lim) s[i] = -INFINITY;
          } else {
            const int lim = gi[t] - j0;
            const int4* t4 = reinterpret_cast<const int4*>(p.t_index + j0 + kb0);
#pragma unroll
            for (int qd = 0; qd < 16; ++qd) {
              int tt[4];
              if (kb0 + 4 * qd + 3 < kmax) {
                const int4 v = __ldg(t4 + qd);
                tt[0] = v.x; tt[1] = v.y; tt[2] = v.z; tt[3] = v.w;
              } else {
#pragma unroll
                for (int e = 0; e < 4; ++e)
                  tt[e] = kb0 + 4 * qd + e < kmax ? p.t_index[j0 + kb0 + 4 * qd + e] : 0;
              }
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const int i = kb0 + 4 * qd + e;
                const bool vis = i < kmax && (i <= lim || tt[e] == ti[t]);
                if (!vis) s[4 * qd + e] = -INFINITY;
              }
            }
          }
        }
      }
      // row max: this lane's two chunks in two chains each, then the partner lane
      float mc[2][2];
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        mc[c][0] = s[32 * c];
        mc[c][1] = s[32 * c + 1];
      }
#pragma unroll
      for (int i = 2; i < 32; i += 2) {
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          mc[c][0] = fmaxf(mc[c][0], s[32 * c + i]);
          mc[c][1] = fmaxf(mc[c][1], s[32 * c + i + 1]);
        }
      }
      float mt = fmaxf(fmaxf(mc[0][0], mc[0][1]) * f[0], fmaxf(mc[1][0], mc[1][1]) * f[1]);
      mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 16));
      const bool need = (m_ref[t] == -INFINITY) || (mt > m_ref[t] + 8.0f);
      const float m_new = need ? fmaxf(mt, m_ref[t]) : m_ref[t];
      if (j > 0 && __any_sync(0xffffffffu, need)) {
        // O_t is final up to P.V(j-1): s_full[t] completed after it. Lane
        // l < 16 rescales dims [0, 64) of its row, lane l + 16 dims [64, 128)
        const float fac = (need && m_ref[t] != -INFINITY) ? ex2(m_ref[t] - m_new) : 1.0f;
#pragma unroll 1
        for (int c = 0; c < 2; ++c) {
          uint32_t o[32];
          tmem_ld_pair32<64>(tO + c * 32, o);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * fac);
          tmem_st_pair32<64>(tO + c * 32, o);
        }
        l[t] *= fac;
      }
      m_ref[t] = m_new;
      const float nm = m_ref[t] == -INFINITY ? 0.0f : -m_ref[t];
      float rs[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const float fc = f[c];
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float x0 = fmaf(s[32 * c + 2 * i], fc, nm), x1 = fmaf(s[32 * c + 2 * i + 1], fc, nm);
          const bool fma_pipe = EXPM == 1 && (i & 3) == 3;
          const float a = fma_pipe ? ex2_fma(x0) : ex2(x0);
          const float b = fma_pipe ? ex2_fma(x1) : ex2(x1);
          rs[i & 3] += a + b;
          pk[i] = pack_bf2(a, b);
        }
        // keys [kb0 + 32c, kb0 + 32c + 32) -> bf16 columns [kb0/2 + 16c, +16):
        // lanes < 16 write columns 16c.., lanes >= 16 columns 32 + 16c..
        tmem_st_pair16<32>(tS + 16 * c, pk);
      }
      tmem_st_wait();
      l[t] += (rs[0] + rs[1]) + (rs[2] + rs[3]);
      tc_fence_before();
      __syncwarp();
      if (lane_id() == 0) mbar_arrive(p_full + 8 * t);
    }
  }
  // the commit after each tile's last P.V, then O / l of this lane's 64 dims
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    const bool fin = ok && nt[t] > 0 &&
                     mbar_wait(s_full + 8 * t, nt[t] & 1, p.err, kDevWaitAccFull);
    if (!__all_sync(0xffffffffu, fin)) continue;
    tc_fence_after();
    const float lt = l[t] + __shfl_xor_sync(0xffffffffu, l[t], 16);
    const float inv = lt > 0.0f ? 1.0f / lt : 0.0f;
    const uint32_t tO = tmem + t * 256 + lane_off + 128;
    __nv_bfloat16* dst = p.out + (long)qi[t] * p.hq * 128 + (long)h * 128 + kb0;
#pragma unroll 1
    for (int c = 0; c < 2; ++c) {
      uint32_t o[32];
      tmem_ld_pair32<64>(tO + c * 32, o);
      tmem_ld_wait();
      if (qi[t] < p.tq) {
        uint4* d4 = reinterpret_cast<uint4*>(dst + c * 32);
#pragma unroll
        for (int qd = 0; qd < 4; ++qd) {
          uint4 v;
          v.x = pack_bf2(__uint_as_float(o[qd * 8 + 0]) * inv, __uint_as_float(o[qd * 8 + 1]) * inv);
          v.y = pack_bf2(__uint_as_float(o[qd * 8 + 2]) * inv, __uint_as_float(o[qd * 8 + 3]) * inv);
          v.z = pack_bf2(__uint_as_float(o[qd * 8 + 4]) * inv, __uint_as_float(o[qd * 8 + 5]) * inv);
          v.w = pack_bf2(__uint_as_float(o[qd * 8 + 6]) * inv, __uint_as_float(o[qd * 8 + 7]) * inv);
          d4[qd] = v;
        }
      }
    }
  }
}

template <bool SAGE, int EXPM, int MODE, bool KS>
__global__ void __launch_bounds__(kThreads, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                const __grid_constant__ CUtensorMap tmV, const __grid_constant__ TcAttnP p)
{
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + kQBytes;
  uint8_t* sV = sK + kStages * kKBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + kStages * kVBytes);
  const uint32_t b0 = smem_u32(bars);
  const uint32_t q_full = b0;
  const uint32_t k_full = b0 + 8;                 // [kStages]
  const uint32_t v_full = k_full + 8 * kStages;
  const uint32_t k_empty = v_full + 8 * kStages;
  const uint32_t v_empty = k_empty + 8 * kStages;
  const uint32_t s_full = v_empty + 8 * kStages;  // [2 tiles]
  const uint32_t p_full = s_full + 16;            // [2 tiles], 128 arrivals
  const uint32_t drain = p_full + 16;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 1 + 4 * kStages + 2 + 2 + 1);
  MaskPlan* plan = reinterpret_cast<MaskPlan*>(bars + 32);
  int* blk_tlo = reinterpret_cast<int*>(bars + 40);   // [kMaxBlk] (block-causal)
  int* blk_thi = blk_tlo + kMaxBlk;

  const int w = (int)warp_id();
  // bidirectional: a 1-D grid of units u = head * (query blocks) + block
  // from p.unit_base, the query blocks of a head side by side (they share
  // its K/V in L2); masked rules: grid (heads, query blocks) with the last
  // query block first -- the longest CTAs start first, so the short ones
  // fill the tail
  const int nqb2 = (p.tq + 2 * kTile - 1) / (2 * kTile);
  const int u0 = (int)blockIdx.x + p.unit_base;
  const int h = MODE == 0 ? u0 / nqb2 : (int)blockIdx.x;
  const int qb = MODE == 0 ? u0 % nqb2 : (int)(gridDim.y - 1 - blockIdx.y);
  const int hk = h / p.G;
  const int q0 = qb * 2 * kTile;
  const int n_all = (p.tk + kBlk - 1) / kBlk;
  const int n_pg = (p.tk + 63) / 64;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(k_full + 8 * s, 1);
      mbar_init(v_full + 8 * s, 1);
      // a K / V stage is free once every issuing warp's MMAs that read it are
      // done; in the release form, once each active tile's softmax has seen
      // the S-ready commit that follows them
      const int act = (q0 < p.tq) + (q0 + kTile < p.tq);
      mbar_init(k_empty + 8 * s, p.release ? act : p.issuers);
      mbar_init(v_empty + 8 * s, p.release ? act : p.issuers);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(s_full + 8 * t, 1);
      // P_t ready: one arrival per softmax thread of the tile, or (key-split
      // layout) one per softmax warp, every warp serving both tiles
      mbar_init(p_full + 8 * t, KS ? 8 : 128);
      // blocks of tile t: none when the tile holds no query row; the causal
      // rule ends at the block of the tile's last row
      const int r_lo = q0 + t * kTile, r_hi = min(r_lo + kTile, p.tq) - 1;
      int nt = r_lo < p.tq ? n_all : 0;
      if (MODE == 1 && nt > 0) nt = min(n_all, (p.q_offset + r_hi) / kBlk + 1);
      plan->n[t] = MODE == 2 ? 0 : nt;
      plan->tlo[t] = INT_MAX;
      plan->thi[t] = INT_MIN;
    }
    mbar_init(drain, p.issuers);
    fence_barrier_init();
  }
  if (w == 0) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  if (threadIdx.x == 32) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // the set-up above overlaps the previous kernel; global memory waits for it
  griddep_launch();
  griddep_wait();
  if constexpr (MODE == 2) {
    // t range of every key block (each warp a block at a time, 4 keys a lane)
    for (int kb = w; kb < n_all; kb += kThreads / 32) {
      int lo = INT_MAX, hi = INT_MIN;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int j = kb * kBlk + q * 32 + (int)lane_id();
        if (j < p.tk) {
          const int tj = p.t_index[j];
          lo = min(lo, tj);
          hi = max(hi, tj);
        }
      }
      lo = __reduce_min_sync(0xffffffffu, lo);
      hi = __reduce_max_sync(0xffffffffu, hi);
      if (lane_id() == 0) {
        blk_tlo[kb] = lo;
        blk_thi[kb] = hi;
      }
    }
    __syncthreads();
    if (w >= 4) {
      // each softmax thread's row: its last block that can hold a visible key
      const int t = (w - 4) >> 2;
      const int qi = q0 + t * kTile + (w & 3) * 32 + (int)lane_id();
      int last = -1, ti = 0;
      if (qi < p.tq) {
        const int gi = p.q_offset + qi;
        ti = p.t_index[gi];
        last = min(gi / kBlk, n_all - 1);
        for (int kb = n_all - 1; kb > last; --kb)
          if (blk_tlo[kb] <= ti && ti <= blk_thi[kb]) {
            last = kb;
            break;
          }
      }
      const bool valid = qi < p.tq;
      last = __reduce_max_sync(0xffffffffu, last);
      const int lo = __reduce_min_sync(0xffffffffu, valid ? ti : INT_MAX);
      const int hi = __reduce_max_sync(0xffffffffu, valid ? ti : INT_MIN);
      if (lane_id() == 0) {
        atomicMax(&plan->n[t], last + 1);
        atomicMin(&plan->tlo[t], lo);
        atomicMax(&plan->thi[t], hi);
      }
    }
    __syncthreads();
  }
  const int n_t0 = plan->n[0], n_t1 = plan->n[1];
  const int n = max(n_t0, n_t1);   // blocks the producer loads
  if (w < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsLow));
    if (w == 0) {
      // ------------------------------------------------------------ producer
      if (lane_id() == 0) {
        const int qrow = h * p.tq + q0;
        if constexpr (SAGE) {
          mbar_arrive_expect_tx(q_full, 2 * kTile * 128);
          for (int t = 0; t < 2; ++t)
            tma_load_2d(smem_u32(sQ + t * kTile * 128), &tmQ, 0, qrow + t * kTile, q_full);
        } else {
          mbar_arrive_expect_tx(q_full, 2 * kTile * 256);
          for (int t = 0; t < 2; ++t)
            for (int d = 0; d < 2; ++d)
              tma_load_2d(smem_u32(sQ + t * kTile * 256 + d * kTile * 128), &tmQ, d * 64,
                          qrow + t * kTile, q_full);
        }
        int nk = 0, nv = 0;   // blocks whose K / V loads were issued
        for (int j = 0; j < n; ++j) {
          const int s = j % kStages;
          const uint32_t ph = (j / kStages) & 1;
          // the block's two pages; past the last page the first one is loaded
          // again (finite data under masked scores)
          const int pg0 = 2 * j, pg1 = min(2 * j + 1, n_pg - 1);
          const int page0 = p.page_table ? p.page_table[pg0] : pg0;
          const int page1 = p.page_table ? p.page_table[pg1] : pg1;
          if (!mbar_wait(k_empty + 8 * s, ph ^ 1, p.err, kDevWaitEmpty)) break;
          uint8_t* k_dst = sK + s * kKBytes;
          if constexpr (SAGE) {
            mbar_arrive_expect_tx(k_full + 8 * s, kBlk * 128);
            const int krow = (int)(hk * p.k8_stride) + j * kBlk;
            tma_load_2d(smem_u32(k_dst), &tmK, 0, krow, k_full + 8 * s);
            tma_load_2d(smem_u32(k_dst + 64 * 128), &tmK, 0, krow + 64, k_full + 8 * s);
          } else {
            mbar_arrive_expect_tx(k_full + 8 * s, kKBytes);
            for (int hf = 0; hf < 2; ++hf) {
              const int krow = ((hf ? page1 : page0) * p.hkv + hk) * 64;
              for (int d = 0; d < 2; ++d)
                tma_load_2d(smem_u32(k_dst + d * kBlk * 128 + hf * 64 * 128), &tmK, d * 64, krow,
                            k_full + 8 * s);
            }
          }
          nk = j + 1;
          if (!mbar_wait(v_empty + 8 * s, ph ^ 1, p.err, kDevWaitEmpty)) break;
          mbar_arrive_expect_tx(v_full + 8 * s, kVBytes);
          for (int hf = 0; hf < 2; ++hf)
            tma_load_2d(smem_u32(sV + s * kVBytes + hf * 128 * 128), &tmV, 0,
                        ((hf ? page1 : page0) * p.hkv + hk) * 128, v_full + 8 * s);
          nv = j + 1;
        }
        // unwinding: every copy issued must land before the CTA may exit
        mbar_wait(q_full, 0, p.err, kDevWaitDrain);
        for (int s = 0; s < kStages; ++s) {
          if (nk > s) {
            const int last = ((nk - 1 - s) / kStages) * kStages + s;
            mbar_wait(k_full + 8 * s, (last / kStages) & 1, p.err, kDevWaitDrain);
          }
          if (nv > s) {
            const int last = ((nv - 1 - s) / kStages) * kStages + s;
            mbar_wait(v_full + 8 * s, (last / kStages) & 1, p.err, kDevWaitDrain);
          }
        }
      }
    } else if ((w == 1 || w == 2) && p.issuers == 2) {
      // ------------------------------------------------------------ MMA, one warp a tile
      // Warp 1 + t issues tile t's MMAs (the key-split softmax's partner). A
      // single issuer's barrier operations after its MMAs return late (the
      // stage commits and the V and P waits between the two tiles took ~700
      // of every ~3900 cycles in a clock trace), and the key-split softmax
      // serves the tiles in turn, so the tiles' MMAs do not interleave: one
      // issuer a tile overlaps each tile's waits with the other's MMAs.
      if (lane_id() == 0) {
        const int t = w - 1;
        const int n_mine = t == 0 ? n_t0 : n_t1;
        const uint32_t id_s = SAGE ? idesc_s8(kTile, kBlk) : idesc_bf16(kTile, kBlk);
        const uint32_t id_o = idesc_bf16(kTile, 128);
        auto issue_s = [&](int j) {
          const uint32_t d = tmem + t * 256;
          const uint32_t kb = smem_u32(sK + (j % kStages) * kKBytes);
          if constexpr (SAGE) {
            const uint32_t a0 = smem_u32(sQ + t * kTile * 128);
  #pragma unroll
            for (int k = 0; k < 4; ++k)
              mma_i8(d, smem_desc_sw128(a0 + k * 32), smem_desc_sw128(kb + k * 32), id_s, k != 0);
          } else {
            const uint32_t a0 = smem_u32(sQ + t * kTile * 256);
  #pragma unroll
            for (int k = 0; k < 8; ++k)
              mma_bf16(d, smem_desc_sw128(a0 + (k >> 2) * kTile * 128 + (k & 3) * 32),
                       smem_desc_sw128(kb + (k >> 2) * kBlk * 128 + (k & 3) * 32), id_s, k != 0);
          }
        };
        bool ok = mbar_wait(q_full, 0, p.err, kDevWaitFull);
        if (ok && n > 0) {
          ok = mbar_wait(k_full, 0, p.err, kDevWaitFull);
          if (ok) {
            tc_fence_after();
            if (n_mine > 0) {
              issue_s(0);
              mma_commit(s_full + 8 * t);
            }
            mma_commit(k_empty);
          }
        }
        // Every block the producer loads is released by both issuers, each
        // only after that fill has landed (the V and next K waits below, also
        // where this tile has no MMA to issue): with two arrivals a phase, a
        // release issued before its fill landed could complete the previous
        // fill's phase alone, while the other tile still reads that fill.
        for (int j = 0; j < n && ok; ++j) {
          const int s = j % kStages, s1 = (j + 1) % kStages;
          const bool mine = j < n_mine;
          if (!mbar_wait_probe(v_full + 8 * s, (j / kStages) & 1, p.err, kDevWaitFull) ||
              (mine && !mbar_wait_probe(p_full + 8 * t, j & 1, p.err, kDevWaitFull))) {
            ok = false;
            break;
          }
          if (mine) {
            tc_fence_after();
            const uint32_t vb = smem_u32(sV + s * kVBytes);
            const uint32_t d = tmem + t * 256 + 128, a = tmem + t * 256;
  #pragma unroll
            for (int k = 0; k < 8; ++k)
              mma_bf16_ts(d, a + k * 8, smem_desc_sw128(vb + (k >> 2) * 128 * 128 + (k & 3) * 32),
                          id_o, (j | k) != 0);
          }
          if (j + 1 < n &&
              !mbar_wait_probe(k_full + 8 * s1, ((j + 1) / kStages) & 1, p.err, kDevWaitFull)) {
            ok = false;
            break;
          }
          if (mine) {
            if (j + 1 < n_mine) {
              tc_fence_after();
              issue_s(j + 1);
            }
            mma_commit(s_full + 8 * t);
          }
          mma_commit(v_empty + 8 * s);
          if (j + 1 < n) mma_commit(k_empty + 8 * s1);
        }
        mma_commit(drain);
        mbar_wait(drain, 0, p.err, kDevWaitDrain);
      }
    } else if (w == 1) {
      // ------------------------------------------------------------ MMA
      if (lane_id() == 0) {
        const uint32_t id_s = SAGE ? idesc_s8(kTile, kBlk) : idesc_bf16(kTile, kBlk);
        const uint32_t id_o = idesc_bf16(kTile, 128);
        const int nt[2] = {n_t0, n_t1};
        auto issue_s = [&](int t, int j) {
          const uint32_t d = tmem + t * 256;
          const uint32_t kb = smem_u32(sK + (j % kStages) * kKBytes);
          if constexpr (SAGE) {
            const uint32_t a0 = smem_u32(sQ + t * kTile * 128);
  #pragma unroll
            for (int k = 0; k < 4; ++k)
              mma_i8(d, smem_desc_sw128(a0 + k * 32), smem_desc_sw128(kb + k * 32), id_s, k != 0);
          } else {
            const uint32_t a0 = smem_u32(sQ + t * kTile * 256);
  #pragma unroll
            for (int k = 0; k < 8; ++k)
              mma_bf16(d, smem_desc_sw128(a0 + (k >> 2) * kTile * 128 + (k & 3) * 32),
                       smem_desc_sw128(kb + (k >> 2) * kBlk * 128 + (k & 3) * 32), id_s, k != 0);
          }
        };
        bool ok = mbar_wait(q_full, 0, p.err, kDevWaitFull);
        if (ok && n > 0) {
          ok = mbar_wait(k_full, 0, p.err, kDevWaitFull);
          if (ok) {
            tc_fence_after();
            for (int t = 0; t < 2; ++t) {
              if (nt[t] == 0) continue;
              issue_s(t, 0);
              mma_commit(s_full + 8 * t);
            }
            if (!p.release) mma_commit(k_empty);
          }
        }
        for (int j = 0; j < n && ok; ++j) {
          const int s = j % kStages, s1 = (j + 1) % kStages;
          if (!mbar_wait_probe(v_full + 8 * s, (j / kStages) & 1, p.err, kDevWaitFull)) break;
          const uint32_t vb = smem_u32(sV + s * kVBytes);
          bool k_next = false;   // K of block j + 1 has landed
          for (int t = 0; t < 2 && ok; ++t) {
            if (j >= nt[t]) continue;
            if (!mbar_wait_probe(p_full + 8 * t, j & 1, p.err, kDevWaitFull)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t d = tmem + t * 256 + 128, a = tmem + t * 256;
  #pragma unroll
            for (int k = 0; k < 8; ++k)
              mma_bf16_ts(d, a + k * 8, smem_desc_sw128(vb + (k >> 2) * 128 * 128 + (k & 3) * 32),
                          id_o, (j | k) != 0);
            if (j + 1 < nt[t]) {
              if (!k_next && !mbar_wait_probe(k_full + 8 * s1, ((j + 1) / kStages) & 1, p.err,
                                              kDevWaitFull)) {
                ok = false;
                break;
              }
              k_next = true;
              tc_fence_after();
              issue_s(t, j + 1);
            }
            mma_commit(s_full + 8 * t);
          }
          if (!ok) break;
          if (!p.release) {
            mma_commit(v_empty + 8 * s);
            // n = max(n_0, n_1): some tile ran block j + 1's S, so its K was waited for
            if (j + 1 < n) mma_commit(k_empty + 8 * s1);
          }
        }
        mma_commit(drain);
        mbar_wait(drain, 0, p.err, kDevWaitDrain);
      }
    }
  } else if constexpr (KS) {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegsHigh));
    softmax_key_split<SAGE, EXPM, MODE>(p, plan, blk_tlo, blk_thi, tmem, s_full, p_full, h, hk, q0,
                                        n_t0, n_t1);
    tc_fence_before();
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegsHigh));
    // ------------------------------------------------------------ softmax
    const int t = (w - 4) >> 2;
    const int wq = w & 3;
    const int row = wq * 32 + (int)lane_id();
    const int qi = q0 + t * kTile + row;
    const int n_mine = t == 0 ? n_t0 : n_t1;
    const uint32_t tS = tmem + t * 256 + ((uint32_t)(wq * 32) << 16);
    const uint32_t tO = tS + 128;
    float sqv = 1.0f;
    if constexpr (SAGE) sqv = (qi < p.tq) ? p.sq[(long)h * p.nqb + qi / 64] : 0.0f;
    // masked rules: this row's position among the keys, its t, and the
    // tile's first position (blocks wholly at or below it are visible)
    const int gi = p.q_offset + qi;
    const int g_first = p.q_offset + q0 + t * kTile;
    int ti = 0;
    bool t_uniform = false;
    if constexpr (MODE == 2) {
      ti = qi < p.tq ? p.t_index[gi] : 0;
      t_uniform = plan->tlo[t] == plan->thi[t];
    }
    // the last 32-key block that holds a key (Sage scales past it are clamped to it)
    const int kb_last = (p.tk - 1) >> 5;
    float m_ref = -INFINITY, l = 0.0f;
    bool ok = true;
    for (int j = 0; j < n_mine; ++j) {
      // warp-uniform: the TMEM loads and stores below are warp-collective
      if (!__all_sync(0xffffffffu, mbar_wait(s_full + 8 * t, j & 1, p.err, kDevWaitAccFull))) {
        ok = false;
        break;
      }
      // release form: the S-ready commit j follows S_t(j) (K block j read)
      // and P.V_t(j - 1) (V block j - 1 read)
      if (p.release && wq == 0 && lane_id() == 0) {
        mbar_arrive(k_empty + 8 * (j % kStages));
        if (j > 0) mbar_arrive(v_empty + 8 * ((j - 1) % kStages));
      }
      tc_fence_after();
      uint32_t r[128];
      tmem_ld32(tS + 0, *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
      tmem_ld32(tS + 32, *reinterpret_cast<uint32_t(*)[32]>(&r[32]));
      tmem_ld32(tS + 64, *reinterpret_cast<uint32_t(*)[32]>(&r[64]));
      tmem_ld32(tS + 96, *reinterpret_cast<uint32_t(*)[32]>(&r[96]));
      tmem_ld_wait();
      // base-2 scale of each 32-key chunk (Sage: the Q block's and the chunk's
      // K block's scales; never zero, so a masked -inf score stays -inf)
      float f[4];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        f[c] = p.scale_log2;
        if constexpr (SAGE)
          f[c] = fmaxf(f[c] * sqv * p.sk[(long)hk * p.nkb + min(4 * j + c, kb_last)], 1e-30f);
      }
      // Sage scores are int32 sums of 128 int8 x int8 products, |S| <=
      // 128 * 127 * 127 < 2^22: adding them to the bits of 1.5 * 2^23 gives
      // the float 1.5 * 2^23 + S exactly, and subtracting 1.5 * 2^23 leaves
      // S -- an integer add and a float add in place of a conversion.
      float s[128];
#pragma unroll
      for (int i = 0; i < 128; ++i) {
        if constexpr (SAGE) s[i] = __int_as_float((int)r[i] + 0x4B400000) - 12582912.0f;
        else s[i] = __uint_as_float(r[i]);
      }
      const int j0 = j * kBlk;
      const int kmax = p.tk - j0;
      if constexpr (MODE == 0) {
        if (kmax < kBlk) {
#pragma unroll
          for (int i = 0; i < 128; ++i)
            if (i >= kmax) s[i] = -INFINITY;
        }
      } else {
        // tile-uniform: is every (row, key) pair of this block visible?
        bool full = kmax >= kBlk && j0 + kBlk - 1 <= g_first;
        if constexpr (MODE == 2)
          full = full || (kmax >= kBlk && t_uniform && blk_tlo[j] == blk_thi[j] &&
                          blk_tlo[j] == plan->tlo[t]);
        if (!full) {
          if constexpr (MODE == 1) {
            const int lim = min(kmax - 1, gi - j0);   // visible columns [0, lim]
#pragma unroll
            for (int i = 0; i < 128; ++i)
              if (i > lim) s[i] = -INFINITY;
          } else {
            const int lim = gi - j0;
            const int4* t4 = reinterpret_cast<const int4*>(p.t_index + j0);
#pragma unroll
            for (int qd = 0; qd < 32; ++qd) {
              int tt[4];
              if (4 * qd + 3 < kmax) {
                const int4 v = __ldg(t4 + qd);
                tt[0] = v.x; tt[1] = v.y; tt[2] = v.z; tt[3] = v.w;
              } else {
#pragma unroll
                for (int e = 0; e < 4; ++e) tt[e] = 4 * qd + e < kmax ? p.t_index[j0 + 4 * qd + e] : 0;
              }
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const int i = 4 * qd + e;
                const bool vis = i < kmax && (i <= lim || tt[e] == ti);
                if (!vis) s[i] = -INFINITY;
              }
            }
          }
        }
      }
      // row maxima of the four 32-key chunks, two independent chains each
      // (one serial chain of 128 would put its latency on the critical path)
      // (three-input max: 15 instructions a chunk instead of 31)
      float mc[4][2];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        mc[c][0] = fmax3(s[32 * c], s[32 * c + 1], s[32 * c + 2]);
        mc[c][1] = fmax3(s[32 * c + 3], s[32 * c + 4], s[32 * c + 5]);
      }
#pragma unroll
      for (int i = 6; i < 32; i += 4) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          mc[c][0] = fmax3(mc[c][0], s[32 * c + i], s[32 * c + i + 1]);
          if (i + 3 < 32) mc[c][1] = fmax3(mc[c][1], s[32 * c + i + 2], s[32 * c + i + 3]);
        }
      }
      const float mt = fmaxf(fmaxf(fmaxf(mc[0][0], mc[0][1]) * f[0], fmaxf(mc[1][0], mc[1][1]) * f[1]),
                             fmaxf(fmaxf(mc[2][0], mc[2][1]) * f[2], fmaxf(mc[3][0], mc[3][1]) * f[3]));
      const bool need = (m_ref == -INFINITY) || (mt > m_ref + 8.0f);
      const float m_new = need ? fmaxf(mt, m_ref) : m_ref;
      if (j > 0 && __any_sync(0xffffffffu, need)) {
        // O_t is final up to P.V(j-1): s_full[t] completed after it
        const float fac = (need && m_ref != -INFINITY) ? ex2(m_ref - m_new) : 1.0f;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t o[32];
          tmem_ld32(tO + c * 32, o);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * fac);
          tmem_st32(tO + c * 32, o);
        }
        l *= fac;
      }
      m_ref = m_new;
      // a row with no visible key yet keeps m_ref = -inf: its exponentials are
      // of -inf scores and give 0 with a zero offset
      const float nm = m_ref == -INFINITY ? 0.0f : -m_ref;
      float rs[4] = {0.0f, 0.0f, 0.0f, 0.0f};   // four independent partial sums
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const float fc = f[c];
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float x0 = fmaf(s[32 * c + 2 * i], fc, nm), x1 = fmaf(s[32 * c + 2 * i + 1], fc, nm);
          // EXPM 1: every fourth pair on the FMA pipe, interleaved with the
          // MUFU ones (i is a constant after unrolling)
          const bool fma_pipe = EXPM == 1 && (i & 3) == 3;
          const float a = fma_pipe ? ex2_fma(x0) : ex2(x0);
          const float b = fma_pipe ? ex2_fma(x1) : ex2(x1);
          rs[i & 3] += a + b;
          pk[i] = pack_bf2(a, b);
        }
        // P chunk c -> columns [16c, 16c+16), whose scores were all read
        tmem_st16(tS + 16 * c, pk);
      }
      tmem_st_wait();
      l += (rs[0] + rs[1]) + (rs[2] + rs[3]);
      tc_fence_before();
      mbar_arrive(p_full + 8 * t);
    }
    // the commit after the last P.V of this tile
    const bool fin = ok && n_mine > 0 &&
                     mbar_wait(s_full + 8 * t, n_mine & 1, p.err, kDevWaitAccFull);
    if (p.release && fin && wq == 0 && lane_id() == 0)
      mbar_arrive(v_empty + 8 * ((n_mine - 1) % kStages));
    if (__all_sync(0xffffffffu, fin)) {
      tc_fence_after();
      const float inv = l > 0.0f ? 1.0f / l : 0.0f;
      __nv_bfloat16* dst = p.out + (long)qi * p.hq * 128 + (long)h * 128;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t o[32];
        tmem_ld32(tO + c * 32, o);
        tmem_ld_wait();
        if (qi < p.tq) {
          uint4* d4 = reinterpret_cast<uint4*>(dst + c * 32);
#pragma unroll
          for (int qd = 0; qd < 4; ++qd) {
            uint4 v;
            v.x = pack_bf2(__uint_as_float(o[qd * 8 + 0]) * inv, __uint_as_float(o[qd * 8 + 1]) * inv);
            v.y = pack_bf2(__uint_as_float(o[qd * 8 + 2]) * inv, __uint_as_float(o[qd * 8 + 3]) * inv);
            v.z = pack_bf2(__uint_as_float(o[qd * 8 + 4]) * inv, __uint_as_float(o[qd * 8 + 5]) * inv);
            v.w = pack_bf2(__uint_as_float(o[qd * 8 + 6]) * inv, __uint_as_float(o[qd * 8 + 7]) * inv);
            d4[qd] = v;
          }
        }
      }
    }
    tc_fence_before();
  }

  __syncthreads();
  if (w == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}


// ---------------------------------------------------------------------
// The bidirectional pass with ONE 128-row tile a CTA. It runs the
// part-empty last round of the two-tile kernel's units (a second launch,
// each unit as two of these CTAs), and the whole pass under
// U15_ATTN_TILES=1 (an A/B form, no faster than the two-tile kernel for the
// full rounds). TMEM holds kSBuf (2
// or 3, U15_ATTN_SBUF) S buffers of 128 columns (block j in buffer
// j % kSBuf, its P written over the buffer's first 64 columns) and O after
// them. The MMA issuer runs S(0) .. S(kSBuf - 1), then P.V(j) followed by
// S(j + kSBuf) into the buffer P.V(j) has just read, so the next blocks' S
// are ready while the softmax works on block j: the tile's chain per block
// is its softmax, with S and P.V on the tensor core beneath it. The
// softmax is the key-split layout (eight warps, two a lane quadrant, 64
// keys a lane). A lazy O rescale first waits for P.V(j - 1) (o_done: two
// slots, block parity; the slot's previous phase, P.V(j - 3), completed
// before S(j) ran). K and V in three stages (224 KB with Q). At 4096 x 32
// heads: 1024 CTAs, 6.92 rounds on 148 SMs (the two-tile kernel: 512, 3.46).
constexpr int kStages1 = 3;
constexpr int kQBytes1 = kTile * 256;   // bf16 Q, one tile; int8 uses half
// + 1024 for the base alignment, + 512 for the mbarriers (at most 23) and the TMEM slot
constexpr int kSmem1 = kQBytes1 + kStages1 * (kKBytes + kVBytes) + 1024 + 512;
static_assert(kSmem1 <= 232448, "one-tile attention: over the 227 KB shared-memory limit");

template <bool SAGE, int kSBuf>
__device__ __forceinline__ void softmax_single(const TcAttnP& p, uint32_t tmem, uint32_t s_full,
                                               uint32_t p_full, uint32_t o_done, uint32_t o_final,
                                               int h, int hk, int q0, int n)
{
  const int w = (int)warp_id();
  const int q4 = w & 3, hf = (w - 4) >> 2;
  const int kh = (int)lane_id() >> 4;   // key half of the block this lane holds
  const int kb0 = 64 * kh;
  const int row = q4 * 32 + hf * 16 + ((int)lane_id() & 15);
  const uint32_t lane_off = (uint32_t)(q4 * 32 + hf * 16) << 16;
  const uint32_t tO = tmem + kSBuf * 128 + lane_off;
  const int qi = q0 + row;
  float sqv = 1.0f;
  if constexpr (SAGE) sqv = (qi < p.tq) ? p.sq[(long)h * p.nqb + qi / 64] : 0.0f;
  const int kb_last = (p.tk - 1) >> 5;
  float m_ref = -INFINITY, l = 0.0f;
  bool ok = true;
  for (int j = 0; j < n; ++j) {
    // warp-uniform: the TMEM loads and stores below are warp-collective
    const int b = j % kSBuf;
    const uint32_t ph = (uint32_t)(j / kSBuf) & 1;
    if (!__all_sync(0xffffffffu, mbar_wait(s_full + 8 * b, ph, p.err, kDevWaitAccFull))) {
      ok = false;
      break;
    }
    tc_fence_after();
    const uint32_t tS = tmem + (uint32_t)b * 128 + lane_off;
    uint32_t r[64];
    tmem_ld_pair64<64>(tS, r);
    tmem_ld_wait();
    float f[2];
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      f[c] = p.scale_log2;
      if constexpr (SAGE)
        f[c] = fmaxf(f[c] * sqv * p.sk[(long)hk * p.nkb + min(4 * j + 2 * kh + c, kb_last)],
                     1e-30f);
    }
    float s[64];
#pragma unroll
    for (int i = 0; i < 64; ++i) {
      if constexpr (SAGE) s[i] = __int_as_float((int)r[i] + 0x4B400000) - 12582912.0f;
      else s[i] = __uint_as_float(r[i]);
    }
    const int kmax = p.tk - j * kBlk;
    if (kmax < kBlk) {
#pragma unroll
      for (int i = 0; i < 64; ++i)
        if (kb0 + i >= kmax) s[i] = -INFINITY;
    }
    float mc[2][2];
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      mc[c][0] = fmax3(s[32 * c], s[32 * c + 1], s[32 * c + 2]);
      mc[c][1] = fmax3(s[32 * c + 3], s[32 * c + 4], s[32 * c + 5]);
    }
#pragma unroll
    for (int i = 6; i < 32; i += 4) {
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        mc[c][0] = fmax3(mc[c][0], s[32 * c + i], s[32 * c + i + 1]);
        if (i + 3 < 32) mc[c][1] = fmax3(mc[c][1], s[32 * c + i + 2], s[32 * c + i + 3]);
      }
    }
    float mt = fmaxf(fmaxf(mc[0][0], mc[0][1]) * f[0], fmaxf(mc[1][0], mc[1][1]) * f[1]);
    mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 16));
    const bool need = (m_ref == -INFINITY) || (mt > m_ref + 8.0f);
    const float m_new = need ? fmaxf(mt, m_ref) : m_ref;
    if (j > 0 && __any_sync(0xffffffffu, need)) {
      // O is final up to P.V(j - 1) once its commit has landed (P.V(j - 3),
      // the slot's previous phase, had before S(j) ran)
      if (!__all_sync(0xffffffffu, mbar_wait(o_done + 8 * ((j - 1) & 1), ((j - 1) >> 1) & 1,
                                             p.err, kDevWaitAccFull))) {
        ok = false;
        break;
      }
      tc_fence_after();
      const float fac = (need && m_ref != -INFINITY) ? ex2(m_ref - m_new) : 1.0f;
#pragma unroll 1
      for (int c = 0; c < 2; ++c) {
        uint32_t o[32];
        tmem_ld_pair32<64>(tO + c * 32, o);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * fac);
        tmem_st_pair32<64>(tO + c * 32, o);
      }
      l *= fac;
    }
    m_ref = m_new;
    const float nm = m_ref == -INFINITY ? 0.0f : -m_ref;
    float rs[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      const float fc = f[c];
      uint32_t pk[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float x0 = fmaf(s[32 * c + 2 * i], fc, nm), x1 = fmaf(s[32 * c + 2 * i + 1], fc, nm);
        const float a = ex2(x0), b1 = ex2(x1);
        rs[i & 3] += a + b1;
        pk[i] = pack_bf2(a, b1);
      }
      // keys [kb0 + 32c, +32) -> bf16 columns [kb0/2 + 16c, +16) of the buffer
      tmem_st_pair16<32>(tS + 16 * c, pk);
    }
    tmem_st_wait();
    l += (rs[0] + rs[1]) + (rs[2] + rs[3]);
    tc_fence_before();
    __syncwarp();
    if (lane_id() == 0) mbar_arrive(p_full + 8 * b);
  }
  // O after the last P.V, then O / l of this lane's 64 dims
  const bool fin = ok && n > 0 && mbar_wait(o_final, 0, p.err, kDevWaitAccFull);
  if (!__all_sync(0xffffffffu, fin)) return;
  tc_fence_after();
  const float lt = l + __shfl_xor_sync(0xffffffffu, l, 16);
  const float inv = lt > 0.0f ? 1.0f / lt : 0.0f;
  __nv_bfloat16* dst = p.out + (long)qi * p.hq * 128 + (long)h * 128 + kb0;
#pragma unroll 1
  for (int c = 0; c < 2; ++c) {
    uint32_t o[32];
    tmem_ld_pair32<64>(tO + c * 32, o);
    tmem_ld_wait();
    if (qi < p.tq) {
      uint4* d4 = reinterpret_cast<uint4*>(dst + c * 32);
#pragma unroll
      for (int qd = 0; qd < 4; ++qd) {
        uint4 v;
        v.x = pack_bf2(__uint_as_float(o[qd * 8 + 0]) * inv, __uint_as_float(o[qd * 8 + 1]) * inv);
        v.y = pack_bf2(__uint_as_float(o[qd * 8 + 2]) * inv, __uint_as_float(o[qd * 8 + 3]) * inv);
        v.z = pack_bf2(__uint_as_float(o[qd * 8 + 4]) * inv, __uint_as_float(o[qd * 8 + 5]) * inv);
        v.w = pack_bf2(__uint_as_float(o[qd * 8 + 6]) * inv, __uint_as_float(o[qd * 8 + 7]) * inv);
        d4[qd] = v;
      }
    }
  }
}


template <bool SAGE, int kSBuf>
__global__ void __launch_bounds__(kThreads, 1)
    attn_tc1_kernel(const __grid_constant__ CUtensorMap tmQ,
                    const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const __grid_constant__ TcAttnP p)
{
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + kQBytes1;
  uint8_t* sV = sK + kStages1 * kKBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + kStages1 * kVBytes);
  const uint32_t b0 = smem_u32(bars);
  const uint32_t q_full = b0;
  const uint32_t k_full = b0 + 8;                  // [kStages1]
  const uint32_t v_full = k_full + 8 * kStages1;
  const uint32_t k_empty = v_full + 8 * kStages1;
  const uint32_t v_empty = k_empty + 8 * kStages1;
  const uint32_t s_full = v_empty + 8 * kStages1;  // [kSBuf]
  const uint32_t p_full = s_full + 8 * kSBuf;      // [kSBuf], one arrival a softmax warp
  const uint32_t o_done = p_full + 8 * kSBuf;      // [2]: P.V(j) completes slot j & 1
  const uint32_t o_final = o_done + 16;            // after the last P.V
  const uint32_t drain = o_final + 8;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 1 + 4 * kStages1 + 2 * kSBuf + 2 + 1 + 1);

  const int w = (int)warp_id();
  // unit t = head * (128-row blocks) + block, from p.unit_base
  const int nqt = (p.tq + kTile - 1) / kTile;
  const int t1 = (int)blockIdx.x + p.unit_base;
  const int h = t1 / nqt, hk = h / p.G;
  const int q0 = (t1 % nqt) * kTile;
  const int n = (p.tk + kBlk - 1) / kBlk;
  const int n_pg = (p.tk + 63) / 64;
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < kStages1; ++s) {
      mbar_init(k_full + 8 * s, 1);
      mbar_init(v_full + 8 * s, 1);
      mbar_init(k_empty + 8 * s, 1);
      mbar_init(v_empty + 8 * s, 1);
    }
    for (int b = 0; b < kSBuf; ++b) {
      mbar_init(s_full + 8 * b, 1);
      mbar_init(p_full + 8 * b, 8);
    }
    mbar_init(o_done, 1);
    mbar_init(o_done + 8, 1);
    mbar_init(o_final, 1);
    mbar_init(drain, 1);
    fence_barrier_init();
  }
  if (w == 0) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  if (threadIdx.x == 32) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // the set-up above overlaps the previous kernel; global memory waits for it
  griddep_launch();
  griddep_wait();
  if (w < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsLow));
    if (w == 0) {
      // ------------------------------------------------------------ producer
      if (lane_id() == 0) {
        const int qrow = h * p.tq + q0;
        if constexpr (SAGE) {
          mbar_arrive_expect_tx(q_full, kTile * 128);
          tma_load_2d(smem_u32(sQ), &tmQ, 0, qrow, q_full);
        } else {
          mbar_arrive_expect_tx(q_full, kTile * 256);
          for (int d = 0; d < 2; ++d)
            tma_load_2d(smem_u32(sQ + d * kTile * 128), &tmQ, d * 64, qrow, q_full);
        }
        int nk = 0, nv = 0;   // blocks whose K / V loads were issued
        for (int j = 0; j < n; ++j) {
          const int s = j % kStages1;
          const uint32_t ph = (j / kStages1) & 1;
          // the block's two pages; past the last page the first one is loaded
          // again (finite data under masked scores)
          const int pg0 = 2 * j, pg1 = min(2 * j + 1, n_pg - 1);
          const int page0 = p.page_table ? p.page_table[pg0] : pg0;
          const int page1 = p.page_table ? p.page_table[pg1] : pg1;
          if (!mbar_wait(k_empty + 8 * s, ph ^ 1, p.err, kDevWaitEmpty)) break;
          uint8_t* k_dst = sK + s * kKBytes;
          if constexpr (SAGE) {
            mbar_arrive_expect_tx(k_full + 8 * s, kBlk * 128);
            const int krow = (int)(hk * p.k8_stride) + j * kBlk;
            tma_load_2d(smem_u32(k_dst), &tmK, 0, krow, k_full + 8 * s);
            tma_load_2d(smem_u32(k_dst + 64 * 128), &tmK, 0, krow + 64, k_full + 8 * s);
          } else {
            mbar_arrive_expect_tx(k_full + 8 * s, kKBytes);
            for (int hf = 0; hf < 2; ++hf) {
              const int krow = ((hf ? page1 : page0) * p.hkv + hk) * 64;
              for (int d = 0; d < 2; ++d)
                tma_load_2d(smem_u32(k_dst + d * kBlk * 128 + hf * 64 * 128), &tmK, d * 64, krow,
                            k_full + 8 * s);
            }
          }
          nk = j + 1;
          if (!mbar_wait(v_empty + 8 * s, ph ^ 1, p.err, kDevWaitEmpty)) break;
          mbar_arrive_expect_tx(v_full + 8 * s, kVBytes);
          for (int hf = 0; hf < 2; ++hf)
            tma_load_2d(smem_u32(sV + s * kVBytes + hf * 128 * 128), &tmV, 0,
                        ((hf ? page1 : page0) * p.hkv + hk) * 128, v_full + 8 * s);
          nv = j + 1;
        }
        // unwinding: every copy issued must land before the CTA may exit
        mbar_wait(q_full, 0, p.err, kDevWaitDrain);
        for (int s = 0; s < kStages1; ++s) {
          if (nk > s) {
            const int last = ((nk - 1 - s) / kStages1) * kStages1 + s;
            mbar_wait(k_full + 8 * s, (last / kStages1) & 1, p.err, kDevWaitDrain);
          }
          if (nv > s) {
            const int last = ((nv - 1 - s) / kStages1) * kStages1 + s;
            mbar_wait(v_full + 8 * s, (last / kStages1) & 1, p.err, kDevWaitDrain);
          }
        }
      }
    } else if (w == 1) {
      // ------------------------------------------------------------ MMA
      // Issue order S(0), S(1), S(2), P.V(0), S(3), P.V(1), S(4), ...:
      // S(j + 3) overwrites P(j)'s buffer and follows P.V(j) on the tensor
      // core. A commit arrives when every earlier MMA of this thread has
      // completed: s_full[b] after S(j), o_done[j & 1] after P.V(j), the
      // stage releases after the MMAs that read the stage.
      if (lane_id() == 0) {
        const uint32_t id_s = SAGE ? idesc_s8(kTile, kBlk) : idesc_bf16(kTile, kBlk);
        const uint32_t id_o = idesc_bf16(kTile, 128);
        auto issue_s = [&](int j) {
          const uint32_t d = tmem + (uint32_t)(j % kSBuf) * 128;
          const uint32_t kb = smem_u32(sK + (j % kStages1) * kKBytes);
          const uint32_t a0 = smem_u32(sQ);
          if constexpr (SAGE) {
  #pragma unroll
            for (int k = 0; k < 4; ++k)
              mma_i8(d, smem_desc_sw128(a0 + k * 32), smem_desc_sw128(kb + k * 32), id_s, k != 0);
          } else {
  #pragma unroll
            for (int k = 0; k < 8; ++k)
              mma_bf16(d, smem_desc_sw128(a0 + (k >> 2) * kTile * 128 + (k & 3) * 32),
                       smem_desc_sw128(kb + (k >> 2) * kBlk * 128 + (k & 3) * 32), id_s, k != 0);
          }
        };
        bool ok = mbar_wait(q_full, 0, p.err, kDevWaitFull);
        for (int j = 0; j < kSBuf && j < n && ok; ++j) {
          const int s = j % kStages1;
          ok = mbar_wait_probe(k_full + 8 * s, (j / kStages1) & 1, p.err, kDevWaitFull);
          if (!ok) break;
          tc_fence_after();
          issue_s(j);
          mma_commit(s_full + 8 * (j % kSBuf));
          mma_commit(k_empty + 8 * s);
        }
        for (int j = 0; j < n && ok; ++j) {
          const int s = j % kStages1, b = j % kSBuf;
          if (!mbar_wait_probe(p_full + 8 * b, (j / kSBuf) & 1, p.err, kDevWaitFull) ||
              !mbar_wait_probe(v_full + 8 * s, (j / kStages1) & 1, p.err, kDevWaitFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t vb = smem_u32(sV + s * kVBytes);
          const uint32_t d = tmem + kSBuf * 128, a = tmem + (uint32_t)b * 128;
  #pragma unroll
          for (int k = 0; k < 8; ++k)
            mma_bf16_ts(d, a + k * 8, smem_desc_sw128(vb + (k >> 2) * 128 * 128 + (k & 3) * 32),
                        id_o, (j | k) != 0);
          mma_commit(o_done + 8 * (j & 1));
          if (j == n - 1) mma_commit(o_final);
          mma_commit(v_empty + 8 * s);
          if (j + kSBuf < n) {
            const int s3 = (j + kSBuf) % kStages1;
            if (!mbar_wait_probe(k_full + 8 * s3, ((j + kSBuf) / kStages1) & 1, p.err,
                                 kDevWaitFull)) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue_s(j + kSBuf);
            mma_commit(s_full + 8 * b);
            mma_commit(k_empty + 8 * s3);
          }
        }
        mma_commit(drain);
        mbar_wait(drain, 0, p.err, kDevWaitDrain);
      }
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegsHigh));
    softmax_single<SAGE, kSBuf>(p, tmem, s_full, p_full, o_done, o_final, h, hk, q0, n);
    tc_fence_before();
  }

  __syncthreads();
  if (w == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}


// SMs of the current device (cached per device)
int device_sms()
{
  static std::atomic<int> cache[64];
  int d = 0;
  if (cudaGetDevice(&d) != cudaSuccess || d < 0 || d >= 64) return 0;
  int v = cache[d].load(std::memory_order_relaxed);
  if (v == 0) {
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, d) != cudaSuccess) return 0;
    cache[d].store(v, std::memory_order_relaxed);
  }
  return v;
}


}  // namespace

bool attention_tc_serves(int mode, int tk, const int32_t* t_index)
{
  if (mode == 0 || mode == 1) return true;
  return mode == 2 && t_index != nullptr && tk <= kMaxBlk * kBlk &&
         (reinterpret_cast<uintptr_t>(t_index) & 15) == 0;
}

int attention_tc(const TcAttnArgs& a, cudaStream_t st, std::string* err)
{
  if (a.hq <= 0 || a.hkv <= 0 || a.hq % a.hkv) {
    *err = "attention: hq must be a positive multiple of hkv";
    return 1;
  }
  if (a.mode < 0 || a.mode > 2) {
    *err = "attention: unknown mode";
    return 1;
  }
  const bool sage = a.q8 != nullptr;
  if (sage && a.mode != 0) {
    *err = "attention: the int8-QK path serves the bidirectional pass only";
    return 1;
  }
  if (a.mode == 2 && !attention_tc_serves(2, a.tk, a.t_index)) {
    *err = "attention (tcgen05): block-causal needs a 16-byte aligned t-index vector and at most " +
           std::to_string(kMaxBlk * kBlk) + " keys";
    return 1;
  }
  if (a.mode != 0 && (a.q_offset < 0 || (a.mode == 2 && (long)a.q_offset + a.tq > a.tk))) {
    *err = "attention: the queries' positions must lie within the key range";
    return 1;
  }
  if (a.tq <= 0 || a.tk <= 0) return 0;
  const int n_pages_needed = (a.tk + 63) / 64;
  if (a.n_pages < n_pages_needed && a.page_table == nullptr) {
    *err = "attention: the page pool holds fewer pages than the key length needs";
    return 1;
  }
  TcAttnP p{};
  p.hq = a.hq;
  p.hkv = a.hkv;
  p.tq = a.tq;
  p.tk = a.tk;
  p.G = a.hq / a.hkv;
  p.q_offset = a.q_offset;
  p.t_index = a.t_index;
  p.scale_log2 = (float)(1.4426950408889634 / std::sqrt(128.0));
  p.page_table = a.page_table;
  p.out = static_cast<__nv_bfloat16*>(a.out);
  p.sq = a.sq;
  p.sk = a.sk;
  p.nqb = (a.tq + 63) / 64;
  p.nkb = 2 * ((a.tk + 63) / 64);   // 32-key K blocks, two per page
  p.k8_stride = (long)p.nkb * 32;
  p.err = a.dev_err;
  const char* iss_env = std::getenv("U15_ATTN_ISSUERS");
  p.issuers = iss_env != nullptr ? (std::atoi(iss_env) == 2 ? 2 : 1) : (a.mode == 2 ? 2 : 1);
  const char* rel_env = std::getenv("U15_ATTN_RELEASE");
  const bool one_row = !(std::getenv("U15_ATTN_KS") ? std::atoi(std::getenv("U15_ATTN_KS")) != 0
                                                     : a.mode == 2);
  // The bidirectional pass's K / V stages are released by the softmax warps
  // (they see the S-ready commit that follows the MMAs reading a stage), so
  // the single issuer commits no stage releases between the tiles' MMAs:
  // 0.321 -> 0.312 ms at 4096 x 4416, Sage unchanged (U15_ATTN_RELEASE=0
  // keeps the issuer's commits). The masked rules' tiles end at different
  // blocks, so they keep them.
  p.release = a.mode == 0 && p.issuers == 1 && one_row &&
              (rel_env == nullptr || std::atoi(rel_env) != 0);
  CUtensorMap mq, mk, mv;
  if (sage) {
    if (make_tma_2d(&mq, a.q8, (uint64_t)a.hq * a.tq, 128, kTile, 1, err)) return 2;
    if (make_tma_2d(&mk, a.k8, (uint64_t)a.hkv * p.k8_stride, 128, 64, 1, err)) return 2;
  } else {
    if (make_tma_2d(&mq, a.q, (uint64_t)a.hq * a.tq, 128, kTile, 2, err)) return 2;
    if (make_tma_2d(&mk, a.k_pages, (uint64_t)a.n_pages * a.hkv * 64, 128, 64, 2, err)) return 2;
  }
  if (make_tma_2d(&mv, a.vt_pages, (uint64_t)a.n_pages * a.hkv * 128, 64, 128, 2, err)) return 2;
  // The exponentials (U15_ATTN_EXP, read per launch for A/B checks): 0 every
  // one a float ex2 on the MUFU; 1 a quarter of them on the FMA pipe (5-10 %
  // slower for bf16, 4 % for Sage, measured).
  static std::atomic<uint64_t> set_attr[20];
  const int nqblk = (a.tq + 2 * kTile - 1) / (2 * kTile);
  const dim3 grid = a.mode == 0 ? dim3(nqblk * a.hq) : dim3(a.hq, nqblk);
  const char* exp_env = std::getenv("U15_ATTN_EXP");
  int expm = exp_env != nullptr ? std::atoi(exp_env) : kDefaultExp;
  if (expm < 0 || expm > 1) expm = kDefaultExp;
  // The softmax layout and the MMA issuers per rule (measured, 4096 x 4416
  // and BASELINE config 4's prefill): the bidirectional and causal rules take
  // one query row a thread with one issuer; the block-causal rule, whose
  // per-element test loads the softmax warps' issue slots, the key-split
  // layout (64 keys a thread, two warps per lane quadrant) with one issuer a
  // tile. U15_ATTN_KS and U15_ATTN_ISSUERS override both (read per launch,
  // for A/B checks).
  const char* ks_env = std::getenv("U15_ATTN_KS");
  const int ks = ks_env != nullptr ? (std::atoi(ks_env) != 0) : (a.mode == 2 ? 1 : 0);
  using KFn = void (*)(CUtensorMap, CUtensorMap, CUtensorMap, TcAttnP);
  static const KFn table[4][2][2] = {
      {{attn_tc_kernel<false, 0, 0, false>, attn_tc_kernel<false, 0, 0, true>},
       {attn_tc_kernel<false, 1, 0, false>, attn_tc_kernel<false, 1, 0, true>}},
      {{attn_tc_kernel<true, 0, 0, false>, attn_tc_kernel<true, 0, 0, true>},
       {attn_tc_kernel<true, 1, 0, false>, attn_tc_kernel<true, 1, 0, true>}},
      {{attn_tc_kernel<false, 0, 1, false>, attn_tc_kernel<false, 0, 1, true>},
       {attn_tc_kernel<false, 1, 1, false>, attn_tc_kernel<false, 1, 1, true>}},
      {{attn_tc_kernel<false, 0, 2, false>, attn_tc_kernel<false, 0, 2, true>},
       {attn_tc_kernel<false, 1, 2, false>, attn_tc_kernel<false, 1, 2, true>}}};
  const int row = sage ? 1 : (a.mode == 0 ? 0 : a.mode + 1);
  // U15_ATTN_TILES=1 (read per launch, for A/B checks): the bidirectional
  // pass with one 128-row tile a CTA and two or three S buffers
  // (U15_ATTN_SBUF=3). Measured in the layer bench against the two-tile
  // kernel: no faster (attention alone -5 % Sage, +-2 % bf16; the layer
  // and the denoise loop unchanged or slower).
  const char* tiles_env = std::getenv("U15_ATTN_TILES");
  const bool single = a.mode == 0 && tiles_env != nullptr && std::atoi(tiles_env) == 1;
  const char* sbuf_env = std::getenv("U15_ATTN_SBUF");
  const int sbuf = sbuf_env != nullptr && std::atoi(sbuf_env) == 3 ? 3 : 2;
  const KFn k_two = table[row][expm][ks];
  const KFn k_one = sbuf == 3 ? (sage ? attn_tc1_kernel<true, 3> : attn_tc1_kernel<false, 3>)
                              : (sage ? attn_tc1_kernel<true, 2> : attn_tc1_kernel<false, 2>);
  const int which_two = (row * 2 + expm) * 2 + ks;
  const int which_one = 16 + (sage ? 1 : 0) + (sbuf == 3 ? 2 : 0);
  // The bidirectional pass's last round: when the two-tile units leave a
  // last round at most half full (and the query count is whole 256-row
  // blocks), its units run as twice as many one-tile CTAs in a second
  // launch, each about 0.58 of a two-tile CTA's time (U15_ATTN_SPLIT=0
  // keeps one launch).
  int split_units = 0;   // two-tile units handed to the one-tile launch
  if (a.mode == 0 && !single && a.tq % (2 * kTile) == 0) {
    const char* sp_env = std::getenv("U15_ATTN_SPLIT");
    if (sp_env == nullptr || std::atoi(sp_env) != 0) {
      const int sms = device_sms();
      const int units = nqblk * a.hq, r = units % sms;
      if (sms > 0 && units > sms && r > 0 && 2 * r <= sms) split_units = r;
    }
  }
  auto launch = [&](KFn kf, int which, int smem, dim3 g, const TcAttnP& pp) {
    if (!smem_attr_once(kf, smem, set_attr[which])) {
      const cudaError_t e0 = cudaGetLastError();
      return e0 == cudaSuccess ? cudaErrorInvalidValue : e0;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = g;
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    cudaError_t e1 = cudaLaunchKernelEx(&cfg, kf, mq, mk, mv, pp);
    if (e1 == cudaSuccess) e1 = cudaGetLastError();
    return e1;
  };
  cudaError_t e = cudaSuccess;
  KFn k = k_two;
  int smem = kSmem;
  p.unit_base = 0;
  if (single) {
    k = k_one;
    smem = kSmem1;
    e = launch(k_one, which_one, kSmem1, dim3(((a.tq + kTile - 1) / kTile) * a.hq), p);
  } else if (split_units > 0) {
    const int units = nqblk * a.hq;
    e = launch(k_two, which_two, kSmem, dim3(units - split_units), p);
    if (e == cudaSuccess) {
      TcAttnP p1 = p;
      p1.unit_base = 2 * (units - split_units);
      k = k_one;
      smem = kSmem1;
      e = launch(k_one, which_one, kSmem1, dim3(2 * split_units), p1);
    }
  } else {
    e = launch(k_two, which_two, kSmem, grid, p);
  }
  if (e != cudaSuccess) {
    cudaFuncAttributes fa{};
    cudaFuncGetAttributes(&fa, k);
    *err = std::string("attention (tcgen05): kernel launch failed: ") + cudaGetErrorString(e) +
           " (registers " + std::to_string(fa.numRegs) + ", max threads " +
           std::to_string(fa.maxThreadsPerBlock) + ", dynamic smem " + std::to_string(smem) + ")";
    return 2;
  }
  return 0;
}

}  // namespace u15
