// The projection GEMM of the MoT layer on sm_100a tensor cores.
//
//   y[m][n] = epilogue( sum_k x[m][k] * W_e[n][k] ),  e = expert of row m
//
// One persistent kernel per call, one CTA per SM, warp-specialised:
//   warp 0      TMA producer: 128x(BK) A tile + 256x(BK) B tile per stage,
//               128-byte swizzle, 4-stage ring in shared memory
//   warp 1      MMA issuer: one thread issues tcgen05.mma (M=128, N=256)
//               into one of two TMEM accumulators (2 x 256 f32 columns)
//   warps 2-5   epilogue: tcgen05.ld the accumulator (one row per thread),
//               apply the fused epilogue, store bf16 to global
// The two TMEM accumulators let the epilogue of tile i overlap the
// main loop of tile i+1.
//
// MoT routing (the reference selects ONE expert per pass,
// src/u15-backbone.cc:189; here one launch serves every segment): the host
// splits the M axis into "units" -- a 128-row block intersected with one
// contiguous token segment -- and each unit names the expert whose weight
// rows (W stacked as [E][N][K]) its B tiles come from. A block that
// straddles a segment boundary appears once per segment and each pass
// stores only its own rows.
//
// bf16: kind::f16, BK = 64 elements (128 bytes), 4 MMAs of K=16 per stage.
// int8: kind::i8, BK = 128 elements (128 bytes), 4 MMAs of K=32 per stage,
//       s32 accumulators, dequantised in the epilogue by the per-token and
//       per-channel scales (acc * s_tok[m] * s_ch[n]).
//
// Epilogues (the reference's separate passes, src/u15-backbone.cc:229-256,
// with their bf16 rounding points kept):
//   STORE   y = bf16(acc [+ bias])
//   RESID   y = bf16(resid + bf16(acc))                       o_proj / down
//   SWIGLU  B rows interleaved in 128-row blocks [gate_j | up_j]:
//           y[:, 128j + c] = bf16(silu(bf16(g)) * bf16(u))    gate|up
#include "u15_common.cuh"
#include "u15_kernels.h"

#include <algorithm>
#include <cstdlib>
#include <mutex>
#include <unordered_map>
#include <vector>

namespace u15 {

namespace {

constexpr int kBM = 128, kBN = 256, kStages = 4, kThreads = 192;
constexpr int kAStage = kBM * 128;   // bytes per A stage (128 rows x 128 B)
constexpr int kBStage = kBN * 128;   // bytes per B stage
constexpr int kSmemBytes = kStages * (kAStage + kBStage) + 1024 /*align*/ + 256 /*bars*/;

struct Unit {
  int m0, row_lo, row_hi, expert;
};

// the pair kernel's L2 policy unless U15_GEMM_L2HINT says otherwise
constexpr int kDefaultL2Hint = 0;
// the pair kernel's k-blocks per stage unless U15_GEMM_KPS says otherwise
constexpr int kDefaultKps = 2;

struct Params {
  int M, N, K;          // N: weight rows per expert (SWIGLU: 2x the output width)
  int n_units, n_nblk, n_kblk;
  int n_full;           // tiles before the split tail (== n_units * n_nblk when none)
  int group;            // tile order: units (row blocks) per group, >= 1
  // row units: a unit_bm-row block intersected with one routing segment,
  // segment-major (segment s holds units [unit_start[s], unit_start[s + 1]))
  int unit_bm;
  int nseg;
  int seg_off[kMaxSeg + 1];
  int seg_expert[kMaxSeg];
  int unit_start[kMaxSeg + 1];
  int l2hint;           // 0 none; 1 B (weights) evict-first; 2 also A evict-last
  int kps;              // pair kernel: k-blocks per pipeline stage, 1, 2 or 3
  void* y;
  long ldy;             // output row stride, elements
  const __nv_bfloat16* resid;
  long ldr;
  const __nv_bfloat16* bias;   // [E][N] or null
  const float* s_tok;          // int8: [M]
  const float* s_ch;           // int8: [E][N]
  int32_t* acc_dump;           // int8 debug: [M][N] raw accumulators, or null
  unsigned* err;
  TpPeers tp;           // kEpiTpReduce
};

// Tile t of a launch. Tiles [0, n_full) are full width; each tile after
// them (the last, partly filled round of the persistent schedule) runs as two
// half-width tiles (half = 0, 1), so that round takes half as long.
struct TileIdx {
  int unit, nb, half;   // half: -1 full width
};

__device__ __forceinline__ TileIdx tile_at(const Params& p, int t)
{
  TileIdx r{0, 0, -1};
  int tt = t;
  if (t >= p.n_full) {
    const int h = t - p.n_full;
    tt = p.n_full + (h >> 1);
    r.half = h & 1;
  }
  // grouped order: the units of one group sweep all column blocks before
  // the next group starts, so a round of the schedule touches `group` row
  // blocks of A and a proportionate share of B
  const int g0 = (tt / (p.group * p.n_nblk)) * p.group;
  const int gs = min(p.group, p.n_units - g0);
  const int rr = tt - g0 * p.n_nblk;
  r.unit = g0 + rr % gs;
  r.nb = rr / gs;
  return r;
}

// Row unit i, computed from the segment table (no per-unit table, so M has
// no limit): its segment s is the last whose first unit is <= i, its block
// the segment's first block plus the offset, its rows the block's rows
// inside the segment.
__device__ __forceinline__ Unit unit_at(const Params& p, int i)
{
  int s = 0;
#pragma unroll 1
  for (int k = 1; k < p.nseg; ++k)
    if (i >= p.unit_start[k]) s = k;
  const int m0 = (p.seg_off[s] / p.unit_bm + (i - p.unit_start[s])) * p.unit_bm;
  return Unit{m0, max(m0, p.seg_off[s]), min(m0 + p.unit_bm, p.seg_off[s + 1]), p.seg_expert[s]};
}

__host__ __device__ __forceinline__ int launch_tiles(const Params& p)
{
  return p.n_full + 2 * (p.n_units * p.n_nblk - p.n_full);
}

template <bool I8>
__device__ __forceinline__ void chunk_values(uint32_t taddr, float (&v)[32], const Params& p,
                                             int row, bool row_ok, int col0, int expert)
{
  uint32_t r[32];
  tmem_ld32(taddr, r);
  tmem_ld_wait();
  if constexpr (I8) {
    const float st = row_ok ? p.s_tok[row] : 0.0f;
    if (p.acc_dump != nullptr && row_ok) {
      int32_t* d = p.acc_dump + (long)row * p.N + col0;
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (col0 + i < p.N) d[i] = (int32_t)r[i];
    }
    const float* sc = p.s_ch + (long)expert * p.N + col0;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const float s = (col0 + i < p.N) ? sc[i] : 0.0f;
      v[i] = ((float)(int32_t)r[i] * st) * s;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
  }
}

// Store 32 bf16 values of one row at columns [col0, col0 + 32) with
// columns >= ncols dropped.
__device__ __forceinline__ void store_row32(__nv_bfloat16* dst, const float (&v)[32], int col0,
                                            int ncols)
{
  if (col0 + 32 <= ncols && ((reinterpret_cast<uintptr_t>(dst) & 15) == 0)) {
    uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint4 o;
      o.x = pack_bf2(v[q * 8 + 0], v[q * 8 + 1]);
      o.y = pack_bf2(v[q * 8 + 2], v[q * 8 + 3]);
      o.z = pack_bf2(v[q * 8 + 4], v[q * 8 + 5]);
      o.w = pack_bf2(v[q * 8 + 6], v[q * 8 + 7]);
      d4[q] = o;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (col0 + i < ncols) dst[i] = f2bf(v[i]);
  }
}

// Store 32 f32 values of one row (columns >= ncols dropped).
__device__ __forceinline__ void store_row32_f32(float* dst, const float (&v)[32], int col0,
                                                int ncols)
{
  if (col0 + 32 <= ncols && ((reinterpret_cast<uintptr_t>(dst) & 15) == 0)) {
    float4* d4 = reinterpret_cast<float4*>(dst);
#pragma unroll
    for (int q = 0; q < 8; ++q) d4[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (col0 + i < ncols) dst[i] = v[i];
  }
}

__device__ __forceinline__ void load_row32(const __nv_bfloat16* src, float (&v)[32], int col0,
                                           int ncols)
{
  if (col0 + 32 <= ncols && ((reinterpret_cast<uintptr_t>(src) & 15) == 0)) {
    const uint4* s4 = reinterpret_cast<const uint4*>(src);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint4 u = s4[q];
      float2 a = unpack_bf2(u.x), b = unpack_bf2(u.y), c = unpack_bf2(u.z), d = unpack_bf2(u.w);
      v[q * 8 + 0] = a.x; v[q * 8 + 1] = a.y; v[q * 8 + 2] = b.x; v[q * 8 + 3] = b.y;
      v[q * 8 + 4] = c.x; v[q * 8 + 5] = c.y; v[q * 8 + 6] = d.x; v[q * 8 + 7] = d.y;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = (col0 + i < ncols) ? bf2f(src[i]) : 0.0f;
  }
}

template <bool I8, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ Params p)
{
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + kStages * kAStage;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sB + kStages * kBStage);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * kStages + 5);

  const uint32_t full0 = smem_u32(bars);
  const uint32_t empty0 = full0 + 8 * kStages;
  const uint32_t accf0 = empty0 + 8 * kStages;
  const uint32_t acce0 = accf0 + 16;
  const uint32_t drain = acce0 + 16;

  const uint32_t w = warp_id();
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(accf0 + 8 * a, 1);
      mbar_init(acce0 + 8 * a, 128);
    }
    mbar_init(drain, 1);
    fence_barrier_init();
  }
  if (w == 0) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  if (threadIdx.x == 32) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int n_tiles = p.n_units * p.n_nblk;
  constexpr int kBK = I8 ? 128 : 64;   // elements per 128-byte row

  if (w == 0) {
    // ---------------- TMA producer ----------------
    if (lane_id() == 0) {
      uint32_t it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < n_tiles && ok; t += gridDim.x) {
        const TileIdx ti = tile_at(p, t);
        const Unit u = unit_at(p, ti.unit);
        const int nb = ti.nb;
        const int brow = u.expert * p.N + nb * kBN;
        for (int kb = 0; kb < p.n_kblk; ++kb, ++it) {
          const uint32_t s = it % kStages, ph = (it / kStages) & 1;
          if (!mbar_wait(empty0 + 8 * s, ph ^ 1, p.err, kDevWaitEmpty)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(full0 + 8 * s, kAStage + kBStage);
          tma_load_2d(smem_u32(sA + s * kAStage), &tmA, kb * kBK, u.m0, full0 + 8 * s);
          tma_load_2d(smem_u32(sB + s * kBStage), &tmB, kb * kBK, brow, full0 + 8 * s);
        }
      }
      // Unwind: every stage's last fill must land before the CTA may exit.
      for (uint32_t s = 0; s < kStages; ++s) {
        if (it > s) {
          const uint32_t last = ((it - 1 - s) / kStages) * kStages + s;
          mbar_wait(full0 + 8 * s, (last / kStages) & 1, p.err, kDevWaitDrain);
        }
      }
    }
  } else if (w == 1) {
    // ---------------- MMA issuer ----------------
    if (lane_id() == 0) {
      const uint32_t idesc = I8 ? idesc_s8(kBM, kBN) : idesc_bf16(kBM, kBN);
      uint32_t it = 0;
      int lt = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < n_tiles && ok; t += gridDim.x, ++lt) {
        const uint32_t acc = lt & 1, aph = (lt >> 1) & 1;
        if (!mbar_wait_probe(acce0 + 8 * acc, aph ^ 1, p.err, kDevWaitAccEmpty)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * kBN;
        for (int kb = 0; kb < p.n_kblk; ++kb, ++it) {
          const uint32_t s = it % kStages, ph = (it / kStages) & 1;
          if (!mbar_wait_probe(full0 + 8 * s, ph, p.err, kDevWaitFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + s * kAStage);
          const uint32_t b0 = smem_u32(sB + s * kBStage);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint64_t ad = smem_desc_sw128(a0 + k * 32);
            const uint64_t bd = smem_desc_sw128(b0 + k * 32);
            if constexpr (I8)
              mma_i8(d_tmem, ad, bd, idesc, (kb | k) != 0);
            else
              mma_bf16(d_tmem, ad, bd, idesc, (kb | k) != 0);
          }
          mma_commit(empty0 + 8 * s);
        }
        if (!ok) break;
        mma_commit(accf0 + 8 * acc);
      }
      // Unwind: all MMAs this thread issued complete before TMEM is freed.
      mma_commit(drain);
      mbar_wait(drain, 0, p.err, kDevWaitDrain);
    }
  } else {
    // ---------------- epilogue (warps 2..5) ----------------
    const int wq = (int)(w & 3);   // TMEM lane quadrant this warp may access
    const int r_in = wq * 32 + (int)lane_id();
    int lt = 0;
    for (int t = blockIdx.x; t < n_tiles; t += gridDim.x, ++lt) {
      const TileIdx ti = tile_at(p, t);
      const Unit u = unit_at(p, ti.unit);
      const int nb = ti.nb;
      const uint32_t acc = lt & 1, aph = (lt >> 1) & 1;
      if (!mbar_wait(accf0 + 8 * acc, aph, p.err, kDevWaitAccFull)) break;
      tc_fence_after();
      const int row = u.m0 + r_in;
      const bool row_ok = row >= u.row_lo && row < u.row_hi;
      const uint32_t tb = tmem_base + acc * kBN + ((uint32_t)(wq * 32) << 16);
      const int n0 = nb * kBN;
      if constexpr (EPI == kEpiSwiglu) {
        const int nout = p.N / 2;
        __nv_bfloat16* yrow = reinterpret_cast<__nv_bfloat16*>(p.y) + (long)row * p.ldy;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          float g[32], v[32];
          chunk_values<I8>(tb + c * 32, g, p, row, row_ok, n0 + c * 32, u.expert);
          chunk_values<I8>(tb + 128 + c * 32, v, p, row, row_ok, n0 + 128 + c * 32, u.expert);
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const float gg = bfround(g[i]), uu = bfround(v[i]);
            g[i] = __fdividef(gg, 1.0f + __expf(-gg)) * uu;
          }
          const int oc = nb * 128 + c * 32;
          if (row_ok) store_row32(yrow + oc, g, oc, nout);
        }
      } else {
        __nv_bfloat16* yrow = reinterpret_cast<__nv_bfloat16*>(p.y) + (long)row * p.ldy;
#pragma unroll 1
        for (int c = 0; c < kBN / 32; ++c) {
          float v[32];
          const int col0 = n0 + c * 32;
          chunk_values<I8>(tb + c * 32, v, p, row, row_ok, col0, u.expert);
          if (!row_ok || col0 >= p.N) continue;
          if (p.bias != nullptr) {
            const __nv_bfloat16* b = p.bias + (long)u.expert * p.N + col0;
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (col0 + i < p.N) v[i] += bf2f(b[i]);
          }
          if constexpr (EPI == kEpiResid) {
            float rr[32];
            load_row32(p.resid + (long)row * p.ldr + col0, rr, col0, p.N);
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = rr[i] + bfround(v[i]);
          }
          if constexpr (EPI == kEpiStoreF32)
            store_row32_f32(reinterpret_cast<float*>(p.y) + (long)row * p.ldy + col0, v, col0, p.N);
          else
            store_row32(yrow + col0, v, col0, p.N);
        }
      }
      tc_fence_before();
      mbar_arrive(acce0 + 8 * acc);
    }
  }

  __syncthreads();
  if (w == 0) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}


// ---------------------------------------------------------------------
// The CTA-pair variant (tcgen05 cta_group::2): one 256x256 tile per pair of
// SMs. CTA r of the pair loads A rows [m0 + 128r, +128) and B rows
// [n0 + 128r, +128) -- half of each operand -- and the leader (r = 0)
// issues M=256 N=256 MMAs that read both CTAs' halves; each CTA's TMEM
// holds its own 128 rows x 256 columns of the accumulator. Per SM and
// k-block that is 32 KB of operands for the same math the single-SM tile
// needs 48 KB for, which is what the L2 -> SM path limits at int8 speed.
// The leader's operand-full and accumulator-empty barriers count both
// CTAs; its commits arrive on both CTAs' stage-empty and accumulator-full
// barriers (multicast commit). No TMA multicast.
// ---------------------------------------------------------------------
constexpr int kStagesP = 6;
constexpr int kAStageP = 128 * 128;   // per CTA: 128 rows x 128 B
constexpr int kBStageP = 128 * 128;
constexpr int kSmemP = kStagesP * (kAStageP + kBStageP) + 1024 + 256;
constexpr int kSmemPTp = kSmemP + 4 * 32 * 32 * 4;   // + the TP epilogue's staging

template <bool I8, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_pair_kernel(const __grid_constant__ CUtensorMap tmA,
                        const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ CUtensorMap tmBh, const __grid_constant__ Params p)
{
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + kStagesP * kAStageP;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sB + kStagesP * kBStageP);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * kStagesP + 5);
  // kEpiTpReduce only (launched with kSmemPTp): 4 warps x [32][32] f32 staging
  float* tp_stage = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(bars) + 256);
  (void)tp_stage;

  const uint32_t full0 = smem_u32(bars);            // leader: count 2 (one per CTA) + tx
  const uint32_t empty0 = full0 + 8 * kStagesP;     // each CTA: leader's multicast commit
  const uint32_t accf0 = empty0 + 8 * kStagesP;     // each CTA: leader's multicast commit
  const uint32_t acce0 = accf0 + 16;                // leader: 256 epilogue threads
  const uint32_t drain = acce0 + 16;                // each CTA: leader's multicast commit

  const uint32_t w = warp_id();
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStagesP; ++s) {
      mbar_init(full0 + 8 * s, 2);
      mbar_init(empty0 + 8 * s, 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(accf0 + 8 * a, 1);
      mbar_init(acce0 + 8 * a, 256);
    }
    mbar_init(drain, 1);
    fence_barrier_init();
  }
  if (w == 0) {
    tmem_alloc_pair(smem_u32(tmem_slot), 512);
    tmem_relinquish_pair();
  }
  if (threadIdx.x == 32) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmBh);
  }
  tc_fence_before();
  cluster_sync();   // barriers of both CTAs initialised before any remote arrive
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // the set-up above overlaps the previous kernel; nothing in global memory
  // is touched before it has completed
  griddep_launch();
  griddep_wait();

  const int n_tiles = launch_tiles(p);
  const int pair = blockIdx.x >> 1, n_pairs = gridDim.x >> 1;
  constexpr int kBK = I8 ? 128 : 64;
  // k-blocks per pipeline stage (1 or 2) and the stages of the ring: the
  // same shared memory as kStagesP stages of one k-block
  const int kps = p.kps;
  const uint32_t nst = kStagesP / kps;

  if (w == 0) {
    // ---------------- TMA producer (both CTAs) ----------------
    if (lane_id() == 0) {
      uint32_t it = 0;
      bool ok = true;
      // the weights stream through L2 once per launch; the activations are
      // read again by every round of the schedule
      const uint64_t pol_b = l2_evict_first_policy(), pol_a = l2_evict_last_policy();
      for (int t = pair; t < n_tiles && ok; t += n_pairs) {
        const TileIdx ti = tile_at(p, t);
        const Unit u = unit_at(p, ti.unit);
        const bool half = ti.half >= 0;
        // B rows this CTA stages: its half of the tile's columns. A
        // half-width SwiGLU tile keeps gate and up paired: CTA 0 takes 64
        // gate rows, CTA 1 the 64 up rows that go with them.
        const int boff = !half                 ? 128 * (int)rank
                         : EPI == kEpiSwiglu   ? 128 * (int)rank + 64 * ti.half
                                               : 128 * ti.half + 64 * (int)rank;
        const int arow = u.m0 + 128 * (int)rank;
        const int brow = u.expert * p.N + ti.nb * 256 + boff;
        const CUtensorMap* mb = half ? &tmBh : &tmB;
        const uint32_t tx = kAStageP + (half ? kBStageP / 2 : kBStageP);
        for (int kb = 0; kb < p.n_kblk; kb += kps, ++it) {
          const uint32_t s = it % nst, ph = (it / nst) & 1;
          if (!mbar_wait(empty0 + 8 * s, ph ^ 1, p.err, kDevWaitEmpty)) {
            ok = false;
            break;
          }
          const int nk = min(kps, p.n_kblk - kb);   // k-blocks in this stage
          const uint32_t fb = mapa_shared(full0 + 8 * s, 0);
          mbar_arrive_expect_tx_cluster(fb, nk * tx);
          for (int hk = 0; hk < nk; ++hk) {
            const uint32_t slot = s * kps + hk;
            const int kx = (kb + hk) * kBK;
            if (p.l2hint >= 2)
              tma_load_2d_pair_hint(smem_u32(sA + slot * kAStageP), &tmA, kx, arow, fb, pol_a);
            else
              tma_load_2d_pair(smem_u32(sA + slot * kAStageP), &tmA, kx, arow, fb);
            if (p.l2hint >= 1)
              tma_load_2d_pair_hint(smem_u32(sB + slot * kBStageP), mb, kx, brow, fb, pol_b);
            else
              tma_load_2d_pair(smem_u32(sB + slot * kBStageP), mb, kx, brow, fb);
          }
        }
      }
      // unwinding (leader): the last fill of every stage, both CTAs' halves,
      // has landed once the leader's full barrier for it completes
      if (leader) {
        for (uint32_t s = 0; s < nst; ++s) {
          if (it > s) {
            const uint32_t last = ((it - 1 - s) / nst) * nst + s;
            mbar_wait(full0 + 8 * s, (last / nst) & 1, p.err, kDevWaitDrain);
          }
        }
      }
    }
  } else if (w == 1) {
    // ---------------- MMA issuer (leader only) ----------------
    if (lane_id() == 0) {
      if (leader) {
        const uint32_t idesc_full = I8 ? idesc_s8(256, 256) : idesc_bf16(256, 256);
        const uint32_t idesc_half = I8 ? idesc_s8(256, 128) : idesc_bf16(256, 128);
        uint32_t it = 0;
        int lt = 0;
        bool ok = true;
        for (int t = pair; t < n_tiles && ok; t += n_pairs, ++lt) {
          const uint32_t idesc = t < p.n_full ? idesc_full : idesc_half;
          const uint32_t acc = lt & 1, aph = (lt >> 1) & 1;
          if (!mbar_wait_cluster_probe(acce0 + 8 * acc, aph ^ 1, p.err, kDevWaitAccEmpty)) break;
          tc_fence_after();
          const uint32_t d_tmem = tmem_base + acc * 256;
          for (int kb = 0; kb < p.n_kblk; kb += kps, ++it) {
            const uint32_t s = it % nst, ph = (it / nst) & 1;
            if (!mbar_wait_probe(full0 + 8 * s, ph, p.err, kDevWaitFull)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const int nk = min(kps, p.n_kblk - kb);
            for (int hk = 0; hk < nk; ++hk) {
              const uint32_t slot = s * kps + hk;
              const uint32_t a0 = smem_u32(sA + slot * kAStageP);
              const uint32_t b0 = smem_u32(sB + slot * kBStageP);
#pragma unroll
              for (int k = 0; k < 4; ++k) {
                const uint64_t ad = smem_desc_sw128(a0 + k * 32);
                const uint64_t bd = smem_desc_sw128(b0 + k * 32);
                if constexpr (I8)
                  mma_i8_pair(d_tmem, ad, bd, idesc, ((kb + hk) | k) != 0);
                else
                  mma_bf16_pair(d_tmem, ad, bd, idesc, ((kb + hk) | k) != 0);
              }
            }
            mma_commit_pair_mc(empty0 + 8 * s, 0x3);
          }
          if (!ok) break;
          mma_commit_pair_mc(accf0 + 8 * acc, 0x3);
        }
        mma_commit_pair_mc(drain, 0x3);
      }
      // both CTAs: every MMA that writes this CTA's TMEM has completed
      mbar_wait(drain, 0, p.err, kDevWaitDrain);
    }
  } else {
    // ---------------- epilogue (warps 2..5, both CTAs) ----------------
    const int wq = (int)(w & 3);
    const int r_in = 128 * (int)rank + wq * 32 + (int)lane_id();
    const uint32_t acce_leader0 = mapa_shared(acce0, 0);
    int lt = 0;
    for (int t = pair; t < n_tiles; t += n_pairs, ++lt) {
      const TileIdx ti = tile_at(p, t);
      const Unit u = unit_at(p, ti.unit);
      const int nb = ti.nb;
      const bool half = ti.half >= 0;
      const uint32_t acc = lt & 1, aph = (lt >> 1) & 1;
      if (!mbar_wait(accf0 + 8 * acc, aph, p.err, kDevWaitAccFull)) break;
      tc_fence_after();
      const int row = u.m0 + r_in;
      const bool row_ok = row >= u.row_lo && row < u.row_hi;
      const uint32_t tb = tmem_base + acc * 256 + ((uint32_t)(wq * 32) << 16);
      if constexpr (EPI == kEpiSwiglu) {
        // accumulator columns [0, gw) are gate rows, [gw, 2 gw) the matching up rows
        const int nout = p.N / 2;
        const int gw = half ? 64 : 128;
        const int gsub = half ? 64 * ti.half : 0;
        __nv_bfloat16* yrow = reinterpret_cast<__nv_bfloat16*>(p.y) + (long)row * p.ldy;
#pragma unroll 1
        for (int c = 0; c < gw / 32; ++c) {
          float g[32], v[32];
          const int gc = nb * 256 + gsub + c * 32;
          chunk_values<I8>(tb + c * 32, g, p, row, row_ok, gc, u.expert);
          chunk_values<I8>(tb + gw + c * 32, v, p, row, row_ok, gc + 128, u.expert);
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const float gg = bfround(g[i]), uu = bfround(v[i]);
            g[i] = __fdividef(gg, 1.0f + __expf(-gg)) * uu;
          }
          const int oc = nb * 128 + gsub + c * 32;
          if (row_ok) store_row32(yrow + oc, g, oc, nout);
        }
      } else if constexpr (EPI == kEpiTpReduce) {
        // Row-parallel product over tensor-parallel ranks.
        // 1) this rank's partial, rounded to bf16 (the exchange's dominant
        //    bytes halved), -> the owner's inbox plane [rank]. A warp's 32
        //    rows x 32 columns of a chunk go through its 4 KB of shared
        //    memory (XOR-swizzled rows) so that every global store
        //    instruction writes 256 contiguous bytes over NVLink.
        const TpPeers& tp = p.tp;
        const int owner = nb % tp.size;
        const int nbo = p.n_nblk / tp.size;
        const long slot = (long)ti.unit * nbo + nb / tp.size;
        const int lane = (int)lane_id();
        float* wsm = tp_stage + wq * 1024;   // [32 rows][32 floats]
        // chunk c of this warp's rows: plane + ((slot*2 + cta)*8 + c)*4096 + (32 wq)*32
        const long tile_off = (slot * 2 + rank) * 8 * 4096 + wq * 32 * 32;
        __nv_bfloat16* mine = tp.inbox[owner] + (long)tp.rank * tp.plane + tile_off;
#pragma unroll 1
        for (int c = 0; c < 8; ++c) {
          float v[32];
          chunk_values<I8>(tb + c * 32, v, p, row, row_ok, nb * 256 + c * 32, u.expert);
#pragma unroll
          for (int k = 0; k < 8; ++k)
            *reinterpret_cast<float4*>(wsm + lane * 32 + ((k ^ (lane & 7)) << 2)) =
                make_float4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
          __syncwarp();
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const int r = 4 * k + (lane >> 3), q4 = lane & 7;
            const float4 f = *reinterpret_cast<const float4*>(wsm + r * 32 + ((q4 ^ (r & 7)) << 2));
            *reinterpret_cast<uint2*>(mine + c * 4096 + r * 32 + q4 * 4) =
                make_uint2(pack_bf2(f.x, f.y), pack_bf2(f.z, f.w));
          }
          __syncwarp();
        }
        tc_fence_before();
        mbar_arrive_cluster(acce_leader0 + 8 * acc);
        named_bar_sync(1, 128);   // this CTA's 128 rows are stored
        unsigned long long* arrive = tp.arrive[owner] + 2 * (long)t + rank;
        if (owner != tp.rank) {
          if (threadIdx.x == 64) {
            __threadfence_system();
            red_release_sys_add(arrive, 1ull);
          }
          continue;
        }
        // 2) owner: wait for the other ranks' partials of these rows, then
        //    x = bf16(x + bf16(f32 sum of the planes)) into every rank's x.
        //    Lanes run along the columns: each plane read is 256 contiguous
        //    bytes, each x store 64 bytes of a row.
        if (threadIdx.x == 64) {
          wait_counter_sys(arrive, (unsigned long long)(tp.size - 1), p.err, kDevWaitPeer);
          *arrive = 0ull;   // ready for the next pass: no rank adds to it before done below
        }
        named_bar_sync(1, 128);
        const __nv_bfloat16* own = tp.inbox[tp.rank] + tile_off;
        const int wrow0 = u.m0 + 128 * (int)rank + wq * 32;   // this warp's first row
        const int q4 = lane & 7;
        // two chunks per pass: 16 independent loads per plane in flight
        // (a serial load -> add -> store chain per element made this epilogue
        // latency-bound)
#pragma unroll 1
        for (int c = 0; c < 8; c += 2) {
          float4 acc4[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) acc4[i] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll 1
          for (int q = 0; q < tp.size; ++q) {
            const __nv_bfloat16* base = own + q * tp.plane + c * 4096;
            uint2 f[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const int r = 4 * (i & 7) + (lane >> 3);
              f[i] = __ldcg(reinterpret_cast<const uint2*>(base + (i >> 3) * 4096 + r * 32 + q4 * 4));
            }
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const float2 a = unpack_bf2(f[i].x), b = unpack_bf2(f[i].y);
              acc4[i].x += a.x;
              acc4[i].y += a.y;
              acc4[i].z += b.x;
              acc4[i].w += b.y;
            }
          }
          const __nv_bfloat16* xme = static_cast<const __nv_bfloat16*>(tp.x[tp.rank]);
          uint2 xr[16];
          bool okr[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int grow = wrow0 + 4 * (i & 7) + (lane >> 3);
            okr[i] = grow >= u.row_lo && grow < u.row_hi;
            const long xo = (long)grow * p.N + nb * 256 + (c + (i >> 3)) * 32 + q4 * 4;
            xr[i] = okr[i] ? __ldcg(reinterpret_cast<const uint2*>(xme + xo)) : make_uint2(0u, 0u);
          }
          uint2 o2[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float2 x01 = unpack_bf2(xr[i].x), x23 = unpack_bf2(xr[i].y);
            o2[i] = make_uint2(pack_bf2(x01.x + bfround(acc4[i].x), x01.y + bfround(acc4[i].y)),
                               pack_bf2(x23.x + bfround(acc4[i].z), x23.y + bfround(acc4[i].w)));
          }
#pragma unroll 1
          for (int q = 0; q < tp.size; ++q) {
            __nv_bfloat16* xq = static_cast<__nv_bfloat16*>(tp.x[q]);
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const int grow = wrow0 + 4 * (i & 7) + (lane >> 3);
              const long xo = (long)grow * p.N + nb * 256 + (c + (i >> 3)) * 32 + q4 * 4;
              if (okr[i]) *reinterpret_cast<uint2*>(xq + xo) = o2[i];
            }
          }
        }
        named_bar_sync(1, 128);   // every rank's copy of these rows is stored
        if (threadIdx.x == 64) {
          __threadfence_system();
          for (int q = 0; q < tp.size; ++q) red_release_sys_add(tp.done[q], 1ull);
        }
        continue;
      } else {
        const int n0 = nb * 256 + (half ? 128 * ti.half : 0);
        const int nchunk = half ? 4 : 8;
        __nv_bfloat16* yrow = reinterpret_cast<__nv_bfloat16*>(p.y) + (long)row * p.ldy;
        // the residual row is fetched one 32-column chunk ahead, so its load
        // latency overlaps the previous chunk (whole, aligned chunks only)
        const __nv_bfloat16* rrow = EPI == kEpiResid ? p.resid + (long)row * p.ldr : nullptr;
        const bool pre = EPI == kEpiResid && row_ok && n0 + nchunk * 32 <= p.N &&
                         (reinterpret_cast<uintptr_t>(rrow + n0) & 15) == 0 && (p.ldr & 7) == 0;
        uint4 rcur[4] = {}, rnext[4] = {};
        if (pre) {
#pragma unroll
          for (int q = 0; q < 4; ++q) rcur[q] = reinterpret_cast<const uint4*>(rrow + n0)[q];
        }
#pragma unroll 1
        for (int c = 0; c < nchunk; ++c) {
          float v[32];
          const int col0 = n0 + c * 32;
          if (pre && c + 1 < nchunk) {
#pragma unroll
            for (int q = 0; q < 4; ++q)
              rnext[q] = reinterpret_cast<const uint4*>(rrow + col0 + 32)[q];
          }
          chunk_values<I8>(tb + c * 32, v, p, row, row_ok, col0, u.expert);
          if (!row_ok || col0 >= p.N) continue;
          if (p.bias != nullptr) {
            const __nv_bfloat16* b = p.bias + (long)u.expert * p.N + col0;
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (col0 + i < p.N) v[i] += bf2f(b[i]);
          }
          if constexpr (EPI == kEpiResid) {
            float rr[32];
            if (pre) {
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                const float2 a = unpack_bf2(rcur[q].x), b = unpack_bf2(rcur[q].y),
                             cc = unpack_bf2(rcur[q].z), d = unpack_bf2(rcur[q].w);
                rr[q * 8 + 0] = a.x; rr[q * 8 + 1] = a.y; rr[q * 8 + 2] = b.x;
                rr[q * 8 + 3] = b.y; rr[q * 8 + 4] = cc.x; rr[q * 8 + 5] = cc.y;
                rr[q * 8 + 6] = d.x; rr[q * 8 + 7] = d.y;
                rcur[q] = rnext[q];
              }
            } else {
              load_row32(rrow + col0, rr, col0, p.N);
            }
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = rr[i] + bfround(v[i]);
          }
          if constexpr (EPI == kEpiStoreF32)
            store_row32_f32(reinterpret_cast<float*>(p.y) + (long)row * p.ldy + col0, v, col0, p.N);
          else
            store_row32(yrow + col0, v, col0, p.N);
        }
      }
      tc_fence_before();
      mbar_arrive_cluster(acce_leader0 + 8 * acc);
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();   // the peer's smem and TMEM stay alive until the pair is done
  if (w == 0) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, 512);
  }
}

// ---------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn()
{
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

struct MapKey {
  const void* ptr;
  uint64_t rows, cols;
  uint32_t box_rows;
  int elsize;
  bool operator==(const MapKey& o) const
  {
    return ptr == o.ptr && rows == o.rows && cols == o.cols && box_rows == o.box_rows &&
           elsize == o.elsize;
  }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const
  {
    return std::hash<const void*>()(k.ptr) ^ (k.rows * 1315423911ull) ^ (k.cols << 7) ^
           ((uint64_t)k.box_rows << 40) ^ ((uint64_t)k.elsize << 56);
  }
};

}  // namespace

// A 2-D [rows][cols] row-major tensor (elsize 2 = bf16, 1 = int8), box of
// 128 bytes x box_rows, 128-byte swizzle, zero fill out of bounds. Cached:
// encoding costs microseconds and a layer calls the same maps every pass.
int make_tma_2d(CUtensorMap* out, const void* ptr, uint64_t rows, uint64_t cols, uint32_t box_rows,
             int elsize, std::string* err)
{
  static std::mutex mu;
  static std::unordered_map<MapKey, CUtensorMap, MapKeyHash> cache;
  const MapKey key{ptr, rows, cols, box_rows, elsize};
  {
    std::lock_guard<std::mutex> g(mu);
    auto it = cache.find(key);
    if (it != cache.end()) {
      *out = it->second;
      return 0;
    }
  }
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) {
    *err = "cuTensorMapEncodeTiled is unavailable (driver too old?)";
    return 1;
  }
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols * (cuuint64_t)elsize};
  const cuuint32_t box[2] = {(cuuint32_t)(128 / elsize), box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r =
      fn(out, elsize == 2 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8, 2,
         const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
         CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    *err = "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")";
    return 1;
  }
  std::lock_guard<std::mutex> g(mu);
  if (cache.size() > 4096) cache.clear();
  cache.emplace(key, *out);
  return 0;
}

namespace {

template <bool I8, int EPI>
int launch_one(const CUtensorMap& ma, const CUtensorMap& mb, const Params& p, int grid,
               cudaStream_t st)
{
  static std::atomic<uint64_t> attr_set;
  auto k = gemm_tc_kernel<I8, EPI>;
  if (!smem_attr_once(k, kSmemBytes, attr_set)) return 2;
  k<<<grid, kThreads, kSmemBytes, st>>>(ma, mb, p);
  return cudaGetLastError() == cudaSuccess ? 0 : 2;
}

// U15_GEMM_NO_SPLIT=1 keeps every tile full width (A/B measurement).
bool no_split()
{
  static const bool v = [] {
    const char* e = std::getenv("U15_GEMM_NO_SPLIT");
    return e != nullptr && *e != '0';
  }();
  return v;
}

// Persistent grid for the CTA-pair kernel: as many pairs as can be resident
// at once. Not every SM has a usable partner, so this can be fewer than
// SMs / 2; launching more pairs than fit would run the excess pairs'
// whole tile lists after the others and double the kernel's time.
template <bool I8, int EPI>
int launch_pair(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mbh, Params p,
                int tiles, cudaStream_t st, bool allow_split = true)
{
  static std::atomic<uint64_t> attr_set;
  static std::atomic<int> max_pairs_dev[64];   // resident pairs, per device (0: not yet known)
  auto k = gemm_tc_pair_kernel<I8, EPI>;
  constexpr int smem = EPI == kEpiTpReduce ? kSmemPTp : kSmemP;
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (!smem_attr_once(k, smem, attr_set)) return 2;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 2;
  int max_pairs = max_pairs_dev[dev & 63].load(std::memory_order_relaxed);
  if (max_pairs <= 0) {
    cfg.gridDim = dim3(2);
    if (cudaOccupancyMaxActiveClusters(&max_pairs, k, &cfg) != cudaSuccess || max_pairs <= 0)
      max_pairs = 64;
    max_pairs_dev[dev & 63].store(max_pairs, std::memory_order_relaxed);
  }
  const int pairs = std::min(tiles, max_pairs);
  // Split tail: when the last round of the persistent schedule would leave
  // at least half the pairs idle, its tiles run as half-width tiles, which
  // all fit in one round of half the length.
  const int rest = tiles % pairs;
  p.n_full = (allow_split && rest > 0 && 2 * rest <= pairs && !no_split()) ? tiles - rest : tiles;
  cfg.gridDim = dim3(2 * pairs);
  cudaLaunchAttribute attrs[2] = {attr[0], {}};
  attrs[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attrs[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attrs;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, k, ma, mb, mbh, p) == cudaSuccess ? 0 : 2;
}

// Which GEMM variant serves a call: the CTA pair by default, the single-SM
// kernel when U15_GEMM_SINGLE is set (A/B measurement) or for tiny M.
bool use_pair(int M)
{
  static const bool single = [] {
    const char* e = std::getenv("U15_GEMM_SINGLE");
    return e != nullptr && *e != '0';
  }();
  return !single && M > 128;
}

}  // namespace

bool pdl_enabled()
{
  const char* e = std::getenv("U15_PDL");
  return e == nullptr || *e != '0';
}

int gemm_tc(const GemmArgs& a, cudaStream_t st, std::string* err)
{
  if (a.M <= 0 || a.N <= 0 || a.K <= 0) {
    *err = "gemm: M, N and K must be positive";
    return 1;
  }
  const int es = a.int8 ? 1 : 2;
  if ((a.K * es) % 16 != 0) {
    *err = "gemm: K * element size must be a multiple of 16 bytes (TMA row stride)";
    return 1;
  }
  if (a.epilogue == kEpiSwiglu && (a.N % 256) != 0) {
    *err = "gemm: the SwiGLU epilogue needs N (gate+up rows) to be a multiple of 256";
    return 1;
  }
  if (a.int8 && (a.s_tok == nullptr || a.s_ch == nullptr)) {
    *err = "gemm: int8 needs the per-token and per-channel scales";
    return 1;
  }
  if (a.epilogue == kEpiResid && a.resid == nullptr) {
    *err = "gemm: the residual epilogue needs a residual input";
    return 1;
  }
  const bool tp = a.epilogue == kEpiTpReduce;
  if (tp && (a.tp == nullptr || a.tp->size < 2 || a.tp->size > kMaxTp || a.N % (256 * a.tp->size) ||
             a.M > a.tp->rows)) {
    *err = "gemm: the tensor-parallel epilogue needs its peers, N a multiple of 256 x ranks "
           "and M within the peers' buffers";
    return 1;
  }
  Params p{};
  p.M = a.M;
  p.N = a.N;
  p.K = a.K;
  p.y = a.y;
  p.ldy = a.ldy > 0 ? a.ldy : (a.epilogue == kEpiSwiglu ? a.N / 2 : a.N);
  p.resid = static_cast<const __nv_bfloat16*>(a.resid);
  p.ldr = a.ldr > 0 ? a.ldr : a.N;
  p.bias = static_cast<const __nv_bfloat16*>(a.bias);
  p.s_tok = a.s_tok;
  p.s_ch = a.s_ch;
  p.acc_dump = a.acc_dump;
  p.err = a.dev_err;
  if (tp) p.tp = *a.tp;

  // Units: 128-row blocks intersected with the routing segments.
  int nseg = a.nseg;
  int off1[2] = {0, a.M}, ex1[1] = {0};
  const int* off = a.seg_off;
  const int* ex = a.seg_expert;
  if (nseg <= 0 || off == nullptr || ex == nullptr) {
    nseg = 1;
    off = off1;
    ex = ex1;
  }
  if (off[0] != 0 || off[nseg] != a.M) {
    *err = "gemm: segments must cover [0, M)";
    return 1;
  }
  const bool pair = tp || use_pair(a.M);   // the fused TP epilogue exists in the pair kernel
  const int bm = pair ? 256 : kBM;
  if (nseg > kMaxSeg) {
    *err = "gemm: at most 8 routing segments";
    return 1;
  }
  // units segment-major: a block that straddles a boundary appears once per
  // segment and each pass stores only its own rows
  p.unit_bm = bm;
  p.nseg = nseg;
  int n_units = 0;
  for (int s = 0; s < nseg; ++s) {
    if (off[s + 1] < off[s]) {
      *err = "gemm: segment offsets must be non-decreasing";
      return 1;
    }
    if (ex[s] < 0 || ex[s] >= a.n_experts) {
      *err = "gemm: segment expert out of range";
      return 1;
    }
    p.seg_off[s] = off[s];
    p.seg_expert[s] = ex[s];
    p.unit_start[s] = n_units;
    if (off[s + 1] > off[s]) n_units += (off[s + 1] + bm - 1) / bm - off[s] / bm;
  }
  p.seg_off[nseg] = off[nseg];
  p.unit_start[nseg] = n_units;
  p.n_units = n_units;
  p.n_nblk = (a.N + kBN - 1) / kBN;
  p.n_full = n_units * p.n_nblk;
  if (tp && (long)n_units * (p.n_nblk / a.tp->size) * 2 * 8 * 4096 > a.tp->plane) {
    *err = "gemm: the pass needs more tile slots than the tensor-parallel planes hold";
    return 1;
  }
  p.group = n_units;
  {
    // U15_GEMM_GROUP (read per launch, for A/B checks): row units per group
    const char* e = std::getenv("U15_GEMM_GROUP");
    const int grp = e != nullptr ? std::atoi(e) : 0;
    if (grp > 0 && grp < n_units) p.group = grp;
  }
  {
    // U15_GEMM_L2HINT (read per launch, for A/B checks): the L2 policy of
    // the pair kernel's operand loads
    const char* e = std::getenv("U15_GEMM_L2HINT");
    p.l2hint = e != nullptr ? std::atoi(e) : kDefaultL2Hint;
  }
  {
    // U15_GEMM_KPS (read per launch, for A/B checks): k-blocks per stage of
    // the pair kernel's ring
    const char* e = std::getenv("U15_GEMM_KPS");
    const int v = e != nullptr ? std::atoi(e) : 0;
    p.kps = v == 1 || v == 2 || v == 3 ? v : kDefaultKps;
  }
  const int bk = a.int8 ? 128 : 64;
  p.n_kblk = (a.K + bk - 1) / bk;

  CUtensorMap ma, mb, mbh;
  if (make_tma_2d(&ma, a.x, (uint64_t)a.M, (uint64_t)a.K, kBM, es, err)) return 2;
  if (make_tma_2d(&mb, a.w, (uint64_t)a.N * a.n_experts, (uint64_t)a.K, pair ? 128 : kBN, es,
                  err))
    return 2;
  if (pair && make_tma_2d(&mbh, a.w, (uint64_t)a.N * a.n_experts, (uint64_t)a.K, 64, es, err))
    return 2;

  const int tiles = p.n_units * p.n_nblk;
  const int sms = a.num_sms > 0 ? a.num_sms : 148;
  int rc;
  if (a.out_tiles != nullptr) *a.out_tiles = tiles;
  if (tp) {
    // every rank enumerates the same full-width tiles (no split tail): the
    // arrival counters are indexed by tile
    rc = a.int8 ? launch_pair<true, kEpiTpReduce>(ma, mb, mbh, p, tiles, st, false)
                : launch_pair<false, kEpiTpReduce>(ma, mb, mbh, p, tiles, st, false);
    if (rc) *err = "gemm (tensor-parallel): kernel launch failed";
    return rc;
  }
  if (pair) {
    if (a.int8) {
      rc = a.epilogue == kEpiResid    ? launch_pair<true, kEpiResid>(ma, mb, mbh, p, tiles, st)
           : a.epilogue == kEpiSwiglu ? launch_pair<true, kEpiSwiglu>(ma, mb, mbh, p, tiles, st)
           : a.epilogue == kEpiStoreF32 ? launch_pair<true, kEpiStoreF32>(ma, mb, mbh, p, tiles, st)
                                      : launch_pair<true, kEpiStore>(ma, mb, mbh, p, tiles, st);
    } else {
      rc = a.epilogue == kEpiResid    ? launch_pair<false, kEpiResid>(ma, mb, mbh, p, tiles, st)
           : a.epilogue == kEpiSwiglu ? launch_pair<false, kEpiSwiglu>(ma, mb, mbh, p, tiles, st)
           : a.epilogue == kEpiStoreF32 ? launch_pair<false, kEpiStoreF32>(ma, mb, mbh, p, tiles, st)
                                      : launch_pair<false, kEpiStore>(ma, mb, mbh, p, tiles, st);
    }
    if (rc) *err = "gemm (CTA pair): kernel launch failed";
    return rc;
  }
  const int grid = std::min(tiles, sms);
  if (a.int8) {
    rc = a.epilogue == kEpiResid    ? launch_one<true, kEpiResid>(ma, mb, p, grid, st)
         : a.epilogue == kEpiSwiglu ? launch_one<true, kEpiSwiglu>(ma, mb, p, grid, st)
         : a.epilogue == kEpiStoreF32 ? launch_one<true, kEpiStoreF32>(ma, mb, p, grid, st)
                                    : launch_one<true, kEpiStore>(ma, mb, p, grid, st);
  } else {
    rc = a.epilogue == kEpiResid    ? launch_one<false, kEpiResid>(ma, mb, p, grid, st)
         : a.epilogue == kEpiSwiglu ? launch_one<false, kEpiSwiglu>(ma, mb, p, grid, st)
         : a.epilogue == kEpiStoreF32 ? launch_one<false, kEpiStoreF32>(ma, mb, p, grid, st)
                                    : launch_one<false, kEpiStore>(ma, mb, p, grid, st);
  }
  if (rc) *err = "gemm: kernel launch failed";
  return rc;
}

namespace {
__global__ void tp_wait_kernel(const unsigned long long* done, unsigned long long target,
                               unsigned* err)
{
  if (threadIdx.x == 0) wait_counter_sys(done, target, err, kDevWaitPeer);
}
}  // namespace

int launch_tp_wait(const unsigned long long* done, unsigned long long target, unsigned* err,
                   cudaStream_t st)
{
  tp_wait_kernel<<<1, 32, 0, st>>>(done, target, err);
  return cudaGetLastError() == cudaSuccess ? 0 : 2;
}

}  // namespace u15
