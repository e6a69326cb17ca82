// Device-side building blocks shared by every kernel in libu15c: bf16
// packing, the device error word, and thin inline-PTX wrappers for the
// sm_100a machinery (mbarrier, TMA bulk-tensor copies, tcgen05 MMA/TMEM).
//
// Every wait in this library is BOUNDED: a spin on an mbarrier gives up
// after the device's wait limit (U15_WAIT_LIMIT_NS, 2 s, unless
// u15c_set_wait_limit set another) of %globaltimer time, records where it
// gave up in the caller-visible error word and returns false, and the
// kernel unwinds (waiting, again bounded, for its own copies and MMAs in
// flight) instead of hanging the GPU. The host reads the word with
// u15c_device_status().
//
// The status block of a device is 16 bytes: word 0 the first error code,
// bytes 8-15 the wait limit in ns (0 = U15_WAIT_LIMIT_NS).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#ifndef U15_WAIT_LIMIT_NS
#define U15_WAIT_LIMIT_NS 2000000000ull   // 2 s: legitimate waits are < 1 ms
#endif

namespace u15 {

// Error codes written into the device error word (first error sticks).
enum DevErr : unsigned {
  kDevOk = 0,
  kDevWaitFull = 0x101,      // MMA waited too long for a TMA stage
  kDevWaitEmpty = 0x102,     // producer waited too long for a free stage
  kDevWaitAccFull = 0x103,   // epilogue waited too long for an accumulator
  kDevWaitAccEmpty = 0x104,  // MMA waited too long for the epilogue
  kDevWaitDrain = 0x105,     // unwinding waited too long for in-flight work
  kDevWaitPeer = 0x106,      // a tensor-parallel rank's partial or result did not arrive
  kDevBadArg = 0x201,        // a kernel saw an argument it cannot serve
};

__device__ __forceinline__ void dev_fail(unsigned* err, unsigned code)
{
  if (err != nullptr) atomicCAS(err, 0u, code);
}

// The wait limit of the device whose status block `err` is (read once per
// wait that outlasts its fast tries).
__device__ __forceinline__ uint64_t wait_limit_ns(const unsigned* err)
{
  if (err == nullptr) return U15_WAIT_LIMIT_NS;
  const uint64_t v = *reinterpret_cast<const volatile uint64_t*>(err + 2);
  return v != 0 ? v : U15_WAIT_LIMIT_NS;
}

// ---------------------------------------------------------------------
// bf16
// ---------------------------------------------------------------------
__device__ __forceinline__ float bf2f(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ __nv_bfloat16 f2bf(float v) { return __float2bfloat16_rn(v); }
// Round a float through bf16 and back (the reference's storage rounding).
__device__ __forceinline__ float bfround(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

__device__ __forceinline__ uint32_t pack_bf2(float lo, float hi)
{
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ float2 unpack_bf2(uint32_t v)
{
  __nv_bfloat162 h = *reinterpret_cast<__nv_bfloat162*>(&v);
  return __bfloat1622float2(h);
}

// Symmetric int8 codes of v at scale s = RN(amax / 127): rn_even(v / s)
// clamped to +-127, equal to the IEEE division rule's codes bit for bit.
// With r = RN(1 / s) (quant_recip), the exact product p = v * r and the exact
// quotient v / s differ by at most |v / s| * 2^-24 <= 7.6e-6, and the IEEE
// quotient by as much again, so p rounds to the same integer as the quotient
// unless p lies within 1.6e-5 of a half-integer. tm = fma(v, r, 1.5 * 2^23)
// rounds p to the nearest integer k (even on ties), and
// d = fma(v, r, 1.5 * 2^23 - tm) is p - k rounded once (|d| <= 0.5), so
// |d| > 0.4999 marks the values within 1e-4 of a half-integer; a group of 8
// holding one takes the division itself. For a normal s, |v| <= amax keeps
// |p| <= 127 * (1 + 2^-23), so the fast code never leaves [-127, 127]; a
// subnormal s (amax < 127 * 2^-126) can be rounded far enough that v / s
// passes 127, so its rows take the clamped division for every value (their
// r = 1 / s is above 2^126). s = 0 (an all-zero row) has r = 0 and codes 0.
// The low byte of tm's bit pattern is the code's low byte.
__device__ __forceinline__ float quant_recip(float s) { return s > 0.0f ? __fdiv_rn(1.0f, s) : 0.0f; }

__device__ __forceinline__ uint32_t code_bits(float v, float r, bool& tie)
{
  const float tm = __fmaf_rn(v, r, 12582912.0f);
  const float d = __fmaf_rn(v, r, 12582912.0f - tm);
  tie |= fabsf(d) > 0.4999f;
  return __float_as_uint(tm);
}

__device__ __forceinline__ uint32_t pack_low_bytes(uint32_t a, uint32_t b, uint32_t c, uint32_t d)
{
  return __byte_perm(__byte_perm(a, b, 0x0040), __byte_perm(c, d, 0x0040), 0x5410);
}

// codes of v[0..8) as 8 bytes, v[0] lowest
__device__ __forceinline__ uint2 quant8(const float* v, float s, float r)
{
  bool tie = r > 8.5070592e37f;   // 2^126: the scale is subnormal
  uint32_t c[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) c[i] = code_bits(v[i], r, tie);
  if (tie) {   // rare: the IEEE quotient of every value of the group
#pragma unroll
    for (int i = 0; i < 8; ++i)
      c[i] = (uint32_t)max(-127, min(127, __float2int_rn(__fdiv_rn(v[i], s))));
  }
  return make_uint2(pack_low_bytes(c[0], c[1], c[2], c[3]), pack_low_bytes(c[4], c[5], c[6], c[7]));
}

// ---------------------------------------------------------------------
// timers / smem addresses
// ---------------------------------------------------------------------
__device__ __forceinline__ uint64_t globaltimer()
{
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// ---------------------------------------------------------------------
// cross-GPU signalling (tensor parallelism over peer memory): 64-bit
// counters in a rank's memory, incremented by its peers with release
// semantics at system scope, read with acquire semantics.
// ---------------------------------------------------------------------
__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p)
{
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_sys_add(unsigned long long* p, unsigned long long v)
{
  asm volatile("red.release.sys.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
// Bounded wait until *p >= target (U15_WAIT_LIMIT_NS): false, with `code` in
// the status word, when it runs out.
__device__ __forceinline__ bool wait_counter_sys(const unsigned long long* p,
                                                 unsigned long long target, unsigned* err,
                                                 unsigned code);
// named barrier over `threads` threads (a multiple of 32) of the CTA
__device__ __forceinline__ void named_bar_sync(int id, int threads)
{
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

__device__ __forceinline__ uint32_t smem_u32(const void* p)
{
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ uint32_t warp_id() { return threadIdx.x >> 5; }
__device__ __forceinline__ uint32_t lane_id() { return threadIdx.x & 31; }

// ---------------------------------------------------------------------
// Programmatic dependent launch. A kernel launched with the PDL attribute
// may be scheduled while the previous kernel of its stream still runs (on
// SMs that kernel has freed); griddep_wait blocks until that kernel has
// completed and its writes are visible, and is a no-op for a kernel launched
// without the attribute. griddep_launch lets the next kernel be scheduled
// once every CTA of this one has issued it (or exited).
// ---------------------------------------------------------------------
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch()
{
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count)
{
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_barrier_init()
{
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar)
{
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes)
{
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity)
{
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Whether the phase with parity `parity` has completed, without waiting.
__device__ __forceinline__ bool mbar_test(uint32_t bar, uint32_t parity)
{
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Wait until the phase with parity `parity` has completed. Bounded: gives up
// after U15_WAIT_LIMIT_NS, records `code` and returns false.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, unsigned* err,
                                          unsigned code)
{
#pragma unroll 1
  for (int i = 0; i < 128; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer(), lim = wait_limit_ns(err);
#pragma unroll 1
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer() - t0 > lim) {
      dev_fail(err, code);
      return false;
    }
  }
}

// mbar_wait for a thread whose barrier is usually complete already: one
// non-blocking probe first. A tcgen05.mma issuer's try_wait returned ~200
// cycles after its call even on a phase completed long before (a clock
// trace of the attention's issuer); the probe returns in a few.
__device__ __forceinline__ bool mbar_wait_probe(uint32_t bar, uint32_t parity, unsigned* err,
                                                unsigned code)
{
  return mbar_test(bar, parity) || mbar_wait(bar, parity, err, code);
}

__device__ __forceinline__ bool wait_counter_sys(const unsigned long long* p,
                                                 unsigned long long target, unsigned* err,
                                                 unsigned code)
{
  if (ld_acquire_sys(p) >= target) return true;
  const uint64_t t0 = globaltimer(), lim = wait_limit_ns(err);
#pragma unroll 1
  while (true) {
    __nanosleep(64);
    if (ld_acquire_sys(p) >= target) return true;
    if (globaltimer() - t0 > lim) {
      dev_fail(err, code);
      return false;
    }
  }
}

// ---------------------------------------------------------------------
// TMA (cp.async.bulk.tensor), no multicast anywhere in this library
// ---------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* m)
{
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}
// 2-D tiled load of box {x: inner, y: outer} at coordinates (x, y) into
// smem, completing `bytes` on the mbarrier. x * elsize must be a multiple
// of 16 bytes (callers pass multiples of the 128-byte swizzle span).
__device__ __forceinline__ void tma_load_2d(uint32_t smem_dst, const CUtensorMap* m, int x,
                                            int y, uint32_t bar)
{
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_dst),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

// ---------------------------------------------------------------------
// tcgen05: TMEM allocation, MMA, commit, loads
// ---------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t slot_smem, uint32_t ncols)
{
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(slot_smem),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish()
{
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols)
{
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f16 (bf16 inputs, f32 acc).
__device__ __forceinline__ void mma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                         uint32_t idesc, uint32_t accumulate)
{
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// The same for kind::i8 (s8 x s8 -> s32).
__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                       uint32_t idesc, uint32_t accumulate)
{
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on an mbarrier once every tcgen05 op this thread issued so far has
// completed.
__device__ __forceinline__ void mma_commit(uint32_t bar)
{
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

// 32 lanes x 32 bits, 32 consecutive columns: thread i of the warp gets
// row (lane base + i), columns [col, col + 32).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32])
{
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor for a K-major operand tile written by TMA
// with 128-byte swizzle: rows of 128 bytes, 8-row (1024-byte) swizzle atoms
// stacked along M/N. LBO is unused for swizzled K-major layouts (set to 1),
// SBO = 1024 bytes, descriptor version 1 (sm100), layout type 2 = 128B
// swizzle. The tile base must be 1024-byte aligned; stepping K inside the
// 128-byte span advances the start address by the step's byte width.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t smem_addr)
{
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr & 0x3FFFFu) >> 4);   // start address [0,14)
  d |= (uint64_t)1 << 16;                          // LBO (unused) [16,30)
  d |= (uint64_t)(1024 >> 4) << 32;                // SBO [32,46)
  d |= (uint64_t)1 << 46;                          // version [46,48)
  d |= (uint64_t)2 << 61;                          // SWIZZLE_128B [61,64)
  return d;
}

// Instruction descriptor: dense, K-major A and B, M x N tile.
//   c_format [4,6): 1 = f32, 2 = s32
//   a_format [7,10) / b_format [10,13): bf16 = 1 (kind::f16); s8 = 1 (kind::i8)
//   n_dim [17,23) = N >> 3; m_dim [24,29) = M >> 4
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N)
{
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) |
         ((uint32_t)(M >> 4) << 24);
}
__host__ __device__ constexpr uint32_t idesc_s8(int M, int N)
{
  return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) |
         ((uint32_t)(M >> 4) << 24);
}

// ---------------------------------------------------------------------
// CTA pairs (cluster of 2, tcgen05 cta_group::2). The even CTA of a pair is
// the leader: it issues the pair's MMAs, and the barriers the MMA waits on
// (operand-full, accumulator-empty) live in its shared memory.
// ---------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank()
{
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// shared::cluster address of `addr` (a shared::cta address) in CTA `rank`.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank)
{
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_sync()
{
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" :::
                   "memory");
}
// Arrivals on a barrier of either CTA of the pair. Relaxed: a release here
// would fence every earlier memory operation at cluster scope on each call
// (a per-k-block stall for the producer), and neither caller needs one --
// the operand bytes are tracked by the TMA transaction count, and the
// epilogue's TMEM reads have completed (tcgen05.wait::ld) before it arrives.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr)
{
  asm volatile("mbarrier.arrive.relaxed.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx_cluster(uint32_t cluster_addr, uint32_t bytes)
{
  asm volatile("mbarrier.arrive.expect_tx.relaxed.cluster.shared::cluster.b64 _, [%0], %1;" ::"r"(
                   cluster_addr),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_cluster(uint32_t bar, uint32_t parity)
{
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_test_cluster(uint32_t bar, uint32_t parity)
{
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait with cluster-scope acquire (for barriers other CTAs arrive on).
__device__ __forceinline__ bool mbar_wait_cluster(uint32_t bar, uint32_t parity, unsigned* err,
                                                  unsigned code)
{
#pragma unroll 1
  for (int i = 0; i < 128; ++i)
    if (mbar_try_wait_cluster(bar, parity)) return true;
  const uint64_t t0 = globaltimer(), lim = wait_limit_ns(err);
#pragma unroll 1
  while (true) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    if (globaltimer() - t0 > lim) {
      dev_fail(err, code);
      return false;
    }
  }
}
// mbar_wait_cluster with one non-blocking probe first (see mbar_wait_probe).
__device__ __forceinline__ bool mbar_wait_cluster_probe(uint32_t bar, uint32_t parity,
                                                        unsigned* err, unsigned code)
{
  return mbar_test_cluster(bar, parity) || mbar_wait_cluster(bar, parity, err, code);
}
// 2-D tiled load into this CTA's shared memory whose completion is counted
// on an mbarrier of either CTA of the pair (no multicast).
__device__ __forceinline__ void tma_load_2d_pair(uint32_t smem_dst, const CUtensorMap* m, int x,
                                                 int y, uint32_t bar_cluster)
{
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_dst),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(x), "r"(y), "r"(bar_cluster)
      : "memory");
}
// L2 eviction-priority policies for cache-hinted loads: streamed operands
// (read once per launch) go first, reused ones stay.
__device__ __forceinline__ uint64_t l2_evict_first_policy()
{
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
__device__ __forceinline__ uint64_t l2_evict_last_policy()
{
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
// tma_load_2d_pair with an L2 cache policy for the bytes it reads.
__device__ __forceinline__ void tma_load_2d_pair_hint(uint32_t smem_dst, const CUtensorMap* m,
                                                      int x, int y, uint32_t bar_cluster,
                                                      uint64_t policy)
{
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_dst),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(x), "r"(y), "r"(bar_cluster), "l"(policy)
      : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t slot_smem, uint32_t ncols)
{
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(slot_smem),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair()
{
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols)
{
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void mma_bf16_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                              uint32_t idesc, uint32_t accumulate)
{
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void mma_i8_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                            uint32_t idesc, uint32_t accumulate)
{
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on the mbarrier at the same offset in every CTA of `mask` once all
// tcgen05 ops this thread issued have completed.
__device__ __forceinline__ void mma_commit_pair_mc(uint32_t bar, uint16_t mask)
{
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], %1;" ::"r"(bar),
      "h"(mask)
      : "memory");
}

}  // namespace u15
