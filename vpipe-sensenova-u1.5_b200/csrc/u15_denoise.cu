// The device half of the denoise step (Generator::generate's step body,
// src/u15-generator.cc:582-705 of the reference), which the reference runs
// on the host in double over H*W*3 floats after a per-branch GPU->host
// round trip:
//   v   = (x_pred - img) / max(1 - t, t_eps)
//   CFG one of four forms, then an optional renorm (global or per token)
//   img += (t_next - t) * v
// Elementwise work in fp64 as the reference does it; the reductions
// (optimized_scale's dot and norm, the renorm norms) are deterministic
// two-stage sums in fp64 over a fixed grid, so a step is bit-reproducible.
//
// Also the pixel packing the stand-in image path uses: channel-last
// [H][W][3] image <-> [tokens][32*32*3] rows ('nhwpqc', the packing the
// reference uses for z, src/u15-ref.cc patchify_channel_last).
#include "u15_capi_internal.h"
#include "u15_common.cuh"

#include <algorithm>
#include <cmath>
#include <random>

namespace {

constexpr int kRedBlocks = 256;   // fixed partial count: deterministic order
constexpr int kRedThreads = 256;
constexpr int kTok = 32;          // pixels per token side

// form / norm codes (include/u15c.h U15C_CFG_*, U15C_NORM_*)
enum { kCfgNone = 0, kCfgImg = 1, kCfgUnc = 2, kCfgBoth = 3 };
enum { kNormNone = 0, kNormGlobal = 1, kNormChannel = 2, kNormZeroStar = 3 };

__global__ void velocity_kernel(const float* __restrict__ xp, const float* __restrict__ img,
                                float* __restrict__ v, long n, double denom)
{
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) v[i] = (float)(((double)xp[i] - (double)img[i]) / denom);
}

__global__ void euler_kernel(float* __restrict__ img, const float* __restrict__ v, long n,
                             double dt)
{
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) img[i] = (float)((double)img[i] + dt * (double)v[i]);
}

// Stage 1: per-block partial sums of a*b and b*b (a, b may alias).
__global__ void __launch_bounds__(kRedThreads)
    dot2_partial(const float* __restrict__ a, const float* __restrict__ b, long n,
                 double* __restrict__ part)
{
  __shared__ double s0[kRedThreads], s1[kRedThreads];
  double d0 = 0.0, d1 = 0.0;
  for (long i = (long)blockIdx.x * kRedThreads + threadIdx.x; i < n;
       i += (long)kRedBlocks * kRedThreads) {
    const double x = a[i], y = b[i];
    d0 += x * y;
    d1 += y * y;
  }
  s0[threadIdx.x] = d0;
  s1[threadIdx.x] = d1;
  __syncthreads();
  for (int o = kRedThreads / 2; o > 0; o >>= 1) {
    if (threadIdx.x < o) {
      s0[threadIdx.x] += s0[threadIdx.x + o];
      s1[threadIdx.x] += s1[threadIdx.x + o];
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    part[2 * blockIdx.x] = s0[0];
    part[2 * blockIdx.x + 1] = s1[0];
  }
}
// Stage 2: one block sums the partials in a fixed order -> res[0..1].
__global__ void __launch_bounds__(kRedThreads) dot2_final(const double* __restrict__ part, double* res)
{
  __shared__ double s0[kRedThreads], s1[kRedThreads];
  s0[threadIdx.x] = part[2 * threadIdx.x];
  s1[threadIdx.x] = part[2 * threadIdx.x + 1];
  __syncthreads();
  for (int o = kRedThreads / 2; o > 0; o >>= 1) {
    if (threadIdx.x < o) {
      s0[threadIdx.x] += s0[threadIdx.x + o];
      s1[threadIdx.x] += s1[threadIdx.x + o];
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    res[0] = s0[0];
    res[1] = s1[0];
  }
}

// The CFG combination (src/u15-generator.cc:596-660). `res` holds the
// zero-star reduction (dot, |v_unc|^2) when form == UNC and norm == ZERO_STAR.
__global__ void cfg_combine_kernel(const float* __restrict__ vc, const float* __restrict__ vu,
                                   const float* __restrict__ vi, float* __restrict__ out, long n,
                                   int form, int norm, double cfg, double icfg, int step,
                                   const double* __restrict__ res)
{
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const double c = vc[i];
  double r;
  if (form == kCfgImg) {
    const double m = vi[i];
    r = m + cfg * (c - m);
  } else if (form == kCfgUnc) {
    const double u = vu[i];
    if (norm == kNormZeroStar) {
      if (step <= 0) {
        r = 0.0;
      } else {
        const double alpha = res[0] / (res[1] + 1e-8);
        const double a = alpha * u;
        r = a + cfg * (c - a);
      }
    } else {
      r = u + cfg * (c - u);
    }
  } else if (form == kCfgBoth) {
    const double u = vu[i], m = vi[i];
    r = u + cfg * (c - m) + icfg * (m - u);
  } else {
    r = c;
  }
  out[i] = (float)r;
}

// Global renorm: out *= min(1, |vc| / (|out| + 1e-8)); nc[1] = |vc|^2 and
// nv[1] = |out|^2 come from dot2 reductions of (vc, vc) and (out, out).
__global__ void scale_kernel(float* __restrict__ out, long n, const double* __restrict__ nc,
                             const double* __restrict__ nv)
{
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  double sc = sqrt(nc[1]) / (sqrt(nv[1]) + 1e-8);
  if (sc > 1.0) sc = 1.0;
  out[i] = (float)(out[i] * sc);
}

// Per-token renorm (src/u15-generator.cc:668-692): one block per 32x32 token,
// 3072 elements gathered by position from the channel-last image.
__global__ void __launch_bounds__(256)
    channel_norm_kernel(const float* __restrict__ vc, float* __restrict__ out, int W, int tw)
{
  const int tok = blockIdx.x, ty = tok / tw, tx = tok % tw;
  __shared__ double s0[256], s1[256];
  double a = 0.0, b = 0.0;
  for (int e = threadIdx.x; e < kTok * kTok * 3; e += 256) {
    const int y = e / (kTok * 3), rem = e % (kTok * 3);
    const long i = ((long)(ty * kTok + y) * W + tx * kTok) * 3 + rem;
    const double c = vc[i], o = out[i];
    a += c * c;
    b += o * o;
  }
  s0[threadIdx.x] = a;
  s1[threadIdx.x] = b;
  __syncthreads();
  for (int o = 128; o > 0; o >>= 1) {
    if (threadIdx.x < o) {
      s0[threadIdx.x] += s0[threadIdx.x + o];
      s1[threadIdx.x] += s1[threadIdx.x + o];
    }
    __syncthreads();
  }
  double sc = sqrt(s0[0]) / (sqrt(s1[0]) + 1e-8);
  if (sc > 1.0) sc = 1.0;
  for (int e = threadIdx.x; e < kTok * kTok * 3; e += 256) {
    const int y = e / (kTok * 3), rem = e % (kTok * 3);
    const long i = ((long)(ty * kTok + y) * W + tx * kTok) * 3 + rem;
    out[i] = (float)(out[i] * sc);
  }
}

// [H][W][3] f32 <-> [th*tw][32*32*3] bf16 rows, 'nhwpqc' (channel last).
__global__ void patchify_kernel(const float* __restrict__ img, __nv_bfloat16* __restrict__ rows,
                                int W, int tw, long n)
{
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const long tok = i / (kTok * kTok * 3);
  const int e = (int)(i % (kTok * kTok * 3));
  const int y = e / (kTok * 3), rem = e % (kTok * 3);
  const int ty = (int)(tok / tw), tx = (int)(tok % tw);
  rows[i] = __float2bfloat16_rn(img[((long)(ty * kTok + y) * W + tx * kTok) * 3 + rem]);
}
__global__ void unpatchify_kernel(const __nv_bfloat16* __restrict__ rows, float* __restrict__ img,
                                  int W, int tw, long n)
{
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const long tok = i / (kTok * kTok * 3);
  const int e = (int)(i % (kTok * kTok * 3));
  const int y = e / (kTok * 3), rem = e % (kTok * 3);
  const int ty = (int)(tok / tw), tx = (int)(tok % tw);
  img[((long)(ty * kTok + y) * W + tx * kTok) * 3 + rem] = __bfloat162float(rows[i]);
}

inline unsigned nb(long n) { return (unsigned)((n + 255) / 256); }

}  // namespace

using u15::fail;

extern "C" {

size_t u15c_cfg_workspace_bytes(void) { return (size_t)(2 * kRedBlocks + 8) * sizeof(double); }

int u15c_velocity(u15c_stream stream, const float* x_pred, const float* img, float* v, long n,
                  double denom)
{
  if (x_pred == nullptr || img == nullptr || v == nullptr || n < 0 || !(denom > 0.0))
    return fail(U15C_EINVAL, "velocity: bad argument");
  if (n == 0) return U15C_OK;
  velocity_kernel<<<nb(n), 256, 0, static_cast<cudaStream_t>(stream)>>>(x_pred, img, v, n, denom);
  return cudaGetLastError() == cudaSuccess ? U15C_OK : fail(U15C_ECUDA, "velocity: launch failed");
}

int u15c_euler(u15c_stream stream, float* img, const float* v, long n, double dt)
{
  if (img == nullptr || v == nullptr || n < 0) return fail(U15C_EINVAL, "euler: bad argument");
  if (n == 0) return U15C_OK;
  euler_kernel<<<nb(n), 256, 0, static_cast<cudaStream_t>(stream)>>>(img, v, n, dt);
  return cudaGetLastError() == cudaSuccess ? U15C_OK : fail(U15C_ECUDA, "euler: launch failed");
}

int u15c_cfg_combine(u15c_stream stream, const float* v_cond, const float* v_unc,
                     const float* v_img, float* out, int H, int W, int form, int norm, double cfg,
                     double icfg, int step, void* workspace)
{
  if (v_cond == nullptr || out == nullptr || workspace == nullptr || H <= 0 || W <= 0)
    return fail(U15C_EINVAL, "cfg_combine: bad argument");
  if (form < kCfgNone || form > kCfgBoth || norm < kNormNone || norm > kNormZeroStar)
    return fail(U15C_EINVAL, "cfg_combine: unknown form or norm");
  if ((form == kCfgImg || form == kCfgBoth) && v_img == nullptr)
    return fail(U15C_EINVAL, "cfg_combine: this form needs the image-conditioned velocity");
  if ((form == kCfgUnc || form == kCfgBoth) && v_unc == nullptr)
    return fail(U15C_EINVAL, "cfg_combine: this form needs the unconditional velocity");
  if (norm == kNormZeroStar && form != kCfgUnc)
    return fail(U15C_EINVAL, "cfg_combine: cfg_zero_star applies to the unconditional form only");
  if (norm == kNormChannel && (H % kTok || W % kTok))
    return fail(U15C_EINVAL, "cfg_combine: the per-token renorm needs H, W multiples of 32");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const long n = (long)H * W * 3;
  double* part = static_cast<double*>(workspace);
  double* res = part + 2 * kRedBlocks;   // res[0..1]: zero-star / |vc|^2, res[2..3]: |out|^2
  if (form == kCfgUnc && norm == kNormZeroStar) {
    dot2_partial<<<kRedBlocks, kRedThreads, 0, st>>>(v_cond, v_unc, n, part);
    dot2_final<<<1, kRedThreads, 0, st>>>(part, res);
  }
  cfg_combine_kernel<<<nb(n), 256, 0, st>>>(v_cond, v_unc, v_img, out, n, form, norm, cfg, icfg,
                                            step, res);
  if (form != kCfgNone && norm == kNormGlobal) {
    dot2_partial<<<kRedBlocks, kRedThreads, 0, st>>>(v_cond, v_cond, n, part);
    dot2_final<<<1, kRedThreads, 0, st>>>(part, res);
    dot2_partial<<<kRedBlocks, kRedThreads, 0, st>>>(out, out, n, part);
    dot2_final<<<1, kRedThreads, 0, st>>>(part, res + 2);
    scale_kernel<<<nb(n), 256, 0, st>>>(out, n, res, res + 2);
  } else if (form != kCfgNone && norm == kNormChannel) {
    channel_norm_kernel<<<(H / kTok) * (W / kTok), 256, 0, st>>>(v_cond, out, W, W / kTok);
  }
  return cudaGetLastError() == cudaSuccess ? U15C_OK : fail(U15C_ECUDA, "cfg_combine: launch failed");
}

int u15c_patchify(u15c_stream stream, const float* img, void* rows, int H, int W)
{
  if (img == nullptr || rows == nullptr || H % kTok || W % kTok || H <= 0 || W <= 0)
    return fail(U15C_EINVAL, "patchify: H and W must be positive multiples of 32");
  const long n = (long)H * W * 3;
  patchify_kernel<<<nb(n), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      img, static_cast<__nv_bfloat16*>(rows), W, W / kTok, n);
  return cudaGetLastError() == cudaSuccess ? U15C_OK : fail(U15C_ECUDA, "patchify: launch failed");
}

int u15c_unpatchify(u15c_stream stream, const void* rows, float* img, int H, int W)
{
  if (img == nullptr || rows == nullptr || H % kTok || W % kTok || H <= 0 || W <= 0)
    return fail(U15C_EINVAL, "unpatchify: H and W must be positive multiples of 32");
  const long n = (long)H * W * 3;
  unpatchify_kernel<<<nb(n), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(rows), img, W, W / kTok, n);
  return cudaGetLastError() == cudaSuccess ? U15C_OK : fail(U15C_ECUDA, "unpatchify: launch failed");
}


// The start image of a render (Generator::generate, src/u15-generator.cc:394-417):
// pixel space, channel-last [H][W][3], one draw per value in that order from
// std::mt19937_64(seed) through std::normal_distribution<float>(0, 1), each
// scaled in double by the resolution's noise scale and rounded to float --
// the reference's own engine and distribution, so the image is the
// reference's for the same seed wherever the C++ standard library is the
// same (the distribution's algorithm is the library's choice).
int u15c_init_noise(uint64_t seed, double noise_scale, float* out, long n)
{
  if (out == nullptr || n < 0) return u15::fail(U15C_EINVAL, "init_noise: bad output");
  std::mt19937_64 rng(seed);
  std::normal_distribution<float> nd(0.0f, 1.0f);
  for (long i = 0; i < n; ++i) out[i] = (float)(noise_scale * nd(rng));
  return U15C_OK;
}

// GenConfig::init_noise_scale (src/u15-config.cc:106-122): sqrt(L / base)
// times noise_scale for the resolution-dependent modes (its square root
// for dynamic_sqrt), noise_scale itself otherwise; capped at max_value.
int u15c_init_noise_scale(int image_tokens, int mode, double noise_scale, double max_value,
                          int base_seq_len, double* out)
{
  if (out == nullptr || image_tokens < 0 || mode < 0 || mode > 2)
    return u15::fail(U15C_EINVAL, "init_noise_scale: bad argument");
  if (mode == U15C_NOISE_CONSTANT) {
    *out = std::min(noise_scale, max_value);
    return U15C_OK;
  }
  const double base = (double)(base_seq_len > 0 ? base_seq_len : 64);
  double v = std::sqrt((double)image_tokens / base) * noise_scale;
  if (mode == U15C_NOISE_DYNAMIC_SQRT) v = std::sqrt(v);
  *out = std::min(v, max_value);
  return U15C_OK;
}

}  // extern "C"
