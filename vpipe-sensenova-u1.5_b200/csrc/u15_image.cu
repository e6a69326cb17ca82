// The image half of a denoise step on the device (ImagePath,
// src/u15-image.cc of the reference; CPU forms in src/u15-ref.cc
// vision_embed / conv_decoder): the patch embedder, the pixel head and the
// timestep + noise-scale embedding. Everything is channel-last, as the
// reference's device path is: the backbone's [tokens][hidden] output is
// already a [th][tw][hidden] map.
//
// The four contractions run on the tcgen05 GEMM (u15_gemm.cu) with its bias
// epilogue:
//   patch linear   [gh*gw][3 p^2]        x [C][3 p^2]        + b   (Conv2d k = s = p)
//   dense linear   [gh*gw/m^2][C m^2]    x [LLM][C m^2]      + b   (Conv2d k = s = m)
//   conv1 3x3      [4 th tw][9 * LLM/4]  x [hid][9 * LLM/4]  + b   (im2col)
//   conv2 3x3      [16 th tw][9 * hid/4] x [192][9 * hid/4]  + b
// and the glue between them is one memory pass each:
//   vision_post    GELU + interleaved 2-D RoPE + the m x m channel-slowest
//                  gather, fused (rounded to bf16 once)
//   ps_hwc         PixelShuffle(2) on a channel-last map (GELU fused for the
//                  conv1 output)
//   im2col3x3      nine contiguous channel runs per output pixel; the conv
//                  weights are repacked at bind time to [cout][ky][kx][cin] to
//                  match (the reference's build_conv_weights_)
//   ps8_out        PixelShuffle(8) into the f32 [H][W][3] image
// The timestep MLP (sinusoid -> Linear -> SiLU -> Linear, twice) is four
// matrix-vector products, one warp per output row, f32 math on the bf16
// weights.
#include "u15_capi_internal.h"
#include "u15_common.cuh"

#include <algorithm>
#include <cmath>
#include <string>
#include <vector>

using u15::cuda_fail;
using u15::DeviceScope;
using u15::fail;

namespace {

using bf16 = __nv_bfloat16;
using u15::pack_bf2;
using u15::unpack_bf2;
inline unsigned nblk(long n, int t) { return (unsigned)((n + t - 1) / t); }

__device__ __forceinline__ float gelu_erf(float v)
{
  return 0.5f * v * (1.0f + erff(v * 0.70710678118654752440f));
}

// img [H][W][3] f32 -> px [gh*gw][3 p^2] bf16, each patch channel-FIRST
// (ci, pi, qi): the patch embedder's input.
__global__ void patchify_cf_kernel(const float* img, bf16* px, int H, int W, int p)
{
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  const int gw = W / p, pin = 3 * p * p;
  const long n = (long)(H / p) * gw * pin;
  if (i >= n) return;
  const long patch = i / pin;
  const int r = (int)(i % pin), ci = r / (p * p), pi = (r / p) % p, qi = r % p;
  const int y = (int)(patch / gw) * p + pi, x = (int)(patch % gw) * p + qi;
  px[i] = __float2bfloat16_rn(img[((long)y * W + x) * 3 + ci]);
}

// emb [gh*gw][C] (patch linear + bias) -> GELU -> rotate pair (2q, 2q+1) of
// the first half by the patch column and of the second half by its row ->
// merged [(gh/m)(gw/m)][C m^2], channel (c, i, j) order. One thread per
// (patch, pair).
__global__ void vision_post_kernel(const bf16* emb, bf16* merged, int gh, int gw, int C, int m,
                                   const float* inv)
{
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  const int pairs = C / 2;
  if (i >= (long)gh * gw * pairs) return;
  const int n = (int)(i / pairs), q = (int)(i % pairs);
  const int row = n / gw, col = n % gw;
  const int quarter = C / 4;
  const bool second = q >= quarter;
  const int k = second ? q - quarter : q;
  const double ang = (double)(second ? row : col) * (double)inv[k];
  double s, c;
  sincos(ang, &s, &c);
  const float a = gelu_erf(__bfloat162float(emb[(long)n * C + 2 * q]));
  const float b = gelu_erf(__bfloat162float(emb[(long)n * C + 2 * q + 1]));
  const float ra = (float)((double)a * c - (double)b * s);
  const float rb = (float)((double)a * s + (double)b * c);
  const int ow = gw / m, tile = C * m * m;
  const int ti = row % m, tj = col % m;
  bf16* o = merged + ((long)(row / m) * ow + col / m) * tile;
  o[((2 * q) * m + ti) * m + tj] = __float2bfloat16_rn(ra);
  o[((2 * q + 1) * m + ti) * m + tj] = __float2bfloat16_rn(rb);
}

// PixelShuffle(r) channel-last: in [H][W][Cin] -> out [H r][W r][Cin / r^2],
// input channel c r^2 + i r + j of pixel (y, x) -> channel c of pixel
// (y r + i, x r + j). One thread per output element; GELU optional.
__global__ void ps_hwc_kernel(const bf16* in, bf16* out, int H, int W, int Cin, int r, int gelu)
{
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  const int Co = Cin / (r * r), OW = W * r;
  if (i >= (long)H * W * Cin) return;
  const int c = (int)(i % Co);
  const long pix = i / Co;
  const int oy = (int)(pix / OW), ox = (int)(pix % OW);
  const int y = oy / r, ii = oy % r, x = ox / r, jj = ox % r;
  float v = __bfloat162float(in[((long)y * W + x) * Cin + c * r * r + ii * r + jj]);
  if (gelu) v = gelu_erf(v);
  out[i] = __float2bfloat16_rn(v);
}

// im2col for a 3x3, padding-1 convolution over in [H][W][C] (C % 8 == 0):
// col [H W][9 C], row = output pixel, columns (ky, kx, c). Each thread moves
// 8 channels (16 bytes).
__global__ void im2col3x3_kernel(const bf16* in, bf16* col, int H, int W, int C)
{
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  const int c8 = C / 8;
  if (i >= (long)H * W * 9 * c8) return;
  const int cc = (int)(i % c8);
  const long r = i / c8;
  const int tap = (int)(r % 9);
  const long pix = r / 9;
  const int y = (int)(pix / W) + tap / 3 - 1, x = (int)(pix % W) + tap % 3 - 1;
  uint4 v = make_uint4(0u, 0u, 0u, 0u);
  if (y >= 0 && y < H && x >= 0 && x < W)
    v = *reinterpret_cast<const uint4*>(in + ((long)y * W + x) * C + cc * 8);
  *reinterpret_cast<uint4*>(col + i * 8) = v;
}

// PixelShuffle(8) of the conv2 output [H][W][192] -> the f32 image
// [8H][8W][3] (the values stay bf16-exact, as the reference's bf16 px_out).
__global__ void ps8_out_kernel(const bf16* in, float* out, int H, int W)
{
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  const int OW = 8 * W;
  if (i >= (long)64 * H * W * 3) return;
  const int c = (int)(i % 3);
  const long pix = i / 3;
  const int oy = (int)(pix / OW), ox = (int)(pix % OW);
  const int y = oy / 8, ii = oy % 8, x = ox / 8, jj = ox % 8;
  out[i] = __bfloat162float(in[((long)y * W + x) * 192 + c * 64 + ii * 8 + jj]);
}

// ---- the same layout moves, a run of values per thread (the forms above
// stay for geometries these do not cover) ----

// patchify for patch 16: one thread per (patch, patch row) reads the row's
// 16 pixels x 3 channels (192 contiguous bytes) and writes the three
// 16-value channel runs of the channel-first patch (32 bytes each).
__global__ void patchify16_kernel(const float* img, bf16* px, int H, int W)
{
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  const int gw = W / 16;
  if (i >= (long)(H / 16) * gw * 16) return;
  const long patch = i / 16;
  const int pi = (int)(i % 16);
  const int y = (int)(patch / gw) * 16 + pi, x0 = (int)(patch % gw) * 16;
  const float4* src = reinterpret_cast<const float4*>(img + ((long)y * W + x0) * 3);
  float v[48];
#pragma unroll
  for (int k = 0; k < 12; ++k) {
    const float4 f = src[k];
    v[4 * k] = f.x;
    v[4 * k + 1] = f.y;
    v[4 * k + 2] = f.z;
    v[4 * k + 3] = f.w;
  }
#pragma unroll
  for (int ci = 0; ci < 3; ++ci) {
    uint32_t w[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) w[q] = pack_bf2(v[(2 * q) * 3 + ci], v[(2 * q + 1) * 3 + ci]);
    uint4* dst = reinterpret_cast<uint4*>(px + patch * 768 + ci * 256 + pi * 16);
    dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
    dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
  }
}

// the vision RoPE's (cos, sin) for every (position, frequency):
// rot[pos][k] = sincos((double)pos * inv[k]), the values vision_post forms
__global__ void vision_rot_kernel(const float* inv, int quarter, int npos, double2* rot)
{
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= npos * quarter) return;
  const int pos = i / quarter, k = i % quarter;
  double sn, cs;
  sincos((double)pos * (double)inv[k], &sn, &cs);
  rot[i] = make_double2(cs, sn);
}

// vision_post for a 2 x 2 merge: one thread per (merged token, channel pair
// q) takes pair q of the token's four patches (GELU, rotation from the
// table) and writes the 8 outputs (channels 2q, 2q+1 x the four patches,
// channel (c, i, j) order) as one 16-byte run.
__global__ void vision_post_m2_kernel(const bf16* emb, bf16* merged, int gh, int gw, int C,
                                      const double2* rot)
{
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  const int pairs = C / 2, ow = gw / 2;
  if (i >= (long)(gh / 2) * ow * pairs) return;
  const long t = i / pairs;
  const int q = (int)(i % pairs);
  const int quarter = C / 4;
  const bool second = q >= quarter;
  const int k = second ? q - quarter : q;
  const int r0 = (int)(t / ow) * 2, c0 = (int)(t % ow) * 2;
  float o[8];
#pragma unroll
  for (int s = 0; s < 4; ++s) {
    const int row = r0 + (s >> 1), col = c0 + (s & 1);
    const float2 ab = unpack_bf2(*reinterpret_cast<const uint32_t*>(
        emb + ((long)row * gw + col) * C + 2 * q));
    const float a = gelu_erf(ab.x), b = gelu_erf(ab.y);
    const double2 r = rot[(long)(second ? row : col) * quarter + k];
    o[s] = (float)((double)a * r.x - (double)b * r.y);
    o[4 + s] = (float)((double)a * r.y + (double)b * r.x);
  }
  *reinterpret_cast<uint4*>(merged + t * (long)C * 4 + 8 * q) =
      make_uint4(pack_bf2(o[0], o[1]), pack_bf2(o[2], o[3]), pack_bf2(o[4], o[5]),
                 pack_bf2(o[6], o[7]));
}

// PixelShuffle(2) channel-last, 8 output channels per thread: reads the 32
// input channels 4c0 .. 4c0 + 31 of one pixel (64 bytes) and writes 8
// channels to each of its 2 x 2 output pixels (16 bytes each); GELU optional.
__global__ void ps2_hwc_kernel(const bf16* in, bf16* out, int H, int W, int Cin, int gelu)
{
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  const int Co = Cin / 4, g = Co / 8;
  if (i >= (long)H * W * g) return;
  const long pix = i / g;
  const int c0 = (int)(i % g) * 8;
  const uint4* src = reinterpret_cast<const uint4*>(in + pix * Cin + 4 * c0);
  float v[32];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const uint4 u = src[k];
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = unpack_bf2(w[j]);
      v[8 * k + 2 * j] = gelu ? gelu_erf(f.x) : f.x;
      v[8 * k + 2 * j + 1] = gelu ? gelu_erf(f.y) : f.y;
    }
  }
  const int y = (int)(pix / W), x = (int)(pix % W);
#pragma unroll
  for (int s = 0; s < 4; ++s) {   // input channel 4c + s -> output pixel (2y + s/2, 2x + s%2)
    uint32_t w[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) w[j] = pack_bf2(v[4 * (2 * j) + s], v[4 * (2 * j + 1) + s]);
    *reinterpret_cast<uint4*>(out + ((long)(2 * y + (s >> 1)) * (2 * W) + 2 * x + (s & 1)) * Co +
                              c0) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

// PixelShuffle(8) to the f32 image, one thread per (input pixel, output row
// ii): reads channels c 64 + 8 ii .. + 8 for c < 3 and writes the 8 output
// pixels x 3 channels of that row (96 contiguous bytes).
__global__ void ps8_row_kernel(const bf16* in, float* out, int H, int W)
{
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long)H * W * 8) return;
  const long pix = i / 8;
  const int ii = (int)(i % 8);
  float v[3][8];
#pragma unroll
  for (int c = 0; c < 3; ++c) {
    const uint4 u = *reinterpret_cast<const uint4*>(in + pix * 192 + c * 64 + ii * 8);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = unpack_bf2(w[j]);
      v[c][2 * j] = f.x;
      v[c][2 * j + 1] = f.y;
    }
  }
  const int y = (int)(pix / W), x = (int)(pix % W);
  float4* dst = reinterpret_cast<float4*>(out + ((long)(8 * y + ii) * (8 * W) + 8 * x) * 3);
#pragma unroll
  for (int k = 0; k < 6; ++k) {
    float e[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int idx = 4 * k + j;   // = 3 jj + c
      e[j] = v[idx % 3][idx / 3];
    }
    dst[k] = make_float4(e[0], e[1], e[2], e[3]);
  }
}

// [H][W][3] model space ([-1, 1]) -> [3][H][W] u8: clamp(x/2 + 1/2) * 255,
// rounded (src/u15-kernels.metal u15_to_u8_planar).
__global__ void to_u8_planar_kernel(const float* px, uint8_t* out, int H, int W)
{
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long)H * W * 3) return;
  const int c = (int)(i % 3);
  const long pix = i / 3;
  const float d = fminf(fmaxf(px[i] * 0.5f + 0.5f, 0.0f), 1.0f);
  out[(long)c * H * W + pix] = (uint8_t)(d * 255.0f + 0.5f);
}

// the timestep sinusoid: [cos(v f_i) | sin(v f_i)], f_i = 1e4^(-i / half)
__global__ void sinusoid_kernel(double v, int dim, float* out)
{
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  const int half = dim / 2;
  if (i >= half) return;
  const double f = exp(-log(10000.0) * (double)i / (double)half);
  double s, c;
  sincos(v * f, &s, &c);
  out[i] = (float)c;
  out[i + half] = (float)s;
}

// y[n] (+)= act(b[n] + sum_k W[n][k] x[k]): one warp per output row,
// W bf16 row-major, x / y f32; act 1 = SiLU; accumulate 1 adds into y.
__global__ void gemv_kernel(const bf16* W, const float* x, const bf16* b, float* y, int N, int K,
                            int act, int accumulate)
{
  const int n = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (n >= N) return;
  const bf16* w = W + (long)n * K;
  float acc = 0.0f;
  for (int k = lane * 2; k < K; k += 64) {
    const float2 wv = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(w + k));
    acc = fmaf(wv.x, x[k], acc);
    acc = fmaf(wv.y, x[k + 1], acc);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) {
    float v = acc + (b ? __bfloat162float(b[n]) : 0.0f);
    if (act == 1) v = v / (1.0f + expf(-v));
    y[n] = accumulate ? y[n] + v : v;
  }
}

// x[r][c] = bf16(x[r][c] + bf16(row[c])) for every row: the timestep row,
// rounded to bf16 as the reference uploads it, added to every image token.
__global__ void add_row_f32_kernel(bf16* x, const float* row, long rows, int dim)
{
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * dim) return;
  const float r = __bfloat162float(__float2bfloat16_rn(row[i % dim]));
  x[i] = __float2bfloat16_rn(__bfloat162float(x[i]) + r);
}

// conv weight [cout][cin][3][3] (f32 / f16 / bf16) -> [cout][9][cin] bf16
__global__ void repack_conv_kernel(const void* src, int dtype, int cout, int cin, bf16* dst)
{
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long)cout * cin * 9) return;
  const int c = (int)(i % cin);
  const long r = i / cin;
  const int k = (int)(r % 9), o = (int)(r / 9);
  const long s = ((long)o * cin + c) * 9 + k;
  float v;
  if (dtype == U15C_DT_F32) v = static_cast<const float*>(src)[s];
  else if (dtype == U15C_DT_F16) v = __half2float(static_cast<const __half*>(src)[s]);
  else v = __bfloat162float(static_cast<const bf16*>(src)[s]);
  dst[i] = __float2bfloat16_rn(v);
}

__global__ void to_bf16_kernel(const void* src, int dtype, long n, bf16* dst)
{
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float v;
  if (dtype == U15C_DT_F32) v = static_cast<const float*>(src)[i];
  else if (dtype == U15C_DT_F16) v = __half2float(static_cast<const __half*>(src)[i]);
  else v = __bfloat162float(static_cast<const bf16*>(src)[i]);
  dst[i] = __float2bfloat16_rn(v);
}

__device__ __forceinline__ uint64_t mix64(uint64_t x)
{
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

// N(0, std) by Box-Muller on a counter hash (seed, stream, index)
__global__ void randn_bf16_kernel(bf16* dst, long n, uint64_t seed, uint64_t stream, float std)
{
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const uint64_t h = mix64(seed ^ mix64(stream * 0x100000001B3ull + (uint64_t)i));
  const float u1 = ((float)(h >> 40) + 1.0f) * (1.0f / 16777217.0f);
  const float u2 = (float)((h >> 16) & 0xFFFFFF) * (1.0f / 16777216.0f);
  dst[i] = __float2bfloat16_rn(std * sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2));
}

}  // namespace

struct u15c_image {
  u15c_image_config cfg{};
  int device = 0;
  // bound weights, bf16; patch/dense per expert (0 und, 1 gen)
  bf16* patch_w = nullptr;   // [2][C][3 p^2]
  bf16* patch_b = nullptr;   // [2][C]
  bf16* dense_w = nullptr;   // [2][LLM][C m^2]
  bf16* dense_b = nullptr;   // [2][LLM]
  bf16* conv1_w = nullptr;   // [hid][9][LLM/4]
  bf16* conv1_b = nullptr;   // [hid]
  bf16* conv2_w = nullptr;   // [192][9][hid/4]
  bf16* conv2_b = nullptr;   // [192]
  bf16* mlp[8] = {};         // tstep w0 b0 w2 b2, nscale w0 b0 w2 b2
  float* inv = nullptr;      // vision RoPE inverse frequencies [C/4]
  double2* rot = nullptr;    // (cos, sin) per (position, frequency), rot_pos positions
  int rot_pos = 0;
  float* tvec = nullptr;     // [dim + 2 LLM] sinusoid | hidden | row
  std::vector<void*> allocs;
  // grow-only scratch
  size_t scratch_bytes = 0;
  void* scratch = nullptr;

  int C() const { return cfg.vision_hidden; }
  int LLM() const { return cfg.llm_hidden; }
  int hid() const { return cfg.head_hidden; }

  template <class T>
  int alloc(T** p, size_t bytes)
  {
    if (cudaMalloc(reinterpret_cast<void**>(p), bytes) != cudaSuccess)
      return fail(U15C_ENOMEM, "image path: out of device memory");
    allocs.push_back(*p);
    return U15C_OK;
  }
  int ensure(size_t bytes)
  {
    if (bytes <= scratch_bytes) return U15C_OK;
    if (scratch) cudaFree(scratch);
    scratch = nullptr;
    scratch_bytes = 0;
    if (cudaMalloc(&scratch, bytes) != cudaSuccess)
      return fail(U15C_ENOMEM, "image path: out of device memory for scratch");
    scratch_bytes = bytes;
    return U15C_OK;
  }
  ~u15c_image()
  {
    if (rot) cudaFree(rot);
    if (scratch) cudaFree(scratch);
    for (void* p : allocs) cudaFree(p);
  }
};

namespace {

int gemm(u15c_image* im, cudaStream_t st, const void* x, const bf16* w, const bf16* b, void* y,
         int M, int K, int N)
{
  u15::GemmArgs a;
  a.x = x;
  a.w = w;
  a.bias = b;
  a.y = y;
  a.M = M;
  a.K = K;
  a.N = N;
  a.epilogue = u15::kEpiStore;
  (void)im;
  return u15::run_gemm(a, st);
}

int launched(const char* what)
{
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? U15C_OK : cuda_fail(e, what);
}

}  // namespace

extern "C" {

int u15c_image_create(const u15c_image_config* cfg, u15c_image** out)
{
  if (cfg == nullptr || out == nullptr) return fail(U15C_EINVAL, "image_create: null argument");
  *out = nullptr;
  const u15c_image_config& c = *cfg;
  if (c.vision_hidden <= 0 || c.vision_hidden % 8 || c.llm_hidden <= 0 || c.llm_hidden % 32 ||
      c.head_hidden <= 0 || c.head_hidden % 32 || c.patch <= 0 || c.merge <= 0 ||
      c.freq_dim <= 0 || c.freq_dim % 2)
    return fail(U15C_EINVAL, "image config: vision_hidden % 8, llm_hidden % 32, head_hidden % 32 "
                             "and an even freq_dim are required");
  if (u15::dev() == nullptr) return U15C_ECUDA;
  auto* im = new u15c_image();
  im->cfg = c;
  cudaGetDevice(&im->device);
  const size_t C = c.vision_hidden, L = c.llm_hidden, pin = 3 * (size_t)c.patch * c.patch;
  const size_t mm = (size_t)c.merge * c.merge, hid = c.head_hidden, D = c.freq_dim;
  int rc = 0;
  rc |= im->alloc(&im->patch_w, 2 * C * pin * 2);
  rc |= im->alloc(&im->patch_b, 2 * C * 2);
  rc |= im->alloc(&im->dense_w, 2 * L * C * mm * 2);
  rc |= im->alloc(&im->dense_b, 2 * L * 2);
  rc |= im->alloc(&im->conv1_w, hid * 9 * (L / 4) * 2);
  rc |= im->alloc(&im->conv1_b, hid * 2);
  rc |= im->alloc(&im->conv2_w, 192 * 9 * (hid / 4) * 2);
  rc |= im->alloc(&im->conv2_b, 192 * 2);
  const size_t mlp_elems[4] = {L * D, L, L * L, L};
  for (int k = 0; k < 8; ++k) rc |= im->alloc(&im->mlp[k], mlp_elems[k % 4] * 2);
  rc |= im->alloc(&im->inv, C / 4 * 4);
  rc |= im->alloc(&im->tvec, (D + 2 * L) * 4);
  if (rc) {
    delete im;
    return U15C_ENOMEM;
  }
  std::vector<float> inv(C / 4);
  for (size_t i = 0; i < C / 4; ++i)
    inv[i] = (float)(1.0 / std::pow(c.vision_theta, (double)(2 * i) / (double)(C / 2)));
  cudaMemcpy(im->inv, inv.data(), inv.size() * 4, cudaMemcpyHostToDevice);
  *out = im;
  return U15C_OK;
}

void u15c_image_destroy(u15c_image* im)
{
  if (im == nullptr) return;
  DeviceScope ds(im->device);
  delete im;
}

int u15c_image_bind(u15c_image* im, u15c_stream stream, int tensor, int expert, const void* src,
                    int dtype, int src_on_host)
{
  if (im == nullptr || src == nullptr) return fail(U15C_EINVAL, "image_bind: null argument");
  if (dtype < 0 || dtype > 2) return fail(U15C_EINVAL, "image_bind: unknown source dtype");
  if (expert < 0 || expert > 1) return fail(U15C_EINVAL, "image_bind: expert must be 0 or 1");
  DeviceScope ds(im->device);
  const size_t C = im->C(), L = im->LLM(), hid = im->hid(), D = im->cfg.freq_dim;
  const size_t pin = 3 * (size_t)im->cfg.patch * im->cfg.patch;
  const size_t mm = (size_t)im->cfg.merge * im->cfg.merge;
  bf16* dst = nullptr;
  size_t n = 0;
  int conv = 0;   // 1: conv1 repack, 2: conv2 repack
  switch (tensor) {
    case U15C_I_PATCH_W: dst = im->patch_w + expert * C * pin; n = C * pin; break;
    case U15C_I_PATCH_B: dst = im->patch_b + expert * C; n = C; break;
    case U15C_I_DENSE_W: dst = im->dense_w + expert * L * C * mm; n = L * C * mm; break;
    case U15C_I_DENSE_B: dst = im->dense_b + expert * L; n = L; break;
    case U15C_I_CONV1_W: dst = im->conv1_w; n = hid * (L / 4) * 9; conv = 1; break;
    case U15C_I_CONV1_B: dst = im->conv1_b; n = hid; break;
    case U15C_I_CONV2_W: dst = im->conv2_w; n = 192 * (hid / 4) * 9; conv = 2; break;
    case U15C_I_CONV2_B: dst = im->conv2_b; n = 192; break;
    default:
      if (tensor >= U15C_I_TSTEP_W0 && tensor <= U15C_I_NSCALE_B2) {
        const int k = tensor - U15C_I_TSTEP_W0;
        const size_t elems[4] = {L * D, L, L * L, L};
        dst = im->mlp[k];
        n = elems[k % 4];
        break;
      }
      return fail(U15C_EINVAL, "image_bind: unknown tensor id");
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t es = dtype == U15C_DT_F32 ? 4 : 2;
  const void* dsrc = src;
  void* staging = nullptr;
  if (src_on_host) {
    if (cudaMalloc(&staging, n * es) != cudaSuccess)
      return fail(U15C_ENOMEM, "image_bind: staging allocation failed");
    const cudaError_t e = cudaMemcpyAsync(staging, src, n * es, cudaMemcpyHostToDevice, st);
    if (e != cudaSuccess) {
      cudaFree(staging);
      return cuda_fail(e, "image_bind: upload");
    }
    dsrc = staging;
  }
  if (conv == 1)
    repack_conv_kernel<<<nblk(n, 256), 256, 0, st>>>(dsrc, dtype, (int)hid, (int)(L / 4), dst);
  else if (conv == 2)
    repack_conv_kernel<<<nblk(n, 256), 256, 0, st>>>(dsrc, dtype, 192, (int)(hid / 4), dst);
  else
    to_bf16_kernel<<<nblk(n, 256), 256, 0, st>>>(dsrc, dtype, (long)n, dst);
  const int rc = launched("image_bind");
  if (staging != nullptr) {
    cudaStreamSynchronize(st);
    cudaFree(staging);
  }
  return rc;
}

int u15c_image_bind_random(u15c_image* im, u15c_stream stream, uint64_t seed, float std)
{
  if (im == nullptr) return fail(U15C_EINVAL, "image_bind_random: null image path");
  DeviceScope ds(im->device);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t C = im->C(), L = im->LLM(), hid = im->hid(), D = im->cfg.freq_dim;
  const size_t pin = 3 * (size_t)im->cfg.patch * im->cfg.patch;
  const size_t mm = (size_t)im->cfg.merge * im->cfg.merge;
  uint64_t sid = 0;
  auto fill = [&](bf16* p, size_t n, float sd) {
    randn_bf16_kernel<<<nblk((long)n, 256), 256, 0, st>>>(p, (long)n, seed, ++sid, sd);
  };
  fill(im->patch_w, 2 * C * pin, std);
  fill(im->patch_b, 2 * C, std);
  fill(im->dense_w, 2 * L * C * mm, std);
  fill(im->dense_b, 2 * L, std);
  fill(im->conv1_w, hid * 9 * (L / 4), std);
  fill(im->conv1_b, hid, std);
  fill(im->conv2_w, 192 * 9 * (hid / 4), std);
  fill(im->conv2_b, 192, std);
  const size_t elems[4] = {L * D, L, L * L, L};
  for (int k = 0; k < 8; ++k) fill(im->mlp[k], elems[k % 4], std);
  return launched("image_bind_random");
}

int u15c_image_patchify(u15c_stream stream, const float* img, void* px, int H, int W, int patch)
{
  if (img == nullptr || px == nullptr || patch <= 0 || H % patch || W % patch || H <= 0 || W <= 0)
    return fail(U15C_EINVAL, "image_patchify: H and W must be positive multiples of the patch");
  if (u15::dev() == nullptr) return U15C_ECUDA;
  const long n = (long)H * W * 3;
  if (patch == 16 && reinterpret_cast<uintptr_t>(img) % 16 == 0)
    patchify16_kernel<<<nblk(n / 48, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        img, static_cast<bf16*>(px), H, W);
  else
    patchify_cf_kernel<<<nblk(n, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        img, static_cast<bf16*>(px), H, W, patch);
  return launched("image_patchify");
}

int u15c_image_embed(u15c_image* im, u15c_stream stream, const void* px, int grid_h, int grid_w,
                     int expert, void* out)
{
  if (im == nullptr || px == nullptr || out == nullptr || grid_h <= 0 || grid_w <= 0)
    return fail(U15C_EINVAL, "image_embed: bad argument");
  const int m = im->cfg.merge;
  if (grid_h % m || grid_w % m)
    return fail(U15C_EINVAL, "image_embed: the patch grid is not a whole number of " +
                                 std::to_string(m) + "x" + std::to_string(m) + " tiles");
  if (expert < 0 || expert > 1) return fail(U15C_EINVAL, "image_embed: expert must be 0 or 1");
  DeviceScope ds(im->device);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int C = im->C(), L = im->LLM(), pin = 3 * im->cfg.patch * im->cfg.patch;
  const long n = (long)grid_h * grid_w;
  const size_t emb_bytes = (size_t)n * C * 2;
  int rc = im->ensure(2 * emb_bytes);
  if (rc) return rc;
  bf16* emb = static_cast<bf16*>(im->scratch);
  bf16* merged = emb + (size_t)n * C;
  if ((rc = gemm(im, st, px, im->patch_w + (size_t)expert * C * pin, im->patch_b + expert * C, emb,
                 (int)n, pin, C)))
    return rc;
  if (m == 2 && C % 16 == 0) {
    // the (cos, sin) table, grown to the grid's largest position on demand
    const int npos = std::max(grid_h, grid_w);
    if (npos > im->rot_pos) {
      if (im->rot) cudaFree(im->rot);
      im->rot = nullptr;
      im->rot_pos = 0;
      if (cudaMalloc(&im->rot, (size_t)npos * (C / 4) * sizeof(double2)) != cudaSuccess)
        return fail(U15C_ENOMEM, "image_embed: out of device memory for the rotation table");
      vision_rot_kernel<<<nblk((long)npos * (C / 4), 256), 256, 0, st>>>(im->inv, C / 4, npos,
                                                                         im->rot);
      // once per growth: later calls may come on other streams
      if (cudaStreamSynchronize(st) != cudaSuccess)
        return cuda_fail(cudaGetLastError(), "image_embed: rotation table");
      im->rot_pos = npos;
    }
    vision_post_m2_kernel<<<nblk(n / 4 * C / 2, 256), 256, 0, st>>>(emb, merged, grid_h, grid_w,
                                                                    C, im->rot);
  } else {
    vision_post_kernel<<<nblk(n * C / 2, 256), 256, 0, st>>>(emb, merged, grid_h, grid_w, C, m,
                                                              im->inv);
  }
  if ((rc = launched("image_embed: vision_post"))) return rc;
  const int rows = (int)(n / (m * m)), K = C * m * m;
  return gemm(im, st, merged, im->dense_w + (size_t)expert * L * K, im->dense_b + expert * L, out,
              rows, K, L);
}

int u15c_image_timestep_row(u15c_image* im, u15c_stream stream, double t, double noise_ratio,
                            float* out)
{
  if (im == nullptr || out == nullptr) return fail(U15C_EINVAL, "image_timestep_row: bad argument");
  DeviceScope ds(im->device);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int L = im->LLM(), D = im->cfg.freq_dim;
  float* sn = im->tvec;
  float* h = im->tvec + D;
  const int wpb = 8;   // warps per block
  for (int e = 0; e < (im->cfg.noise_scale_embedding ? 2 : 1); ++e) {
    bf16* const* w = im->mlp + 4 * e;
    sinusoid_kernel<<<nblk(D / 2, 128), 128, 0, st>>>(e == 0 ? t : noise_ratio, D, sn);
    gemv_kernel<<<nblk(L, wpb), 32 * wpb, 0, st>>>(w[0], sn, w[1], h, L, D, 1, 0);
    gemv_kernel<<<nblk(L, wpb), 32 * wpb, 0, st>>>(w[2], h, w[3], out, L, L, 0, e);
  }
  return launched("image_timestep_row");
}

int u15c_image_add_timestep(u15c_image* im, u15c_stream stream, void* x, int rows, double t,
                            double noise_ratio)
{
  if (im == nullptr || x == nullptr || rows <= 0)
    return fail(U15C_EINVAL, "image_add_timestep: bad argument");
  DeviceScope ds(im->device);
  float* row = im->tvec + im->cfg.freq_dim + im->LLM();
  int rc = u15c_image_timestep_row(im, stream, t, noise_ratio, row);
  if (rc) return rc;
  const long n = (long)rows * im->LLM();
  add_row_f32_kernel<<<nblk(n, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<bf16*>(x), row, rows, im->LLM());
  return launched("image_add_timestep");
}

int u15c_image_decode(u15c_image* im, u15c_stream stream, const void* hidden, int th, int tw,
                      float* out_px)
{
  if (im == nullptr || hidden == nullptr || out_px == nullptr || th <= 0 || tw <= 0)
    return fail(U15C_EINVAL, "image_decode: bad argument");
  DeviceScope ds(im->device);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int L = im->LLM(), hid = im->hid();
  const int c1 = L / 4, c2 = hid / 4;
  const long p1 = 4L * th * tw, p2 = 16L * th * tw;   // pixels of conv1 / conv2
  const size_t a_el = (size_t)p1 * c1, col_el = std::max((size_t)p1 * 9 * c1, (size_t)p2 * 9 * c2);
  const size_t b_el = (size_t)p1 * hid, c_el = (size_t)p2 * c2, e_el = (size_t)p2 * 192;
  int rc = im->ensure((std::max(a_el, c_el) + col_el + std::max(b_el, e_el)) * 2);
  if (rc) return rc;
  bf16* a = static_cast<bf16*>(im->scratch);            // PS(2) input of a conv
  bf16* col = a + std::max(a_el, c_el);
  bf16* b = col + col_el;                               // a conv's output
  // PS(2): [th][tw][L] -> [2th][2tw][L/4]; conv1 (+ bias) -> [2th][2tw][hid]
  if (L % 32 == 0)
    ps2_hwc_kernel<<<nblk((long)th * tw * (L / 32), 256), 256, 0, st>>>(
        static_cast<const bf16*>(hidden), a, th, tw, L, 0);
  else
    ps_hwc_kernel<<<nblk((long)th * tw * L, 256), 256, 0, st>>>(static_cast<const bf16*>(hidden),
                                                                a, th, tw, L, 2, 0);
  im2col3x3_kernel<<<nblk(p1 * 9 * (c1 / 8), 256), 256, 0, st>>>(a, col, 2 * th, 2 * tw, c1);
  if ((rc = launched("image_decode: conv1 gather"))) return rc;
  if ((rc = gemm(im, st, col, im->conv1_w, im->conv1_b, b, (int)p1, 9 * c1, hid))) return rc;
  // GELU + PS(2): [2th][2tw][hid] -> [4th][4tw][hid/4]; conv2 (+ bias) -> [4th][4tw][192]
  if (hid % 32 == 0)
    ps2_hwc_kernel<<<nblk(p1 * (hid / 32), 256), 256, 0, st>>>(b, a, 2 * th, 2 * tw, hid, 1);
  else
    ps_hwc_kernel<<<nblk(p1 * hid, 256), 256, 0, st>>>(b, a, 2 * th, 2 * tw, hid, 2, 1);
  im2col3x3_kernel<<<nblk(p2 * 9 * (c2 / 8), 256), 256, 0, st>>>(a, col, 4 * th, 4 * tw, c2);
  if ((rc = launched("image_decode: conv2 gather"))) return rc;
  if ((rc = gemm(im, st, col, im->conv2_w, im->conv2_b, b, (int)p2, 9 * c2, 192))) return rc;
  // PS(8) -> [32th][32tw][3]
  if (reinterpret_cast<uintptr_t>(out_px) % 16 == 0)
    ps8_row_kernel<<<nblk(p2 * 8, 256), 256, 0, st>>>(b, out_px, 4 * th, 4 * tw);
  else
    ps8_out_kernel<<<nblk(p2 * 192, 256), 256, 0, st>>>(b, out_px, 4 * th, 4 * tw);
  return launched("image_decode: pixel shuffle");
}

int u15c_image_to_u8_planar(u15c_stream stream, const float* px, uint8_t* out, int H, int W)
{
  if (px == nullptr || out == nullptr || H <= 0 || W <= 0)
    return fail(U15C_EINVAL, "image_to_u8_planar: bad argument");
  if (u15::dev() == nullptr) return U15C_ECUDA;
  to_u8_planar_kernel<<<nblk((long)H * W * 3, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      px, out, H, W);
  return launched("image_to_u8_planar");
}

}  // extern "C"
