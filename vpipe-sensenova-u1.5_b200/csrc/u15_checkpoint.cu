// The checkpoint's affine-quantized matrices (the reference's w8g64 / w4
// packs, src/u15-weights.cc:248-325 bind_matrix_): u32 codes [N][K*bits/32]
// with per-group scales and biases [N][K/group], value = scale * code +
// bias. The B200 path dequantizes them once, at bind time, into the bound
// bf16 layout; the W8A8 twin is then requantized per output channel by
// u15c_model_finalize, the form the int8 tensor-core GEMM consumes.
#include "u15_capi_internal.h"
#include "u15_common.cuh"

#include <cuda_fp16.h>

using u15::cuda_fail;
using u15::fail;

namespace {

using bf16 = __nv_bfloat16;

__device__ __forceinline__ float scalar_as_bf16(const void* p, int dtype, long i)
{
  // the pack's scales and biases reach the kernel as bf16 (the reference
  // binds them through bind_bf16_), rounded to nearest even from F16 / F32
  float v;
  if (dtype == U15C_DT_F16) v = __half2float(static_cast<const __half*>(p)[i]);
  else if (dtype == U15C_DT_F32) v = static_cast<const float*>(p)[i];
  else return __bfloat162float(static_cast<const bf16*>(p)[i]);
  return __bfloat162float(__float2bfloat16_rn(v));
}

// one thread per output element: w[n][k] = bf16(scale * code + bias), the
// product and the sum rounded separately (no fused multiply-add), so a
// host restatement in f32 reproduces it bit for bit
__global__ void dequant_affine_kernel(const uint32_t* codes, const void* scales,
                                      const void* biases, int sdtype, int N, int K, int bits,
                                      int group, bf16* out)
{
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long)N * K) return;
  const int n = (int)(i / K), k = (int)(i % K);
  const int per = 32 / bits;
  const uint32_t word = codes[(long)n * (K / per) + k / per];
  const uint32_t code = (word >> ((k % per) * bits)) & ((1u << bits) - 1u);
  const long g = (long)n * (K / group) + k / group;
  const float s = scalar_as_bf16(scales, sdtype, g), b = scalar_as_bf16(biases, sdtype, g);
  out[i] = __float2bfloat16_rn(__fadd_rn(__fmul_rn(s, (float)code), b));
}

}  // namespace

extern "C" {

int u15c_dequant_affine(u15c_stream stream, const uint32_t* codes, const void* scales,
                        const void* biases, int scale_dtype, int N, int K, int bits, int group,
                        void* out)
{
  if (codes == nullptr || scales == nullptr || biases == nullptr || out == nullptr || N <= 0 ||
      K <= 0)
    return fail(U15C_EINVAL, "dequant_affine: bad argument");
  if ((bits != 4 && bits != 8) || (group != 32 && group != 64) || K % group || K % (32 / bits))
    return fail(U15C_EINVAL, "dequant_affine: packs are w4 / w8 with groups of 32 / 64 "
                             "dividing K (src/u15-weights.cc:270-283)");
  if (scale_dtype < 0 || scale_dtype > 2)
    return fail(U15C_EINVAL, "dequant_affine: unknown scale dtype");
  if (u15::dev() == nullptr) return U15C_ECUDA;
  const long n = (long)N * K;
  dequant_affine_kernel<<<(unsigned)((n + 255) / 256), 256, 0,
                          static_cast<cudaStream_t>(stream)>>>(
      codes, scales, biases, scale_dtype, N, K, bits, group, static_cast<bf16*>(out));
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? U15C_OK : cuda_fail(e, "dequant_affine launch");
}

}  // extern "C"
