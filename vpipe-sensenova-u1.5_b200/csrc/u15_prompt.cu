// The prefill's inputs from token ids (src/u15-generator.cc:308-392 of the
// reference): the token-embedding gather, the (t, h, w) position rule of
// Prompt::thw_indexes (src/u15-prompt.cc:349-386), and the splice of the
// reference images' patch embeddings over their <IMG_CONTEXT> rows.
#include "u15_capi_internal.h"
#include "u15_common.cuh"

#include <vector>

using u15::cuda_fail;
using u15::fail;

namespace {

using bf16 = __nv_bfloat16;

// out[i] = table[ids[i]] row by row, 8 bf16 per thread; an id outside
// [0, vocab) yields a zero row and records kDevBadArg in the status word.
__global__ void embed_gather_kernel(const bf16* table, int vocab, int hidden, const int32_t* ids,
                                    int n, bf16* out, unsigned* err)
{
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  const int h8 = hidden / 8;
  if (i >= (long)n * h8) return;
  const int r = (int)(i / h8), c = (int)(i % h8);
  const int id = ids[r];
  uint4 v = make_uint4(0u, 0u, 0u, 0u);
  if (id >= 0 && id < vocab)
    v = *reinterpret_cast<const uint4*>(table + (long)id * hidden + c * 8);
  else if (c == 0)
    u15::dev_fail(err, u15::kDevBadArg);
  *reinterpret_cast<uint4*>(out + (long)r * hidden + c * 8) = v;
}

}  // namespace

extern "C" {

int u15c_embed_tokens(u15c_stream stream, const void* table, int vocab, int hidden,
                      const int32_t* ids, int n, void* out)
{
  if (table == nullptr || ids == nullptr || out == nullptr || vocab <= 0 || n <= 0 ||
      hidden <= 0 || hidden % 8)
    return fail(U15C_EINVAL, "embed_tokens: bad argument (hidden must be a multiple of 8)");
  u15::DevState* d = u15::dev();
  if (d == nullptr) return U15C_ECUDA;
  const long work = (long)n * (hidden / 8);
  embed_gather_kernel<<<(unsigned)((work + 255) / 256), 256, 0,
                        static_cast<cudaStream_t>(stream)>>>(
      static_cast<const bf16*>(table), vocab, hidden, ids, n, static_cast<bf16*>(out), d->err);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? U15C_OK : cuda_fail(e, "embed_tokens launch");
}

int u15c_thw_indexes(const int32_t* ids, int n, int img_id, int img_ctx_id, const int* grid_hw,
                     int n_imgs, int32_t* t, int32_t* h, int32_t* w)
{
  if (ids == nullptr || t == nullptr || h == nullptr || w == nullptr || n < 0 || n_imgs < 0 ||
      (n_imgs > 0 && grid_hw == nullptr))
    return fail(U15C_EINVAL, "thw_indexes: bad argument");
  // One pass over the prompt. The sequence position steps on every token
  // outside an image's context run and once more on the token that follows
  // an <img> marker, so all of a run's tokens share the position one past
  // their marker's. Context tokens also take the next cell of their
  // image's merged grid (half the patch grid each way), row by row; an
  // image whose grid is exhausted (or empty) hands over to the next one,
  // and context tokens beyond the last image keep row and column 0.
  int pos = -1;
  int image = 0;   // the image whose grid the next context token fills
  int cell = 0;    // the next free cell of that grid
  auto grid_cells = [&](int k) { return (grid_hw[2 * k] / 2) * (grid_hw[2 * k + 1] / 2); };
  for (int i = 0; i < n; ++i) {
    const bool context = ids[i] == img_ctx_id;
    const bool after_marker = i > 0 && ids[i - 1] == img_id;
    pos += (after_marker ? 1 : 0) + (context ? 0 : 1);
    t[i] = pos;
    h[i] = 0;
    w[i] = 0;
    if (!context) continue;
    while (image < n_imgs && cell >= grid_cells(image)) {
      ++image;
      cell = 0;
    }
    if (image >= n_imgs) continue;
    const int cols = grid_hw[2 * image + 1] / 2;
    if (cols <= 0) return fail(U15C_EINVAL, "thw_indexes: an image grid is smaller than 2x2");
    h[i] = cell / cols;
    w[i] = cell % cols;
    ++cell;
  }
  return U15C_OK;
}

int u15c_splice_image_rows(u15c_stream stream, void* x, int hidden, const int32_t* ids_host,
                           int n, int img_ctx_id, const void* const* image_embeds,
                           const int* image_tokens, int n_imgs)
{
  if (x == nullptr || ids_host == nullptr || n <= 0 || hidden <= 0 || n_imgs < 0 ||
      (n_imgs > 0 && (image_embeds == nullptr || image_tokens == nullptr)))
    return fail(U15C_EINVAL, "splice_image_rows: bad argument");
  if (u15::dev() == nullptr) return U15C_ECUDA;
  // each image's context tokens are one contiguous run in the prompt
  // (<img> <IMG_CONTEXT> x tokens </img>): one copy per image
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int i = 0;
  for (int img = 0; img < n_imgs; ++img) {
    while (i < n && ids_host[i] != img_ctx_id) ++i;
    int j = i;
    while (j < n && ids_host[j] == img_ctx_id && j - i < image_tokens[img]) ++j;
    if (j - i != image_tokens[img])
      return fail(U15C_EINVAL, "splice_image_rows: image " + std::to_string(img) + " has " +
                                   std::to_string(image_tokens[img]) + " tokens but its context "
                                   "run in the prompt has " + std::to_string(j - i));
    const size_t bytes = (size_t)(j - i) * hidden * 2;
    const cudaError_t e = cudaMemcpyAsync(static_cast<bf16*>(x) + (size_t)i * hidden,
                                          image_embeds[img], bytes, cudaMemcpyDeviceToDevice, st);
    if (e != cudaSuccess) return cuda_fail(e, "splice_image_rows copy");
    i = j;
  }
  return U15C_OK;
}

}  // extern "C"
