// The C ABI (include/u15c.h): argument validation, error strings and the
// per-device state, over the launchers in u15_gemm.cu, u15_attn.cu and
// u15_elem.cu. The model half (weights, KV cache, backbone) is in
// u15_model.cu.
#include "u15_capi_internal.h"

#include <cmath>
#include <cstring>
#include <mutex>

namespace u15 {

thread_local std::string g_last_error;

int fail(int code, const std::string& msg)
{
  g_last_error = msg;
  return code;
}

int cuda_fail(cudaError_t e, const char* what)
{
  return fail(U15C_ECUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

namespace {
constexpr int kMaxDev = 64;
constexpr size_t kStatusBytes = 16;
DevState g_dev[kMaxDev];
std::mutex g_dev_mu;
}  // namespace

int dev_init(int device)
{
  if (device < 0 || device >= kMaxDev) return fail(U15C_EINVAL, "device index out of range");
  std::lock_guard<std::mutex> g(g_dev_mu);
  DevState& d = g_dev[device];
  if (d.ready) return U15C_OK;
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
  cudaDeviceProp prop;
  e = cudaGetDeviceProperties(&prop, device);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceProperties");
  if (prop.major != 10)
    return fail(U15C_EINVAL, std::string("libu15c is built for sm_100a (B200); device is ") +
                                 prop.name + " sm_" + std::to_string(prop.major) +
                                 std::to_string(prop.minor));
  d.sms = prop.multiProcessorCount;
  // the status block: the first error code, then the wait limit (0 = default)
  e = cudaMalloc(&d.err, kStatusBytes);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(status word)");
  e = cudaMemset(d.err, 0, kStatusBytes);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemset(status word)");
  d.ready = true;
  return U15C_OK;
}

DevState* dev()
{
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess) {
    fail(U15C_ECUDA, "cudaGetDevice failed");
    return nullptr;
  }
  if (!g_dev[device].ready && dev_init(device) != U15C_OK) return nullptr;
  return &g_dev[device];
}

bool fill_seg(SegInfo* s, const int* off, const int* ex, int nseg, int rows, int n_experts,
              std::string* err)
{
  if (nseg <= 0 || off == nullptr || ex == nullptr) {
    s->nseg = 1;
    s->off[0] = 0;
    s->off[1] = rows;
    s->expert[0] = 0;
    return true;
  }
  if (nseg > kMaxSeg) {
    *err = "at most 8 routing segments";
    return false;
  }
  if (off[0] != 0 || off[nseg] != rows) {
    *err = "segments must cover [0, rows)";
    return false;
  }
  s->nseg = nseg;
  for (int i = 0; i <= nseg; ++i) s->off[i] = off[i];
  for (int i = 0; i < nseg; ++i) {
    if (ex[i] < 0 || ex[i] >= n_experts) {
      *err = "segment expert out of range";
      return false;
    }
    if (off[i + 1] < off[i]) {
      *err = "segment offsets must be non-decreasing";
      return false;
    }
    s->expert[i] = ex[i];
  }
  return true;
}

KvView kv_view(void* k, void* v, const int32_t* page_table, int cap, int hkv)
{
  KvView kv;
  kv.k = k;
  kv.v = v;
  kv.page_table = page_table;
  if (page_table == nullptr) {
    kv.page_stride = (long)kPageTokens * kHeadDim;
    kv.head_stride = (long)cap * kHeadDim;
  } else {
    kv.page_stride = (long)hkv * kPageTokens * kHeadDim;
    kv.head_stride = (long)kPageTokens * kHeadDim;
  }
  return kv;
}

// Sage workspace: int8 Q [hq][tq][128], int8 smoothed K [hkv][npg * 64][128]
// (rows past tk zero), Q scales [hq][ceil(tq / 64)], K scales [hkv][2 * npg]
// (one per 32-key block), K-mean page partials [hkv][npg][128].
size_t sage_bytes(int hq, int hkv, int tq, int tk)
{
  const size_t nqb = (size_t)(tq + 63) / 64, npg = (size_t)(tk + 63) / 64;
  auto al = [](size_t b) { return (b + 255) & ~(size_t)255; };
  return al((size_t)hq * tq * 128) + al((size_t)hkv * npg * 64 * 128) + al(4 * hq * nqb) +
         al(4 * hkv * 2 * npg) + al(4 * (size_t)hkv * npg * 128);
}

SageWs sage_split(void* ws, int hq, int hkv, int tq, int tk)
{
  const size_t nqb = (size_t)(tq + 63) / 64, npg = (size_t)(tk + 63) / 64;
  auto al = [](size_t b) { return (b + 255) & ~(size_t)255; };
  uint8_t* p = static_cast<uint8_t*>(ws);
  SageWs s;
  s.q8 = reinterpret_cast<int8_t*>(p);
  p += al((size_t)hq * tq * 128);
  s.k8 = reinterpret_cast<int8_t*>(p);
  p += al((size_t)hkv * npg * 64 * 128);
  s.sq = reinterpret_cast<float*>(p);
  p += al(4 * hq * nqb);
  s.sk = reinterpret_cast<float*>(p);
  p += al(4 * hkv * 2 * npg);
  s.kmean = reinterpret_cast<float*>(p);
  return s;
}

int check_attention(int hq, int hkv, int tq, int tk, int mode, int q_offset,
                    const int32_t* t_index, bool sage, bool legacy)
{
  if (hq <= 0 || hkv <= 0 || hq % hkv != 0)
    return fail(U15C_EINVAL, "attention: hq must be a positive multiple of hkv");
  if (legacy && (hq / hkv > 8 || 128 % (hq / hkv) != 0))
    return fail(U15C_EINVAL, "attention: GQA group size must divide 128 and be at most 8");
  if (tq < 0 || tk < 0)
    return fail(U15C_EINVAL, "attention: token counts must be non-negative");
  if (mode < 0 || mode > 2) return fail(U15C_EINVAL, "attention: unknown mode");
  if (sage && mode != 0)
    return fail(U15C_EINVAL, "attention: Sage serves the bidirectional pass only");
  if (mode == 2 && t_index == nullptr)
    return fail(U15C_EINVAL, "attention: block-causal needs the t-index vector");
  if (mode != 0 && (q_offset < 0 || (mode == 2 && tq > 0 && (long)q_offset + tq > tk)))
    return fail(U15C_EINVAL, "attention: the queries' positions must lie within the key range");
  return U15C_OK;
}

int run_attention(cudaStream_t st, const void* q, const KvView& kv, void* out, int hq, int hkv,
                  int tq, int tk, int mode, int q_offset, const int32_t* t_index, void* sage_ws)
{
  DevState* d = dev();
  if (d == nullptr) return U15C_ECUDA;
  if (q == nullptr || kv.k == nullptr || kv.v == nullptr || out == nullptr)
    return fail(U15C_EINVAL, "attention: null buffer");
  int rc = check_attention(hq, hkv, tq, tk, mode, q_offset, t_index, sage_ws != nullptr, true);
  if (rc) return rc;
  AttnArgs a;
  a.q = q;
  a.kv = kv;
  a.out = out;
  a.hq = hq;
  a.hkv = hkv;
  a.tq = tq;
  a.tk = tk;
  a.mode = mode;
  a.q_offset = q_offset;
  a.t_index = t_index;
  a.dev_err = d->err;
  std::string err;
  if (sage_ws != nullptr) {
    SageWs s = sage_split(sage_ws, hq, hkv, tq, tk);
    if (sage_prepare(q, kv, hq, hkv, tq, tk, s.q8, s.k8, s.sq, s.sk, s.kmean, st, &err))
      return fail(U15C_ECUDA, err);
    a.q8 = s.q8;
    a.k8 = s.k8;
    a.sq = s.sq;
    a.sk = s.sk;
  }
  rc = attention(a, st, &err);
  if (rc) return fail(rc == 1 ? U15C_EINVAL : U15C_ECUDA, err);
  return U15C_OK;
}

int run_attention_tc(cudaStream_t st, const void* q, const KvView& kv, int n_pages, void* out,
                     int hq, int hkv, int tq, int tk, int mode, int q_offset,
                     const int32_t* t_index, void* sage_ws)
{
  DevState* d = dev();
  if (d == nullptr) return U15C_ECUDA;
  if (q == nullptr || kv.k == nullptr || kv.v == nullptr || out == nullptr)
    return fail(U15C_EINVAL, "attention: null buffer");
  if (!kv.v_t || kv.page_stride != (long)hkv * kPageTokens * kHeadDim ||
      kv.head_stride != (long)kPageTokens * kHeadDim)
    return fail(U15C_EINVAL, "attention: the tcgen05 path needs the paged layout with transposed V");
  if ((tk + kPageTokens - 1) / kPageTokens > n_pages)
    return fail(U15C_EINVAL, "attention: key length exceeds the page pool");
  if (!attention_tc_serves(mode, tk, t_index))
    return run_attention(st, q, kv, out, hq, hkv, tq, tk, mode, q_offset, t_index, sage_ws);
  int rc = check_attention(hq, hkv, tq, tk, mode, q_offset, t_index, sage_ws != nullptr, false);
  if (rc) return rc;
  TcAttnArgs a;
  a.q = q;
  a.k_pages = kv.k;
  a.vt_pages = kv.v;
  a.page_table = kv.page_table;
  a.n_pages = n_pages;
  a.out = out;
  a.hq = hq;
  a.hkv = hkv;
  a.tq = tq;
  a.tk = tk;
  a.mode = mode;
  a.q_offset = q_offset;
  a.t_index = t_index;
  a.dev_err = d->err;
  std::string err;
  if (sage_ws != nullptr) {
    SageWs s = sage_split(sage_ws, hq, hkv, tq, tk);
    if (sage_prepare(q, kv, hq, hkv, tq, tk, s.q8, s.k8, s.sq, s.sk, s.kmean, st, &err))
      return fail(U15C_ECUDA, err);
    a.q8 = s.q8;
    a.k8 = s.k8;
    a.sq = s.sq;
    a.sk = s.sk;
  }
  rc = attention_tc(a, st, &err);
  if (rc) return fail(rc == 1 ? U15C_EINVAL : U15C_ECUDA, err);
  return U15C_OK;
}

int run_gemm(GemmArgs& a, cudaStream_t st)
{
  DevState* d = dev();
  if (d == nullptr) return U15C_ECUDA;
  if (a.x == nullptr || a.w == nullptr || (a.y == nullptr && a.epilogue != kEpiTpReduce))
    return fail(U15C_EINVAL, "gemm: null buffer");
  a.dev_err = d->err;
  a.num_sms = d->sms;
  std::string err;
  const int rc = gemm_tc(a, st, &err);
  if (rc) return fail(rc == 1 ? U15C_EINVAL : U15C_ECUDA, err);
  return U15C_OK;
}

}  // namespace u15

using namespace u15;

#define ST(s) static_cast<cudaStream_t>(s)
#define LAUNCH(expr, what)                                              \
  do {                                                                  \
    if (dev() == nullptr) return U15C_ECUDA;                            \
    if ((expr) != 0) return fail(U15C_ECUDA, what ": launch failed");   \
    return U15C_OK;                                                     \
  } while (0)

extern "C" {

const char* u15c_last_error(void) { return g_last_error.c_str(); }
const char* u15c_version(void) { return "u15c 0.1 (sm_100a)"; }

int u15c_init(int device, unsigned flags)
{
  (void)flags;
  const int rc = dev_init(device);
  if (rc) return rc;
  const cudaError_t e = cudaSetDevice(device);
  return e == cudaSuccess ? U15C_OK : cuda_fail(e, "cudaSetDevice");
}

int u15c_device_status(int device, unsigned* code)
{
  if (device < 0 || device >= 64 || code == nullptr) return fail(U15C_EINVAL, "bad argument");
  int cur = 0;
  cudaGetDevice(&cur);
  if (cur != device) cudaSetDevice(device);
  DevState* d = dev();
  int rc = U15C_OK;
  if (d == nullptr) {
    rc = U15C_ECUDA;
  } else {
    unsigned v = 0;
    cudaError_t e = cudaMemcpy(&v, d->err, sizeof(unsigned), cudaMemcpyDeviceToHost);
    if (e == cudaSuccess) e = cudaMemset(d->err, 0, sizeof(unsigned));
    if (e != cudaSuccess) rc = cuda_fail(e, "reading the status word");
    *code = v;
  }
  if (cur != device) cudaSetDevice(cur);
  return rc;
}

int u15c_set_wait_limit(int device, unsigned long long ns)
{
  if (device < 0 || device >= 64) return fail(U15C_EINVAL, "device index out of range");
  int cur = 0;
  cudaGetDevice(&cur);
  int rc = dev_init(device);
  if (rc == U15C_OK) {
    const uint64_t v = ns;
    cudaError_t e = cudaSetDevice(device);
    if (e == cudaSuccess)
      e = cudaMemcpy(reinterpret_cast<uint8_t*>(g_dev[device].err) + 8, &v, sizeof v,
                     cudaMemcpyHostToDevice);
    if (e != cudaSuccess) rc = cuda_fail(e, "setting the wait limit");
  }
  cudaSetDevice(cur);
  return rc;
}

int u15c_wait_counter(u15c_stream stream, const unsigned long long* counter,
                      unsigned long long target)
{
  if (counter == nullptr) return fail(U15C_EINVAL, "wait_counter: null counter");
  DevState* d = dev();
  if (d == nullptr) return U15C_ECUDA;
  if (launch_tp_wait(counter, target, d->err, ST(stream)))
    return fail(U15C_ECUDA, "wait_counter: kernel launch failed");
  return U15C_OK;
}

int u15c_sync(u15c_stream stream)
{
  cudaError_t e = cudaStreamSynchronize(ST(stream));
  if (e != cudaSuccess) return cuda_fail(e, "cudaStreamSynchronize");
  int device = 0;
  cudaGetDevice(&device);
  unsigned code = 0;
  const int rc = u15c_device_status(device, &code);
  if (rc) return rc;
  if (code != 0) {
    char buf[96];
    std::snprintf(buf, sizeof buf, "a kernel's bounded wait ran out (status 0x%x)", code);
    return fail(U15C_EDEVICE, buf);
  }
  return U15C_OK;
}

// ---------------------------------------------------------------- GEMMs
int u15c_linear_bf16(u15c_stream stream, const void* x, const void* w, const void* bias, void* y,
                     int M, int K, int N)
{
  GemmArgs a;
  a.x = x;
  a.w = w;
  a.bias = bias;
  a.y = y;
  a.M = M;
  a.K = K;
  a.N = N;
  return run_gemm(a, ST(stream));
}

int u15c_mot_linear_bf16(u15c_stream stream, const void* x, const void* w_stack, int n_experts,
                         const int* seg_off, const int* seg_expert, int nseg, int epilogue,
                         const void* bias, const void* resid, void* y, int M, int K, int N)
{
  if (epilogue < 0 || epilogue > 2) return fail(U15C_EINVAL, "unknown epilogue");
  GemmArgs a;
  a.x = x;
  a.w = w_stack;
  a.n_experts = n_experts;
  a.seg_off = seg_off;
  a.seg_expert = seg_expert;
  a.nseg = nseg;
  a.epilogue = epilogue;
  a.bias = bias;
  a.resid = resid;
  a.y = y;
  a.M = M;
  a.K = K;
  a.N = N;
  return run_gemm(a, ST(stream));
}

int u15c_quant_rows_i8(u15c_stream stream, const void* x, int8_t* q, float* scale, int rows,
                       int cols)
{
  if (x == nullptr || q == nullptr || scale == nullptr || cols <= 0 || cols % 8)
    return fail(U15C_EINVAL, "quant_rows_i8: null buffer or cols not a multiple of 8");
  LAUNCH(launch_quant_rows(x, q, scale, rows, cols, ST(stream)), "quant_rows_i8");
}

int u15c_linear_i8(u15c_stream stream, const int8_t* xq, const float* s_tok, const int8_t* wq,
                   const float* s_ch, const void* bias, void* y, int32_t* acc_dump, int M, int K,
                   int N)
{
  GemmArgs a;
  a.int8 = true;
  a.x = xq;
  a.w = wq;
  a.s_tok = s_tok;
  a.s_ch = s_ch;
  a.bias = bias;
  a.y = y;
  a.acc_dump = acc_dump;
  a.M = M;
  a.K = K;
  a.N = N;
  return run_gemm(a, ST(stream));
}

int u15c_mot_linear_i8(u15c_stream stream, const int8_t* xq, const float* s_tok,
                       const int8_t* wq_stack, const float* s_ch_stack, int n_experts,
                       const int* seg_off, const int* seg_expert, int nseg, int epilogue,
                       const void* resid, void* y, int32_t* acc_dump, int M, int K, int N)
{
  if (epilogue < 0 || epilogue > 2) return fail(U15C_EINVAL, "unknown epilogue");
  GemmArgs a;
  a.int8 = true;
  a.x = xq;
  a.w = wq_stack;
  a.s_tok = s_tok;
  a.s_ch = s_ch_stack;
  a.n_experts = n_experts;
  a.seg_off = seg_off;
  a.seg_expert = seg_expert;
  a.nseg = nseg;
  a.epilogue = epilogue;
  a.resid = resid;
  a.y = y;
  a.acc_dump = acc_dump;
  a.M = M;
  a.K = K;
  a.N = N;
  return run_gemm(a, ST(stream));
}

// ---------------------------------------------------------------- norms etc.
int u15c_rms_norm(u15c_stream stream, const void* x, const void* w, void* y, int rows, int dim,
                  float eps)
{
  return u15c_mot_rms_norm(stream, x, w, 1, nullptr, nullptr, 0, y, rows, dim, eps);
}

int u15c_mot_rms_norm(u15c_stream stream, const void* x, const void* w_stack, int n_experts,
                      const int* seg_off, const int* seg_expert, int nseg, void* y, int rows,
                      int dim, float eps)
{
  if (x == nullptr || w_stack == nullptr || y == nullptr || dim <= 0 || dim % 8)
    return fail(U15C_EINVAL, "rms_norm: null buffer or dim not a multiple of 8");
  SegInfo seg;
  std::string err;
  if (!fill_seg(&seg, seg_off, seg_expert, nseg, rows, n_experts, &err))
    return fail(U15C_EINVAL, "rms_norm: " + err);
  LAUNCH(launch_rms_norm(x, w_stack, y, rows, dim, eps, seg, ST(stream)), "rms_norm");
}

int u15c_mot_rms_norm_quant_i8(u15c_stream stream, const void* x, const void* w_stack,
                               int n_experts, const int* seg_off, const int* seg_expert, int nseg,
                               int8_t* q, float* scale, int rows, int dim, float eps)
{
  if (x == nullptr || w_stack == nullptr || q == nullptr || scale == nullptr || dim <= 0 ||
      dim % 8 || dim > 4096)
    return fail(U15C_EINVAL, "rms_norm_quant: null buffer, or dim not a multiple of 8 up to 4096");
  SegInfo seg;
  std::string err;
  if (!fill_seg(&seg, seg_off, seg_expert, nseg, rows, n_experts, &err))
    return fail(U15C_EINVAL, "rms_norm_quant: " + err);
  LAUNCH(launch_rms_norm_quant(x, w_stack, q, scale, rows, dim, eps, seg, ST(stream)),
         "rms_norm_quant");
}

int u15c_split_qk_norm(u15c_stream stream, void* x, const void* w_t, const void* w_hw, int heads,
                       int tokens, int head_dim, float eps)
{
  if (head_dim != 128) return fail(U15C_EINVAL, "split_qk_norm: head_dim must be 128");
  if (x == nullptr || w_t == nullptr || w_hw == nullptr)
    return fail(U15C_EINVAL, "split_qk_norm: null buffer");
  LAUNCH(launch_split_qk_norm(x, w_t, w_hw, heads, tokens, eps, ST(stream)), "split_qk_norm");
}

int u15c_split_rope(u15c_stream stream, void* x, const float* cos_tab, const float* sin_tab,
                    int heads, int tokens, int head_dim, int d_t, int d_h)
{
  if (head_dim != 128 || d_t != 64 || d_h != 32)
    return fail(U15C_EINVAL, "split_rope: the t/h/w ranges must be 64/32/32 of a 128 head");
  if (x == nullptr || cos_tab == nullptr || sin_tab == nullptr)
    return fail(U15C_EINVAL, "split_rope: null buffer");
  LAUNCH(launch_split_rope(x, cos_tab, sin_tab, heads, tokens, ST(stream)), "split_rope");
}

int u15c_build_rope_tables(u15c_stream stream, const int32_t* pos_t, const int32_t* pos_h,
                           const int32_t* pos_w, int tokens, int head_dim, int d_t, int d_h,
                           double theta_t, double theta_hw, float* cos_tab, float* sin_tab)
{
  if (head_dim != 128 || d_t + 2 * d_h != 128 || d_t % 2 || d_h % 2)
    return fail(U15C_EINVAL, "build_rope_tables: ranges must tile a 128 head");
  if (pos_t == nullptr || pos_h == nullptr || pos_w == nullptr || cos_tab == nullptr ||
      sin_tab == nullptr)
    return fail(U15C_EINVAL, "build_rope_tables: null buffer");
  LAUNCH(launch_rope_tables(pos_t, pos_h, pos_w, tokens, d_t, d_h, theta_t, theta_hw, cos_tab,
                            sin_tab, ST(stream)),
         "build_rope_tables");
}

int u15c_qkv_post(u15c_stream stream, const void* qkv, const void* norms_stack, int n_experts,
                  const int* seg_off, const int* seg_expert, int nseg, const float* cos_tab,
                  const float* sin_tab, void* q_out, void* k_cache, void* v_cache,
                  const int32_t* page_table, int cap, int heads, int kv_heads, int T, int kv_off,
                  float eps)
{
  if (qkv == nullptr || norms_stack == nullptr || cos_tab == nullptr || sin_tab == nullptr ||
      q_out == nullptr || k_cache == nullptr || v_cache == nullptr)
    return fail(U15C_EINVAL, "qkv_post: null buffer");
  if (page_table == nullptr && kv_off + T > cap)
    return fail(U15C_EINVAL, "qkv_post: KV cache too small for kv_off + T");
  SegInfo seg;
  std::string err;
  if (!fill_seg(&seg, seg_off, seg_expert, nseg, T, n_experts, &err))
    return fail(U15C_EINVAL, "qkv_post: " + err);
  const KvView kv = kv_view(k_cache, v_cache, page_table, cap, kv_heads);
  LAUNCH(launch_qkv_post(qkv, norms_stack, cos_tab, sin_tab, q_out, kv, T, heads, kv_heads,
                         kv_off, eps, seg, ST(stream)),
         "qkv_post");
}

int u15c_transpose_thd(u15c_stream stream, const void* in, void* out, int T, int H, int D)
{
  if (in == nullptr || out == nullptr || D % 8) return fail(U15C_EINVAL, "transpose_thd: bad args");
  LAUNCH(launch_transpose(in, out, T, H, D, true, ST(stream)), "transpose_thd");
}

int u15c_transpose_htd(u15c_stream stream, const void* in, void* out, int T, int H, int D)
{
  if (in == nullptr || out == nullptr || D % 8) return fail(U15C_EINVAL, "transpose_htd: bad args");
  LAUNCH(launch_transpose(in, out, T, H, D, false, ST(stream)), "transpose_htd");
}

int u15c_transpose_into_cache(u15c_stream stream, const void* in, void* cache, int T, int H,
                              int D, int cap, int offset)
{
  if (D != 128) return fail(U15C_EINVAL, "transpose_into_cache: head_dim must be 128");
  if (in == nullptr || cache == nullptr || offset < 0 || offset + T > cap)
    return fail(U15C_EINVAL, "transpose_into_cache: cache too small for offset + T");
  LAUNCH(launch_kv_append(in, cache, nullptr, (long)kPageTokens * 128, (long)cap * 128, T, H,
                          offset, ST(stream)),
         "transpose_into_cache");
}

int u15c_kv_append(u15c_stream stream, const void* in, void* pages, const int32_t* page_table,
                   int T, int H, int offset)
{
  if (in == nullptr || pages == nullptr || page_table == nullptr || offset < 0)
    return fail(U15C_EINVAL, "kv_append: null buffer");
  LAUNCH(launch_kv_append(in, pages, page_table, (long)H * kPageTokens * 128,
                          (long)kPageTokens * 128, T, H, offset, ST(stream)),
         "kv_append");
}

// ---------------------------------------------------------------- elementwise
int u15c_swiglu(u15c_stream stream, const void* gate, const void* up, void* y, int rows, int inter)
{
  const long n = (long)rows * inter;
  if (gate == nullptr || up == nullptr || y == nullptr || n % 8)
    return fail(U15C_EINVAL, "swiglu: null buffer or size not a multiple of 8");
  LAUNCH(launch_swiglu(gate, up, y, n, ST(stream)), "swiglu");
}

int u15c_add(u15c_stream stream, void* dst, const void* src, long n)
{
  if (dst == nullptr || src == nullptr || n % 8)
    return fail(U15C_EINVAL, "add: null buffer or n not a multiple of 8");
  LAUNCH(launch_add(dst, src, n, ST(stream)), "add");
}

int u15c_add_row(u15c_stream stream, void* dst, const void* row, int rows, int dim)
{
  if (dst == nullptr || row == nullptr || dim % 8)
    return fail(U15C_EINVAL, "add_row: null buffer or dim not a multiple of 8");
  LAUNCH(launch_add_row(dst, row, rows, dim, ST(stream)), "add_row");
}

int u15c_silu(u15c_stream stream, void* x, long n)
{
  if (x == nullptr || n % 8) return fail(U15C_EINVAL, "silu: null buffer or n not a multiple of 8");
  LAUNCH(launch_silu(x, n, ST(stream)), "silu");
}

// ---------------------------------------------------------------- attention
size_t u15c_sage_workspace_bytes(int hq, int hkv, int tq, int tk)
{
  return sage_bytes(hq, hkv, tq, tk);
}

int u15c_attention(u15c_stream stream, const void* q, const void* k, const void* v,
                   const int32_t* page_table, int cap, void* out, int hq, int hkv, int tq, int tk,
                   int head_dim, int mode, int q_offset, const int32_t* t_index, void* sage_ws)
{
  if (head_dim != 128) return fail(U15C_EINVAL, "attention: head_dim must be 128");
  if (page_table == nullptr && tk > cap)
    return fail(U15C_EINVAL, "attention: key length exceeds the cache capacity");
  return run_attention(ST(stream), q, kv_view(const_cast<void*>(k), const_cast<void*>(v),
                                              page_table, cap, hkv),
                       out, hq, hkv, tq, tk, mode, q_offset, t_index, sage_ws);
}

int u15c_attention_paged(u15c_stream stream, const void* q, const void* k_pages,
                         const void* vt_pages, const int32_t* page_table, int n_pages, void* out,
                         int hq, int hkv, int tq, int tk, int head_dim, int mode, int q_offset,
                         const int32_t* t_index, void* sage_ws)
{
  if (head_dim != 128) return fail(U15C_EINVAL, "attention: head_dim must be 128");
  if (n_pages <= 0) return fail(U15C_EINVAL, "attention: n_pages must be positive");
  KvView kv;
  kv.k = const_cast<void*>(k_pages);
  kv.v = const_cast<void*>(vt_pages);
  kv.page_table = page_table;
  kv.page_stride = (long)hkv * kPageTokens * kHeadDim;
  kv.head_stride = (long)kPageTokens * kHeadDim;
  kv.v_t = true;
  return run_attention_tc(ST(stream), q, kv, n_pages, out, hq, hkv, tq, tk, mode, q_offset,
                          t_index, sage_ws);
}

int u15c_sdpa(u15c_stream stream, const void* q, const void* k, const void* v, void* out, int hq,
              int hkv, int tq, int tk, int d, int cap, int causal, int q_offset)
{
  return u15c_attention(stream, q, k, v, nullptr, cap, out, hq, hkv, tq, tk, d,
                        causal ? U15C_ATTN_CAUSAL : U15C_ATTN_BIDIRECTIONAL, q_offset, nullptr,
                        nullptr);
}

int u15c_sdpa_steel(u15c_stream stream, const void* q, const void* k, const void* v, void* out,
                    int hq, int hkv, int tq, int tk, int d, int cap, void* sage_ws)
{
  return u15c_attention(stream, q, k, v, nullptr, cap, out, hq, hkv, tq, tk, d,
                        U15C_ATTN_BIDIRECTIONAL, 0, nullptr, sage_ws);
}

int u15c_sdpa_block_causal(u15c_stream stream, const void* q, const void* k, const void* v,
                           void* out, const int32_t* t_index, int hq, int hkv, int tq, int tk,
                           int d, int cap, int q_offset)
{
  return u15c_attention(stream, q, k, v, nullptr, cap, out, hq, hkv, tq, tk, d,
                        U15C_ATTN_BLOCK_CAUSAL, q_offset, t_index, nullptr);
}

}  // extern "C"
