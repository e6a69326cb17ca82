// u15c_attention_sage_static: the Sage int8-QK attention with its workspace
// (int8 Q and K copies, block scales, the K channel means) in a fixed
// device array compiled into this library, for callers that cannot
// allocate device memory themselves -- a host that plans all of its device
// memory before the first call and may not grow it afterwards (the vpipe
// stage declares its scratch during planning), a process whose free device
// memory is already reserved by another allocator, or a latency-bound
// caller that cannot take cudaMalloc/cudaFree's implicit synchronisation.
//
// The array holds kStaticSageBytes (24 MiB) on every GPU that loads this
// library, until the process exits. Requests whose workspace would exceed
// it are refused with U15C_EINVAL before anything is launched.
//
// Set-up: the first call on a device (with that device current) resolves
// the array's device address with cudaGetSymbolAddress and caches it; that
// first call should come before any stream capture on that device. Later
// calls do no set-up.
//
// Every call uses the same array, which keeps the previous call's contents.
// The prologue rewrites every byte the attention kernel reads (Q codes for
// the rows in use, all K rows including the zero padding of the last block,
// every scale and channel mean), so nothing needs clearing between calls.
// Calls that overlap on the GPU (other streams, other host threads) race on
// the array: serialise them.
//
// No cudaMalloc, cudaFree or allocating library routine is called here.
#include "u15_capi_internal.h"

#include <mutex>

namespace {

constexpr size_t kStaticSageBytes = 24ull << 20;
constexpr int kMaxDevices = 64;

__device__ __align__(256) unsigned char g_sage_static[kStaticSageBytes];

void* g_static_addr[kMaxDevices] = {};
std::mutex g_static_mu;

// Device address of g_sage_static on the current device (set up once).
int static_workspace(void** out)
{
  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) return u15::cuda_fail(e, "cudaGetDevice");
  if (device < 0 || device >= kMaxDevices) return u15::fail(U15C_EINVAL, "device index out of range");
  std::lock_guard<std::mutex> g(g_static_mu);
  if (g_static_addr[device] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_sage_static);
    if (e != cudaSuccess) return u15::cuda_fail(e, "cudaGetSymbolAddress(static Sage workspace)");
    g_static_addr[device] = p;
  }
  *out = g_static_addr[device];
  return U15C_OK;
}

}  // namespace

extern "C" {

int u15c_attention_sage_static(u15c_stream stream, const void* q, const void* k, const void* v,
                               const int32_t* page_table, int cap, void* out, int hq, int hkv,
                               int tq, int tk, int head_dim)
{
  if (head_dim != 128) return u15::fail(U15C_EINVAL, "attention: head_dim must be 128");
  if (q == nullptr || k == nullptr || v == nullptr || out == nullptr)
    return u15::fail(U15C_EINVAL, "attention: null buffer");
  // every refusal comes before anything is launched or the array is touched
  int rc = u15::check_attention(hq, hkv, tq, tk, 0, 0, nullptr, true, true);
  if (rc) return rc;
  if (page_table == nullptr && tk > cap)
    return u15::fail(U15C_EINVAL, "attention: key length exceeds the cache capacity");
  const size_t need = u15::sage_bytes(hq, hkv, tq, tk);
  if (need > kStaticSageBytes)
    return u15::fail(U15C_EINVAL, "attention: this geometry needs " + std::to_string(need) +
                                      " bytes of Sage workspace; the static workspace holds " +
                                      std::to_string(kStaticSageBytes) +
                                      " (use u15c_attention with a caller-provided workspace)");
  if (tq == 0 || tk == 0) return U15C_OK;
  void* ws = nullptr;
  rc = static_workspace(&ws);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const u15::KvView kv =
      u15::kv_view(const_cast<void*>(k), const_cast<void*>(v), page_table, cap, hkv);
  const u15::SageWs s = u15::sage_split(ws, hq, hkv, tq, tk);
  std::string err;
  if (u15::sage_prepare(q, kv, hq, hkv, tq, tk, s.q8, s.k8, s.sq, s.sk, s.kmean, st, &err))
    return u15::fail(U15C_ECUDA, err);
  u15::AttnArgs a;
  a.q = q;
  a.kv = kv;
  a.out = out;
  a.hq = hq;
  a.hkv = hkv;
  a.tq = tq;
  a.tk = tk;
  a.mode = 0;
  a.q8 = s.q8;
  a.k8 = s.k8;
  a.sq = s.sq;
  a.sk = s.sk;
  rc = u15::attention(a, st, &err);
  if (rc) return u15::fail(rc == 1 ? U15C_EINVAL : U15C_ECUDA, err);
  return U15C_OK;
}

}  // extern "C"
