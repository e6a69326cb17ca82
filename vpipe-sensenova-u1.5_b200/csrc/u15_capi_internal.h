// Shared internals of the C ABI implementation (u15_capi.cu, u15_model.cu).
#pragma once

#include "../../include/u15c.h"
#include "u15_kernels.h"

#include <cuda_runtime.h>

#include <string>

namespace u15 {

struct DevState {
  bool ready = false;
  int sms = 148;
  unsigned* err = nullptr;   // device status block: watchdog code, then the wait limit
};

// Set this thread's last error and return `code`.
int fail(int code, const std::string& msg);
int cuda_fail(cudaError_t e, const char* what);

int dev_init(int device);

// Runs the enclosing C-ABI call on `device` (the one its model was created
// on) and gives the caller back its own current device on return, so a
// handle used from a thread or process whose current device differs still
// launches where its memory lives.
struct DeviceScope {
  int prev = -1;
  explicit DeviceScope(int device)
  {
    int cur = 0;
    if (cudaGetDevice(&cur) == cudaSuccess && cur != device && cudaSetDevice(device) == cudaSuccess)
      prev = cur;
  }
  ~DeviceScope()
  {
    if (prev >= 0) cudaSetDevice(prev);
  }
  DeviceScope(const DeviceScope&) = delete;
  DeviceScope& operator=(const DeviceScope&) = delete;
};
DevState* dev();   // state of the current device, initialised on first use

bool fill_seg(SegInfo* s, const int* off, const int* ex, int nseg, int rows, int n_experts,
              std::string* err);
KvView kv_view(void* k, void* v, const int32_t* page_table, int cap, int hkv);

struct SageWs {
  int8_t* q8;
  int8_t* k8;
  float* sq;
  float* sk;
  float* kmean;
};
size_t sage_bytes(int hq, int hkv, int tq, int tk);
SageWs sage_split(void* ws, int hq, int hkv, int tq, int tk);

// The checks every attention entry makes before it launches anything (the
// Sage prologue included): head counts and, for the mma.sync kernel
// (`legacy`), its GQA group limit; the rule, its t-index vector and the
// queries' place among the keys. U15C_OK or the refusal (message set).
int check_attention(int hq, int hkv, int tq, int tk, int mode, int q_offset,
                    const int32_t* t_index, bool sage, bool legacy);
// The mma.sync kernel: any K/V layout (contiguous, paged, transposed V).
int run_attention(cudaStream_t st, const void* q, const KvView& kv, void* out, int hq, int hkv,
                  int tq, int tk, int mode, int q_offset, const int32_t* t_index, void* sage_ws);
int run_gemm(GemmArgs& a, cudaStream_t st);
// The tcgen05 kernel over a paged cache with transposed V pages (the model's
// layout): every rule, Sage (bidirectional) when sage_ws is non-null. A
// block-causal call the kernel does not serve (an unaligned t-index vector,
// more than 32768 keys) runs on the mma.sync kernel.
int run_attention_tc(cudaStream_t st, const void* q, const KvView& kv, int n_pages, void* out,
                     int hq, int hkv, int tq, int tk, int mode, int q_offset,
                     const int32_t* t_index, void* sage_ws);

}  // namespace u15
