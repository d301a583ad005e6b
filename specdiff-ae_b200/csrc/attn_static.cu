// Verify attention with no caller workspace and no allocation per call: the
// split-KV partials go to a fixed 24 MiB device array of this library.
//
// The array's address is resolved once per device (cudaGetSymbolAddress with
// that device current) on the first call there; that call must come before
// any stream capture.  Calls on one device share the array, so they must not
// overlap (serialise them on one stream).  Nothing in the array needs to
// start at zero: every partial row the merge reads is written by the same
// launch first.  Requests needing more than the array holds are rejected
// with TV_ERR_WORKSPACE before anything is launched.
#include <cuda_runtime.h>

#include <mutex>

#include "common.cuh"
#include "specverify.h"

namespace {

constexpr size_t kStaticScratchBytes = size_t(24) << 20;
constexpr int kMaxDevices = 64;

__device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

std::mutex g_static_mu;
void* g_static_addr[kMaxDevices] = {};

}  // namespace

extern "C" int tv_verify_attn_static(const tv_attn_args* a, void* stream) {
  if (!a) return TV_ERR_NULL;
  size_t need = 0;
  const int rc = tv_attn_workspace_size(a, &need);
  if (rc != TV_OK) return rc;
  if (need > kStaticScratchBytes) return TV_ERR_WORKSPACE;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return tv::record_cuda_error(e);
  if (dev < 0 || dev >= kMaxDevices) return TV_ERR_UNSUPPORTED;
  void* base = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_static_mu);
    if (!g_static_addr[dev]) {
      void* ptr = nullptr;
      e = cudaGetSymbolAddress(&ptr, g_static_scratch);
      if (e != cudaSuccess) return tv::record_cuda_error(e);
      g_static_addr[dev] = ptr;
    }
    base = g_static_addr[dev];
  }
  tv_attn_args b = *a;
  b.workspace = base;
  b.workspace_bytes = kStaticScratchBytes;
  return tv_verify_attn(&b, stream);
}
