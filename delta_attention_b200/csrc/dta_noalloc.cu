// dta_decode_noalloc: the decode path of dta_decode with its scratch (the
// split-K partials) held in a file-scope device array instead of a caller
// workspace, for callers that cannot allocate device memory (see the header).
#include <cuda_runtime.h>
#include <stddef.h>

#include <mutex>

#include "delta_attention_b200.h"
#include "dta_internal.h"

namespace {

// One array per device that loads this library; shared by every call.
static __device__ __align__(256) unsigned char g_decode_scratch[DTA_DECODE_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
void* g_scratch_addr[kMaxDevices] = {};
std::mutex g_scratch_mu;

// Device address of g_decode_scratch on the current device.  In host code the
// array's name is only a host-side stand-in, so the address is looked up with
// cudaGetSymbolAddress once per device (that device current) and cached.
int scratch_for_current_device(void** out) {
  // an unsupported device is reported as such, before any symbol lookup
  int sms = 0;
  const int st = dta::check_device(&sms);
  if (st != DTA_OK) return st;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return dta::fail_cuda(e);
  if (dev < 0 || dev >= kMaxDevices) return DTA_ERR_UNSUPPORTED_DEVICE;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    if ((e = cudaGetSymbolAddress(&p, g_decode_scratch)) != cudaSuccess) return dta::fail_cuda(e);
    if (p == nullptr) return dta::fail_cuda(cudaErrorInvalidSymbol);
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return DTA_OK;
}

}  // namespace

extern "C" int dta_decode_noalloc(const dta_decode_args* args, void* stream) {
  if (!args) return DTA_ERR_INVALID_ARG;
  dta_decode_args a = *args;
  a.workspace = nullptr;
  a.workspace_bytes = 0;
  const size_t need = dta_decode_workspace_size(&a);
  if (need == 0) return dta_decode(&a, stream);  // invalid arguments: dta_decode reports which
  if (need > (size_t)DTA_DECODE_NOALLOC_SCRATCH_BYTES) return DTA_ERR_SCRATCH_LIMIT;
  void* scratch = nullptr;
  const int st = scratch_for_current_device(&scratch);
  if (st != DTA_OK) return st;
  a.workspace = scratch;
  a.workspace_bytes = DTA_DECODE_NOALLOC_SCRATCH_BYTES;
  return dta_decode(&a, stream);
}
