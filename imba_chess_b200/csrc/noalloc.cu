// imba_step_noalloc: the jagged decode / prefill step for callers that cannot
// allocate device memory themselves.
//
// Who needs it: a host that embeds this library inside a runtime that owns all
// of the GPU's memory up front (a serving framework whose caching allocator
// must see every byte, or a process started with a fixed memory budget) and
// therefore may not call cudaMalloc or hand the library a freshly allocated
// workspace at decode time; or a small C/C++ engine driver that wants a fixed
// footprint decided at load time.  imba_step needs a caller-provided
// workspace; this variant uses a scratch array compiled into the library.
//
// The scratch is one file-scope device array of IMBA_NOALLOC_SCRATCH_BYTES.
// Every GPU that loads the library holds it until the process exits.  Its
// device address is looked up once per device (cudaGetSymbolAddress, with
// that device current) on the first call made on the device and cached; make
// that first call before any stream capture.  All calls share the array: two
// calls that overlap on the GPU (different streams, or different host threads
// on one device) race on it and must be serialised by the caller.  No part of
// the scratch needs to start at zero: every scratch byte the step reads is
// written earlier in the same call, so the previous call's contents are never
// observed.
#include <mutex>

#include "common.cuh"

namespace {

static __device__ __align__(256) unsigned char g_noalloc_scratch[IMBA_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_addr[kMaxDevices] = {};

// Device address of the scratch array on the current device.
imba_status_t scratch_for_current_device(void** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) return IMBA_ERR_CUDA;
  if (dev < 0 || dev >= kMaxDevices) return IMBA_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) return IMBA_ERR_CUDA;
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return IMBA_OK;
}

}  // namespace

extern "C" imba_status_t imba_step_noalloc(const imba_model* model, const imba_step_desc* step,
                                           const imba_pool_desc* pool, void* stream) {
  if (!model || !step || step->num_rows < 0) return IMBA_ERR_ARG;
  const size_t need = imba_step_workspace_bytes(model, step->num_rows);
  if (need > (size_t)IMBA_NOALLOC_SCRATCH_BYTES) return IMBA_ERR_OOM;  // too many rows for the fixed scratch
  void* scratch = nullptr;
  const imba_status_t s = scratch_for_current_device(&scratch);
  if (s != IMBA_OK) return s;
  return imba_step(model, step, pool, scratch, (size_t)IMBA_NOALLOC_SCRATCH_BYTES, stream);
}
