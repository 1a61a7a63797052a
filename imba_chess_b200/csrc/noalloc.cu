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
// With lazy module loading (the CUDA default) the array is placed on a device
// when this module is first used there, and stays until the process exits.
// imba_model_create does that on the handle's device (noalloc_prepare_device
// below), so the array is resident before any step runs, while the caller can
// still allocate.  Every imba_step_noalloc call looks the array's device
// address up again (cudaGetSymbolAddress, cheap once the module is loaded),
// so no address is cached across a device reset.  All calls share the array:
// two calls that overlap on the GPU (different streams, or different host
// threads on one device) race on it and must be serialised by the caller.
// No part of the scratch needs to start at zero: every scratch byte the step
// reads is written earlier in the same call (the attention work-queue
// counters are cleared by the step itself), so the previous call's contents
// are never observed.
#include "common.cuh"

namespace {

static __device__ __align__(256) unsigned char g_noalloc_scratch[IMBA_NOALLOC_SCRATCH_BYTES];

// Device address of the scratch array on the current device.
imba_status_t scratch_for_current_device(void** out) {
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
  if (e != cudaSuccess || p == nullptr) {
    cudaGetLastError();
    return IMBA_ERR_CUDA;
  }
  *out = p;
  return IMBA_OK;
}

}  // namespace

namespace imba {

// Places the scratch array on the current device (loads this module there).
imba_status_t noalloc_prepare_device() {
  void* p = nullptr;
  return scratch_for_current_device(&p);
}

}  // namespace imba

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
