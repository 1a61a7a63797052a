// imba_selftest_wait_timeout: the library's bounded device-side wait, run on
// an mbarrier that nothing ever arrives at, so a host can check its handling
// of device-side timeouts (IMBA_ERR_TIMEOUT in the status word, the context
// still usable afterwards) without hanging or faulting a GPU.  The wait is
// the one every pipelined kernel of the library uses (tc::mbar_wait_for);
// here its limit is the caller's instead of the production 2 s.
#include "kernels.cuh"
#include "tc_ptx.cuh"

namespace imba {
namespace {

__global__ void wait_timeout_kernel(uint64_t limit_ns, int32_t* status) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    tc::mbar_init(&bar, 1);
    tc::fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) tc::mbar_wait_for(&bar, 0, status, limit_ns);  // never completes: times out
  __syncthreads();
}

}  // namespace
}  // namespace imba

extern "C" imba_status_t imba_selftest_wait_timeout(int64_t limit_ns, int32_t* status, void* stream) {
  if (!status || limit_ns <= 0 || limit_ns > 10000000000ll) return IMBA_ERR_ARG;
  imba::wait_timeout_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>((uint64_t)limit_ns, status);
  return cudaGetLastError() == cudaSuccess ? IMBA_OK : IMBA_ERR_CUDA;
}
