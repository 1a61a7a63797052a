// Placeholder until the tcgen05 kernel lands: no shape is handled here, so
// every GEMM takes the SIMT path.
#include "gemm_tc.cuh"

namespace imba {

imba_status_t gemm_tc_prepare(imba_model*) { return IMBA_OK; }

template <typename T>
bool gemm_tc_launch_uvqk(const imba_model*, int, int, const T*, const EpiUVQK<T>&, cudaStream_t, cudaError_t*) {
  return false;
}
template <typename T>
bool gemm_tc_launch_out(const imba_model*, int, int, const T*, const EpiResidual&, cudaStream_t, cudaError_t*) {
  return false;
}
template <typename T>
bool gemm_tc_launch_policy(const imba_model*, int, const T*, const T*, float*, cudaStream_t, cudaError_t*) {
  return false;
}
template bool gemm_tc_launch_uvqk<float>(const imba_model*, int, int, const float*, const EpiUVQK<float>&, cudaStream_t, cudaError_t*);
template bool gemm_tc_launch_uvqk<bf16>(const imba_model*, int, int, const bf16*, const EpiUVQK<bf16>&, cudaStream_t, cudaError_t*);
template bool gemm_tc_launch_out<float>(const imba_model*, int, int, const float*, const EpiResidual&, cudaStream_t, cudaError_t*);
template bool gemm_tc_launch_out<bf16>(const imba_model*, int, int, const bf16*, const EpiResidual&, cudaStream_t, cudaError_t*);
template bool gemm_tc_launch_policy<float>(const imba_model*, int, const float*, const float*, float*, cudaStream_t, cudaError_t*);
template bool gemm_tc_launch_policy<bf16>(const imba_model*, int, const bf16*, const bf16*, float*, cudaStream_t, cudaError_t*);

}  // namespace imba
