// Tensor-core (tcgen05 + TMA) GEMMs of the bf16 step.  Each launcher returns
// false when the handle has no tensor-core state (fp32 handles, or the SIMT
// GEMM test hook); the caller then runs the SIMT GEMM for an fp32 or hooked
// handle and reports IMBA_ERR_UNSUPPORTED otherwise.  When it returns true,
// *err holds the launch status.
#pragma once

#include "epilogues.cuh"

namespace imba {

// Encodes the weights' TMA descriptors once per model (bf16 models only);
// IMBA_ERR_UNSUPPORTED / IMBA_ERR_ARG when a bf16 handle's weights cannot be
// served by the tensor-core GEMMs.
imba_status_t gemm_tc_prepare(imba_model* m);
void gemm_tc_release(imba_model* m);

template <typename T>
bool gemm_tc_launch_uvqk(const imba_model* m, int layer, int rows, const T* xn, const EpiUVQK<T>& epi,
                         cudaStream_t s, cudaError_t* err);
template <typename T>
bool gemm_tc_launch_out(const imba_model* m, int layer, int rows, const T* gated, const EpiResidual& epi,
                        int32_t* status, cudaStream_t s, cudaError_t* err);
template <typename T>
bool gemm_tc_launch_policy(const imba_model* m, int rows, const T* xf3, const EpiStore& epi, int32_t* status,
                           cudaStream_t s, cudaError_t* err);
// Board projection + embeddings: pooled3 [rows, 192] split bf16 against the
// handle's [d, 192] split copy of the projection.
bool gemm_tc_launch_content(const imba_model* m, int rows, const bf16* pooled3, const EpiContent& epi,
                            int32_t* status, cudaStream_t s, cudaError_t* err);
template <typename T>
bool gemm_tc_launch_value(const imba_model* m, int rows, const T* xin, int lda, const EpiBiasSilu& epi,
                          int32_t* status, cudaStream_t s, cudaError_t* err);

}  // namespace imba
