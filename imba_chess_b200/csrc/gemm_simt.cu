// fp32-accumulating SIMT GEMM, acc = A[M, K] . W[N, K]^T, with a fused
// epilogue.  This is the exact-fp32 path (the fp32 parity mode, max abs error
// 1e-4) and the fallback for shapes the tensor-core kernel does not take.
// 64 x 64 output tile per 256-thread CTA, 4 x 4 outputs per thread, K staged
// through shared memory in 16-wide slices.
#include "epilogues.cuh"

namespace imba {
namespace {

constexpr int kBM = 64, kBN = 64, kBK = 16;

template <typename TA, typename TW, class Epi>
__global__ void __launch_bounds__(256) gemm_simt_kernel(const TA* __restrict__ A, int lda, const TW* __restrict__ W,
                                                        int ldw, int M, int N, int K, Epi epi) {
  pdl_wait();
  pdl_trigger();
  __shared__ float As[kBK][kBM + 4];
  __shared__ float Ws[kBK][kBN + 4];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int m0 = blockIdx.y * kBM, n0 = blockIdx.x * kBN;
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;

  for (int k0 = 0; k0 < K; k0 += kBK) {
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const int i = threadIdx.x + 256 * t;
      const int row = i / kBK, k = i % kBK;
      const int gk = k0 + k;
      const int gm = m0 + row, gn = n0 + row;
      As[k][row] = (gm < M && gk < K) ? to_f(A[(size_t)gm * lda + gk]) : 0.f;
      Ws[k][row] = (gn < N && gk < K) ? to_f(W[(size_t)gn * ldw + gk]) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < kBK; ++k) {
      float a[4], w[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[k][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) w[j] = Ws[k][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], w[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = m0 + ty * 4 + i;
    if (r >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int c = n0 + tx * 4 + j;
      if (c < N) epi(r, c, acc[i][j]);
    }
  }
}

}  // namespace

template <typename TA, typename TW, class Epi>
cudaError_t launch_gemm_simt(const TA* A, int lda, const TW* W, int ldw, int M, int N, int K, Epi epi,
                             cudaStream_t s) {
  if (M <= 0 || N <= 0) return cudaSuccess;
  dim3 grid((N + kBN - 1) / kBN, (M + kBM - 1) / kBM);
  return launch_pdl(gemm_simt_kernel<TA, TW, Epi>, grid, dim3(256), 0, s, A, lda, W, ldw, M, N, K, epi);
}

#define IMBA_INST(TA, TW, EPI) \
  template cudaError_t launch_gemm_simt<TA, TW, EPI>(const TA*, int, const TW*, int, int, int, int, EPI, cudaStream_t);
IMBA_INST(float, float, EpiUVQK<float>)
IMBA_INST(bf16, bf16, EpiUVQK<bf16>)
IMBA_INST(float, float, EpiResidual)
IMBA_INST(bf16, bf16, EpiResidual)
IMBA_INST(float, float, EpiStore)
IMBA_INST(float, float, EpiBiasSilu)
IMBA_INST(bf16, bf16, EpiBiasSilu)
IMBA_INST(float, float, EpiContent)
IMBA_INST(bf16, bf16, EpiContent)
#undef IMBA_INST

}  // namespace imba
