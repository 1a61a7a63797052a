// Content embedding of decode/prefill tokens (fp32 SIMT):
//   board vector  = BoardSquareEncoder(piece_square_table[piece*64 + square])
//                   (src/imba_chess/model/hstu_model.py:118-179, :275-278)
//   content       = board + seq + turn + castle + ep + halfmove + fullmove
//                   + prev_move embeddings, side ids clamped to their tables
//                   (hstu_model.py:283-335)
//   x             = content * sqrt(d) + pos_emb[min(pos, max_pos - 1)]
//                   (src/imba_chess/model/position_embedding.py:52-62)
// One CTA per board: the 64 x 64 square activations stay in shared memory
// through both square-attention blocks, the mean pool and the projection.
#include "common.cuh"

namespace imba {
namespace {

constexpr int kSq = 64;
constexpr int kDim = IMBA_BOARD_DIM;
constexpr int kHeads = 4;
constexpr int kHd = kDim / kHeads;
constexpr int kLd = kDim + 1;          // padded row stride of 64-wide buffers
constexpr int kLdBig = 3 * kDim + 1;   // padded row stride of the qkv buffer
constexpr int kThreads = 256;

struct BlockParams {
  const float *an_w, *an_b, *qkv_w, *ao_w, *mn_w, *mn_b, *m0_w, *m0_b, *m2_w, *m2_b;
};

__device__ BlockParams block_params(const float* p, int b) {
  const float* q = p + (size_t)b * IMBA_BOARD_BLOCK_FLOATS;
  BlockParams r;
  r.an_w = q; q += 64;
  r.an_b = q; q += 64;
  r.qkv_w = q; q += 192 * 64;
  r.ao_w = q; q += 64 * 64;
  r.mn_w = q; q += 64;
  r.mn_b = q; q += 64;
  r.m0_w = q; q += 128 * 64;
  r.m0_b = q; q += 128;
  r.m2_w = q; q += 64 * 128;
  r.m2_b = q;
  return r;
}

// Affine LayerNorm (eps 1e-5) of 64 rows of 64: one warp per row.
__device__ void ln64(const float* in, float* out, const float* w, const float* b) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = warp; i < kSq; i += kThreads / 32) {
    float a = in[i * kLd + lane], c = in[i * kLd + lane + 32];
    float mu = warp_sum(a + c) * (1.0f / 64.0f);
    float da = a - mu, dc = c - mu;
    float var = warp_sum(da * da + dc * dc) * (1.0f / 64.0f);
    float rs = 1.0f / sqrtf(var + 1e-5f);
    out[i * kLd + lane] = da * rs * w[lane] + b[lane];
    out[i * kLd + lane + 32] = dc * rs * w[lane + 32] + b[lane + 32];
  }
}

enum { kStore = 0, kAdd = 1, kBiasSilu = 2, kBiasAdd = 3 };

// out[i][j] (op)= sum_k in[i][k] * W[j][k] for 64 rows, N columns, K inputs.
template <int K, int MODE>
__device__ void linear64(const float* in, int ld_in, const float* __restrict__ W, int N,
                         const float* __restrict__ bias, float* out, int ld_out) {
  for (int o = threadIdx.x; o < 16 * N; o += kThreads) {
    const int j = o % N, i0 = (o / N) * 4;
    const float* w = W + (size_t)j * K;
    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll 8
    for (int k = 0; k < K; ++k) {
      const float wk = __ldg(w + k);
      a0 = fmaf(in[(i0 + 0) * ld_in + k], wk, a0);
      a1 = fmaf(in[(i0 + 1) * ld_in + k], wk, a1);
      a2 = fmaf(in[(i0 + 2) * ld_in + k], wk, a2);
      a3 = fmaf(in[(i0 + 3) * ld_in + k], wk, a3);
    }
    float acc[4] = {a0, a1, a2, a3};
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      float* dst = out + (i0 + r) * ld_out + j;
      if (MODE == kStore) *dst = acc[r];
      if (MODE == kAdd) *dst += acc[r];
      if (MODE == kBiasSilu) *dst = silu_f(acc[r] + bias[j]);
      if (MODE == kBiasAdd) *dst += acc[r] + bias[j];
    }
  }
}

__global__ void __launch_bounds__(kThreads) embed_kernel(imba_model_desc md, imba_step_desc st, float* x_out) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ float sm[];
  float* X = sm;                 // [64][kLd] residual
  float* Hn = X + kSq * kLd;     // [64][kLd] LN output / attention output
  float* S = Hn + kSq * kLd;     // [64][kLd] scores of one head
  float* big = S + kSq * kLd;    // [64][kLdBig] qkv, or [64][129] MLP hidden
  __shared__ float pooled[kDim];

  const int r = blockIdx.x;
  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;

  // Gather the joint (piece, square) rows.
  for (int i = tid; i < kSq * kDim; i += kThreads) {
    const int s = i / kDim, c = i % kDim;
    int p = st.piece_ids[(size_t)r * kSq + s];
    if (p > 12) {
      report(st.status, IMBA_ERR_RANGE);
      p = 0;
    }
    X[s * kLd + c] = __ldg(md.piece_square + (size_t)(p * 64 + s) * kDim + c);
  }
  __syncthreads();

  for (int b = 0; b < 2; ++b) {
    const BlockParams bp = block_params(md.board_params, b);
    ln64(X, Hn, bp.an_w, bp.an_b);
    __syncthreads();
    linear64<kDim, kStore>(Hn, kLd, bp.qkv_w, 3 * kDim, nullptr, big, kLdBig);
    __syncthreads();
    for (int h = 0; h < kHeads; ++h) {
      // S = q_h k_h^T / sqrt(16)
      for (int o = tid; o < kSq * kSq; o += kThreads) {
        const int i = o / kSq, j = o % kSq;
        const float* qi = big + i * kLdBig + h * kHd;
        const float* kj = big + j * kLdBig + kDim + h * kHd;
        float s = 0.f;
#pragma unroll
        for (int e = 0; e < kHd; ++e) s = fmaf(qi[e], kj[e], s);
        S[i * kLd + j] = s * 0.25f;
      }
      __syncthreads();
      for (int i = warp; i < kSq; i += kThreads / 32) {
        float a = S[i * kLd + lane], c = S[i * kLd + lane + 32];
        float mx = warp_max(fmaxf(a, c));
        a = expf(a - mx);
        c = expf(c - mx);
        float inv = 1.0f / warp_sum(a + c);
        S[i * kLd + lane] = a * inv;
        S[i * kLd + lane + 32] = c * inv;
      }
      __syncthreads();
      for (int o = tid; o < kSq * kHd; o += kThreads) {
        const int i = o / kHd, e = o % kHd;
        float acc = 0.f;
        for (int j = 0; j < kSq; ++j) acc = fmaf(S[i * kLd + j], big[j * kLdBig + 2 * kDim + h * kHd + e], acc);
        Hn[i * kLd + h * kHd + e] = acc;
      }
      __syncthreads();
    }
    linear64<kDim, kAdd>(Hn, kLd, bp.ao_w, kDim, nullptr, X, kLd);
    __syncthreads();
    ln64(X, Hn, bp.mn_w, bp.mn_b);
    __syncthreads();
    linear64<kDim, kBiasSilu>(Hn, kLd, bp.m0_w, 2 * kDim, bp.m0_b, big, 2 * kDim + 1);
    __syncthreads();
    linear64<2 * kDim, kBiasAdd>(big, 2 * kDim + 1, bp.m2_w, kDim, bp.m2_b, X, kLd);
    __syncthreads();
  }
  const float* fin = md.board_params + 2 * IMBA_BOARD_BLOCK_FLOATS;
  ln64(X, Hn, fin, fin + 64);
  __syncthreads();
  if (tid < kDim) {
    float s = 0.f;
    for (int i = 0; i < kSq; ++i) s += Hn[i * kLd + tid];
    pooled[tid] = s * (1.0f / 64.0f);
  }
  __syncthreads();

  // Projection to d, side embeddings, position embedding.
  const int d = md.model_dim;
  const int32_t* ids = st.side_ids + (size_t)r * IMBA_NUM_SIDE_IDS;
  auto clampid = [&](int v, int n) {
    return v < 0 ? 0 : (v >= n ? n - 1 : v);
  };
  const int i_seq = clampid(ids[0], 2), i_turn = clampid(ids[1], 2), i_castle = clampid(ids[2], 16);
  const int i_ep = clampid(ids[3], 9), i_half = clampid(ids[4], md.halfmove_vocab);
  const int i_full = clampid(ids[5], md.fullmove_vocab), i_prev = clampid(ids[6], md.vocab);
  int pos = st.positions[r];
  if (pos < 0) {
    report(st.status, IMBA_ERR_RANGE);
    pos = 0;
  }
  if (pos > md.max_pos - 1) pos = md.max_pos - 1;
  const float scale = sqrtf((float)d);
  for (int j = tid; j < d; j += kThreads) {
    const float* w = md.board_out_w + (size_t)j * kDim;
    float acc = 0.f;
#pragma unroll 8
    for (int c = 0; c < kDim; ++c) acc = fmaf(pooled[c], __ldg(w + c), acc);
    float v = acc + md.board_out_b[j];
    v += md.emb_seq[(size_t)i_seq * d + j];
    v += md.emb_turn[(size_t)i_turn * d + j];
    v += md.emb_castle[(size_t)i_castle * d + j];
    v += md.emb_ep[(size_t)i_ep * d + j];
    v += md.emb_halfmove[(size_t)i_half * d + j];
    v += md.emb_fullmove[(size_t)i_full * d + j];
    v += md.emb_prev_move[(size_t)i_prev * d + j];
    x_out[(size_t)r * d + j] = v * scale + md.emb_pos[(size_t)pos * d + j];
  }
}

}  // namespace

size_t embed_smem_bytes() { return sizeof(float) * (3 * kSq * kLd + kSq * kLdBig); }

cudaError_t launch_embed(const imba_model_desc& md, const imba_step_desc& st, float* x, cudaStream_t s) {
  const size_t smem = embed_smem_bytes();
  cudaError_t e = cudaFuncSetAttribute(embed_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  return launch_pdl(embed_kernel, dim3(st.num_rows), dim3(kThreads), smem, s, md, st, x);
}

}  // namespace imba
