// Board encoder on the tensor cores (bf16 models): the two pre-LN square-
// attention blocks over the 64 squares of each position, the final LayerNorm
// and the mean over squares (src/imba_chess/model/hstu_model.py:118-179,
// :275-278).  Output: the pooled 64-vector of every board as the split bf16
// operand [hi | lo | hi] (192 values, hi + lo = the fp32 mean to ~2^-16); the
// 64 -> d projection (against [W_hi | W_hi | W_lo]) and the side / position
// embeddings follow in a GEMM epilogue.
//
// Persistent CTAs of 16 warps hold both blocks' weights in shared memory
// (bf16, padded rows) and process four boards per iteration: warp w owns
// squares 16*(w%4) .. +15 of board w/4.  Every product is an
// mma.sync.m16n8k16 (bf16 in, fp32 accumulate).  The residual stream stays in
// fp32 registers in the accumulator layout; LayerNorms reduce across the four
// lanes that share a row; accumulators convert directly into the next
// product's A fragments.  Per block and head: S = Q K^T (queries pre-scaled
// by log2(e) / 4, keys of the own board from shared memory), fp32 softmax in
// the log2 domain, O = P V, and the head's 16 output columns go straight
// through their slice of the output projection into the residual; the MLP
// (64 -> 128 -> 64, SiLU) runs in two 64-wide halves accumulating into the
// residual too.  Keeping only one head's state live holds a warp to 128
// registers, so 16 warps (four boards) share an SM.
#include "kernels.cuh"

namespace imba {
namespace {

constexpr int kThreads = 512;
constexpr int kBoardsPerIter = 4;
constexpr int LD64 = 72;    // padded bf16 row stride for 64-wide rows
constexpr int LD128 = 136;  // padded bf16 row stride for 128-wide rows

// bf16 element offsets of one block's weights in shared memory.
constexpr int kOffQKV = 0;                       // [192][72]
constexpr int kOffOut = kOffQKV + 192 * LD64;    // [64][72]
constexpr int kOffW1 = kOffOut + 64 * LD64;      // [128][72]
constexpr int kOffW2 = kOffW1 + 128 * LD64;      // [64][136]
constexpr int kBlockW = kOffW2 + 64 * LD128;     // elements per block
constexpr int kKV = kBoardsPerIter * 64 * LD64;  // one of sK / sV
// fp32 parameters per block: attn_norm w,b | mlp_norm w,b | b1 (128) | b2 (64)
constexpr int kBlockP = 64 * 4 + 128 + 64;
constexpr size_t kSmemBytes = (size_t)(2 * kBlockW + 2 * kKV) * 2 + (size_t)(2 * kBlockP + 128) * 4 +
                              (size_t)kBoardsPerIter * 4 * 64 * 4;

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const bf16* p) {
  const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(p));
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(a));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const bf16* p) {
  const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(p));
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(a));
}

// acc[nt] (+)= A(16 x 64, four k-chunks) . W[n0 + 8 nt .. , 0..63]^T for
// NT n-tiles (NT even), W row-major [n][k] with row stride ld.
template <int NT>
__device__ __forceinline__ void gemm_k64(float (&acc)[NT][4], const uint32_t (&a)[4][4], const bf16* W, int ld,
                                         int n0, int kofs, int lane) {
  const int r = lane & 7, m = lane >> 3;
#pragma unroll
  for (int kc = 0; kc < 4; ++kc) {
#pragma unroll
    for (int nt = 0; nt < NT; nt += 2) {
      uint32_t b[4];
      // matrices: (n, k), (n, k+8), (n+8, k), (n+8, k+8)
      ldsm_x4(b, W + (size_t)(n0 + 8 * nt + r + 8 * (m >> 1)) * ld + kofs + 16 * kc + 8 * (m & 1));
      mma16816(acc[nt], a[kc], b[0], b[1]);
      mma16816(acc[nt + 1], a[kc], b[2], b[3]);
    }
  }
}

// acc[nt] += A(16 x 16, one k-chunk) . W[n0 + 8 nt .., kofs .. kofs + 15]^T.
template <int NT>
__device__ __forceinline__ void gemm_k16(float (&acc)[NT][4], const uint32_t (&a)[4], const bf16* W, int ld, int n0,
                                         int kofs, int lane) {
  const int r = lane & 7, m = lane >> 3;
#pragma unroll
  for (int nt = 0; nt < NT; nt += 2) {
    uint32_t b[4];
    ldsm_x4(b, W + (size_t)(n0 + 8 * nt + r + 8 * (m >> 1)) * ld + kofs + 8 * (m & 1));
    mma16816(acc[nt], a, b[0], b[1]);
    mma16816(acc[nt + 1], a, b[2], b[3]);
  }
}

__device__ __forceinline__ float exp2_approx(float x) {  // hardware ex2
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Accumulator tiles (8 n-tiles = 64 columns) -> bf16 A fragments (4 k-chunks).
__device__ __forceinline__ void to_afrag(const float (&c)[8][4], uint32_t (&a)[4][4]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    a[j][0] = pack_bf16(c[2 * j][0], c[2 * j][1]);
    a[j][1] = pack_bf16(c[2 * j][2], c[2 * j][3]);
    a[j][2] = pack_bf16(c[2 * j + 1][0], c[2 * j + 1][1]);
    a[j][3] = pack_bf16(c[2 * j + 1][2], c[2 * j + 1][3]);
  }
}

// Affine LayerNorm (eps 1e-5) of the 16 x 64 residual tile (accumulator
// layout: this lane holds rows g and g+8, columns 8n + 2t, +1).
__device__ __forceinline__ void layer_norm(const float (&x)[8][4], const float* w, const float* b, int t,
                                           float (&y)[8][4]) {
  float s0 = 0.f, s1 = 0.f;
#pragma unroll
  for (int n = 0; n < 8; ++n) {
    s0 += x[n][0] + x[n][1];
    s1 += x[n][2] + x[n][3];
  }
  s0 += __shfl_xor_sync(0xffffffffu, s0, 1);
  s0 += __shfl_xor_sync(0xffffffffu, s0, 2);
  s1 += __shfl_xor_sync(0xffffffffu, s1, 1);
  s1 += __shfl_xor_sync(0xffffffffu, s1, 2);
  const float mu0 = s0 * (1.0f / 64.0f), mu1 = s1 * (1.0f / 64.0f);
  float q0 = 0.f, q1 = 0.f;
#pragma unroll
  for (int n = 0; n < 8; ++n) {
    q0 += (x[n][0] - mu0) * (x[n][0] - mu0) + (x[n][1] - mu0) * (x[n][1] - mu0);
    q1 += (x[n][2] - mu1) * (x[n][2] - mu1) + (x[n][3] - mu1) * (x[n][3] - mu1);
  }
  q0 += __shfl_xor_sync(0xffffffffu, q0, 1);
  q0 += __shfl_xor_sync(0xffffffffu, q0, 2);
  q1 += __shfl_xor_sync(0xffffffffu, q1, 1);
  q1 += __shfl_xor_sync(0xffffffffu, q1, 2);
  const float r0 = 1.0f / sqrtf(q0 * (1.0f / 64.0f) + 1e-5f), r1 = 1.0f / sqrtf(q1 * (1.0f / 64.0f) + 1e-5f);
#pragma unroll
  for (int n = 0; n < 8; ++n) {
    const int c = 8 * n + 2 * t;
    y[n][0] = (x[n][0] - mu0) * r0 * w[c] + b[c];
    y[n][1] = (x[n][1] - mu0) * r0 * w[c + 1] + b[c + 1];
    y[n][2] = (x[n][2] - mu1) * r1 * w[c] + b[c];
    y[n][3] = (x[n][3] - mu1) * r1 * w[c + 1] + b[c + 1];
  }
}

// Barrier of one board's four warps (named barrier board + 1, 128 threads):
// the boards of a CTA share only read-only weights, so each advances on its
// own instead of waiting for the slowest board at every phase.
__device__ __forceinline__ void board_barrier(int board) {
  asm volatile("bar.sync %0, 128;" ::"r"(board + 1) : "memory");
}

__device__ __forceinline__ void zero(float (&c)[8][4]) {
#pragma unroll
  for (int n = 0; n < 8; ++n) c[n][0] = c[n][1] = c[n][2] = c[n][3] = 0.f;
}

// Store an accumulator tile as bf16 rows [16][64] of a [64][LD64] board buffer.
__device__ __forceinline__ void store_rows(const float (&c)[8][4], bf16* dst, int row0, int g, int t) {
#pragma unroll
  for (int n = 0; n < 8; ++n) {
    const int col = 8 * n + 2 * t;
    *reinterpret_cast<uint32_t*>(dst + (size_t)(row0 + g) * LD64 + col) = pack_bf16(c[n][0], c[n][1]);
    *reinterpret_cast<uint32_t*>(dst + (size_t)(row0 + g + 8) * LD64 + col) = pack_bf16(c[n][2], c[n][3]);
  }
}

__global__ void __launch_bounds__(kThreads, 1)
    board_mma_kernel(const float* __restrict__ table, const float* __restrict__ params,
                     const uint8_t* __restrict__ piece_ids, int rows, bf16* __restrict__ pooled_out,
                     int32_t* status) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  bf16* sW = reinterpret_cast<bf16*>(smem_raw);       // 2 blocks of weights
  bf16* sK = sW + 2 * kBlockW;                          // [2 boards][64][72]
  bf16* sV = sK + kKV;
  float* sP = reinterpret_cast<float*>(sV + kKV);       // 2 blocks of fp32 params, then final LN w,b
  float* sPool = sP + 2 * kBlockP + 128;                // [kBoardsPerIter boards][4 warps][64]

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int board_slot = warp >> 2, wq = warp & 3;
  const int row0 = 16 * wq;  // first square of this warp

  // ---- weights -> shared memory (once per CTA) ----
  for (int b = 0; b < 2; ++b) {
    const float* p = params + (size_t)b * IMBA_BOARD_BLOCK_FLOATS;
    const float *an_w = p, *an_b = p + 64, *qkv = p + 128, *ao = qkv + 192 * 64, *mn_w = ao + 64 * 64,
                *mn_b = mn_w + 64, *w1 = mn_b + 64, *b1 = w1 + 128 * 64, *w2 = b1 + 128, *b2 = w2 + 64 * 128;
    bf16* W = sW + (size_t)b * kBlockW;
    for (int i = tid; i < 192 * 64; i += kThreads) W[kOffQKV + (i >> 6) * LD64 + (i & 63)] = __float2bfloat16_rn(qkv[i]);
    for (int i = tid; i < 64 * 64; i += kThreads) W[kOffOut + (i >> 6) * LD64 + (i & 63)] = __float2bfloat16_rn(ao[i]);
    for (int i = tid; i < 128 * 64; i += kThreads) W[kOffW1 + (i >> 6) * LD64 + (i & 63)] = __float2bfloat16_rn(w1[i]);
    for (int i = tid; i < 64 * 128; i += kThreads) W[kOffW2 + (i >> 7) * LD128 + (i & 127)] = __float2bfloat16_rn(w2[i]);
    float* P = sP + (size_t)b * kBlockP;
    for (int i = tid; i < 64; i += kThreads) {
      P[i] = an_w[i];
      P[64 + i] = an_b[i];
      P[128 + i] = mn_w[i];
      P[192 + i] = mn_b[i];
      P[256 + 128 + i] = b2[i];
    }
    for (int i = tid; i < 128; i += kThreads) P[256 + i] = b1[i];
  }
  {
    const float* fin = params + 2 * IMBA_BOARD_BLOCK_FLOATS;
    for (int i = tid; i < 128; i += kThreads) sP[2 * kBlockP + i] = fin[i];
  }
  // The weights above are step-invariant; piece ids and the pooled output
  // are ordered after the previous kernel of the stream.
  pdl_wait();
  pdl_trigger();
  __syncthreads();

  const int pairs = (rows + kBoardsPerIter - 1) / kBoardsPerIter;
  for (int pair = blockIdx.x; pair < pairs; pair += gridDim.x) {
    const int r = pair * kBoardsPerIter + board_slot;
    const bool live = r < rows;
    // ---- gather the joint (piece, square) embeddings ----
    float x[8][4];
    {
      int sq0 = row0 + g, sq1 = row0 + g + 8;
      int p0 = live ? piece_ids[(size_t)r * 64 + sq0] : 0, p1 = live ? piece_ids[(size_t)r * 64 + sq1] : 0;
      if (p0 > 12 || p1 > 12) {
        report(status, IMBA_ERR_RANGE);
        p0 = p0 > 12 ? 0 : p0;
        p1 = p1 > 12 ? 0 : p1;
      }
      const float* e0 = table + (size_t)(p0 * 64 + sq0) * 64;
      const float* e1 = table + (size_t)(p1 * 64 + sq1) * 64;
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        const float2 v0 = __ldg(reinterpret_cast<const float2*>(e0 + 8 * n + 2 * t));
        const float2 v1 = __ldg(reinterpret_cast<const float2*>(e1 + 8 * n + 2 * t));
        x[n][0] = v0.x;
        x[n][1] = v0.y;
        x[n][2] = v1.x;
        x[n][3] = v1.y;
      }
    }
    bf16* myK = sK + (size_t)board_slot * 64 * LD64;
    bf16* myV = sV + (size_t)board_slot * 64 * LD64;
#pragma unroll 1
    for (int blk = 0; blk < 2; ++blk) {
      const bf16* W = sW + (size_t)blk * kBlockW;
      const float* P = sP + (size_t)blk * kBlockP;
      uint32_t ha[4][4];
      {
        float y[8][4];
        layer_norm(x, P, P + 64, t, y);
        to_afrag(y, ha);
      }
      uint32_t qa[4][4];
      {
        // Q, pre-scaled by log2(e) / sqrt(16) so that the scores come out in
        // the log2 domain; K and V go to the board's shared buffers.
        constexpr float kQScale = 0.25f * 1.4426950408889634f;
        // K and V first, so that the Q fragments are live only from here on.
        float acc[8][4];
        zero(acc);
        gemm_k64<8>(acc, ha, W + kOffQKV, LD64, 64, 0, lane);
        store_rows(acc, myK, row0, g, t);
        zero(acc);
        gemm_k64<8>(acc, ha, W + kOffQKV, LD64, 128, 0, lane);
        store_rows(acc, myV, row0, g, t);
        zero(acc);
        gemm_k64<8>(acc, ha, W + kOffQKV, LD64, 0, 0, lane);
#pragma unroll
        for (int n = 0; n < 8; ++n) {
          acc[n][0] *= kQScale;
          acc[n][1] *= kQScale;
          acc[n][2] *= kQScale;
          acc[n][3] *= kQScale;
        }
        to_afrag(acc, qa);
      }
      board_barrier(board_slot);
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        float s[8][4];
        zero(s);
        const int rr = lane & 7, m = lane >> 3;
#pragma unroll
        for (int nt = 0; nt < 8; nt += 2) {
          uint32_t b[4];
          // keys 8nt.. (and +8), dims 16h .. 16h+15
          ldsm_x4(b, myK + (size_t)(8 * nt + rr + 8 * (m >> 1)) * LD64 + 16 * h + 8 * (m & 1));
          mma16816(s[nt], qa[h], b[0], b[1]);
          mma16816(s[nt + 1], qa[h], b[2], b[3]);
        }
        float m0 = -INFINITY, m1 = -INFINITY;
#pragma unroll
        for (int n = 0; n < 8; ++n) {
          m0 = fmaxf(m0, fmaxf(s[n][0], s[n][1]));
          m1 = fmaxf(m1, fmaxf(s[n][2], s[n][3]));
        }
        m0 = fmaxf(m0, __shfl_xor_sync(0xffffffffu, m0, 1));
        m0 = fmaxf(m0, __shfl_xor_sync(0xffffffffu, m0, 2));
        m1 = fmaxf(m1, __shfl_xor_sync(0xffffffffu, m1, 1));
        m1 = fmaxf(m1, __shfl_xor_sync(0xffffffffu, m1, 2));
        float l0 = 0.f, l1 = 0.f;
#pragma unroll
        for (int n = 0; n < 8; ++n) {
          s[n][0] = exp2_approx(s[n][0] - m0);
          s[n][1] = exp2_approx(s[n][1] - m0);
          s[n][2] = exp2_approx(s[n][2] - m1);
          s[n][3] = exp2_approx(s[n][3] - m1);
          l0 += s[n][0] + s[n][1];
          l1 += s[n][2] + s[n][3];
        }
        l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
        l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
        l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
        l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
        uint32_t pa[4][4];
        to_afrag(s, pa);
        float oh[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
        for (int kc = 0; kc < 4; ++kc) {
          uint32_t b[4];
          // keys 16kc + (0..7 | 8..15), dims 16h + (0..7 | 8..15), transposed
          ldsm_x4_t(b, myV + (size_t)(16 * kc + rr + 8 * (m & 1)) * LD64 + 16 * h + 8 * (m >> 1));
          mma16816(oh[0], pa[kc], b[0], b[1]);
          mma16816(oh[1], pa[kc], b[2], b[3]);
        }
        const float i0 = __frcp_rn(l0), i1 = __frcp_rn(l1);
        // The head's output (16 x 16) as one A k-chunk, through its slice of
        // the output projection into the residual.
        uint32_t oa[4];
        oa[0] = pack_bf16(oh[0][0] * i0, oh[0][1] * i0);
        oa[1] = pack_bf16(oh[0][2] * i1, oh[0][3] * i1);
        oa[2] = pack_bf16(oh[1][0] * i0, oh[1][1] * i0);
        oa[3] = pack_bf16(oh[1][2] * i1, oh[1][3] * i1);
        gemm_k16<8>(x, oa, W + kOffOut, LD64, 0, 16 * h, lane);  // x += o_h . Wout[:, 16h .. 16h+15]^T
      }
      board_barrier(board_slot);  // the board's K / V are reused by the next block
      {
        float y[8][4];
        layer_norm(x, P + 128, P + 192, t, y);
        to_afrag(y, ha);
      }
      const float* b1 = P + 256;
      const float* b2 = P + 256 + 128;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        float acc[8][4];
        zero(acc);
        gemm_k64<8>(acc, ha, W + kOffW1, LD64, 64 * half, 0, lane);
#pragma unroll
        for (int n = 0; n < 8; ++n) {
          const int c = 64 * half + 8 * n + 2 * t;
          acc[n][0] = silu_tanh(acc[n][0] + b1[c]);
          acc[n][1] = silu_tanh(acc[n][1] + b1[c + 1]);
          acc[n][2] = silu_tanh(acc[n][2] + b1[c]);
          acc[n][3] = silu_tanh(acc[n][3] + b1[c + 1]);
        }
        uint32_t ma[4][4];
        to_afrag(acc, ma);
        gemm_k64<8>(x, ma, W + kOffW2, LD128, 0, 64 * half, lane);  // x += silu(.) . W2[:, half]^T
      }
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        const int c = 8 * n + 2 * t;
        x[n][0] += b2[c];
        x[n][1] += b2[c + 1];
        x[n][2] += b2[c];
        x[n][3] += b2[c + 1];
      }
    }
    // ---- final LayerNorm and mean over the 64 squares ----
    {
      float y[8][4];
      const float* fin = sP + 2 * kBlockP;
      layer_norm(x, fin, fin + 64, t, y);
      float cs[8][2];
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        cs[n][0] = y[n][0] + y[n][2];
        cs[n][1] = y[n][1] + y[n][3];
#pragma unroll
        for (int o2 = 4; o2 < 32; o2 <<= 1) {
          cs[n][0] += __shfl_xor_sync(0xffffffffu, cs[n][0], o2);
          cs[n][1] += __shfl_xor_sync(0xffffffffu, cs[n][1], o2);
        }
      }
      if (g == 0) {
        float* dst = sPool + (size_t)(board_slot * 4 + wq) * 64;
#pragma unroll
        for (int n = 0; n < 8; ++n) {
          dst[8 * n + 2 * t] = cs[n][0];
          dst[8 * n + 2 * t + 1] = cs[n][1];
        }
      }
    }
    board_barrier(board_slot);
    if (live && wq == 0) {
      const float* src = sPool + (size_t)board_slot * 4 * 64;
      for (int c = lane; c < 64; c += 32) {
        const float s = src[c] + src[64 + c] + src[128 + c] + src[192 + c];
        const float v = s * (1.0f / 64.0f);
        const bf16 hi = __float2bfloat16_rn(v), lo = __float2bfloat16_rn(v - __bfloat162float(hi));
        bf16* o = pooled_out + (size_t)r * 3 * 64;
        o[c] = hi;
        o[64 + c] = lo;
        o[128 + c] = hi;
      }
    }
    board_barrier(board_slot);
  }
}

// [d, 64] fp32 projection -> [d, 192] bf16 [W_hi | W_hi | W_lo].
__global__ void split_board_proj_kernel(const float* __restrict__ w, int d, bf16* __restrict__ out) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= d * 64) return;
  const int row = i >> 6, c = i & 63;
  const float v = w[i];
  const bf16 hi = __float2bfloat16_rn(v), lo = __float2bfloat16_rn(v - __bfloat162float(hi));
  bf16* o = out + (size_t)row * 192;
  o[c] = hi;
  o[64 + c] = hi;
  o[128 + c] = lo;
}

}  // namespace

cudaError_t build_board_proj_split(const imba_model_desc& md, bf16* out, cudaStream_t s) {
  const int n = md.model_dim * 64;
  split_board_proj_kernel<<<(n + 255) / 256, 256, 0, s>>>(md.board_out_w, md.model_dim, out);
  return cudaGetLastError();
}

cudaError_t launch_board_mma(const imba_model_desc& md, const imba_step_desc& st, bf16* pooled, cudaStream_t s) {
  if (st.num_rows <= 0) return cudaSuccess;
  cudaError_t e = cudaFuncSetAttribute(board_mma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes);
  if (e != cudaSuccess) return e;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int pairs = (st.num_rows + kBoardsPerIter - 1) / kBoardsPerIter;
  const int grid = pairs < sms ? pairs : sms;
  return launch_pdl(board_mma_kernel, dim3(grid), dim3(kThreads), kSmemBytes, s, md.piece_square, md.board_params,
                    st.piece_ids, st.num_rows, pooled, st.status);
}

}  // namespace imba
