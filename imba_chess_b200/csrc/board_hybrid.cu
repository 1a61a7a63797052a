// Board encoder for bf16 models: the two pre-LN square-attention
// blocks over the 64 squares of each position, the final LayerNorm and the
// mean over squares (src/imba_chess/model/hstu_model.py:118-179, :275-278).
// Output: the pooled 64-vector of every board as the split bf16 operand
// [hi | lo | hi] (192 values, hi + lo = the fp32 mean to ~2^-16); the
// 64 -> d projection and the side / position embeddings follow in a GEMM
// epilogue.
//
// The dense projections go to the 5th-generation tensor cores, the per-board
// attention stays in registers:
//   * a tile is two boards = 128 square rows, the M of one tcgen05.mma; a
//     persistent CTA of 16 warps runs two tiles (warps 0-7, 8-15) so one
//     tile's LayerNorm / softmax work overlaps the other's MMAs;
//   * [Q|K|V] = LN1(x) Wqkv^T (N192), hidden = LN2(x) W1^T (N128) and
//     hidden' W2^T (N64, K128) are tcgen05.mma from shared memory (bf16,
//     K-major, 128-byte swizzle) into TMEM columns [256 t, 256 t + 256) of
//     tile t, issued by one thread of the tile;
//   * warp w of tile t owns rows 32 (w % 4) + 16 ((w / 4) % 2) .. +15, i.e.
//     16 squares of board (w % 4) / 2, and reads them from TMEM with the
//     16x256b shape, which lands in the mma.sync accumulator layout (this
//     lane: rows g and g + 8, columns 8 n + 2 t, +1);
//   * per head, S = Q K^T, the fp32 softmax in the log2 domain and O = P V are
//     mma.sync.m16n8k16 on the board's K / V in shared memory, and the head's
//     16 outputs go straight through their slice of the output projection
//     (mma.sync) into the fp32 residual, which stays in registers.
// Operands staged by the threads (LN outputs, SiLU hidden, K, V) are written
// with stmatrix into the swizzled layout; each MMA follows a 256-thread
// barrier of the tile (after fence.proxy.async and tcgen05.fence), and the
// tile waits on an mbarrier the MMA's commit arrives on.  Waits are bounded:
// after a timeout no further MMA is issued, every later wait returns at once,
// every thread still takes the same barriers and the status word holds the
// error.
#include "kernels.cuh"
#include "tc_ptx.cuh"

namespace imba {
namespace {

constexpr int kThreads = 512;
constexpr uint32_t kTmemCols = 512;

// Byte offsets inside the 1024-aligned shared window.
constexpr uint32_t kWBlock = 65536;     // one block's weights:
constexpr uint32_t kOffWqkv = 0;        //   [192 x 64] Wq | Wk | Wv rows
constexpr uint32_t kOffW1 = 24576;      //   [128 x 64]
constexpr uint32_t kOffW2 = 40960;      //   [64 x 128], two 64-wide atom columns 8 KB apart
constexpr uint32_t kOffWo = 57344;      //   [64 x 64] output projection (mma.sync B operand)
constexpr uint32_t kOffTile = 2 * kWBlock;  // 32 KB per tile: LN output [128 x 64] at +0, or
constexpr uint32_t kTileBytes = 32768;      // K / V of board b at +16 KB b, +8 KB, or hidden [128 x 128]
constexpr uint32_t kOffPar = kOffTile + 2 * kTileBytes;
constexpr int kParBlock = 448;  // ln1 w, b | (unused 128) | b1' (128, folded and halved) | b2 (64)
constexpr int kParFinal = 2 * kParBlock;
constexpr uint32_t kOffPool = kOffPar + (2 * kParBlock + 128) * 4;  // [4 boards][4 warps][64] floats
constexpr uint32_t kOffBar = kOffPool + 4 * 4 * 64 * 4;             // one mbarrier per tile
constexpr uint32_t kOffMisc = kOffBar + 2 * 8;                      // TMEM base, abort flag
constexpr size_t kSmemBytes = kOffMisc + 16 + 1024;                 // + alignment slack

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Byte offset of 16-byte chunk j (0..7) of row n in a K-major tile with the
// 128-byte swizzle (8-row / 1024-byte atoms).
__device__ __forceinline__ uint32_t sw(int n, int j) {
  return (uint32_t)((n >> 3) * 1024 + (n & 7) * 128 + (((j ^ n) & 7) << 4));
}

__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t a) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(a));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], uint32_t a) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(a));
}
__device__ __forceinline__ void stsm_x4(uint32_t a, const uint32_t (&r)[4]) {
  asm volatile("stmatrix.sync.aligned.m8n8.x4.shared.b16 [%0], {%1,%2,%3,%4};\n" ::"r"(a), "r"(r[0]), "r"(r[1]),
               "r"(r[2]), "r"(r[3])
               : "memory");
}

// Hardware 2^x on a bf16 pair (the probabilities are bf16 operands of P V).
__device__ __forceinline__ uint32_t exp2_bf16x2(uint32_t x) {
  uint32_t y;
  asm("ex2.approx.ftz.bf16x2 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}

// SiLU of a bf16 pair given h = v / 2: h (1 + tanh(h)) with the hardware
// tanh (the hidden activations are bf16 operands of the second MLP product;
// W1 and b1 are staged halved, which is exact).
__device__ __forceinline__ uint32_t silu_half_bf16x2(float h0, float h1) {
  const uint32_t h = pack_bf16(h0, h1);
  uint32_t t, y;
  asm("tanh.approx.bf16x2 %0, %1;" : "=r"(t) : "r"(h));
  asm("fma.rn.bf16x2 %0, %1, %2, %1;" : "=r"(y) : "r"(h), "r"(t));
  return y;
}
constexpr uint32_t kOnesBf16x2 = 0x3F803F80u;  // (1.0, 1.0)

__device__ __forceinline__ float rcp_approx(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 16 TMEM lanes x 64 fp32 columns in the mma.sync accumulator layout:
// c[n] = (lane g, column 8 n + 2 t, +1), (lane g + 8, same columns).
__device__ __forceinline__ void tmem_ld_frag(uint32_t taddr, float (&c)[8][4]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.16x256b.x8.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int n = 0; n < 8; ++n) {
    c[n][0] = __uint_as_float(r[4 * n]);
    c[n][1] = __uint_as_float(r[4 * n + 1]);
    c[n][2] = __uint_as_float(r[4 * n + 2]);
    c[n][3] = __uint_as_float(r[4 * n + 3]);
  }
}

// 16 TMEM lanes x 16 fp32 columns, times `scale`, as one bf16 A fragment
// (k-chunk) of the mma.sync layout.
__device__ __forceinline__ void tmem_ld_afrag16(uint32_t taddr, float scale, uint32_t (&a)[4]) {
  uint32_t r[8];
  asm volatile(
      "tcgen05.ld.sync.aligned.16x256b.x2.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
      : "r"(taddr)
      : "memory");
  a[0] = pack_bf16(scale * __uint_as_float(r[0]), scale * __uint_as_float(r[1]));
  a[1] = pack_bf16(scale * __uint_as_float(r[2]), scale * __uint_as_float(r[3]));
  a[2] = pack_bf16(scale * __uint_as_float(r[4]), scale * __uint_as_float(r[5]));
  a[3] = pack_bf16(scale * __uint_as_float(r[6]), scale * __uint_as_float(r[7]));
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

// Store this warp's 16 x 64 bf16 fragments (A-fragment order) as rows
// row0 .. row0 + 15 of a swizzled K-major tile at byte address base.
__device__ __forceinline__ void store_tile(uint32_t base, const uint32_t (&a)[4][4], int row0, int lane) {
  const int mi = lane >> 3, ri = lane & 7;
  const int row = row0 + ri + 8 * (mi & 1);
#pragma unroll
  for (int j = 0; j < 4; ++j) stsm_x4(base + sw(row, 2 * j + (mi >> 1)), a[j]);
}

// Affine LayerNorm (eps 1e-5) of the 16 x 64 residual tile in the
// accumulator layout; the four lanes of a row combine their partial sums.
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
  const float r0 = rsqrtf(q0 * (1.0f / 64.0f) + 1e-5f), r1 = rsqrtf(q1 * (1.0f / 64.0f) + 1e-5f);
#pragma unroll
  for (int n = 0; n < 8; ++n) {
    const int c = 8 * n + 2 * t;
    y[n][0] = (x[n][0] - mu0) * r0 * w[c] + b[c];
    y[n][1] = (x[n][1] - mu0) * r0 * w[c + 1] + b[c + 1];
    y[n][2] = (x[n][2] - mu1) * r1 * w[c] + b[c];
    y[n][3] = (x[n][3] - mu1) * r1 * w[c + 1] + b[c + 1];
  }
}

// LayerNorm without the affine part, (x - mean) / std: used where the
// affine weights are folded into what follows (the MLP's first product, the
// pooled mean).
__device__ __forceinline__ void layer_norm_plain(const float (&x)[8][4], float (&y)[8][4]) {
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
  const float r0 = rsqrtf(q0 * (1.0f / 64.0f) + 1e-5f), r1 = rsqrtf(q1 * (1.0f / 64.0f) + 1e-5f);
  const float z0 = -mu0 * r0, z1 = -mu1 * r1;
#pragma unroll
  for (int n = 0; n < 8; ++n) {
    y[n][0] = fmaf(x[n][0], r0, z0);
    y[n][1] = fmaf(x[n][1], r0, z0);
    y[n][2] = fmaf(x[n][2], r1, z1);
    y[n][3] = fmaf(x[n][3], r1, z1);
  }
}

__device__ __forceinline__ void zero(float (&c)[8][4]) {
#pragma unroll
  for (int n = 0; n < 8; ++n) c[n][0] = c[n][1] = c[n][2] = c[n][3] = 0.f;
}

// Barrier of one board's four warps (ids 1-4, 128 threads) and of one tile's
// eight warps (ids 5-6, 256 threads).
__device__ __forceinline__ void board_barrier(int board) {
  asm volatile("bar.sync %0, 128;" ::"r"(board + 1) : "memory");
}
__device__ __forceinline__ void tile_barrier(int tile) {
  asm volatile("bar.sync %0, 256;" ::"r"(tile + 5) : "memory");
}

// fp32 [rows, kdim] row-major, times `scale` and (when given) the per-input
// factors colw[k] -> bf16 K-major swizzled tile (64-wide atom columns
// rows * 128 bytes apart).
__device__ void stage_weights(uint32_t dst, const float* __restrict__ w, int rows, int kdim, int tid,
                              float scale = 1.f, const float* __restrict__ colw = nullptr) {
  const int cpr = kdim >> 3;
  for (int i = tid; i < rows * cpr; i += kThreads) {
    const int n = i / cpr, j = i - n * cpr;
    const float* s = w + (size_t)n * kdim + 8 * j;
    float f[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) f[k] = scale * __ldg(s + k) * (colw ? __ldg(colw + 8 * j + k) : 1.f);
    uint32_t p[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) p[k] = pack_bf16(f[2 * k], f[2 * k + 1]);
    asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(dst + (uint32_t)(j >> 3) * (uint32_t)(rows * 128) +
                                                                 sw(n, j & 7)),
                 "r"(p[0]), "r"(p[1]), "r"(p[2]), "r"(p[3])
                 : "memory");
  }
}

__global__ void __launch_bounds__(kThreads, 1)
    board_hybrid_kernel(const float* __restrict__ table, const float* __restrict__ params,
                        const uint8_t* __restrict__ piece_ids, int rows, bf16* __restrict__ pooled_out,
                        int32_t* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sb = tc::smem_u32(sm);
  float* sPar = reinterpret_cast<float*>(sm + kOffPar);
  float* sPool = reinterpret_cast<float*>(sm + kOffPool);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + kOffBar);
  uint32_t* sTmem = reinterpret_cast<uint32_t*>(sm + kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + kOffMisc + 4);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int tile = warp >> 3, wt = warp & 7, quad = warp & 3;
  const int r0 = 32 * quad + 16 * (wt >> 2);  // this warp's first row of the tile
  const int bt = quad >> 1;                    // board of the tile
  const int sq0 = r0 & 63;                     // first square of the board
  const int wib = (quad & 1) + 2 * (wt >> 2);  // warp index within the board (0..3)
  const int bslot = 2 * tile + bt;             // board slot of the CTA (0..3)

  // ---- weights -> shared memory (step-invariant, before the PDL wait) ----
  for (int b = 0; b < 2; ++b) {
    const float* p = params + (size_t)b * IMBA_BOARD_BLOCK_FLOATS;
    const float *an_w = p, *an_b = p + 64, *qkv = p + 128, *ao = qkv + 192 * 64, *mn_w = ao + 64 * 64,
                *mn_b = mn_w + 64, *w1 = mn_b + 64, *b1 = w1 + 128 * 64, *w2 = b1 + 128, *b2 = w2 + 64 * 128;
    const uint32_t wb = sb + (uint32_t)b * kWBlock;
    stage_weights(wb + kOffWqkv, qkv, 192, 64, tid);
    // The MLP LayerNorm's affine part folds into the first product:
    // W1 diag(w) and b1 + W1 b, both halved (the SiLU takes v / 2).
    stage_weights(wb + kOffW1, w1, 128, 64, tid, 0.5f, mn_w);
    stage_weights(wb + kOffW2, w2, 64, 128, tid);
    stage_weights(wb + kOffWo, ao, 64, 64, tid);
    float* P = sPar + b * kParBlock;
    for (int i = tid; i < 64; i += kThreads) {
      P[i] = an_w[i];
      P[64 + i] = an_b[i];
      P[384 + i] = b2[i];
    }
    for (int i = tid; i < 128; i += kThreads) {
      float acc = b1[i];
      for (int k = 0; k < 64; ++k) acc = fmaf(w1[(size_t)i * 64 + k], mn_b[k], acc);
      P[256 + i] = 0.5f * acc;
    }
  }
  for (int i = tid; i < 128; i += kThreads) sPar[kParFinal + i] = params[2 * IMBA_BOARD_BLOCK_FLOATS + i];
  if (tid == 0) {
    tc::mbar_init(&bars[0], 1);
    tc::mbar_init(&bars[1], 1);
    *abort_flag = 0;
    tc::fence_mbar_init();
  }
  if (warp == 0) {
    tc::tmem_alloc(sTmem, kTmemCols);
    tc::tmem_relinquish();
  }
  tc::fence_proxy_async_smem();  // the staged weights are read by the tensor cores
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem_tile = *sTmem + 256u * (uint32_t)tile;
  const uint32_t tl = tmem_tile + ((uint32_t)r0 << 16);  // this warp's 16 lanes
  const uint32_t tb = sb + kOffTile + (uint32_t)tile * kTileBytes;
  const uint32_t kb = tb + 16384u * (uint32_t)bt, vb = kb + 8192u;  // this board's K and V
  const bool issuer = wt == 0 && lane == 0;
  // Piece ids and the pooled output are ordered after the previous kernel.
  pdl_wait();
  pdl_trigger();

  uint32_t phase = 0;
  bool dead = false;
  // One tile-wide hand-off: operands written (generic proxy) and TMEM reads
  // done, then the issuing thread runs `issue` and commits to the tile's
  // mbarrier, which every thread of the tile waits on.
  auto handoff = [&](auto issue) {
    tc::fence_proxy_async_smem();
    tc::fence_before_sync();
    tile_barrier(tile);
    if (issuer && !dead) {
      tc::fence_after_sync();
      issue();
      tc::umma_commit(&bars[tile]);
    }
    if (!dead && !tc::mbar_wait_or_abort(&bars[tile], phase, status, abort_flag)) dead = true;
    phase ^= 1;
    tc::fence_after_sync();
  };
  constexpr uint32_t idN192 = tc::idesc_bf16_f32(128, 192), idN128 = tc::idesc_bf16_f32(128, 128),
                     idN64 = tc::idesc_bf16_f32(128, 64);
  const uint64_t dT = tc::smem_desc_k128(sm + kOffTile + tile * kTileBytes);

  const int iters = (rows + 3) >> 2;
  const int s0 = sq0 + g, s1 = sq0 + g + 8;  // this lane's squares
  // Piece ids are loaded one iteration ahead (two registers), so that only
  // the embedding gather waits on memory at the start of an iteration.
  int pn0 = 0, pn1 = 0;
  if (4 * (int)blockIdx.x + bslot < rows) {
    pn0 = piece_ids[(size_t)(4 * blockIdx.x + bslot) * 64 + s0];
    pn1 = piece_ids[(size_t)(4 * blockIdx.x + bslot) * 64 + s1];
  }
  for (int it = blockIdx.x; it < iters; it += gridDim.x) {
    const int r = 4 * it + bslot;
    const bool live = r < rows;
    int p0 = pn0, p1 = pn1;
    if (r + 4 * (int)gridDim.x < rows) {
      pn0 = piece_ids[(size_t)(r + 4 * gridDim.x) * 64 + s0];
      pn1 = piece_ids[(size_t)(r + 4 * gridDim.x) * 64 + s1];
    }
    // ---- gather the joint (piece, square) embeddings ----
    float x[8][4];
    {
      if (p0 > 12 || p1 > 12) {
        report(status, IMBA_ERR_RANGE);
        p0 = p0 > 12 ? 0 : p0;
        p1 = p1 > 12 ? 0 : p1;
      }
      const float* e0 = table + (size_t)(p0 * 64 + s0) * 64;
      const float* e1 = table + (size_t)(p1 * 64 + s1) * 64;
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
#pragma unroll 1
    for (int blk = 0; blk < 2; ++blk) {
      const uint32_t wb = sb + (uint32_t)blk * kWBlock;
      const uint8_t* wbp = sm + blk * kWBlock;
      const float* P = sPar + blk * kParBlock;
      {  // LN1 -> tile rows (A operand of the QKV projection)
        float y[8][4];
        uint32_t a[4][4];
        layer_norm(x, P, P + 64, t, y);
        to_afrag(y, a);
        store_tile(tb, a, r0, lane);
      }
      handoff([&] {
        const uint64_t dW = tc::smem_desc_k128(wbp + kOffWqkv);
#pragma unroll
        for (int k = 0; k < 4; ++k) tc::umma_f16(tmem_tile, dT + 2 * k, dW + 2 * k, idN192, k);
      });
      {  // K and V rows of the board -> shared memory
        float acc[8][4];
        uint32_t a[4][4];
        tmem_ld_frag(tl + 64, acc);
        to_afrag(acc, a);
        store_tile(kb, a, sq0, lane);
        tmem_ld_frag(tl + 128, acc);
        to_afrag(acc, a);
        store_tile(vb, a, sq0, lane);
      }
      board_barrier(bslot);  // the board's K / V are complete
      const int rr = lane & 7, m = lane >> 3;
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        // The head's Q columns stay in TMEM until the MLP product: read as
        // the A fragment, pre-scaled by log2(e) / sqrt(16) so that the scores
        // come out in the log2 domain.
        uint32_t qh[4];
        tmem_ld_afrag16(tl + 16 * h, 0.25f * 1.4426950408889634f, qh);
        float s[8][4];
        zero(s);
#pragma unroll
        for (int nt = 0; nt < 8; nt += 2) {
          uint32_t b[4];
          // keys 8 nt .. (and +8), dims 16 h .. 16 h + 15
          ldsm_x4(b, kb + sw(8 * nt + rr + 8 * (m >> 1), 2 * h + (m & 1)));
          mma16816(s[nt], qh, b[0], b[1]);
          mma16816(s[nt + 1], qh, b[2], b[3]);
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
        // P = 2^(s - m) as bf16 A fragments; the row sums come from the same
        // bf16 values through a third product against a column of ones.
        uint32_t pa[4][4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          pa[j][0] = exp2_bf16x2(pack_bf16(s[2 * j][0] - m0, s[2 * j][1] - m0));
          pa[j][1] = exp2_bf16x2(pack_bf16(s[2 * j][2] - m1, s[2 * j][3] - m1));
          pa[j][2] = exp2_bf16x2(pack_bf16(s[2 * j + 1][0] - m0, s[2 * j + 1][1] - m0));
          pa[j][3] = exp2_bf16x2(pack_bf16(s[2 * j + 1][2] - m1, s[2 * j + 1][3] - m1));
        }
        float oh[3][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
        for (int kc = 0; kc < 4; ++kc) {
          uint32_t b[4];
          // keys 16 kc + (0..7 | 8..15), dims 16 h + (0..7 | 8..15), transposed
          ldsm_x4_t(b, vb + sw(16 * kc + rr + 8 * (m & 1), 2 * h + (m >> 1)));
          mma16816(oh[0], pa[kc], b[0], b[1]);
          mma16816(oh[1], pa[kc], b[2], b[3]);
          mma16816(oh[2], pa[kc], kOnesBf16x2, kOnesBf16x2);
        }
        const float i0 = rcp_approx(oh[2][0]), i1 = rcp_approx(oh[2][2]);
        // The head's output (16 x 16) as one A k-chunk, through its slice of
        // the output projection into the residual.
        uint32_t oa[4];
        oa[0] = pack_bf16(oh[0][0] * i0, oh[0][1] * i0);
        oa[1] = pack_bf16(oh[0][2] * i1, oh[0][3] * i1);
        oa[2] = pack_bf16(oh[1][0] * i0, oh[1][1] * i0);
        oa[3] = pack_bf16(oh[1][2] * i1, oh[1][3] * i1);
#pragma unroll
        for (int nt = 0; nt < 8; nt += 2) {
          uint32_t b[4];
          ldsm_x4(b, wb + kOffWo + sw(8 * nt + rr + 8 * (m >> 1), 2 * h + (m & 1)));
          mma16816(x[nt], oa, b[0], b[1]);  // x += o_h . Wout[:, 16 h .. 16 h + 15]^T
          mma16816(x[nt + 1], oa, b[2], b[3]);
        }
      }
      // LN2 output overwrites the first board's K / V: the whole tile is done
      // with its attention first.
      tile_barrier(tile);
      {
        float y[8][4];
        uint32_t a[4][4];
        layer_norm_plain(x, y);
        to_afrag(y, a);
        store_tile(tb, a, r0, lane);
      }
      handoff([&] {
        const uint64_t dW = tc::smem_desc_k128(wbp + kOffW1);
#pragma unroll
        for (int k = 0; k < 4; ++k) tc::umma_f16(tmem_tile, dT + 2 * k, dW + 2 * k, idN128, k);
      });
      {  // hidden = SiLU(v), v / 2 = . + b1 / 2 (halved W1, b1) -> tile (two 64-wide atom columns)
        const float* b1 = P + 256;
#pragma unroll 1
        for (int half = 0; half < 2; ++half) {
          float acc[8][4];
          uint32_t a[4][4];
          tmem_ld_frag(tl + 64 * half, acc);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float2 c0 = *reinterpret_cast<const float2*>(b1 + 64 * half + 16 * j + 2 * t);
            const float2 c1 = *reinterpret_cast<const float2*>(b1 + 64 * half + 16 * j + 8 + 2 * t);
            a[j][0] = silu_half_bf16x2(acc[2 * j][0] + c0.x, acc[2 * j][1] + c0.y);
            a[j][1] = silu_half_bf16x2(acc[2 * j][2] + c0.x, acc[2 * j][3] + c0.y);
            a[j][2] = silu_half_bf16x2(acc[2 * j + 1][0] + c1.x, acc[2 * j + 1][1] + c1.y);
            a[j][3] = silu_half_bf16x2(acc[2 * j + 1][2] + c1.x, acc[2 * j + 1][3] + c1.y);
          }
          store_tile(tb + 16384u * half, a, r0, lane);
        }
      }
      handoff([&] {
        const uint64_t dW = tc::smem_desc_k128(wbp + kOffW2);
#pragma unroll
        for (int k = 0; k < 8; ++k)
          tc::umma_f16(tmem_tile + 192, dT + (k >> 2) * (16384 >> 4) + 2 * (k & 3),
                       dW + (k >> 2) * (8192 >> 4) + 2 * (k & 3), idN64, k);
      });
      {  // x += . + b2
        const float* b2 = P + 384;
        float acc[8][4];
        tmem_ld_frag(tl + 192, acc);
#pragma unroll
        for (int n = 0; n < 8; ++n) {
          const int c = 8 * n + 2 * t;
          x[n][0] += acc[n][0] + b2[c];
          x[n][1] += acc[n][1] + b2[c + 1];
          x[n][2] += acc[n][2] + b2[c];
          x[n][3] += acc[n][3] + b2[c + 1];
        }
      }
    }
    // ---- final LayerNorm and mean over the 64 squares ----
    {
      float y[8][4];
      layer_norm_plain(x, y);  // the affine part applies to the mean
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
        float* dst = sPool + (size_t)(bslot * 4 + wib) * 64;
#pragma unroll
        for (int n = 0; n < 8; ++n) {
          dst[8 * n + 2 * t] = cs[n][0];
          dst[8 * n + 2 * t + 1] = cs[n][1];
        }
      }
    }
    board_barrier(bslot);
    if (live && wib == 0) {
      const float* src = sPool + (size_t)bslot * 4 * 64;
      for (int c = lane; c < 64; c += 32) {
        const float s = src[c] + src[64 + c] + src[128 + c] + src[192 + c];
        const float v = fmaf(s * (1.0f / 64.0f), sPar[kParFinal + c], sPar[kParFinal + 64 + c]);
        const bf16 hi = __float2bfloat16_rn(v), lo = __float2bfloat16_rn(v - __bfloat162float(hi));
        bf16* o = pooled_out + (size_t)r * 3 * 64;
        o[c] = hi;
        o[64 + c] = lo;
        o[128 + c] = hi;
      }
    }
    board_barrier(bslot);
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    tc::fence_after_sync();
    tc::tmem_dealloc(*sTmem, kTmemCols);
  }
}

// [d, 64] fp32 board projection -> [d, 192] bf16 [W_hi | W_hi | W_lo], the
// content GEMM's B operand against the pooled [p_hi | p_lo | p_hi].
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

cudaError_t launch_board_hybrid(const imba_model_desc& md, const imba_step_desc& st, bf16* pooled,
                                cudaStream_t s) {
  if (st.num_rows <= 0) return cudaSuccess;
  cudaError_t e =
      cudaFuncSetAttribute(board_hybrid_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes);
  if (e != cudaSuccess) return e;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int iters = (st.num_rows + 3) / 4;
  const int grid = iters < sms ? iters : sms;
  return launch_pdl(board_hybrid_kernel, dim3(grid), dim3(kThreads), kSmemBytes, s, md.piece_square,
                    md.board_params, st.piece_ids, st.num_rows, pooled, st.status);
}

}  // namespace imba
