// Board encoder on the 5th-generation tensor cores (bf16 models): the two
// pre-LN square-attention blocks over the 64 squares of each position, the
// final LayerNorm and the mean over squares (src/imba_chess/model/
// hstu_model.py:118-179, :275-278).  Output: the pooled 64-vector of every
// board as the split bf16 operand [hi | lo | hi] (192 values), like the
// mma.sync encoder in board_mma.cu; the projection follows in a GEMM.
//
// A tile is two boards = 128 square rows, the M of one tcgen05.mma.  One
// persistent CTA per SM holds both blocks' weights in shared memory (bf16,
// K-major, 128-byte swizzle) and 512 TMEM columns.  Warp 8 issues every
// tcgen05.mma from one thread; warps 0-7 own the rows: warp w reads TMEM
// lanes 32 (w % 4) .. +31 and columns half w / 4 of each 64-wide row, so a
// row lives in two threads that combine LayerNorm / softmax partials through
// shared memory.  The fp32 residual stays in those threads' registers.
//
// Per block and tile:
//   LN1 -> H (smem)  | [Q|K] = H [Wq;Wk]^T  (M128 N128 K64)
//                    | V^T  = [Wv;*] H^T    (dims on TMEM lanes 0-63, keys on columns)
//   Q (scaled by log2(e)/4), K, V^T -> smem bf16
//   per head h: S_h = Q_h K_h^T (K16, both boards' keys; a row reads its own
//   board's 64), fp32 softmax in the log2 domain, P_h (normalised) -> smem,
//   O_h = P_h V^T_{b,h} for b = 0, 1 (N16; a row reads its board's result);
//   S of the next heads is issued while a head's softmax runs
//   O -> smem | x += O Wout^T | LN2 -> H | hidden = SiLU(H W1^T + b1) -> smem
//   | x += hidden W2^T + b2
// Hand-offs: ALU threads arrive on an mbarrier (count 256) after writing an
// operand (fence.proxy.async) or reading TMEM (tcgen05.fence); the MMA
// thread commits each group to an mbarrier the ALU threads wait on.  Every
// wait is bounded; after a failed wait all later waits return at once and
// every thread still runs the same sequence of named barriers.
#include "kernels.cuh"
#include "tc_ptx.cuh"

namespace imba {
namespace {

constexpr int kAluWarps = 8;
constexpr int kThreads = (kAluWarps + 1) * 32;
constexpr uint32_t kTmemCols = 512;

// Byte offsets inside the 1024-aligned shared window.
constexpr uint32_t kWBlock = 65536;  // one block's weights
constexpr uint32_t kOffWQK = 0;      // [128 x 64]  Wq rows 0-63, Wk rows 64-127
constexpr uint32_t kOffWV = 16384;   // [64 x 64]   Wv (rows 64-127 of the A tile read Wout)
constexpr uint32_t kOffWOut = 24576; // [64 x 64]
constexpr uint32_t kOffW1 = 32768;   // [128 x 64]
constexpr uint32_t kOffW2 = 49152;   // [64 x 128]  two 64-wide atom columns, 8 KB apart
constexpr uint32_t kOffH = 2 * kWBlock;      // [128 x 64] LN output | P of odd heads | O
constexpr uint32_t kOffQ = kOffH + 16384;    // [128 x 64] Q | hidden columns 0-63
constexpr uint32_t kOffK = kOffQ + 16384;    // [128 x 64] K | hidden columns 64-127
constexpr uint32_t kOffVT = kOffK + 16384;   // [64 dims x 128 keys], board b's keys in atom column b
constexpr uint32_t kOffP0 = kOffVT + 16384;  // [128 x 64] P of even heads
constexpr uint32_t kOffPar = kOffP0 + 16384; // fp32 parameters
constexpr int kParBlock = 448;               // ln1 w, b | ln2 w, b | b1 (128) | b2 (64)
constexpr int kParFinal = 2 * kParBlock;     // final LN w, b
constexpr uint32_t kOffXch = kOffPar + (2 * kParBlock + 128) * 4;  // [2][2 halves][128 rows] float2
constexpr uint32_t kOffPool = kOffXch + 2 * 2 * 128 * 8;            // [2 boards][2 warps][64] floats
constexpr uint32_t kOffBar = kOffPool + 2 * 2 * 64 * 4;
constexpr int kBarReady = 0, kBarP0 = 1, kBarM = 3, kBarS0 = 4, kBarPV0 = 6, kNumBars = 8;
constexpr uint32_t kOffMisc = kOffBar + kNumBars * 8;  // TMEM base, abort flag
constexpr size_t kSmemBytes = kOffMisc + 16 + 1024;    // + alignment slack

// TMEM columns (fp32 accumulators, 128 lanes = the tile's rows).
constexpr uint32_t kColQK = 0;    // [Q | K] of a block, then S of even heads, then hidden
constexpr uint32_t kColVT = 128;  // V^T (lanes 0-63), then S of odd heads, then W2 output
constexpr uint32_t kColO = 256;   // O: head h, board b at 256 + 32 h + 16 b
constexpr uint32_t kColOut = 384; // out-projection

__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Byte offset of 16-byte chunk j (0..7) of row n in a K-major tile with the
// 128-byte swizzle (8-row / 1024-byte atoms, the TMA SWIZZLE_128B layout).
__device__ __forceinline__ uint32_t sw(int n, int j) {
  return (uint32_t)((n >> 3) * 1024 + (n & 7) * 128 + (((j ^ n) & 7) << 4));
}

__device__ __forceinline__ void st_chunk(uint32_t addr, const float* v) {
  asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(pack2(v[0], v[1])),
               "r"(pack2(v[2], v[3])), "r"(pack2(v[4], v[5])), "r"(pack2(v[6], v[7]))
               : "memory");
}

__device__ __forceinline__ float exp2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 32 lanes x 16 consecutive fp32 columns: thread t gets lane (base + t).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Two 32-column TMEM loads (32 lanes each, thread t gets lane base + t) and
// one wait.
__device__ __forceinline__ void tmem_ld64(uint32_t a0, uint32_t a1, float (&v)[64]) {
  uint32_t r[64];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%64];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, "
      "%48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63}, [%65];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]),
        "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]),
        "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]),
        "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]),
        "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
      : "r"(a0), "r"(a1)
      : "memory");
#pragma unroll
  for (int i = 0; i < 64; ++i) v[i] = __uint_as_float(r[i]);
}
// Two 16-column TMEM loads into v[0..15], v[16..31], one wait.
__device__ __forceinline__ void tmem_ld16x2(uint32_t a0, uint32_t a1, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%32];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%33];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(a0), "r"(a1)
      : "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Pairwise (tree) reductions of 32 values: five dependent steps instead of 31.
__device__ __forceinline__ float sum32(const float (&v)[32]) {
  float t[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) t[i] = v[i] + v[i + 16];
#pragma unroll
  for (int w = 8; w >= 1; w >>= 1) {
#pragma unroll
    for (int i = 0; i < w; ++i) t[i] += t[i + w];
  }
  return t[0];
}
__device__ __forceinline__ float max32(const float (&v)[32]) {
  float t[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) t[i] = fmaxf(v[i], v[i + 16]);
#pragma unroll
  for (int w = 8; w >= 1; w >>= 1) {
#pragma unroll
    for (int i = 0; i < w; ++i) t[i] = fmaxf(t[i], t[i + w]);
  }
  return t[0];
}

__device__ __forceinline__ void alu_sync() { asm volatile("bar.sync 2, 256;" ::: "memory"); }

// fp32 [rows, kdim] row-major -> bf16 K-major swizzled tile (64-wide atom
// columns rows * 128 bytes apart).
__device__ void stage_weights(uint32_t dst, const float* __restrict__ w, int rows, int kdim, int tid) {
  const int cpr = kdim >> 3;
  for (int i = tid; i < rows * cpr; i += kThreads) {
    const int n = i / cpr, j = i - n * cpr;
    const float4 a = __ldg(reinterpret_cast<const float4*>(w + (size_t)n * kdim + 8 * j));
    const float4 b = __ldg(reinterpret_cast<const float4*>(w + (size_t)n * kdim + 8 * j + 4));
    const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    st_chunk(dst + (uint32_t)(j >> 3) * (uint32_t)(rows * 128) + sw(n, j & 7), v);
  }
}

__global__ void __launch_bounds__(kThreads, 1)
    board_tc_kernel(const float* __restrict__ table, const float* __restrict__ params,
                    const uint8_t* __restrict__ piece_ids, int rows, bf16* __restrict__ pooled_out,
                    int32_t* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sb = tc::smem_u32(sm);
  float* sPar = reinterpret_cast<float*>(sm + kOffPar);
  float2* sXch = reinterpret_cast<float2*>(sm + kOffXch);
  float* sPool = reinterpret_cast<float*>(sm + kOffPool);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + kOffBar);
  uint32_t* sTmem = reinterpret_cast<uint32_t*>(sm + kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + kOffMisc + 4);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int tiles = (rows + 1) >> 1;

  // ---- weights -> shared memory (step-invariant, before the PDL wait) ----
  for (int b = 0; b < 2; ++b) {
    const float* p = params + (size_t)b * IMBA_BOARD_BLOCK_FLOATS;
    const float *an_w = p, *an_b = p + 64, *qkv = p + 128, *ao = qkv + 192 * 64, *mn_w = ao + 64 * 64,
                *mn_b = mn_w + 64, *w1 = mn_b + 64, *b1 = w1 + 128 * 64, *w2 = b1 + 128, *b2 = w2 + 64 * 128;
    const uint32_t wb = sb + (uint32_t)b * kWBlock;
    stage_weights(wb + kOffWQK, qkv, 128, 64, tid);
    stage_weights(wb + kOffWV, qkv + 128 * 64, 64, 64, tid);
    stage_weights(wb + kOffWOut, ao, 64, 64, tid);
    stage_weights(wb + kOffW1, w1, 128, 64, tid);
    stage_weights(wb + kOffW2, w2, 64, 128, tid);
    float* P = sPar + b * kParBlock;
    for (int i = tid; i < 64; i += kThreads) {
      P[i] = an_w[i];
      P[64 + i] = an_b[i];
      P[128 + i] = mn_w[i];
      P[192 + i] = mn_b[i];
      P[384 + i] = b2[i];
    }
    for (int i = tid; i < 128; i += kThreads) P[256 + i] = b1[i];
  }
  for (int i = tid; i < 128; i += kThreads) sPar[kParFinal + i] = params[2 * IMBA_BOARD_BLOCK_FLOATS + i];
  if (tid == 0) {
    tc::mbar_init(&bars[kBarReady], 256);
    tc::mbar_init(&bars[kBarP0], 256);
    tc::mbar_init(&bars[kBarP0 + 1], 256);
    for (int i = kBarM; i < kNumBars; ++i) tc::mbar_init(&bars[i], 1);
    *abort_flag = 0;
    tc::fence_mbar_init();
  }
  if (warp == kAluWarps) {
    tc::tmem_alloc(sTmem, kTmemCols);
    tc::tmem_relinquish();
  }
  tc::fence_proxy_async_smem();  // the staged weights are read by the tensor cores
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *sTmem;
  // Piece ids and the pooled output are ordered after the previous kernel.
  pdl_wait();
  pdl_trigger();

  if (warp < kAluWarps) {
    // ================= row threads =================
    const int q = warp & 3, c = warp >> 2;
    const int r = 32 * q + lane, bt = q >> 1, sq = r & 63;
    const uint32_t tl = tmem + ((uint32_t)(32 * q) << 16);
    int xk = 0;  // exchange buffer parity
    // Partner exchange: this thread's value for the row's other half.
    auto exch = [&](float2 v) -> float2 {
      sXch[((xk & 1) * 2 + c) * 128 + r] = v;
      asm volatile("bar.sync %0, 64;" ::"r"(3 + q) : "memory");
      const float2 o = sXch[((xk & 1) * 2 + (c ^ 1)) * 128 + r];
      ++xk;
      return o;
    };
    // Two-pass LayerNorm (eps 1e-5) of the row's 64 values; this thread's 32.
    auto ln_half = [&](const float (&x)[32], const float* w, const float* b, float (&y)[32]) {
      float s = sum32(x);
      s += exch(make_float2(s, 0.f)).x;
      const float mu = s * (1.0f / 64.0f);
#pragma unroll
      for (int i = 0; i < 32; ++i) y[i] = (x[i] - mu) * (x[i] - mu);
      float v = sum32(y);
      v += exch(make_float2(v, 0.f)).x;
      const float rs = 1.0f / sqrtf(v * (1.0f / 64.0f) + 1e-5f);
#pragma unroll
      for (int i = 0; i < 32; ++i) y[i] = (x[i] - mu) * rs * w[i] + b[i];
    };
    // Once a wait fails (timeout, or another role's abort) every later wait
    // returns at once: the threads keep the same sequence of barriers and
    // finish with the error in the status word.
    bool dead = false;
    auto mwait = [&](int bi, uint32_t parity) {
      if (!tc::mbar_wait_or_abort(&bars[bi], parity, status, abort_flag)) dead = true;
      tc::fence_after_sync();
    };
    auto handoff = [&](int bi) {
      tc::fence_before_sync();
      tc::fence_proxy_async_smem();
      tc::mbar_arrive(&bars[bi]);
    };
    // This thread's 32 embedding values of its square in the tile.
    auto x_src = [&](int tile) -> const float4* {
      int board = 2 * tile + bt;
      if (board >= rows) board = rows - 1;
      int p = piece_ids[(size_t)board * 64 + sq];
      if (p > 12) {
        report(status, IMBA_ERR_RANGE);
        p = 0;
      }
      return reinterpret_cast<const float4*>(table + (size_t)(p * 64 + sq) * 64 + 32 * c);
    };
    auto load_x = [&](const float4* e, float (&dst)[32]) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float4 v = __ldg(e + i);
        dst[4 * i] = v.x;
        dst[4 * i + 1] = v.y;
        dst[4 * i + 2] = v.z;
        dst[4 * i + 3] = v.w;
      }
    };
    constexpr float kQScale = 0.25f * 1.4426950408889634f;  // log2(e) / sqrt(16)
    float x[32];
    int tile = blockIdx.x;
    if (tile < tiles) load_x(x_src(tile), x);
    for (; tile < tiles; tile += gridDim.x) {
      // The next tile's rows go to L1 while this one runs.
      const float4* xnext = tile + (int)gridDim.x < tiles ? x_src(tile + gridDim.x) : nullptr;
      if (xnext) asm volatile("prefetch.global.L1 [%0];" ::"l"(xnext));
#pragma unroll 1
      for (int blk = 0; blk < 2; ++blk) {
        const float* P = sPar + blk * kParBlock;
        {  // LN1 -> H
          float y[32];
          ln_half(x, P + 32 * c, P + 64 + 32 * c, y);
#pragma unroll
          for (int j = 0; j < 4; ++j) st_chunk(sb + kOffH + sw(r, 4 * c + j), y + 8 * j);
          handoff(kBarReady);
        }
        mwait(kBarM, 0);
        {  // Q (scaled) or K rows; V^T rows on lanes 0-63
          float v[64];
          tmem_ld64(tl + kColQK + 64 * c, tl + kColQK + 64 * c + 32, v);
          const float qs = c ? 1.0f : kQScale;
#pragma unroll
          for (int i = 0; i < 64; ++i) v[i] *= qs;
          const uint32_t dst = sb + (c ? kOffK : kOffQ);
#pragma unroll
          for (int j = 0; j < 8; ++j) st_chunk(dst + sw(r, j), v + 8 * j);
          if (q < 2) {
            tmem_ld64(tl + kColVT + 64 * c, tl + kColVT + 64 * c + 32, v);
#pragma unroll
            for (int j = 0; j < 8; ++j) st_chunk(sb + kOffVT + 8192u * c + sw(r, j), v + 8 * j);
          }
          handoff(kBarReady);
        }
#pragma unroll 1
        for (int h = 0; h < 4; ++h) {
          const int hb = h & 1;
          mwait(kBarS0 + hb, (h >> 1) & 1);
          float s[32];
          tc::tmem_ld32(tl + 128 * hb + 64 * bt + 32 * c, s);
          const float m = max32(s);
#pragma unroll
          for (int i = 0; i < 32; ++i) s[i] = exp2_approx(s[i] - m);
          const float l = sum32(s);
          const float2 o = exch(make_float2(m, l));
          const float M = fmaxf(m, o.x);
          const float fa = exp2_approx(m - M), fb = exp2_approx(o.x - M);
          const float f = fa / (l * fa + o.y * fb);
#pragma unroll
          for (int i = 0; i < 32; ++i) s[i] *= f;
          // P of head h - 2 (same buffer) must have been consumed.
          if (h >= 2) mwait(kBarPV0 + hb, 0);
          const uint32_t pb = sb + (hb ? kOffH : kOffP0);
#pragma unroll
          for (int j = 0; j < 4; ++j) st_chunk(pb + sw(r, 4 * c + j), s + 8 * j);
          handoff(kBarP0 + hb);
        }
        {  // O -> smem (the H buffer); PV of heads 3 and 2 done
          mwait(kBarPV0 + 1, 1);
          mwait(kBarPV0, 1);
          float o[32];
          tmem_ld16x2(tl + kColO + 64 * c + 16 * bt, tl + kColO + 64 * c + 32 + 16 * bt, o);
#pragma unroll
          for (int j = 0; j < 4; ++j) st_chunk(sb + kOffH + sw(r, 4 * c + j), o + 8 * j);
          handoff(kBarReady);
        }
        mwait(kBarM, 1);
        {  // x += O Wout^T; LN2 -> H
          float d[32];
          tc::tmem_ld32(tl + kColOut + 32 * c, d);
#pragma unroll
          for (int i = 0; i < 32; ++i) x[i] += d[i];
          float y[32];
          ln_half(x, P + 128 + 32 * c, P + 192 + 32 * c, y);
#pragma unroll
          for (int j = 0; j < 4; ++j) st_chunk(sb + kOffH + sw(r, 4 * c + j), y + 8 * j);
          handoff(kBarReady);
        }
        mwait(kBarM, 0);
        {  // hidden = SiLU(H W1^T + b1): this thread's 64 columns, one atom column
          float v[64];
          tmem_ld64(tl + kColQK + 64 * c, tl + kColQK + 64 * c + 32, v);
          const float* b1 = P + 256 + 64 * c;
#pragma unroll
          for (int i = 0; i < 64; ++i) v[i] = silu_tanh(v[i] + b1[i]);
          const uint32_t dst = sb + (c ? kOffK : kOffQ);
#pragma unroll
          for (int j = 0; j < 8; ++j) st_chunk(dst + sw(r, j), v + 8 * j);
          handoff(kBarReady);
        }
        mwait(kBarM, 1);
        {  // x += hidden W2^T + b2
          float d[32];
          tc::tmem_ld32(tl + kColVT + 32 * c, d);
          const float* b2 = P + 384 + 32 * c;
#pragma unroll
          for (int i = 0; i < 32; ++i) x[i] += d[i] + b2[i];
        }
      }
      // ---- final LayerNorm, mean over the board's 64 squares ----
      {
        float y[32];
        ln_half(x, sPar + kParFinal + 32 * c, sPar + kParFinal + 64 + 32 * c, y);
        // Column sums over the warp's 32 rows: after the halving steps lane L
        // holds column L of this thread's 32.
#pragma unroll
        for (int wd = 16; wd >= 1; wd >>= 1) {
          const bool up = (lane & wd) != 0;
#pragma unroll
          for (int i = 0; i < wd; ++i) {
            const float send = up ? y[i] : y[i + wd];
            const float keep = up ? y[i + wd] : y[i];
            y[i] = keep + __shfl_xor_sync(0xffffffffu, send, wd);
          }
        }
        sPool[(bt * 2 + (q & 1)) * 64 + 32 * c + lane] = y[0];
        alu_sync();
        const int board = 2 * tile + bt;
        if ((q & 1) == 0 && board < rows) {
          const int col = 32 * c + lane;
          const float v = (sPool[(bt * 2) * 64 + col] + sPool[(bt * 2 + 1) * 64 + col]) * (1.0f / 64.0f);
          const bf16 hi = __float2bfloat16_rn(v), lo = __float2bfloat16_rn(v - __bfloat162float(hi));
          bf16* o = pooled_out + (size_t)board * 192;
          o[col] = hi;
          o[64 + col] = lo;
          o[128 + col] = hi;
        }
      }
      if (xnext) load_x(xnext, x);
    }
  } else {
    // ================= MMA warp (one issuing thread) =================
    const uint32_t idN128 = tc::idesc_bf16_f32(128, 128), idN64 = tc::idesc_bf16_f32(128, 64),
                   idN16 = tc::idesc_bf16_f32(128, 16);
    const uint64_t dH = tc::smem_desc_k128(sm + kOffH), dQ = tc::smem_desc_k128(sm + kOffQ),
                   dK = tc::smem_desc_k128(sm + kOffK), dVT = tc::smem_desc_k128(sm + kOffVT),
                   dP0 = tc::smem_desc_k128(sm + kOffP0);
    uint32_t rp = 0;  // phases of the ready barrier consumed
    bool dead = false;
    // After a failed wait nothing more is issued; the loop runs out at once.
    auto rwait = [&](int bi, uint32_t parity) -> bool {
      if (!dead && !__all_sync(0xffffffffu, tc::mbar_wait_or_abort(&bars[bi], parity, status, abort_flag)))
        dead = true;
      tc::fence_after_sync();
      return !dead && lane == 0;
    };
    for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
#pragma unroll 1
      for (int blk = 0; blk < 2; ++blk) {
        const uint8_t* wbp = sm + (uint32_t)blk * kWBlock;
        const uint64_t dWQK = tc::smem_desc_k128(wbp + kOffWQK), dWV = tc::smem_desc_k128(wbp + kOffWV),
                       dWOut = tc::smem_desc_k128(wbp + kOffWOut), dW1 = tc::smem_desc_k128(wbp + kOffW1),
                       dW2 = tc::smem_desc_k128(wbp + kOffW2);
        if (rwait(kBarReady, rp++ & 1)) {  // [Q | K] and V^T
          for (int k = 0; k < 4; ++k) tc::umma_f16(tmem + kColQK, dH + 2 * k, dWQK + 2 * k, idN128, k);
          for (int k = 0; k < 4; ++k) tc::umma_f16(tmem + kColVT, dWV + 2 * k, dH + 2 * k, idN128, k);
          tc::umma_commit(&bars[kBarM]);
        }
        __syncwarp();
        if (rwait(kBarReady, rp++ & 1)) {  // S of heads 0 and 1
          for (int h = 0; h < 2; ++h) {
            tc::umma_f16(tmem + 128 * h, dQ + 2 * h, dK + 2 * h, idN128, 0);
            tc::umma_commit(&bars[kBarS0 + h]);
          }
        }
        __syncwarp();
        for (int h = 0; h < 4; ++h) {
          const int hb = h & 1;
          if (rwait(kBarP0 + hb, (h >> 1) & 1)) {
            const uint64_t dP = hb ? dH : dP0;
            for (int b = 0; b < 2; ++b) {
              const uint64_t dV = dVT + ((8192u * b + 2048u * h) >> 4);
              for (int k = 0; k < 4; ++k)
                tc::umma_f16(tmem + kColO + 32 * h + 16 * b, dP + 2 * k, dV + 2 * k, idN16, k);
            }
            tc::umma_commit(&bars[kBarPV0 + hb]);
            if (h < 2) {  // S of head h + 2 into the columns head h has released
              tc::umma_f16(tmem + 128 * hb, dQ + 2 * (h + 2), dK + 2 * (h + 2), idN128, 0);
              tc::umma_commit(&bars[kBarS0 + hb]);
            }
          }
          __syncwarp();
        }
        if (rwait(kBarReady, rp++ & 1)) {  // O Wout^T
          for (int k = 0; k < 4; ++k) tc::umma_f16(tmem + kColOut, dH + 2 * k, dWOut + 2 * k, idN64, k);
          tc::umma_commit(&bars[kBarM]);
        }
        __syncwarp();
        if (rwait(kBarReady, rp++ & 1)) {  // H W1^T
          for (int k = 0; k < 4; ++k) tc::umma_f16(tmem + kColQK, dH + 2 * k, dW1 + 2 * k, idN128, k);
          tc::umma_commit(&bars[kBarM]);
        }
        __syncwarp();
        if (rwait(kBarReady, rp++ & 1)) {  // hidden W2^T (K = 128: two atom columns)
          for (int k = 0; k < 8; ++k)
            tc::umma_f16(tmem + kColVT, dQ + (k >> 2) * (16384 >> 4) + 2 * (k & 3),
                         dW2 + (k >> 2) * (8192 >> 4) + 2 * (k & 3), idN64, k);
          tc::umma_commit(&bars[kBarM]);
        }
        __syncwarp();
      }
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == kAluWarps) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace

bool board_tc_applies(const imba_model_desc& md) {
  return md.dtype == IMBA_DTYPE_BF16 && (reinterpret_cast<uintptr_t>(md.board_params) & 15) == 0 &&
         (reinterpret_cast<uintptr_t>(md.piece_square) & 15) == 0;
}

cudaError_t launch_board_tc(const imba_model_desc& md, const imba_step_desc& st, bf16* pooled, cudaStream_t s) {
  if (st.num_rows <= 0) return cudaSuccess;
  cudaError_t e = cudaFuncSetAttribute(board_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes);
  if (e != cudaSuccess) return e;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int tiles = (st.num_rows + 1) / 2;
  const int grid = tiles < sms ? tiles : sms;
  return launch_pdl(board_tc_kernel, dim3(grid), dim3(kThreads), kSmemBytes, s, md.piece_square, md.board_params,
                    st.piece_ids, st.num_rows, pooled, st.status);
}

}  // namespace imba
