// GEMM epilogues of the decode step.  Every GEMM computes
//   acc[r, c] = sum_k A[r, k] * W[c, k]      (W in nn.Linear [out, in] layout)
// and hands each fp32 accumulator to one of these functors.
#pragma once

#include "common.cuh"

namespace imba {

// Store 32 consecutive values (16-byte aligned destination) as 128-bit stores.
__device__ __forceinline__ void store32(float* dst, const float (&v)[32]) {
  float4* d = reinterpret_cast<float4*>(dst);
#pragma unroll
  for (int i = 0; i < 8; ++i) d[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
}
__device__ __forceinline__ void store32(bf16* dst, const float (&v)[32]) {
  uint32_t w[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
    w[i] = *reinterpret_cast<uint32_t*>(&h);
  }
  uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int i = 0; i < 4; ++i) d[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
}

// uvqk projection epilogue: SiLU, then the reference's split order u | v | q | k
// (src/imba_chess/model/hstu_attention.py:310-325).  u goes to the fp32 gate
// buffer, q to the query buffer, and k / v straight into the row's slot of the
// paged KV pool (the KV append, fused).
template <typename T>
struct EpiUVQK {
  float* u;
  T* q;
  T* pool;
  const int32_t* dst_slot;
  PoolGeom g;
  int layer;
  int32_t* status;

  __device__ __forceinline__ void operator()(int r, int c, float acc) const {
    const float y = silu_f(acc);
    const int hdv = g.H * g.dv, hdq = g.H * g.dqk;
    if (c < hdv) {
      u[(size_t)r * hdv + c] = y;
      return;
    }
    c -= hdv;
    if (c < hdv) {
      const int64_t slot = dst_slot[r];
      if (slot < 0 || slot >= g.num_slots) {
        report(status, IMBA_ERR_RANGE);
        return;
      }
      pool[g.v_off(slot, layer, c / g.dv) + (c % g.dv)] = from_f<T>(y);
      return;
    }
    c -= hdv;
    if (c < hdq) {
      q[(size_t)r * hdq + c] = from_f<T>(y);
      return;
    }
    c -= hdq;
    const int64_t slot = dst_slot[r];
    if (slot < 0 || slot >= g.num_slots) {
      report(status, IMBA_ERR_RANGE);
      return;
    }
    pool[g.k_off(slot, layer, c / g.dqk) + (c % g.dqk)] = from_f<T>(y);
  }

  // Per-row state of the tensor-core epilogue: the row's KV slot, loaded once per tile.
  struct Ctx {
    int64_t slot;
  };
  __device__ __forceinline__ Ctx begin(int r, int /*n0*/, int /*bn*/) const { return Ctx{(int64_t)dst_slot[r]}; }

  // 32 consecutive columns starting at c0 (a multiple of 32; d_qk and d_v
  // are multiples of 32, so a chunk never straddles a head or a region).
  __device__ __forceinline__ void chunk32(const Ctx& cx, int r, int c0, int N, const float (&a)[32]) const {
    if (c0 >= N) return;
    float y[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) y[i] = silu_tanh(a[i]);
    const int hdv = g.H * g.dv, hdq = g.H * g.dqk;
    if (c0 < hdv) {
      store32(u + (size_t)r * hdv + c0, y);
      return;
    }
    int c = c0 - hdv;
    if (c >= hdv && c - hdv < hdq) {
      store32(q + (size_t)r * hdq + (c - hdv), y);
      return;
    }
    const int64_t slot = cx.slot;
    if (slot < 0 || slot >= g.num_slots) {
      report(status, IMBA_ERR_RANGE);
      return;
    }
    if (c < hdv) {
      store32(pool + g.v_off(slot, layer, c / g.dv) + (c % g.dv), y);
    } else {
      c -= hdv + hdq;
      store32(pool + g.k_off(slot, layer, c / g.dqk) + (c % g.dqk), y);
    }
  }
};

// Output projection epilogue: x = (acc + bias) + x   (hstu_attention.py:423)
struct EpiResidual {
  float* x;
  const float* bias;
  int ld;
  __device__ __forceinline__ void operator()(int r, int c, float acc) const {
    float* p = x + (size_t)r * ld + c;
    *p = (acc + bias[c]) + *p;
  }
  // The tile's residual lines are prefetched into L1 when the row starts.
  struct Ctx {};
  __device__ __forceinline__ Ctx begin(int r, int n0, int bn) const {
    const float* p = x + (size_t)r * ld + n0;
    for (int c = 0; c < bn && n0 + c < ld; c += 32)
      asm volatile("prefetch.global.L1 [%0];" ::"l"(p + c));
    return Ctx{};
  }
  // All loads are issued before any store: interleaving each load after the
  // previous store of the same row serialises them (the compiler cannot prove
  // x and bias do not alias) and was measured ~30x slower.
  __device__ __forceinline__ void chunk32(const Ctx&, int r, int c0, int N, const float (&a)[32]) const {
    if (c0 >= N) return;
    float4* p = reinterpret_cast<float4*>(x + (size_t)r * ld + c0);
    const float4* b = reinterpret_cast<const float4*>(bias + c0);
    float4 xv[8], bv[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      xv[i] = p[i];
      bv[i] = __ldg(b + i);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      xv[i].x = (a[4 * i] + bv[i].x) + xv[i].x;
      xv[i].y = (a[4 * i + 1] + bv[i].y) + xv[i].y;
      xv[i].z = (a[4 * i + 2] + bv[i].z) + xv[i].z;
      xv[i].w = (a[4 * i + 3] + bv[i].w) + xv[i].w;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) p[i] = xv[i];
  }
};

struct EpiStore {
  float* out;
  int ld;
  __device__ __forceinline__ void operator()(int r, int c, float acc) const { out[(size_t)r * ld + c] = acc; }
  struct Ctx {};
  __device__ __forceinline__ Ctx begin(int, int, int) const { return Ctx{}; }
  // The policy row stride (vocab floats) is even but not a multiple of 4:
  // full chunks use 8-byte stores, the ragged last chunk scalar stores.
  __device__ __forceinline__ void chunk32(const Ctx&, int r, int c0, int N, const float (&a)[32]) const {
    float* o = out + (size_t)r * ld + c0;
    if (c0 + 32 <= N && ((reinterpret_cast<uintptr_t>(o) & 7) == 0)) {
      float2* o2 = reinterpret_cast<float2*>(o);
#pragma unroll
      for (int i = 0; i < 16; ++i) o2[i] = make_float2(a[2 * i], a[2 * i + 1]);
      return;
    }
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (c0 + i < N) o[i] = a[i];
  }
};

// Adds into an existing fp32 output (split-precision passes).
struct EpiAccumulate {
  float* out;
  int ld;
  __device__ __forceinline__ void operator()(int r, int c, float acc) const { out[(size_t)r * ld + c] += acc; }
};

// Value-head hidden layer: SiLU(acc + bias)   (hstu_model.py:252-257)
struct EpiBiasSilu {
  float* out;
  const float* bias;
  int ld;
  __device__ __forceinline__ void operator()(int r, int c, float acc) const {
    out[(size_t)r * ld + c] = silu_f(acc + bias[c]);
  }
  struct Ctx {};
  __device__ __forceinline__ Ctx begin(int, int, int) const { return Ctx{}; }
  __device__ __forceinline__ void chunk32(const Ctx&, int r, int c0, int N, const float (&a)[32]) const {
    if (c0 >= N) return;
    float y[32];
    const float4* b = reinterpret_cast<const float4*>(bias + c0);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 bv = __ldg(b + i);
      y[4 * i] = silu_f(a[4 * i] + bv.x);
      y[4 * i + 1] = silu_f(a[4 * i + 1] + bv.y);
      y[4 * i + 2] = silu_f(a[4 * i + 2] + bv.z);
      y[4 * i + 3] = silu_f(a[4 * i + 3] + bv.w);
    }
    store32(out + (size_t)r * ld + c0, y);
  }
};

// Content embedding epilogue (bf16 models): acc = pooled . board_out^T, then
// x = (acc + b_out + seq + turn + castle + ep + halfmove + fullmove + prev_move)
//     * sqrt(d) + pos_emb[min(pos, max_pos - 1)]
// with side ids clamped to their tables (hstu_model.py:275-335;
// position_embedding.py:52-62).
struct EpiContent {
  float* x;
  const imba_model_desc* md;  // device copy not needed: pointers and sizes only
  const float* bias;
  const float *seq, *turn, *castle, *ep, *half, *full, *prev, *pos_emb;
  const int32_t* side_ids;
  const int32_t* positions;
  int d, halfmove_vocab, fullmove_vocab, vocab, max_pos;
  float scale;
  int32_t* status;

  __device__ __forceinline__ static int clampi(int v, int n) { return v < 0 ? 0 : (v >= n ? n - 1 : v); }
  __device__ __forceinline__ void operator()(int r, int c, float acc) const {
    const int32_t* ids = side_ids + (size_t)r * IMBA_NUM_SIDE_IDS;
    float v = acc + bias[c];
    v += seq[(size_t)clampi(ids[0], 2) * d + c];
    v += turn[(size_t)clampi(ids[1], 2) * d + c];
    v += castle[(size_t)clampi(ids[2], 16) * d + c];
    v += ep[(size_t)clampi(ids[3], 9) * d + c];
    v += half[(size_t)clampi(ids[4], halfmove_vocab) * d + c];
    v += full[(size_t)clampi(ids[5], fullmove_vocab) * d + c];
    v += prev[(size_t)clampi(ids[6], vocab) * d + c];
    int p = positions[r];
    if (p < 0) {
      report(status, IMBA_ERR_RANGE);
      p = 0;
    }
    if (p > max_pos - 1) p = max_pos - 1;
    x[(size_t)r * d + c] = v * scale + pos_emb[(size_t)p * d + c];
  }
};

}  // namespace imba
