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

  // 32 consecutive columns starting at c0 (a multiple of 32; d_qk and d_v
  // are multiples of 32, so a chunk never straddles a head or a region).
  __device__ __forceinline__ void chunk32(int r, int c0, int /*N*/, const float (&a)[32]) const {
    float y[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) y[i] = silu_f(a[i]);
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
    const int64_t slot = dst_slot[r];
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
  __device__ __forceinline__ void chunk32(int r, int c0, int N, const float (&a)[32]) const {
    if (c0 >= N) return;
    float4* p = reinterpret_cast<float4*>(x + (size_t)r * ld + c0);
    const float4* b = reinterpret_cast<const float4*>(bias + c0);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float4 xv = p[i];
      const float4 bv = b[i];
      xv.x = (a[4 * i] + bv.x) + xv.x;
      xv.y = (a[4 * i + 1] + bv.y) + xv.y;
      xv.z = (a[4 * i + 2] + bv.z) + xv.z;
      xv.w = (a[4 * i + 3] + bv.w) + xv.w;
      p[i] = xv;
    }
  }
};

struct EpiStore {
  float* out;
  int ld;
  __device__ __forceinline__ void operator()(int r, int c, float acc) const { out[(size_t)r * ld + c] = acc; }
  // Scalar stores: the policy row stride (vocab floats) is not 16-byte aligned.
  __device__ __forceinline__ void chunk32(int r, int c0, int N, const float (&a)[32]) const {
    float* o = out + (size_t)r * ld;
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (c0 + i < N) o[c0 + i] = a[i];
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
  __device__ __forceinline__ void chunk32(int r, int c0, int N, const float (&a)[32]) const {
    if (c0 >= N) return;
    float y[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) y[i] = silu_f(a[i] + bias[c0 + i]);
    store32(out + (size_t)r * ld + c0, y);
  }
};

}  // namespace imba
