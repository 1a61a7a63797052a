// GEMM epilogues of the decode step.  Every GEMM computes
//   acc[r, c] = sum_k A[r, k] * W[c, k]      (W in nn.Linear [out, in] layout)
// and hands each fp32 accumulator to one of these functors.
#pragma once

#include "common.cuh"

namespace imba {

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
};

struct EpiStore {
  float* out;
  int ld;
  __device__ __forceinline__ void operator()(int r, int c, float acc) const { out[(size_t)r * ld + c] = acc; }
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
};

}  // namespace imba
