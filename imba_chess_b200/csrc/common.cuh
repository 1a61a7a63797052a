// Shared device helpers and the internal model / workspace structures of the
// imba_b200 library.  Device code only uses the fp32 and bf16 storage types;
// every reduction and every softmax is carried out in fp32 (fp64 for the
// legal-move log-softmax, which the reference computes in float64).
#pragma once

#include <utility>

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "imba_b200.h"

namespace imba {

using bf16 = __nv_bfloat16;

__device__ __forceinline__ float to_f(float x) { return x; }
__device__ __forceinline__ float to_f(bf16 x) { return __bfloat162float(x); }

template <typename T>
__device__ __forceinline__ T from_f(float x);
template <>
__device__ __forceinline__ float from_f<float>(float x) { return x; }
template <>
__device__ __forceinline__ bf16 from_f<bf16>(float x) { return __float2bfloat16_rn(x); }

__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + expf(-x)); }
// SiLU with the fast exponential / division intrinsics (bf16 tensor-core epilogues).
// Programmatic dependent launch.  Step kernels are launched with
// launch_pdl(), so a kernel may begin (CTA scheduling, barrier / TMEM set-up,
// reads of weights and host-written step metadata) while the previous kernel
// of the stream finishes.  pdl_wait() returns once that kernel has completed
// and its writes are visible; every step kernel calls it before touching
// memory that an earlier kernel of the step writes or reads, which keeps the
// completion order transitive along the stream.  pdl_trigger() lets the next
// kernel be scheduled.  Both are no-ops for kernels launched without the
// attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ float silu_fast(float x) { return __fdividef(x, 1.0f + __expf(-x)); }
// x * sigmoid(x) with sigmoid(x) = (1 + tanh(x / 2)) / 2 on the hardware tanh
// (one MUFU op instead of an exponential and a reciprocal; relative error
// ~2^-11, used where the result is rounded to bf16 or gates bf16 data).
__device__ __forceinline__ float silu_tanh(float x) {
  const float h = 0.5f * x;
  float th;
  asm("tanh.approx.f32 %0, %1;" : "=f"(th) : "f"(h));
  return fmaf(h, th, h);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// First error wins; later errors never overwrite it.
__device__ __forceinline__ void report(int32_t* status, int32_t code) {
  if (status) atomicCAS(status, 0, code);
}

// Geometry of the paged KV pool for one model.
struct PoolGeom {
  int64_t page_stride;   // elements per page (all layers)
  int64_t layer_stride;  // elements per layer within a page
  int64_t v_offset;      // offset of the V block within a layer block
  int64_t num_slots;     // num_pages * IMBA_PAGE_TOKENS
  int H, dqk, dv;

  // Element offset of token slot `slot`, layer `l`, head `h`, K block.
  __host__ __device__ __forceinline__ int64_t k_off(int64_t slot, int l, int h) const {
    return (slot / IMBA_PAGE_TOKENS) * page_stride + (int64_t)l * layer_stride +
           ((int64_t)h * IMBA_PAGE_TOKENS + (slot % IMBA_PAGE_TOKENS)) * dqk;
  }
  __host__ __device__ __forceinline__ int64_t v_off(int64_t slot, int l, int h) const {
    return (slot / IMBA_PAGE_TOKENS) * page_stride + (int64_t)l * layer_stride + v_offset +
           ((int64_t)h * IMBA_PAGE_TOKENS + (slot % IMBA_PAGE_TOKENS)) * dv;
  }
};

// Element strides [a, b, head, dim] of a dense K or V source (imba_kv_scatter_indexed).
struct KVStrides {
  int64_t k[4];
  int64_t v[4];
};

}  // namespace imba

// The opaque handle behind imba_model*.
struct imba_model {
  imba_model_desc d;
  int uvqk_n;         // 2 H (d_v + d_qk)
  void* tc = nullptr;  // tensor-core GEMM state (TMA descriptors of the weights), or null
  // Test hooks of bf16 handles (imba_model_desc.flags): the SIMT kernel of a
  // component instead of its tensor-core kernel, for cross-checks.
  bool simt_gemm = false;
  bool simt_attn = false;
  bool simt_board = false;
  // bf16 models with the tensor-core board encoder: [d, 192] bf16 split copy
  // of the board projection (device memory owned by the handle), or null.
  void* board_proj3 = nullptr;
  imba::PoolGeom geom(int64_t num_pages) const {
    imba::PoolGeom g;
    g.H = d.num_heads;
    g.dqk = d.attention_dim;
    g.dv = d.linear_dim;
    g.v_offset = (int64_t)d.num_heads * IMBA_PAGE_TOKENS * d.attention_dim;
    g.layer_stride = (int64_t)d.num_heads * IMBA_PAGE_TOKENS * (d.attention_dim + d.linear_dim);
    g.page_stride = g.layer_stride * d.num_layers;
    g.num_slots = num_pages * IMBA_PAGE_TOKENS;
    return g;
  }
};

namespace imba {

// Scratch buffers carved out of the caller's workspace for one step.
// Work-queue counters per step: one per (layer, attention head group).
constexpr int kCountersPerLayer = 16;
constexpr int kNumCounters = IMBA_MAX_LAYERS * kCountersPerLayer;
// One resolved attention work item (<= 32 rows of one chunk), int32 words:
// written once per step by the item pass, read by every layer's attention.
constexpr int kAttnRecInts = 296;

struct Workspace {
  float* x;        // [R, d]      residual stream
  void* xn;        // [R, d]      LN(x), model dtype
  void* u;         // [R, H dv]   gate (post-SiLU u), model dtype
  void* q;         // [R, H dqk]  queries, model dtype
  float* attn;     // [R, H dv]   attention output
  void* gated;     // [R, H dv]   LN(attn) * u, model dtype
  float* xf32;     // [R, d]      final LN output, fp32
  void* xf3;       // [R, 3d]     bf16 only: final LN output as [hi | lo | hi]
  float* hval;     // [R, d/2]    value-head hidden
  float* logits;   // [R, vocab]  used when the caller passes no logits buffer
  void* pooled;    // [R, 192]    bf16 models: mean-pooled board-encoder output, split bf16
  int* counters;   // [kNumCounters] work-queue counters, zeroed at the start of every step
  int* recs;       // [2 R][kAttnRecInts] bf16 models: resolved attention work items
  float2* ml;      // [R, H]      bf16 models: (max, sum) of each row's pages-only attention pass
  size_t bytes;
};

Workspace carve_workspace(const imba_model* m, int32_t rows, void* base);

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                              Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace imba
