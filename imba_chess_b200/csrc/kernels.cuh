// Launch functions of the step kernels (one translation unit each).
#pragma once

#include "epilogues.cuh"

namespace imba {

struct AttnArgs {
  const void* q;        // [R, H dqk] model dtype
  const void* pool;     // paged KV pool, model dtype
  PoolGeom g;
  int layer;
  const float* ps_w;    // [H, 2 max_pos - 1]
  int max_pos;
  float scale;          // 1 / sqrt(d_qk)
  imba_step_desc st;
  float* out;           // [R, H dv]
  int* counters;        // this layer's work-queue counters (zero at launch)
};

cudaError_t launch_embed(const imba_model_desc& md, const imba_step_desc& st, float* x, cudaStream_t s);
// Board encoder -> pooled [R, 192] split bf16 ([hi | lo | hi] of the mean):
// tcgen05 projections + mma.sync per-head attention (board_hybrid.cu).
cudaError_t launch_board_hybrid(const imba_model_desc& md, const imba_step_desc& st, bf16* pooled, cudaStream_t s);
// [d, 64] fp32 board projection -> [d, 192] bf16 [W_hi | W_hi | W_lo].
cudaError_t build_board_proj_split(const imba_model_desc& md, bf16* out, cudaStream_t s);
template <typename T>
cudaError_t launch_ln_rows(const float* x, int rows, int n, float eps, T* out, cudaStream_t s);
template <typename T>
cudaError_t launch_gate(const float* attn, const T* u, int rows, int n, T* out, cudaStream_t s);
// The same with the attention output already rounded to bf16 (n a multiple of 128).
cudaError_t launch_gate_bf16(const bf16* attn, const bf16* u, int rows, int n, bf16* out, cudaStream_t s);
template <typename T>
cudaError_t launch_final_ln(const float* x, int rows, int n, const float* w, const float* b, float* out32, T* out3,
                            cudaStream_t s);
// logits == nullptr: legal logits as fp32 gathers of x32 . policy_w32[id] (scratch: [R, vocab] floats).
cudaError_t launch_value_legal(const imba_model_desc& md, const imba_step_desc& st, const float* hval,
                               const float* logits, const float* x32, float* scratch, cudaStream_t s);
template <typename T>
cudaError_t launch_kv_copy(const PoolGeom& g, T* pool, int layer, int n, const int32_t* slots, T* dk, T* dv,
                           int to_pool, int32_t* status, cudaStream_t s);
template <typename T>
cudaError_t launch_kv_scatter_indexed(const PoolGeom& g, T* pool, int layer, int n, const int32_t* slots,
                                      const int32_t* ia, const int32_t* ib, const T* sk, const T* sv,
                                      const KVStrides& st, int32_t* status, cudaStream_t s);
template <typename TA, typename TW, class Epi>
cudaError_t launch_gemm_simt(const TA* A, int lda, const TW* W, int ldw, int M, int N, int K, Epi epi,
                             cudaStream_t s);
template <typename T>
cudaError_t launch_attn_simt(const AttnArgs& a, cudaStream_t s);
// Tensor-core paged attention (bf16, head dims 64); false when it does not
// apply.  With every head in one CTA it also applies the attention-output
// norm and the u gate, writes `gated` and sets *fused.
// recs: this step's resolved work items, written once per step by
// launch_attn_items ([2 num_chunks][kAttnRecInts]).
cudaError_t launch_attn_items(const imba_step_desc& st, const PoolGeom& g, int* recs, cudaStream_t s);
bool launch_attn_page(const AttnArgs& a, int num_layers, const imba_model_desc& md, int64_t num_pages,
                      const bf16* u, bf16* gated, const int* recs, cudaStream_t s, cudaError_t* err, bool* fused,
                      float2* ml = nullptr);
// After launch_attn_page with `ml` (the pages only): the rows' extra keys,
// the attention-output norm and the u gate (H <= 8).
cudaError_t launch_attn_combine(const AttnArgs& a, const float2* ml, const bf16* u, bf16* gated, cudaStream_t s);
// Jagged prefill attention (tcgen05; bf16, head dims 64, an even head
// count): for steps without extra keys.  Writes O rounded to bf16 over a.out
// ([R, H dv] bf16 in its first half; the norm / gate is a separate pass,
// launch_gate_bf16); false when it does not apply.
bool launch_attn_prefill(const AttnArgs& a, int num_layers, int64_t num_pages, const int* recs, cudaStream_t s,
                         cudaError_t* err);

// Places imba_step_noalloc's scratch array on the current device (noalloc.cu).
imba_status_t noalloc_prepare_device();

}  // namespace imba
