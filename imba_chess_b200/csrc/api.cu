// C ABI entry points: handle lifetime, workspace sizing and the per-step
// launch sequence (embedding -> L x [LN, uvqk GEMM + KV append, paged
// attention, gate, output GEMM + residual] -> heads -> legal projection).
// Mirrors HSTUChessModel.forward_decode_grouped / forward
// (src/imba_chess/model/hstu_model.py:337-374, :651-752).
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <new>
#include <type_traits>

#include "gemm_tc.cuh"
#include "kernels.cuh"

namespace imba {

namespace {

constexpr size_t kAlign = 256;
inline size_t align_up(size_t x) { return (x + kAlign - 1) / kAlign * kAlign; }

inline size_t dtype_bytes(int dtype) { return dtype == IMBA_DTYPE_BF16 ? 2 : 4; }

size_t workspace_layout(const imba_model* m, int32_t rows, void* base, Workspace* ws) {
  const imba_model_desc& d = m->d;
  const size_t R = (size_t)(rows > 0 ? rows : 0);
  const size_t eb = dtype_bytes(d.dtype);
  const size_t hdv = (size_t)d.num_heads * d.linear_dim, hdq = (size_t)d.num_heads * d.attention_dim;
  size_t off = 0;
  char* b = static_cast<char*>(base);
  auto take = [&](size_t bytes) -> void* {
    void* p = b ? b + off : nullptr;
    off += align_up(bytes);
    return p;
  };
  Workspace w{};
  w.x = static_cast<float*>(take(R * d.model_dim * 4));
  w.xn = take(R * d.model_dim * eb);
  w.u = take(R * hdv * eb);
  w.q = take(R * hdq * eb);
  w.attn = static_cast<float*>(take(R * hdv * 4));
  w.gated = take(R * hdv * eb);
  w.xf32 = static_cast<float*>(take(R * d.model_dim * 4));
  w.xf3 = take(d.dtype == IMBA_DTYPE_BF16 ? R * 3 * d.model_dim * 2 : 0);
  w.hval = static_cast<float*>(take(R * (d.model_dim / 2 + 1) * 4));
  w.logits = static_cast<float*>(take(R * d.vocab * 4));
  w.pooled = take(d.dtype == IMBA_DTYPE_BF16 ? R * 3 * IMBA_BOARD_DIM * 2 : 0);
  w.counters = static_cast<int*>(take(kNumCounters * sizeof(int)));
  // paged attention work items: at most one chunk per row, two records per chunk
  w.recs = static_cast<int*>(take(d.dtype == IMBA_DTYPE_BF16 ? 2 * R * kAttnRecInts * sizeof(int) : 0));
  // per row and head (max, sum) of the paged attention's pages-only pass
  w.ml = static_cast<float2*>(take(d.dtype == IMBA_DTYPE_BF16 ? R * d.num_heads * sizeof(float2) : 0));
  w.bytes = off;
  if (ws) *ws = w;
  return off;
}

imba_status_t validate_desc(const imba_model_desc* d) {
  if (!d) return IMBA_ERR_ARG;
  if (d->model_dim <= 0 || d->model_dim > 1024 || d->model_dim % 2) return IMBA_ERR_UNSUPPORTED;
  if (d->num_layers <= 0 || d->num_layers > IMBA_MAX_LAYERS) return IMBA_ERR_UNSUPPORTED;
  if (d->num_heads <= 0 || d->attention_dim <= 0 || d->attention_dim > 64 || d->linear_dim <= 0 ||
      d->linear_dim > 64)
    return IMBA_ERR_UNSUPPORTED;
  if ((int64_t)d->num_heads * d->linear_dim > 1024) return IMBA_ERR_UNSUPPORTED;
  if (d->vocab <= 0 || d->max_pos <= 0 || d->halfmove_vocab <= 0 || d->fullmove_vocab <= 0) return IMBA_ERR_ARG;
  if (d->dtype != IMBA_DTYPE_F32 && d->dtype != IMBA_DTYPE_BF16) return IMBA_ERR_ARG;
  if (d->flags & ~(IMBA_FLAG_SIMT_GEMM | IMBA_FLAG_SIMT_ATTN | IMBA_FLAG_SIMT_BOARD)) return IMBA_ERR_ARG;
  const void* req[] = {d->piece_square, d->board_params, d->board_out_w, d->board_out_b, d->emb_seq,
                       d->emb_turn,     d->emb_castle,   d->emb_ep,      d->emb_halfmove, d->emb_fullmove,
                       d->emb_prev_move, d->emb_pos,     d->final_norm_w, d->final_norm_b, d->policy_w,
                       d->policy_w32};
  for (const void* p : req)
    if (!p) return IMBA_ERR_ARG;
  for (int l = 0; l < d->num_layers; ++l)
    if (!d->uvqk_w[l] || !d->o_w[l] || !d->o_b[l] || !d->ps_w[l]) return IMBA_ERR_ARG;
  if (d->has_value_head && (!d->value0_w || !d->value0_b || !d->value2_w || !d->value2_b)) return IMBA_ERR_ARG;
  return IMBA_OK;
}

// Shapes the bf16 tensor-core kernels cover: the GEMM tiles (d and H dv
// multiples of 128, the uvqk width a multiple of 256) and the paged
// attention (head dims 64 / 64, at most 16 head groups of 8).
bool bf16_shape_supported(const imba_model_desc& d, bool simt_gemm, bool simt_attn) {
  const int hdv = d.num_heads * d.linear_dim;
  const int uvqk_n = 2 * d.num_heads * (d.linear_dim + d.attention_dim);
  const bool gemm_ok = d.model_dim % 128 == 0 && hdv % 128 == 0 && uvqk_n % 256 == 0 && d.attention_dim % 32 == 0 &&
                       d.linear_dim % 32 == 0;
  const bool attn_ok = d.attention_dim == 64 && d.linear_dim == 64 && d.num_heads <= 128;
  return (simt_gemm || gemm_ok) && (simt_attn || attn_ok);
}

imba_status_t validate_step(const imba_model* m, const imba_step_desc* st, const imba_pool_desc* pool) {
  if (!st || !pool) return IMBA_ERR_ARG;
  if (st->num_rows < 0 || st->num_groups < 0 || st->num_chunks < 0 || st->num_legal < 0 || st->num_extra < 0 ||
      st->num_group_pages < 0)
    return IMBA_ERR_ARG;
  if (st->num_rows == 0) return IMBA_OK;
  if (st->num_chunks > st->num_rows) return IMBA_ERR_ARG;  // every chunk holds at least one row
  if (!pool->base || pool->num_pages <= 0) return IMBA_ERR_ARG;
  if (reinterpret_cast<uintptr_t>(pool->base) & 255) return IMBA_ERR_ARG;  // TMA views need aligned bases
  if (pool->num_pages > (int64_t)INT32_MAX / IMBA_PAGE_TOKENS) return IMBA_ERR_RANGE;
  const void* req[] = {st->piece_ids, st->side_ids, st->positions, st->row_vis, st->row_extra_off,
                       st->row_dst_slot, st->row_perm};
  for (const void* p : req)
    if (!p) return IMBA_ERR_ARG;
  if (st->num_chunks > 0 && (!st->chunk_group || !st->chunk_row_off || !st->chunk_nrows || !st->group_page_off))
    return IMBA_ERR_ARG;
  if (st->num_group_pages > 0 && !st->group_pages) return IMBA_ERR_ARG;
  if (st->num_extra > 0 && (!st->extra_slot || !st->extra_pos)) return IMBA_ERR_ARG;
  if (st->legal_off && st->num_legal > 0 && !st->legal_ids) return IMBA_ERR_ARG;
  if ((st->legal_logits || st->legal_logprob) && !st->legal_off) return IMBA_ERR_ARG;
  (void)m;
  return IMBA_OK;
}

// Records phase-boundary events when profiling; a no-op otherwise.
struct PhaseMarks {
  void* const* ev = nullptr;
  int n = 0;
  int next = 0;
  cudaError_t mark(cudaStream_t s) {
    if (!ev) return cudaSuccess;
    if (next >= n) return cudaErrorInvalidValue;
    return cudaEventRecord(static_cast<cudaEvent_t>(ev[next++]), s);
  }
};

template <typename T>
imba_status_t run_step(const imba_model* m, const imba_step_desc& st, const imba_pool_desc& pool, Workspace& w,
                       cudaStream_t s, PhaseMarks& pm) {
  const imba_model_desc& md = m->d;
  const int R = st.num_rows, d = md.model_dim, H = md.num_heads;
  const int hdv = H * md.linear_dim;
  const PoolGeom g = m->geom(pool.num_pages);
  T* poolp = static_cast<T*>(pool.base);
  cudaError_t e;
#define IMBA_CK(...)               \
  do {                             \
    e = (__VA_ARGS__);             \
    if (e != cudaSuccess) return IMBA_ERR_CUDA; \
  } while (0)

  IMBA_CK(pm.mark(s));
  IMBA_CK(cudaMemsetAsync(w.counters, 0, kNumCounters * sizeof(int), s));
  // The paged attention's work items, resolved once for every layer.
  const bool paged_attn = md.dtype == IMBA_DTYPE_BF16 && !m->simt_attn;
  if (paged_attn) IMBA_CK(launch_attn_items(st, g, w.recs, s));
  // A step whose rows find every key in their groups' pages and that has
  // several rows per group on average (a jagged prefill of documents) runs
  // the prefill attention kernel; decode waves (every row has extra keys)
  // and short root extensions run the paged decode kernel.
  const bool prefill_attn = paged_attn && st.num_extra == 0 && st.num_rows >= 4 * st.num_groups;
  // Decode steps whose rows carry suffix chains (extra keys beyond
  // themselves) or whose groups have few rows run the paged kernel over the
  // pages only and fold the extra keys, norm and gate into a per-row pass
  // (attn_combine): the per-item extra-key and norm work then leaves the
  // kernel's critical path.  Sibling waves (many rows per group, one extra
  // key each) keep the fused kernel.
  const bool partial_attn = paged_attn && !prefill_attn && md.num_heads <= 8 &&
                            (st.num_extra > st.num_rows || st.num_rows < 4 * st.num_groups);
  // bf16 handles run the tensor-core kernels; a launcher that declines
  // (returns false) is an error unless a SIMT test hook selected the SIMT
  // kernel of that component (imba_model_desc.flags).
  const bool tc_gemm = md.dtype == IMBA_DTYPE_BF16 && !m->simt_gemm;
  if (md.dtype == IMBA_DTYPE_BF16 && !m->simt_board) {
    // tensor-core board encoder -> pooled [R, 192] split bf16; projection + embeddings in the GEMM epilogue
    IMBA_CK(launch_board_hybrid(md, st, static_cast<bf16*>(w.pooled), s));
    EpiContent ec{w.x, nullptr, md.board_out_b, md.emb_seq, md.emb_turn, md.emb_castle, md.emb_ep, md.emb_halfmove,
                  md.emb_fullmove, md.emb_prev_move, md.emb_pos, st.side_ids, st.positions, d, md.halfmove_vocab,
                  md.fullmove_vocab, md.vocab, md.max_pos, sqrtf((float)d), st.status};
    const bf16* p3 = static_cast<const bf16*>(w.pooled);
    if (!gemm_tc_launch_content(m, R, p3, ec, st.status, s, &e)) {
      if (tc_gemm) return IMBA_ERR_UNSUPPORTED;
      IMBA_CK(launch_gemm_simt<bf16, bf16, EpiContent>(p3, 3 * IMBA_BOARD_DIM, static_cast<const bf16*>(m->board_proj3),
                                                       3 * IMBA_BOARD_DIM, R, d, 3 * IMBA_BOARD_DIM, ec, s));
    } else if (e != cudaSuccess) {
      return IMBA_ERR_CUDA;
    }
  } else {
    IMBA_CK(launch_embed(md, st, w.x, s));
  }
  IMBA_CK(pm.mark(s));
  for (int l = 0; l < md.num_layers; ++l) {
    IMBA_CK(launch_ln_rows<T>(w.x, R, d, 1e-6f, static_cast<T*>(w.xn), s));
    IMBA_CK(pm.mark(s));
    EpiUVQK<T> epi{static_cast<T*>(w.u), static_cast<T*>(w.q), poolp, st.row_dst_slot, g, l, st.status};
    if (!gemm_tc_launch_uvqk(m, l, R, static_cast<const T*>(w.xn), epi, s, &e)) {
      if (tc_gemm) return IMBA_ERR_UNSUPPORTED;
      IMBA_CK(launch_gemm_simt<T, T, EpiUVQK<T>>(static_cast<const T*>(w.xn), d,
                                                static_cast<const T*>(md.uvqk_w[l]), d, R, m->uvqk_n, d, epi, s));
    } else if (e != cudaSuccess) {
      return IMBA_ERR_CUDA;
    }
    IMBA_CK(pm.mark(s));
    AttnArgs aa{w.q, pool.base, g, l, md.ps_w[l], md.max_pos, 1.0f / sqrtf((float)md.attention_dim), st, w.attn,
                w.counters + l * kCountersPerLayer};
    bool fused = false;
    bf16* gated_bf = std::is_same<T, bf16>::value ? reinterpret_cast<bf16*>(w.gated) : nullptr;
    bool gate_bf16 = false;  // the attention output was stored as bf16
    if (prefill_attn && launch_attn_prefill(aa, md.num_layers, pool.num_pages, w.recs, s, &e)) {
      if (e != cudaSuccess) return IMBA_ERR_CUDA;
      gate_bf16 = true;
    } else if (partial_attn && launch_attn_page(aa, md.num_layers, md, pool.num_pages,
                                                         static_cast<const bf16*>(w.u), nullptr, w.recs, s, &e,
                                                         &fused, w.ml)) {
      if (e != cudaSuccess) return IMBA_ERR_CUDA;
      IMBA_CK(launch_attn_combine(aa, w.ml, static_cast<const bf16*>(w.u), gated_bf, s));
      fused = true;
    } else if (!paged_attn || !launch_attn_page(aa, md.num_layers, md, pool.num_pages, static_cast<const bf16*>(w.u),
                                                gated_bf, w.recs, s, &e, &fused)) {
      if (md.dtype == IMBA_DTYPE_BF16 && !m->simt_attn) return IMBA_ERR_UNSUPPORTED;
      IMBA_CK(launch_attn_simt<T>(aa, s));
    } else if (e != cudaSuccess) {
      return IMBA_ERR_CUDA;
    }
    IMBA_CK(pm.mark(s));
    if (gate_bf16)
      IMBA_CK(launch_gate_bf16(reinterpret_cast<const bf16*>(w.attn), static_cast<const bf16*>(w.u), R, hdv,
                               static_cast<bf16*>(w.gated), s));
    else if (!fused)
      IMBA_CK(launch_gate<T>(w.attn, static_cast<const T*>(w.u), R, hdv, static_cast<T*>(w.gated), s));
    IMBA_CK(pm.mark(s));
    EpiResidual er{w.x, md.o_b[l], d};
    if (!gemm_tc_launch_out(m, l, R, static_cast<const T*>(w.gated), er, st.status, s, &e)) {
      if (tc_gemm) return IMBA_ERR_UNSUPPORTED;
      IMBA_CK(launch_gemm_simt<T, T, EpiResidual>(static_cast<const T*>(w.gated), hdv,
                                                  static_cast<const T*>(md.o_w[l]), hdv, R, d, hdv, er, s));
    } else if (e != cudaSuccess) {
      return IMBA_ERR_CUDA;
    }
    IMBA_CK(pm.mark(s));
  }
  const bool bf = md.dtype == IMBA_DTYPE_BF16;
  IMBA_CK(launch_final_ln<T>(w.x, R, d, md.final_norm_w, md.final_norm_b, w.xf32,
                             bf ? static_cast<T*>(w.xf3) : nullptr, s));
  IMBA_CK(pm.mark(s));
  if (st.hidden) IMBA_CK(cudaMemcpyAsync(st.hidden, w.x, (size_t)R * d * 4, cudaMemcpyDeviceToDevice, s));
  // The full policy projection runs only when the caller asks for all
  // logits; otherwise the legal entries are gathered in the value / legal
  // pass (exact fp32 dot products).
  float* logits = st.logits;
  if (st.logits) {
    if (!gemm_tc_launch_policy(m, R, static_cast<const T*>(w.xf3), EpiStore{logits, md.vocab}, st.status, s, &e)) {
      if (tc_gemm) return IMBA_ERR_UNSUPPORTED;
      IMBA_CK(launch_gemm_simt<float, float, EpiStore>(w.xf32, d, md.policy_w32, d, R, md.vocab, d,
                                                       EpiStore{logits, md.vocab}, s));
    } else if (e != cudaSuccess) {
      return IMBA_ERR_CUDA;
    }
  }
  IMBA_CK(pm.mark(s));
  if (md.has_value_head) {
    const int hd = d / 2;
    EpiBiasSilu eb{w.hval, md.value0_b, hd};
    // bf16: the first d columns of [x_hi | x_lo | x_hi]; fp32: the fp32 final-LN output.
    const T* xin = bf ? static_cast<const T*>(w.xf3) : reinterpret_cast<const T*>(w.xf32);
    const int lda = bf ? 3 * d : d;
    if (!gemm_tc_launch_value(m, R, xin, lda, eb, st.status, s, &e)) {
      if (tc_gemm) return IMBA_ERR_UNSUPPORTED;
      IMBA_CK(launch_gemm_simt<T, T, EpiBiasSilu>(xin, lda, static_cast<const T*>(md.value0_w), d, R, hd, d, eb, s));
    } else if (e != cudaSuccess) {
      return IMBA_ERR_CUDA;
    }
  }
  IMBA_CK(pm.mark(s));
  IMBA_CK(launch_value_legal(md, st, w.hval, logits, w.xf32, w.logits, s));
  IMBA_CK(pm.mark(s));
#undef IMBA_CK
  return IMBA_OK;
}

}  // namespace

Workspace carve_workspace(const imba_model* m, int32_t rows, void* base) {
  Workspace w;
  workspace_layout(m, rows, base, &w);
  return w;
}

}  // namespace imba

extern "C" {

int32_t imba_version(void) { return 1; }
int32_t imba_abi_size(int32_t which) {
  switch (which) {
    case 0: return (int32_t)sizeof(imba_model_desc);
    case 1: return (int32_t)sizeof(imba_step_desc);
    case 2: return (int32_t)sizeof(imba_pool_desc);
    default: return -1;
  }
}
int32_t imba_device_arch(void) { return 1000; }

imba_status_t imba_model_create(const imba_model_desc* desc, imba_model** out) {
  if (!out) return IMBA_ERR_ARG;
  *out = nullptr;
  const imba_status_t v = imba::validate_desc(desc);
  if (v != IMBA_OK) return v;
  // imba_step_noalloc's scratch array is placed on this device now, while the
  // caller can still allocate, not at the first allocation-free step.
  const imba_status_t na = imba::noalloc_prepare_device();
  if (na != IMBA_OK) return na;
  imba_model* m = new (std::nothrow) imba_model();
  if (!m) return IMBA_ERR_OOM;
  m->d = *desc;
  m->uvqk_n = 2 * desc->num_heads * (desc->linear_dim + desc->attention_dim);
  m->simt_gemm = (desc->flags & IMBA_FLAG_SIMT_GEMM) != 0;
  m->simt_attn = (desc->flags & IMBA_FLAG_SIMT_ATTN) != 0;
  m->simt_board = (desc->flags & IMBA_FLAG_SIMT_BOARD) != 0;
  if (desc->dtype == IMBA_DTYPE_BF16 && !imba::bf16_shape_supported(*desc, m->simt_gemm, m->simt_attn)) {
    delete m;
    return IMBA_ERR_UNSUPPORTED;
  }
  if (desc->dtype == IMBA_DTYPE_BF16 && !m->simt_board) {
    // Split bf16 copy of the board projection for the content GEMM.
    void* w3 = nullptr;
    if (cudaMalloc(&w3, (size_t)desc->model_dim * 3 * IMBA_BOARD_DIM * sizeof(imba::bf16)) != cudaSuccess) {
      cudaGetLastError();
      delete m;
      return IMBA_ERR_OOM;
    }
    if (imba::build_board_proj_split(m->d, static_cast<imba::bf16*>(w3), 0) != cudaSuccess ||
        cudaStreamSynchronize(0) != cudaSuccess) {
      cudaGetLastError();
      cudaFree(w3);
      delete m;
      return IMBA_ERR_CUDA;
    }
    m->board_proj3 = w3;
  }
  const imba_status_t t = imba::gemm_tc_prepare(m);
  if (t != IMBA_OK) {
    if (m->board_proj3) cudaFree(m->board_proj3);
    delete m;
    return t;
  }
  *out = m;
  return IMBA_OK;
}

void imba_model_destroy(imba_model* model) {
  if (!model) return;
  imba::gemm_tc_release(model);
  if (model->board_proj3) cudaFree(model->board_proj3);
  delete model;
}

size_t imba_step_workspace_bytes(const imba_model* model, int32_t max_rows) {
  if (!model || max_rows < 0) return 0;
  return imba::workspace_layout(model, max_rows, nullptr, nullptr);
}

int32_t imba_profile_event_count(const imba_model* model) {
  return model ? 2 + 5 * model->d.num_layers + 4 : 0;
}

static imba_status_t step_impl(const imba_model* model, const imba_step_desc* step, const imba_pool_desc* pool,
                               void* workspace, size_t workspace_bytes, void* stream, imba::PhaseMarks pm) {
  if (!model) return IMBA_ERR_ARG;
  const imba_status_t v = imba::validate_step(model, step, pool);
  if (v != IMBA_OK) return v;
  if (step->num_rows == 0) return IMBA_OK;
  const size_t need = imba::workspace_layout(model, step->num_rows, nullptr, nullptr);
  if (!workspace || workspace_bytes < need) return IMBA_ERR_OOM;
  if (reinterpret_cast<uintptr_t>(workspace) & 255) return IMBA_ERR_ARG;  // buffers are carved 256-aligned
  imba::Workspace w = imba::carve_workspace(model, step->num_rows, workspace);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (model->d.dtype == IMBA_DTYPE_BF16) return imba::run_step<imba::bf16>(model, *step, *pool, w, s, pm);
  return imba::run_step<float>(model, *step, *pool, w, s, pm);
}

imba_status_t imba_step(const imba_model* model, const imba_step_desc* step, const imba_pool_desc* pool,
                        void* workspace, size_t workspace_bytes, void* stream) {
  return step_impl(model, step, pool, workspace, workspace_bytes, stream, imba::PhaseMarks{});
}

imba_status_t imba_step_profiled(const imba_model* model, const imba_step_desc* step, const imba_pool_desc* pool,
                                 void* workspace, size_t workspace_bytes, void* stream, void* const* events,
                                 int32_t num_events) {
  if (!model || !events || num_events != imba_profile_event_count(model)) return IMBA_ERR_ARG;
  for (int i = 0; i < num_events; ++i)
    if (!events[i]) return IMBA_ERR_ARG;
  imba::PhaseMarks pm;
  pm.ev = events;
  pm.n = num_events;
  return step_impl(model, step, pool, workspace, workspace_bytes, stream, pm);
}

static imba_status_t kv_copy(const imba_model* model, const imba_pool_desc* pool, int32_t layer, int32_t n,
                             const int32_t* slots, void* dk, void* dv, int to_pool, int32_t* status, void* stream) {
  if (!model || !pool || !pool->base || pool->num_pages <= 0) return IMBA_ERR_ARG;
  if (layer < 0 || layer >= model->d.num_layers || n < 0) return IMBA_ERR_RANGE;
  if (n == 0) return IMBA_OK;
  if (!slots || !dk || !dv) return IMBA_ERR_ARG;
  const imba::PoolGeom g = model->geom(pool->num_pages);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  if (model->d.dtype == IMBA_DTYPE_BF16)
    e = imba::launch_kv_copy<imba::bf16>(g, static_cast<imba::bf16*>(pool->base), layer, n, slots,
                                         static_cast<imba::bf16*>(dk), static_cast<imba::bf16*>(dv), to_pool, status, s);
  else
    e = imba::launch_kv_copy<float>(g, static_cast<float*>(pool->base), layer, n, slots, static_cast<float*>(dk),
                                    static_cast<float*>(dv), to_pool, status, s);
  return e == cudaSuccess ? IMBA_OK : IMBA_ERR_CUDA;
}

imba_status_t imba_kv_scatter(const imba_model* model, const imba_pool_desc* pool, int32_t layer, int32_t n,
                              const int32_t* slots, const void* dense_k, const void* dense_v, int32_t* status,
                              void* stream) {
  return kv_copy(model, pool, layer, n, slots, const_cast<void*>(dense_k), const_cast<void*>(dense_v), 1, status,
                 stream);
}

imba_status_t imba_kv_scatter_indexed(const imba_model* model, const imba_pool_desc* pool, int32_t layer, int32_t n,
                                      const int32_t* slots, const int32_t* src_a, const int32_t* src_b,
                                      const void* src_k, const void* src_v, const int64_t* strides_k,
                                      const int64_t* strides_v, int32_t* status, void* stream) {
  if (!model || !pool || !pool->base || pool->num_pages <= 0) return IMBA_ERR_ARG;
  if (layer < 0 || layer >= model->d.num_layers || n < 0) return IMBA_ERR_RANGE;
  if (n == 0) return IMBA_OK;
  if (!slots || !src_a || !src_b || !src_k || !src_v || !strides_k || !strides_v) return IMBA_ERR_ARG;
  imba::KVStrides st;
  for (int i = 0; i < 4; ++i) {
    st.k[i] = strides_k[i];
    st.v[i] = strides_v[i];
  }
  const imba::PoolGeom g = model->geom(pool->num_pages);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  if (model->d.dtype == IMBA_DTYPE_BF16)
    e = imba::launch_kv_scatter_indexed<imba::bf16>(g, static_cast<imba::bf16*>(pool->base), layer, n, slots, src_a,
                                                    src_b, static_cast<const imba::bf16*>(src_k),
                                                    static_cast<const imba::bf16*>(src_v), st, status, s);
  else
    e = imba::launch_kv_scatter_indexed<float>(g, static_cast<float*>(pool->base), layer, n, slots, src_a, src_b,
                                               static_cast<const float*>(src_k), static_cast<const float*>(src_v), st,
                                               status, s);
  return e == cudaSuccess ? IMBA_OK : IMBA_ERR_CUDA;
}

imba_status_t imba_kv_gather(const imba_model* model, const imba_pool_desc* pool, int32_t layer, int32_t n,
                             const int32_t* slots, void* dense_k, void* dense_v, int32_t* status, void* stream) {
  return kv_copy(model, pool, layer, n, slots, dense_k, dense_v, 0, status, stream);
}

}  // extern "C"
