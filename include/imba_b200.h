/*
 * imba_b200.h - C ABI of the B200 (sm_100a) HSTU chess inference library.
 *
 * The library evaluates the HSTU chess model's one-token decode step and its
 * jagged prefix prefill against a paged, device-resident KV pool.  It
 * replaces the torch op sequences behind the reference's model decode API:
 *
 *   HSTUChessModel.forward(return_kv=True)   src/imba_chess/model/hstu_model.py:337-374
 *   HSTUChessModel.forward_decode            src/imba_chess/model/hstu_model.py:600-649
 *   HSTUChessModel.forward_decode_grouped    src/imba_chess/model/hstu_model.py:651-752
 *   SequentialTransductionUnitJagged.*       src/imba_chess/model/hstu_attention.py:81-424
 *   _KVArena append / gather_suffix          src/imba_chess/eval/actor_server.py:206-280
 *   _gather_legal_logits / _batched_value_stm src/imba_chess/eval/actor_server.py:168-203
 *   _log_softmax_f32                         src/imba_chess/eval/actor_worker.py:267-291
 *
 * Conventions
 *  - Every pointer inside a descriptor is a DEVICE pointer on the device that
 *    is current when the call is made, unless a field says otherwise.
 *  - Entry points never allocate device memory, never synchronise the host
 *    with the device and never trap.  Scratch space is a caller-provided
 *    workspace sized by imba_step_workspace_bytes().
 *  - Argument errors found on the host return IMBA_ERR_ARG / IMBA_ERR_RANGE
 *    before anything is launched.  Errors found on the device (an index out
 *    of range, a wait that ran out) are written to the optional device status
 *    word; the kernel skips the offending access and keeps going.  The caller
 *    reads the status after its own next synchronisation point.
 *  - One imba_model handle may be used from one host thread at a time; any
 *    number of handles may coexist.  The library keeps no hidden globals.
 */
#ifndef IMBA_B200_H_
#define IMBA_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define IMBA_API __attribute__((visibility("default")))
#else
#define IMBA_API
#endif

typedef int32_t imba_status_t;
#define IMBA_OK 0
#define IMBA_ERR_ARG 1          /* malformed descriptor (null pointer, bad size) */
#define IMBA_ERR_RANGE 2        /* an index outside its table or pool             */
#define IMBA_ERR_OOM 3          /* workspace smaller than required                */
#define IMBA_ERR_TIMEOUT 4      /* a bounded device-side wait ran out             */
#define IMBA_ERR_CUDA 5         /* a CUDA runtime call failed                     */
#define IMBA_ERR_UNSUPPORTED 6  /* shape not supported by the selected kernels    */

#define IMBA_DTYPE_F32 0        /* fp32 weights, activations and KV pool          */
#define IMBA_DTYPE_BF16 1       /* bf16 GEMM operands and KV pool, fp32 residual  */

/* imba_model_desc.flags: test hooks that replace one tensor-core component of
 * a bf16 handle by its fp32-accumulating SIMT kernel, so a test can compare
 * the two on identical inputs.  Production handles pass 0. */
#define IMBA_FLAG_SIMT_GEMM 1   /* projections, heads: SIMT GEMMs                 */
#define IMBA_FLAG_SIMT_ATTN 2   /* attention: SIMT kernel + separate gate pass    */
#define IMBA_FLAG_SIMT_BOARD 4  /* board encoder + content: fp32 SIMT kernel      */

#define IMBA_MAX_LAYERS 32
#define IMBA_PAGE_TOKENS 16     /* tokens per KV page                              */
#define IMBA_CHUNK_ROWS 64      /* max query rows in one attention work item      */
#define IMBA_BOARD_DIM 64
#define IMBA_NUM_SIDE_IDS 7     /* seq, turn, castle, ep, halfmove, fullmove, prev */

/* Model weights.  Every tensor keeps the reference's nn.Module layout
 * ([out, in] for linear layers) and is owned by the caller, which keeps it
 * alive for the lifetime of the handle.  "wdt" marks tensors stored in the
 * model dtype (fp32 or bf16); the rest are fp32. */
typedef struct imba_model_desc {
  int32_t model_dim;        /* d                                   */
  int32_t num_layers;       /* L  (<= IMBA_MAX_LAYERS)             */
  int32_t num_heads;        /* H                                   */
  int32_t attention_dim;    /* d_qk per head                       */
  int32_t linear_dim;       /* d_v per head                        */
  int32_t vocab;            /* move vocab (policy width)           */
  int32_t max_pos;          /* max_position_embeddings             */
  int32_t halfmove_vocab;
  int32_t fullmove_vocab;
  int32_t has_value_head;
  int32_t dtype;            /* IMBA_DTYPE_*                        */
  int32_t flags;            /* IMBA_FLAG_* (0 for normal use)      */

  /* content embedding (hstu_model.py:209-228, :275-335) */
  const float* piece_square;   /* [832, 64]                                */
  const float* board_params;   /* packed board-encoder blocks, see below   */
  const float* board_out_w;    /* [d, 64]                                  */
  const float* board_out_b;    /* [d]                                      */
  const float* emb_seq;        /* [2, d]                                   */
  const float* emb_turn;       /* [2, d]                                   */
  const float* emb_castle;     /* [16, d]                                  */
  const float* emb_ep;         /* [9, d]                                   */
  const float* emb_halfmove;   /* [halfmove_vocab, d]                      */
  const float* emb_fullmove;   /* [fullmove_vocab, d]                      */
  const float* emb_prev_move;  /* [vocab, d] (tied with the policy head)   */
  const float* emb_pos;        /* [max_pos, d]                             */

  /* STU layers (hstu_attention.py:30-49) */
  const void* uvqk_w[IMBA_MAX_LAYERS];  /* wdt [2H(d_v+d_qk), d], rows u|v|q|k */
  const void* o_w[IMBA_MAX_LAYERS];     /* wdt [d, H d_v]                      */
  const float* o_b[IMBA_MAX_LAYERS];    /* [d]                                 */
  const float* ps_w[IMBA_MAX_LAYERS];   /* [H, 2 max_pos - 1]                  */

  /* heads (hstu_model.py:245-260) */
  const float* final_norm_w;   /* [d] */
  const float* final_norm_b;   /* [d] */
  const void* policy_w;        /* fp32: [vocab, d]; bf16: [vocab, 3d] = [hi | hi | lo] where
                                  hi = bf16(w) and lo = bf16(w - hi), so that one K = 3d GEMM
                                  against [x_hi | x_lo | x_hi] gives x.w to ~16 mantissa bits */
  const float* policy_w32;     /* [vocab, d] fp32 copy (the exact-precision path) */
  const void* value0_w;        /* wdt [d/2, d]   (NULL when no value head) */
  const float* value0_b;       /* [d/2]                                    */
  const float* value2_w;       /* [3, d/2]                                 */
  const float* value2_b;       /* [3]                                      */
} imba_model_desc;

/* Packed board-encoder block parameters (fp32), per block b in {0, 1}:
 *   attn_norm.w[64] attn_norm.b[64] qkv.w[192*64] attn_out.w[64*64]
 *   mlp_norm.w[64] mlp_norm.b[64] mlp0.w[128*64] mlp0.b[128]
 *   mlp2.w[64*128] mlp2.b[64]
 * followed by final_norm.w[64] final_norm.b[64]
 * (hstu_model.py:118-179). */
#define IMBA_BOARD_BLOCK_FLOATS (64 + 64 + 192 * 64 + 64 * 64 + 64 + 64 + 128 * 64 + 128 + 64 * 128 + 64)
#define IMBA_BOARD_PARAM_FLOATS (2 * IMBA_BOARD_BLOCK_FLOATS + 128)

typedef struct imba_model imba_model;

/* Paged KV pool: num_pages pages; a page holds IMBA_PAGE_TOKENS tokens of
 * every layer, laid out [page][layer][ K: H x 16 x d_qk | V: H x 16 x d_v ]
 * in the model dtype.  A token's physical slot is page * 16 + offset. */
typedef struct imba_pool_desc {
  void* base;
  int64_t num_pages;
} imba_pool_desc;

/* One jagged step: R query rows, each a new token of some sequence group.
 * Decode, grouped decode, prefill and incremental prefill are all steps:
 *  - row r attends to the first row_vis[r] tokens of its group's page list
 *    (positions 0..row_vis[r]-1), then to its "extra" keys (explicit slots
 *    with explicit positions: a decode row's suffix chain and itself);
 *  - row r's own k/v are written to slot row_dst_slot[r] BEFORE attention,
 *    so a prefill row that sees its own slot through row_vis needs no extra;
 *  - the relative bias uses key position minus positions[r] (unclamped);
 *    the position embedding clamps positions[r] to max_pos - 1.
 * Attention work is given as chunks of <= IMBA_CHUNK_ROWS rows of one group:
 * chunk c covers row_perm[chunk_row_off[c] .. chunk_row_off[c] + chunk_nrows[c]).
 * A step has at most num_rows chunks (IMBA_ERR_ARG otherwise). */
typedef struct imba_step_desc {
  int32_t num_rows;
  int32_t num_groups;
  int32_t num_chunks;
  int32_t num_legal;             /* total legal ids (length of legal_ids)  */
  int32_t num_extra;             /* total extra keys (length of extra_*)   */
  int32_t num_group_pages;       /* length of group_pages                  */

  const uint8_t* piece_ids;      /* [R, 64] values 0..12                        */
  const int32_t* side_ids;       /* [R, 7] seq, turn, castle, ep, half, full, prev */
  const int32_t* positions;      /* [R]                                         */

  const int32_t* row_vis;        /* [R]                                         */
  const int32_t* row_extra_off;  /* [R + 1] CSR offsets into extra_*            */
  const int32_t* extra_slot;     /* physical slot of each extra key             */
  const int32_t* extra_pos;      /* absolute position of each extra key         */
  const int32_t* row_dst_slot;   /* [R]                                         */
  const int32_t* group_page_off; /* [G + 1] CSR offsets into group_pages        */
  const int32_t* group_pages;    /* page ids, in sequence order                 */
  const int32_t* chunk_group;    /* [C]                                         */
  const int32_t* chunk_row_off;  /* [C]                                         */
  const int32_t* chunk_nrows;    /* [C]                                         */
  const int32_t* row_perm;       /* [R] rows grouped by chunk                   */

  const int32_t* legal_off;      /* [R + 1] CSR offsets into legal_ids, or NULL */
  const int32_t* legal_ids;      /* move ids in each row's given order          */

  float* logits;                 /* [R, vocab] or NULL                          */
  float* value_logits;           /* [R, 3] or NULL                              */
  float* value_stm;              /* [R] p(win) - p(loss), or NULL               */
  float* legal_logits;           /* [num_legal] raw logits at legal ids, or NULL*/
  float* legal_logprob;          /* [num_legal] log-softmax over each row's ids */
  float* hidden;                 /* [R, d] final residual stream, or NULL       */
  int32_t* status;               /* device status word (IMBA_* code), or NULL   */
} imba_step_desc;

/* Library version and the compiled device architecture (e.g. 1000 for sm_100a). */
IMBA_API int32_t imba_version(void);
/* sizeof() of the descriptor structs as compiled into the library
 * (0: imba_model_desc, 1: imba_step_desc, 2: imba_pool_desc), so a binding
 * can refuse a library built against a different header. */
IMBA_API int32_t imba_abi_size(int32_t which);
IMBA_API int32_t imba_device_arch(void);

/* Validate a model description and build a handle on the current device.
 * bf16 handles encode their TMA descriptors here and keep one small device
 * copy of the board projection split into bf16 hi / lo parts ([d, 192]
 * bf16, freed by imba_model_destroy).  A bf16 handle runs only on the
 * tensor-core kernels (unless desc->flags selects a SIMT test hook): it needs
 * head dims 64 / 64, d and H x 64 multiples of 128 and 2 H x 128 a multiple
 * of 256; other shapes return IMBA_ERR_UNSUPPORTED (fp32 handles take any
 * shape within the limits above). */
IMBA_API imba_status_t imba_model_create(const imba_model_desc* desc, imba_model** out);
IMBA_API void imba_model_destroy(imba_model* model);

/* Bytes of workspace imba_step needs for up to max_rows rows. */
IMBA_API size_t imba_step_workspace_bytes(const imba_model* model, int32_t max_rows);

/* Run one jagged step: content embedding, L STU layers (writing every row's
 * k/v into the pool), heads, legal-id projection.  Enqueued on `stream`. */
IMBA_API imba_status_t imba_step(const imba_model* model, const imba_step_desc* step,
                        const imba_pool_desc* pool, void* workspace,
                        size_t workspace_bytes, void* stream);

/* Allocation-free step.  No counterpart in the reference: it exists for hosts
 * that may not allocate GPU memory at decode time (a runtime whose allocator
 * owns all device memory, or an engine driver with a fixed footprint) and so
 * cannot supply imba_step's workspace.  It runs imba_step on a scratch array
 * of IMBA_NOALLOC_SCRATCH_BYTES compiled into the library and calls no
 * allocator.  imba_model_create places that array on the handle's device (it
 * then stays there until the process exits), so the allocation-free calls
 * that follow need no set-up; the array's address is looked up on every call
 * (no address outlives a device reset).  Returns IMBA_ERR_OOM, launching
 * nothing, when imba_step_workspace_bytes(model, step->num_rows) exceeds that
 * size (about 335 rows at d512 / 8 layers).  All calls share the array and
 * it keeps the last call's contents (no step reads scratch it did not write
 * first): calls that overlap on the GPU race and must be serialised by the
 * caller. */
#define IMBA_NOALLOC_SCRATCH_BYTES (8u << 20)
IMBA_API imba_status_t imba_step_noalloc(const imba_model* model, const imba_step_desc* step,
                                         const imba_pool_desc* pool, void* stream);

/* Per-phase timing.  imba_step_profiled is imba_step that additionally
 * records caller-created CUDA events (cudaEvent_t handles) on `stream` at
 * every phase boundary, in this order:
 *   [0] start, [1] after the content embedding,
 *   per layer l: [2+5l] input LN, [3+5l] uvqk GEMM + KV append,
 *                [4+5l] attention, [5+5l] gate, [6+5l] output GEMM,
 *   then final LN, policy GEMM, value GEMM, value/legal kernel.
 * num_events must equal imba_profile_event_count(model). */
IMBA_API int32_t imba_profile_event_count(const imba_model* model);
IMBA_API imba_status_t imba_step_profiled(const imba_model* model, const imba_step_desc* step,
                                          const imba_pool_desc* pool, void* workspace,
                                          size_t workspace_bytes, void* stream,
                                          void* const* events, int32_t num_events);

/* Dense strided K / V rows of one layer into pool slots, in the model dtype,
 * without an intermediate copy: row r (< n) goes to slot slots[r]; its
 * element (head h, dim e) is read from
 *   src_k[src_a[r] * strides_k[0] + src_b[r] * strides_k[1] + h * strides_k[2] + e * strides_k[3]]
 * (strides in elements; src_v likewise).  With (src_a, src_b) = (group,
 * token) this stages the reference's padded [G, H, maxP, d] prefix stack
 * (hstu_model.py:651-752, merged_executors.py:187-196), with (row, column)
 * its [B, H, s, d] suffix tensors.  Slots outside the pool are skipped and
 * reported in the status word (IMBA_ERR_RANGE). */
IMBA_API imba_status_t imba_kv_scatter_indexed(const imba_model* model, const imba_pool_desc* pool, int32_t layer,
                                               int32_t n, const int32_t* slots, const int32_t* src_a,
                                               const int32_t* src_b, const void* src_k, const void* src_v,
                                               const int64_t* strides_k, const int64_t* strides_v, int32_t* status,
                                               void* stream);

/* Failure-path self-test.  Launches one CTA on `stream` that runs the
 * library's bounded device-side wait (the one every pipelined kernel uses,
 * 2 s in production) on an mbarrier nothing arrives at, with the given limit
 * (0 < limit_ns <= 10 s).  The wait runs out, the kernel writes
 * IMBA_ERR_TIMEOUT to the device status word `status` and returns, leaving
 * the context usable.  No counterpart in the reference (whose decode path has
 * no device-side waits); it lets a host test the device-timeout error path
 * without hanging a GPU. */
IMBA_API imba_status_t imba_selftest_wait_timeout(int64_t limit_ns, int32_t* status, void* stream);

/* KV page kernels for dense <-> paged conversion (the reference's dense
 * prefix/suffix tensors, hstu_model.py:651-752).  `dense_k` is [n, H, d_qk]
 * and `dense_v` is [n, H, d_v] for one layer, in the model dtype; `slots`
 * gives each row's physical slot. */
IMBA_API imba_status_t imba_kv_scatter(const imba_model* model, const imba_pool_desc* pool,
                              int32_t layer, int32_t n, const int32_t* slots,
                              const void* dense_k, const void* dense_v,
                              int32_t* status, void* stream);
IMBA_API imba_status_t imba_kv_gather(const imba_model* model, const imba_pool_desc* pool,
                             int32_t layer, int32_t n, const int32_t* slots,
                             void* dense_k, void* dense_v, int32_t* status,
                             void* stream);

#ifdef __cplusplus
}
#endif

#endif /* IMBA_B200_H_ */
