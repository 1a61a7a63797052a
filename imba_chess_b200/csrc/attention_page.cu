// Grouped paged-KV decode / prefill attention on the tensor cores (bf16
// models, d_qk = d_v = 64), with the attention-output LayerNorm and the u
// gate fused into its epilogue.
//
// Persistent: one CTA per SM (per head group when H > 8) pulls work items
// from a per-layer atomic counter.  An item is <= 32 query rows of one
// sequence group (a chunk; a 64-row chunk is two items) and HC heads (all of
// them when H <= 8).  Warp roles:
//   * the producer warp (index 2 HC) claims the next chunk, resolves its
//     rows' metadata (row ids, visible prefix, query positions, extra-key
//     offsets and the first extra tile's owners) into one of two item
//     buffers, then streams the group's visible KV pages: per 16-token page
//     two TMA tiled loads (K rows of the HC heads, then their V rows:
//     [HC x 16, 64] bf16 with the 128-byte swizzle) into a ring of stages
//     with one "full" (transaction bytes) and one "empty" (one arrive per
//     consumer warp) mbarrier per stage.  It runs ahead into the next item
//     while the consumers finish the current one, so the metadata and page
//     latency of an item overlaps the previous item's math.
//   * consumer warps 0 .. 2 HC - 1: warp w owns local head w / 2 and query
//     rows 16 (w % 2) .. +15 of the item.  The item's queries are staged
//     once in a swizzled shared tile (cp.async) and read per page with
//     ldmatrix, which keeps a warp's registers to its softmax state and O.
// Every page is read from HBM once per item and serves every sibling row and
// every head.  Per page a consumer warp computes S = Q K^T (mma.sync
// m16n8k16, fp32 accumulate), scales it, adds the relative-position bias
// ps_w[h, clamp(k - q + max - 1)], masks keys beyond each row's visible
// prefix, updates the fp32 online softmax in registers and accumulates
// O += P V.  The rows' extra keys (each row's suffix chain and the row
// itself: scattered arena slots, usually one to a few per row) are folded in
// per row afterwards: the four lanes that share a row split the 64-dim dot
// product (a quad reduction), update the row's online softmax and add p v to
// their O columns, reading K / V straight from the pool.
// Epilogue: O / l; when the CTA holds every head, O is staged in shared
// memory and after one barrier each warp takes whole rows: LayerNorm over the
// row's H dv outputs (no affine, eps 1e-6, warp reductions) times u, stored
// in bf16 for the output projection; otherwise fp32 O is stored and the gate
// runs as its own pass.
// Every wait is bounded; a timeout sets the status word and ends the CTA.
// Semantics: src/imba_chess/model/hstu_attention.py :64-76, :81-132,
// :134-148, :327-413 (attention), :185-190 (norm and gate).
#include <cuda_fp16.h>

#include <type_traits>

#include "kernels.cuh"
#include "tc_ptx.cuh"

namespace imba {
namespace {

constexpr int kHalfRows = 32;                                 // query rows per item
constexpr int kMaxHC = 8;                                     // heads per CTA
constexpr int kPageBytes = IMBA_PAGE_TOKENS * 128;            // 16 tokens x 64 bf16 of one head
constexpr size_t kSmemMax = 227 * 1024;                       // dynamic shared memory per CTA
constexpr int kMaxStages = 8;
constexpr int kMetaBytes = 8192;
constexpr int kMaxThreads = (2 * kMaxHC + 1) * 32;

// Item buffer (int32 words): header, then per-row arrays.
constexpr int kItN = 0;        // rows in the item (-1: no more items)
constexpr int kItNpg = 1;      // visible pages (ceil of the longest row's prefix / 16)
constexpr int kItRows = 8;     // [32] global row ids
constexpr int kItVis = 40;     // [32] visible prefix tokens
constexpr int kItQpos = 72;    // [32] query positions
constexpr int kItXoff = 104;   // [32] first extra of the row
constexpr int kItXcnt = 136;   // [32] extras of the row
constexpr int kItX0slot = 168; // [32] pool slot of the row's first extra (-1: none)
constexpr int kItX0pos = 200;  // [32] its position
constexpr int kItemInts = 232;

struct PageParams {
  AttnArgs a;
  int num_layers;
  int hc;         // heads per CTA
  int stages;
  const bf16* u;  // [R, H dv]
  bf16* gated;    // [R, H dv]: fused norm + gate output (nullptr: store fp32 O to a.out)
};

// Row stride (floats) of the staged O tile: 4 floats of padding keep the
// per-lane float2 writes of eight different rows in different banks.
__host__ __device__ constexpr int otile_ld(int hdv) { return hdv + 4; }
__host__ __device__ constexpr int otile_bytes(int hdv) { return kHalfRows * otile_ld(hdv) * 4; }

__device__ __forceinline__ int bias_index(int kpos, int qpos, int max_pos) {
  int idx = kpos - qpos + (max_pos - 1);
  idx = idx < 0 ? 0 : idx;
  return idx > 2 * max_pos - 2 ? 2 * max_pos - 2 : idx;
}

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

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t saddr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(saddr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], uint32_t saddr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(saddr));
}

// Byte offset of (token t < 16, 16-byte chunk j of its 128-byte row) in one
// head's 2 KB page block, 128-byte swizzle (blocks start 1024-aligned).
__device__ __forceinline__ uint32_t blk_off(int t, int j) { return (uint32_t)(t * 128 + ((j ^ (t & 7)) << 4)); }

__device__ __forceinline__ void bar_consumers(int nthreads) {
  asm volatile("bar.sync 1, %0;" ::"r"(nthreads) : "memory");
}
// Consumer-warp barrier that also ORs a predicate over the participants.
__device__ __forceinline__ bool bar_consumers_or(int nthreads, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, 1, %2, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}\n"
      : "=r"(r)
      : "r"((uint32_t)pred), "r"(nthreads)
      : "memory");
  return r != 0;
}

// Scores are kept in the log2 domain: s2 = (q.k) * scale * log2(e) +
// bias * log2(e), weights 2^(s2 - max), which is the same softmax as
// exp(s - max) with one multiply less per element.
constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ float exp2_approx(float x) {  // hardware ex2; 2^-inf = +0
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Relative-position bias lookups log2(e) * ps_w[h, idx]: from a per-CTA fp16
// copy of the CTA's rows (pre-multiplied by log2(e)) in shared memory, or
// from global memory when that copy does not fit (long position tables).
struct BiasShared {
  const __half* p;
  __device__ __forceinline__ float operator()(int idx) const { return __half2float(p[idx]); }
};
struct BiasGlobal {
  const float* p;
  __device__ __forceinline__ float operator()(int idx) const { return __ldg(p + idx) * kLog2e; }
};

// Running softmax state of one 16-row block for this lane's two rows
// (16 b + g and 16 b + g + 8, g = lane / 4).  l0 / l1 are this lane's
// partial row sums (its 4 key columns of every block); the quad's partials
// are added once, before normalisation.
struct RowState {
  float o[8][4];
  float m0, m1, l0, l1;
};

// Scale / bias / mask one 16-row x 16-key score block, update the online
// softmax of its rows and return P as the bf16 A fragment of P V.
// Keys are prefix tokens t0 .. t0 + 15; kFast: every key is visible to both
// rows and no bias index needs clamping (the common case of a full page).
// scale2 = scale * log2(e).
template <bool kFast, class Bias>
__device__ __forceinline__ void softmax16(RowState& rs, float (&sc)[2][4], uint32_t (&pa)[4], int t0, int vis0,
                                          int vis1, int qp0, int qp1, const Bias& psw, float scale2, int max_pos,
                                          int t) {
  float mx0 = -INFINITY, mx1 = -INFINITY;
  if (kFast) {
    const int b0 = t0 - qp0 + max_pos - 1 + 2 * t, b1 = t0 - qp1 + max_pos - 1 + 2 * t;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        sc[nt][e] = fmaf(sc[nt][e], scale2, psw(b0 + 8 * nt + e));
        sc[nt][2 + e] = fmaf(sc[nt][2 + e], scale2, psw(b1 + 8 * nt + e));
        mx0 = fmaxf(mx0, sc[nt][e]);
        mx1 = fmaxf(mx1, sc[nt][2 + e]);
      }
    }
  } else {
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int kpos = t0 + 8 * nt + 2 * t + e;
        const bool v0 = kpos < vis0, v1 = kpos < vis1;
        sc[nt][e] = v0 ? fmaf(sc[nt][e], scale2, psw(bias_index(kpos, qp0, max_pos))) : -INFINITY;
        sc[nt][2 + e] = v1 ? fmaf(sc[nt][2 + e], scale2, psw(bias_index(kpos, qp1, max_pos))) : -INFINITY;
        mx0 = fmaxf(mx0, sc[nt][e]);
        mx1 = fmaxf(mx1, sc[nt][2 + e]);
      }
    }
  }
  mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
  mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
  mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
  mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
  const float mn0 = fmaxf(rs.m0, mx0), mn1 = fmaxf(rs.m1, mx1);
  // A row with no visible key yet keeps max -inf; 0 stands in as the
  // exponent base so that every weight (and the old state's factor) is 0.
  const float ms0 = mn0 == -INFINITY ? 0.f : mn0, ms1 = mn1 == -INFINITY ? 0.f : mn1;
  const float c0 = exp2_approx(rs.m0 - ms0), c1 = exp2_approx(rs.m1 - ms1);
  float ps0 = 0.f, ps1 = 0.f;
#pragma unroll
  for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      sc[nt][e] = exp2_approx(sc[nt][e] - ms0);
      sc[nt][2 + e] = exp2_approx(sc[nt][2 + e] - ms1);
      ps0 += sc[nt][e];
      ps1 += sc[nt][2 + e];
    }
  }
  rs.l0 = fmaf(rs.l0, c0, ps0);
  rs.l1 = fmaf(rs.l1, c1, ps1);
  rs.m0 = mn0;
  rs.m1 = mn1;
  // Rescale O only when some row's running max moved (factor != 1).
  if (!__all_sync(0xffffffffu, c0 == 1.f && c1 == 1.f)) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      rs.o[j][0] *= c0;
      rs.o[j][1] *= c0;
      rs.o[j][2] *= c1;
      rs.o[j][3] *= c1;
    }
  }
  pa[0] = pack_bf16(sc[0][0], sc[0][1]);
  pa[1] = pack_bf16(sc[0][2], sc[0][3]);
  pa[2] = pack_bf16(sc[1][0], sc[1][1]);
  pa[3] = pack_bf16(sc[1][2], sc[1][3]);
}

// One 16-key block for the warp's 16 query rows: S = Q K^T (Q fragments
// read from the shared Q tile with ldmatrix), softmax16, O += P V.
template <bool kFast, class Bias>
__device__ __forceinline__ void step16(RowState& rs, uint32_t qb, uint32_t kb, uint32_t vb, int t0, int vis0,
                                       int vis1, int qp0, int qp1, const Bias& psw, float scale2, int max_pos,
                                       int lane) {
  const int t = lane & 3, r8 = lane & 7, mm = lane >> 3;
  float sc[2][4];
#pragma unroll
  for (int j = 0; j < 2; ++j) sc[j][0] = sc[j][1] = sc[j][2] = sc[j][3] = 0.f;
#pragma unroll
  for (int kc = 0; kc < 4; ++kc) {
    uint32_t qa[4], f[4];
    ldsm_x4(qa, qb + blk_off(lane & 15, 2 * kc + (lane >> 4)));
    ldsm_x4(f, kb + blk_off(r8 + 8 * (mm >> 1), 2 * kc + (mm & 1)));
    mma16816(sc[0], qa, f[0], f[1]);
    mma16816(sc[1], qa, f[2], f[3]);
  }
  uint32_t pa[4];
  softmax16<kFast, Bias>(rs, sc, pa, t0, vis0, vis1, qp0, qp1, psw, scale2, max_pos, t);
#pragma unroll
  for (int np = 0; np < 4; ++np) {
    uint32_t f[4];
    ldsm_x4_t(f, vb + blk_off(r8 + 8 * (mm & 1), 2 * np + (mm >> 1)));
    mma16816(rs.o[2 * np], pa, f[0], f[1]);
    mma16816(rs.o[2 * np + 1], pa, f[2], f[3]);
  }
}

// Fold one extra key (pool slot, position) into one row's online softmax.
// The row's four lanes (t = 0..3) each take 16 of the 64 dims of q . k and
// reduce across the quad; ol / oh: this lane's O columns 8 j + 2 t, +1 of the
// row.  active is uniform across the quad.
template <class Bias>
__device__ __forceinline__ void extra_key(float& m, float& l, float (&o)[8][4], int ci, bool active, uint32_t qrow,
                                          int qrow_sw, const bf16* kp, const bf16* vp, int kpos, int qpos,
                                          const Bias& psw, float scale2, int max_pos, int t) {
  float part = 0.f;
  uint4 kv[2] = {make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0)};
  if (active) {
    kv[0] = __ldg(reinterpret_cast<const uint4*>(kp + 16 * t));
    kv[1] = __ldg(reinterpret_cast<const uint4*>(kp + 16 * t + 8));
  }
  uint32_t vv[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) vv[j] = active ? __ldg(reinterpret_cast<const uint32_t*>(vp + 8 * j + 2 * t)) : 0u;
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    uint4 qv;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(qv.x), "=r"(qv.y), "=r"(qv.z), "=r"(qv.w)
                 : "r"(qrow + (uint32_t)(((2 * t + c) ^ qrow_sw) << 4)));
    const uint32_t qw[4] = {qv.x, qv.y, qv.z, qv.w};
    const uint32_t kw[4] = {kv[c].x, kv[c].y, kv[c].z, kv[c].w};
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const float2 qf = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&qw[w]));
      const float2 kf = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&kw[w]));
      part = fmaf(qf.x, kf.x, part);
      part = fmaf(qf.y, kf.y, part);
    }
  }
  part += __shfl_xor_sync(0xffffffffu, part, 1);
  part += __shfl_xor_sync(0xffffffffu, part, 2);
  if (!active) return;
  const float s2 = fmaf(part, scale2, psw(bias_index(kpos, qpos, max_pos)));
  const float mn = fmaxf(m, s2);
  const float c = exp2_approx(m - mn), p = exp2_approx(s2 - mn);
  m = mn;
  l = fmaf(l, c, t == 0 ? p : 0.f);  // the quad's partial sums: one lane counts the key
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float2 vf = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&vv[j]));
    o[j][2 * ci] = fmaf(o[j][2 * ci], c, p * vf.x);
    o[j][2 * ci + 1] = fmaf(o[j][2 * ci + 1], c, p * vf.y);
  }
}

template <bool kSmemBias>
__global__ void __launch_bounds__(kMaxThreads, 1)
    attn_page_kernel(const __grid_constant__ CUtensorMap kvmap, const PageParams prm) {
  const AttnArgs& a = prm.a;
  const imba_step_desc& st = a.st;
  const int HC = prm.hc, S = prm.stages;
  const int ncw = 2 * HC, nct = ncw * 32;  // consumer warps (head, row block) / threads
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int H = a.g.H;
  constexpr int D = 64;
  const int hdv = H * D;
  const int h0 = blockIdx.z * HC;
  const int stage_bytes = 2 * HC * kPageBytes;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = base;                                    // S stages: [K: HC x 2 KB][V: HC x 2 KB]
  uint8_t* qtile = ring + S * stage_bytes;                 // [HC][32 rows][128 B] queries, 128-byte swizzle
  const int bias_w = 2 * a.max_pos - 1;                    // ps_w row length
  // Fused epilogue: the item's O [32 rows][H dv + 4] fp32, staged.
  float* otile = reinterpret_cast<float*>(qtile + HC * kHalfRows * 128);
  const int otile_size = prm.gated ? otile_bytes(hdv) : 0;
  __half* bias_s = reinterpret_cast<__half*>(qtile + HC * kHalfRows * 128 + otile_size);  // [HC][bias_w] (kSmemBias)
  const int bias_bytes = kSmemBias ? (HC * bias_w * 2 + 15) / 16 * 16 : 0;
  int* items = reinterpret_cast<int*>(reinterpret_cast<uint8_t*>(bias_s) + bias_bytes);  // [2][kItemInts]
  int* misc = items + 2 * kItemInts;                       // [0] abort flag, [1] pad
  uint64_t* full = reinterpret_cast<uint64_t*>(misc + 2);           // 8-byte aligned: even int count precedes
  uint64_t* empty = full + kMaxStages;
  uint64_t* item_full = empty + kMaxStages;
  uint64_t* item_empty = item_full + 2;
  volatile int* abort_flag = misc;

  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], ncw);
    }
    for (int b = 0; b < 2; ++b) {
      tc::mbar_init(&item_full[b], 1);
      tc::mbar_init(&item_empty[b], ncw);
    }
    misc[0] = 0;
    tc::fence_mbar_init();
  }
  __syncthreads();

  if (warp == ncw) {
    // ---------------- producer ----------------
    const int64_t num_pages = a.g.num_slots / IMBA_PAGE_TOKENS;
    int* ctr = a.counters + blockIdx.z;
    int next_c = 0;
    if (lane == 0) next_c = atomicAdd(ctr, 1);
    int c = 0, half = 0, nhalves = 0, off0 = 0, n_chunk = 0, pg0 = 0, cap = 0;
    int it = 0, pc = 0;
    while (true) {
      if (++half >= nhalves) {  // claim the next non-empty chunk
        half = 0;
        nhalves = 0;
        while (true) {
          c = __shfl_sync(0xffffffffu, next_c, 0);
          if (c >= st.num_chunks) break;
          if (lane == 0) next_c = atomicAdd(ctr, 1);  // consumed on the next claim
          int v = 0;
          if (lane == 0) v = st.chunk_group[c];
          else if (lane == 1) v = st.chunk_row_off[c];
          else if (lane == 2) v = st.chunk_nrows[c];
          const int grp = __shfl_sync(0xffffffffu, v, 0);
          off0 = __shfl_sync(0xffffffffu, v, 1);
          n_chunk = __shfl_sync(0xffffffffu, v, 2);
          if (grp < 0 || grp >= st.num_groups || n_chunk < 0 || n_chunk > IMBA_CHUNK_ROWS || off0 < 0 ||
              off0 + n_chunk > st.num_rows) {
            if (lane == 0) report(st.status, IMBA_ERR_RANGE);
            continue;
          }
          int pv = 0;
          if (lane < 2) pv = st.group_page_off[grp + lane];
          pg0 = __shfl_sync(0xffffffffu, pv, 0);
          const int pg1 = __shfl_sync(0xffffffffu, pv, 1);
          if (pg0 < 0 || pg1 < pg0 || pg1 > st.num_group_pages) {
            if (lane == 0) report(st.status, IMBA_ERR_RANGE);
            pg0 = 0;
            cap = 0;
          } else {
            cap = (pg1 - pg0) * IMBA_PAGE_TOKENS;
          }
          nhalves = (n_chunk + kHalfRows - 1) / kHalfRows;
          if (nhalves > 0) break;
        }
      }
      const int ib = it & 1;
      int* item = items + ib * kItemInts;
      if (it >= 2) {  // the consumers release a buffer after the item's epilogue
        int ok = 1;
        if (lane == 0) ok = tc::mbar_wait_or_abort(&item_empty[ib], ((it >> 1) - 1) & 1, st.status, abort_flag);
        if (!__shfl_sync(0xffffffffu, ok, 0)) return;
      }
      if (c >= st.num_chunks) {
        if (lane == 0) {
          item[kItN] = -1;
          tc::mbar_arrive(&item_full[ib]);
        }
        return;
      }
      // Rows of this item, one lane per row.
      const int n = n_chunk - half * kHalfRows < kHalfRows ? n_chunk - half * kHalfRows : kHalfRows;
      const int off = off0 + half * kHalfRows;
      int r = -1, v = 0, qp = 0, e0 = 0, cnt = 0;
      if (lane < n) {
        r = st.row_perm[off + lane];
        if (r < 0 || r >= st.num_rows) {
          report(st.status, IMBA_ERR_RANGE);
          r = 0;
        }
        v = st.row_vis[r];
        qp = st.positions[r];
        e0 = st.row_extra_off[r];
        int e1 = st.row_extra_off[r + 1];
        if (v < 0 || v > cap) {
          report(st.status, IMBA_ERR_RANGE);
          v = v < 0 ? 0 : cap;
        }
        if (e0 < 0 || e1 < e0 || e1 > st.num_extra) {
          report(st.status, IMBA_ERR_RANGE);
          e1 = e0 = 0;
        }
        cnt = e1 - e0;
      }
      int vm = v;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) vm = max(vm, __shfl_xor_sync(0xffffffffu, vm, o));
      const int npg = (vm + IMBA_PAGE_TOKENS - 1) / IMBA_PAGE_TOKENS;
      item[kItRows + lane] = r;
      item[kItVis + lane] = v;
      item[kItQpos + lane] = qp;
      item[kItXoff + lane] = e0;
      item[kItXcnt + lane] = cnt;
      {
        int slot0 = -1, pos0 = 0;
        if (cnt > 0) {
          slot0 = st.extra_slot[e0];
          pos0 = st.extra_pos[e0];
          if (slot0 < 0 || slot0 >= a.g.num_slots) {
            report(st.status, IMBA_ERR_RANGE);
            slot0 = -1;
          }
        }
        item[kItX0slot + lane] = slot0;
        item[kItX0pos + lane] = pos0;
      }
      if (lane == 0) {
        item[kItN] = n;
        item[kItNpg] = npg;
      }
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&item_full[ib]);
      // The pages may hold KV written by the preceding projection kernel.
      pdl_wait();
      // Stream the visible pages through the ring.
      for (int b0 = 0; b0 < npg; b0 += 32) {
        int pg = 0;
        if (b0 + lane < npg) {
          pg = st.group_pages[pg0 + b0 + lane];
          if (pg < 0 || pg >= num_pages) {
            report(st.status, IMBA_ERR_RANGE);
            pg = 0;
          }
        }
        const int cnt2 = npg - b0 < 32 ? npg - b0 : 32;
        for (int k = 0; k < cnt2; ++k) {
          const int page = __shfl_sync(0xffffffffu, pg, k);
          int ok = 1;
          if (lane == 0) {
            const int s = pc % S;
            if (pc >= S) ok = tc::mbar_wait_or_abort(&empty[s], ((pc / S) - 1) & 1, st.status, abort_flag);
            if (ok) {
              uint8_t* dst = ring + s * stage_bytes;
              const int rowK = ((page * prm.num_layers + a.layer) * 2 * H + h0) * IMBA_PAGE_TOKENS;
              const int rowV = rowK + H * IMBA_PAGE_TOKENS;
              tc::mbar_arrive_expect_tx(&full[s], stage_bytes);
              tc::tma_load_2d(dst, &kvmap, &full[s], 0, rowK);
              tc::tma_load_2d(dst + HC * kPageBytes, &kvmap, &full[s], 0, rowV);
            }
          }
          if (!__shfl_sync(0xffffffffu, ok, 0)) return;
          ++pc;
        }
      }
      ++it;
    }
  }

  // ---------------- consumers ----------------
  const int hl = warp >> 1, rb = warp & 1, h = h0 + hl;
  const int g = lane >> 2, t = lane & 3;
  const int rl0 = 16 * rb + g, rl1 = rl0 + 8;
  if (kSmemBias) {  // fp16 copy of this CTA's ps_w rows (contiguous heads h0 .. h0 + HC - 1)
    const float* src = a.ps_w + (size_t)h0 * bias_w;
    const int total = HC * bias_w;
    // Each thread loads 8 values before converting and storing them, so the
    // loads of a round are in flight together.
    for (int base = tid * 8; base < total; base += nct * 8) {
      float v[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) v[k] = base + k < total ? __ldg(src + base + k) : 0.f;
#pragma unroll
      for (int k = 0; k < 8; ++k)
        if (base + k < total) bias_s[base + k] = __float2half_rn(v[k] * kLog2e);
    }
    // visible to every consumer warp after the first item's barrier
  }
  // The bias table (weights) and the producer's first item (host-written step
  // metadata) overlap the previous kernel; queries, u, the rows' own K / V
  // and the outputs are ordered after it.
  pdl_wait();
  pdl_trigger();
  using Bias = typename std::conditional<kSmemBias, BiasShared, BiasGlobal>::type;
  Bias psw;
  if constexpr (kSmemBias) psw.p = bias_s + (size_t)hl * bias_w;
  else psw.p = a.ps_w + (size_t)h * bias_w;
  const bf16* Pool = static_cast<const bf16*>(a.pool);
  const bf16* Q = static_cast<const bf16*>(a.q);
  const uint32_t ring_base = tc::smem_u32(ring), qtb = tc::smem_u32(qtile);
  const uint32_t qb = qtb + hl * (kHalfRows * 128) + rb * (16 * 128);  // this warp's 16 query rows

  int pc = 0;
  for (int it = 0;; ++it) {
    const int ib = it & 1;
    const int* item = items + ib * kItemInts;
    const bool ok_item =
        __all_sync(0xffffffffu, tc::mbar_wait_or_abort(&item_full[ib], (it >> 1) & 1, st.status, abort_flag));
    if (bar_consumers_or(nct, !ok_item)) {
      *abort_flag = 1;
      return;
    }
    const int n = item[kItN];
    if (n < 0) return;
    const int npg = item[kItNpg];
    // Query tile of the item: row r, head hh, 16-byte chunk c8 (rows past n are zero).
    for (int idx = tid; idx < kHalfRows * HC * 8; idx += nct) {
      const int c8 = idx & 7, rest = idx >> 3;
      const int hh = rest % HC, row = rest / HC;
      const uint32_t dst = qtb + hh * (kHalfRows * 128) + blk_off(row, c8);
      if (row < n) {
        const bf16* src = Q + (size_t)item[kItRows + row] * (H * D) + (h0 + hh) * D + 8 * c8;
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(dst), "l"(src) : "memory");
      } else {
        asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};\n" ::"r"(dst), "r"(0u) : "memory");
      }
    }
    asm volatile("cp.async.commit_group;\n" ::: "memory");
    // Bring the K / V lines of each row's first extra key (usually the row
    // itself, written by the preceding projection) into L1 while the pages
    // stream: lane t of a quad takes (row rl0 | rl1) x (K | V).
    {
      const int rl = (t & 1) ? rl1 : rl0;
      const int slot = rl < n ? item[kItX0slot + rl] : -1;
      if (slot >= 0) {
        const bf16* ln = Pool + ((t & 2) ? a.g.v_off(slot, a.layer, h) : a.g.k_off(slot, a.layer, h));
        asm volatile("prefetch.global.L1 [%0];" ::"l"(ln));
      }
    }
    const bool live = 16 * rb < n;
    // Rows past n mirror row 0 (never stored): they keep the fast path and
    // every bias index of a full page in range.
    const int vis0 = item[kItVis + (rl0 < n ? rl0 : 0)], vis1 = item[kItVis + (rl1 < n ? rl1 : 0)];
    const int qp0 = item[kItQpos + (rl0 < n ? rl0 : 0)], qp1 = item[kItQpos + (rl1 < n ? rl1 : 0)];
    const float scale2 = a.scale * kLog2e;
    // Pages [fast_lo, fast_hi) are fully visible to every row of the warp and
    // need no bias-index clamping (warp-uniform bounds).
    int fast_lo = max(max(qp0, qp1) - a.max_pos + 1, 0);
    int fast_hi = min(min(vis0, vis1), min(qp0, qp1) + a.max_pos);
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      fast_lo = max(fast_lo, __shfl_xor_sync(0xffffffffu, fast_lo, o));
      fast_hi = min(fast_hi, __shfl_xor_sync(0xffffffffu, fast_hi, o));
    }
    int wvis = max(vis0, vis1);  // pages past every row of this warp are skipped
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) wvis = max(wvis, __shfl_xor_sync(0xffffffffu, wvis, o));
    asm volatile("cp.async.wait_group 0;\n" ::: "memory");
    bar_consumers(nct);  // the query tile is complete
    RowState rs;
#pragma unroll
    for (int j = 0; j < 8; ++j) rs.o[j][0] = rs.o[j][1] = rs.o[j][2] = rs.o[j][3] = 0.f;
    rs.m0 = rs.m1 = -INFINITY;
    rs.l0 = rs.l1 = 0.f;

    bool aborted = false;
    for (int p = 0; p < npg; ++p, ++pc) {
      const int s = pc % S;
      const bool ok = __all_sync(0xffffffffu, tc::mbar_wait_or_abort(&full[s], (pc / S) & 1, st.status, abort_flag));
      if (!ok) {
        aborted = true;
        break;
      }
      if (live && p * IMBA_PAGE_TOKENS < wvis) {
        const uint32_t kb = ring_base + s * stage_bytes + hl * kPageBytes;
        const int t0 = p * IMBA_PAGE_TOKENS;
        if (t0 >= fast_lo && t0 + IMBA_PAGE_TOKENS <= fast_hi)
          step16<true, Bias>(rs, qb, kb, kb + HC * kPageBytes, t0, vis0, vis1, qp0, qp1, psw, scale2, a.max_pos,
                             lane);
        else
          step16<false, Bias>(rs, qb, kb, kb + HC * kPageBytes, t0, vis0, vis1, qp0, qp1, psw, scale2, a.max_pos,
                              lane);
      }
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&empty[s]);
    }
    // Every consumer warp reaches this barrier, aborted or not, so the
    // decision to stop is uniform and no warp waits at a later barrier.
    if (bar_consumers_or(nct, aborted)) {
      *abort_flag = 1;
      asm volatile("cp.async.wait_all;\n" ::: "memory");
      return;  // the status word already holds the timeout
    }
    // Extra keys, per row: the suffix chain and the row itself.
    {
      const int c0 = rl0 < n ? item[kItXcnt + rl0] : 0, c1 = rl1 < n ? item[kItXcnt + rl1] : 0;
      const int o0 = item[kItXoff + rl0], o1 = item[kItXoff + rl1];
      int emax = max(c0, c1);
#pragma unroll
      for (int o = 4; o < 32; o <<= 1) emax = max(emax, __shfl_xor_sync(0xffffffffu, emax, o));
      const uint32_t qr0 = qb + g * 128, qr1 = qb + (g + 8) * 128;  // rows rl0, rl1 of the query tile
      for (int e = 0; e < emax; ++e) {
#pragma unroll
        for (int ci = 0; ci < 2; ++ci) {
          const int cnt = ci ? c1 : c0;
          int slot = -1, kpos = 0;
          if (e == 0) {  // resolved (and range-checked) by the producer
            const int rl = ci ? rl1 : rl0;
            if (cnt > 0) {
              slot = item[kItX0slot + rl];
              kpos = item[kItX0pos + rl];
            }
          } else if (e < cnt) {
            const int xi = (ci ? o1 : o0) + e;
            slot = st.extra_slot[xi];
            kpos = st.extra_pos[xi];
            if (slot < 0 || slot >= a.g.num_slots) {
              report(st.status, IMBA_ERR_RANGE);
              slot = -1;
            }
          }
          const bool act = slot >= 0;
          const bf16* kp = Pool + (act ? a.g.k_off(slot, a.layer, h) : 0);
          const bf16* vp = Pool + (act ? a.g.v_off(slot, a.layer, h) : 0);
          if (ci == 0)
            extra_key(rs.m0, rs.l0, rs.o, 0, act, qr0, g & 7, kp, vp, kpos, qp0, psw, scale2, a.max_pos, t);
          else
            extra_key(rs.m1, rs.l1, rs.o, 1, act, qr1, (g + 8) & 7, kp, vp, kpos, qp1, psw, scale2, a.max_pos, t);
        }
      }
    }

    // ---- epilogue: this lane holds rows rl0 / rl1, columns 8 j + 2 t, +1 ----
    rs.l0 += __shfl_xor_sync(0xffffffffu, rs.l0, 1);  // the quad's partial row sums
    rs.l0 += __shfl_xor_sync(0xffffffffu, rs.l0, 2);
    rs.l1 += __shfl_xor_sync(0xffffffffu, rs.l1, 1);
    rs.l1 += __shfl_xor_sync(0xffffffffu, rs.l1, 2);
    const float i0 = rs.l0 > 0.f ? 1.0f / rs.l0 : 0.f, i1 = rs.l1 > 0.f ? 1.0f / rs.l1 : 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      rs.o[j][0] *= i0;
      rs.o[j][1] *= i0;
      rs.o[j][2] *= i1;
      rs.o[j][3] *= i1;
    }
    const int r0 = rl0 < n ? item[kItRows + rl0] : -1, r1 = rl1 < n ? item[kItRows + rl1] : -1;
    if (prm.gated == nullptr) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int col = h * D + 8 * j + 2 * t;
        if (r0 >= 0) *reinterpret_cast<float2*>(a.out + (size_t)r0 * hdv + col) = make_float2(rs.o[j][0], rs.o[j][1]);
        if (r1 >= 0) *reinterpret_cast<float2*>(a.out + (size_t)r1 * hdv + col) = make_float2(rs.o[j][2], rs.o[j][3]);
      }
    } else {
      // LayerNorm over the row's H dv outputs, then the gate by u: O goes to
      // the shared O tile, and after one barrier each warp normalises whole
      // rows (2 of the 32) with warp reductions; u and the gated output move
      // as coalesced 8-byte pieces.  The u loads are issued first.
      // Lane l owns columns 128 k + 4 l .. +3 (k < 4) of a row; warp w
      // normalises rows w, w + 2 HC, ... (two rows when HC = 8).
      const int ld = otile_ld(hdv);
      auto col_ok = [&](int k) { return 128 * k + 4 * lane < hdv; };
      uint2 uw[2][4];  // u of this warp's first two rows, loaded before the barrier
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int rr = warp + i * ncw;
        const int gr = rr < n ? item[kItRows + rr] : -1;
#pragma unroll
        for (int k = 0; k < 4; ++k)
          uw[i][k] = (gr >= 0 && col_ok(k))
                         ? __ldg(reinterpret_cast<const uint2*>(prm.u + (size_t)gr * hdv + 128 * k + 4 * lane))
                         : make_uint2(0u, 0u);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int col = hl * D + 8 * j + 2 * t;
        *reinterpret_cast<float2*>(otile + rl0 * ld + col) = make_float2(rs.o[j][0], rs.o[j][1]);
        *reinterpret_cast<float2*>(otile + rl1 * ld + col) = make_float2(rs.o[j][2], rs.o[j][3]);
      }
      bar_consumers(nct);
      for (int i = 0, rr = warp; rr < n; ++i, rr += ncw) {
        const int gr = item[kItRows + rr];
        uint2 ur[4];
#pragma unroll
        for (int k = 0; k < 4; ++k)
          ur[k] = i < 2 ? (i ? uw[1][k] : uw[0][k])
                        : (col_ok(k) ? __ldg(reinterpret_cast<const uint2*>(prm.u + (size_t)gr * hdv + 128 * k +
                                                                            4 * lane))
                                     : make_uint2(0u, 0u));
        float4 v[4];
        float sum = 0.f;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          v[k] = col_ok(k) ? *reinterpret_cast<const float4*>(otile + rr * ld + 128 * k + 4 * lane)
                           : make_float4(0.f, 0.f, 0.f, 0.f);
          sum += (v[k].x + v[k].y) + (v[k].z + v[k].w);
        }
        const float mu = warp_sum(sum) / (float)hdv;
        float sq = 0.f;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          if (col_ok(k))
            sq += (v[k].x - mu) * (v[k].x - mu) + (v[k].y - mu) * (v[k].y - mu) + (v[k].z - mu) * (v[k].z - mu) +
                  (v[k].w - mu) * (v[k].w - mu);
        }
        const float rsd = 1.0f / sqrtf(warp_sum(sq) / (float)hdv + 1e-6f);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          if (!col_ok(k)) continue;
          const float2 u01 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&ur[k].x));
          const float2 u23 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&ur[k].y));
          uint2 o;
          o.x = pack_bf16(u01.x * ((v[k].x - mu) * rsd), u01.y * ((v[k].y - mu) * rsd));
          o.y = pack_bf16(u23.x * ((v[k].z - mu) * rsd), u23.y * ((v[k].w - mu) * rsd));
          *reinterpret_cast<uint2*>(prm.gated + (size_t)gr * hdv + 128 * k + 4 * lane) = o;
        }
      }
    }
    __syncwarp();
    if (lane == 0) tc::mbar_arrive(&item_empty[ib]);  // this warp is done with the item buffer
  }
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

}  // namespace

// Returns false (nothing launched) when the model / pool cannot use this
// kernel.  *fused is set when the norm + gate was done in the epilogue (the
// caller then skips its gate pass).  a.counters[0 .. H / hc) must be zero.
bool launch_attn_page(const AttnArgs& a, int num_layers, const imba_model_desc& md, int64_t num_pages,
                      const bf16* u, bf16* gated, cudaStream_t s, cudaError_t* err, bool* fused) {
  *fused = false;
  if (md.dtype != IMBA_DTYPE_BF16 || md.attention_dim != 64 || md.linear_dim != 64) return false;
  const int H = md.num_heads;
  int hc = H < kMaxHC ? H : kMaxHC;
  while (H % hc) --hc;  // largest divisor of H up to 8
  if (H / hc > kCountersPerLayer || !a.counters) return false;
  const bool fuse = hc == H && gated != nullptr;
  if (a.st.num_chunks <= 0) {
    *err = cudaSuccess;
    *fused = fuse;
    return true;
  }
  // TMA view of the pool: 2D [num_pages * L * 2H * 16 rows, 64 columns] bf16;
  // one box = one page's 16 rows of hc consecutive heads.
  const uint64_t rows = (uint64_t)num_pages * num_layers * 2 * H * IMBA_PAGE_TOKENS;
  if (rows > (uint64_t)INT32_MAX) return false;
  EncodeTiledFn enc = encode_fn();
  if (!enc || (reinterpret_cast<uintptr_t>(a.pool) & 15)) return false;
  CUtensorMap map;
  const cuuint64_t dims[2] = {64, rows};
  const cuuint64_t strides[1] = {128};
  const cuuint32_t box[2] = {64, (cuuint32_t)(hc * IMBA_PAGE_TOKENS)};
  const cuuint32_t estr[2] = {1, 1};
  if (enc(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(a.pool), dims, strides, box, estr,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return false;
  // Shared memory: alignment slack, KV ring, query tile, optional fp16 bias
  // table, item buffers and barriers.  The bias table is
  // kept in shared memory when at least 3 ring stages still fit.
  const size_t stage_bytes = 2 * (size_t)hc * kPageBytes;
  const size_t fixed = 1024 + (size_t)hc * kHalfRows * 128 + (fuse ? (size_t)otile_bytes(H * 64) : 0) + kMetaBytes;
  const size_t bias_bytes = ((size_t)hc * (2 * md.max_pos - 1) * 2 + 15) / 16 * 16;
  const bool smem_bias = fixed + bias_bytes + 3 * stage_bytes <= kSmemMax;
  size_t stages = (kSmemMax - fixed - (smem_bias ? bias_bytes : 0)) / stage_bytes;
  stages = stages > kMaxStages ? kMaxStages : stages;
  if (stages < 2) return false;
  const size_t smem = fixed + (smem_bias ? bias_bytes : 0) + stages * stage_bytes;
  auto kern = smem_bias ? attn_page_kernel<true> : attn_page_kernel<false>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) {
    *err = e;
    return true;
  }
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  PageParams prm{a, num_layers, hc, (int)stages, u, fuse ? gated : nullptr};
  const int ctas = a.st.num_chunks < sms ? a.st.num_chunks : sms;
  dim3 grid(ctas, 1, H / hc);
  *err = launch_pdl(kern, grid, dim3((2 * hc + 1) * 32), smem, s, map, prm);
  *fused = fuse && *err == cudaSuccess;
  return true;
}

}  // namespace imba
