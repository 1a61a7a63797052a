// Grouped paged-KV decode attention on the tensor cores (bf16 models,
// d_qk = d_v = 64), with the attention-output LayerNorm and the u gate fused
// into its epilogue.  It also runs steps without extra keys that have few
// rows per group (root extensions); jagged prefills of whole documents run
// attention_prefill.cu.
//
// Work items.  An item is <= 32 query rows of one chunk (a 64-row chunk is
// two items) and HC heads (all of them when H <= 8).  Once per step the item
// pass (attn_items_kernel) resolves every item's metadata into one record of
// kAttnRecInts words: row ids, visible prefix lengths, query positions,
// extra-key offsets and counts, the first extra key's slot and position, and
// the group's first page ids.  Every layer's attention then fetches a record
// with one bulk copy instead of a chain of dependent global loads.
//
// The attention kernel is persistent: one CTA per SM (per head group when
// H > 8) pulls chunks from a per-layer atomic counter.  Warp roles, every
// hand-off an mbarrier or a named barrier:
//   * the producer warp (index 2 HC) claims a chunk (at once while the queue
//     is far from its end, then when the consumers near the end of the
//     previous item's pages), bulk-copies its record into one of four item
//     buffers and streams the item's visible KV pages: per 16-token page two TMA tiled
//     loads (K rows of the HC heads, then their V rows: [HC x 16, 64] bf16
//     with the 128-byte swizzle) into a ring of stages with one "full"
//     (transaction bytes) and one "empty" (one arrive per consumer warp)
//     mbarrier per stage.  It runs ahead into the next item while the
//     consumers finish the current one.
//   * consumer warps 0 .. 2 HC - 1: warp w owns local head w / 2 and query
//     rows 16 (w % 2) .. +15 of the item.  The queries sit in one of two
//     swizzled shared tiles: while an item's epilogue runs, the consumers
//     copy the next item's queries (cp.async) into the other tile, so an
//     item starts with its queries in place.  Per page a warp computes
//     S = Q K^T (mma.sync m16n8k16, fp32 accumulate; Q fragments by
//     ldmatrix), scales it, adds the relative-position bias
//     ps_w[h, clamp(k - q + max - 1)], masks keys beyond each row's visible
//     prefix, updates the fp32 online softmax in registers and accumulates
//     O += P V.  The rows' extra keys (each row's suffix chain and the row
//     itself: scattered arena slots, usually one to a few per row) are folded
//     in afterwards: the four lanes that share a row split the 64-dim dot
//     product (a quad reduction), update the row's online softmax and add
//     p v to their O columns, reading K / V straight from the pool.
// Every page is read from HBM once per item and serves every sibling row and
// every head.
// Epilogue: O / l.  With every head in the CTA, O (rounded to bf16, as the
// reference's bf16 attention output is) overwrites the warp's own query rows
// in the tile, and after one barrier each warp takes whole rows: LayerNorm
// over the row's H dv outputs (no affine, eps 1e-6, warp reductions) times u,
// stored in bf16 for the output projection.  With more than 8 heads fp32 O
// is stored and the gate runs as its own pass.
// Every wait is bounded; a timeout sets the status word and ends the CTA.
// Semantics: src/imba_chess/model/hstu_attention.py :64-76, :81-132,
// :134-148, :327-413 (attention), :185-190 (norm and gate).
#include <cuda_fp16.h>

#include <type_traits>

#include "attn_common.cuh"
#include "kernels.cuh"
#include "tc_ptx.cuh"

namespace imba {
namespace {

constexpr int kHalfRows = 32;                          // query rows per item
constexpr int kMaxHC = 8;                              // heads per CTA
constexpr int kPageBytes = IMBA_PAGE_TOKENS * 128;     // 16 tokens x 64 bf16 of one head
constexpr int kHeadTile = kHalfRows * 128;             // one head's 32 query / O rows (bytes)
constexpr size_t kSmemMax = 227 * 1024;                // dynamic shared memory per CTA
constexpr int kMaxStages = 8;
constexpr int kItemBufs = 4;
constexpr int kMaxThreads = (2 * kMaxHC + 1) * 32;

constexpr int kRows = kHalfRows;

struct PageParams {
  AttnArgs a;
  int num_layers;
  int hc;            // heads per CTA
  int stages;
  const bf16* u;     // [R, H dv]
  bf16* gated;       // [R, H dv]: fused norm + gate output (nullptr: store fp32 O to a.out)
  const int* recs;   // [2 C][kAttnRecInts]: record c = chunk c's first 32 rows, C + c its second
  float2* ml;        // [R, H] or null: the pages only; O / l, and (max, sum) per row and head,
                     // for attn_combine (extra keys, norm, gate)
};

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

// Byte offset of (row t, 16-byte chunk j of its 128-byte row) in a tile of
// 128-byte rows with the 128-byte swizzle (tiles start 1024-aligned): a
// page's 16 K or V rows of one head, or a head's 32 query / O rows.
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

// Relative-position bias lookups log2(e) * ps_w[h, idx]: from a per-CTA fp16
// copy of the CTA's rows (pre-multiplied by log2(e)) in shared memory, or
// from global memory when that copy does not fit (long position tables).
struct BiasShared {
  const __half* p;
  __device__ __forceinline__ float operator()(int idx) const { return __half2float(p[idx]); }
  // entries idx and idx + 1 (one 4-byte load when idx is even: rows start
  // 4-byte aligned)
  __device__ __forceinline__ float2 pair(int idx) const {
    if (idx & 1) return make_float2(__half2float(p[idx]), __half2float(p[idx + 1]));
    return __half22float2(*reinterpret_cast<const __half2*>(p + idx));
  }
};
struct BiasGlobal {
  const float* p;
  __device__ __forceinline__ float operator()(int idx) const { return __ldg(p + idx) * kLog2e; }
  __device__ __forceinline__ float2 pair(int idx) const {
    return make_float2(__ldg(p + idx) * kLog2e, __ldg(p + idx + 1) * kLog2e);
  }
};

// The online softmax keeps a reference max per row and rescales O and the
// row sums only when a score exceeds it by more than 2^kLazyLog2: weights
// are then at most 2^kLazyLog2 (exact in the fp32 sums and in bf16 P), and
// most pages skip the cross-lane max and the rescale.
constexpr float kLazyLog2 = 8.0f;

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
// rows and no bias index needs clamping (the common case of a full page);
// kUni (with kFast): the warp's rows share one query position, so the four
// bias values of this lane's key columns serve both rows.
// scale2 = scale * log2(e).
template <bool kFast, bool kUni, class Bias>
__device__ __forceinline__ void softmax16(RowState& rs, float (&sc)[2][4], uint32_t (&pa)[4], int t0, int vis0,
                                          int vis1, int qp0, int qp1, const Bias& psw, float scale2, int max_pos,
                                          int t) {
  if (kFast && kUni) {
    const int b0 = t0 - qp0 + max_pos - 1 + 2 * t;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      const float2 bp = psw.pair(b0 + 8 * nt);
      sc[nt][0] = fmaf(sc[nt][0], scale2, bp.x);
      sc[nt][1] = fmaf(sc[nt][1], scale2, bp.y);
      sc[nt][2] = fmaf(sc[nt][2], scale2, bp.x);
      sc[nt][3] = fmaf(sc[nt][3], scale2, bp.y);
    }
  } else if (kFast) {
    const int b0 = t0 - qp0 + max_pos - 1 + 2 * t, b1 = t0 - qp1 + max_pos - 1 + 2 * t;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        sc[nt][e] = fmaf(sc[nt][e], scale2, psw(b0 + 8 * nt + e));
        sc[nt][2 + e] = fmaf(sc[nt][2 + e], scale2, psw(b1 + 8 * nt + e));
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
      }
    }
  }
  float mx0 = fmaxf(fmaxf(sc[0][0], sc[0][1]), fmaxf(sc[1][0], sc[1][1]));
  float mx1 = fmaxf(fmaxf(sc[0][2], sc[0][3]), fmaxf(sc[1][2], sc[1][3]));
  if (__any_sync(0xffffffffu, mx0 > rs.m0 + kLazyLog2 || mx1 > rs.m1 + kLazyLog2)) {
    // New reference max (exact over the row's quad); O and the sums follow.
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float mn0 = fmaxf(rs.m0, mx0), mn1 = fmaxf(rs.m1, mx1);
    // A row with no visible key yet keeps max -inf; 0 stands in as the
    // exponent base so that the old state's factor is 0.
    const float c0 = exp2_approx(rs.m0 - (mn0 == -INFINITY ? 0.f : mn0));
    const float c1 = exp2_approx(rs.m1 - (mn1 == -INFINITY ? 0.f : mn1));
    rs.l0 *= c0;
    rs.l1 *= c1;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      rs.o[j][0] *= c0;
      rs.o[j][1] *= c0;
      rs.o[j][2] *= c1;
      rs.o[j][3] *= c1;
    }
    rs.m0 = mn0;
    rs.m1 = mn1;
  }
  const float ms0 = rs.m0 == -INFINITY ? 0.f : rs.m0, ms1 = rs.m1 == -INFINITY ? 0.f : rs.m1;
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
  rs.l0 += ps0;
  rs.l1 += ps1;
  pa[0] = pack_bf16(sc[0][0], sc[0][1]);
  pa[1] = pack_bf16(sc[0][2], sc[0][3]);
  pa[2] = pack_bf16(sc[1][0], sc[1][1]);
  pa[3] = pack_bf16(sc[1][2], sc[1][3]);
}

// One 16-key block for the warp's 16 query rows: S = Q K^T (Q fragments
// read from the shared Q tile with ldmatrix), softmax16, O += P V.
template <bool kFast, bool kUni, class Bias>
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
  softmax16<kFast, kUni, Bias>(rs, sc, pa, t0, vis0, vis1, qp0, qp1, psw, scale2, max_pos, t);
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

// ---------------------------------------------------------------------------
// Item pass: one warp per record.  Record k < C: chunk k's rows 0..31;
// record C + k: its rows 32..63 (n = 0 when the chunk has <= 32 rows).
// Every index is range-checked here (IMBA_ERR_RANGE, clamped), so the
// attention kernel trusts the records.
__global__ void __launch_bounds__(128) attn_items_kernel(const imba_step_desc st, const PoolGeom g, int* recs) {
  const int lane = threadIdx.x & 31;
  const int k = blockIdx.x * 4 + (threadIdx.x >> 5);
  const int C = st.num_chunks;
  pdl_wait();
  pdl_trigger();
  if (k >= 2 * C) return;
  const int c = k < C ? k : k - C, half = k < C ? 0 : 1;
  int* rec = recs + (size_t)k * kAttnRecInts;
  int v0 = 0;
  if (lane == 0) v0 = st.chunk_group[c];
  else if (lane == 1) v0 = st.chunk_row_off[c];
  else if (lane == 2) v0 = st.chunk_nrows[c];
  const int grp = __shfl_sync(0xffffffffu, v0, 0);
  const int off0 = __shfl_sync(0xffffffffu, v0, 1);
  int n_chunk = __shfl_sync(0xffffffffu, v0, 2);
  int pg0 = 0, cap = 0;
  if (grp < 0 || grp >= st.num_groups || n_chunk < 0 || n_chunk > IMBA_CHUNK_ROWS || off0 < 0 ||
      off0 + n_chunk > st.num_rows) {
    if (lane == 0) report(st.status, IMBA_ERR_RANGE);
    n_chunk = 0;
  } else {
    int pv = 0;
    if (lane < 2) pv = st.group_page_off[grp + lane];
    pg0 = __shfl_sync(0xffffffffu, pv, 0);
    const int pg1 = __shfl_sync(0xffffffffu, pv, 1);
    if (pg0 < 0 || pg1 < pg0 || pg1 > st.num_group_pages) {
      if (lane == 0) report(st.status, IMBA_ERR_RANGE);
      pg0 = 0;
    } else {
      cap = (pg1 - pg0) * IMBA_PAGE_TOKENS;
    }
  }
  int n = n_chunk - half * kRows;
  n = n < 0 ? 0 : (n > kRows ? kRows : n);
  const int off = off0 + half * kRows;
  int r = -1, v = 0, qp = 0, e0 = 0, cnt = 0, slot0 = -1, pos0 = 0;
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
    if (cnt > 0) {
      slot0 = st.extra_slot[e0];
      pos0 = st.extra_pos[e0];
      if (slot0 < 0 || slot0 >= g.num_slots) {
        report(st.status, IMBA_ERR_RANGE);
        slot0 = -1;
      }
    }
  }
  int vm = v;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) vm = max(vm, __shfl_xor_sync(0xffffffffu, vm, o));
  const int npg = (vm + IMBA_PAGE_TOKENS - 1) / IMBA_PAGE_TOKENS;
  const int64_t num_pages = g.num_slots / IMBA_PAGE_TOKENS;
  rec[kRecRows + lane] = r;
  rec[kRecVis + lane] = v;
  rec[kRecQpos + lane] = qp;
  rec[kRecXoff + lane] = e0;
  rec[kRecXcnt + lane] = cnt;
  rec[kRecX0slot + lane] = slot0;
  rec[kRecX0pos + lane] = pos0;
  for (int p = lane; p < kRecMaxPages; p += 32) {
    int pg = 0;
    if (p < npg) {
      pg = st.group_pages[pg0 + p];
      if (pg < 0 || pg >= num_pages) {
        report(st.status, IMBA_ERR_RANGE);
        pg = 0;
      }
    }
    rec[kRecPages + p] = pg;
  }
  const int r0 = __shfl_sync(0xffffffffu, r, 0);
  const bool contig = __all_sync(0xffffffffu, lane >= n || r == r0 + lane);
  if (lane < 8) {
    int h = 0;
    if (lane == kRecN) h = n;
    else if (lane == kRecNpg) h = npg;
    else if (lane == kRecPg0) h = pg0;
    else if (lane == kRecHalves) h = (n_chunk + kRows - 1) / kRows;
    else if (lane == kRecContig) h = contig ? 1 : 0;
    rec[lane] = h;
  }
}

#ifndef IMBA_CLAIM_EARLY
#define IMBA_CLAIM_EARLY 2
#endif
#ifndef IMBA_CLAIM_LEAD
#define IMBA_CLAIM_LEAD(n) ((n) <= 8 ? 3 : ((n) <= 16 ? 2 : 0))
#endif
// Pages before the end of an item at which its CTA claims the next chunk,
// by the item's row count.
__device__ __forceinline__ int claim_lead(int n) { return IMBA_CLAIM_LEAD(n); }

template <bool kSmemBias>
__global__ void __launch_bounds__(kMaxThreads, 1)
    attn_page_kernel(const __grid_constant__ CUtensorMap kvmap, const PageParams prm) {
  const AttnArgs& a = prm.a;
  const imba_step_desc& st = a.st;
  const int HC = prm.hc, S = prm.stages;
  const bool fused = prm.gated != nullptr;
  const int ncw = 2 * HC, nct = ncw * 32;  // consumer warps (head, row block) / threads
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int H = a.g.H;
  constexpr int D = 64;
  const int hdv = H * D;
  const int h0 = blockIdx.z * HC;
  const int stage_bytes = 2 * HC * kPageBytes;
  const int q_bytes = HC * kHeadTile;  // one query tile: [HC][32 rows][128 B]

  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = base;                                  // S stages: [K: HC x 2 KB][V: HC x 2 KB]
  uint8_t* qtile = ring + S * stage_bytes;               // [2] query tiles, 128-byte swizzle
  const int bias_w = 2 * a.max_pos - 1;                  // ps_w row length (odd)
  const int bias_ld = bias_w + 1;                        // its row stride in shared memory: even, so that
                                                         // pairs at even indices are 4-byte aligned
  __half* bias_s = reinterpret_cast<__half*>(qtile + 2 * q_bytes);  // [HC][bias_ld] (kSmemBias)
  const int bias_bytes = kSmemBias ? (HC * bias_ld * 2 + 15) / 16 * 16 : 0;
  int* items = reinterpret_cast<int*>(reinterpret_cast<uint8_t*>(bias_s) + bias_bytes);  // [kItemBufs][rec]
  int* misc = items + kItemBufs * kAttnRecInts;          // [0] abort flag, [1] pad
  uint64_t* full = reinterpret_cast<uint64_t*>(misc + 2);  // 8-byte aligned: even int count precedes
  uint64_t* empty = full + kMaxStages;
  uint64_t* item_full = empty + kMaxStages;
  uint64_t* item_empty = item_full + kItemBufs;
  volatile int* abort_flag = misc;

  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], ncw);
    }
    for (int b = 0; b < kItemBufs; ++b) {
      tc::mbar_init(&item_full[b], 1);
      tc::mbar_init(&item_empty[b], ncw);
    }
    misc[0] = 0;
    tc::fence_mbar_init();
  }
  __syncthreads();

  if (warp == ncw) {
    // ---------------- producer ----------------
    // Its j-th item goes to buffer j % kItemBufs.
    const int64_t num_pages = a.g.num_slots / IMBA_PAGE_TOKENS;
    const int C = st.num_chunks;
    int* ctr = a.counters + blockIdx.z;
    // Every kernel of a step waits for its predecessor before it lets its
    // dependents launch, so once this CTA runs, every kernel before the
    // preceding one has completed: the item pass's records and the zeroed
    // counters are readable now.  The pages hold KV of the preceding
    // projection: the first page waits for it.
    bool waited = false;
    auto claim = [&]() {
      int c = 0;
      if (lane == 0) c = atomicAdd(ctr, 1);
      return __shfl_sync(0xffffffffu, c, 0);
    };
    // lane 0: buffer of item j free again (item j - kItemBufs released by the consumers)
    auto buffer_free = [&](int j) -> bool {
      return j < kItemBufs ||
             tc::mbar_wait_park_or_abort(&item_empty[j % kItemBufs], ((j / kItemBufs) - 1) & 1, st.status, abort_flag);
    };
    auto load_record = [&](int j, int rec) {  // lane 0
      const int b = j % kItemBufs;
      tc::mbar_arrive_expect_tx(&item_full[b], kRecBytes);
      tc::bulk_load(items + b * kAttnRecInts, prm.recs + (size_t)rec * kAttnRecInts, kRecBytes, &item_full[b]);
    };
    auto put_end = [&](int j) {  // lane 0: no more items
      const int b = j % kItemBufs;
      items[b * kAttnRecInts + kRecN] = -1;
      tc::mbar_arrive(&item_full[b]);
    };
    int c = claim();
    if (c >= C) {
      if (lane == 0) put_end(0);
      return;
    }
    if (lane == 0) load_record(0, c);
    int j = 0, pc = 0, half = 0;
    while (true) {
      const int b = j % kItemBufs;
      int ok = 1;
      if (lane == 0) ok = tc::mbar_wait_park_or_abort(&item_full[b], (j / kItemBufs) & 1, st.status, abort_flag);
      if (!__shfl_sync(0xffffffffu, ok, 0)) return;
      const int* item = items + b * kAttnRecInts;
      const int npg = item[kRecNpg], pg0 = item[kRecPg0], nhalves = item[kRecHalves];
      if (!waited) {
        pdl_wait();
        waited = true;
      }
      // Stream the visible pages through the ring.
      for (int b0 = 0; b0 < npg; b0 += 32) {
        int pg = 0;
        if (b0 + lane < npg) {
          if (b0 + lane < kRecMaxPages) {
            pg = item[kRecPages + b0 + lane];
          } else {
            pg = st.group_pages[pg0 + b0 + lane];
            if (pg < 0 || pg >= num_pages) {
              report(st.status, IMBA_ERR_RANGE);
              pg = 0;
            }
          }
        }
        const int cnt2 = npg - b0 < 32 ? npg - b0 : 32;
        for (int k = 0; k < cnt2; ++k) {
          const int page = __shfl_sync(0xffffffffu, pg, k);
          int ok2 = 1;
          if (lane == 0) {
            const int s = pc % S;
            if (pc >= S) ok2 = tc::mbar_wait_park_or_abort(&empty[s], ((pc / S) - 1) & 1, st.status, abort_flag);
            if (ok2) {
              uint8_t* dst = ring + s * stage_bytes;
              const int rowK = ((page * prm.num_layers + a.layer) * 2 * H + h0) * IMBA_PAGE_TOKENS;
              const int rowV = rowK + H * IMBA_PAGE_TOKENS;
              tc::mbar_arrive_expect_tx(&full[s], stage_bytes);
              tc::tma_load_2d(dst, &kvmap, &full[s], 0, rowK);
              tc::tma_load_2d(dst + HC * kPageBytes, &kvmap, &full[s], 0, rowV);
            }
          }
          if (!__shfl_sync(0xffffffffu, ok2, 0)) return;
          ++pc;
        }
      }
      // The next chunk is claimed when the consumers release this item's
      // page claim_lead(n) from its end: early enough that the next item's
      // record and first pages arrive before the consumers finish this one
      // (a small item has little work after its pages), late enough that a
      // CTA which stays busy for a while does not take work that another CTA
      // would start sooner from the longest-first queue.  Page q's release is
      // the (q / S)-th phase of its stage's empty barrier; while page q + S
      // is not issued (lead < S) that barrier is at most one phase past it.
      // A lead of npg or S or more claims at once (page q, if any, was
      // released before page q + S was issued).
      // While more than IMBA_CLAIM_EARLY chunks per CTA remain, the tail is far
      // off and the claim goes out at once.
      const int lead = C - c > IMBA_CLAIM_EARLY * (int)gridDim.x ? S : claim_lead(item[kRecN]);
      ok = 1;
      if (lane == 0 && lead < npg && lead < S) {
        const int q = pc - 1 - lead;
        ok = tc::mbar_wait_park_or_abort(&empty[q % S], (q / S) & 1, st.status, abort_flag);
      }
      if (!__shfl_sync(0xffffffffu, ok, 0)) return;
      int next = -1, next_half = 0;
      if (half == 0 && nhalves > 1) {
        next = C + c;
        next_half = 1;
      } else {
        c = claim();
        if (c < C) next = c;
      }
      ok = 1;
      if (lane == 0) {
        ok = buffer_free(j + 1);
        if (ok) {
          if (next >= 0) load_record(j + 1, next);
          else put_end(j + 1);
        }
      }
      if (!__shfl_sync(0xffffffffu, ok, 0)) return;
      ++j;
      half = next_half;
      if (next < 0) return;  // item j is the end marker
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
    for (int b = tid * 8; b < total; b += nct * 8) {
      float v[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) v[k] = b + k < total ? __ldg(src + b + k) : 0.f;
#pragma unroll
      for (int k = 0; k < 8; ++k)
        if (b + k < total) bias_s[(b + k) / bias_w * bias_ld + (b + k) % bias_w] = __float2half_rn(v[k] * kLog2e);
    }
    // visible to every consumer warp after the first item's barrier
  }
  // The bias table (weights) overlaps the previous kernel; queries, u, the
  // rows' own K / V and the outputs are ordered after it.
  pdl_wait();
  pdl_trigger();
  using Bias = typename std::conditional<kSmemBias, BiasShared, BiasGlobal>::type;
  Bias psw;
  if constexpr (kSmemBias) psw.p = bias_s + (size_t)hl * bias_ld;
  else psw.p = a.ps_w + (size_t)h * bias_w;
  const bf16* Pool = static_cast<const bf16*>(a.pool);
  const bf16* Q = static_cast<const bf16*>(a.q);
  const uint32_t ring_base = tc::smem_u32(ring), qtb = tc::smem_u32(qtile);
  const float scale2 = a.scale * kLog2e;

  // Queries of an item (record rec, n rows) into query tile `tile`: row r,
  // head hh, 16-byte chunk c8; rows past n are zero-filled by the copy
  // itself (source size 0).  Consecutive threads read consecutive chunks of
  // a row.
  auto copy_queries = [&](const int* rec, int n, int tile) {
    const uint32_t dst0 = qtb + tile * q_bytes;
    for (int idx = tid; idx < kHalfRows * HC * 8; idx += nct) {
      const int c8 = idx & 7, rest = idx >> 3;
      const int hh = rest % HC, row = rest / HC;
      const bool live = row < n;
      const bf16* src = Q + (live ? (size_t)rec[kRecRows + row] * (H * D) + (h0 + hh) * D + 8 * c8 : 0);
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst0 + hh * kHeadTile + blk_off(row, c8)),
                   "l"(src), "r"(live ? 16u : 0u)
                   : "memory");
    }
    asm volatile("cp.async.commit_group;\n" ::: "memory");
  };

  // The first item's record and queries.
  bool ok_next = __all_sync(0xffffffffu, tc::mbar_wait_park_or_abort(&item_full[0], 0, st.status, abort_flag));
  if (ok_next && items[kRecN] > 0) copy_queries(items, items[kRecN], 0);
  int pc = 0;
  for (int j = 0;; ++j) {
    const int b = j % kItemBufs, tile = j & 1;
    const int* item = items + b * kAttnRecInts;
    asm volatile("cp.async.wait_group 0;\n" ::: "memory");
    // The item's queries (and, at j = 0, the bias table) are visible to every
    // consumer warp past this barrier; a failed record wait anywhere stops all.
    if (bar_consumers_or(nct, !ok_next)) {
      *abort_flag = 1;
      return;
    }
    const int n = item[kRecN];
    if (n < 0) return;
    const int npg = item[kRecNpg];
    const uint32_t qb = qtb + tile * q_bytes + hl * kHeadTile + rb * (16 * 128);  // this warp's 16 query rows
    // Bring the K / V lines of each row's first extra key (usually the row
    // itself, written by the preceding projection) into L1 while the pages
    // stream: lane t of a quad takes (row rl0 | rl1) x (K | V).
    {
      const int rl = (t & 1) ? rl1 : rl0;
      const int slot = rl < n ? item[kRecX0slot + rl] : -1;
      if (slot >= 0) {
        const bf16* ln = Pool + ((t & 2) ? a.g.v_off(slot, a.layer, h) : a.g.k_off(slot, a.layer, h));
        asm volatile("prefetch.global.L1 [%0];" ::"l"(ln));
      }
    }
    const bool live = 16 * rb < n;
    // Rows past n mirror row 0 (never stored): they keep the fast path and
    // every bias index of a full page in range.
    const int vis0 = item[kRecVis + (rl0 < n ? rl0 : 0)], vis1 = item[kRecVis + (rl1 < n ? rl1 : 0)];
    const int qp0 = item[kRecQpos + (rl0 < n ? rl0 : 0)], qp1 = item[kRecQpos + (rl1 < n ? rl1 : 0)];
    // Pages [fast_lo, fast_hi) are fully visible to every row of the warp and
    // need no bias-index clamping (warp-uniform bounds).
    int fast_lo = max(max(qp0, qp1) - a.max_pos + 1, 0);
    int fast_hi = min(min(vis0, vis1), min(qp0, qp1) + a.max_pos);
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      fast_lo = max(fast_lo, __shfl_xor_sync(0xffffffffu, fast_lo, o));
      fast_hi = min(fast_hi, __shfl_xor_sync(0xffffffffu, fast_hi, o));
    }
    // The warp's rows share one query position (siblings of one parent).
    const int qp_lane0 = __shfl_sync(0xffffffffu, qp0, 0);  // every lane takes part in the shuffle
    const bool uni = __all_sync(0xffffffffu, qp0 == qp1 && qp0 == qp_lane0);
    int wvis = max(vis0, vis1);  // pages past every row of this warp are skipped
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) wvis = max(wvis, __shfl_xor_sync(0xffffffffu, wvis, o));
    RowState rs;
#pragma unroll
    for (int q = 0; q < 8; ++q) rs.o[q][0] = rs.o[q][1] = rs.o[q][2] = rs.o[q][3] = 0.f;
    rs.m0 = rs.m1 = -INFINITY;
    rs.l0 = rs.l1 = 0.f;

    bool aborted = false;
    for (int p = 0; p < npg; ++p, ++pc) {
      const int s = pc % S;
      const bool ok = __all_sync(0xffffffffu, tc::mbar_wait_park_or_abort(&full[s], (pc / S) & 1, st.status, abort_flag));
      if (!ok) {
        aborted = true;
        break;
      }
      if (live && p * IMBA_PAGE_TOKENS < wvis) {
        const uint32_t kb = ring_base + s * stage_bytes + hl * kPageBytes;
        const int t0 = p * IMBA_PAGE_TOKENS;
        if (t0 >= fast_lo && t0 + IMBA_PAGE_TOKENS <= fast_hi) {
          if (uni)
            step16<true, true, Bias>(rs, qb, kb, kb + HC * kPageBytes, t0, vis0, vis1, qp0, qp1, psw, scale2,
                                     a.max_pos, lane);
          else
            step16<true, false, Bias>(rs, qb, kb, kb + HC * kPageBytes, t0, vis0, vis1, qp0, qp1, psw, scale2,
                                      a.max_pos, lane);
        } else {
          step16<false, false, Bias>(rs, qb, kb, kb + HC * kPageBytes, t0, vis0, vis1, qp0, qp1, psw, scale2,
                                     a.max_pos, lane);
        }
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
    if (!prm.ml) {
      const int c0 = rl0 < n ? item[kRecXcnt + rl0] : 0, c1 = rl1 < n ? item[kRecXcnt + rl1] : 0;
      const int o0 = item[kRecXoff + rl0], o1 = item[kRecXoff + rl1];
      int emax = max(c0, c1);
#pragma unroll
      for (int o = 4; o < 32; o <<= 1) emax = max(emax, __shfl_xor_sync(0xffffffffu, emax, o));
      const uint32_t qr0 = qb + g * 128, qr1 = qb + (g + 8) * 128;  // rows rl0, rl1 of the query tile
      for (int e = 0; e < emax; ++e) {
#pragma unroll
        for (int ci = 0; ci < 2; ++ci) {
          const int cnt = ci ? c1 : c0;
          int slot = -1, kpos = 0;
          if (e == 0) {  // resolved (and range-checked) by the item pass
            const int rl = ci ? rl1 : rl0;
            if (cnt > 0) {
              slot = item[kRecX0slot + rl];
              kpos = item[kRecX0pos + rl];
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

    // The next item's queries go into the other tile (its previous contents,
    // the item before this one, were last read before this item's first
    // barrier) while this item's epilogue runs.
    {
      const int jn = j + 1, bn = jn % kItemBufs;
      ok_next = __all_sync(0xffffffffu,
                           tc::mbar_wait_park_or_abort(&item_full[bn], (jn / kItemBufs) & 1, st.status, abort_flag));
      const int nn = ok_next ? items[bn * kAttnRecInts + kRecN] : 0;
      if (nn > 0) copy_queries(items + bn * kAttnRecInts, nn, jn & 1);
    }
    // ---- epilogue: this lane holds rows rl0 / rl1, columns 8 q + 2 t, +1 ----
    rs.l0 += __shfl_xor_sync(0xffffffffu, rs.l0, 1);  // the quad's partial row sums
    rs.l0 += __shfl_xor_sync(0xffffffffu, rs.l0, 2);
    rs.l1 += __shfl_xor_sync(0xffffffffu, rs.l1, 1);
    rs.l1 += __shfl_xor_sync(0xffffffffu, rs.l1, 2);
    const float i0 = rs.l0 > 0.f ? 1.0f / rs.l0 : 0.f, i1 = rs.l1 > 0.f ? 1.0f / rs.l1 : 0.f;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      rs.o[q][0] *= i0;
      rs.o[q][1] *= i0;
      rs.o[q][2] *= i1;
      rs.o[q][3] *= i1;
    }
    if (!fused) {
      const int r0 = rl0 < n ? item[kRecRows + rl0] : -1, r1 = rl1 < n ? item[kRecRows + rl1] : -1;
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const int col = h * D + 8 * q + 2 * t;
        if (r0 >= 0) *reinterpret_cast<float2*>(a.out + (size_t)r0 * hdv + col) = make_float2(rs.o[q][0], rs.o[q][1]);
        if (r1 >= 0) *reinterpret_cast<float2*>(a.out + (size_t)r1 * hdv + col) = make_float2(rs.o[q][2], rs.o[q][3]);
      }
      if (prm.ml && t == 0) {
        if (r0 >= 0) prm.ml[(size_t)r0 * H + h] = make_float2(rs.m0, rs.l0);
        if (r1 >= 0) prm.ml[(size_t)r1 * H + h] = make_float2(rs.m1, rs.l1);
      }
    } else {
      // O (bf16) over this warp's own query rows of the tile, then, after one
      // barrier, LayerNorm over each row's H dv outputs times u, whole rows
      // per warp: warp w takes rows w, w + 2 HC, ...; lane l takes 16-byte
      // chunks l and l + 32 of a row (chunk c: head c / 8, columns 8 (c % 8)).
      const uint32_t ot = qtb + tile * q_bytes;
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        asm volatile("st.shared.u32 [%0], %1;" ::"r"(ot + hl * kHeadTile + blk_off(rl0, q) + 4 * t),
                     "r"(pack_bf16(rs.o[q][0], rs.o[q][1]))
                     : "memory");
        asm volatile("st.shared.u32 [%0], %1;" ::"r"(ot + hl * kHeadTile + blk_off(rl1, q) + 4 * t),
                     "r"(pack_bf16(rs.o[q][2], rs.o[q][3]))
                     : "memory");
      }
      const int nck = H * 8;  // 16-byte chunks per row
      uint4 un[2] = {make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0)};  // u of this warp's first row
      {
        const int gr = warp < n ? item[kRecRows + warp] : -1;
#pragma unroll
        for (int c2 = 0; c2 < 2; ++c2)
          if (gr >= 0 && lane + 32 * c2 < nck)
            un[c2] = __ldg(reinterpret_cast<const uint4*>(prm.u + (size_t)gr * hdv + 8 * (lane + 32 * c2)));
      }
      bar_consumers(nct);
      for (int rr = warp; rr < n; rr += ncw) {
        const int gr = item[kRecRows + rr];
        const uint4 ur[2] = {un[0], un[1]};
        const int rn = rr + ncw;  // this warp's next row: its u load overlaps this row
        const int grn = rn < n ? item[kRecRows + rn] : -1;
#pragma unroll
        for (int c2 = 0; c2 < 2; ++c2)
          un[c2] = (grn >= 0 && lane + 32 * c2 < nck)
                       ? __ldg(reinterpret_cast<const uint4*>(prm.u + (size_t)grn * hdv + 8 * (lane + 32 * c2)))
                       : make_uint4(0, 0, 0, 0);
        float v[2][8];
        float sum = 0.f;
#pragma unroll
        for (int c2 = 0; c2 < 2; ++c2) {
          const int ck = lane + 32 * c2;
          uint4 w = make_uint4(0, 0, 0, 0);
          if (ck < nck)
            asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                         : "=r"(w.x), "=r"(w.y), "=r"(w.z), "=r"(w.w)
                         : "r"(ot + (ck >> 3) * kHeadTile + blk_off(rr, ck & 7)));
          const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&ww[e]));
            v[c2][2 * e] = f.x;
            v[c2][2 * e + 1] = f.y;
            sum += f.x + f.y;
          }
        }
        const float mu = warp_sum(sum) / (float)hdv;
        float sq = 0.f;
#pragma unroll
        for (int c2 = 0; c2 < 2; ++c2) {
          if (lane + 32 * c2 < nck)
#pragma unroll
            for (int e = 0; e < 8; ++e) sq += (v[c2][e] - mu) * (v[c2][e] - mu);
        }
        const float rsd = 1.0f / sqrtf(warp_sum(sq) / (float)hdv + 1e-6f);
#pragma unroll
        for (int c2 = 0; c2 < 2; ++c2) {
          const int ck = lane + 32 * c2;
          if (ck >= nck) continue;
          const uint32_t uu[4] = {ur[c2].x, ur[c2].y, ur[c2].z, ur[c2].w};
          uint32_t o[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 uf = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&uu[e]));
            o[e] = pack_bf16(uf.x * ((v[c2][2 * e] - mu) * rsd), uf.y * ((v[c2][2 * e + 1] - mu) * rsd));
          }
          *reinterpret_cast<uint4*>(prm.gated + (size_t)gr * hdv + 8 * ck) = make_uint4(o[0], o[1], o[2], o[3]);
        }
      }
    }
    __syncwarp();
    if (lane == 0) tc::mbar_arrive(&item_empty[b]);  // this warp is done with the item buffer
  }
}

}  // namespace

cudaError_t launch_attn_items(const imba_step_desc& st, const PoolGeom& g, int* recs, cudaStream_t s) {
  if (st.num_chunks <= 0) return cudaSuccess;
  const int warps = 2 * st.num_chunks;
  return launch_pdl(attn_items_kernel, dim3((warps + 3) / 4), dim3(128), 0, s, st, g, recs);
}

// Returns false (nothing launched) when the model / pool cannot use this
// kernel.  *fused is set when the norm + gate was done in the epilogue (the
// caller then skips its gate pass).  a.counters[0 .. H / hc) must be zero and
// recs must hold this step's item records (launch_attn_items).
bool launch_attn_page(const AttnArgs& a, int num_layers, const imba_model_desc& md, int64_t num_pages,
                      const bf16* u, bf16* gated, const int* recs, cudaStream_t s, cudaError_t* err, bool* fused,
                      float2* ml) {
  *fused = false;
  if (md.dtype != IMBA_DTYPE_BF16 || md.attention_dim != 64 || md.linear_dim != 64) return false;
  const int H = md.num_heads;
  int hc = H < kMaxHC ? H : kMaxHC;
  while (H % hc) --hc;  // largest divisor of H up to 8
  if (H / hc > kCountersPerLayer || !a.counters || !recs) return false;
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
  EncodeTiledFn enc = attn_encode_fn();
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
  // Shared memory: alignment slack, KV ring, the two query tiles, optional
  // fp16 bias table, item buffers and barriers.  The bias table is kept in
  // shared memory when at least 3 ring stages still fit.
  const size_t stage_bytes = 2 * (size_t)hc * kPageBytes;
  const size_t meta = kItemBufs * (size_t)kRecBytes + 2 * 4 + (2 * kMaxStages + 2 * kItemBufs) * 8;
  const size_t fixed = 1024 + 2 * (size_t)hc * kHeadTile + meta;
  const size_t bias_bytes = ((size_t)hc * (2 * md.max_pos) * 2 + 15) / 16 * 16;  // rows padded to even length
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
  PageParams prm{a, num_layers, hc, (int)stages, u, fuse ? gated : nullptr, recs, fuse ? nullptr : ml};
  const int ctas = a.st.num_chunks < sms ? a.st.num_chunks : sms;
  dim3 grid(ctas, 1, H / hc);
  *err = launch_pdl(kern, grid, dim3((2 * hc + 1) * 32), smem, s, map, prm);
  *fused = fuse && *err == cudaSuccess;
  return true;
}

namespace {

// The rest of a row's attention after the page kernel's partial pass: its
// extra keys (suffix chain and itself) folded into each head's softmax
// state, O rounded to bf16, the LayerNorm over the row's H dv outputs (no
// affine, eps 1e-6) and the u gate.  One warp per row, H <= 8: lane l takes
// head l / 4 and dims 16 (l % 4) .. +15.
__global__ void __launch_bounds__(256) attn_combine_kernel(const AttnArgs a, const float2* __restrict__ ml,
                                                           const bf16* __restrict__ u, bf16* __restrict__ gated) {
  pdl_wait();
  pdl_trigger();
  const imba_step_desc& st = a.st;
  const int r = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5), lane = threadIdx.x & 31;
  if (r >= st.num_rows) return;
  const int H = a.g.H, hdv = H * 64;
  const int hh = lane >> 2, part = lane & 3;
  const bool on = hh < H;
  const int col = hh * 64 + 16 * part;
  float o[16];
  float m = -INFINITY, l = 0.f;
  if (on) {
    const float4* op = reinterpret_cast<const float4*>(a.out + (size_t)r * hdv + col);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float4 v = op[i];
      o[4 * i] = v.x;
      o[4 * i + 1] = v.y;
      o[4 * i + 2] = v.z;
      o[4 * i + 3] = v.w;
    }
    const float2 s = ml[(size_t)r * H + hh];
    m = s.x;
    l = s.y;
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i) o[i] = 0.f;
  }
  // O back to the unnormalised sum relative to m.
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i] *= l;
  int e0 = st.row_extra_off[r], e1 = st.row_extra_off[r + 1];
  if (e0 < 0 || e1 < e0 || e1 > st.num_extra) {
    report(st.status, IMBA_ERR_RANGE);
    e0 = e1 = 0;
  }
  if (e1 > e0) {
    const int qpos = st.positions[r];
    const float scale2 = a.scale * kLog2e;
    uint4 qv[2] = {make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0)};
    if (on) {
      const uint4* qp = reinterpret_cast<const uint4*>(static_cast<const bf16*>(a.q) + (size_t)r * hdv + col);
      qv[0] = __ldg(qp);
      qv[1] = __ldg(qp + 1);
    }
    const bf16* pool = static_cast<const bf16*>(a.pool);
    for (int e = e0; e < e1; ++e) {
      int slot = st.extra_slot[e];
      const int kpos = st.extra_pos[e];
      if (slot < 0 || slot >= a.g.num_slots) {
        report(st.status, IMBA_ERR_RANGE);
        continue;  // uniform across the warp
      }
      float dot = 0.f;
      float vv[16];
      if (on) {
        const uint4* kp = reinterpret_cast<const uint4*>(pool + a.g.k_off(slot, a.layer, hh) + 16 * part);
        const uint4* vp = reinterpret_cast<const uint4*>(pool + a.g.v_off(slot, a.layer, hh) + 16 * part);
        const uint4 k2[2] = {__ldg(kp), __ldg(kp + 1)}, v2[2] = {__ldg(vp), __ldg(vp + 1)};
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const uint32_t qw[4] = {qv[c].x, qv[c].y, qv[c].z, qv[c].w}, kw[4] = {k2[c].x, k2[c].y, k2[c].z, k2[c].w};
          const uint32_t vw[4] = {v2[c].x, v2[c].y, v2[c].z, v2[c].w};
#pragma unroll
          for (int w = 0; w < 4; ++w) {
            const float2 qf = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&qw[w]));
            const float2 kf = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&kw[w]));
            const float2 vf = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&vw[w]));
            dot = fmaf(qf.x, kf.x, dot);
            dot = fmaf(qf.y, kf.y, dot);
            vv[8 * c + 2 * w] = vf.x;
            vv[8 * c + 2 * w + 1] = vf.y;
          }
        }
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) vv[i] = 0.f;
      }
      dot += __shfl_xor_sync(0xffffffffu, dot, 1);
      dot += __shfl_xor_sync(0xffffffffu, dot, 2);
      if (on) {
        const float sx = fmaf(dot, scale2, __ldg(a.ps_w + (size_t)hh * (2 * a.max_pos - 1) +
                                                  bias_index(kpos, qpos, a.max_pos)) * kLog2e);
        const float mn = fmaxf(m, sx);
        const float c = exp2_approx(m - mn), p = exp2_approx(sx - mn);
        l = fmaf(l, c, p);
#pragma unroll
        for (int i = 0; i < 16; ++i) o[i] = fmaf(o[i], c, p * vv[i]);
        m = mn;
      }
    }
  }
  const float inv = l > 0.f ? 1.0f / l : 0.f;
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    o[i] = __bfloat162float(__float2bfloat16_rn(o[i] * inv));  // the attention output's type
    sum += o[i];
  }
  const float mu = warp_sum(sum) / (float)hdv;
  float q2 = 0.f;
  if (on) {
#pragma unroll
    for (int i = 0; i < 16; ++i) q2 += (o[i] - mu) * (o[i] - mu);
  }
  const float rstd = rsqrtf(warp_sum(q2) / (float)hdv + 1e-6f);
  if (on) {
    const uint4* up = reinterpret_cast<const uint4*>(u + (size_t)r * hdv + col);
    uint4* gp = reinterpret_cast<uint4*>(gated + (size_t)r * hdv + col);
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      const uint4 uv = __ldg(up + c);
      const uint32_t uw[4] = {uv.x, uv.y, uv.z, uv.w};
      uint32_t g[4];
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        const float2 uf = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&uw[w]));
        g[w] = pack_bf16(uf.x * ((o[8 * c + 2 * w] - mu) * rstd), uf.y * ((o[8 * c + 2 * w + 1] - mu) * rstd));
      }
      gp[c] = make_uint4(g[0], g[1], g[2], g[3]);
    }
  }
}

}  // namespace

cudaError_t launch_attn_combine(const AttnArgs& a, const float2* ml, const bf16* u, bf16* gated, cudaStream_t s) {
  if (a.g.H > 8 || a.st.num_rows <= 0) return a.st.num_rows <= 0 ? cudaSuccess : cudaErrorInvalidValue;
  const int blocks = (a.st.num_rows + 7) / 8;
  return launch_pdl(attn_combine_kernel, dim3(blocks), dim3(256), 0, s, a, ml, u, gated);
}

}  // namespace imba
