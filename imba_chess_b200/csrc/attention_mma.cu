// Grouped paged-KV decode / prefill attention on the tensor cores (bf16
// models, d_qk = d_v = 64).
//
// One CTA per (chunk of <= 64 query rows of one sequence group, group of
// heads).  For each of its heads the CTA streams the group's KV pages in
// 64-token tiles (four 16-token pages): per page one TMA tiled load brings
// its 16 K rows and one its 16 V rows of this (layer, head) into shared
// memory with the 128-byte swizzle.  The (head, tile) sequence flows through
// one double-buffered ring (one mbarrier per stage, bounded waits), so the
// next head's tiles load while the current head computes.  Each tile is
// loaded ONCE and serves every sibling row of the chunk: warp w owns query
// rows 16w..16w+15; S = Q K^T (mma.sync m16n8k16, fp32 accumulate), scale,
// relative-position bias ps_w[h, clamp(k - q + max - 1)], per-row visibility
// mask, fp32 online softmax in registers, O += P V.  The rows' extra keys
// (each row's suffix chain and the row itself, scattered arena slots) are
// gathered with cp.async into 64-key tiles of the same swizzled layout and go
// through the same loop with an ownership mask (key j is visible to row r
// only if it is one of r's extras).  Semantics: src/imba_chess/model/
// hstu_attention.py :64-76, :81-132, :134-148, :327-413.
#include "kernels.cuh"
#include "tc_ptx.cuh"

namespace imba {
namespace {

constexpr int kRows = IMBA_CHUNK_ROWS;  // 64
constexpr int kTileTok = 64;
constexpr int kPagesPerTile = kTileTok / IMBA_PAGE_TOKENS;    // 4
constexpr int kBlockBytes = IMBA_PAGE_TOKENS * 64 * 2;        // 16 rows x 128 B
constexpr int kStageBytes = 2 * kPagesPerTile * kBlockBytes;  // K blocks then V blocks
constexpr int kStages = 2;
constexpr int kThreads = 128;

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

// Byte offset of (token t of a 64-token tile, 16-byte chunk j of its 128-byte
// row) in a K or V half-stage: page block t/16, row t%16, 128-byte swizzle.
__device__ __forceinline__ uint32_t tile_off(int t, int j) {
  return (uint32_t)((t >> 4) * kBlockBytes + (t & 15) * 128 + ((j ^ (t & 7)) << 4));
}

struct AttnMmaParams {
  AttnArgs a;
  int num_layers;
  int heads_per_cta;
};

// Running softmax state of this lane's two rows (rl0 = 16w + g, rl1 = rl0 + 8).
struct RowState {
  float o[8][4];
  float m0, m1, l0, l1;
};

// One 64-key tile: S = Q K^T, mask / scale / bias, online softmax, O += P V.
// is_extra: keys are gathered extras (owner / position per key in smem);
// otherwise prefix tokens t0 .. t0 + 63 visible below each row's limit.
__device__ __forceinline__ void tile_step(RowState& rs, const uint32_t (&qa)[4][4], uint32_t kb, bool is_extra,
                                          int t0, int vis0, int vis1, int qp0, int qp1, int rl0, int rl1,
                                          const int* x_owner, const int* x_pos, const float* __restrict__ psw,
                                          float scale, int max_pos, int lane) {
  const int t = lane & 3, r8 = lane & 7, mm = lane >> 3;
  const uint32_t vb = kb + kPagesPerTile * kBlockBytes;
  float sc[8][4];
#pragma unroll
  for (int j = 0; j < 8; ++j) sc[j][0] = sc[j][1] = sc[j][2] = sc[j][3] = 0.f;
#pragma unroll
  for (int kc = 0; kc < 4; ++kc) {
#pragma unroll
    for (int nt = 0; nt < 8; nt += 2) {
      uint32_t b[4];
      ldsm_x4(b, kb + tile_off(8 * nt + r8 + 8 * (mm >> 1), 2 * kc + (mm & 1)));
      mma16816(sc[nt], qa[kc], b[0], b[1]);
      mma16816(sc[nt + 1], qa[kc], b[2], b[3]);
    }
  }
  float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
  for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int j = 8 * nt + 2 * t + e;
      bool v0, v1;
      int kpos;
      if (!is_extra) {
        kpos = t0 + j;
        v0 = kpos < vis0;
        v1 = kpos < vis1;
      } else {
        const int own = x_owner[j];
        kpos = x_pos[j];
        v0 = own == rl0;
        v1 = own == rl1;
      }
      sc[nt][e] = v0 ? sc[nt][e] * scale + __ldg(psw + bias_index(kpos, qp0, max_pos)) : -INFINITY;
      sc[nt][2 + e] = v1 ? sc[nt][2 + e] * scale + __ldg(psw + bias_index(kpos, qp1, max_pos)) : -INFINITY;
      mx0 = fmaxf(mx0, sc[nt][e]);
      mx1 = fmaxf(mx1, sc[nt][2 + e]);
    }
  }
  mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
  mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
  mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
  mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
  const float mn0 = fmaxf(rs.m0, mx0), mn1 = fmaxf(rs.m1, mx1);
  const float c0 = mn0 == -INFINITY ? 1.f : (rs.m0 == -INFINITY ? 0.f : __expf(rs.m0 - mn0));
  const float c1 = mn1 == -INFINITY ? 1.f : (rs.m1 == -INFINITY ? 0.f : __expf(rs.m1 - mn1));
  float ps0 = 0.f, ps1 = 0.f;
#pragma unroll
  for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const float p0 = sc[nt][e] == -INFINITY ? 0.f : __expf(sc[nt][e] - mn0);
      const float p1 = sc[nt][2 + e] == -INFINITY ? 0.f : __expf(sc[nt][2 + e] - mn1);
      sc[nt][e] = p0;
      sc[nt][2 + e] = p1;
      ps0 += p0;
      ps1 += p1;
    }
  }
  ps0 += __shfl_xor_sync(0xffffffffu, ps0, 1);
  ps0 += __shfl_xor_sync(0xffffffffu, ps0, 2);
  ps1 += __shfl_xor_sync(0xffffffffu, ps1, 1);
  ps1 += __shfl_xor_sync(0xffffffffu, ps1, 2);
  rs.l0 = rs.l0 * c0 + ps0;
  rs.l1 = rs.l1 * c1 + ps1;
  rs.m0 = mn0;
  rs.m1 = mn1;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    rs.o[j][0] *= c0;
    rs.o[j][1] *= c0;
    rs.o[j][2] *= c1;
    rs.o[j][3] *= c1;
  }
  uint32_t pa[4][4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    pa[j][0] = pack_bf16(sc[2 * j][0], sc[2 * j][1]);
    pa[j][1] = pack_bf16(sc[2 * j][2], sc[2 * j][3]);
    pa[j][2] = pack_bf16(sc[2 * j + 1][0], sc[2 * j + 1][1]);
    pa[j][3] = pack_bf16(sc[2 * j + 1][2], sc[2 * j + 1][3]);
  }
#pragma unroll
  for (int kc = 0; kc < 4; ++kc) {
#pragma unroll
    for (int np = 0; np < 4; ++np) {
      uint32_t b[4];
      ldsm_x4_t(b, vb + tile_off(16 * kc + r8 + 8 * (mm & 1), 2 * np + (mm >> 1)));
      mma16816(rs.o[2 * np], pa[kc], b[0], b[1]);
      mma16816(rs.o[2 * np + 1], pa[kc], b[2], b[3]);
    }
  }
}

__global__ void __launch_bounds__(kThreads, 3)
    attn_mma_kernel(const __grid_constant__ CUtensorMap kvmap, const AttnMmaParams prm) {
  const AttnArgs& a = prm.a;
  const imba_step_desc& st = a.st;
  const int c = blockIdx.x;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int H = a.g.H;
  constexpr int D = 64;
  const int h0 = blockIdx.y * prm.heads_per_cta;
  const int h1 = h0 + prm.heads_per_cta < H ? h0 + prm.heads_per_cta : H;
  const int nh = h1 - h0;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* stages = base;                                        // kStages x kStageBytes (prefix tiles)
  uint8_t* xstage = stages + kStages * kStageBytes;              // one gathered extra-key tile
  int* x_owner = reinterpret_cast<int*>(xstage + kStageBytes);   // [64] local row owning each extra key
  int* x_pos = x_owner + kTileTok;                               // [64] its position
  int* x_start = x_pos + kTileTok;                               // [65] exclusive scan of extras per row
  uint64_t* full = reinterpret_cast<uint64_t*>(x_start + kRows + 2);  // 8-byte aligned: 194 ints precede
  __shared__ int rows_s[kRows], vis_s[kRows], qpos_s[kRows], xoff_s[kRows], xcnt_s[kRows];
  __shared__ int vmax_s;

  const int grp = st.chunk_group[c];
  const int off = st.chunk_row_off[c];
  const int n = st.chunk_nrows[c];
  if (nh <= 0 || grp < 0 || grp >= st.num_groups || n < 0 || n > kRows || off < 0 || off + n > st.num_rows) {
    if (tid == 0 && nh > 0) report(st.status, IMBA_ERR_RANGE);
    return;
  }
  int pg0 = st.group_page_off[grp], pg1 = st.group_page_off[grp + 1];
  if (pg0 < 0 || pg1 < pg0 || pg1 > st.num_group_pages) {
    if (tid == 0) report(st.status, IMBA_ERR_RANGE);
    pg0 = pg1 = 0;
  }
  const int npages = pg1 - pg0;
  const int cap = npages * IMBA_PAGE_TOKENS;
  const int64_t num_pages = a.g.num_slots / IMBA_PAGE_TOKENS;

  if (tid == 0) {
    vmax_s = 0;
    for (int s = 0; s < kStages; ++s) tc::mbar_init(&full[s], 1);
    tc::fence_mbar_init();
  }
  __syncthreads();
  // Per-row metadata, one thread per row (independent loads).
  if (tid < kRows) {
    int r = -1, v = 0, qp = 0, e0 = 0, e1 = 0;
    if (tid < n) {
      r = st.row_perm[off + tid];
      if (r < 0 || r >= st.num_rows) {
        report(st.status, IMBA_ERR_RANGE);
        r = 0;
      }
      v = st.row_vis[r];
      qp = st.positions[r];
      e0 = st.row_extra_off[r];
      e1 = st.row_extra_off[r + 1];
      if (v < 0 || v > cap) {
        report(st.status, IMBA_ERR_RANGE);
        v = v < 0 ? 0 : cap;
      }
      if (e0 < 0 || e1 < e0 || e1 > st.num_extra) {
        report(st.status, IMBA_ERR_RANGE);
        e1 = e0 = 0;
      }
      atomicMax(&vmax_s, v);
    }
    rows_s[tid] = r;
    vis_s[tid] = v;
    qpos_s[tid] = qp;
    xoff_s[tid] = e0;
    xcnt_s[tid] = e1 - e0;
  }
  __syncthreads();
  if (warp == 0) {  // exclusive scan of the 64 per-row extra counts, two per lane
    const int c0 = xcnt_s[2 * lane], c1 = xcnt_s[2 * lane + 1];
    int incl = c0 + c1;
#pragma unroll
    for (int o2 = 1; o2 < 32; o2 <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o2);
      if (lane >= o2) incl += v;
    }
    const int excl = incl - c0 - c1;
    x_start[2 * lane] = excl;
    x_start[2 * lane + 1] = excl + c0;
    if (lane == 31) x_start[kRows] = incl;
  }
  __syncthreads();
  const int ntiles = (vmax_s + kTileTok - 1) / kTileTok;
  const int n_extra = x_start[kRows];
  const int xtiles = (n_extra + kTileTok - 1) / kTileTok;
  const int total_p = nh * ntiles;  // prefix (head, tile) items

  // TMA issue of prefix item p (head h0 + p / ntiles, tile p % ntiles) into stage p % kStages.
  auto issue = [&](int p) {
    const int s = p % kStages;
    const int h = h0 + p / ntiles, ti = p % ntiles;
    uint8_t* dst = stages + s * kStageBytes;
    int pages[kPagesPerTile];
#pragma unroll
    for (int q = 0; q < kPagesPerTile; ++q) {
      const int idx = ti * kPagesPerTile + q;
      pages[q] = st.group_pages[pg0 + (idx < npages ? idx : 0)];
    }
    tc::mbar_arrive_expect_tx(&full[s], kStageBytes);
#pragma unroll
    for (int q = 0; q < kPagesPerTile; ++q) {
      int page = pages[q];
      if (page < 0 || page >= num_pages) {
        report(st.status, IMBA_ERR_RANGE);
        page = 0;
      }
      const int rowK = ((page * prm.num_layers + a.layer) * 2 * H + h) * IMBA_PAGE_TOKENS;
      const int rowV = rowK + H * IMBA_PAGE_TOKENS;
      tc::tma_load_2d(dst + q * kBlockBytes, &kvmap, &full[s], 0, rowK);
      tc::tma_load_2d(dst + kPagesPerTile * kBlockBytes + q * kBlockBytes, &kvmap, &full[s], 0, rowV);
    }
  };
  if (tid == 0) {
    for (int p = 0; p < kStages && p < total_p; ++p) issue(p);
  }

  // Gather extra-key tile xt of head h into xstage with cp.async; records each
  // key's owner row and position (the same for every head).
  const bf16* Pool = static_cast<const bf16*>(a.pool);
  auto gather_extras = [&](int h, int xt) {
    for (int idx = tid; idx < kTileTok * 16; idx += kThreads) {
      const int j = idx >> 4, part = idx & 15;  // key j, 16-byte chunk part (0..7 K, 8..15 V)
      const int q = xt * kTileTok + j;
      const uint32_t dst = static_cast<uint32_t>(__cvta_generic_to_shared(xstage)) +
                           (part < 8 ? 0u : (uint32_t)(kPagesPerTile * kBlockBytes)) + tile_off(j, part & 7);
      int64_t slot = -1;
      if (q < n_extra) {
        int lo = 0, hi = n;  // owner: last rr with x_start[rr] <= q
        while (hi - lo > 1) {
          const int mid = (lo + hi) >> 1;
          if (x_start[mid] <= q) lo = mid; else hi = mid;
        }
        const int xi = xoff_s[lo] + (q - x_start[lo]);
        slot = st.extra_slot[xi];
        if (slot < 0 || slot >= a.g.num_slots) {
          if (part == 0) report(st.status, IMBA_ERR_RANGE);
          slot = -1;
        }
        if (part == 0) {
          x_owner[j] = slot >= 0 ? lo : -1;
          x_pos[j] = st.extra_pos[xi];
        }
      } else if (part == 0) {
        x_owner[j] = -1;
        x_pos[j] = 0;
      }
      if (slot >= 0) {
        const bf16* src = Pool + (part < 8 ? a.g.k_off(slot, a.layer, h) : a.g.v_off(slot, a.layer, h)) +
                          8 * (part & 7);
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(dst), "l"(src) : "memory");
      } else {
        asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};\n" ::"r"(dst), "r"(0u) : "memory");
      }
    }
    asm volatile("cp.async.commit_group;\n" ::: "memory");
  };
  if (xtiles > 0) gather_extras(h0, 0);

  const int rl0 = 16 * warp + g, rl1 = rl0 + 8;
  const bool warp_live = 16 * warp < n;
  const int vis0 = rl0 < n ? vis_s[rl0] : 0, vis1 = rl1 < n ? vis_s[rl1] : 0;
  const int qp0 = rl0 < n ? qpos_s[rl0] : 0, qp1 = rl1 < n ? qpos_s[rl1] : 0;
  const bf16* Q = static_cast<const bf16*>(a.q);
  const uint32_t stage_base = static_cast<uint32_t>(__cvta_generic_to_shared(stages));
  const uint32_t xbase = static_cast<uint32_t>(__cvta_generic_to_shared(xstage));
  bool aborted = false;

  for (int hh = 0; hh < nh && !aborted; ++hh) {
    const int h = h0 + hh;
    const float* psw = a.ps_w + (size_t)h * (2 * a.max_pos - 1);
    uint32_t qa[4][4];
    {
      const bf16* q0 = rl0 < n ? Q + (size_t)rows_s[rl0] * (H * D) + h * D : nullptr;
      const bf16* q1 = rl1 < n ? Q + (size_t)rows_s[rl1] * (H * D) + h * D : nullptr;
#pragma unroll
      for (int kc = 0; kc < 4; ++kc) {
        const int col = 16 * kc + 2 * t;
        qa[kc][0] = q0 ? *reinterpret_cast<const uint32_t*>(q0 + col) : 0u;
        qa[kc][1] = q1 ? *reinterpret_cast<const uint32_t*>(q1 + col) : 0u;
        qa[kc][2] = q0 ? *reinterpret_cast<const uint32_t*>(q0 + col + 8) : 0u;
        qa[kc][3] = q1 ? *reinterpret_cast<const uint32_t*>(q1 + col + 8) : 0u;
      }
    }
    RowState rs;
#pragma unroll
    for (int j = 0; j < 8; ++j) rs.o[j][0] = rs.o[j][1] = rs.o[j][2] = rs.o[j][3] = 0.f;
    rs.m0 = rs.m1 = -INFINITY;
    rs.l0 = rs.l1 = 0.f;

    for (int ti = 0; ti < ntiles; ++ti) {
      const int p = hh * ntiles + ti, s = p % kStages;
      bool ok = tc::mbar_wait(&full[s], (p / kStages) & 1, st.status);
      ok = __syncthreads_and(ok);
      if (!ok) {
        aborted = true;
        break;
      }
      if (warp_live)
        tile_step(rs, qa, stage_base + s * kStageBytes, false, ti * kTileTok, vis0, vis1, qp0, qp1, rl0, rl1,
                  x_owner, x_pos, psw, a.scale, a.max_pos, lane);
      __syncthreads();  // every warp is done with stage s
      if (tid == 0 && p + kStages < total_p) issue(p + kStages);
    }
    if (aborted) break;
    for (int xt = 0; xt < xtiles; ++xt) {
      asm volatile("cp.async.wait_all;\n" ::: "memory");
      __syncthreads();
      if (warp_live)
        tile_step(rs, qa, xbase, true, 0, 0, 0, qp0, qp1, rl0, rl1, x_owner, x_pos, psw, a.scale, a.max_pos, lane);
      __syncthreads();
      if (xt + 1 < xtiles) gather_extras(h, xt + 1);
      else if (hh + 1 < nh) gather_extras(h + 1, 0);
    }
    // Normalise and store: this lane holds rows rl0 / rl1, columns 8j + 2t, +1.
    if (warp_live) {
      const float i0 = rs.l0 > 0.f ? 1.0f / rs.l0 : 0.f, i1 = rs.l1 > 0.f ? 1.0f / rs.l1 : 0.f;
      float* out0 = rl0 < n ? a.out + (size_t)rows_s[rl0] * (H * D) + h * D : nullptr;
      float* out1 = rl1 < n ? a.out + (size_t)rows_s[rl1] * (H * D) + h * D : nullptr;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int col = 8 * j + 2 * t;
        if (out0) *reinterpret_cast<float2*>(out0 + col) = make_float2(rs.o[j][0] * i0, rs.o[j][1] * i0);
        if (out1) *reinterpret_cast<float2*>(out1 + col) = make_float2(rs.o[j][2] * i1, rs.o[j][3] * i1);
      }
    }
  }
  if (aborted) asm volatile("cp.async.wait_all;\n" ::: "memory");
}

// TMA view of the pool: 2D [num_pages * L * 2H * 16 rows, 64 columns] bf16.
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

constexpr size_t kSmemBytes =
    1024 + (kStages + 1) * kStageBytes + sizeof(int) * (2 * kTileTok + kRows + 2) + kStages * 8;

}  // namespace

// Returns false (nothing launched) when the model / pool cannot use this kernel.
bool launch_attn_mma(const AttnArgs& a, int num_layers, const imba_model_desc& md, int64_t num_pages,
                     cudaStream_t s, cudaError_t* err) {
  if (md.dtype != IMBA_DTYPE_BF16 || md.attention_dim != 64 || md.linear_dim != 64) return false;
  if (a.st.num_chunks <= 0) {
    *err = cudaSuccess;
    return true;
  }
  const uint64_t rows = (uint64_t)num_pages * num_layers * 2 * md.num_heads * IMBA_PAGE_TOKENS;
  if (rows > (uint64_t)INT32_MAX) return false;
  EncodeTiledFn enc = encode_fn();
  if (!enc || (reinterpret_cast<uintptr_t>(a.pool) & 15)) return false;
  CUtensorMap map;
  const cuuint64_t dims[2] = {64, rows};
  const cuuint64_t strides[1] = {128};
  const cuuint32_t box[2] = {64, IMBA_PAGE_TOKENS};
  const cuuint32_t estr[2] = {1, 1};
  if (enc(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(a.pool), dims, strides, box, estr,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return false;
  cudaError_t e =
      cudaFuncSetAttribute(attn_mma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes);
  if (e != cudaSuccess) {
    *err = e;
    return true;
  }
  // Heads per CTA: enough CTAs to fill the machine (~4 per SM); when the
  // chunks alone do, each CTA takes more heads (one prologue, a longer TMA
  // stream).
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int H = md.num_heads;
  int groups = (4 * sms + a.st.num_chunks - 1) / a.st.num_chunks;
  groups = groups < 1 ? 1 : (groups > H ? H : groups);
  const int hpc = (H + groups - 1) / groups;
  const int gy = (H + hpc - 1) / hpc;
  AttnMmaParams prm{a, num_layers, hpc};
  dim3 grid(a.st.num_chunks, gy);
  attn_mma_kernel<<<grid, kThreads, kSmemBytes, s>>>(map, prm);
  *err = cudaGetLastError();
  return true;
}

}  // namespace imba
