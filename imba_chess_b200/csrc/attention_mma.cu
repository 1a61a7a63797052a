// Grouped paged-KV decode / prefill attention on the tensor cores (bf16
// models, d_qk = d_v = 64).
//
// One CTA per (chunk of <= 64 query rows of one sequence group, head).  The
// group's KV pages are streamed in 64-token tiles (four 16-token pages); for
// every page one TMA tiled load brings its 16 K rows and one its 16 V rows of
// this (layer, head) into shared memory with the 128-byte swizzle
// (double-buffered, one mbarrier per stage, bounded waits).  Each tile is
// loaded ONCE and serves every sibling row of the chunk: warp w owns query
// rows 16w..16w+15; S = Q K^T (mma.sync m16n8k16, fp32 accumulate), scale,
// relative-position bias ps_w[h, clamp(k - q + max - 1)], per-row visibility
// mask, fp32 online softmax in registers, O += P V.  The rows' extra keys
// (suffix chain and the row itself) are folded in afterwards per row, exactly
// as in the SIMT kernel.  Semantics: src/imba_chess/model/hstu_attention.py
// :64-76, :81-132, :134-148, :327-413.
#include "kernels.cuh"
#include "tc_ptx.cuh"

namespace imba {
namespace {

constexpr int kRows = IMBA_CHUNK_ROWS;  // 64
constexpr int kTileTok = 64;
constexpr int kPagesPerTile = kTileTok / IMBA_PAGE_TOKENS;  // 4
constexpr int kBlockBytes = IMBA_PAGE_TOKENS * 64 * 2;      // 16 rows x 128 B
constexpr int kStageBytes = 2 * kPagesPerTile * kBlockBytes;  // K blocks then V blocks
constexpr int kStages = 2;
constexpr int kLdO = 65;

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
};

__global__ void __launch_bounds__(128)
    attn_mma_kernel(const __grid_constant__ CUtensorMap kvmap, const AttnMmaParams prm) {
  const AttnArgs& a = prm.a;
  const imba_step_desc& st = a.st;
  const int c = blockIdx.x, h = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int H = a.g.H;
  constexpr int D = 64;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* stages = base;                                           // kStages x kStageBytes
  float* O_s = reinterpret_cast<float*>(stages + kStages * kStageBytes);  // [64][65]
  float* m_s = O_s + kRows * kLdO;
  float* l_s = m_s + kRows;
  float* psw = l_s + kRows;  // [2 max_pos - 1]
  uint64_t* full = reinterpret_cast<uint64_t*>(
      (reinterpret_cast<uintptr_t>(psw + 2 * a.max_pos - 1) + 7) & ~uintptr_t(7));
  __shared__ int rows_s[kRows], vis_s[kRows], qpos_s[kRows];
  __shared__ int vmax_s;

  const int grp = st.chunk_group[c];
  const int off = st.chunk_row_off[c];
  const int n = st.chunk_nrows[c];
  if (grp < 0 || grp >= st.num_groups || n < 0 || n > kRows || off < 0 || off + n > st.num_rows) {
    if (tid == 0) report(st.status, IMBA_ERR_RANGE);
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
  for (int i = tid; i < 2 * a.max_pos - 1; i += 128) psw[i] = a.ps_w[(size_t)h * (2 * a.max_pos - 1) + i];
  __syncthreads();
  if (tid < kRows) {
    int r = -1, v = 0, qp = 0;
    if (tid < n) {
      r = st.row_perm[off + tid];
      if (r < 0 || r >= st.num_rows) {
        report(st.status, IMBA_ERR_RANGE);
        r = 0;
      }
      v = st.row_vis[r];
      if (v < 0 || v > cap) {
        report(st.status, IMBA_ERR_RANGE);
        v = v < 0 ? 0 : cap;
      }
      qp = st.positions[r];
      atomicMax(&vmax_s, v);
    }
    rows_s[tid] = r;
    vis_s[tid] = v;
    qpos_s[tid] = qp;
  }
  __syncthreads();
  const int vmax = vmax_s;
  const int ntiles = (vmax + kTileTok - 1) / kTileTok;

  // TMA issue of tile i into stage i % kStages (thread 0 only).
  auto issue = [&](int i) {
    const int s = i % kStages;
    uint8_t* dst = stages + s * kStageBytes;
    tc::mbar_arrive_expect_tx(&full[s], kStageBytes);
    for (int p = 0; p < kPagesPerTile; ++p) {
      const int idx = i * kPagesPerTile + p;
      int page = st.group_pages[pg0 + (idx < npages ? idx : 0)];
      if (page < 0 || page >= num_pages) {
        report(st.status, IMBA_ERR_RANGE);
        page = 0;
      }
      const int rowK = ((page * prm.num_layers + a.layer) * 2 * H + h) * IMBA_PAGE_TOKENS;
      const int rowV = rowK + H * IMBA_PAGE_TOKENS;
      tc::tma_load_2d(dst + p * kBlockBytes, &kvmap, &full[s], 0, rowK);
      tc::tma_load_2d(dst + kPagesPerTile * kBlockBytes + p * kBlockBytes, &kvmap, &full[s], 0, rowV);
    }
  };
  if (tid == 0) {
    for (int i = 0; i < kStages && i < ntiles; ++i) issue(i);
  }

  // Query fragments of this warp's 16 rows.
  const int rl0 = 16 * warp + g, rl1 = rl0 + 8;
  const bool warp_live = 16 * warp < n;
  uint32_t qa[4][4];
  {
    const bf16* Q = static_cast<const bf16*>(a.q);
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
  const int vis0 = rl0 < n ? vis_s[rl0] : 0, vis1 = rl1 < n ? vis_s[rl1] : 0;
  const int qp0 = rl0 < n ? qpos_s[rl0] : 0, qp1 = rl1 < n ? qpos_s[rl1] : 0;
  float o[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  const int r8 = lane & 7, mm = lane >> 3;

  for (int i = 0; i < ntiles; ++i) {
    const int s = i % kStages;
    bool ok = tc::mbar_wait(&full[s], (i / kStages) & 1, st.status);
    ok = __syncthreads_and(ok);
    if (!ok) break;
    if (warp_live) {
      const uint32_t kb = static_cast<uint32_t>(__cvta_generic_to_shared(stages + s * kStageBytes));
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
      // scale, bias, visibility; running max
      const int t0 = i * kTileTok;
      float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int key = t0 + 8 * nt + 2 * t + e;
          sc[nt][e] = key < vis0 ? sc[nt][e] * a.scale + psw[bias_index(key, qp0, a.max_pos)] : -INFINITY;
          sc[nt][2 + e] = key < vis1 ? sc[nt][2 + e] * a.scale + psw[bias_index(key, qp1, a.max_pos)] : -INFINITY;
          mx0 = fmaxf(mx0, sc[nt][e]);
          mx1 = fmaxf(mx1, sc[nt][2 + e]);
        }
      }
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
      const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
      const float c0 = (mn0 == -INFINITY || m0 == -INFINITY) ? (mn0 == -INFINITY ? 1.f : 0.f) : expf(m0 - mn0);
      const float c1 = (mn1 == -INFINITY || m1 == -INFINITY) ? (mn1 == -INFINITY ? 1.f : 0.f) : expf(m1 - mn1);
      float ps0 = 0.f, ps1 = 0.f;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float p0 = sc[nt][e] == -INFINITY ? 0.f : expf(sc[nt][e] - mn0);
          const float p1 = sc[nt][2 + e] == -INFINITY ? 0.f : expf(sc[nt][2 + e] - mn1);
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
      l0 = l0 * c0 + ps0;
      l1 = l1 * c1 + ps1;
      m0 = mn0;
      m1 = mn1;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        o[j][0] *= c0;
        o[j][1] *= c0;
        o[j][2] *= c1;
        o[j][3] *= c1;
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
          mma16816(o[2 * np], pa[kc], b[0], b[1]);
          mma16816(o[2 * np + 1], pa[kc], b[2], b[3]);
        }
      }
    }
    __syncthreads();  // every warp is done with stage s
    if (tid == 0 && i + kStages < ntiles) issue(i + kStages);
  }

  // Unnormalised prefix state -> shared memory, one row per warp afterwards.
  if (warp_live) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int col = 8 * j + 2 * t;
      O_s[rl0 * kLdO + col] = o[j][0];
      O_s[rl0 * kLdO + col + 1] = o[j][1];
      O_s[rl1 * kLdO + col] = o[j][2];
      O_s[rl1 * kLdO + col + 1] = o[j][3];
    }
    if (t == 0) {
      m_s[rl0] = m0;
      l_s[rl0] = l0;
      m_s[rl1] = m1;
      l_s[rl1] = l1;
    }
  }
  __syncthreads();

  const bf16* P = static_cast<const bf16*>(a.pool);
  const bf16* Q = static_cast<const bf16*>(a.q);
  for (int rr = warp; rr < n; rr += 4) {
    const int r = rows_s[rr];
    int e0 = st.row_extra_off[r], e1 = st.row_extra_off[r + 1];
    if (e0 < 0 || e1 < e0 || e1 > st.num_extra) {
      if (lane == 0) report(st.status, IMBA_ERR_RANGE);
      e0 = e1 = 0;
    }
    float m = m_s[rr], l = l_s[rr];
    float o0 = O_s[rr * kLdO + lane], o1 = O_s[rr * kLdO + lane + 32];
    const bf16* qr = Q + (size_t)r * (H * D) + h * D;
    const float q0 = __bfloat162float(qr[lane]), q1 = __bfloat162float(qr[lane + 32]);
    for (int x = e0; x < e1; ++x) {
      const int64_t slot = st.extra_slot[x];
      if (slot < 0 || slot >= a.g.num_slots) {
        if (lane == 0) report(st.status, IMBA_ERR_RANGE);
        continue;
      }
      const bf16* kp = P + a.g.k_off(slot, a.layer, h);
      const bf16* vp = P + a.g.v_off(slot, a.layer, h);
      float d = q0 * __bfloat162float(kp[lane]);
      d = fmaf(q1, __bfloat162float(kp[lane + 32]), d);
      d = warp_sum(d);
      const float sx = d * a.scale + psw[bias_index(st.extra_pos[x], qpos_s[rr], a.max_pos)];
      const float mnew = fmaxf(m, sx);
      const float cr = (m == -INFINITY) ? 0.f : expf(m - mnew);
      const float p = expf(sx - mnew);
      l = l * cr + p;
      o0 = o0 * cr + p * __bfloat162float(vp[lane]);
      o1 = o1 * cr + p * __bfloat162float(vp[lane + 32]);
      m = mnew;
    }
    const float inv = l > 0.f ? 1.0f / l : 0.f;
    float* outr = a.out + (size_t)r * (H * D) + h * D;
    outr[lane] = o0 * inv;
    outr[lane + 32] = o1 * inv;
  }
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

}  // namespace

size_t attn_mma_smem_bytes(int max_pos) {
  return 1024 + kStages * kStageBytes + sizeof(float) * (kRows * kLdO + 2 * kRows + 2 * max_pos - 1) + 8 +
         kStages * 8;
}

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
  const size_t smem = attn_mma_smem_bytes(md.max_pos);
  if (smem > 200 * 1024) return false;
  cudaError_t e = cudaFuncSetAttribute(attn_mma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) {
    *err = e;
    return true;
  }
  AttnMmaParams prm{a, num_layers};
  dim3 grid(a.st.num_chunks, md.num_heads);
  attn_mma_kernel<<<grid, 128, smem, s>>>(map, prm);
  *err = cudaGetLastError();
  return true;
}

}  // namespace imba
