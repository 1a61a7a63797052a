// Grouped paged-KV decode / prefill attention, SIMT fp32 math (exact path).
//
// For one chunk of <= 64 query rows of one sequence group and one head, the
// CTA streams the group's KV pages in 32-token tiles ONCE and reuses each
// tile for every row of the chunk (all sibling queries of a parent share the
// parent's prefix).  Per row the key set is
//   [first row_vis tokens of the group | the row's extra keys (suffix chain
//    and the row's own token)]
// with score = (q . k) / sqrt(d_qk) + ps_w[h, clamp(k_pos - q_pos + max - 1,
// 0, 2 max - 2)] and an fp32 online softmax, which equals the reference's
// concatenated [prefix | masked suffix | self] softmax
// (src/imba_chess/model/hstu_attention.py:134-148, :327-413) and its causal
// prefill form (hstu_attention.py:64-76, :81-132).
#include "kernels.cuh"

namespace imba {

namespace {

constexpr int kRows = IMBA_CHUNK_ROWS;  // 64
constexpr int kTile = 32;
constexpr int kLd = 65;
constexpr int kLdP = kTile + 1;

__device__ __forceinline__ int bias_index(int kpos, int qpos, int max_pos) {
  int idx = kpos - qpos + (max_pos - 1);
  idx = idx < 0 ? 0 : idx;
  return idx > 2 * max_pos - 2 ? 2 * max_pos - 2 : idx;
}

template <typename T>
__global__ void __launch_bounds__(128) attn_simt_kernel(AttnArgs a) {
  pdl_wait();
  pdl_trigger();
  const int c = blockIdx.x, h = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int dqk = a.g.dqk, dv = a.g.dv;
  const imba_step_desc& st = a.st;
  extern __shared__ float sm[];
  float* qs = sm;                   // [64][65]
  float* acc = qs + kRows * kLd;    // [64][65]
  float* kt = acc + kRows * kLd;    // [32][65]
  float* vt = kt + kTile * kLd;     // [32][65]
  float* pt = vt + kTile * kLd;     // [64][33]
  float* mrow = pt + kRows * kLdP;  // [64]
  float* lrow = mrow + kRows;       // [64]
  float* crow = lrow + kRows;       // [64]
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
  const int cap = (pg1 - pg0) * IMBA_PAGE_TOKENS;
  const float* psw = a.ps_w + (size_t)h * (2 * a.max_pos - 1);
  const T* Q = static_cast<const T*>(a.q);
  const T* P = static_cast<const T*>(a.pool);
  const int64_t num_pages = a.g.num_slots / IMBA_PAGE_TOKENS;

  if (tid == 0) vmax_s = 0;
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
    mrow[tid] = -INFINITY;
    lrow[tid] = 0.f;
  }
  __syncthreads();
  for (int i = tid; i < kRows * 64; i += 128) {
    const int rr = i >> 6, e = i & 63;
    float qv = 0.f;
    if (rr < n && e < dqk) qv = to_f(Q[(size_t)rows_s[rr] * (a.g.H * dqk) + h * dqk + e]);
    qs[rr * kLd + e] = qv;
    acc[rr * kLd + e] = 0.f;
  }
  __syncthreads();

  const int vmax = vmax_s;
  for (int t0 = 0; t0 < vmax; t0 += kTile) {
    for (int i = tid; i < kTile * 64; i += 128) {
      const int j = i >> 6, e = i & 63;
      const int tt = t0 + j;
      float kv = 0.f, vv = 0.f;
      if (tt < vmax) {
        const int page = st.group_pages[pg0 + tt / IMBA_PAGE_TOKENS];
        if (page < 0 || page >= num_pages) {
          report(st.status, IMBA_ERR_RANGE);
        } else {
          const int64_t slot = (int64_t)page * IMBA_PAGE_TOKENS + tt % IMBA_PAGE_TOKENS;
          if (e < dqk) kv = to_f(P[a.g.k_off(slot, a.layer, h) + e]);
          if (e < dv) vv = to_f(P[a.g.v_off(slot, a.layer, h) + e]);
        }
      }
      kt[j * kLd + e] = kv;
      vt[j * kLd + e] = vv;
    }
    __syncthreads();
    for (int i = tid; i < kRows * kTile; i += 128) {
      const int rr = i >> 5, j = i & 31;
      float s = -INFINITY;
      if (rr < n && t0 + j < vis_s[rr]) {
        float d = 0.f;
        for (int e = 0; e < dqk; ++e) d = fmaf(qs[rr * kLd + e], kt[j * kLd + e], d);
        s = d * a.scale + psw[bias_index(t0 + j, qpos_s[rr], a.max_pos)];
      }
      pt[rr * kLdP + j] = s;
    }
    __syncthreads();
    for (int rr = warp; rr < n; rr += 4) {
      const float s = pt[rr * kLdP + lane];
      const float mold = mrow[rr];
      const float mnew = fmaxf(mold, warp_max(s));
      float p = 0.f, cr = 1.f;
      if (mnew != -INFINITY) {
        p = (s == -INFINITY) ? 0.f : expf(s - mnew);
        cr = (mold == -INFINITY) ? 0.f : expf(mold - mnew);
      }
      const float sum = warp_sum(p);
      pt[rr * kLdP + lane] = p;
      if (lane == 0) {
        lrow[rr] = lrow[rr] * cr + sum;
        mrow[rr] = mnew;
        crow[rr] = cr;
      }
    }
    __syncthreads();
    for (int i = tid; i < kRows * 64; i += 128) {
      const int rr = i >> 6, e = i & 63;
      if (rr >= n || e >= dv) continue;
      float o = acc[rr * kLd + e] * crow[rr];
#pragma unroll 8
      for (int j = 0; j < kTile; ++j) o = fmaf(pt[rr * kLdP + j], vt[j * kLd + e], o);
      acc[rr * kLd + e] = o;
    }
    __syncthreads();
  }

  // Per-row extra keys (suffix chain, then the row's own token), then finalize.
  for (int rr = warp; rr < n; rr += 4) {
    const int r = rows_s[rr];
    int e0 = st.row_extra_off[r], e1 = st.row_extra_off[r + 1];
    if (e0 < 0 || e1 < e0 || e1 > st.num_extra) {
      if (lane == 0) report(st.status, IMBA_ERR_RANGE);
      e0 = e1 = 0;
    }
    float m = mrow[rr], l = lrow[rr];
    float o0 = (lane < dv) ? acc[rr * kLd + lane] : 0.f;
    float o1 = (lane + 32 < dv) ? acc[rr * kLd + lane + 32] : 0.f;
    const float q0 = qs[rr * kLd + lane], q1 = qs[rr * kLd + lane + 32];
    for (int x = e0; x < e1; ++x) {
      const int64_t slot = st.extra_slot[x];
      if (slot < 0 || slot >= a.g.num_slots) {
        if (lane == 0) report(st.status, IMBA_ERR_RANGE);
        continue;
      }
      const T* kp = P + a.g.k_off(slot, a.layer, h);
      const T* vp = P + a.g.v_off(slot, a.layer, h);
      float d = 0.f;
      if (lane < dqk) d = q0 * to_f(kp[lane]);
      if (lane + 32 < dqk) d = fmaf(q1, to_f(kp[lane + 32]), d);
      d = warp_sum(d);
      const float s = d * a.scale + psw[bias_index(st.extra_pos[x], qpos_s[rr], a.max_pos)];
      const float mnew = fmaxf(m, s);
      const float cr = (m == -INFINITY) ? 0.f : expf(m - mnew);
      const float p = expf(s - mnew);
      l = l * cr + p;
      o0 = o0 * cr + (lane < dv ? p * to_f(vp[lane]) : 0.f);
      o1 = o1 * cr + (lane + 32 < dv ? p * to_f(vp[lane + 32]) : 0.f);
      m = mnew;
    }
    const float inv = l > 0.f ? 1.0f / l : 0.f;
    float* outr = a.out + (size_t)r * (a.g.H * dv) + h * dv;
    if (lane < dv) outr[lane] = o0 * inv;
    if (lane + 32 < dv) outr[lane + 32] = o1 * inv;
  }
}

}  // namespace

size_t attn_simt_smem_bytes() {
  return sizeof(float) * (2 * kRows * kLd + 2 * kTile * kLd + kRows * kLdP + 3 * kRows);
}

template <typename T>
cudaError_t launch_attn_simt(const AttnArgs& a, cudaStream_t s) {
  if (a.st.num_chunks <= 0) return cudaSuccess;
  const size_t smem = attn_simt_smem_bytes();
  cudaError_t e = cudaFuncSetAttribute(attn_simt_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  dim3 grid(a.st.num_chunks, a.g.H);
  return launch_pdl(attn_simt_kernel<T>, grid, dim3(128), smem, s, a);
}
template cudaError_t launch_attn_simt<float>(const AttnArgs&, cudaStream_t);
template cudaError_t launch_attn_simt<bf16>(const AttnArgs&, cudaStream_t);

}  // namespace imba
