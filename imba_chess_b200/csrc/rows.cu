// Row-wise kernels of the decode step (one warp per row, fp32 math):
//  - input LayerNorm of an STU layer (no affine, eps 1e-6), cast to the GEMM
//    operand dtype                       (src/imba_chess/model/hstu_attention.py:51-52, :309)
//  - attention-output LayerNorm (no affine, eps 1e-6) gated by u
//                                        (hstu_attention.py:54-57, :415-421)
//  - final LayerNorm (affine, eps 1e-5)  (src/imba_chess/model/hstu_model.py:245, :745)
//  - value head output layer, p(win) - p(loss), legal-id gather and the
//    legal-move log-softmax             (hstu_model.py:252-260;
//    src/imba_chess/eval/actor_server.py:168-203; actor_worker.py:267-291)
//  - dense <-> paged KV copies for one layer.
#include "common.cuh"

namespace imba {
namespace {

constexpr int kMaxPerLane = 32;  // supports row widths up to 1024

template <typename TOut>
__global__ void ln_rows_kernel(const float* __restrict__ x, int rows, int n, float eps, TOut* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= rows) return;
  const float* xr = x + (size_t)warp * n;
  float v[kMaxPerLane];
  float s = 0.f;
  const int per = (n + 31) / 32;
#pragma unroll
  for (int i = 0; i < kMaxPerLane; ++i) {
    const int c = lane + 32 * i;
    v[i] = (i < per && c < n) ? xr[c] : 0.f;
    s += v[i];
  }
  const float mu = warp_sum(s) / n;
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxPerLane; ++i) {
    const int c = lane + 32 * i;
    if (i < per && c < n) q += (v[i] - mu) * (v[i] - mu);
  }
  const float rs = 1.0f / sqrtf(warp_sum(q) / n + eps);
  TOut* o = out + (size_t)warp * n;
#pragma unroll
  for (int i = 0; i < kMaxPerLane; ++i) {
    const int c = lane + 32 * i;
    if (i < per && c < n) o[c] = from_f<TOut>((v[i] - mu) * rs);
  }
}

template <typename TOut>
__global__ void gate_kernel(const float* __restrict__ attn, const TOut* __restrict__ u, int rows, int n,
                            TOut* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= rows) return;
  const float* ar = attn + (size_t)warp * n;
  const TOut* ur = u + (size_t)warp * n;
  float v[kMaxPerLane];
  float s = 0.f;
  const int per = (n + 31) / 32;
#pragma unroll
  for (int i = 0; i < kMaxPerLane; ++i) {
    const int c = lane + 32 * i;
    v[i] = (i < per && c < n) ? ar[c] : 0.f;
    s += v[i];
  }
  const float mu = warp_sum(s) / n;
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxPerLane; ++i) {
    const int c = lane + 32 * i;
    if (i < per && c < n) q += (v[i] - mu) * (v[i] - mu);
  }
  const float rs = 1.0f / sqrtf(warp_sum(q) / n + 1e-6f);
  TOut* o = out + (size_t)warp * n;
#pragma unroll
  for (int i = 0; i < kMaxPerLane; ++i) {
    const int c = lane + 32 * i;
    if (i < per && c < n) o[c] = from_f<TOut>(to_f(ur[c]) * ((v[i] - mu) * rs));
  }
}

// Final affine LayerNorm.  Writes fp32 and, for bf16 models, the split
// operand [hi | lo | hi] (hi = bf16(y), lo = bf16(y - hi)) of the
// split-precision policy GEMM; its first n columns are the value head's input.
template <typename T>
__global__ void final_ln_kernel(const float* __restrict__ x, int rows, int n, const float* __restrict__ w,
                                const float* __restrict__ b, float* __restrict__ out32, T* __restrict__ out3) {
  pdl_wait();
  pdl_trigger();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= rows) return;
  const float* xr = x + (size_t)warp * n;
  float v[kMaxPerLane];
  float s = 0.f;
  const int per = (n + 31) / 32;
#pragma unroll
  for (int i = 0; i < kMaxPerLane; ++i) {
    const int c = lane + 32 * i;
    v[i] = (i < per && c < n) ? xr[c] : 0.f;
    s += v[i];
  }
  const float mu = warp_sum(s) / n;
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxPerLane; ++i) {
    const int c = lane + 32 * i;
    if (i < per && c < n) q += (v[i] - mu) * (v[i] - mu);
  }
  const float rs = 1.0f / sqrtf(warp_sum(q) / n + 1e-5f);
#pragma unroll
  for (int i = 0; i < kMaxPerLane; ++i) {
    const int c = lane + 32 * i;
    if (i < per && c < n) {
      const float y = (v[i] - mu) * rs * w[c] + b[c];
      const size_t o = (size_t)warp * n + c;
      out32[o] = y;
      if (out3) {
        const T hi = from_f<T>(y);
        T* r3 = out3 + (size_t)warp * 3 * n;
        r3[c] = hi;
        r3[n + c] = from_f<T>(y - to_f(hi));
        r3[2 * n + c] = hi;
      }
    }
  }
}

// ---- 128-bit variants (row width a multiple of 128, at most 1024) --------
// Lane l holds columns 128 i + 4 l .. +3 for i < n / 128.
constexpr int kMaxVec = 8;

__device__ __forceinline__ float4 load4(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ float4 load4(const bf16* p) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  const float2 lo = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
  const float2 hi = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
  return make_float4(lo.x, lo.y, hi.x, hi.y);
}
__device__ __forceinline__ void store4(float* p, float a, float b, float c, float d) {
  *reinterpret_cast<float4*>(p) = make_float4(a, b, c, d);
}
__device__ __forceinline__ void store4(bf16* p, float a, float b, float c, float d) {
  __nv_bfloat162 lo = __floats2bfloat162_rn(a, b), hi = __floats2bfloat162_rn(c, d);
  uint2 u;
  u.x = *reinterpret_cast<uint32_t*>(&lo);
  u.y = *reinterpret_cast<uint32_t*>(&hi);
  *reinterpret_cast<uint2*>(p) = u;
}

// mean and 1/sqrt(var + eps) of a row held as float4 chunks.
__device__ __forceinline__ void row_stats4(const float4 (&v)[kMaxVec], int nv, int n, float eps, float& mu,
                                           float& rs) {
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxVec; ++i)
    if (i < nv) s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
  mu = warp_sum(s) / n;
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxVec; ++i)
    if (i < nv) {
      const float a = v[i].x - mu, b = v[i].y - mu, c = v[i].z - mu, d = v[i].w - mu;
      q += (a * a + b * b) + (c * c + d * d);
    }
  rs = 1.0f / sqrtf(warp_sum(q) / n + eps);
}

template <typename TOut>
__global__ void ln_rows4_kernel(const float* __restrict__ x, int rows, int n, float eps, TOut* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= rows) return;
  const int nv = n >> 7;
  const float* xr = x + (size_t)warp * n + 4 * lane;
  float4 v[kMaxVec];
#pragma unroll
  for (int i = 0; i < kMaxVec; ++i)
    if (i < nv) v[i] = *reinterpret_cast<const float4*>(xr + 128 * i);
  float mu, rs;
  row_stats4(v, nv, n, eps, mu, rs);
  TOut* o = out + (size_t)warp * n + 4 * lane;
#pragma unroll
  for (int i = 0; i < kMaxVec; ++i)
    if (i < nv)
      store4(o + 128 * i, (v[i].x - mu) * rs, (v[i].y - mu) * rs, (v[i].z - mu) * rs, (v[i].w - mu) * rs);
}

template <typename TIn, typename TOut>
__global__ void gate4_kernel(const TIn* __restrict__ attn, const TOut* __restrict__ u, int rows, int n,
                             TOut* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= rows) return;
  const int nv = n >> 7;
  const TIn* ar = attn + (size_t)warp * n + 4 * lane;
  const TOut* ur = u + (size_t)warp * n + 4 * lane;
  float4 v[kMaxVec], w[kMaxVec];
#pragma unroll
  for (int i = 0; i < kMaxVec; ++i)
    if (i < nv) {
      v[i] = load4(ar + 128 * i);
      w[i] = load4(ur + 128 * i);
    }
  float mu, rs;
  row_stats4(v, nv, n, 1e-6f, mu, rs);
  TOut* o = out + (size_t)warp * n + 4 * lane;
#pragma unroll
  for (int i = 0; i < kMaxVec; ++i)
    if (i < nv)
      store4(o + 128 * i, w[i].x * ((v[i].x - mu) * rs), w[i].y * ((v[i].y - mu) * rs),
             w[i].z * ((v[i].z - mu) * rs), w[i].w * ((v[i].w - mu) * rs));
}

template <typename T>
__global__ void final_ln4_kernel(const float* __restrict__ x, int rows, int n, const float* __restrict__ w,
                                 const float* __restrict__ b, float* __restrict__ out32, T* __restrict__ out3) {
  pdl_wait();
  pdl_trigger();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= rows) return;
  const int nv = n >> 7;
  const float* xr = x + (size_t)warp * n + 4 * lane;
  float4 v[kMaxVec];
#pragma unroll
  for (int i = 0; i < kMaxVec; ++i)
    if (i < nv) v[i] = *reinterpret_cast<const float4*>(xr + 128 * i);
  float mu, rs;
  row_stats4(v, nv, n, 1e-5f, mu, rs);
#pragma unroll
  for (int i = 0; i < kMaxVec; ++i)
    if (i < nv) {
      const int c = 128 * i + 4 * lane;
      const float4 wv = *reinterpret_cast<const float4*>(w + c);
      const float4 bv = *reinterpret_cast<const float4*>(b + c);
      const float y0 = (v[i].x - mu) * rs * wv.x + bv.x, y1 = (v[i].y - mu) * rs * wv.y + bv.y;
      const float y2 = (v[i].z - mu) * rs * wv.z + bv.z, y3 = (v[i].w - mu) * rs * wv.w + bv.w;
      store4(out32 + (size_t)warp * n + c, y0, y1, y2, y3);
      if (out3) {
        T* r3 = out3 + (size_t)warp * 3 * n + c;
        const float h0 = to_f(from_f<T>(y0)), h1 = to_f(from_f<T>(y1)), h2 = to_f(from_f<T>(y2)),
                    h3 = to_f(from_f<T>(y3));
        store4(r3, h0, h1, h2, h3);
        store4(r3 + n, y0 - h0, y1 - h1, y2 - h2, y3 - h3);
        store4(r3 + 2 * n, h0, h1, h2, h3);
      }
    }
}

// Value output layer + v + legal projection, one warp per row.  With
// logits == nullptr the row's legal logits are computed here as exact fp32
// dot products of the final-LN output x32 with the fp32 policy rows of the
// legal ids (the reference's _gather_legal_logits,
// src/imba_chess/eval/actor_server.py:176-203, only reads those entries of
// the full projection), staged in scratch[r * vocab ..].
__global__ void value_legal_kernel(imba_model_desc md, imba_step_desc st, const float* __restrict__ hval,
                                   const float* __restrict__ logits, const float* __restrict__ x32,
                                   float* __restrict__ scratch) {
  pdl_wait();
  pdl_trigger();
  const int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (r >= st.num_rows) return;
  if (md.has_value_head) {
    const int hd = md.model_dim / 2;
    const float* hr = hval + (size_t)r * hd;
    float z[3];
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      float a = 0.f;
      for (int c = lane; c < hd; c += 32) a = fmaf(hr[c], md.value2_w[(size_t)j * hd + c], a);
      z[j] = warp_sum(a) + md.value2_b[j];
    }
    if (lane == 0) {
      if (st.value_logits) {
        st.value_logits[(size_t)r * 3 + 0] = z[0];
        st.value_logits[(size_t)r * 3 + 1] = z[1];
        st.value_logits[(size_t)r * 3 + 2] = z[2];
      }
      if (st.value_stm) {
        const float m = fmaxf(z[0], fmaxf(z[1], z[2]));
        const float e0 = expf(z[0] - m), e1 = expf(z[1] - m), e2 = expf(z[2] - m);
        const float sum = e0 + e1 + e2;
        st.value_stm[r] = e2 / sum - e0 / sum;
      }
    }
  } else if (lane == 0) {
    // No value head: the reference serves a zero placeholder (uniform softmax, v = 0).
    if (st.value_logits) {
      st.value_logits[(size_t)r * 3 + 0] = 0.f;
      st.value_logits[(size_t)r * 3 + 1] = 0.f;
      st.value_logits[(size_t)r * 3 + 2] = 0.f;
    }
    if (st.value_stm) st.value_stm[r] = 0.f;
  }
  if (!st.legal_off) return;
  const int a = st.legal_off[r], b = st.legal_off[r + 1];
  if (a < 0 || b < a || b > st.num_legal) {
    if (lane == 0) report(st.status, IMBA_ERR_RANGE);
    return;
  }
  const bool gather = logits == nullptr;
  float* sr = scratch + (size_t)r * md.vocab;  // gather mode: legal logit of entry i at sr[i - a]
  if (gather) {
    const int d = md.model_dim;
    const float* xr = x32 + (size_t)r * d;
    const float* W = md.policy_w32;
    const bool vec = (d & 127) == 0 && d <= 128 * kMaxVec;
    float4 xv[kMaxVec];
#pragma unroll
    for (int k = 0; k < kMaxVec; ++k)
      xv[k] = vec && 128 * k < d ? *reinterpret_cast<const float4*>(xr + 128 * k + 4 * lane) : make_float4(0, 0, 0, 0);
    for (int base = a; base < b; base += 4) {  // four legal ids per round, their loads in flight together
      const float* wr[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        wr[q] = nullptr;
        if (base + q < b) {
          int id = st.legal_ids[base + q];
          if (id < 0 || id >= md.vocab) {
            if (lane == 0) report(st.status, IMBA_ERR_RANGE);
            id = 0;
          }
          wr[q] = W + (size_t)id * d;
        }
      }
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
      if (vec) {
#pragma unroll
        for (int k = 0; k < kMaxVec; ++k) {
          if (128 * k >= d) break;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            if (!wr[q]) continue;
            const float4 w = __ldg(reinterpret_cast<const float4*>(wr[q] + 128 * k + 4 * lane));
            acc[q] = fmaf(xv[k].x, w.x, fmaf(xv[k].y, w.y, fmaf(xv[k].z, w.z, fmaf(xv[k].w, w.w, acc[q]))));
          }
        }
      } else {
        for (int c = lane; c < d; c += 32) {
          const float xc = xr[c];
#pragma unroll
          for (int q = 0; q < 4; ++q)
            if (wr[q]) acc[q] = fmaf(xc, __ldg(wr[q] + c), acc[q]);
        }
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) acc[q] = warp_sum(acc[q]);
      if (lane == 0) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          if (base + q >= b) break;
          sr[base + q - a] = acc[q];
          if (st.legal_logits) st.legal_logits[base + q] = acc[q];
        }
      }
    }
    __syncwarp();
  }
  const float* lr = logits + (size_t)r * md.vocab;
  auto legal_logit = [&](int i) -> float {
    if (gather) return sr[i - a];
    int id = st.legal_ids[i];
    id = (id < 0 || id >= md.vocab) ? 0 : id;
    return lr[id];
  };
  float mx = -INFINITY;
  for (int i = a + lane; i < b; i += 32) {
    if (!gather) {
      const int id = st.legal_ids[i];
      if (id < 0 || id >= md.vocab) report(st.status, IMBA_ERR_RANGE);
    }
    const float v = legal_logit(i);
    if (st.legal_logits && !gather) st.legal_logits[i] = v;
    mx = fmaxf(mx, v);
  }
  mx = warp_max(mx);
  if (!st.legal_logprob || b == a) return;
  double se = 0.0;
  for (int i = a + lane; i < b; i += 32) se += exp((double)legal_logit(i) - (double)mx);
  const double lse = log(warp_sum_d(se));
  for (int i = a + lane; i < b; i += 32) st.legal_logprob[i] = (float)(((double)legal_logit(i) - (double)mx) - lse);
}

template <typename T>
__global__ void kv_copy_kernel(PoolGeom g, T* pool, int layer, int n, const int32_t* __restrict__ slots,
                               T* dk, T* dv, int to_pool, int32_t* status) {
  const int r = blockIdx.x;
  if (r >= n) return;
  const int64_t slot = slots[r];
  if (slot < 0 || slot >= g.num_slots) {
    if (threadIdx.x == 0) report(status, IMBA_ERR_RANGE);
    return;
  }
  const int nk = g.H * g.dqk, nv = g.H * g.dv;
  for (int i = threadIdx.x; i < nk + nv; i += blockDim.x) {
    if (i < nk) {
      const int h = i / g.dqk, e = i % g.dqk;
      T* p = pool + g.k_off(slot, layer, h) + e;
      T* q = dk + (size_t)r * nk + i;
      if (to_pool) *p = *q; else *q = *p;
    } else {
      const int j = i - nk, h = j / g.dv, e = j % g.dv;
      T* p = pool + g.v_off(slot, layer, h) + e;
      T* q = dv + (size_t)r * nv + j;
      if (to_pool) *p = *q; else *q = *p;
    }
  }
}

// Dense strided K / V rows -> pool slots: row r's element (h, e) comes from
// src[a[r] * s[0] + b[r] * s[1] + h * s[2] + e * s[3]] (elements).  One CTA
// per row.
template <typename T>
__global__ void kv_scatter_indexed_kernel(PoolGeom g, T* pool, int layer, int n, const int32_t* __restrict__ slots,
                                          const int32_t* __restrict__ ia, const int32_t* __restrict__ ib,
                                          const T* __restrict__ sk, const T* __restrict__ sv, KVStrides st,
                                          int32_t* status) {
  const int r = blockIdx.x;
  if (r >= n) return;
  const int64_t slot = slots[r];
  if (slot < 0 || slot >= g.num_slots) {
    if (threadIdx.x == 0) report(status, IMBA_ERR_RANGE);
    return;
  }
  const int64_t a = ia[r], b = ib[r];
  const int nk = g.H * g.dqk, nv = g.H * g.dv;
  for (int i = threadIdx.x; i < nk + nv; i += blockDim.x) {
    if (i < nk) {
      const int h = i / g.dqk, e = i % g.dqk;
      pool[g.k_off(slot, layer, h) + e] = sk[a * st.k[0] + b * st.k[1] + h * st.k[2] + e * st.k[3]];
    } else {
      const int j = i - nk, h = j / g.dv, e = j % g.dv;
      pool[g.v_off(slot, layer, h) + e] = sv[a * st.v[0] + b * st.v[1] + h * st.v[2] + e * st.v[3]];
    }
  }
}

inline int warp_blocks(int rows) { return (rows + 7) / 8; }  // 8 warps per 256-thread block

}  // namespace

template <typename T>
cudaError_t launch_ln_rows(const float* x, int rows, int n, float eps, T* out, cudaStream_t s) {
  if (n % 128 == 0 && n <= 128 * kMaxVec)
    return launch_pdl(ln_rows4_kernel<T>, dim3(warp_blocks(rows)), dim3(256), 0, s, x, rows, n, eps, out);
  return launch_pdl(ln_rows_kernel<T>, dim3(warp_blocks(rows)), dim3(256), 0, s, x, rows, n, eps, out);
}
template cudaError_t launch_ln_rows<float>(const float*, int, int, float, float*, cudaStream_t);
template cudaError_t launch_ln_rows<bf16>(const float*, int, int, float, bf16*, cudaStream_t);

template <typename T>
cudaError_t launch_gate(const float* attn, const T* u, int rows, int n, T* out, cudaStream_t s) {
  if (n % 128 == 0 && n <= 128 * kMaxVec)
    return launch_pdl(gate4_kernel<float, T>, dim3(warp_blocks(rows)), dim3(256), 0, s, attn, u, rows, n, out);
  return launch_pdl(gate_kernel<T>, dim3(warp_blocks(rows)), dim3(256), 0, s, attn, u, rows, n, out);
}
template cudaError_t launch_gate<float>(const float*, const float*, int, int, float*, cudaStream_t);
template cudaError_t launch_gate<bf16>(const float*, const bf16*, int, int, bf16*, cudaStream_t);

cudaError_t launch_gate_bf16(const bf16* attn, const bf16* u, int rows, int n, bf16* out, cudaStream_t s) {
  if (n % 128 || n > 128 * kMaxVec) return cudaErrorInvalidValue;
  return launch_pdl(gate4_kernel<bf16, bf16>, dim3(warp_blocks(rows)), dim3(256), 0, s, attn, u, rows, n, out);
}

template <typename T>
cudaError_t launch_final_ln(const float* x, int rows, int n, const float* w, const float* b, float* out32, T* out3,
                            cudaStream_t s) {
  if (n % 128 == 0 && n <= 128 * kMaxVec)
    return launch_pdl(final_ln4_kernel<T>, dim3(warp_blocks(rows)), dim3(256), 0, s, x, rows, n, w, b, out32, out3);
  return launch_pdl(final_ln_kernel<T>, dim3(warp_blocks(rows)), dim3(256), 0, s, x, rows, n, w, b, out32, out3);
}
template cudaError_t launch_final_ln<float>(const float*, int, int, const float*, const float*, float*, float*,
                                            cudaStream_t);
template cudaError_t launch_final_ln<bf16>(const float*, int, int, const float*, const float*, float*, bf16*,
                                           cudaStream_t);

cudaError_t launch_value_legal(const imba_model_desc& md, const imba_step_desc& st, const float* hval,
                               const float* logits, const float* x32, float* scratch, cudaStream_t s) {
  return launch_pdl(value_legal_kernel, dim3(warp_blocks(st.num_rows)), dim3(256), 0, s, md, st, hval, logits, x32,
                    scratch);
}

template <typename T>
cudaError_t launch_kv_copy(const PoolGeom& g, T* pool, int layer, int n, const int32_t* slots, T* dk, T* dv,
                           int to_pool, int32_t* status, cudaStream_t s) {
  kv_copy_kernel<T><<<n, 128, 0, s>>>(g, pool, layer, n, slots, dk, dv, to_pool, status);
  return cudaGetLastError();
}
template cudaError_t launch_kv_copy<float>(const PoolGeom&, float*, int, int, const int32_t*, float*, float*, int,
                                           int32_t*, cudaStream_t);

template <typename T>
cudaError_t launch_kv_scatter_indexed(const PoolGeom& g, T* pool, int layer, int n, const int32_t* slots,
                                      const int32_t* ia, const int32_t* ib, const T* sk, const T* sv,
                                      const KVStrides& st, int32_t* status, cudaStream_t s) {
  kv_scatter_indexed_kernel<T><<<n, 128, 0, s>>>(g, pool, layer, n, slots, ia, ib, sk, sv, st, status);
  return cudaGetLastError();
}
template cudaError_t launch_kv_scatter_indexed<float>(const PoolGeom&, float*, int, int, const int32_t*,
                                                      const int32_t*, const int32_t*, const float*, const float*,
                                                      const KVStrides&, int32_t*, cudaStream_t);
template cudaError_t launch_kv_scatter_indexed<bf16>(const PoolGeom&, bf16*, int, int, const int32_t*, const int32_t*,
                                                     const int32_t*, const bf16*, const bf16*, const KVStrides&,
                                                     int32_t*, cudaStream_t);
template cudaError_t launch_kv_copy<bf16>(const PoolGeom&, bf16*, int, int, const int32_t*, bf16*, bf16*, int,
                                          int32_t*, cudaStream_t);

}  // namespace imba
