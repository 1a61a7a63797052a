// GEMM epilogues of the decode step.  Every GEMM computes
//   acc[r, c] = sum_k A[r, k] * W[c, k]      (W in nn.Linear [out, in] layout)
// and hands each fp32 accumulator to one of these functors.
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace imba {

// Store 32 consecutive values (16-byte aligned destination) as 128-bit stores.
__device__ __forceinline__ void store32(float* dst, const float (&v)[32]) {
  float4* d = reinterpret_cast<float4*>(dst);
#pragma unroll
  for (int i = 0; i < 8; ++i) d[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
}
__device__ __forceinline__ void store32(bf16* dst, const float (&v)[32]) {
  uint32_t w[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
    w[i] = *reinterpret_cast<uint32_t*>(&h);
  }
  uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int i = 0; i < 4; ++i) d[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
}

// Staged epilogues (kStaged): the tensor-core GEMM hands each epilogue warp
// a 32 x 32 accumulator chunk (rows row0 .. row0 + 31, columns c0 .. c0 + 31)
// in shared memory, element (r, c) at s[r * 32 + (c ^ r)] (conflict-free for
// both the row-per-lane writes and the reads below), plus one per-row tag.
// Lane l takes columns 4 (l & 7) .. +3 of rows (l >> 3) + 4 k, k = 0..7, so
// the eight lanes of a row group write one row's 32 columns contiguously:
// one or two full lines per row instead of eight 16-byte pieces from eight
// different rows per instruction.
__device__ __forceinline__ float4 staged4(const float* s, int r, int c4) {
  return make_float4(s[r * 32 + ((c4) ^ r)], s[r * 32 + ((c4 + 1) ^ r)], s[r * 32 + ((c4 + 2) ^ r)],
                     s[r * 32 + ((c4 + 3) ^ r)]);
}
__device__ __forceinline__ void put4(float* p, float a, float b, float c, float d) {
  *reinterpret_cast<float4*>(p) = make_float4(a, b, c, d);
}
__device__ __forceinline__ void put4(bf16* p, float a, float b, float c, float d) {
  __nv_bfloat162 lo = __floats2bfloat162_rn(a, b), hi = __floats2bfloat162_rn(c, d);
  uint2 v;
  v.x = *reinterpret_cast<uint32_t*>(&lo);
  v.y = *reinterpret_cast<uint32_t*>(&hi);
  *reinterpret_cast<uint2*>(p) = v;
}

// uvqk projection epilogue: SiLU, then the reference's split order u | v | q | k
// (src/imba_chess/model/hstu_attention.py:310-325).  u goes to the gate input
// buffer, q to the query buffer (both in the model dtype), and k / v straight
// into the row's slot of the paged KV pool (the KV append, fused).
template <typename T>
struct EpiUVQK {
  T* u;
  T* q;
  T* pool;
  const int32_t* dst_slot;
  PoolGeom g;
  int layer;
  int32_t* status;
  // Tensor-core path (bf16): u and q are written as [32 rows x 64 columns]
  // boxes by TMA stores from a 128-byte-swizzled staging tile (bf16 [R, H dv]
  // and [R, H dqk], encoded per launch); v and k go to the pool per thread.
  CUtensorMap u_map, q_map;
  static constexpr bool kBoxStore = true;
  // 1: column c0 lies in u, 2: in q, 0: in v or k (pool rows).
  __device__ __forceinline__ int box_region(int c0) const {
    const int hdv = g.H * g.dv, hdq = g.H * g.dqk;
    if (c0 < hdv) return 1;
    if (c0 >= 2 * hdv && c0 < 2 * hdv + hdq) return 2;
    return 0;
  }
  __device__ __forceinline__ const CUtensorMap* box_map(int region) const { return region == 1 ? &u_map : &q_map; }
  __device__ __forceinline__ int box_x(int region, int c0) const {
    return region == 1 ? c0 : c0 - 2 * g.H * g.dv;
  }
  // SiLU of one row's 32 columns (thread = row = lane of the box), as bf16
  // into 16-byte chunks 4 h .. 4 h + 3 of the row's 128 bytes, 128-byte
  // swizzle (chunk j of row r at j ^ (r % 8)).
  __device__ __forceinline__ void box_stage32(uint8_t* box, int h, const float (&a)[32], int lane) const {
    const uint32_t base = static_cast<uint32_t>(__cvta_generic_to_shared(box)) + lane * 128;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint32_t w[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        __nv_bfloat162 p = __floats2bfloat162_rn(silu_tanh(a[8 * j + 2 * k]), silu_tanh(a[8 * j + 2 * k + 1]));
        w[k] = *reinterpret_cast<uint32_t*>(&p);
      }
      const uint32_t dst = base + ((((uint32_t)(4 * h + j)) ^ (uint32_t)(lane & 7)) << 4);
      asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(dst), "r"(w[0]), "r"(w[1]), "r"(w[2]), "r"(w[3])
                   : "memory");
    }
  }

  __device__ __forceinline__ void operator()(int r, int c, float acc) const {
    const float y = silu_f(acc);
    const int hdv = g.H * g.dv, hdq = g.H * g.dqk;
    if (c < hdv) {
      u[(size_t)r * hdv + c] = from_f<T>(y);
      return;
    }
    c -= hdv;
    if (c < hdv) {
      const int64_t slot = dst_slot[r];
      if (slot < 0 || slot >= g.num_slots) {
        report(status, IMBA_ERR_RANGE);
        return;
      }
      pool[g.v_off(slot, layer, c / g.dv) + (c % g.dv)] = from_f<T>(y);
      return;
    }
    c -= hdv;
    if (c < hdq) {
      q[(size_t)r * hdq + c] = from_f<T>(y);
      return;
    }
    c -= hdq;
    const int64_t slot = dst_slot[r];
    if (slot < 0 || slot >= g.num_slots) {
      report(status, IMBA_ERR_RANGE);
      return;
    }
    pool[g.k_off(slot, layer, c / g.dqk) + (c % g.dqk)] = from_f<T>(y);
  }

  // Per-row state of the tensor-core epilogue: the row's KV slot, loaded once per tile.
  struct Ctx {
    int64_t slot;
  };
  __device__ __forceinline__ Ctx begin(int r, int /*n0*/, int /*bn*/) const { return Ctx{(int64_t)dst_slot[r]}; }

  // Per-thread rows (kStaged false): a staged 32 x 32 chunk variant of this
  // epilogue measured slower (its stores are 64-128 B per row and chunk; the
  // staging round trip and the per-row slot lookups cost more than they save).
  static constexpr bool kStaged = false;

  // 32 consecutive columns starting at c0 (a multiple of 32; d_qk and d_v
  // are multiples of 32, so a chunk never straddles a head or a region).
  __device__ __forceinline__ void chunk32(const Ctx& cx, int r, int c0, int N, const float (&a)[32]) const {
    if (c0 >= N) return;
    float y[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) y[i] = silu_tanh(a[i]);
    const int hdv = g.H * g.dv, hdq = g.H * g.dqk;
    if (c0 < hdv) {
      store32(u + (size_t)r * hdv + c0, y);
      return;
    }
    int c = c0 - hdv;
    if (c >= hdv && c - hdv < hdq) {
      store32(q + (size_t)r * hdq + (c - hdv), y);
      return;
    }
    const int64_t slot = cx.slot;
    if (slot < 0 || slot >= g.num_slots) {
      report(status, IMBA_ERR_RANGE);
      return;
    }
    if (c < hdv) {
      store32(pool + g.v_off(slot, layer, c / g.dv) + (c % g.dv), y);
    } else {
      c -= hdv + hdq;
      store32(pool + g.k_off(slot, layer, c / g.dqk) + (c % g.dqk), y);
    }
  }
};

// Output projection epilogue: x = (acc + bias) + x   (hstu_attention.py:423)
struct EpiResidual {
  float* x;
  const float* bias;
  int ld;
  __device__ __forceinline__ void operator()(int r, int c, float acc) const {
    float* p = x + (size_t)r * ld + c;
    *p = (acc + bias[c]) + *p;
  }
  // The tile's residual lines are prefetched into L1 when the row starts.
  struct Ctx {};
  __device__ __forceinline__ Ctx begin(int r, int n0, int bn) const {
    const float* p = x + (size_t)r * ld + n0;
    for (int c = 0; c < bn && n0 + c < ld; c += 32)
      asm volatile("prefetch.global.L1 [%0];" ::"l"(p + c));
    return Ctx{};
  }
  static constexpr bool kStaged = true;
  static constexpr bool kBoxStore = false;
  __device__ __forceinline__ int row_tag(int) const { return 0; }
  // Staged chunk (see staged4): all residual and bias loads are issued
  // before any store (the compiler cannot prove x and bias do not alias).
  __device__ __forceinline__ void tile32(const float* s, const int*, int row0, int c0, int M, int N,
                                         int lane) const {
    if (c0 >= N) return;
    const int cg = 4 * (lane & 7), r4 = lane >> 3;
    const float4 b = __ldg(reinterpret_cast<const float4*>(bias + c0 + cg));
    float* xc = x + (size_t)(row0 + r4) * ld + c0 + cg;  // row r4 of the chunk; rows step by 4
#pragma unroll 1
    for (int k0 = 0; k0 < 8; k0 += 4) {  // two batches of four rows (bounded register use)
      float4 xv[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int row = row0 + r4 + 4 * (k0 + k);
        xv[k] = row < M ? *reinterpret_cast<const float4*>(xc + (size_t)(4 * (k0 + k)) * ld) : make_float4(0, 0, 0, 0);
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int rr = r4 + 4 * (k0 + k), row = row0 + rr;
        if (row >= M) continue;
        const float4 a = staged4(s, rr, cg);
        put4(xc + (size_t)(4 * (k0 + k)) * ld, (a.x + b.x) + xv[k].x, (a.y + b.y) + xv[k].y, (a.z + b.z) + xv[k].z,
             (a.w + b.w) + xv[k].w);
      }
    }
  }
  // All loads are issued before any store: interleaving each load after the
  // previous store of the same row serialises them (the compiler cannot prove
  // x and bias do not alias) and was measured ~30x slower.
  __device__ __forceinline__ void chunk32(const Ctx&, int r, int c0, int N, const float (&a)[32]) const {
    if (c0 >= N) return;
    float4* p = reinterpret_cast<float4*>(x + (size_t)r * ld + c0);
    const float4* b = reinterpret_cast<const float4*>(bias + c0);
    float4 xv[8], bv[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      xv[i] = p[i];
      bv[i] = __ldg(b + i);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      xv[i].x = (a[4 * i] + bv[i].x) + xv[i].x;
      xv[i].y = (a[4 * i + 1] + bv[i].y) + xv[i].y;
      xv[i].z = (a[4 * i + 2] + bv[i].z) + xv[i].z;
      xv[i].w = (a[4 * i + 3] + bv[i].w) + xv[i].w;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) p[i] = xv[i];
  }
};

struct EpiStore {
  static constexpr bool kStaged = false;
  static constexpr bool kBoxStore = false;
  float* out;
  int ld;
  __device__ __forceinline__ void operator()(int r, int c, float acc) const { out[(size_t)r * ld + c] = acc; }
  struct Ctx {};
  __device__ __forceinline__ Ctx begin(int, int, int) const { return Ctx{}; }
  // The policy row stride (vocab floats) is even but not a multiple of 4:
  // full chunks use 8-byte stores, the ragged last chunk scalar stores.
  __device__ __forceinline__ void chunk32(const Ctx&, int r, int c0, int N, const float (&a)[32]) const {
    float* o = out + (size_t)r * ld + c0;
    if (c0 + 32 <= N && ((reinterpret_cast<uintptr_t>(o) & 7) == 0)) {
      float2* o2 = reinterpret_cast<float2*>(o);
#pragma unroll
      for (int i = 0; i < 16; ++i) o2[i] = make_float2(a[2 * i], a[2 * i + 1]);
      return;
    }
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (c0 + i < N) o[i] = a[i];
  }
};

// Adds into an existing fp32 output (split-precision passes).
struct EpiAccumulate {
  float* out;
  int ld;
  __device__ __forceinline__ void operator()(int r, int c, float acc) const { out[(size_t)r * ld + c] += acc; }
};

// Value-head hidden layer: SiLU(acc + bias)   (hstu_model.py:252-257)
struct EpiBiasSilu {
  static constexpr bool kBoxStore = false;
  static constexpr bool kStaged = false;
  float* out;
  const float* bias;
  int ld;
  __device__ __forceinline__ void operator()(int r, int c, float acc) const {
    out[(size_t)r * ld + c] = silu_f(acc + bias[c]);
  }
  struct Ctx {};
  __device__ __forceinline__ Ctx begin(int, int, int) const { return Ctx{}; }
  __device__ __forceinline__ void chunk32(const Ctx&, int r, int c0, int N, const float (&a)[32]) const {
    if (c0 >= N) return;
    float y[32];
    const float4* b = reinterpret_cast<const float4*>(bias + c0);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 bv = __ldg(b + i);
      y[4 * i] = silu_f(a[4 * i] + bv.x);
      y[4 * i + 1] = silu_f(a[4 * i + 1] + bv.y);
      y[4 * i + 2] = silu_f(a[4 * i + 2] + bv.z);
      y[4 * i + 3] = silu_f(a[4 * i + 3] + bv.w);
    }
    store32(out + (size_t)r * ld + c0, y);
  }
};

// Content embedding epilogue (bf16 models): acc = pooled . board_out^T, then
// x = (acc + b_out + seq + turn + castle + ep + halfmove + fullmove + prev_move)
//     * sqrt(d) + pos_emb[min(pos, max_pos - 1)]
// with side ids clamped to their tables (hstu_model.py:275-335;
// position_embedding.py:52-62).
struct EpiContent {
  float* x;
  const imba_model_desc* md;  // device copy not needed: pointers and sizes only
  const float* bias;
  const float *seq, *turn, *castle, *ep, *half, *full, *prev, *pos_emb;
  const int32_t* side_ids;
  const int32_t* positions;
  int d, halfmove_vocab, fullmove_vocab, vocab, max_pos;
  float scale;
  int32_t* status;

  static constexpr bool kStaged = false;
  static constexpr bool kBoxStore = false;
  __device__ __forceinline__ static int clampi(int v, int n) { return v < 0 ? 0 : (v >= n ? n - 1 : v); }
  // Tensor-core epilogue: the row's seven side-embedding rows and its
  // position row, resolved once per tile.
  struct Ctx {
    const float* e[7];
    const float* pos;
  };
  __device__ __forceinline__ Ctx begin(int r, int, int) const {
    const int32_t* ids = side_ids + (size_t)r * IMBA_NUM_SIDE_IDS;
    Ctx cx;
    cx.e[0] = seq + (size_t)clampi(ids[0], 2) * d;
    cx.e[1] = turn + (size_t)clampi(ids[1], 2) * d;
    cx.e[2] = castle + (size_t)clampi(ids[2], 16) * d;
    cx.e[3] = ep + (size_t)clampi(ids[3], 9) * d;
    cx.e[4] = half + (size_t)clampi(ids[4], halfmove_vocab) * d;
    cx.e[5] = full + (size_t)clampi(ids[5], fullmove_vocab) * d;
    cx.e[6] = prev + (size_t)clampi(ids[6], vocab) * d;
    int p = positions[r];
    if (p < 0) {
      report(status, IMBA_ERR_RANGE);
      p = 0;
    }
    if (p > max_pos - 1) p = max_pos - 1;
    cx.pos = pos_emb + (size_t)p * d;
    return cx;
  }
  // 32 columns of one row, in the same summation order as operator(); the
  // tables are read through the read-only path (never written by a step).
  __device__ __forceinline__ void chunk32(const Ctx& cx, int r, int c0, int N, const float (&a)[32]) const {
    if (c0 >= N) return;
    float* xr = x + (size_t)r * d + c0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int c = c0 + 4 * i;
      const float4 b = __ldg(reinterpret_cast<const float4*>(bias + c));
      float4 v = make_float4(a[4 * i] + b.x, a[4 * i + 1] + b.y, a[4 * i + 2] + b.z, a[4 * i + 3] + b.w);
#pragma unroll
      for (int k = 0; k < 7; ++k) {
        const float4 e = __ldg(reinterpret_cast<const float4*>(cx.e[k] + c));
        v.x += e.x;
        v.y += e.y;
        v.z += e.z;
        v.w += e.w;
      }
      const float4 pe = __ldg(reinterpret_cast<const float4*>(cx.pos + c));
      *reinterpret_cast<float4*>(xr + 4 * i) =
          make_float4(v.x * scale + pe.x, v.y * scale + pe.y, v.z * scale + pe.z, v.w * scale + pe.w);
    }
  }
  __device__ __forceinline__ void operator()(int r, int c, float acc) const {
    const int32_t* ids = side_ids + (size_t)r * IMBA_NUM_SIDE_IDS;
    float v = acc + bias[c];
    v += seq[(size_t)clampi(ids[0], 2) * d + c];
    v += turn[(size_t)clampi(ids[1], 2) * d + c];
    v += castle[(size_t)clampi(ids[2], 16) * d + c];
    v += ep[(size_t)clampi(ids[3], 9) * d + c];
    v += half[(size_t)clampi(ids[4], halfmove_vocab) * d + c];
    v += full[(size_t)clampi(ids[5], fullmove_vocab) * d + c];
    v += prev[(size_t)clampi(ids[6], vocab) * d + c];
    int p = positions[r];
    if (p < 0) {
      report(status, IMBA_ERR_RANGE);
      p = 0;
    }
    if (p > max_pos - 1) p = max_pos - 1;
    x[(size_t)r * d + c] = v * scale + pos_emb[(size_t)p * d + c];
  }
};

}  // namespace imba
