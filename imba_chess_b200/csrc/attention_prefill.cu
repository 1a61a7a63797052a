// Jagged prefill attention on the tcgen05 tensor cores (bf16 models,
// d_qk = d_v = 64).  It serves the steps whose rows find all their keys in
// their groups' pages (no extra keys): a prefill of whole documents packed
// into one jagged batch, where row i of a document sees the document's keys
// up to its own position, with the relative-position bias.
//
// Work units.  A unit is one chunk (<= 64 consecutive rows of one group,
// described by the item pass's two 32-row records) and one pair of heads.
// The unit's tensor-core tiles stack the pair: rows 0-63 of the M = 128 tile
// are the chunk's rows for the first head, rows 64-127 for the second.
//   S' = Q' K'^T  Q' [128 x 64 dims]; K' [64 x 64 dims] = two pages' keys of
//                 both heads, column 32 p + 16 hh + t = token t of page p for
//                 head hh (one TMA box per page covers both heads' rows).
//   O' += P' V'   P' [128 x 64] bf16, a row non-zero only in its own head's
//                 columns; V' [64 keys' x 64 dims] in the same key order,
//                 read as an MN-major operand; O' accumulates in TMEM.
// Half of each product is the other head's unused part: tensor-pipe time
// the unit has to spare.  The work is the causal triangle in 32-key blocks:
// each block of a chunk is loaded once and serves 64 rows of two heads.
//
// Warp roles (192 threads, two CTAs per SM; grid z = head pair, so a CTA
// keeps its pair's fp32 bias rows in shared memory):
//   * warp 4 (one lane): claims chunks from the pair's counter, bulk-copies
//     the chunk's two records into one of two unit buffers (the next unit's
//     as soon as a buffer frees up, while the current unit's blocks stream),
//     loads the unit's query tile by TMA when its rows are consecutive (a
//     prefill's are) once the previous unit's last S' is done, and streams
//     its 2-page blocks through a 3-stage TMA ring (K' then V', 16 KB a
//     stage).
//   * warp 5 (one lane): issues S' of block b + 1 as soon as the softmax has
//     read S' of block b, then P' V' of block b once its P' is in shared
//     memory; tcgen05.commit releases the ring stage and signals O'.
//   * warps 0-3: thread i owns tile row i (TMEM lane i).  It copies its
//     query row (when the unit's rows are not consecutive), reads its 32
//     scores per block from TMEM, adds the bias, masks keys past its visible
//     prefix and keeps the online softmax (lazy rescale: O' in TMEM is
//     rescaled only when the max grows by more than 2^8), writes its P' row,
//     and at the end stores O / l as bf16 rows (the attention output's
//     type); the attention-output norm and u gate then run as their own pass.
// Every wait is bounded; a timeout sets the status word and the CTA drains
// its copies and MMAs before freeing TMEM.
// Semantics: src/imba_chess/model/hstu_attention.py:64-76 (bias),
// :81-132 (document-causal flex_attention with the position score_mod).
#include "attn_common.cuh"
#include "kernels.cuh"
#include "tc_ptx.cuh"

namespace imba {
namespace {

constexpr int kThreads = 192;
constexpr int kStages = 3;
constexpr uint32_t kStageBytes = 16384;  // K' (64 rows x 128 B) then V' (64 rows x 128 B)
constexpr uint32_t kTileBytes = 16384;   // Q' or P': 128 rows x 128 B, 128-byte swizzle
constexpr uint32_t kOffQ = kStages * kStageBytes;
constexpr uint32_t kOffP = kOffQ + kTileBytes;
constexpr uint32_t kOffBias = kOffP + kTileBytes;
constexpr uint32_t kTmemCols = 128;  // S' [0, 64), O' [64, 128)
constexpr int kUnitInts = 2 * kAttnRecInts;
constexpr int kNumBars = 18;
constexpr size_t kSmemMax = 227 * 1024;
constexpr float kLazy = 8.0f;  // log2 of the largest weight before a rescale

struct PrefillParams {
  AttnArgs a;
  int num_layers;
  uint32_t bias_bytes;  // fp32 bias rows of the pair, padded to 16 bytes
  const int* recs;      // [2 C][kAttnRecInts]
  int q_tma;            // 1: qmap views the queries (TMA query tiles for consecutive rows)
};

// Blocks of a unit (two pages each) from its two records.
__device__ __forceinline__ int unit_blocks(const int* ub) {
  const int npa = ub[kRecNpg], npb = ub[kAttnRecInts + kRecNpg];
  return ((npa > npb ? npa : npb) + 1) >> 1;
}
// The unit's 64 rows are consecutive row ids from its first row: its query
// tile is two TMA boxes (one per head); otherwise the softmax warps copy it.
__device__ __forceinline__ bool unit_q_tma(const int* ub, int q_tma) {
  const int* rb = ub + kAttnRecInts;
  return q_tma && ub[kRecN] > 0 && ub[kRecContig] &&
         (rb[kRecN] == 0 || (rb[kRecContig] && rb[kRecRows] == ub[kRecRows] + 32));
}

__device__ __forceinline__ uint32_t pack2_bf16(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

__global__ void __launch_bounds__(kThreads, 2)
    attn_prefill_kernel(const __grid_constant__ CUtensorMap kvmap, const __grid_constant__ CUtensorMap qmap,
                        const PrefillParams prm) {
  const AttnArgs& a = prm.a;
  const imba_step_desc& st = a.st;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int H = a.g.H, h0 = 2 * (int)blockIdx.z;
  const int C = st.num_chunks;
  const int bias_w = 2 * a.max_pos - 1;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = sm;
  uint8_t* qt = sm + kOffQ;
  uint8_t* pt = sm + kOffP;
  float* bias_s = reinterpret_cast<float*>(sm + kOffBias);  // [2][bias_w]
  int* units = reinterpret_cast<int*>(sm + kOffBias + prm.bias_bytes);  // [2][kUnitInts]
  int* unit_id = units + 2 * kUnitInts;                                  // [2] chunk, -1: no more units
  int* misc = unit_id + 2;                                               // [0] abort flag, [1] TMEM base
  uint64_t* bars = reinterpret_cast<uint64_t*>(misc + 2);               // 8-aligned (16-aligned + 4752)
  uint64_t* full = bars;             // [kStages] ring stage loaded (transaction bytes)
  uint64_t* empty = bars + 3;        // [kStages] ring stage consumed (MMA commit)
  uint64_t* s_full = bars + 6;       // S' of a block in TMEM (commit)
  uint64_t* s_free = bars + 7;       // S' read by the four softmax warps
  uint64_t* p_full = bars + 8;       // P' of a block written by the four softmax warps
  uint64_t* o_done = bars + 9;       // P' V' of a block complete (commit)
  uint64_t* q_full = bars + 10;      // Q' of a unit loaded by TMA (transaction bytes)
  uint64_t* q_copy = bars + 11;      // Q' of a unit copied by the four softmax warps
  uint64_t* q_empty = bars + 12;     // the last S' of a unit issued and complete (commit)
  uint64_t* unit_full = bars + 13;   // [2] unit buffer loaded
  uint64_t* unit_empty = bars + 15;  // [2] unit buffer released (4 softmax warps + MMA lane)
  uint64_t* drain = bars + 17;       // the MMA lane's last commit
  volatile int* abort_flag = misc;

  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], 1);
    }
    tc::mbar_init(s_full, 1);
    tc::mbar_init(s_free, 4);
    tc::mbar_init(p_full, 4);
    tc::mbar_init(o_done, 1);
    tc::mbar_init(q_full, 1);
    tc::mbar_init(q_copy, 4);
    tc::mbar_init(q_empty, 1);
    for (int b = 0; b < 2; ++b) {
      tc::mbar_init(&unit_full[b], 1);
      tc::mbar_init(&unit_empty[b], 5);
    }
    tc::mbar_init(drain, 1);
    misc[0] = 0;
    tc::fence_mbar_init();
  }
  if (warp == 0) {
    tc::tmem_alloc(reinterpret_cast<uint32_t*>(&misc[1]), kTmemCols);
    tc::tmem_relinquish();
  }
  // The pair's bias rows (weights: read before the programmatic wait), and a
  // zero P' tile: a row's other-head columns stay zero for the whole kernel.
  {
    // rows h0 and h0 + 1 of ps_w are contiguous; 8 loads in flight per thread
    const float* src = a.ps_w + (size_t)h0 * bias_w;
    const int total = 2 * bias_w;
    for (int i = tid * 8; i < total; i += kThreads * 8) {
      float v[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) v[k] = i + k < total ? __ldg(src + i + k) : 0.f;
#pragma unroll
      for (int k = 0; k < 8; ++k)
        if (i + k < total) bias_s[i + k] = v[k] * kLog2e;
    }
  }
  for (uint32_t o = (uint32_t)tid * 16; o < kTileBytes; o += kThreads * 16)
    *reinterpret_cast<uint4*>(pt + o) = make_uint4(0, 0, 0, 0);
  tc::fence_proxy_async_smem();
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = static_cast<uint32_t>(misc[1]);
  // Queries, pages and records are written by earlier kernels of the step.
  pdl_wait();
  pdl_trigger();

  auto wait = [&](uint64_t* bar, uint32_t parity) {
    return tc::mbar_wait_park_or_abort(bar, parity, st.status, abort_flag);
  };

  if (warp == 4) {
    // ---------------- producer ----------------
    if (lane == 0) {
      int* ctr = a.counters + blockIdx.z;
      const int64_t num_pages = a.g.num_slots / IMBA_PAGE_TOKENS;
      uint32_t kc = 0;  // blocks issued by this CTA
      int qn = 0;       // units with blocks so far (phases of q_empty)
      // Claim a chunk for unit jj and start copying its records into buffer
      // jj & 1 (free); at the end of the queue write the end marker instead.
      auto request = [&](int jj) {
        const int b = jj & 1;
        const int c = atomicAdd(ctr, 1);
        if (c >= C) {
          unit_id[b] = -1;
          tc::mbar_arrive(&unit_full[b]);
          return false;
        }
        unit_id[b] = c;
        int* ub = units + b * kUnitInts;
        tc::mbar_arrive_expect_tx(&unit_full[b], 2 * kRecBytes);
        tc::bulk_load(ub, prm.recs + (size_t)c * kAttnRecInts, kRecBytes, &unit_full[b]);
        tc::bulk_load(ub + kAttnRecInts, prm.recs + (size_t)(C + c) * kAttnRecInts, kRecBytes, &unit_full[b]);
        return true;
      };
      bool more = request(0), ok = true;
      for (int j = 0; more && ok; ++j) {
        const int b = j & 1;
        if (!wait(&unit_full[b], (j >> 1) & 1)) break;
        // Unit j + 1 is requested as soon as its buffer (unit j - 1's) is
        // released, so its records travel while this unit's blocks stream.
        bool requested = false, next_more = false;
        auto request_next = [&](bool block) {
          if (requested) return true;
          if (j >= 1) {
            const uint32_t par = (((j + 1) >> 1) - 1) & 1;  // unit j - 1's use of the buffer
            if (block) {
              if (!wait(&unit_empty[(j + 1) & 1], par)) return false;
            } else if (!tc::mbar_try_wait(&unit_empty[(j + 1) & 1], par)) {
              return true;  // not yet: ask again after the next block
            }
          }
          next_more = request(j + 1);
          requested = true;
          return true;
        };
        if (!request_next(false)) break;
        const int* ub = units + b * kUnitInts;
        const int npa = ub[kRecNpg], npb = ub[kAttnRecInts + kRecNpg];
        const int* rp = npb > npa ? ub + kAttnRecInts : ub;  // the record that lists more pages
        const int npg = npa > npb ? npa : npb, pg0 = ub[kRecPg0];
        auto page_at = [&](int p) {
          if (p < kRecMaxPages) return rp[kRecPages + p];
          int pg = st.group_pages[pg0 + p];  // p < the group's page count (item pass)
          if (pg < 0 || pg >= num_pages) {
            report(st.status, IMBA_ERR_RANGE);
            pg = 0;
          }
          return pg;
        };
        if (npg > 0) {
          if (unit_q_tma(ub, prm.q_tma)) {
            // Q' once the previous unit's S' products are done with it.
            if (qn > 0 && !wait(q_empty, (qn - 1) & 1)) break;
            const int row0 = ub[kRecRows];
            tc::mbar_arrive_expect_tx(q_full, kTileBytes);
            tc::tma_load_2d(qt, &qmap, q_full, h0 * 64, row0);
            tc::tma_load_2d(qt + kTileBytes / 2, &qmap, q_full, (h0 + 1) * 64, row0);
          }
          ++qn;
        }
        for (int p = 0; p < npg; p += 2, ++kc) {
          const int s = kc % kStages;
          if (kc >= kStages && !wait(&empty[s], ((kc / kStages) - 1) & 1)) {
            ok = false;
            break;
          }
          // An odd last page repeats the first: finite V' rows under zero P'.
          const int pa = page_at(p), pb = p + 1 < npg ? page_at(p + 1) : pa;
          const int ka = ((pa * prm.num_layers + a.layer) * 2 * H + h0) * IMBA_PAGE_TOKENS;
          const int kb = ((pb * prm.num_layers + a.layer) * 2 * H + h0) * IMBA_PAGE_TOKENS;
          uint8_t* dst = ring + s * kStageBytes;
          tc::mbar_arrive_expect_tx(&full[s], kStageBytes);
          tc::tma_load_2d(dst, &kvmap, &full[s], 0, ka);
          tc::tma_load_2d(dst + 4096, &kvmap, &full[s], 0, kb);
          tc::tma_load_2d(dst + 8192, &kvmap, &full[s], 0, ka + H * IMBA_PAGE_TOKENS);
          tc::tma_load_2d(dst + 12288, &kvmap, &full[s], 0, kb + H * IMBA_PAGE_TOKENS);
          if (!request_next(false)) {
            ok = false;
            break;
          }
        }
        if (!ok || !request_next(true)) break;
        more = next_more;
      }
      // Loads still in flight land before the CTA ends (bounded waits).
      for (uint32_t k = kc > kStages ? kc - kStages : 0; k < kc; ++k)
        tc::mbar_wait_for(&full[k % kStages], (k / kStages) & 1, st.status, tc::kWaitNs);
    }
    __syncwarp();
  } else if (warp == 5) {
    // ---------------- MMA issue ----------------
    if (lane == 0) {
      constexpr uint32_t idS = tc::idesc_bf16_f32(128, 64);
      constexpr uint32_t idPV = tc::idesc_bf16_f32(128, 64) | tc::kIdescBMajorMN;
      const uint64_t dQ = tc::smem_desc_k128(qt), dP = tc::smem_desc_k128(pt);
      // S' of block k; the unit's last S' also releases Q'.
      auto issue_s = [&](uint32_t k, bool last) {
        const int s = k % kStages;
        if (!wait(&full[s], (k / kStages) & 1)) return false;
        if (k > 0 && !wait(s_free, (k - 1) & 1)) return false;  // S' of block k - 1 has been read
        tc::fence_after_sync();
        const uint64_t dK = tc::smem_desc_k128(ring + s * kStageBytes);
#pragma unroll
        for (int i = 0; i < 4; ++i) tc::umma_f16(tmem, dQ + 2 * i, dK + 2 * i, idS, i);
        tc::umma_commit(s_full);
        if (last) tc::umma_commit(q_empty);
        return true;
      };
      uint32_t kc = 0;
      int nq_tma = 0, nq_copy = 0;
      bool ok = true;
      for (int j = 0; ok; ++j) {
        const int b = j & 1;
        if (!wait(&unit_full[b], (j >> 1) & 1) || unit_id[b] < 0) break;
        const int* ub = units + b * kUnitInts;
        const int nblk = unit_blocks(ub);
        if (nblk > 0) {
          ok = unit_q_tma(ub, prm.q_tma) ? wait(q_full, nq_tma++ & 1) : wait(q_copy, nq_copy++ & 1);
          ok = ok && issue_s(kc, nblk == 1);
          for (int blk = 0; ok && blk < nblk; ++blk, ++kc) {
            if (blk + 1 < nblk && !issue_s(kc + 1, blk + 2 == nblk)) {
              ok = false;
              break;
            }
            if (!wait(p_full, kc & 1)) {
              ok = false;
              break;
            }
            tc::fence_after_sync();
            const int s = kc % kStages;
            const uint64_t dV = tc::smem_desc_k128(ring + s * kStageBytes + 8192);
#pragma unroll
            for (int i = 0; i < 4; ++i) tc::umma_f16(tmem + 64, dP + 2 * i, dV + 128 * i, idPV, (blk | i) != 0);
            tc::umma_commit(&empty[s]);
            tc::umma_commit(o_done);
          }
        }
        if (ok) tc::mbar_arrive(&unit_empty[b]);
      }
      // Every MMA issued here completes before TMEM is freed.
      tc::umma_commit(drain);
      tc::mbar_wait_for(drain, 0, st.status, tc::kWaitNs);
    }
    __syncwarp();
  } else {
    // ---------------- softmax / epilogue: thread = tile row ----------------
    const int hh = warp >> 1, half = warp & 1, h = h0 + hh;
    const int trow = 32 * warp + lane;
    const uint32_t tl = tmem + ((uint32_t)(32 * warp) << 16);  // this warp's TMEM lanes
    const uint32_t qrow = tc::smem_u32(qt) + trow * 128, prow = tc::smem_u32(pt) + trow * 128;
    const uint32_t sw = (uint32_t)(trow & 7);
    const float* brow = bias_s + hh * bias_w;
    const float scale2 = a.scale * kLog2e;
    const int HD = H * 64, bmax = 2 * a.max_pos - 2;
    uint32_t kc = 0;
    bool ok = true;
    for (int j = 0; ok; ++j) {
      const int b = j & 1;
      if (!__all_sync(0xffffffffu, wait(&unit_full[b], (j >> 1) & 1)) || unit_id[b] < 0) break;
      const int* ub = units + b * kUnitInts;
      const int* rec = ub + half * kAttnRecInts;
      const int nblk = unit_blocks(ub);
      const int n = rec[kRecN];
      const bool valid = lane < n;
      const int r = valid ? rec[kRecRows + lane] : 0;
      const int vis = valid ? rec[kRecVis + lane] : 0;
      const int qp = valid ? rec[kRecQpos + lane] : 0;
      float l = 0.f, m_ref = -INFINITY;
      if (nblk > 0 && !unit_q_tma(ub, prm.q_tma)) {
        // This row's query (zeros past the chunk's rows) -> Q'.  The
        // previous unit's S' products are complete: this warp waited for
        // its last block's scores.
        const bf16* src = static_cast<const bf16*>(a.q) + (size_t)r * HD + h * 64;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const uint32_t dst = qrow + (((uint32_t)c ^ sw) << 4);
          if (valid)
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(dst), "l"(src + 8 * c) : "memory");
          else
            asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(dst), "r"(0) : "memory");
        }
        asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;\n" ::: "memory");
        tc::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(q_copy);
      }
      for (int blk = 0; blk < nblk; ++blk, ++kc) {
        if (!__all_sync(0xffffffffu, wait(s_full, kc & 1))) {
          ok = false;
          break;
        }
        tc::fence_after_sync();
        uint32_t sr[2][16];
        tc::tmem_ld16_async(tl + 16 * hh, sr[0]);       // page 0 of the block, this head's 16 keys
        tc::tmem_ld16_async(tl + 32 + 16 * hh, sr[1]);  // page 1
        tc::tmem_wait_ld();
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(s_free);  // the MMA lane may overwrite S'
        // Scores in the log2 domain; keys at or past the row's visible
        // prefix get -inf.
        const int t0 = 32 * blk, nv = vis - t0, bi = t0 - qp + a.max_pos - 1;
        float x[32];
        if (bi >= 0 && bi + 31 <= bmax) {
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const float v = fmaf(__uint_as_float(sr[e >> 4][e & 15]), scale2, brow[bi + e]);
            x[e] = e < nv ? v : -INFINITY;
          }
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            int idx = bi + e;
            idx = idx < 0 ? 0 : (idx > bmax ? bmax : idx);
            const float v = fmaf(__uint_as_float(sr[e >> 4][e & 15]), scale2, brow[idx]);
            x[e] = e < nv ? v : -INFINITY;
          }
        }
        float mb = x[0];
#pragma unroll
        for (int e = 1; e < 32; ++e) mb = fmaxf(mb, x[e]);
        bool o_ready = blk == 0;  // no earlier P' V' of this unit to wait for
        if (__any_sync(0xffffffffu, mb > m_ref + kLazy)) {
          const float m_new = fmaxf(m_ref, mb);
          const float corr = m_new == -INFINITY ? 1.f : exp2_approx(m_ref - m_new);
          l *= corr;
          if (blk > 0) {  // O' holds the earlier blocks: scale it once the last P V is done
            if (!__all_sync(0xffffffffu, wait(o_done, (kc - 1) & 1))) {
              ok = false;
              break;
            }
            o_ready = true;
            tc::fence_after_sync();
#pragma unroll
            for (int hp = 0; hp < 2; ++hp) {
              float ov[32];
              tc::tmem_ld32(tl + 64 + 32 * hp, ov);
#pragma unroll
              for (int i = 0; i < 32; ++i) ov[i] *= corr;
              tc::tmem_st32(tl + 64 + 32 * hp, ov);
            }
          }
          m_ref = m_new;
        }
        const float mu = m_ref == -INFINITY ? 0.f : m_ref;
        uint32_t pw[16];
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          const float p0 = exp2_approx(x[e] - mu), p1 = exp2_approx(x[e + 1] - mu);
          l += p0 + p1;
          pw[e >> 1] = pack2_bf16(p0, p1);
        }
        // P' of the previous block has been consumed before it is overwritten.
        if (!o_ready && !__all_sync(0xffffffffu, wait(o_done, (kc - 1) & 1))) {
          ok = false;
          break;
        }
        // This head's columns of the row: 16-byte chunks 4 p + 2 hh (+1).
#pragma unroll
        for (int p = 0; p < 2; ++p)
#pragma unroll
          for (int hf = 0; hf < 2; ++hf) {
            const uint32_t c = (uint32_t)(4 * p + 2 * hh + hf);
            const uint32_t* w = pw + 8 * p + 4 * hf;
            asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(prow + ((c ^ sw) << 4)), "r"(w[0]),
                         "r"(w[1]), "r"(w[2]), "r"(w[3])
                         : "memory");
          }
        tc::fence_proxy_async_smem();
        tc::fence_before_sync();  // a rescaled O' is in place before the next P' V'
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(p_full);
      }
      if (!ok) break;
      // Epilogue: O / l (fp32) for the row's head.
      if (nblk > 0) {
        if (!__all_sync(0xffffffffu, wait(o_done, (kc - 1) & 1))) break;
        tc::fence_after_sync();
      }
      const float inv = l > 0.f ? 1.0f / l : 0.f;
      uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<bf16*>(a.out) + (size_t)r * HD + h * 64);
#pragma unroll
      for (int hp = 0; hp < 2; ++hp) {
        float ov[32];
        if (nblk > 0) {
          tc::tmem_ld32(tl + 64 + 32 * hp, ov);
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) ov[i] = 0.f;
        }
        if (valid) {
#pragma unroll
          for (int i = 0; i < 32; i += 8)
            dst[4 * hp + i / 8] = make_uint4(pack2_bf16(ov[i] * inv, ov[i + 1] * inv),
                                             pack2_bf16(ov[i + 2] * inv, ov[i + 3] * inv),
                                             pack2_bf16(ov[i + 4] * inv, ov[i + 5] * inv),
                                             pack2_bf16(ov[i + 6] * inv, ov[i + 7] * inv));
        }
      }
      tc::fence_before_sync();  // O' read before the next unit's first P' V' overwrites it
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&unit_empty[b]);
    }
    asm volatile("cp.async.wait_all;\n" ::: "memory");
  }

  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace

bool launch_attn_prefill(const AttnArgs& a, int num_layers, int64_t num_pages, const int* recs, cudaStream_t s,
                         cudaError_t* err) {
  const int H = a.g.H;
  if (a.g.dqk != 64 || a.g.dv != 64 || H % 2 || H / 2 > kCountersPerLayer || !a.counters || !recs ||
      a.st.num_extra != 0 || a.max_pos < 1)
    return false;
  if (a.st.num_chunks <= 0) {
    *err = cudaSuccess;
    return true;
  }
  // TMA view of the pool: 2D [num_pages * L * 2H * 16 rows, 64 columns] bf16;
  // one box = one page's 16 rows of two consecutive heads.
  const uint64_t rows = (uint64_t)num_pages * num_layers * 2 * H * IMBA_PAGE_TOKENS;
  if (rows > (uint64_t)INT32_MAX) return false;
  EncodeTiledFn enc = attn_encode_fn();
  if (!enc || (reinterpret_cast<uintptr_t>(a.pool) & 15) || (reinterpret_cast<uintptr_t>(a.q) & 15)) return false;
  CUtensorMap map;
  const cuuint64_t dims[2] = {64, rows};
  const cuuint64_t strides[1] = {128};
  const cuuint32_t box[2] = {64, 2 * IMBA_PAGE_TOKENS};
  const cuuint32_t estr[2] = {1, 1};
  if (enc(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(a.pool), dims, strides, box, estr,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return false;
  // TMA view of the queries: 2D [R rows, H * 64 columns] bf16; one box = 64
  // rows of one head.
  CUtensorMap qmap;
  const int R = a.st.num_rows;
  const cuuint64_t qdims[2] = {(cuuint64_t)H * 64, (cuuint64_t)(R > 0 ? R : 1)};
  const cuuint64_t qstrides[1] = {(cuuint64_t)H * 64 * 2};
  const cuuint32_t qbox[2] = {64, 64};
  const int q_tma = enc(&qmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(a.q), qdims, qstrides, qbox,
                        estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
  const uint32_t bias_bytes = (uint32_t)((2 * (2 * (size_t)a.max_pos - 1) * 4 + 15) / 16 * 16);
  const size_t smem = 1024 + kOffBias + bias_bytes + 2 * kUnitInts * 4 + 2 * 4 + 2 * 4 + kNumBars * 8;
  if (smem > kSmemMax) return false;
  cudaError_t e = cudaFuncSetAttribute(attn_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  // The whole unified L1 as shared memory, so that two CTAs fit on an SM.
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(attn_prefill_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                             (int)cudaSharedmemCarveoutMaxShared);
  if (e != cudaSuccess) {
    *err = e;
    return true;
  }
  int dev = 0, sms = 148, smem_sm = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
  // CTAs per SM by shared memory (1 KB reserved per CTA) and registers
  // (launch bounds: two); the work queue balances any CTA that starts late.
  int per_sm = (int)((size_t)smem_sm / (smem + 1024));
  per_sm = per_sm > 2 ? 2 : (per_sm < 1 ? 1 : per_sm);
  const int pairs = H / 2;
  int ctas = per_sm * sms / pairs;
  ctas = ctas < 1 ? 1 : ctas;
  ctas = a.st.num_chunks < ctas ? a.st.num_chunks : ctas;
  PrefillParams prm{a, num_layers, bias_bytes, recs, q_tma};
  *err = launch_pdl(attn_prefill_kernel, dim3(ctas, 1, pairs), dim3(kThreads), smem, s, map, qmap, prm);
  return true;
}

}  // namespace imba
