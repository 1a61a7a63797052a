// Pieces shared by the two tensor-core attention kernels (attention_page.cu:
// grouped decode, and prefill steps with few rows per group;
// attention_prefill.cu: jagged prefill): the per-step item records, the
// relative-position bias index and the log2-domain softmax helpers.
#pragma once

#include <cuda.h>
#include <mutex>

#include "common.cuh"

namespace imba {

// Item record (int32 words; kAttnRecInts * 4 bytes, a multiple of 16):
// <= 32 query rows of one chunk, resolved once per step by the item pass.
constexpr int kRecN = 0;        // rows in the item (0: nothing to do; -1 in a buffer: no more items)
constexpr int kRecNpg = 1;      // visible pages (ceil of the longest row's prefix / 16)
constexpr int kRecPg0 = 2;      // first entry of the group's page list
constexpr int kRecHalves = 3;   // items of the chunk (record of its first half)
constexpr int kRecContig = 4;   // 1: the rows are consecutive row ids rows[0] + i
constexpr int kRecRows = 8;     // [32] global row ids
constexpr int kRecVis = 40;     // [32] visible prefix tokens
constexpr int kRecQpos = 72;    // [32] query positions
constexpr int kRecXoff = 104;   // [32] first extra of the row
constexpr int kRecXcnt = 136;   // [32] extras of the row
constexpr int kRecX0slot = 168; // [32] pool slot of the row's first extra (-1: none)
constexpr int kRecX0pos = 200;  // [32] its position
constexpr int kRecPages = 232;  // [kRecMaxPages] the group's first page ids
constexpr int kRecMaxPages = 64;
constexpr uint32_t kRecBytes = kAttnRecInts * 4;
static_assert(kRecPages + kRecMaxPages == kAttnRecInts, "record layout");
static_assert(kRecBytes % 16 == 0, "bulk copies move multiples of 16 bytes");

// Relative-position bias column: clamp(k - q + max_pos - 1, 0, 2 max_pos - 2)
// (the reference's _position_score_mod / _relative_bias).
__device__ __forceinline__ int bias_index(int kpos, int qpos, int max_pos) {
  int idx = kpos - qpos + (max_pos - 1);
  idx = idx < 0 ? 0 : idx;
  return idx > 2 * max_pos - 2 ? 2 * max_pos - 2 : idx;
}

// Scores are kept in the log2 domain, s2 = log2(e) (q . k / sqrt(d) + bias),
// and weights are 2^(s2 - max): the same softmax as exp(s - max) with one
// multiply less per element.
constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ float exp2_approx(float x) {  // hardware ex2; 2^-inf = +0
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// cuTensorMapEncodeTiled through the runtime's driver entry point (null when
// the driver has none).
inline EncodeTiledFn attn_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

}  // namespace imba
