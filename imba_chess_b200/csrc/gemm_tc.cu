// bf16 tensor-core GEMM for sm_100a: acc[M, N] = A[M, K] . W[N, K]^T with a
// fused epilogue, on the 5th-generation tensor cores.
//
// Output tiles are 128 x BN; both operands are K-major.  A persistent grid (one
// CTA per SM) walks the tiles; TMA copies 128 x 64 (A) and BN x 64 (W) bf16
// tiles into shared memory with the 128-byte swizzle through a STAGES-deep
// ring guarded by full / empty mbarriers.  Warp 0 (one thread) issues the TMA
// copies, warp 1 (one thread) issues tcgen05.mma (M = 128, N = BN, K = 16 per
// instruction) into one of two TMEM accumulators and releases each stage with
// tcgen05.commit; 8 or 16 epilogue warps read the other accumulator back
// (TMEM lane quadrant = warp % 4 = tile rows; two or four warps per quadrant,
// one column slice each) and hand 32-column chunks to the epilogue functor,
// so tile i's epilogue overlaps tile i + 1's main loop.
// Out-of-range rows / columns of A / W are zero-filled by TMA and skipped by
// the epilogue.
//
// Used for the STU projections (uvqk with SiLU + KV append; output projection
// with bias + residual), the split-precision policy GEMM and the value-head
// hidden layer (hstu_attention.py:307-325, :415-424; hstu_model.py:745-751).
#include <mutex>
#include <new>

#include "gemm_tc.cuh"
#include "tc_ptx.cuh"

namespace imba {
namespace {

constexpr int kBM = 128;
constexpr int kBK = 64;

// Epilogue warps: 8 (two per TMEM lane quadrant, one column half each).  16
// warps measured no faster for the per-thread epilogues (their limit is the
// SM's store path, not latency).
template <bool STAGED>
__host__ __device__ constexpr int epi_warps() { return 8; }
template <bool STAGED>
__host__ __device__ constexpr int gemm_threads() { return 64 + 32 * epi_warps<STAGED>(); }
// Staged epilogues: per epilogue warp a swizzled fp32 32 x 32 chunk plus 32
// per-row tags.
constexpr size_t kStageFloats = 32 * 32 + 32;

// Box-stored epilogues: per epilogue warp one 4 KB staging box (32 rows x
// 128 B, 128-byte swizzle) for its TMA stores, 1024-aligned after the ring.
constexpr size_t kBoxBytes = 32 * 128;

template <int BN, int STAGES, bool STAGED, bool BOX = false>
struct TileShape {
  static constexpr uint32_t kABytes = kBM * kBK * 2;
  static constexpr uint32_t kBBytes = BN * kBK * 2;
  static constexpr size_t kSmem = 1024 + STAGES * (kABytes + kBBytes) + (BOX ? epi_warps<STAGED>() * kBoxBytes : 0) +
                                  (2 * STAGES + 4) * 8 + 16 + (STAGED ? epi_warps<STAGED>() * kStageFloats * 4 : 0);
};

// Persistent, warp-specialised: CTA b handles tiles b, b + gridDim.x, ...
// (tile t -> m-tile t % mt, n-tile t / mt).  Warp 0 streams A / W tiles
// through the smem ring; warp 1 issues the MMAs of tile i into TMEM buffer
// i % 2 (2 x BN columns) and signals acc_full; the epilogue warps drain buffer i % 2
// while tile i + 1 is being loaded and multiplied, then signal acc_empty.
template <int BN, int STAGES, class Epi>
__global__ void __launch_bounds__(gemm_threads<Epi::kStaged>(), 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, int M, int N,
                   int K, const __grid_constant__ Epi epi, int32_t* status) {
  using S = TileShape<BN, STAGES, Epi::kStaged, Epi::kBoxStore>;
  constexpr int kEpiWarps = epi_warps<Epi::kStaged>();
  constexpr int kColGroups = kEpiWarps / 4;  // warps per TMEM lane quadrant
  constexpr int kCols = BN / kColGroups;      // columns per epilogue warp
  static_assert(kCols % 32 == 0, "epilogue column slice must be a multiple of 32");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * S::kABytes;
  uint8_t* boxes = sB + STAGES * S::kBBytes;  // kEpiWarps x kBoxBytes (box-stored epilogues)
  uint64_t* full = reinterpret_cast<uint64_t*>(boxes + (Epi::kBoxStore ? kEpiWarps * kBoxBytes : 0));
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  float* staging = reinterpret_cast<float*>(tmem_slot + 4);  // kEpiWarps x kStageFloats (staged epilogues)
  __shared__ int abort_flag;
  volatile int* abort = &abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int KB = K / kBK;
  const int mt = (M + kBM - 1) / kBM, ntl = (N + BN - 1) / BN;
  const int tiles = mt * ntl;

  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int s = 0; s < STAGES; ++s) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      tc::mbar_init(&acc_full[b], 1);
      tc::mbar_init(&acc_empty[b], kEpiWarps);
    }
    tc::fence_mbar_init();
    tc::prefetch_tmap(&tmA);
    tc::prefetch_tmap(&tmB);
  }
  if (warp == 1) {
    tc::tmem_alloc(tmem_slot, 2 * BN);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  // Barrier / TMEM set-up and descriptor prefetch overlap the previous
  // kernel; operand loads and epilogue memory accesses are ordered after it.
  pdl_wait();
  pdl_trigger();

  if (warp == 0) {
    if (lane == 0) {  // TMA producer
      int it = 0;
      for (int tile = blockIdx.x; tile < tiles && !*abort; tile += gridDim.x) {
        const int m0 = (tile % mt) * kBM, n0 = (tile / mt) * BN;
        for (int kb = 0; kb < KB; ++kb, ++it) {
          const int s = it % STAGES;
          if (it >= STAGES && !tc::mbar_wait_or_abort(&empty[s], ((it / STAGES) - 1) & 1, status, abort)) break;
          tc::mbar_arrive_expect_tx(&full[s], S::kABytes + S::kBBytes);
          tc::tma_load_2d(sA + s * S::kABytes, &tmA, &full[s], kb * kBK, m0);
          tc::tma_load_2d(sB + s * S::kBBytes, &tmB, &full[s], kb * kBK, n0);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {  // MMA issuer
      constexpr uint32_t idesc = tc::idesc_bf16_f32(kBM, BN);
      int it = 0, i = 0;
      for (int tile = blockIdx.x; tile < tiles && !*abort; tile += gridDim.x, ++i) {
        const int b = i & 1;
        if (i >= 2 && !tc::mbar_wait_or_abort(&acc_empty[b], ((i >> 1) - 1) & 1, status, abort)) break;
        tc::fence_after_sync();
        const uint32_t d = tmem + b * BN;
        bool ok = true;
        for (int kb = 0; kb < KB; ++kb, ++it) {
          const int s = it % STAGES;
          if (!tc::mbar_wait_or_abort(&full[s], (it / STAGES) & 1, status, abort)) {
            ok = false;
            break;
          }
          tc::fence_after_sync();
          const uint64_t ad = tc::smem_desc_k128(sA + s * S::kABytes);
          const uint64_t bd = tc::smem_desc_k128(sB + s * S::kBBytes);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) tc::umma_f16(d, ad + 2 * k, bd + 2 * k, idesc, (kb | k) != 0);
          tc::umma_commit(&empty[s]);
        }
        tc::umma_commit(&acc_full[b]);  // fires once the tile's MMAs (or those issued) complete
        if (!ok) break;
      }
    }
  } else {  // epilogue warps: two per TMEM lane quadrant, one per column half
    const int quad = warp & 3;  // TMEM lane quadrant this warp may access
    const int c_lo = ((warp - 2) >> 2) * kCols;  // kColGroups warps per quadrant, one slice each
    const uint32_t lane_base = static_cast<uint32_t>(quad * 32) << 16;
    bool box_pending = false;  // a TMA store of this warp may still be reading its box
    int i = 0;
    for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++i) {
      const int b = i & 1;
      bool ok = tc::mbar_wait_or_abort(&acc_full[b], (i >> 1) & 1, status, abort);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc::fence_after_sync();
      const int m0 = (tile % mt) * kBM, n0 = (tile / mt) * BN;
      const int row = m0 + quad * 32 + lane;
      if constexpr (Epi::kStaged) {
        // TMEM -> registers (thread = row) -> swizzled shared chunk -> rows
        // written by groups of eight lanes.
        float* stg = staging + (size_t)(warp - 2) * kStageFloats;
        int* tags = reinterpret_cast<int*>(stg + 32 * 32);
        tags[lane] = row < M ? epi.row_tag(row) : 0;
#pragma unroll 1
        for (int c = c_lo; c < c_lo + kCols; c += 32) {
          float v[32];
          tc::tmem_ld32(tmem + b * BN + lane_base + c, v);
#pragma unroll
          for (int k = 0; k < 32; ++k) stg[lane * 32 + (k ^ lane)] = v[k];
          __syncwarp();
          epi.tile32(stg, tags, m0 + quad * 32, n0 + c, M, N, lane);
          __syncwarp();
        }
      } else {
        int region = 0;
        if constexpr (Epi::kBoxStore) region = epi.box_region(n0 + c_lo);
        if (region != 0) {
          if constexpr (Epi::kBoxStore) {
            // 64-column boxes of this warp's 32 rows: TMEM -> SiLU -> bf16 ->
            // swizzled staging box -> one TMA store (rows past M are clipped).
            uint8_t* box = boxes + (size_t)(warp - 2) * kBoxBytes;
#pragma unroll 1
            for (int cb = 0; cb < kCols; cb += 64) {
              if (box_pending) {  // the previous store from this box must have read it
                if (lane == 0) tc::bulk_wait_read_all();
                __syncwarp();
              }
#pragma unroll 1
              for (int h = 0; h < 2; ++h) {
                float v[32];
                tc::tmem_ld32(tmem + b * BN + lane_base + c_lo + cb + 32 * h, v);
                epi.box_stage32(box, h, v, lane);
              }
              tc::fence_proxy_async_smem();
              __syncwarp();
              if (lane == 0) {
                tc::tma_store_2d(epi.box_map(region), box, epi.box_x(region, n0 + c_lo + cb), m0 + quad * 32);
                tc::bulk_commit();
              }
              box_pending = true;
            }
          }
        } else {
          typename Epi::Ctx cx{};
          if (row < M) cx = epi.begin(row, n0 + c_lo, kCols);
#pragma unroll 1
          for (int c = c_lo; c < c_lo + kCols; c += 32) {
            float v[32];
            tc::tmem_ld32(tmem + b * BN + lane_base + c, v);
            if (row < M && n0 + c < N) epi.chunk32(cx, row, n0 + c, N, v);
          }
        }
      }
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&acc_empty[b]);
    }
    if (box_pending && lane == 0) tc::bulk_wait_all();  // stores complete before the CTA exits
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 1) tc::tmem_dealloc(tmem, 2 * BN);
}

// ---------------------------------------------------------------------------
// Host side: TMA descriptors.
// ---------------------------------------------------------------------------
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
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

// K-major bf16 operand [rows, cols] with the given row stride; 64 x box_rows
// boxes, 128-byte swizzle, zero fill out of range.
bool make_map(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t row_stride_bytes,
              uint32_t box_rows) {
  EncodeTiledFn enc = encode_fn();
  if (!enc || !base || rows == 0 || cols == 0) return false;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (row_stride_bytes & 15)) return false;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {row_stride_bytes};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(kBK), box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

constexpr int kBNWide = 256;
constexpr int kBNNarrow = 128;

struct TCState {
  CUtensorMap uvqk[IMBA_MAX_LAYERS];
  CUtensorMap o[IMBA_MAX_LAYERS];
  CUtensorMap policy;
  CUtensorMap value;
  CUtensorMap content;  // [d, 192] split board projection
  bool has_value = false;
  bool has_content = false;
};

int sm_count() {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms;
}

template <int BN, class Epi>
cudaError_t launch(const CUtensorMap& ta, const CUtensorMap& tb, int M, int N, int K, const Epi& epi, int32_t* status,
                   cudaStream_t s) {
  constexpr int kSt = BN == 256 ? 4 : 6;
  using S = TileShape<BN, kSt, Epi::kStaged, Epi::kBoxStore>;
  auto kern = gemm_tc_kernel<BN, kSt, Epi>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)S::kSmem);
  if (e != cudaSuccess) return e;
  const int tiles = ((M + kBM - 1) / kBM) * ((N + BN - 1) / BN);
  const int sms = sm_count();
  const int grid = tiles < sms ? tiles : sms;
  return launch_pdl(kern, dim3(grid), dim3(gemm_threads<Epi::kStaged>()), S::kSmem, s, ta, tb, M, N, K, epi, status);
}

}  // namespace

imba_status_t gemm_tc_prepare(imba_model* m) {
  const imba_model_desc& d = m->d;
  m->tc = nullptr;
  // fp32 handles, and bf16 handles whose SIMT-GEMM test hook is set, run the
  // SIMT GEMMs.  Any other bf16 handle must get every tensor map encoded.
  if (d.dtype != IMBA_DTYPE_BF16 || m->simt_gemm) return IMBA_OK;
  const int hdv = d.num_heads * d.linear_dim;
  const bool shapes_ok = d.model_dim % 64 == 0 && hdv % 64 == 0 && d.attention_dim % 32 == 0 &&
                         d.linear_dim % 32 == 0 && m->uvqk_n % kBNWide == 0 && d.model_dim % kBNNarrow == 0 &&
                         (d.model_dim / 2) % 32 == 0;
  if (!shapes_ok) return IMBA_ERR_UNSUPPORTED;
  if (!encode_fn()) return IMBA_ERR_CUDA;  // no cuTensorMapEncodeTiled in this driver
  TCState* t = new (std::nothrow) TCState();
  if (!t) return IMBA_ERR_OOM;
  bool ok = true;
  for (int l = 0; l < d.num_layers && ok; ++l) {
    ok = make_map(&t->uvqk[l], d.uvqk_w[l], m->uvqk_n, d.model_dim, (uint64_t)d.model_dim * 2, kBNWide) &&
         make_map(&t->o[l], d.o_w[l], d.model_dim, hdv, (uint64_t)hdv * 2, kBNNarrow);
  }
  ok = ok && make_map(&t->policy, d.policy_w, d.vocab, 3 * d.model_dim, (uint64_t)3 * d.model_dim * 2, kBNWide);
  if (ok && d.has_value_head) {
    ok = make_map(&t->value, d.value0_w, d.model_dim / 2, d.model_dim, (uint64_t)d.model_dim * 2, kBNNarrow);
    t->has_value = ok;
  }
  if (ok && m->board_proj3) {
    ok = make_map(&t->content, m->board_proj3, d.model_dim, 192, 192 * 2, kBNNarrow);
    t->has_content = ok;
  }
  if (!ok) {  // a weight tensor the TMA cannot address (alignment, stride)
    delete t;
    return IMBA_ERR_ARG;
  }
  m->tc = t;
  return IMBA_OK;
}

void gemm_tc_release(imba_model* m) {
  delete static_cast<TCState*>(m->tc);
  m->tc = nullptr;
}

template <>
bool gemm_tc_launch_uvqk<bf16>(const imba_model* m, int layer, int rows, const bf16* xn, const EpiUVQK<bf16>& epi,
                               cudaStream_t s, cudaError_t* err) {
  const TCState* t = static_cast<const TCState*>(m->tc);
  if (!t || rows <= 0) return false;
  CUtensorMap ta;
  if (!make_map(&ta, xn, rows, m->d.model_dim, (uint64_t)m->d.model_dim * 2, kBM)) return false;
  // u / q as [rows, H d] bf16 with 64 x 32 boxes for the epilogue's TMA stores.
  EpiUVQK<bf16> e = epi;
  const int hdv = m->d.num_heads * m->d.linear_dim, hdq = m->d.num_heads * m->d.attention_dim;
  if (!make_map(&e.u_map, e.u, rows, hdv, (uint64_t)hdv * 2, 32) ||
      !make_map(&e.q_map, e.q, rows, hdq, (uint64_t)hdq * 2, 32))
    return false;
  *err = launch<kBNWide>(ta, t->uvqk[layer], rows, m->uvqk_n, m->d.model_dim, e, epi.status, s);
  return true;
}

bool gemm_tc_launch_content(const imba_model* m, int rows, const bf16* pooled3, const EpiContent& epi,
                            int32_t* status, cudaStream_t s, cudaError_t* err) {
  const TCState* t = static_cast<const TCState*>(m->tc);
  if (!t || !t->has_content || rows <= 0) return false;
  CUtensorMap ta;
  if (!make_map(&ta, pooled3, rows, 192, 192 * 2, kBM)) return false;
  *err = launch<kBNNarrow>(ta, t->content, rows, m->d.model_dim, 192, epi, status, s);
  return true;
}

template <>
bool gemm_tc_launch_out<bf16>(const imba_model* m, int layer, int rows, const bf16* gated, const EpiResidual& epi,
                              int32_t* status, cudaStream_t s, cudaError_t* err) {
  const TCState* t = static_cast<const TCState*>(m->tc);
  if (!t || rows <= 0) return false;
  const int hdv = m->d.num_heads * m->d.linear_dim;
  CUtensorMap ta;
  if (!make_map(&ta, gated, rows, hdv, (uint64_t)hdv * 2, kBM)) return false;
  *err = launch<kBNNarrow>(ta, t->o[layer], rows, m->d.model_dim, hdv, epi, status, s);
  return true;
}

template <>
bool gemm_tc_launch_policy<bf16>(const imba_model* m, int rows, const bf16* xf3, const EpiStore& epi,
                                 int32_t* status, cudaStream_t s, cudaError_t* err) {
  const TCState* t = static_cast<const TCState*>(m->tc);
  if (!t || rows <= 0) return false;
  const int k3 = 3 * m->d.model_dim;
  CUtensorMap ta;
  if (!make_map(&ta, xf3, rows, k3, (uint64_t)k3 * 2, kBM)) return false;
  *err = launch<kBNWide>(ta, t->policy, rows, m->d.vocab, k3, epi, status, s);
  return true;
}

template <>
bool gemm_tc_launch_value<bf16>(const imba_model* m, int rows, const bf16* xin, int lda, const EpiBiasSilu& epi,
                                int32_t* status, cudaStream_t s, cudaError_t* err) {
  const TCState* t = static_cast<const TCState*>(m->tc);
  if (!t || !t->has_value || rows <= 0) return false;
  CUtensorMap ta;
  if (!make_map(&ta, xin, rows, m->d.model_dim, (uint64_t)lda * 2, kBM)) return false;
  *err = launch<kBNNarrow>(ta, t->value, rows, m->d.model_dim / 2, m->d.model_dim, epi, status, s);
  return true;
}

// fp32 models always take the SIMT path.
template <>
bool gemm_tc_launch_uvqk<float>(const imba_model*, int, int, const float*, const EpiUVQK<float>&, cudaStream_t,
                                cudaError_t*) {
  return false;
}
template <>
bool gemm_tc_launch_out<float>(const imba_model*, int, int, const float*, const EpiResidual&, int32_t*, cudaStream_t,
                               cudaError_t*) {
  return false;
}
template <>
bool gemm_tc_launch_policy<float>(const imba_model*, int, const float*, const EpiStore&, int32_t*, cudaStream_t,
                                  cudaError_t*) {
  return false;
}
template <>
bool gemm_tc_launch_value<float>(const imba_model*, int, const float*, int, const EpiBiasSilu&, int32_t*,
                                 cudaStream_t, cudaError_t*) {
  return false;
}

}  // namespace imba
