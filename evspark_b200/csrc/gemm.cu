// Dense projections Y = X · Wᵀ for the verify block.
//
// bf16 path (tcgen05): "swap-AB" weight streaming.  The weight tile (128 output rows x
// 64 K, TMA, 128-byte swizzle) is the MMA A operand, the activation tile (NT tokens x 64 K)
// is the B operand, the fp32 accumulator [128 x NT] lives in TMEM.  One elected thread
// issues TMA, one issues tcgen05.mma, four warps drain TMEM.  A fixed split of K (chosen
// from N and K only, never from the token count) spreads each GEMM over >= 148 CTAs;
// partial sums land in ws[split][token][row] and the consumer kernel adds them in split
// order, so every token row is computed by the same arithmetic whatever the batch size.
//
// fp32 path (SIMT): one warp per output row, lanes stride K, fixed butterfly reduction.
#include "internal.hpp"

namespace {

constexpr int A_STAGE_BYTES = GEMM_BM * GEMM_BK * 2;  // 16 KiB

template <int NT>
struct TcCfg {
  static constexpr int B_STAGE_BYTES = NT * GEMM_BK * 2;
  static constexpr int STAGES = NT <= 16 ? 5 : (NT <= 64 ? 4 : 3);
  static constexpr int STAGE_BYTES = A_STAGE_BYTES + B_STAGE_BYTES;
  static constexpr int TMEM_COLS = NT < 32 ? 32 : NT;
  static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 + 256;
};

template <int NT>
__global__ void __launch_bounds__(192, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmA2,
                   const __grid_constant__ CUtensorMap tmB, float* __restrict__ ws, int N, int K, int M, int splits,
                   int dual, EvsDevErr* err) {
  using C = TcCfg<NT>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + C::STAGES * A_STAGE_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::STAGES * C::STAGE_BYTES);
  uint64_t* empty = full + C::STAGES;
  uint64_t* accum = empty + C::STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x, split = blockIdx.y, ttile = blockIdx.z;
  const int kblocks = K / GEMM_BK;
  const int kb_begin = static_cast<int>(static_cast<long long>(kblocks) * split / splits);
  const int kb_end = static_cast<int>(static_cast<long long>(kblocks) * (split + 1) / splits);
  const int nkb = kb_end - kb_begin;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accum, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
    if (dual) prefetch_tmap(&tmA2);
    for (int i = 0; i < nkb; ++i) {
      const int s = i % C::STAGES;
      const uint32_t ph = (i / C::STAGES) & 1;
      if (i >= C::STAGES && !mbar_wait_bounded(&empty[s], ph ^ 1, err, EVS_K_GEMM_TC, 1)) break;
      mbar_arrive_expect_tx(&full[s], C::STAGE_BYTES);
      const int kx = (kb_begin + i) * GEMM_BK;
      uint8_t* a_dst = sA + s * A_STAGE_BYTES;
      if (dual) {
        tma_load_2d(&tmA, &full[s], a_dst, kx, tile * (GEMM_BM / 2));
        tma_load_2d(&tmA2, &full[s], a_dst + A_STAGE_BYTES / 2, kx, tile * (GEMM_BM / 2));
      } else {
        tma_load_2d(&tmA, &full[s], a_dst, kx, tile * GEMM_BM);
      }
      tma_load_2d(&tmB, &full[s], sB + s * C::B_STAGE_BYTES, kx, ttile * NT);
    }
  } else if (warp == 1 && lane == 0) {
    constexpr uint32_t idesc = umma_idesc_bf16(GEMM_BM, NT);
    for (int i = 0; i < nkb; ++i) {
      const int s = i % C::STAGES;
      const uint32_t ph = (i / C::STAGES) & 1;
      if (!mbar_wait_bounded(&full[s], ph, err, EVS_K_GEMM_TC, 2)) break;
      tc_fence_after();
      const uint32_t a0 = smem_u32(sA + s * A_STAGE_BYTES);
      const uint32_t b0 = smem_u32(sB + s * C::B_STAGE_BYTES);
#pragma unroll
      for (int j = 0; j < GEMM_BK / 16; ++j) {
        tc_mma_f16(tmem_base, umma_desc_sw128(a0 + j * 32), umma_desc_sw128(b0 + j * 32), idesc,
                   (i | j) != 0 ? 1u : 0u);
      }
      tc_commit(&empty[s]);
    }
    tc_commit(accum);
  } else if (warp >= 2) {
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    const bool ok = mbar_wait_bounded(accum, 0, err, EVS_K_GEMM_TC, 3);
    tc_fence_after();
    if (ok) {
      const int row = tile * GEMM_BM + q * 32 + lane;
#pragma unroll
      for (int c0 = 0; c0 < NT; c0 += 16) {
        float v[16];
        tmem_ld_32x32b_x16(tmem_base + (static_cast<uint32_t>(q * 32) << 16) + c0, v);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int tok = ttile * NT + c0 + j;
          if (tok < M) ws[(static_cast<size_t>(split) * M + tok) * N + row] = v[j];
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

template <typename TW, typename TX>
__global__ void __launch_bounds__(128) gemm_simt_kernel(const TW* __restrict__ W, const TW* __restrict__ W2,
                                                        const TX* __restrict__ X, int ldx, float* __restrict__ ws,
                                                        int N, int K, int M, int splits, int dual) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n = blockIdx.x * 4 + warp;
  if (n >= N) return;
  const TW* wrow;
  if (dual) {
    const int t = n / GEMM_BM, r = n % GEMM_BM;
    wrow = r < GEMM_BM / 2 ? W + static_cast<size_t>(t * (GEMM_BM / 2) + r) * K
                           : W2 + static_cast<size_t>(t * (GEMM_BM / 2) + r - GEMM_BM / 2) * K;
  } else {
    wrow = W + static_cast<size_t>(n) * K;
  }
  const int split = blockIdx.y;
  const int k0 = static_cast<int>(static_cast<long long>(K) * split / splits);
  const int k1 = static_cast<int>(static_cast<long long>(K) * (split + 1) / splits);
  constexpr int TG = 8;
  for (int t0 = 0; t0 < M; t0 += TG) {
    float acc[TG];
#pragma unroll
    for (int j = 0; j < TG; ++j) acc[j] = 0.f;
    for (int k = k0 + lane; k < k1; k += 32) {
      const float w = to_f32(wrow[k]);
#pragma unroll
      for (int j = 0; j < TG; ++j)
        if (t0 + j < M) acc[j] = fmaf(w, to_f32(X[static_cast<size_t>(t0 + j) * ldx + k]), acc[j]);
    }
#pragma unroll
    for (int j = 0; j < TG; ++j) acc[j] = warp_sum(acc[j]);
    if (lane == 0) {
#pragma unroll
      for (int j = 0; j < TG; ++j)
        if (t0 + j < M) ws[(static_cast<size_t>(split) * M + t0 + j) * N + n] = acc[j];
    }
  }
}

typedef CUresult (*PFN_encodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                    const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                    CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

PFN_encodeTiled get_encode() {
  static PFN_encodeTiled fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_encodeTiled>(p);
  }
  return fn;
}

template <int NT>
int launch_tc(const CUtensorMap* tmA, const CUtensorMap* tmA2, const CUtensorMap* tmB, const GemmPlan& p, float* ws,
              EvsDevErr* err, cudaStream_t st) {
  using C = TcCfg<NT>;
  static bool attr_set = false;
  if (!attr_set) {
    EVS_CUDA_TRY(cudaFuncSetAttribute(gemm_tc_kernel<NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
    attr_set = true;
  }
  dim3 grid(p.N / GEMM_BM, p.splits, (p.M + NT - 1) / NT);
  gemm_tc_kernel<NT><<<grid, 192, C::SMEM, st>>>(*tmA, tmA2 ? *tmA2 : *tmA, *tmB, ws, p.N, p.K, p.M, p.splits,
                                                  p.dual, err);
  EVS_CUDA_TRY(cudaGetLastError());
  evs_count_launch(1);
  return EVS_OK;
}

}  // namespace

int make_tmap_2d_bf16(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint64_t row_stride_bytes,
                      uint32_t box_inner, uint32_t box_outer) {
  PFN_encodeTiled enc = get_encode();
  if (enc == nullptr) {
    evs_set_last_error(EVS_ECUDA, "cuTensorMapEncodeTiled entry point unavailable");
    return EVS_ECUDA;
  }
  EVS_CHECK_ARG(reinterpret_cast<uintptr_t>(base) % 16 == 0, "TMA base address must be 16-byte aligned");
  EVS_CHECK_ARG(row_stride_bytes % 16 == 0, "TMA row stride must be a multiple of 16 bytes");
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    evs_set_last_error(EVS_ECUDA, "cuTensorMapEncodeTiled failed");
    return EVS_ECUDA;
  }
  return EVS_OK;
}

// Split count depends only on (N, K): at least 148 work units for one token tile.
GemmPlan gemm_plan(const evs_model* m, int N, int K, int M, int dual) {
  GemmPlan p{N, K, M, 1, dual};
  if (m->cfg.dtype != EVS_DTYPE_BF16) return p;
  const int kblocks = K / GEMM_BK;
  const int tiles = N / GEMM_BM;
  int splits = 1;
  while (tiles * splits < 148 && splits < kblocks) ++splits;
  p.splits = splits;
  return p;
}

int launch_gemm_tc(const CUtensorMap* tmA, const CUtensorMap* tmA2, const CUtensorMap* tmB, const GemmPlan& p,
                   float* ws, EvsDevErr* err, cudaStream_t st) {
  EVS_CHECK_ARG(p.N % GEMM_BM == 0 && p.K % GEMM_BK == 0, "tcgen05 GEMM needs N % 128 == 0 and K % 64 == 0");
  EVS_CHECK_ARG(p.splits >= 1 && p.splits <= p.K / GEMM_BK, "bad split count");
  if (p.M <= 0) return EVS_OK;
  return launch_tc<TOK_TILE>(tmA, tmA2, tmB, p, ws, err, st);
}

int launch_gemm_simt(const void* W, const void* W2, const void* X, int ldx, int dtype, const GemmPlan& p, float* ws,
                     cudaStream_t st) {
  if (p.M <= 0) return EVS_OK;
  dim3 grid((p.N + 3) / 4, p.splits);
  if (dtype == EVS_DTYPE_BF16) {
    gemm_simt_kernel<__nv_bfloat16, __nv_bfloat16><<<grid, 128, 0, st>>>(
        static_cast<const __nv_bfloat16*>(W), static_cast<const __nv_bfloat16*>(W2),
        static_cast<const __nv_bfloat16*>(X), ldx, ws, p.N, p.K, p.M, p.splits, p.dual);
  } else {
    gemm_simt_kernel<float, float><<<grid, 128, 0, st>>>(static_cast<const float*>(W),
                                                         static_cast<const float*>(W2),
                                                         static_cast<const float*>(X), ldx, ws, p.N, p.K, p.M,
                                                         p.splits, p.dual);
  }
  EVS_CUDA_TRY(cudaGetLastError());
  evs_count_launch(1);
  return EVS_OK;
}
