// Dense projections Y = X · Wᵀ for the verify block.
//
// bf16 path (tcgen05): "swap-AB" weight streaming.  The weight tile (128 output rows x
// 64 K, TMA, 128-byte swizzle) is the MMA A operand, the activation tile (NT tokens x 64 K)
// is the B operand, the fp32 accumulator [128 x NT] lives in TMEM.  One elected thread
// issues TMA, one issues tcgen05.mma, four warps drain TMEM.  A fixed split of K (chosen
// from N and K only, never from the token count) spreads each GEMM over up to 3 x 148 CTAs;
// partial sums land in ws[split][token][row] and the consumer kernel adds them in split
// order, so every token row is computed by the same arithmetic whatever the batch size.
//
// fp32 path (CUDA cores): register-tiled 64x32 tiles through shared memory, fixed split of K.
#include <algorithm>

#include "internal.hpp"

namespace {

constexpr int A_STAGE_BYTES = GEMM_BM * GEMM_BK * 2;  // 16 KiB

template <int NT>
struct TcCfg {
  static constexpr int B_STAGE_BYTES = NT * GEMM_BK * 2;
  // NT = 16: 4 stages (~75 KB): three CTAs per SM, and room beside the next kernel's CTAs
  static constexpr int STAGES = NT <= 16 ? 4 : (NT <= 64 ? 4 : 3);
  static constexpr int STAGE_BYTES = A_STAGE_BYTES + B_STAGE_BYTES;
  static constexpr int TMEM_COLS = NT < 32 ? 32 : NT;
  static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 + 256;
};

template <int NT>
__global__ void __launch_bounds__(192, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmA2,
                   const __grid_constant__ CUtensorMap tmB, float* __restrict__ ws, int N, int K, int M, int splits,
                   int dual, __nv_bfloat16* __restrict__ act, int ld_act, EvsDevErr* err) {
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
  // token tile fastest: the CTAs that share a weight tile run side by side and share its L2 lines
  const int ttile = blockIdx.x, tile = blockIdx.y, split = blockIdx.z;
  const int kblocks = K / GEMM_BK;
  const int kb_begin = static_cast<int>(static_cast<long long>(kblocks) * split / splits);
  const int kb_end = static_cast<int>(static_cast<long long>(kblocks) * (split + 1) / splits);
  const int nkb = kb_end - kb_begin;
  pdl_trigger();

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
    // the weights stream through once per forward: evict them first, so that the states, caches
    // and partial sums of the small kernels stay in L2
    const uint64_t pol = l2_policy_evict_first();
    auto load_a = [&](int i, int s) {
      const int kx = (kb_begin + i) * GEMM_BK;
      uint8_t* a_dst = sA + s * A_STAGE_BYTES;
      if (dual) {
        tma_load_2d_hint(&tmA, &full[s], a_dst, kx, tile * (GEMM_BM / 2), pol);
        tma_load_2d_hint(&tmA2, &full[s], a_dst + A_STAGE_BYTES / 2, kx, tile * (GEMM_BM / 2), pol);
      } else {
        tma_load_2d_hint(&tmA, &full[s], a_dst, kx, tile * GEMM_BM, pol);
      }
    };
    auto load_b = [&](int i, int s) {
      tma_load_2d(&tmB, &full[s], sB + s * C::B_STAGE_BYTES, (kb_begin + i) * GEMM_BK, ttile * NT);
    };
    // the weights do not depend on earlier kernels: fill every stage with them before waiting
    // for the kernel that produces the activations (programmatic dependent launch)
    const int pre = nkb < C::STAGES ? nkb : C::STAGES;
    for (int i = 0; i < pre; ++i) {
      mbar_arrive_expect_tx(&full[i], C::STAGE_BYTES);
      load_a(i, i);
    }
    pdl_wait();
    for (int i = 0; i < pre; ++i) load_b(i, i);
    for (int i = pre; i < nkb; ++i) {
      const int s = i % C::STAGES;
      const uint32_t ph = (i / C::STAGES) & 1;
      if (!mbar_wait_bounded(&empty[s], ph ^ 1, err, EVS_K_GEMM_TC, 1)) break;
      mbar_arrive_expect_tx(&full[s], C::STAGE_BYTES);
      load_a(i, s);
      load_b(i, s);
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
    pdl_wait();  // (already satisfied: the MMAs consumed activations loaded after the wait)
    if (ok && act != nullptr) {
      // fused SwiGLU (dual tile, one split): TMEM lanes 0-63 hold w1 features tile*64 + r, lanes
      // 64-127 the same w2 features; the w2 half goes through the idle stage memory to the w1 half,
      // which writes silu(g1) * g2 as the bf16 activation of the w3 projection
      float* g2s = reinterpret_cast<float*>(sA);  // [64][NT + 1]; every stage has been consumed
      float v[NT];
#pragma unroll
      for (int c0 = 0; c0 < NT; c0 += 16)
        tmem_ld_32x32b_x16(tmem_base + (static_cast<uint32_t>(q * 32) << 16) + c0,
                           *reinterpret_cast<float(*)[16]>(v + c0));
      tmem_ld_wait();
      if (q >= 2) {
#pragma unroll
        for (int j = 0; j < NT; ++j) g2s[((q - 2) * 32 + lane) * (NT + 1) + j] = v[j];
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");  // the four epilogue warps
      if (q < 2) {
        const int f = tile * 64 + q * 32 + lane;
#pragma unroll
        for (int j = 0; j < NT; ++j) {
          const int tok = ttile * NT + j;
          if (tok < M)
            act[static_cast<size_t>(tok) * ld_act + f] = __float2bfloat16_rn(swiglu_gate(v[j], g2s[(q * 32 + lane) * (NT + 1) + j]));
        }
      }
    } else if (ok) {
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

// Large token counts (prefill): the CTA of (token tile, weight tile) walks every split of the
// fixed split plan in order.  Each split is accumulated from zero in its own TMEM buffer by the same
// MMA sequence as in gemm_tc_kernel, and the epilogue adds the splits into a running fp32 sum
// (0 + s0 + s1 + ..., the consumers' order of additions).  The sum is stored as the only split:
// a consumer reading one split computes 0 + sum = sum, so every row gets the bits of the split-K
// path without writing and re-reading the per-split partial sums.  Two TMEM buffers alternate:
// the MMA of split s + 2 waits until the epilogue has read split s.
constexpr int SER_NT = 128;   // wide token tile (GEMM_NT[2])
constexpr int SER_NT_N = 96;  // narrow token tile (GEMM_NT[3])
// two CTAs per SM (registers <= 168): one CTA's epilogue and another's main loop overlap
template <int NT>
__global__ void __launch_bounds__(192, 2)
    gemm_tc_serial_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmA2,
                          const __grid_constant__ CUtensorMap tmB, float* __restrict__ ws, int N, int K, int M,
                          int splits, int dual, EvsDevErr* err) {
  using C = TcCfg<NT>;
  constexpr uint32_t TMEM_SER = 2 * NT <= 128 ? 128 : 256;  // two accumulators, a power of two
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + C::STAGES * A_STAGE_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::STAGES * C::STAGE_BYTES);
  uint64_t* empty = full + C::STAGES;
  uint64_t* accf = empty + C::STAGES;  // [2] split accumulated
  uint64_t* acce = accf + 2;           // [2] split read by the epilogue
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acce + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ttile = blockIdx.x, tile = blockIdx.y;
  const int kblocks = K / GEMM_BK;
  pdl_trigger();

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accf[b], 1);
      mbar_init(&acce[b], 128);
    }
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_SER);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0 && lane == 0) {
    // every k-block in order (the splits' ranges concatenated)
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
    if (dual) prefetch_tmap(&tmA2);
    const uint64_t pol = l2_policy_evict_first();
    auto load_a = [&](int kb, int s) {
      const int kx = kb * GEMM_BK;
      uint8_t* a_dst = sA + s * A_STAGE_BYTES;
      if (dual) {
        tma_load_2d_hint(&tmA, &full[s], a_dst, kx, tile * (GEMM_BM / 2), pol);
        tma_load_2d_hint(&tmA2, &full[s], a_dst + A_STAGE_BYTES / 2, kx, tile * (GEMM_BM / 2), pol);
      } else {
        tma_load_2d_hint(&tmA, &full[s], a_dst, kx, tile * GEMM_BM, pol);
      }
    };
    auto load_b = [&](int kb, int s) {
      tma_load_2d(&tmB, &full[s], sB + s * C::B_STAGE_BYTES, kb * GEMM_BK, ttile * NT);
    };
    const int pre = kblocks < C::STAGES ? kblocks : C::STAGES;
    for (int i = 0; i < pre; ++i) {
      mbar_arrive_expect_tx(&full[i], C::STAGE_BYTES);
      load_a(i, i);
    }
    pdl_wait();
    for (int i = 0; i < pre; ++i) load_b(i, i);
    for (int i = pre; i < kblocks; ++i) {
      const int s = i % C::STAGES;
      if (!mbar_wait_bounded(&empty[s], ((i / C::STAGES) & 1) ^ 1, err, EVS_K_GEMM_TC, 41)) break;
      mbar_arrive_expect_tx(&full[s], C::STAGE_BYTES);
      load_a(i, s);
      load_b(i, s);
    }
  } else if (warp == 1 && lane == 0) {
    constexpr uint32_t idesc = umma_idesc_bf16(GEMM_BM, NT);
    bool ok = true;
    for (int sp = 0; sp < splits && ok; ++sp) {
      const int kb0 = static_cast<int>(static_cast<long long>(kblocks) * sp / splits);
      const int kb1 = static_cast<int>(static_cast<long long>(kblocks) * (sp + 1) / splits);
      const int buf = sp & 1;
      if (sp >= 2 && !mbar_wait_bounded(&acce[buf], ((sp >> 1) - 1) & 1, err, EVS_K_GEMM_TC, 42)) break;
      tc_fence_after();
      for (int kb = kb0; kb < kb1; ++kb) {
        const int s = kb % C::STAGES;
        if (!mbar_wait_bounded(&full[s], (kb / C::STAGES) & 1, err, EVS_K_GEMM_TC, 43)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t a0 = smem_u32(sA + s * A_STAGE_BYTES);
        const uint32_t b0 = smem_u32(sB + s * C::B_STAGE_BYTES);
#pragma unroll
        for (int j = 0; j < GEMM_BK / 16; ++j)
          tc_mma_f16(tmem_base + buf * NT, umma_desc_sw128(a0 + j * 32), umma_desc_sw128(b0 + j * 32), idesc,
                     (kb != kb0 || j != 0) ? 1u : 0u);
        tc_commit(&empty[s]);
      }
      if (ok) tc_commit(&accf[buf]);
    }
  } else if (warp >= 2) {
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    float sum[NT];
#pragma unroll
    for (int j = 0; j < NT; ++j) sum[j] = 0.f;
    bool ok = true;
    for (int sp = 0; sp < splits; ++sp) {
      const int buf = sp & 1;
      ok = mbar_wait_bounded(&accf[buf], (sp >> 1) & 1, err, EVS_K_GEMM_TC, 44);
      if (!ok) break;
      tc_fence_after();
#pragma unroll
      for (int c0 = 0; c0 < NT; c0 += 16) {
        float v[16];
        tmem_ld_32x32b_x16(tmem_base + (static_cast<uint32_t>(q * 32) << 16) + buf * NT + c0, v);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 16; ++j) sum[c0 + j] += v[j];
      }
      tc_fence_before();
      asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&acce[buf])) : "memory");
    }
    pdl_wait();  // (already satisfied: the MMAs consumed activations loaded after the wait)
    if (ok) {
      const int row = tile * GEMM_BM + q * 32 + lane;
#pragma unroll
      for (int j = 0; j < NT; ++j) {
        const int tok = ttile * NT + j;
        if (tok < M) ws[static_cast<size_t>(tok) * N + row] = sum[j];
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_SER);
  }
}

// fp32 projection for few token rows (the drafter, fp32 targets): CTA = 8 warps x 4 weight rows,
// one split of K (SK_KC <= 1024 columns) and up to 16 token rows.  The token rows of the split are
// staged in shared memory with 16-byte asynchronous copies; each warp streams its 4 weight rows
// with coalesced float4 loads (lane l takes columns 4l..4l+3 of every 128) and keeps 4 x 16
// accumulators.  Lane partials are summed in lane order through shared memory, so an output's
// arithmetic does not depend on its token slot or on M (row invariance).  Partials go to
// ws[split][row][col]; dual: virtual row v is w_{(v % 128) / 64} feature (v / 128) * 64 + v % 64.
constexpr int SK_WARPS = 8, SK_R = 4, SK_ROWS = SK_WARPS * SK_R, SK_TOK = 16, SK_KC_MAX = 1024;
constexpr size_t SK_SMEM = sizeof(float) * SK_TOK * SK_KC_MAX;  // also holds 8 x 64 x 32 lane partials

// One CTA's work: weight rows n0 .. n0+SK_ROWS-1, split sp, token groups z0, z0 + zs, ... below
// M_rows.  xrow(m) is token row m of the activations.
template <typename XRow>
__device__ __forceinline__ void skinny_cta(const float* __restrict__ W, const float* __restrict__ W2, XRow xrow,
                                           float* __restrict__ ws, int N, int K, int M, int kc, int dual, int M_rows,
                                           int n0, int sp, int z0, int zs, float* sk_sm) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int m0 = z0 * SK_TOK; m0 < M_rows; m0 += zs * SK_TOK) {
    if (m0 != z0 * SK_TOK) __syncthreads();  // the previous group's partials are read
    const int mt = min(SK_TOK, M_rows - m0);
    const int kb = sp * kc, ke = min(K, kb + kc);  // this CTA's K range, staged SK_KC_MAX columns at a time
    const float* wr[SK_R];
#pragma unroll
    for (int i = 0; i < SK_R; ++i) {
      const int v = n0 + warp * SK_R + i;
      const int vr = v < N ? v : N - 1;
      if (dual) {
        const int f = (vr / 128) * 64 + (vr % 64);
        wr[i] = ((vr % 128) < 64 ? W : W2) + static_cast<size_t>(f) * K;
      } else {
        wr[i] = W + static_cast<size_t>(vr) * K;
      }
    }
    float acc[SK_R][SK_TOK];
#pragma unroll
    for (int i = 0; i < SK_R; ++i)
#pragma unroll
      for (int m = 0; m < SK_TOK; ++m) acc[i][m] = 0.f;
    for (int cb = kb; cb < ke; cb += SK_KC_MAX) {
      const int kw = min(SK_KC_MAX, ke - cb);  // multiple of 4
      // stage X[m0 .. m0+mt)[cb .. cb+kw) as xs[m][k - cb] (row stride SK_KC_MAX)
      const int c4 = kw / 4;
      if (cb != kb) __syncthreads();  // every warp is done with the previous stage
      for (int i = threadIdx.x; i < mt * c4; i += blockDim.x) {
        const int m = i / c4, c = i - m * c4;
        cp_async16(sk_sm + m * SK_KC_MAX + 4 * c, xrow(m0 + m) + cb + 4 * c);
      }
      cp_async_commit();
      cp_async_wait<0>();
      __syncthreads();
#pragma unroll 2
      for (int k = 4 * lane; k < kw; k += 128) {
        float4 w4[SK_R];
#pragma unroll
        for (int i = 0; i < SK_R; ++i) w4[i] = __ldg(reinterpret_cast<const float4*>(wr[i] + cb + k));
#pragma unroll
        for (int m = 0; m < SK_TOK; ++m) {
          if (m < mt) {
            const float4 x4 = *reinterpret_cast<const float4*>(sk_sm + m * SK_KC_MAX + k);
#pragma unroll
            for (int i = 0; i < SK_R; ++i) {
              acc[i][m] = fmaf(w4[i].x, x4.x, acc[i][m]);
              acc[i][m] = fmaf(w4[i].y, x4.y, acc[i][m]);
              acc[i][m] = fmaf(w4[i].z, x4.z, acc[i][m]);
              acc[i][m] = fmaf(w4[i].w, x4.w, acc[i][m]);
            }
          }
        }
      }
    }
    __syncthreads();  // xs no longer needed: reuse it for the lane partials
    float* red = sk_sm + warp * (SK_R * SK_TOK * 32);
#pragma unroll
    for (int i = 0; i < SK_R; ++i)
#pragma unroll
      for (int m = 0; m < SK_TOK; ++m) {
        const int v = i * SK_TOK + m;
        red[v * 32 + (lane ^ (v & 31))] = acc[i][m];
      }
    __syncwarp();
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int v = lane + 32 * h;
      const int i = v / SK_TOK, m = v % SK_TOK;
      float sum = 0.f;
      for (int j = 0; j < 32; ++j) sum += red[v * 32 + (j ^ (v & 31))];
      const int n = n0 + warp * SK_R + i;
      if (m < mt && n < N) ws[(static_cast<size_t>(sp) * M + m0 + m) * N + n] = sum;
    }
  }
}


__global__ void __launch_bounds__(SK_WARPS * 32) gemm_skinny_f32_kernel(const float* __restrict__ W,
                                                                        const float* __restrict__ W2,
                                                                        const float* __restrict__ X, int ldx,
                                                                        float* __restrict__ ws, int N, int K, int M,
                                                                        int kc, int dual,
                                                                        const int32_t* __restrict__ m_dev) {
  extern __shared__ __align__(16) float sk_sm[];
  pdl_trigger();
  pdl_wait();
  // a device-side row count (rows decided by an earlier kernel): token groups past it have no work
  // (M stays the partial buffers' row stride).  The grid may hold fewer token groups than M: a CTA
  // then takes groups blockIdx.z, blockIdx.z + gridDim.z, ... (the arithmetic of a group is the same)
  const int M_rows = m_dev != nullptr ? min(M, *m_dev) : M;
  skinny_cta(W, W2, [&](int m) { return X + static_cast<size_t>(m) * ldx; }, ws, N, K, M, kc, dual, M_rows,
             static_cast<int>(blockIdx.x) * SK_ROWS, static_cast<int>(blockIdx.y), static_cast<int>(blockIdx.z),
             static_cast<int>(gridDim.z), sk_sm);
}

// Several projections of the same shape (N x K, one plan) in one launch: job j = blockIdx.x / tiles
// runs gemm_skinny_f32_kernel's CTA on its own weights, rows and partial buffer.  Token row m of a
// job is row m of X0 below msplit and row m - msplit of X1 from there.
__global__ void __launch_bounds__(SK_WARPS * 32) gemm_skinny_f32_jobs_kernel(const __grid_constant__ SkJobs jobs,
                                                                             int tiles, int N, int K, int ldx,
                                                                             int kc) {
  extern __shared__ __align__(16) float sk_sm[];
  pdl_trigger();
  pdl_wait();
  const int j = static_cast<int>(blockIdx.x) / tiles, tile = static_cast<int>(blockIdx.x) - j * tiles;
  const SkJob& J = jobs.j[j];
  const int M_rows = J.m_dev != nullptr ? min(J.M, *J.m_dev) : J.M;
  const float* X0 = J.X0;
  const float* X1 = J.X1;
  const int ms = J.msplit;
  skinny_cta(J.W, J.W,
             [&](int m) { return m < ms ? X0 + static_cast<size_t>(m) * ldx : X1 + static_cast<size_t>(m - ms) * ldx; },
             J.ws, N, K, J.M, kc, 0, M_rows, tile * SK_ROWS, static_cast<int>(blockIdx.y),
             static_cast<int>(blockIdx.z), static_cast<int>(gridDim.z), sk_sm);
}

__global__ void reduce_splits_kernel(const float* __restrict__ ws, int splits, int MN, const float* __restrict__ bias,
                                     int N, float* __restrict__ out, const int32_t* __restrict__ m_dev) {
  pdl_trigger();
  pdl_wait();
  // grid-stride over the rows below the device-side count (the grid may cover fewer)
  const int lim = m_dev != nullptr ? min(MN, *m_dev * N) : MN;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < lim; i += gridDim.x * blockDim.x) {
    float acc = split_sum(ws + i, MN, splits);
    out[i] = bias ? acc + bias[i % N] : acc;
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
              EvsDevErr* err, cudaStream_t st, bool pdl, __nv_bfloat16* act, int ld_act) {
  static_assert(NT % 16 == 0 && NT <= 256, "UMMA N");
  using C = TcCfg<NT>;
  static std::atomic<unsigned long long> attr_devs{0};
  EVS_TRY(smem_attr_once(attr_devs, reinterpret_cast<const void*>(gemm_tc_kernel<NT>), C::SMEM));
  dim3 grid((p.M + NT - 1) / NT, p.N / GEMM_BM, p.splits);
  EVS_CUDA_TRY(evs_launch(gemm_tc_kernel<NT>, grid, dim3(192), C::SMEM, st, pdl, *tmA, tmA2 ? *tmA2 : *tmA, *tmB,
                          ws, p.N, p.K, p.M, p.splits, p.dual, act, ld_act, err));
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
  if (m->cfg.dtype != EVS_DTYPE_BF16) return gemm_plan_f32(N, K, M, dual);
  const int kblocks = K / GEMM_BK;
  const int tiles = N / GEMM_BM;
  // as many splits as keep every CTA resident at once (three per SM at the 16-token tile): more
  // CTAs streaming the same bytes, each over fewer k-blocks.  From N and K only (row invariance).
  int splits = 1;
  while (tiles * (splits + 1) <= 3 * 148 && splits < kblocks && splits < 16) ++splits;
  p.splits = splits;
  return p;
}

// fp32 projection plan, from N and K only: K chunks of at most 1024 columns (multiples of 128),
// shrunk until one token group gives >= 2 CTAs per SM
GemmPlan gemm_plan_f32(int N, int K, int M, int dual) {
  GemmPlan p{N, K, M, 1, dual};
  const int tiles = (N + SK_ROWS - 1) / SK_ROWS;
  int kc = std::min(SK_KC_MAX, (K + 127) / 128 * 128);
  while (kc > 128 && tiles * ((K + kc - 1) / kc) < 296) kc -= 128;
  p.kchunk = kc;
  p.splits = (K + kc - 1) / kc;
  return p;
}

// drafter projections: one split (no reduction launch) when the GEMM has at least 128 row tiles;
// otherwise K is split until about two CTAs per SM stream it (K chunks of at least 128 columns)
GemmPlan gemm_plan_f32_drafter(int N, int K, int M) {
  GemmPlan p{N, K, M, 1, 0};
  const int tiles = (N + SK_ROWS - 1) / SK_ROWS;
  int splits = 1;
  while (tiles < 128 && tiles * splits < 296 && splits < K / 128) ++splits;
  p.kchunk = (K + splits - 1) / splits;
  p.kchunk = (p.kchunk + 127) / 128 * 128;
  p.splits = (K + p.kchunk - 1) / p.kchunk;
  return p;
}

// Whether a projection of M token rows runs gemm_tc_serial_kernel: many token rows (a prefill
// chunk), and at least one wave of (token tile, weight tile) CTAs.  The choice changes no bit.
bool gemm_serial(const GemmPlan& p) {
  const long long ctas = static_cast<long long>((p.M + SER_NT - 1) / SER_NT) * (p.N / GEMM_BM);
  return p.M >= 512 && p.splits > 1 && ctas >= 148;
}

int launch_gemm_tc_serial(const CUtensorMap* tmA, const CUtensorMap* tmA2, const CUtensorMap* tmB, const GemmPlan& p,
                          float* ws, EvsDevErr* err, cudaStream_t st, bool pdl) {
  EVS_CHECK_ARG(p.N % GEMM_BM == 0 && p.K % GEMM_BK == 0, "tcgen05 GEMM needs N % 128 == 0 and K % 64 == 0");
  EVS_CHECK_ARG(p.splits >= 1 && p.splits <= p.K / GEMM_BK, "bad split count");
  if (p.M <= 0) return EVS_OK;
  static_assert(GEMM_NT[2] == SER_NT && GEMM_NT[3] == SER_NT_N, "the serial kernel's token tiles");
  // the narrow token tile when its CTAs take no more rounds (two CTAs per SM) than the wide tile's:
  // each CTA then does three quarters of the work (measured at 832 rows: -4 % on the in-, out- and
  // w3 projections; the w1/w2 projection, one round more with it, +8 %).  The tile changes no bit
  // (every token row runs the same MMA sequence and the same additions).
  const long long tiles = p.N / GEMM_BM, slots = 2LL * 148;
  auto rounds = [&](int nt) { return (static_cast<long long>((p.M + nt - 1) / nt) * tiles + slots - 1) / slots; };
  const bool narrow = rounds(SER_NT_N) <= rounds(SER_NT);
  auto launch = [&](auto kern, int nt, size_t smem, const CUtensorMap* tb, std::atomic<unsigned long long>& attr) -> int {
    EVS_TRY(smem_attr_once(attr, reinterpret_cast<const void*>(kern), static_cast<int>(smem)));
    dim3 grid((p.M + nt - 1) / nt, p.N / GEMM_BM, 1);
    EVS_CUDA_TRY(evs_launch(kern, grid, dim3(192), smem, st, pdl, *tmA, tmA2 ? *tmA2 : *tmA, *tb, ws, p.N, p.K, p.M,
                            p.splits, p.dual, err));
    evs_count_launch(1);
    return EVS_OK;
  };
  static std::atomic<unsigned long long> attr_w{0}, attr_n{0};
  if (narrow)
    return launch(gemm_tc_serial_kernel<SER_NT_N>, SER_NT_N, TcCfg<SER_NT_N>::SMEM, &tmB[3], attr_n);
  return launch(gemm_tc_serial_kernel<SER_NT>, SER_NT, TcCfg<SER_NT>::SMEM, &tmB[2], attr_w);
}

int gemm_tile_index(int M) { return M <= GEMM_NT[0] ? 0 : (M <= GEMM_NT[1] ? 1 : 2); }

int launch_gemm_tc(const CUtensorMap* tmA, const CUtensorMap* tmA2, const CUtensorMap* tmB, const GemmPlan& p,
                   float* ws, EvsDevErr* err, cudaStream_t st, bool pdl, void* swiglu_act, int ld_act) {
  EVS_CHECK_ARG(swiglu_act == nullptr || (p.dual && p.splits == 1), "fused SwiGLU needs the dual tile and one split");
  EVS_CHECK_ARG(p.N % GEMM_BM == 0 && p.K % GEMM_BK == 0, "tcgen05 GEMM needs N % 128 == 0 and K % 64 == 0");
  EVS_CHECK_ARG(p.splits >= 1 && p.splits <= p.K / GEMM_BK, "bad split count");
  if (p.M <= 0) return EVS_OK;
  switch (gemm_tile_index(p.M)) {
    case 0: return launch_tc<GEMM_NT[0]>(tmA, tmA2, &tmB[0], p, ws, err, st, pdl, static_cast<__nv_bfloat16*>(swiglu_act), ld_act);
    case 1: return launch_tc<GEMM_NT[1]>(tmA, tmA2, &tmB[1], p, ws, err, st, pdl, static_cast<__nv_bfloat16*>(swiglu_act), ld_act);
    default: return launch_tc<GEMM_NT[2]>(tmA, tmA2, &tmB[2], p, ws, err, st, pdl, static_cast<__nv_bfloat16*>(swiglu_act), ld_act);
  }
}

int launch_gemm_simt(const void* W, const void* W2, const void* X, int ldx, int dtype, const GemmPlan& p, float* ws,
                     cudaStream_t st, bool pdl, const int32_t* m_dev, int m_hint) {
  if (p.M <= 0) return EVS_OK;
  EVS_CHECK_ARG(dtype == EVS_DTYPE_FP32, "CUDA-core projection is fp32 only");
  EVS_CHECK_ARG(p.K % 4 == 0 && ldx % 4 == 0 && reinterpret_cast<uintptr_t>(X) % 16 == 0 &&
                    reinterpret_cast<uintptr_t>(W) % 16 == 0,
                "fp32 projection needs K and the row stride multiples of 4 and 16-byte aligned operands");
  EVS_CHECK_ARG(p.kchunk > 0 && p.kchunk % 128 == 0 && p.splits * p.kchunk >= p.K, "bad fp32 projection plan");
  static std::atomic<unsigned long long> attr_devs{0};
  EVS_TRY(smem_attr_once(attr_devs, reinterpret_cast<const void*>(gemm_skinny_f32_kernel), static_cast<int>(SK_SMEM)));
  const size_t smem = SK_SMEM;
  // with a device-side row count, token groups for about m_hint rows (the CTAs walk the rest)
  const int ngroups = (p.M + SK_TOK - 1) / SK_TOK;
  const int zg = m_dev != nullptr && m_hint > 0 ? std::min(ngroups, (m_hint + SK_TOK - 1) / SK_TOK) : ngroups;
  dim3 grid((p.N + SK_ROWS - 1) / SK_ROWS, p.splits, zg);
  EVS_CUDA_TRY(evs_launch(gemm_skinny_f32_kernel, grid, dim3(SK_WARPS * 32), smem, st, pdl,
                          static_cast<const float*>(W), static_cast<const float*>(W2 ? W2 : W),
                          static_cast<const float*>(X), ldx, ws, p.N, p.K, p.M, p.kchunk, p.dual, m_dev));
  evs_count_launch(1);
  return EVS_OK;
}

int launch_gemm_simt_jobs(const SkJobs& jobs, int n_jobs, int ldx, const GemmPlan& p, cudaStream_t st, bool pdl,
                          int m_hint) {
  EVS_CHECK_ARG(n_jobs >= 1 && n_jobs <= SK_MAX_JOBS, "1 to 3 projection jobs");
  EVS_CHECK_ARG(p.K % 4 == 0 && ldx % 4 == 0 && p.N % SK_ROWS == 0, "fp32 projection jobs need K, ldx % 4 and N % 32");
  EVS_CHECK_ARG(p.kchunk > 0 && p.kchunk % 128 == 0 && p.splits * p.kchunk >= p.K, "bad fp32 projection plan");
  int groups = 0;
  for (int j = 0; j < n_jobs; ++j) {
    const SkJob& J = jobs.j[j];
    EVS_CHECK_ARG(J.W && J.X0 && J.ws && J.M >= 0 && (J.X1 || J.msplit >= J.M), "bad projection job");
    EVS_CHECK_ARG(reinterpret_cast<uintptr_t>(J.W) % 16 == 0 && reinterpret_cast<uintptr_t>(J.X0) % 16 == 0 &&
                      reinterpret_cast<uintptr_t>(J.X1) % 16 == 0,
                  "fp32 projection jobs need 16-byte aligned operands");
    const int rows = J.m_dev != nullptr && m_hint > 0 ? std::min(J.M, m_hint) : J.M;
    groups = std::max(groups, (rows + SK_TOK - 1) / SK_TOK);
  }
  if (groups == 0) return EVS_OK;
  static std::atomic<unsigned long long> attr_devs{0};
  EVS_TRY(smem_attr_once(attr_devs, reinterpret_cast<const void*>(gemm_skinny_f32_jobs_kernel),
                         static_cast<int>(SK_SMEM)));
  const int tiles = p.N / SK_ROWS;
  dim3 grid(tiles * n_jobs, p.splits, groups);
  EVS_CUDA_TRY(evs_launch(gemm_skinny_f32_jobs_kernel, grid, dim3(SK_WARPS * 32), SK_SMEM, st, pdl, jobs, tiles, p.N,
                          p.K, ldx, p.kchunk));
  evs_count_launch(1);
  return EVS_OK;
}

int launch_reduce_splits(const float* ws, int splits, int M, int N, const float* bias, float* out, cudaStream_t st,
                         bool pdl, const int32_t* m_dev, int m_hint) {
  const int MN = M * N;
  if (MN <= 0) return EVS_OK;
  const int rows = m_dev != nullptr && m_hint > 0 ? std::min(M, m_hint) : M;
  EVS_CUDA_TRY(evs_launch(reduce_splits_kernel, dim3((rows * N + 255) / 256), dim3(256), 0, st, pdl, ws, splits, MN,
                          bias, N, out, m_dev));
  evs_count_launch(1);
  return EVS_OK;
}
