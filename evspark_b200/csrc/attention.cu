// Causal multi-head attention of T new queries per row over the KV cache (vortex layout
// [B, Lmax, 2, H, Dh]), bottom-right aligned: query t of row b sits at absolute position
// P = len[b] + t and sees keys 0..P (evspark/specdec/block/chunk.py:34-35; the reference reaches
// flash_attn_with_kvcache through the model forward).
//
//   rope_append_kernel   qkv partials -> rotate-half RoPE (fp64 angle) -> q_rot, K/V cache append
//   attn_block_kernel    one CTA per (64-key block, head, row) staged in shared memory:
//                        partial (max, sum, acc) per query
//   attn_combine_kernel  folds the partials of blocks 0..P/64 in block order
//   attn_fused_kernel    chunks longer than the split-KV query cap (prefill): the same per-block
//                        partials and the same fold inside one CTA per (16 queries, head, row)
//
// Blocks are aligned at absolute key positions and folded in a fixed order, so a query's result
// does not depend on how many other queries share the call (native T=1 == verify T=γ+1).
#include <math_constants.h>

#include <algorithm>

#include "internal.hpp"

namespace {

template <typename TD>
__global__ void rope_append_kernel(const float* __restrict__ ws, int splits, int M, int T, int d, int H, int Dh,
                                   double log_base, const int32_t* __restrict__ len, int Lmax, TD* __restrict__ qrot,
                                   TD* __restrict__ kv, EvsDevErr* err) {
  pdl_trigger();
  pdl_wait();
  const int row = blockIdx.x, h = blockIdx.y, j = threadIdx.x;
  const int half = Dh / 2;
  if (j >= half) return;
  const int b = row / T, t = row % T;
  const int P = len[b] + t;
  if (P >= Lmax) {
    if (j == 0) evs_record_error(err, EVS_ERANGE, EVS_K_ATTN, row);
    return;
  }
  const int N = 3 * d;
  auto val = [&](int c) {
    return round_to<TD>(split_sum(ws + static_cast<size_t>(row) * N + c, static_cast<size_t>(M) * N, splits));
  };
  const int c1 = h * Dh + j, c2 = c1 + half;
  const float q1 = val(c1), q2 = val(c2);
  const float k1 = val(d + c1), k2 = val(d + c2);
  const float v1 = val(2 * d + c1), v2 = val(2 * d + c2);
  const double inv_freq = exp(-(2.0 * j / Dh) * log_base);
  double sn, cs;
  sincos(static_cast<double>(P) * inv_freq, &sn, &cs);
  const float c = static_cast<float>(cs), s = static_cast<float>(sn);
  TD* qo = qrot + static_cast<size_t>(row) * d;
  qo[c1] = from_f32<TD>(q1 * c - q2 * s);
  qo[c2] = from_f32<TD>(q2 * c + q1 * s);
  const size_t HD = static_cast<size_t>(H) * Dh;
  TD* kdst = kv + ((static_cast<size_t>(b) * Lmax + P) * 2 + 0) * HD;
  TD* vdst = kdst + HD;
  kdst[c1] = from_f32<TD>(k1 * c - k2 * s);
  kdst[c2] = from_f32<TD>(k2 * c + k1 * s);
  vdst[c1] = from_f32<TD>(v1);
  vdst[c2] = from_f32<TD>(v2);
}

constexpr int QT = 16;           // queries per pass over the staged keys
constexpr int ATTN_THREADS = 128;
constexpr int QK_Q = QT / (ATTN_THREADS / ATTN_BLOCK);  // queries per thread in the score pass
constexpr int PV_QMAX = 8;       // queries per thread in P.V (head_dim <= 128)

// shared memory of both attention kernels: K and V rows padded by 16 bytes (conflict-free
// row-per-thread reads and 8-row matrix loads), fp32 queries, scores, the P.V tile of the tensor-core
// path and per-query stats (+ the running fold of the fused kernel)
template <typename TD>
__host__ __device__ constexpr size_t attn_smem_bytes(int Dh) {
  return sizeof(TD) * (2 * static_cast<size_t>(ATTN_BLOCK) * (Dh + 16 / sizeof(TD))) +
         sizeof(float) * (2 * static_cast<size_t>(QT) * Dh + static_cast<size_t>(QT) * ATTN_BLOCK + 6 * QT);
}

template <typename TD>
struct AttnSmem {
  TD* Ks;
  TD* Vs;
  float* qs;
  float* S;
  float* stt;   // [2 QT]: block max, block sum
  float* fold;  // [4 QT]: running max, running sum, scale of the old accumulator, scale of the block
  float* O;     // [QT][Dh]: P.V of the tensor-core path
  int kpad;     // row stride of K and V (elements)
  __device__ AttnSmem(unsigned char* raw, int Dh) {
    constexpr int EPC = 16 / sizeof(TD);
    kpad = Dh + EPC;
    Ks = reinterpret_cast<TD*>(raw);
    Vs = Ks + ATTN_BLOCK * kpad;
    qs = reinterpret_cast<float*>(Vs + ATTN_BLOCK * kpad);
    S = qs + QT * Dh;
    stt = S + QT * ATTN_BLOCK;
    fold = stt + 2 * QT;
    O = fold + 4 * QT;
  }
};

// 16-byte asynchronous copies of the K rows [0, nk) of one key block (one commit group)
template <typename TD>
__device__ __forceinline__ void stage_k(const AttnSmem<TD>& sm, const TD* kb, size_t HD, int Dh, int nk) {
  constexpr int EPC = 16 / sizeof(TD);
  const int cpr = Dh / EPC;
  for (int i = threadIdx.x; i < nk * cpr; i += ATTN_THREADS) {
    const int r = i / cpr, c = i - r * cpr;
    cp_async16(sm.Ks + r * sm.kpad + c * EPC, kb + static_cast<size_t>(r) * 2 * HD + c * EPC);
  }
  cp_async_commit();
}
// ... and of its V rows (one commit group); V rows past the block's keys are zero: P is zero
// there, and 0 times stale data could be NaN
template <typename TD>
__device__ __forceinline__ void stage_v(const AttnSmem<TD>& sm, const TD* kb, size_t HD, int Dh, int nk) {
  constexpr int EPC = 16 / sizeof(TD);
  const int cpr = Dh / EPC;
  for (int i = threadIdx.x; i < nk * cpr; i += ATTN_THREADS) {
    const int r = i / cpr, c = i - r * cpr;
    cp_async16(sm.Vs + r * sm.kpad + c * EPC, kb + static_cast<size_t>(r) * 2 * HD + HD + c * EPC);
  }
  cp_async_commit();
  for (int i = nk * cpr + threadIdx.x; i < ATTN_BLOCK * cpr; i += ATTN_THREADS) {
    const int r = i / cpr, c = i - r * cpr;
    *reinterpret_cast<uint4*>(sm.Vs + r * sm.kpad + c * EPC) = make_uint4(0u, 0u, 0u, 0u);
  }
}
template <typename TD>
__device__ __forceinline__ void stage_kv(const AttnSmem<TD>& sm, const TD* kb, size_t HD, int Dh, int nk) {
  stage_k(sm, kb, HD, Dh, nk);
  stage_v(sm, kb, HD, Dh, nk);
}

// query rows per block pass and the bf16 query tile's padded row (272 B for Dh = 128: the MMA
// fragment loads of 8 rows x 4 lanes hit 32 distinct banks)
__host__ __device__ constexpr int qb_pad(int Dh) { return Dh + 8; }

// nq query rows (head slice of Dh values, row stride ld elements) into shared memory with 16-byte
// loads, up to four per thread in flight: fp32 sm.qs[nq][Dh] (fp32 data), or for bf16 data the
// bf16 rows themselves in sm.qs viewed as bf16[QT][qb_pad(Dh)], rows nq..QT-1 zero
template <typename TD>
__device__ __forceinline__ void stage_q(const AttnSmem<TD>& sm, const TD* src, size_t ld, int nq, int Dh) {
  constexpr int EPC = 16 / sizeof(TD);
  const int cpr = Dh / EPC, n = nq * cpr;
  if constexpr (sizeof(TD) == 2) {
    TD* qb = reinterpret_cast<TD*>(sm.qs);
    const int qp = qb_pad(Dh);
    for (int i = threadIdx.x; i < QT * cpr; i += ATTN_THREADS) {
      const int t = i / cpr, c = i - t * cpr;
      *reinterpret_cast<uint4*>(qb + t * qp + c * EPC) =
          t < nq ? *reinterpret_cast<const uint4*>(src + t * ld + c * EPC) : make_uint4(0u, 0u, 0u, 0u);
    }
    return;
  }
  for (int i0 = threadIdx.x; i0 < n; i0 += 4 * ATTN_THREADS) {
    uint4 raw[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int i = i0 + k * ATTN_THREADS;
      if (i < n) {
        const int t = i / cpr, c = i - t * cpr;
        raw[k] = *reinterpret_cast<const uint4*>(src + t * ld + c * EPC);
      }
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int i = i0 + k * ATTN_THREADS;
      if (i < n) {
        const int t = i / cpr, c = i - t * cpr;
        float* dst = sm.qs + t * Dh + c * EPC;
        if constexpr (sizeof(TD) == 2) {
          const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&raw[k]);
          const float2 f0 = __bfloat1622float2(h2[0]), f1 = __bfloat1622float2(h2[1]);
          const float2 f2 = __bfloat1622float2(h2[2]), f3 = __bfloat1622float2(h2[3]);
          reinterpret_cast<float4*>(dst)[0] = make_float4(f0.x, f0.y, f1.x, f1.y);
          reinterpret_cast<float4*>(dst)[1] = make_float4(f2.x, f2.y, f3.x, f3.y);
        } else {
          *reinterpret_cast<uint4*>(dst) = raw[k];
        }
      }
    }
  }
}

// scores of one key block: thread = one key x QK_Q queries; keys past a query's position -> -inf
// bf16 x bf16 -> fp32 tensor-core MMA, m16n8k16, A row-major, B column-major
__device__ __forceinline__ void mma_bf16_16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

template <typename TD>
__device__ __forceinline__ void block_scores(const AttnSmem<TD>& sm, int Dh, int nk, int nq, int k0, int P0,
                                             float scale) {
  if constexpr (sizeof(TD) == 2) {
    // S[16 queries][64 keys] = Q K^T on the tensor cores (bf16 inputs are exact, fp32
    // accumulation; a query row's result does not depend on the other rows).  Warp w: keys
    // 16w .. 16w+15 as two 8-key tiles, Dh / 16 steps of K.
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, gid = lane >> 2, tig = lane & 3;
    const TD* qb = reinterpret_cast<const TD*>(sm.qs);
    const int qp = qb_pad(Dh);
    float c[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) c[nt][e] = 0.f;
    for (int kc = tig * 2; kc < Dh; kc += 16) {
      const uint32_t a0 = *reinterpret_cast<const uint32_t*>(qb + gid * qp + kc);
      const uint32_t a1 = *reinterpret_cast<const uint32_t*>(qb + (gid + 8) * qp + kc);
      const uint32_t a2 = *reinterpret_cast<const uint32_t*>(qb + gid * qp + kc + 8);
      const uint32_t a3 = *reinterpret_cast<const uint32_t*>(qb + (gid + 8) * qp + kc + 8);
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        const TD* kr = sm.Ks + (warp * 16 + nt * 8 + gid) * sm.kpad;
        mma_bf16_16816(c[nt], a0, a1, a2, a3, *reinterpret_cast<const uint32_t*>(kr + kc),
                       *reinterpret_cast<const uint32_t*>(kr + kc + 8));
      }
    }
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int t = gid + (e >> 1) * 8, key = warp * 16 + nt * 8 + tig * 2 + (e & 1);
        if (t < nq) {
          const bool vis = key < nk && k0 + key <= P0 + t;  // P0: position of query 0 of the pass
          sm.S[t * ATTN_BLOCK + key] = vis ? c[nt][e] * scale : -CUDART_INF_F;
        }
      }
    return;
  }
  constexpr int EPC = 16 / sizeof(TD);
  const int key = threadIdx.x % ATTN_BLOCK, qh = threadIdx.x / ATTN_BLOCK;
  float acc[QK_Q];
#pragma unroll
  for (int u = 0; u < QK_Q; ++u) acc[u] = 0.f;
  const int u0 = qh * QK_Q;
  if (key < nk && u0 < nq) {
    const TD* kr = sm.Ks + key * sm.kpad;
    for (int c0 = 0; c0 < Dh; c0 += EPC) {
      float kf[EPC];
      if constexpr (sizeof(TD) == 2) {
        const uint4 raw = *reinterpret_cast<const uint4*>(kr + c0);
        const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f2 = __bfloat1622float2(h2[e]);
          kf[2 * e] = f2.x;
          kf[2 * e + 1] = f2.y;
        }
      } else {
        const float4 raw = *reinterpret_cast<const float4*>(kr + c0);
        kf[0] = raw.x;
        kf[1] = raw.y;
        kf[2] = raw.z;
        kf[3] = raw.w;
      }
#pragma unroll
      for (int u = 0; u < QK_Q; ++u) {
        if (u0 + u < nq) {
          const float* qr = sm.qs + (u0 + u) * Dh + c0;
#pragma unroll
          for (int e = 0; e < EPC; e += 4) {
            const float4 q4 = *reinterpret_cast<const float4*>(qr + e);
            acc[u] = fmaf(q4.x, kf[e], acc[u]);
            acc[u] = fmaf(q4.y, kf[e + 1], acc[u]);
            acc[u] = fmaf(q4.z, kf[e + 2], acc[u]);
            acc[u] = fmaf(q4.w, kf[e + 3], acc[u]);
          }
        }
      }
    }
  }
#pragma unroll
  for (int u = 0; u < QK_Q; ++u) {
    const int t = u0 + u;
    if (t < nq) {
      const bool vis = key < nk && k0 + key <= P0 + t;  // P0: position of query 0 of the pass
      sm.S[t * ATTN_BLOCK + key] = vis ? acc[u] * scale : -CUDART_INF_F;
    }
  }
}

// per query: block max, p = exp(s - max) in place, block sum -> stt.  Eight lanes per query (keys
// 8k8 .. 8k8+7 on lane k8, summed in key order, then across the eight lanes by butterfly), four
// queries per warp: the 16 query rows of a pass in one round.
template <typename TD>
__device__ __forceinline__ void block_softmax(const AttnSmem<TD>& sm, int nq) {
  static_assert(ATTN_BLOCK == 64 && QT == 16 && ATTN_THREADS == 128, "layout of the softmax pass");
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, k8 = lane & 7;
  const int t = warp * 4 + (lane >> 3);
  const bool live = t < nq;
  float* Sr = sm.S + t * ATTN_BLOCK + 8 * k8;
  float v[8];
  if (live) {
    const float4 x0 = reinterpret_cast<const float4*>(Sr)[0], x1 = reinterpret_cast<const float4*>(Sr)[1];
    v[0] = x0.x; v[1] = x0.y; v[2] = x0.z; v[3] = x0.w;
    v[4] = x1.x; v[5] = x1.y; v[6] = x1.z; v[7] = x1.w;
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = -CUDART_INF_F;
  }
  float mx = v[0];
#pragma unroll
  for (int i = 1; i < 8; ++i) mx = fmaxf(mx, v[i]);
#pragma unroll
  for (int o = 4; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float l = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    v[i] = (mx == -CUDART_INF_F || v[i] == -CUDART_INF_F) ? 0.f : expf(v[i] - mx);
    l += v[i];
  }
#pragma unroll
  for (int o = 4; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
  if (live) {
    reinterpret_cast<float4*>(Sr)[0] = make_float4(v[0], v[1], v[2], v[3]);
    reinterpret_cast<float4*>(Sr)[1] = make_float4(v[4], v[5], v[6], v[7]);
    if (k8 == 0) {
      sm.stt[2 * t] = mx;
      sm.stt[2 * t + 1] = l;
    }
  }
}

// two 8x8 bf16 matrices from shared memory, transposed (rows addressed by lanes 0-15)
__device__ __forceinline__ void ldmatrix_x2_trans(uint32_t& r0, uint32_t& r1, const void* row_addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0, %1}, [%2];"
               : "=r"(r0), "=r"(r1)
               : "r"(smem_u32(row_addr)));
}
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

// P.V of one key block: head columns 2*pi, 2*pi+1 for queries g, g+groups, ...
template <typename TD>
__device__ __forceinline__ void block_pv(const AttnSmem<TD>& sm, int Dh, int nk, int nq, float (&a0)[PV_QMAX],
                                         float (&a1)[PV_QMAX]) {
  const int npair = Dh / 2, groups = ATTN_THREADS / npair;
  const int pi = threadIdx.x % npair, g = threadIdx.x / npair;
  if constexpr (sizeof(TD) == 2) {
    // O[16][Dh] = P V on the tensor cores.  P (fp32) enters as two bf16 parts hi + lo (P = hi + lo
    // to ~16 bits), V exactly; fp32 accumulation.  Warp w: head columns [w*Dh/4, (w+1)*Dh/4) as
    // 8-column tiles, 16 keys per step (V^T fragments by transposed 8x8 matrix loads).
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, gid = lane >> 2, tig = lane & 3;
    const int ntw = Dh / 32;  // 8-column tiles per warp (<= 4)
    float c[4][4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) c[j][e] = 0.f;
#pragma unroll
    for (int ks = 0; ks < ATTN_BLOCK / 16; ++ks) {
      const float* S0 = sm.S + gid * ATTN_BLOCK + ks * 16 + 2 * tig;
      const float* S1 = S0 + 8 * ATTN_BLOCK;
      const float p[8] = {S0[0], S0[1], S1[0], S1[1], S0[8], S0[9], S1[8], S1[9]};
      uint32_t hi[4], lo[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const __nv_bfloat16 h0 = __float2bfloat16_rn(p[2 * e]), h1 = __float2bfloat16_rn(p[2 * e + 1]);
        const __nv_bfloat162 hh = __halves2bfloat162(h0, h1);
        hi[e] = *reinterpret_cast<const uint32_t*>(&hh);
        lo[e] = pack_bf16x2(p[2 * e] - __bfloat162float(h0), p[2 * e + 1] - __bfloat162float(h1));
      }
      const TD* vrow = sm.Vs + (ks * 16 + (lane >> 3 & 1) * 8 + (lane & 7)) * sm.kpad;
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (j < ntw) {
          uint32_t b0, b1;
          ldmatrix_x2_trans(b0, b1, vrow + (warp * ntw + j) * 8);
          mma_bf16_16816(c[j], hi[0], hi[1], hi[2], hi[3], b0, b1);
          mma_bf16_16816(c[j], lo[0], lo[1], lo[2], lo[3], b0, b1);
        }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (j < ntw) {
        const int col = (warp * ntw + j) * 8 + 2 * tig;
        sm.O[gid * Dh + col] = c[j][0];
        sm.O[gid * Dh + col + 1] = c[j][1];
        sm.O[(gid + 8) * Dh + col] = c[j][2];
        sm.O[(gid + 8) * Dh + col + 1] = c[j][3];
      }
    __syncthreads();
#pragma unroll
    for (int q = 0; q < PV_QMAX; ++q) {
      const int t = g + q * groups;
      a0[q] = t < QT ? sm.O[t * Dh + 2 * pi] : 0.f;
      a1[q] = t < QT ? sm.O[t * Dh + 2 * pi + 1] : 0.f;
    }
    __syncthreads();  // O is rewritten by the next block
    return;
  }
#pragma unroll
  for (int q = 0; q < PV_QMAX; ++q) a0[q] = a1[q] = 0.f;
  for (int i0 = 0; i0 < nk; i0 += 4) {  // keys in order, four per float4 of P
    float4 p4[PV_QMAX];
#pragma unroll
    for (int q = 0; q < PV_QMAX; ++q) {
      const int t = g + q * groups;
      p4[q] = t < nq ? *reinterpret_cast<const float4*>(sm.S + t * ATTN_BLOCK + i0) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int i = i0 + k;
      if (i < nk) {
        float v0, v1;
        if constexpr (sizeof(TD) == 2) {
          const float2 f2 = __bfloat1622float2(reinterpret_cast<const __nv_bfloat162*>(sm.Vs + i * sm.kpad)[pi]);
          v0 = f2.x;
          v1 = f2.y;
        } else {
          const float2 f2 = reinterpret_cast<const float2*>(sm.Vs + i * sm.kpad)[pi];
          v0 = f2.x;
          v1 = f2.y;
        }
#pragma unroll
        for (int q = 0; q < PV_QMAX; ++q) {
          const int t = g + q * groups;
          if (t < nq) {
            const float pv = k == 0 ? p4[q].x : (k == 1 ? p4[q].y : (k == 2 ? p4[q].z : p4[q].w));
            a0[q] = fmaf(pv, v0, a0[q]);
            a1[q] = fmaf(pv, v1, a1[q]);
          }
        }
      }
    }
  }
}

// fold of block j's (max mj, sum lj) into the running (m, l): the scales of the old accumulator
// (a) and of the block (bj); acc' = acc * a + acc_j * bj.  Blocks with mj = -inf are skipped.
__device__ __forceinline__ void fold_stats(float& m, float& l, float mj, float lj, float& a, float& bj) {
  const float mn = fmaxf(m, mj);
  a = m == -CUDART_INF_F ? 0.f : expf(m - mn);
  bj = expf(mj - mn);
  l = fmaf(l, a, __fmul_rn(lj, bj));
  m = mn;
}
__device__ __forceinline__ float fold_acc(float acc, float a, float accj, float bj) {
  return fmaf(acc, a, __fmul_rn(accj, bj));
}

// Split-KV (chunks of at most QT queries, i.e. one pass): grid (block groups, H, B), ATTN_THREADS
// threads.  A CTA walks bpc consecutive ATTN_BLOCK-key blocks of one head; for each it computes the
// scores, softmax and P.V and writes, for each query whose position reaches the block, the block's
// partial (acc, max, sum).  The next block's K is in flight while this block's softmax and P.V
// run, its V while this block's partials are written.  Keys past a query's position score -inf
// and contribute exact zeros, so a query's partial does not depend on how many queries share the
// call, nor on bpc.
template <typename TD>
__global__ void __launch_bounds__(ATTN_THREADS) attn_block_kernel(const TD* __restrict__ qrot,
                                                                 const TD* __restrict__ kv,
                                                                 const int32_t* __restrict__ len, int T, int d,
                                                                 int H, int Dh, int Lmax, int nblk_cap, int tcap,
                                                                 int bpc, float scale, float* __restrict__ part) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ __align__(16) unsigned char attn_sm[];
  const int h = blockIdx.y, b = blockIdx.z;
  const int L0 = len[b];
  const int Lend = L0 + T;
  const int nq = T;  // T <= QT
  const int j_begin = blockIdx.x * bpc;
  const int j_end = min(j_begin + bpc, (Lend + ATTN_BLOCK - 1) / ATTN_BLOCK);
  if (j_begin >= j_end) return;
  AttnSmem<TD> sm(attn_sm, Dh);
  const size_t HD = static_cast<size_t>(H) * Dh;
  const TD* kvb = kv + static_cast<size_t>(b) * Lmax * 2 * HD + static_cast<size_t>(h) * Dh;
  auto nk_of = [&](int j) { return min(ATTN_BLOCK, Lend - j * ATTN_BLOCK); };
  stage_k(sm, kvb + static_cast<size_t>(j_begin) * ATTN_BLOCK * 2 * HD, HD, Dh, nk_of(j_begin));
  stage_v(sm, kvb + static_cast<size_t>(j_begin) * ATTN_BLOCK * 2 * HD, HD, Dh, nk_of(j_begin));
  stage_q(sm, qrot + static_cast<size_t>(b * T) * d + h * Dh, d, nq, Dh);
  const int npair = Dh / 2, groups = ATTN_THREADS / npair;
  const int pi = threadIdx.x % npair, g = threadIdx.x / npair;
  for (int j = j_begin; j < j_end; ++j) {
    const int k0 = j * ATTN_BLOCK, nk = nk_of(j);
    const bool more = j + 1 < j_end;
    cp_async_wait<1>();  // K of block j (its V may still be in flight)
    __syncthreads();
    block_scores(sm, Dh, nk, nq, k0, L0, scale);
    __syncthreads();  // K of block j no longer read
    if (more) stage_k(sm, kvb + static_cast<size_t>(j + 1) * ATTN_BLOCK * 2 * HD, HD, Dh, nk_of(j + 1));
    block_softmax(sm, nq);
    if (more)
      cp_async_wait<1>();  // V of block j (the next K may still be in flight)
    else
      cp_async_wait<0>();
    __syncthreads();
    float a0[PV_QMAX], a1[PV_QMAX];
    block_pv(sm, Dh, nk, nq, a0, a1);
    __syncthreads();  // V of block j no longer read
    if (more) stage_v(sm, kvb + static_cast<size_t>(j + 1) * ATTN_BLOCK * 2 * HD, HD, Dh, nk_of(j + 1));
#pragma unroll
    for (int q = 0; q < PV_QMAX; ++q) {
      const int t = g + q * groups;
      if (t < nq && L0 + t >= k0) {
        float* pd = part + ((((static_cast<size_t>(b) * H + h) * nblk_cap + j) * tcap + t) * (Dh + 2));
        pd[2 * pi] = a0[q];
        pd[2 * pi + 1] = a1[q];
        if (pi == 0) {
          pd[Dh] = sm.stt[2 * t];
          pd[Dh + 1] = sm.stt[2 * t + 1];
        }
      }
    }
  }
  cp_async_wait<0>();  // no copy may outlive the CTA
}

template <typename TD>
__global__ void attn_combine_kernel(const float* __restrict__ part, const int32_t* __restrict__ len, int T, int d,
                                    int H, int Dh, int nblk_cap, int tcap, TD* __restrict__ out, int ld_out) {
  pdl_trigger();
  pdl_wait();
  const int row = blockIdx.x, h = blockIdx.y, dd = threadIdx.x;
  if (dd >= Dh) return;
  const int b = row / T, t = row % T;
  const int P = len[b] + t;
  const int jmax = P / ATTN_BLOCK;
  float m = -CUDART_INF_F, l = 0.f, acc = 0.f;
  const float* pb = part + ((static_cast<size_t>(b) * H + h) * nblk_cap * tcap + t) * (Dh + 2);
  const size_t jstride = static_cast<size_t>(tcap) * (Dh + 2);
  for (int j0 = 0; j0 <= jmax; j0 += 4) {  // four blocks' loads in flight, folded in block order
    float mj[4], lj[4], aj[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      if (j0 + k <= jmax) {
        const float* pj = pb + (j0 + k) * jstride;
        mj[k] = pj[Dh];
        lj[k] = pj[Dh + 1];
        aj[k] = pj[dd];
      }
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      if (j0 + k > jmax || mj[k] == -CUDART_INF_F) continue;
      float a, bj;
      fold_stats(m, l, mj[k], lj[k], a, bj);
      acc = fold_acc(acc, a, aj[k], bj);
    }
  }
  out[static_cast<size_t>(row) * ld_out + h * Dh + dd] = from_f32<TD>(acc / l);
}

// Fused (chunks of more than tcap queries, i.e. prefill): grid (query tiles of QT, H, B).  A CTA
// walks the key blocks 0 .. (last query's position) / ATTN_BLOCK in order and computes each
// block's partial with the split-KV kernel's arithmetic (block_scores / block_softmax / block_pv),
// then folds it as the combine kernel does (fold_stats / fold_acc), so every query's output equals
// the split-KV + combine result bit for bit, with no partial buffer and any chunk length.
template <typename TD>
__global__ void __launch_bounds__(ATTN_THREADS) attn_fused_kernel(const TD* __restrict__ qrot,
                                                                 const TD* __restrict__ kv,
                                                                 const int32_t* __restrict__ len, int T, int d,
                                                                 int H, int Dh, int Lmax, float scale,
                                                                 TD* __restrict__ out, int ld_out) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ __align__(16) unsigned char attn_sm[];
  const int tq0 = blockIdx.x * QT, h = blockIdx.y, b = blockIdx.z;
  const int nq = min(QT, T - tq0);
  const int L0 = len[b];
  const int Lend = L0 + T;
  AttnSmem<TD> sm(attn_sm, Dh);
  const size_t HD = static_cast<size_t>(H) * Dh;
  const int npair = Dh / 2, groups = ATTN_THREADS / npair;
  const int pi = threadIdx.x % npair, g = threadIdx.x / npair;
  stage_q(sm, qrot + static_cast<size_t>(b * T + tq0) * d + h * Dh, d, nq, Dh);
  for (int t = threadIdx.x; t < QT; t += ATTN_THREADS) {
    sm.fold[4 * t] = -CUDART_INF_F;
    sm.fold[4 * t + 1] = 0.f;
  }
  float c0[PV_QMAX], c1[PV_QMAX];  // running accumulators (the combine kernel's acc)
#pragma unroll
  for (int q = 0; q < PV_QMAX; ++q) c0[q] = c1[q] = 0.f;
  const int jlast = (L0 + tq0 + nq - 1) / ATTN_BLOCK;
  for (int j = 0; j <= jlast; ++j) {
    const int k0 = j * ATTN_BLOCK;
    const int nk = min(ATTN_BLOCK, Lend - k0);
    __syncthreads();  // the previous block's K/V/S are no longer read
    stage_kv(sm, kv + (static_cast<size_t>(b) * Lmax + k0) * 2 * HD + static_cast<size_t>(h) * Dh, HD, Dh, nk);
    cp_async_wait<0>();
    __syncthreads();
    block_scores(sm, Dh, nk, nq, k0, L0 + tq0, scale);
    __syncthreads();
    block_softmax(sm, nq);
    __syncthreads();
    for (int t = threadIdx.x; t < nq; t += ATTN_THREADS) {
      const float mj = sm.stt[2 * t];
      float* f = sm.fold + 4 * t;
      if (mj == -CUDART_INF_F) {  // the block lies past this query: the combine skips it
        f[2] = 1.f;
        f[3] = 0.f;
        continue;
      }
      float m = f[0], l = f[1], a, bj;
      fold_stats(m, l, mj, sm.stt[2 * t + 1], a, bj);
      f[0] = m;
      f[1] = l;
      f[2] = a;
      f[3] = bj;
    }
    __syncthreads();
    float a0[PV_QMAX], a1[PV_QMAX];
    block_pv(sm, Dh, nk, nq, a0, a1);
#pragma unroll
    for (int q = 0; q < PV_QMAX; ++q) {
      const int t = g + q * groups;
      if (t < nq && sm.stt[2 * t] != -CUDART_INF_F) {
        const float a = sm.fold[4 * t + 2], bj = sm.fold[4 * t + 3];
        c0[q] = fold_acc(c0[q], a, a0[q], bj);
        c1[q] = fold_acc(c1[q], a, a1[q], bj);
      }
    }
  }
#pragma unroll
  for (int q = 0; q < PV_QMAX; ++q) {
    const int t = g + q * groups;
    if (t < nq) {
      const float l = sm.fold[4 * t + 1];
      TD* o = out + static_cast<size_t>(b * T + tq0 + t) * ld_out + h * Dh + 2 * pi;
      o[0] = from_f32<TD>(c0[q] / l);
      o[1] = from_f32<TD>(c1[q] / l);
    }
  }
}

template <typename TD>
int launch_attention_t(const evs_model* m, evs_state* s, int layer, int B, int T, int splits, int kv_blocks,
                       cudaStream_t st) {
  const int d = m->dl, H = m->Hl, Dh = m->cfg.head_dim;  // this rank's channels and heads
  const int M = B * T;
  TD* kv = static_cast<TD*>(s->kv[layer]);
  TD* qrot = static_cast<TD*>(s->qrot);
  const bool pdl = s->use_pdl();
  EVS_CUDA_TRY(evs_launch(rope_append_kernel<TD>, dim3(M, H), dim3(Dh / 2), 0, st, pdl,
                          static_cast<const float*>(s->ws), splits, M, T, d, H, Dh, log(m->cfg.rope_base),
                          static_cast<const int32_t*>(s->d_len), s->max_seqlen, qrot, kv, s->d_err));
  const size_t smem = attn_smem_bytes<TD>(Dh);
  EVS_CHECK_RANGE(smem <= 227 * 1024, "head_dim too large for the staged attention block");
  const float scale = 1.0f / sqrtf(static_cast<float>(Dh));
  if (T > s->attn_tcap) {
    EVS_CUDA_TRY(cudaFuncSetAttribute(attn_fused_kernel<TD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      static_cast<int>(smem)));
    EVS_CUDA_TRY(evs_launch(attn_fused_kernel<TD>, dim3((T + QT - 1) / QT, H, B), dim3(ATTN_THREADS), smem, st, pdl,
                            static_cast<const TD*>(qrot), static_cast<const TD*>(kv),
                            static_cast<const int32_t*>(s->d_len), T, d, H, Dh, s->max_seqlen, scale,
                            static_cast<TD*>(s->act), s->ld_act));
    evs_count_launch(2);
    return EVS_OK;
  }
  EVS_CUDA_TRY(cudaFuncSetAttribute(attn_block_kernel<TD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    static_cast<int>(smem)));
  // key blocks per CTA: one while the grid has fewer than ~16 CTAs per SM, more for long contexts
  // (the arithmetic of a block does not depend on it)
  EVS_CHECK_ARG(T <= QT, "split-KV attention takes at most QT queries per call");
  static int n_sm = 0;
  if (n_sm == 0) EVS_CUDA_TRY(cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, m->device));
  const long long want = 16LL * n_sm;
  const int bpc = static_cast<int>(std::max<long long>(1, (static_cast<long long>(kv_blocks) * H * B + want - 1) / want));
  EVS_CUDA_TRY(evs_launch(attn_block_kernel<TD>, dim3((kv_blocks + bpc - 1) / bpc, H, B), dim3(ATTN_THREADS), smem, st,
                          pdl, static_cast<const TD*>(qrot), static_cast<const TD*>(kv),
                          static_cast<const int32_t*>(s->d_len), T, d, H, Dh, s->max_seqlen, s->attn_blocks,
                          s->attn_tcap, bpc, scale, s->attn_part));
  EVS_CUDA_TRY(evs_launch(attn_combine_kernel<TD>, dim3(M, H), dim3(Dh), 0, st, pdl,
                          static_cast<const float*>(s->attn_part), static_cast<const int32_t*>(s->d_len), T, d, H,
                          Dh, s->attn_blocks, s->attn_tcap, static_cast<TD*>(s->act), s->ld_act));
  evs_count_launch(3);
  return EVS_OK;
}

}  // namespace

int launch_attention(const evs_model* m, evs_state* s, int layer, int B, int T, int splits, int kv_blocks,
                     cudaStream_t st) {
  // P.V gives each thread two head columns and at most PV_QMAX of the QT queries of a pass
  EVS_CHECK_ARG(m->cfg.head_dim >= 32 && m->cfg.head_dim <= 128 && 256 % m->cfg.head_dim == 0,
                "head_dim must be 32, 64 or 128");
  EVS_CHECK_RANGE(kv_blocks >= 1 && kv_blocks <= s->attn_blocks, "KV length beyond max_seqlen");
  if (m->cfg.dtype == EVS_DTYPE_BF16) return launch_attention_t<__nv_bfloat16>(m, s, layer, B, T, splits, kv_blocks, st);
  return launch_attention_t<float>(m, s, layer, B, T, splits, kv_blocks, st);
}
