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
#include <cmath>

#include "internal.hpp"

namespace {

template <typename TD>
__global__ void rope_append_kernel(const float* __restrict__ ws, int splits, int M, int T, int d, int H, int Dh,
                                   double log_base, const int32_t* __restrict__ len, int Lmax, TD* __restrict__ qrot,
                                   TD* __restrict__ kv, EvsDevErr* err) {
  pdl_trigger();
  const int row = blockIdx.x, h = blockIdx.y, j = threadIdx.x;
  const int half = Dh / 2;
  if (j >= half) return;
  const double inv_freq = exp(-(2.0 * j / Dh) * log_base);  // depends on no earlier kernel
  pdl_wait();
  const int b = row / T, t = row % T;
  // the projection's partial sums do not depend on the state length: their loads go first
  const int N = 3 * d;
  auto val = [&](int c) {
    return round_to<TD>(split_sum(ws + static_cast<size_t>(row) * N + c, static_cast<size_t>(M) * N, splits));
  };
  const int c1 = h * Dh + j, c2 = c1 + half;
  const float q1 = val(c1), q2 = val(c2);
  const float k1 = val(d + c1), k2 = val(d + c2);
  const float v1 = val(2 * d + c1), v2 = val(2 * d + c2);
  const int P = len[b] + t;
  if (P >= Lmax) {
    if (j == 0) evs_record_error(err, EVS_ERANGE, EVS_K_ATTN, row);
    return;
  }
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
constexpr int QK_Q = QT / (ATTN_THREADS / ATTN_BLOCK);  // queries per thread in the fp32 score pass
constexpr int PV_QMAX = 8;       // queries per thread in the fp32 P.V (head_dim <= 128)
constexpr int ACC_N = 16;        // P.V accumulators per thread (both paths)
// row stride of the scores (floats): 4 floats of padding keep the softmax's quarter-warp float4
// loads and the 8-row matrix loads of P on distinct banks.  For bf16 data the softmax pass
// overwrites each score row with P's bf16 parts, hi in bytes 0-127 and lo in bytes 128-255 of the
// row (PLD bf16 elements per row).
constexpr int SLD = ATTN_BLOCK + 4;
constexpr int PLD = 2 * SLD;

// query rows per block pass and the bf16 query tile's padded row (272 B for Dh = 128: the MMA
// fragment loads of 8 rows x 4 lanes hit 32 distinct banks)
__host__ __device__ constexpr int qb_pad(int Dh) { return Dh + 8; }

// shared memory of both attention kernels: K and V rows padded by 16 bytes (conflict-free
// row-per-thread reads and 8-row matrix loads); the queries (fp32 rows, or bf16 rows padded to
// qb_pad); the scores; for bf16 data the bf16 hi and lo parts of P; per-query stats (+ the running
// folds of the fused kernel)
template <typename TD>
__host__ __device__ constexpr size_t attn_q_bytes(int Dh) {
  return sizeof(TD) == 2 ? 2 * static_cast<size_t>(QT) * qb_pad(Dh) : 4 * static_cast<size_t>(QT) * Dh;
}
template <typename TD>
__host__ __device__ constexpr size_t attn_smem_bytes(int Dh) {
  return sizeof(TD) * (2 * static_cast<size_t>(ATTN_BLOCK) * (Dh + 16 / sizeof(TD))) + attn_q_bytes<TD>(Dh) +
         4 * static_cast<size_t>(QT) * SLD + sizeof(float) * 10 * QT;
}

template <typename TD>
struct AttnSmem {
  TD* Ks;
  TD* Vs;
  float* qs;            // fp32 queries [QT][Dh], or bf16 query rows [QT][qb_pad(Dh)]
  float* S;             // [QT][SLD]: scores; after the softmax pass p = 2^(s - max) (fp32 path)
  __nv_bfloat16* Ph;    // [QT][PLD] over S: bf16 parts of p, p = hi + lo to ~16 bits (bf16 path)
  __nv_bfloat16* Pl;    // Ph + 64
  float* stt;    // [2 QT]: block max, block sum
  float* fold;   // [4 QT]: running max, running sum, scale of the old accumulator, scale of the block
  float* gfold;  // [4 QT]: the same for the current fold group (fused kernel)
  int kpad;      // row stride of K and V (elements)
  __device__ AttnSmem(unsigned char* raw, int Dh) {
    constexpr int EPC = 16 / sizeof(TD);
    kpad = Dh + EPC;
    Ks = reinterpret_cast<TD*>(raw);
    Vs = Ks + ATTN_BLOCK * kpad;
    unsigned char* q = reinterpret_cast<unsigned char*>(Vs + ATTN_BLOCK * kpad);
    qs = reinterpret_cast<float*>(q);
    q += attn_q_bytes<TD>(Dh);
    S = reinterpret_cast<float*>(q);
    q += 4 * QT * SLD;
    Ph = reinterpret_cast<__nv_bfloat16*>(S);
    Pl = Ph + ATTN_BLOCK;
    stt = reinterpret_cast<float*>(q);
    fold = stt + 2 * QT;
    gfold = fold + 4 * QT;
  }
};

// The P.V accumulators of a thread: ACC_N values, pairs (i, i + 1) of one query row and two
// adjacent head columns.  bf16 path: the m16n8k16 fragments, i = 4 j + e -> row gid + 8 (e / 2),
// column (warp ntw + j) 8 + 2 tig + e % 2 (ntw = Dh / 32 tiles per warp).  fp32 path: i = 2 q + e
// -> row g + q groups, column 2 pi + e.
template <typename TD>
__device__ __forceinline__ int acc_row(int i, int Dh) {
  if constexpr (sizeof(TD) == 2) {
    return ((threadIdx.x & 31) >> 2) + 8 * ((i & 3) >> 1);
  } else {
    const int npair = Dh / 2, groups = ATTN_THREADS / npair;
    return static_cast<int>(threadIdx.x) / npair + (i >> 1) * groups;
  }
}
template <typename TD>
__device__ __forceinline__ int acc_col(int i, int Dh) {
  if constexpr (sizeof(TD) == 2) {
    const int warp = threadIdx.x >> 5, tig = threadIdx.x & 3, ntw = Dh / 32;
    return (warp * ntw + (i >> 2)) * 8 + 2 * tig + (i & 1);
  } else {
    return 2 * (static_cast<int>(threadIdx.x) % (Dh / 2)) + (i & 1);
  }
}
template <typename TD>
__device__ __forceinline__ bool acc_live(int i, int Dh) {
  if constexpr (sizeof(TD) == 2) return (i >> 2) < Dh / 32;
  return acc_row<TD>(i, Dh) < QT;
}

// 16-byte asynchronous copies of the K rows [0, nk) of one key block (one commit group)
// (a thread copies chunk c of rows r0, r0 + rs, ...: 16-byte chunks per row divide ATTN_THREADS)
template <typename TD>
__device__ __forceinline__ void stage_k(const AttnSmem<TD>& sm, const TD* kb, size_t HD, int Dh, int nk) {
  constexpr int EPC = 16 / sizeof(TD);
  const int cpr = Dh / EPC, rs = ATTN_THREADS / cpr;
  const int r0 = threadIdx.x / cpr, c = threadIdx.x - r0 * cpr;
  for (int r = r0; r < nk; r += rs)
    cp_async16(sm.Ks + r * sm.kpad + c * EPC, kb + static_cast<size_t>(r) * 2 * HD + c * EPC);
  cp_async_commit();
}
// ... and of its V rows (one commit group); V rows past the block's keys are zero: P is zero
// there, and 0 times stale data could be NaN
template <typename TD>
__device__ __forceinline__ void stage_v(const AttnSmem<TD>& sm, const TD* kb, size_t HD, int Dh, int nk) {
  constexpr int EPC = 16 / sizeof(TD);
  const int cpr = Dh / EPC, rs = ATTN_THREADS / cpr;
  const int r0 = threadIdx.x / cpr, c = threadIdx.x - r0 * cpr;
  int r = r0;
  for (; r < nk; r += rs) cp_async16(sm.Vs + r * sm.kpad + c * EPC, kb + static_cast<size_t>(r) * 2 * HD + HD + c * EPC);
  cp_async_commit();
  for (; r < ATTN_BLOCK; r += rs) *reinterpret_cast<uint4*>(sm.Vs + r * sm.kpad + c * EPC) = make_uint4(0u, 0u, 0u, 0u);
}
template <typename TD>
__device__ __forceinline__ void stage_kv(const AttnSmem<TD>& sm, const TD* kb, size_t HD, int Dh, int nk) {
  stage_k(sm, kb, HD, Dh, nk);
  stage_v(sm, kb, HD, Dh, nk);
}

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

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
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
      for (int hh = 0; hh < 2; ++hh) {
        const int t = gid + hh * 8, key = warp * 16 + nt * 8 + tig * 2;
        if (t < nq) {  // P0: position of query 0 of the pass
          const bool v0 = key < nk && k0 + key <= P0 + t, v1 = key + 1 < nk && k0 + key + 1 <= P0 + t;
          *reinterpret_cast<float2*>(sm.S + t * SLD + key) =
              make_float2(v0 ? c[nt][2 * hh] * scale : -CUDART_INF_F, v1 ? c[nt][2 * hh + 1] * scale : -CUDART_INF_F);
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
      sm.S[t * SLD + key] = vis ? acc[u] * scale : -CUDART_INF_F;
    }
  }
}

// per query: block max, p = 2^(s - max), block sum -> stt.  Eight lanes per query: lane k8
// takes keys 4 k8 .. 4 k8 + 3 and 32 + 4 k8 .. 32 + 4 k8 + 3 (two float4, a quarter-warp on distinct
// banks) and sums its eight p in that order, then the eight lanes are summed by butterfly; four
// queries per warp, the 16 query rows of a pass in one round.  p goes back in place (fp32 path)
// or as its bf16 parts hi = bf16(p), lo = bf16(p - hi) (bf16 path, the P.V operand).  Rows past
// nq get p = 0.
template <typename TD>
__device__ __forceinline__ void block_softmax(const AttnSmem<TD>& sm, int nq) {
  static_assert(ATTN_BLOCK == 64 && QT == 16 && ATTN_THREADS == 128, "layout of the softmax pass");
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, k8 = lane & 7;
  const int t = warp * 4 + (lane >> 3);
  const bool live = t < nq;
  float* Sr = sm.S + t * SLD + 4 * k8;
  float v[8];
  if (live) {
    const float4 x0 = *reinterpret_cast<const float4*>(Sr), x1 = *reinterpret_cast<const float4*>(Sr + 32);
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
    v[i] = (mx == -CUDART_INF_F || v[i] == -CUDART_INF_F) ? 0.f : exp2f(v[i] - mx);
    l += v[i];
  }
#pragma unroll
  for (int o = 4; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
  if constexpr (sizeof(TD) == 2) {
#pragma unroll
    for (int hq = 0; hq < 2; ++hq) {
      uint32_t hi[2], lo[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const float p0 = v[4 * hq + 2 * e], p1 = v[4 * hq + 2 * e + 1];
        const __nv_bfloat16 h0 = __float2bfloat16_rn(p0), h1 = __float2bfloat16_rn(p1);
        const __nv_bfloat162 hh = __halves2bfloat162(h0, h1);
        hi[e] = *reinterpret_cast<const uint32_t*>(&hh);
        lo[e] = pack_bf16x2(p0 - __bfloat162float(h0), p1 - __bfloat162float(h1));
      }
      // (row t of P overlays row t of S, read by this warp only, before the shuffles above)
      const int off = t * PLD + 4 * k8 + 32 * hq;
      *reinterpret_cast<uint2*>(sm.Ph + off) = make_uint2(hi[0], hi[1]);
      *reinterpret_cast<uint2*>(sm.Pl + off) = make_uint2(lo[0], lo[1]);
    }
  } else if (live) {
    *reinterpret_cast<float4*>(Sr) = make_float4(v[0], v[1], v[2], v[3]);
    *reinterpret_cast<float4*>(Sr + 32) = make_float4(v[4], v[5], v[6], v[7]);
  }
  if (live && k8 == 0) {
    sm.stt[2 * t] = mx;
    sm.stt[2 * t + 1] = l;
  }
}

// two 8x8 bf16 matrices from shared memory, transposed (rows addressed by lanes 0-15)
__device__ __forceinline__ void ldmatrix_x2_trans(uint32_t& r0, uint32_t& r1, const void* row_addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0, %1}, [%2];"
               : "=r"(r0), "=r"(r1)
               : "r"(smem_u32(row_addr)));
}

// four 8x8 bf16 matrices from shared memory (rows addressed by lanes 0-31): the A fragment of
// one m16n8k16 step
__device__ __forceinline__ void ldmatrix_x4(uint32_t (&r)[4], const void* row_addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(row_addr)));
}

// P.V of one key block into the thread's ACC_N accumulators (layout: acc_row / acc_col)
template <typename TD>
__device__ __forceinline__ void block_pv(const AttnSmem<TD>& sm, int Dh, int nk, int nq, float (&acc)[ACC_N]) {
  if constexpr (sizeof(TD) == 2) {
    // O[16][Dh] = P V on the tensor cores.  P enters as its bf16 parts hi + lo (written by the
    // softmax pass), V exactly; fp32 accumulation.  Warp w: head columns [w Dh/4, (w+1) Dh/4) as
    // 8-column tiles, 16 keys per step (P by 8x8 matrix loads, V^T by transposed ones).
    (void)nk;
    (void)nq;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ntw = Dh / 32;  // 8-column tiles per warp (<= 4)
    float c[4][4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) c[j][e] = 0.f;
    const int prow = (lane & 7) + ((lane >> 3) & 1) * 8, pcol = (lane >> 4) * 8;
#pragma unroll
    for (int ks = 0; ks < ATTN_BLOCK / 16; ++ks) {
      uint32_t hi[4], lo[4];
      ldmatrix_x4(hi, sm.Ph + prow * PLD + ks * 16 + pcol);
      ldmatrix_x4(lo, sm.Pl + prow * PLD + ks * 16 + pcol);
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
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[4 * j + e] = c[j][e];
    return;
  }
  const int npair = Dh / 2, groups = ATTN_THREADS / npair;
  const int pi = threadIdx.x % npair, g = threadIdx.x / npair;
  float a0[PV_QMAX], a1[PV_QMAX];
#pragma unroll
  for (int q = 0; q < PV_QMAX; ++q) a0[q] = a1[q] = 0.f;
  for (int i0 = 0; i0 < nk; i0 += 4) {  // keys in order, four per float4 of P
    float4 p4[PV_QMAX];
#pragma unroll
    for (int q = 0; q < PV_QMAX; ++q) {
      const int t = g + q * groups;
      p4[q] = t < nq ? *reinterpret_cast<const float4*>(sm.S + t * SLD + i0) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int i = i0 + k;
      if (i < nk) {
        const float2 f2 = reinterpret_cast<const float2*>(sm.Vs + i * sm.kpad)[pi];
#pragma unroll
        for (int q = 0; q < PV_QMAX; ++q) {
          const int t = g + q * groups;
          if (t < nq) {
            const float pv = k == 0 ? p4[q].x : (k == 1 ? p4[q].y : (k == 2 ? p4[q].z : p4[q].w));
            a0[q] = fmaf(pv, f2.x, a0[q]);
            a1[q] = fmaf(pv, f2.y, a1[q]);
          }
        }
      }
    }
  }
#pragma unroll
  for (int q = 0; q < PV_QMAX; ++q) {
    acc[2 * q] = a0[q];
    acc[2 * q + 1] = a1[q];
  }
}

// fold of block j's (max mj, sum lj) into the running (m, l): the scales of the old accumulator
// (a) and of the block (bj); acc' = acc * a + acc_j * bj.  Blocks with mj = -inf are skipped.
__device__ __forceinline__ void fold_stats(float& m, float& l, float mj, float lj, float& a, float& bj) {
  const float mn = fmaxf(m, mj);
  a = m == -CUDART_INF_F ? 0.f : exp2f(m - mn);
  bj = exp2f(mj - mn);
  l = fmaf(l, a, __fmul_rn(lj, bj));
  m = mn;
}
__device__ __forceinline__ float fold_acc(float acc, float a, float accj, float bj) {
  return fmaf(acc, a, __fmul_rn(accj, bj));
}

// The fold order of a query's key blocks (the same in the split-KV combine and the fused kernel):
// the blocks of each group of ATTN_GROUP consecutive blocks (aligned at absolute block indices) in
// block order, from an empty accumulator; then the groups in group order.  Folding one group's
// result into the empty accumulator is exact, so contexts of one group fold block by block.
constexpr int ATTN_GROUP = 16;
// per-block partials of contexts up to this many blocks are folded on both levels by the combine
// kernel alone (a sequential fold per query, as short as the group fold kernel's launch)
constexpr int ATTN_COMBINE_BLOCKS = 64;

// Split-KV (chunks of at most QT queries, i.e. one pass): grid (block ranges, H, B), ATTN_THREADS
// threads.  A CTA walks bpc consecutive ATTN_BLOCK-key blocks of one head; for each it computes the
// scores, softmax and P.V.  The next block's K is in flight while this block's softmax and P.V
// run, its V while this block's results are stored.  Keys past a query's position score -inf and
// contribute exact zeros, so a query's result does not depend on how many queries share the call,
// nor on bpc.  Stored per query whose position reaches the block:
//   group_fold = 0: every block's partial (acc, max, sum) in its slot;
//   group_fold = 1 (bpc a multiple of ATTN_GROUP, so the range covers whole groups): the blocks of
//     each group folded in block order from an empty accumulator, the group's (acc, max, sum) in
//     the slot of its first block, which is what attn_group_fold_kernel makes of the partials.
template <typename TD>
__global__ void __launch_bounds__(ATTN_THREADS, 5) attn_block_kernel(const TD* __restrict__ qrot,
                                                                 const TD* __restrict__ kv,
                                                                 const int32_t* __restrict__ len, int T, int d,
                                                                 int H, int Dh, int Lmax, int nblk_cap, int tcap,
                                                                 int bpc, int group_fold, float scale,
                                                                 float* __restrict__ part) {
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
  float gc[ACC_N];  // group_fold: the running accumulator of the current group
#pragma unroll
  for (int i = 0; i < ACC_N; ++i) gc[i] = 0.f;
  for (int t = threadIdx.x; t < QT; t += ATTN_THREADS) {
    sm.gfold[4 * t] = -CUDART_INF_F;
    sm.gfold[4 * t + 1] = 0.f;
  }
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
    if (group_fold) {  // the block's stats folded into the group's (as the fused kernel does)
      for (int t = threadIdx.x; t < nq; t += ATTN_THREADS) {
        const float mj = sm.stt[2 * t];
        float* f = sm.gfold + 4 * t;
        if (mj == -CUDART_INF_F) {
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
    }
    float acc[ACC_N];
    block_pv(sm, Dh, nk, nq, acc);
    __syncthreads();  // V of block j no longer read; the group stats updated
    if (more) stage_v(sm, kvb + static_cast<size_t>(j + 1) * ATTN_BLOCK * 2 * HD, HD, Dh, nk_of(j + 1));
    if (!group_fold) {
#pragma unroll
      for (int i = 0; i < ACC_N; i += 2) {
        const int t = acc_row<TD>(i, Dh), col = acc_col<TD>(i, Dh);
        if (acc_live<TD>(i, Dh) && t < nq && L0 + t >= k0) {
          float* pd = part + ((((static_cast<size_t>(b) * H + h) * nblk_cap + j) * tcap + t) * (Dh + 2));
          *reinterpret_cast<float2*>(pd + col) = make_float2(acc[i], acc[i + 1]);
          if (col == 0) {
            pd[Dh] = sm.stt[2 * t];
            pd[Dh + 1] = sm.stt[2 * t + 1];
          }
        }
      }
      continue;
    }
#pragma unroll
    for (int i = 0; i < ACC_N; i += 2) {
      const int t = acc_row<TD>(i, Dh);
      if (acc_live<TD>(i, Dh) && t < nq && sm.stt[2 * t] != -CUDART_INF_F) {
        const float a = sm.gfold[4 * t + 2], bj = sm.gfold[4 * t + 3];
        gc[i] = fold_acc(gc[i], a, acc[i], bj);
        gc[i + 1] = fold_acc(gc[i + 1], a, acc[i + 1], bj);
      }
    }
    if (j % ATTN_GROUP == ATTN_GROUP - 1 || j + 1 == j_end) {
      // the group's result into the slot of its first block (queries the group reaches), then the
      // group emptied
      const int jg = j - j % ATTN_GROUP;
#pragma unroll
      for (int i = 0; i < ACC_N; i += 2) {
        const int t = acc_row<TD>(i, Dh), col = acc_col<TD>(i, Dh);
        if (acc_live<TD>(i, Dh) && t < nq && L0 + t >= jg * ATTN_BLOCK) {
          float* pd = part + ((((static_cast<size_t>(b) * H + h) * nblk_cap + jg) * tcap + t) * (Dh + 2));
          *reinterpret_cast<float2*>(pd + col) = make_float2(gc[i], gc[i + 1]);
          if (col == 0) {
            pd[Dh] = sm.gfold[4 * t];
            pd[Dh + 1] = sm.gfold[4 * t + 1];
          }
        }
        gc[i] = gc[i + 1] = 0.f;
      }
      __syncthreads();  // the group stats are read
      for (int t = threadIdx.x; t < QT; t += ATTN_THREADS) {
        sm.gfold[4 * t] = -CUDART_INF_F;
        sm.gfold[4 * t + 1] = 0.f;
      }
    }
  }
  cp_async_wait<0>();  // no copy may outlive the CTA
}

// partials of blocks jb, jb + jstep, jb + 2 jstep, ... <= jend folded in that order (eight loads
// in flight); blocks with max -inf (past the query) are skipped
__device__ __forceinline__ void fold_blocks(const float* pb, size_t jstride, int Dh, int dd, int jb, int jend,
                                            int jstep, float& m, float& l, float& acc) {
  constexpr int FB = 16;  // block partials loaded per batch (folded in block order)
  for (int j0 = jb; j0 <= jend; j0 += FB * jstep) {
    float mj[FB], lj[FB], aj[FB];
#pragma unroll
    for (int k = 0; k < FB; ++k) {
      const int j = j0 + k * jstep;
      if (j <= jend) {
        const float* pj = pb + j * jstride;
        mj[k] = pj[Dh];
        lj[k] = pj[Dh + 1];
        aj[k] = pj[dd];
      }
    }
#pragma unroll
    for (int k = 0; k < FB; ++k) {
      if (j0 + k * jstep > jend || mj[k] == -CUDART_INF_F) continue;
      float a, bj;
      fold_stats(m, l, mj[k], lj[k], a, bj);
      acc = fold_acc(acc, a, aj[k], bj);
    }
  }
}

// Contexts of more than one group: group g's blocks folded in block order, in place, into the
// partial slot of its first block.  grid (M, H, groups), Dh threads.
__global__ void attn_group_fold_kernel(float* __restrict__ part, const int32_t* __restrict__ len, int T, int H,
                                       int Dh, int nblk_cap, int tcap) {
  pdl_trigger();
  pdl_wait();
  const int row = blockIdx.x, h = blockIdx.y, grp = blockIdx.z, dd = threadIdx.x;
  const int b = row / T, t = row % T;
  const int jmax = (len[b] + t) / ATTN_BLOCK;
  const int jb = grp * ATTN_GROUP;
  if (jb > jmax) return;  // the whole group lies past this query
  float* pb = part + ((static_cast<size_t>(b) * H + h) * nblk_cap * tcap + t) * (Dh + 2);
  const size_t jstride = static_cast<size_t>(tcap) * (Dh + 2);
  float m = -CUDART_INF_F, l = 0.f, acc = 0.f;
  if (dd < Dh) fold_blocks(pb, jstride, Dh, dd, jb, min(jmax, jb + ATTN_GROUP - 1), 1, m, l, acc);
  __syncthreads();  // every thread has read the group's statistics
  float* pg = pb + jb * jstride;
  if (dd < Dh) pg[dd] = acc;
  if (dd == 0) {
    pg[Dh] = m;
    pg[Dh + 1] = l;
  }
}

// grid (M, H), Dh threads: the query's partial slots j = 0, jstep, 2 jstep, ... <= its last block
// folded in order (jstep = 1: the blocks of a one-group context; ATTN_GROUP: the group results).
// jstep = 0: per-block partials of a context of a few groups, both levels of the fold here (each
// group's blocks from an empty accumulator, then the group into the total: attn_group_fold_kernel
// followed by jstep = ATTN_GROUP, without its launch).
template <typename TD>
__global__ void attn_combine_kernel(const float* __restrict__ part, const int32_t* __restrict__ len, int T, int d,
                                    int H, int Dh, int nblk_cap, int tcap, int jstep, TD* __restrict__ out,
                                    int ld_out) {
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
  if (jstep > 0) {
    fold_blocks(pb, jstride, Dh, dd, 0, jmax, jstep, m, l, acc);
  } else {
    for (int jb = 0; jb <= jmax; jb += ATTN_GROUP) {
      float gm = -CUDART_INF_F, gl = 0.f, ga = 0.f;
      fold_blocks(pb, jstride, Dh, dd, jb, min(jmax, jb + ATTN_GROUP - 1), 1, gm, gl, ga);
      if (gm == -CUDART_INF_F) continue;
      float a, bg;
      fold_stats(m, l, gm, gl, a, bg);
      acc = fold_acc(acc, a, ga, bg);
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
__global__ void __launch_bounds__(ATTN_THREADS, 4) attn_fused_kernel(const TD* __restrict__ qrot,
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
  stage_q(sm, qrot + static_cast<size_t>(b * T + tq0) * d + h * Dh, d, nq, Dh);
  for (int t = threadIdx.x; t < QT; t += ATTN_THREADS) {
    sm.fold[4 * t] = sm.gfold[4 * t] = -CUDART_INF_F;
    sm.fold[4 * t + 1] = sm.gfold[4 * t + 1] = 0.f;
  }
  // running accumulators: of the whole fold (cc) and of the current fold group (gc)
  float cc[ACC_N], gc[ACC_N];
#pragma unroll
  for (int i = 0; i < ACC_N; ++i) cc[i] = gc[i] = 0.f;
  const int jlast = (L0 + tq0 + nq - 1) / ATTN_BLOCK;
  // K and V of the next block in flight while this block computes (as in attn_block_kernel)
  const TD* kvb = kv + static_cast<size_t>(b) * Lmax * 2 * HD + static_cast<size_t>(h) * Dh;
  auto nk_of = [&](int j) { return min(ATTN_BLOCK, Lend - j * ATTN_BLOCK); };
  stage_k(sm, kvb, HD, Dh, nk_of(0));
  stage_v(sm, kvb, HD, Dh, nk_of(0));
  for (int j = 0; j <= jlast; ++j) {
    const int k0 = j * ATTN_BLOCK;
    const int nk = nk_of(j);
    const bool more = j < jlast;
    cp_async_wait<1>();  // K of block j (its V may still be in flight)
    __syncthreads();
    block_scores(sm, Dh, nk, nq, k0, L0 + tq0, scale);
    __syncthreads();  // K of block j no longer read
    if (more) stage_k(sm, kvb + static_cast<size_t>(j + 1) * ATTN_BLOCK * 2 * HD, HD, Dh, nk_of(j + 1));
    block_softmax(sm, nq);
    if (more)
      cp_async_wait<1>();  // V of block j (the next K may still be in flight)
    else
      cp_async_wait<0>();
    __syncthreads();
    for (int t = threadIdx.x; t < nq; t += ATTN_THREADS) {
      const float mj = sm.stt[2 * t];
      float* f = sm.gfold + 4 * t;
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
    float acc[ACC_N];
    block_pv(sm, Dh, nk, nq, acc);
    __syncthreads();  // V of block j no longer read
    if (more) stage_v(sm, kvb + static_cast<size_t>(j + 1) * ATTN_BLOCK * 2 * HD, HD, Dh, nk_of(j + 1));
#pragma unroll
    for (int i = 0; i < ACC_N; i += 2) {
      const int t = acc_row<TD>(i, Dh);
      if (acc_live<TD>(i, Dh) && t < nq && sm.stt[2 * t] != -CUDART_INF_F) {
        const float a = sm.gfold[4 * t + 2], bj = sm.gfold[4 * t + 3];
        gc[i] = fold_acc(gc[i], a, acc[i], bj);
        gc[i + 1] = fold_acc(gc[i + 1], a, acc[i + 1], bj);
      }
    }
    if (j % ATTN_GROUP == ATTN_GROUP - 1 || j == jlast) {
      // the group's result folded into the whole fold (a group past a query is skipped, as the
      // combine skips it), then the group accumulator emptied
      __syncthreads();
      for (int t = threadIdx.x; t < nq; t += ATTN_THREADS) {
        float* f = sm.fold + 4 * t;
        float* gf = sm.gfold + 4 * t;
        const float gm = gf[0], gl = gf[1];
        gf[0] = -CUDART_INF_F;
        gf[1] = 0.f;
        if (gm == -CUDART_INF_F) {
          f[3] = -1.f;  // no fold for this query
          continue;
        }
        float m = f[0], l = f[1], a, bg;
        fold_stats(m, l, gm, gl, a, bg);
        f[0] = m;
        f[1] = l;
        f[2] = a;
        f[3] = bg;
      }
      __syncthreads();
#pragma unroll
      for (int i = 0; i < ACC_N; i += 2) {
        const int t = acc_row<TD>(i, Dh);
        if (acc_live<TD>(i, Dh) && t < nq && sm.fold[4 * t + 3] >= 0.f) {
          const float a = sm.fold[4 * t + 2], bg = sm.fold[4 * t + 3];
          cc[i] = fold_acc(cc[i], a, gc[i], bg);
          cc[i + 1] = fold_acc(cc[i + 1], a, gc[i + 1], bg);
        }
        gc[i] = gc[i + 1] = 0.f;
      }
    }
  }
#pragma unroll
  for (int i = 0; i < ACC_N; i += 2) {
    const int t = acc_row<TD>(i, Dh);
    if (acc_live<TD>(i, Dh) && t < nq) {
      const float l = sm.fold[4 * t + 1];
      TD* o = out + static_cast<size_t>(b * T + tq0 + t) * ld_out + h * Dh + acc_col<TD>(i, Dh);
      o[0] = from_f32<TD>(cc[i] / l);
      o[1] = from_f32<TD>(cc[i + 1] / l);
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
  // scores in the base-2 domain: s = (q.k / sqrt(Dh)) log2(e), p = 2^(s - max), the same softmax
  const float scale = static_cast<float>(1.4426950408889634 / std::sqrt(static_cast<double>(Dh)));
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
  int bpc = static_cast<int>(std::max<long long>(1, (static_cast<long long>(kv_blocks) * H * B + want - 1) / want));
  // long contexts: whole groups per CTA, folded in the CTA (no per-block partials, no group fold
  // kernel); the bits are those of the per-block path
  const int group_fold = bpc >= ATTN_GROUP / 2 ? 1 : 0;
  if (group_fold) bpc = (bpc + ATTN_GROUP - 1) / ATTN_GROUP * ATTN_GROUP;
  EVS_CUDA_TRY(evs_launch(attn_block_kernel<TD>, dim3((kv_blocks + bpc - 1) / bpc, H, B), dim3(ATTN_THREADS), smem, st,
                          pdl, static_cast<const TD*>(qrot), static_cast<const TD*>(kv),
                          static_cast<const int32_t*>(s->d_len), T, d, H, Dh, s->max_seqlen, s->attn_blocks,
                          s->attn_tcap, bpc, group_fold, scale, s->attn_part));
  int jstep = 1;
  if (group_fold) {
    jstep = ATTN_GROUP;
  } else if (kv_blocks > ATTN_GROUP && kv_blocks <= ATTN_COMBINE_BLOCKS) {
    jstep = 0;  // a few groups: both fold levels in the combine
  } else if (kv_blocks > ATTN_GROUP) {
    const int ngroups = (kv_blocks + ATTN_GROUP - 1) / ATTN_GROUP;
    EVS_CUDA_TRY(evs_launch(attn_group_fold_kernel, dim3(M, H, ngroups), dim3(Dh), 0, st, pdl, s->attn_part,
                            static_cast<const int32_t*>(s->d_len), T, H, Dh, s->attn_blocks, s->attn_tcap));
    evs_count_launch(1);
    jstep = ATTN_GROUP;
  }
  EVS_CUDA_TRY(evs_launch(attn_combine_kernel<TD>, dim3(M, H), dim3(Dh), 0, st, pdl,
                          static_cast<const float*>(s->attn_part), static_cast<const int32_t*>(s->d_len), T, d, H,
                          Dh, s->attn_blocks, s->attn_tcap, jstep, static_cast<TD*>(s->act), s->ld_act));
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
