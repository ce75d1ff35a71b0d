// γ-parallel neural drafter on the device (fp32), batched over independent rows.
//
// trunk (evspark/specdec/block/neural_draft.py:157-197, evspark/train/drafter.py:208-409):
//   H_ctx = RMSNorm(ctx_proj(last min(ctx_window, len) injection-layer outputs))
//   h = in_proj(embed([anchor, MASK x (γ'-1)])) + pos
//   2 x DraftLayer: Pre-LN attention over [H_ctx ; H_d] (ctx fully visible, drafts causal) + MLP(SiLU)
//   U = (final_ln(h) out_proj) · embedᵀ · H^-1/2
// serial head (neural_draft.py:200-259): q_k = softmax(U_k + B[x_{k-1}]), greedy argmax of q or
//   a draw from q' = apply_transform(log q, T, top_k) with one host uniform per position;
//   conf = σ(conf_w [h ; in_proj(embed(prev))]).
// The context comes straight from the state's capture ring (written by the target forward), so
// drafting needs no host copy of hidden states.
#include <algorithm>
#include <cstring>
#include <string>

#include "internal.hpp"
#include "sampling.cuh"

struct evs_drafter {
  evs_drafter_config cfg;
  int max_batch = 0;
  int CW = 0;  // context rows per batch row (= ctx_window)
  bool finalized = false;
  const float* t[EVS_D_LAYER0 + EVS_D_MAX_LAYERS * EVS_D_PER_LAYER] = {nullptr};
  int64_t numel[EVS_D_LAYER0 + EVS_D_MAX_LAYERS * EVS_D_PER_LAYER] = {0};
  float *ctx_in = nullptr, *ctx = nullptr, *h = nullptr, *xb = nullptr, *q = nullptr;
  float *kb = nullptr, *vb = nullptr, *y = nullptr, *tmp = nullptr, *m1 = nullptr;
  float *z = nullptr, *U = nullptr;
  // in_proj(embed[v]) + in_proj.bias for every token v [V][d], formed once at finalize by the same
  // projection and epilogue as a round's rows (a token's row does not depend on the other rows), so
  // the draft rows [anchor, MASK...] and the confidence head's in_proj(embed(prev)) are gathers
  float* tok_in = nullptr;
  // context rows are projected once per position: the k and v rows of every layer ([n_layers][B]
  // [DR_CR][d], slot = position % DR_CR), with the position and the capture tag of the ring row they
  // came from; a call projects only the rows whose slot does not hold the current (position, tag)
  float *ck = nullptr, *cv = nullptr;
  int32_t* cpos = nullptr;              // [B][DR_CR], -1 = empty
  unsigned long long* ctag = nullptr;   // [B][DR_CR]
  int32_t* cmap = nullptr;              // [B * CW][2]: (row, position) of this call's rows to project
  int32_t* ccount = nullptr;            // [2]: those rows; plus the B * g draft rows
  int64_t* prev = nullptr;
  float* ws = nullptr;  // split-K partials of the projections
  size_t ws_floats = 0;
  void* block = nullptr;
};

namespace {

using namespace evs_sampling;

struct RingPtrs {
  const float* p[4];
};

constexpr int DR_CR = 128;  // cache slots per row: covers the ctx_window (<= 64) positions a call reads
constexpr int DRAFT_ATTN_ROWS_MIN_B = 4;  // rows from which one attention CTA per (head, row) serves all queries
                                          // (fewer rows: one CTA per (head, row, query))

// Which context rows of a call lack a current projection: row b reads positions L-n .. L-1
// (n = min(CW, L)); position P is current when its slot holds P with the capture tag that the
// state's ring row at P carries now.  One CTA: the flags, an exclusive scan in (row, position)
// order, the map of rows to project, and the counts [rows, rows + B*g].
__global__ void __launch_bounds__(1024) ctx_plan_kernel(const int32_t* __restrict__ len, int B, int CW, int g,
                                                        const unsigned long long* __restrict__ cap_tag, int ring_len,
                                                        const int32_t* __restrict__ cpos,
                                                        const unsigned long long* __restrict__ ctag,
                                                        int32_t* __restrict__ cmap, int32_t* __restrict__ ccount) {
  pdl_trigger();
  pdl_wait();
  __shared__ int wsum[32];
  __shared__ int base, pass_total;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  if (threadIdx.x == 0) base = 0;
  __syncthreads();
  const int items = B * CW;
  for (int i0 = 0; i0 < items; i0 += blockDim.x) {
    const int i = i0 + threadIdx.x;
    int need = 0, b = 0, P = 0;
    if (i < items) {
      b = i / CW;
      const int j = i - b * CW, L = len[b], n = min(CW, L);
      if (j < n) {
        P = L - n + j;
        const int slot = P % DR_CR;
        need = !(cpos[b * DR_CR + slot] == P &&
                 ctag[b * DR_CR + slot] == cap_tag[static_cast<size_t>(b) * ring_len + P % ring_len]);
      }
    }
    const unsigned bal = __ballot_sync(0xffffffffu, need);
    if (lane == 0) wsum[warp] = __popc(bal);
    __syncthreads();
    if (warp == 0) {
      const int v = lane < nw ? wsum[lane] : 0;
      int x = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
      }
      if (lane < nw) wsum[lane] = x - v;  // exclusive prefix of the warps
      if (lane == 31) pass_total = x;
    }
    __syncthreads();
    if (need) {
      const int idx = base + wsum[warp] + __popc(bal & ((1u << lane) - 1u));
      cmap[2 * idx] = b;
      cmap[2 * idx + 1] = P;
    }
    __syncthreads();
    if (threadIdx.x == 0) base += pass_total;
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    ccount[0] = base;
    ccount[1] = base + B * g;
  }
}

// the ring rows (injection-layer outputs, n_inject rings concatenated) of the rows to project
__global__ void gather_ctx_rows_kernel(RingPtrs rings, int n_inject, int ring_len, int H,
                                       const int32_t* __restrict__ cmap, const int32_t* __restrict__ ccount,
                                       float* __restrict__ out) {
  pdl_trigger();
  pdl_wait();
  const int r = blockIdx.x;
  if (r >= ccount[0]) return;
  const int b = cmap[2 * r], P = cmap[2 * r + 1];
  float* dst = out + static_cast<size_t>(r) * n_inject * H;
  for (int c = 0; c < n_inject; ++c) {
    const float4* src = reinterpret_cast<const float4*>(rings.p[c] + (static_cast<size_t>(b) * ring_len + P % ring_len) * H);
    float4* d4 = reinterpret_cast<float4*>(dst + c * H);
    for (int e = threadIdx.x; e < H / 4; e += blockDim.x) d4[e] = src[e];
  }
}

// Split-K partials of a projection summed in split order (reduce_splits_kernel's additions), then
// the drafter's elementwise step after that projection (acc = the sum, t = row % g):
//   EPI_BIAS_NORM   out = RMSNorm(acc + bias)                     context rows
//   EPI_IN_NORM     h = (acc + bias) + pos[t]; out = RMSNorm(h)   in-projection and the first pre-norm
//   EPI_RESID_NORM  h = h + (acc (+ bias)); out = RMSNorm(h)      attention / MLP output, next norm
//   EPI_BIAS_SILU   out = silu(acc + bias)                        MLP hidden layer
//   EPI_BIAS        out = acc + bias                              out-projection, conf in-projection
//   EPI_SCALE       out = acc * s                                 logits scale H^-1/2
// RMSNorm(v) = scale * (v / sqrt(mean(v²) + eps)), the sum of squares per thread over columns
// tid, tid + 256, ..., then the warp butterfly and the warps in order.  The norm modes run one CTA
// per row; the others one thread per element.
//   EPI_TOK_IN_NORM h = tok_in[id] + pos[t]; out = RMSNorm(h)     EPI_IN_NORM from the token table
//                   (id = anchor[b] at t = 0, mask_id after it): the same values, no projection
enum DraftEpi { EPI_BIAS_NORM, EPI_IN_NORM, EPI_RESID_NORM, EPI_BIAS_SILU, EPI_BIAS, EPI_SCALE, EPI_TOK_IN_NORM };
constexpr int EPI_THREADS = 256;
constexpr int EPI_VPT = 4;  // norm modes: columns per thread per pass
constexpr int EPI_SB = 8;   // norm modes: splits per batch of loads
struct DraftEpiArgs {
  const float* ws;  // partials [splits][M][N]
  int splits, M, N;
  const float* bias;
  const float* pos;  // EPI_IN_NORM: [g][N] position rows (t = row % g)
  int g;
  float* h;  // residual stream [M][N] (EPI_IN_NORM writes it, EPI_RESID_NORM updates it)
  const float* scale;
  float* out;
  float eps, s;
  const float* tok_in;      // EPI_TOK_IN_NORM: the token table [V][N]
  const int64_t* anchor;    // ... the anchor of each batch row
  int mask_id;
  const int32_t* m_dev;     // optional device-side row count (rows past it are skipped)
};

template <int MODE>
__global__ void __launch_bounds__(EPI_THREADS) draft_epi_kernel(DraftEpiArgs a) {
  pdl_trigger();
  pdl_wait();
  const size_t MN = static_cast<size_t>(a.M) * a.N;
  if constexpr (MODE == EPI_BIAS_NORM || MODE == EPI_IN_NORM || MODE == EPI_RESID_NORM || MODE == EPI_TOK_IN_NORM) {
    extern __shared__ float vrow[];  // the row before the norm
    __shared__ float red[33];
    const int N = a.N;
    const int M_rows = a.m_dev != nullptr ? min(a.M, *a.m_dev) : a.M;
    for (int row = blockIdx.x; row < M_rows; row += gridDim.x) {
    if (row != static_cast<int>(blockIdx.x)) __syncthreads();  // the previous row's vrow and red are read
    const size_t r0 = static_cast<size_t>(row) * N;
    float ss = 0.f;
    // EPI_VPT columns c = tid + 256 j per pass; the split loads of all of them are in flight together
    for (int c0 = 0; c0 < N; c0 += EPI_THREADS * EPI_VPT) {
      float acc[EPI_VPT], hv[EPI_VPT];
#pragma unroll
      for (int j = 0; j < EPI_VPT; ++j) {
        acc[j] = 0.f;
        const int c = c0 + threadIdx.x + j * EPI_THREADS;
        if (MODE == EPI_RESID_NORM && c < N) hv[j] = a.h[r0 + c];
      }
      if constexpr (MODE == EPI_TOK_IN_NORM) {
        const int t = row % a.g;
        const int64_t id = t == 0 ? a.anchor[row / a.g] : a.mask_id;
#pragma unroll
        for (int j = 0; j < EPI_VPT; ++j) {
          const int c = c0 + threadIdx.x + j * EPI_THREADS;
          if (c < N) acc[j] = a.tok_in[static_cast<size_t>(id) * N + c];
        }
      }
      for (int s0 = 0; s0 < (MODE == EPI_TOK_IN_NORM ? 0 : a.splits); s0 += EPI_SB) {
        float v[EPI_VPT][EPI_SB];
#pragma unroll
        for (int j = 0; j < EPI_VPT; ++j)
#pragma unroll
          for (int k = 0; k < EPI_SB; ++k) {
            const int c = c0 + threadIdx.x + j * EPI_THREADS;
            if (c < N && s0 + k < a.splits) v[j][k] = __ldcg(a.ws + static_cast<size_t>(s0 + k) * MN + r0 + c);
          }
#pragma unroll
        for (int j = 0; j < EPI_VPT; ++j)
#pragma unroll
          for (int k = 0; k < EPI_SB; ++k)
            if (s0 + k < a.splits) acc[j] += v[j][k];
      }
#pragma unroll
      for (int j = 0; j < EPI_VPT; ++j) {
        const int c = c0 + threadIdx.x + j * EPI_THREADS;
        if (c >= N) break;
        float v;
        if constexpr (MODE == EPI_BIAS_NORM) {
          v = acc[j] + a.bias[c];
        } else if constexpr (MODE == EPI_IN_NORM) {
          v = acc[j] + a.bias[c];
          v = v + a.pos[static_cast<size_t>(row % a.g) * N + c];
          a.h[r0 + c] = v;
        } else if constexpr (MODE == EPI_TOK_IN_NORM) {
          v = acc[j] + a.pos[static_cast<size_t>(row % a.g) * N + c];  // acc = in_proj(embed) + bias
          a.h[r0 + c] = v;
        } else {
          const float x = a.bias ? acc[j] + a.bias[c] : acc[j];
          v = hv[j] + x;
          a.h[r0 + c] = v;
        }
        vrow[c] = v;
        ss = fmaf(v, v, ss);
      }
    }
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x == 0) {
      float t = 0.f;
      for (int w = 0; w < EPI_THREADS / 32; ++w) t += red[w];
      red[32] = t;
    }
    __syncthreads();
    const float rms = sqrtf(red[32] / static_cast<float>(N) + a.eps);
    float* o = a.out + r0;
    for (int c = threadIdx.x; c < N; c += EPI_THREADS) o[c] = a.scale[c] * (vrow[c] / rms);
    }
  } else {
    const size_t i = static_cast<size_t>(blockIdx.x) * EPI_THREADS + threadIdx.x;
    if (i >= MN) return;
    const float acc = split_sum(a.ws + i, MN, a.splits);
    if constexpr (MODE == EPI_BIAS_SILU) {
      const float v = acc + a.bias[i % a.N];
      a.out[i] = v / (1.0f + expf(-v));
    } else if constexpr (MODE == EPI_BIAS) {
      a.out[i] = acc + a.bias[i % a.N];
    } else {
      a.out[i] = acc * a.s;
    }
  }
}

// rows of the k / v projections: [the B*g draft rows (xb) ; the context rows to project]
// The q, k and v partial sums of one layer, each added in split order (reduce_splits_kernel's
// additions; blockIdx.y = 0, 1, 2 for q, k, v).  q and the draft rows (below Bg) of k and v go to
// out[]; the context rows of k and v (row Bg + r is the r-th context row of this call, cmap) go
// straight into their cache slots, and after the last layer the slots get the rows' positions and
// capture tags, after which those rows are current for later calls.
struct QkvRed {
  const float* ws[3];  // [splits][M_j][N]
  float* out[3];
  int M[3];
};
__global__ void qkv_reduce_kernel(const __grid_constant__ QkvRed a, int splits, int N, int Bg,
                                  const int32_t* __restrict__ ccount, const int32_t* __restrict__ cmap,
                                  float* __restrict__ ck, float* __restrict__ cv, int last,
                                  const unsigned long long* __restrict__ cap_tag, int ring_len,
                                  int32_t* __restrict__ cpos, unsigned long long* __restrict__ ctag) {
  pdl_trigger();
  pdl_wait();
  const int j = static_cast<int>(blockIdx.y);
  const int M = a.M[j];
  const size_t MN = static_cast<size_t>(M) * N;
  // rows with work: q's Bg; for k and v the draft rows and this call's context rows (ccount[1])
  const int rows = (j == 0 || ccount == nullptr) ? M : min(M, ccount[1]);
  const int lim = rows * N;
  const float* ws = a.ws[j];
  float* out = a.out[j];
  float* cache = j == 1 ? ck : cv;
  for (int i = static_cast<int>(blockIdx.x * blockDim.x + threadIdx.x); i < lim;
       i += static_cast<int>(gridDim.x * blockDim.x)) {
    const float acc = split_sum(ws + i, MN, splits);
    const int row = i / N;
    if (j == 0 || row < Bg) {
      out[i] = acc;
      continue;
    }
    const int r = row - Bg, col = i - row * N;
    const int b = cmap[2 * r], P = cmap[2 * r + 1];
    const int slot = P % DR_CR;
    cache[(static_cast<size_t>(b) * DR_CR + slot) * N + col] = acc;
    if (last && j == 2 && col == 0) {
      cpos[b * DR_CR + slot] = P;
      ctag[b * DR_CR + slot] = cap_tag[static_cast<size_t>(b) * ring_len + P % ring_len];
    }
  }
}

// one CTA per (query t, head, row b); 128 threads; keys = the row's context positions L-n .. L-1
// (n = min(CW, L), their k/v from the cache slots) and the drafts <= t, in that order
__global__ void __launch_bounds__(128) draft_attn_kernel(const float* q, const float* kd, const float* vd,
                                                         const float* ck, const float* cv, const int32_t* len,
                                                         int with_ctx, int CW, int g, int d, int heads, float* y) {
  pdl_trigger();
  pdl_wait();
  __shared__ float sc[256];
  __shared__ float red[8];
  const int t = blockIdx.x, hh = blockIdx.y, b = blockIdx.z;
  const int hd = d / heads;
  const int L = len[b];
  const int nctx = with_ctx ? min(CW, L) : 0;
  const int nk = CW + g;
  const float scale = rsqrtf(static_cast<float>(hd));
  const float* qr = q + (static_cast<size_t>(b) * g + t) * d + hh * hd;
  auto krow = [&](const float* cbuf, const float* dbuf, int j) -> const float* {
    return j < CW ? cbuf + (static_cast<size_t>(b) * DR_CR + (L - nctx + j) % DR_CR) * d + hh * hd
                  : dbuf + (static_cast<size_t>(b) * g + j - CW) * d + hh * hd;
  };
  for (int j = threadIdx.x; j < nk; j += blockDim.x) {
    const bool vis = j < CW ? j < nctx : (j - CW) <= t;
    float s = -CUDART_INF_F;
    if (vis) {
      const float* kr = krow(ck, kd, j);
      float acc = 0.f;
      for (int e = 0; e < hd; ++e) acc = fmaf(qr[e], kr[e], acc);
      s = acc * scale;
    }
    sc[j] = s;
  }
  __syncthreads();
  float m = -CUDART_INF_F;
  for (int j = threadIdx.x; j < nk; j += blockDim.x) m = fmaxf(m, sc[j]);
  m = warp_max(m);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  m = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
  __syncthreads();
  float l = 0.f;
  for (int j = threadIdx.x; j < nk; j += blockDim.x) {
    const float p = sc[j] == -CUDART_INF_F ? 0.f : expf(sc[j] - m);
    sc[j] = p;
    l += p;
  }
  l = warp_sum(l);
  if ((threadIdx.x & 31) == 0) red[4 + (threadIdx.x >> 5)] = l;
  __syncthreads();
  l = (red[4] + red[5]) + (red[6] + red[7]);
  for (int e = threadIdx.x; e < hd; e += blockDim.x) {
    float acc = 0.f;
    // a key with p = 0 (invisible, or underflowed) adds exactly nothing: its row is not read
    for (int j = 0; j < nk; ++j)
      if (sc[j] != 0.f) acc = fmaf(sc[j], krow(cv, vd, j)[e], acc);
    y[(static_cast<size_t>(b) * g + t) * d + hh * hd + e] = acc / l;
  }
}

// Many rows: one CTA per (head, row b) for all g queries, with the row's visible k/v rows staged
// once in shared memory (K rows padded to hd + 1 floats: a thread per key reads its own row without
// bank conflicts).  Each query runs draft_attn_kernel's arithmetic, thread for thread (same key per
// thread, same reductions, same add order), so the two kernels give the same bits.
__global__ void __launch_bounds__(128) draft_attn_rows_kernel(const float* q, const float* kd, const float* vd,
                                                              const float* ck, const float* cv, const int32_t* len,
                                                              int with_ctx, int CW, int g, int d, int heads, int qpc,
                                                              float* y) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ __align__(16) float da_sm[];
  __shared__ float red[8];
  const int hh = blockIdx.x, b = blockIdx.y;
  // this CTA's queries t0 .. t1-1 (blockIdx.z chunk of qpc); the draft keys up to t1-1 are staged
  const int t0 = blockIdx.z * qpc, t1 = min(g, t0 + qpc);
  const int hd = d / heads;
  const int L = len[b];
  const int nctx = with_ctx ? min(CW, L) : 0;
  const int nk = CW + g;
  const float scale = rsqrtf(static_cast<float>(hd));
  float* Ks = da_sm;                                // [nk][hd + 1]
  float* Vs = Ks + (nk * (hd + 1) + 3) / 4 * 4;     // [nk][hd], 16-byte aligned
  float* Qs = Vs + nk * hd;           // [g][hd]
  float* sc = Qs + g * hd;            // [nk]
  auto krow = [&](const float* cbuf, const float* dbuf, int j) -> const float* {
    return j < CW ? cbuf + (static_cast<size_t>(b) * DR_CR + (L - nctx + j) % DR_CR) * d + hh * hd
                  : dbuf + (static_cast<size_t>(b) * g + j - CW) * d + hh * hd;
  };
  // 16-byte loads, eight per thread in flight (context slots before position 0 are never visible
  // and never read)
  const int h4 = hd / 4, n4 = (CW + t1) * h4;
  for (int i0 = threadIdx.x; i0 < n4; i0 += 8 * blockDim.x) {
    float4 kx[8], vx[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i = i0 + u * blockDim.x, j = i / h4, e4 = i - j * h4;
      if (i < n4 && !(j < CW && j >= nctx)) {
        kx[u] = *reinterpret_cast<const float4*>(krow(ck, kd, j) + 4 * e4);
        vx[u] = *reinterpret_cast<const float4*>(krow(cv, vd, j) + 4 * e4);
      }
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i = i0 + u * blockDim.x, j = i / h4, e4 = i - j * h4;
      if (i < n4 && !(j < CW && j >= nctx)) {
        float* kd4 = Ks + j * (hd + 1) + 4 * e4;
        kd4[0] = kx[u].x;
        kd4[1] = kx[u].y;
        kd4[2] = kx[u].z;
        kd4[3] = kx[u].w;
        *reinterpret_cast<float4*>(Vs + j * hd + 4 * e4) = vx[u];
      }
    }
  }
  for (int i = threadIdx.x; i < (t1 - t0) * h4; i += blockDim.x) {
    const int t = i / h4, e4 = i - t * h4;
    *reinterpret_cast<float4*>(Qs + 4 * i) =
        *reinterpret_cast<const float4*>(q + (static_cast<size_t>(b) * g + t0 + t) * d + hh * hd + 4 * e4);
  }
  __syncthreads();
  for (int t = t0; t < t1; ++t) {
    const float* qr = Qs + (t - t0) * hd;
    for (int j = threadIdx.x; j < nk; j += blockDim.x) {
      const bool vis = j < CW ? j < nctx : (j - CW) <= t;
      float s = -CUDART_INF_F;
      if (vis) {
        const float* kr = Ks + j * (hd + 1);
        float acc = 0.f;
        for (int e = 0; e < hd; ++e) acc = fmaf(qr[e], kr[e], acc);
        s = acc * scale;
      }
      sc[j] = s;
    }
    __syncthreads();
    float m = -CUDART_INF_F;
    for (int j = threadIdx.x; j < nk; j += blockDim.x) m = fmaxf(m, sc[j]);
    m = warp_max(m);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    m = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
    __syncthreads();
    float l = 0.f;
    for (int j = threadIdx.x; j < nk; j += blockDim.x) {
      const float p = sc[j] == -CUDART_INF_F ? 0.f : expf(sc[j] - m);
      sc[j] = p;
      l += p;
    }
    l = warp_sum(l);
    if ((threadIdx.x & 31) == 0) red[4 + (threadIdx.x >> 5)] = l;
    __syncthreads();
    l = (red[4] + red[5]) + (red[6] + red[7]);
    for (int e = threadIdx.x; e < hd; e += blockDim.x) {
      float acc = 0.f;
      for (int j = 0; j < nk; ++j)
        if (sc[j] != 0.f) acc = fmaf(sc[j], Vs[j * hd + e], acc);
      y[(static_cast<size_t>(b) * g + t) * d + hh * hd + e] = acc / l;
    }
    __syncthreads();  // sc and red are rewritten by the next query
  }
}

// serial Markov head for V = 128 * NL (NL = 1, 2, 4), with the warp-level layout of
// warp_pw_sum / warp_argmax16 (sampling.cuh) for the sums, argmax and top-k; only the
// left-to-right cumulative sum of sampling runs sequentially, in shared memory.
// 4 warps: the elementwise fp32/fp64 math of a step is spread over 128 threads (element i on
// thread i % 128), through shared memory; warp 0 gathers the row into the pairwise-sum layout
// above (lane L: elements leaf*128 + j + 8t) for the sums, argmax and top-k.
template <int NL>
__global__ void __launch_bounds__(128) serial_head_warp_kernel(const float* U, const float* markov,
                                                              const int64_t* anchor, int g, int greedy,
                                                              double temperature, int top_k, const double* u,
                                                              const int64_t* forced, int64_t* tokens, double* qout,
                                                              int64_t* prev_ids) {
  pdl_trigger();
  constexpr int V = 128 * NL;
  constexpr int PT = V / 128;  // elements per thread in the elementwise phases
  {
    // the Markov table rows are read one dependent step at a time: pull the table into L2 first
    constexpr unsigned TB = V * V * 4, CHUNK = 16384;
    for (unsigned off = threadIdx.x * CHUNK; off < TB; off += blockDim.x * CHUNK)
      asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(reinterpret_cast<const char*>(markov) + off),
                   "r"(CHUNK)
                   : "memory");
  }
  pdl_wait();
  __shared__ double row[V];
  __shared__ double cval[V];  // sampling: nonzero weights (then their prefix sums) in index order
  __shared__ int cidx[V];     // ... and their indices
  __shared__ double su[EVS_RETAIN_MAX];
  __shared__ long long sfo[EVS_RETAIN_MAX];
  __shared__ float fred[4];
  __shared__ double dsh[2];
  __shared__ int ish[1];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, leaf = lane >> 3, j = lane & 7;
  const bool act = leaf < NL;
  const int base = act ? leaf * 128 + j : 0;
  const int b = blockIdx.x;
  const unsigned full = 0xffffffffu;
  int prev = static_cast<int>(anchor[b]);
  // per-step inputs up front: the uniforms and forced tokens of every step
  for (int i = tid; i < g; i += blockDim.x) {
    su[i] = (!greedy && u != nullptr) ? u[static_cast<size_t>(b) * g + i] : 0.0;
    sfo[i] = forced != nullptr ? forced[static_cast<size_t>(b) * g + i] : -1;
  }
  __syncthreads();
  for (int k = 0; k < g; ++k) {
    const float* Ur = U + (static_cast<size_t>(b) * g + k) * V;
    const float* Br = markov + static_cast<size_t>(prev) * V;
    // q_k = softmax(U_k + B[prev]) in fp32
    float lg[PT];
    float mx = -CUDART_INF_F;
#pragma unroll
    for (int s2 = 0; s2 < PT; ++s2) {
      lg[s2] = Ur[tid + 128 * s2] + Br[tid + 128 * s2];
      mx = fmaxf(mx, lg[s2]);
    }
    mx = warp_max(mx);
    if (lane == 0) fred[warp] = mx;
    __syncthreads();
    mx = fmaxf(fmaxf(fred[0], fred[1]), fmaxf(fred[2], fred[3]));
    __syncthreads();
    float ss = 0.f;
#pragma unroll
    for (int s2 = 0; s2 < PT; ++s2) {
      lg[s2] = expf(lg[s2] - mx);
      ss += lg[s2];
    }
    ss = warp_sum(ss);
    if (lane == 0) fred[warp] = ss;
    __syncthreads();
    ss = (fred[0] + fred[1]) + (fred[2] + fred[3]);
    double* qo = qout + (static_cast<size_t>(b) * g + k) * V;
    int tok = 0;
    if (greedy) {
#pragma unroll
      for (int s2 = 0; s2 < PT; ++s2) {
        const double e = static_cast<double>(lg[s2] / ss);
        row[tid + 128 * s2] = e;
        qo[tid + 128 * s2] = e;
      }
      __syncthreads();
      if (warp == 0) {
        double e[16];
#pragma unroll
        for (int t = 0; t < 16; ++t) e[t] = act ? row[base + 8 * t] : -CUDART_INF;
        tok = warp_argmax16(e, base, nullptr);
        if (lane == 0) ish[0] = tok;
      }
      __syncthreads();
      tok = ish[0];
    } else {
      // q' = apply_transform(log q): log on the support, -inf elsewhere, / temperature
      const bool onehot = temperature <= 0.0;
#pragma unroll
      for (int s2 = 0; s2 < PT; ++s2) {
        const double e = static_cast<double>(lg[s2] / ss);
        const double x = e > 0.0 ? log(e) : -CUDART_INF;
        row[tid + 128 * s2] = onehot ? x : x / temperature;
      }
      __syncthreads();
      double p[16];
      if (warp == 0) {
        double x[16];
#pragma unroll
        for (int t = 0; t < 16; ++t) x[t] = act ? row[base + 8 * t] : -CUDART_INF;
        double xm;
        const int am = warp_argmax16(x, base, &xm);
        if (lane == 0) {
          dsh[0] = xm;
          ish[0] = am;
        }
      }
      __syncthreads();
      if (onehot) {
        const int am = ish[0];
#pragma unroll
        for (int s2 = 0; s2 < PT; ++s2) row[tid + 128 * s2] = (tid + 128 * s2 == am) ? 1.0 : 0.0;
      } else {
        const double xm = dsh[0];
#pragma unroll
        for (int s2 = 0; s2 < PT; ++s2) row[tid + 128 * s2] = exp(row[tid + 128 * s2] - xm);
      }
      __syncthreads();
      if (!onehot) {
        // normalise: the pairwise sum in warp 0's layout, then every thread divides its elements
        if (warp == 0) {
#pragma unroll
          for (int t = 0; t < 16; ++t) p[t] = act ? row[base + 8 * t] : 0.0;
          const double z = warp_pw_sum<NL>(p, lane);
          if (lane == 0) dsh[1] = z;
        }
        __syncthreads();
        const double z = dsh[1];
        const bool bad = !(z > 0.0) || !isfinite(z);
#pragma unroll
        for (int s2 = 0; s2 < PT; ++s2) row[tid + 128 * s2] = bad ? 1.0 / V : row[tid + 128 * s2] / z;
        __syncthreads();
      }
      if (warp == 0) {
#pragma unroll
        for (int t = 0; t < 16; ++t) p[t] = act ? row[base + 8 * t] : 0.0;
        if (!onehot) {
          if (top_k > 0 && top_k < V) {
            unsigned keep = 0;
            double m[16];
#pragma unroll
            for (int t = 0; t < 16; ++t) m[t] = act ? p[t] : -CUDART_INF;
            for (int r = 0; r < top_k; ++r) {
              const int am = warp_argmax16(m, base, nullptr);
#pragma unroll
              for (int t = 0; t < 16; ++t)
                if (act && base + 8 * t == am) {
                  keep |= 1u << t;
                  m[t] = -CUDART_INF;
                }
            }
#pragma unroll
            for (int t = 0; t < 16; ++t) m[t] = (keep >> t & 1u) ? p[t] : 0.0;
            const double ms = warp_pw_sum<NL>(m, lane);
            const bool bad2 = !(ms > 0.0) || !isfinite(ms);
            // the kept weights / ms: at most top_k per warp and usually at most one per lane, so the
            // lanes divide their r-th kept weight in round r (warp-uniform rounds, no per-slot branch)
            int rounds = __popc(keep);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) rounds = max(rounds, __shfl_xor_sync(full, rounds, o));
            double pk[16];
#pragma unroll
            for (int t = 0; t < 16; ++t) pk[t] = 0.0;
            unsigned rem = keep;
            for (int r = 0; r < rounds; ++r) {
              const int ts = rem != 0u ? __ffs(rem) - 1 : -1;
              double x = 0.0;
#pragma unroll
              for (int t = 0; t < 16; ++t)
                if (t == ts) x = m[t];
              const double y = bad2 ? 1.0 / top_k : x / ms;
#pragma unroll
              for (int t = 0; t < 16; ++t)
                if (t == ts) pk[t] = y;
              rem &= rem - 1u;
            }
#pragma unroll
            for (int t = 0; t < 16; ++t) p[t] = (keep >> t & 1u) ? pk[t] : 0.0;
          }
        }
        // the q' row out, then sample_categorical(q'): clip, normalise (pairwise), cumsum, inverse CDF
        double w[16];
#pragma unroll
        for (int t = 0; t < 16; ++t) {
          if (act) qo[base + 8 * t] = p[t];
          w[t] = fmax(p[t], 0.0);
        }
        const double s = warp_pw_sum<NL>(w, lane);
        const bool bad = !(s > 0.0) || !isfinite(s);
        __syncwarp();
        // the weights in index order (1/V each when their sum is unusable)
#pragma unroll
        for (int t = 0; t < 16; ++t)
          if (act) row[base + 8 * t] = bad ? 1.0 / V : w[t];
        __syncwarp();
        // cumsum + inverse CDF.  Adding a zero leaves the running sum unchanged, so the prefix
        // sums are those of the nonzero weights in index order: the nonzero weights are compacted in
        // index order (round i holds indices 32i .. 32i+31, a ballot gives each its place) and
        // normalised there, one division per lane (an entry whose quotient underflows to 0 only
        // repeats the prefix before it, which cannot be the first to exceed u); lane 0 sums them in
        // order, and since the prefixes never decrease, the count of prefix / last <= u is the index
        // of the first nonzero that fails it
        int nnz = 0;
#pragma unroll
        for (int i = 0; i < V / 32; ++i) {
          const double v = row[i * 32 + lane];
          const unsigned nzm = __ballot_sync(full, v != 0.0);
          if (v != 0.0) {
            const int pos = nnz + __popc(nzm & ((1u << lane) - 1u));
            cval[pos] = v;
            cidx[pos] = i * 32 + lane;
          }
          nnz += __popc(nzm);
        }
        __syncwarp();
        if (!bad)
          for (int n = lane; n < nnz; n += 32) cval[n] = cval[n] / s;
        __syncwarp();
        if (lane == 0) {
          double c = 0.0;
          for (int n = 0; n < nnz; ++n) {
            c += cval[n];
            cval[n] = c;
          }
        }
        __syncwarp();
        const double last = cval[nnz - 1];  // nnz >= 1: the normalised weights sum to about 1
        const double uu = su[k];
        int first = nnz;
        for (int n = lane; n < nnz; n += 32)
          if (!(cval[n] / last <= uu)) {
            first = n;
            break;
          }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) first = min(first, __shfl_xor_sync(full, first, o));
        const int cnt = first < nnz ? cidx[first] : V;
        if (lane == 0) ish[0] = cnt < V ? cnt : V - 1;
      }
      __syncthreads();
      tok = ish[0];
    }
    if (sfo[k] >= 0) tok = static_cast<int>(sfo[k]);  // negative: not forced
    if (tid == 0) {
      tokens[static_cast<size_t>(b) * g + k] = tok;
      prev_ids[static_cast<size_t>(b) * g + k] = prev;
    }
    prev = tok;
    __syncthreads();  // row / fred / ish are reused by the next step
  }
}

// serial Markov head, one CTA per row
__global__ void __launch_bounds__(256) serial_head_kernel(const float* U, const float* markov, const int64_t* anchor,
                                                          int g, int V, int greedy, double temperature, int top_k,
                                                          const double* u, const int64_t* forced, int64_t* tokens,
                                                          double* qout, int64_t* prev_ids) {
  pdl_trigger();
  pdl_wait();
  __shared__ float lg[VMAX];
  __shared__ double e[VMAX], row[VMAX], masked[VMAX];
  __shared__ int keep[VMAX];
  __shared__ SampScratch sc;
  __shared__ float fred[9];
  __shared__ int s_prev;
  const int b = blockIdx.x;
  if (threadIdx.x == 0) s_prev = static_cast<int>(anchor[b]);
  __syncthreads();
  for (int k = 0; k < g; ++k) {
    const int prev = s_prev;
    const float* Ur = U + (static_cast<size_t>(b) * g + k) * V;
    const float* Br = markov + static_cast<size_t>(prev) * V;
    // q_k = softmax(U_k + B[prev]) in fp32
    float mx = -CUDART_INF_F;
    for (int v = threadIdx.x; v < V; v += blockDim.x) {
      lg[v] = Ur[v] + Br[v];
      mx = fmaxf(mx, lg[v]);
    }
    mx = warp_max(mx);
    if ((threadIdx.x & 31) == 0) fred[threadIdx.x >> 5] = mx;
    __syncthreads();
    if (threadIdx.x == 0) {
      float m2 = fred[0];
      for (int w = 1; w < static_cast<int>(blockDim.x >> 5); ++w) m2 = fmaxf(m2, fred[w]);
      fred[8] = m2;
    }
    __syncthreads();
    mx = fred[8];
    __syncthreads();
    float ssum = 0.f;
    for (int v = threadIdx.x; v < V; v += blockDim.x) {
      lg[v] = expf(lg[v] - mx);
      ssum += lg[v];
    }
    ssum = warp_sum(ssum);
    if ((threadIdx.x & 31) == 0) fred[threadIdx.x >> 5] = ssum;
    __syncthreads();
    if (threadIdx.x == 0) {
      float s2 = 0.f;
      for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) s2 += fred[w];
      fred[8] = s2;
    }
    __syncthreads();
    const float zs = fred[8];
    for (int v = threadIdx.x; v < V; v += blockDim.x) e[v] = static_cast<double>(lg[v] / zs);
    __syncthreads();
    double* qo = qout + (static_cast<size_t>(b) * g + k) * V;
    int tok;
    if (greedy) {
      tok = block_argmax(e, V, &sc);
      for (int v = threadIdx.x; v < V; v += blockDim.x) qo[v] = e[v];
    } else {
      // q' = apply_transform(log q): log on the support, -inf elsewhere
      for (int v = threadIdx.x; v < V; v += blockDim.x) row[v] = e[v] > 0.0 ? log(e[v]) : -CUDART_INF;
      __syncthreads();
      transform_row(row, V, temperature, top_k, masked, keep, e, &sc);
      for (int v = threadIdx.x; v < V; v += blockDim.x) {
        qo[v] = masked[v];
        row[v] = fmax(masked[v], 0.0);
      }
      __syncthreads();
      tok = block_sample_clipped(row, V, u[static_cast<size_t>(b) * g + k], &sc);
    }
    if (threadIdx.x == 0) {
      if (forced != nullptr && forced[static_cast<size_t>(b) * g + k] >= 0)  // negative: not forced
        tok = static_cast<int>(forced[static_cast<size_t>(b) * g + k]);
      tokens[static_cast<size_t>(b) * g + k] = tok;
      prev_ids[static_cast<size_t>(b) * g + k] = prev;
      s_prev = tok;
    }
    __syncthreads();
  }
}

// conf[row] = sigmoid([h ; tok_in[prev[row]]] · w + bias); one warp per row
__global__ void conf_kernel(const float* h, const float* tok_in, const int64_t* prev, const float* w,
                            const float* bias, int d, int rows, float* conf) {
  pdl_trigger();
  pdl_wait();
  const int row = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float* pe = tok_in + static_cast<size_t>(prev[row]) * d;
  float acc = 0.f;
  // lane's elements c = lane, lane + 32, ... in order; sixteen of them (and their weights) loaded
  // at a time
  for (int c0 = lane; c0 < 2 * d; c0 += 32 * 16) {
    float x[16], wv[16];
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      const int c = c0 + 32 * k;
      if (c < 2 * d) {
        x[k] = c < d ? h[static_cast<size_t>(row) * d + c] : pe[c - d];
        wv[k] = w[c];
      }
    }
#pragma unroll
    for (int k = 0; k < 16; ++k)
      if (c0 + 32 * k < 2 * d) acc = fmaf(x[k], wv[k], acc);
  }
  acc = warp_sum(acc);
  if (lane == 0) conf[row] = 1.0f / (1.0f + expf(-(acc + bias[0])));
}

int64_t drafter_numel(const evs_drafter_config& c, int id) {
  const int64_t d = c.d_model, H = c.target_hidden, V = c.vocab_size, hid = static_cast<int64_t>(c.mlp_mult) * d;
  switch (id) {
    case EVS_D_EMBED: return V * H;
    case EVS_D_IN_W: return d * H;
    case EVS_D_IN_B: return d;
    case EVS_D_OUT_W: return H * d;
    case EVS_D_OUT_B: return H;
    case EVS_D_POS: return static_cast<int64_t>(c.gamma) * d;
    case EVS_D_CTX_W: return c.n_inject > 0 ? d * c.n_inject * H : 0;
    case EVS_D_CTX_B:
    case EVS_D_CTX_NORM: return c.n_inject > 0 ? d : 0;
    case EVS_D_FINAL_LN: return d;
    case EVS_D_MARKOV: return V * V;
    case EVS_D_CONF_W: return 2 * d;
    case EVS_D_CONF_B: return 1;
    default: break;
  }
  if (id < EVS_D_LAYER0) return 0;
  const int l = (id - EVS_D_LAYER0) / EVS_D_PER_LAYER, r = (id - EVS_D_LAYER0) % EVS_D_PER_LAYER;
  if (l >= c.n_layers) return 0;
  switch (r) {
    case EVS_D_LN1:
    case EVS_D_LN2:
    case EVS_D_MLP2_B: return d;
    case EVS_D_Q:
    case EVS_D_K:
    case EVS_D_V:
    case EVS_D_O: return d * d;
    case EVS_D_MLP0_W: return hid * d;
    case EVS_D_MLP0_B: return hid;
    case EVS_D_MLP2_W: return d * hid;
    default: return 0;
  }
}

// out[M][N] = X W^T (fp32, split-K partials reduced in split order); m_dev: optional device-side
// row count at most M
// m_hint: the row count the grids are sized for when m_dev is given (the kernels walk any rows
// beyond it), so that a launch sized for the largest count does not carry idle CTAs
inline unsigned blocks_for(size_t n, int t) { return static_cast<unsigned>((n + t - 1) / t); }

// projection partials into the workspace (no reduction), then the fused epilogue `mode` over them
int sgemm_epi(evs_drafter* dr, const float* W, const float* X, int ldx, int N, int K, int M, int mode,
              DraftEpiArgs e, cudaStream_t st, int m_hint = 0) {
  const GemmPlan p = gemm_plan_f32_drafter(N, K, M);
  EVS_CHECK_RANGE(static_cast<size_t>(p.splits) * M * N <= dr->ws_floats, "drafter workspace too small");
  EVS_TRY(launch_gemm_simt(W, nullptr, X, ldx, EVS_DTYPE_FP32, p, dr->ws, st, true, e.m_dev, m_hint));
  e.ws = dr->ws;
  e.splits = p.splits;
  e.M = M;
  e.N = N;
  const bool norm = mode == EPI_BIAS_NORM || mode == EPI_IN_NORM || mode == EPI_RESID_NORM || mode == EPI_TOK_IN_NORM;
  const int rows = e.m_dev != nullptr && m_hint > 0 ? std::min(M, m_hint) : M;  // (norm CTAs walk the rest)
  EVS_CHECK_ARG(norm || e.m_dev == nullptr || m_hint <= 0, "a row hint needs a norm epilogue");
  const dim3 grid = norm ? dim3(rows) : dim3(blocks_for(static_cast<size_t>(M) * N, EPI_THREADS));
  const size_t smem = norm ? sizeof(float) * N : 0;
  EVS_CHECK_ARG(smem <= 48 * 1024, "drafter width too large for the fused norm");
  switch (mode) {
    case EPI_BIAS_NORM: EVS_CUDA_TRY(evs_launch(draft_epi_kernel<EPI_BIAS_NORM>, grid, dim3(EPI_THREADS), smem, st, true, e)); break;
    case EPI_IN_NORM: EVS_CUDA_TRY(evs_launch(draft_epi_kernel<EPI_IN_NORM>, grid, dim3(EPI_THREADS), smem, st, true, e)); break;
    case EPI_RESID_NORM: EVS_CUDA_TRY(evs_launch(draft_epi_kernel<EPI_RESID_NORM>, grid, dim3(EPI_THREADS), smem, st, true, e)); break;
    case EPI_TOK_IN_NORM: EVS_CUDA_TRY(evs_launch(draft_epi_kernel<EPI_TOK_IN_NORM>, grid, dim3(EPI_THREADS), smem, st, true, e)); break;
    case EPI_BIAS_SILU: EVS_CUDA_TRY(evs_launch(draft_epi_kernel<EPI_BIAS_SILU>, grid, dim3(EPI_THREADS), 0, st, true, e)); break;
    case EPI_BIAS: EVS_CUDA_TRY(evs_launch(draft_epi_kernel<EPI_BIAS>, grid, dim3(EPI_THREADS), 0, st, true, e)); break;
    default: EVS_CUDA_TRY(evs_launch(draft_epi_kernel<EPI_SCALE>, grid, dim3(EPI_THREADS), 0, st, true, e)); break;
  }
  evs_count_launch(1);
  return EVS_OK;
}

DraftEpiArgs epi(const float* bias, float* out, const float* scale = nullptr, float* h = nullptr,
                 const float* pos = nullptr, int g = 1, float eps = 1e-6f, float sc = 1.f) {
  DraftEpiArgs e{};
  e.bias = bias;
  e.out = out;
  e.scale = scale;
  e.h = h;
  e.pos = pos;
  e.g = g;
  e.eps = eps;
  e.s = sc;
  return e;
}

}  // namespace

extern "C" {

int evs_drafter_create(const evs_drafter_config* cfg, int max_batch, evs_drafter** out) {
  EVS_CHECK_ARG(cfg && out, "null argument");
  const evs_drafter_config& c = *cfg;
  EVS_CHECK_ARG(c.n_layers >= 0 && c.n_layers <= EVS_D_MAX_LAYERS, "drafter n_layers outside [0, 8]");
  EVS_CHECK_ARG(c.n_heads >= 1 && c.d_model % c.n_heads == 0, "d_model must divide into heads");
  EVS_CHECK_ARG(c.gamma >= 1 && c.gamma <= 64, "drafter gamma outside [1, 64]");
  EVS_CHECK_ARG(c.ctx_window >= 1 && c.ctx_window <= 64, "ctx_window outside [1, 64]");
  EVS_CHECK_ARG(c.vocab_size >= 1 && c.vocab_size <= VMAX, "vocab outside [1, 1024]");
  EVS_CHECK_ARG(c.n_inject >= 0 && c.n_inject <= 4, "n_inject outside [0, 4]");
  EVS_CHECK_ARG(max_batch >= 1, "max_batch must be >= 1");
  EVS_CHECK_ARG(c.ctx_window + c.gamma <= 256, "ctx_window + gamma must be <= 256");
  evs_drafter* dr = new evs_drafter();
  dr->cfg = c;
  dr->max_batch = max_batch;
  dr->CW = c.ctx_window;
  const size_t B = max_batch, g = c.gamma, d = c.d_model, H = c.target_hidden, V = c.vocab_size;
  const size_t CW = dr->CW, hid = static_cast<size_t>(c.mlp_mult) * d;
  const size_t nI = c.n_inject > 0 ? c.n_inject : 1;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off = (off + bytes + 255) & ~size_t(255);
    return o;
  };
  const size_t o_ctx_in = take(4 * B * CW * nI * H), o_ctx = take(4 * B * CW * d);
  const size_t o_h = take(4 * B * g * d), o_xb = take(4 * B * g * d), o_q = take(4 * B * g * d);
  const size_t o_kb = take(4 * B * (CW + g) * d), o_vb = take(4 * B * (CW + g) * d);
  const size_t o_y = take(4 * B * g * d), o_tmp = take(4 * B * g * d), o_m1 = take(4 * B * g * hid);
  const size_t o_z = take(4 * B * g * H), o_U = take(4 * B * g * V);
  const size_t o_prev = take(8 * B * g), o_tok = take(4 * V * d);
  const size_t nL = c.n_layers, cache_rows = B * DR_CR;
  const size_t o_ck = take(4 * nL * cache_rows * d), o_cv = take(4 * nL * cache_rows * d);
  const size_t o_cpos = take(4 * cache_rows), o_ctag = take(8 * cache_rows), o_cmap = take(8 * B * CW),
               o_ccount = take(8);
  // largest split-K partial buffer over the drafter's projections
  size_t wsf = 0;
  auto need = [&](size_t M_, size_t N_, size_t K_) {
    const GemmPlan p = gemm_plan_f32_drafter(static_cast<int>(N_), static_cast<int>(K_), static_cast<int>(M_));
    wsf = std::max(wsf, static_cast<size_t>(p.splits) * M_ * N_);
  };
  need(B * CW, d, nI * H);
  need(B * g, d, H);
  need(B * g, d, d);
  need(B * (CW + g), d, d);
  need(B * g, hid, d);
  need(B * g, d, hid);
  need(B * g, H, d);
  need(B * g, V, H);
  need(V, d, H);  // the token table
  {
    // q, k and v of one layer side by side: the draft rows, twice the draft + context rows
    const GemmPlan p = gemm_plan_f32_drafter(static_cast<int>(d), static_cast<int>(d), static_cast<int>(B * (CW + g)));
    wsf = std::max(wsf, static_cast<size_t>(p.splits) * (B * g + 2 * B * (CW + g)) * d);
  }
  const size_t o_ws = take(4 * wsf);
  if (cudaMalloc(&dr->block, off) != cudaSuccess) {
    cudaGetLastError();
    delete dr;
    evs_set_last_error(EVS_ECUDA, "cudaMalloc of the drafter scratch failed");
    return EVS_ECUDA;
  }
  char* base = static_cast<char*>(dr->block);
  dr->ctx_in = reinterpret_cast<float*>(base + o_ctx_in);
  dr->ctx = reinterpret_cast<float*>(base + o_ctx);
  dr->h = reinterpret_cast<float*>(base + o_h);
  dr->xb = reinterpret_cast<float*>(base + o_xb);
  dr->q = reinterpret_cast<float*>(base + o_q);
  dr->kb = reinterpret_cast<float*>(base + o_kb);
  dr->vb = reinterpret_cast<float*>(base + o_vb);
  dr->y = reinterpret_cast<float*>(base + o_y);
  dr->tmp = reinterpret_cast<float*>(base + o_tmp);
  dr->m1 = reinterpret_cast<float*>(base + o_m1);
  dr->z = reinterpret_cast<float*>(base + o_z);
  dr->U = reinterpret_cast<float*>(base + o_U);
  dr->prev = reinterpret_cast<int64_t*>(base + o_prev);
  dr->tok_in = reinterpret_cast<float*>(base + o_tok);
  dr->ck = reinterpret_cast<float*>(base + o_ck);
  dr->cv = reinterpret_cast<float*>(base + o_cv);
  dr->cpos = reinterpret_cast<int32_t*>(base + o_cpos);
  dr->ctag = reinterpret_cast<unsigned long long*>(base + o_ctag);
  dr->cmap = reinterpret_cast<int32_t*>(base + o_cmap);
  dr->ccount = reinterpret_cast<int32_t*>(base + o_ccount);
  dr->ws = reinterpret_cast<float*>(base + o_ws);
  dr->ws_floats = wsf;
  EVS_CUDA_TRY(cudaMemset(dr->block, 0, off));
  EVS_CUDA_TRY(cudaMemset(dr->cpos, 0xff, 4 * cache_rows));  // every slot empty (-1)
  *out = dr;
  return EVS_OK;
}

int evs_drafter_set_tensor(evs_drafter* dr, int id, const void* dev_ptr, int64_t numel) {
  EVS_CHECK_ARG(dr && dev_ptr, "null argument");
  EVS_CHECK_ARG(id >= 0 && id < EVS_D_LAYER0 + EVS_D_MAX_LAYERS * EVS_D_PER_LAYER, "tensor id out of range");
  const int64_t want = drafter_numel(dr->cfg, id);
  EVS_CHECK_ARG(want > 0, "tensor id not used by this drafter");
  EVS_CHECK_ARG(want == numel, "drafter tensor numel mismatch");
  dr->t[id] = static_cast<const float*>(dev_ptr);
  dr->numel[id] = numel;
  return EVS_OK;
}

int evs_drafter_finalize(evs_drafter* dr) {
  EVS_CHECK_ARG(dr != nullptr, "null drafter");
  for (int id = 0; id < EVS_D_LAYER0 + EVS_D_MAX_LAYERS * EVS_D_PER_LAYER; ++id) {
    if (drafter_numel(dr->cfg, id) > 0 && dr->t[id] == nullptr) {
      evs_set_last_error(EVS_EINVAL, ("drafter tensor " + std::to_string(id) + " not set").c_str());
      return EVS_EINVAL;
    }
  }
  // the token table: every embedding row through in_proj (+ bias), the rows a round would form
  const evs_drafter_config& c = dr->cfg;
  cudaStream_t st = nullptr;
  EVS_CUDA_TRY(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
  const int r = sgemm_epi(dr, dr->t[EVS_D_IN_W], dr->t[EVS_D_EMBED], c.target_hidden, c.d_model, c.target_hidden,
                          c.vocab_size, EPI_BIAS, epi(dr->t[EVS_D_IN_B], dr->tok_in), st);
  const cudaError_t e = cudaStreamSynchronize(st);
  cudaStreamDestroy(st);
  EVS_TRY(r);
  EVS_CUDA_TRY(e);
  dr->finalized = true;
  return EVS_OK;
}

void evs_drafter_destroy(evs_drafter* dr) {
  if (dr == nullptr) return;
  if (dr->block) cudaFree(dr->block);
  delete dr;
}

int evs_draft_propose(evs_drafter* dr, const evs_state* s, const int64_t* anchor, int batch, int gamma, int greedy,
                      double temperature, int top_k, const double* u, const int64_t* forced, int64_t* tokens,
                      double* qrows, float* conf, float* U_out, cudaStream_t st) {
  EVS_CHECK_ARG(dr && s && anchor && tokens && qrows && conf, "null argument");
  EVS_CHECK_ARG(dr->finalized, "drafter not finalized");
  const evs_drafter_config& c = dr->cfg;
  if (gamma < 1 || gamma > c.gamma) {
    evs_set_last_error(EVS_EINVAL, ("decode γ'=" + std::to_string(gamma) + " must satisfy 1 <= γ' <= training γ=" +
                                    std::to_string(c.gamma))
                                       .c_str());
    return EVS_EINVAL;
  }
  EVS_CHECK_ARG(batch >= 1 && batch <= dr->max_batch && batch <= s->max_batch, "batch outside drafter/state limits");
  EVS_CHECK_ARG(greedy || u != nullptr, "sampling needs uniforms");
  EVS_CHECK_ARG(c.n_inject <= s->m->n_capture, "state has fewer capture rings than n_inject");
  EVS_CHECK_ARG(c.n_inject == 0 || c.target_hidden == s->m->cfg.d_model, "drafter target_hidden != model d_model");
  EVS_CHECK_RANGE(s->ring_len - s->max_chunk >= dr->CW, "capture ring shorter than the drafter context window");
  const int B = batch, g = gamma, d = c.d_model, H = c.target_hidden, V = c.vocab_size, CW = dr->CW;
  const int hid = c.mlp_mult * d, rows = B * g;
  const size_t B_cap = static_cast<size_t>(dr->max_batch);  // the cache's row stride
  const float eps = 1e-6f;
  const float* const* T = dr->t;
  // ---- context: H_ctx = RMSNorm(ctx_proj(the injection-layer outputs at the last n positions)),
  // projected here only for positions whose k/v rows are not cached yet (the plan's rows, compacted)
  const int Bg = B * g;
  if (c.n_inject > 0) {
    EVS_CHECK_ARG(s->cap_tag != nullptr, "state has no capture tags");
    EVS_CUDA_TRY(evs_launch(ctx_plan_kernel, dim3(1), dim3(1024), 0, st, true, static_cast<const int32_t*>(s->d_len), B,
                            CW, g, static_cast<const unsigned long long*>(s->cap_tag), s->ring_len,
                            static_cast<const int32_t*>(dr->cpos), static_cast<const unsigned long long*>(dr->ctag),
                            dr->cmap, dr->ccount));
    RingPtrs rg;
    for (int k = 0; k < 4; ++k) rg.p[k] = s->cap_ring[k];
    EVS_CHECK_ARG(H % 4 == 0, "target_hidden must be a multiple of 4");
    EVS_CUDA_TRY(evs_launch(gather_ctx_rows_kernel, dim3(B * CW), dim3(256), 0, st, true, rg, c.n_inject, s->ring_len,
                            H, static_cast<const int32_t*>(dr->cmap), static_cast<const int32_t*>(dr->ccount),
                            dr->ctx_in));
    DraftEpiArgs e = epi(T[EVS_D_CTX_B], dr->ctx, T[EVS_D_CTX_NORM], nullptr, nullptr, 1, eps);
    e.m_dev = dr->ccount;
    // grids for about two new context positions per row (a speculative round accepts k + 1)
    EVS_TRY(sgemm_epi(dr, T[EVS_D_CTX_W], dr->ctx_in, c.n_inject * H, d, c.n_inject * H, B * CW, EPI_BIAS_NORM, e,
                      st, std::min(B * CW, 2 * B + 16)));
  }
  // ---- h = in_proj(embed([anchor, MASK...])) + pos (rows of the token table), and the first
  // layer's pre-norm of h into xb ----
  const float* ln1_0 = c.n_layers > 0 ? T[EVS_D_LAYER0 + EVS_D_LN1] : T[EVS_D_FINAL_LN];
  {
    DraftEpiArgs e = epi(nullptr, dr->xb, ln1_0, dr->h, T[EVS_D_POS], g, eps);
    e.tok_in = dr->tok_in;
    e.anchor = anchor;
    e.mask_id = c.mask_id;
    e.M = rows;
    e.N = d;
    e.splits = 0;
    EVS_CUDA_TRY(evs_launch(draft_epi_kernel<EPI_TOK_IN_NORM>, dim3(rows), dim3(EPI_THREADS), sizeof(float) * d, st,
                            true, e));
  }
  for (int l = 0; l < c.n_layers; ++l) {
    const float* const* L = T + EVS_D_LAYER0 + l * EVS_D_PER_LAYER;
    // the norm after this layer's MLP: the next layer's pre-norm, or the final norm
    const float* next_ln = l + 1 < c.n_layers ? T[EVS_D_LAYER0 + (l + 1) * EVS_D_PER_LAYER + EVS_D_LN1] : T[EVS_D_FINAL_LN];
    // q, k and v in one launch (each its own rows: q the draft rows; k and v the draft rows, then
    // the context rows to project), then one reduction that also stores those context rows' k and
    // v in the cache
    const bool ctxr = c.n_inject > 0;
    const int kv_rows = ctxr ? Bg + B * CW : Bg;
    const int32_t* kv_m = ctxr ? dr->ccount + 1 : nullptr;
    const int kv_hint = ctxr ? std::min(kv_rows, Bg + 2 * B + 16) : 0;
    float* ckl = dr->ck + static_cast<size_t>(l) * B_cap * DR_CR * d;
    float* cvl = dr->cv + static_cast<size_t>(l) * B_cap * DR_CR * d;
    {
      const GemmPlan p = gemm_plan_f32_drafter(d, d, kv_rows);
      const size_t sq = static_cast<size_t>(p.splits) * Bg * d, skv = static_cast<size_t>(p.splits) * kv_rows * d;
      EVS_CHECK_RANGE(sq + 2 * skv <= dr->ws_floats, "drafter workspace too small");
      SkJobs jobs{};
      jobs.j[0] = SkJob{L[EVS_D_Q], dr->xb, nullptr, dr->ws, nullptr, Bg, Bg};
      jobs.j[1] = SkJob{L[EVS_D_K], dr->xb, dr->ctx, dr->ws + sq, kv_m, Bg, kv_rows};
      jobs.j[2] = SkJob{L[EVS_D_V], dr->xb, dr->ctx, dr->ws + sq + skv, kv_m, Bg, kv_rows};
      EVS_TRY(launch_gemm_simt_jobs(jobs, 3, d, p, st, true, kv_hint));
      QkvRed qr{};
      qr.ws[0] = dr->ws;
      qr.ws[1] = dr->ws + sq;
      qr.ws[2] = dr->ws + sq + skv;
      qr.out[0] = dr->q;
      qr.out[1] = dr->kb;
      qr.out[2] = dr->vb;
      qr.M[0] = Bg;
      qr.M[1] = qr.M[2] = kv_rows;
      const int red_rows = std::max(Bg, ctxr ? kv_hint : kv_rows);
      EVS_CUDA_TRY(evs_launch(qkv_reduce_kernel, dim3(blocks_for(static_cast<size_t>(red_rows) * d, 256), 3), dim3(256),
                              0, st, true, qr, p.splits, d, Bg, ctxr ? static_cast<const int32_t*>(dr->ccount) : nullptr,
                              static_cast<const int32_t*>(dr->cmap), ckl, cvl, static_cast<int>(l == c.n_layers - 1),
                              static_cast<const unsigned long long*>(s->cap_tag), s->ring_len, dr->cpos, dr->ctag));
      evs_count_launch(1);
    }
    const int hd = d / c.n_heads, nk = CW + g;
    const size_t rows_smem =
        sizeof(float) * ((static_cast<size_t>(nk) * (hd + 1) + 3) / 4 * 4 + static_cast<size_t>(nk) * hd + g * hd + nk);
    if (rows_smem <= 48 * 1024 && hd % 4 == 0 && d % 4 == 0) {
      // few rows: one CTA per query as well (the staging is repeated, the CTAs run side by side)
      const int qpc = B >= DRAFT_ATTN_ROWS_MIN_B ? g : 1;
      EVS_CUDA_TRY(evs_launch(draft_attn_rows_kernel, dim3(c.n_heads, B, (g + qpc - 1) / qpc), dim3(128), rows_smem,
                              st, true, static_cast<const float*>(dr->q), static_cast<const float*>(dr->kb),
                              static_cast<const float*>(dr->vb), static_cast<const float*>(ckl),
                              static_cast<const float*>(cvl), static_cast<const int32_t*>(s->d_len),
                              static_cast<int>(ctxr), CW, g, d, c.n_heads, qpc, dr->y));
    } else {
      EVS_CUDA_TRY(evs_launch(draft_attn_kernel, dim3(dim3(g, c.n_heads, B)), dim3(128), 0, st, true,
                              static_cast<const float*>(dr->q), static_cast<const float*>(dr->kb),
                              static_cast<const float*>(dr->vb), static_cast<const float*>(ckl),
                              static_cast<const float*>(cvl), static_cast<const int32_t*>(s->d_len),
                              static_cast<int>(ctxr), CW, g, d, c.n_heads, dr->y));
    }
    // h += out_proj(y); xb = pre-MLP norm of h
    EVS_TRY(sgemm_epi(dr, L[EVS_D_O], dr->y, d, d, d, rows, EPI_RESID_NORM,
                      epi(nullptr, dr->xb, L[EVS_D_LN2], dr->h, nullptr, 1, eps), st));
    EVS_TRY(sgemm_epi(dr, L[EVS_D_MLP0_W], dr->xb, d, hid, d, rows, EPI_BIAS_SILU, epi(L[EVS_D_MLP0_B], dr->m1), st));
    // h += mlp2(m1) + bias; xb = next pre-norm (the final norm after the last layer)
    EVS_TRY(sgemm_epi(dr, L[EVS_D_MLP2_W], dr->m1, hid, d, hid, rows, EPI_RESID_NORM,
                      epi(L[EVS_D_MLP2_B], dr->xb, next_ln, dr->h, nullptr, 1, eps), st));
  }
  // ---- U = (final_ln(h) out_proj) embedᵀ H^-1/2 (xb holds final_ln(h)) ----
  EVS_TRY(sgemm_epi(dr, T[EVS_D_OUT_W], dr->xb, d, H, d, rows, EPI_BIAS, epi(T[EVS_D_OUT_B], dr->z), st));
  EVS_TRY(sgemm_epi(dr, T[EVS_D_EMBED], dr->z, H, V, H, rows, EPI_SCALE,
                    epi(nullptr, dr->U, nullptr, nullptr, nullptr, 1, eps, 1.0f / sqrtf(static_cast<float>(H))), st));
  // ---- serial Markov head ----
  if ((V == 512 || V == 256 || V == 128) && g <= EVS_RETAIN_MAX) {  // per-step inputs held in shared memory
    auto head = V == 512 ? serial_head_warp_kernel<4> : (V == 256 ? serial_head_warp_kernel<2> : serial_head_warp_kernel<1>);
    EVS_CUDA_TRY(evs_launch(head, dim3(B), dim3(128), 0, st, true, dr->U, T[EVS_D_MARKOV], anchor, g, greedy,
                            temperature, top_k, u, forced, tokens, qrows, dr->prev));
  } else {
    EVS_CUDA_TRY(evs_launch(serial_head_kernel, dim3(B), dim3(256), 0, st, true, dr->U, T[EVS_D_MARKOV], anchor, g, V,
                            greedy, temperature, top_k, u, forced, tokens, qrows, dr->prev));
  }
  // ---- confidence: σ(conf_w [final_ln(h) ; in_proj(embed(prev))]), the second half from the table ----
  EVS_CUDA_TRY(evs_launch(conf_kernel, dim3(blocks_for(rows, 4)), dim3(128), 0, st, true, dr->xb, dr->tok_in, dr->prev,
                          T[EVS_D_CONF_W], T[EVS_D_CONF_B], d, rows, conf));
  // kernels of this call that count nowhere else (projections, their fused epilogues and the q/k/v
  // reduction count themselves): context plan + gather, draft rows, attention per layer, serial
  // head, conf
  evs_count_launch((c.n_inject > 0 ? 2 : 0) + 1 + c.n_layers + 2);
  if (U_out != nullptr)
    EVS_CUDA_TRY(cudaMemcpyAsync(U_out, dr->U, sizeof(float) * rows * V, cudaMemcpyDeviceToDevice, st));
  EVS_CUDA_TRY(cudaGetLastError());
  return EVS_OK;
}

}  // extern "C"
