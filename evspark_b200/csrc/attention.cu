// Causal multi-head attention of T new queries per row over the KV cache (vortex layout
// [B, Lmax, 2, H, Dh]), bottom-right aligned: query t of row b sits at absolute position
// P = len[b] + t and sees keys 0..P (evspark/specdec/block/chunk.py:34-35; the reference reaches
// flash_attn_with_kvcache through the model forward).
//
//   rope_append_kernel   qkv partials -> rotate-half RoPE (fp64 angle) -> q_rot, K/V cache append
//   attn_block_kernel    one CTA per (256-key block, head, row): partial (max, sum, acc) per query
//   attn_combine_kernel  folds the partials of blocks 0..P/256 in block order
//
// Blocks are aligned at absolute key positions and folded in a fixed order, so a query's result
// does not depend on how many other queries share the call (native T=1 == verify T=γ+1).
#include <math_constants.h>

#include "internal.hpp"

namespace {

template <typename TD>
__global__ void rope_append_kernel(const float* __restrict__ ws, int splits, int M, int T, int d, int H, int Dh,
                                   double log_base, const int32_t* __restrict__ len, int Lmax, TD* __restrict__ qrot,
                                   TD* __restrict__ kv, EvsDevErr* err) {
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
    float acc = 0.f;
    for (int sp = 0; sp < splits; ++sp) acc += ws[(static_cast<size_t>(sp) * M + row) * N + c];
    return round_to<TD>(acc);
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

constexpr int QG = 8;  // queries per score pass

// grid (blocks, H, B); 256 threads; smem: q[T][Dh] + S[T][256] + stats[2T]
template <typename TD>
__global__ void __launch_bounds__(256) attn_block_kernel(const TD* __restrict__ qrot, const TD* __restrict__ kv,
                                                        const int32_t* __restrict__ len, int T, int d, int H, int Dh,
                                                        int Lmax, int nblk_cap, int tcap, float scale,
                                                        float* __restrict__ part) {
  extern __shared__ float sm[];
  const int j = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int L0 = len[b];
  const int Lend = L0 + T;
  const int k0 = j * ATTN_BLOCK;
  if (k0 >= Lend) return;
  const int nk = min(ATTN_BLOCK, Lend - k0);
  float* qs = sm;                 // [T][Dh]
  float* S = qs + T * Dh;         // [T][ATTN_BLOCK]
  float* st = S + T * ATTN_BLOCK; // [T][2]
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  for (int i = tid; i < T * Dh; i += blockDim.x) {
    const int t = i / Dh, dd = i % Dh;
    qs[i] = to_f32(qrot[static_cast<size_t>(b * T + t) * d + h * Dh + dd]);
  }
  __syncthreads();
  const size_t HD = static_cast<size_t>(H) * Dh;
  if (tid < nk) {
    const int kk = k0 + tid;
    const TD* kp = kv + ((static_cast<size_t>(b) * Lmax + kk) * 2 + 0) * HD + h * Dh;
    for (int tg = 0; tg < T; tg += QG) {
      float acc[QG];
#pragma unroll
      for (int u = 0; u < QG; ++u) acc[u] = 0.f;
      for (int dd = 0; dd < Dh; ++dd) {
        const float kvv = to_f32(kp[dd]);
#pragma unroll
        for (int u = 0; u < QG; ++u)
          if (tg + u < T) acc[u] = fmaf(qs[(tg + u) * Dh + dd], kvv, acc[u]);
      }
#pragma unroll
      for (int u = 0; u < QG; ++u) {
        const int t = tg + u;
        if (t < T) S[t * ATTN_BLOCK + tid] = kk <= L0 + t ? acc[u] * scale : -CUDART_INF_F;
      }
    }
  }
  __syncthreads();
  for (int t = warp; t < T; t += blockDim.x / 32) {
    float m = -CUDART_INF_F;
    for (int i = lane; i < nk; i += 32) m = fmaxf(m, S[t * ATTN_BLOCK + i]);
    m = warp_max(m);
    float l = 0.f;
    for (int i = lane; i < nk; i += 32) {
      const float sv = S[t * ATTN_BLOCK + i];
      const float pv = (m == -CUDART_INF_F || sv == -CUDART_INF_F) ? 0.f : expf(sv - m);
      S[t * ATTN_BLOCK + i] = pv;
      l += pv;
    }
    l = warp_sum(l);
    if (lane == 0) {
      st[2 * t] = m;
      st[2 * t + 1] = l;
    }
  }
  __syncthreads();
  const int groups = blockDim.x / Dh;
  const int dd = tid % Dh, g = tid / Dh;
  if (g < groups) {
    for (int t = g; t < T; t += groups) {
      float acc = 0.f;
      for (int i = 0; i < nk; ++i) {
        const TD* vp = kv + ((static_cast<size_t>(b) * Lmax + k0 + i) * 2 + 1) * HD + h * Dh;
        acc = fmaf(S[t * ATTN_BLOCK + i], to_f32(vp[dd]), acc);
      }
      float* pd = part + ((((static_cast<size_t>(b) * H + h) * nblk_cap + j) * tcap + t) * (Dh + 2));
      pd[dd] = acc;
      if (dd == 0) {
        pd[Dh] = st[2 * t];
        pd[Dh + 1] = st[2 * t + 1];
      }
    }
  }
}

template <typename TD>
__global__ void attn_combine_kernel(const float* __restrict__ part, const int32_t* __restrict__ len, int T, int d,
                                    int H, int Dh, int nblk_cap, int tcap, TD* __restrict__ out, int ld_out) {
  const int row = blockIdx.x, h = blockIdx.y, dd = threadIdx.x;
  if (dd >= Dh) return;
  const int b = row / T, t = row % T;
  const int P = len[b] + t;
  const int jmax = P / ATTN_BLOCK;
  float m = -CUDART_INF_F, l = 0.f, acc = 0.f;
  for (int j = 0; j <= jmax; ++j) {
    const float* pj = part + ((((static_cast<size_t>(b) * H + h) * nblk_cap + j) * tcap + t) * (Dh + 2));
    const float mj = pj[Dh];
    if (mj == -CUDART_INF_F) continue;
    const float mn = fmaxf(m, mj);
    const float a = m == -CUDART_INF_F ? 0.f : expf(m - mn);
    const float bj = expf(mj - mn);
    l = l * a + pj[Dh + 1] * bj;
    acc = acc * a + pj[dd] * bj;
    m = mn;
  }
  out[static_cast<size_t>(row) * ld_out + h * Dh + dd] = from_f32<TD>(acc / l);
}

template <typename TD>
int launch_attention_t(const evs_model* m, evs_state* s, int layer, int B, int T, int splits, int kv_blocks,
                       cudaStream_t st) {
  const int d = m->cfg.d_model, H = m->cfg.n_heads, Dh = m->cfg.head_dim;
  const int M = B * T;
  TD* kv = static_cast<TD*>(s->kv[layer]);
  TD* qrot = static_cast<TD*>(s->qrot);
  rope_append_kernel<TD><<<dim3(M, H), Dh / 2, 0, st>>>(s->ws, splits, M, T, d, H, Dh, log(m->cfg.rope_base),
                                                        s->d_len, s->max_seqlen, qrot, kv, s->d_err);
  EVS_CUDA_TRY(cudaGetLastError());
  const size_t smem = sizeof(float) * (static_cast<size_t>(T) * Dh + static_cast<size_t>(T) * ATTN_BLOCK + 2 * T);
  EVS_CHECK_RANGE(smem <= 200 * 1024, "too many queries per attention call");
  EVS_CUDA_TRY(cudaFuncSetAttribute(attn_block_kernel<TD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    static_cast<int>(smem)));
  attn_block_kernel<TD><<<dim3(kv_blocks, H, B), 256, smem, st>>>(
      qrot, kv, s->d_len, T, d, H, Dh, s->max_seqlen, s->attn_blocks, s->max_chunk, 1.0f / sqrtf(static_cast<float>(Dh)),
      s->attn_part);
  EVS_CUDA_TRY(cudaGetLastError());
  attn_combine_kernel<TD><<<dim3(M, H), Dh, 0, st>>>(s->attn_part, s->d_len, T, d, H, Dh, s->attn_blocks,
                                                     s->max_chunk, static_cast<TD*>(s->act), s->ld_act);
  EVS_CUDA_TRY(cudaGetLastError());
  evs_count_launch(3);
  return EVS_OK;
}

}  // namespace

int launch_attention(const evs_model* m, evs_state* s, int layer, int B, int T, int splits, int kv_blocks,
                     cudaStream_t st) {
  EVS_CHECK_ARG(m->cfg.head_dim % 2 == 0 && m->cfg.head_dim <= 256 && 256 % m->cfg.head_dim == 0,
                "head_dim must divide 256");
  EVS_CHECK_RANGE(kv_blocks >= 1 && kv_blocks <= s->attn_blocks, "KV length beyond max_seqlen");
  if (m->cfg.dtype == EVS_DTYPE_BF16) return launch_attention_t<__nv_bfloat16>(m, s, layer, B, T, splits, kv_blocks, st);
  return launch_attention_t<float>(m, s, layer, B, T, splits, kv_blocks, st);
}
