// Hyena mixer of one layer for a chunk of T tokens per row, fused end to end:
//   in-projection partials (split-K, fixed order) -> data-dtype u [T, 3d]
//   -> outer causal FIR (K0 = 3) over all 3d channels with the carried history
//   -> de-interleave (channel 3h+j -> group j) into x2, x1, v;  x1v = x1 * v
//   -> inner FIR (SE: K=7 unflipped; MR: K=128 flipped + gated bias D·x1v)  [hyena_fir_kernel]
//      or modal IIR s_t = p∘s_{t-1} + x1v_t, y = x2∘(Σ R s_t + D x1v_t)      [hyena_iir_kernel]
// (evspark/specdec/block/chunk.py:162-295).
//
// Tap rule of the step path (chunk.py:88-125): with c = min(P, K-1) inputs of history at
// absolute position P, an unflipped filter weights the input of age a by w[c - a], a flipped
// one by w[a].  Prefill (zero-padded parallel convolution) uses w[K-1-a] for unflipped filters.
//
// State never moves on rollback: FIR inputs live in per-row rings indexed by absolute position
// (slot = P mod cap), IIR states in per-position slots; evs_rollback only rewrites lengths.
#include "internal.hpp"

namespace {

constexpr int CH = 32;  // channels per CTA

template <typename TD>
struct HyArgs {
  const float* ws;
  int splits, M, T, d;
  TD* outer_ring;
  int cap_o;
  const float* short_w;
  int K0;
  TD* inner_ring;
  int cap_i;
  const float* inner_w;
  int K;
  const float* D;
  const float* poles;
  const float* residues;
  float* s_all;
  int S, slots;
  const int32_t* len;
  const int32_t* iir_cur;
  int prefill, retain;
  TD* y;
  int ld_y;
};

// data-dtype value of the in-projection output (channel c of a token row)
template <typename TD>
__device__ __forceinline__ float u_chunk(const HyArgs<TD>& a, int row, int c) {
  float acc = 0.f;
  for (int sp = 0; sp < a.splits; ++sp) acc += a.ws[(static_cast<size_t>(sp) * a.M + row) * (3 * a.d) + c];
  return round_to<TD>(acc);
}

// outer-FIR input at absolute position P of row b (inside the chunk or in the ring)
template <typename TD>
__device__ __forceinline__ float u_at(const HyArgs<TD>& a, int b, int L0, int P, int c) {
  if (P >= L0) return u_chunk(a, b * a.T + (P - L0), c);
  return to_f32(a.outer_ring[(static_cast<size_t>(b) * a.cap_o + (P % a.cap_o)) * (3 * a.d) + c]);
}

// outer FIR (unflipped, K0 taps) for channel c at absolute position P
template <typename TD>
__device__ __forceinline__ float outer_fir(const HyArgs<TD>& a, int b, int L0, int P, int c, float u_now) {
  const int K0 = a.K0;
  const int cs = min(P, K0 - 1);
  const int base = a.prefill ? K0 - 1 : cs;
  const float* w = a.short_w + static_cast<size_t>(c) * K0;
  float z = 0.f;
  for (int age = cs; age >= 1; --age) z = fmaf(w[base - age], u_at(a, b, L0, P - age, c), z);
  return fmaf(w[base], u_now, z);
}

// grid (d / 32, B); 128 threads; dynamic smem: hist[(K-1)+T][32] + x2[T][32] + taps[K][32]
template <typename TD, bool FLIP>
__global__ void __launch_bounds__(128) hyena_fir_kernel(HyArgs<TD> a) {
  extern __shared__ float sm[];
  const int K = a.K, T = a.T, H = K - 1;
  float* hist = sm;                  // [(H + T)][CH]
  float* x2s = hist + (H + T) * CH;  // [T][CH]
  float* taps = x2s + T * CH;        // [K][CH]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h0 = blockIdx.x * CH, b = blockIdx.y;
  const int h = h0 + lane;
  const int L0 = a.len[b];

  // history window of x1v (positions L0-H .. L0-1) and taps, transposed to [*][channel]
  for (int i = threadIdx.x; i < H * CH; i += blockDim.x) {
    const int r = i / CH, cc = i % CH;
    const int P = L0 - H + r;
    hist[r * CH + cc] =
        P >= 0 ? to_f32(a.inner_ring[(static_cast<size_t>(b) * a.cap_i + (P % a.cap_i)) * a.d + h0 + cc]) : 0.f;
  }
  for (int i = threadIdx.x; i < K * CH; i += blockDim.x) {
    const int cc = i / K, j = i % K;
    taps[j * CH + cc] = a.inner_w[static_cast<size_t>(h0 + cc) * K + j];
  }
  // phase 1: outer FIR, de-interleave, x1v for every chunk position
  for (int t = warp; t < T; t += 4) {
    const int P = L0 + t, row = b * T + t;
    float zq[3];
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      const int c = 3 * h + j;
      const float un = u_chunk(a, row, c);
      a.outer_ring[(static_cast<size_t>(b) * a.cap_o + (P % a.cap_o)) * (3 * a.d) + c] = from_f32<TD>(un);
      zq[j] = round_to<TD>(outer_fir(a, b, L0, P, c, un));
    }
    const float x1v = round_to<TD>(zq[1] * zq[2]);
    hist[(H + t) * CH + lane] = x1v;
    x2s[t * CH + lane] = zq[0];
    a.inner_ring[(static_cast<size_t>(b) * a.cap_i + (P % a.cap_i)) * a.d + h] = from_f32<TD>(x1v);
  }
  __syncthreads();
  // phase 2: inner FIR over [history | chunk]
  const float Dh = FLIP ? a.D[h] : 0.f;
  for (int t = warp; t < T; t += 4) {
    const int P = L0 + t;
    const int cs = min(P, H);
    float z = 0.f;
    if (FLIP) {
      for (int age = cs; age >= 0; --age) z = fmaf(taps[age * CH + lane], hist[(H + t - age) * CH + lane], z);
      z = fmaf(Dh, hist[(H + t) * CH + lane], z);
    } else {
      const int base = a.prefill ? H : cs;
      for (int age = cs; age >= 0; --age)
        z = fmaf(taps[(base - age) * CH + lane], hist[(H + t - age) * CH + lane], z);
    }
    const float yv = round_to<TD>(x2s[t * CH + lane] * round_to<TD>(z));
    a.y[static_cast<size_t>(b * T + t) * a.ld_y + h] = from_f32<TD>(yv);
  }
}

// grid (d / 32, B); 128 threads = 32 channels x 4 pole groups (S / 4 poles each)
template <typename TD, int SPT>
__global__ void __launch_bounds__(128) hyena_iir_kernel(HyArgs<TD> a) {
  const int q = threadIdx.x & 3;
  const int h = blockIdx.x * CH + (threadIdx.x >> 2);
  const int b = blockIdx.y;
  const int T = a.T, S = a.S, d = a.d;
  const int L0 = a.len[b];
  float p[SPT], r[SPT], s[SPT];
  const float* src = a.s_all + ((static_cast<size_t>(b) * a.slots + a.iir_cur[b]) * d + h) * S + q * SPT;
#pragma unroll
  for (int j = 0; j < SPT; ++j) {
    p[j] = a.poles[static_cast<size_t>(h) * S + q * SPT + j];
    r[j] = a.residues[static_cast<size_t>(h) * S + q * SPT + j];
    s[j] = L0 > 0 ? src[j] : 0.f;
  }
  const float Dh = a.D[h];
  for (int t = 0; t < T; ++t) {
    const int P = L0 + t, row = b * T + t;
    float zq[3];
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      const int c = 3 * h + j;
      const float un = u_chunk(a, row, c);
      if (q == 0)
        a.outer_ring[(static_cast<size_t>(b) * a.cap_o + (P % a.cap_o)) * (3 * d) + c] = from_f32<TD>(un);
      zq[j] = round_to<TD>(outer_fir(a, b, L0, P, c, un));
    }
    const float x1v = round_to<TD>(zq[1] * zq[2]);
    float part = 0.f;
#pragma unroll
    for (int j = 0; j < SPT; ++j) {
      s[j] = fmaf(p[j], s[j], x1v);
      part = fmaf(r[j], s[j], part);
    }
    part += __shfl_xor_sync(0xffffffffu, part, 1);
    part += __shfl_xor_sync(0xffffffffu, part, 2);
    if (q == 0) {
      const float yv = round_to<TD>(zq[0] * (part + Dh * x1v));
      a.y[static_cast<size_t>(row) * a.ld_y + h] = from_f32<TD>(yv);
    }
    if (a.retain) {
      float* dst = a.s_all + ((static_cast<size_t>(b) * a.slots + t) * d + h) * S + q * SPT;
#pragma unroll
      for (int j = 0; j < SPT; ++j) dst[j] = s[j];
    }
  }
  if (!a.retain) {
    // final state into slot 0 (this thread read its old slot before writing anything)
    float* dst = a.s_all + ((static_cast<size_t>(b) * a.slots + 0) * d + h) * S + q * SPT;
#pragma unroll
    for (int j = 0; j < SPT; ++j) dst[j] = s[j];
  }
}

__global__ void rollback_kernel(int32_t* len, const int32_t* len0, int32_t* iir_cur, const int32_t* chunk,
                                const int32_t* k, int B, EvsDevErr* err) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  const int kk = k[b], c = chunk[0];
  if (c <= 0 || kk < 0 || kk >= c) {
    evs_record_error(err, EVS_ERANGE, EVS_K_HYENA, b);
    return;
  }
  len[b] = len0[b] + kk + 1;
  iir_cur[b] = kk;
}

template <typename TD>
__global__ void export_ring_kernel(const TD* ring, int cap, int C, int row, const int32_t* len, int width,
                                   float* dst) {
  const int L = len[row];
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < C * width; i += gridDim.x * blockDim.x) {
    const int c = i / width, j = i % width;
    const int P = L - width + j;
    dst[i] = P >= 0 ? to_f32(ring[(static_cast<size_t>(row) * cap + (P % cap)) * C + c]) : 0.f;
  }
}

__global__ void export_iir_kernel(const float* s_all, int slots, int d, int S, int row, const int32_t* iir_cur,
                                  const int32_t* len, float* dst) {
  const int cur = iir_cur[row];
  const bool empty = len[row] == 0;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < d * S; i += gridDim.x * blockDim.x)
    dst[i] = empty ? 0.f : s_all[(static_cast<size_t>(row) * slots + cur) * d * S + i];
}

template <typename TD>
__global__ void export_kv_kernel(const TD* kv, int Lmax, int HD2, int row, const int32_t* len, int width, TD* dst) {
  const int L = len[row];
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < width * HD2; i += gridDim.x * blockDim.x) {
    const int j = i / HD2, e = i % HD2;
    const int P = L - width + j;
    dst[i] = P >= 0 ? kv[(static_cast<size_t>(row) * Lmax + P) * HD2 + e] : from_f32<TD>(0.f);
  }
}

template <typename TD>
int launch_hyena_t(const evs_model* m, evs_state* s, int layer, int B, int T, int splits, int prefill, int retain,
                   cudaStream_t st) {
  const LayerDev& L = m->L[layer];
  const HyenaDev& hy = s->hy[layer];
  const int d = m->cfg.d_model;
  HyArgs<TD> a;
  a.ws = s->ws;
  a.splits = splits;
  a.M = B * T;
  a.T = T;
  a.d = d;
  a.outer_ring = static_cast<TD*>(hy.outer_ring);
  a.cap_o = s->cap_outer;
  a.short_w = static_cast<const float*>(L.short_w);
  a.K0 = m->cfg.short_filter_length;
  a.inner_ring = static_cast<TD*>(hy.inner_ring);
  a.cap_i = L.kind == EVS_LAYER_HCM ? s->cap_hcm : s->cap_hcs;
  a.inner_w = static_cast<const float*>(L.inner_w);
  a.K = L.kind == EVS_LAYER_HCM ? m->cfg.hcm_filter_length : m->cfg.hcs_filter_length;
  a.D = static_cast<const float*>(L.D);
  a.poles = L.poles;
  a.residues = static_cast<const float*>(L.residues);
  a.s_all = hy.s_all;
  a.S = m->cfg.state_size;
  a.slots = s->iir_slots;
  a.len = s->d_len;
  a.iir_cur = s->d_iir_cur;
  a.prefill = prefill;
  a.retain = retain;
  a.y = static_cast<TD*>(s->act);
  a.ld_y = s->ld_act;
  dim3 grid(d / CH, B);
  if (L.kind == EVS_LAYER_HCL) {
    switch (a.S / 4) {
      case 4: hyena_iir_kernel<TD, 4><<<grid, 128, 0, st>>>(a); break;
      case 8: hyena_iir_kernel<TD, 8><<<grid, 128, 0, st>>>(a); break;
      case 2: hyena_iir_kernel<TD, 2><<<grid, 128, 0, st>>>(a); break;
      case 1: hyena_iir_kernel<TD, 1><<<grid, 128, 0, st>>>(a); break;
      default: EVS_CHECK_ARG(false, "state_size must be 4, 8, 16 or 32");
    }
  } else {
    const size_t smem = sizeof(float) * (static_cast<size_t>(a.K - 1 + T) * CH + T * CH + a.K * CH);
    EVS_CHECK_RANGE(smem <= 200 * 1024, "chunk too long for the FIR shared-memory window");
    if (L.kind == EVS_LAYER_HCM) {
      EVS_CUDA_TRY(cudaFuncSetAttribute(hyena_fir_kernel<TD, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        static_cast<int>(smem)));
      hyena_fir_kernel<TD, true><<<grid, 128, smem, st>>>(a);
    } else {
      EVS_CUDA_TRY(cudaFuncSetAttribute(hyena_fir_kernel<TD, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        static_cast<int>(smem)));
      hyena_fir_kernel<TD, false><<<grid, 128, smem, st>>>(a);
    }
  }
  EVS_CUDA_TRY(cudaGetLastError());
  evs_count_launch(1);
  return EVS_OK;
}

}  // namespace

int launch_hyena(const evs_model* m, evs_state* s, int layer, int B, int T, int splits, int prefill, int retain,
                 cudaStream_t st) {
  EVS_CHECK_ARG(m->cfg.d_model % CH == 0, "d_model must be a multiple of 32");
  if (m->cfg.dtype == EVS_DTYPE_BF16)
    return launch_hyena_t<__nv_bfloat16>(m, s, layer, B, T, splits, prefill, retain, st);
  return launch_hyena_t<float>(m, s, layer, B, T, splits, prefill, retain, st);
}

int launch_rollback(evs_state* s, const int32_t* k, int B, cudaStream_t st) {
  rollback_kernel<<<(B + 127) / 128, 128, 0, st>>>(s->d_len, s->d_len0, s->d_iir_cur, s->d_chunk, k, B, s->d_err);
  EVS_CUDA_TRY(cudaGetLastError());
  evs_count_launch(1);
  return EVS_OK;
}

int launch_state_export(const evs_state* s, int layer, int which, int row, int width, void* dst, cudaStream_t st) {
  const evs_model* m = s->m;
  const int d = m->cfg.d_model;
  const HyenaDev& hy = s->hy[layer];
  const bool bf = m->cfg.dtype == EVS_DTYPE_BF16;
  if (which == 0 || which == 1) {
    const void* ring = which == 0 ? hy.outer_ring : hy.inner_ring;
    const int cap = which == 0 ? s->cap_outer : (m->L[layer].kind == EVS_LAYER_HCM ? s->cap_hcm : s->cap_hcs);
    const int C = which == 0 ? 3 * d : d;
    EVS_CHECK_ARG(ring != nullptr, "layer has no such FIR state");
    float* out = static_cast<float*>(dst);
    if (bf)
      export_ring_kernel<__nv_bfloat16><<<64, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(ring), cap, C, row,
                                                            s->d_len, width, out);
    else
      export_ring_kernel<float><<<64, 256, 0, st>>>(static_cast<const float*>(ring), cap, C, row, s->d_len, width,
                                                    out);
  } else if (which == 2) {
    EVS_CHECK_ARG(hy.s_all != nullptr, "layer has no IIR state");
    export_iir_kernel<<<64, 256, 0, st>>>(hy.s_all, s->iir_slots, d, m->cfg.state_size, row, s->d_iir_cur,
                                          s->d_len, static_cast<float*>(dst));
  } else if (which == 3) {
    EVS_CHECK_ARG(s->kv[layer] != nullptr, "layer has no KV cache");
    const int HD2 = 2 * m->cfg.n_heads * m->cfg.head_dim;
    if (bf)
      export_kv_kernel<__nv_bfloat16><<<64, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(s->kv[layer]),
                                                          s->max_seqlen, HD2, row, s->d_len, width,
                                                          static_cast<__nv_bfloat16*>(dst));
    else
      export_kv_kernel<float><<<64, 256, 0, st>>>(static_cast<const float*>(s->kv[layer]), s->max_seqlen, HD2, row,
                                                  s->d_len, width, static_cast<float*>(dst));
  } else {
    EVS_CHECK_ARG(false, "unknown export kind");
  }
  EVS_CUDA_TRY(cudaGetLastError());
  evs_count_launch(1);
  return EVS_OK;
}
