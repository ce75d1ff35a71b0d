// Row-wise kernels between the GEMMs: embedding + pre-norm, split-K reduction + residual
// add + RMSNorm (+ drafter-context capture), SwiGLU gating, logits, per-row bookkeeping.
// Every reduction runs in a fixed order that does not depend on the number of token rows.
#include "internal.hpp"

namespace {

constexpr int ROW_THREADS = 256;

// sum over the block in a fixed order (per-thread strided partial -> butterfly -> warps in order)
__device__ float block_sum_fixed(float v, float* red) {
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (threadIdx.x == 0) {
    float s = 0.f;
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) s += red[w];
    red[32] = s;
  }
  __syncthreads();
  const float out = red[32];
  __syncthreads();
  return out;
}

template <typename TD>
__global__ void __launch_bounds__(ROW_THREADS) embed_norm_kernel(const int64_t* __restrict__ ids,
                                                                 const TD* __restrict__ embed,
                                                                 const float* __restrict__ scale,
                                                                 float* __restrict__ resid, TD* __restrict__ act,
                                                                 int ld_act, int d, int V, float eps,
                                                                 EvsDevErr* err) {
  __shared__ float red[33];
  const int row = blockIdx.x;
  int64_t id = ids[row];
  if (id < 0 || id >= V) {
    if (threadIdx.x == 0) evs_record_error(err, EVS_ERANGE, EVS_K_ROW, row);
    id = 0;
  }
  float ss = 0.f;
  for (int c = threadIdx.x; c < d; c += ROW_THREADS) {
    const float v = to_f32(embed[id * d + c]);
    resid[static_cast<size_t>(row) * d + c] = v;
    ss = fmaf(v, v, ss);
  }
  ss = block_sum_fixed(ss, red);
  const float inv = 1.0f / sqrtf(ss / static_cast<float>(d) + eps);
  for (int c = threadIdx.x; c < d; c += ROW_THREADS) {
    const float v = resid[static_cast<size_t>(row) * d + c];
    act[static_cast<size_t>(row) * ld_act + c] = from_f32<TD>(v * inv * scale[c]);
  }
}

template <typename TD>
__global__ void __launch_bounds__(ROW_THREADS) res_add_norm_kernel(
    const float* __restrict__ ws, int splits, int M, float* __restrict__ resid, const float* __restrict__ scale,
    TD* __restrict__ act, int ld_act, int d, float eps, float* __restrict__ ring, int ring_len,
    const int32_t* __restrict__ len, int T) {
  __shared__ float red[33];
  const int row = blockIdx.x;
  const int b = row / T, t = row % T;
  float* cap = nullptr;
  if (ring != nullptr && t >= T - ring_len) {
    const int P = len[b] + t;
    cap = ring + (static_cast<size_t>(b) * ring_len + P % ring_len) * d;
  }
  float ss = 0.f;
  for (int c = threadIdx.x; c < d; c += ROW_THREADS) {
    float acc = 0.f;
    for (int sp = 0; sp < splits; ++sp) acc += ws[(static_cast<size_t>(sp) * M + row) * d + c];
    const float v = resid[static_cast<size_t>(row) * d + c] + acc;
    resid[static_cast<size_t>(row) * d + c] = v;
    if (cap != nullptr) cap[c] = v;
    ss = fmaf(v, v, ss);
  }
  ss = block_sum_fixed(ss, red);
  const float inv = 1.0f / sqrtf(ss / static_cast<float>(d) + eps);
  for (int c = threadIdx.x; c < d; c += ROW_THREADS) {
    const float v = resid[static_cast<size_t>(row) * d + c];
    act[static_cast<size_t>(row) * ld_act + c] = from_f32<TD>(v * inv * scale[c]);
  }
}

// ws holds the dual GEMM: virtual row (f / 64) * 128 + j * 64 + f % 64 is w_{j+1} feature f
template <typename TD>
__global__ void __launch_bounds__(ROW_THREADS) swiglu_kernel(const float* __restrict__ ws, int splits, int M, int F,
                                                            TD* __restrict__ act, int ld_act) {
  const int row = blockIdx.y;
  const int f = blockIdx.x * ROW_THREADS + threadIdx.x;
  if (f >= F) return;
  const int N2 = 2 * F;
  const int v1 = (f / 64) * 128 + (f % 64), v2 = v1 + 64;
  float g1 = 0.f, g2 = 0.f;
  for (int sp = 0; sp < splits; ++sp) {
    const float* r = ws + (static_cast<size_t>(sp) * M + row) * N2;
    g1 += r[v1];
    g2 += r[v2];
  }
  const float sig = 1.0f / (1.0f + expf(-g1));
  act[static_cast<size_t>(row) * ld_act + f] = from_f32<TD>(g1 * sig * g2);
}

__global__ void logits_kernel(const float* __restrict__ ws, int splits, int M, int V, int T, int out_T, int t0,
                              int last_only, float* __restrict__ out) {
  const int row = blockIdx.y;
  const int v = blockIdx.x * blockDim.x + threadIdx.x;
  if (v >= V) return;
  const int t = row % T;
  if (last_only && t != T - 1) return;
  float acc = 0.f;
  for (int sp = 0; sp < splits; ++sp) acc += ws[(static_cast<size_t>(sp) * M + row) * V + v];
  const int b = row / T;
  const size_t orow = last_only ? static_cast<size_t>(b) : static_cast<size_t>(b) * out_T + t0 + t;
  out[orow * V + v] = acc;
}

__global__ void bookkeeping_kernel(int32_t* len, int32_t* len0, int32_t* iir_cur, int32_t* chunk, int B, int T,
                                   int retain) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b < B) {
    const int old = len[b];
    len0[b] = old;
    len[b] = old + T;
    iir_cur[b] = retain ? T - 1 : 0;
  }
  if (b == 0) chunk[0] = retain ? T : 0;
}

__global__ void poles_kernel(const float* lp, float* p, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) p[i] = expf(lp[i]);
}

}  // namespace

int launch_embed_norm(const evs_model* m, evs_state* s, const int64_t* ids, int M, const float* scale,
                      cudaStream_t st) {
  const int d = m->cfg.d_model;
  if (m->cfg.dtype == EVS_DTYPE_BF16)
    embed_norm_kernel<__nv_bfloat16><<<M, ROW_THREADS, 0, st>>>(
        ids, static_cast<const __nv_bfloat16*>(m->embed), scale, s->resid, static_cast<__nv_bfloat16*>(s->act),
        s->ld_act, d, m->cfg.vocab_size, m->cfg.eps, s->d_err);
  else
    embed_norm_kernel<float><<<M, ROW_THREADS, 0, st>>>(ids, static_cast<const float*>(m->embed), scale, s->resid,
                                                        static_cast<float*>(s->act), s->ld_act, d,
                                                        m->cfg.vocab_size, m->cfg.eps, s->d_err);
  EVS_CUDA_TRY(cudaGetLastError());
  evs_count_launch(1);
  return EVS_OK;
}

int launch_res_add_norm(const evs_model* m, evs_state* s, int M, int splits, const float* scale, int capture_slot,
                        int T, cudaStream_t st) {
  const int d = m->cfg.d_model;
  float* ring = capture_slot >= 0 ? s->cap_ring[capture_slot] : nullptr;
  if (m->cfg.dtype == EVS_DTYPE_BF16)
    res_add_norm_kernel<__nv_bfloat16><<<M, ROW_THREADS, 0, st>>>(
        s->ws, splits, M, s->resid, scale, static_cast<__nv_bfloat16*>(s->act), s->ld_act, d, m->cfg.eps, ring,
        s->ring_len, s->d_len, T);
  else
    res_add_norm_kernel<float><<<M, ROW_THREADS, 0, st>>>(s->ws, splits, M, s->resid, scale,
                                                          static_cast<float*>(s->act), s->ld_act, d, m->cfg.eps,
                                                          ring, s->ring_len, s->d_len, T);
  EVS_CUDA_TRY(cudaGetLastError());
  evs_count_launch(1);
  return EVS_OK;
}

int launch_swiglu(const evs_model* m, evs_state* s, int M, int splits, cudaStream_t st) {
  const int F = m->cfg.mlp_inner;
  dim3 grid((F + ROW_THREADS - 1) / ROW_THREADS, M);
  if (m->cfg.dtype == EVS_DTYPE_BF16)
    swiglu_kernel<__nv_bfloat16><<<grid, ROW_THREADS, 0, st>>>(s->ws, splits, M, F,
                                                                static_cast<__nv_bfloat16*>(s->act), s->ld_act);
  else
    swiglu_kernel<float><<<grid, ROW_THREADS, 0, st>>>(s->ws, splits, M, F, static_cast<float*>(s->act), s->ld_act);
  EVS_CUDA_TRY(cudaGetLastError());
  evs_count_launch(1);
  return EVS_OK;
}

int launch_logits(const evs_model* m, evs_state* s, int M, int T, int splits, float* logits, int out_T, int t0,
                  int last_only, cudaStream_t st) {
  const int V = m->cfg.vocab_size;
  dim3 grid((V + 255) / 256, M);
  logits_kernel<<<grid, 256, 0, st>>>(s->ws, splits, M, V, T, out_T, t0, last_only, logits);
  EVS_CUDA_TRY(cudaGetLastError());
  evs_count_launch(1);
  return EVS_OK;
}

int launch_bookkeeping(evs_state* s, int B, int T, int retain, cudaStream_t st) {
  bookkeeping_kernel<<<(B + 127) / 128, 128, 0, st>>>(s->d_len, s->d_len0, s->d_iir_cur, s->d_chunk, B, T, retain);
  EVS_CUDA_TRY(cudaGetLastError());
  evs_count_launch(1);
  return EVS_OK;
}

int launch_poles(const float* log_poles, float* poles, int n, cudaStream_t st) {
  poles_kernel<<<(n + 255) / 256, 256, 0, st>>>(log_poles, poles, n);
  EVS_CUDA_TRY(cudaGetLastError());
  evs_count_launch(1);
  return EVS_OK;
}
