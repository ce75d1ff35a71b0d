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
  float *ctx_in = nullptr, *ctx = nullptr, *emb = nullptr, *h = nullptr, *xb = nullptr, *q = nullptr;
  float *kv_in = nullptr, *kb = nullptr, *vb = nullptr, *y = nullptr, *tmp = nullptr, *m1 = nullptr;
  float *z = nullptr, *U = nullptr, *pe = nullptr;
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

__global__ void gather_ctx_kernel(RingPtrs rings, int n_inject, int ring_len, int H, const int32_t* len, int CW,
                                  float* out) {
  const int j = blockIdx.x, b = blockIdx.y;
  const int L = len[b];
  const int n = min(CW, L);
  const int K = n_inject * H;
  float* dst = out + (static_cast<size_t>(b) * CW + j) * K;
  if (j >= n) {
    for (int e = threadIdx.x; e < K; e += blockDim.x) dst[e] = 0.f;
    return;
  }
  const int P = L - n + j;
  for (int c = 0; c < n_inject; ++c) {
    const float* src = rings.p[c] + (static_cast<size_t>(b) * ring_len + P % ring_len) * H;
    for (int e = threadIdx.x; e < H; e += blockDim.x) dst[c * H + e] = src[e];
  }
}

// out = scale * (v / sqrt(mean(v²) + eps)), v = x (+ bias); one CTA per row
__global__ void bias_rmsnorm_kernel(const float* x, const float* bias, const float* scale, float* out, int d,
                                    float eps) {
  __shared__ float red[33];
  const int row = blockIdx.x;
  const float* xr = x + static_cast<size_t>(row) * d;
  float ss = 0.f;
  for (int c = threadIdx.x; c < d; c += blockDim.x) {
    const float v = bias ? xr[c] + bias[c] : xr[c];
    ss = fmaf(v, v, ss);
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    float s = 0.f;
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) s += red[w];
    red[32] = s;
  }
  __syncthreads();
  const float rms = sqrtf(red[32] / static_cast<float>(d) + eps);
  float* o = out + static_cast<size_t>(row) * d;
  for (int c = threadIdx.x; c < d; c += blockDim.x) {
    const float v = bias ? xr[c] + bias[c] : xr[c];
    o[c] = scale[c] * (v / rms);
  }
}

// rows b*g + t: embed[t == 0 ? anchor[b] : mask]  or embed[ids[b*g + t]] when ids is given
__global__ void embed_rows_kernel(const float* embed, int H, const int64_t* anchor, const int64_t* ids, int g,
                                  int mask_id, float* out) {
  const int row = blockIdx.x;
  const int b = row / g, t = row % g;
  const int64_t id = ids ? ids[row] : (t == 0 ? anchor[b] : mask_id);
  const float* src = embed + static_cast<size_t>(id) * H;
  float* dst = out + static_cast<size_t>(row) * H;
  for (int e = threadIdx.x; e < H; e += blockDim.x) dst[e] = src[e];
}

// x[row] = (x[row] + bias) + pos[t]   (pos may be null)
__global__ void bias_pos_kernel(float* x, const float* bias, const float* pos, int g, int d, int rows) {
  const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= static_cast<size_t>(rows) * d) return;
  const int row = static_cast<int>(i / d), c = static_cast<int>(i % d);
  float v = x[i] + bias[c];
  if (pos) v = v + pos[(row % g) * d + c];
  x[i] = v;
}

// h += (x (+ bias))
__global__ void residual_add_kernel(float* h, const float* x, const float* bias, int d, int rows) {
  const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= static_cast<size_t>(rows) * d) return;
  const float v = bias ? x[i] + bias[i % d] : x[i];
  h[i] = h[i] + v;
}

__global__ void bias_silu_kernel(float* x, const float* bias, int n, int rows) {
  const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= static_cast<size_t>(rows) * n) return;
  const float v = x[i] + bias[i % n];
  x[i] = v / (1.0f + expf(-v));
}

__global__ void scale_kernel(float* x, float s, size_t n) {
  const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n) x[i] = x[i] * s;
}

// kv_in[b] = [ctx[b] (CW rows) ; xb[b] (g rows)]
__global__ void build_kv_kernel(const float* ctx, const float* xb, int CW, int g, int d, float* out) {
  const int j = blockIdx.x, b = blockIdx.y;
  const float* src = j < CW ? ctx + (static_cast<size_t>(b) * CW + j) * d : xb + (static_cast<size_t>(b) * g + j - CW) * d;
  float* dst = out + (static_cast<size_t>(b) * (CW + g) + j) * d;
  for (int c = threadIdx.x; c < d; c += blockDim.x) dst[c] = src[c];
}

// one CTA per (query t, head, row b); 128 threads; keys = ctx rows j < n_ctx(b) and drafts <= t
__global__ void __launch_bounds__(128) draft_attn_kernel(const float* q, const float* kb, const float* vb,
                                                         const int32_t* len, int CW, int g, int d, int heads,
                                                         float* y) {
  __shared__ float sc[256];
  __shared__ float red[8];
  const int t = blockIdx.x, hh = blockIdx.y, b = blockIdx.z;
  const int hd = d / heads;
  const int nctx = min(CW, len[b]);
  const int nk = CW + g;
  const float scale = rsqrtf(static_cast<float>(hd));
  const float* qr = q + (static_cast<size_t>(b) * g + t) * d + hh * hd;
  for (int j = threadIdx.x; j < nk; j += blockDim.x) {
    const bool vis = j < CW ? j < nctx : (j - CW) <= t;
    float s = -CUDART_INF_F;
    if (vis) {
      const float* kr = kb + (static_cast<size_t>(b) * nk + j) * d + hh * hd;
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
    for (int j = 0; j < nk; ++j) acc = fmaf(sc[j], vb[(static_cast<size_t>(b) * nk + j) * d + hh * hd + e], acc);
    y[(static_cast<size_t>(b) * g + t) * d + hh * hd + e] = acc / l;
  }
}

// serial Markov head, one CTA per row
__global__ void __launch_bounds__(256) serial_head_kernel(const float* U, const float* markov, const int64_t* anchor,
                                                          int g, int V, int greedy, double temperature, int top_k,
                                                          const double* u, const int64_t* forced, int64_t* tokens,
                                                          double* qout, int64_t* prev_ids) {
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

// conf[row] = sigmoid([h ; pe] · w + bias); one warp per row
__global__ void conf_kernel(const float* h, const float* pe, const float* w, const float* bias, int d, int rows,
                            float* conf) {
  const int row = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  float acc = 0.f;
  for (int c = lane; c < 2 * d; c += 32) {
    const float x = c < d ? h[static_cast<size_t>(row) * d + c] : pe[static_cast<size_t>(row) * d + c - d];
    acc = fmaf(x, w[c], acc);
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

// out[M][N] = X W^T (fp32, split-K partials reduced in split order)
int sgemm(evs_drafter* dr, const float* W, const float* X, int ldx, float* out, int N, int K, int M,
          cudaStream_t st) {
  const GemmPlan p = gemm_plan_f32(N, K, M, 0);
  EVS_CHECK_RANGE(static_cast<size_t>(p.splits) * M * N <= dr->ws_floats, "drafter workspace too small");
  if (p.splits == 1) return launch_gemm_simt(W, nullptr, X, ldx, EVS_DTYPE_FP32, p, out, st);
  EVS_TRY(launch_gemm_simt(W, nullptr, X, ldx, EVS_DTYPE_FP32, p, dr->ws, st));
  return launch_reduce_splits(dr->ws, p.splits, M, N, nullptr, out, st);
}

inline unsigned blocks_for(size_t n, int t) { return static_cast<unsigned>((n + t - 1) / t); }

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
  const size_t o_ctx_in = take(4 * B * CW * nI * H), o_ctx = take(4 * B * CW * d), o_emb = take(4 * B * g * H);
  const size_t o_h = take(4 * B * g * d), o_xb = take(4 * B * g * d), o_q = take(4 * B * g * d);
  const size_t o_kv = take(4 * B * (CW + g) * d), o_kb = take(4 * B * (CW + g) * d), o_vb = take(4 * B * (CW + g) * d);
  const size_t o_y = take(4 * B * g * d), o_tmp = take(4 * B * g * d), o_m1 = take(4 * B * g * hid);
  const size_t o_z = take(4 * B * g * H), o_U = take(4 * B * g * V), o_pe = take(4 * B * g * d);
  const size_t o_prev = take(8 * B * g);
  // largest split-K partial buffer over the drafter's projections
  size_t wsf = 0;
  auto need = [&](size_t M_, size_t N_, size_t K_) {
    const GemmPlan p = gemm_plan_f32(static_cast<int>(N_), static_cast<int>(K_), static_cast<int>(M_), 0);
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
  dr->emb = reinterpret_cast<float*>(base + o_emb);
  dr->h = reinterpret_cast<float*>(base + o_h);
  dr->xb = reinterpret_cast<float*>(base + o_xb);
  dr->q = reinterpret_cast<float*>(base + o_q);
  dr->kv_in = reinterpret_cast<float*>(base + o_kv);
  dr->kb = reinterpret_cast<float*>(base + o_kb);
  dr->vb = reinterpret_cast<float*>(base + o_vb);
  dr->y = reinterpret_cast<float*>(base + o_y);
  dr->tmp = reinterpret_cast<float*>(base + o_tmp);
  dr->m1 = reinterpret_cast<float*>(base + o_m1);
  dr->z = reinterpret_cast<float*>(base + o_z);
  dr->U = reinterpret_cast<float*>(base + o_U);
  dr->pe = reinterpret_cast<float*>(base + o_pe);
  dr->prev = reinterpret_cast<int64_t*>(base + o_prev);
  dr->ws = reinterpret_cast<float*>(base + o_ws);
  dr->ws_floats = wsf;
  EVS_CUDA_TRY(cudaMemset(dr->block, 0, off));
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
  const int hid = c.mlp_mult * d, nk = CW + g, rows = B * g;
  const float eps = 1e-6f;
  const float* const* T = dr->t;
  // ---- context: H_ctx = RMSNorm(ctx_proj(last rows of the capture ring)) ----
  if (c.n_inject > 0) {
    RingPtrs rg;
    for (int k = 0; k < 4; ++k) rg.p[k] = s->cap_ring[k];
    gather_ctx_kernel<<<dim3(CW, B), 256, 0, st>>>(rg, c.n_inject, s->ring_len, H, s->d_len, CW, dr->ctx_in);
    EVS_CUDA_TRY(cudaGetLastError());
    EVS_TRY(sgemm(dr, T[EVS_D_CTX_W], dr->ctx_in, c.n_inject * H, dr->kb, d, c.n_inject * H, B * CW, st));
    bias_rmsnorm_kernel<<<B * CW, 256, 0, st>>>(dr->kb, T[EVS_D_CTX_B], T[EVS_D_CTX_NORM], dr->ctx, d, eps);
  } else {
    EVS_CUDA_TRY(cudaMemsetAsync(dr->ctx, 0, sizeof(float) * B * CW * d, st));
  }
  // the draft attention reads the context length from the state; without injection it is empty
  const int32_t* ctx_len = c.n_inject > 0 ? s->d_len : reinterpret_cast<const int32_t*>(dr->prev);
  if (c.n_inject == 0) EVS_CUDA_TRY(cudaMemsetAsync(dr->prev, 0, sizeof(int32_t) * B, st));
  // ---- h = in_proj(embed([anchor, MASK...])) + pos ----
  embed_rows_kernel<<<rows, 256, 0, st>>>(T[EVS_D_EMBED], H, anchor, nullptr, g, c.mask_id, dr->emb);
  EVS_TRY(sgemm(dr, T[EVS_D_IN_W], dr->emb, H, dr->h, d, H, rows, st));
  bias_pos_kernel<<<blocks_for(static_cast<size_t>(rows) * d, 256), 256, 0, st>>>(dr->h, T[EVS_D_IN_B], T[EVS_D_POS],
                                                                                 g, d, rows);
  for (int l = 0; l < c.n_layers; ++l) {
    const float* const* L = T + EVS_D_LAYER0 + l * EVS_D_PER_LAYER;
    bias_rmsnorm_kernel<<<rows, 256, 0, st>>>(dr->h, nullptr, L[EVS_D_LN1], dr->xb, d, eps);
    EVS_TRY(sgemm(dr, L[EVS_D_Q], dr->xb, d, dr->q, d, d, rows, st));
    build_kv_kernel<<<dim3(nk, B), 256, 0, st>>>(dr->ctx, dr->xb, CW, g, d, dr->kv_in);
    EVS_TRY(sgemm(dr, L[EVS_D_K], dr->kv_in, d, dr->kb, d, d, B * nk, st));
    EVS_TRY(sgemm(dr, L[EVS_D_V], dr->kv_in, d, dr->vb, d, d, B * nk, st));
    draft_attn_kernel<<<dim3(g, c.n_heads, B), 128, 0, st>>>(dr->q, dr->kb, dr->vb, ctx_len, CW, g, d, c.n_heads,
                                                            dr->y);
    EVS_TRY(sgemm(dr, L[EVS_D_O], dr->y, d, dr->tmp, d, d, rows, st));
    residual_add_kernel<<<blocks_for(static_cast<size_t>(rows) * d, 256), 256, 0, st>>>(dr->h, dr->tmp, nullptr, d,
                                                                                        rows);
    bias_rmsnorm_kernel<<<rows, 256, 0, st>>>(dr->h, nullptr, L[EVS_D_LN2], dr->xb, d, eps);
    EVS_TRY(sgemm(dr, L[EVS_D_MLP0_W], dr->xb, d, dr->m1, hid, d, rows, st));
    bias_silu_kernel<<<blocks_for(static_cast<size_t>(rows) * hid, 256), 256, 0, st>>>(dr->m1, L[EVS_D_MLP0_B], hid,
                                                                                      rows);
    EVS_TRY(sgemm(dr, L[EVS_D_MLP2_W], dr->m1, hid, dr->tmp, d, hid, rows, st));
    residual_add_kernel<<<blocks_for(static_cast<size_t>(rows) * d, 256), 256, 0, st>>>(dr->h, dr->tmp,
                                                                                        L[EVS_D_MLP2_B], d, rows);
  }
  // ---- U = (final_ln(h) out_proj) embedᵀ H^-1/2 ----
  bias_rmsnorm_kernel<<<rows, 256, 0, st>>>(dr->h, nullptr, T[EVS_D_FINAL_LN], dr->xb, d, eps);
  EVS_TRY(sgemm(dr, T[EVS_D_OUT_W], dr->xb, d, dr->z, H, d, rows, st));
  bias_pos_kernel<<<blocks_for(static_cast<size_t>(rows) * H, 256), 256, 0, st>>>(dr->z, T[EVS_D_OUT_B], nullptr, g,
                                                                                 H, rows);
  EVS_TRY(sgemm(dr, T[EVS_D_EMBED], dr->z, H, dr->U, V, H, rows, st));
  scale_kernel<<<blocks_for(static_cast<size_t>(rows) * V, 256), 256, 0, st>>>(
      dr->U, 1.0f / sqrtf(static_cast<float>(H)), static_cast<size_t>(rows) * V);
  // ---- serial Markov head ----
  serial_head_kernel<<<B, 256, 0, st>>>(dr->U, T[EVS_D_MARKOV], anchor, g, V, greedy, temperature, top_k, u, forced,
                                        tokens, qrows, dr->prev);
  // ---- confidence: σ(conf_w [final_ln(h) ; in_proj(embed(prev))]) ----
  embed_rows_kernel<<<rows, 256, 0, st>>>(T[EVS_D_EMBED], H, nullptr, dr->prev, g, 0, dr->emb);
  EVS_TRY(sgemm(dr, T[EVS_D_IN_W], dr->emb, H, dr->pe, d, H, rows, st));
  bias_pos_kernel<<<blocks_for(static_cast<size_t>(rows) * d, 256), 256, 0, st>>>(dr->pe, T[EVS_D_IN_B], nullptr, g,
                                                                                 d, rows);
  conf_kernel<<<blocks_for(rows, 4), 128, 0, st>>>(dr->xb, dr->pe, T[EVS_D_CONF_W], T[EVS_D_CONF_B], d, rows, conf);
  // non-GEMM kernels of this call (the projections count themselves): context gather + norm,
  // embed + bias/pos, 7 per layer, final norm + bias + scale, serial head, conf embed + bias + dot
  evs_count_launch((c.n_inject > 0 ? 2 : 0) + 2 + 7 * c.n_layers + 3 + 4);
  if (U_out != nullptr)
    EVS_CUDA_TRY(cudaMemcpyAsync(U_out, dr->U, sizeof(float) * rows * V, cudaMemcpyDeviceToDevice, st));
  EVS_CUDA_TRY(cudaGetLastError());
  return EVS_OK;
}

}  // extern "C"
