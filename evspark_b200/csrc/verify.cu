// Sampling transform and Leviathan verification on the device, fp64 decision math.
//
// apply_transform (evspark/specdec/transforms.py:18-64): logits/T, max-subtracted exp,
//   normalise, keep the top-k by (-p, index), renormalise; T <= 0 -> one-hot argmax.
// verify_round (evspark/specdec/verifier.py:54-123): for each draft position draw r and accept
//   iff r < min(1, p(x)/q(x)); on the first rejection sample norm(max(0, p - q)) (p itself when
//   that mass underflows); if everything is accepted sample the bonus token from p_{γ+1}.
// verify_round_greedy (verifier.py:126-176): accept iff x == argmax p (lowest index on ties).
// sample_categorical (verifier.py:28-40): clip at 0, normalise (uniform when the mass is 0 or
//   not finite), inverse CDF with one uniform: the first index whose cumulative sum / total > u.
//
// All fp64 row sums use pairwise summation (blocks of 128 with eight running partials, halves
// split at a multiple of 8) and cumulative sums run left to right, so that for the same inputs
// the normalised rows are the ones numpy produces.
#include "internal.hpp"
#include "sampling.cuh"

namespace {

using namespace evs_sampling;

// one CTA per row
__global__ void __launch_bounds__(256) transform_kernel(const void* __restrict__ logits, int f64, int V,
                                                        double temperature, int top_k, double* __restrict__ probs) {
  __shared__ double e[VMAX], masked[VMAX];
  __shared__ int keep[VMAX];
  __shared__ SampScratch sc;
  const int r = blockIdx.x;
  if (f64) {
    const double* lg = static_cast<const double*>(logits) + static_cast<size_t>(r) * V;
    for (int i = threadIdx.x; i < V; i += blockDim.x) e[i] = lg[i];
  } else {
    const float* lg = static_cast<const float*>(logits) + static_cast<size_t>(r) * V;
    for (int i = threadIdx.x; i < V; i += blockDim.x) e[i] = static_cast<double>(lg[i]);
  }
  __syncthreads();
  transform_row(e, V, temperature, top_k, probs + static_cast<size_t>(r) * V, keep, masked, &sc);
}

// V = 128 NL: one warp per row in the warp layout of warp_pw_sum (lane L holds elements
// leaf * 128 + j + 8t), every reduction a warp shuffle, no block barrier; element by element the
// operations of transform_row, and its sums and argmaxes in the same order, so the same bits.
template <int NL>
__global__ void __launch_bounds__(32) transform_warp_kernel(const void* __restrict__ logits, int f64,
                                                            double temperature, int top_k,
                                                            double* __restrict__ probs) {
  constexpr int V = 128 * NL;
  const int r = blockIdx.x, lane = threadIdx.x, leaf = lane >> 3, j = lane & 7;
  const bool act = leaf < NL;
  const int base = act ? leaf * 128 + j : 0;
  double e[16];
#pragma unroll
  for (int t = 0; t < 16; ++t) {
    const size_t i = static_cast<size_t>(r) * V + base + 8 * t;
    e[t] = !act ? -CUDART_INF
                : (f64 ? static_cast<const double*>(logits)[i] : static_cast<double>(static_cast<const float*>(logits)[i]));
  }
  double* out = probs + static_cast<size_t>(r) * V;
  if (temperature <= 0.0) {
    const int am = warp_argmax16(e, base, nullptr);
#pragma unroll
    for (int t = 0; t < 16; ++t)
      if (act) out[base + 8 * t] = base + 8 * t == am ? 1.0 : 0.0;
    return;
  }
#pragma unroll
  for (int t = 0; t < 16; ++t)
    if (act) e[t] = e[t] / temperature;
  double mx;
  warp_argmax16(e, base, &mx);
#pragma unroll
  for (int t = 0; t < 16; ++t) e[t] = act ? exp(e[t] - mx) : 0.0;
  const double z = warp_pw_sum<NL>(e, lane);
  const bool bad = !(z > 0.0) || !isfinite(z);
#pragma unroll
  for (int t = 0; t < 16; ++t) e[t] = act ? (bad ? 1.0 / V : e[t] / z) : 0.0;
  if (top_k <= 0 || top_k >= V) {
#pragma unroll
    for (int t = 0; t < 16; ++t)
      if (act) out[base + 8 * t] = e[t];
    return;
  }
  unsigned keep = 0;
  double m[16];
#pragma unroll
  for (int t = 0; t < 16; ++t) m[t] = act ? e[t] : -CUDART_INF;
  for (int k = 0; k < top_k; ++k) {
    const int am2 = warp_argmax16(m, base, nullptr);
#pragma unroll
    for (int t = 0; t < 16; ++t)
      if (act && base + 8 * t == am2) {
        keep |= 1u << t;
        m[t] = -CUDART_INF;
      }
  }
#pragma unroll
  for (int t = 0; t < 16; ++t) m[t] = (keep >> t & 1u) ? e[t] : 0.0;
  const double ms = warp_pw_sum<NL>(m, lane);
  const bool bad2 = !(ms > 0.0) || !isfinite(ms);
#pragma unroll
  for (int t = 0; t < 16; ++t)
    if (act) out[base + 8 * t] = (keep >> t & 1u) ? (bad2 ? 1.0 / top_k : m[t] / ms) : 0.0;
}

// one CTA per row b; every block-wide helper is called by all threads (uniform control flow)
__global__ void __launch_bounds__(256) verify_kernel(const double* __restrict__ p, const double* __restrict__ q,
                                                     const int64_t* __restrict__ x, const double* __restrict__ u,
                                                     int gamma, int V, int greedy, int32_t* __restrict__ accepted,
                                                     int64_t* __restrict__ tokens, int32_t* __restrict__ info) {
  __shared__ double w[VMAX];
  __shared__ SampScratch sc;
  __shared__ int s_done, s_acc, s_ui;
  const int b = blockIdx.x;
  const double* pb = p + static_cast<size_t>(b) * (gamma + 1) * V;
  const double* qb = q ? q + static_cast<size_t>(b) * gamma * V : nullptr;
  const int64_t* xb = x + static_cast<size_t>(b) * gamma;
  const double* ub = u ? u + static_cast<size_t>(b) * (gamma + 1) : nullptr;
  int64_t* tb = tokens + static_cast<size_t>(b) * (gamma + 1);
  if (threadIdx.x == 0) {
    s_done = 0;
    s_acc = 0;
    s_ui = 0;
  }
  for (int i = threadIdx.x; i <= gamma; i += blockDim.x) tb[i] = -1;
  __syncthreads();
  int tok = -1, from_res = 0, fb = 0;
  for (int i = 0; i < gamma; ++i) {
    const double* pi = pb + static_cast<size_t>(i) * V;
    const int64_t xi = xb[i];
    if (greedy) {
      const int am = block_argmax(pi, V, &sc);
      if (xi != am) {
        tok = am;
        from_res = 1;
        break;
      }
      if (threadIdx.x == 0) tb[i] = am;
      continue;
    }
    const double* qi = qb + static_cast<size_t>(i) * V;
    const double r = ub[i];  // draw i is the accept test of position i
    const bool ok = xi >= 0 && xi < V && r < accept_prob(pi[xi], qi[xi]);
    if (ok) {
      if (threadIdx.x == 0) tb[i] = xi;
      continue;
    }
    // first rejection: sample norm(max(0, p - q)), or p when that mass underflows
    for (int v = threadIdx.x; v < V; v += blockDim.x) w[v] = fmax(pi[v] - qi[v], 0.0);
    __syncthreads();
    const double mass = block_pairwise_sum(w, V, &sc);
    fb = (!(mass > 0.0) || !isfinite(mass)) ? 1 : 0;
    if (fb) {
      for (int v = threadIdx.x; v < V; v += blockDim.x) w[v] = fmax(pi[v], 0.0);
      __syncthreads();
    }
    tok = block_sample_clipped(w, V, ub[i + 1], &sc);
    from_res = 1;
    if (threadIdx.x == 0) {
      s_acc = i;
      s_ui = i + 2;
      s_done = 1;
    }
    break;
  }
  __syncthreads();
  int acc_len, used;
  if (greedy) {
    // tokens accepted so far are the prefix written above
    acc_len = 0;
    while (acc_len < gamma && tb[acc_len] >= 0) ++acc_len;
    if (tok < 0) tok = block_argmax(pb + static_cast<size_t>(gamma) * V, V, &sc);
    used = 0;
  } else if (!s_done) {
    const double* pg = pb + static_cast<size_t>(gamma) * V;
    for (int v = threadIdx.x; v < V; v += blockDim.x) w[v] = fmax(pg[v], 0.0);
    __syncthreads();
    tok = block_sample_clipped(w, V, ub[gamma], &sc);
    acc_len = gamma;
    used = gamma + 1;
  } else {
    acc_len = s_acc;
    used = s_ui;
  }
  if (threadIdx.x == 0) {
    tb[acc_len] = tok;
    accepted[b] = acc_len;
    info[3 * b + 0] = from_res;
    info[3 * b + 1] = fb;
    info[3 * b + 2] = used;
  }
}

__global__ void __launch_bounds__(256) sample_kernel(const double* __restrict__ rows, int V,
                                                     const double* __restrict__ u, int64_t* __restrict__ out) {
  __shared__ double w[VMAX];
  __shared__ SampScratch sc;
  const int r = blockIdx.x;
  const double* row = rows + static_cast<size_t>(r) * V;
  for (int v = threadIdx.x; v < V; v += blockDim.x) w[v] = fmax(row[v], 0.0);
  __syncthreads();
  const int idx = block_sample_clipped(w, V, u[r], &sc);
  if (threadIdx.x == 0) out[r] = idx;
}

// dst = as_prob_row(src): clip at 0 and normalise (numpy pairwise sum), uniform when the mass is
// zero or not finite.  src may be global or shared; dst shared.  Whole block.
__device__ inline void as_prob_row(const double* src, double* dst, int V, SampScratch* sc) {
  for (int v = threadIdx.x; v < V; v += blockDim.x) dst[v] = fmax(src[v], 0.0);
  __syncthreads();
  const double s = block_pairwise_sum(dst, V, sc);
  const bool bad = !(s > 0.0) || !isfinite(s);
  for (int v = threadIdx.x; v < V; v += blockDim.x) dst[v] = bad ? 1.0 / V : dst[v] / s;
  __syncthreads();
}

// SpecInfer multi-candidate verification of B drafts of one stream (evspark/specdec/verifier.py:
// 212-319).  Candidates that agree with the accepted prefix stay live; position i is tested
// against the first live candidate's target and draft rows; each live candidate in order gets one
// uniform, and a rejection replaces the working distribution by norm(max(0, work - q_lead)) (p_lead
// when that mass underflows).  No candidate accepted: sample the working distribution.  All γ
// accepted: sample the bonus from p_lead[γ].  Greedy: argmax of p_lead[i] (raw logits) against the
// candidates.  One CTA; u holds up to γB + 1 uniforms, used in order.
// out tokens [γ+1]; info = {accepted, from_residual, fallback, uniforms consumed, winner}
__global__ void __launch_bounds__(256) multicand_kernel(const double* __restrict__ p, const double* __restrict__ q,
                                                        const int64_t* __restrict__ x, const double* __restrict__ u,
                                                        int B, int gamma, int V, int greedy,
                                                        int64_t* __restrict__ tokens, int32_t* __restrict__ info) {
  __shared__ double pi[VMAX], qi[VMAX], work[VMAX], tmp[VMAX];
  __shared__ SampScratch sc;
  __shared__ unsigned live_s;
  __shared__ int chosen_s;
  const int g1 = gamma + 1;
  unsigned live = B >= 32 ? 0xffffffffu : ((1u << B) - 1u);
  int used = 0, acc = gamma, from_res = 0, fb = 0, tok = -1;
  auto lead_of = [](unsigned m) { return __ffs(static_cast<int>(m)) - 1; };
  for (int i = 0; i < gamma; ++i) {
    const int lead = lead_of(live);
    const double* prow = p + (static_cast<size_t>(lead) * g1 + i) * V;
    if (greedy) {
      const int t = block_argmax(prow, V, &sc);
      unsigned m = 0;
      for (int b = 0; b < B; ++b)
        if ((live >> b & 1u) && x[static_cast<size_t>(b) * gamma + i] == t) m |= 1u << b;
      if (threadIdx.x == 0) tokens[i] = t;
      if (m == 0) {
        tok = t;
        acc = i;
        from_res = 1;
        break;
      }
      live = m;
      continue;
    }
    as_prob_row(prow, pi, V, &sc);
    as_prob_row(q + (static_cast<size_t>(lead) * gamma + i) * V, qi, V, &sc);
    for (int v = threadIdx.x; v < V; v += blockDim.x) work[v] = pi[v];
    __syncthreads();
    int chosen = -1;
    for (int b = 0; b < B; ++b) {
      if (!(live >> b & 1u)) continue;
      const int64_t xx = x[static_cast<size_t>(b) * gamma + i];
      const double r = u[used++];
      if (xx >= 0 && xx < V && r < accept_prob(work[xx], qi[xx])) {
        chosen = static_cast<int>(xx);
        break;
      }
      for (int v = threadIdx.x; v < V; v += blockDim.x) tmp[v] = fmax(work[v] - qi[v], 0.0);
      __syncthreads();
      const double mass = block_pairwise_sum(tmp, V, &sc);
      if (!(mass > 0.0) || !isfinite(mass)) {
        fb = 1;
        as_prob_row(pi, work, V, &sc);
        break;
      }
      for (int v = threadIdx.x; v < V; v += blockDim.x) work[v] = tmp[v] / mass;
      __syncthreads();
    }
    if (chosen < 0) {
      // sample_categorical(work): clip, normalise, inverse CDF
      for (int v = threadIdx.x; v < V; v += blockDim.x) tmp[v] = fmax(work[v], 0.0);
      __syncthreads();
      tok = block_sample_clipped(tmp, V, u[used++], &sc);
      acc = i;
      from_res = 1;
      break;
    }
    if (threadIdx.x == 0) tokens[i] = chosen;
    unsigned m = 0;
    for (int b = 0; b < B; ++b)
      if ((live >> b & 1u) && x[static_cast<size_t>(b) * gamma + i] == chosen) m |= 1u << b;
    live = m;
  }
  const int lead = lead_of(live);
  if (tok < 0) {  // every position accepted: the bonus from the lead candidate's last row
    const double* prow = p + (static_cast<size_t>(lead) * g1 + gamma) * V;
    if (greedy) {
      tok = block_argmax(prow, V, &sc);
    } else {
      as_prob_row(prow, work, V, &sc);
      for (int v = threadIdx.x; v < V; v += blockDim.x) tmp[v] = fmax(work[v], 0.0);
      __syncthreads();
      tok = block_sample_clipped(tmp, V, u[used++], &sc);
    }
  }
  (void)live_s;
  (void)chosen_s;
  if (threadIdx.x == 0) {
    tokens[acc] = tok;
    info[0] = acc;
    info[1] = from_res;
    info[2] = fb;
    info[3] = used;
    info[4] = lead;
  }
}

}  // namespace

int launch_transform(const void* logits, int logits_fp64, int rows, int V, double temperature, int top_k,
                     double* probs, cudaStream_t st) {
  EVS_CHECK_ARG(V > 0 && V <= VMAX, "vocabulary must be in [1, 1024]");
  if (rows <= 0) return EVS_OK;
  if (V == 512)
    transform_warp_kernel<4><<<rows, 32, 0, st>>>(logits, logits_fp64, temperature, top_k, probs);
  else if (V == 256)
    transform_warp_kernel<2><<<rows, 32, 0, st>>>(logits, logits_fp64, temperature, top_k, probs);
  else if (V == 128)
    transform_warp_kernel<1><<<rows, 32, 0, st>>>(logits, logits_fp64, temperature, top_k, probs);
  else
    transform_kernel<<<rows, 256, 0, st>>>(logits, logits_fp64, V, temperature, top_k, probs);
  EVS_CUDA_TRY(cudaGetLastError());
  evs_count_launch(1);
  return EVS_OK;
}

int launch_verify(const double* p, const double* q, const int64_t* x, const double* u, int B, int gamma, int V,
                  int greedy, int32_t* accepted, int64_t* tokens, int32_t* info, cudaStream_t st) {
  EVS_CHECK_ARG(V > 0 && V <= VMAX, "vocabulary must be in [1, 1024]");
  EVS_CHECK_ARG(gamma >= 1, "gamma must be >= 1");
  EVS_CHECK_ARG(greedy || (q != nullptr && u != nullptr), "sampling verification needs q and uniforms");
  if (B <= 0) return EVS_OK;
  verify_kernel<<<B, 256, 0, st>>>(p, q, x, u, gamma, V, greedy, accepted, tokens, info);
  EVS_CUDA_TRY(cudaGetLastError());
  evs_count_launch(1);
  return EVS_OK;
}

int launch_verify_multicand(const double* p, const double* q, const int64_t* x, const double* u, int B, int gamma,
                            int V, int greedy, int64_t* tokens, int32_t* info, cudaStream_t st) {
  EVS_CHECK_ARG(V > 0 && V <= VMAX, "vocabulary must be in [1, 1024]");
  EVS_CHECK_ARG(gamma >= 1, "gamma must be >= 1");
  EVS_CHECK_ARG(B >= 1 && B <= 32, "n_candidates must be in [1, 32]");
  EVS_CHECK_ARG(greedy || (q != nullptr && u != nullptr), "sampling verification needs q and uniforms");
  multicand_kernel<<<1, 256, 0, st>>>(p, q, x, u, B, gamma, V, greedy, tokens, info);
  EVS_CUDA_TRY(cudaGetLastError());
  evs_count_launch(1);
  return EVS_OK;
}

int launch_sample(const double* rows, int n, int V, const double* u, int64_t* out, cudaStream_t st) {
  EVS_CHECK_ARG(V > 0 && V <= VMAX, "vocabulary must be in [1, 1024]");
  if (n <= 0) return EVS_OK;
  sample_kernel<<<n, 256, 0, st>>>(rows, V, u, out);
  EVS_CUDA_TRY(cudaGetLastError());
  evs_count_launch(1);
  return EVS_OK;
}
