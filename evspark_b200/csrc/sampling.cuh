// fp64 sampling helpers shared by the verifier and the drafter's serial head.
//
// Row sums use pairwise summation (blocks of 128 with eight running partials, halves split at a
// multiple of 8) and cumulative sums run left to right, so that for the same inputs the
// normalised rows equal the ones numpy produces (evspark/specdec/verifier.py:28-40 and
// evspark/specdec/transforms.py:18-64 are written against numpy).
#pragma once

#include <math_constants.h>

#include "common.cuh"

namespace evs_sampling {

constexpr int VMAX = 1024;

// pairwise sum of a[0..n) (8-way unrolled base case of 128 elements)
__device__ inline double pairwise_sum(const double* a, int n) {
  if (n < 8) {
    double r = 0.0;
    for (int i = 0; i < n; ++i) r += a[i];
    return r;
  }
  if (n <= 128) {
    double r[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) r[j] = a[j];
    int i = 8;
    for (; i < n - (n % 8); i += 8) {
#pragma unroll
      for (int j = 0; j < 8; ++j) r[j] += a[i + j];
    }
    double res = ((r[0] + r[1]) + (r[2] + r[3])) + ((r[4] + r[5]) + (r[6] + r[7]));
    for (; i < n; ++i) res += a[i];
    return res;
  }
  int n2 = n / 2;
  n2 -= n2 % 8;
  return pairwise_sum(a, n2) + pairwise_sum(a + n2, n - n2);
}

// index of the max (lowest index on ties) of row[0..V), whole block participates
__device__ inline int block_argmax(const double* row, int V, double* sv, int* si) {
  double best = 0.0;
  int bi = -1;
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    const double v = row[i];
    if (bi < 0 || v > best) {  // i grows, so ties keep the lower index
      best = v;
      bi = i;
    }
  }
  sv[threadIdx.x] = best;
  si[threadIdx.x] = bi;
  __syncthreads();
  for (int s = blockDim.x / 2; s > 0; s >>= 1) {
    if (threadIdx.x < s) {
      const double ov = sv[threadIdx.x + s], mv = sv[threadIdx.x];
      const int oi = si[threadIdx.x + s], mi = si[threadIdx.x];
      if (oi >= 0 && (mi < 0 || ov > mv || (ov == mv && oi < mi))) {
        sv[threadIdx.x] = ov;
        si[threadIdx.x] = oi;
      }
    }
    __syncthreads();
  }
  const int out = si[0];
  __syncthreads();
  return out;
}

// thread 0 only: sample_categorical(row, u) with row already clipped at 0 in `w` (length V)
__device__ inline int sample_clipped(double* w, int V, double u) {
  const double s = pairwise_sum(w, V);
  if (!(s > 0.0) || !isfinite(s)) {
    for (int i = 0; i < V; ++i) w[i] = 1.0 / V;
  } else {
    for (int i = 0; i < V; ++i) w[i] = w[i] / s;
  }
  double c = 0.0;
  for (int i = 0; i < V; ++i) {
    c += w[i];
    w[i] = c;
  }
  const double last = w[V - 1];
  int idx = 0;
  for (int i = 0; i < V; ++i) {
    if (w[i] / last <= u) idx = i + 1;
  }
  return idx < V ? idx : V - 1;
}

__device__ inline double accept_prob(double px, double qx) {
  if (qx > 0.0) {
    const double r = px / qx;
    if (!isfinite(r)) return 0.0;
    return r >= 1.0 ? 1.0 : r;
  }
  return px > 0.0 ? 1.0 : 0.0;
}


// apply_transform of the fp64 row e[0..V) (in shared memory; overwritten) into out (global or
// shared).  Whole block participates.  keep / masked / sv / si are shared scratch of V / 256.
__device__ inline void transform_row(double* e, int V, double temperature, int top_k, double* out, int* keep,
                                     double* masked, double* sv, int* si, double* scal) {
  if (temperature <= 0.0) {
    const int am = block_argmax(e, V, sv, si);
    for (int i = threadIdx.x; i < V; i += blockDim.x) out[i] = i == am ? 1.0 : 0.0;
    __syncthreads();
    return;
  }
  for (int i = threadIdx.x; i < V; i += blockDim.x) e[i] = e[i] / temperature;
  __syncthreads();
  const int am = block_argmax(e, V, sv, si);
  const double mx = e[am];
  __syncthreads();
  for (int i = threadIdx.x; i < V; i += blockDim.x) e[i] = exp(e[i] - mx);
  __syncthreads();
  if (threadIdx.x == 0) scal[0] = pairwise_sum(e, V);
  __syncthreads();
  const double z = scal[0];
  const bool bad = !(z > 0.0) || !isfinite(z);
  for (int i = threadIdx.x; i < V; i += blockDim.x) e[i] = bad ? 1.0 / V : e[i] / z;
  __syncthreads();
  if (top_k <= 0 || top_k >= V) {
    for (int i = threadIdx.x; i < V; i += blockDim.x) out[i] = e[i];
    __syncthreads();
    return;
  }
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    keep[i] = 0;
    masked[i] = e[i];
  }
  __syncthreads();
  for (int k = 0; k < top_k; ++k) {
    const int am2 = block_argmax(masked, V, sv, si);
    if (threadIdx.x == 0) {
      keep[am2] = 1;
      masked[am2] = -CUDART_INF;
    }
    __syncthreads();
  }
  for (int i = threadIdx.x; i < V; i += blockDim.x) masked[i] = keep[i] ? e[i] : 0.0;
  __syncthreads();
  if (threadIdx.x == 0) scal[0] = pairwise_sum(masked, V);
  __syncthreads();
  const double ms = scal[0];
  const bool bad2 = !(ms > 0.0) || !isfinite(ms);
  for (int i = threadIdx.x; i < V; i += blockDim.x) out[i] = keep[i] ? (bad2 ? 1.0 / top_k : masked[i] / ms) : 0.0;
  __syncthreads();
}

}  // namespace evs_sampling
