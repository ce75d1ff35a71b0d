// fp64 sampling helpers shared by the verifier and the drafter's serial head.
//
// Row sums use pairwise summation — blocks of at most 128 values summed with eight running
// partials combined as ((r0+r1)+(r2+r3))+((r4+r5)+(r6+r7)), larger ranges split in two at a
// multiple of 8 — and cumulative sums run left to right, so that for the same inputs the
// normalised rows and the inverse-CDF draws equal numpy's (evspark/specdec/verifier.py:28-40 and
// evspark/specdec/transforms.py:18-64 are written against numpy).  The leaves of the summation
// tree are evaluated by groups of eight threads in parallel; only the cumulative sum is serial.
#pragma once

#include <math_constants.h>

#include "common.cuh"

namespace evs_sampling {

constexpr int VMAX = 1024;
constexpr int MAX_LEAVES = 16;  // VMAX / 64

// scratch the helpers share (one per block, in shared memory)
struct SampScratch {
  double leaf[MAX_LEAVES];
  double dv[32];
  int iv[32];
  double scal[2];
  int icount;
  int cidx[VMAX];  // sampling: indices of the nonzero weights, in index order
};

// leaf ranges of the pairwise-summation tree of n values, left to right
__device__ inline int pw_leaves(int n, int* start, int* len) {
  int cnt = 0;
  // explicit stack of (offset, size), processed depth-first left to right
  int so[32], ss[32], top = 0;
  so[0] = 0;
  ss[0] = n;
  top = 1;
  while (top > 0) {
    --top;
    const int o = so[top], m = ss[top];
    if (m <= 128) {
      start[cnt] = o;
      len[cnt] = m;
      ++cnt;
    } else {
      int n2 = m / 2;
      n2 -= n2 % 8;
      // push right then left so the left range is processed first
      so[top] = o + n2;
      ss[top] = m - n2;
      ++top;
      so[top] = o;
      ss[top] = n2;
      ++top;
    }
  }
  return cnt;
}

__device__ inline double pw_combine(const double* leaf, int n, int* idx) {
  if (n <= 128) return leaf[(*idx)++];
  int n2 = n / 2;
  n2 -= n2 % 8;
  const double a = pw_combine(leaf, n2, idx);
  const double b = pw_combine(leaf, n - n2, idx);
  return a + b;
}

// numpy-identical pairwise sum of a[0..n) (n <= VMAX); whole block participates, >= 128 threads
__device__ inline double block_pairwise_sum(const double* a, int n, SampScratch* sc) {
  int start[MAX_LEAVES], len[MAX_LEAVES];
  const int nl = pw_leaves(n, start, len);
  const int t = threadIdx.x;
  const int leaf = t >> 3, j = t & 7;
  // every thread of the first nl*8 takes part (others idle); groups of 8 are warp-aligned
  double r = 0.0;
  if (leaf < nl) {
    const double* b = a + start[leaf];
    const int m = len[leaf];
    if (m >= 8) {
      r = b[j];
      for (int i = 8 + j; i < m - (m % 8); i += 8) r += b[i];
    } else if (j == 0) {
      for (int i = 0; i < m; ++i) r += b[i];
    }
  }
  // ((r0+r1)+(r2+r3))+((r4+r5)+(r6+r7)) within each group of 8 lanes
  const unsigned full = 0xffffffffu;
  double o = __shfl_xor_sync(full, r, 1);
  r = (j & 1) ? o + r : r + o;
  o = __shfl_xor_sync(full, r, 2);
  r = (j & 2) ? o + r : r + o;
  o = __shfl_xor_sync(full, r, 4);
  r = (j & 4) ? o + r : r + o;
  if (leaf < nl && j == 0) {
    const int m = len[leaf];
    if (m >= 8) {
      const double* b = a + start[leaf];
      for (int i = m - (m % 8); i < m; ++i) r += b[i];
    }
    sc->leaf[leaf] = r;
  }
  __syncthreads();
  if (t == 0) {
    int idx = 0;
    sc->scal[0] = nl == 1 ? sc->leaf[0] : pw_combine(sc->leaf, n, &idx);
  }
  __syncthreads();
  const double out = sc->scal[0];
  __syncthreads();
  return out;
}

__device__ inline double accept_prob(double px, double qx) {
  if (qx > 0.0) {
    const double r = px / qx;
    if (!isfinite(r)) return 0.0;
    return r >= 1.0 ? 1.0 : r;
  }
  return px > 0.0 ? 1.0 : 0.0;
}

// index of the max (lowest index on ties) of row[0..V); whole block participates
__device__ inline int block_argmax(const double* row, int V, SampScratch* sc) {
  double best = 0.0;
  int bi = -1;
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    const double v = row[i];
    if (bi < 0 || v > best) {  // i grows, so ties keep the lower index
      best = v;
      bi = i;
    }
  }
  const unsigned full = 0xffffffffu;
  for (int o = 16; o > 0; o >>= 1) {
    const double ov = __shfl_xor_sync(full, best, o);
    const int oi = __shfl_xor_sync(full, bi, o);
    if (oi >= 0 && (bi < 0 || ov > best || (ov == best && oi < bi))) {
      best = ov;
      bi = oi;
    }
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  if (lane == 0) {
    sc->dv[warp] = best;
    sc->iv[warp] = bi;
  }
  __syncthreads();
  if (warp == 0) {
    best = lane < nw ? sc->dv[lane] : 0.0;
    bi = lane < nw ? sc->iv[lane] : -1;
    for (int o = 16; o > 0; o >>= 1) {
      const double ov = __shfl_xor_sync(full, best, o);
      const int oi = __shfl_xor_sync(full, bi, o);
      if (oi >= 0 && (bi < 0 || ov > best || (ov == best && oi < bi))) {
        best = ov;
        bi = oi;
      }
    }
    if (lane == 0) sc->iv[0] = bi;
  }
  __syncthreads();
  const int out = sc->iv[0];
  __syncthreads();
  return out;
}

// sample_categorical(w, u) with w already clipped at 0 (w is overwritten); whole block.  numpy:
// cumsum left to right, then the count of prefixes with prefix / total <= u.  Adding +0 leaves a
// running sum unchanged, so the prefixes are those of the nonzero weights in index order: warp 0
// compacts them (in place, a ballot per 32 indices), lane 0 sums them in order, and since the
// prefixes never decrease the count is the index of the first nonzero whose prefix / total > u
// (every index before it has a prefix at most the previous one's), or V if there is none.
__device__ inline int block_sample_clipped(double* w, int V, double u, SampScratch* sc) {
  const double s = block_pairwise_sum(w, V, sc);
  const bool bad = !(s > 0.0) || !isfinite(s);
  for (int i = threadIdx.x; i < V; i += blockDim.x) w[i] = bad ? 1.0 / V : w[i] / s;
  __syncthreads();
  if (threadIdx.x < 32) {
    const unsigned full = 0xffffffffu;
    const int lane = threadIdx.x;
    int nnz = 0;
    for (int i0 = 0; i0 < V; i0 += 32) {
      const int i = i0 + lane;
      const double v = i < V ? w[i] : 0.0;
      const unsigned m = __ballot_sync(full, v != 0.0);
      if (v != 0.0) {
        const int pos = nnz + __popc(m & ((1u << lane) - 1u));
        w[pos] = v;  // pos <= i: this round's values were read above, later rounds read higher indices
        sc->cidx[pos] = i;
      }
      nnz += __popc(m);
    }
    __syncwarp();
    if (lane == 0) {
      double c = 0.0;
      for (int n = 0; n < nnz; ++n) {
        c += w[n];
        w[n] = c;
      }
    }
    __syncwarp();
    const double last = nnz > 0 ? w[nnz - 1] : 0.0;
    int first = nnz;
    for (int n = lane; n < nnz; n += 32)
      if (!(w[n] / last <= u)) {
        first = n;
        break;
      }
    for (int o = 16; o > 0; o >>= 1) first = min(first, __shfl_xor_sync(full, first, o));
    if (lane == 0) sc->icount = first < nnz ? sc->cidx[first] : V;
  }
  __syncthreads();
  const int idx = sc->icount;
  __syncthreads();
  return idx < V ? idx : V - 1;
}

// Warp-level forms for V = 128 * NL (NL = 1, 2, 4): lane L holds the 16 elements
// leaf * 128 + j + 8t (leaf = L / 8, j = L % 8, t = 0..15) in registers, exactly the slots of the
// pairwise sum above (8 running partials per 128-element leaf), so a sum is formed as lane-local
// partials in t order -> ((r0+r1)+(r2+r3))+((r4+r5)+(r6+r7)) over the 8 lanes of a leaf -> the leaf
// tree, the same additions as block_pairwise_sum.  Argmax is by warp shuffles (lowest index on
// ties), as block_argmax.
template <int NL>
__device__ __forceinline__ double warp_pw_sum(const double (&v)[16], int lane) {
  double r = 0.0;
#pragma unroll
  for (int t = 0; t < 16; ++t) r += v[t];
  const unsigned full = 0xffffffffu;
  r = r + __shfl_xor_sync(full, r, 1);
  r = r + __shfl_xor_sync(full, r, 2);
  r = r + __shfl_xor_sync(full, r, 4);  // every lane of a leaf: that leaf's sum
  if (NL >= 2) r = r + __shfl_xor_sync(full, r, 8);
  if (NL >= 4) r = r + __shfl_xor_sync(full, r, 16);
  (void)lane;
  return r;
}

// index of the max of the row (lowest index on ties); every lane gets it
__device__ __forceinline__ int warp_argmax16(const double (&v)[16], int base, double* best_out) {
  double best = v[0];
  int bi = base;
#pragma unroll
  for (int t = 1; t < 16; ++t)
    if (v[t] > best) {  // indices grow with t: ties keep the lower index
      best = v[t];
      bi = base + 8 * t;
    }
  const unsigned full = 0xffffffffu;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const double ov = __shfl_xor_sync(full, best, o);
    const int oi = __shfl_xor_sync(full, bi, o);
    if (ov > best || (ov == best && oi < bi)) {
      best = ov;
      bi = oi;
    }
  }
  if (best_out) *best_out = best;
  return bi;
}

// apply_transform of the fp64 row e[0..V) (shared memory; overwritten) into out (global or
// shared).  Whole block participates.  keep / masked: shared scratch of V.
__device__ inline void transform_row(double* e, int V, double temperature, int top_k, double* out, int* keep,
                                     double* masked, SampScratch* sc) {
  if (temperature <= 0.0) {
    const int am = block_argmax(e, V, sc);
    for (int i = threadIdx.x; i < V; i += blockDim.x) out[i] = i == am ? 1.0 : 0.0;
    __syncthreads();
    return;
  }
  for (int i = threadIdx.x; i < V; i += blockDim.x) e[i] = e[i] / temperature;
  __syncthreads();
  const int am = block_argmax(e, V, sc);
  const double mx = e[am];
  __syncthreads();
  for (int i = threadIdx.x; i < V; i += blockDim.x) e[i] = exp(e[i] - mx);
  __syncthreads();
  const double z = block_pairwise_sum(e, V, sc);
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
    const int am2 = block_argmax(masked, V, sc);
    if (threadIdx.x == 0) {
      keep[am2] = 1;
      masked[am2] = -CUDART_INF;
    }
    __syncthreads();
  }
  for (int i = threadIdx.x; i < V; i += blockDim.x) masked[i] = keep[i] ? e[i] : 0.0;
  __syncthreads();
  const double ms = block_pairwise_sum(masked, V, sc);
  const bool bad2 = !(ms > 0.0) || !isfinite(ms);
  for (int i = threadIdx.x; i < V; i += blockDim.x) out[i] = keep[i] ? (bad2 ? 1.0 / top_k : masked[i] / ms) : 0.0;
  __syncthreads();
}

}  // namespace evs_sampling
