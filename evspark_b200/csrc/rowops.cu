// Row-wise kernels between the GEMMs: embedding + pre-norm, split-K reduction + residual
// add + RMSNorm (+ drafter-context capture), SwiGLU gating, logits, per-row bookkeeping.
// Every reduction runs in a fixed order that does not depend on the number of token rows.
#include <cooperative_groups.h>

#include <algorithm>

#include "internal.hpp"

namespace cg = cooperative_groups;

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
  pdl_trigger();
  pdl_wait();
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

// A cluster of NORM_CL CTAs per token row: CTA r owns columns [r*d/NORM_CL, (r+1)*d/NORM_CL) as
// float4s held in registers.  Split partials are summed in split order, the residual updated (and
// captured), and the row's sum of squares formed as: per-thread components in order -> warp
// butterfly -> warps in order -> cluster ranks in order (read through distributed shared memory),
// so every CTA of the cluster sees the same value and the result does not depend on M.
constexpr int NORM_CL = 8;
constexpr int NORM_THREADS = 128;
constexpr int NORM_VPT = 4;  // float4s per thread: d <= NORM_CL * NORM_THREADS * 4 * NORM_VPT = 16384

template <typename TD>
__device__ inline void store4(TD* dst, float4 v) {
  if constexpr (sizeof(TD) == 2) {
    __nv_bfloat162 lo = __floats2bfloat162_rn(v.x, v.y), hi = __floats2bfloat162_rn(v.z, v.w);
    uint2 u;
    u.x = *reinterpret_cast<uint32_t*>(&lo);
    u.y = *reinterpret_cast<uint32_t*>(&hi);
    *reinterpret_cast<uint2*>(dst) = u;
  } else {
    *reinterpret_cast<float4*>(dst) = v;
  }
}

// TP: the partial sums come from parts.R ranks (channel sharding), one summed partial per rank.
// Thread r polls rank r's flag and every rank's float4 of a column is loaded before the rank-order
// adds, so a reduction costs one NVLink round trip for the flags and one for the data, not R each.
template <typename TD, bool TP>
__global__ void __cluster_dims__(NORM_CL, 1, 1) __launch_bounds__(NORM_THREADS)
    res_add_norm_kernel(TpPartials parts, int splits, int M, float* __restrict__ resid,
                        const float* __restrict__ scale, TD* __restrict__ act, int ld_act, int d, float eps,
                        float* __restrict__ ring, int ring_len, const int32_t* __restrict__ len, int T,
                        unsigned long long* __restrict__ tags, const unsigned long long* __restrict__ fwd_seq,
                        unsigned long long tag_hi, EvsDevErr* err) {
  pdl_trigger();
  cg::cluster_group cluster = cg::this_cluster();
  // first phase of a cluster barrier: its wait (before the first store into a peer's shared memory)
  // guarantees that every CTA of the cluster has started
  cluster_arrive_relaxed();
  const int rank = static_cast<int>(cluster.block_rank());
  const int cpc = d / NORM_CL, n4 = cpc / 4;
  const int c_base = rank * cpc;
  // the norm weight is a weight (no earlier kernel writes it): load it before the wait
  float4 sc[NORM_VPT];
#pragma unroll
  for (int v = 0; v < NORM_VPT; ++v) {
    const int c4 = threadIdx.x + v * NORM_THREADS;
    if (c4 < n4) sc[v] = __ldg(reinterpret_cast<const float4*>(scale + c_base + c4 * 4));
  }
  pdl_wait();
  if constexpr (TP) {
    // every rank's partial sums of this reduction are published once its flag reaches the epoch;
    // thread r waits for rank r (on a timeout the sums below use whatever the buffers hold and the
    // error word reports it)
    const int r = threadIdx.x;
    const long long* f = nullptr;
#pragma unroll
    for (int q = 0; q < EVS_TP_MAX; ++q)
      if (q == r && q < parts.R) f = parts.flag[q];
    if (f != nullptr && ld_acquire_sys(f) < parts.epoch) {
      const uint64_t t0 = globaltimer_ns();
      while (ld_acquire_sys(f) < parts.epoch) {
        if (globaltimer_ns() - t0 > EVS_WAIT_LIMIT_NS) {
          evs_record_error(err, EVS_ETIMEOUT, EVS_K_ROW, 1000 + r);
          break;
        }
      }
    }
    __syncthreads();
  }
  __shared__ float red[NORM_THREADS / 32];
  __shared__ float ss_all[NORM_CL];  // every CTA's sum of squares, stored here by its owner
  const int row = blockIdx.y;
  const int b = row / T, t = row % T;
  float* cap = nullptr;
  if (ring != nullptr && t >= T - ring_len) {
    const int P = len[b] + t;
    cap = ring + (static_cast<size_t>(b) * ring_len + P % ring_len) * d;
    if (tags != nullptr && rank == 0 && threadIdx.x == 0)
      tags[static_cast<size_t>(b) * ring_len + P % ring_len] = evs_capture_tag(tag_hi, b, *fwd_seq);
  }
  float4 r[NORM_VPT];
  float ss = 0.f;
  // the residual values first, so that their loads are in flight with the partial sums'
  float4 xr[NORM_VPT];
#pragma unroll
  for (int v = 0; v < NORM_VPT; ++v) {
    const int c4 = threadIdx.x + v * NORM_THREADS;
    if (c4 < n4) xr[v] = *reinterpret_cast<const float4*>(resid + static_cast<size_t>(row) * d + c_base + c4 * 4);
  }
  // TP: every rank's partial (one summed split each) for two column groups at a time, all in flight
  constexpr int TPV = 2;
  float4 tp_acc[NORM_VPT];
  if constexpr (TP) {
#pragma unroll
    for (int v0 = 0; v0 < NORM_VPT; v0 += TPV) {
      float4 pv[TPV][EVS_TP_MAX];
#pragma unroll
      for (int v = v0; v < v0 + TPV; ++v) {
        const int c4 = threadIdx.x + v * NORM_THREADS;
#pragma unroll
        for (int q = 0; q < EVS_TP_MAX; ++q)
          if (c4 < n4 && q < parts.R)
            pv[v - v0][q] = __ldcv(reinterpret_cast<const float4*>(parts.buf[q] + static_cast<size_t>(row) * d +
                                                                    c_base + c4 * 4));
      }
#pragma unroll
      for (int v = v0; v < v0 + TPV; ++v) {
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int q = 0; q < EVS_TP_MAX; ++q)  // ranks in rank order
          if (q < parts.R) {
            acc.x += pv[v - v0][q].x;
            acc.y += pv[v - v0][q].y;
            acc.z += pv[v - v0][q].z;
            acc.w += pv[v - v0][q].w;
          }
        tp_acc[v] = acc;
      }
    }
  }
#pragma unroll
  for (int v = 0; v < NORM_VPT; ++v) {
    const int c4 = threadIdx.x + v * NORM_THREADS;
    if (c4 < n4) {
      const int c = c_base + c4 * 4;
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      if constexpr (TP) {
        acc = tp_acc[v];
      } else {
        // one rank: its splits in split order
        split_sum4<false>(acc, parts.buf[0] + static_cast<size_t>(row) * d + c, static_cast<size_t>(M) * d, splits);
      }
      float4* rp = reinterpret_cast<float4*>(resid + static_cast<size_t>(row) * d + c);
      float4 x = xr[v];
      x.x += acc.x;
      x.y += acc.y;
      x.z += acc.z;
      x.w += acc.w;
      *rp = x;
      if (cap != nullptr) *reinterpret_cast<float4*>(cap + c) = x;
      ss = fmaf(x.x, x.x, ss);
      ss = fmaf(x.y, x.y, ss);
      ss = fmaf(x.z, x.z, ss);
      ss = fmaf(x.w, x.w, ss);
      r[v] = x;
    }
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  cluster_wait();  // every CTA of the cluster has started
  if (threadIdx.x == 0) {
    float a = 0.f;
    for (int w = 0; w < NORM_THREADS / 32; ++w) a += red[w];
    // this CTA's sum into slot `rank` of every CTA's ss_all (its own included)
#pragma unroll
    for (int q = 0; q < NORM_CL; ++q) *cluster.map_shared_rank(&ss_all[rank], q) = a;
  }
  cluster.sync();  // every CTA's sums have arrived; no shared memory of a peer is touched after this
  float tot = 0.f;
  for (int q = 0; q < NORM_CL; ++q) tot += ss_all[q];
  const float inv = 1.0f / sqrtf(tot / static_cast<float>(d) + eps);
#pragma unroll
  for (int v = 0; v < NORM_VPT; ++v) {
    const int c4 = threadIdx.x + v * NORM_THREADS;
    if (c4 < n4) {
      const int c = c_base + c4 * 4;
      const float4 x = r[v];
      store4<TD>(act + static_cast<size_t>(row) * ld_act + c,
                 make_float4(x.x * inv * sc[v].x, x.y * inv * sc[v].y, x.z * inv * sc[v].z, x.w * inv * sc[v].w));
    }
  }
}

// Many token rows of one split without channel sharding (the serial-split projections): a cluster
// walks NORM_RPC consecutive rows with the next row's residual and partial sums in flight while the
// current row's sum of squares is reduced.  A row's arithmetic is res_add_norm_kernel's (0 + the
// split, the residual added, the same reduction order), so both kernels give the same bits.
constexpr int NORM_RPC = 4;
template <typename TD>
__global__ void __cluster_dims__(NORM_CL, 1, 1) __launch_bounds__(NORM_THREADS)
    res_add_norm_rows_kernel(const float* __restrict__ part, int M, float* __restrict__ resid,
                             const float* __restrict__ scale, TD* __restrict__ act, int ld_act, int d, float eps,
                             float* __restrict__ ring, int ring_len, const int32_t* __restrict__ len, int T,
                             unsigned long long* __restrict__ tags, const unsigned long long* __restrict__ fwd_seq,
                             unsigned long long tag_hi) {
  pdl_trigger();
  cg::cluster_group cluster = cg::this_cluster();
  cluster_arrive_relaxed();  // its wait, before the first remote store: every peer has started
  const int rank = static_cast<int>(cluster.block_rank());
  const int cpc = d / NORM_CL, n4 = cpc / 4;
  const int c_base = rank * cpc;
  float4 sc[NORM_VPT];
#pragma unroll
  for (int v = 0; v < NORM_VPT; ++v) {
    const int c4 = threadIdx.x + v * NORM_THREADS;
    if (c4 < n4) sc[v] = __ldg(reinterpret_cast<const float4*>(scale + c_base + c4 * 4));
  }
  pdl_wait();
  __shared__ float red[NORM_THREADS / 32];
  // every CTA's sum of squares, stored here by its owner; rows alternate between the two halves, so
  // a peer's store for row i + 2 (after row i + 1's barrier) never meets this CTA's reads of row i
  __shared__ float ss_all[2][NORM_CL];
  const int row0 = blockIdx.y * NORM_RPC, row_end = min(M, row0 + NORM_RPC);
  float4 xr[NORM_VPT], pv[NORM_VPT];
  auto load_row = [&](int row, float4 (&x)[NORM_VPT], float4 (&q)[NORM_VPT]) {
#pragma unroll
    for (int v = 0; v < NORM_VPT; ++v) {
      const int c4 = threadIdx.x + v * NORM_THREADS;
      if (c4 < n4) {
        const size_t o = static_cast<size_t>(row) * d + c_base + c4 * 4;
        x[v] = *reinterpret_cast<const float4*>(resid + o);
        q[v] = *reinterpret_cast<const float4*>(part + o);
      }
    }
  };
  load_row(row0, xr, pv);
  for (int row = row0; row < row_end; ++row) {
    float4 xn[NORM_VPT], pn[NORM_VPT];
    if (row + 1 < row_end) load_row(row + 1, xn, pn);
    const int b = row / T, t = row % T;
    float* cap = nullptr;
    if (ring != nullptr && t >= T - ring_len) {
      const int P = len[b] + t;
      cap = ring + (static_cast<size_t>(b) * ring_len + P % ring_len) * d;
      if (tags != nullptr && rank == 0 && threadIdx.x == 0)
        tags[static_cast<size_t>(b) * ring_len + P % ring_len] = evs_capture_tag(tag_hi, b, *fwd_seq);
    }
    float4 r[NORM_VPT];
    float ss = 0.f;
#pragma unroll
    for (int v = 0; v < NORM_VPT; ++v) {
      const int c4 = threadIdx.x + v * NORM_THREADS;
      if (c4 < n4) {
        const int c = c_base + c4 * 4;
        float4 x = xr[v];
        x.x += 0.f + pv[v].x;
        x.y += 0.f + pv[v].y;
        x.z += 0.f + pv[v].z;
        x.w += 0.f + pv[v].w;
        *reinterpret_cast<float4*>(resid + static_cast<size_t>(row) * d + c) = x;
        if (cap != nullptr) *reinterpret_cast<float4*>(cap + c) = x;
        ss = fmaf(x.x, x.x, ss);
        ss = fmaf(x.y, x.y, ss);
        ss = fmaf(x.z, x.z, ss);
        ss = fmaf(x.w, x.w, ss);
        r[v] = x;
      }
    }
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (row == row0) cluster_wait();
    float* slots = ss_all[(row - row0) & 1];
    if (threadIdx.x == 0) {
      float a = 0.f;
      for (int w = 0; w < NORM_THREADS / 32; ++w) a += red[w];
#pragma unroll
      for (int q = 0; q < NORM_CL; ++q) *cluster.map_shared_rank(&slots[rank], q) = a;
    }
    cluster.sync();  // every CTA's sum of this row has arrived
    float tot = 0.f;
    for (int q = 0; q < NORM_CL; ++q) tot += slots[q];
    const float inv = 1.0f / sqrtf(tot / static_cast<float>(d) + eps);
#pragma unroll
    for (int v = 0; v < NORM_VPT; ++v) {
      const int c4 = threadIdx.x + v * NORM_THREADS;
      if (c4 < n4) {
        const int c = c_base + c4 * 4;
        const float4 x = r[v];
        store4<TD>(act + static_cast<size_t>(row) * ld_act + c,
                   make_float4(x.x * inv * sc[v].x, x.y * inv * sc[v].y, x.z * inv * sc[v].z, x.w * inv * sc[v].w));
      }
    }
#pragma unroll
    for (int v = 0; v < NORM_VPT; ++v) {
      xr[v] = xn[v];
      pv[v] = pn[v];
    }
  }
}

// ws holds the dual GEMM: virtual row (f / 64) * 128 + j * 64 + f % 64 is w_{j+1} feature f.
// Each thread gates four consecutive features (one float4 of each half) of RPT token rows
// (rows blockIdx.y * RPT ..; their loads in flight together when the projection left one split).
template <typename TD, int RPT>
__global__ void __launch_bounds__(ROW_THREADS) swiglu_kernel(const float* __restrict__ ws, int splits, int M, int F,
                                                            TD* __restrict__ act, int ld_act) {
  pdl_trigger();
  pdl_wait();
  const int f = (blockIdx.x * ROW_THREADS + threadIdx.x) * 4;
  if (f >= F) return;
  const int N2 = 2 * F;
  const int v1 = (f / 64) * 128 + (f % 64), v2 = v1 + 64;
  float4 g1[RPT], g2[RPT];
#pragma unroll
  for (int i = 0; i < RPT; ++i) {
    const int row = blockIdx.y * RPT + i;
    g1[i] = g2[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (row < M) {
      const float* r = ws + static_cast<size_t>(row) * N2;
      split_sum4<false>(g1[i], r + v1, static_cast<size_t>(M) * N2, splits);
      split_sum4<false>(g2[i], r + v2, static_cast<size_t>(M) * N2, splits);
    }
  }
#pragma unroll
  for (int i = 0; i < RPT; ++i) {
    const int row = blockIdx.y * RPT + i;
    if (row < M)
      store4<TD>(act + static_cast<size_t>(row) * ld_act + f,
                 make_float4(swiglu_gate(g1[i].x, g2[i].x), swiglu_gate(g1[i].y, g2[i].y),
                             swiglu_gate(g1[i].z, g2[i].z), swiglu_gate(g1[i].w, g2[i].w)));
  }
}

__global__ void logits_kernel(const float* __restrict__ ws, int splits, int M, int V, int T, int out_T, int t0,
                              int last_only, float* __restrict__ out) {
  pdl_trigger();
  pdl_wait();
  const int row = blockIdx.y;
  const int v = blockIdx.x * blockDim.x + threadIdx.x;
  if (v >= V) return;
  const int t = row % T;
  if (last_only && t != T - 1) return;
  const float acc = split_sum(ws + static_cast<size_t>(row) * V + v, static_cast<size_t>(M) * V, splits);
  const int b = row / T;
  const size_t orow = last_only ? static_cast<size_t>(b) : static_cast<size_t>(b) * out_T + t0 + t;
  out[orow * V + v] = acc;
}

__global__ void bookkeeping_kernel(int32_t* len, int32_t* len0, int32_t* iir_cur, int32_t* chunk, int B, int T,
                                   int retain, unsigned long long* fwd_seq) {
  pdl_trigger();
  pdl_wait();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b < B) {
    const int old = len[b];
    len0[b] = old;
    len[b] = old + T;
    iir_cur[b] = retain ? T - 1 : 0;
  }
  if (b == 0) {
    chunk[0] = retain ? T : 0;
    *fwd_seq += 1;  // the next forward's capture rows get a new tag
  }
}

// publish this rank's partial sums (written by the preceding projection) to the peers
// This rank's split partials of a row-parallel projection summed in split order into split 0
// (in place, float4 per thread), then the epoch published: each CTA fences its sums at system
// scope and counts itself in; the last one resets the counter and stores the epoch with a
// system-scope release.  The peers then read one partial buffer per rank instead of every split.
__global__ void tp_reduce_signal_kernel(float4* __restrict__ buf, int splits, int n4, unsigned* counter,
                                        long long* flag, long long epoch) {
  pdl_trigger();
  pdl_wait();
  if (splits > 1) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += gridDim.x * blockDim.x) {
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int sp = 0; sp < splits; ++sp) {
        const float4 v = buf[static_cast<size_t>(sp) * n4 + i];
        acc.x += v.x;
        acc.y += v.y;
        acc.z += v.z;
        acc.w += v.w;
      }
      buf[i] = acc;
    }
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0 && atomicAdd(counter, 1u) == gridDim.x - 1) {
    *counter = 0u;
    __threadfence_system();
    st_release_sys(flag, epoch);
  }
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
    EVS_CUDA_TRY(evs_launch(embed_norm_kernel<__nv_bfloat16>, dim3(M), dim3(ROW_THREADS), 0, st, s->use_pdl(), ids,
                            static_cast<const __nv_bfloat16*>(m->embed), scale, s->resid,
                            static_cast<__nv_bfloat16*>(s->act), s->ld_act, d, m->cfg.vocab_size, m->cfg.eps,
                            s->d_err));
  else
    EVS_CUDA_TRY(evs_launch(embed_norm_kernel<float>, dim3(M), dim3(ROW_THREADS), 0, st, s->use_pdl(), ids,
                            static_cast<const float*>(m->embed), scale, s->resid, static_cast<float*>(s->act),
                            s->ld_act, d, m->cfg.vocab_size, m->cfg.eps, s->d_err));
  evs_count_launch(1);
  return EVS_OK;
}

int launch_res_add_norm(const evs_model* m, evs_state* s, int M, int splits, const TpPartials& parts,
                        const float* scale, int capture_slot, int T, cudaStream_t st) {
  const int d = m->cfg.d_model;
  float* ring = capture_slot >= 0 ? s->cap_ring[capture_slot] : nullptr;
  EVS_CHECK_ARG(d % (NORM_CL * 4) == 0 && d <= NORM_CL * NORM_THREADS * 4 * NORM_VPT && s->ld_act % 4 == 0,
                "d_model must be a multiple of 32 and at most 16384");
  EVS_CHECK_ARG(parts.R >= 1 && parts.R <= EVS_TP_MAX, "bad partial-sum ranks");
  if (parts.R == 1 && splits == 1 && M >= 512) {
    const dim3 grid(NORM_CL, (M + NORM_RPC - 1) / NORM_RPC);
    const unsigned long long* seq = static_cast<const unsigned long long*>(s->d_fwd_seq);
    unsigned long long* tg = ring ? s->cap_tag : nullptr;
    const int32_t* ln = static_cast<const int32_t*>(s->d_len);
    if (m->cfg.dtype == EVS_DTYPE_BF16)
      EVS_CUDA_TRY(evs_launch(res_add_norm_rows_kernel<__nv_bfloat16>, grid, dim3(NORM_THREADS), 0, st, s->use_pdl(),
                              parts.buf[0], M, s->resid, scale, static_cast<__nv_bfloat16*>(s->act), s->ld_act, d,
                              m->cfg.eps, ring, s->ring_len, ln, T, tg, seq, s->tag_hi));
    else
      EVS_CUDA_TRY(evs_launch(res_add_norm_rows_kernel<float>, grid, dim3(NORM_THREADS), 0, st, s->use_pdl(),
                              parts.buf[0], M, s->resid, scale, static_cast<float*>(s->act), s->ld_act, d, m->cfg.eps,
                              ring, s->ring_len, ln, T, tg, seq, s->tag_hi));
    evs_count_launch(1);
    return EVS_OK;
  }
  const bool tp = parts.R > 1;
  EVS_CHECK_ARG(!tp || splits == 1, "channel-sharded partial sums must be pre-summed to one split per rank");
  if (m->cfg.dtype == EVS_DTYPE_BF16)
    EVS_CUDA_TRY(evs_launch(tp ? res_add_norm_kernel<__nv_bfloat16, true> : res_add_norm_kernel<__nv_bfloat16, false>,
                            dim3(NORM_CL, M), dim3(NORM_THREADS), 0, st, s->use_pdl(), parts, splits, M, s->resid,
                            scale, static_cast<__nv_bfloat16*>(s->act), s->ld_act, d, m->cfg.eps, ring, s->ring_len,
                            static_cast<const int32_t*>(s->d_len), T, ring ? s->cap_tag : nullptr,
                            static_cast<const unsigned long long*>(s->d_fwd_seq), s->tag_hi, s->d_err));
  else
    EVS_CUDA_TRY(evs_launch(tp ? res_add_norm_kernel<float, true> : res_add_norm_kernel<float, false>,
                            dim3(NORM_CL, M), dim3(NORM_THREADS), 0, st, s->use_pdl(), parts, splits, M, s->resid,
                            scale, static_cast<float*>(s->act), s->ld_act, d, m->cfg.eps, ring, s->ring_len,
                            static_cast<const int32_t*>(s->d_len), T, ring ? s->cap_tag : nullptr,
                            static_cast<const unsigned long long*>(s->d_fwd_seq), s->tag_hi, s->d_err));
  evs_count_launch(1);
  return EVS_OK;
}

int launch_swiglu(const evs_model* m, evs_state* s, int M, int splits, cudaStream_t st) {
  const int F = m->Fl;  // this rank's MLP features
  EVS_CHECK_ARG(F % 64 == 0, "mlp_inner must be a multiple of 64");
  // many rows of one split (the serial-split projection): four rows per thread, their loads in flight
  const bool four = M >= 256 && splits == 1;
  const int rpt = four ? 4 : 1;
  dim3 grid((F / 4 + ROW_THREADS - 1) / ROW_THREADS, (M + rpt - 1) / rpt);
  if (m->cfg.dtype == EVS_DTYPE_BF16)
    EVS_CUDA_TRY(evs_launch(four ? swiglu_kernel<__nv_bfloat16, 4> : swiglu_kernel<__nv_bfloat16, 1>, grid,
                            dim3(ROW_THREADS), 0, st, s->use_pdl(), static_cast<const float*>(s->ws), splits, M, F,
                            static_cast<__nv_bfloat16*>(s->act), s->ld_act));
  else
    EVS_CUDA_TRY(evs_launch(four ? swiglu_kernel<float, 4> : swiglu_kernel<float, 1>, grid, dim3(ROW_THREADS), 0, st,
                            s->use_pdl(), static_cast<const float*>(s->ws), splits, M, F,
                            static_cast<float*>(s->act), s->ld_act));
  evs_count_launch(1);
  return EVS_OK;
}

int launch_logits(const evs_model* m, evs_state* s, int M, int T, int splits, float* logits, int out_T, int t0,
                  int last_only, cudaStream_t st) {
  const int V = m->cfg.vocab_size;
  dim3 grid((V + 255) / 256, M);
  EVS_CUDA_TRY(evs_launch(logits_kernel, grid, dim3(256), 0, st, s->use_pdl(), static_cast<const float*>(s->ws),
                          splits, M, V, T, out_T, t0, last_only, logits));
  evs_count_launch(1);
  return EVS_OK;
}

int launch_bookkeeping(evs_state* s, int B, int T, int retain, cudaStream_t st) {
  EVS_CUDA_TRY(evs_launch(bookkeeping_kernel, dim3((B + 127) / 128), dim3(128), 0, st, s->use_pdl(), s->d_len,
                          s->d_len0, s->d_iir_cur, s->d_chunk, B, T, retain, s->d_fwd_seq));
  evs_count_launch(1);
  return EVS_OK;
}

int launch_tp_reduce_signal(evs_state* s, float* buf, int splits, int M, long long epoch, cudaStream_t st) {
  char* tail = s->tp_base[s->m->tp_rank] + 2 * s->tp_buf_bytes;  // [epoch flag | ... | arrival counter]
  long long* flag = reinterpret_cast<long long*>(tail);
  unsigned* counter = reinterpret_cast<unsigned*>(tail + 64);
  const int d = s->m->cfg.d_model;
  EVS_CHECK_ARG(d % 4 == 0, "d_model must be a multiple of 4");
  const int n4 = M * d / 4;
  const int blocks = splits > 1 ? std::min((n4 + 255) / 256, 2 * 148) : 1;
  EVS_CUDA_TRY(evs_launch(tp_reduce_signal_kernel, dim3(blocks), dim3(256), 0, st, s->use_pdl(),
                          reinterpret_cast<float4*>(buf), splits, n4, counter, flag, epoch));
  evs_count_launch(1);
  return EVS_OK;
}

int launch_poles(const float* log_poles, float* poles, int n, cudaStream_t st) {
  poles_kernel<<<(n + 255) / 256, 256, 0, st>>>(log_poles, poles, n);
  EVS_CUDA_TRY(cudaGetLastError());
  evs_count_launch(1);
  return EVS_OK;
}
