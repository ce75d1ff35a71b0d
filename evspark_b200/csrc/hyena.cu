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

constexpr int CH = 32;          // output channels per CTA (96 interleaved in-projection channels)
constexpr int C3 = 3 * CH;
constexpr int TS = 32;          // chunk positions per pass
constexpr int UW = 64;          // outer-FIR input window in shared memory (positions mod UW)
constexpr int HY_THREADS = 128;      // IIR kernel: 32 channels x 4 pole groups
constexpr int HY_FIR_THREADS = 512;  // FIR kernel: 16 warps, one chunk position per warp at a time

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

// n element copies dst(i) <- src(i) with four loads in flight per thread before the stores
template <typename LoadF, typename StoreF>
__device__ __forceinline__ void batched_copy(int n, LoadF ld, StoreF stf) {
  for (int i0 = threadIdx.x; i0 < n; i0 += 4 * blockDim.x) {
    float v[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int i = i0 + k * blockDim.x;
      if (i < n) v[k] = ld(i);
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int i = i0 + k * blockDim.x;
      if (i < n) stf(i, v[k]);
    }
  }
}

// Stage the outer-FIR history (positions L0-K0+1 .. L0-1 of the outer ring) and the outer taps
// of channels 3h0 .. 3h0+95 in shared memory.
template <typename TD>
__device__ void outer_stage(const HyArgs<TD>& a, int b, int L0, int h0, float* uw, float* wo) {
  const size_t N3 = 3 * static_cast<size_t>(a.d);
  const int c0 = 3 * h0, Hh = a.K0 - 1;
  const TD* ring = a.outer_ring;
  const int cap = a.cap_o;
  batched_copy(
      Hh * C3,
      [&](int i) {
        const int r = i / C3, cc = i - r * C3;
        const int P = L0 - Hh + r;
        return P >= 0 ? to_f32(ring[(static_cast<size_t>(b) * cap + (P % cap)) * N3 + c0 + cc]) : 0.f;
      },
      [&](int i, float v) {
        const int r = i / C3, cc = i - r * C3;
        const int P = L0 - Hh + r;
        if (P >= 0) uw[(P & (UW - 1)) * C3 + cc] = v;
      });
  const float* sw = a.short_w + static_cast<size_t>(c0) * a.K0;
  batched_copy(C3 * a.K0, [&](int i) { return __ldg(sw + i); }, [&](int i, float v) { wo[i] = v; });
}

// The in-projection partials of a pass loaded ahead of the state lengths, which they do not
// depend on: the thread's float4 chunks i = tid + k * blockDim (k < PK) of every split (at most
// PS).  ok is false when the pass has more splits or chunks; outer_pass then loads them itself.
constexpr int PS = 4;
template <int PK>
struct OuterPre {
  float4 v[PS][PK];
  bool ok;
};
template <typename TD, int PK>
__device__ __forceinline__ void outer_preload(const HyArgs<TD>& a, int b, int h0, int t0, int ns, OuterPre<PK>& pre) {
  constexpr int Q = C3 / 4;
  const int n4 = ns * Q;
  pre.ok = a.splits <= PS && n4 <= PK * static_cast<int>(blockDim.x);
  if (!pre.ok) return;
  const size_t N3 = 3 * static_cast<size_t>(a.d);
  const size_t split_stride = static_cast<size_t>(a.M) * N3;
#pragma unroll
  for (int u = 0; u < PS; ++u)
#pragma unroll
    for (int k = 0; k < PK; ++k) {
      const int i = threadIdx.x + k * blockDim.x;
      if (u < a.splits && i < n4) {
        const int t = i / Q, q4 = i - t * Q;
        pre.v[u][k] = __ldg(reinterpret_cast<const float4*>(a.ws + u * split_stride +
                                                            static_cast<size_t>(b * a.T + t0 + t) * N3 + 3 * h0) + q4);
      }
    }
}

// u of chunk i (float4 q4 of position t) into the outer ring and the window uw
template <typename TD>
__device__ __forceinline__ void outer_store_u(const HyArgs<TD>& a, int b, int L0, int h0, int t0, int i, float4 acc,
                                              float* uw) {
  constexpr int Q = C3 / 4;
  const size_t N3 = 3 * static_cast<size_t>(a.d);
  const int t = i / Q, q4 = i - t * Q;
  const int P = L0 + t0 + t;
  const float4 un = make_float4(round_to<TD>(acc.x), round_to<TD>(acc.y), round_to<TD>(acc.z), round_to<TD>(acc.w));
  *reinterpret_cast<float4*>(uw + (P & (UW - 1)) * C3 + 4 * q4) = un;
  TD* dst = a.outer_ring + (static_cast<size_t>(b) * a.cap_o + (P % a.cap_o)) * N3 + 3 * h0 + 4 * q4;
  dst[0] = from_f32<TD>(un.x);
  dst[1] = from_f32<TD>(un.y);
  dst[2] = from_f32<TD>(un.z);
  dst[3] = from_f32<TD>(un.w);
}

// One pass over chunk positions t0 .. t0+ns-1 of row b: in-projection values u (sum of the
// split partials in split order, rounded to the data dtype) into the outer ring and the window uw,
// then the outer FIR outputs z (rounded) into zs[ns][96].  Starts and ends with a block barrier.
// pre: this pass's partials loaded by outer_preload (the same chunks per thread, the same order
// of additions), or null.
template <typename TD, int PK = 1>
__device__ void outer_pass(const HyArgs<TD>& a, int b, int L0, int h0, int t0, int ns, float* uw, const float* wo,
                           float* zs, const OuterPre<PK>* pre = nullptr) {
  const size_t N3 = 3 * static_cast<size_t>(a.d);
  const size_t split_stride = static_cast<size_t>(a.M) * N3;
  const int c0 = 3 * h0;
  constexpr int Q = C3 / 4;  // float4s per position
  const int n4 = ns * Q;
  __syncthreads();  // the previous pass has finished reading uw / zs
  if (pre != nullptr && pre->ok) {
#pragma unroll
    for (int k = 0; k < PK; ++k) {
      const int i = threadIdx.x + k * blockDim.x;
      if (i < n4) {
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int u = 0; u < PS; ++u)
          if (u < a.splits) {
            acc.x += pre->v[u][k].x;
            acc.y += pre->v[u][k].y;
            acc.z += pre->v[u][k].z;
            acc.w += pre->v[u][k].w;
          }
        outer_store_u(a, b, L0, h0, t0, i, acc, uw);
      }
    }
  }
  for (int i0 = threadIdx.x; i0 < ((pre != nullptr && pre->ok) ? 0 : n4); i0 += 4 * blockDim.x) {
    float4 acc[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) acc[k] = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int s0 = 0; s0 < a.splits; s0 += 2) {  // two splits x four chunks of loads in flight
      float4 v[2][4];
#pragma unroll
      for (int u = 0; u < 2; ++u)
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int i = i0 + k * blockDim.x;
          if (s0 + u < a.splits && i < n4) {
            const int t = i / Q, q4 = i - t * Q;
            v[u][k] = __ldg(reinterpret_cast<const float4*>(a.ws + (s0 + u) * split_stride +
                                                            static_cast<size_t>(b * a.T + t0 + t) * N3 + c0) + q4);
          }
        }
#pragma unroll
      for (int u = 0; u < 2; ++u)
        if (s0 + u < a.splits) {
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            acc[k].x += v[u][k].x;
            acc[k].y += v[u][k].y;
            acc[k].z += v[u][k].z;
            acc[k].w += v[u][k].w;
          }
        }
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int i = i0 + k * blockDim.x;
      if (i < n4) outer_store_u(a, b, L0, h0, t0, i, acc[k], uw);
    }
  }
  __syncthreads();
  const int K0 = a.K0;
  for (int i = threadIdx.x; i < ns * C3; i += blockDim.x) {
    const int t = i / C3, cc = i - t * C3;
    const int P = L0 + t0 + t;
    const int cs = min(P, K0 - 1);
    const int base = a.prefill ? K0 - 1 : cs;
    const float* w = wo + cc * K0;
    float z = 0.f;
    for (int age = cs; age >= 1; --age) z = fmaf(w[base - age], uw[((P - age) & (UW - 1)) * C3 + cc], z);
    z = fmaf(w[base], uw[(P & (UW - 1)) * C3 + cc], z);
    zs[t * C3 + cc] = round_to<TD>(z);
  }
  __syncthreads();
}

// tap row stride in shared memory: a multiple of 4 floats whose quarter is odd, so that eight
// lanes reading 16 bytes from eight consecutive rows hit distinct banks
__host__ __device__ constexpr int tap_stride(int K) {
  const int k4 = (K + 3) / 4;
  return 4 * ((k4 & 1) ? k4 : k4 + 1);
}

// grid (d / 32, B), 128 threads.  Shared memory: uw[UW][96] f32 | zs[TS][96] f32 | wo[96][K0] f32 |
// taps[32][tap_stride(K)] f32 | hist[win][32] TD (x1v by position mod win) | x2s[TS][32] f32
template <typename TD, bool FLIP>
__global__ void __launch_bounds__(HY_FIR_THREADS) hyena_fir_kernel(HyArgs<TD> a, int win) {
  pdl_trigger();
  extern __shared__ __align__(16) float sm[];
  const int K = a.K, H = K - 1, KS = tap_stride(K), T = a.T;
  float* uw = sm;
  float* zs = uw + UW * C3;
  float* wo = zs + TS * C3;
  float* taps = wo + C3 * a.K0;
  TD* hist = reinterpret_cast<TD*>(taps + CH * KS);
  float* x2s = reinterpret_cast<float*>(hist + win * CH);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h0 = blockIdx.x * CH, b = blockIdx.y;
  const int wm = win - 1;
  // the filter taps are weights (no earlier kernel writes them): fetch them before waiting for
  // the in-projection, asynchronously when K % 4 == 0
  const float* iw = a.inner_w + static_cast<size_t>(h0) * K;
  if (K % 4 == 0) {
    const int k4 = K / 4;
    for (int i = threadIdx.x; i < CH * k4; i += blockDim.x) {
      const int cc = i / k4, j = i - cc * k4;
      cp_async16(taps + cc * KS + 4 * j, iw + cc * K + 4 * j);
    }
  } else {
    batched_copy(CH * K, [&](int i) { return __ldg(iw + i); },
                 [&](int i, float v) { taps[(i / K) * KS + i % K] = v; });
  }
  cp_async_commit();
  pdl_wait();
  OuterPre<1> pre;
  outer_preload(a, b, h0, 0, min(TS, T), pre);
  const int L0 = a.len[b];
  // inner-FIR history rows, asynchronously
  constexpr int EPC = 16 / sizeof(TD);
  constexpr int RC = CH / EPC;  // 16-byte chunks per history row
  for (int i = threadIdx.x; i < H * RC; i += blockDim.x) {
    const int r = i / RC, c = i - r * RC;
    const int P = L0 - H + r;
    if (P >= 0)
      cp_async16(hist + (P & wm) * CH + c * EPC,
                 a.inner_ring + (static_cast<size_t>(b) * a.cap_i + (P % a.cap_i)) * a.d + h0 + c * EPC);
  }
  cp_async_commit();
  outer_stage(a, b, L0, h0, uw, wo);
  const float Dg = FLIP ? a.D[h0 + lane] : 0.f;
  const float* tp = taps + lane * KS;
  for (int t0 = 0; t0 < T; t0 += TS) {
    const int ns = min(TS, T - t0);
    outer_pass(a, b, L0, h0, t0, ns, uw, wo, zs, t0 == 0 ? &pre : nullptr);
    if (t0 == 0) {
      cp_async_wait<0>();
      __syncthreads();
    }
    // de-interleave (channel 3h+j -> group j): x2 = z[3h], x1v = z[3h+1] * z[3h+2]
    for (int i = threadIdx.x; i < ns * CH; i += blockDim.x) {
      const int t = i / CH, cc = i - t * CH;
      const int P = L0 + t0 + t;
      const float* zr = zs + t * C3 + 3 * cc;
      const float x1v = round_to<TD>(zr[1] * zr[2]);
      hist[(P & wm) * CH + cc] = from_f32<TD>(x1v);
      x2s[t * CH + cc] = zr[0];
      a.inner_ring[(static_cast<size_t>(b) * a.cap_i + (P % a.cap_i)) * a.d + h0 + cc] = from_f32<TD>(x1v);
    }
    __syncthreads();
    // inner FIR, lane = channel, one position per warp at a time, ages in descending order
    for (int t = warp; t < ns; t += HY_FIR_THREADS / 32) {
      const int P = L0 + t0 + t;
      const int cs = min(P, H);
      float z = 0.f;
      if (FLIP) {
        for (int a4 = cs >> 2; a4 >= 0; --a4) {
          const float4 w4 = *reinterpret_cast<const float4*>(tp + 4 * a4);
          const float wv[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
          for (int e = 3; e >= 0; --e) {
            const int age = 4 * a4 + e;
            if (age <= cs) z = fmaf(wv[e], to_f32(hist[((P - age) & wm) * CH + lane]), z);
          }
        }
        z = fmaf(Dg, to_f32(hist[(P & wm) * CH + lane]), z);
      } else {
        const int base = a.prefill ? H : cs;
        for (int age = cs; age >= 0; --age) z = fmaf(tp[base - age], to_f32(hist[((P - age) & wm) * CH + lane]), z);
      }
      const float yv = round_to<TD>(x2s[t * CH + lane] * round_to<TD>(z));
      a.y[static_cast<size_t>(b * T + t0 + t) * a.ld_y + h0 + lane] = from_f32<TD>(yv);
    }
  }
  if (T <= 0) cp_async_wait<0>();
}

template <int SPT>
__device__ __forceinline__ void load_vec(const float* src, float* v) {
  if constexpr (SPT % 4 == 0) {
#pragma unroll
    for (int j = 0; j < SPT; j += 4) {
      const float4 f = *reinterpret_cast<const float4*>(src + j);
      v[j] = f.x;
      v[j + 1] = f.y;
      v[j + 2] = f.z;
      v[j + 3] = f.w;
    }
  } else {
#pragma unroll
    for (int j = 0; j < SPT; ++j) v[j] = src[j];
  }
}

template <int SPT>
__device__ __forceinline__ void store_vec(float* dst, const float* v) {
  if constexpr (SPT % 4 == 0) {
#pragma unroll
    for (int j = 0; j < SPT; j += 4) *reinterpret_cast<float4*>(dst + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
  } else {
#pragma unroll
    for (int j = 0; j < SPT; ++j) dst[j] = v[j];
  }
}

// grid (d / 32, B), 128 threads = 32 channels x 4 pole groups (SPT = S / 4 poles each).
// Shared memory (floats): uw[UW][96] | zs[TS][96] | wo[96][K0]
template <typename TD, int SPT>
__global__ void __launch_bounds__(HY_THREADS) hyena_iir_kernel(HyArgs<TD> a) {
  pdl_trigger();
  extern __shared__ __align__(16) float sm[];
  float* uw = sm;
  float* zs = uw + UW * C3;
  float* wo = zs + TS * C3;
  const int q = threadIdx.x & 3, hl = threadIdx.x >> 2;
  const int h0 = blockIdx.x * CH, h = h0 + hl;
  const int b = blockIdx.y;
  const int T = a.T, S = a.S, d = a.d;
  // poles, residues and D are weights (no earlier kernel writes them): load before the wait
  float p[SPT], r[SPT], s[SPT];
  load_vec<SPT>(a.poles + static_cast<size_t>(h) * S + q * SPT, p);
  load_vec<SPT>(a.residues + static_cast<size_t>(h) * S + q * SPT, r);
  const float Dg = a.D[h];
  pdl_wait();
  OuterPre<3> pre;
  outer_preload(a, b, h0, 0, min(TS, T), pre);
  const int L0 = a.len[b];
  const int cur = a.iir_cur[b];  // loaded with the length: the state load below waits for one round trip
  if (L0 > 0) {
    load_vec<SPT>(a.s_all + ((static_cast<size_t>(b) * a.slots + cur) * d + h) * S + q * SPT, s);
  } else {
#pragma unroll
    for (int j = 0; j < SPT; ++j) s[j] = 0.f;
  }
  outer_stage(a, b, L0, h0, uw, wo);
  __syncthreads();
  for (int t0 = 0; t0 < T; t0 += TS) {
    const int ns = min(TS, T - t0);
    outer_pass(a, b, L0, h0, t0, ns, uw, wo, zs, t0 == 0 ? &pre : nullptr);
    for (int t = 0; t < ns; ++t) {
      const float* zr = zs + t * C3 + 3 * hl;
      const float x1v = round_to<TD>(zr[1] * zr[2]);
      float part = 0.f;
#pragma unroll
      for (int j = 0; j < SPT; ++j) {
        s[j] = fmaf(p[j], s[j], x1v);
        part = fmaf(r[j], s[j], part);
      }
      part += __shfl_xor_sync(0xffffffffu, part, 1);
      part += __shfl_xor_sync(0xffffffffu, part, 2);
      if (q == 0) {
        const float yv = round_to<TD>(zr[0] * (part + Dg * x1v));
        a.y[static_cast<size_t>(b * T + t0 + t) * a.ld_y + h] = from_f32<TD>(yv);
      }
      if (a.retain) store_vec<SPT>(a.s_all + ((static_cast<size_t>(b) * a.slots + t0 + t) * d + h) * S + q * SPT, s);
    }
    __syncthreads();
  }
  // final state into slot 0 (this thread read its old slot before writing anything)
  if (!a.retain) store_vec<SPT>(a.s_all + ((static_cast<size_t>(b) * a.slots + 0) * d + h) * S + q * SPT, s);
}

// ---------------------------------------------------------------------------------------------
// Decode kernels (chunks of at most DEC_T tokens: verify blocks and native steps of any batch).
// One thread owns one output channel h of one row b for every position of the chunk, so the
// in-projection sum, the outer FIR, the de-interleave, x1v and the inner FIR / IIR run in the
// thread's registers with no block barrier between them, and a launch has d x B threads (warps of
// 32 consecutive channels, coalesced on every buffer).  Every value is formed by the same float
// operations in the same order as in hyena_fir_kernel / hyena_iir_kernel (in-projection splits in
// split order; FIR ages oldest first, one fmaf each; the IIR residue sum over four groups of four
// poles, added pairwise), so the two paths give the same bits and the chunking of a sequence
// still changes no result.
// ---------------------------------------------------------------------------------------------
constexpr int DEC_T = 16;     // chunk positions held in registers
constexpr int DEC_ROWS = 4;   // rows per CTA (one warp each); the taps are staged once per CTA
constexpr int DEC_K0 = 3;     // outer short filter length of the decode path
// batches from this many rows take the decode path: with fewer, its d x B threads leave the GPU
// idle and the general kernels (16 warps per 32 channels) finish sooner; the bits are the same
constexpr int DEC_MIN_ROWS = 4;

// 4-element stores of rounded values (bf16: one 8-byte store)
template <typename TD>
__device__ __forceinline__ void store4_td(TD* dst, float a, float b, float c, float d) {
  if constexpr (sizeof(TD) == 2) {
    const __nv_bfloat162 lo = __floats2bfloat162_rn(a, b), hi = __floats2bfloat162_rn(c, d);
    uint2 u;
    u.x = *reinterpret_cast<const uint32_t*>(&lo);
    u.y = *reinterpret_cast<const uint32_t*>(&hi);
    *reinterpret_cast<uint2*>(dst) = u;
  } else {
    *reinterpret_cast<float4*>(dst) = make_float4(a, b, c, d);
  }
}

// Outer pass of the warp's 32 output channels h0 .. h0+31 of row b (lane = channel h0 + lane):
// u (the 96 interleaved in-projection channels 3h0 .. 3h0+95, splits summed in split order,
// rounded) into the outer ring, then per lane the outer FIR (oldest age first) of its channels
// 3h+j, rounded, x2 = z[3h] and x1v = round(z[3h+1] * z[3h+2]) for positions L0 .. L0+T-1.  The
// split partials are loaded as float4s by lanes 0..23 (one 16-byte chunk of the 96 channels each,
// every position of a split in flight) and handed to the channel lanes through `ub` (the warp's
// [DEC_T][96] TD buffer in shared memory: the rounded values are exact in TD).
template <typename TD, int DT>
__device__ __forceinline__ void dec_outer(const HyArgs<TD>& a, int b, int h0, int lane, int L0,
                                          const float (&wo)[3 * DEC_K0], TD* ub, float (&x2)[DT],
                                          float (&x1v)[DT]) {
  const int N3 = 3 * a.d;
  const size_t split_stride = static_cast<size_t>(a.M) * N3;
  const int T = a.T;
  const int cmask = a.cap_o - 1;  // the ring capacity is a power of two
  TD* ring = a.outer_ring + static_cast<size_t>(b) * a.cap_o * N3 + 3 * h0;
  // u window of the lane's channels: uw[j][0..1] = u at positions P-2, P-1 (zero before position 0)
  float uw[3][DEC_K0 - 1];
#pragma unroll
  for (int r = 0; r < DEC_K0 - 1; ++r) {
    const int P = L0 - (DEC_K0 - 1) + r;
#pragma unroll
    for (int j = 0; j < 3; ++j)
      uw[j][r] = P >= 0 ? to_f32(ring[static_cast<size_t>(P & cmask) * N3 + 3 * lane + j]) : 0.f;
  }
  if (lane < 24) {
    // positions t >= T load row T-1 again (unconditional loads stay in one block, all in flight)
    // and are never used
    float4 u4[DT];
#pragma unroll
    for (int t = 0; t < DT; ++t) u4[t] = make_float4(0.f, 0.f, 0.f, 0.f);
    const float* src = a.ws + static_cast<size_t>(b) * T * N3 + 3 * h0 + 4 * lane;
    for (int sp = 0; sp < a.splits; ++sp) {
      const float* ss = src + sp * split_stride;
#pragma unroll
      for (int t = 0; t < DT; ++t) {
        const float4 v = __ldg(reinterpret_cast<const float4*>(ss + static_cast<size_t>(min(t, T - 1)) * N3));
        u4[t].x += v.x;
        u4[t].y += v.y;
        u4[t].z += v.z;
        u4[t].w += v.w;
      }
    }
#pragma unroll
    for (int t = 0; t < DT; ++t) {
      const float r0 = round_to<TD>(u4[t].x), r1 = round_to<TD>(u4[t].y), r2 = round_to<TD>(u4[t].z),
                  r3 = round_to<TD>(u4[t].w);
      store4_td<TD>(ub + t * 96 + 4 * lane, r0, r1, r2, r3);
      if (t < T) store4_td<TD>(ring + static_cast<size_t>((L0 + t) & cmask) * N3 + 4 * lane, r0, r1, r2, r3);
    }
  }
  __syncwarp();
#pragma unroll
  for (int t = 0; t < DT; ++t) {
    x2[t] = 0.f;
    x1v[t] = 0.f;
    if (t < T) {
      const int P = L0 + t;
      float zq[3];
      const int cs = min(P, DEC_K0 - 1);
      const int base = a.prefill ? DEC_K0 - 1 : cs;
#pragma unroll
      for (int j = 0; j < 3; ++j) {
        const float un = to_f32(ub[t * 96 + 3 * lane + j]);
        // the weights of ages 2, 1, 0 are w[base-2], w[base-1], w[base] (selected, not indexed, so
        // that they stay in registers); age 2 appears only when cs = 2, where base = 2
        const float w0 = wo[j * DEC_K0], w1 = wo[j * DEC_K0 + 1], w2 = wo[j * DEC_K0 + 2];
        const float wb = base == 2 ? w1 : w0;
        const float wc = base == 2 ? w2 : (base == 1 ? w1 : w0);
        float z = 0.f;
        if (cs >= 2) z = fmaf(w0, uw[j][0], z);
        if (cs >= 1) z = fmaf(wb, uw[j][1], z);
        z = fmaf(wc, un, z);
        zq[j] = round_to<TD>(z);
        uw[j][0] = uw[j][1];
        uw[j][1] = un;
      }
      x2[t] = zq[0];
      x1v[t] = round_to<TD>(zq[1] * zq[2]);
    }
  }
}

// grid (d / 32, ceil(B / DEC_ROWS)), block (32, DEC_ROWS).  KI = inner filter length (7 or 128);
// DT = positions held in registers (the chunk length 13 of a verify block, or DT).  Shared
// memory: taps[32][tap_stride(KI)] f32 (channel c's weight of age a at taps[c][a]) | per warp
// x2s[DT][32] f32 (the gates, kept out of registers during the inner FIR) | per warp
// hist[KI-1+DT][32] TD (x1v by position, the oldest history position first) | per warp
// ub[DT][96] TD (the outer pass's exchange).
template <int KI, int DT, typename TD>
constexpr size_t fir_dec_smem() {
  return sizeof(float) * 32 * tap_stride(KI) + sizeof(float) * DEC_ROWS * DT * 32 +
         sizeof(TD) * DEC_ROWS * (KI - 1 + DT) * 32 + sizeof(TD) * DEC_ROWS * DT * 96;
}
template <typename TD, bool FLIP, int KI, int DT>
__global__ void __launch_bounds__(32 * DEC_ROWS) hyena_fir_dec_kernel(HyArgs<TD> a) {
  pdl_trigger();
  constexpr int H = KI - 1, WROWS = H + DT, KS = tap_stride(KI);
  extern __shared__ __align__(16) float sm[];
  float* taps = sm;
  float* x2s = taps + 32 * KS + threadIdx.y * DT * 32;
  TD* hist = reinterpret_cast<TD*>(taps + 32 * KS + DEC_ROWS * DT * 32) + threadIdx.y * WROWS * 32;
  TD* ub = reinterpret_cast<TD*>(taps + 32 * KS + DEC_ROWS * DT * 32) + DEC_ROWS * WROWS * 32 + threadIdx.y * DT * 96;
  const int lane = threadIdx.x, h0 = blockIdx.x * 32, h = h0 + lane;
  const int b = blockIdx.y * DEC_ROWS + threadIdx.y;
  // the taps are weights: stage them before waiting for the in-projection.  The full-window weight
  // of age a is w[a] for the flipped filter (the rows as they are: asynchronous 16-byte copies) and
  // w[K-1-a] otherwise (reversed rows)
  const float* iw = a.inner_w + static_cast<size_t>(h0) * KI;
  if constexpr (FLIP && KI % 4 == 0) {
    for (int i = threadIdx.y * 32 + lane; i < 32 * (KI / 4); i += 32 * DEC_ROWS) {
      const int c = i / (KI / 4), j = i - c * (KI / 4);
      cp_async16(taps + c * KS + 4 * j, iw + c * KI + 4 * j);
    }
    cp_async_commit();
  } else {
    for (int i = threadIdx.y * 32 + lane; i < 32 * KI; i += 32 * DEC_ROWS) {
      const int c = i / KI, k = i - c * KI;
      taps[c * KS + (FLIP ? k : H - k)] = __ldg(iw + i);
    }
  }
  for (int i = threadIdx.y * 32 + lane; i < 32 * (KS - KI); i += 32 * DEC_ROWS)
    taps[(i / (KS - KI)) * KS + KI + i % (KS - KI)] = 0.f;  // the padding a float4 read may touch
  float wo[3 * DEC_K0];
#pragma unroll
  for (int i = 0; i < 3 * DEC_K0; ++i) wo[i] = __ldg(a.short_w + static_cast<size_t>(3 * h) * DEC_K0 + i);
  const float Dg = FLIP ? __ldg(a.D + h) : 0.f;
  pdl_wait();
  if constexpr (FLIP && KI % 4 == 0) cp_async_wait<0>();
  __syncthreads();  // taps staged
  if (b >= a.M / a.T) return;
  const int L0 = a.len[b];
  const int T = a.T;
  // x1v history of the warp's 32 channels, positions L0-H .. L0-1 (zero before position 0), copied
  // asynchronously while the outer pass runs: one 16-byte chunk per copy, every copy in flight
  constexpr int CPR = 32 * static_cast<int>(sizeof(TD)) / 16;  // 16-byte chunks per history row
  const TD* ring_row = a.inner_ring + static_cast<size_t>(b) * a.cap_i * a.d + h0;
  for (int i = lane; i < H * CPR; i += 32) {
    const int r = i / CPR, c = i - r * CPR;
    const int P = L0 - H + r;
    TD* dst = hist + r * 32 + c * (16 / sizeof(TD));
    if (P >= 0)
      cp_async16(dst, ring_row + static_cast<size_t>(P & (a.cap_i - 1)) * a.d + c * (16 / sizeof(TD)));
    else
      *reinterpret_cast<int4*>(dst) = make_int4(0, 0, 0, 0);
  }
  cp_async_commit();
  {
    float x2[DT], x1v[DT];
    dec_outer<TD, DT>(a, b, h0, lane, L0, wo, ub, x2, x1v);
    TD* ring_w = a.inner_ring + static_cast<size_t>(b) * a.cap_i * a.d + h;
#pragma unroll
    for (int t = 0; t < DT; ++t) {
      // x1v is rounded to TD: its history copy holds it exactly; x2 waits in shared memory
      hist[(H + t) * 32 + lane] = from_f32<TD>(x1v[t]);
      x2s[t * 32 + lane] = x2[t];
      if (t < T) ring_w[static_cast<size_t>((L0 + t) & (a.cap_i - 1)) * a.d] = from_f32<TD>(x1v[t]);
    }
  }
  cp_async_wait<0>();
  __syncwarp();  // the history rows the other lanes copied
  float acc[DT];
#pragma unroll
  for (int t = 0; t < DT; ++t) acc[t] = 0.f;
  if (FLIP || a.prefill || L0 >= H) {
    // every position uses the full window (positions before 0 hold zeros, which add nothing):
    // acc[t] += w(age) * x(L0 + t - age) for age = H .. 0, the window rotating one position a step
    float win[DT];
#pragma unroll
    for (int t = 0; t < DT; ++t) win[t] = to_f32(hist[t * 32 + lane]);
    const float* tp = taps + lane * KS;
#pragma unroll
    for (int a4 = H / 4; a4 >= 0; --a4) {
      const float4 w4 = *reinterpret_cast<const float4*>(tp + 4 * a4);
      const float wv[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
      for (int e = 3; e >= 0; --e) {
        const int age = 4 * a4 + e;
        if (age > H) continue;
#pragma unroll
        for (int t = 0; t < DT; ++t) acc[t] = fmaf(wv[e], win[t], acc[t]);
        if (age > 0) {
#pragma unroll
          for (int t = 0; t < DT - 1; ++t) win[t] = win[t + 1];
          win[DT - 1] = to_f32(hist[(H + DT - age) * 32 + lane]);
        }
      }
    }
  } else {
    // unflipped filter on a history shorter than K-1 (a sequence's first positions outside
    // prefill): position P weights age a by w[min(P, K-1) - a]
    const float* wr = a.inner_w + static_cast<size_t>(h) * KI;
#pragma unroll
    for (int t = 0; t < DT; ++t) {
      if (t < T) {
        const int P = L0 + t, cs = min(P, H);
        float z = 0.f;
        for (int age = cs; age >= 0; --age) z = fmaf(__ldg(wr + cs - age), to_f32(hist[(H + t - age) * 32 + lane]), z);
        acc[t] = z;
      }
    }
  }
#pragma unroll
  for (int t = 0; t < DT; ++t) {
    if (t < T) {
      float z = acc[t];
      if (FLIP) z = fmaf(Dg, to_f32(hist[(H + t) * 32 + lane]), z);
      const float yv = round_to<TD>(x2s[t * 32 + lane] * round_to<TD>(z));
      a.y[static_cast<size_t>(b * T + t) * a.ld_y + h] = from_f32<TD>(yv);
    }
  }
}

// Outer pass of the IIR decode kernel: the warp's 8 output channels h0 .. h0+7 of row b, four
// lanes per channel (lane = 4 ch + q).  The 24 interleaved in-projection channels 3h0 .. 3h0+23 of
// every position are loaded as float4s spread over all lanes (three per lane and split, splits
// summed in split order), rounded, written to the outer ring and handed over through `ub` (the
// warp's [DEC_T][24] TD buffer); then every lane runs its channel's outer FIR with the arithmetic of
// dec_outer (the four lanes of a channel compute the same values).
template <typename TD>
__device__ __forceinline__ void dec_outer8(const HyArgs<TD>& a, int b, int h0, int ch, int lane, int L0,
                                           const float (&wo)[3 * DEC_K0], TD* ub, float (&x2)[DEC_T],
                                           float (&x1v)[DEC_T]) {
  constexpr int C4 = 6;  // float4 chunks of the 24 channels
  const int N3 = 3 * a.d;
  const size_t split_stride = static_cast<size_t>(a.M) * N3;
  const int T = a.T;
  const int cmask = a.cap_o - 1;  // the ring capacity is a power of two
  TD* ring = a.outer_ring + static_cast<size_t>(b) * a.cap_o * N3 + 3 * h0;
  float uw[3][DEC_K0 - 1];
#pragma unroll
  for (int r = 0; r < DEC_K0 - 1; ++r) {
    const int P = L0 - (DEC_K0 - 1) + r;
#pragma unroll
    for (int j = 0; j < 3; ++j)
      uw[j][r] = P >= 0 ? to_f32(ring[static_cast<size_t>(P & cmask) * N3 + 3 * ch + j]) : 0.f;
  }
  {
    // item i = t * C4 + c (position t, chunk c); lane takes i = lane, lane + 32, lane + 64; positions
    // t >= T load row T-1 again (all loads in flight) and are never used
    float4 u4[3];
#pragma unroll
    for (int k = 0; k < 3; ++k) u4[k] = make_float4(0.f, 0.f, 0.f, 0.f);
    const float* src = a.ws + static_cast<size_t>(b) * T * N3 + 3 * h0;
    for (int sp = 0; sp < a.splits; ++sp) {
      const float* ss = src + sp * split_stride;
#pragma unroll
      for (int k = 0; k < 3; ++k) {
        const int i = lane + 32 * k, t = i / C4, c = i - t * C4;
        const float4 v = __ldg(reinterpret_cast<const float4*>(ss + static_cast<size_t>(min(t, T - 1)) * N3 + 4 * c));
        u4[k].x += v.x;
        u4[k].y += v.y;
        u4[k].z += v.z;
        u4[k].w += v.w;
      }
    }
#pragma unroll
    for (int k = 0; k < 3; ++k) {
      const int i = lane + 32 * k, t = i / C4, c = i - t * C4;
      const float r0 = round_to<TD>(u4[k].x), r1 = round_to<TD>(u4[k].y), r2 = round_to<TD>(u4[k].z),
                  r3 = round_to<TD>(u4[k].w);
      store4_td<TD>(ub + t * 24 + 4 * c, r0, r1, r2, r3);
      if (t < T) store4_td<TD>(ring + static_cast<size_t>((L0 + t) & cmask) * N3 + 4 * c, r0, r1, r2, r3);
    }
  }
  __syncwarp();
#pragma unroll
  for (int t = 0; t < DEC_T; ++t) {
    x2[t] = 0.f;
    x1v[t] = 0.f;
    if (t < T) {
      const int P = L0 + t;
      float zq[3];
      const int cs = min(P, DEC_K0 - 1);
      const int base = a.prefill ? DEC_K0 - 1 : cs;
#pragma unroll
      for (int j = 0; j < 3; ++j) {
        const float un = to_f32(ub[t * 24 + 3 * ch + j]);
        const float w0 = wo[j * DEC_K0], w1 = wo[j * DEC_K0 + 1], w2 = wo[j * DEC_K0 + 2];
        const float wb = base == 2 ? w1 : w0;
        const float wc = base == 2 ? w2 : (base == 1 ? w1 : w0);
        float z = 0.f;
        if (cs >= 2) z = fmaf(w0, uw[j][0], z);
        if (cs >= 1) z = fmaf(wb, uw[j][1], z);
        z = fmaf(wc, un, z);
        zq[j] = round_to<TD>(z);
        uw[j][0] = uw[j][1];
        uw[j][1] = un;
      }
      x2[t] = zq[0];
      x1v[t] = round_to<TD>(zq[1] * zq[2]);
    }
  }
}

// grid (d / 8, ceil(B / DEC_ROWS)), block (32, DEC_ROWS): four lanes per channel and row, lane q
// holding poles 4q .. 4q+3 (the four pole-group threads of hyena_iir_kernel); the residue sum is
// ((group 0 + group 1) + (group 2 + group 3)) by two butterfly steps, as in the general kernel.
// The poles and residues (weights) are loaded before the dependency wait.  Shared memory: per warp
// ub[DEC_T][24] TD.
template <typename TD>
__global__ void __launch_bounds__(32 * DEC_ROWS) hyena_iir_dec_kernel(HyArgs<TD> a) {
  pdl_trigger();
  constexpr int S = 16;
  extern __shared__ __align__(16) float sm[];
  const int lane = threadIdx.x, ch = lane >> 2, q = lane & 3;
  const int h0 = blockIdx.x * 8, h = h0 + ch;
  const int b = blockIdx.y * DEC_ROWS + threadIdx.y;
  const int d = a.d;
  TD* ub = reinterpret_cast<TD*>(sm) + threadIdx.y * DEC_T * 24;
  float p[4], r[4];
  load_vec<4>(a.poles + static_cast<size_t>(h) * S + 4 * q, p);
  load_vec<4>(a.residues + static_cast<size_t>(h) * S + 4 * q, r);
  float wo[3 * DEC_K0];
#pragma unroll
  for (int i = 0; i < 3 * DEC_K0; ++i) wo[i] = __ldg(a.short_w + static_cast<size_t>(3 * h) * DEC_K0 + i);
  const float Dg = a.D[h];
  pdl_wait();
  if (b >= a.M / a.T) return;  // (whole warps: b is the warp's row)
  const int L0 = a.len[b];
  // the carried state first, so that its loads are in flight with the outer pass
  float st[4];
  if (L0 > 0) {
    load_vec<4>(a.s_all + ((static_cast<size_t>(b) * a.slots + a.iir_cur[b]) * d + h) * S + 4 * q, st);
  } else {
#pragma unroll
    for (int j = 0; j < 4; ++j) st[j] = 0.f;
  }
  float x2[DEC_T], x1v[DEC_T];
  dec_outer8(a, b, h0, ch, lane, L0, wo, ub, x2, x1v);
#pragma unroll
  for (int t = 0; t < DEC_T; ++t) {
    if (t < a.T) {
      float part = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        st[j] = fmaf(p[j], st[j], x1v[t]);
        part = fmaf(r[j], st[j], part);
      }
      const float pair = part + __shfl_xor_sync(0xffffffffu, part, 1);
      const float tot = pair + __shfl_xor_sync(0xffffffffu, pair, 2);
      if (q == 0) {
        const float yv = round_to<TD>(x2[t] * (tot + Dg * x1v[t]));
        a.y[static_cast<size_t>(b * a.T + t) * a.ld_y + h] = from_f32<TD>(yv);
      }
      if (a.retain) store_vec<4>(a.s_all + ((static_cast<size_t>(b) * a.slots + t) * d + h) * S + 4 * q, st);
    }
  }
  if (!a.retain) store_vec<4>(a.s_all + ((static_cast<size_t>(b) * a.slots + 0) * d + h) * S + 4 * q, st);
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
  const int d = m->dl;  // this rank's channels
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
  EVS_CHECK_ARG(a.K0 >= 1 && a.K0 - 1 + TS <= UW, "short filter too long for the outer-FIR window");
  // chunks of at most DEC_T tokens with the Evo2 filter shapes: the register-resident decode path
  // (same bits as the general kernels below)
  const bool dec_shape = B >= DEC_MIN_ROWS && T <= DEC_T && a.K0 == DEC_K0 &&
                         (L.kind == EVS_LAYER_HCL ? a.S == 16 : (a.K == 7 || a.K == 128));
  if (dec_shape) {
    const dim3 dgrid(d / 32, (B + DEC_ROWS - 1) / DEC_ROWS), dblock(32, DEC_ROWS);
    if (L.kind == EVS_LAYER_HCL) {
      EVS_CHECK_ARG(d % 8 == 0, "IIR channels must be a multiple of 8");
      EVS_CUDA_TRY(evs_launch(hyena_iir_dec_kernel<TD>, dim3(d / 8, (B + DEC_ROWS - 1) / DEC_ROWS), dblock,
                              sizeof(TD) * DEC_ROWS * DEC_T * 24, st, s->use_pdl(), a));
    } else {
      auto launch = [&](auto kern, size_t smem) -> int {
        EVS_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
        EVS_CUDA_TRY(evs_launch(kern, dgrid, dblock, smem, st, s->use_pdl(), a));
        return EVS_OK;
      };
      // 13 positions (a verify block of gamma = 12) held exactly, else DEC_T with the tail unused
      const bool t13 = T == 13;
      const bool flip = L.kind == EVS_LAYER_HCM;
      if (a.K == 128) {
        if (flip)
          EVS_TRY(t13 ? launch(hyena_fir_dec_kernel<TD, true, 128, 13>, fir_dec_smem<128, 13, TD>())
                      : launch(hyena_fir_dec_kernel<TD, true, 128, DEC_T>, fir_dec_smem<128, DEC_T, TD>()));
        else
          EVS_TRY(t13 ? launch(hyena_fir_dec_kernel<TD, false, 128, 13>, fir_dec_smem<128, 13, TD>())
                      : launch(hyena_fir_dec_kernel<TD, false, 128, DEC_T>, fir_dec_smem<128, DEC_T, TD>()));
      } else {
        if (flip)
          EVS_TRY(t13 ? launch(hyena_fir_dec_kernel<TD, true, 7, 13>, fir_dec_smem<7, 13, TD>())
                      : launch(hyena_fir_dec_kernel<TD, true, 7, DEC_T>, fir_dec_smem<7, DEC_T, TD>()));
        else
          EVS_TRY(t13 ? launch(hyena_fir_dec_kernel<TD, false, 7, 13>, fir_dec_smem<7, 13, TD>())
                      : launch(hyena_fir_dec_kernel<TD, false, 7, DEC_T>, fir_dec_smem<7, DEC_T, TD>()));
      }
    }
    EVS_CUDA_TRY(cudaGetLastError());
    evs_count_launch(1);
    return EVS_OK;
  }
  dim3 grid(d / CH, B);
  const size_t outer_floats = static_cast<size_t>(UW) * C3 + TS * C3 + C3 * a.K0;
  if (L.kind == EVS_LAYER_HCL) {
    const size_t smem = sizeof(float) * outer_floats;
    auto launch = [&](auto kern) -> int {
      EVS_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
      EVS_CUDA_TRY(evs_launch(kern, grid, dim3(HY_THREADS), smem, st, s->use_pdl(), a));
      return EVS_OK;
    };
    switch (a.S / 4) {
      case 4: EVS_TRY(launch(hyena_iir_kernel<TD, 4>)); break;
      case 8: EVS_TRY(launch(hyena_iir_kernel<TD, 8>)); break;
      case 2: EVS_TRY(launch(hyena_iir_kernel<TD, 2>)); break;
      case 1: EVS_TRY(launch(hyena_iir_kernel<TD, 1>)); break;
      default: EVS_CHECK_ARG(false, "state_size must be 4, 8, 16 or 32");
    }
  } else {
    int win = 1;
    while (win < a.K - 1 + TS) win <<= 1;
    const size_t smem = sizeof(float) * (outer_floats + static_cast<size_t>(CH) * tap_stride(a.K) + TS * CH) +
                        sizeof(TD) * static_cast<size_t>(win) * CH;
    EVS_CHECK_RANGE(smem <= 220 * 1024, "FIR filter too long for the shared-memory window");
    auto launch = [&](auto kern) -> int {
      EVS_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
      EVS_CUDA_TRY(evs_launch(kern, grid, dim3(HY_FIR_THREADS), smem, st, s->use_pdl(), a, win));
      return EVS_OK;
    };
    if (L.kind == EVS_LAYER_HCM)
      EVS_TRY(launch(hyena_fir_kernel<TD, true>));
    else
      EVS_TRY(launch(hyena_fir_kernel<TD, false>));
  }
  EVS_CUDA_TRY(cudaGetLastError());
  evs_count_launch(1);
  return EVS_OK;
}

}  // namespace

int launch_hyena(const evs_model* m, evs_state* s, int layer, int B, int T, int splits, int prefill, int retain,
                 cudaStream_t st) {
  EVS_CHECK_ARG(m->dl % CH == 0, "d_model / tp_world must be a multiple of 32");
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
  const int d = m->dl;  // this rank's channels
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
    const int HD2 = 2 * m->Hl * m->cfg.head_dim;
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
