// evs_gemm_bf16_noalloc: the split-K tcgen05 projection for callers that must not allocate.
//
// Some hosts cannot call cudaMalloc at the moment they need a projection: a serving engine that
// has already carved all device memory into its own pool, code running while a stream is being
// captured (allocation would end the capture), or a plugin whose host forbids allocation after
// start-up.  For them this entry point keeps its split-K partial sums in a fixed file-scope device
// array instead of caller- or library-allocated scratch.
//
// Limits and behaviour:
//   * the array holds EVS_NOALLOC_SCRATCH_FLOATS fp32 values (4 MiB); a call needs
//     splits * M * N of them and is rejected with EVS_ERANGE beyond that;
//   * every GPU that loads the library keeps the array until the process exits;
//   * each call fully overwrites the part of the array it uses before reading it, so nothing
//     has to start at zero; the array keeps the last call's partial sums;
//   * all calls share the one array: calls that may overlap on the GPU (different streams
//     without ordering, different host threads) race on it — serialise them;
//   * the first call on a device looks up the array's device address with
//     cudaGetSymbolAddress (the array's name in host code is only a host-side stand-in); make
//     that first call before any stream capture begins;
//   * a file-scope device error word sits beside the array: each call clears it, the projection
//     records a timed-out wait there, and the reduction then writes NaN to every output value
//     instead of adding partial sums that a previous call may have left behind.
#include <mutex>
#include <string>

#include "internal.hpp"

#define EVS_NOALLOC_SCRATCH_FLOATS (1u << 20)

static __device__ __align__(256) float g_noalloc_scratch[EVS_NOALLOC_SCRATCH_FLOATS];
static __device__ EvsDevErr g_noalloc_err;

namespace {

constexpr int kMaxDevices = 64;
std::mutex g_mu;
float* g_scratch_dev[kMaxDevices] = {nullptr};
EvsDevErr* g_err_dev[kMaxDevices] = {nullptr};

int symbol_address(void** p, const void* symbol) {
  const cudaError_t e = cudaGetSymbolAddress(p, symbol);
  if (e != cudaSuccess || *p == nullptr) {
    evs_set_last_error(EVS_ECUDA, e != cudaSuccess ? cudaGetErrorString(e) : "null symbol address");
    return EVS_ECUDA;
  }
  return EVS_OK;
}

// device addresses of g_noalloc_scratch and g_noalloc_err on the current device (looked up once
// per device, with that device current)
int noalloc_buffers(float** ws, EvsDevErr** err) {
  int dev = 0;
  EVS_CUDA_TRY(cudaGetDevice(&dev));
  EVS_CHECK_RANGE(dev >= 0 && dev < kMaxDevices, "device index beyond the no-alloc scratch table");
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_scratch_dev[dev] == nullptr) {
    void *p = nullptr, *q = nullptr;
    EVS_TRY(symbol_address(&p, reinterpret_cast<const void*>(&g_noalloc_scratch)));
    EVS_TRY(symbol_address(&q, reinterpret_cast<const void*>(&g_noalloc_err)));
    g_err_dev[dev] = static_cast<EvsDevErr*>(q);
    g_scratch_dev[dev] = static_cast<float*>(p);
  }
  *ws = g_scratch_dev[dev];
  *err = g_err_dev[dev];
  return EVS_OK;
}

// out[m][n] = sum over splits, in split order, of the partials [split][m][n]; NaN everywhere when
// the projection recorded an error (its partial sums may be incomplete or a previous call's)
__global__ void noalloc_reduce_kernel(const float* __restrict__ ws, int splits, int MN, const EvsDevErr* err,
                                      float* __restrict__ out) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= MN) return;
  if (err->code != 0) {
    out[i] = __int_as_float(0x7fc00000);
    return;
  }
  float acc = 0.f;
  for (int sp = 0; sp < splits; ++sp) acc += ws[static_cast<size_t>(sp) * MN + i];
  out[i] = acc;
}

}  // namespace

extern "C" EVS_API int evs_gemm_bf16_noalloc(const void* W, const void* X, float* out, int N, int K, int M,
                                            cudaStream_t st) {
  EVS_CHECK_ARG(W && X && out, "null argument");
  EVS_CHECK_ARG(N % GEMM_BM == 0 && K % GEMM_BK == 0 && M >= 1 && M <= 4096, "bad GEMM shape");
  GemmPlan p{N, K, M, 1, 0};
  const int kblocks = K / GEMM_BK, tiles = N / GEMM_BM;
  while (tiles * p.splits < 148 && p.splits < kblocks) ++p.splits;
  const size_t need = static_cast<size_t>(p.splits) * M * N;
  if (need > EVS_NOALLOC_SCRATCH_FLOATS) {
    evs_set_last_error(EVS_ERANGE,
                       ("evs_gemm_bf16_noalloc: needs " + std::to_string(need) +
                        " fp32 scratch values (splits*M*N), the fixed array holds " +
                        std::to_string(EVS_NOALLOC_SCRATCH_FLOATS))
                           .c_str());
    return EVS_ERANGE;
  }
  float* ws = nullptr;
  EvsDevErr* err = nullptr;
  EVS_TRY(noalloc_buffers(&ws, &err));
  EVS_CUDA_TRY(cudaMemsetAsync(err, 0, sizeof(EvsDevErr), st));
  CUtensorMap ta, tb[3];
  EVS_TRY(make_tmap_2d_bf16(&ta, W, K, N, static_cast<uint64_t>(K) * 2, GEMM_BK, GEMM_BM));
  for (int t = 0; t < 3; ++t)
    EVS_TRY(make_tmap_2d_bf16(&tb[t], X, K, M, static_cast<uint64_t>(K) * 2, GEMM_BK, GEMM_NT[t]));
  EVS_TRY(launch_gemm_tc(&ta, nullptr, tb, p, ws, err, st));
  const int MN = M * N;
  noalloc_reduce_kernel<<<(MN + 255) / 256, 256, 0, st>>>(ws, p.splits, MN, err, out);
  EVS_CUDA_TRY(cudaGetLastError());
  evs_count_launch(1);
  return EVS_OK;
}
