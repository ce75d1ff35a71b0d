// Internal structures of libevspark_sm100 (not part of the C ABI).
#pragma once

#include <atomic>
#include <vector>

#include "common.cuh"

// A kernel's dynamic shared-memory opt-in (cudaFuncSetAttribute) belongs to one device context:
// each launch site keeps a bit per device that has it, set once per device, any thread.
inline int smem_attr_once(std::atomic<unsigned long long>& done, const void* kern, int bytes) {
  int dev = 0;
  EVS_CUDA_TRY(cudaGetDevice(&dev));
  const unsigned long long bit = dev < 64 ? (1ull << dev) : 0ull;
  if (bit != 0 && (done.load(std::memory_order_acquire) & bit) != 0) return EVS_OK;
  EVS_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  done.fetch_or(bit, std::memory_order_acq_rel);
  return EVS_OK;
}

// GEMM tile geometry (tcgen05 path): 128 weight rows x 64 K per stage, tokens per MMA = NT
constexpr int GEMM_BM = 128;
constexpr int GEMM_BK = 64;
constexpr int TOK_TILE = 16;  // token rows per decode tile (MMA N)
// token tiles (MMA N) of the projection kernel, chosen from the token count M; index 3 is the
// serial-split kernel's narrow tile (its wide tile is GEMM_NT[2])
constexpr int GEMM_NT[4] = {16, 64, 128, 96};
constexpr int GEMM_NMAPS = 4;  // activation maps per operand (box rows GEMM_NT[i])
constexpr int ATTN_BLOCK = 64;  // keys per attention partial (aligned at absolute positions)
constexpr int EVS_TP_MAX = 8;   // channel-sharding ranks
constexpr int ATTN_TCAP = 16;   // split-KV attention handles chunks of at most this many queries
constexpr int EVS_RETAIN_MAX = 64;  // tokens per row of a retained forward (per-position IIR slots)

// HBM layout of the per-sequence state ------------------------------------
//   outer FIR history ring   [B][cap_outer][3d]   data dtype  (positions mod cap_outer)
//   inner FIR history ring   [B][cap_inner][d]    data dtype  (SE / MR layers)
//   IIR per-position states  [B][iir_slots][d][S] fp32        (slot = block index)
//   KV cache                 [B][Lmax][2][H][Dh]  data dtype
//   capture ring             [B][ring_len][d]     fp32        (injection-layer outputs)
struct LayerDev {
  int kind = 0;
  const void* pre_norm = nullptr;
  const void* post_norm = nullptr;
  const void* w_in = nullptr;
  const void* short_w = nullptr;
  const void* inner_w = nullptr;
  const void* D = nullptr;
  const void* log_poles = nullptr;
  const void* residues = nullptr;
  const void* w_out = nullptr;
  const void* w_qkv = nullptr;
  const void* w_o = nullptr;
  const void* w1 = nullptr;
  const void* w2 = nullptr;
  const void* w3 = nullptr;
  float* poles = nullptr;  // owned: exp(log_poles) fp32 [d, S]
  CUtensorMap tm_in, tm_out, tm_qkv, tm_o, tm_w1, tm_w2, tm_w3;
  int64_t numel[EVS_W_NUM_SLOTS] = {0};
};

struct evs_model {
  evs_model_config cfg;
  int device = 0;
  // channel sharding: this rank's Hyena channels, attention heads and MLP features
  int tp_world = 1, tp_rank = 0;
  int dl = 0, Hl = 0, Fl = 0;
  bool finalized = false;
  const void* embed = nullptr;
  const void* final_norm = nullptr;
  int64_t embed_numel = 0, final_norm_numel = 0;
  CUtensorMap tm_embed;
  LayerDev L[EVS_MAX_LAYERS];
  int n_capture = 0;
  int capture_layer[4] = {-1, -1, -1, -1};
  size_t elem() const { return cfg.dtype == EVS_DTYPE_BF16 ? 2 : 4; }
  int capture_slot(int layer) const {
    for (int c = 0; c < n_capture; ++c)
      if (capture_layer[c] == layer) return c;
    return -1;
  }
};

struct HyenaDev {
  void* outer_ring = nullptr;
  void* inner_ring = nullptr;
  float* s_all = nullptr;
};

struct evs_state {
  const evs_model* m = nullptr;
  int max_batch = 0, max_seqlen = 0, max_chunk = 0;
  int cap_outer = 0, cap_hcs = 0, cap_hcm = 0, iir_slots = 0, ring_len = 0;
  int m_cap = 0;      // max token rows per call = max_batch * max_chunk (padded to TOK_TILE)
  int ld_act = 0;     // row stride (elements) of the activation buffer = max(d, F)
  size_t ws_floats = 0;  // capacity of the split-K workspace
  int attn_blocks = 0;   // ceil(max_seqlen / ATTN_BLOCK)
  int attn_tcap = 0;     // queries per call of the split-KV attention (longer chunks use the fused kernel)
  // per-row bookkeeping (device truth) and a host upper bound of the lengths
  int32_t* d_len = nullptr;      // [B] tokens consumed
  int32_t* d_len0 = nullptr;     // [B] lengths before the last retained forward
  int32_t* d_iir_cur = nullptr;  // [B] IIR slot holding the current state
  int32_t* d_chunk = nullptr;    // [1] length of the last retained chunk (0: no stash)
  std::vector<int32_t> h_len;    // host upper bound of d_len
  int h_chunk = 0;               // host copy of the last retained chunk length
  HyenaDev hy[EVS_MAX_LAYERS];
  void* kv[EVS_MAX_LAYERS] = {nullptr};
  float* cap_ring[4] = {nullptr, nullptr, nullptr, nullptr};
  // capture tags [B][ring_len]: which forward wrote each capture-ring row (state id, row, forward
  // sequence number; every capture layer of a forward gets the same tag), so that a consumer that
  // keeps values derived from ring rows (the drafter's projected context) can tell them current
  unsigned long long* cap_tag = nullptr;
  unsigned long long* d_fwd_seq = nullptr;  // [1] forwards run on this state (device counter)
  unsigned long long tag_hi = 0;            // this state's id, in the tag's top bits
  // scratch
  float* resid = nullptr;      // [m_cap][d] fp32 residual stream
  void* act = nullptr;         // [m_cap][ld_act] data dtype: GEMM B operand
  float* ws = nullptr;         // split-K partials [splits][m][n] fp32
  void* qrot = nullptr;        // [m_cap][d] data dtype rotated queries
  float* attn_part = nullptr;  // [B][H][attn_blocks][attn_tcap][Dh+2] fp32
  int64_t* ids_scratch = nullptr;  // [m_cap] chunk ids of a strided prefill
  EvsDevErr* d_err = nullptr;
  // channel sharding: partial sums of the row-parallel projections, double-buffered, and an
  // epoch flag, in one region shared with the peers over CUDA IPC (tp_base[rank] = own region)
  void* tp_region = nullptr;
  size_t tp_buf_bytes = 0;  // one of the two partial-sum buffers (splits x m_cap x d fp32)
  char* tp_base[EVS_TP_MAX] = {nullptr};
  bool tp_connected = false;
  long long tp_epoch = 0;  // row-parallel reductions issued so far (same count on every rank)
  // activation buffer as GEMM B operand, K = d, K = local F and K = local d, box rows GEMM_NT[i]
  CUtensorMap tm_act_d[GEMM_NMAPS], tm_act_f[GEMM_NMAPS], tm_act_l[GEMM_NMAPS];
  // bf16: the w1/w2 projection's fused SwiGLU output [m_cap][F] (its own buffer: the projection's
  // other CTAs still read act while one CTA's epilogue writes), read by w3 through tm_gate
  void* gate = nullptr;
  CUtensorMap tm_gate[GEMM_NMAPS];
  // profiling (evs_profile_start / evs_profile_stop)
  struct ProfRec {
    int kind;
    cudaEvent_t a, b;
    double bytes;
  };
  bool prof = false;
  bool pdl = true;  // programmatic dependent launch inside a forward (off while profiling)
  bool use_pdl() const { return pdl && !prof; }
  std::vector<ProfRec> prof_recs;
  std::vector<cudaEvent_t> ev_pool;
  size_t ev_used = 0;
  std::vector<void*> owned;        // [0] persistent arenas, [1] scratch
  std::vector<size_t> owned_bytes;
};

// ---- launchers (stream-ordered; return EVS_* status) ----
// GEMM partial sums ws[split][tok][n] over the weight rows; dual: w1/w2 interleaved per 64 rows
struct GemmPlan {
  int N, K, M, splits, dual;
  int kchunk = 0;  // fp32 path: K columns per split (multiple of 128)
};
GemmPlan gemm_plan(const evs_model* m, int N, int K, int M, int dual);
GemmPlan gemm_plan_f32(int N, int K, int M, int dual);
GemmPlan gemm_plan_f32_drafter(int N, int K, int M);
// out[m][n] = sum of the split partials (in split order) + bias[n]
int launch_reduce_splits(const float* ws, int splits, int M, int N, const float* bias, float* out, cudaStream_t st,
                         bool pdl = false, const int32_t* m_dev = nullptr,
                         int m_hint = 0);
// pdl: launch with programmatic stream serialization (see pdl_wait)
// tmB: three maps of the activations with box rows GEMM_NT[0..2]; the tile is chosen from p.M
int gemm_tile_index(int M);
// swiglu_act: with the dual w1/w2 tile and one split, write silu(w1 x) * (w2 x) as bf16 rows of
// stride ld_act there instead of partial sums to ws
int launch_gemm_tc(const CUtensorMap* tmA, const CUtensorMap* tmA2, const CUtensorMap* tmB, const GemmPlan& p,
                   float* ws, EvsDevErr* err, cudaStream_t st, bool pdl = false, void* swiglu_act = nullptr,
                   int ld_act = 0);
// large token counts: every split in one CTA per (token tile, weight tile), the splits' sum stored
// as the only split (the same bits as the split partials summed in order); see gemm_serial
bool gemm_serial(const GemmPlan& p);
int launch_gemm_tc_serial(const CUtensorMap* tmA, const CUtensorMap* tmA2, const CUtensorMap* tmB, const GemmPlan& p,
                          float* ws, EvsDevErr* err, cudaStream_t st, bool pdl = false);
// m_dev: optional device-side row count (at most p.M, which sizes the grid)
int launch_gemm_simt(const void* W, const void* W2, const void* X, int ldx, int dtype, const GemmPlan& p, float* ws,
                     cudaStream_t st, bool pdl = false, const int32_t* m_dev = nullptr, int m_hint = 0);
// several fp32 projections of one shape and plan in one launch (at most SK_MAX_JOBS): job j
// computes the partials of W_j x row m into its own ws_j[split][M_j][N], row m being X0[m] below
// msplit and X1[m - msplit] from there; each CTA does gemm_skinny_f32_kernel's arithmetic
constexpr int SK_MAX_JOBS = 3;
struct SkJob {
  const float* W;
  const float* X0;
  const float* X1;
  float* ws;
  const int32_t* m_dev;  // optional device-side row count
  int msplit, M;
};
struct SkJobs {
  SkJob j[SK_MAX_JOBS];
};
int launch_gemm_simt_jobs(const SkJobs& jobs, int n_jobs, int ldx, const GemmPlan& p, cudaStream_t st, bool pdl,
                          int m_hint = 0);
int make_tmap_2d_bf16(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint64_t row_stride_bytes,
                      uint32_t box_inner, uint32_t box_outer);

// row kernels
int launch_embed_norm(const evs_model* m, evs_state* s, const int64_t* ids, int M, const float* scale,
                      cudaStream_t st);
// partial sums a residual + RMSNorm adds, rank by rank in rank order: buf[r] + split x M x d fp32;
// for R > 1 the kernel first waits (bounded) until every rank's flag has reached epoch
struct TpPartials {
  const float* buf[EVS_TP_MAX];
  const long long* flag[EVS_TP_MAX];
  int R;
  long long epoch;
};
int launch_res_add_norm(const evs_model* m, evs_state* s, int M, int splits, const TpPartials& parts,
                        const float* scale, int capture_slot, int T, cudaStream_t st);
// capture tag of row b: state id | row | forward sequence number
constexpr int EVS_TAG_SEQ_BITS = 34, EVS_TAG_ROW_BITS = 10;
__host__ __device__ inline unsigned long long evs_capture_tag(unsigned long long tag_hi, int b,
                                                              unsigned long long seq) {
  return tag_hi | (static_cast<unsigned long long>(b) << EVS_TAG_SEQ_BITS) |
         (seq & ((1ull << EVS_TAG_SEQ_BITS) - 1));
}
// publish this rank's partial sums of reduction `epoch` to the peers (after the producing kernel)
int launch_tp_reduce_signal(evs_state* s, float* buf, int splits, int M, long long epoch, cudaStream_t st);
int launch_swiglu(const evs_model* m, evs_state* s, int M, int splits, cudaStream_t st);
// logits rows go to out[(b * out_T + t0 + t) * V] (or out[b * V] for the last row when last_only)
int launch_logits(const evs_model* m, evs_state* s, int M, int T, int splits, float* logits, int out_T, int t0,
                  int last_only, cudaStream_t st);
int launch_bookkeeping(evs_state* s, int B, int T, int retain, cudaStream_t st);
int launch_poles(const float* log_poles, float* poles, int n, cudaStream_t st);

// Hyena mixer (outer FIR + inner FIR / IIR), reads in-projection partials from s->ws
int launch_hyena(const evs_model* m, evs_state* s, int layer, int B, int T, int splits, int prefill, int retain,
                 cudaStream_t st);
int launch_rollback(evs_state* s, const int32_t* k, int B, cudaStream_t st);
int launch_state_export(const evs_state* s, int layer, int which, int row, int width, void* dst, cudaStream_t st);

// attention: rope + KV append + split-KV partials + ordered combine (output into s->act)
int launch_attention(const evs_model* m, evs_state* s, int layer, int B, int T, int splits, int kv_blocks,
                     cudaStream_t st);

// verification
int launch_transform(const void* logits, int logits_fp64, int rows, int V, double temperature, int top_k,
                     double* probs, cudaStream_t st);
int launch_sample(const double* rows, int n, int V, const double* u, int64_t* out, cudaStream_t st);
int launch_verify(const double* p, const double* q, const int64_t* x, const double* u, int B, int gamma, int V,
                  int greedy, int32_t* accepted, int64_t* tokens, int32_t* info, cudaStream_t st);
int launch_verify_multicand(const double* p, const double* q, const int64_t* x, const double* u, int B, int gamma,
                            int V, int greedy, int64_t* tokens, int32_t* info, cudaStream_t st);
