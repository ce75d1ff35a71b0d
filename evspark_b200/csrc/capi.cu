// C ABI entry points: model / state handles and the layer-loop orchestration of one forward.
#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <cstring>
#include <string>

#include "internal.hpp"

namespace {

thread_local std::string g_last_error = "";

int next_pow2(int x) {
  int p = 1;
  while (p < x) p <<= 1;
  return p;
}

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// element count of a slot on this rank (0 = slot unused); sharded slots use the local widths
int64_t expected_numel(const evs_model* m, int kind, int slot) {
  const evs_model_config& c = m->cfg;
  const int64_t D = c.d_model, d = m->dl, F = m->Fl, S = c.state_size;
  const bool hy = kind != EVS_LAYER_MHA;
  switch (slot) {
    case EVS_W_PRE_NORM:
    case EVS_W_POST_NORM: return D;
    case EVS_W_IN: return hy ? 3 * d * D : 0;
    case EVS_W_SHORT: return hy ? 3 * d * c.short_filter_length : 0;
    case EVS_W_INNER:
      return kind == EVS_LAYER_HCS ? d * c.hcs_filter_length : (kind == EVS_LAYER_HCM ? d * c.hcm_filter_length : 0);
    case EVS_W_D: return (kind == EVS_LAYER_HCM || kind == EVS_LAYER_HCL) ? d : 0;
    case EVS_W_LOG_POLES:
    case EVS_W_RESIDUES: return kind == EVS_LAYER_HCL ? d * S : 0;
    case EVS_W_OUT: return hy ? D * d : 0;
    case EVS_W_QKV: return hy ? 0 : 3 * d * D;
    case EVS_W_O: return hy ? 0 : D * d;
    case EVS_W_W1:
    case EVS_W_W2: return F * D;
    case EVS_W_W3: return D * F;
    default: return 0;
  }
}

const void** slot_ptr(LayerDev& L, int slot) {
  switch (slot) {
    case EVS_W_PRE_NORM: return &L.pre_norm;
    case EVS_W_POST_NORM: return &L.post_norm;
    case EVS_W_IN: return &L.w_in;
    case EVS_W_SHORT: return &L.short_w;
    case EVS_W_INNER: return &L.inner_w;
    case EVS_W_D: return &L.D;
    case EVS_W_LOG_POLES: return &L.log_poles;
    case EVS_W_RESIDUES: return &L.residues;
    case EVS_W_OUT: return &L.w_out;
    case EVS_W_QKV: return &L.w_qkv;
    case EVS_W_O: return &L.w_o;
    case EVS_W_W1: return &L.w1;
    case EVS_W_W2: return &L.w2;
    case EVS_W_W3: return &L.w3;
    default: return nullptr;
  }
}

// one GEMM: bf16 -> tcgen05 (TMA maps), fp32 -> SIMT
// out: partial sums [splits][M][N] (s->ws, or a shared buffer of a row-parallel projection)
int gemm(const evs_model* m, evs_state* s, const CUtensorMap* tA, const CUtensorMap* tA2, const void* W,
         const void* W2, int N, int K, int M, int dual, float* out, size_t out_floats, cudaStream_t st, int* splits,
         const CUtensorMap* tB_override = nullptr) {
  GemmPlan p = gemm_plan(m, N, K, M, dual);
  EVS_CHECK_RANGE(static_cast<size_t>(p.splits) * M * N <= out_floats, "split-K workspace too small");
  *splits = p.splits;
  if (m->cfg.dtype == EVS_DTYPE_BF16) {
    const CUtensorMap* tB =
        tB_override ? tB_override : (K == m->cfg.d_model ? s->tm_act_d : (K == m->Fl ? s->tm_act_f : s->tm_act_l));
    if (m->tp_world == 1 && gemm_serial(p)) {
      *splits = 1;  // the splits' sum, stored as one split
      return launch_gemm_tc_serial(tA, tA2, tB, p, out, s->d_err, st, s->use_pdl());
    }
    return launch_gemm_tc(tA, tA2, tB, p, out, s->d_err, st, s->use_pdl());
  }
  return launch_gemm_simt(W, W2, s->act, s->ld_act, m->cfg.dtype, p, out, st, s->use_pdl());
}

cudaEvent_t take_event(evs_state* s) {
  if (s->ev_used == s->ev_pool.size()) {
    cudaEvent_t e;
    if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
    s->ev_pool.push_back(e);
  }
  return s->ev_pool[s->ev_used++];
}

// run fn(); when profiling, bracket it with events on the stream and record its algorithmic bytes
template <typename F>
int timed(evs_state* s, cudaStream_t st, int kind, double bytes, F&& fn) {
  if (!s->prof) return fn();
  cudaEvent_t a = take_event(s), b = take_event(s);
  if (a == nullptr || b == nullptr) return fn();
  cudaEventRecord(a, st);
  const int r = fn();
  cudaEventRecord(b, st);
  s->prof_recs.push_back({kind, a, b, bytes});
  return r;
}

int run_forward(const evs_model* m, evs_state* s, const int64_t* ids, int B, int T, int prefill, int retain,
                float* logits, int out_T, int t0, int last_only, cudaStream_t st) {
  const evs_model_config& c = m->cfg;
  // d: residual width; dl, F, H: this rank's Hyena channels, MLP features and heads
  const int d = c.d_model, dl = m->dl, F = m->Fl, V = c.vocab_size;
  const bool tp = m->tp_world > 1;
  EVS_CHECK_ARG(!tp || s->tp_connected, "channel-sharded state not connected to its peers (evs_state_tp_connect)");
  EVS_CHECK_ARG(B >= 1 && B <= s->max_batch, "batch outside [1, max_batch]");
  EVS_CHECK_ARG(T >= 1 && T <= s->max_chunk, "chunk length outside [1, max_chunk]");
  EVS_CHECK_ARG(!retain || T <= s->iir_slots, "a retained forward holds at most 64 tokens per row");
  int maxlen = 0;
  for (int b = 0; b < B; ++b) maxlen = std::max(maxlen, s->h_len[b]);
  EVS_CHECK_RANGE(maxlen + T <= s->max_seqlen, "sequence would exceed max_seqlen");
  const int M = B * T;
  const int kv_blocks = (maxlen + T + ATTN_BLOCK - 1) / ATTN_BLOCK;
  const double el = static_cast<double>(m->elem());
  const int H = m->Hl, Dh = c.head_dim, S = c.state_size;
  int sp = 1;
  // one projection, timed with its algorithmic bytes (weights + activations in + fp32 partials out)
  const CUtensorMap* w3_act = nullptr;  // set when the w1/w2 projection wrote the fused SwiGLU output
  auto G = [&](const CUtensorMap* tA, const CUtensorMap* tA2, const void* W, const void* W2, int N, int K, int dual,
               float* out = nullptr, size_t out_floats = 0, const CUtensorMap* tB = nullptr) {
    const GemmPlan pl = gemm_plan(m, N, K, M, dual);
    const double bytes = (static_cast<double>(N) * K + static_cast<double>(M) * K) * el + 4.0 * pl.splits * M * N;
    float* o = out != nullptr ? out : s->ws;
    const size_t of = out != nullptr ? out_floats : s->ws_floats;
    return timed(s, st, EVS_PROF_GEMM, bytes,
                 [&] { return gemm(m, s, tA, tA2, W, W2, N, K, M, dual, o, of, st, &sp, tB); });
  };
  // row-parallel projection [d x K] whose partial sums the next residual + RMSNorm adds up: with
  // channel sharding it writes to the shared buffer of reduction `epoch` and signals the peers
  TpPartials parts{};
  auto RP = [&](const CUtensorMap* tA, const void* W, int K, const CUtensorMap* tB = nullptr) -> int {
    parts = TpPartials{};
    if (!tp) {
      EVS_TRY(G(tA, nullptr, W, nullptr, d, K, 0, nullptr, 0, tB));
      parts.R = 1;
      parts.buf[0] = s->ws;
      return EVS_OK;
    }
    const long long epoch = ++s->tp_epoch;
    const size_t boff = static_cast<size_t>(epoch & 1) * s->tp_buf_bytes;
    float* mine = reinterpret_cast<float*>(s->tp_base[m->tp_rank] + boff);
    EVS_TRY(G(tA, nullptr, W, nullptr, d, K, 0, mine, s->tp_buf_bytes / sizeof(float), tB));
    // this rank's splits summed into split 0, then published: the consumer reads one partial per rank
    EVS_TRY(launch_tp_reduce_signal(s, mine, sp, M, epoch, st));
    sp = 1;
    parts.R = m->tp_world;
    parts.epoch = epoch;
    for (int r = 0; r < m->tp_world; ++r) {
      parts.buf[r] = reinterpret_cast<const float*>(s->tp_base[r] + boff);
      parts.flag[r] = reinterpret_cast<const long long*>(s->tp_base[r] + 2 * s->tp_buf_bytes);
    }
    return EVS_OK;
  };
  const double row_bytes = static_cast<double>(M) * d * (8.0 + el);
  EVS_TRY(timed(s, st, EVS_PROF_ROW, row_bytes,
                [&] { return launch_embed_norm(m, s, ids, M, static_cast<const float*>(m->L[0].pre_norm), st); }));
  for (int i = 0; i < c.n_layers; ++i) {
    const LayerDev& L = m->L[i];
    if (L.kind == EVS_LAYER_MHA) {
      EVS_TRY(G(&L.tm_qkv, nullptr, L.w_qkv, nullptr, 3 * dl, d, 0));
      const double kv_bytes = 2.0 * B * (maxlen + T) * H * Dh * el + 4.0 * sp * M * 3 * dl + 2.0 * M * dl * el;
      EVS_TRY(timed(s, st, EVS_PROF_ATTN, kv_bytes, [&] { return launch_attention(m, s, i, B, T, sp, kv_blocks, st); }));
      EVS_TRY(RP(&L.tm_o, L.w_o, dl));
    } else {
      EVS_TRY(G(&L.tm_in, nullptr, L.w_in, nullptr, 3 * dl, d, 0));
      const int K = L.kind == EVS_LAYER_HCM ? c.hcm_filter_length : c.hcs_filter_length;
      const int K0 = c.short_filter_length;
      // u in + y out + outer history read/write + taps; inner FIR history or IIR states
      double hb = B * ((2.0 * T * 3 * dl + (K0 - 1) * 3.0 * dl + T * dl) * el) + 3.0 * dl * K0 * 4;
      if (L.kind == EVS_LAYER_HCL)
        hb += B * (static_cast<double>(dl) * S * 4 * (1 + (retain ? T : 1))) + 3.0 * dl * S * 4;
      else
        hb += B * ((K - 1.0 + T) * dl * el) + static_cast<double>(dl) * K * 4;
      EVS_TRY(timed(s, st, EVS_PROF_HYENA, hb, [&] { return launch_hyena(m, s, i, B, T, sp, prefill, retain, st); }));
      EVS_TRY(RP(&L.tm_out, L.w_out, dl));
    }
    EVS_TRY(timed(s, st, EVS_PROF_ROW, row_bytes + 4.0 * sp * M * d * parts.R, [&] {
      return launch_res_add_norm(m, s, M, sp, parts, static_cast<const float*>(L.post_norm), -1, T, st);
    }));
    if (c.dtype == EVS_DTYPE_BF16 && gemm_plan(m, 2 * F, d, M, 1).splits == 1) {
      // one split: the w1/w2 projection applies the SwiGLU gate in its epilogue
      const GemmPlan pl = gemm_plan(m, 2 * F, d, M, 1);
      const double bytes = (2.0 * F * d + static_cast<double>(M) * d) * el + M * F * el;
      EVS_TRY(timed(s, st, EVS_PROF_GEMM, bytes, [&] {
        const CUtensorMap* tB = s->tm_act_d;
        return launch_gemm_tc(&L.tm_w1, &L.tm_w2, tB, pl, s->ws, s->d_err, st, s->use_pdl(), s->gate, F);
      }));
      w3_act = s->tm_gate;
    } else {
      w3_act = nullptr;
      EVS_TRY(G(&L.tm_w1, &L.tm_w2, L.w1, L.w2, 2 * F, d, 1));
      EVS_TRY(timed(s, st, EVS_PROF_ROW, 8.0 * sp * M * F + M * F * el, [&] { return launch_swiglu(m, s, M, sp, st); }));
    }
    EVS_TRY(RP(&L.tm_w3, L.w3, F, w3_act));
    const float* next = static_cast<const float*>(i + 1 < c.n_layers ? m->L[i + 1].pre_norm : m->final_norm);
    EVS_TRY(timed(s, st, EVS_PROF_ROW, row_bytes + 4.0 * sp * M * d * parts.R,
                  [&] { return launch_res_add_norm(m, s, M, sp, parts, next, m->capture_slot(i), T, st); }));
  }
  if (logits != nullptr) {
    EVS_TRY(G(&m->tm_embed, nullptr, m->embed, nullptr, V, d, 0));
    EVS_TRY(timed(s, st, EVS_PROF_ROW, 4.0 * (sp + 1) * M * V,
                  [&] { return launch_logits(m, s, M, T, sp, logits, out_T, t0, last_only, st); }));
  }
  EVS_TRY(launch_bookkeeping(s, B, T, retain, st));
  for (int b = 0; b < B; ++b) s->h_len[b] += T;
  s->h_chunk = retain ? T : 0;
  return EVS_OK;
}

}  // namespace

namespace {
std::atomic<long long> g_launches{0};
}

void evs_count_launch(int n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

void evs_set_last_error(int code, const char* msg) {
  (void)code;
  g_last_error = msg ? msg : "";
}

extern "C" {

int evs_version(void) { return 1; }

const char* evs_last_error(void) { return g_last_error.c_str(); }

int evs_device_check(void) {
  int dev = 0, n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
    cudaGetLastError();
    evs_set_last_error(EVS_ENODEV, "no CUDA device visible");
    return EVS_ENODEV;
  }
  EVS_CUDA_TRY(cudaGetDevice(&dev));
  int major = 0, minor = 0;
  EVS_CUDA_TRY(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev));
  EVS_CUDA_TRY(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev));
  if (major != 10 || minor != 0) {
    evs_set_last_error(EVS_ENODEV, "libevspark_sm100 needs an sm_100 (B200) device");
    return EVS_ENODEV;
  }
  return EVS_OK;
}

int evs_model_create(const evs_model_config* cfg, evs_model** out) {
  EVS_CHECK_ARG(cfg != nullptr && out != nullptr, "null argument");
  const evs_model_config& c = *cfg;
  EVS_CHECK_ARG(c.n_layers >= 1 && c.n_layers <= EVS_MAX_LAYERS, "n_layers outside [1, 64]");
  EVS_CHECK_ARG(c.d_model % 32 == 0 && c.n_heads * c.head_dim == c.d_model, "bad d_model / heads");
  EVS_CHECK_ARG(c.dtype == EVS_DTYPE_FP32 || c.dtype == EVS_DTYPE_BF16, "dtype must be fp32 or bf16");
  EVS_CHECK_ARG(c.mlp_inner % 64 == 0, "mlp_inner must be a multiple of 64");
  EVS_CHECK_ARG(c.vocab_size >= 1 && c.vocab_size <= 1024, "vocab_size outside [1, 1024]");
  EVS_CHECK_ARG(c.short_filter_length >= 1 && c.hcs_filter_length >= 1 && c.hcm_filter_length >= 1,
                "bad filter lengths");
  EVS_CHECK_ARG(c.state_size % 4 == 0 && c.state_size <= 32, "state_size must be 4, 8, 16 or 32");
  if (c.dtype == EVS_DTYPE_BF16)
    EVS_CHECK_ARG(c.d_model % 128 == 0 && c.vocab_size % 128 == 0,
                  "bf16 models need d_model and vocab_size multiples of 128");
  for (int i = 0; i < c.n_layers; ++i)
    EVS_CHECK_ARG(c.layer_kind[i] >= 0 && c.layer_kind[i] <= 3, "unknown layer kind");
  const int tw = c.tp_world > 1 ? c.tp_world : 1;
  EVS_CHECK_ARG(tw <= EVS_TP_MAX && c.tp_rank >= 0 && c.tp_rank < tw, "tp_rank / tp_world out of range");
  EVS_CHECK_ARG(c.n_heads % tw == 0 && c.mlp_inner % (64 * tw) == 0 && (c.d_model / tw) % 32 == 0,
                "heads, mlp_inner / 64 and d_model / 32 must divide by tp_world");
  if (tw > 1)
    EVS_CHECK_ARG(c.dtype == EVS_DTYPE_BF16 && (c.d_model / tw) % 128 == 0,
                  "channel sharding needs a bf16 model with d_model / tp_world a multiple of 128");
  evs_model* m = new evs_model();
  m->cfg = c;
  m->tp_world = tw;
  m->tp_rank = tw > 1 ? c.tp_rank : 0;
  m->dl = c.d_model / tw;
  m->Hl = c.n_heads / tw;
  m->Fl = c.mlp_inner / tw;
  EVS_CUDA_TRY(cudaGetDevice(&m->device));
  for (int i = 0; i < c.n_layers; ++i) m->L[i].kind = c.layer_kind[i];
  for (int k = 0; k < 4; ++k) {
    const int l = c.capture_layers[k];
    if (l >= 0) {
      if (l >= c.n_layers) {
        delete m;
        evs_set_last_error(EVS_EINVAL, "capture layer outside the model");
        return EVS_EINVAL;
      }
      m->capture_layer[m->n_capture++] = l;
    }
  }
  *out = m;
  return EVS_OK;
}

int evs_model_set_tensor(evs_model* m, int layer, int slot, const void* dev_ptr, int64_t numel) {
  EVS_CHECK_ARG(m != nullptr && dev_ptr != nullptr, "null argument");
  EVS_CHECK_ARG(!m->finalized, "model already finalized");
  const evs_model_config& c = m->cfg;
  if (layer < 0) {
    if (slot == EVS_W_EMBED) {
      EVS_CHECK_ARG(numel == static_cast<int64_t>(c.vocab_size) * c.d_model, "embed numel mismatch");
      m->embed = dev_ptr;
      m->embed_numel = numel;
      return EVS_OK;
    }
    if (slot == EVS_W_FINAL_NORM) {
      EVS_CHECK_ARG(numel == c.d_model, "final_norm numel mismatch");
      m->final_norm = dev_ptr;
      m->final_norm_numel = numel;
      return EVS_OK;
    }
    EVS_CHECK_ARG(false, "model-level slot must be EVS_W_EMBED or EVS_W_FINAL_NORM");
  }
  EVS_CHECK_ARG(layer < c.n_layers, "layer index out of range");
  EVS_CHECK_ARG(slot >= EVS_W_PRE_NORM && slot < EVS_W_NUM_SLOTS, "bad slot");
  LayerDev& L = m->L[layer];
  const int64_t want = expected_numel(m, L.kind, slot);
  EVS_CHECK_ARG(want > 0, "slot not used by this layer kind");
  EVS_CHECK_ARG(numel == want, "tensor numel does not match the slot shape");
  *slot_ptr(L, slot) = dev_ptr;
  L.numel[slot] = numel;
  return EVS_OK;
}

int evs_model_finalize(evs_model* m) {
  EVS_CHECK_ARG(m != nullptr, "null model");
  if (m->finalized) return EVS_OK;
  const evs_model_config& c = m->cfg;
  const int d = c.d_model, dl = m->dl, F = m->Fl, V = c.vocab_size;
  EVS_CHECK_ARG(m->embed && m->final_norm, "embed / final_norm not set");
  for (int i = 0; i < c.n_layers; ++i) {
    LayerDev& L = m->L[i];
    for (int slot = EVS_W_PRE_NORM; slot < EVS_W_NUM_SLOTS; ++slot) {
      if (expected_numel(m, L.kind, slot) > 0 && *slot_ptr(L, slot) == nullptr) {
        evs_set_last_error(EVS_EINVAL, ("layer " + std::to_string(i) + " slot " + std::to_string(slot) +
                                        " not set").c_str());
        return EVS_EINVAL;
      }
    }
    if (L.kind == EVS_LAYER_HCL) {
      EVS_CUDA_TRY(cudaMalloc(&L.poles, sizeof(float) * dl * c.state_size));
      EVS_TRY(launch_poles(static_cast<const float*>(L.log_poles), L.poles, dl * c.state_size, 0));
    }
    if (c.dtype == EVS_DTYPE_BF16) {
      // local shapes: column-parallel [3 dl, d] / [Fl, d], row-parallel [d, dl] / [d, Fl]
      if (L.kind == EVS_LAYER_MHA) {
        EVS_TRY(make_tmap_2d_bf16(&L.tm_qkv, L.w_qkv, d, 3 * dl, d * 2, GEMM_BK, GEMM_BM));
        EVS_TRY(make_tmap_2d_bf16(&L.tm_o, L.w_o, dl, d, dl * 2, GEMM_BK, GEMM_BM));
      } else {
        EVS_TRY(make_tmap_2d_bf16(&L.tm_in, L.w_in, d, 3 * dl, d * 2, GEMM_BK, GEMM_BM));
        EVS_TRY(make_tmap_2d_bf16(&L.tm_out, L.w_out, dl, d, dl * 2, GEMM_BK, GEMM_BM));
      }
      EVS_TRY(make_tmap_2d_bf16(&L.tm_w1, L.w1, d, F, d * 2, GEMM_BK, GEMM_BM / 2));
      EVS_TRY(make_tmap_2d_bf16(&L.tm_w2, L.w2, d, F, d * 2, GEMM_BK, GEMM_BM / 2));
      EVS_TRY(make_tmap_2d_bf16(&L.tm_w3, L.w3, F, d, static_cast<uint64_t>(F) * 2, GEMM_BK, GEMM_BM));
    }
  }
  if (c.dtype == EVS_DTYPE_BF16) EVS_TRY(make_tmap_2d_bf16(&m->tm_embed, m->embed, d, V, d * 2, GEMM_BK, GEMM_BM));
  EVS_CUDA_TRY(cudaDeviceSynchronize());
  m->finalized = true;
  return EVS_OK;
}

void evs_model_destroy(evs_model* m) {
  if (m == nullptr) return;
  for (int i = 0; i < m->cfg.n_layers; ++i)
    if (m->L[i].poles) cudaFree(m->L[i].poles);
  delete m;
}

// Persistent per-row arenas live in one allocation (owned[0]); scratch in owned[1].
int evs_state_create(const evs_model* m, int max_batch, int max_seqlen, int max_chunk, evs_state** out) {
  EVS_CHECK_ARG(m != nullptr && out != nullptr, "null argument");
  EVS_CHECK_ARG(m->finalized, "model not finalized");
  EVS_CHECK_ARG(max_batch >= 1 && max_seqlen >= 2 && max_chunk >= 1, "bad state sizes");
  const evs_model_config& c = m->cfg;
  // d: residual width; dl, H, F: this rank's Hyena channels, heads and MLP features
  const int d = c.d_model, dl = m->dl, F = m->Fl, H = m->Hl, Dh = c.head_dim, S = c.state_size;
  const size_t el = m->elem();
  evs_state* s = new evs_state();
  s->m = m;
  s->max_batch = max_batch;
  s->max_seqlen = max_seqlen;
  s->max_chunk = max_chunk;
  // EVS_NO_PDL=1 serialises the kernels of a forward (programmatic dependent launch off)
  s->pdl = std::getenv("EVS_NO_PDL") == nullptr;
  s->cap_outer = next_pow2(c.short_filter_length - 1 + max_chunk);
  s->cap_hcs = next_pow2(c.hcs_filter_length - 1 + max_chunk);
  s->cap_hcm = next_pow2(c.hcm_filter_length - 1 + max_chunk);
  // per-position IIR states are kept only for retained (verify) forwards of at most EVS_RETAIN_MAX
  s->iir_slots = std::min(max_chunk, EVS_RETAIN_MAX);
  s->ring_len = next_pow2(64 + max_chunk);
  s->m_cap = (max_batch * max_chunk + TOK_TILE - 1) / TOK_TILE * TOK_TILE;
  s->ld_act = std::max(d, F);
  s->attn_blocks = (max_seqlen + ATTN_BLOCK - 1) / ATTN_BLOCK;
  s->attn_tcap = std::min(max_chunk, ATTN_TCAP);
  s->h_len.assign(max_batch, 0);
  const size_t B = max_batch;

  // ---- persistent arenas ----
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off = align256(off + bytes);
    return o;
  };
  const size_t o_len = take(4 * B), o_len0 = take(4 * B), o_cur = take(4 * B), o_chunk = take(4);
  size_t o_outer[EVS_MAX_LAYERS], o_inner[EVS_MAX_LAYERS], o_iir[EVS_MAX_LAYERS], o_kv[EVS_MAX_LAYERS];
  for (int i = 0; i < c.n_layers; ++i) {
    const int k = c.layer_kind[i];
    o_outer[i] = o_inner[i] = o_iir[i] = o_kv[i] = SIZE_MAX;
    if (k == EVS_LAYER_MHA) {
      o_kv[i] = take(B * max_seqlen * 2 * H * Dh * el);
    } else {
      o_outer[i] = take(B * s->cap_outer * 3 * dl * el);
      if (k == EVS_LAYER_HCS) o_inner[i] = take(B * s->cap_hcs * dl * el);
      if (k == EVS_LAYER_HCM) o_inner[i] = take(B * s->cap_hcm * dl * el);
      if (k == EVS_LAYER_HCL) o_iir[i] = take(B * s->iir_slots * dl * S * sizeof(float));
    }
  }
  size_t o_ring[4];
  for (int k = 0; k < m->n_capture; ++k) o_ring[k] = take(B * s->ring_len * d * sizeof(float));
  const size_t o_tag = m->n_capture > 0 ? take(B * s->ring_len * sizeof(unsigned long long)) : SIZE_MAX;
  const size_t o_seq = take(sizeof(unsigned long long));
  void* pers = nullptr;
  if (cudaMalloc(&pers, off) != cudaSuccess) {
    cudaGetLastError();
    delete s;
    evs_set_last_error(EVS_ECUDA, "cudaMalloc of the state arenas failed");
    return EVS_ECUDA;
  }
  s->owned.push_back(pers);
  s->owned_bytes.push_back(off);
  char* base = static_cast<char*>(pers);
  s->d_len = reinterpret_cast<int32_t*>(base + o_len);
  s->d_len0 = reinterpret_cast<int32_t*>(base + o_len0);
  s->d_iir_cur = reinterpret_cast<int32_t*>(base + o_cur);
  s->d_chunk = reinterpret_cast<int32_t*>(base + o_chunk);
  for (int i = 0; i < c.n_layers; ++i) {
    if (o_outer[i] != SIZE_MAX) s->hy[i].outer_ring = base + o_outer[i];
    if (o_inner[i] != SIZE_MAX) s->hy[i].inner_ring = base + o_inner[i];
    if (o_iir[i] != SIZE_MAX) s->hy[i].s_all = reinterpret_cast<float*>(base + o_iir[i]);
    if (o_kv[i] != SIZE_MAX) s->kv[i] = base + o_kv[i];
  }
  for (int k = 0; k < m->n_capture; ++k) s->cap_ring[k] = reinterpret_cast<float*>(base + o_ring[k]);
  if (o_tag != SIZE_MAX) s->cap_tag = reinterpret_cast<unsigned long long*>(base + o_tag);
  s->d_fwd_seq = reinterpret_cast<unsigned long long*>(base + o_seq);
  {
    static std::atomic<unsigned long long> next_id{1};
    const unsigned long long id = next_id.fetch_add(1) & ((1ull << (64 - EVS_TAG_SEQ_BITS - EVS_TAG_ROW_BITS)) - 1);
    s->tag_hi = (id == 0 ? 1ull : id) << (EVS_TAG_SEQ_BITS + EVS_TAG_ROW_BITS);
  }

  // ---- scratch ----
  size_t ws_cols = 0;
  auto plan_cols = [&](int N, int K, int dual) {
    GemmPlan p = gemm_plan(m, N, K, s->m_cap, dual);
    ws_cols = std::max(ws_cols, static_cast<size_t>(p.splits) * N);
  };
  plan_cols(3 * dl, d, 0);
  plan_cols(d, dl, 0);
  plan_cols(2 * F, d, 1);
  plan_cols(d, F, 0);
  plan_cols(c.vocab_size, d, 0);
  s->ws_floats = ws_cols * s->m_cap;
  // row-parallel partial sums exchanged with the peers: two buffers of splits x m_cap x d fp32
  if (m->tp_world > 1) {
    size_t rp = 0;
    rp = std::max(rp, static_cast<size_t>(gemm_plan(m, d, dl, s->m_cap, 0).splits));
    rp = std::max(rp, static_cast<size_t>(gemm_plan(m, d, F, s->m_cap, 0).splits));
    s->tp_buf_bytes = align256(rp * s->m_cap * d * sizeof(float));
  }
  bool any_mha = false;
  for (int i = 0; i < c.n_layers; ++i) any_mha |= c.layer_kind[i] == EVS_LAYER_MHA;
  off = 0;
  const size_t o_resid = take(static_cast<size_t>(s->m_cap) * d * 4);
  const size_t o_act = take(static_cast<size_t>(s->m_cap) * s->ld_act * el);
  const size_t o_ws = take(s->ws_floats * 4);
  const size_t o_qrot = take(static_cast<size_t>(s->m_cap) * dl * el);
  const size_t o_part = any_mha ? take(B * H * s->attn_blocks * s->attn_tcap * (Dh + 2) * 4) : SIZE_MAX;
  const size_t o_ids = take(static_cast<size_t>(s->m_cap) * 8);
  const size_t o_gate = c.dtype == EVS_DTYPE_BF16 ? take(static_cast<size_t>(s->m_cap) * F * 2) : SIZE_MAX;
  const size_t o_err = take(sizeof(EvsDevErr));
  void* scr = nullptr;
  if (cudaMalloc(&scr, off) != cudaSuccess) {
    cudaGetLastError();
    cudaFree(pers);
    delete s;
    evs_set_last_error(EVS_ECUDA, "cudaMalloc of the state scratch failed");
    return EVS_ECUDA;
  }
  s->owned.push_back(scr);
  s->owned_bytes.push_back(off);
  base = static_cast<char*>(scr);
  s->resid = reinterpret_cast<float*>(base + o_resid);
  s->act = base + o_act;
  s->ws = reinterpret_cast<float*>(base + o_ws);
  s->qrot = base + o_qrot;
  if (o_part != SIZE_MAX) s->attn_part = reinterpret_cast<float*>(base + o_part);
  s->ids_scratch = reinterpret_cast<int64_t*>(base + o_ids);
  if (o_gate != SIZE_MAX) s->gate = base + o_gate;
  s->d_err = reinterpret_cast<EvsDevErr*>(base + o_err);
  EVS_CUDA_TRY(cudaMemset(pers, 0, s->owned_bytes[0]));
  EVS_CUDA_TRY(cudaMemset(scr, 0, s->owned_bytes[1]));
  if (m->tp_world > 1) {
    // [buffer 0 | buffer 1 | epoch flag]; its own allocation so that it can be shared over IPC
    const size_t bytes = 2 * s->tp_buf_bytes + 256;
    if (cudaMalloc(&s->tp_region, bytes) != cudaSuccess) {
      cudaGetLastError();
      for (void* p : s->owned) cudaFree(p);
      delete s;
      evs_set_last_error(EVS_ECUDA, "cudaMalloc of the shared partial-sum region failed");
      return EVS_ECUDA;
    }
    EVS_CUDA_TRY(cudaMemset(s->tp_region, 0, bytes));
    s->tp_base[m->tp_rank] = static_cast<char*>(s->tp_region);
  }
  if (c.dtype == EVS_DTYPE_BF16) {
    for (int t = 0; t < GEMM_NMAPS; ++t) {
      const uint64_t ld = static_cast<uint64_t>(s->ld_act) * 2;
      EVS_TRY(make_tmap_2d_bf16(&s->tm_act_d[t], s->act, d, s->m_cap, ld, GEMM_BK, GEMM_NT[t]));
      EVS_TRY(make_tmap_2d_bf16(&s->tm_act_f[t], s->act, F, s->m_cap, ld, GEMM_BK, GEMM_NT[t]));
      EVS_TRY(make_tmap_2d_bf16(&s->tm_act_l[t], s->act, dl, s->m_cap, ld, GEMM_BK, GEMM_NT[t]));
      EVS_TRY(make_tmap_2d_bf16(&s->tm_gate[t], s->gate, F, s->m_cap, static_cast<uint64_t>(F) * 2, GEMM_BK,
                                GEMM_NT[t]));
    }
  }
  EVS_CUDA_TRY(cudaDeviceSynchronize());
  *out = s;
  return EVS_OK;
}

void evs_state_destroy(evs_state* s) {
  if (s == nullptr) return;
  if (s->tp_connected) evs_state_tp_disconnect(s);
  for (cudaEvent_t e : s->ev_pool) cudaEventDestroy(e);
  for (void* p : s->owned) cudaFree(p);
  if (s->tp_region) cudaFree(s->tp_region);
  delete s;
}

int evs_state_tp_handle(const evs_state* s, void* handle64) {
  EVS_CHECK_ARG(s && handle64, "null argument");
  EVS_CHECK_ARG(s->tp_region != nullptr, "state of a model without channel sharding");
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
  cudaIpcMemHandle_t h;
  EVS_CUDA_TRY(cudaIpcGetMemHandle(&h, s->tp_region));
  std::memcpy(handle64, &h, sizeof(h));
  return EVS_OK;
}

int evs_state_tp_connect(evs_state* s, const void* handles, int world) {
  EVS_CHECK_ARG(s && handles, "null argument");
  EVS_CHECK_ARG(s->tp_region != nullptr, "state of a model without channel sharding");
  EVS_CHECK_ARG(world == s->m->tp_world, "handle count != tp_world");
  EVS_CHECK_ARG(!s->tp_connected, "state already connected");
  for (int r = 0; r < world; ++r) {
    if (r == s->m->tp_rank) continue;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, static_cast<const char*>(handles) + 64 * r, sizeof(h));
    void* p = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      for (int q = 0; q < r; ++q)
        if (q != s->m->tp_rank && s->tp_base[q]) {
          cudaIpcCloseMemHandle(s->tp_base[q]);
          s->tp_base[q] = nullptr;
        }
      evs_set_last_error(EVS_ECUDA, (std::string("cudaIpcOpenMemHandle: ") + cudaGetErrorString(e)).c_str());
      return EVS_ECUDA;
    }
    s->tp_base[r] = static_cast<char*>(p);
  }
  s->tp_connected = true;
  return EVS_OK;
}

int evs_state_tp_disconnect(evs_state* s) {
  EVS_CHECK_ARG(s != nullptr, "null state");
  if (!s->tp_connected) return EVS_OK;
  for (int r = 0; r < s->m->tp_world; ++r)
    if (r != s->m->tp_rank && s->tp_base[r]) {
      cudaIpcCloseMemHandle(s->tp_base[r]);
      s->tp_base[r] = nullptr;
    }
  s->tp_connected = false;
  return EVS_OK;
}

int evs_state_reset(evs_state* s, cudaStream_t st) {
  EVS_CHECK_ARG(s != nullptr, "null state");
  EVS_CUDA_TRY(cudaMemsetAsync(s->d_len, 0, 4 * s->max_batch, st));
  EVS_CUDA_TRY(cudaMemsetAsync(s->d_len0, 0, 4 * s->max_batch, st));
  EVS_CUDA_TRY(cudaMemsetAsync(s->d_iir_cur, 0, 4 * s->max_batch, st));
  EVS_CUDA_TRY(cudaMemsetAsync(s->d_chunk, 0, 4, st));
  std::fill(s->h_len.begin(), s->h_len.end(), 0);
  s->h_chunk = 0;
  return EVS_OK;
}

int evs_state_copy(evs_state* dst, const evs_state* src, cudaStream_t st) {
  EVS_CHECK_ARG(dst && src && dst->m == src->m, "states of different models");
  EVS_CHECK_ARG(dst->max_batch == src->max_batch && dst->max_seqlen == src->max_seqlen &&
                    dst->max_chunk == src->max_chunk,
                "states of different sizes");
  EVS_CUDA_TRY(cudaMemcpyAsync(dst->owned[0], src->owned[0], src->owned_bytes[0], cudaMemcpyDeviceToDevice, st));
  dst->h_len = src->h_len;
  dst->h_chunk = src->h_chunk;
  return EVS_OK;
}

int evs_state_get_lengths(const evs_state* s, int32_t* host_lengths, int batch, cudaStream_t st) {
  EVS_CHECK_ARG(s && host_lengths && batch >= 1 && batch <= s->max_batch, "bad arguments");
  EVS_CUDA_TRY(cudaMemcpyAsync(host_lengths, s->d_len, 4 * batch, cudaMemcpyDeviceToHost, st));
  EVS_CUDA_TRY(cudaStreamSynchronize(st));
  evs_state* ms = const_cast<evs_state*>(s);
  for (int b = 0; b < batch; ++b) ms->h_len[b] = host_lengths[b];
  return EVS_OK;
}

int evs_state_set_lengths(evs_state* s, const int32_t* host_lengths, int batch, cudaStream_t st) {
  EVS_CHECK_ARG(s && host_lengths && batch >= 1 && batch <= s->max_batch, "bad arguments");
  for (int b = 0; b < batch; ++b)
    EVS_CHECK_RANGE(host_lengths[b] >= 0 && host_lengths[b] <= s->max_seqlen, "length outside [0, max_seqlen]");
  EVS_CUDA_TRY(cudaMemcpyAsync(s->d_len, host_lengths, 4 * batch, cudaMemcpyHostToDevice, st));
  EVS_CUDA_TRY(cudaStreamSynchronize(st));
  for (int b = 0; b < batch; ++b) s->h_len[b] = host_lengths[b];
  return EVS_OK;
}

int evs_state_note_lengths(evs_state* s, const int32_t* host_lengths, int batch) {
  EVS_CHECK_ARG(s && host_lengths && batch >= 1 && batch <= s->max_batch, "bad arguments");
  for (int b = 0; b < batch; ++b) {
    EVS_CHECK_RANGE(host_lengths[b] >= 0 && host_lengths[b] <= s->max_seqlen, "length outside [0, max_seqlen]");
    s->h_len[b] = host_lengths[b];
  }
  return EVS_OK;
}

namespace {
// copy every per-row arena of row src into row dst (KV: first kv_len positions)
int copy_row(evs_state* s, int src, int dst, cudaStream_t st) {
  const evs_model* m = s->m;
  const evs_model_config& c = m->cfg;
  const int d = m->dl;  // this rank's channels (the capture ring below is full width)
  const size_t el = m->elem();
  auto cp = [&](void* base, size_t row_bytes, size_t bytes) -> int {
    char* b = static_cast<char*>(base);
    EVS_CUDA_TRY(cudaMemcpyAsync(b + dst * row_bytes, b + src * row_bytes, bytes, cudaMemcpyDeviceToDevice, st));
    return EVS_OK;
  };
  for (int i = 0; i < c.n_layers; ++i) {
    const HyenaDev& hy = s->hy[i];
    if (hy.outer_ring) EVS_TRY(cp(hy.outer_ring, s->cap_outer * 3ull * d * el, s->cap_outer * 3ull * d * el));
    if (hy.inner_ring) {
      const size_t cap = c.layer_kind[i] == EVS_LAYER_HCM ? s->cap_hcm : s->cap_hcs;
      EVS_TRY(cp(hy.inner_ring, cap * d * el, cap * d * el));
    }
    if (hy.s_all) {
      const size_t rb = static_cast<size_t>(s->iir_slots) * d * c.state_size * 4;
      EVS_TRY(cp(hy.s_all, rb, rb));
    }
    if (s->kv[i]) {
      const size_t pos = 2ull * m->Hl * c.head_dim * el;
      EVS_TRY(cp(s->kv[i], pos * s->max_seqlen, pos * std::min(s->h_len[src], s->max_seqlen)));
    }
  }
  for (int k = 0; k < m->n_capture; ++k) {
    const size_t rb = static_cast<size_t>(s->ring_len) * c.d_model * 4;
    EVS_TRY(cp(s->cap_ring[k], rb, rb));
  }
  if (s->cap_tag) {
    const size_t rb = static_cast<size_t>(s->ring_len) * sizeof(unsigned long long);
    EVS_TRY(cp(s->cap_tag, rb, rb));
  }
  EVS_TRY(cp(s->d_len, 4, 4));
  EVS_TRY(cp(s->d_len0, 4, 4));
  EVS_TRY(cp(s->d_iir_cur, 4, 4));
  s->h_len[dst] = s->h_len[src];
  return EVS_OK;
}
}  // namespace

int evs_state_expand(evs_state* s, int batch, cudaStream_t st) {
  EVS_CHECK_ARG(s != nullptr, "null state");
  EVS_CHECK_ARG(batch >= 1 && batch <= s->max_batch, "batch outside [1, max_batch]");
  for (int b = 1; b < batch; ++b) EVS_TRY(copy_row(s, 0, b, st));
  return EVS_OK;
}

int evs_state_collapse(evs_state* s, int idx, cudaStream_t st) {
  EVS_CHECK_ARG(s != nullptr, "null state");
  EVS_CHECK_RANGE(idx >= 0 && idx < s->max_batch, "row index out of range");
  if (idx != 0) EVS_TRY(copy_row(s, idx, 0, st));
  return EVS_OK;
}

int evs_state_export(const evs_state* s, int layer, int which, int row, int width, void* dst, cudaStream_t st) {
  EVS_CHECK_ARG(s && dst, "null argument");
  EVS_CHECK_ARG(layer >= 0 && layer < s->m->cfg.n_layers, "layer out of range");
  EVS_CHECK_RANGE(row >= 0 && row < s->max_batch, "row out of range");
  EVS_CHECK_RANGE(width >= 0 && width <= s->max_seqlen, "width out of range");
  return launch_state_export(s, layer, which, row, width, dst, st);
}

int evs_state_capture_ring(const evs_state* s, int c, float** dev_ptr, int* ring_len) {
  EVS_CHECK_ARG(s && dev_ptr && ring_len, "null argument");
  EVS_CHECK_RANGE(c >= 0 && c < s->m->n_capture, "capture slot out of range");
  *dev_ptr = s->cap_ring[c];
  *ring_len = s->ring_len;
  return EVS_OK;
}

int evs_prefill(const evs_model* m, evs_state* s, const int64_t* ids, int batch, int T, float* logits,
                int last_only, cudaStream_t st) {
  EVS_CHECK_ARG(m && s && ids && s->m == m, "bad arguments");
  EVS_CHECK_ARG(batch >= 1 && batch <= s->max_batch && T >= 1, "bad batch / length");
  for (int b = 0; b < batch; ++b) EVS_CHECK_ARG(s->h_len[b] == 0, "prefill requires an empty state");
  for (int t0 = 0; t0 < T; t0 += s->max_chunk) {
    const int tc = std::min(s->max_chunk, T - t0);
    const int64_t* chunk = ids + t0;
    if (batch > 1 || t0 > 0) {
      EVS_CUDA_TRY(cudaMemcpy2DAsync(s->ids_scratch, tc * sizeof(int64_t), ids + t0, T * sizeof(int64_t),
                                     tc * sizeof(int64_t), batch, cudaMemcpyDeviceToDevice, st));
      chunk = s->ids_scratch;
    }
    const bool last_chunk = t0 + tc == T;
    float* lg = (logits != nullptr && (!last_only || last_chunk)) ? logits : nullptr;
    EVS_TRY(run_forward(m, s, chunk, batch, tc, 1, 0, lg, T, t0, last_only, st));
  }
  return EVS_OK;
}

int evs_forward(const evs_model* m, evs_state* s, const int64_t* ids, int batch, int T, int retain, float* logits,
                cudaStream_t st) {
  EVS_CHECK_ARG(m && s && ids && s->m == m, "bad arguments");
  for (int b = 0; b < batch && b < s->max_batch; ++b)
    EVS_CHECK_ARG(s->h_len[b] > 0, "forward needs a prefilled state (call evs_prefill first)");
  return run_forward(m, s, ids, batch, T, 0, retain ? 1 : 0, logits, T, 0, 0, st);
}

int evs_rollback(evs_state* s, const int32_t* k, int batch, cudaStream_t st) {
  EVS_CHECK_ARG(s && k, "null argument");
  EVS_CHECK_ARG(batch >= 1 && batch <= s->max_batch, "batch outside [1, max_batch]");
  EVS_CHECK_RANGE(s->h_chunk > 0, "no retained forward to roll back");
  return launch_rollback(s, k, batch, st);
}

int evs_transform(const void* logits, int logits_fp64, int rows, int V, double temperature, int top_k, double* probs,
                  cudaStream_t st) {
  EVS_CHECK_ARG(logits && probs, "null argument");
  return launch_transform(logits, logits_fp64, rows, V, temperature, top_k, probs, st);
}

int evs_verify(const double* p, const double* q, const int64_t* x, const double* u, int batch, int gamma, int V,
               int greedy, int32_t* accepted, int64_t* tokens, int32_t* info, cudaStream_t st) {
  EVS_CHECK_ARG(p && x && accepted && tokens && info, "null argument");
  return launch_verify(p, q, x, u, batch, gamma, V, greedy, accepted, tokens, info, st);
}

int evs_verify_multicand(const double* p, const double* q, const int64_t* x, const double* u, int n_candidates,
                         int gamma, int V, int greedy, int64_t* tokens, int32_t* info, cudaStream_t st) {
  EVS_CHECK_ARG(p && x && tokens && info, "null argument");
  return launch_verify_multicand(p, q, x, u, n_candidates, gamma, V, greedy, tokens, info, st);
}

int evs_sample(const double* rows, int n, int V, const double* u, int64_t* out, cudaStream_t st) {
  EVS_CHECK_ARG(rows && u && out, "null argument");
  return launch_sample(rows, n, V, u, out, st);
}

int evs_gemm_bf16(const void* W, const void* X, float* out, int N, int K, int M, int splits, cudaStream_t st) {
  EVS_CHECK_ARG(W && X && out, "null argument");
  EVS_CHECK_ARG(N % GEMM_BM == 0 && K % GEMM_BK == 0 && M >= 1 && M <= 4096, "bad GEMM shape");
  CUtensorMap ta, tb[3];
  EVS_TRY(make_tmap_2d_bf16(&ta, W, K, N, static_cast<uint64_t>(K) * 2, GEMM_BK, GEMM_BM));
  for (int t = 0; t < 3; ++t)
    EVS_TRY(make_tmap_2d_bf16(&tb[t], X, K, M, static_cast<uint64_t>(K) * 2, GEMM_BK, GEMM_NT[t]));
  GemmPlan p{N, K, M, 1, 0};
  if (splits <= 0) {
    const int kblocks = K / GEMM_BK, tiles = N / GEMM_BM;
    while (tiles * p.splits < 148 && p.splits < kblocks) ++p.splits;
  } else {
    p.splits = splits;
  }
  EVS_CHECK_ARG(p.splits == 1, "evs_gemm_bf16 writes out directly: use splits == 1 or <= 0 with one split");
  return launch_gemm_tc(&ta, nullptr, tb, p, out, nullptr, st);
}

int evs_profile_start(evs_state* s) {
  EVS_CHECK_ARG(s != nullptr, "null state");
  s->prof = true;
  s->prof_recs.clear();
  s->ev_used = 0;
  return EVS_OK;
}

int evs_profile_stop(evs_state* s, int64_t* launches, double* ms, double* bytes) {
  EVS_CHECK_ARG(s && launches && ms && bytes, "null argument");
  for (int k = 0; k < EVS_PROF_KINDS; ++k) {
    launches[k] = 0;
    ms[k] = 0.0;
    bytes[k] = 0.0;
  }
  if (!s->prof_recs.empty()) EVS_CUDA_TRY(cudaEventSynchronize(s->prof_recs.back().b));
  for (const auto& r : s->prof_recs) {
    float t = 0.f;
    EVS_CUDA_TRY(cudaEventElapsedTime(&t, r.a, r.b));
    launches[r.kind] += 1;
    ms[r.kind] += t;
    bytes[r.kind] += r.bytes;
  }
  s->prof = false;
  s->prof_recs.clear();
  s->ev_used = 0;
  return EVS_OK;
}

int64_t evs_launch_count(void) { return g_launches.load(); }

int evs_get_device_error(const evs_state* s, int32_t* code, int32_t* where, int32_t* info) {
  EVS_CHECK_ARG(s && code && where && info, "null argument");
  EvsDevErr e;
  EVS_CUDA_TRY(cudaMemcpy(&e, s->d_err, sizeof(e), cudaMemcpyDeviceToHost));
  *code = e.code;
  *where = e.where;
  *info = e.info;
  return EVS_OK;
}

int evs_clear_device_error(evs_state* s, cudaStream_t st) {
  EVS_CHECK_ARG(s != nullptr, "null state");
  EVS_CUDA_TRY(cudaMemsetAsync(s->d_err, 0, sizeof(EvsDevErr), st));
  return EVS_OK;
}

}  // extern "C"
