/*
 * evspark_sm100.h — C ABI of libevspark_sm100.so, the B200 (sm_100a) block-verification
 * hot path of EvSpark (lossless speculative decoding for StripedHyena2 / Evo2).
 *
 * Plain C: opaque handles, raw device pointers, sizes and a cudaStream_t.  Every
 * entry point returns an int status (EVS_OK == 0); evs_last_error() gives the message.
 * Device buffers are caller-owned unless a *_create call says otherwise.  Nothing here
 * allocates inside the per-round calls (evs_forward / evs_rollback / evs_verify /
 * evs_transform / evs_draft_propose): the state and drafter handles own all scratch.
 *
 * Reference interfaces replaced (paths inside the EvSpark project):
 *   HyenaCascade chunk forward + block_forward      evspark/specdec/block/chunk.py:162-295,
 *                                                     evspark/specdec/block/driver.py:179-226
 *   prefill                                          evspark/specdec/block/driver.py:49-60
 *   step_forward_reference (native T=1 path)         evspark/specdec/block/driver.py:229-240
 *   slice_states_to_accept / ChunkStash              evspark/specdec/block/slice.py:33-191
 *   clone_inference_params / expand / collapse       evspark/specdec/block/driver.py:40-46, 96-176
 *   apply_transform                                  evspark/specdec/transforms.py:18-64
 *   verify_round / verify_round_greedy               evspark/specdec/verifier.py:54-176
 *   trunk_forward / serial_sample / propose_block    evspark/specdec/block/neural_draft.py:157-363
 *   HiddenCapture (injection-layer context ring)     evspark/specdec/block/neural_draft.py:51-154
 */
#ifndef EVSPARK_SM100_H
#define EVSPARK_SM100_H

#include <stdint.h>
#include <cuda_runtime.h>

#if defined(__GNUC__)
#define EVS_API __attribute__((visibility("default")))
#else
#define EVS_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes (the Python shim maps them to ValueError / RuntimeError) ---- */
#define EVS_OK 0
#define EVS_EINVAL 1    /* bad argument or shape                              -> ValueError   */
#define EVS_ERANGE 2    /* index / length outside the allowed range           -> ValueError   */
#define EVS_ETIMEOUT 3  /* a bounded device wait gave up (error word set)     -> RuntimeError */
#define EVS_ECUDA 4     /* a CUDA runtime/driver call failed                  -> RuntimeError */
#define EVS_ENODEV 5    /* no sm_100 device visible                           -> RuntimeError */
#define EVS_EDEVICE 6   /* a kernel reported an internal consistency failure  -> RuntimeError */

#define EVS_MAX_LAYERS 64

/* layer kinds (evspark_b200.config.LAYER_CODE) */
#define EVS_LAYER_HCS 0 /* Hyena-SE: inner FIR K=7, unflipped               */
#define EVS_LAYER_HCM 1 /* Hyena-MR: inner FIR K=128, flipped, gated bias D  */
#define EVS_LAYER_HCL 2 /* Hyena-LI: modal IIR, real poles                   */
#define EVS_LAYER_MHA 3 /* multi-head attention with KV cache                */

#define EVS_DTYPE_FP32 0
#define EVS_DTYPE_BF16 1

/* per-layer tensor slots for evs_model_set_tensor (layer = -1 for model-level tensors) */
enum evs_slot {
  EVS_W_EMBED = 0,      /* [V, d] data dtype (tied unembedding)  layer -1 */
  EVS_W_FINAL_NORM = 1, /* [d] fp32                                layer -1 */
  EVS_W_PRE_NORM = 2,   /* [d] fp32 */
  EVS_W_POST_NORM = 3,  /* [d] fp32 */
  EVS_W_IN = 4,         /* [3d, d] data dtype (Hyena in-projection) */
  EVS_W_SHORT = 5,      /* [3d, K0] fp32 outer FIR taps */
  EVS_W_INNER = 6,      /* [d, K] fp32 inner FIR taps (SE/MR) */
  EVS_W_D = 7,          /* [d] fp32 (MR gated bias, LI skip) */
  EVS_W_LOG_POLES = 8,  /* [d, S] fp32 */
  EVS_W_RESIDUES = 9,   /* [d, S] fp32 */
  EVS_W_OUT = 10,       /* [d, d] data dtype */
  EVS_W_QKV = 11,       /* [3d, d] data dtype */
  EVS_W_O = 12,         /* [d, d] data dtype */
  EVS_W_W1 = 13,        /* [F, d] data dtype */
  EVS_W_W2 = 14,        /* [F, d] data dtype */
  EVS_W_W3 = 15,        /* [d, F] data dtype */
  EVS_W_NUM_SLOTS = 16
};

typedef struct evs_model_config {
  int32_t vocab_size, d_model, n_layers, n_heads, head_dim, mlp_inner, state_size;
  int32_t short_filter_length, hcs_filter_length, hcm_filter_length;
  int32_t dtype; /* EVS_DTYPE_* : storage type of activations and GEMM weights */
  float eps, rope_base;
  int32_t layer_kind[EVS_MAX_LAYERS];
  /* blocks whose output (residual stream, fp32) feeds the drafter context ring; -1 = unused */
  int32_t capture_layers[4];
  /* channel sharding over tp_world GPUs (0 or 1 = one GPU).  Rank tp_rank holds d_model/tp_world
   * Hyena channels (in-projection rows 3h..3h+2, filters, poles), n_heads/tp_world heads and
   * mlp_inner/tp_world MLP features; out-/o-projection and w3 are row-parallel and their partial
   * sums are added across ranks by the following residual + RMSNorm.  Norms, embedding and
   * unembedding are replicated (evspark has no sharded target; this follows the depthwise-filter
   * channel split of Evo2-40B inference). */
  int32_t tp_world, tp_rank;
} evs_model_config;

typedef struct evs_model evs_model;
typedef struct evs_state evs_state;
typedef struct evs_drafter evs_drafter;

/* ---- library ---- */
EVS_API int evs_version(void);
EVS_API const char* evs_last_error(void);
/* EVS_OK when the current device is sm_100 (B200); EVS_ENODEV otherwise */
EVS_API int evs_device_check(void);

/* ---- target model (weights are caller-owned device memory, never copied) ----
 * replaces vortex StripedHyena construction + Evo2 weight loading (evspark/api.py:94-98) */
EVS_API int evs_model_create(const evs_model_config* cfg, evs_model** out);
EVS_API int evs_model_set_tensor(evs_model* m, int layer, int slot, const void* dev_ptr, int64_t numel);
/* validates every slot, builds TMA tensor maps and derived constants (poles = exp(log_poles)) */
EVS_API int evs_model_finalize(evs_model* m);
EVS_API void evs_model_destroy(evs_model* m);

/* ---- per-sequence state: FIR history rings, per-position IIR states, KV cache, lengths ----
 * replaces model.initialize_inference_params (evspark/specdec/block/loop.py:341).
 * max_chunk bounds the tokens of one evs_forward call (prefill is chunked internally). */
EVS_API int evs_state_create(const evs_model* m, int max_batch, int max_seqlen, int max_chunk, evs_state** out);
EVS_API void evs_state_destroy(evs_state* s);
/* zero the lengths of every row (an empty cache; prefill may follow) */
EVS_API int evs_state_reset(evs_state* s, cudaStream_t stream);
/* full copy of every arena (clone_inference_params, driver.py:40-46) */
EVS_API int evs_state_copy(evs_state* dst, const evs_state* src, cudaStream_t stream);
/* per-row consumed lengths (device-resident truth) -> host, and host -> device */
EVS_API int evs_state_get_lengths(const evs_state* s, int32_t* host_lengths, int batch, cudaStream_t stream);
EVS_API int evs_state_set_lengths(evs_state* s, const int32_t* host_lengths, int batch, cudaStream_t stream);
/* host-side note of the exact lengths after a device-side evs_rollback whose k the caller also
 * knows: tightens the library's host bound (used for max_seqlen checks and attention grid sizes);
 * no device traffic.  Lengths must not be below the device truth. */
EVS_API int evs_state_note_lengths(evs_state* s, const int32_t* host_lengths, int batch);
/* replicate row 0 into rows [1, batch) (expand_inference_params, driver.py:96-142) */
EVS_API int evs_state_expand(evs_state* s, int batch, cudaStream_t stream);
/* move row idx into row 0 (collapse_inference_params, driver.py:145-176) */
EVS_API int evs_state_collapse(evs_state* s, int idx, cudaStream_t stream);
/* vortex-layout export for tests/snapshots (snapshot_states, driver.py:243-278):
 * which = 0 outer FIR state [3d, width] fp32, 1 inner FIR state [d, width] fp32,
 *         2 IIR state [d, state_size] fp32, 3 KV rows [width, 2, H, Dh] in the data dtype;
 * dst is device memory */
EVS_API int evs_state_export(const evs_state* s, int layer, int which, int row, int width, void* dst,
                     cudaStream_t stream);
/* device address of the drafter-context ring of capture slot c: [max_batch, ring_len, d] fp32,
 * row P mod ring_len holds the injection-layer output at absolute position P */
EVS_API int evs_state_capture_ring(const evs_state* s, int c, float** dev_ptr, int* ring_len);

/* ---- channel sharding (tp_world > 1): every rank's state shares one device region (partial
 * sums of the row-parallel projections, double-buffered, and an epoch flag) with its peers over
 * CUDA IPC.  Call evs_state_tp_handle on every rank, exchange the 64-byte handles (rank order),
 * then evs_state_tp_connect on every rank before the first forward.  Before destroying a state,
 * synchronise, call evs_state_tp_disconnect on every rank, and wait for all ranks to get there.
 * No reference counterpart: the reference runs one GPU per model (evspark/api.py:94-98). */
EVS_API int evs_state_tp_handle(const evs_state* s, void* handle64);
EVS_API int evs_state_tp_connect(evs_state* s, const void* handles, int world);
EVS_API int evs_state_tp_disconnect(evs_state* s);

/* ---- forward passes ----
 * ids: device int64 [batch, T] (row-major).  logits: device fp32 [batch, T, V] or NULL.
 * evs_prefill (driver.py:49-60): empty state -> parallel-prefill semantics (zero-padded
 *   causal FIR); last_only != 0 writes logits only for the final position ([batch, V]).
 * evs_forward (driver.py:179-226 / 229-240): continue from the current state (block verify when
 *   T = γ+1, native step when T = 1).  retain != 0 keeps every per-position state so that
 *   evs_rollback is a pure slice (ChunkStash, slice.py:33-52). */
EVS_API int evs_prefill(const evs_model* m, evs_state* s, const int64_t* ids, int batch, int T, float* logits,
                int last_only, cudaStream_t stream);
EVS_API int evs_forward(const evs_model* m, evs_state* s, const int64_t* ids, int batch, int T, int retain,
                float* logits, cudaStream_t stream);
/* roll every row back to block index k[b] of the last retained evs_forward (device int32 [batch])
 * (slice_states_to_accept, slice.py:117-191); zero data movement: per-row ring heads, IIR slot
 * index and KV length are updated */
EVS_API int evs_rollback(evs_state* s, const int32_t* k, int batch, cudaStream_t stream);

/* ---- sampling transform and verification (fp64 decision math) ---- */
/* probs[r] = apply_transform(logits[r], temperature, top_k) for r < rows; probs fp64 [rows, V]
 * (transforms.py:18-64).  logits [rows, V] are fp32 (logits_fp64 == 0) or fp64 (!= 0, may hold -inf). */
EVS_API int evs_transform(const void* logits, int logits_fp64, int rows, int V, double temperature, int top_k,
                          double* probs, cudaStream_t stream);
/* Leviathan verification of `batch` independent rounds (verifier.py:54-176).
 * p fp64 [batch, γ+1, V] target rows (transformed probabilities, or raw logits when greedy),
 * q fp64 [batch, γ, V] draft rows (unused when greedy), x int64 [batch, γ] draft tokens,
 * u fp64 [batch, γ+1] uniforms in draw order (a round consumes a prefix of them).
 * Outputs: accepted int32 [batch], tokens int64 [batch, γ+1] (-1 padded),
 * info int32 [batch, 3] = {from_residual, fallback, uniforms consumed}. */
EVS_API int evs_verify(const double* p, const double* q, const int64_t* x, const double* u, int batch, int gamma, int V,
               int greedy, int32_t* accepted, int64_t* tokens, int32_t* info, cudaStream_t stream);

/* sample_categorical (verifier.py:37-40) for n rows: clip at 0, normalise, inverse CDF with u[r];
 * rows fp64 [n, V], u fp64 [n], out int64 [n] */
/* SpecInfer multi-candidate verification of n_candidates drafts of one stream; replaces
 * verify_round_multicand / verify_round_greedy_multicand (evspark/specdec/verifier.py:212-319).
 * p [n, γ+1, V] target rows (transformed probabilities; greedy: raw logits), q [n, γ, V], x [n, γ],
 * u: at least γ·n + 1 uniforms, used in order.  tokens [γ+1] receives the accepted prefix and the
 * correction / bonus; info = {accepted, from_residual, fallback, uniforms consumed, winner row}. */
EVS_API int evs_verify_multicand(const double* p, const double* q, const int64_t* x, const double* u, int n_candidates,
                                 int gamma, int V, int greedy, int64_t* tokens, int32_t* info, cudaStream_t stream);
EVS_API int evs_sample(const double* rows, int n, int V, const double* u, int64_t* out, cudaStream_t stream);

/* Dense projection used inside evs_forward, exposed for tests and benchmarks:
 * out[m][n] = sum_k X[m][k] * W[n][k], bf16 inputs, fp32 accumulate/output, tcgen05 path.
 * W [N, K], X [M, K] row-major device bf16 (16-byte aligned, N % 128 == 0, K % 64 == 0,
 * M <= 4096); out fp32 [M, N].  splits <= 0 picks the same K split as evs_forward. */
EVS_API int evs_gemm_bf16(const void* W, const void* X, float* out, int N, int K, int M, int splits,
                  cudaStream_t stream);

/* The split-K projection above for callers that cannot allocate device memory when they need it
 * (a host that has handed all device memory to its own pool, code running during stream capture,
 * plugins barred from allocating after start-up).  No counterpart in the reference.  Partial sums
 * go to one fixed 4 MiB file-scope device array (1,048,576 fp32; each GPU that loads the library
 * holds it until exit) instead of allocated scratch.  The K split is the smallest `splits` with
 * (N / 128) * splits >= 148, at most K / 64; calls whose splits * M * N exceeds 1,048,576 fail with
 * EVS_ERANGE.  No cudaMalloc/cudaFree.  The first call on a device looks up the array's address —
 * make it before any stream capture.  All calls share the array (last call's contents remain):
 * calls that may overlap on the GPU race.  If a wait inside the projection times out, every output
 * value is NaN. */
EVS_API int evs_gemm_bf16_noalloc(const void* W, const void* X, float* out, int N, int K, int M,
                                  cudaStream_t stream);

/* ---- γ-parallel drafter (fp32; evspark/train/drafter.py Drafter parameters) ---- */
typedef struct evs_drafter_config {
  int32_t d_model, n_layers, n_heads, gamma, n_inject, target_hidden, vocab_size, mask_id, ctx_window,
      mlp_mult;
} evs_drafter_config;

/* drafter tensor ids (parameter names of the reference Drafter, evspark/train/drafter.py:274-336);
 * layer l tensors are EVS_D_LAYER0 + l * EVS_D_PER_LAYER + {LN1, Q, K, V, O, LN2, MLP0_W, MLP0_B,
 * MLP2_W, MLP2_B} */
enum evs_drafter_tensor {
  EVS_D_EMBED = 0,    /* embed.weight     [V, H]   (frozen target embedding, fp32) */
  EVS_D_IN_W = 1,     /* in_proj.weight   [d, H] */
  EVS_D_IN_B = 2,     /* in_proj.bias     [d] */
  EVS_D_OUT_W = 3,    /* out_proj.weight  [H, d] */
  EVS_D_OUT_B = 4,    /* out_proj.bias    [H] */
  EVS_D_POS = 5,      /* pos.weight       [gamma, d] */
  EVS_D_CTX_W = 6,    /* ctx_proj.weight  [d, n_inject*H] */
  EVS_D_CTX_B = 7,    /* ctx_proj.bias    [d] */
  EVS_D_CTX_NORM = 8, /* ctx_norm.scale   [d] */
  EVS_D_FINAL_LN = 9, /* final_ln.scale   [d] */
  EVS_D_MARKOV = 10,  /* markov           [V, V] */
  EVS_D_CONF_W = 11,  /* conf_w.weight    [1, 2d] */
  EVS_D_CONF_B = 12,  /* conf_w.bias      [1] */
  EVS_D_LAYER0 = 16,
  EVS_D_PER_LAYER = 10,
  EVS_D_LN1 = 0, EVS_D_Q = 1, EVS_D_K = 2, EVS_D_V = 3, EVS_D_O = 4, EVS_D_LN2 = 5,
  EVS_D_MLP0_W = 6, EVS_D_MLP0_B = 7, EVS_D_MLP2_W = 8, EVS_D_MLP2_B = 9
};
#define EVS_D_MAX_LAYERS 8
/* (NeuralDraftModel.from_checkpoint, neural_draft.py:285-303) */
EVS_API int evs_drafter_create(const evs_drafter_config* cfg, int max_batch, evs_drafter** out);
EVS_API int evs_drafter_set_tensor(evs_drafter* d, int tensor_id, const void* dev_ptr, int64_t numel);
EVS_API int evs_drafter_finalize(evs_drafter* d);
EVS_API void evs_drafter_destroy(evs_drafter* d);
/* One drafting round per row (propose_block, neural_draft.py:323-363): context = the last
 * min(ctx_window, len) captured rows of the state, trunk over [anchor, MASK x (γ'-1)], then the
 * serial Markov head.  anchor int64 [batch]; u fp64 [batch, γ'] uniforms (sampling);
 * forced int64 [batch, γ'] or NULL.  Outputs: tokens int64 [batch, γ'], q fp64 [batch, γ', V]
 * (q' rows when sampling, raw q when greedy), conf fp32 [batch, γ'], U fp32 [batch, γ', V]
 * trunk logits (may be NULL). */
EVS_API int evs_draft_propose(evs_drafter* d, const evs_state* s, const int64_t* anchor, int batch, int gamma,
                      int greedy, double temperature, int top_k, const double* u, const int64_t* forced,
                      int64_t* tokens, double* q, float* conf, float* U, cudaStream_t stream);

/* ---- tracing ----
 * evs_profile_start arms per-launch CUDA events inside evs_prefill / evs_forward on the call's
 * stream; evs_profile_stop synchronises and returns, per kernel group (EVS_PROF_*), the number of
 * launches, their summed device time (ms) and their algorithmic HBM bytes. */
#define EVS_PROF_GEMM 0  /* tcgen05 / SIMT projections                */
#define EVS_PROF_HYENA 1 /* fused outer FIR + inner FIR / modal IIR    */
#define EVS_PROF_ATTN 2  /* RoPE + KV append + attention + combine     */
#define EVS_PROF_ROW 3   /* embedding, residual + norm, SwiGLU, logits */
#define EVS_PROF_KINDS 4
EVS_API int evs_profile_start(evs_state* s);
EVS_API int evs_profile_stop(evs_state* s, int64_t* launches, double* ms, double* bytes);
/* number of kernels this library has launched in the process (all entry points) */
EVS_API int64_t evs_launch_count(void);

/* ---- device error word ---- */
EVS_API int evs_get_device_error(const evs_state* s, int32_t* code, int32_t* where, int32_t* info);
EVS_API int evs_clear_device_error(evs_state* s, cudaStream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* EVSPARK_SM100_H */
