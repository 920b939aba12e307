/*
 * diffusorrt_b200 — C ABI of the B200 (sm_100a) denoising-decode engine.
 *
 * This library is the native provider behind the DiffusorRT SDK's `cuda_native` route: the
 * SDK imports `diffusorrt_runtime` lazily (python/src/edllm/model.py:888-920) and drives a
 * device session through start_device / propose_device / commit_device / execute_window /
 * device_metrics (python/src/edllm/backends/device_runtime.py:140-183, 354-363). Each entry
 * point below replaces one of those calls; the Python module diffusorrt_b200.runtime binds
 * them with ctypes under the same names.
 *
 * Conventions
 *   - Every function returns a drt_status. The values 0..4 are the reference AbiStatus
 *     (python/src/edllm/abi/forward.py:20-25); DRT_DEVICE_TIMEOUT is added for a bounded
 *     device wait that ran out. drt_last_error() describes the last failure of this thread.
 *   - Host pointers are borrowed for the duration of the call (Ownership.BORROWED,
 *     python/src/edllm/abi/buffers.py:37-40). Device memory is owned by the library.
 *   - A session is single-threaded (python/src/edllm/abi/handles.py:28): calls on one session
 *     must not overlap. Different sessions may run on different threads.
 *   - Kernel-level entry points take device pointers and a cudaStream_t passed as void*.
 */
#ifndef DIFFUSORRT_B200_H_
#define DIFFUSORRT_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ABI version; must equal the reference ABI_VERSION (python/src/edllm/abi/__init__.py:14). */
#define DRT_ABI_VERSION_MAJOR 0
#define DRT_ABI_VERSION_MINOR 1
#define DRT_ABI_VERSION_PATCH 0

typedef enum drt_status {
  DRT_OK = 0,                 /* AbiStatus.OK */
  DRT_VERSION_MISMATCH = 1,   /* AbiStatus.VERSION_MISMATCH */
  DRT_INVALID_ARGUMENT = 2,   /* AbiStatus.INVALID_ARGUMENT */
  DRT_UNSUPPORTED = 3,        /* AbiStatus.UNSUPPORTED */
  DRT_INTERNAL_ERROR = 4,     /* AbiStatus.INTERNAL_ERROR */
  DRT_DEVICE_TIMEOUT = 5      /* a bounded device wait expired; the context stays usable */
} drt_status;

/* Decode strategies and commit policies: the ABI integers of
 * python/src/edllm/abi/enums.py:14-31. Only these are served by a device session. */
#define DRT_STRATEGY_BLOCK_THRESHOLD 0
#define DRT_STRATEGY_D2F_BLOCK_PIPELINE 2
#define DRT_STRATEGY_ENTROPY_COUNT 5
#define DRT_STRATEGY_BD3_FIXED_QUOTA 7
#define DRT_COMMIT_THRESHOLD 2
#define DRT_COMMIT_FIXED_QUOTA 3
/* Attention mask kinds: python/src/edllm/abi/enums.py:40-43. */
#define DRT_MASK_BIDIRECTIONAL 0
#define DRT_MASK_D2F_HYBRID 1

/* Selector modes. */
#define DRT_SELECT_MAX_PROB 0   /* TopConfidence: raw softmax max-probability */
#define DRT_SELECT_NEG_ENTROPY 1 /* NegEntropy: sum p log(p + 1e-10) of softmax(x / T) */

/* Step certification bits (drt_step_trace.tie, drt_metrics counters). */
#define DRT_TIE_NEAR 1
#define DRT_TIE_EXACT 2

/* Tensor parallelism (one Dream-7B request across 2/4/8 GPUs): one rank's shard of the model.
 * Attention heads are split by K/V head; when there are more ranks than K/V heads, the ranks
 * sharing a K/V head each project it and split its query heads. MLP intermediate columns are split
 * in 64-column units. Embedding, norms and the lm_head weight are replicated; a session whose peers
 * are mapped splits the lm_head's work by vocabulary (drt_session_tp_vocab_parallel). */
typedef struct drt_tp_shard {
  int32_t rank, world;
  int32_t q_head0, q_heads;    /* global query heads [q_head0, q_head0 + q_heads) */
  int32_t kv_head0, kv_heads;  /* global K/V heads [kv_head0, kv_head0 + kv_heads) */
  int32_t inter0, inter;       /* intermediate columns [inter0, inter0 + inter) of gate/up/down */
} drt_tp_shard;
#define DRT_TP_ID_BYTES 128
#define DRT_TP_HANDLE_BYTES 64

typedef struct drt_model drt_model;
typedef struct drt_session drt_session;

/* Model geometry: python/src/edllm/abi/lifetimes.py ModelGeometry plus the architecture
 * flags of python/src/edllm/model_definitions.py:417-448. */
typedef struct drt_model_config {
  int32_t layer_count;
  int32_t hidden_size;
  int32_t attention_heads;
  int32_t num_kv_heads;
  int32_t head_dim;          /* must be 128 */
  int32_t intermediate_size;
  int32_t vocab_size;
  int32_t qk_norm;           /* Qwen3 per-head QK RMSNorm */
  int32_t qkv_bias;          /* q/k/v projection bias (Qwen2 / Dream) */
  int32_t tied_lm_head;      /* lm_head.weight is model.embed_tokens.weight */
  float rms_norm_eps;
  float rope_theta;
  int32_t max_seq;           /* K/V capacity in positions */
  int32_t max_prefill_rows;  /* rows per prefill chunk (activation capacity) */
  int32_t logits_shift;      /* 1: dream_ar_shift (position p is scored from the logits of row
                                max(p - 1, 0), mlx_ops.shift_logits_for_dream); 0: row p itself */
} drt_model_config;

/* Session config: the keys RuntimeHandle._generate_cuda_native passes to
 * runtime.session(...) (python/src/edllm/model.py:1055-1066). */
typedef struct drt_session_config {
  int32_t decode_strategy;     /* DRT_STRATEGY_* */
  int32_t commit_policy;       /* DRT_COMMIT_* */
  int32_t attention_mask_kind; /* DRT_MASK_* */
  int32_t block_size;
  int32_t steps;
  int32_t max_tokens;
} drt_session_config;

/* Device-resident decode request (drt_session_generate). */
typedef struct drt_generate_params {
  int32_t decode_strategy;     /* DRT_STRATEGY_BD3_FIXED_QUOTA, _BLOCK_THRESHOLD, _D2F_BLOCK_PIPELINE or _ENTROPY_COUNT */
  int32_t steps;               /* requested denoising steps (the loop's iteration limit) */
  int32_t block_size;
  int32_t max_tokens;          /* generated canvas length */
  int32_t mask_token_id;
  int32_t eos_token_id;
  double confidence_threshold; /* block threshold tau (conf >= tau); D2F pipeline tau_conf (conf > tau) */
  int32_t rounds_per_block;    /* block threshold: per-block round budget, 0 = none */
  int32_t trace_steps;         /* record up to this many drt_step_trace entries */
  /* entropy_count (full-canvas masked diffusion): EntropyCountStrategy(temperature, top_p, eps),
   * python/src/edllm/backends/diffusion_runtime.py:2079-2110. */
  double temperature;          /* entropy_count: NegEntropy logits / T (<= 0: no scaling);
                                  bd3_fixed_quota: sampling temperature (0: argmax), as drt_selector_sample;
                                  block_threshold and d2f_block_pipeline: must be 0 */
  double top_p;                /* nucleus mass (>= 1: no nucleus) */
  double eps;                  /* last timestep of linspace(1, eps, steps + 1) */
  uint64_t seed;               /* bd3_fixed_quota at temperature > 0: keys the draws */
  int32_t mask_origin;         /* d2f mask geometry origin: 0 = absolute blocks from position 0 (the
                                  BD3LM graph), -1 = the prompt length (prompt bidirectional, blocks
                                  counted from it: the Dream D2F graph), else that position */
  /* d2f_block_pipeline (D2FBlockPipelineCommit, python/src/edllm/backends/diffusion_runtime.py:1416-1704):
   * a new block joins the window when the last appended block's decoded ratio is >= add_threshold;
   * block j is fully activated when block j - 1's ratio is >= activate_threshold. Both in (0, 1]
   * (the reference defaults are 0.1 and 0.95). The prompt length minus the mask origin must be a
   * multiple of block_size, so that the pipeline's blocks are the attention's blocks. */
  double add_threshold;
  double activate_threshold;
} drt_generate_params;

typedef struct drt_generate_result {
  int32_t forward_count;
  int32_t iteration_count;
  int32_t committed_token_count;
  int32_t near_tie_steps;
  int32_t exact_tie_steps;
  int32_t stopped;
  int32_t canvas_len;
  float prefill_ms;            /* device time of the prompt prefill */
  float decode_ms;             /* device time of all denoising steps */
  float total_ms;              /* device time from the prompt upload to the canvas download */
  int32_t kernel_launches;     /* kernels this call launched (prefill + graph replays) */
  float host_enqueue_ms;       /* host wall time spent enqueueing the denoising steps */
} drt_generate_result;

/* One recorded denoising step (device-resident loop). */
typedef struct drt_step_trace {
  int32_t step, n_frontier, n_chosen, tie;
  int32_t frontier_pos[64];
  int32_t token[64];
  double conf[64];
  uint64_t chosen_mask;
} drt_step_trace;

typedef struct drt_metrics {
  int64_t forward_count;
  int64_t forwarded_rows;
  int64_t prefill_rows;
  int64_t committed_token_count;
  int64_t near_tie_steps;
  int64_t exact_tie_steps;
  double forward_ms_total;     /* device time of proposes / steps */
  int64_t device_bytes;        /* device memory held by the session */
} drt_metrics;

/* ------------------------------------------------------------------ library */
/* Reference: python/src/edllm/abi/__init__.py:14 (ABI_VERSION). */
int drt_abi_version(int32_t* major, int32_t* minor, int32_t* patch);
/* Text of the last error raised on this thread ("" if none). */
const char* drt_last_error(void);
/* Number of visible CUDA devices (0 on a host without a GPU). */
int drt_device_count(int32_t* count);

/* ------------------------------------------------------------------ model (weights) */
/* Reference: diffusorrt_runtime.Runtime(package_dir, engine_config, precision, device_ordinal)
 * (python/src/edllm/model.py:873-920). Allocates device weights for `config`. */
int drt_model_create(const drt_model_config* config, int32_t device_ordinal, drt_model** out);
/* Seeded synthetic weights (counter-based generator, reproducible bit for bit on the host):
 * linears N(0, linear_std^2)-shaped, embedding embed_std, biases bias_std, norms 1. */
int drt_model_init_synthetic(drt_model* model, uint64_t seed, float linear_std, float embed_std, float bias_std);
/* Load one tensor by its package key (python/src/edllm/graph/emitter.py:88-276 names, e.g.
 * "model.layers.3.self_attn.q_proj.weight", "model.norm.weight", "lm_head.weight").
 * data: host bf16 (dtype 0) or f32 (dtype 1) [rows x cols], row-major. */
int drt_model_set_tensor(drt_model* model, const char* key, const void* data, int32_t dtype, int64_t rows, int64_t cols);
/* Copy one tensor back to the host as bf16 (dtype 0) or f32 (dtype 1). */
int drt_model_get_tensor(drt_model* model, const char* key, void* data, int32_t dtype, int64_t rows, int64_t cols);
/* RoPE half tables cos/sin [n_pos x head_dim/2] f32, as built by the reference
 * (python/src/edllm/backends/mlx_forward.py:1566-1595). */
int drt_model_set_rope(drt_model* model, const float* cos_half, const float* sin_half, int32_t n_pos);
int64_t drt_model_device_bytes(const drt_model* model);
/* Quantize every layer linear (q/k/v/o, gate/up, down) and lm_head in groups of 64 inputs; the
 * embedding stays bf16. Call again after drt_model_set_tensor to refresh the copies. group_size 64
 * only (else DRT_UNSUPPORTED).
 *  bits 4: 4-bit affine (reference _quantize_linear_weights, mlx_dream.py:2090-2108, keys
 *    :2033-2087); later forwards follow the quantized-matmul output contract (no bf16 rounding of
 *    linear outputs, mlx_ops.py:108-117).
 *  bits 8: the CUDA int8_weight_only precision (device_runtime.py:19-56, engine_config
 *    linear_quant_bits 8): int8 weights with one absmax scale per group; bf16 activations, f32
 *    accumulation and bf16-rounded outputs, as the bf16 linears.
 * The quantizers' rounding rules are defined in diffusorrt_b200/csrc/quant.cuh. */
int drt_model_quantize(drt_model* model, int32_t bits, int32_t group_size);
void drt_model_destroy(drt_model* model);
/* Shard of rank `rank` in a group of `world` (host only; no device call). */
int drt_tp_shard_geometry(const drt_model_config* config, int32_t rank, int32_t world, drt_tp_shard* out);
/* The value a row-split linear raises in the peers' flag arrays for forward `epoch`, layer `layer`,
 * which = 0 (o_proj) or 1 (down_proj); reducers wait for a value >= it. Host only: exposed so the
 * epoch / tag arithmetic can be checked without a GPU (every flag of one epoch lies below every flag
 * of the next for any layer count a session accepts). */
uint64_t drt_tp_flag_value(uint64_t epoch, int32_t layer, int32_t which);
/* A new NCCL unique id (DRT_TP_ID_BYTES bytes) for drt_model_create_tp; made by one rank and
 * shared with the others by the caller (torch.distributed in the Python binding). */
int drt_tp_unique_id(uint8_t* id);
/* drt_model_create for one rank's shard, joined to the group's NCCL communicator (blocks until
 * every rank has joined). Weights: drt_model_init_synthetic fills the shard's block of the same
 * logical tensors a whole model gets; drt_model_set_tensor takes FULL logical tensors and keeps the
 * shard's block. Sessions on a sharded model serve entropy_count only: the layer forward
 * all-reduces the f32 o_proj and down_proj partials over the group, then adds bf16(sum) to the
 * replicated residual, so every rank holds the same hidden state, logits and selections. */
int drt_model_create_tp(const drt_model_config* config, int32_t device_ordinal, int32_t rank, int32_t world,
                        const uint8_t* nccl_id, drt_model** out);

/* ------------------------------------------------------------------ session */
/* Reference: Runtime.session(session_config) (python/src/edllm/model.py:1055-1067). */
int drt_session_open(drt_model* model, const drt_session_config* config, drt_session** out);
/* Reference: session.start_device(x, prompt_len, block_size, mask_token_id, exact_kv, steps,
 * memory_budget_bytes, temperature, seed) (python/src/edllm/backends/device_runtime.py:140-150).
 * `prompt_len` is the mask-geometry origin (0 for BD3's absolute blocks).
 * exact_kv != 0: each propose reuses the K/V of the frozen prefix computed by earlier forwards (exact
 * under the d2f_hybrid mask); exact_kv == 0: each propose recomputes the whole window's K/V (the
 * reference's cache-off shape; `forwarded` then counts the whole window). A bidirectional
 * (entropy_count) session refuses exact_kv (DRT_INVALID_ARGUMENT, as device_runtime.py:125-126) and
 * decodes through drt_session_generate only (start_device returns DRT_UNSUPPORTED).
 * temperature > 0 (bd3_fixed_quota only; block_threshold refuses it): each propose draws every
 * frontier row's token as drt_selector_sample does, keyed by `seed`, the propose's index since
 * start_device and the row's position; the score is the raw probability of the drawn token. */
int drt_session_start(drt_session* s, const int32_t* x, int32_t n, int32_t prompt_len, int32_t block_size,
                      int32_t mask_token_id, int32_t exact_kv, int32_t steps, int64_t memory_budget_bytes,
                      double temperature, uint64_t seed);
/* Reference: session.propose_device(frontier, window_end=, frozen_prefix=) -> (scores,
 * token_ids, forwarded) in frontier order (device_runtime.py:152-178). scores: f64 raw
 * max-probability; token_ids: argmax; forwarded: rows computed by this forward. */
int drt_session_propose(drt_session* s, const int32_t* frontier, int32_t n_frontier, int32_t window_end,
                        int32_t frozen_prefix, double* scores, int32_t* token_ids, int32_t* forwarded);
/* Reference: session.commit_device(positions, token_ids) (diffusion_runtime.py:749-753). */
int drt_session_commit(drt_session* s, const int32_t* positions, const int32_t* token_ids, int32_t n);
/* Reference: session.execute_window(token_ids, scope, mask_geometry=(prompt_len, block_size))
 * (device_runtime.py:354-363): selection-ready f32 logits [n_scope x vocab] of the scope
 * rows, in scope order. No cache: the whole window is forwarded. */
int drt_session_execute_window(drt_session* s, const int32_t* token_ids, int32_t n_tokens, const int32_t* scope,
                               int32_t n_scope, int32_t prompt_len, int32_t block_size, float* logits,
                               int32_t* forwarded_rows);
/* Whole request on the device: prefill, then CUDA-graph denoising steps whose plan, score,
 * select and commit all run on the GPU. prompt/out are host buffers; out receives the final
 * canvas (prompt + max_tokens). trace (optional, host) receives params->trace_steps entries. */
int drt_session_generate(drt_session* s, const drt_generate_params* params, const int32_t* prompt,
                         int32_t prompt_len, int32_t* out, drt_generate_result* result, drt_step_trace* trace);
/* Tensor-parallel sessions over peer memory: each rank's session owns a receive buffer for the
 * o_proj / down_proj partials of every rank. drt_session_tp_handle gives its CUDA IPC handle
 * (DRT_TP_HANDLE_BYTES); after the caller has gathered every rank's handle (rank order),
 * drt_session_tp_connect maps the peers' buffers. From then on each such linear stores its f32
 * partial straight into every rank's buffer over NVLink from its epilogue and a flag-gated kernel
 * adds bf16(sum) to the residual (no NCCL call on the data path). Without it the session uses the
 * NCCL all-reduce. Both calls are collective over the group. */
int drt_session_tp_handle(drt_session* s, void* handle);
int drt_session_tp_connect(drt_session* s, const void* handles, int32_t world);
/* Vocabulary-parallel lm_head of a connected tensor-parallel session (no counterpart in the
 * reference, which runs on one device; the multi-GPU Dream benchmark configuration splits the
 * lm_head by vocabulary): rank r projects vocabulary tiles [r T / w, (r + 1) T / w) of the T 128-row tiles and its
 * epilogue stores them into every rank's logits over NVLink, so every rank's selector sees the
 * whole row, bit-identical to one GPU's. On by default once drt_session_tp_connect has mapped the
 * peers (for a bf16 model whose vocabulary is a multiple of 128 with at least one tile per rank);
 * enable = 0 makes every rank project the whole vocabulary again. Collective: every rank passes
 * the same value before its next request. Used by the entropy_count (Dream) step. */
int drt_session_tp_vocab_parallel(drt_session* s, int32_t enable);
/* Failure-handling drill (no counterpart in the reference, whose ABI reports failures as
 * INTERNAL_ERROR, python/src/edllm/abi/forward.py:20-25): runs, on the session's stream, the bounded
 * wait a tensor-parallel reducer makes for a peer's partials, on a flag that nothing raises — what a
 * rank sees when a peer has stopped. It returns DRT_DEVICE_TIMEOUT once the device wait limit (2 s)
 * has passed; no GPU fault is raised, and the session, its stream and the context stay usable. */
int drt_session_peer_wait_drill(drt_session* s);
/* entropy_count transfer schedule (EntropyCountCommit.plan, diffusion_runtime.py:921-937):
 * timesteps = linspace(1, eps, steps + 1) in float32, transfer[s] = int(N * (1 - t[s+1] / t[s]))
 * (all N remaining on the last step) for s < steps, from n_masked masked positions, N falling by
 * each step's transfer. 0 marks a skipped step and every step after the canvas is full. Host only. */
int drt_entropy_count_schedule(int32_t n_masked, int32_t steps, double eps, int32_t* transfer);
/* Reference: session.device_metrics() (python/src/edllm/model.py:1087). */
int drt_session_metrics(drt_session* s, drt_metrics* out);
/* Raw device pointers of the session's K/V cache planes (tests): K [L*nkv][max_seq][128],
 * V^T [L*nkv][128][max_seq], both bf16. */
int drt_session_kv_pointers(drt_session* s, void** k_cache, void** vt_cache);
void drt_session_close(drt_session* s);

/* ------------------------------------------------------------------ kernels (device pointers) */
/* Fused selector over rows of f32 logits (reference _raw_max_prob_rows_exact,
 * diffusion_runtime.py:179-192, and _entropy_confidence without top-p, :90-114).
 * conf[r] (f64) and token[r] (i32) for r < n_rows. scratch: see drt_selector_scratch_bytes. */
size_t drt_selector_scratch_bytes(int32_t n_rows, int32_t vocab);
int drt_selector_rows(const float* logits, int64_t ld, int32_t n_rows, int32_t vocab, int32_t mode,
                      double temperature, void* scratch, double* conf, int32_t* token, void* stream);
/* The selector over gathered rows: row r reads logits row row_index[r] (device int32), the way the
 * reference scores only the masked frontier (diffusion_runtime.py:1946-1949 gathers the masked
 * rows, then _raw_max_prob_confidence :136-165 / _entropy_confidence :90-114 score them).
 * Same scratch, modes and outputs as drt_selector_rows. */
int drt_selector_gather(const float* logits, int64_t ld, const int32_t* row_index, int32_t n_rows, int32_t vocab,
                        int32_t mode, double temperature, void* scratch, double* conf, int32_t* token, void* stream);
/* NegEntropy confidence with a top-p nucleus (_entropy_confidence, diffusion_runtime.py:90-114, with
 * _top_p_filter :358-370 and _softmax :373-378) of the rows row_index[r] (NULL: row r) of f32 logits
 * [.., ld]: conf[r] = f32(sum p' log(p' + 1e-10)) over the nucleus-renormalised softmax of x / T
 * (stored as f64), token[r] = its argmax. exclude_token (-1: none) is scored as -inf
 * (_exclude_mask_token, :256-282). tie (optional) gets DRT_TIE_NEAR when a cumulative mass at the
 * nucleus cut is within tie_rel of top_p, DRT_TIE_EXACT when the cut keeps part of a tied maximum. */
int drt_selector_topp(const float* logits, int64_t ld, const int32_t* row_index, int32_t n_rows, int32_t vocab,
                      double temperature, double top_p, int32_t exclude_token, double tie_rel, double* conf,
                      int32_t* token, int32_t* tie, void* stream);
/* The selector's exp for non-positive arguments (table-driven, Tang 1989), y[i] = exp(x[i]) for
 * x[i] <= 0, on device arrays; exposed so its accuracy against CUDA's exp can be tested. */
int drt_exp_nonpos(const double* x, double* y, int64_t n, void* stream);
/* Temperature sampling over rows (row_index NULL: row r) of f32 logits, the reference's
 * _sampled_max_prob_confidence with sampling_noise (diffusion_runtime.py:195-253): token[r] = the
 * first argmax over v of f64(x_v) + T * f64(g_v), g = -log(-log u) in float32 with u from a splitmix64
 * hash of (seed, forward, positions[r] (device int32), v); conf[r] = exp(x_tok - max) / S in f64.
 * tie (optional) gets DRT_TIE_NEAR where the two best keys lie within 2^-16 T, the most a last-bit
 * difference of the float32 logs can move a key. Scratch: drt_selector_scratch_bytes. */
int drt_selector_sample(const float* logits, int64_t ld, const int32_t* row_index, int32_t n_rows, int32_t vocab,
                        double temperature, uint64_t seed, int32_t forward, const int32_t* positions, void* scratch,
                        double* conf, int32_t* token, int32_t* tie, void* stream);
/* Commit choices for a batch of confidence runs: item b owns rows offsets[b] .. offsets[b + 1]
 * (device int32, n_items + 1 entries). mode 0 = top-k (_topk_count_choices,
 * diffusion_runtime.py:290-299: the k highest, lowest row first among equals), mode 1 =
 * threshold (_threshold_choices, :302-314: conf >= tau, else the first argmax). Writes
 * chosen[row] in {0, 1} and tie[b]: bit 1 when the deciding gap (k-th vs (k+1)-th, |conf - tau|,
 * or top-1 vs top-2 without a hit) is within tie_rel relative, bit 2 when it is an exact tie. */
int drt_select_choices(const double* conf, const int32_t* offsets, int32_t n_items, int32_t mode, int32_t k, double tau,
                       double tie_rel, int32_t* chosen, int32_t* tie, void* stream);
/* The same selector without any device allocation, for callers that may not allocate device
 * memory: a host whose GPU memory is owned by its own pool or fixed budget (outside of which it
 * may not cudaMalloc), or a latency-critical caller that cannot afford cudaMalloc's implicit
 * synchronization. No counterpart in the reference. The scratch is one static device array of
 * about 0.81 MB that every GPU loading this library keeps until exit; calls are limited to
 * n_rows <= 1024 and vocab <= 262144 (larger calls fail with DRT_INVALID_ARGUMENT). The first call
 * in each CUDA context looks up the array's device address (cached under the context's id, so a
 * context made after cudaDeviceReset, or a second context on the same device, looks it up again),
 * so make that first call before any stream capture. All calls share the array: calls that overlap
 * on the GPU (other streams, other threads) race and must be serialized by the caller. */
int drt_selector_rows_noalloc(const float* logits, int64_t ld, int32_t n_rows, int32_t vocab, int32_t mode,
                              double temperature, double* conf, int32_t* token, void* stream);
/* y = x @ W^T on the tensor cores with the MLX rounding contract (bf16 output rounding when
 * round_bf16 != 0). x [rows x K] bf16, w [n x K] bf16, y [rows x n] f32; n % 128 == 0,
 * K % 64 == 0; splits in {1, 2, 4, 8, 16} (split-K CTAs of a tile form one thread-block cluster
 * and reduce through distributed shared memory, so scratch may be NULL and
 * drt_linear_scratch_bytes returns 0). */
/* 4-bit affine quantization of a bf16 weight w [rows x K] (device pointers): q [rows x K/2] packed
 * nibbles (input 2j in the low nibble of byte j), scale / bias [rows x K/64] bf16 (quant.cuh). */
int drt_quantize_q4(const void* w, int64_t rows, int32_t K, void* q, void* scale, void* bias, void* stream);
/* y = x @ dequant(q, scale, bias)^T for rows <= 64: x bf16 [rows x K], y f32 [rows x n] (no output
 * rounding, the quantized-matmul contract); n % 128 == 0, K % 64 == 0, splits in {1, 2, 4, 8, 16}
 * with at most 8 groups of 64 inputs per split. The decode linear's quantized instantiation. */
int drt_linear_q4(const void* x, const void* q, const void* scale, const void* bias, float* y, int32_t rows, int32_t n,
                  int32_t K, int32_t splits, void* stream);
/* int8 weight-only quantization of a bf16 weight w [rows x K] (device pointers): q [rows x K] bytes
 * holding the signed weight + 128, scale [rows x K/64] bf16 (absmax / 127) and bias = -128 * scale,
 * the affine form the decode linear dequantizes (quant.cuh). */
int drt_quantize_q8(const void* w, int64_t rows, int32_t K, void* q, void* scale, void* bias, void* stream);
/* y = x @ dequant(q, scale, bias)^T for rows <= 64 with the int8 weight-only contract (bf16 dequantized
 * weights, f32 accumulation, outputs rounded to bf16 and widened to f32); shapes as drt_linear_q4. */
int drt_linear_q8(const void* x, const void* q, const void* scale, const void* bias, float* y, int32_t rows, int32_t n,
                  int32_t K, int32_t splits, void* stream);
size_t drt_linear_scratch_bytes(int32_t rows, int32_t n, int32_t K, int32_t splits);
int drt_linear_bf16(const void* x, const void* w, float* y, int32_t rows, int32_t n, int32_t K, int32_t splits,
                    int32_t round_bf16, void* scratch, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* DIFFUSORRT_B200_H_ */
