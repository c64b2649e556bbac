/*
 * lewm_b200.h -- C ABI of the B200 (sm_100a) LeWM iCEM planning hot path.
 *
 * Plain pointers and sizes only. Every tensor pointer is a CUDA device pointer
 * on the context's device unless a comment says otherwise; float tensors are
 * contiguous row-major float32. Calls are asynchronous on the given stream
 * (a cudaStream_t passed as void*; NULL = legacy default stream) and the
 * caller owns every buffer. One context per device; a context is not
 * thread-safe without external locking, and its calls share its workspace, so
 * calls on one context must be ordered on the GPU (one stream, or streams the
 * caller orders with events).
 *
 * lewm_plan (without a trace or injected noise) and lewm_model_cost_grad capture
 * their launches into a CUDA graph on the first call of each shape, on a stream
 * of the context, and replay that graph on later calls (LEWM_NO_GRAPH=1 turns
 * this off): do not call them while the given stream is being captured.
 *
 * The reference (antoinenguyen27/lewm-flash) is pure PyTorch and has no FFI;
 * each entry point below replaces one Python interface of its planning path,
 * cited as file:line in that project.
 */
#ifndef LEWM_B200_H
#define LEWM_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define LEWM_ABI_VERSION 3

#if defined(__GNUC__)
#define LEWM_API __attribute__((visibility("default")))
#else
#define LEWM_API
#endif

typedef enum lewm_status {
  LEWM_OK = 0,
  LEWM_INVALID_ARG = 1,       /* bad pointer, size or option (reference: ValueError) */
  LEWM_UNSUPPORTED_SHAPE = 2, /* a model / plan shape the kernels are not built for */
  LEWM_DEVICE_TIMEOUT = 3,    /* a bounded device-side wait expired */
  LEWM_NUMERIC_NAN = 4,       /* NaN in a plan's final costs */
  LEWM_CUDA_ERROR = 5,        /* CUDA runtime error; see lewm_last_error */
  LEWM_OUT_OF_MEMORY = 6
} lewm_status;

typedef struct lewm_ctx lewm_ctx;

/* Predictor + action-encoder shape (reference lewm/module.py:189-285).
 * Supported: dim in {192, 384}, dim_head == 64, heads <= 16, mlp_dim and
 * embed_hidden multiples of 128, action_dim and smoothed_dim <= 16,
 * num_frames <= 8. pred_proj (JEPA.predict, lewm/jepa.py:106-114): Identity
 * (pred_proj_hidden == 0), or the MLP head of lewm/module.py:217-240 at dim 192
 * with a hidden width that is a multiple of 256 and LayerNorm / BatchNorm1d
 * (eval, eps 1e-5) / no norm. */
typedef struct lewm_model_desc {
  int32_t dim;
  int32_t depth;
  int32_t heads;
  int32_t dim_head;
  int32_t mlp_dim;
  int32_t action_dim;
  int32_t smoothed_dim;
  int32_t embed_hidden;
  int32_t num_frames;
  int32_t pred_proj_hidden; /* 0: Identity */
  int32_t pred_proj_norm;   /* 0 none, 1 LayerNorm, 2 BatchNorm1d (eval) */
} lewm_model_desc;

/* Number of float32 values lewm_create expects for `desc`. The weights are the
 * reference JEPA state-dict tensors (predictor.*, action_encoder.*, pred_proj.*)
 * concatenated in this order, each row-major:
 *   predictor.pos_embedding
 *   for each layer l: adaLN_modulation.1.weight, .bias, attn.norm.weight, .bias,
 *     attn.to_qkv.weight, attn.to_out.0.weight, .bias, mlp.net.0.weight, .bias,
 *     mlp.net.1.weight, .bias, mlp.net.4.weight, .bias
 *   transformer.norm.weight, .bias
 *   action_encoder.patch_embed.weight, .bias, embed.0.weight, .bias, embed.2.weight, .bias
 *   with an MLP head: pred_proj.net.0.weight, .bias, then net.1.weight, .bias (LayerNorm)
 *     or net.1.weight, .bias, .running_mean, .running_var (BatchNorm1d), then
 *     net.3.weight, .bias
 * (host memory). */
LEWM_API size_t lewm_weight_count(const lewm_model_desc* desc);

/* Build a context on `device`: validates `desc`, packs `weights` (HOST float32,
 * `n_floats` values, lewm_weight_count order) into bf16 tensor-core tiles and
 * uploads them. Replaces loading the reference JEPA predictor onto the GPU
 * (reference tools/benchmarks/lewm_plan_benchmark.py:1855-1857). */
LEWM_API lewm_status lewm_create(lewm_ctx** out, const lewm_model_desc* desc, const float* weights, size_t n_floats,
                        int device);
LEWM_API void lewm_destroy(lewm_ctx* ctx);
/* Message of the last failing call on `ctx` ("" if none). NULL ctx: last lewm_create failure. */
LEWM_API const char* lewm_last_error(const lewm_ctx* ctx);

/* Model-cost arithmetic of a context (reference JEPA.set_model_cost_autocast,
 * lewm/jepa.py:65-86, whose modes are "none" and "bf16"). */
#define LEWM_AUTOCAST_NONE 0 /* float32 throughout: the reference without autocast */
#define LEWM_AUTOCAST_BF16 1 /* bf16 tensor-core GEMMs, fp32 norms / residual / cost (the default) */

/* Select the arithmetic of every later lewm_model_cost / lewm_plan / lewm_profile_plan on
 * `ctx`. LEWM_AUTOCAST_BF16 (the default of a new context) runs the tcgen05 kernels;
 * LEWM_AUTOCAST_NONE runs the same model in float32 on CUDA cores (tiled SIMT GEMMs with
 * fused epilogues, two-pass LayerNorms, erf GELU): the reference's float32 costs within its
 * 1e-5 exactness tolerance (tools/benchmarks/check_lewm_cache_exactness.py:783-784), at a
 * fraction of the bf16 throughput. Any other mode: LEWM_INVALID_ARG. Synchronizes the
 * context's device and drops its captured plan graphs. */
LEWM_API lewm_status lewm_set_model_cost_autocast(lewm_ctx* ctx, int32_t mode);

/* Terminal latent cost of each action candidate.
 * Replaces JEPA.get_cost_from_embeddings(emb, goal_emb, action_candidates, history_size)
 * (reference lewm/jepa.py:302-317), i.e. rollout_from_embeddings (:262-300) and
 * cost_from_rollout (:246-260), computed with bf16 tensor-core GEMMs and fp32
 * norms/residuals/cost, or in float32 throughout under LEWM_AUTOCAST_NONE.
 *   emb   (B,H,D) if emb_per_sample == 0, else (B,S,H,D)
 *   goal  (B,D)   if goal_per_sample == 0, else (B,S,D): the last goal row
 *   cand  (B,S,T,A)
 *   costs_out (B,S)
 * 1 <= H <= T, 1 <= history_size <= num_frames. */
LEWM_API lewm_status lewm_model_cost(lewm_ctx* ctx, const float* emb, int32_t emb_per_sample, int32_t H, const float* goal,
                            int32_t goal_per_sample, const float* cand, int32_t B, int32_t S, int32_t T,
                            int32_t history_size, float* costs_out, void* stream);

/* Model costs and their gradient with respect to the action candidates: the gradient
 * CEM-GD's refinement steps on (reference lewm/solvers/cem_gd.py:459-606 takes torch
 * autograd of JEPA.get_cost_from_embeddings, lewm/jepa.py:302-317). Float32 forward and
 * reverse pass on CUDA cores whatever the context's autocast mode (a bf16 rollout has no
 * useful gradient at this precision). Arguments as lewm_model_cost, plus
 *   cost_weights (B,S) device, or NULL for all ones: w in d(sum_c w_c cost_c) / d cand;
 *     candidates are independent, so grad_out[c] = w_c * d cost_c / d cand_c
 *   grad_out (B,S,T,A)
 * The embeddings and the goal are constants (no gradient). Needs an Identity pred_proj
 * (LEWM_UNSUPPORTED_SHAPE otherwise) and B*S*T <= 2^22. Keeps the forward's activations
 * in a context buffer that grows to the largest call (about 1.5 MB per candidate at
 * width 192, T 5, window 3). */
LEWM_API lewm_status lewm_model_cost_grad(lewm_ctx* ctx, const float* emb, int32_t emb_per_sample, int32_t H,
                                          const float* goal, int32_t goal_per_sample, const float* cand, int32_t B,
                                          int32_t S, int32_t T, int32_t history_size, const float* cost_weights,
                                          float* costs_out, float* grad_out, void* stream);

/* iCEM solver options (reference ICEMSolver.__init__, lewm/solvers/icem.py:258-322). */
typedef struct lewm_plan_desc {
  int32_t n_envs;           /* B */
  int32_t horizon;          /* T */
  int32_t history;          /* H (rows of emb per env) */
  int32_t history_size;     /* predictor window (JEPA default 3) */
  int32_t num_samples;      /* S */
  int32_t topk;             /* k */
  int32_t n_steps;          /* iCEM iterations */
  double sample_decay;      /* >= 1 (a Python float in the reference) */
  int32_t bucket;           /* sample_count_bucket_size >= 0 */
  int32_t elite_retention;  /* >= 0 */
  float beta;               /* colored-noise exponent: 0 white, 1 pink, 2 brown */
  int32_t time_axis_raw;    /* 1: color over horizon*action_block raw steps; 0: over horizon */
  int32_t action_block;     /* >= 1 */
  float momentum_alpha;     /* [0, 1) */
  int32_t return_best_elite;
  int32_t clip_actions;     /* clamp to action_low/high */
  uint64_t seed;            /* Philox key word 0 */
  uint64_t plan_index;      /* Philox key word 1: a new stream per plan call */
  /* NULL: the sample count of iteration i follows the schedule of
   * ICEMSolver.sample_count_for_step (num_samples, sample_decay, bucket).
   * Else a HOST array of n_steps counts, each in [topk, num_samples], used as
   * given: the sample counts of an arbitrary list of noise tensors, as the
   * reference's run_static_icem_chain accepts (lewm/solvers/icem_static_compile.py:61-114). */
  const int32_t* sample_counts;
} lewm_plan_desc;

/* LEWM_ABI_VERSION of the loaded library (a binding checks it against the header it was written for). */
LEWM_API int32_t lewm_abi_version(void);

/* Per-iteration device outputs for solver callbacks / debugging (any may be NULL).
 * i = iteration, S = num_samples (rows past the iteration's sample count are unset). */
typedef struct lewm_plan_trace {
  float* costs;       /* [n_steps][B][S] */
  int32_t* topk_idx;  /* [n_steps][B][k] ascending cost */
  float* topk_val;    /* [n_steps][B][k] */
  float* mean;        /* [n_steps][B][T][A] after refit */
  float* std;         /* [n_steps][B][T][A] after refit */
  float* candidates;  /* [n_steps][B][S][T][A] */
} lewm_plan_trace;

/* Sample counts of every iteration (reference ICEMSolver.sample_counts,
 * lewm/solvers/icem.py:377-394). Writes min(n_steps, cap) counts; returns the
 * total model-cost evaluations per env in *evals_out (may be NULL). HOST memory. */
LEWM_API lewm_status lewm_sample_counts(const lewm_plan_desc* plan, int32_t* counts_out, int32_t cap, int64_t* evals_out);

/* One full iCEM solve for B independent envs, with no host round trip.
 * Replaces the per-env-batch iteration loop of ICEMSolver.solve
 * (lewm/solvers/icem.py:501-588) and the tensor-only run_static_icem_chain
 * (lewm/solvers/icem_static_compile.py:61-114).
 *   emb (B,H,D), goal (B,D), init_mean/init_std (B,T,A)
 *   noise_steps: NULL -> in-kernel Philox colored noise; else n_steps device
 *     pointers (a HOST array of device pointers), step i of shape
 *     (B, counts[i], T, A): the reference's post-coloring noise ("injection mode")
 *   action_low/high (A) device, used when clip_actions
 *   actions_out (B,T,A): final mean, or the best elite if return_best_elite
 *   std_out (B,T,A), final_cost_out (B): mean of the last top-k costs
 *   trace: optional per-iteration outputs. */
LEWM_API lewm_status lewm_plan(lewm_ctx* ctx, const lewm_plan_desc* plan, const float* emb, const float* goal,
                      const float* init_mean, const float* init_std, const float* const* noise_steps,
                      const float* action_low, const float* action_high, float* actions_out, float* std_out,
                      float* final_cost_out, const lewm_plan_trace* trace, void* stream);

/* One elite selection + refit step on given costs (reference
 * lewm/solvers/icem.py:543-563, lewm/solvers/icem_static_compile.py:95-107).
 *   costs (B,S), cand (B,S,T,A), mean/std (B,T,A) updated in place,
 *   topk_idx (B,k) / topk_val (B,k) ascending (ties: lower index), best (B,T,A),
 *   final_cost (B). */
LEWM_API lewm_status lewm_topk_refit(lewm_ctx* ctx, const float* costs, const float* cand, int32_t B, int32_t S, int32_t T,
                            int32_t A, int32_t k, float momentum_alpha, float* mean, float* std, int32_t* topk_idx,
                            float* topk_val, float* best, float* final_cost, void* stream);

/* Candidate sampling alone (tests / diagnostics): candidates of iteration
 * `iter` for the given mean/std, no elite injection. Reference
 * make_colored_noise (lewm/solvers/icem.py:185-250) + :523-527.
 * mean/std (B,T,A), injected_noise (B,S,T,A) or NULL, out (B,S,T,A), with
 * B = plan->n_envs, T = plan->horizon and A the context's model action_dim
 * (the buffers are not self-describing: a caller must size them with that A). */
LEWM_API lewm_status lewm_sample_candidates(lewm_ctx* ctx, const lewm_plan_desc* plan, int32_t S, int32_t iter,
                                   const float* mean, const float* std, const float* injected_noise,
                                   const float* action_low, const float* action_high, float* out, void* stream);

/* Candidate sampling that allocates nothing. No counterpart in the reference:
 * it serves callers that cannot allocate device memory where they sample (all
 * memory handed to their own pool, or no context at hand). Same candidates as
 * lewm_sample_candidates for the same plan fields, S, iter, mean and std, on
 * device `device` for an action dimension `action_dim`; no context.
 *   Scratch: one fixed array of 65,792 bytes per device inside the library
 *   (a coloring matrix of at most 128 x 128 plus the Philox key); a colored
 *   time length (horizon*action_block for raw time, else horizon) above 128,
 *   or horizon*action_dim above 128, returns LEWM_UNSUPPORTED_SHAPE.
 *   The first call on a device looks up that array's address (and may load
 *   the module there): make it before any stream capture. The address is kept
 *   for the life of the process: after cudaDeviceReset on a device, do not call
 *   this entry point on that device again.
 *   Calls that overlap on the GPU (unordered streams) share the scratch and
 *   race; order them on one stream or with events.
 *   Errors: text from lewm_last_error(NULL). */
LEWM_API lewm_status lewm_sample_candidates_noalloc(const lewm_plan_desc* plan, int32_t action_dim, int32_t S,
                                           int32_t iter, const float* mean, const float* std,
                                           const float* injected_noise, const float* action_low,
                                           const float* action_high, float* out, int32_t device, void* stream);

/* The real n x n matrix W with irfft(rfft(x) * scale, n) == W x, scale_f = (f/n)^(-beta/2),
 * scale_0 = scale_1: the temporal coloring of _colored_noise_along_time
 * (lewm/solvers/icem.py:173-182) as a matrix. HOST memory, row-major. */
LEWM_API lewm_status lewm_coloring_matrix(int32_t n, double beta, double* out);

/* Kernel classes reported by lewm_profile_plan, in array order. */
#define LEWM_KERNEL_CLASSES 14 /* embed, adaln, qkv_attn, out_proj, fc1, fc2, final, sample, refit, prep0, \
                                  ffn (fused FC1 + GELU + FC2), ln_operand (per-tile GEMM operand), \
                                  tile_call (all layers of a predictor call per row tile), \
                                  fp32_cost (a whole float32 model cost, LEWM_AUTOCAST_NONE) */

/* Run one plan (in-kernel noise) with a CUDA event pair around every kernel
 * launch, synchronize, and report per kernel class: summed device ms,
 * algorithmic FLOPs (valid rows x GEMM shape) and launch count. HOST output
 * arrays of LEWM_KERNEL_CLASSES entries. Diagnostics only: the events
 * serialize launches, so use lewm_plan for timing whole plans. No reference
 * counterpart (the reference profiles with torch.profiler,
 * tools/benchmarks/lewm_plan_benchmark.py:1455-1475). */
LEWM_API lewm_status lewm_profile_plan(lewm_ctx* ctx, const lewm_plan_desc* plan, const float* emb, const float* goal,
                                       const float* init_mean, const float* init_std, double* ms_out,
                                       double* flops_out, int32_t* launches_out, void* stream);

/* Synchronize `stream`, then read and clear the device status word of `ctx`:
 * LEWM_DEVICE_TIMEOUT if any bounded wait expired since the last call, else
 * LEWM_NUMERIC_NAN if a plan since the last call produced a NaN final cost. */
LEWM_API lewm_status lewm_sync_status(lewm_ctx* ctx, void* stream);

/* Time limit of every bounded device-side wait (mbarrier phases of bulk copies and
 * MMA completion) in kernels launched on `ctx` from now on, in nanoseconds of
 * %globaltimer; 0 restores the default of 2 s. A wait that runs out sets the
 * timeout bit of the context's status word, the kernel skips its dependent work,
 * releases its tensor memory and returns; lewm_sync_status then reports
 * LEWM_DEVICE_TIMEOUT. No reference counterpart (the reference's PyTorch kernels
 * have no bounded waits). Takes effect for kernels enqueued after it returns; it
 * synchronizes the context's device. */
LEWM_API lewm_status lewm_set_wait_limit(lewm_ctx* ctx, uint64_t limit_ns);

/* Failure-detection self-test: enqueue on `stream` one device wait on a barrier that
 * nothing ever completes, bounded by the context's wait limit. When it runs out the
 * kernel sets the timeout bit and returns (nothing else is in flight), so the next
 * lewm_sync_status reports LEWM_DEVICE_TIMEOUT and the context stays usable. Set a
 * short limit first (lewm_set_wait_limit), or the call takes the 2 s default. No
 * reference counterpart. */
LEWM_API lewm_status lewm_wait_selftest(lewm_ctx* ctx, void* stream);

/* ------------------------------------------------------------------ observation encoder
 * The pixels -> embedding step in front of planning: JEPA.encode
 * (lewm/jepa.py:88-104), i.e. the CLS row of a transformers ViTModel
 * (stable-pretraining 0.1.7 `vit_hf`, tools/benchmarks/stage_lewm_weights.py:72-78)
 * followed by the projector MLP (lewm/module.py:217-240). Reached by the planner
 * through JEPA._ensure_cost_embeddings (lewm/jepa.py:319-345). */
typedef struct lewm_encoder lewm_encoder;

/* Supported: hidden == 192 with heads == hidden / 64, image_size a multiple of
 * patch_size, (image_size / patch_size)^2 + 1 <= 272 tokens, channels x patch^2
 * <= 2048, mlp_dim a multiple of 192 or 256, proj_hidden a positive multiple of
 * 256, proj_out == 192. */
typedef struct lewm_encoder_desc {
  int32_t image_size;  /* ViTConfig.image_size (224) */
  int32_t patch_size;  /* ViTConfig.patch_size (14) */
  int32_t channels;    /* ViTConfig.num_channels (3) */
  int32_t hidden;      /* ViTConfig.hidden_size (192) */
  int32_t depth;       /* ViTConfig.num_hidden_layers (12) */
  int32_t heads;       /* ViTConfig.num_attention_heads (3) */
  int32_t mlp_dim;     /* ViTConfig.intermediate_size (768) */
  float ln_eps;        /* ViTConfig.layer_norm_eps (1e-12) */
  int32_t proj_hidden; /* projector MLP hidden width (2048) */
  int32_t proj_out;    /* projector output width (192) */
  int32_t proj_norm;   /* projector norm: 0 none, 1 LayerNorm, 2 BatchNorm1d (eval) */
  float proj_eps;      /* projector norm eps (1e-5) */
} lewm_encoder_desc;

/* Float32 values lewm_encoder_create expects (0 for an unsupported desc): the
 * ViTModel and projector state-dict tensors concatenated in this order, each
 * row-major:
 *   embeddings.cls_token, embeddings.position_embeddings,
 *   embeddings.patch_embeddings.projection.weight, .bias
 *   for each layer l (encoder.layer.l.): layernorm_before.weight, .bias,
 *     attention.attention.query.weight, .bias, .key.weight, .bias, .value.weight, .bias,
 *     attention.output.dense.weight, .bias, layernorm_after.weight, .bias,
 *     intermediate.dense.weight, .bias, output.dense.weight, .bias
 *   layernorm.weight, .bias
 *   projector net.0.weight, .bias; norm (LayerNorm: weight, bias; BatchNorm1d:
 *     weight, bias, running_mean, running_var; none: nothing); net.3.weight, .bias */
LEWM_API size_t lewm_encoder_weight_count(const lewm_encoder_desc* desc);

/* Validate `desc`, pack `weights` (HOST float32) into bf16 tensor-core tiles on
 * `device` (BatchNorm folded into the first projector Linear). Replaces building
 * and loading the reference encoder + projector (tools/benchmarks/stage_lewm_weights.py:61-103). */
LEWM_API lewm_status lewm_encoder_create(lewm_encoder** out, const lewm_encoder_desc* desc, const float* weights,
                                         size_t n_floats, int device);

/* emb_out[n_images][proj_out] = projector(ViT(pixels)[:, 0]) for pixels
 * [n_images][channels][image_size][image_size] (already normalized, as JEPA.encode
 * receives them). Device pointers; emb_out 16-byte aligned; n_images <= 65535.
 * Asynchronous on `stream`; grows the encoder's workspace on first use of a larger
 * batch. */
LEWM_API lewm_status lewm_encode(lewm_encoder* enc, const float* pixels, int32_t n_images, float* emb_out,
                                 void* stream);

/* lewm_encode from raw uint8 frames [n_images][image_size][image_size][channels]
 * (height, width, channel; device memory): each sample is normalized in the first
 * kernel as (u * float32(1/255) - mean[c]) / std[c] (mean, std: HOST arrays of
 * `channels` floats, channels <= 4), the arithmetic of the policy image transform
 * ToDtype(float32, scale=True) + Normalize (lewm/eval.py:17-26) for frames already at
 * image_size (its Resize is then the identity). Bit-identical to lewm_encode on the
 * transformed float pixels, with a quarter of the input bytes. */
LEWM_API lewm_status lewm_encode_u8(lewm_encoder* enc, const uint8_t* frames, int32_t n_images, const float* mean,
                                    const float* std, float* emb_out, void* stream);

/* Synchronize `stream`, then read and clear the encoder's device status word. */
LEWM_API lewm_status lewm_encoder_sync_status(lewm_encoder* enc, void* stream);
LEWM_API const char* lewm_encoder_last_error(const lewm_encoder* enc);
LEWM_API void lewm_encoder_destroy(lewm_encoder* enc);

#ifdef __cplusplus
}
#endif

#endif /* LEWM_B200_H */
