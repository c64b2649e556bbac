// Internal layouts shared by the kernels and the C-ABI layer.
//
// Device memory layout (all bf16 operand tiles are K-major, 128-byte
// swizzled [rows x 64] blocks, so one bulk copy lands a block ready for
// tcgen05.mma):
//
//   weights (read-only, packed once by lewm_create)
//     qkv  [L][heads][D/64]      blocks of [192 x 64]   rows = q|k|v of one head
//     wout [L][4][inner/64]      blocks of [D/4 x 64]
//     w1   [L][mlp/128][D/64]    blocks of [128 x 64]
//     w2   [L][4][mlp/64]        blocks of [D/4 x 64]
//     wada [L*6D/NT_ADA][D/64]   blocks of [NT_ADA x 64]   (all layers stacked)
//     we2  [eh/128][2]           blocks of [D x 64]        (Embedder Linear 2)
//   activations (per plan / model-cost call)
//     act_a [ceil(NC*T/128)][D/64] blocks of [128 x 64]  SiLU(action embedding)
//     mod   [NC*T][L*6D] bf16   AdaLN shift/scale/gate per (candidate, time, layer)
//     x     [tiles][128][D] fp32  residual stream of one window
//     attn  [tiles][inner/64] blocks of [128 x 64]  attention output
//     h     [tiles][mlp/64]   blocks of [128 x 64]  GELU(FFN hidden)
//     pred  [NC][T-H+1][D] fp32  predicted embeddings appended to the history
//
// A window tile holds floor(128 / w) whole candidates (w = window tokens),
// row = local_candidate * w + position, so attention never crosses tiles.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdlib>
#include <utility>
#include <vector>

namespace lewm {

constexpr int kDimHead = 64;
constexpr int kTileM = 128;

struct DevWeights {
  const __nv_bfloat16* qkv;
  const __nv_bfloat16* wout;
  const __nv_bfloat16* wout_wide;  // out-proj [L][inner/64][D x 64] (all outputs per K block; D 192 only)
  const __nv_bfloat16* w1;
  const __nv_bfloat16* w2;
  const __nv_bfloat16* wada;
  const __nv_bfloat16* we2;
  const float* pos;        // [frames][D]
  const float* ada_b;      // [L][6D]
  const float* attn_ln_w;  // [L][D]
  const float* attn_ln_b;  // [L][D]
  const float* out_b;      // [L][D]
  const float* ffn_ln_w;   // [L][D]
  const float* ffn_ln_b;   // [L][D]
  const float* b1;         // [L][mlp]
  const float* b2;         // [L][D]
  const float* fin_w;      // [D]
  const float* fin_b;      // [D]
  const float* conv_w;     // [A'][A]
  const float* conv_b;     // [A']
  const float* e1_w;       // [eh][A']
  const float* e1_b;       // [eh]
  const float* e2_b;       // [D]
  // FC1 / FC2 re-blocked for the fused call kernel (width 192, MLP 768): [L][4 quarters][3]
  // blocks of [192 x 64]: FC1 rows = the quarter's 192 hidden units over K block kb of D;
  // FC2 rows = the 192 outputs over hidden columns [192 q + 64 kb, +64).
  const __nv_bfloat16* w1s;
  const __nv_bfloat16* w2s;
};

struct ModelDims {
  int D, L, heads, inner, mlp, A, As, eh, frames;
  int pp_hidden, pp_norm;  // pred_proj MLP head hidden width (0: Identity) and norm kind
};

// One predictor call of the rollout over every candidate.
// Tile groups per head of the persistent QKV + attention kernel (16 heads x 9 = 144 CTAs).
constexpr int kQkvGroups = 9;

struct CallGeom {
  int n_cand;   // candidates in flight (envs * samples)
  int S;        // samples per env (candidate -> env mapping)
  int T, H;     // horizon, history length
  int w;        // window tokens
  int start;    // history index of window position 0
  int cpt;      // candidates per tile
  int n_tiles;  // window tiles
  int rows8;    // rows of a tile that operand copies move: cpt * w rounded up to 8 (<= 128)
  int ln_prebuilt;  // 1: QKV / FC1 operands are built by k_ln_operand and bulk-copied
  int ffn_fused;    // 1: FC1 + GELU + FC2 run as one kernel per (tile, hidden quarter)
  int fc2_parts;    // K parts of FC2's partial sums (4 hidden quarters at D 192 / MLP 768, else 2),
                    // the same on both FFN paths so a row's result does not depend on the batch
  int outproj_wide; // 1: out-proj CTAs compute all D columns (N = D) of one K half
  int qkv_persistent;  // 1: QKV + attention by head-resident CTAs looping over prebuilt tiles
  int call;     // prediction slot written by this call
  int last;     // 1: final call, write costs
  // Window of the next call (k_final prepares its layer-0 inputs); unused when last.
  int next_w, next_start, next_cpt;
  // Rows of each candidate this call processes: the whole window (rpc = w, pos0 = 0) or, on
  // a growing-window call whose earlier positions the calls before already ran through the
  // layers (their inputs and outputs do not change while the window only grows: causal
  // attention, fixed positions), just the new last position (rpc = 1, pos0 = w - 1), whose
  // attention reads the earlier positions' keys and values from the cache (kv_read).
  int rpc, pos0;
  int kv_read;   // 1: keys / values of positions < pos0 come from RolloutBufs::kvc
  int kv_write;  // 1: this call's rows store their keys / values there (the next call reads them)
  int next_rpc, next_pos0;
};

struct RolloutBufs {
  const float* emb;   // (B,H,D) or (NC,H,D)
  int emb_per_cand;
  const float* goal;  // (B,D) or (NC,D)
  int goal_per_cand;
  const float* cand;  // (NC,T,A)
  __nv_bfloat16* act_a;
  __nv_bfloat16* mod;
  float* x;        // residual stream of this call's window before each layer, [tiles][128][D]
  float* xn;       // residual stream of the next call's window (k_final writes it)
  float* xs;       // residual after the attention half of a layer, [tiles][128][D]
  float* part_a;   // out-proj partial sums, [2][tiles][128][D]
  float* part_b;   // FC2 partial sums, [2 or 4][tiles][128][D]
  size_t part_stride;  // floats between consecutive partials of part_a / part_b
  __nv_bfloat16* a_op; // GEMM operand built by k_ln_operand, [tiles][D/64][128x64] pre-swizzled
  __nv_bfloat16* attn;
  __nv_bfloat16* h;
  float* pred;
  float* costs;
  // Keys and values of growing-window positions per layer, candidate, position, head:
  // [L][n_cand][kvc_pos][heads][k 64 | v 64] fp32 (the row format of the attention's
  // shared k/v scratch). Null with kvc_pos 0 when no call of the rollout reads it.
  float* kvc;
  int kvc_pos;
  // pred_proj head (null: Identity): k_final writes the final-LayerNorm rows of the calls'
  // new predictions into pp_in ([n_cand / 128][D / 64][128 x 64] bf16 operand blocks, row =
  // candidate); after the head, k_final_post reads the head's fp32 output rows pp_out [n_cand][D].
  __nv_bfloat16* pp_in;
  const float* pp_out;
};

// Optional per-launch event profiler (host side). When `on`, every launch site
// records an event pair and the algorithmic FLOPs of that launch under a kernel
// class; lewm_profile_plan sums them after a synchronize.
enum KernelClass { KC_EMBED = 0, KC_ADALN, KC_QKV_ATTN, KC_OUT, KC_FC1, KC_FC2, KC_FINAL, KC_SAMPLE, KC_REFIT,
                   KC_PREP0, KC_FFN, KC_LN_OP, KC_TILE_CALL, KC_F32_COST, KC_COUNT };
struct Prof {
  bool on = false;
  struct Rec {
    int cls;
    double flops;
    cudaEvent_t a, b;
  };
  std::vector<Rec> recs;
  std::vector<cudaEvent_t> pool;
  size_t used = 0;
  cudaEvent_t take() {
    if (used == pool.size()) {
      cudaEvent_t e;
      cudaEventCreate(&e);
      pool.push_back(e);
    }
    return pool[used++];
  }
  void begin(cudaStream_t s) {
    if (!on) return;
    cur_a = take();
    cudaEventRecord(cur_a, s);
  }
  void end(int cls, double flops, cudaStream_t s) {
    if (!on) return;
    cudaEvent_t b = take();
    cudaEventRecord(b, s);
    recs.push_back(Rec{cls, flops, cur_a, b});
  }
  void reset() {
    recs.clear();
    used = 0;
  }
  ~Prof() {
    for (auto e : pool) cudaEventDestroy(e);
  }
  cudaEvent_t cur_a = nullptr;
};

// Launch with programmatic stream serialization (the kernel calls griddep_wait()
// before touching its predecessor's output). LEWM_NO_PDL=1 turns it off.
// Per-thread switch used while the event profiler is on: events recorded between
// programmatically dependent launches would break their ordering, so profiled
// plans launch every kernel with plain stream ordering.
inline bool& pdl_suppressed() {
  static thread_local bool off = false;
  return off;
}
inline bool pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("LEWM_NO_PDL");
    return !(v && v[0] == '1');
  }();
  return on && !pdl_suppressed();
}
// Launch with programmatic stream serialization (unless disabled or profiling).
template <typename... KArgs, typename... Args>
cudaError_t launch_k(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  int n = 0;
  if (pdl_enabled()) {
    at[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = at;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// Launchers (rollout_kernels.cu). All asynchronous on `st`; `prof` may be null.
cudaError_t launch_embed(const ModelDims& md, const DevWeights& w, const float* cand, int rows, __nv_bfloat16* eh,
                         __nv_bfloat16* act_a, uint32_t* status, cudaStream_t st, Prof* prof);
cudaError_t launch_adaln(const ModelDims& md, const DevWeights& w, int rows, const __nv_bfloat16* act_a,
                         __nv_bfloat16* mod, uint32_t* status, cudaStream_t st, Prof* prof);
cudaError_t launch_call(const ModelDims& md, const DevWeights& w, const CallGeom& g, const RolloutBufs& b,
                        uint32_t* status, cudaStream_t st, Prof* prof);
// Layer-0 residual rows (history + position) of the first predictor call of a rollout.
cudaError_t launch_prep0(const ModelDims& md, const DevWeights& w, const CallGeom& g, const RolloutBufs& b,
                         cudaStream_t st, Prof* prof);
// With a pred_proj head: the second half of a call's final step once the head has written
// b.pp_out (cost on the last call, else the prediction's history slot and the next call's
// layer-0 rows).
cudaError_t launch_final_post(const ModelDims& md, const DevWeights& w, const CallGeom& g, const RolloutBufs& b,
                              cudaStream_t st, Prof* prof);

// iCEM kernels (icem_kernels.cu).
struct SampleParams {
  int B, S, T, A;
  int noise_kind;     // 0 white, 1 raw-time colored, 2 block colored
  int raw_block;      // action_block for raw-time coloring
  int ncol;           // colored time length (T*block or T)
  const float* W;     // [ncol][ncol] coloring matrix (fp32)
  const float* noise; // injected noise (B,S,T,A) or null
  const uint32_t* rng;  // device [seed, plan index] (Philox key), read at run time
  uint32_t iter;
  const float* mean;  // (B,T,A)
  const float* stdv;  // (B,T,A)
  const float* elites;  // (B,elite_stride,T,A) previous sorted elites
  int elite_stride;
  int n_inject;       // slots 1..n_inject take elites 0..n_inject-1
  const float* low;   // (A) or null
  const float* high;
  float* cand;        // (B,S,T,A)
};
cudaError_t launch_sample(const SampleParams& p, cudaStream_t st);
cudaError_t launch_set_rng(uint32_t* rng, uint32_t seed, uint32_t plan, cudaStream_t st);
// One wait on an mbarrier that nothing arrives on: expires after the status block's limit.
cudaError_t launch_wait_selftest(uint32_t* status, cudaStream_t st);

// One predictor call, all layers, for tiles of 40 candidates x 3 window rows
// (tile_call.cu). Width 192, 16 heads, MLP 768, a full window of 3 from the first call.
struct TileCallParams {
  int n_cand;         // candidates (envs x samples)
  int S;              // samples per env
  int T, H;           // horizon, history rows
  int start;          // history index of window position 0 (H + call - 3)
  int call;           // prediction slot this call writes
  int last;           // 1: write costs instead of the prediction
  int npred;          // prediction slots per candidate (T - H + 1)
  int layers;
  int goal_per_cand;
  const float* emb;   // (B, H, D)
  const float* goal;  // (B, D) or (n_cand, D)
  const __nv_bfloat16* mod;  // AdaLN modulation rows [n_cand * T][L * 6D]
  float* pred;        // [n_cand][npred][D]
  float* costs;       // [n_cand]
  uint32_t* status;
};
cudaError_t launch_tile_call(const DevWeights& w, const TileCallParams& p, cudaStream_t st);
int tile_call_candidates_per_tile();
void tile_call_describe(char* buf, size_t n);  // launch resources, for error messages

// MLP head at input / output width 192 (reference lewm/module.py:217-240): Linear(192 -> P),
// LayerNorm / BatchNorm1d (eval) / none, GELU, Linear(P -> 192); the predictor's pred_proj.
// Runs on the encoder's projector kernels (encoder.cu).
struct MlpHead {
  int P = 0;     // hidden width, a multiple of 256
  int norm = 0;  // 0 none, 1 LayerNorm, 2 BatchNorm1d (folded into scale / shift)
  float eps = 1e-5f;
  void* d_w = nullptr;
  const __nv_bfloat16* w1 = nullptr;  // [P / 256][3][256 x 64] blocks
  const __nv_bfloat16* w2 = nullptr;  // [P / 64][192 x 64] blocks
  const float* scale = nullptr;  // [P] BatchNorm scale (1 otherwise)
  const float* shift = nullptr;  // [P] first Linear's bias, BatchNorm-folded
  const float* ln_g = nullptr;   // [P] LayerNorm affine (norm == 1)
  const float* ln_b = nullptr;
  const float* b2 = nullptr;     // [192]
};
// Host weights in state-dict order: net.0.weight [P x 192], net.0.bias, norm parameters
// (LayerNorm: weight, bias; BatchNorm1d: weight, bias, running_mean, running_var),
// net.3.weight [192 x P], net.3.bias.
size_t mlp_head_floats(int P, int norm);
cudaError_t mlp_head_create(MlpHead* h, const float* w, int P, int norm, float eps);
void mlp_head_destroy(MlpHead* h);
// out[n_rows][192] (fp32) = head(rows of in_op), in_op: [ceil(n_rows / 128)][3][128 x 64]
// bf16 operand blocks; hid_op: [tiles][P / 64][128 x 64]; hid32: [tiles * 128][P] (LayerNorm only).
cudaError_t mlp_head_run(const MlpHead& h, const __nv_bfloat16* in_op, int n_rows, __nv_bfloat16* hid_op,
                         float* hid32, float* out, uint32_t* status, cudaStream_t st);

// fp32 model cost (fp32_path.cu): the predictor's float32 weights as given (row-major
// state-dict tensors) and the float32 activations of one evaluation.
struct F32Layer {
  const float *ada_w, *ada_b;          // [6D][D], [6D]
  const float *attn_ln_w, *attn_ln_b;  // [D]
  const float *qkv_w;                  // [3 inner][D]
  const float *out_w, *out_b;          // [D][inner], [D]
  const float *ffn_ln_w, *ffn_ln_b;    // [D]
  const float *w1, *b1;                // [mlp][D], [mlp]
  const float *w2, *b2;                // [D][mlp], [D]
};
struct F32Weights {
  const float* pos = nullptr;  // [frames][D]
  std::vector<F32Layer> layers;
  const float *fin_w = nullptr, *fin_b = nullptr;
  const float *conv_w = nullptr, *conv_b = nullptr;  // [A'][A], [A']
  const float *e1_w = nullptr, *e1_b = nullptr;      // [eh][A'], [eh]
  const float *e2_w = nullptr, *e2_b = nullptr;      // [D][eh], [D]
  // pred_proj MLP head: first Linear (bias only with LayerNorm), LayerNorm affine, or the
  // per-column scale / shift of BatchNorm (eval) with the Linear's bias folded in (scale 1,
  // shift = bias without a norm), second Linear.
  const float *pp_w1 = nullptr, *pp_b1 = nullptr, *pp_ln_g = nullptr, *pp_ln_b = nullptr;
  const float *pp_scale = nullptr, *pp_shift = nullptr, *pp_w2 = nullptr, *pp_b2 = nullptr;
  const float* ada_stack = nullptr;    // [L * 6D][D]: every layer's adaLN Linear weight, stacked
  const float* ada_b_stack = nullptr;  // [L * 6D]: their biases
};
struct F32Work {
  float *act, *eh, *sact;  // [NC*T] x A' / eh / D: Embedder activations, sact = SiLU(action embedding)
  float* mod;              // [NC*T][L*6D] AdaLN modulation
  float *x, *a;            // [NC*w][D] residual stream, LayerNorm-modulated operand
  float *qkv, *att, *hid;  // [NC*w] x 3 inner / inner / mlp
  float* y;                // [NC][D] final-LayerNorm (and head) output of a call
  float* pred;             // [NC][T-H+1][D] predictions appended to the history
  float* pph;              // [NC][P] pred_proj hidden rows
  int* row_tok;            // [NC*w] modulation row (candidate * T + history index) of each row
  float* part;             // [4][NC*w][D] split-K partial sums of the gated-residual GEMMs
  float* kv;               // [L][NC][HS-1][2 inner] keys / values of growing-window positions
};
// Floats of F32Work for n_cand candidates, horizon T, window <= frames (pointers into one block).
size_t f32_work_floats(const ModelDims& m, size_t n_cand, size_t T);
F32Work f32_work_carve(const ModelDims& m, size_t n_cand, size_t T, float* base);
// What the reverse pass of the fp32 model cost reads, recorded by the forward: per predictor
// call (rows = candidates x window, row = candidate * w + position), per layer.
struct F32TapeCall {
  int rows = 0, w = 0, start = 0;
  int* row_tok = nullptr;  // [rows] modulation row of each row
  float* x_in = nullptr;   // [L][rows][D] residual entering the layer
  float* qkv = nullptr;    // [L][rows][3 inner]
  float* o = nullptr;      // [L][rows][D] out-projection output (with bias), before its gate
  float* x_mid = nullptr;  // [L][rows][D] residual after the attention half
  float* f1 = nullptr;     // [L][rows][mlp] FC1 output (with bias), before GELU
  float* f2 = nullptr;     // [L][rows][D] FC2 output (with bias), before its gate
  float* x_out = nullptr;  // [rows][D] residual after the last layer
};
struct F32Tape {
  float* h1 = nullptr;  // [NC*T][eh] Embedder hidden layer before SiLU
  float* e = nullptr;   // [NC*T][D] action embedding before SiLU
  float* y = nullptr;   // [NC][D] final-LayerNorm output of the last call
  std::vector<F32TapeCall> calls;
};
// Gradient buffers of the reverse pass (d = d loss / d ...).
struct F32GradWork {
  float *dX, *dF, *dF1, *dA, *dAtt, *dQKV;  // [NC*w] x D / D / mlp / D / inner / 3 inner
  float *dY, *dpred;                        // [NC][D], [NC][T-H+1][D]
  float *dmod, *de, *dh1, *da1;             // [NC*T] x L*6D / D / eh / A'
  float* part;                              // split-reduction partial sums of the dY . W GEMMs
  size_t part_floats;
  // staged inputs and outputs of a graph-replayed pass: emb, goal, candidates, cost weights,
  // costs, gradient
  float *in_emb, *in_goal, *in_cand, *in_w, *out_cost, *out_grad;
};
// Floats of the tape + gradient buffers of one evaluation; carve them from `base`.
size_t f32_grad_floats(const ModelDims& m, int NC, int T, int H, int HS);
void f32_grad_carve(const ModelDims& m, int NC, int T, int H, int HS, float* base, F32Tape* tape, F32GradWork* gw);
// `tape` null: plain forward. Else the forward also records the tape (pred_proj Identity).
cudaError_t run_model_cost_fp32(const ModelDims& m, const F32Weights& w, const F32Work& ws, const float* emb,
                                int emb_pc, int H, const float* goal, int goal_pc, const float* cand, int B, int S,
                                int T, int HS, float* costs, cudaStream_t st, const F32Tape* tape = nullptr);
// costs and grad (B,S,T,A) = cost_weight[c] * d cost[c] / d cand[c] (weights null: 1), float32 forward
// and reverse over the recorded tape; pred_proj Identity.
cudaError_t run_model_cost_grad_fp32(const ModelDims& m, const F32Weights& w, const F32Work& ws, const F32Tape& tape,
                                     const F32GradWork& gw, const float* emb, int emb_pc, int H, const float* goal,
                                     int goal_pc, const float* cand, int B, int S, int T, int HS,
                                     const float* cost_weights, float* costs, float* grad, cudaStream_t st);

// Sets the thread's error text that lewm_last_error(NULL) returns (context-free calls).
void set_noctx_error(const char* msg);

struct RefitParams {
  int B, S, T, A, k, R;
  const float* costs;   // (B,S)
  const float* cand;    // (B,S,T,A)
  float* mean;          // (B,T,A) in/out
  float* stdv;          // (B,T,A) in/out
  float alpha;          // momentum
  float* elites;        // (B,R,T,A) out: R best elites, ascending cost
  float* best;          // (B,T,A) out: best elite
  float* final_cost;    // (B) out: mean of the k smallest costs
  int32_t* topk_idx;    // (B,k) out or null
  float* topk_val;      // (B,k) out or null
  uint32_t* nan_status; // status block: LEWM_DEV_NAN is set when a final cost is NaN (or null: no check)
};
cudaError_t launch_refit(const RefitParams& p, cudaStream_t st);

}  // namespace lewm
