// C ABI of the LeWM iCEM hot path: argument checks, weight packing, workspace
// management and the launch sequence of one model-cost call / one plan.
#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/lewm_b200.h"
#include "lewm_common.cuh"
#include "lewm_internal.h"

using namespace lewm;

static_assert(KC_COUNT == LEWM_KERNEL_CLASSES, "kernel classes of lewm_profile_plan");

namespace {

thread_local std::string g_create_error;

size_t round_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

uint16_t f2bf(float f) {  // round to nearest even
  uint32_t u;
  std::memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return 0x7fc0;
  u += 0x7fffu + ((u >> 16) & 1u);
  return static_cast<uint16_t>(u >> 16);
}

uint32_t sw128(uint32_t r, uint32_t k) { return r * 128u + ((((k >> 3) ^ (r & 7u)) << 4) | ((k & 7u) << 1)); }

struct Workspace {
  void* base = nullptr;
  size_t bytes = 0;
  float* cand = nullptr;
  __nv_bfloat16* act_a = nullptr;
  __nv_bfloat16* eh = nullptr;   // embedder hidden layer, pre-swizzled [row tile][eh/64] blocks
  __nv_bfloat16* mod = nullptr;
  float* x = nullptr;    // two residual buffers: predictor calls alternate between them
  float* x2 = nullptr;
  float* xs = nullptr;   // residual after the attention half of a layer
  float* part_a = nullptr;  // out-proj partial sums (two K halves)
  float* part_b = nullptr;  // FC2 partial sums (CallGeom::fc2_parts K parts: 2 halves or 4 hidden quarters)
  size_t part_stride = 0;
  __nv_bfloat16* a_op = nullptr;  // QKV / FC1 operand built once per tile
  __nv_bfloat16* attn = nullptr;
  __nv_bfloat16* h = nullptr;
  float* pred = nullptr;
  float* costs = nullptr;
  float* kvc = nullptr;      // growing-window key / value cache (RolloutBufs::kvc)
  // plan state
  float* mean = nullptr;
  float* stdv = nullptr;
  float* elites = nullptr;
  float* best = nullptr;
  float* fcost = nullptr;
  float* W = nullptr;
  uint32_t* rng = nullptr;   // [seed, plan index]
  __nv_bfloat16* pp_in = nullptr;   // pred_proj head: operand, hidden operand, LayerNorm rows, output rows
  __nv_bfloat16* pp_hid = nullptr;
  float* pp_hid32 = nullptr;
  float* pp_out = nullptr;
  F32Work f32{};             // fp32 model-cost activations (carved when the context computes in fp32)
  float* emb_in = nullptr;   // staged plan inputs (graph path)
  float* goal_in = nullptr;
  float* lohi = nullptr;     // action low | high
};

struct WsReq {
  size_t n_cand, T, A, D, L, tiles, heads, mlp, npred, B, R, ncol, kvpos;
  // fp32 model-cost activations for this many candidates and horizon (0: none), sized by the
  // float32 requests alone so that bf16 calls of many candidates do not size them
  size_t f32_nc = 0, f32_T = 0;
  bool operator<=(const WsReq& o) const {
    return n_cand <= o.n_cand && T <= o.T && tiles <= o.tiles && npred <= o.npred && B <= o.B && R <= o.R &&
           ncol <= o.ncol && kvpos <= o.kvpos && f32_nc <= o.f32_nc && f32_T <= o.f32_T;
  }
};

// Growing-window key / value cache (CallGeom::kv_read); LEWM_KV_CACHE=0 recomputes every
// window position in every call instead.
bool kv_cache_on() {
  static const bool on = [] {
    const char* v = std::getenv("LEWM_KV_CACHE");
    return v ? std::atoi(v) != 0 : true;
  }();
  return on;
}

// Positions per candidate the cache holds for a rollout with history H and window HS: the
// calls before the window first slides write positions 0 .. HS - 2; none when the first
// call's window is already full.
int kv_positions(int H, int HS) { return (kv_cache_on() && H + 1 <= HS) ? HS - 1 : 0; }

}  // namespace

struct lewm_ctx {
  int device = 0;
  lewm_model_desc desc{};
  ModelDims md{};
  std::string err;
  void* d_weights = nullptr;
  DevWeights w{};
  int autocast = 1;           // model-cost arithmetic: 1 bf16 tensor cores (default), 0 float32
  void* d_w32 = nullptr;      // float32 weights of the fp32 model cost
  F32Weights w32;
  float* d_grad = nullptr;    // tape + gradient buffers of lewm_model_cost_grad
  size_t grad_floats = 0;
  std::map<std::vector<int>, cudaGraphExec_t> grad_graphs;  // one executable graph per gradient shape
  MlpHead pp{};  // pred_proj MLP head (P == 0: Identity)
  uint32_t* d_status = nullptr;
  Workspace ws;
  WsReq cap{};
  bool have_ws = false;
  Prof prof;                  // per-launch event profiler (lewm_profile_plan)
  cudaStream_t cap_stream = nullptr;  // plan graphs are captured and replayed here
  cudaEvent_t ev_in = nullptr, ev_out = nullptr;
  std::map<std::vector<double>, cudaGraphExec_t> graphs;  // one executable graph per plan shape
  int tile_target = 1;        // row tiles a small predictor call is spread over
  int tile_call_min = -1;     // fused call kernel from this many candidates (-1: 8000, 0: never)
  int sm_count = 148;         // streaming multiprocessors of the device
  std::vector<float> W_host;  // last uploaded coloring matrix
  int W_n = -1;
  float W_beta = -1.f;
};

namespace {

lewm_status fail(lewm_ctx* c, lewm_status s, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  if (c)
    c->err = buf;
  else
    g_create_error = buf;
  return s;
}

#define LEWM_CK(ctx, call)                                                                               \
  do {                                                                                                   \
    cudaError_t e_ = (call);                                                                             \
    if (e_ != cudaSuccess)                                                                               \
      return fail(ctx, e_ == cudaErrorMemoryAllocation ? LEWM_OUT_OF_MEMORY : LEWM_CUDA_ERROR, "%s: %s", \
                  #call, cudaGetErrorString(e_));                                                        \
  } while (0)

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

lewm_status check_desc(const lewm_model_desc* d, ModelDims* md) {
  if (!d) return fail(nullptr, LEWM_INVALID_ARG, "desc is NULL");
  if (d->dim <= 0 || d->depth <= 0 || d->heads <= 0 || d->dim_head <= 0 || d->mlp_dim <= 0 || d->action_dim <= 0 ||
      d->smoothed_dim <= 0 || d->embed_hidden <= 0 || d->num_frames <= 0 || d->pred_proj_hidden < 0)
    return fail(nullptr, LEWM_INVALID_ARG, "model dimensions must be positive");
  if (d->dim != 192 && d->dim != 384)
    return fail(nullptr, LEWM_UNSUPPORTED_SHAPE, "dim=%d unsupported (built for 192, 384)", d->dim);
  if (d->dim_head != 64) return fail(nullptr, LEWM_UNSUPPORTED_SHAPE, "dim_head=%d unsupported (64)", d->dim_head);
  if (d->heads > 16) return fail(nullptr, LEWM_UNSUPPORTED_SHAPE, "heads=%d > 16", d->heads);
  if (d->mlp_dim % 128 || d->embed_hidden % 128)
    return fail(nullptr, LEWM_UNSUPPORTED_SHAPE, "mlp_dim and embed_hidden must be multiples of 128");
  if (d->action_dim > 16 || d->smoothed_dim > 16)
    return fail(nullptr, LEWM_UNSUPPORTED_SHAPE, "action_dim/smoothed_dim must be <= 16");
  if (d->num_frames > 8) return fail(nullptr, LEWM_UNSUPPORTED_SHAPE, "num_frames must be <= 8");
  if (d->pred_proj_hidden != 0) {  // MLP head: runs on the 192-wide projector kernels
    if (d->dim != 192 || d->pred_proj_hidden % 256 != 0)
      return fail(nullptr, LEWM_UNSUPPORTED_SHAPE,
                  "pred_proj MLP head needs dim 192 and a hidden width that is a multiple of 256 (got %d, %d)",
                  d->dim, d->pred_proj_hidden);
    if (d->pred_proj_norm < 0 || d->pred_proj_norm > 2)
      return fail(nullptr, LEWM_INVALID_ARG, "pred_proj_norm must be 0, 1 or 2, got %d", d->pred_proj_norm);
  }
  md->D = d->dim;
  md->L = d->depth;
  md->heads = d->heads;
  md->inner = d->heads * 64;
  md->mlp = d->mlp_dim;
  md->A = d->action_dim;
  md->As = d->smoothed_dim;
  md->eh = d->embed_hidden;
  md->frames = d->num_frames;
  md->pp_hidden = d->pred_proj_hidden;
  md->pp_norm = d->pred_proj_norm;
  return LEWM_OK;
}

size_t weight_count(const ModelDims& m) {
  const size_t D = m.D;
  size_t n = (size_t)m.frames * D;
  const size_t per_layer = 6 * D * D + 6 * D + 2 * D + 3 * (size_t)m.inner * D + D * m.inner + D + 2 * D +
                           (size_t)m.mlp * D + m.mlp + D * m.mlp + D;
  n += per_layer * m.L;
  n += 2 * D;
  n += (size_t)m.As * m.A + m.As + (size_t)m.eh * m.As + m.eh + D * m.eh + D;
  if (m.pp_hidden) n += mlp_head_floats(m.pp_hidden, m.pp_norm);
  return n;
}

// Pack rows `rowmap(r)` (r < nrows) and columns [64*kb, 64*kb+64) of W (rows x K) into a
// swizzled [nrows x 64] bf16 block.
template <class RowMap>
void pack_block(uint8_t* dst, const float* W, int K, int nrows, int kb, RowMap rowmap) {
  for (int r = 0; r < nrows; ++r) {
    const float* src = W + (size_t)rowmap(r) * K;
    for (int k = 0; k < 64; ++k) {
      const int col = kb * 64 + k;
      const uint16_t v = col < K ? f2bf(src[col]) : 0;
      std::memcpy(dst + sw128(r, k), &v, 2);
    }
  }
}

lewm_status pack_weights(lewm_ctx* c, const float* wts, size_t n) {
  const ModelDims& m = c->md;
  const int D = m.D, L = m.L, KB = D / 64, NT = D / 4, NKI = m.inner / 64, NKM = m.mlp / 64;
  const int NT_ADA = (D == 192) ? 192 : 128;
  // Walk the canonical order.
  const float* p = wts;
  auto take = [&](size_t k) {
    const float* q = p;
    p += k;
    return q;
  };
  const float* pos = take((size_t)m.frames * D);
  std::vector<const float*> ada_w(L), ada_b(L), aln_w(L), aln_b(L), qkv_w(L), out_w(L), out_b(L), fln_w(L),
      fln_b(L), w1(L), b1(L), w2(L), b2(L);
  for (int l = 0; l < L; ++l) {
    ada_w[l] = take((size_t)6 * D * D);
    ada_b[l] = take(6 * D);
    aln_w[l] = take(D);
    aln_b[l] = take(D);
    qkv_w[l] = take((size_t)3 * m.inner * D);
    out_w[l] = take((size_t)D * m.inner);
    out_b[l] = take(D);
    fln_w[l] = take(D);
    fln_b[l] = take(D);
    w1[l] = take((size_t)m.mlp * D);
    b1[l] = take(m.mlp);
    w2[l] = take((size_t)D * m.mlp);
    b2[l] = take(D);
  }
  const float* fin_w = take(D);
  const float* fin_b = take(D);
  const float* conv_w = take((size_t)m.As * m.A);
  const float* conv_b = take(m.As);
  const float* e1_w = take((size_t)m.eh * m.As);
  const float* e1_b = take(m.eh);
  const float* e2_w = take((size_t)D * m.eh);
  const float* e2_b = take(D);
  const float* pp_w = m.pp_hidden ? take(mlp_head_floats(m.pp_hidden, m.pp_norm)) : nullptr;
  if ((size_t)(p - wts) != n) return fail(c, LEWM_INVALID_ARG, "weight walk mismatch");
  if (pp_w) LEWM_CK(c, mlp_head_create(&c->pp, pp_w, m.pp_hidden, m.pp_norm, 1e-5f));

  std::vector<uint8_t> buf;
  auto alloc = [&](size_t bytes) {
    const size_t off = round_up(buf.size(), 1024);
    buf.resize(off + bytes);
    return off;
  };
  const size_t blkA = 128 * 128;  // [128 x 64] block bytes
  const size_t o_qkv = alloc((size_t)L * m.heads * KB * 192 * 128);
  const size_t o_wout = alloc((size_t)L * 4 * NKI * NT * 128);
  const size_t o_wout_w = D == 192 ? alloc((size_t)L * NKI * D * 128) : 0;
  const size_t o_w1 = alloc((size_t)L * (m.mlp / 128) * KB * blkA);
  const size_t o_w2 = alloc((size_t)L * 4 * NKM * NT * 128);
  const bool tile_w = D == 192 && m.mlp == 768;  // FC1 / FC2 blocks of the fused call kernel
  const size_t o_w1s = tile_w ? alloc((size_t)L * 12 * 192 * 128) : 0;
  const size_t o_w2s = tile_w ? alloc((size_t)L * 12 * 192 * 128) : 0;
  const size_t n_ada_tiles = (size_t)L * 6 * D / NT_ADA;
  const size_t o_wada = alloc(n_ada_tiles * KB * NT_ADA * 128);
  const size_t o_we2 = alloc((size_t)(m.eh / 128) * 2 * D * 128);
  auto fvec = [&](const std::vector<const float*>& parts, size_t each) {
    const size_t off = alloc(parts.size() * each * 4);
    for (size_t i = 0; i < parts.size(); ++i) std::memcpy(buf.data() + off + i * each * 4, parts[i], each * 4);
    return off;
  };
  const size_t o_pos = fvec({pos}, (size_t)m.frames * D);
  const size_t o_adab = fvec(ada_b, 6 * D);
  const size_t o_alnw = fvec(aln_w, D), o_alnb = fvec(aln_b, D);
  const size_t o_outb = fvec(out_b, D);
  const size_t o_flnw = fvec(fln_w, D), o_flnb = fvec(fln_b, D);
  const size_t o_b1 = fvec(b1, m.mlp), o_b2 = fvec(b2, D);
  const size_t o_finw = fvec({fin_w}, D), o_finb = fvec({fin_b}, D);
  const size_t o_convw = fvec({conv_w}, (size_t)m.As * m.A), o_convb = fvec({conv_b}, m.As);
  const size_t o_e1w = fvec({e1_w}, (size_t)m.eh * m.As), o_e1b = fvec({e1_b}, m.eh), o_e2b = fvec({e2_b}, D);

  for (int l = 0; l < L; ++l) {
    for (int h = 0; h < m.heads; ++h)
      for (int kb = 0; kb < KB; ++kb) {
        uint8_t* dst = buf.data() + o_qkv + ((size_t)(l * m.heads + h) * KB + kb) * 192 * 128;
        pack_block(dst, qkv_w[l], D, 192, kb, [&](int r) { return (r / 64) * m.inner + h * 64 + (r % 64); });
      }
    for (int nt = 0; nt < 4; ++nt)
      for (int kb = 0; kb < NKI; ++kb) {
        uint8_t* dst = buf.data() + o_wout + ((size_t)(l * 4 + nt) * NKI + kb) * NT * 128;
        pack_block(dst, out_w[l], m.inner, NT, kb, [&](int r) { return nt * NT + r; });
      }
    if (D == 192)
      for (int kb = 0; kb < NKI; ++kb) {
        uint8_t* dst = buf.data() + o_wout_w + ((size_t)l * NKI + kb) * D * 128;
        pack_block(dst, out_w[l], m.inner, D, kb, [&](int r) { return r; });
      }
    for (int nt = 0; nt < m.mlp / 128; ++nt)
      for (int kb = 0; kb < KB; ++kb) {
        uint8_t* dst = buf.data() + o_w1 + ((size_t)(l * (m.mlp / 128) + nt) * KB + kb) * blkA;
        pack_block(dst, w1[l], D, 128, kb, [&](int r) { return nt * 128 + r; });
      }
    for (int nt = 0; nt < 4; ++nt)
      for (int kb = 0; kb < NKM; ++kb) {
        uint8_t* dst = buf.data() + o_w2 + ((size_t)(l * 4 + nt) * NKM + kb) * NT * 128;
        pack_block(dst, w2[l], m.mlp, NT, kb, [&](int r) { return nt * NT + r; });
      }
    if (tile_w)
      for (int q = 0; q < 4; ++q)
        for (int kb = 0; kb < 3; ++kb) {
          const size_t blk = ((size_t)(l * 4 + q) * 3 + kb) * 192 * 128;
          pack_block(buf.data() + o_w1s + blk, w1[l], D, 192, kb, [&](int r) { return 192 * q + r; });
          pack_block(buf.data() + o_w2s + blk, w2[l], m.mlp, 192, 3 * q + kb, [&](int r) { return r; });
        }
  }
  for (size_t t = 0; t < n_ada_tiles; ++t)
    for (int kb = 0; kb < KB; ++kb) {
      uint8_t* dst = buf.data() + o_wada + (t * KB + kb) * NT_ADA * 128;
      for (int r = 0; r < NT_ADA; ++r) {
        const size_t R = t * NT_ADA + r;
        const float* src = ada_w[R / (6 * D)] + (R % (6 * D)) * D;
        for (int k = 0; k < 64; ++k) {
          const uint16_t v = f2bf(src[kb * 64 + k]);
          std::memcpy(dst + sw128(r, k), &v, 2);
        }
      }
    }
  for (int ch = 0; ch < m.eh / 128; ++ch)
    for (int kb = 0; kb < 2; ++kb) {
      uint8_t* dst = buf.data() + o_we2 + ((size_t)ch * 2 + kb) * D * 128;
      for (int r = 0; r < D; ++r)
        for (int k = 0; k < 64; ++k) {
          const uint16_t v = f2bf(e2_w[(size_t)r * m.eh + ch * 128 + kb * 64 + k]);
          std::memcpy(dst + sw128(r, k), &v, 2);
        }
    }

  LEWM_CK(c, cudaMalloc(&c->d_weights, buf.size()));
  LEWM_CK(c, cudaMemcpy(c->d_weights, buf.data(), buf.size(), cudaMemcpyHostToDevice));
  auto* base = static_cast<uint8_t*>(c->d_weights);
  auto bf = [&](size_t o) { return reinterpret_cast<const __nv_bfloat16*>(base + o); };
  auto fl = [&](size_t o) { return reinterpret_cast<const float*>(base + o); };
  c->w = DevWeights{bf(o_qkv), bf(o_wout), D == 192 ? bf(o_wout_w) : nullptr, bf(o_w1), bf(o_w2), bf(o_wada), bf(o_we2), fl(o_pos), fl(o_adab),
                    fl(o_alnw), fl(o_alnb), fl(o_outb), fl(o_flnw), fl(o_flnb), fl(o_b1), fl(o_b2), fl(o_finw),
                    fl(o_finb), fl(o_convw), fl(o_convb), fl(o_e1w), fl(o_e1b), fl(o_e2b),
                    tile_w ? bf(o_w1s) : nullptr, tile_w ? bf(o_w2s) : nullptr};
  return LEWM_OK;
}

// Candidates per row tile and tile count of a predictor call with window w. A tile
// holds whole candidates (at most 128 rows). A call with few candidates is spread
// over up to `target` tiles (one wave of the one-head-per-CTA QKV kernel), so each
// CTA of the streamed-operand GEMMs moves fewer rows; a large call uses full tiles.
// The float32 weights of the fp32 model cost: each tensor of the canonical host array at a
// 16-byte aligned offset (so the GEMMs' 16-byte loads apply), plus [2P] per-column scale /
// shift of a pred_proj head without a LayerNorm (BatchNorm1d in eval folded with the first
// Linear's bias, computed in double; scale 1, shift = bias with no norm).
lewm_status upload_f32_weights(lewm_ctx* c, const float* wts, size_t n) {
  const ModelDims& m = c->md;
  const size_t D = m.D, P = m.pp_hidden;
  std::vector<float> stage;
  size_t src = 0;
  std::vector<std::pair<const float**, size_t>> fix;  // pointer to set, staged offset
  auto place = [&](const float* data, size_t k) {
    const size_t off = round_up(stage.size(), 4);
    stage.resize(off + k);
    std::memcpy(stage.data() + off, data, k * 4);
    return off;
  };
  auto take = [&](const float** dst, size_t k) {
    fix.emplace_back(dst, place(wts + src, k));
    src += k;
  };
  auto skip = [&](size_t k) { src += k; };
  F32Weights& w = c->w32;
  take(&w.pos, (size_t)m.frames * D);
  w.layers.assign(m.L, F32Layer{});
  std::vector<const float*> ada_src(m.L);
  for (int l = 0; l < m.L; ++l) {
    F32Layer& lw = w.layers[l];
    ada_src[l] = wts + src;
    take(&lw.ada_w, 6 * D * D);
    take(&lw.ada_b, 6 * D);
    take(&lw.attn_ln_w, D);
    take(&lw.attn_ln_b, D);
    take(&lw.qkv_w, 3 * (size_t)m.inner * D);
    take(&lw.out_w, D * m.inner);
    take(&lw.out_b, D);
    take(&lw.ffn_ln_w, D);
    take(&lw.ffn_ln_b, D);
    take(&lw.w1, (size_t)m.mlp * D);
    take(&lw.b1, m.mlp);
    take(&lw.w2, D * m.mlp);
    take(&lw.b2, D);
  }
  take(&w.fin_w, D);
  take(&w.fin_b, D);
  take(&w.conv_w, (size_t)m.As * m.A);
  take(&w.conv_b, m.As);
  take(&w.e1_w, (size_t)m.eh * m.As);
  take(&w.e1_b, m.eh);
  take(&w.e2_w, D * m.eh);
  take(&w.e2_b, D);
  if (P) {  // net.0.weight, net.0.bias, norm parameters, net.3.weight, net.3.bias
    take(&w.pp_w1, P * D);
    const float* hb = wts + src;
    take(&w.pp_b1, P);
    if (m.pp_norm == 1) {
      take(&w.pp_ln_g, P);
      take(&w.pp_ln_b, P);
    } else {
      std::vector<float> scale(P, 1.f), shift(hb, hb + P);
      if (m.pp_norm == 2) {  // BatchNorm1d weight, bias, running mean, running var
        const float *g = wts + src, *bb = g + P, *mu = bb + P, *var = mu + P;
        for (size_t j = 0; j < P; ++j) {
          const double sc = (double)g[j] / std::sqrt((double)var[j] + 1e-5);
          scale[j] = (float)sc;
          shift[j] = (float)(((double)hb[j] - mu[j]) * sc + bb[j]);
        }
        skip(4 * P);
      }
      fix.emplace_back(&w.pp_scale, place(scale.data(), P));
      fix.emplace_back(&w.pp_shift, place(shift.data(), P));
    }
    take(&w.pp_w2, D * P);
    take(&w.pp_b2, D);
  }
  if (src != n) return fail(c, LEWM_INVALID_ARG, "fp32 weight walk mismatch");
  {  // every layer's adaLN weight and bias stacked, [L * 6D][D] and [L * 6D]: one GEMM for the
     // modulation of all layers, and one for its reverse pass
    const size_t per = 6 * D * D, off = round_up(stage.size(), 4);
    stage.resize(off + per * m.L);
    for (int l = 0; l < m.L; ++l) std::memcpy(stage.data() + off + per * l, ada_src[l], per * 4);
    fix.emplace_back(&w.ada_stack, off);
    const size_t offb = round_up(stage.size(), 4);
    stage.resize(offb + 6 * D * m.L);
    for (int l = 0; l < m.L; ++l) std::memcpy(stage.data() + offb + 6 * D * l, ada_src[l] + per, 6 * D * 4);
    fix.emplace_back(&w.ada_b_stack, offb);
  }
  LEWM_CK(c, cudaMalloc(&c->d_w32, stage.size() * 4));
  LEWM_CK(c, cudaMemcpy(c->d_w32, stage.data(), stage.size() * 4, cudaMemcpyHostToDevice));
  for (auto& f : fix) *f.first = static_cast<const float*>(c->d_w32) + f.second;
  return LEWM_OK;
}

void tile_geom(int n_cand, int w, int target, int* cpt, int* n_tiles) {
  const int cmax = 128 / w;
  int nt = (n_cand + cmax - 1) / cmax;
  nt = std::max(nt, std::min(n_cand, target));
  const int c = (n_cand + nt - 1) / nt;
  *cpt = c;
  *n_tiles = (n_cand + c - 1) / c;
}

int window_tiles(int n_cand, int w, int target) {
  int cpt, nt;
  tile_geom(n_cand, w, target, &cpt, &nt);
  return nt;
}

void clear_graphs(lewm_ctx* c) {
  for (auto& kv : c->graphs) cudaGraphExecDestroy(kv.second);
  c->graphs.clear();
  for (auto& kv : c->grad_graphs) cudaGraphExecDestroy(kv.second);
  c->grad_graphs.clear();
}

lewm_status ensure_ws(lewm_ctx* c, const WsReq& need_in) {
  WsReq need = need_in;
  if (c->autocast == 0) {  // float32 model costs of this request
    need.f32_nc = std::max(need.f32_nc, need.n_cand);
    need.f32_T = std::max(need.f32_T, need.T);
  }
  if (c->have_ws && need <= c->cap) return LEWM_OK;
  WsReq r = need;
  if (c->have_ws) {  // grow monotonically
    r.n_cand = std::max(r.n_cand, c->cap.n_cand);
    r.T = std::max(r.T, c->cap.T);
    r.tiles = std::max(r.tiles, c->cap.tiles);
    r.npred = std::max(r.npred, c->cap.npred);
    r.B = std::max(r.B, c->cap.B);
    r.R = std::max(r.R, c->cap.R);
    r.ncol = std::max(r.ncol, c->cap.ncol);
    r.kvpos = std::max(r.kvpos, c->cap.kvpos);
    r.f32_nc = std::max(r.f32_nc, c->cap.f32_nc);
    r.f32_T = std::max(r.f32_T, c->cap.f32_T);
    clear_graphs(c);
    cudaFree(c->ws.base);
    c->ws = Workspace{};
    c->have_ws = false;
  }
  const ModelDims& m = c->md;
  const size_t rows_e = r.n_cand * r.T;
  const size_t tiles_e = (rows_e + 127) / 128;
  size_t off = 0;
  auto carve = [&](size_t bytes) {
    const size_t o = off;
    off = round_up(off + std::max<size_t>(bytes, 16), 1024);
    return o;
  };
  const size_t o_cand = carve(r.n_cand * r.T * m.A * 4);
  const size_t o_act = carve(tiles_e * (m.D / 64) * 128 * 64 * 2);
  const size_t o_eh = carve(tiles_e * (m.eh / 64) * 128 * 64 * 2);
  const size_t o_mod = carve(rows_e * (size_t)m.L * 6 * m.D * 2);
  const size_t o_x = carve(r.tiles * 128 * (size_t)m.D * 4);
  const size_t o_x2 = carve(r.tiles * 128 * (size_t)m.D * 4);
  const size_t o_xs = carve(r.tiles * 128 * (size_t)m.D * 4);
  const size_t o_part_a = carve(2 * r.tiles * 128 * (size_t)m.D * 4);
  const size_t o_part_b = carve(4 * r.tiles * 128 * (size_t)m.D * 4);
  const size_t o_aop = carve(r.tiles * 128 * (size_t)m.D * 2);
  const size_t o_attn = carve(r.tiles * (size_t)(m.inner / 64) * 128 * 64 * 2);
  const size_t o_h = carve(r.tiles * (size_t)(m.mlp / 64) * 128 * 64 * 2);
  const size_t o_pred = carve(r.n_cand * r.npred * (size_t)m.D * 4);
  const size_t o_costs = carve(r.n_cand * 4);
  const size_t o_kvc = carve((size_t)m.L * r.n_cand * r.kvpos * m.heads * 128 * 4);
  const size_t ta = r.T * m.A;
  const size_t o_mean = carve(r.B * ta * 4);
  const size_t o_std = carve(r.B * ta * 4);
  const size_t o_el = carve(r.B * std::max<size_t>(r.R, 1) * ta * 4);
  const size_t o_best = carve(r.B * ta * 4);
  const size_t o_fc = carve(r.B * 4);
  const size_t o_W = carve(std::max<size_t>(r.ncol, 1) * std::max<size_t>(r.ncol, 1) * 4);
  const size_t o_rng = carve(16);
  const size_t o_embin = carve(r.B * r.T * (size_t)m.D * 4);
  const size_t o_goalin = carve(r.B * (size_t)m.D * 4);
  const size_t o_lohi = carve(2 * (size_t)m.A * 4);
  const size_t pp_tiles = m.pp_hidden ? (r.n_cand + 127) / 128 : 0;
  const size_t o_ppin = carve(pp_tiles * (m.D / 64) * 128 * 64 * 2);
  const size_t o_pphid = carve(pp_tiles * (size_t)(m.pp_hidden / 64) * 128 * 64 * 2);
  const size_t o_pph32 = carve(m.pp_norm == 1 ? pp_tiles * 128 * (size_t)m.pp_hidden * 4 : 0);
  const size_t o_ppout = carve(m.pp_hidden ? r.n_cand * (size_t)m.D * 4 : 0);
  const size_t o_f32 = carve(r.f32_nc ? f32_work_floats(m, r.f32_nc, r.f32_T) * 4 : 0);
  void* base = nullptr;
  LEWM_CK(c, cudaMalloc(&base, off));
  auto* b = static_cast<uint8_t*>(base);
  Workspace& ws = c->ws;
  ws.base = base;
  ws.bytes = off;
  ws.cand = reinterpret_cast<float*>(b + o_cand);
  ws.act_a = reinterpret_cast<__nv_bfloat16*>(b + o_act);
  ws.eh = reinterpret_cast<__nv_bfloat16*>(b + o_eh);
  ws.mod = reinterpret_cast<__nv_bfloat16*>(b + o_mod);
  ws.x = reinterpret_cast<float*>(b + o_x);
  ws.x2 = reinterpret_cast<float*>(b + o_x2);
  ws.xs = reinterpret_cast<float*>(b + o_xs);
  ws.part_a = reinterpret_cast<float*>(b + o_part_a);
  ws.part_b = reinterpret_cast<float*>(b + o_part_b);
  ws.part_stride = r.tiles * 128 * (size_t)m.D;
  ws.a_op = reinterpret_cast<__nv_bfloat16*>(b + o_aop);
  ws.attn = reinterpret_cast<__nv_bfloat16*>(b + o_attn);
  ws.h = reinterpret_cast<__nv_bfloat16*>(b + o_h);
  ws.pred = reinterpret_cast<float*>(b + o_pred);
  ws.costs = reinterpret_cast<float*>(b + o_costs);
  ws.kvc = reinterpret_cast<float*>(b + o_kvc);
  ws.mean = reinterpret_cast<float*>(b + o_mean);
  ws.stdv = reinterpret_cast<float*>(b + o_std);
  ws.elites = reinterpret_cast<float*>(b + o_el);
  ws.best = reinterpret_cast<float*>(b + o_best);
  ws.fcost = reinterpret_cast<float*>(b + o_fc);
  ws.W = reinterpret_cast<float*>(b + o_W);
  ws.rng = reinterpret_cast<uint32_t*>(b + o_rng);
  ws.emb_in = reinterpret_cast<float*>(b + o_embin);
  ws.goal_in = reinterpret_cast<float*>(b + o_goalin);
  ws.lohi = reinterpret_cast<float*>(b + o_lohi);
  ws.pp_in = reinterpret_cast<__nv_bfloat16*>(b + o_ppin);
  ws.pp_hid = reinterpret_cast<__nv_bfloat16*>(b + o_pphid);
  ws.pp_hid32 = reinterpret_cast<float*>(b + o_pph32);
  ws.pp_out = reinterpret_cast<float*>(b + o_ppout);
  if (r.f32_nc) ws.f32 = f32_work_carve(m, r.f32_nc, r.f32_T, reinterpret_cast<float*>(b + o_f32));
  c->cap = r;
  c->have_ws = true;
  c->W_n = -1;
  return LEWM_OK;
}

// The fused call kernel (tile_call.cu) covers width 192 / 16 heads / MLP 768 / 6 layers
// without a pred_proj head, calls whose window of 3 is full (history index H + k >= 3 at
// call k: every call when H >= 3, the later calls of a history-1 or -2 rollout, whose
// earlier growing-window calls stay on the per-layer kernels), observation embeddings per
// env, and calls of at least LEWM_TILE_CALL_MIN candidates (default 8000, where it
// overtakes the per-layer kernels: measured 641 -> 696 plans/s at 64 envs, 669 -> 844 at 256
// envs; 0 disables it).
bool use_tile_call(const lewm_ctx* c, int NC, int H, int HS, int emb_pc, int call) {
  const int min_cand = c->tile_call_min;
  const ModelDims& m = c->md;
  if (min_cand == 0) return false;
  const int need = min_cand > 0 ? min_cand : 8000;
  return m.D == 192 && m.heads == 16 && m.mlp == 768 && m.pp_hidden == 0 && m.frames >= 3 && HS == 3 &&
         H + call >= 3 && !emb_pc && c->w.w1s != nullptr && NC >= need;
}

// Algorithmic FLOPs of one model-cost evaluation: the GEMMs over the rows each computes
// (Embedder and AdaLN over every token; every predictor call over its whole window; the
// pred_proj head over the new predictions).
double model_cost_flops(const ModelDims& m, int NC, int T, int H, int HS) {
  const double NT = (double)NC * T;
  double f = 2.0 * NT * ((double)m.A * m.As + (double)m.As * m.eh + (double)m.eh * m.D + (double)m.L * 6 * m.D * m.D);
  for (int k = 0; k < T - H + 1; ++k) {
    const int end = H + k, w = end - std::max(0, end - HS);
    f += 2.0 * NC * w * m.L * ((double)m.D * 3 * m.inner + (double)m.inner * m.D + 2.0 * m.D * m.mlp);
    f += 2.0 * NC * m.D * 2.0 * m.pp_hidden;
  }
  return f;
}

// Launch sequence of one model-cost evaluation over n_cand = B*S candidates.
lewm_status run_model_cost(lewm_ctx* c, const float* emb, int emb_pc, int H, const float* goal, int goal_pc,
                           const float* cand, int B, int S, int T, int HS, float* costs, cudaStream_t st) {
  const ModelDims& m = c->md;
  const int NC = B * S;
  const int rows = NC * T;
  if (c->autocast == 0) {  // float32 arithmetic throughout (no autocast): CUDA-core kernels
    c->prof.begin(st);
    LEWM_CK(c, run_model_cost_fp32(m, c->w32, c->ws.f32, emb, emb_pc, H, goal, goal_pc, cand, B, S, T, HS, costs, st));
    c->prof.end(KC_F32_COST, model_cost_flops(m, NC, T, H, HS), st);
    return LEWM_OK;
  }
  LEWM_CK(c, launch_embed(m, c->w, cand, rows, c->ws.eh, c->ws.act_a, c->d_status, st, &c->prof));
  LEWM_CK(c, launch_adaln(m, c->w, rows, c->ws.act_a, c->ws.mod, c->d_status, st, &c->prof));
  RolloutBufs b{emb,        emb_pc,    goal,      goal_pc, cand,      c->ws.act_a, c->ws.mod,
                c->ws.x,    c->ws.x2,  c->ws.xs,  c->ws.part_a, c->ws.part_b, c->ws.part_stride, c->ws.a_op,
                c->ws.attn, c->ws.h,
                c->ws.pred, costs, c->ws.kvc, kv_positions(H, HS),
                m.pp_hidden ? c->ws.pp_in : nullptr, m.pp_hidden ? c->ws.pp_out : nullptr};
  const int n_calls = T - H + 1;
  // Batched regime: one fused kernel per predictor call with a full window (all layers per
  // row tile); it builds its layer-0 rows from the embeddings and the earlier predictions.
  auto tile_call = [&](int k) -> lewm_status {
    TileCallParams tp{};
    tp.n_cand = NC;
    tp.S = S;
    tp.T = T;
    tp.H = H;
    tp.start = H + k - 3;
    tp.call = k;
    tp.last = k == n_calls - 1 ? 1 : 0;
    tp.npred = n_calls;
    tp.layers = m.L;
    tp.goal_per_cand = goal_pc;
    tp.emb = emb;
    tp.goal = goal;
    tp.mod = c->ws.mod;
    tp.pred = c->ws.pred;
    tp.costs = costs;
    tp.status = c->d_status;
    c->prof.begin(st);
    const cudaError_t te = launch_tile_call(c->w, tp, st);
    if (te != cudaSuccess) {
      char info[256];
      tile_call_describe(info, sizeof info);
      return fail(c, LEWM_CUDA_ERROR, "fused call kernel launch: %s (%s)", cudaGetErrorString(te), info);
    }
    c->prof.end(KC_TILE_CALL, 2.0 * NC * 3 * m.L * (double)(m.D * 3 * m.inner + m.inner * m.D + 2 * m.D * m.mlp),
                st);
    return LEWM_OK;
  };
  if (use_tile_call(c, NC, H, HS, emb_pc, 0)) {  // every call
    for (int k = 0; k < n_calls; ++k) {
      const lewm_status ts = tile_call(k);
      if (ts != LEWM_OK) return ts;
    }
    return LEWM_OK;
  }
  auto geom = [&](int k) {
    const int end = H + k;
    const int start = std::max(0, end - HS);
    const int w = end - start;
    // While the window only grows (start stays 0) a call's earlier positions are those of
    // the call before, with the same inputs and outputs: such a call runs only its new last
    // position, its attention reading the earlier keys / values from the cache that the
    // calls before wrote.
    const bool kv_read = kv_cache_on() && k >= 1 && end <= HS;
    const bool kv_write = kv_cache_on() && k + 1 < n_calls && end + 1 <= HS;
    const int rpc = kv_read ? 1 : w;
    int cpt, nt;
    tile_geom(NC, rpc, c->tile_target, &cpt, &nt);
    const int rows8 = std::min(128, (cpt * rpc + 7) & ~7);
    // Operands of tiles with more rows than one pass of the in-kernel build (512 threads,
    // D/12 per row) are built once per tile by a separate kernel.
    static const int pre_rows = [] {
      const char* v = std::getenv("LEWM_PREBUILT_ROWS");
      return v ? std::atoi(v) : -1;
    }();
    const int ln_prebuilt = rows8 > (pre_rows >= 0 ? pre_rows : 512 / (m.D / 12)) ? 1 : 0;
    // FC1 + GELU + FC2 fused into one kernel at width 192 / MLP 768: one CTA per (tile,
    // 192 hidden units). Used where it is fastest: tiles of at most 32 rows (operand built
    // in the kernel), and calls with enough tiles to fill the SMs (4 CTAs per tile;
    // throughput-bound, measured 387 -> 499 plans/s at 64 envs). A few large tiles keep
    // the two-kernel path (FC1 over 24 CTAs per tile, then the FC2 partial GEMM): more
    // CTAs in flight for a latency-bound call. LEWM_FFN_FUSED=0 keeps the two-kernel
    // path everywhere.
    static const int ffn_env = [] {
      const char* v = std::getenv("LEWM_FFN_FUSED");
      return v ? std::atoi(v) : 1;
    }();
    const int fc2_parts = (m.D == 192 && m.mlp == 4 * 192) ? 4 : 2;
    const bool ffn_small = !ln_prebuilt && rows8 <= 64;
    const bool ffn_many = nt * 4 >= c->sm_count;
    const int ffn_fused = (ffn_env != 0 && fc2_parts == 4 && (ffn_small || ffn_many)) ? 1 : 0;
    // Out-projection: 4 N pieces of D/4 x 2 K halves per tile (8 CTAs: latency), or, once
    // the calls' tiles fill the SMs with 2 CTAs each, all D columns per CTA (N = 192 runs
    // at the tensor pipe's peak rate, N = 48 on its per-instruction floor). Same K order
    // per output element either way, so the same bits.
    const int outproj_wide = (m.D == 192 && nt * 2 >= c->sm_count) ? 1 : 0;
    CallGeom g{};  // fields by name: a field added to CallGeom cannot shift the others
    g.n_cand = NC;
    g.S = S;
    g.T = T;
    g.H = H;
    g.w = w;
    g.start = start;
    g.cpt = cpt;
    g.n_tiles = nt;
    g.rows8 = rows8;
    g.ln_prebuilt = ln_prebuilt;
    g.ffn_fused = ffn_fused;
    g.fc2_parts = fc2_parts;
    g.outproj_wide = outproj_wide;
    g.call = k;
    g.last = k == n_calls - 1 ? 1 : 0;
    g.next_w = 1;
    g.next_start = 0;
    g.next_cpt = 128;
    // QKV + attention by head-resident CTAs (16 heads x kQkvGroups tile groups) once the
    // operands are prebuilt and every group has at least 4 tiles; LEWM_QKV_PERSISTENT=0 keeps
    // one CTA per (tile, head) everywhere.
    static const int qkv_env = [] {
      const char* v = std::getenv("LEWM_QKV_PERSISTENT");
      return v ? std::atoi(v) : 1;
    }();
    g.qkv_persistent = (qkv_env != 0 && m.D == 192 && m.heads == 16 && ln_prebuilt && nt >= 4 * kQkvGroups) ? 1 : 0;
    g.rpc = rpc;
    g.pos0 = w - rpc;
    g.kv_read = kv_read ? 1 : 0;
    g.kv_write = kv_write ? 1 : 0;
    g.next_rpc = 1;
    g.next_pos0 = 0;
    return g;
  };
  for (int k = 0; k < n_calls; ++k) {
    if (use_tile_call(c, NC, H, HS, emb_pc, k)) {  // a full window from this call on
      const lewm_status ts = tile_call(k);
      if (ts != LEWM_OK) return ts;
      continue;
    }
    CallGeom g = geom(k);
    if (k + 1 < n_calls) {
      const CallGeom gn = geom(k + 1);
      g.next_w = gn.w;
      g.next_start = gn.start;
      g.next_cpt = gn.cpt;
      g.next_rpc = gn.rpc;
      g.next_pos0 = gn.pos0;
    }
    // Calls alternate residual buffers: k_final of call k writes call k+1's layer-0 rows.
    b.x = (k & 1) ? c->ws.x2 : c->ws.x;
    b.xn = (k & 1) ? c->ws.x : c->ws.x2;
    if (k == 0) LEWM_CK(c, launch_prep0(m, c->w, g, b, st, &c->prof));
    LEWM_CK(c, launch_call(m, c->w, g, b, c->d_status, st, &c->prof));
    if (m.pp_hidden) {  // pred_proj on the new predictions (JEPA.predict, lewm/jepa.py:106-114)
      LEWM_CK(c, mlp_head_run(c->pp, c->ws.pp_in, NC, c->ws.pp_hid, c->ws.pp_hid32, c->ws.pp_out, c->d_status, st));
      LEWM_CK(c, launch_final_post(m, c->w, g, b, st, &c->prof));
    }
  }
  return LEWM_OK;
}

int max_call_tiles(int NC, int T, int H, int HS, int target) {
  int t = 1;
  for (int k = 0; k < T - H + 1; ++k) {
    const int end = H + k;
    t = std::max(t, window_tiles(NC, end - std::max(0, end - HS), target));
  }
  return t;
}

void coloring_matrix(int n, double beta, double* W) {
  // W[t][u] = irfft(rfft(e_u) * scale)[t]; scale_f = (f/n)^(-beta/2) for f >= 1, scale_0 = scale_1.
  std::vector<double> s(n / 2 + 1);
  for (int f = 1; f <= n / 2; ++f) s[f] = std::pow((double)f / n, -beta / 2.0);
  s[0] = (n / 2 >= 1) ? s[1] : 1.0;
  const double pi = 3.14159265358979323846;
  for (int t = 0; t < n; ++t)
    for (int u = 0; u < n; ++u) {
      const int d = t - u;
      double acc = s[0];
      for (int f = 1; f <= n / 2; ++f) {
        const double wgt = (2 * f == n) ? 1.0 : 2.0;
        acc += wgt * s[f] * std::cos(2.0 * pi * f * d / n);
      }
      W[t * n + u] = acc / n;
    }
}

lewm_status check_plan(lewm_ctx* c, const lewm_plan_desc* p) {
  if (!p) return fail(c, LEWM_INVALID_ARG, "plan desc is NULL");
  if (p->topk <= 0) return fail(c, LEWM_INVALID_ARG, "topk must be positive, got %d", p->topk);
  if (p->num_samples < p->topk)
    return fail(c, LEWM_INVALID_ARG, "num_samples=%d must be >= topk=%d", p->num_samples, p->topk);
  if (p->n_steps <= 0) return fail(c, LEWM_INVALID_ARG, "n_steps must be positive, got %d", p->n_steps);
  if (p->elite_retention < 0)
    return fail(c, LEWM_INVALID_ARG, "elite_retention must be non-negative, got %d", p->elite_retention);
  if (!(p->momentum_alpha >= 0.f && p->momentum_alpha < 1.f))
    return fail(c, LEWM_INVALID_ARG, "momentum_alpha must satisfy 0 <= alpha < 1, got %g", p->momentum_alpha);
  if (!(p->sample_decay >= 1.0)) return fail(c, LEWM_INVALID_ARG, "sample_decay must be >= 1.0, got %g", p->sample_decay);
  if (p->sample_counts)
    for (int i = 0; i < p->n_steps; ++i)
      if (p->sample_counts[i] < p->topk || p->sample_counts[i] > p->num_samples)
        return fail(c, LEWM_INVALID_ARG, "sample_counts[%d]=%d must lie in [topk=%d, num_samples=%d]", i,
                    p->sample_counts[i], p->topk, p->num_samples);
  if (p->bucket < 0) return fail(c, LEWM_INVALID_ARG, "sample_count_bucket_size must be non-negative, got %d", p->bucket);
  if (p->action_block <= 0) return fail(c, LEWM_INVALID_ARG, "action_block must be positive, got %d", p->action_block);
  if (!(p->beta >= 0.f)) return fail(c, LEWM_INVALID_ARG, "beta must be >= 0");
  if (p->n_envs <= 0 || p->horizon <= 0 || p->history <= 0 || p->history > p->horizon || p->history_size <= 0)
    return fail(c, LEWM_INVALID_ARG, "need n_envs > 0 and 1 <= history <= horizon, history_size >= 1");
  if (c) {
    if (p->history_size > c->md.frames)
      return fail(c, LEWM_UNSUPPORTED_SHAPE, "history_size=%d exceeds num_frames=%d", p->history_size, c->md.frames);
    if (p->horizon * c->md.A > 128) return fail(c, LEWM_UNSUPPORTED_SHAPE, "horizon*action_dim must be <= 128");
    if (p->beta > 0.f && p->time_axis_raw && p->action_block > 1) {
      if (c->md.A % p->action_block)
        return fail(c, LEWM_INVALID_ARG, "action_dim=%d is not divisible by action_block=%d", c->md.A,
                    p->action_block);
      if (p->horizon * p->action_block > 128) return fail(c, LEWM_UNSUPPORTED_SHAPE, "horizon*action_block > 128");
    }
    if (p->num_samples > 4096) return fail(c, LEWM_UNSUPPORTED_SHAPE, "num_samples must be <= 4096");
    if (p->topk > 512) return fail(c, LEWM_UNSUPPORTED_SHAPE, "topk must be <= 512");
  }
  return LEWM_OK;
}

std::vector<int> counts_of(const lewm_plan_desc* p) {
  if (p->sample_counts) return std::vector<int>(p->sample_counts, p->sample_counts + p->n_steps);
  std::vector<int> out(p->n_steps);
  for (int s = 0; s < p->n_steps; ++s) {
    int count;
    if (p->sample_decay == 1.0) {
      count = p->num_samples;
    } else {
      const int decayed = (int)std::ceil(p->num_samples * std::pow(p->sample_decay, (double)-s));
      count = std::max(decayed, std::min(p->num_samples, 2 * p->topk));
      if (p->bucket > 0)
        count = std::min(p->num_samples, (int)std::ceil((double)count / p->bucket) * p->bucket);
    }
    out[s] = count;
  }
  return out;
}

// Noise layout of make_colored_noise for this plan: kind and colored length.
void noise_kind(const lewm_ctx* c, const lewm_plan_desc* p, int* kind, int* ncol) {
  if (p->beta <= 0.f) {
    *kind = 0;
    *ncol = 0;
    return;
  }
  if (p->time_axis_raw && p->action_block > 1) {
    *kind = 1;
    *ncol = p->horizon * p->action_block;
  } else {
    *kind = 2;
    *ncol = p->horizon;
  }
  if (*ncol <= 1) {
    *kind = 0;
    *ncol = 0;
  }
  (void)c;
}

lewm_status upload_W(lewm_ctx* c, const lewm_plan_desc* p, int ncol, cudaStream_t st) {
  if (ncol <= 1) return LEWM_OK;
  if (c->W_n == ncol && c->W_beta == p->beta) return LEWM_OK;
  std::vector<double> Wd((size_t)ncol * ncol);
  coloring_matrix(ncol, p->beta, Wd.data());
  c->W_host.assign(Wd.begin(), Wd.end());
  LEWM_CK(c, cudaMemcpyAsync(c->ws.W, c->W_host.data(), c->W_host.size() * 4, cudaMemcpyHostToDevice, st));
  LEWM_CK(c, cudaStreamSynchronize(st));  // W_host may be rewritten by a later call
  c->W_n = ncol;
  c->W_beta = p->beta;
  return LEWM_OK;
}

struct PlanIO {
  const float* emb;
  const float* goal;
  const float* low;
  const float* high;
};

bool graphs_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("LEWM_NO_GRAPH");
    return !(v && v[0] == '1');
  }();
  return on;
}

std::vector<double> plan_key(const lewm_plan_desc* p, int kind, int ncol) {
  std::vector<double> key{(double)p->n_envs, (double)p->horizon, (double)p->history, (double)p->history_size,
                          (double)p->num_samples, (double)p->topk, (double)p->n_steps, p->sample_decay,
                          (double)p->bucket, (double)p->elite_retention, (double)kind, (double)ncol,
                          (double)p->action_block, (double)p->momentum_alpha, (double)p->return_best_elite,
                          (double)p->clip_actions, p->sample_counts ? 1.0 : 0.0};
  if (p->sample_counts)
    for (int i = 0; i < p->n_steps; ++i) key.push_back((double)p->sample_counts[i]);
  return key;
}

// Every launch of one plan: per iteration sample -> model cost -> top-k/refit.
// Reads the distribution from ws.mean / ws.stdv (set by the caller) and leaves the
// result there; the Philox key is read from ws.rng at run time.
lewm_status plan_iterations(lewm_ctx* c, const lewm_plan_desc* p, const std::vector<int>& counts, int kind,
                            int ncol, const PlanIO& io, const float* const* noise_steps,
                            const lewm_plan_trace* trace, cudaStream_t st) {
  const ModelDims& m = c->md;
  Workspace& ws = c->ws;
  const int B = p->n_envs, T = p->horizon, A = m.A, TA = T * A, k = p->topk;
  const int R = std::min(p->elite_retention, k);
  for (int it = 0; it < p->n_steps; ++it) {
    const int St = counts[it];
    const int n_inject = (it > 0 && p->elite_retention > 0) ? std::min(R, St - 1) : 0;
    SampleParams sp{};
    sp.B = B;
    sp.S = St;
    sp.T = T;
    sp.A = A;
    sp.noise_kind = kind;
    sp.raw_block = p->action_block;
    sp.ncol = ncol;
    sp.W = ws.W;
    sp.noise = noise_steps ? noise_steps[it] : nullptr;
    sp.rng = ws.rng;
    sp.iter = (uint32_t)it;
    sp.mean = ws.mean;
    sp.stdv = ws.stdv;
    sp.elites = ws.elites;
    sp.elite_stride = std::max(R, 1);
    sp.n_inject = std::max(n_inject, 0);
    sp.low = io.low;
    sp.high = io.high;
    sp.cand = ws.cand;
    c->prof.begin(st);
    LEWM_CK(c, launch_sample(sp, st));
    c->prof.end(KC_SAMPLE, 0.0, st);
    lewm_status s = run_model_cost(c, io.emb, 0, p->history, io.goal, 0, ws.cand, B, St, T, p->history_size,
                                   ws.costs, st);
    if (s != LEWM_OK) return s;
    RefitParams rp{};
    rp.B = B;
    rp.S = St;
    rp.T = T;
    rp.A = A;
    rp.k = k;
    rp.R = R;
    rp.costs = ws.costs;
    rp.cand = ws.cand;
    rp.mean = ws.mean;
    rp.stdv = ws.stdv;
    rp.alpha = p->momentum_alpha;
    rp.elites = ws.elites;
    rp.best = ws.best;
    rp.final_cost = ws.fcost;
    rp.topk_idx = (trace && trace->topk_idx) ? trace->topk_idx + (size_t)it * B * k : nullptr;
    rp.topk_val = (trace && trace->topk_val) ? trace->topk_val + (size_t)it * B * k : nullptr;
    rp.nan_status = (it == p->n_steps - 1) ? c->d_status : nullptr;  // the plan's final costs
    c->prof.begin(st);
    LEWM_CK(c, launch_refit(rp, st));
    c->prof.end(KC_REFIT, 0.0, st);
    if (trace) {
      const size_t S = p->num_samples;
      if (trace->costs)
        LEWM_CK(c, cudaMemcpy2DAsync(trace->costs + (size_t)it * B * S, S * 4, ws.costs, (size_t)St * 4,
                                     (size_t)St * 4, B, cudaMemcpyDeviceToDevice, st));
      if (trace->candidates)
        LEWM_CK(c, cudaMemcpy2DAsync(trace->candidates + (size_t)it * B * S * TA, S * TA * 4, ws.cand,
                                     (size_t)St * TA * 4, (size_t)St * TA * 4, B, cudaMemcpyDeviceToDevice, st));
      if (trace->mean)
        LEWM_CK(c, cudaMemcpyAsync(trace->mean + (size_t)it * B * TA, ws.mean, (size_t)B * TA * 4,
                                   cudaMemcpyDeviceToDevice, st));
      if (trace->std)
        LEWM_CK(c, cudaMemcpyAsync(trace->std + (size_t)it * B * TA, ws.stdv, (size_t)B * TA * 4,
                                   cudaMemcpyDeviceToDevice, st));
    }
  }
  return LEWM_OK;
}

lewm_status copy_plan_outputs(lewm_ctx* c, const lewm_plan_desc* p, float* actions_out, float* std_out,
                              float* final_cost_out, cudaStream_t st) {
  const size_t bta = (size_t)p->n_envs * p->horizon * c->md.A * 4;
  LEWM_CK(c, cudaMemcpyAsync(actions_out, p->return_best_elite ? c->ws.best : c->ws.mean, bta,
                             cudaMemcpyDeviceToDevice, st));
  LEWM_CK(c, cudaMemcpyAsync(std_out, c->ws.stdv, bta, cudaMemcpyDeviceToDevice, st));
  LEWM_CK(c, cudaMemcpyAsync(final_cost_out, c->ws.fcost, (size_t)p->n_envs * 4, cudaMemcpyDeviceToDevice, st));
  return LEWM_OK;
}

}  // namespace

namespace lewm {
void set_noctx_error(const char* msg) { g_create_error = msg; }
}  // namespace lewm

extern "C" {

size_t lewm_weight_count(const lewm_model_desc* desc) {
  ModelDims md{};
  if (check_desc(desc, &md) != LEWM_OK) return 0;
  return weight_count(md);
}

lewm_status lewm_create(lewm_ctx** out, const lewm_model_desc* desc, const float* weights, size_t n_floats,
                        int device) {
  if (!out) return fail(nullptr, LEWM_INVALID_ARG, "out is NULL");
  *out = nullptr;
  ModelDims md{};
  lewm_status s = check_desc(desc, &md);
  if (s != LEWM_OK) return s;
  if (!weights) return fail(nullptr, LEWM_INVALID_ARG, "weights is NULL");
  if (n_floats != weight_count(md))
    return fail(nullptr, LEWM_INVALID_ARG, "expected %zu weight floats, got %zu", weight_count(md), n_floats);
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev)
    return fail(nullptr, LEWM_CUDA_ERROR, "no CUDA device %d", device);
  DeviceGuard g(device);
  cudaDeviceProp prop{};
  cudaGetDeviceProperties(&prop, device);
  if (prop.major != 10) return fail(nullptr, LEWM_UNSUPPORTED_SHAPE, "device %d is sm_%d%d, need sm_100", device, prop.major, prop.minor);
  auto* c = new lewm_ctx();
  c->device = device;
  c->desc = *desc;
  c->md = md;
  // Small calls spread over about two thirds of one QKV wave (SMs / heads): the SMs
  // left free let the next kernel's CTAs launch early and prefetch their weights
  // (measured on B200, the 1-env 300-sample plan: 6 tiles 18.25 ms, 4 tiles 19.42 ms,
  // 8 tiles 19.04 ms, 3 tiles 19.70 ms, 12 tiles 22.83 ms).
  c->tile_target = std::max(1, prop.multiProcessorCount / md.heads * 2 / 3);
  c->sm_count = prop.multiProcessorCount;
  if (const char* tt = std::getenv("LEWM_TILE_TARGET")) {  // tuning override
    const int v = std::atoi(tt);
    if (v > 0) c->tile_target = v;
  }
  if (const char* tm = std::getenv("LEWM_TILE_CALL_MIN")) c->tile_call_min = std::atoi(tm);  // read per context
  s = pack_weights(c, weights, n_floats);
  if (s == LEWM_OK) s = upload_f32_weights(c, weights, n_floats);
  if (s == LEWM_OK && cudaMalloc(&c->d_status, kStatusBytes) != cudaSuccess) s = fail(c, LEWM_CUDA_ERROR, "status alloc");
  if (s == LEWM_OK && cudaMemset(c->d_status, 0, kStatusBytes) != cudaSuccess)
    s = fail(c, LEWM_CUDA_ERROR, "status memset");
  if (s == LEWM_OK && (cudaStreamCreateWithFlags(&c->cap_stream, cudaStreamNonBlocking) != cudaSuccess ||
                       cudaEventCreateWithFlags(&c->ev_in, cudaEventDisableTiming) != cudaSuccess ||
                       cudaEventCreateWithFlags(&c->ev_out, cudaEventDisableTiming) != cudaSuccess))
    s = fail(c, LEWM_CUDA_ERROR, "stream/event creation");
  if (s != LEWM_OK) {
    g_create_error = c->err;
    lewm_destroy(c);
    return s;
  }
  *out = c;
  return LEWM_OK;
}

void lewm_destroy(lewm_ctx* c) {
  if (!c) return;
  DeviceGuard g(c->device);
  if (c->cap_stream) cudaStreamSynchronize(c->cap_stream);
  clear_graphs(c);
  if (c->ev_in) cudaEventDestroy(c->ev_in);
  if (c->ev_out) cudaEventDestroy(c->ev_out);
  if (c->cap_stream) cudaStreamDestroy(c->cap_stream);
  if (c->ws.base) cudaFree(c->ws.base);
  if (c->d_weights) cudaFree(c->d_weights);
  if (c->d_w32) cudaFree(c->d_w32);
  if (c->d_grad) cudaFree(c->d_grad);
  mlp_head_destroy(&c->pp);
  if (c->d_status) cudaFree(c->d_status);
  delete c;
}

const char* lewm_last_error(const lewm_ctx* c) { return c ? c->err.c_str() : g_create_error.c_str(); }

lewm_status lewm_model_cost(lewm_ctx* c, const float* emb, int32_t emb_per_sample, int32_t H, const float* goal,
                            int32_t goal_per_sample, const float* cand, int32_t B, int32_t S, int32_t T,
                            int32_t history_size, float* costs_out, void* stream) {
  if (!c) return fail(nullptr, LEWM_INVALID_ARG, "ctx is NULL");
  c->err.clear();
  if (!emb || !goal || !cand || !costs_out) return fail(c, LEWM_INVALID_ARG, "NULL tensor pointer");
  if (B <= 0 || S <= 0 || T <= 0 || H <= 0 || H > T || history_size <= 0)
    return fail(c, LEWM_INVALID_ARG, "need B,S,T > 0 and 1 <= H <= T, got B=%d S=%d T=%d H=%d", B, S, T, H);
  if (history_size > c->md.frames)
    return fail(c, LEWM_UNSUPPORTED_SHAPE, "history_size=%d exceeds num_frames=%d", history_size, c->md.frames);
  if ((int64_t)B * S * T > (1ll << 26)) return fail(c, LEWM_UNSUPPORTED_SHAPE, "B*S*T too large");
  DeviceGuard g(c->device);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int NC = B * S;
  WsReq need{(size_t)NC, (size_t)T, (size_t)c->md.A, (size_t)c->md.D, (size_t)c->md.L,
             (size_t)max_call_tiles(NC, T, H, history_size, c->tile_target), (size_t)c->md.heads, (size_t)c->md.mlp,
             (size_t)(T - H + 1), 1, 0, 0, (size_t)kv_positions(H, history_size)};
  lewm_status s = ensure_ws(c, need);
  if (s != LEWM_OK) return s;
  return run_model_cost(c, emb, emb_per_sample != 0, H, goal, goal_per_sample != 0, cand, B, S, T, history_size,
                        costs_out, st);
}

lewm_status lewm_model_cost_grad(lewm_ctx* c, const float* emb, int32_t emb_per_sample, int32_t H, const float* goal,
                                 int32_t goal_per_sample, const float* cand, int32_t B, int32_t S, int32_t T,
                                 int32_t history_size, const float* cost_weights, float* costs_out, float* grad_out,
                                 void* stream) {
  if (!c) return fail(nullptr, LEWM_INVALID_ARG, "ctx is NULL");
  c->err.clear();
  if (!emb || !goal || !cand || !costs_out || !grad_out) return fail(c, LEWM_INVALID_ARG, "NULL tensor pointer");
  if (B <= 0 || S <= 0 || T <= 0 || H <= 0 || H > T || history_size <= 0)
    return fail(c, LEWM_INVALID_ARG, "need B,S,T > 0 and 1 <= H <= T, got B=%d S=%d T=%d H=%d", B, S, T, H);
  if (history_size > c->md.frames)
    return fail(c, LEWM_UNSUPPORTED_SHAPE, "history_size=%d exceeds num_frames=%d", history_size, c->md.frames);
  if (c->md.pp_hidden)
    return fail(c, LEWM_UNSUPPORTED_SHAPE, "the model-cost gradient covers an Identity pred_proj only");
  if ((int64_t)B * S * T > (1ll << 22)) return fail(c, LEWM_UNSUPPORTED_SHAPE, "B*S*T too large for the gradient");
  DeviceGuard g(c->device);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int NC = B * S;
  WsReq need{(size_t)NC, (size_t)T, (size_t)c->md.A, (size_t)c->md.D, (size_t)c->md.L,
             (size_t)max_call_tiles(NC, T, H, history_size, c->tile_target), (size_t)c->md.heads, (size_t)c->md.mlp,
             (size_t)(T - H + 1), 1, 0, 0, (size_t)kv_positions(H, history_size)};
  need.f32_nc = (size_t)NC;
  need.f32_T = (size_t)T;
  lewm_status s = ensure_ws(c, need);
  if (s != LEWM_OK) return s;
  const size_t nf = f32_grad_floats(c->md, NC, T, H, history_size);
  if (nf > c->grad_floats) {  // grows; cudaFree waits for the work that used the old buffers
    for (auto& kv : c->grad_graphs) cudaGraphExecDestroy(kv.second);
    c->grad_graphs.clear();
    if (c->d_grad) cudaFree(c->d_grad);
    c->d_grad = nullptr;
    c->grad_floats = 0;
    LEWM_CK(c, cudaMalloc(&c->d_grad, nf * 4));
    c->grad_floats = nf;
  }
  F32Tape tape;
  F32GradWork gw{};
  f32_grad_carve(c->md, NC, T, H, history_size, c->d_grad, &tape, &gw);
  const bool emb_pc = emb_per_sample != 0, goal_pc = goal_per_sample != 0;
  if (c->prof.on || !graphs_enabled()) {
    LEWM_CK(c, run_model_cost_grad_fp32(c->md, c->w32, c->ws.f32, tape, gw, emb, emb_pc, H, goal, goal_pc, cand, B,
                                        S, T, history_size, cost_weights, costs_out, grad_out, st));
    return LEWM_OK;
  }
  // Graph path (the pass is ~640 small launches): stage the inputs into the gradient buffer so
  // the captured pass is pointer-stable, replay the cached graph of this shape, copy out.
  const ModelDims& m = c->md;
  const size_t n_emb = (size_t)(emb_pc ? NC : B) * H * m.D, n_goal = (size_t)(goal_pc ? NC : B) * m.D;
  const size_t n_cand = (size_t)NC * T * m.A;
  cudaStream_t cs = c->cap_stream;
  LEWM_CK(c, cudaEventRecord(c->ev_in, st));
  LEWM_CK(c, cudaStreamWaitEvent(cs, c->ev_in, 0));
  LEWM_CK(c, cudaMemcpyAsync(gw.in_emb, emb, n_emb * 4, cudaMemcpyDeviceToDevice, cs));
  LEWM_CK(c, cudaMemcpyAsync(gw.in_goal, goal, n_goal * 4, cudaMemcpyDeviceToDevice, cs));
  LEWM_CK(c, cudaMemcpyAsync(gw.in_cand, cand, n_cand * 4, cudaMemcpyDeviceToDevice, cs));
  if (cost_weights) LEWM_CK(c, cudaMemcpyAsync(gw.in_w, cost_weights, (size_t)NC * 4, cudaMemcpyDeviceToDevice, cs));
  const std::vector<int> key{B, S, T, H, history_size, emb_pc ? 1 : 0, goal_pc ? 1 : 0, cost_weights ? 1 : 0};
  auto it = c->grad_graphs.find(key);
  if (it == c->grad_graphs.end()) {
    cudaGraph_t graph = nullptr;
    LEWM_CK(c, cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal));
    const cudaError_t re = run_model_cost_grad_fp32(m, c->w32, c->ws.f32, tape, gw, gw.in_emb, emb_pc, H, gw.in_goal,
                                                    goal_pc, gw.in_cand, B, S, T, history_size,
                                                    cost_weights ? gw.in_w : nullptr, gw.out_cost, gw.out_grad, cs);
    const cudaError_t ce = cudaStreamEndCapture(cs, &graph);
    if (re != cudaSuccess || ce != cudaSuccess) {
      if (graph) cudaGraphDestroy(graph);
      return fail(c, LEWM_CUDA_ERROR, "gradient graph capture: %s",
                  cudaGetErrorString(re != cudaSuccess ? re : ce));
    }
    cudaGraphExec_t exec = nullptr;
    const cudaError_t ie = cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    if (ie != cudaSuccess) return fail(c, LEWM_CUDA_ERROR, "gradient graph instantiate: %s", cudaGetErrorString(ie));
    it = c->grad_graphs.emplace(key, exec).first;
  }
  LEWM_CK(c, cudaGraphLaunch(it->second, cs));
  LEWM_CK(c, cudaMemcpyAsync(costs_out, gw.out_cost, (size_t)NC * 4, cudaMemcpyDeviceToDevice, cs));
  LEWM_CK(c, cudaMemcpyAsync(grad_out, gw.out_grad, n_cand * 4, cudaMemcpyDeviceToDevice, cs));
  LEWM_CK(c, cudaEventRecord(c->ev_out, cs));
  LEWM_CK(c, cudaStreamWaitEvent(st, c->ev_out, 0));
  return LEWM_OK;
}

lewm_status lewm_sample_counts(const lewm_plan_desc* plan, int32_t* counts_out, int32_t cap, int64_t* evals_out) {
  lewm_status s = check_plan(nullptr, plan);
  if (s != LEWM_OK) return s;
  const std::vector<int> cs = counts_of(plan);
  int64_t tot = 0;
  for (size_t i = 0; i < cs.size(); ++i) {
    if (counts_out && (int32_t)i < cap) counts_out[i] = cs[i];
    tot += cs[i];
  }
  if (evals_out) *evals_out = tot;
  return LEWM_OK;
}

lewm_status lewm_plan(lewm_ctx* c, const lewm_plan_desc* p, const float* emb, const float* goal,
                      const float* init_mean, const float* init_std, const float* const* noise_steps,
                      const float* action_low, const float* action_high, float* actions_out, float* std_out,
                      float* final_cost_out, const lewm_plan_trace* trace, void* stream) {
  if (!c) return fail(nullptr, LEWM_INVALID_ARG, "ctx is NULL");
  c->err.clear();
  lewm_status s = check_plan(c, p);
  if (s != LEWM_OK) return s;
  if (!emb || !goal || !init_mean || !init_std || !actions_out || !std_out || !final_cost_out)
    return fail(c, LEWM_INVALID_ARG, "NULL tensor pointer");
  if (p->clip_actions && (!action_low || !action_high))
    return fail(c, LEWM_INVALID_ARG, "clip_actions needs action_low and action_high");
  if (noise_steps)
    for (int i = 0; i < p->n_steps; ++i)
      if (!noise_steps[i]) return fail(c, LEWM_INVALID_ARG, "noise_steps[%d] is NULL", i);
  DeviceGuard g(c->device);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const ModelDims& m = c->md;
  const int B = p->n_envs, T = p->horizon, A = m.A, TA = T * A, H = p->history;
  const std::vector<int> counts = counts_of(p);
  const int Smax = *std::max_element(counts.begin(), counts.end());
  if ((int64_t)B * Smax * T > (1ll << 26)) return fail(c, LEWM_UNSUPPORTED_SHAPE, "n_envs*num_samples*T too large");
  int kind, ncol;
  noise_kind(c, p, &kind, &ncol);
  const int R = std::min(p->elite_retention, p->topk);
  const int NC = B * Smax;
  WsReq need{(size_t)NC, (size_t)T, (size_t)A, (size_t)m.D, (size_t)m.L,
             (size_t)max_call_tiles(NC, T, H, p->history_size, c->tile_target), (size_t)m.heads, (size_t)m.mlp,
             (size_t)(T - H + 1), (size_t)B, (size_t)R, (size_t)std::max(ncol, 1),
             (size_t)kv_positions(H, p->history_size)};
  s = ensure_ws(c, need);
  if (s != LEWM_OK) return s;
  Workspace& ws = c->ws;
  s = upload_W(c, p, ncol, st);
  if (s != LEWM_OK) return s;
  const uint32_t seed = (uint32_t)(p->seed & 0xffffffffu), plan = (uint32_t)(p->plan_index & 0xffffffffu);
  const bool use_graph = !noise_steps && !trace && !c->prof.on && graphs_enabled();
  if (!use_graph) {
    LEWM_CK(c, cudaMemcpyAsync(ws.mean, init_mean, (size_t)B * TA * 4, cudaMemcpyDeviceToDevice, st));
    LEWM_CK(c, cudaMemcpyAsync(ws.stdv, init_std, (size_t)B * TA * 4, cudaMemcpyDeviceToDevice, st));
    LEWM_CK(c, launch_set_rng(ws.rng, seed, plan, st));
    PlanIO io{emb, goal, p->clip_actions ? action_low : nullptr, p->clip_actions ? action_high : nullptr};
    s = plan_iterations(c, p, counts, kind, ncol, io, noise_steps, trace, st);
    if (s != LEWM_OK) return s;
    return copy_plan_outputs(c, p, actions_out, std_out, final_cost_out, st);
  }
  // Graph path: stage the inputs into workspace buffers so the captured plan is
  // pointer-stable, replay the cached graph for this plan shape, copy outputs back.
  cudaStream_t cs = c->cap_stream;
  LEWM_CK(c, cudaEventRecord(c->ev_in, st));
  LEWM_CK(c, cudaStreamWaitEvent(cs, c->ev_in, 0));
  LEWM_CK(c, cudaMemcpyAsync(ws.emb_in, emb, (size_t)B * H * m.D * 4, cudaMemcpyDeviceToDevice, cs));
  LEWM_CK(c, cudaMemcpyAsync(ws.goal_in, goal, (size_t)B * m.D * 4, cudaMemcpyDeviceToDevice, cs));
  LEWM_CK(c, cudaMemcpyAsync(ws.mean, init_mean, (size_t)B * TA * 4, cudaMemcpyDeviceToDevice, cs));
  LEWM_CK(c, cudaMemcpyAsync(ws.stdv, init_std, (size_t)B * TA * 4, cudaMemcpyDeviceToDevice, cs));
  if (p->clip_actions) {
    LEWM_CK(c, cudaMemcpyAsync(ws.lohi, action_low, (size_t)A * 4, cudaMemcpyDeviceToDevice, cs));
    LEWM_CK(c, cudaMemcpyAsync(ws.lohi + A, action_high, (size_t)A * 4, cudaMemcpyDeviceToDevice, cs));
  }
  LEWM_CK(c, launch_set_rng(ws.rng, seed, plan, cs));
  const std::vector<double> key = plan_key(p, kind, ncol);
  auto it = c->graphs.find(key);
  if (it == c->graphs.end()) {
    cudaGraph_t graph = nullptr;
    LEWM_CK(c, cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal));
    PlanIO io{ws.emb_in, ws.goal_in, p->clip_actions ? ws.lohi : nullptr, p->clip_actions ? ws.lohi + A : nullptr};
    s = plan_iterations(c, p, counts, kind, ncol, io, nullptr, nullptr, cs);
    const cudaError_t ce = cudaStreamEndCapture(cs, &graph);
    if (s != LEWM_OK) {
      if (graph) cudaGraphDestroy(graph);
      return s;
    }
    if (ce != cudaSuccess) {
      if (graph) cudaGraphDestroy(graph);
      return fail(c, LEWM_CUDA_ERROR, "plan graph capture: %s", cudaGetErrorString(ce));
    }
    cudaGraphExec_t exec = nullptr;
    const cudaError_t ie = cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    if (ie != cudaSuccess) return fail(c, LEWM_CUDA_ERROR, "plan graph instantiate: %s", cudaGetErrorString(ie));
    it = c->graphs.emplace(key, exec).first;
  }
  LEWM_CK(c, cudaGraphLaunch(it->second, cs));
  s = copy_plan_outputs(c, p, actions_out, std_out, final_cost_out, cs);
  if (s != LEWM_OK) return s;
  LEWM_CK(c, cudaEventRecord(c->ev_out, cs));
  LEWM_CK(c, cudaStreamWaitEvent(st, c->ev_out, 0));
  return LEWM_OK;
}

lewm_status lewm_topk_refit(lewm_ctx* c, const float* costs, const float* cand, int32_t B, int32_t S, int32_t T,
                            int32_t A, int32_t k, float momentum_alpha, float* mean, float* std, int32_t* topk_idx,
                            float* topk_val, float* best, float* final_cost, void* stream) {
  if (!c) return fail(nullptr, LEWM_INVALID_ARG, "ctx is NULL");
  c->err.clear();
  if (!costs || !cand || !mean || !std || !best || !final_cost) return fail(c, LEWM_INVALID_ARG, "NULL tensor pointer");
  if (B <= 0 || S <= 0 || T <= 0 || A <= 0 || k <= 0 || k > S)
    return fail(c, LEWM_INVALID_ARG, "need B,S,T,A > 0 and 1 <= k <= S");
  if (S > 4096 || T * A > 128 || k > 512) return fail(c, LEWM_UNSUPPORTED_SHAPE, "S <= 4096, T*A <= 128, k <= 512");
  if (!(momentum_alpha >= 0.f && momentum_alpha < 1.f)) return fail(c, LEWM_INVALID_ARG, "0 <= momentum_alpha < 1");
  DeviceGuard g(c->device);
  RefitParams rp{};
  rp.B = B;
  rp.S = S;
  rp.T = T;
  rp.A = A;
  rp.k = k;
  rp.R = 0;
  rp.costs = costs;
  rp.cand = cand;
  rp.mean = mean;
  rp.stdv = std;
  rp.alpha = momentum_alpha;
  rp.elites = nullptr;
  rp.best = best;
  rp.final_cost = final_cost;
  rp.topk_idx = topk_idx;
  rp.topk_val = topk_val;
  LEWM_CK(c, launch_refit(rp, static_cast<cudaStream_t>(stream)));
  return LEWM_OK;
}

lewm_status lewm_sample_candidates(lewm_ctx* c, const lewm_plan_desc* p, int32_t S, int32_t iter,
                                   const float* mean, const float* std, const float* injected_noise,
                                   const float* action_low, const float* action_high, float* out, void* stream) {
  if (!c) return fail(nullptr, LEWM_INVALID_ARG, "ctx is NULL");
  c->err.clear();
  lewm_status s = check_plan(c, p);
  if (s != LEWM_OK) return s;
  if (!mean || !std || !out || S <= 0 || iter < 0) return fail(c, LEWM_INVALID_ARG, "bad sample arguments");
  if (p->clip_actions && (!action_low || !action_high))
    return fail(c, LEWM_INVALID_ARG, "clip_actions needs action_low and action_high");
  DeviceGuard g(c->device);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int kind, ncol;
  noise_kind(c, p, &kind, &ncol);
  WsReq need{1, (size_t)p->horizon, (size_t)c->md.A, (size_t)c->md.D, (size_t)c->md.L, 1, (size_t)c->md.heads,
             (size_t)c->md.mlp, 1, 1, 0, (size_t)std::max(ncol, 1), 0};
  s = ensure_ws(c, need);
  if (s != LEWM_OK) return s;
  s = upload_W(c, p, ncol, st);
  if (s != LEWM_OK) return s;
  SampleParams sp{};
  sp.B = p->n_envs;
  sp.S = S;
  sp.T = p->horizon;
  sp.A = c->md.A;
  sp.noise_kind = kind;
  sp.raw_block = p->action_block;
  sp.ncol = ncol;
  sp.W = c->ws.W;
  sp.noise = injected_noise;
  LEWM_CK(c, launch_set_rng(c->ws.rng, (uint32_t)(p->seed & 0xffffffffu), (uint32_t)(p->plan_index & 0xffffffffu),
                            st));
  sp.rng = c->ws.rng;
  sp.iter = (uint32_t)iter;
  sp.mean = mean;
  sp.stdv = std;
  sp.elites = nullptr;
  sp.elite_stride = 1;
  sp.n_inject = 0;
  sp.low = p->clip_actions ? action_low : nullptr;
  sp.high = p->clip_actions ? action_high : nullptr;
  sp.cand = out;
  LEWM_CK(c, launch_sample(sp, st));
  return LEWM_OK;
}

lewm_status lewm_sync_status(lewm_ctx* c, void* stream) {
  if (!c) return fail(nullptr, LEWM_INVALID_ARG, "ctx is NULL");
  DeviceGuard g(c->device);
  LEWM_CK(c, cudaStreamSynchronize(static_cast<cudaStream_t>(stream)));
  if (c->cap_stream) LEWM_CK(c, cudaStreamSynchronize(c->cap_stream));
  LEWM_CK(c, cudaGetLastError());
  uint32_t v = 0;
  LEWM_CK(c, cudaMemcpy(&v, c->d_status, 4, cudaMemcpyDeviceToHost));
  if (v) {
    LEWM_CK(c, cudaMemset(c->d_status, 0, 4));
    if (v & (LEWM_DEV_TIMEOUT | LEWM_DEV_BADARG))
      return fail(c, LEWM_DEVICE_TIMEOUT, "device status 0x%x: a bounded device wait expired", v);
    return fail(c, LEWM_NUMERIC_NAN, "device status 0x%x: a plan produced a NaN final cost", v);
  }
  return LEWM_OK;
}

lewm_status lewm_set_wait_limit(lewm_ctx* c, uint64_t limit_ns) {
  if (!c) return fail(nullptr, LEWM_INVALID_ARG, "ctx is NULL");
  DeviceGuard g(c->device);
  LEWM_CK(c, cudaDeviceSynchronize());
  LEWM_CK(c, cudaMemcpy(reinterpret_cast<uint8_t*>(c->d_status) + 8, &limit_ns, 8, cudaMemcpyHostToDevice));
  return LEWM_OK;
}

lewm_status lewm_wait_selftest(lewm_ctx* c, void* stream) {
  if (!c) return fail(nullptr, LEWM_INVALID_ARG, "ctx is NULL");
  DeviceGuard g(c->device);
  LEWM_CK(c, launch_wait_selftest(c->d_status, static_cast<cudaStream_t>(stream)));
  return LEWM_OK;
}

int32_t lewm_abi_version(void) { return LEWM_ABI_VERSION; }

lewm_status lewm_set_model_cost_autocast(lewm_ctx* c, int32_t mode) {
  if (!c) return fail(nullptr, LEWM_INVALID_ARG, "ctx is NULL");
  c->err.clear();
  if (mode != LEWM_AUTOCAST_NONE && mode != LEWM_AUTOCAST_BF16)
    return fail(c, LEWM_INVALID_ARG, "Unsupported model_cost_autocast mode: %d (0 none, 1 bf16)", mode);
  if (mode == c->autocast) return LEWM_OK;
  DeviceGuard g(c->device);
  LEWM_CK(c, cudaDeviceSynchronize());
  clear_graphs(c);  // captured plans hold the other arithmetic's launches
  c->autocast = mode;
  return LEWM_OK;
}

lewm_status lewm_profile_plan(lewm_ctx* c, const lewm_plan_desc* p, const float* emb, const float* goal,
                              const float* init_mean, const float* init_std, double* ms_out, double* flops_out,
                              int32_t* launches_out, void* stream) {
  if (!c) return fail(nullptr, LEWM_INVALID_ARG, "ctx is NULL");
  if (!ms_out || !flops_out || !launches_out) return fail(c, LEWM_INVALID_ARG, "NULL output array");
  if (!p) return fail(c, LEWM_INVALID_ARG, "plan desc is NULL");
  DeviceGuard g(c->device);
  const int B = p->n_envs, TA = p->horizon * c->md.A;
  float *act = nullptr, *sd = nullptr, *fc = nullptr;
  LEWM_CK(c, cudaMalloc(&act, (size_t)B * TA * 4 * 2 + (size_t)B * 4));
  sd = act + (size_t)B * TA;
  fc = sd + (size_t)B * TA;
  c->prof.reset();
  c->prof.on = true;
  pdl_suppressed() = true;
  lewm_status s = lewm_plan(c, p, emb, goal, init_mean, init_std, nullptr, nullptr, nullptr, act, sd, fc, nullptr,
                            stream);
  pdl_suppressed() = false;
  c->prof.on = false;
  cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
  cudaFree(act);
  if (s != LEWM_OK) return s;
  if (e != cudaSuccess) return fail(c, LEWM_CUDA_ERROR, "profile sync: %s", cudaGetErrorString(e));
  for (int k = 0; k < KC_COUNT; ++k) {
    ms_out[k] = 0;
    flops_out[k] = 0;
    launches_out[k] = 0;
  }
  for (const auto& r : c->prof.recs) {
    float ms = 0.f;
    cudaEventElapsedTime(&ms, r.a, r.b);
    ms_out[r.cls] += ms;
    flops_out[r.cls] += r.flops;
    launches_out[r.cls] += 1;
  }
  c->prof.reset();
  return LEWM_OK;
}

lewm_status lewm_coloring_matrix(int32_t n, double beta, double* out) {
  if (n <= 0 || !out || !(beta >= 0.0)) return fail(nullptr, LEWM_INVALID_ARG, "bad coloring_matrix arguments");
  if (beta <= 0.0 || n <= 1) {
    for (int i = 0; i < n * n; ++i) out[i] = (i / n == i % n) ? 1.0 : 0.0;
    return LEWM_OK;
  }
  coloring_matrix(n, beta, out);
  return LEWM_OK;
}

}  // extern "C"
