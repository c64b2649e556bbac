// fp32 precision mode of the model cost: the reference's float32 arithmetic
// (get_cost_from_embeddings without autocast, lewm/jepa.py:302-317) on CUDA cores.
//
// Same algorithm and data flow as the bf16 path (Embedder, AdaLN modulation for every
// token and layer, per call the window rows through the ConditionalBlocks, final
// LayerNorm, cost or history slot), but every operand and accumulator is float32: a
// tiled SIMT GEMM (no tensor cores, fixed K order) with fused epilogues, LayerNorms with
// two-pass moments, exact-erf GELU and expf-based SiLU / softmax. It exists for the
// reference's float32 exactness gate (tools/benchmarks/check_lewm_cache_exactness.py:
// 783-784) and its fp32 CEM configuration; the bf16 tensor-core path is the fast one.
#include <cmath>

#include "lewm_common.cuh"
#include "lewm_internal.h"

namespace lewm {
namespace {

constexpr int GB_M = 64, GB_N = 64, GB_K = 32, G_THREADS = 256;

enum GemmEpi { GE_BIAS = 0, GE_SILU = 1, GE_GELU = 2, GE_RESID = 3 };

__device__ __forceinline__ float gelu_erf(float x) { return 0.5f * x * (1.0f + erff(x * 0.70710678118654752f)); }

// C[M x N] = A[M x K] . W[N x K]^T + bias, then the epilogue:
//   GE_BIAS  C = acc + bias                  GE_SILU  C = silu(acc + bias)
//   GE_GELU  C = gelu(acc + bias)            GE_RESID X += gate . (acc + bias), in place,
//   gate = mod[row_tok[m] * mod_ld + gate_off + n]
// 64 x 64 output tile per CTA, 4 x 4 outputs per thread, K in slabs of 32 staged through
// shared memory (transposed, so the inner loop reads float4s). The next slab's global loads
// are issued into registers before the current slab's FMAs (one slab in flight: the kernel
// is bound by load latency at the planner's few hundred rows). VEC: 16-byte loads (K, lda
// multiples of 4 and 16-byte aligned A / W), else scalar loads. Every output sums its K
// products in increasing k, one fmaf each, whatever the grid.
template <int EPI, bool VEC>
__global__ void __launch_bounds__(G_THREADS) k_sgemm(const float* __restrict__ A, int lda, const float* __restrict__ W,
                                                     int K, const float* __restrict__ bias, float* __restrict__ C, int ldc,
                                                     int M, int N, const float* __restrict__ mod,
                                                     const int* __restrict__ row_tok, int mod_ld, int gate_off) {
  __shared__ __align__(16) float sA[GB_K][GB_M + 4];
  __shared__ __align__(16) float sW[GB_K][GB_N + 4];
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int m0 = blockIdx.y * GB_M, n0 = blockIdx.x * GB_N;
  // Per slab each thread moves 8 A values and 8 W values: VEC as 2 float4 (row s / 8,
  // k 4 (s % 8)), scalar as 8 floats (row s / 32, k s % 32), s = tid + 256 q.
  float ra[8], rw[8];
  auto load = [&](int k0) {
    if constexpr (VEC) {
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const int sl = tid + q * G_THREADS, r = sl >> 3, k = k0 + (sl & 7) * 4;
        const int m = m0 + r, n = n0 + r;
        float4 a = make_float4(0.f, 0.f, 0.f, 0.f), w = a;
        if (m < M && k < K) a = *reinterpret_cast<const float4*>(A + (size_t)m * lda + k);
        if (n < N && k < K) w = *reinterpret_cast<const float4*>(W + (size_t)n * K + k);
        ra[4 * q] = a.x, ra[4 * q + 1] = a.y, ra[4 * q + 2] = a.z, ra[4 * q + 3] = a.w;
        rw[4 * q] = w.x, rw[4 * q + 1] = w.y, rw[4 * q + 2] = w.z, rw[4 * q + 3] = w.w;
      }
    } else {
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const int sl = tid + q * G_THREADS, r = sl >> 5, k = k0 + (sl & 31);
        const int m = m0 + r, n = n0 + r;
        ra[q] = (m < M && k < K) ? A[(size_t)m * lda + k] : 0.f;
        rw[q] = (n < N && k < K) ? W[(size_t)n * K + k] : 0.f;
      }
    }
  };
  auto store = [&]() {
    if constexpr (VEC) {
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const int sl = tid + q * G_THREADS, r = sl >> 3, kk = (sl & 7) * 4;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          sA[kk + j][r] = ra[4 * q + j];
          sW[kk + j][r] = rw[4 * q + j];
        }
      }
    } else {
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const int sl = tid + q * G_THREADS, r = sl >> 5, kk = sl & 31;
        sA[kk][r] = ra[q];
        sW[kk][r] = rw[q];
      }
    }
  };
  float acc[4][4] = {};
  load(0);
  store();
  __syncthreads();
  for (int k0 = 0; k0 < K; k0 += GB_K) {
    const bool more = k0 + GB_K < K;
    if (more) load(k0 + GB_K);
#pragma unroll
    for (int kk = 0; kk < GB_K; ++kk) {
      const float4 a = *reinterpret_cast<const float4*>(&sA[kk][ty * 4]);
      const float4 b = *reinterpret_cast<const float4*>(&sW[kk][tx * 4]);
      const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    __syncthreads();
    if (more) {
      store();
      __syncthreads();
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int m = m0 + ty * 4 + i;
    if (m >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = n0 + tx * 4 + j;
      if (n >= N) continue;
      const float v = acc[i][j] + (bias ? bias[n] : 0.f);
      if constexpr (EPI == GE_BIAS) C[(size_t)m * ldc + n] = v;
      if constexpr (EPI == GE_SILU) C[(size_t)m * ldc + n] = v / (1.0f + expf(-v));
      if constexpr (EPI == GE_GELU) C[(size_t)m * ldc + n] = gelu_erf(v);
      if constexpr (EPI == GE_RESID) {
        const float gt = mod[(size_t)row_tok[m] * mod_ld + gate_off + n];
        C[(size_t)m * ldc + n] += gt * v;
      }
    }
  }
}

// One warp per row of `width` (<= 2048) floats: mean, then variance (two passes).
__device__ __forceinline__ float2 warp_moments(const float* row, int width) {
  float s = 0.f;
  for (int c = threadIdx.x & 31; c < width; c += 32) s += row[c];
  const float mean = warp_sum(s) / width;
  float q = 0.f;
  for (int c = threadIdx.x & 31; c < width; c += 32) {
    const float d = row[c] - mean;
    q += d * d;
  }
  return make_float2(mean, warp_sum(q) / width);
}

// out = LN_{g,b}(LN(x) * (1 + scale) + shift): AdaLN modulate (eps 1e-6, no affine) then the
// block's LayerNorm (eps 1e-5), width D; scratch h in `out` between the passes.
__global__ void __launch_bounds__(256) k_ln_mod32(const float* __restrict__ X, int rows, int D,
                                                  const int* __restrict__ row_tok, const float* __restrict__ mod,
                                                  int mod_ld, int shift_off, int scale_off, const float* __restrict__ g,
                                                  const float* __restrict__ b, float* __restrict__ out) {
  const int r = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (r >= rows) return;
  const float* x = X + (size_t)r * D;
  float* o = out + (size_t)r * D;
  const float* mrow = mod + (size_t)row_tok[r] * mod_ld;
  const float2 mv = warp_moments(x, D);
  const float rstd = 1.0f / sqrtf(mv.y + 1e-6f);
  for (int c = lane; c < D; c += 32) {
    const float y = (x[c] - mv.x) * rstd;
    o[c] = y * (1.0f + mrow[scale_off + c]) + mrow[shift_off + c];
  }
  __syncwarp();
  const float2 m2 = warp_moments(o, D);
  const float r2 = 1.0f / sqrtf(m2.y + 1e-5f);
  for (int c = lane; c < D; c += 32) o[c] = (o[c] - m2.x) * r2 * g[c] + b[c];
}

// In-place LayerNorm of `width`-wide rows (eps, optional affine), then optional GELU:
// the pred_proj head's LayerNorm over its hidden width.
__global__ void __launch_bounds__(256) k_row_ln32(float* __restrict__ X, int rows, int width, float eps,
                                                  const float* __restrict__ g, const float* __restrict__ b, int gelu) {
  const int r = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (r >= rows) return;
  float* x = X + (size_t)r * width;
  const float2 mv = warp_moments(x, width);
  const float rstd = 1.0f / sqrtf(mv.y + eps);
  for (int c = lane; c < width; c += 32) {
    float v = (x[c] - mv.x) * rstd;
    if (g) v = v * g[c] + b[c];
    x[c] = gelu ? gelu_erf(v) : v;
  }
}

// x = scale . x + shift per column, then GELU (the folded eval BatchNorm1d of a pred_proj head).
__global__ void k_col_affine_gelu32(float* __restrict__ X, size_t n, int width, const float* __restrict__ scale,
                                    const float* __restrict__ shift) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const int c = (int)(i % width);
    X[i] = gelu_erf(X[i] * scale[c] + shift[c]);
  }
}

// Causal window attention (scale 1/8, softmax over the window's positions <= the row's):
// one warp per (row, head), rows = candidate * w + position; qkv rows [3 * inner].
__global__ void __launch_bounds__(256) k_attn32(const float* __restrict__ qkv, int rows, int w, int heads,
                                                float* __restrict__ out) {
  const int item = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (item >= rows * heads) return;
  const int r = item / heads, h = item % heads;
  const int inner = heads * 64, pos = r % w, base = r - pos;
  const float* q = qkv + (size_t)r * 3 * inner + h * 64;
  float s[8];
  float mx = -INFINITY;
  for (int j = 0; j <= pos; ++j) {
    const float* k = qkv + (size_t)(base + j) * 3 * inner + inner + h * 64;
    const float d = warp_sum(q[lane] * k[lane] + q[32 + lane] * k[32 + lane]) * 0.125f;
    s[j] = d;
    mx = fmaxf(mx, d);
  }
  float den = 0.f;
  for (int j = 0; j <= pos; ++j) {
    s[j] = expf(s[j] - mx);
    den += s[j];
  }
  float o0 = 0.f, o1 = 0.f;
  for (int j = 0; j <= pos; ++j) {
    const float* v = qkv + (size_t)(base + j) * 3 * inner + 2 * inner + h * 64;
    o0 = fmaf(s[j], v[lane], o0);
    o1 = fmaf(s[j], v[32 + lane], o1);
  }
  float* dst = out + (size_t)r * inner + h * 64;
  dst[lane] = o0 / den;
  dst[32 + lane] = o1 / den;
}

// Layer-0 rows of one call: x[cand * w + p] = history entry (observation embedding or an
// earlier prediction) + position embedding p; row_tok = the token's modulation row.
__global__ void k_rows_init32(const float* __restrict__ emb, int emb_per_cand, const float* __restrict__ pred,
                              const float* __restrict__ pos, int n_cand, int S, int T, int H, int w, int start,
                              int npred, int D, float* __restrict__ X, int* __restrict__ row_tok) {
  const int r = blockIdx.x;
  if (r >= n_cand * w) return;
  const int cand = r / w, p = r % w, j = start + p;
  const float* src = j < H ? emb + ((size_t)(emb_per_cand ? cand : cand / S) * H + j) * D
                           : pred + ((size_t)cand * npred + (j - H)) * D;
  for (int c = threadIdx.x; c < D; c += blockDim.x) X[(size_t)r * D + c] = src[c] + pos[p * D + c];
  if (threadIdx.x == 0) row_tok[r] = cand * T + j;
}

// Final LayerNorm (eps 1e-5, affine) of each candidate's last window row, into y.
__global__ void __launch_bounds__(256) k_final_ln32(const float* __restrict__ X, int n_cand, int w, int D,
                                                    const float* __restrict__ g, const float* __restrict__ b,
                                                    float* __restrict__ y) {
  const int cand = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (cand >= n_cand) return;
  const float* x = X + ((size_t)cand * w + w - 1) * D;
  const float2 mv = warp_moments(x, D);
  const float rstd = 1.0f / sqrtf(mv.y + 1e-5f);
  for (int c = lane; c < D; c += 32) y[(size_t)cand * D + c] = (x[c] - mv.x) * rstd * g[c] + b[c];
}

// The call's prediction: history slot (earlier calls) or squared distance to the goal (last).
__global__ void __launch_bounds__(256) k_emit32(const float* __restrict__ y, int n_cand, int D, int last, int call,
                                                int npred, float* __restrict__ pred, const float* __restrict__ goal,
                                                int goal_per_cand, int S, float* __restrict__ costs) {
  const int cand = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (cand >= n_cand) return;
  const float* yr = y + (size_t)cand * D;
  if (!last) {
    for (int c = lane; c < D; c += 32) pred[((size_t)cand * npred + call) * D + c] = yr[c];
    return;
  }
  const float* gr = goal + (size_t)(goal_per_cand ? cand : cand / S) * D;
  float acc = 0.f;
  for (int c = lane; c < D; c += 32) {
    const float d = yr[c] - gr[c];
    acc += d * d;
  }
  acc = warp_sum(acc);
  if (lane == 0) costs[cand] = acc;
}

template <int EPI>
cudaError_t sgemm(const float* A, int lda, const float* W, int K, const float* bias, float* C, int ldc, int M, int N,
                  cudaStream_t st, const float* mod = nullptr, const int* row_tok = nullptr, int mod_ld = 0,
                  int gate_off = 0) {
  const dim3 grid((N + GB_N - 1) / GB_N, (M + GB_M - 1) / GB_M);
  const bool vec = K % 4 == 0 && lda % 4 == 0 && (reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(W)) % 16 == 0;
  if (vec)
    k_sgemm<EPI, true><<<grid, G_THREADS, 0, st>>>(A, lda, W, K, bias, C, ldc, M, N, mod, row_tok, mod_ld, gate_off);
  else
    k_sgemm<EPI, false><<<grid, G_THREADS, 0, st>>>(A, lda, W, K, bias, C, ldc, M, N, mod, row_tok, mod_ld, gate_off);
  return cudaGetLastError();
}

}  // namespace

#define F32_TRY(x)                            \
  do {                                        \
    const cudaError_t e_ = (x);               \
    if (e_ != cudaSuccess) return e_;         \
  } while (0)

cudaError_t run_model_cost_fp32(const ModelDims& m, const F32Weights& w, const F32Work& ws, const float* emb,
                                int emb_pc, int H, const float* goal, int goal_pc, const float* cand, int B, int S,
                                int T, int HS, float* costs, cudaStream_t st) {
  const int NC = B * S, NT = NC * T, D = m.D, L = m.L, inner = m.inner;
  const int mod_ld = L * 6 * D;
  // Embedder (lewm/module.py:189-214): Conv1d(k = 1) -> Linear -> SiLU -> Linear; the blocks
  // use SiLU(act_emb) (the first layer of adaLN_modulation), so that is what is kept.
  F32_TRY(sgemm<GE_BIAS>(cand, m.A, w.conv_w, m.A, w.conv_b, ws.act, m.As, NT, m.As, st));
  F32_TRY(sgemm<GE_SILU>(ws.act, m.As, w.e1_w, m.As, w.e1_b, ws.eh, m.eh, NT, m.eh, st));
  F32_TRY(sgemm<GE_SILU>(ws.eh, m.eh, w.e2_w, m.eh, w.e2_b, ws.sact, D, NT, D, st));
  for (int l = 0; l < L; ++l)  // AdaLN modulation of every token and layer
    F32_TRY(sgemm<GE_BIAS>(ws.sact, D, w.layers[l].ada_w, D, w.layers[l].ada_b, ws.mod + l * 6 * D, mod_ld, NT,
                           6 * D, st));
  const int n_calls = T - H + 1;
  for (int k = 0; k < n_calls; ++k) {
    const int end = H + k, start = end > HS ? end - HS : 0, wlen = end - start;
    const int rows = NC * wlen;
    k_rows_init32<<<rows, 64, 0, st>>>(emb, emb_pc, ws.pred, w.pos, NC, S, T, H, wlen, start, n_calls, D, ws.x,
                                       ws.row_tok);
    F32_TRY(cudaGetLastError());
    const int lnb = (rows + 7) / 8;
    for (int l = 0; l < L; ++l) {  // ConditionalBlock (lewm/module.py:88-111)
      const F32Layer& lw = w.layers[l];
      const int mo = l * 6 * D;  // shift_msa | scale_msa | gate_msa | shift_mlp | scale_mlp | gate_mlp
      k_ln_mod32<<<lnb, 256, 0, st>>>(ws.x, rows, D, ws.row_tok, ws.mod, mod_ld, mo, mo + D, lw.attn_ln_w,
                                      lw.attn_ln_b, ws.a);
      F32_TRY(sgemm<GE_BIAS>(ws.a, D, lw.qkv_w, D, nullptr, ws.qkv, 3 * inner, rows, 3 * inner, st));
      k_attn32<<<(rows * m.heads + 7) / 8, 256, 0, st>>>(ws.qkv, rows, wlen, m.heads, ws.att);
      F32_TRY(sgemm<GE_RESID>(ws.att, inner, lw.out_w, inner, lw.out_b, ws.x, D, rows, D, st, ws.mod, ws.row_tok,
                              mod_ld, mo + 2 * D));
      k_ln_mod32<<<lnb, 256, 0, st>>>(ws.x, rows, D, ws.row_tok, ws.mod, mod_ld, mo + 3 * D, mo + 4 * D, lw.ffn_ln_w,
                                      lw.ffn_ln_b, ws.a);
      F32_TRY(sgemm<GE_GELU>(ws.a, D, lw.w1, D, lw.b1, ws.hid, m.mlp, rows, m.mlp, st));
      F32_TRY(sgemm<GE_RESID>(ws.hid, m.mlp, lw.w2, m.mlp, lw.b2, ws.x, D, rows, D, st, ws.mod, ws.row_tok, mod_ld,
                              mo + 5 * D));
    }
    k_final_ln32<<<(NC + 7) / 8, 256, 0, st>>>(ws.x, NC, wlen, D, w.fin_w, w.fin_b, ws.y);
    F32_TRY(cudaGetLastError());
    if (m.pp_hidden) {  // pred_proj MLP head on the new predictions (lewm/jepa.py:106-114)
      const int P = m.pp_hidden;
      if (m.pp_norm == 1) {
        F32_TRY(sgemm<GE_BIAS>(ws.y, D, w.pp_w1, D, w.pp_b1, ws.pph, P, NC, P, st));
        k_row_ln32<<<(NC + 7) / 8, 256, 0, st>>>(ws.pph, NC, P, 1e-5f, w.pp_ln_g, w.pp_ln_b, 1);
      } else {
        F32_TRY(sgemm<GE_BIAS>(ws.y, D, w.pp_w1, D, nullptr, ws.pph, P, NC, P, st));
        k_col_affine_gelu32<<<1024, 256, 0, st>>>(ws.pph, (size_t)NC * P, P, w.pp_scale, w.pp_shift);
      }
      F32_TRY(cudaGetLastError());
      F32_TRY(sgemm<GE_BIAS>(ws.pph, P, w.pp_w2, P, w.pp_b2, ws.y, D, NC, D, st));
    }
    k_emit32<<<(NC + 7) / 8, 256, 0, st>>>(ws.y, NC, D, k == n_calls - 1 ? 1 : 0, k, n_calls, ws.pred, goal, goal_pc,
                                           S, costs);
    F32_TRY(cudaGetLastError());
  }
  return cudaSuccess;
}

}  // namespace lewm

namespace lewm {

namespace {
// The F32Work arrays in carve order (floats each, 16-float aligned).
template <class F>
void f32_layout(const ModelDims& m, size_t NC, size_t T, F&& f) {
  const size_t NT = NC * T, NW = NC * m.frames;
  auto al = [](size_t n) { return (n + 15) / 16 * 16; };
  f(0, al(NT * m.As));
  f(1, al(NT * m.eh));
  f(2, al(NT * m.D));
  f(3, al(NT * (size_t)m.L * 6 * m.D));
  f(4, al(NW * m.D));
  f(5, al(NW * m.D));
  f(6, al(NW * 3 * (size_t)m.inner));
  f(7, al(NW * m.inner));
  f(8, al(NW * m.mlp));
  f(9, al(NC * m.D));
  f(10, al(NC * T * m.D));
  f(11, al(NC * (size_t)m.pp_hidden));
  f(12, al(NW));  // row_tok (int32)
}
}  // namespace

size_t f32_work_floats(const ModelDims& m, size_t n_cand, size_t T) {
  size_t n = 0;
  f32_layout(m, n_cand, T, [&](int, size_t k) { n += k; });
  return n;
}

F32Work f32_work_carve(const ModelDims& m, size_t n_cand, size_t T, float* base) {
  float* p[13];
  size_t off = 0;
  f32_layout(m, n_cand, T, [&](int i, size_t k) {
    p[i] = base + off;
    off += k;
  });
  F32Work w{};
  w.act = p[0];
  w.eh = p[1];
  w.sact = p[2];
  w.mod = p[3];
  w.x = p[4];
  w.a = p[5];
  w.qkv = p[6];
  w.att = p[7];
  w.hid = p[8];
  w.y = p[9];
  w.pred = p[10];
  w.pph = p[11];
  w.row_tok = reinterpret_cast<int*>(p[12]);
  return w;
}

}  // namespace lewm
