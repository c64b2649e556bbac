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
#include <algorithm>
#include <cmath>

#include "lewm_common.cuh"
#include "lewm_internal.h"

#define F32_TRY(x)                            \
  do {                                        \
    const cudaError_t e_ = (x);               \
    if (e_ != cudaSuccess) return e_;         \
  } while (0)

namespace lewm {
namespace {
// Launch of a float32-path kernel. As a programmatic dependent launch (unless LEWM_NO_PDL=1 or
// LEWM_FP32_PDL=0) the grid is set up while the kernel before drains; every kernel waits for
// its predecessor (griddepcontrol.wait) before its first access and never triggers early, so
// the next grid's CTAs take no SM slots while this one runs.
bool fp32_pdl() {
  static const bool on = [] {
    const char* v = std::getenv("LEWM_FP32_PDL");
    return !(v && v[0] == '0');
  }();
  return on && pdl_enabled();
}
// 64 x 32 GEMM tiles where 64 x 64 ones number fewer than the SMs, 32 x 32 where 64 x 32 ones
// fill fewer than half of them (LEWM_FP32_NARROW=0: never; the same bits either way).
bool narrow_tiles() {
  static const bool on = [] {
    const char* v = std::getenv("LEWM_FP32_NARROW");
    return !(v && v[0] == '0');
  }();
  return on;
}
template <typename... KArgs, typename... Args>
cudaError_t launch_f32(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args&&... args) {
  if (fp32_pdl()) return launch_k(kern, grid, block, smem, st, std::forward<Args>(args)...);
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}
}  // namespace
}  // namespace lewm

namespace lewm {
namespace {

constexpr int GB_M = 64, GB_N = 64, GB_K = 32, G_THREADS = 256;
// K chunks of the gated-residual GEMMs (out-projection K = inner, FC2 K = mlp; N = D): their
// grids are N / 64 x rows / 64 CTAs, a few dozen at the planner's sizes, each walking K in
// dependent slabs. Always 4 chunks, whatever the batch, so a row's sum order (and bits) do
// not depend on the rows around it.
constexpr int kSplitK = 4;

enum GemmEpi { GE_BIAS = 0, GE_SILU = 1, GE_GELU = 2, GE_RESID = 3 };

// Column of element (k, r) in a transposed K slab [GB_K][rows + 4]: r XOR 4 ((k / 4) % 8).
// The loaders write 4 consecutive k of one row per thread and 8 threads per row, so without
// it a warp's 32 stores hit 8 banks (4-way conflicts); with it all 32 banks. The XOR keeps
// groups of 4 columns together, so the inner loop's float4 reads stay whole.
__device__ __forceinline__ int slab_col(int k, int r) { return r ^ (((k >> 2) & 7) << 2); }

__device__ __forceinline__ float gelu_erf(float x) { return 0.5f * x * (1.0f + erff(x * 0.70710678118654752f)); }

// C[M x N] = A[M x K] . W[N x K]^T + bias, then the epilogue:
//   GE_BIAS  C = acc + bias                  GE_SILU  C = silu(acc + bias)
//   GE_GELU  C = gelu(acc + bias)            GE_RESID X += gate . (acc + bias), in place,
//   gate = mod[row_tok[m] * mod_ld + gate_off + n]
// and, when `save` is set, save[m][n] = acc + bias (an [M][N] array) for the reverse pass.
// BM x BN output tile per CTA (64 x 64; 64 x 32 or 32 x 32 where larger tiles leave SMs idle),
// BM / 16 x BN / 16 outputs per thread, K in slabs of 32 staged through shared memory
// (transposed, so the inner loop reads float4s / float2s). The next slab's global loads are issued into registers
// before the current slab's FMAs (one slab in flight: the kernel is bound by load latency at
// the planner's few hundred rows). VEC: 16-byte loads (K, lda multiples of 4 and 16-byte
// aligned A / W), else scalar loads. Every output sums its K products in increasing k, one
// fmaf each, whatever the grid or the tile width.
template <int EPI, bool VEC, int BN = GB_N, int BM = GB_M>
__global__ void __launch_bounds__(G_THREADS) k_sgemm(const float* __restrict__ A, int lda, const float* __restrict__ W,
                                                     int K, const float* __restrict__ bias, float* __restrict__ C, int ldc,
                                                     int M, int N, const float* __restrict__ mod,
                                                     const int* __restrict__ row_tok, int mod_ld, int gate_off,
                                                     float* __restrict__ save, int kc, float* __restrict__ part) {
  static_assert((BN == 64 || BN == 32) && (BM == 64 || BM == 32), "tile shape");
  constexpr int TN = BN / 16;       // output columns per thread
  constexpr int TM = BM / 16;       // output rows per thread
  constexpr int WV = BN / 32;       // W float4 loads per thread and slab (VEC)
  constexpr int AV = BM / 32;       // A float4 loads per thread and slab (VEC)
  griddep_wait();  // launched as a programmatic dependent: wait for the kernel before
  __shared__ __align__(16) float sA[GB_K][BM + 4];
  __shared__ __align__(16) float sW[GB_K][BN + 4];
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  // K range of this CTA: all of K, or chunk blockIdx.z of kc (a multiple of GB_K) when split.
  const int kbeg = blockIdx.z * kc, kend = min(K, kbeg + kc);
  // Per slab each thread moves BM / 8 A values and BN / 8 W values: VEC as float4s (row s / 8,
  // k 4 (s % 8)), scalar as floats (row s / 32, k s % 32), s = tid + 256 q.
  float ra[BM / 8], rw[BN / 8];
  auto load = [&](int k0) {
    if constexpr (VEC) {
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const int sl = tid + q * G_THREADS, r = sl >> 3, k = k0 + (sl & 7) * 4;
        const int m = m0 + r, n = n0 + r;
        if (q < AV) {
          float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
          if (m < M && k < kend) a = *reinterpret_cast<const float4*>(A + (size_t)m * lda + k);
          ra[4 * q] = a.x, ra[4 * q + 1] = a.y, ra[4 * q + 2] = a.z, ra[4 * q + 3] = a.w;
        }
        if (q < WV) {
          float4 w = make_float4(0.f, 0.f, 0.f, 0.f);
          if (n < N && k < kend) w = *reinterpret_cast<const float4*>(W + (size_t)n * K + k);
          rw[4 * q] = w.x, rw[4 * q + 1] = w.y, rw[4 * q + 2] = w.z, rw[4 * q + 3] = w.w;
        }
      }
    } else {
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const int sl = tid + q * G_THREADS, r = sl >> 5, k = k0 + (sl & 31);
        const int m = m0 + r, n = n0 + r;
        if (q < BM / 8) ra[q] = (m < M && k < kend) ? A[(size_t)m * lda + k] : 0.f;
        if (q < BN / 8) rw[q] = (n < N && k < kend) ? W[(size_t)n * K + k] : 0.f;
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
          if (q < AV) sA[kk + j][slab_col(kk + j, r)] = ra[4 * q + j];
          if (q < WV) sW[kk + j][slab_col(kk + j, r)] = rw[4 * q + j];
        }
      }
    } else {
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const int sl = tid + q * G_THREADS, r = sl >> 5, kk = sl & 31;
        if (q < BM / 8) sA[kk][slab_col(kk, r)] = ra[q];
        if (q < BN / 8) sW[kk][slab_col(kk, r)] = rw[q];
      }
    }
  };
  float acc[TM][TN] = {};
  load(kbeg);
  store();
  __syncthreads();
  for (int k0 = kbeg; k0 < kend; k0 += GB_K) {
    const bool more = k0 + GB_K < kend;
    if (more) load(k0 + GB_K);
#pragma unroll
    for (int kk = 0; kk < GB_K; ++kk) {
      float av[TM], bv[TN];
      if constexpr (TM == 4) {
        const float4 a = *reinterpret_cast<const float4*>(&sA[kk][slab_col(kk, ty * 4)]);
        av[0] = a.x, av[1] = a.y, av[2] = a.z, av[3] = a.w;
      } else {
        const float2 a = *reinterpret_cast<const float2*>(&sA[kk][slab_col(kk, ty * 2)]);
        av[0] = a.x, av[1] = a.y;
      }
      if constexpr (TN == 4) {
        const float4 b = *reinterpret_cast<const float4*>(&sW[kk][slab_col(kk, tx * 4)]);
        bv[0] = b.x, bv[1] = b.y, bv[2] = b.z, bv[3] = b.w;
      } else {
        const float2 b = *reinterpret_cast<const float2*>(&sW[kk][slab_col(kk, tx * 2)]);
        bv[0] = b.x, bv[1] = b.y;
      }
#pragma unroll
      for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    __syncthreads();
    if (more) {
      store();
      __syncthreads();
    }
  }
#pragma unroll
  for (int i = 0; i < TM; ++i) {
    const int m = m0 + ty * TM + i;
    if (m >= M) continue;
#pragma unroll
    for (int j = 0; j < TN; ++j) {
      const int n = n0 + tx * TN + j;
      if (n >= N) continue;
      if (part) {  // split K: this chunk's raw sum; k_splitk_resid32 applies the epilogue
        part[((size_t)blockIdx.z * M + m) * N + n] = acc[i][j];
        continue;
      }
      const float v = acc[i][j] + (bias ? bias[n] : 0.f);
      if (save) save[(size_t)m * N + n] = v;  // pre-activation / branch output for the reverse pass
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
  griddep_wait();  // launched as a programmatic dependent: wait for the kernel before
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
  griddep_wait();  // launched as a programmatic dependent: wait for the kernel before
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
  griddep_wait();  // launched as a programmatic dependent: wait for the kernel before
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const int c = (int)(i % width);
    X[i] = gelu_erf(X[i] * scale[c] + shift[c]);
  }
}

// Causal window attention (scale 1/8, softmax over the window's positions <= the row's):
// one warp per (row, head); qkv rows [3 * inner]. A call runs rpc rows per candidate, the
// window positions pos0 .. pos0 + rpc - 1 (row = candidate * rpc + position - pos0); the
// keys / values of the positions before pos0 come from the cache kv [candidate][kv_pos]
// [k inner | v inner] of this layer (a growing-window call whose earlier positions the calls
// before ran with the same inputs).
__global__ void __launch_bounds__(256) k_attn32(const float* __restrict__ qkv, int rows, int rpc, int pos0, int heads,
                                                const float* __restrict__ kv, int kv_pos, float* __restrict__ out) {
  griddep_wait();  // launched as a programmatic dependent: wait for the kernel before
  const int item = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (item >= rows * heads) return;
  const int r = item / heads, h = item % heads;
  const int inner = heads * 64, cand = r / rpc, pos = pos0 + r % rpc, base = r - (pos - pos0);
  const float* q = qkv + (size_t)r * 3 * inner + h * 64;
  auto key = [&](int j) {
    return j < pos0 ? kv + ((size_t)cand * kv_pos + j) * 2 * inner + h * 64
                    : qkv + (size_t)(base + j - pos0) * 3 * inner + inner + h * 64;
  };
  auto val = [&](int j) {
    return j < pos0 ? kv + ((size_t)cand * kv_pos + j) * 2 * inner + inner + h * 64
                    : qkv + (size_t)(base + j - pos0) * 3 * inner + 2 * inner + h * 64;
  };
  float s[8];
  float mx = -INFINITY;
  for (int j = 0; j <= pos; ++j) {
    const float* k = key(j);
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
    const float* v = val(j);
    o0 = fmaf(s[j], v[lane], o0);
    o1 = fmaf(s[j], v[32 + lane], o1);
  }
  float* dst = out + (size_t)r * inner + h * 64;
  dst[lane] = o0 / den;
  dst[32 + lane] = o1 / den;
}

// The keys / values of this call's rows at window positions below kv_pos into the cache
// kv [candidate][kv_pos][k inner | v inner] (one block per row).
__global__ void k_kv_store32(const float* __restrict__ qkv, int rows, int rpc, int pos0, int inner, int kv_pos,
                             float* __restrict__ kv) {
  griddep_wait();  // launched as a programmatic dependent: wait for the kernel before
  const int r = blockIdx.x;
  if (r >= rows) return;
  const int cand = r / rpc, pos = pos0 + r % rpc;
  if (pos >= kv_pos) return;
  const float* src = qkv + (size_t)r * 3 * inner + inner;
  float* dst = kv + ((size_t)cand * kv_pos + pos) * 2 * inner;
  for (int c = threadIdx.x; c < 2 * inner; c += blockDim.x) dst[c] = src[c];
}

// Layer-0 rows of one call: x[cand * rpc + p - pos0] = history entry (observation embedding
// or an earlier prediction) + position embedding p for the window positions p = pos0 ..
// pos0 + rpc - 1 the call runs; row_tok = the token's modulation row.
__global__ void k_rows_init32(const float* __restrict__ emb, int emb_per_cand, const float* __restrict__ pred,
                              const float* __restrict__ pos, int n_cand, int S, int T, int H, int rpc, int pos0,
                              int start, int npred, int D, float* __restrict__ X, int* __restrict__ row_tok) {
  griddep_wait();  // launched as a programmatic dependent: wait for the kernel before
  const int r = blockIdx.x;
  if (r >= n_cand * rpc) return;
  const int cand = r / rpc, p = pos0 + r % rpc, j = start + p;
  const float* src = j < H ? emb + ((size_t)(emb_per_cand ? cand : cand / S) * H + j) * D
                           : pred + ((size_t)cand * npred + (j - H)) * D;
  for (int c = threadIdx.x; c < D; c += blockDim.x) X[(size_t)r * D + c] = src[c] + pos[p * D + c];
  if (threadIdx.x == 0) row_tok[r] = cand * T + j;
}

// Final LayerNorm (eps 1e-5, affine) of each candidate's last window row, into y.
__global__ void __launch_bounds__(256) k_final_ln32(const float* __restrict__ X, int n_cand, int w, int D,
                                                    const float* __restrict__ g, const float* __restrict__ b,
                                                    float* __restrict__ y) {
  griddep_wait();  // launched as a programmatic dependent: wait for the kernel before
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
  griddep_wait();  // launched as a programmatic dependent: wait for the kernel before
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

// The same GEMM as k_sgemm for the wide, many-row cases (QKV, AdaLN, FC1, the Embedder):
// 128 x 128 output tile per 256-thread CTA, 8 x 8 outputs per thread (half the shared-memory
// loads per FMA of the 4 x 4 tile), K in slabs of 32 with the next slab prefetched into
// registers. Each output still sums its K products in increasing k with one fmaf each, so
// the results are bit-identical to k_sgemm's; the launcher picks the tile by grid size only.
// Epilogues GE_BIAS / GE_SILU / GE_GELU (and `save`).
constexpr int GL_M = 128, GL_N = 128;

template <int EPI, bool VEC>
__global__ void __launch_bounds__(G_THREADS, 2) k_sgemm_wide(const float* __restrict__ A, int lda,
                                                          const float* __restrict__ W, int K,
                                                          const float* __restrict__ bias, float* __restrict__ C,
                                                          int ldc, int M, int N, float* __restrict__ save) {
  griddep_wait();  // launched as a programmatic dependent: wait for the kernel before
  __shared__ __align__(16) float sA[GB_K][GL_M + 4];
  __shared__ __align__(16) float sW[GB_K][GL_N + 4];
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int m0 = blockIdx.y * GL_M, n0 = blockIdx.x * GL_N;
  // Per slab each thread moves 16 A values and 16 W values: VEC as 4 float4 (row s / 8, k
  // 4 (s % 8)), scalar as 16 floats (row s / 32, k s % 32), s = tid + 256 q.
  float ra[16], rw[16];
  auto load = [&](int k0) {
    if constexpr (VEC) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
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
      for (int q = 0; q < 16; ++q) {
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
      for (int q = 0; q < 4; ++q) {
        const int sl = tid + q * G_THREADS, r = sl >> 3, kk = (sl & 7) * 4;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          sA[kk + j][r] = ra[4 * q + j];
          sW[kk + j][r] = rw[4 * q + j];
        }
      }
    } else {
#pragma unroll
      for (int q = 0; q < 16; ++q) {
        const int sl = tid + q * G_THREADS, r = sl >> 5, kk = sl & 31;
        sA[kk][r] = ra[q];
        sW[kk][r] = rw[q];
      }
    }
  };
  float acc[8][8] = {};
  load(0);
  store();
  __syncthreads();
  for (int k0 = 0; k0 < K; k0 += GB_K) {
    const bool more = k0 + GB_K < K;
    if (more) load(k0 + GB_K);
#pragma unroll
    for (int kk = 0; kk < GB_K; ++kk) {
      const float4 a0 = *reinterpret_cast<const float4*>(&sA[kk][ty * 8]);
      const float4 a1 = *reinterpret_cast<const float4*>(&sA[kk][ty * 8 + 4]);
      const float4 b0 = *reinterpret_cast<const float4*>(&sW[kk][tx * 8]);
      const float4 b1 = *reinterpret_cast<const float4*>(&sW[kk][tx * 8 + 4]);
      const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    __syncthreads();
    if (more) {
      store();
      __syncthreads();
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int m = m0 + ty * 8 + i;
    if (m >= M) continue;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int n = n0 + tx * 8 + j;
      if (n >= N) continue;
      const float v = acc[i][j] + (bias ? bias[n] : 0.f);
      if (save) save[(size_t)m * N + n] = v;
      if constexpr (EPI == GE_BIAS) C[(size_t)m * ldc + n] = v;
      if constexpr (EPI == GE_SILU) C[(size_t)m * ldc + n] = v / (1.0f + expf(-v));
      if constexpr (EPI == GE_GELU) C[(size_t)m * ldc + n] = gelu_erf(v);
    }
  }
}

// Split-K epilogue of the gated residual: v = bias + sum_z part[z] (z ascending), save = v,
// X += gate . v (one thread per output).
__global__ void k_splitk_resid32(const float* __restrict__ part, int splits, int M, int N,
                                 const float* __restrict__ bias, float* __restrict__ X, int ldc,
                                 const float* __restrict__ mod, const int* __restrict__ row_tok, int mod_ld,
                                 int gate_off, float* __restrict__ save) {
  griddep_wait();  // launched as a programmatic dependent: wait for the kernel before
  const size_t n_out = (size_t)M * N;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n_out; i += (size_t)gridDim.x * blockDim.x) {
    const int m = (int)(i / N), n = (int)(i % N);
    float v = part[i];
    for (int z = 1; z < splits; ++z) v += part[z * n_out + i];
    v += bias ? bias[n] : 0.f;
    if (save) save[i] = v;
    X[(size_t)m * ldc + n] += mod[(size_t)row_tok[m] * mod_ld + gate_off + n] * v;
  }
}

template <int EPI>
cudaError_t sgemm(const float* A, int lda, const float* W, int K, const float* bias, float* C, int ldc, int M, int N,
                  cudaStream_t st, const float* mod = nullptr, const int* row_tok = nullptr, int mod_ld = 0,
                  int gate_off = 0, float* save = nullptr, float* part = nullptr, int splits = 1) {
  if (EPI != GE_RESID || !part) splits = 1;  // split K only where k_splitk_resid32 finishes the epilogue
  if constexpr (EPI != GE_RESID) {
    // The 128 x 128 tile where it still fills the SMs (same bits as the 64 x 64 one).
    const dim3 wide((N + GL_N - 1) / GL_N, (M + GL_M - 1) / GL_M);
    if ((size_t)wide.x * wide.y >= 2 * 148) {
      const bool v = K % 4 == 0 && lda % 4 == 0 &&
                     (reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(W)) % 16 == 0;
      if (v)
        F32_TRY(launch_f32(k_sgemm_wide<EPI, true>, dim3(wide), dim3(G_THREADS), 0, st, A, lda, W, K, bias, C, ldc, M,
                         N, save));
      else
        F32_TRY(launch_f32(k_sgemm_wide<EPI, false>, dim3(wide), dim3(G_THREADS), 0, st, A, lda, W, K, bias, C, ldc, M,
                         N, save));
      return cudaGetLastError();
    }
  }
  const int kc = splits > 1 ? ((K + splits - 1) / splits + GB_K - 1) / GB_K * GB_K : K;
  const int nz = (K + kc - 1) / kc;
  const dim3 grid((N + GB_N - 1) / GB_N, (M + GB_M - 1) / GB_M, nz);
  float* pp = nz > 1 ? part : nullptr;
  const bool vec = K % 4 == 0 && lda % 4 == 0 && (reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(W)) % 16 == 0;
  const dim3 g6432((N + 31) / 32, grid.y, grid.z), g3232(g6432.x, (M + 31) / 32, grid.z);
  if (narrow_tiles() && (size_t)g6432.x * g6432.y * g6432.z < 74) {
    // 64 x 32 tiles would fill fewer than half the SMs: 32 x 32 tiles (same bits). At 120
    // tiles of 64 x 32 (FC1 and the residual GEMMs of 300 rows) 32 x 32 measured slower.
    if (vec)
      F32_TRY(launch_f32(k_sgemm<EPI, true, 32, 32>, g3232, dim3(G_THREADS), 0, st, A, lda, W, K, bias, C, ldc, M, N,
                         mod, row_tok, mod_ld, gate_off, save, kc, pp));
    else
      F32_TRY(launch_f32(k_sgemm<EPI, false, 32, 32>, g3232, dim3(G_THREADS), 0, st, A, lda, W, K, bias, C, ldc, M,
                         N, mod, row_tok, mod_ld, gate_off, save, kc, pp));
  } else if (narrow_tiles() && (size_t)grid.x * grid.y * grid.z < 148) {
    // Fewer 64 x 64 tiles than SMs: 64 x 32 tiles, twice the CTAs (same bits).
    if (vec)
      F32_TRY(launch_f32(k_sgemm<EPI, true, 32>, g6432, dim3(G_THREADS), 0, st, A, lda, W, K, bias, C, ldc, M, N, mod,
                         row_tok, mod_ld, gate_off, save, kc, pp));
    else
      F32_TRY(launch_f32(k_sgemm<EPI, false, 32>, g6432, dim3(G_THREADS), 0, st, A, lda, W, K, bias, C, ldc, M, N,
                         mod, row_tok, mod_ld, gate_off, save, kc, pp));
  } else if (vec)
    F32_TRY(launch_f32(k_sgemm<EPI, true>, dim3(grid), dim3(G_THREADS), 0, st, A, lda, W, K, bias, C, ldc, M, N, mod,
                     row_tok, mod_ld, gate_off, save, kc, pp));
  else
    F32_TRY(launch_f32(k_sgemm<EPI, false>, dim3(grid), dim3(G_THREADS), 0, st, A, lda, W, K, bias, C, ldc, M, N, mod,
                     row_tok, mod_ld, gate_off, save, kc, pp));
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess || !pp) return e;
  const size_t n_out = (size_t)M * N;
  const int blocks = (int)std::min<size_t>((n_out + 255) / 256, 148 * 16);
  F32_TRY(launch_f32(k_splitk_resid32, dim3(blocks), dim3(256), 0, st, pp, nz, M, N, bias, C, ldc, mod, row_tok,
                   mod_ld, gate_off, save));
  return cudaGetLastError();
}

}  // namespace

cudaError_t run_model_cost_fp32(const ModelDims& m, const F32Weights& w, const F32Work& ws, const float* emb,
                                int emb_pc, int H, const float* goal, int goal_pc, const float* cand, int B, int S,
                                int T, int HS, float* costs, cudaStream_t st, const F32Tape* tape) {
  const int NC = B * S, NT = NC * T, D = m.D, L = m.L, inner = m.inner;
  const int mod_ld = L * 6 * D;
  // Embedder (lewm/module.py:189-214): Conv1d(k = 1) -> Linear -> SiLU -> Linear; the blocks
  // use SiLU(act_emb) (the first layer of adaLN_modulation), so that is what is kept.
  F32_TRY(sgemm<GE_BIAS>(cand, m.A, w.conv_w, m.A, w.conv_b, ws.act, m.As, NT, m.As, st));
  F32_TRY(sgemm<GE_SILU>(ws.act, m.As, w.e1_w, m.As, w.e1_b, ws.eh, m.eh, NT, m.eh, st, nullptr, nullptr, 0, 0,
                         tape ? tape->h1 : nullptr));
  F32_TRY(sgemm<GE_SILU>(ws.eh, m.eh, w.e2_w, m.eh, w.e2_b, ws.sact, D, NT, D, st, nullptr, nullptr, 0, 0,
                         tape ? tape->e : nullptr));
  // AdaLN modulation of every token and layer: one GEMM over the stacked layer weights, whose
  // output rows are the [L * 6D] modulation rows
  F32_TRY(sgemm<GE_BIAS>(ws.sact, D, w.ada_stack, D, w.ada_b_stack, ws.mod, mod_ld, NT, mod_ld, st));
  const int n_calls = T - H + 1;
  // Growing-window key / value cache (no tape): while the window only grows, a call's
  // earlier positions have the inputs, and so the outputs, of the call before (causal
  // attention, fixed positions), so the call runs only its new last position and reads the
  // earlier keys / values from the cache the calls before wrote: the same bits as running
  // the whole window. The taped forward runs every window row (its reverse pass needs them).
  const int kv_pos = (!tape && H + 1 <= HS) ? HS - 1 : 0;
  for (int k = 0; k < n_calls; ++k) {
    const int end = H + k, start = end > HS ? end - HS : 0, wlen = end - start;
    const bool kv_read = kv_pos > 0 && k >= 1 && end <= HS;
    const bool kv_write = kv_pos > 0 && k + 1 < n_calls && end + 1 <= HS;
    const int rpc = kv_read ? 1 : wlen, pos0 = wlen - rpc;
    const int rows = NC * rpc;
    const F32TapeCall* tc = tape ? &tape->calls[k] : nullptr;
    int* row_tok = tc ? tc->row_tok : ws.row_tok;
    const size_t RD = (size_t)rows * D;
    F32_TRY(launch_f32(k_rows_init32, dim3(rows), dim3(64), 0, st, emb, emb_pc, ws.pred, w.pos, NC, S, T, H, rpc, pos0,
                     start, n_calls, D, ws.x, row_tok));
    const int lnb = (rows + 7) / 8;
    for (int l = 0; l < L; ++l) {  // ConditionalBlock (lewm/module.py:88-111)
      const F32Layer& lw = w.layers[l];
      const int mo = l * 6 * D;  // shift_msa | scale_msa | gate_msa | shift_mlp | scale_mlp | gate_mlp
      float* qkv = tc ? tc->qkv + (size_t)l * rows * 3 * inner : ws.qkv;
      if (tc) F32_TRY(cudaMemcpyAsync(tc->x_in + l * RD, ws.x, RD * 4, cudaMemcpyDeviceToDevice, st));
      F32_TRY(launch_f32(k_ln_mod32, dim3(lnb), dim3(256), 0, st, ws.x, rows, D, row_tok, ws.mod, mod_ld, mo, mo + D,
                       lw.attn_ln_w, lw.attn_ln_b, ws.a));
      F32_TRY(sgemm<GE_BIAS>(ws.a, D, lw.qkv_w, D, nullptr, qkv, 3 * inner, rows, 3 * inner, st));
      float* kv_l = ws.kv + (size_t)l * NC * kv_pos * 2 * inner;
      if (kv_write) {
        F32_TRY(launch_f32(k_kv_store32, dim3(rows), dim3(128), 0, st, qkv, rows, rpc, pos0, inner, kv_pos, kv_l));
      }
      F32_TRY(launch_f32(k_attn32, dim3((rows * m.heads + 7) / 8), dim3(256), 0, st, qkv, rows, rpc, pos0, m.heads,
                       kv_l, kv_pos, ws.att));
      F32_TRY(sgemm<GE_RESID>(ws.att, inner, lw.out_w, inner, lw.out_b, ws.x, D, rows, D, st, ws.mod, row_tok, mod_ld,
                              mo + 2 * D, tc ? tc->o + l * RD : nullptr, ws.part, kSplitK));
      if (tc) F32_TRY(cudaMemcpyAsync(tc->x_mid + l * RD, ws.x, RD * 4, cudaMemcpyDeviceToDevice, st));
      F32_TRY(launch_f32(k_ln_mod32, dim3(lnb), dim3(256), 0, st, ws.x, rows, D, row_tok, ws.mod, mod_ld, mo + 3 * D,
                       mo + 4 * D, lw.ffn_ln_w, lw.ffn_ln_b, ws.a));
      F32_TRY(sgemm<GE_GELU>(ws.a, D, lw.w1, D, lw.b1, ws.hid, m.mlp, rows, m.mlp, st, nullptr, nullptr, 0, 0,
                             tc ? tc->f1 + (size_t)l * rows * m.mlp : nullptr));
      F32_TRY(sgemm<GE_RESID>(ws.hid, m.mlp, lw.w2, m.mlp, lw.b2, ws.x, D, rows, D, st, ws.mod, row_tok, mod_ld,
                              mo + 5 * D, tc ? tc->f2 + l * RD : nullptr, ws.part, kSplitK));
    }
    if (tc) F32_TRY(cudaMemcpyAsync(tc->x_out, ws.x, RD * 4, cudaMemcpyDeviceToDevice, st));
    F32_TRY(launch_f32(k_final_ln32, dim3((NC + 7) / 8), dim3(256), 0, st, ws.x, NC, rpc, D, w.fin_w, w.fin_b, ws.y));
    if (m.pp_hidden) {  // pred_proj MLP head on the new predictions (lewm/jepa.py:106-114)
      const int P = m.pp_hidden;
      if (m.pp_norm == 1) {
        F32_TRY(sgemm<GE_BIAS>(ws.y, D, w.pp_w1, D, w.pp_b1, ws.pph, P, NC, P, st));
        F32_TRY(launch_f32(k_row_ln32, dim3((NC + 7) / 8), dim3(256), 0, st, ws.pph, NC, P, 1e-5f, w.pp_ln_g,
                         w.pp_ln_b, 1));
      } else {
        F32_TRY(sgemm<GE_BIAS>(ws.y, D, w.pp_w1, D, nullptr, ws.pph, P, NC, P, st));
        F32_TRY(launch_f32(k_col_affine_gelu32, dim3(1024), dim3(256), 0, st, ws.pph, (size_t)NC * P, P, w.pp_scale,
                         w.pp_shift));
      }
      F32_TRY(cudaGetLastError());
      F32_TRY(sgemm<GE_BIAS>(ws.pph, P, w.pp_w2, P, w.pp_b2, ws.y, D, NC, D, st));
    }
    F32_TRY(launch_f32(k_emit32, dim3((NC + 7) / 8), dim3(256), 0, st, ws.y, NC, D, k == n_calls - 1 ? 1 : 0, k,
                     n_calls, ws.pred, goal, goal_pc, S, costs));
    if (tape && k == n_calls - 1)
      F32_TRY(cudaMemcpyAsync(tape->y, ws.y, (size_t)NC * D * 4, cudaMemcpyDeviceToDevice, st));
  }
  return cudaSuccess;
}

}  // namespace lewm

namespace lewm {

// ------------------------------------------------------------------------------------------
// Reverse mode: d cost / d action candidates, the gradient CEM-GD steps on (reference
// lewm/solvers/cem_gd.py:459-606 takes torch autograd of get_cost_from_embeddings,
// lewm/jepa.py:302-317). Float32 throughout, over the activations the forward recorded.
namespace {

enum NnEpi { NE_STORE = 0, NE_GELU_BWD = 1, NE_SILU_BWD = 2 };

// d/dx of the exact GELU 0.5 x (1 + erf(x / sqrt 2)): Phi(x) + x phi(x).
__device__ __forceinline__ float gelu_erf_grad(float x) {
  const float cdf = 0.5f * (1.0f + erff(x * 0.70710678118654752f));
  return cdf + x * 0.39894228040143268f * expf(-0.5f * x * x);
}
// d/dx of x sigmoid(x): sigmoid(x) (1 + x (1 - sigmoid(x))).
__device__ __forceinline__ float silu_grad(float x) {
  const float sg = 1.0f / (1.0f + expf(-x));
  return sg * (1.0f + x * (1.0f - sg));
}

// C[M x Kout] = A[M x Nin] . Bm[Nin x Kout] (Bm row-major with row stride Kout: a Linear's
// [out][in] weight, so C = dY . W is the input gradient of y = x . W^T), then the epilogue:
// NE_STORE C = acc; NE_GELU_BWD / NE_SILU_BWD C = acc * f'(pre[m][c]). Same tiling, slab
// prefetch and fixed summation order as k_sgemm; VEC: 16-byte loads of A and Bm.
template <int EPI, bool VEC, int BN = GB_N, int BM = GB_M>
__global__ void __launch_bounds__(G_THREADS) k_sgemm_nn(const float* __restrict__ A, int lda, const float* __restrict__ Bm,
                                                        int Nin, int Kout, float* __restrict__ C, int ldc, int M,
                                                        const float* __restrict__ pre, int ldp, int kc,
                                                        float* __restrict__ part) {
  static_assert((BN == 64 || BN == 32) && (BM == 64 || BM == 32), "tile shape");
  constexpr int TN = BN / 16, TM = BM / 16;  // outputs per thread
  constexpr int AV = BM / 32, BV = BN / 32;  // float4 loads per thread and slab (VEC)
  constexpr int BQ = BN / 4;                 // float4s per Bm row of the tile
  griddep_wait();  // launched as a programmatic dependent: wait for the kernel before
  __shared__ __align__(16) float sA[GB_K][BM + 4];
  __shared__ __align__(16) float sB[GB_K][BN + 4];
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int m0 = blockIdx.y * BM, c0 = blockIdx.x * BN;
  const int nbeg = blockIdx.z * kc, nend = min(Nin, nbeg + kc);  // reduction chunk of this CTA
  float ra[BM / 8], rb[BN / 8];
  auto load = [&](int n0) {
    if constexpr (VEC) {
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const int sl = tid + q * G_THREADS;
        if (q < AV) {
          const int r = sl >> 3, n = n0 + (sl & 7) * 4, m = m0 + r;
          float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
          if (m < M && n < nend) a = *reinterpret_cast<const float4*>(A + (size_t)m * lda + n);
          ra[4 * q] = a.x, ra[4 * q + 1] = a.y, ra[4 * q + 2] = a.z, ra[4 * q + 3] = a.w;
        }
        if (q < BV) {
          const int rr = sl / BQ, c = c0 + (sl % BQ) * 4, nb = n0 + rr;
          float4 b = make_float4(0.f, 0.f, 0.f, 0.f);
          if (nb < nend && c < Kout) b = *reinterpret_cast<const float4*>(Bm + (size_t)nb * Kout + c);
          rb[4 * q] = b.x, rb[4 * q + 1] = b.y, rb[4 * q + 2] = b.z, rb[4 * q + 3] = b.w;
        }
      }
    } else {
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const int sl = tid + q * G_THREADS;
        if (q < BM / 8) {
          const int r = sl >> 5, n = n0 + (sl & 31), m = m0 + r;
          ra[q] = (m < M && n < nend) ? A[(size_t)m * lda + n] : 0.f;
        }
        if (q < BN / 8) {
          const int rr = sl / BN, c = c0 + (sl % BN), nb = n0 + rr;
          rb[q] = (nb < nend && c < Kout) ? Bm[(size_t)nb * Kout + c] : 0.f;
        }
      }
    }
  };
  auto store = [&]() {
    if constexpr (VEC) {
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const int sl = tid + q * G_THREADS;
        if (q < AV) {
          const int r = sl >> 3, kk = (sl & 7) * 4;
#pragma unroll
          for (int j = 0; j < 4; ++j) sA[kk + j][slab_col(kk + j, r)] = ra[4 * q + j];
        }
        if (q < BV)
          *reinterpret_cast<float4*>(&sB[sl / BQ][(sl % BQ) * 4]) =
              make_float4(rb[4 * q], rb[4 * q + 1], rb[4 * q + 2], rb[4 * q + 3]);
      }
    } else {
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const int sl = tid + q * G_THREADS;
        if (q < BM / 8) sA[sl & 31][slab_col(sl & 31, sl >> 5)] = ra[q];
        if (q < BN / 8) sB[sl / BN][sl % BN] = rb[q];
      }
    }
  };
  float acc[TM][TN] = {};
  load(nbeg);
  store();
  __syncthreads();
  for (int n0 = nbeg; n0 < nend; n0 += GB_K) {
    const bool more = n0 + GB_K < nend;
    if (more) load(n0 + GB_K);
#pragma unroll
    for (int kk = 0; kk < GB_K; ++kk) {
      float av[TM], bv[TN];
      if constexpr (TM == 4) {
        const float4 a = *reinterpret_cast<const float4*>(&sA[kk][slab_col(kk, ty * 4)]);
        av[0] = a.x, av[1] = a.y, av[2] = a.z, av[3] = a.w;
      } else {
        const float2 a = *reinterpret_cast<const float2*>(&sA[kk][slab_col(kk, ty * 2)]);
        av[0] = a.x, av[1] = a.y;
      }
      if constexpr (TN == 4) {
        const float4 b = *reinterpret_cast<const float4*>(&sB[kk][tx * 4]);
        bv[0] = b.x, bv[1] = b.y, bv[2] = b.z, bv[3] = b.w;
      } else {
        const float2 b = *reinterpret_cast<const float2*>(&sB[kk][tx * 2]);
        bv[0] = b.x, bv[1] = b.y;
      }
#pragma unroll
      for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    __syncthreads();
    if (more) {
      store();
      __syncthreads();
    }
  }
#pragma unroll
  for (int i = 0; i < TM; ++i) {
    const int m = m0 + ty * TM + i;
    if (m >= M) continue;
#pragma unroll
    for (int j = 0; j < TN; ++j) {
      const int c = c0 + tx * TN + j;
      if (c >= Kout) continue;
      if (part) {  // split reduction: this chunk's raw sum; k_splitk_nn32 finishes
        part[((size_t)blockIdx.z * M + m) * Kout + c] = acc[i][j];
        continue;
      }
      float v = acc[i][j];
      if constexpr (EPI == NE_GELU_BWD) v *= gelu_erf_grad(pre[(size_t)m * ldp + c]);
      if constexpr (EPI == NE_SILU_BWD) v *= silu_grad(pre[(size_t)m * ldp + c]);
      C[(size_t)m * ldc + c] = v;
    }
  }
}

// Split-reduction epilogue of k_sgemm_nn: v = sum_z part[z] (z ascending), then the epilogue.
template <int EPI>
__global__ void k_splitk_nn32(const float* __restrict__ part, int splits, int M, int Kout, float* __restrict__ C,
                              int ldc, const float* __restrict__ pre, int ldp) {
  griddep_wait();  // launched as a programmatic dependent: wait for the kernel before
  const size_t n_out = (size_t)M * Kout;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n_out; i += (size_t)gridDim.x * blockDim.x) {
    const int m = (int)(i / Kout), c = (int)(i % Kout);
    float v = part[i];
    for (int z = 1; z < splits; ++z) v += part[z * n_out + i];
    if constexpr (EPI == NE_GELU_BWD) v *= gelu_erf_grad(pre[(size_t)m * ldp + c]);
    if constexpr (EPI == NE_SILU_BWD) v *= silu_grad(pre[(size_t)m * ldp + c]);
    C[(size_t)m * ldc + c] = v;
  }
}

// Reduction chunks of dY . W as a function of the reduction length alone (one chunk per 256,
// at most kMaxNnSplits), so a row's sum order does not depend on the batch: the long
// reductions (3 inner, the stacked adaLN 6 D L, mlp) would otherwise walk 24-216 dependent
// slabs in a few CTAs.
constexpr int kMaxNnSplits = 16;
int nn_splits(int Nin) { return std::max(1, std::min(kMaxNnSplits, Nin / 256)); }

template <int EPI>
cudaError_t sgemm_nn(const float* A, int lda, const float* Bm, int Nin, int Kout, float* C, int ldc, int M,
                     cudaStream_t st, const F32GradWork& gw, const float* pre = nullptr, int ldp = 0) {
  const int splits = nn_splits(Nin);
  const int kc = ((Nin + splits - 1) / splits + GB_K - 1) / GB_K * GB_K;
  const int nz = (Nin + kc - 1) / kc;
  // The partials must fit gw.part; the reductions it is sized for always do (output width D).
  if (nz > 1 && (size_t)nz * M * Kout > gw.part_floats) return cudaErrorInvalidValue;
  float* pp = nz > 1 ? gw.part : nullptr;
  const dim3 grid((Kout + GB_N - 1) / GB_N, (M + GB_M - 1) / GB_M, nz);
  const bool vec = Nin % 4 == 0 && lda % 4 == 0 && Kout % 4 == 0 &&
                   (reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(Bm)) % 16 == 0;
  // Narrower tiles on grids that leave SMs idle, as in sgemm (same bits).
  const dim3 g6432((Kout + 31) / 32, grid.y, nz), g3232(g6432.x, (M + 31) / 32, nz);
  if (narrow_tiles() && (size_t)g6432.x * g6432.y * g6432.z < 74) {
    if (vec)
      F32_TRY(launch_f32(k_sgemm_nn<EPI, true, 32, 32>, g3232, dim3(G_THREADS), 0, st, A, lda, Bm, Nin, Kout, C, ldc,
                         M, pre, ldp, kc, pp));
    else
      F32_TRY(launch_f32(k_sgemm_nn<EPI, false, 32, 32>, g3232, dim3(G_THREADS), 0, st, A, lda, Bm, Nin, Kout, C,
                         ldc, M, pre, ldp, kc, pp));
  } else if (narrow_tiles() && (size_t)grid.x * grid.y * grid.z < 148) {
    if (vec)
      F32_TRY(launch_f32(k_sgemm_nn<EPI, true, 32>, g6432, dim3(G_THREADS), 0, st, A, lda, Bm, Nin, Kout, C, ldc, M,
                         pre, ldp, kc, pp));
    else
      F32_TRY(launch_f32(k_sgemm_nn<EPI, false, 32>, g6432, dim3(G_THREADS), 0, st, A, lda, Bm, Nin, Kout, C, ldc,
                         M, pre, ldp, kc, pp));
  } else if (vec)
    F32_TRY(launch_f32(k_sgemm_nn<EPI, true>, dim3(grid), dim3(G_THREADS), 0, st, A, lda, Bm, Nin, Kout, C, ldc, M,
                     pre, ldp, kc, pp));
  else
    F32_TRY(launch_f32(k_sgemm_nn<EPI, false>, dim3(grid), dim3(G_THREADS), 0, st, A, lda, Bm, Nin, Kout, C, ldc, M,
                     pre, ldp, kc, pp));
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess || !pp) return e;
  const size_t n_out = (size_t)M * Kout;
  const int blocks = (int)std::min<size_t>((n_out + 255) / 256, 148 * 16);
  F32_TRY(launch_f32(k_splitk_nn32<EPI>, dim3(blocks), dim3(256), 0, st, pp, nz, M, Kout, C, ldc, pre, ldp));
  return cudaGetLastError();
}

// dY[c] = 2 (y[c] - goal) * weight[c]: d of weight . sum_d (y - goal)^2 (lewm/jepa.py:246-260).
__global__ void __launch_bounds__(256) k_seed32(const float* __restrict__ y, const float* __restrict__ goal,
                                                int goal_per_cand, int S, const float* __restrict__ weights,
                                                int n_cand, int D, float* __restrict__ dY) {
  griddep_wait();  // launched as a programmatic dependent: wait for the kernel before
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n_cand * D) return;
  const int cand = i / D, c = i % D;
  const float g = goal[(size_t)(goal_per_cand ? cand : cand / S) * D + c];
  dY[i] = 2.0f * (y[i] - g) * (weights ? weights[cand] : 1.0f);
}

// Final LayerNorm (affine, eps 1e-5) of each candidate's last window row: dX[last row] =
// LN backward of dy (row stride dy_ld); the other rows of dX stay as they are (zero).
__global__ void __launch_bounds__(256) k_final_ln_bwd32(const float* __restrict__ X, int n_cand, int w, int D,
                                                        const float* __restrict__ g, const float* __restrict__ dy,
                                                        int dy_ld, float* __restrict__ dX) {
  griddep_wait();  // launched as a programmatic dependent: wait for the kernel before
  const int cand = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (cand >= n_cand) return;
  const size_t row = (size_t)cand * w + w - 1;
  const float* x = X + row * D;
  const float2 mv = warp_moments(x, D);
  const float rstd = 1.0f / sqrtf(mv.y + 1e-5f);
  const float* d = dy + (size_t)cand * dy_ld;
  float sa = 0.f, sb = 0.f;
  for (int c = lane; c < D; c += 32) {
    const float dh = d[c] * g[c], xh = (x[c] - mv.x) * rstd;
    sa += dh;
    sb += dh * xh;
  }
  sa = warp_sum(sa) / D;
  sb = warp_sum(sb) / D;
  for (int c = lane; c < D; c += 32) {
    const float dh = d[c] * g[c], xh = (x[c] - mv.x) * rstd;
    dX[row * D + c] = rstd * (dh - sa - xh * sb);
  }
}

// Gated residual x += gate . F: dF = dX . gate and dmod[token][gate] += dX . F. A call's rows
// hold distinct tokens, so no two threads of a launch touch one dmod element.
__global__ void k_gate_bwd32(const float* __restrict__ dX, const float* __restrict__ F, const int* __restrict__ row_tok,
                             const float* __restrict__ mod, float* __restrict__ dmod, int mod_ld, int gate_off,
                             int rows, int D, float* __restrict__ dF) {
  griddep_wait();  // launched as a programmatic dependent: wait for the kernel before
  const size_t n = (size_t)rows * D;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const int r = (int)(i / D), c = (int)(i % D);
    const size_t mi = (size_t)row_tok[r] * mod_ld + gate_off + c;
    const float dx = dX[i];
    dF[i] = dx * mod[mi];
    dmod[mi] += dx * F[i];
  }
}

// Reverse of a = LN_{g,b}(LN(x) (1 + scale) + shift) (k_ln_mod32): from dA, recompute u = LN(x)
// and h, then dmod[shift] += dh, dmod[scale] += dh . u and dX += LN backward of dh . (1 + scale).
// One warp per row, NV = D / 32 values per lane.
template <int NV>
__global__ void __launch_bounds__(256) k_ln_mod_bwd32(const float* __restrict__ X, const float* __restrict__ dA,
                                                      int rows, const int* __restrict__ row_tok,
                                                      const float* __restrict__ mod, float* __restrict__ dmod,
                                                      int mod_ld, int shift_off, int scale_off,
                                                      const float* __restrict__ g, float* __restrict__ dX) {
  griddep_wait();  // launched as a programmatic dependent: wait for the kernel before
  constexpr int D = NV * 32;
  const int r = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (r >= rows) return;
  const float* x = X + (size_t)r * D;
  const size_t mrow = (size_t)row_tok[r] * mod_ld;
  const float2 mv = warp_moments(x, D);
  const float rstd1 = 1.0f / sqrtf(mv.y + 1e-6f);
  float u[NV], h[NV], sc[NV];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = lane + 32 * i;
    u[i] = (x[c] - mv.x) * rstd1;
    sc[i] = mod[mrow + scale_off + c];
    h[i] = u[i] * (1.0f + sc[i]) + mod[mrow + shift_off + c];
    s += h[i];
  }
  const float mean2 = warp_sum(s) / D;
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) q += (h[i] - mean2) * (h[i] - mean2);
  const float rstd2 = 1.0f / sqrtf(warp_sum(q) / D + 1e-5f);
  float sa = 0.f, sb = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = lane + 32 * i;
    const float ah = (h[i] - mean2) * rstd2, dah = dA[(size_t)r * D + c] * g[c];
    h[i] = ah;  // h now holds the normalised h
    sa += dah;
    sb += dah * ah;
  }
  sa = warp_sum(sa) / D;
  sb = warp_sum(sb) / D;
  float ta = 0.f, tb = 0.f;
  float du[NV];
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = lane + 32 * i;
    const float dah = dA[(size_t)r * D + c] * g[c];
    const float dh = rstd2 * (dah - sa - h[i] * sb);
    dmod[mrow + shift_off + c] += dh;
    dmod[mrow + scale_off + c] += dh * u[i];
    du[i] = dh * (1.0f + sc[i]);
    ta += du[i];
    tb += du[i] * u[i];
  }
  ta = warp_sum(ta) / D;
  tb = warp_sum(tb) / D;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = lane + 32 * i;
    dX[(size_t)r * D + c] += rstd1 * (du[i] - ta - u[i] * tb);
  }
}

// Reverse of the causal window attention (k_attn32): one warp per (candidate, head) walks
// the candidate's w rows, recomputes each row's softmax P and accumulates
// dq = 1/8 sum_j dS_j k_j, dk_j += 1/8 dS_j q, dv_j += P_j dO with dS_j = P_j (dP_j - sum P dP).
__global__ void __launch_bounds__(256) k_attn_bwd32(const float* __restrict__ qkv, const float* __restrict__ dO,
                                                    int n_cand, int w, int heads, float* __restrict__ dQKV) {
  griddep_wait();  // launched as a programmatic dependent: wait for the kernel before
  const int item = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (item >= n_cand * heads) return;
  const int cand = item / heads, hd = item % heads, inner = heads * 64, ld = 3 * inner;
  const size_t base = (size_t)cand * w;
  float dk0[8], dk1[8], dv0[8], dv1[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) dk0[j] = dk1[j] = dv0[j] = dv1[j] = 0.f;
  for (int p = 0; p < w; ++p) {
    const float* q = qkv + (base + p) * ld + hd * 64;
    const float q0 = q[lane], q1 = q[32 + lane];
    float P[8], dP[8];
    float mx = -INFINITY;
    for (int j = 0; j <= p; ++j) {
      const float* k = qkv + (base + j) * ld + inner + hd * 64;
      P[j] = warp_sum(q0 * k[lane] + q1 * k[32 + lane]) * 0.125f;
      mx = fmaxf(mx, P[j]);
    }
    float den = 0.f;
    for (int j = 0; j <= p; ++j) {
      P[j] = expf(P[j] - mx);
      den += P[j];
    }
    const float* o = dO + (base + p) * inner + hd * 64;
    const float o0 = o[lane], o1 = o[32 + lane];
    float spd = 0.f;
    for (int j = 0; j <= p; ++j) {
      P[j] /= den;
      const float* v = qkv + (base + j) * ld + 2 * inner + hd * 64;
      dP[j] = warp_sum(o0 * v[lane] + o1 * v[32 + lane]);
      spd += P[j] * dP[j];
    }
    float dq0 = 0.f, dq1 = 0.f;
    for (int j = 0; j <= p; ++j) {
      const float* k = qkv + (base + j) * ld + inner + hd * 64;
      const float ds = P[j] * (dP[j] - spd) * 0.125f;
      dq0 = fmaf(ds, k[lane], dq0);
      dq1 = fmaf(ds, k[32 + lane], dq1);
#pragma unroll
      for (int jj = 0; jj < 8; ++jj)
        if (jj == j) {  // register-resident accumulators: static indices only
          dk0[jj] = fmaf(ds, q0, dk0[jj]);
          dk1[jj] = fmaf(ds, q1, dk1[jj]);
          dv0[jj] = fmaf(P[j], o0, dv0[jj]);
          dv1[jj] = fmaf(P[j], o1, dv1[jj]);
        }
    }
    float* dq = dQKV + (base + p) * ld + hd * 64;
    dq[lane] = dq0;
    dq[32 + lane] = dq1;
  }
#pragma unroll
  for (int j = 0; j < 8; ++j)
    if (j < w) {
      float* d = dQKV + (base + j) * ld + hd * 64;
      d[inner + lane] = dk0[j];
      d[inner + 32 + lane] = dk1[j];
      d[2 * inner + lane] = dv0[j];
      d[2 * inner + 32 + lane] = dv1[j];
    }
}

// Layer-0 rows were history + position: rows holding an earlier prediction (history index
// j >= H) pass their gradient to that prediction, dpred[cand][j - H] += dX[row].
__global__ void k_hist_bwd32(const float* __restrict__ dX, int n_cand, int w, int start, int H, int npred, int D,
                             float* __restrict__ dpred) {
  griddep_wait();  // launched as a programmatic dependent: wait for the kernel before
  const int r = blockIdx.x;
  if (r >= n_cand * w) return;
  const int cand = r / w, j = start + r % w;
  if (j < H) return;
  float* dst = dpred + ((size_t)cand * npred + (j - H)) * D;
  for (int c = threadIdx.x; c < D; c += blockDim.x) dst[c] += dX[(size_t)r * D + c];
}

cudaError_t ln_mod_bwd(int D, const float* X, const float* dA, int rows, const int* row_tok, const float* mod,
                       float* dmod, int mod_ld, int shift_off, int scale_off, const float* g, float* dX,
                       cudaStream_t st) {
  const int blocks = (rows + 7) / 8;
  if (D == 192)
    F32_TRY(launch_f32(k_ln_mod_bwd32<6>, dim3(blocks), dim3(256), 0, st, X, dA, rows, row_tok, mod, dmod, mod_ld,
                     shift_off, scale_off, g, dX));
  else if (D == 384)
    F32_TRY(launch_f32(k_ln_mod_bwd32<12>, dim3(blocks), dim3(256), 0, st, X, dA, rows, row_tok, mod, dmod, mod_ld,
                     shift_off, scale_off, g, dX));
  else
    return cudaErrorInvalidValue;
  return cudaGetLastError();
}

int ew_blocks(size_t n) { return (int)std::min<size_t>((n + 255) / 256, 148 * 16); }

}  // namespace

cudaError_t run_model_cost_grad_fp32(const ModelDims& m, const F32Weights& w, const F32Work& ws, const F32Tape& tape,
                                     const F32GradWork& gw, const float* emb, int emb_pc, int H, const float* goal,
                                     int goal_pc, const float* cand, int B, int S, int T, int HS,
                                     const float* cost_weights, float* costs, float* grad, cudaStream_t st) {
  if (m.pp_hidden) return cudaErrorInvalidValue;  // the reverse pass covers an Identity pred_proj
  const int NC = B * S, NT = NC * T, D = m.D, L = m.L, inner = m.inner, mlp = m.mlp;
  const int mod_ld = L * 6 * D, n_calls = T - H + 1;
  F32_TRY(run_model_cost_fp32(m, w, ws, emb, emb_pc, H, goal, goal_pc, cand, B, S, T, HS, costs, st, &tape));
  F32_TRY(cudaMemsetAsync(gw.dmod, 0, (size_t)NT * mod_ld * 4, st));
  F32_TRY(cudaMemsetAsync(gw.dpred, 0, (size_t)NC * n_calls * D * 4, st));
  F32_TRY(launch_f32(k_seed32, dim3((NC * D + 255) / 256), dim3(256), 0, st, tape.y, goal, goal_pc, S, cost_weights,
                   NC, D, gw.dY));
  for (int k = n_calls - 1; k >= 0; --k) {  // calls in reverse: later windows read earlier predictions
    const F32TapeCall& tc = tape.calls[k];
    const int R = tc.rows;
    const size_t RD = (size_t)R * D;
    F32_TRY(cudaMemsetAsync(gw.dX, 0, RD * 4, st));
    const bool last = k == n_calls - 1;
    F32_TRY(launch_f32(k_final_ln_bwd32, dim3((NC + 7) / 8), dim3(256), 0, st, tc.x_out, NC, tc.w, D, w.fin_w,
                     last ? gw.dY : gw.dpred + (size_t)k * D, last ? D : n_calls * D, gw.dX));
    for (int l = L - 1; l >= 0; --l) {
      const F32Layer& lw = w.layers[l];
      const int mo = l * 6 * D;
      // x += gate_mlp . FFN(a2): FFN(a2) = GELU(a2 W1^T + b1) W2^T + b2
      F32_TRY(launch_f32(k_gate_bwd32, dim3(ew_blocks(RD)), dim3(256), 0, st, gw.dX, tc.f2 + l * RD, tc.row_tok,
                       ws.mod, gw.dmod, mod_ld, mo + 5 * D, R, D, gw.dF));
      F32_TRY(sgemm_nn<NE_GELU_BWD>(gw.dF, D, lw.w2, D, mlp, gw.dF1, mlp, R, st, gw, tc.f1 + (size_t)l * R * mlp,
                                    mlp));
      F32_TRY(sgemm_nn<NE_STORE>(gw.dF1, mlp, lw.w1, mlp, D, gw.dA, D, R, st, gw));
      F32_TRY(ln_mod_bwd(D, tc.x_mid + l * RD, gw.dA, R, tc.row_tok, ws.mod, gw.dmod, mod_ld, mo + 3 * D, mo + 4 * D,
                         lw.ffn_ln_w, gw.dX, st));
      // x += gate_msa . (attention(a) W_out^T + b_out), attention over q | k | v = a W_qkv^T
      F32_TRY(launch_f32(k_gate_bwd32, dim3(ew_blocks(RD)), dim3(256), 0, st, gw.dX, tc.o + l * RD, tc.row_tok, ws.mod,
                       gw.dmod, mod_ld, mo + 2 * D, R, D, gw.dF));
      F32_TRY(sgemm_nn<NE_STORE>(gw.dF, D, lw.out_w, D, inner, gw.dAtt, inner, R, st, gw));
      F32_TRY(launch_f32(k_attn_bwd32, dim3((NC * m.heads + 7) / 8), dim3(256), 0, st,
                       tc.qkv + (size_t)l * R * 3 * inner, gw.dAtt, NC, tc.w, m.heads, gw.dQKV));
      F32_TRY(sgemm_nn<NE_STORE>(gw.dQKV, 3 * inner, lw.qkv_w, 3 * inner, D, gw.dA, D, R, st, gw));
      F32_TRY(ln_mod_bwd(D, tc.x_in + l * RD, gw.dA, R, tc.row_tok, ws.mod, gw.dmod, mod_ld, mo, mo + D,
                         lw.attn_ln_w, gw.dX, st));
    }
    F32_TRY(launch_f32(k_hist_bwd32, dim3(R), dim3(64), 0, st, gw.dX, NC, tc.w, tc.start, H, n_calls, D, gw.dpred));
  }
  // mod = SiLU(e) W_ada^T + b_ada for every layer; e = SiLU(h1) W_e2^T + b_e2; h1 = a1 W_e1^T + b_e1;
  // a1 = cand W_conv^T + b_conv (Embedder, lewm/module.py:205-214).
  F32_TRY(sgemm_nn<NE_SILU_BWD>(gw.dmod, mod_ld, w.ada_stack, mod_ld, D, gw.de, D, NT, st, gw, tape.e, D));
  F32_TRY(sgemm_nn<NE_SILU_BWD>(gw.de, D, w.e2_w, D, m.eh, gw.dh1, m.eh, NT, st, gw, tape.h1, m.eh));
  F32_TRY(sgemm_nn<NE_STORE>(gw.dh1, m.eh, w.e1_w, m.eh, m.As, gw.da1, m.As, NT, st, gw));
  F32_TRY(sgemm_nn<NE_STORE>(gw.da1, m.As, w.conv_w, m.As, m.A, grad, m.A, NT, st, gw));
  return cudaSuccess;
}

namespace {
// Tape and gradient buffers of one evaluation, in carve order (16-float aligned).
size_t grad_walk(const ModelDims& m, int NC, int T, int H, int HS, float* base, F32Tape* tape, F32GradWork* gw) {
  size_t off = 0;
  auto take = [&](size_t n) {
    float* p = base ? base + off : nullptr;
    off += (n + 15) / 16 * 16;
    return p;
  };
  const size_t NT = (size_t)NC * T, D = m.D, I = m.inner, L = m.L, mlp = m.mlp;
  const int n_calls = T - H + 1;
  F32Tape t;
  t.h1 = take(NT * m.eh);
  t.e = take(NT * D);
  t.y = take((size_t)NC * D);
  t.calls.resize(n_calls);
  size_t maxR = 1;
  for (int k = 0; k < n_calls; ++k) {
    F32TapeCall& c = t.calls[k];
    const int end = H + k;
    c.start = end > HS ? end - HS : 0;
    c.w = end - c.start;
    c.rows = NC * c.w;
    const size_t R = c.rows;
    maxR = std::max(maxR, R);
    c.row_tok = reinterpret_cast<int*>(take(R));
    c.x_in = take(L * R * D);
    c.qkv = take(L * R * 3 * I);
    c.o = take(L * R * D);
    c.x_mid = take(L * R * D);
    c.f1 = take(L * R * mlp);
    c.f2 = take(L * R * D);
    c.x_out = take(R * D);
  }
  F32GradWork g{};
  g.dX = take(maxR * D);
  g.dF = take(maxR * D);
  g.dF1 = take(maxR * mlp);
  g.dA = take(maxR * D);
  g.dAtt = take(maxR * I);
  g.dQKV = take(maxR * 3 * I);
  g.dY = take((size_t)NC * D);
  g.dpred = take((size_t)NC * n_calls * D);
  g.dmod = take(NT * L * 6 * D);
  g.de = take(NT * D);
  g.dh1 = take(NT * m.eh);
  g.da1 = take(NT * m.As);
  // split-reduction partials of dY . W: the split reductions (q|k|v, mlp, stacked adaLN, eh) all
  // produce rows of width D or A' <= D
  g.part_floats = (size_t)kMaxNnSplits * std::max(maxR, NT) * std::max<size_t>(D, m.As);
  g.part = take(g.part_floats);
  g.in_emb = take((size_t)NC * H * D);  // per-candidate embeddings at most
  g.in_goal = take((size_t)NC * D);
  g.in_cand = take(NT * m.A);
  g.in_w = take((size_t)NC);
  g.out_cost = take((size_t)NC);
  g.out_grad = take(NT * m.A);
  if (tape) *tape = std::move(t);
  if (gw) *gw = g;
  return off;
}
}  // namespace

size_t f32_grad_floats(const ModelDims& m, int NC, int T, int H, int HS) {
  return grad_walk(m, NC, T, H, HS, nullptr, nullptr, nullptr);
}

void f32_grad_carve(const ModelDims& m, int NC, int T, int H, int HS, float* base, F32Tape* tape, F32GradWork* gw) {
  grad_walk(m, NC, T, H, HS, base, tape, gw);
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
  f(13, al((size_t)kSplitK * NW * m.D));  // split-K partial sums
  f(14, al((size_t)m.L * NC * (m.frames - 1) * 2 * m.inner));  // growing-window key / value cache
}
}  // namespace

size_t f32_work_floats(const ModelDims& m, size_t n_cand, size_t T) {
  size_t n = 0;
  f32_layout(m, n_cand, T, [&](int, size_t k) { n += k; });
  return n;
}

F32Work f32_work_carve(const ModelDims& m, size_t n_cand, size_t T, float* base) {
  float* p[15];
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
  w.part = p[13];
  w.kv = p[14];
  return w;
}

}  // namespace lewm
