// iCEM sampling and elite refit kernels for sm_100a.
//
// k_sample: one warp per (env, candidate) builds the candidate action sequence
//   cand = noise * std + mean (reference lewm/solvers/icem.py:523), slot 0 = mean
//   (:524), slots 1..n_inject = previous sorted elites (:421-432), optional clamp
//   (:526-527). Noise is either injected (the reference's post-coloring noise
//   tensors) or drawn in-kernel: Philox4x32-10 normals (Box-Muller), colored by
//   a fixed real matrix W that equals rfft -> scale -> irfft
//   (lewm/solvers/icem.py:173-182), then divided by the unbiased std over time
//   (clamped at 1e-8, :148-150), laid out as in make_colored_noise (:185-250).
// k_refit: one CTA per env sorts (cost, index) keys with a bitonic network in
//   shared memory (ascending; ties -> lower index; NaN last), gathers the k
//   elites and refits mean / unbiased std with optional momentum
//   (lewm/solvers/icem.py:543-563), keeps the best elite (:551) and the mean
//   of the k smallest costs (:580).
#include "lewm_common.cuh"
#include "lewm_internal.h"

namespace lewm {
namespace {

constexpr int kMaxTA = 128;   // horizon * action_dim
constexpr int kMaxCol = 128;  // colored time length

struct Philox4 {
  uint32_t x, y, z, w;
};

__device__ __forceinline__ Philox4 philox4x32_10(Philox4 c, uint32_t k0, uint32_t k1) {
#pragma unroll
  for (int i = 0; i < 10; ++i) {
    const uint32_t lo0 = 0xD2511F53u * c.x, hi0 = __umulhi(0xD2511F53u, c.x);
    const uint32_t lo1 = 0xCD9E8D57u * c.z, hi1 = __umulhi(0xCD9E8D57u, c.z);
    c = Philox4{hi1 ^ c.y ^ k0, lo1, hi0 ^ c.w ^ k1, lo0};
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  return c;
}

// Draw d of (plan, it, env, cand): counter (d/4, cand, env, it), key (seed, plan).
__device__ __forceinline__ void normals4(uint32_t blk, uint32_t cand, uint32_t env, uint32_t it, uint32_t seed,
                                         uint32_t plan, float* out) {
  const Philox4 r = philox4x32_10(Philox4{blk, cand, env, it}, seed, plan);
  const float u1a = ((float)r.x + 1.0f) * 2.3283064365386963e-10f;  // (0, 1]
  const float u2a = (float)r.y * 2.3283064365386963e-10f;           // [0, 1)
  const float u1b = ((float)r.z + 1.0f) * 2.3283064365386963e-10f;
  const float u2b = (float)r.w * 2.3283064365386963e-10f;
  const float ra = sqrtf(-2.0f * logf(u1a)), rb = sqrtf(-2.0f * logf(u1b));
  float sa, ca, sb, cb;
  sincospif(2.0f * u2a, &sa, &ca);
  sincospif(2.0f * u2b, &sb, &cb);
  out[0] = ra * ca;
  out[1] = ra * sa;
  out[2] = rb * cb;
  out[3] = rb * sb;
}

// One warp per candidate: lane k draws Philox block k (normals 4k .. 4k+3, the same
// counter layout as a single thread would use), lanes split the coloring matvec over
// time steps, and the unbiased std over time is a warp reduction.
constexpr int kSampleWarps = 4;  // candidates per 128-thread CTA

__global__ void __launch_bounds__(32 * kSampleWarps) k_sample(SampleParams p) {
  __shared__ float wn_s[kSampleWarps][kMaxTA];
  __shared__ float v_s[kSampleWarps][kMaxTA];
  griddep_wait();
  griddep_launch();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gid = blockIdx.x * kSampleWarps + warp;
  if (gid >= p.B * p.S) return;  // whole warp
  const int env = gid / p.S, c = gid - env * p.S;
  const int TA = p.T * p.A;
  const float* mean = p.mean + (size_t)env * TA;
  const float* sd = p.stdv + (size_t)env * TA;
  float* out = p.cand + (size_t)gid * TA;
  float* wn = wn_s[warp];
  float* v = v_s[warp];
  if (c == 0) {
    for (int i = lane; i < TA; i += 32) v[i] = mean[i];
  } else if (c <= p.n_inject) {
    const float* e = p.elites + ((size_t)env * p.elite_stride + (c - 1)) * TA;
    for (int i = lane; i < TA; i += 32) v[i] = e[i];
  } else if (p.noise) {
    const float* nz = p.noise + (size_t)gid * TA;
    for (int i = lane; i < TA; i += 32) v[i] = nz[i] * sd[i] + mean[i];
  } else {
    // White draws in the reference's randn layout: [channel][time].
    const int chans = (p.noise_kind == 1) ? p.A / p.raw_block : p.A;
    const int ncol = (p.noise_kind == 0) ? p.T : p.ncol;
    const int n = chans * ncol;
    for (int blk = lane; 4 * blk < n; blk += 32) {
      float r4[4];
      normals4((uint32_t)blk, (uint32_t)c, (uint32_t)env, p.iter, p.rng[0], p.rng[1], r4);
#pragma unroll
      for (int q = 0; q < 4; ++q)
        if (4 * blk + q < n) wn[4 * blk + q] = r4[q];
    }
    __syncwarp();
    if (p.noise_kind == 0) {
      // white (B,S,T,A): draw d -> (t, a) = (d / A, d % A)
      for (int i = lane; i < TA; i += 32) v[i] = wn[i] * sd[i] + mean[i];
    } else {
      for (int ch = 0; ch < chans; ++ch) {
        float colv[kMaxCol / 32];
        float s = 0.f;
#pragma unroll
        for (int k = 0; k < kMaxCol / 32; ++k) {
          const int t = lane + 32 * k;
          float acc = 0.f;
          if (t < ncol) {
            const float* wr = p.W + t * ncol;
            for (int u = 0; u < ncol; ++u) acc += wr[u] * wn[ch * ncol + u];
          }
          colv[k] = acc;
          s += acc;
        }
        const float mu = warp_sum(s) / ncol;
        float q = 0.f;
#pragma unroll
        for (int k = 0; k < kMaxCol / 32; ++k)
          if (lane + 32 * k < ncol) q += (colv[k] - mu) * (colv[k] - mu);
        const float sdv = fmaxf(sqrtf(warp_sum(q) / (float)(ncol - 1)), 1e-8f);
#pragma unroll
        for (int k = 0; k < kMaxCol / 32; ++k) {
          const int t = lane + 32 * k;
          if (t < ncol) {
            int ts, a;
            if (p.noise_kind == 1) {  // raw time: (t, ch) -> solver step t / block, dim (t % block) * chans + ch
              ts = t / p.raw_block;
              a = (t - ts * p.raw_block) * chans + ch;
            } else {  // block: channel ch is action dim, t is solver step
              ts = t;
              a = ch;
            }
            const int i = ts * p.A + a;
            v[i] = (colv[k] / sdv) * sd[i] + mean[i];
          }
        }
      }
    }
  }
  __syncwarp();
  for (int i = lane; i < TA; i += 32) {
    float x = v[i];
    if (p.low) x = fminf(fmaxf(x, p.low[i % p.A]), p.high[i % p.A]);
    out[i] = x;
  }
}

__device__ __forceinline__ uint32_t order_key(float f) {
  if (isnan(f)) return 0xFFFFFFFFu;
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

constexpr int kRefitThreads = 512;
constexpr int kMaxSort = 4096;

__global__ void __launch_bounds__(kRefitThreads) k_refit(RefitParams p) {
  __shared__ unsigned long long keys[kMaxSort];
  griddep_wait();
  griddep_launch();
  const int env = blockIdx.x, tid = threadIdx.x;
  int P = 1;
  while (P < p.S) P <<= 1;
  const float* costs = p.costs + (size_t)env * p.S;
  for (int i = tid; i < P; i += kRefitThreads) {
    const uint32_t k = (i < p.S) ? order_key(costs[i]) : 0xFFFFFFFFu;
    keys[i] = ((unsigned long long)k << 32) | (unsigned)i;
  }
  __syncthreads();
  for (int size = 2; size <= P; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = tid; i < P; i += kRefitThreads) {
        const int j = i ^ stride;
        if (j > i) {
          const bool up = (i & size) == 0;
          const unsigned long long a = keys[i], b = keys[j];
          if ((a > b) == up) {
            keys[i] = b;
            keys[j] = a;
          }
        }
      }
      __syncthreads();
    }
  }
  const int TA = p.T * p.A;
  const float* cand = p.cand + (size_t)env * p.S * TA;
  if (tid < p.k) {
    const int idx = (int)(keys[tid] & 0xFFFFFFFFull);
    if (p.topk_idx) p.topk_idx[(size_t)env * p.k + tid] = idx;
    if (p.topk_val) p.topk_val[(size_t)env * p.k + tid] = costs[idx];
  }
  if (tid == 0) {
    float s = 0.f;
    for (int i = 0; i < p.k; ++i) s += costs[(int)(keys[i] & 0xFFFFFFFFull)];
    const float fc = s / (float)p.k;
    p.final_cost[env] = fc;
    if (p.nan_status && fc != fc) atomicOr(p.nan_status, LEWM_DEV_NAN);
  }
  for (int e = tid; e < p.R * TA; e += kRefitThreads) {
    const int i = e / TA, d = e - i * TA;
    const int idx = (int)(keys[i] & 0xFFFFFFFFull);
    p.elites[((size_t)env * p.R + i) * TA + d] = cand[(size_t)idx * TA + d];
  }
  if (tid < TA) {
    const int d = tid;
    float s = 0.f;
    for (int i = 0; i < p.k; ++i) s += cand[(size_t)(keys[i] & 0xFFFFFFFFull) * TA + d];
    const float mu = s / (float)p.k;
    float q = 0.f;
    for (int i = 0; i < p.k; ++i) {
      const float dv = cand[(size_t)(keys[i] & 0xFFFFFFFFull) * TA + d] - mu;
      q += dv * dv;
    }
    const float sdv = sqrtf(q / (float)(p.k - 1));
    const size_t o = (size_t)env * TA + d;
    p.best[o] = cand[(size_t)(keys[0] & 0xFFFFFFFFull) * TA + d];
    if (p.alpha != 0.f) {
      p.mean[o] = p.alpha * p.mean[o] + (1.0f - p.alpha) * mu;
      p.stdv[o] = p.alpha * p.stdv[o] + (1.0f - p.alpha) * sdv;
    } else {
      p.mean[o] = mu;
      p.stdv[o] = sdv;
    }
  }
}

__global__ void k_set_rng(uint32_t* rng, uint32_t seed, uint32_t plan) {
  griddep_wait();
  griddep_launch();
  rng[0] = seed;
  rng[1] = plan;
}

// Bounded-wait self-test: one thread waits on an mbarrier that nothing ever arrives
// on (no copy or MMA is attached to it), with the wait limit of the context's status
// block. The wait runs out, sets LEWM_DEV_TIMEOUT in the status word and the kernel
// returns; nothing else is in flight, so the context stays usable.
__global__ void k_wait_selftest(uint32_t* status) {
  __shared__ uint64_t bar;
  mbar_init(&bar, 1);
  fence_mbar_init();
  mbar_wait(&bar, 0, status);
}

}  // namespace

cudaError_t launch_wait_selftest(uint32_t* status, cudaStream_t st) {
  k_wait_selftest<<<1, 1, 0, st>>>(status);
  return cudaGetLastError();
}

cudaError_t launch_set_rng(uint32_t* rng, uint32_t seed, uint32_t plan, cudaStream_t st) {
  return launch_k(k_set_rng, dim3(1), dim3(1), 0, st, rng, seed, plan);
}

cudaError_t launch_sample(const SampleParams& p, cudaStream_t st) {
  if (p.T * p.A > kMaxTA || p.ncol > kMaxCol) return cudaErrorInvalidValue;
  const int n = p.B * p.S;
  return launch_k(k_sample, dim3((n + kSampleWarps - 1) / kSampleWarps), dim3(32 * kSampleWarps), 0, st, p);
}

cudaError_t launch_refit(const RefitParams& p, cudaStream_t st) {
  if (p.S > kMaxSort || p.T * p.A > kMaxTA || p.k > p.S || p.k < 1 || p.k > kRefitThreads) return cudaErrorInvalidValue;
  return launch_k(k_refit, dim3(p.B), dim3(kRefitThreads), 0, st, p);
}

}  // namespace lewm
