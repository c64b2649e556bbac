// Candidate sampling that allocates no device memory.
//
// lewm_sample_candidates keeps the coloring matrix W and the Philox key in a
// per-context workspace that lewm_create / the first call allocate with
// cudaMalloc. Some hosts cannot allocate at the point where they sample: a
// caller that has handed all of its device memory to its own pool, one that
// runs inside a region where allocation is forbidden, or one that only holds
// raw device pointers and no context. lewm_sample_candidates_noalloc serves
// them. It needs no context and keeps its scratch in one fixed-size array that
// is part of the loaded module, so it calls no cudaMalloc, cudaFree or any
// allocating library routine.
//
// Scratch: kScratchFloats floats (65,792 bytes) per device, holding a
// coloring matrix of at most kMaxCol x kMaxCol (kMaxCol = 128 colored time
// steps) followed by the two Philox key words. Requests whose colored time
// length exceeds kMaxCol are rejected with LEWM_UNSUPPORTED_SHAPE.
//
// Set-up: the first call on a device, made with that device current, resolves
// the scratch array's device address with cudaGetSymbolAddress (this may load
// the module on that device) and caches it. Make that first call before any
// stream capture. Later calls only launch two kernels. The cached address belongs to
// the device's primary context: a caller that destroys that context
// (cudaDeviceReset) must not call this entry point on that device again in the
// same process, since the cache would hand the kernels a stale address.
//
// Zero state: nothing in the scratch has to start at zero. Each call first
// rewrites every scratch word the sampler will read (the ncol x ncol matrix and
// the key) in a fill kernel on the caller's stream, and the sampler reads them
// only after that kernel has finished.
//
// Concurrency: the scratch is shared by every call on a device. Two calls whose
// work overlaps on the GPU (different streams without ordering between them)
// race on it and can produce wrong candidates. Calls on one stream, or streams
// ordered by events, are safe.
#include <cuda_runtime.h>

#include <climits>
#include <cstdarg>
#include <cmath>
#include <cstdio>
#include <mutex>

#include "lewm_b200.h"
#include "lewm_common.cuh"
#include "lewm_internal.h"

namespace lewm {
namespace {

constexpr int kMaxCol = 128;
constexpr int kMaxTA = 128;
constexpr int kKeyOffset = kMaxCol * kMaxCol;   // floats before the key words
constexpr int kScratchFloats = kKeyOffset + 64;  // key padded to 256 bytes
constexpr int kMaxDevices = 64;

static __device__ __align__(256) float g_sample_scratch[kScratchFloats];

// W[t][u] = (1/n) * (s_0 + sum_{f=1}^{n/2} w_f s_f cos(2 pi f (t - u) / n)), the
// real matrix of rfft -> scale by s_f = (f/n)^(-beta/2) (s_0 = s_1) -> irfft,
// with w_f = 1 at the Nyquist bin of even n and 2 otherwise
// (reference lewm/solvers/icem.py:173-182). Block t writes row t; the row is a
// cyclic shift of one column vector that each block forms in shared memory in
// double precision. Block 0 also stores the Philox key.
__global__ void __launch_bounds__(128) k_fill_sample_scratch(float* scratch, int n, double beta, uint32_t seed,
                                                             uint32_t plan) {
  griddep_wait();
  __shared__ float col[kMaxCol];
  const double pi = 3.14159265358979323846;
  for (int d = threadIdx.x; d < n; d += blockDim.x) {
    const double s1 = pow(1.0 / n, -beta / 2.0);
    double acc = s1;  // s_0 = s_1
    for (int f = 1; f <= n / 2; ++f) {
      const double w = (2 * f == n) ? 1.0 : 2.0;
      acc += w * pow((double)f / n, -beta / 2.0) * cos(2.0 * pi * f * d / n);
    }
    col[d] = (float)(acc / n);
  }
  __syncthreads();
  const int t = blockIdx.x;
  for (int u = threadIdx.x; u < n; u += blockDim.x) {
    const int d = t - u < 0 ? t - u + n : t - u;
    scratch[t * n + u] = col[d];
  }
  if (t == 0 && threadIdx.x == 0) {
    scratch[kKeyOffset] = __uint_as_float(seed);
    scratch[kKeyOffset + 1] = __uint_as_float(plan);
  }
}

std::mutex g_scratch_mu;
float* g_scratch_ptr[kMaxDevices] = {};

// Device address of this device's scratch; resolved once per device with the
// device current.
cudaError_t scratch_for_device(int dev, float** out) {
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_sample_scratch);
    if (e != cudaSuccess) return e;
    g_scratch_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_scratch_ptr[dev];
  return cudaSuccess;
}

lewm_status noalloc_fail(lewm_status s, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  set_noctx_error(buf);
  return s;
}

struct DeviceSwitch {
  int prev = -1;
  cudaError_t err = cudaSuccess;
  explicit DeviceSwitch(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    err = cudaSetDevice(dev);
  }
  ~DeviceSwitch() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

}  // namespace
}  // namespace lewm

using namespace lewm;

extern "C" lewm_status lewm_sample_candidates_noalloc(const lewm_plan_desc* p, int32_t action_dim, int32_t S,
                                                      int32_t iter, const float* mean, const float* std,
                                                      const float* injected_noise, const float* action_low,
                                                      const float* action_high, float* out, int32_t device,
                                                      void* stream) {
  set_noctx_error("");
  if (!p) return noalloc_fail(LEWM_INVALID_ARG, "plan desc is NULL");
  if (!mean || !std || !out) return noalloc_fail(LEWM_INVALID_ARG, "mean, std and out must be non-NULL");
  if (p->n_envs <= 0 || p->horizon <= 0 || action_dim <= 0 || S <= 0 || iter < 0)
    return noalloc_fail(LEWM_INVALID_ARG, "need n_envs, horizon, action_dim, S > 0 and iter >= 0");
  if (p->action_block <= 0) return noalloc_fail(LEWM_INVALID_ARG, "action_block must be positive, got %d", p->action_block);
  if (!(p->beta >= 0.f)) return noalloc_fail(LEWM_INVALID_ARG, "beta must be >= 0");
  if (p->clip_actions && (!action_low || !action_high))
    return noalloc_fail(LEWM_INVALID_ARG, "clip_actions needs action_low and action_high");
  if ((int64_t)p->horizon * action_dim > kMaxTA)
    return noalloc_fail(LEWM_UNSUPPORTED_SHAPE, "horizon*action_dim=%lld exceeds %d",
                        (long long)p->horizon * action_dim, kMaxTA);
  if ((int64_t)p->n_envs * S > (int64_t)INT_MAX - 127)
    return noalloc_fail(LEWM_UNSUPPORTED_SHAPE, "n_envs*S too large");
  if (device < 0 || device >= kMaxDevices) return noalloc_fail(LEWM_INVALID_ARG, "bad device %d", device);

  // Noise layout of make_colored_noise (reference lewm/solvers/icem.py:185-250).
  int kind = 0, ncol = 0;
  if (p->beta > 0.f) {
    if (p->time_axis_raw && p->action_block > 1) {
      if (action_dim % p->action_block)
        return noalloc_fail(LEWM_INVALID_ARG, "action_dim=%d is not divisible by action_block=%d", action_dim,
                            p->action_block);
      if ((int64_t)p->horizon * p->action_block > kMaxCol)
        return noalloc_fail(LEWM_UNSUPPORTED_SHAPE,
                            "colored time length horizon*action_block=%lld exceeds the fixed scratch limit of %d",
                            (long long)p->horizon * p->action_block, kMaxCol);
      kind = 1;
      ncol = p->horizon * p->action_block;
    } else {
      if (p->horizon > kMaxCol)
        return noalloc_fail(LEWM_UNSUPPORTED_SHAPE, "colored time length horizon=%d exceeds the fixed scratch limit of %d",
                            p->horizon, kMaxCol);
      kind = 2;
      ncol = p->horizon;
    }
    if (ncol <= 1) {
      kind = 0;
      ncol = 0;
    }
  }

  DeviceSwitch ds(device);
  if (ds.err != cudaSuccess) return noalloc_fail(LEWM_CUDA_ERROR, "cudaSetDevice(%d): %s", device, cudaGetErrorString(ds.err));
  float* scratch = nullptr;
  cudaError_t e = scratch_for_device(device, &scratch);
  if (e != cudaSuccess)
    return noalloc_fail(LEWM_CUDA_ERROR, "cudaGetSymbolAddress(scratch): %s", cudaGetErrorString(e));
  cudaStream_t st = static_cast<cudaStream_t>(stream);

  // A plain launch: the fill kernel starts only after earlier work on the
  // stream (including a previous call's sampler) has finished with the scratch.
  k_fill_sample_scratch<<<dim3(ncol > 0 ? ncol : 1), dim3(128), 0, st>>>(
      scratch, ncol > 0 ? ncol : 1, (double)p->beta, (uint32_t)(p->seed & 0xffffffffu),
      (uint32_t)(p->plan_index & 0xffffffffu));
  e = cudaGetLastError();
  if (e != cudaSuccess) return noalloc_fail(LEWM_CUDA_ERROR, "fill kernel launch: %s", cudaGetErrorString(e));

  SampleParams sp{};
  sp.B = p->n_envs;
  sp.S = S;
  sp.T = p->horizon;
  sp.A = action_dim;
  sp.noise_kind = kind;
  sp.raw_block = p->action_block;
  sp.ncol = ncol;
  sp.W = scratch;
  sp.noise = injected_noise;
  sp.rng = reinterpret_cast<const uint32_t*>(scratch + kKeyOffset);
  sp.iter = (uint32_t)iter;
  sp.mean = mean;
  sp.stdv = std;
  sp.elites = nullptr;
  sp.elite_stride = 1;
  sp.n_inject = 0;
  sp.low = p->clip_actions ? action_low : nullptr;
  sp.high = p->clip_actions ? action_high : nullptr;
  sp.cand = out;
  e = launch_sample(sp, st);
  if (e != cudaSuccess) return noalloc_fail(LEWM_CUDA_ERROR, "sample launch: %s", cudaGetErrorString(e));
  return LEWM_OK;
}
