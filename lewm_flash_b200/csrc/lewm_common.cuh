// sm_100a building blocks: mbarriers, bulk (TMA) copies, tcgen05 MMA / TMEM,
// the 128-byte-swizzled K-major operand layout, and bounded waits.
//
// Every wait here has a time limit (%globaltimer); on expiry it sets
// LEWM_DEV_TIMEOUT in the context's device status word and returns false so
// the kernel can release TMEM and exit instead of hanging the GPU.
//
// Status block (16 bytes of device memory per context, 8-byte aligned):
//   word 0      status bits (LEWM_DEV_*), read and cleared by the host
//   word 1      unused
//   words 2-3   wait limit in ns (uint64; 0 = kWaitLimitNs), set by the host
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace lewm {

// ----------------------------------------------------------------- status bits
constexpr uint32_t LEWM_DEV_TIMEOUT = 1u;   // a bounded wait gave up
constexpr uint32_t LEWM_DEV_BADARG = 2u;    // a kernel saw an impossible index
constexpr uint32_t LEWM_DEV_NAN = 4u;       // a plan's final cost was NaN
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // default: 2 s per wait
constexpr size_t kStatusBytes = 16;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ----------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// Barrier `id` (1..15) among `nthreads` threads (whole warps) of the CTA.
__device__ __forceinline__ void named_bar(uint32_t id, uint32_t nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}
// The wait limit stored in the status block (read only once a wait has not
// completed on its first try).
__device__ __forceinline__ uint64_t wait_limit_ns(const uint32_t* status) {
  const uint64_t v = *reinterpret_cast<const volatile uint64_t*>(status + 2);
  return v ? v : kWaitLimitNs;
}

// Wait for phase `parity` of `bar` to complete, at most the status block's wait limit.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t* status) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  const uint64_t limit = wait_limit_ns(status);
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (global_timer_ns() - t0 > limit) {
      atomicOr(status, LEWM_DEV_TIMEOUT);
      return false;
    }
  }
}

// Wait for the MMA-completion barrier in warp 0 only; every other thread blocks on the
// CTA barrier instead of polling the mbarrier, whose shared-memory word the tensor
// core's operand reads would otherwise share with hundreds of pollers. `flag` is a
// spare shared word that carries warp 0's result.
__device__ __forceinline__ bool cta_wait_mma(uint64_t* bar, uint32_t* status, uint32_t* flag,
                                             uint32_t parity = 0) {
  if (threadIdx.x < 32) {
    const bool ok = mbar_wait(bar, parity, status);
    if (threadIdx.x == 0) *flag = ok ? 1u : 0u;
  }
  __syncthreads();
  return *flag != 0u;
}

// ----------------------------------------------------------------- bulk copies (TMA engine, 1-D)
// global -> shared, completes `bytes` of transaction count on `bar`.
// dst/src 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
// shared -> global, tracked by the issuing thread's bulk group.
__device__ __forceinline__ void bulk_s2g(void* gdst, const void* smem_src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(gdst),
               "r"(smem_u32(smem_src)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// Wait until the shared-memory sources of every committed bulk store have been read
// (the global writes complete on their own and are visible at grid completion).
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// Make generic-proxy shared-memory writes visible to the async proxy (MMA / bulk copy).
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// ----------------------------------------------------------------- tcgen05 / TMEM
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {  // whole warp
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {  // whole warp
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {  // whole warp
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, bf16 inputs, fp32 accumulate.
__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on `bar` once every MMA issued so far by this thread has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 TMEM lanes x 16 consecutive 32-bit columns; thread i of the warp gets lane (base lane + i).
// Each load waits for its own completion inside the same asm statement, so no use of
// the destination registers can be scheduled before the data is there.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float* v) {
  uint32_t r[8];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];\n\t"
               "tcgen05.wait::ld.sync.aligned;"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_ld4(uint32_t taddr, float* v) {
  uint32_t r[4];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];\n\t"
               "tcgen05.wait::ld.sync.aligned;"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] = __uint_as_float(r[i]);
}
// N consecutive columns (N a multiple of 4) into v, then wait.
template <int N>
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, float* v) {
  int c = 0;
#pragma unroll
  for (; c + 16 <= N; c += 16) tmem_ld16(taddr + c, v + c);
  if constexpr ((N % 16) >= 8) {
    tmem_ld8(taddr + (N / 16) * 16, v + (N / 16) * 16);
  }
  if constexpr ((N % 8) == 4) {
    tmem_ld4(taddr + N - 4, v + N - 4);
  }
  tmem_ld_wait();
}

// ----------------------------------------------------------------- programmatic dependent launch
// Kernels launched with programmatic stream serialization may start before their
// predecessor finishes; everything that reads the predecessor's output must come
// after griddep_wait(). griddep_launch() lets the next kernel start its own prologue.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Instruction descriptor for kind::f16: bf16 A and B (both K-major), fp32 D, shape M x N.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N) {
  return (1u << 4)                              // D format: f32
         | (1u << 7)                            // A format: bf16
         | (1u << 10)                           // B format: bf16
         | (static_cast<uint32_t>(N >> 3) << 17)  // N / 8
         | (static_cast<uint32_t>(M >> 4) << 24); // M / 16
}

// Shared-memory matrix descriptor for a K-major operand in the 128-byte
// swizzle layout: rows of 64 bf16 (128 B), 8-row atoms of 1024 B stacked
// contiguously. `saddr` is the shared address of the first element of the
// 16-element K slice being addressed (atom base + 32 B * slice).
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t saddr) {
  uint64_t d = static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(1u) << 16;            // leading byte offset (unused for swizzled K-major)
  d |= static_cast<uint64_t>(1024u >> 4) << 32;    // stride byte offset: 8 rows x 128 B
  d |= static_cast<uint64_t>(1u) << 46;            // descriptor version for sm_100
  d |= static_cast<uint64_t>(2u) << 61;            // SWIZZLE_128B
  return d;
}

// Byte offset of element (r, k), k < 64, inside one [R x 64] bf16 block in
// the 128-byte swizzle layout (16-byte chunk index XOR row % 8).
__host__ __device__ __forceinline__ uint32_t sw128_off(uint32_t r, uint32_t k) {
  return r * 128u + ((((k >> 3) ^ (r & 7u)) << 4) | ((k & 7u) << 1));
}

// Issue the MMAs of D[128 x N] (+)= A[128 x 64*nkb] * B[N x 64*nkb]^T where A and
// B are stored as consecutive [rows x 64] swizzled blocks. Single thread.
__device__ __forceinline__ void umma_tile(uint32_t d_tmem, uint32_t a_base, uint32_t a_block_bytes,
                                          uint32_t b_base, uint32_t b_block_bytes, int kb0, int nkb,
                                          uint32_t idesc, bool accumulate) {
  for (int kb = 0; kb < nkb; ++kb) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint64_t ad = sdesc_sw128(a_base + (kb0 + kb) * a_block_bytes + j * 32);
      const uint64_t bd = sdesc_sw128(b_base + (kb0 + kb) * b_block_bytes + j * 32);
      umma_bf16(d_tmem, ad, bd, idesc, (accumulate || kb > 0 || j > 0) ? 1u : 0u);
    }
  }
}

// ----------------------------------------------------------------- math helpers
__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + expf(-x)); }
// Exact-form GELU, x * Phi(x), with Phi from the complementary error function of
// Abramowitz & Stegun, Handbook of Mathematical Functions, formula 7.1.26:
// erfc(z) ~= t (a1 + t (a2 + t (a3 + t (a4 + t a5)))) exp(-z^2), t = 1 / (1 + p z), z >= 0,
// |error| <= 1.5e-7. Against the exact GELU the float result is within 4.3e-7 absolute
// over [-10, 10], far below the bf16 rounding of the hidden activations it feeds. The
// negative branch uses erfc directly (no 1 - erf cancellation). About a third of the
// instructions of an erff-based form: the FFN epilogues are issue-bound on it.
__device__ __forceinline__ float gelu_f(float x) {
  const float z = fabsf(x) * 0.70710678118654752440f;
  const float t = __fdividef(1.0f, fmaf(0.3275911f, z, 1.0f));
  const float poly =
      t * fmaf(t, fmaf(t, fmaf(t, fmaf(t, 1.061405429f, -1.453152027f), 1.421413741f), -0.284496736f), 0.254829592f);
  const float tail = 0.5f * poly * __expf(-z * z);  // Phi(-|x|)
  return x * (x >= 0.f ? 1.0f - tail : tail);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ float2 unpack_bf16x2(uint32_t u) {
  __nv_bfloat162 h = *reinterpret_cast<__nv_bfloat162*>(&u);
  return __bfloat1622float2(h);
}

}  // namespace lewm
