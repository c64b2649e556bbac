// One predictor call of the rollout, all layers, in one kernel: the batched regime.
//
// Reference: the per-call body of rollout_from_embeddings (lewm/jepa.py:262-300):
// ARPredictor.forward (lewm/module.py:244-285, position add), the Transformer's
// ConditionalBlocks (:88-111: AdaLN modulate, Attention :56-85, FeedForward :38-53),
// the final LayerNorm (:183), then the new prediction's history slot or, on the last
// call, cost_from_rollout (lewm/jepa.py:246-260).
//
// Work split: a CTA owns one row tile of 40 candidates x 3 window rows for the whole
// call. Rows sit quadrant-aligned so a candidate's window never crosses a TMEM lane
// quadrant: row r = 32 q + 3 c + pos for the candidate c (0..9) of quadrant q; rows
// 30 and 31 of each quadrant are idle. The fp32 residual stream of the tile stays in
// the registers of the 16 epilogue warps (warp w: quadrant w & 3, columns
// [48 (w >> 2), +48)) across all layers; nothing but the inputs, the modulation rows
// and the weights is read, and nothing but the call's prediction or cost is written.
//
// Roles (18 warps):
//   warp 16  producer: streams the layer weights as [192 x 64] bf16 blocks (24 KB)
//            through a 4-slot shared-memory ring, two copies per instruction;
//   warp 17  MMA issuer: tcgen05.mma M 128 x N 192 into TMEM (columns [0, 192) QKV of
//            one head or one FC1 quarter, [192, 384) the out-projection / FC2
//            accumulator), operands in 128-byte-swizzled K-major shared memory;
//   warps 0-15  epilogue: LayerNorm + modulate + LayerNorm into the bf16 A operand,
//            causal window attention per head (k / v exchanged in shared memory),
//            residual updates, bias + GELU into the FC2 operand, final LayerNorm, cost.
// Per layer the MMA order is QKV(0), then for each head h >= 1 QKV(h) and the
// out-projection of head h - 1 (K = 64 into the accumulator), out-projection(15),
// FC1(0), then FC1(q) and FC2(q - 1) for q = 1..3, FC2(3); the producer streams the
// weight blocks in exactly that order (88 blocks, 2.1 MB per layer, L2-resident).
//
// Synchronisation: mbarriers throughout (ring full / empty; epilogue -> MMA arrivals
// of one lane per warp after a proxy fence; MMA -> epilogue through tcgen05.commit);
// every wait is bounded by the context's wait limit and, once any wait of the CTA has
// expired, every later wait returns at once, so the CTA drains and exits. Control flow
// (barriers, loop trip counts) never depends on that outcome.
#include <cstdio>

#include "lewm_common.cuh"
#include "lewm_internal.h"

namespace lewm {
namespace {

constexpr int D = 192, HEADS = 16, MLP = 768, WIN = 3;
constexpr int CAND_PER_QUAD = 10;
constexpr int EPI_THREADS = 512;
constexpr int PRODUCER_WARP = 16, MMA_WARP = 17;
constexpr int THREADS = 18 * 32;
constexpr int RING = 4;
constexpr int B_BLK = 192 * 128;  // bytes of a [192 x 64] bf16 weight block
constexpr int A_BLK = 128 * 128;  // bytes of a [128 x 64] bf16 operand block
constexpr int BLOCKS_PER_LAYER = 88;
constexpr int KV_ROW = 256;       // bytes per row of the k / v exchange: k 64 | v 64 bf16
constexpr uint32_t COL_QKV = 0, COL_OUT = 192, COL_STASH = 384;

constexpr int OFF_A = 0;                              // 3 operand blocks (LayerNorm output)
constexpr int OFF_RING = OFF_A + 3 * A_BLK;           // weight ring
constexpr int OFF_SCR = OFF_RING + RING * B_BLK;      // attention scratch | FC2 operand (hidden)
constexpr int OFF_KV = OFF_SCR;                       // [128][256 B]: k 64 | v 64 bf16, chunks swizzled
constexpr int OFF_SO = OFF_SCR + 128 * KV_ROW;        // 2 attention-output operand blocks
// [2 buffers][4 parts][3 positions][128] partial scores; the LayerNorm moments ([2][4][128]
// float2) share the region (the two phases never overlap).
constexpr int OFF_SPART = OFF_SO + 2 * A_BLK;
constexpr int OFF_STATS = OFF_SPART;
constexpr int OFF_BAR = OFF_SPART + 2 * 4 * WIN * 128 * 4;
constexpr int SMEM_BYTES = 1024 + OFF_BAR + 256;
static_assert(OFF_SO % 1024 == 0 && OFF_SCR % 1024 == 0, "operand blocks need 1024-byte alignment");
static_assert(2 * 4 * 128 * 8 <= OFF_BAR - OFF_STATS, "moment scratch must fit the score region");
static_assert(3 * A_BLK <= OFF_BAR - OFF_SCR, "hidden operand must fit the scratch region");
static_assert(SMEM_BYTES <= 232448, "shared memory");

enum Bar {
  B_FULL = 0,       // [4] ring slot loaded (producer arrive_expect_tx + copy bytes)
  B_EMPTY = 4,      // [4] ring slot consumed (tcgen05.commit)
  B_A_READY = 8,    // A operand written (16 epilogue warps)
  B_QKV_FULL = 9,   // QKV(h) in TMEM (commit)
  B_QKV_FREE = 10,  // QKV(h) read out of TMEM (16 warps), h < 15
  B_O_READY = 11,   // [2] attention output block written (16 warps)
  B_O_FREE = 13,    // [2] out-projection of that block done (commit)
  B_OUT_FULL = 15,  // out-projection accumulator complete (commit)
  B_FC1_FULL = 16,  // FC1(q) in TMEM (commit)
  B_FC1_FREE = 17,  // FC1(q) read out of TMEM (16 warps), q < 3
  B_HID_READY = 18, // FC2 operand of quarter q written (16 warps)
  B_HID_FREE = 19,  // FC2(q) done (commit)
  B_DRAIN = 20,     // every MMA of the CTA done (commit), before TMEM is released
  B_COUNT = 21
};

// The four warps of one TMEM lane quadrant (the four column parts of the same 32 rows).
__device__ __forceinline__ void bar_quad(int quad) { named_bar(2 + quad, 128); }

// mbarrier.try_wait with a suspend-time hint: the waiting thread sleeps until the phase
// completes or `hint_ns` elapse, instead of spinning and taking issue slots from the warps
// that do the work on its sub-partition.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

// Bounded wait that gives up at once when another wait of the CTA has expired.
__device__ __forceinline__ bool tc_wait(uint64_t* bar, uint32_t parity, uint32_t* status, volatile int* abort) {
  if (mbar_try_wait(bar, parity)) return true;
  if (*abort) return false;
  const uint64_t t0 = global_timer_ns();
  const uint64_t limit = wait_limit_ns(status);
  while (true) {
    if (mbar_try_wait_sleep(bar, parity, 1000000u)) return true;
    if (*abort) return false;
    if (global_timer_ns() - t0 > limit) {
      atomicOr(status, LEWM_DEV_TIMEOUT);
      *abort = 1;
      return false;
    }
  }
}

// Lane 0 of the warp waits; the warp continues together with its result.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, uint32_t* status, volatile int* abort,
                                          int lane) {
  int ok = 1;
  if (lane == 0) ok = tc_wait(bar, parity, status, abort) ? 1 : 0;
  ok = __shfl_sync(0xffffffffu, ok, 0);
  __syncwarp();
  return ok != 0;
}

// One arrival per epilogue warp, after the warp's shared-memory writes are visible to
// the tensor core (async proxy) and its TMEM reads have completed.
__device__ __forceinline__ void warp_arrive(uint64_t* bar, int lane) {
  fence_async_smem();
  tc_fence_before();
  __syncwarp();
  if (lane == 0) mbar_arrive(bar);
}

// Weight block `blk` (0..87) of layer `l`, in the MMA consumption order.
__device__ __forceinline__ const __nv_bfloat16* weight_block(const DevWeights& w, int l, int blk) {
  constexpr size_t E = 192 * 64;  // elements per block
  int kind, idx, kb;              // kind 0 QKV(idx), 1 out-projection(idx), 2 FC1(idx), 3 FC2(idx)
  if (blk < 3) {
    kind = 0; idx = 0; kb = blk;
  } else if (blk < 63) {
    const int u = blk - 3, t = u & 3;
    if (t < 3) { kind = 0; idx = 1 + (u >> 2); kb = t; }
    else { kind = 1; idx = u >> 2; kb = 0; }
  } else if (blk == 63) {
    kind = 1; idx = 15; kb = 0;
  } else if (blk < 67) {
    kind = 2; idx = 0; kb = blk - 64;
  } else if (blk < 85) {
    const int u = blk - 67, q = 1 + u / 6, t = u % 6;
    if (t < 3) { kind = 2; idx = q; kb = t; }
    else { kind = 3; idx = q - 1; kb = t - 3; }
  } else {
    kind = 3; idx = 3; kb = blk - 85;
  }
  switch (kind) {
    case 0: return w.qkv + ((size_t)(l * HEADS + idx) * 3 + kb) * E;
    case 1: return w.wout_wide + ((size_t)l * HEADS + idx) * E;
    case 2: return w.w1s + ((size_t)(l * 4 + idx) * 3 + kb) * E;
    default: return w.w2s + ((size_t)(l * 4 + idx) * 3 + kb) * E;
  }
}

// MMAs of one 64-wide K block: D[128 x 192] (+)= A block . B block^T, 4 steps of K 16.
__device__ __forceinline__ void mma_kblock(uint32_t d, uint32_t a, uint32_t b, bool acc) {
  constexpr uint32_t idesc = idesc_bf16(128, 192);
  uint64_t ad = sdesc_sw128(a), bd = sdesc_sw128(b);
#pragma unroll
  for (int j = 0; j < 4; ++j) umma_bf16(d, ad + 2 * j, bd + 2 * j, idesc, (acc || j > 0) ? 1u : 0u);
}

// 32 TMEM lanes x 16 columns from registers (tcgen05.st); completes before it returns.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};\n\t"
      "tcgen05.wait::st.sync.aligned;" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
      "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
      "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15]))
      : "memory");
}

// The thread's 48-column residual slice: columns [0, 16) in registers (xr), [16, 48) in
// TMEM columns [384 + 32 part, +32) (the stash): registers are the epilogue's limit.
// Chunk t (16 columns) of the slice into v.
__device__ __forceinline__ void load_chunk(int t, const float* xr, uint32_t tstash, float* v) {
  if (t == 0) {
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = xr[i];
  } else {
    tmem_ld16(tstash + 16 * (t - 1), v);
  }
}
__device__ __forceinline__ void store_chunk(int t, float* xr, uint32_t tstash, const float* v) {
  if (t == 0) {
#pragma unroll
    for (int i = 0; i < 16; ++i) xr[i] = v[i];
  } else {
    tmem_st16(tstash + 16 * (t - 1), v);
  }
}

struct RowCtx {
  int r;        // tile row (TMEM lane)
  int part;     // column part 0..3: residual columns [48 part, 48 part + 48)
  int cand;     // candidate index over all envs
  int pos;      // window position 0..2
  bool valid;
  int tok;      // cand * T + history index (modulation row)
};

// Row moments from the four parts' own (mean, M2) over 48 columns each (Chan et al.'s
// pairwise combination): mean of the part means, M2 = sum M2_p + 48 sum (mean_p - mean)^2.
// One exchange through the two-buffer scratch (`red` counts uses). Returns (mean, var).
__device__ __forceinline__ float2 row_moments(float mean_p, float m2_p, float* stats, int& red, const RowCtx& rc) {
  float2* s = reinterpret_cast<float2*>(stats) + (red & 1) * 512;
  ++red;
  s[rc.part * 128 + rc.r] = make_float2(mean_p, m2_p);
  bar_quad(rc.r >> 5);
  const float2 a = s[rc.r], b = s[128 + rc.r], c = s[256 + rc.r], d = s[384 + rc.r];
  const float mean = ((a.x + b.x) + (c.x + d.x)) * 0.25f;
  const float da = a.x - mean, db = b.x - mean, dc = c.x - mean, dd = d.x - mean;
  const float m2 = ((a.y + b.y) + (c.y + d.y)) + 48.0f * ((da * da + db * db) + (dc * dc + dd * dd));
  return make_float2(mean, m2 * (1.0f / D));
}
// Sum of one value over the row's four parts.
__device__ __forceinline__ float row_sum(float v, float* stats, int& red, const RowCtx& rc) {
  float2* s = reinterpret_cast<float2*>(stats) + (red & 1) * 512;
  ++red;
  s[rc.part * 128 + rc.r] = make_float2(v, 0.f);
  bar_quad(rc.r >> 5);
  return (s[rc.r].x + s[128 + rc.r].x) + (s[256 + rc.r].x + s[384 + rc.r].x);
}

__device__ __forceinline__ void unpack2(uint32_t u, float* f) {
  f[0] = __uint_as_float(u << 16);
  f[1] = __uint_as_float(u & 0xffff0000u);
}
__device__ __forceinline__ void unpack8(const uint4 u, float* f) {
  unpack2(u.x, f);
  unpack2(u.y, f + 2);
  unpack2(u.z, f + 4);
  unpack2(u.w, f + 6);
}
__device__ __forceinline__ void ldg8(const float* p, float* f) {
  const float4 a = __ldg(reinterpret_cast<const float4*>(p));
  const float4 b = __ldg(reinterpret_cast<const float4*>(p + 4));
  f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
}

// bf16(LN_{g,b}(LN(x) * (1 + scale) + shift)) into the three operand blocks at `op`:
// first LayerNorm eps 1e-6 without affine (AdaLN modulate, lewm/module.py:105-111),
// second the block's own LayerNorm (eps 1e-5, affine). shift / scale: this row's
// modulation columns (bf16) for the thread's part, or null for an idle row. Two-pass
// moments; h = y * (1 + scale) + shift is recomputed per pass (modulation rows hit L1).
__device__ __forceinline__ void mod_chunk8(const __nv_bfloat16* shift, const __nv_bfloat16* scale, int c, float* sh,
                                           float* sc) {
  if (shift) {
    unpack8(__ldg(reinterpret_cast<const uint4*>(shift + c)), sh);
    unpack8(__ldg(reinterpret_cast<const uint4*>(scale + c)), sc);
  } else {
#pragma unroll
    for (int e = 0; e < 8; ++e) sh[e] = sc[e] = 0.f;
  }
}

__device__ __forceinline__ void ln_modulate_operand(const float* xr, uint32_t ts, const __nv_bfloat16* shift,
                                                    const __nv_bfloat16* scale, const float* __restrict__ g,
                                                    const float* __restrict__ bb, uint8_t* op, float* stats, int& red,
                                                    const RowCtx& rc) {
  const int c0 = 48 * rc.part;
  // moments of x (two passes over the thread's 48 columns, one exchange)
  float s = 0.f;
#pragma unroll
  for (int t = 0; t < 3; ++t) {
    float v[16];
    load_chunk(t, xr, ts, v);
#pragma unroll
    for (int i = 0; i < 16; ++i) s += v[i];
  }
  const float mp = s * (1.0f / 48);
  float q = 0.f;
#pragma unroll
  for (int t = 0; t < 3; ++t) {
    float v[16];
    load_chunk(t, xr, ts, v);
#pragma unroll
    for (int i = 0; i < 16; ++i) q += (v[i] - mp) * (v[i] - mp);
  }
  const float2 mv1 = row_moments(mp, q, stats, red, rc);
  const float m1 = mv1.x, r1 = rsqrtf(mv1.y + 1e-6f);
  // h = LN(x) * (1 + scale) + shift: its moments in one pass (sum and sum of squares over the
  // thread's 48 columns, then the exact pairwise combination across parts), recomputed for
  // the output pass.
  float hs = 0.f, hss = 0.f;
#pragma unroll
  for (int t = 0; t < 3; ++t) {
    float v[16];
    load_chunk(t, xr, ts, v);
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      float sh[8], sc[8];
      mod_chunk8(shift, scale, 16 * t + 8 * e, sh, sc);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float y = (v[8 * e + k] - m1) * r1;
        const float h = fmaf(y, sc[k], y) + sh[k];
        hs += h;
        hss = fmaf(h, h, hss);
      }
    }
  }
  const float hp = hs * (1.0f / 48);
  const float2 mv2 = row_moments(hp, fmaxf(hss - hs * hp, 0.f), stats, red, rc);
  const float m2 = mv2.x, r2 = rsqrtf(mv2.y + 1e-5f);
#pragma unroll
  for (int t = 0; t < 3; ++t) {
    float v[16];
    load_chunk(t, xr, ts, v);
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      float sh[8], sc[8], gg[8], bv[8], o[8];
      mod_chunk8(shift, scale, 16 * t + 8 * e, sh, sc);
      const int c = c0 + 16 * t + 8 * e;
      ldg8(g + c, gg);
      ldg8(bb + c, bv);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float y = (v[8 * e + k] - m1) * r1;
        const float h = fmaf(y, sc[k], y) + sh[k];
        o[k] = fmaf((h - m2) * r2, gg[k], bv[k]);
      }
      const uint4 u = make_uint4(pack_bf16x2(o[0], o[1]), pack_bf16x2(o[2], o[3]), pack_bf16x2(o[4], o[5]),
                                 pack_bf16x2(o[6], o[7]));
      *reinterpret_cast<uint4*>(op + (c >> 6) * A_BLK + sw128_off(rc.r, c & 63)) = u;
    }
  }
}

// x += gate * (acc + bias) for the thread's 48 columns, acc read from TMEM.
__device__ __forceinline__ void residual_update(float* xr, uint32_t ts, uint32_t tacc, const __nv_bfloat16* gate,
                                                const float* __restrict__ bias, const RowCtx& rc) {
  const int c0 = 48 * rc.part;
#pragma unroll
  for (int t = 0; t < 3; ++t) {
    float a[16], v[16];
    tmem_ld16(tacc + 16 * t, a);
    load_chunk(t, xr, ts, v);
#pragma unroll
    for (int e = 0; e < 16; e += 8) {
      float gt[8], bv[8];
      if (gate)
        unpack8(__ldg(reinterpret_cast<const uint4*>(gate + 16 * t + e)), gt);
      else
#pragma unroll
        for (int k = 0; k < 8; ++k) gt[k] = 0.f;
      ldg8(bias + c0 + 16 * t + e, bv);
#pragma unroll
      for (int k = 0; k < 8; ++k) v[e + k] = fmaf(gt[k], a[e + k] + bv[k], v[e + k]);
    }
    store_chunk(t, xr, ts, v);
  }
}

}  // namespace

__global__ void __maxnreg__(96) k_tile_call(DevWeights w, TileCallParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem + OFF_A;
  uint8_t* ring = smem + OFF_RING;
  uint8_t* sKV = smem + OFF_KV;
  uint8_t* sO = smem + OFF_SO;
  uint8_t* sHid = smem + OFF_SCR;
  float* spart = reinterpret_cast<float*>(smem + OFF_SPART);
  float* stats = reinterpret_cast<float*>(smem + OFF_STATS);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + B_COUNT);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int tile = blockIdx.x;
  uint32_t* status = p.status;

  if (tid == 0) {
    for (int s = 0; s < RING; ++s) {
      mbar_init(&bars[B_FULL + s], 1);
      mbar_init(&bars[B_EMPTY + s], 1);
    }
    mbar_init(&bars[B_A_READY], 16);
    mbar_init(&bars[B_QKV_FULL], 1);
    mbar_init(&bars[B_QKV_FREE], 16);
    mbar_init(&bars[B_O_READY], 16);
    mbar_init(&bars[B_O_READY + 1], 16);
    mbar_init(&bars[B_O_FREE], 1);
    mbar_init(&bars[B_O_FREE + 1], 1);
    mbar_init(&bars[B_OUT_FULL], 1);
    mbar_init(&bars[B_FC1_FULL], 1);
    mbar_init(&bars[B_FC1_FREE], 16);
    mbar_init(&bars[B_HID_READY], 16);
    mbar_init(&bars[B_HID_FREE], 1);
    mbar_init(&bars[B_DRAIN], 1);
    *abort = 0;
    fence_mbar_init();
  }
  if (warp == MMA_WARP) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int L = p.layers;
  const int total_blocks = L * BLOCKS_PER_LAYER;

  int issued = 0;  // producer: ring blocks whose copies were issued
  if (warp == PRODUCER_WARP) {
    // Weights only: the producer may start before the previous kernel has finished.
    for (int g = 0; g < total_blocks; g += 2) {
      const int s0 = g % RING, use = g / RING;
      bool ok = true;
      if (lane == 0 && use > 0) {
        ok = tc_wait(&bars[B_EMPTY + s0], (use - 1) & 1, status, abort) &&
             tc_wait(&bars[B_EMPTY + s0 + 1], (use - 1) & 1, status, abort);
      }
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      if (!ok) break;
      if (lane == 0) {
        mbar_arrive_expect_tx(&bars[B_FULL + s0], B_BLK);
        mbar_arrive_expect_tx(&bars[B_FULL + s0 + 1], B_BLK);
      }
      __syncwarp();
      if (lane < 2) {
        const int gg = g + lane;
        bulk_g2s(ring + (s0 + lane) * B_BLK, weight_block(w, gg / BLOCKS_PER_LAYER, gg % BLOCKS_PER_LAYER), B_BLK,
                 &bars[B_FULL + s0 + lane]);
      }
      __syncwarp();
      issued = g + 2;
    }
    griddep_wait();
    griddep_launch();
  } else if (warp == MMA_WARP) {
    griddep_wait();
    griddep_launch();
    int g = 0;  // ring block counter
    auto take = [&](int& slot) -> bool {
      slot = g % RING;
      const bool ok = warp_wait(&bars[B_FULL + slot], (g / RING) & 1, status, abort, lane);
      tc_fence_after();
      return ok;
    };
    auto release = [&](int slot) {
      if (lane == 0) umma_commit(&bars[B_EMPTY + slot]);
      __syncwarp();
      ++g;
    };
    const uint32_t aA = smem_u32(sA), aRing = smem_u32(ring), aO = smem_u32(sO), aHid = smem_u32(sHid);
    for (int l = 0; l < L; ++l) {
      bool ok = warp_wait(&bars[B_A_READY], (2 * l) & 1, status, abort, lane);
      tc_fence_after();
      // QKV(h) for h = 0..15, with the out-projection of head h - 1 after QKV(h).
      for (int h = 0; h < HEADS; ++h) {
        if (h > 0) {
          ok = warp_wait(&bars[B_QKV_FREE], (15 * l + h - 1) & 1, status, abort, lane) && ok;
          tc_fence_after();
        }
        for (int kb = 0; kb < 3; ++kb) {
          int slot;
          ok = take(slot) && ok;
          if (lane == 0 && ok) mma_kblock(tmem + COL_QKV, aA + kb * A_BLK, aRing + slot * B_BLK, kb > 0);
          release(slot);
        }
        if (lane == 0) umma_commit(&bars[B_QKV_FULL]);
        __syncwarp();
        if (h > 0) {
          const int hp = h - 1, b = hp & 1;
          ok = warp_wait(&bars[B_O_READY + b], (8 * l + hp / 2) & 1, status, abort, lane) && ok;
          tc_fence_after();
          int slot;
          ok = take(slot) && ok;
          if (lane == 0 && ok) mma_kblock(tmem + COL_OUT, aO + b * A_BLK, aRing + slot * B_BLK, hp > 0);
          release(slot);
          if (lane == 0) umma_commit(&bars[B_O_FREE + b]);
          __syncwarp();
        }
      }
      {  // out-projection of head 15
        ok = warp_wait(&bars[B_O_READY + 1], (8 * l + 7) & 1, status, abort, lane) && ok;
        tc_fence_after();
        int slot;
        ok = take(slot) && ok;
        if (lane == 0 && ok) mma_kblock(tmem + COL_OUT, aO + A_BLK, aRing + slot * B_BLK, true);
        release(slot);
        if (lane == 0) {
          umma_commit(&bars[B_O_FREE + 1]);
          umma_commit(&bars[B_OUT_FULL]);
        }
        __syncwarp();
      }
      // Feed-forward: FC1 quarter q into [0, 192), FC2 quarter q accumulating into [192, 384).
      ok = warp_wait(&bars[B_A_READY], (2 * l + 1) & 1, status, abort, lane) && ok;
      tc_fence_after();
      for (int q = 0; q <= 4; ++q) {
        if (q < 4) {
          if (q > 0) {
            ok = warp_wait(&bars[B_FC1_FREE], (3 * l + q - 1) & 1, status, abort, lane) && ok;
            tc_fence_after();
          }
          for (int kb = 0; kb < 3; ++kb) {
            int slot;
            ok = take(slot) && ok;
            if (lane == 0 && ok) mma_kblock(tmem + COL_QKV, aA + kb * A_BLK, aRing + slot * B_BLK, kb > 0);
            release(slot);
          }
          if (lane == 0) umma_commit(&bars[B_FC1_FULL]);
          __syncwarp();
        }
        if (q > 0) {
          const int qp = q - 1;
          ok = warp_wait(&bars[B_HID_READY], (4 * l + qp) & 1, status, abort, lane) && ok;
          tc_fence_after();
          for (int kb = 0; kb < 3; ++kb) {
            int slot;
            ok = take(slot) && ok;
            if (lane == 0 && ok)
              mma_kblock(tmem + COL_OUT, aHid + kb * A_BLK, aRing + slot * B_BLK, qp > 0 || kb > 0);
            release(slot);
          }
          if (lane == 0) umma_commit(&bars[B_HID_FREE]);
          __syncwarp();
        }
      }
    }
  } else if (warp < 16) {
    // ------------------------------------------------------------ epilogue warps
    RowCtx rc;
    const int quad = warp & 3;
    rc.part = warp >> 2;
    rc.r = 32 * quad + lane;
    const int cl = CAND_PER_QUAD * quad + lane / WIN;
    rc.pos = lane % WIN;
    rc.cand = tile * (4 * CAND_PER_QUAD) + cl;
    rc.valid = lane < CAND_PER_QUAD * WIN && rc.cand < p.n_cand;
    const int j = p.start + rc.pos;  // history index of the row
    rc.tok = rc.cand * p.T + j;
    const int c0 = 48 * rc.part;
    const uint32_t tlane = tmem + ((uint32_t)(32 * quad) << 16);
    const uint32_t tstash = tlane + COL_STASH + 32 * rc.part;
    const size_t mod_cols = (size_t)L * 6 * D;
    const __nv_bfloat16* mrow = rc.valid ? p.mod + (size_t)rc.tok * mod_cols : nullptr;
    int red = 0;
    griddep_wait();
    griddep_launch();
    // Layer-0 rows: the history entry (observation embedding or an earlier prediction)
    // plus the position embedding (lewm/module.py:276-280).
    float xr[16];  // residual columns [c0, c0 + 16); [c0 + 16, c0 + 48) in the TMEM stash
    {
      const float* src = nullptr;
      if (rc.valid) {
        const int e = rc.cand / p.S;
        src = j < p.H ? p.emb + ((size_t)e * p.H + j) * D : p.pred + ((size_t)rc.cand * p.npred + (j - p.H)) * D;
      }
#pragma unroll
      for (int t = 0; t < 3; ++t) {
        float v[16];
#pragma unroll
        for (int i = 0; i < 16; i += 4) {
          float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
          if (src) {
            a = *reinterpret_cast<const float4*>(src + c0 + 16 * t + i);
            const float4 pe = __ldg(reinterpret_cast<const float4*>(w.pos + rc.pos * D + c0 + 16 * t + i));
            a.x += pe.x; a.y += pe.y; a.z += pe.z; a.w += pe.w;
          }
          v[i] = a.x; v[i + 1] = a.y; v[i + 2] = a.z; v[i + 3] = a.w;
        }
        store_chunk(t, xr, tstash, v);
      }
    }
    const int npos = rc.valid ? rc.pos : 0;  // earlier window positions this row attends to
    const int base = rc.r - rc.pos;           // tile row of window position 0
    for (int l = 0; l < L; ++l) {
      const __nv_bfloat16* ml = mrow ? mrow + (size_t)l * 6 * D + c0 : nullptr;
      // ---- attention half: A = attn.norm(LN1(x) * (1 + scale_msa) + shift_msa)
      ln_modulate_operand(xr, tstash, ml, ml ? ml + D : nullptr, w.attn_ln_w + l * D, w.attn_ln_b + l * D, sA, stats,
                          red, rc);
      warp_arrive(&bars[B_A_READY], lane);
      for (int h = 0; h < HEADS; ++h) {
        warp_wait(&bars[B_QKV_FULL], (16 * l + h) & 1, status, abort, lane);
        tc_fence_after();
        // Part p owns head dims [8p, 8p + 8) and [32 + 8p, 40 + 8p) of q, k and v.
        float q[16], kk[16], vv[16];
        const uint32_t tr = tlane + COL_QKV + rc.part * 8;
        tmem_ld8(tr, q);
        tmem_ld8(tr + 32, q + 8);
        tmem_ld8(tr + 64, kk);
        tmem_ld8(tr + 96, kk + 8);
        tmem_ld8(tr + 128, vv);
        tmem_ld8(tr + 160, vv + 8);
        if (h < HEADS - 1) warp_arrive(&bars[B_QKV_FREE], lane);
        // k and v of every row, bf16 (the precision of the reference's autocast attention) for
        // the window-mates, fp32 for the row itself, exchanged through shared memory. A candidate's window rows are lanes of this warp
        // and the part's dims are this warp's, so the exchange needs only warp barriers.
        uint8_t* kvr = sKV + rc.r * KV_ROW;
        const int sw = rc.r & 7;  // 16-byte chunk swizzle of the row
        __syncwarp();             // window-mates are done reading the previous head's k / v
        *reinterpret_cast<uint4*>(kvr + (((2 * rc.part) ^ sw) << 4)) =
            make_uint4(pack_bf16x2(kk[0], kk[1]), pack_bf16x2(kk[2], kk[3]), pack_bf16x2(kk[4], kk[5]),
                       pack_bf16x2(kk[6], kk[7]));
        *reinterpret_cast<uint4*>(kvr + (((2 * rc.part + 1) ^ sw) << 4)) =
            make_uint4(pack_bf16x2(kk[8], kk[9]), pack_bf16x2(kk[10], kk[11]), pack_bf16x2(kk[12], kk[13]),
                       pack_bf16x2(kk[14], kk[15]));
        *reinterpret_cast<uint4*>(kvr + (((8 + 2 * rc.part) ^ sw) << 4)) =
            make_uint4(pack_bf16x2(vv[0], vv[1]), pack_bf16x2(vv[2], vv[3]), pack_bf16x2(vv[4], vv[5]),
                       pack_bf16x2(vv[6], vv[7]));
        *reinterpret_cast<uint4*>(kvr + (((9 + 2 * rc.part) ^ sw) << 4)) =
            make_uint4(pack_bf16x2(vv[8], vv[9]), pack_bf16x2(vv[10], vv[11]), pack_bf16x2(vv[12], vv[13]),
                       pack_bf16x2(vv[14], vv[15]));
        __syncwarp();
        float* sp = spart + (h & 1) * (4 * WIN * 128);  // double-buffered partial scores
        // Partial scores q . k_j over this part's 16 dims for j <= pos (the row's own k from
        // registers, the window-mates' from the exchange).
        {
          float d = 0.f;
#pragma unroll
          for (int t = 0; t < 16; ++t) d = fmaf(q[t], kk[t], d);
          sp[(rc.part * WIN + npos) * 128 + rc.r] = d;
        }
#pragma unroll 1
        for (int jj = 0; jj < npos; ++jj) {
          const int rj = base + jj;
          const uint8_t* kr = sKV + rj * KV_ROW;
          float kf[16];
          unpack8(*reinterpret_cast<const uint4*>(kr + (((2 * rc.part) ^ (rj & 7)) << 4)), kf);
          unpack8(*reinterpret_cast<const uint4*>(kr + (((2 * rc.part + 1) ^ (rj & 7)) << 4)), kf + 8);
          float d = 0.f;
#pragma unroll
          for (int t = 0; t < 16; ++t) d = fmaf(q[t], kf[t], d);
          sp[(rc.part * WIN + jj) * 128 + rc.r] = d;
        }
        bar_quad(quad);
        // One pass of online softmax (scale 1/8 = dim_head^-0.5) and the weighted sum of v.
        float mx = -INFINITY, den = 0.f, o[16];
#pragma unroll
        for (int t = 0; t < 16; ++t) o[t] = 0.f;
#pragma unroll 1
        for (int jj = 0; jj <= npos; ++jj) {
          const float sj = ((sp[(0 * WIN + jj) * 128 + rc.r] + sp[(1 * WIN + jj) * 128 + rc.r]) +
                            (sp[(2 * WIN + jj) * 128 + rc.r] + sp[(3 * WIN + jj) * 128 + rc.r])) *
                           0.125f;
          const float mnew = fmaxf(mx, sj);
          const float sc = __expf(mx - mnew);
          const float pj = __expf(sj - mnew);
          den = den * sc + pj;
          mx = mnew;
          float vf[16];
          if (jj < npos) {
            const int rj = base + jj;
            const uint8_t* vr = sKV + rj * KV_ROW;
            unpack8(*reinterpret_cast<const uint4*>(vr + (((8 + 2 * rc.part) ^ (rj & 7)) << 4)), vf);
            unpack8(*reinterpret_cast<const uint4*>(vr + (((9 + 2 * rc.part) ^ (rj & 7)) << 4)), vf + 8);
          } else {
#pragma unroll
            for (int t = 0; t < 16; ++t) vf[t] = vv[t];
          }
#pragma unroll
          for (int t = 0; t < 16; ++t) o[t] = fmaf(pj, vf[t], o[t] * sc);
        }
        const float inv = rc.valid ? 1.0f / den : 0.f;
        const int b = h & 1;
        if (h >= 2) warp_wait(&bars[B_O_FREE + b], (8 * l + (h - 2) / 2) & 1, status, abort, lane);
        uint8_t* ob = sO + b * A_BLK;
        *reinterpret_cast<uint4*>(ob + sw128_off(rc.r, rc.part * 8)) =
            make_uint4(pack_bf16x2(o[0] * inv, o[1] * inv), pack_bf16x2(o[2] * inv, o[3] * inv),
                       pack_bf16x2(o[4] * inv, o[5] * inv), pack_bf16x2(o[6] * inv, o[7] * inv));
        *reinterpret_cast<uint4*>(ob + sw128_off(rc.r, 32 + rc.part * 8)) =
            make_uint4(pack_bf16x2(o[8] * inv, o[9] * inv), pack_bf16x2(o[10] * inv, o[11] * inv),
                       pack_bf16x2(o[12] * inv, o[13] * inv), pack_bf16x2(o[14] * inv, o[15] * inv));
        warp_arrive(&bars[B_O_READY + b], lane);
      }
      // ---- x += gate_msa * (out-projection + bias)
      warp_wait(&bars[B_OUT_FULL], l & 1, status, abort, lane);
      tc_fence_after();
      residual_update(xr, tstash, tlane + COL_OUT + c0, ml ? ml + 2 * D : nullptr, w.out_b + l * D, rc);
      // ---- feed-forward half: A = ffn.norm(LN2(x) * (1 + scale_mlp) + shift_mlp)
      ln_modulate_operand(xr, tstash, ml ? ml + 3 * D : nullptr, ml ? ml + 4 * D : nullptr, w.ffn_ln_w + l * D,
                          w.ffn_ln_b + l * D, sA, stats, red, rc);
      warp_arrive(&bars[B_A_READY], lane);
      for (int q = 0; q < 4; ++q) {
        warp_wait(&bars[B_FC1_FULL], (4 * l + q) & 1, status, abort, lane);
        tc_fence_after();
        // hidden units 192 q + [48 part, +48): bias, GELU, bf16 (packed, 24 registers)
        uint32_t hp[24];
#pragma unroll
        for (int t = 0; t < 3; ++t) {
          float a[16];
          tmem_ld16(tlane + COL_QKV + c0 + 16 * t, a);
          const float* b1 = w.b1 + l * MLP + 192 * q + c0 + 16 * t;
          float bv[16];
          ldg8(b1, bv);
          ldg8(b1 + 8, bv + 8);
#pragma unroll
          for (int e = 0; e < 16; e += 2)
            hp[8 * t + e / 2] = pack_bf16x2(gelu_f(a[e] + bv[e]), gelu_f(a[e + 1] + bv[e + 1]));
        }
        if (q < 3) warp_arrive(&bars[B_FC1_FREE], lane);
        if (q > 0) warp_wait(&bars[B_HID_FREE], (4 * l + q - 1) & 1, status, abort, lane);
#pragma unroll
        for (int t = 0; t < 6; ++t) {
          const int c = c0 + 8 * t;
          *reinterpret_cast<uint4*>(sHid + (c >> 6) * A_BLK + sw128_off(rc.r, c & 63)) =
              make_uint4(hp[4 * t], hp[4 * t + 1], hp[4 * t + 2], hp[4 * t + 3]);
        }
        warp_arrive(&bars[B_HID_READY], lane);
      }
      // ---- x += gate_mlp * (FC2 + bias)
      warp_wait(&bars[B_HID_FREE], (4 * l + 3) & 1, status, abort, lane);
      tc_fence_after();
      residual_update(xr, tstash, tlane + COL_OUT + c0, ml ? ml + 5 * D : nullptr, w.b2 + l * D, rc);
    }
    // ---- final LayerNorm (lewm/module.py:183) of the window's last row: the call's prediction
    float sum = 0.f;
#pragma unroll
    for (int t = 0; t < 3; ++t) {
      float v[16];
      load_chunk(t, xr, tstash, v);
#pragma unroll
      for (int i = 0; i < 16; ++i) sum += v[i];
    }
    const float mpart = sum * (1.0f / 48);
    float qv = 0.f;
#pragma unroll
    for (int t = 0; t < 3; ++t) {
      float v[16];
      load_chunk(t, xr, tstash, v);
#pragma unroll
      for (int i = 0; i < 16; ++i) qv += (v[i] - mpart) * (v[i] - mpart);
    }
    const float2 mvf = row_moments(mpart, qv, stats, red, rc);
    const float mean = mvf.x, rstd = rsqrtf(mvf.y + 1e-5f);
    const bool out_row = rc.valid && rc.pos == WIN - 1;
    float acc = 0.f;
    const float* gr = nullptr;
    float* dst = nullptr;
    if (out_row) {
      if (p.last)
        gr = p.goal + (size_t)(p.goal_per_cand ? rc.cand : rc.cand / p.S) * D + c0;
      else
        dst = p.pred + ((size_t)rc.cand * p.npred + p.call) * D + c0;
    }
#pragma unroll
    for (int t = 0; t < 3; ++t) {
      float v[16];
      load_chunk(t, xr, tstash, v);
      float fw[16], fb[16];
      ldg8(w.fin_w + c0 + 16 * t, fw);
      ldg8(w.fin_w + c0 + 16 * t + 8, fw + 8);
      ldg8(w.fin_b + c0 + 16 * t, fb);
      ldg8(w.fin_b + c0 + 16 * t + 8, fb + 8);
#pragma unroll
      for (int i = 0; i < 16; ++i) v[i] = fmaf((v[i] - mean) * rstd, fw[i], fb[i]);
      if (gr) {  // cost_from_rollout: squared distance to the goal's last row
#pragma unroll
        for (int i = 0; i < 16; ++i) acc += (v[i] - gr[16 * t + i]) * (v[i] - gr[16 * t + i]);
      }
      if (dst) {
#pragma unroll
        for (int i = 0; i < 16; i += 4)
          *reinterpret_cast<float4*>(dst + 16 * t + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
      }
    }
    if (p.last) {
      const float tot = row_sum(acc, stats, red, rc);
      if (out_row && rc.part == 0) p.costs[rc.cand] = tot;
    }
  }
  // Drain. Normally every copy has been consumed and every MMA has completed by now. After
  // an expired wait, the producer waits (bounded) for the last copy issued into each ring
  // slot to land, and the MMA warp for its MMAs to complete, before shared memory and
  // TMEM are released.
  if (warp == PRODUCER_WARP && lane == 0 && *abort) {
    for (int g = issued - RING > 0 ? issued - RING : 0; g < issued; ++g) {
      const uint64_t t0 = global_timer_ns();
      while (!mbar_try_wait(&bars[B_FULL + g % RING], (g / RING) & 1) &&
             global_timer_ns() - t0 < wait_limit_ns(status)) {
      }
    }
  }
  if (warp == MMA_WARP) {
    if (lane == 0) {
      umma_commit(&bars[B_DRAIN]);
      const uint64_t t0 = global_timer_ns();
      while (!mbar_try_wait(&bars[B_DRAIN], 0) && global_timer_ns() - t0 < wait_limit_ns(status)) {
      }
    }
    __syncwarp();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == MMA_WARP) tmem_dealloc(tmem, 512);
}

cudaError_t launch_tile_call(const DevWeights& w, const TileCallParams& p, cudaStream_t st) {
  const cudaError_t e = cudaFuncSetAttribute(k_tile_call, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
  if (e != cudaSuccess) return e;
  const int tiles = (p.n_cand + 4 * CAND_PER_QUAD - 1) / (4 * CAND_PER_QUAD);
  return launch_k(k_tile_call, dim3(tiles), dim3(THREADS), SMEM_BYTES, st, w, p);
}

int tile_call_candidates_per_tile() { return 4 * CAND_PER_QUAD; }

void tile_call_describe(char* buf, size_t n) {
  cudaFuncAttributes a{};
  cudaFuncGetAttributes(&a, k_tile_call);
  snprintf(buf, n, "k_tile_call: %d registers, max %d threads per block, %d threads, %zu + %d bytes shared memory",
           a.numRegs, a.maxThreadsPerBlock, THREADS, a.sharedSizeBytes, SMEM_BYTES);
}

}  // namespace lewm
