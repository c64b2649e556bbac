// LeWM predictor rollout kernels for sm_100a.
//
// One model-cost evaluation (reference JEPA.get_cost_from_embeddings,
// lewm/jepa.py:302-317) is:
//   k_embed   Embedder (lewm/module.py:205-214) + SiLU for every (candidate, time)
//   k_adaln   AdaLN modulation Linear (lewm/module.py:98-100) for every layer at once;
//             it depends only on the actions, so it is hoisted out of the
//             autoregressive chain and computed once per candidate and time step
//   per predictor call (lewm/jepa.py:284-298), per layer (lewm/module.py:105-111):
//     k_qkv_attn  LN1 -> modulate -> attn.norm -> QKV GEMM (one head per CTA)
//                 -> causal attention over the window (lewm/module.py:75-85)
//     k_resid_gemm (out-proj) GEMM + bias, * gate_msa, + residual
//     k_fc1       LN2 -> modulate -> FFN LayerNorm -> FC1 GEMM + bias -> GELU
//     k_resid_gemm (FC2) GEMM + bias, * gate_mlp, + residual
//   k_final     final LayerNorm (lewm/module.py:183) on each window's last token,
//               then append to the history or score against the goal
//               (cost_from_rollout, lewm/jepa.py:246-260)
//
// GEMMs run on tcgen05 (bf16 in, fp32 accumulate in TMEM); operands arrive in
// shared memory by bulk copy of pre-swizzled blocks; LayerNorm, modulation,
// bias, GELU, gates, residuals and the cost are fp32 in prologues/epilogues.
//
// Latency structure: every kernel is launched with programmatic stream
// serialization. Before griddep_wait() a kernel only initialises barriers,
// allocates TMEM and starts the bulk copies of its weight tiles, so that part
// overlaps the previous kernel. Row work (LayerNorm prologues, attention) is
// split over several threads per row and accumulator columns over the four
// warps that share a TMEM lane quadrant, so no thread walks a long serial chain.
#include <algorithm>

#include "lewm_common.cuh"
#include "lewm_internal.h"

namespace lewm {
namespace {

constexpr int kBlk = 16384;           // bytes of one [128 x 64] bf16 block
constexpr int kBlkElems = 128 * 64;   // elements of one [128 x 64] block
constexpr int kMaxWindow = 8;
constexpr int kScratchStride = 193;   // floats per row of the q|k|v scratch
constexpr int kThreads = 512;         // 16 warps: 4 per TMEM lane quadrant

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

template <int D>
struct Cfg {
  static constexpr int KB = D / 64;
  static constexpr int NT_OUT = D / 4;            // out-proj / FC2 N tile (4 tiles per row block)
  static constexpr int NT_ADA = (D == 192) ? 192 : 128;
  static constexpr int TMEM_OUT = (NT_OUT <= 64) ? 64 : 128;
  static constexpr int TMEM_EMB = (D <= 256) ? 256 : 512;
  static constexpr int QKV_ST = (KB < 3) ? KB : 3;
  static constexpr int RES_ST = 6;                // K-ring depth of the streamed-A GEMMs
  static constexpr int TPR = D / 48;              // LayerNorm threads per row (48 columns each)
  static constexpr int RPP = kThreads / TPR;      // rows per LayerNorm pass
};

struct RowMap {
  bool valid;
  int cand, pos, tok;  // tok = cand*T + history index
};
__device__ __forceinline__ RowMap map_row(const CallGeom& g, int tile, int r) {
  RowMap m;
  const int cl = r / g.w;
  m.pos = r - cl * g.w;
  m.cand = tile * g.cpt + cl;
  m.valid = (cl < g.cpt) && (m.cand < g.n_cand);
  m.tok = m.cand * g.T + g.start + m.pos;
  return m;
}

// ---------------------------------------------------------------- row prologue
// TPR threads per row; thread q holds float4 chunks j = q + TPR*i (i < 12), i.e.
// columns 4j..4j+3. A-row (bf16, swizzled) = LN_affine(LN(x)*(1+scale)+shift).
// Every lane runs the group shuffles; invalid rows compute on zeros and store zeros.
template <int D>
__device__ __forceinline__ void ln_mod_ln_part(bool valid, const float* __restrict__ xrow,
                                               const float* __restrict__ addrow,
                                               const __nv_bfloat16* __restrict__ shift,
                                               const __nv_bfloat16* __restrict__ scale,
                                               const float* __restrict__ g, const float* __restrict__ bb,
                                               uint8_t* a_smem, int r, int q, float* __restrict__ xout) {
  constexpr int TPR = Cfg<D>::TPR;
  constexpr int NC = 12;
  float4 v[NC];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < NC; ++i) {
    const int c = 4 * (q + TPR * i);
    float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
    if (valid) {
      t = *reinterpret_cast<const float4*>(xrow + c);
      if (addrow) {
        const float4 a = *reinterpret_cast<const float4*>(addrow + c);
        t.x += a.x;
        t.y += a.y;
        t.z += a.z;
        t.w += a.w;
      }
      if (xout) *reinterpret_cast<float4*>(xout + c) = t;
    }
    v[i] = t;
    s += (t.x + t.y) + (t.z + t.w);
  }
#pragma unroll
  for (int o = TPR / 2; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  const float mean = s * (1.0f / D);
  float q2 = 0.f;
#pragma unroll
  for (int i = 0; i < NC; ++i) {
    const float a = v[i].x - mean, b = v[i].y - mean, c = v[i].z - mean, d = v[i].w - mean;
    q2 += (a * a + b * b) + (c * c + d * d);
  }
#pragma unroll
  for (int o = TPR / 2; o > 0; o >>= 1) q2 += __shfl_xor_sync(0xffffffffu, q2, o);
  const float rstd = rsqrtf(q2 * (1.0f / D) + 1e-6f);
  float s2 = 0.f;
#pragma unroll
  for (int i = 0; i < NC; ++i) {
    const int c = 4 * (q + TPR * i);
    float2 sh01 = make_float2(0.f, 0.f), sh23 = sh01, sc01 = sh01, sc23 = sh01;
    if (valid) {
      const uint2 sh = *reinterpret_cast<const uint2*>(shift + c);
      const uint2 sc = *reinterpret_cast<const uint2*>(scale + c);
      sh01 = unpack_bf16x2(sh.x);
      sh23 = unpack_bf16x2(sh.y);
      sc01 = unpack_bf16x2(sc.x);
      sc23 = unpack_bf16x2(sc.y);
    }
    v[i].x = (v[i].x - mean) * rstd * (1.0f + sc01.x) + sh01.x;
    v[i].y = (v[i].y - mean) * rstd * (1.0f + sc01.y) + sh01.y;
    v[i].z = (v[i].z - mean) * rstd * (1.0f + sc23.x) + sh23.x;
    v[i].w = (v[i].w - mean) * rstd * (1.0f + sc23.y) + sh23.y;
    s2 += (v[i].x + v[i].y) + (v[i].z + v[i].w);
  }
#pragma unroll
  for (int o = TPR / 2; o > 0; o >>= 1) s2 += __shfl_xor_sync(0xffffffffu, s2, o);
  const float mean2 = s2 * (1.0f / D);
  float q3 = 0.f;
#pragma unroll
  for (int i = 0; i < NC; ++i) {
    const float a = v[i].x - mean2, b = v[i].y - mean2, c = v[i].z - mean2, d = v[i].w - mean2;
    q3 += (a * a + b * b) + (c * c + d * d);
  }
#pragma unroll
  for (int o = TPR / 2; o > 0; o >>= 1) q3 += __shfl_xor_sync(0xffffffffu, q3, o);
  const float rstd2 = rsqrtf(q3 * (1.0f / D) + 1e-5f);
#pragma unroll
  for (int i = 0; i < NC; ++i) {
    const int c = 4 * (q + TPR * i);
    uint2 out = make_uint2(0u, 0u);
    if (valid) {
      const float4 gg = *reinterpret_cast<const float4*>(g + c);
      const float4 b4 = *reinterpret_cast<const float4*>(bb + c);
      out.x = pack_bf16x2((v[i].x - mean2) * rstd2 * gg.x + b4.x, (v[i].y - mean2) * rstd2 * gg.y + b4.y);
      out.y = pack_bf16x2((v[i].z - mean2) * rstd2 * gg.z + b4.z, (v[i].w - mean2) * rstd2 * gg.w + b4.w);
    }
    *reinterpret_cast<uint2*>(a_smem + (c >> 6) * kBlk + sw128_off(r, c & 63)) = out;
  }
}

// ---------------------------------------------------------------- Embedder + SiLU
// act_a[row] = bf16(SiLU(Linear2(SiLU(Linear1(Conv1x1(a)))))), rows = candidate*T + t.
template <int D>
__global__ void __launch_bounds__(256) k_embed(DevWeights w, ModelDims md, const float* __restrict__ cand, int rows,
                                               __nv_bfloat16* __restrict__ act_a, uint32_t* status) {
  using C = Cfg<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* sA1 = smem;                     // 2 blocks [128 x 64]
  uint8_t* sB = smem + 2 * kBlk;           // 2 blocks [D x 64]
  uint8_t* sOut = smem;                    // KB blocks, aliases sA1/sB after the last MMA
  float* actc = reinterpret_cast<float*>(smem + 2 * kBlk + 2 * D * 128);  // [128][16]
  uint64_t* bars = reinterpret_cast<uint64_t*>(actc + 128 * 16);
  uint64_t* bar_b = bars;
  uint64_t* bar_mma = bars + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2);

  const int tid = threadIdx.x, warp = tid >> 5;
  const int row0 = blockIdx.x * 128;
  if (tid == 0) {
    mbar_init(bar_b, 1);
    mbar_init(bar_mma, 1);
    fence_mbar_init();
    mbar_arrive_expect_tx(bar_b, 2 * D * 128);
    bulk_g2s(sB, w.we2, D * 128, bar_b);
    bulk_g2s(sB + D * 128, w.we2 + (size_t)D * 64, D * 128, bar_b);
  }
  __syncwarp();
  if (warp == 0) {
    tmem_alloc(tmem_slot, C::TMEM_EMB);
    tmem_relinquish();
  }
  griddep_wait();
  griddep_launch();
  for (int idx = tid; idx < 128 * 16; idx += 256) {
    const int r = idx >> 4, o = idx & 15;
    const int row = row0 + r;
    float v = 0.f;
    if (o < md.As && row < rows) {
      v = w.conv_b[o];
      const float* a = cand + (size_t)row * md.A;
      for (int i = 0; i < md.A; ++i) v += w.conv_w[o * md.A + i] * a[i];
    }
    actc[idx] = v;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int nch = md.eh / 128;
  bool ok = true;
  for (int c = 0; c < nch; ++c) {
    if (c > 0) {
      ok = mbar_wait(bar_mma, (c - 1) & 1, status) && ok;
      if (tid == 0) {
        mbar_arrive_expect_tx(bar_b, 2 * D * 128);
        bulk_g2s(sB, w.we2 + (size_t)(c * 2) * D * 64, D * 128, bar_b);
        bulk_g2s(sB + D * 128, w.we2 + (size_t)(c * 2 + 1) * D * 64, D * 128, bar_b);
      }
    }
    {
      const int k = tid & 127;
      const int hk = c * 128 + k;
      float wv[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) wv[i] = (i < md.As) ? w.e1_w[hk * md.As + i] : 0.f;
      const float bias = w.e1_b[hk];
      uint8_t* blk = sA1 + (k >> 6) * kBlk;
      for (int r = tid >> 7; r < 128; r += 2) {
        float acc = bias;
#pragma unroll
        for (int i = 0; i < 16; ++i) acc += wv[i] * actc[r * 16 + i];
        *reinterpret_cast<__nv_bfloat16*>(blk + sw128_off(r, k & 63)) = __float2bfloat16_rn(silu_f(acc));
      }
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (tid == 0) {
      if (mbar_wait(bar_b, c & 1, status)) {
        tc_fence_after();
        const uint32_t idesc = idesc_bf16(128, 192);
        for (int kb = 0; kb < 2; ++kb) {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint64_t ad = sdesc_sw128(smem_u32(sA1) + kb * kBlk + j * 32);
#pragma unroll
            for (int nh = 0; nh < D / 192; ++nh) {
              const uint64_t bd = sdesc_sw128(smem_u32(sB) + kb * D * 128 + nh * 192 * 128 + j * 32);
              umma_bf16(tmem + nh * 192, ad, bd, idesc, (c | kb | j) ? 1u : 0u);
            }
          }
        }
      }
      umma_commit(bar_mma);
    }
  }
  ok = mbar_wait(bar_mma, (nch - 1) & 1, status) && ok;
  __syncwarp();
  tc_fence_after();
  {
    const int r = tid & 127;
    const int half = tid >> 7;
    const uint32_t taddr = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    const bool valid = ok && (row0 + r < rows);
    for (int c0 = half * (D / 2); c0 < (half + 1) * (D / 2); c0 += 16) {
      float v[16];
      tmem_ld16(taddr + c0, v);
#pragma unroll
      for (int i = 0; i < 16; i += 2) {
        const int c = c0 + i;
        const float a0 = valid ? silu_f(v[i] + w.e2_b[c]) : 0.f;
        const float a1 = valid ? silu_f(v[i + 1] + w.e2_b[c + 1]) : 0.f;
        *reinterpret_cast<uint32_t*>(sOut + (c >> 6) * kBlk + sw128_off(r, c & 63)) = pack_bf16x2(a0, a1);
      }
    }
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  if (tid == 0) {
    for (int kb = 0; kb < C::KB; ++kb)
      bulk_s2g(act_a + ((size_t)blockIdx.x * C::KB + kb) * kBlkElems, sOut + kb * kBlk, kBlk);
    bulk_commit();
    bulk_wait_all();
  }
  __syncwarp();
  if (warp == 0) tmem_dealloc(tmem, C::TMEM_EMB);
}

// ---------------------------------------------------------------- AdaLN modulation
// mod[row, n] = bf16(act_a[row] . Wada[n] + b[n]) for n over all layers' 6*D outputs.
template <int D>
__global__ void __launch_bounds__(kThreads) k_adaln(DevWeights w, ModelDims md, int rows,
                                                    const __nv_bfloat16* __restrict__ act_a,
                                                    __nv_bfloat16* __restrict__ mod, uint32_t* status) {
  using C = Cfg<D>;
  constexpr int NT = C::NT_ADA;
  constexpr int CW = NT / 4;  // columns per warp
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* sA = smem;
  uint8_t* sB = smem + C::KB * kBlk;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sB + C::KB * NT * 128);  // [0] weights, [1] mma, [2] act
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 3);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int tile = blockIdx.x, nt = blockIdx.y;
  if (tid == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    mbar_init(&bars[2], 1);
    fence_mbar_init();
    mbar_arrive_expect_tx(&bars[0], C::KB * NT * 128);
    for (int kb = 0; kb < C::KB; ++kb)
      bulk_g2s(sB + kb * NT * 128, w.wada + ((size_t)nt * C::KB + kb) * NT * 64, NT * 128, &bars[0]);
  }
  __syncwarp();
  if (warp == 0) {
    tmem_alloc(tmem_slot, 256);
    tmem_relinquish();
  }
  griddep_wait();
  griddep_launch();
  if (tid == 0) {
    mbar_arrive_expect_tx(&bars[2], C::KB * kBlk);
    for (int kb = 0; kb < C::KB; ++kb)
      bulk_g2s(sA + kb * kBlk, act_a + ((size_t)tile * C::KB + kb) * kBlkElems, kBlk, &bars[2]);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (tid == 0) {
    if (mbar_wait(&bars[0], 0, status) && mbar_wait(&bars[2], 0, status)) {
      tc_fence_after();
      umma_tile(tmem, smem_u32(sA), kBlk, smem_u32(sB), NT * 128, 0, C::KB, idesc_bf16(128, NT), false);
    }
    umma_commit(&bars[1]);
  }
  const bool ok = mbar_wait(&bars[1], 0, status);
  __syncwarp();
  tc_fence_after();
  const int quad = warp & 3, slice = warp >> 2;
  const int row = tile * 128 + quad * 32 + lane;
  const int ncols = md.L * 6 * D;
  const uint32_t taddr = tmem + ((uint32_t)(quad * 32) << 16) + slice * CW;
  float v[CW];
  tmem_ld_cols<CW>(taddr, v);
  if (ok && row < rows) {
    const int n0 = nt * NT + slice * CW;
    uint4* dst = reinterpret_cast<uint4*>(mod + (size_t)row * ncols + n0);
#pragma unroll
    for (int i = 0; i < CW / 8; ++i) {
      uint32_t pk[4];
#pragma unroll
      for (int k = 0; k < 4; ++k)
        pk[k] = pack_bf16x2(v[8 * i + 2 * k] + w.ada_b[n0 + 8 * i + 2 * k],
                            v[8 * i + 2 * k + 1] + w.ada_b[n0 + 8 * i + 2 * k + 1]);
      dst[i] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
    }
  }
  tc_fence_before();
  __syncthreads();
  __syncwarp();
  if (warp == 0) tmem_dealloc(tmem, 256);
}

// ---------------------------------------------------------------- QKV + attention
template <int D>
__global__ void __launch_bounds__(kThreads) k_qkv_attn(DevWeights w, ModelDims md, CallGeom g, RolloutBufs b,
                                                       int layer, uint32_t* status) {
  using C = Cfg<D>;
  constexpr int KB = C::KB;
  constexpr int ST = C::QKV_ST;
  constexpr int B_BLK = 192 * 128;
  constexpr int R1 = KB * kBlk + ST * B_BLK;
  constexpr int SCR = 128 * kScratchStride * 4;
  constexpr int R1S = ((R1 > SCR ? R1 : SCR) + 1023) & ~1023;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* sA = smem;
  uint8_t* sB = smem + KB * kBlk;
  float* scr = reinterpret_cast<float*>(smem);  // aliases sA/sB after the MMA
  uint8_t* sO = smem + R1S;
  uint64_t* full = reinterpret_cast<uint64_t*>(sO + kBlk);
  uint64_t* empty = full + ST;
  uint64_t* bar_mma = empty + ST;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_mma + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int tile = blockIdx.x, head = blockIdx.y;
  const __nv_bfloat16* wq = w.qkv + (size_t)((layer * md.heads + head) * KB) * (192 * 64);
  const int ncols = md.L * 6 * D;

  if (tid == 0) {
    for (int s = 0; s < ST; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(bar_mma, 1);
    fence_mbar_init();
    for (int s = 0; s < ST; ++s) {
      mbar_arrive_expect_tx(&full[s], B_BLK);
      bulk_g2s(sB + s * B_BLK, wq + (size_t)s * 192 * 64, B_BLK, &full[s]);
    }
  }
  __syncwarp();
  if (warp == 0) {
    tmem_alloc(tmem_slot, 256);
    tmem_relinquish();
  }
  griddep_wait();
  griddep_launch();
  // Prologue: window rows -> LN1 -> modulate(shift_msa, scale_msa) -> attn.norm -> bf16 A.
  const int NPRED = g.T - g.H + 1;
  for (int r = tid / C::TPR; r < 128; r += C::RPP) {
    const int q = tid % C::TPR;
    const RowMap m = map_row(g, tile, r);
    const __nv_bfloat16* mrow = b.mod + (size_t)(m.valid ? m.tok : 0) * ncols + layer * 6 * D;
    float* xdst = b.x + ((size_t)tile * 128 + r) * D;
    if (layer == 0) {
      const float* src = b.emb;
      if (m.valid) {
        const int j = g.start + m.pos;
        if (j < g.H) {
          const int e = b.emb_per_cand ? m.cand : (m.cand / g.S);
          src = b.emb + ((size_t)e * g.H + j) * D;
        } else {
          src = b.pred + ((size_t)m.cand * NPRED + (j - g.H)) * D;
        }
      }
      ln_mod_ln_part<D>(m.valid, src, w.pos + m.pos * D, mrow, mrow + D, w.attn_ln_w + layer * D,
                        w.attn_ln_b + layer * D, sA, r, q, head == 0 ? xdst : nullptr);
    } else {
      ln_mod_ln_part<D>(m.valid, xdst, nullptr, mrow, mrow + D, w.attn_ln_w + layer * D, w.attn_ln_b + layer * D,
                        sA, r, q, nullptr);
    }
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (tid == 0) {
    const uint32_t idesc = idesc_bf16(128, 192);
    for (int kb = 0; kb < KB; ++kb) {
      const int s = kb % ST;
      if (!mbar_wait(&full[s], (kb / ST) & 1, status)) break;
      tc_fence_after();
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint64_t ad = sdesc_sw128(smem_u32(sA) + kb * kBlk + j * 32);
        const uint64_t bd = sdesc_sw128(smem_u32(sB) + s * B_BLK + j * 32);
        umma_bf16(tmem, ad, bd, idesc, (kb | j) ? 1u : 0u);
      }
      umma_commit(&empty[s]);
      if (kb + ST < KB) {
        if (!mbar_wait(&empty[s], (kb / ST) & 1, status)) break;
        mbar_arrive_expect_tx(&full[s], B_BLK);
        bulk_g2s(sB + s * B_BLK, wq + (size_t)(kb + ST) * 192 * 64, B_BLK, &full[s]);
      }
    }
    umma_commit(bar_mma);
  }
  const bool ok = mbar_wait(bar_mma, 0, status);
  __syncwarp();
  tc_fence_after();
  {  // q|k|v of this head -> scratch rows (fp32); warp slice s owns columns [48s, 48s+48)
    const int quad = warp & 3, slice = warp >> 2;
    const int r = quad * 32 + lane;
    const uint32_t taddr = tmem + ((uint32_t)(quad * 32) << 16) + slice * 48;
    float v[48];
    tmem_ld_cols<48>(taddr, v);
    float* srow = scr + r * kScratchStride + slice * 48;
#pragma unroll
    for (int i = 0; i < 48; ++i) srow[i] = v[i];
  }
  __syncthreads();
  {  // causal softmax(q k^T / 8) v within the candidate's window; 4 threads per row, 16 dims each
    const int r = tid >> 2, part = tid & 3;
    const RowMap m = map_row(g, tile, r);
    const bool valid = ok && m.valid;
    const int base = r - m.pos;
    const float* qr = scr + r * kScratchStride + part * 16;
    float sc[kMaxWindow];
    float mx = -INFINITY;
    for (int j = 0; j < g.w; ++j) {
      float d = 0.f;
      if (valid && j <= m.pos) {
        const float* kr = scr + (base + j) * kScratchStride + 64 + part * 16;
#pragma unroll
        for (int t = 0; t < 16; ++t) d += qr[t] * kr[t];
      }
      d += __shfl_xor_sync(0xffffffffu, d, 1);
      d += __shfl_xor_sync(0xffffffffu, d, 2);
      sc[j] = d * 0.125f;
      if (j <= m.pos) mx = fmaxf(mx, sc[j]);
    }
    float den = 0.f;
    for (int j = 0; j < g.w; ++j) {
      sc[j] = (j <= m.pos) ? expf(sc[j] - mx) : 0.f;
      den += sc[j];
    }
    const float inv = 1.0f / den;
    float o[16];
#pragma unroll
    for (int t = 0; t < 16; ++t) o[t] = 0.f;
    if (valid) {
      for (int j = 0; j <= m.pos; ++j) {
        const float* vr = scr + (base + j) * kScratchStride + 128 + part * 16;
#pragma unroll
        for (int t = 0; t < 16; ++t) o[t] += sc[j] * vr[t];
      }
    }
    uint4 lo, hi;
    lo.x = pack_bf16x2(o[0] * inv, o[1] * inv);
    lo.y = pack_bf16x2(o[2] * inv, o[3] * inv);
    lo.z = pack_bf16x2(o[4] * inv, o[5] * inv);
    lo.w = pack_bf16x2(o[6] * inv, o[7] * inv);
    hi.x = pack_bf16x2(o[8] * inv, o[9] * inv);
    hi.y = pack_bf16x2(o[10] * inv, o[11] * inv);
    hi.z = pack_bf16x2(o[12] * inv, o[13] * inv);
    hi.w = pack_bf16x2(o[14] * inv, o[15] * inv);
    if (!valid) lo = hi = make_uint4(0u, 0u, 0u, 0u);
    *reinterpret_cast<uint4*>(sO + sw128_off(r, part * 16)) = lo;
    *reinterpret_cast<uint4*>(sO + sw128_off(r, part * 16 + 8)) = hi;
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  if (tid == 0) {
    bulk_s2g(b.attn + ((size_t)tile * md.heads + head) * kBlkElems, sO, kBlk);
    bulk_commit();
    bulk_wait_all();
  }
  __syncwarp();
  if (warp == 0) tmem_dealloc(tmem, 256);
}

// ---------------------------------------------------------------- streamed-K GEMM with residual epilogue
// x[:, n-tile] += gate * (A . B^T + bias), A streamed from pre-swizzled global tiles.
// Used for the attention out-projection (gate_msa) and FC2 (gate_mlp).
template <int D>
__global__ void __launch_bounds__(kThreads) k_resid_gemm(const __nv_bfloat16* __restrict__ gA, int nkb,
                                                         const __nv_bfloat16* __restrict__ gB,
                                                         const float* __restrict__ bias, int gate_chunk, CallGeom g,
                                                         RolloutBufs b, ModelDims md, int layer, uint32_t* status) {
  using C = Cfg<D>;
  constexpr int NT = C::NT_OUT;
  constexpr int CW = NT / 4;
  constexpr int ST = C::RES_ST;
  constexpr int B_BLK = NT * 128;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* sA = smem;
  uint8_t* sB = smem + ST * kBlk;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + ST * B_BLK);
  uint64_t* empty = full + ST;
  uint64_t* bar_mma = empty + ST;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_mma + 1);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int tile = blockIdx.x, nt = blockIdx.y;
  const __nv_bfloat16* tA = gA + (size_t)tile * nkb * kBlkElems;
  const __nv_bfloat16* tB = gB + (size_t)nt * nkb * NT * 64;
  const int pre = ST < nkb ? ST : nkb;
  if (tid == 0) {
    for (int s = 0; s < ST; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(bar_mma, 1);
    fence_mbar_init();
    for (int s = 0; s < pre; ++s) {  // weights first: they do not depend on the previous kernel
      mbar_arrive_expect_tx(&full[s], kBlk + B_BLK);
      bulk_g2s(sB + s * B_BLK, tB + (size_t)s * NT * 64, B_BLK, &full[s]);
    }
  }
  __syncwarp();
  if (warp == 0) {
    tmem_alloc(tmem_slot, C::TMEM_OUT);
    tmem_relinquish();
  }
  griddep_wait();
  griddep_launch();
  if (tid == 0)
    for (int s = 0; s < pre; ++s) bulk_g2s(sA + s * kBlk, tA + (size_t)s * kBlkElems, kBlk, &full[s]);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (tid == 0) {
    const uint32_t idesc = idesc_bf16(128, NT);
    for (int kb = 0; kb < nkb; ++kb) {
      const int s = kb % ST;
      if (!mbar_wait(&full[s], (kb / ST) & 1, status)) break;
      tc_fence_after();
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint64_t ad = sdesc_sw128(smem_u32(sA) + s * kBlk + j * 32);
        const uint64_t bd = sdesc_sw128(smem_u32(sB) + s * B_BLK + j * 32);
        umma_bf16(tmem, ad, bd, idesc, (kb | j) ? 1u : 0u);
      }
      umma_commit(&empty[s]);
      // Refill the stage the previous MMA group used once that group is done.
      if (kb >= 1 && kb - 1 + ST < nkb) {
        const int ps = (kb - 1) % ST;
        if (!mbar_wait(&empty[ps], ((kb - 1) / ST) & 1, status)) break;
        const int nk = kb - 1 + ST;
        mbar_arrive_expect_tx(&full[ps], kBlk + B_BLK);
        bulk_g2s(sA + ps * kBlk, tA + (size_t)nk * kBlkElems, kBlk, &full[ps]);
        bulk_g2s(sB + ps * B_BLK, tB + (size_t)nk * NT * 64, B_BLK, &full[ps]);
      }
    }
    umma_commit(bar_mma);
  }
  const bool ok = mbar_wait(bar_mma, 0, status);
  __syncwarp();
  tc_fence_after();
  const int quad = warp & 3, slice = warp >> 2;
  const int r = quad * 32 + lane;
  const RowMap m = map_row(g, tile, r);
  const uint32_t taddr = tmem + ((uint32_t)(quad * 32) << 16) + slice * CW;
  float v[CW];
  tmem_ld_cols<CW>(taddr, v);
  if (ok && m.valid) {
    const int ncols = md.L * 6 * D;
    const int c0 = nt * NT + slice * CW;
    float* xrow = b.x + ((size_t)tile * 128 + r) * D + c0;
    const __nv_bfloat16* gate = b.mod + (size_t)m.tok * ncols + layer * 6 * D + gate_chunk * D + c0;
    const float* bs = bias + c0;
#pragma unroll
    for (int i = 0; i < CW; i += 4) {
      const uint2 gt = *reinterpret_cast<const uint2*>(gate + i);
      const float2 g01 = unpack_bf16x2(gt.x), g23 = unpack_bf16x2(gt.y);
      const float4 b4 = *reinterpret_cast<const float4*>(bs + i);
      float4 xv = *reinterpret_cast<float4*>(xrow + i);
      xv.x += g01.x * (v[i] + b4.x);
      xv.y += g01.y * (v[i + 1] + b4.y);
      xv.z += g23.x * (v[i + 2] + b4.z);
      xv.w += g23.y * (v[i + 3] + b4.w);
      *reinterpret_cast<float4*>(xrow + i) = xv;
    }
  }
  tc_fence_before();
  __syncthreads();
  __syncwarp();
  if (warp == 0) tmem_dealloc(tmem, C::TMEM_OUT);
}

// ---------------------------------------------------------------- FC1 + GELU
template <int D>
__global__ void __launch_bounds__(kThreads) k_fc1(DevWeights w, ModelDims md, CallGeom g, RolloutBufs b, int layer,
                                                  uint32_t* status) {
  using C = Cfg<D>;
  constexpr int KB = C::KB;
  constexpr int ST = C::QKV_ST;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* sA = smem;
  uint8_t* sB = smem + KB * kBlk;
  uint8_t* sO = smem;  // 2 blocks, aliases sA after the MMA
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + ST * kBlk);
  uint64_t* empty = full + ST;
  uint64_t* bar_mma = empty + ST;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_mma + 1);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int tile = blockIdx.x, nt = blockIdx.y;
  const int nmlp = md.mlp / 128;
  const __nv_bfloat16* wb = w.w1 + (size_t)((layer * nmlp + nt) * KB) * kBlkElems;
  const int ncols = md.L * 6 * D;
  if (tid == 0) {
    for (int s = 0; s < ST; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(bar_mma, 1);
    fence_mbar_init();
    for (int s = 0; s < ST; ++s) {
      mbar_arrive_expect_tx(&full[s], kBlk);
      bulk_g2s(sB + s * kBlk, wb + (size_t)s * kBlkElems, kBlk, &full[s]);
    }
  }
  __syncwarp();
  if (warp == 0) {
    tmem_alloc(tmem_slot, 128);
    tmem_relinquish();
  }
  griddep_wait();
  griddep_launch();
  for (int r = tid / C::TPR; r < 128; r += C::RPP) {
    const int q = tid % C::TPR;
    const RowMap m = map_row(g, tile, r);
    const __nv_bfloat16* mrow = b.mod + (size_t)(m.valid ? m.tok : 0) * ncols + layer * 6 * D;
    ln_mod_ln_part<D>(m.valid, b.x + ((size_t)tile * 128 + r) * D, nullptr, mrow + 3 * D, mrow + 4 * D,
                      w.ffn_ln_w + layer * D, w.ffn_ln_b + layer * D, sA, r, q, nullptr);
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (tid == 0) {
    const uint32_t idesc = idesc_bf16(128, 128);
    for (int kb = 0; kb < KB; ++kb) {
      const int s = kb % ST;
      if (!mbar_wait(&full[s], (kb / ST) & 1, status)) break;
      tc_fence_after();
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint64_t ad = sdesc_sw128(smem_u32(sA) + kb * kBlk + j * 32);
        const uint64_t bd = sdesc_sw128(smem_u32(sB) + s * kBlk + j * 32);
        umma_bf16(tmem, ad, bd, idesc, (kb | j) ? 1u : 0u);
      }
      umma_commit(&empty[s]);
      if (kb + ST < KB) {
        if (!mbar_wait(&empty[s], (kb / ST) & 1, status)) break;
        mbar_arrive_expect_tx(&full[s], kBlk);
        bulk_g2s(sB + s * kBlk, wb + (size_t)(kb + ST) * kBlkElems, kBlk, &full[s]);
      }
    }
    umma_commit(bar_mma);
  }
  const bool ok = mbar_wait(bar_mma, 0, status);
  __syncwarp();
  tc_fence_after();
  {  // warp slice s owns hidden columns [32s, 32s+32) of this 128-wide chunk
    const int quad = warp & 3, slice = warp >> 2;
    const int r = quad * 32 + lane;
    const RowMap m = map_row(g, tile, r);
    const bool valid = ok && m.valid;
    const uint32_t taddr = tmem + ((uint32_t)(quad * 32) << 16) + slice * 32;
    const float* bs = w.b1 + layer * md.mlp + nt * 128 + slice * 32;
    float v[32];
    tmem_ld_cols<32>(taddr, v);
#pragma unroll
    for (int i = 0; i < 32; i += 8) {
      uint4 pk = make_uint4(0u, 0u, 0u, 0u);
      if (valid) {
        pk.x = pack_bf16x2(gelu_f(v[i] + bs[i]), gelu_f(v[i + 1] + bs[i + 1]));
        pk.y = pack_bf16x2(gelu_f(v[i + 2] + bs[i + 2]), gelu_f(v[i + 3] + bs[i + 3]));
        pk.z = pack_bf16x2(gelu_f(v[i + 4] + bs[i + 4]), gelu_f(v[i + 5] + bs[i + 5]));
        pk.w = pack_bf16x2(gelu_f(v[i + 6] + bs[i + 6]), gelu_f(v[i + 7] + bs[i + 7]));
      }
      const int c = slice * 32 + i;
      *reinterpret_cast<uint4*>(sO + (c >> 6) * kBlk + sw128_off(r, c & 63)) = pk;
    }
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  if (tid == 0) {
    const int nkm = md.mlp / 64;
    bulk_s2g(b.h + ((size_t)tile * nkm + 2 * nt) * kBlkElems, sO, kBlk);
    bulk_s2g(b.h + ((size_t)tile * nkm + 2 * nt + 1) * kBlkElems, sO + kBlk, kBlk);
    bulk_commit();
    bulk_wait_all();
  }
  __syncwarp();
  if (warp == 0) tmem_dealloc(tmem, 128);
}

// ---------------------------------------------------------------- final LayerNorm + history / cost
template <int D>
__global__ void __launch_bounds__(128) k_final(DevWeights w, CallGeom g, RolloutBufs b) {
  griddep_wait();
  griddep_launch();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cand = blockIdx.x * 4 + warp;
  if (cand >= g.n_cand) return;
  const int tile = cand / g.cpt;
  const int r = (cand - tile * g.cpt) * g.w + (g.w - 1);
  const float* xr = b.x + ((size_t)tile * 128 + r) * D;
  constexpr int NP = D / 64;
  float2 v[NP];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < NP; ++i) {
    v[i] = *reinterpret_cast<const float2*>(xr + 64 * i + 2 * lane);
    s += v[i].x + v[i].y;
  }
  const float mean = warp_sum(s) * (1.0f / D);
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < NP; ++i) {
    const float dx = v[i].x - mean, dy = v[i].y - mean;
    q += dx * dx + dy * dy;
  }
  const float rstd = rsqrtf(warp_sum(q) * (1.0f / D) + 1e-5f);
#pragma unroll
  for (int i = 0; i < NP; ++i) {
    const int c = 64 * i + 2 * lane;
    v[i].x = (v[i].x - mean) * rstd * w.fin_w[c] + w.fin_b[c];
    v[i].y = (v[i].y - mean) * rstd * w.fin_w[c + 1] + w.fin_b[c + 1];
  }
  if (g.last) {
    const int e = b.goal_per_cand ? cand : cand / g.S;
    const float* gr = b.goal + (size_t)e * D;
    float acc = 0.f;
#pragma unroll
    for (int i = 0; i < NP; ++i) {
      const int c = 64 * i + 2 * lane;
      const float dx = v[i].x - gr[c], dy = v[i].y - gr[c + 1];
      acc += dx * dx + dy * dy;
    }
    acc = warp_sum(acc);
    if (lane == 0) b.costs[cand] = acc;
  } else {
    const int NPred = g.T - g.H + 1;
    float* dst = b.pred + ((size_t)cand * NPred + g.call) * D;
#pragma unroll
    for (int i = 0; i < NP; ++i) *reinterpret_cast<float2*>(dst + 64 * i + 2 * lane) = v[i];
  }
}

// ---------------------------------------------------------------- shared-memory sizes
template <int D>
constexpr int smem_embed() { return 1024 + 2 * kBlk + 2 * D * 128 + 128 * 16 * 4 + 64; }
template <int D>
constexpr int smem_adaln() { return 1024 + Cfg<D>::KB * (kBlk + Cfg<D>::NT_ADA * 128) + 64; }
template <int D>
constexpr int smem_qkv() {
  constexpr int R1 = Cfg<D>::KB * kBlk + Cfg<D>::QKV_ST * 192 * 128;
  constexpr int SCR = 128 * kScratchStride * 4;
  constexpr int R1S = ((R1 > SCR ? R1 : SCR) + 1023) & ~1023;
  return 1024 + R1S + kBlk + 128;
}
template <int D>
constexpr int smem_resid() { return 1024 + Cfg<D>::RES_ST * (kBlk + Cfg<D>::NT_OUT * 128) + 128; }
template <int D>
constexpr int smem_fc1() { return 1024 + Cfg<D>::KB * kBlk + Cfg<D>::QKV_ST * kBlk + 128; }

static_assert(smem_qkv<192>() <= 232448 && smem_qkv<384>() <= 232448, "qkv smem");
static_assert(smem_embed<384>() <= 232448 && smem_adaln<384>() <= 232448, "embed/adaln smem");
static_assert(smem_fc1<384>() <= 232448 && smem_resid<384>() <= 232448, "fc smem");

template <int D>
cudaError_t set_smem_attrs() {
  static bool done = false;  // per process; attributes are per device function
  if (done) return cudaSuccess;
  cudaError_t e;
  if ((e = cudaFuncSetAttribute(k_embed<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_embed<D>()))) return e;
  if ((e = cudaFuncSetAttribute(k_adaln<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_adaln<D>()))) return e;
  if ((e = cudaFuncSetAttribute(k_qkv_attn<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_qkv<D>()))) return e;
  if ((e = cudaFuncSetAttribute(k_resid_gemm<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_resid<D>())))
    return e;
  if ((e = cudaFuncSetAttribute(k_fc1<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_fc1<D>()))) return e;
  done = true;
  return cudaSuccess;
}

template <int D>
cudaError_t embed_impl(const ModelDims& md, const DevWeights& w, const float* cand, int rows, __nv_bfloat16* act_a,
                       uint32_t* status, cudaStream_t st, Prof* prof) {
  cudaError_t e = set_smem_attrs<D>();
  if (e) return e;
  const int tiles = (rows + 127) / 128;
  if (prof) prof->begin(st);
  e = launch_k(k_embed<D>, dim3(tiles), dim3(256), smem_embed<D>(), st, w, md, cand, rows, act_a, status);
  if (prof) prof->end(KC_EMBED, 2.0 * rows * ((double)md.A * md.As + (double)md.As * md.eh + (double)md.eh * D), st);
  return e;
}

template <int D>
cudaError_t adaln_impl(const ModelDims& md, const DevWeights& w, int rows, const __nv_bfloat16* act_a,
                       __nv_bfloat16* mod, uint32_t* status, cudaStream_t st, Prof* prof) {
  cudaError_t e = set_smem_attrs<D>();
  if (e) return e;
  const int tiles = (rows + 127) / 128;
  const int ntiles = md.L * 6 * D / Cfg<D>::NT_ADA;
  if (prof) prof->begin(st);
  e = launch_k(k_adaln<D>, dim3(tiles, ntiles), dim3(kThreads), smem_adaln<D>(), st, w, md, rows, act_a, mod, status);
  if (prof) prof->end(KC_ADALN, 2.0 * rows * (double)D * md.L * 6 * D, st);
  return e;
}

template <int D>
cudaError_t call_impl(const ModelDims& md, const DevWeights& w, const CallGeom& g, const RolloutBufs& b,
                      uint32_t* status, cudaStream_t st, Prof* prof) {
  cudaError_t e = set_smem_attrs<D>();
  if (e) return e;
  const int nkb_inner = md.inner / 64, nkb_mlp = md.mlp / 64;
  const double rows = (double)g.n_cand * g.w;  // valid window rows
#define LEWM_TRY(x)                         \
  do {                                      \
    if ((e = (x)) != cudaSuccess) return e; \
  } while (0)
  for (int l = 0; l < md.L; ++l) {
    if (prof) prof->begin(st);
    LEWM_TRY(launch_k(k_qkv_attn<D>, dim3(g.n_tiles, md.heads), dim3(kThreads), smem_qkv<D>(), st, w, md, g, b, l,
                      status));
    if (prof) prof->end(KC_QKV_ATTN, 2.0 * rows * D * 3 * md.inner + 4.0 * rows * g.w * md.inner, st);
    if (prof) prof->begin(st);
    LEWM_TRY(launch_k(k_resid_gemm<D>, dim3(g.n_tiles, 4), dim3(kThreads), smem_resid<D>(), st,
                      (const __nv_bfloat16*)b.attn, nkb_inner,
                      (const __nv_bfloat16*)(w.wout + (size_t)l * 4 * nkb_inner * Cfg<D>::NT_OUT * 64),
                      (const float*)(w.out_b + l * D), 2, g, b, md, l, status));
    if (prof) prof->end(KC_OUT, 2.0 * rows * md.inner * D, st);
    if (prof) prof->begin(st);
    LEWM_TRY(launch_k(k_fc1<D>, dim3(g.n_tiles, md.mlp / 128), dim3(kThreads), smem_fc1<D>(), st, w, md, g, b, l,
                      status));
    if (prof) prof->end(KC_FC1, 2.0 * rows * D * md.mlp, st);
    if (prof) prof->begin(st);
    LEWM_TRY(launch_k(k_resid_gemm<D>, dim3(g.n_tiles, 4), dim3(kThreads), smem_resid<D>(), st,
                      (const __nv_bfloat16*)b.h, nkb_mlp,
                      (const __nv_bfloat16*)(w.w2 + (size_t)l * 4 * nkb_mlp * Cfg<D>::NT_OUT * 64),
                      (const float*)(w.b2 + l * D), 5, g, b, md, l, status));
    if (prof) prof->end(KC_FC2, 2.0 * rows * md.mlp * D, st);
  }
  if (prof) prof->begin(st);
  LEWM_TRY(launch_k(k_final<D>, dim3((g.n_cand + 3) / 4), dim3(128), 0, st, w, g, b));
  if (prof) prof->end(KC_FINAL, 0.0, st);
#undef LEWM_TRY
  return cudaSuccess;
}

}  // namespace

cudaError_t launch_embed(const ModelDims& md, const DevWeights& w, const float* cand, int rows,
                         __nv_bfloat16* act_a, uint32_t* status, cudaStream_t st, Prof* prof) {
  if (md.D == 192) return embed_impl<192>(md, w, cand, rows, act_a, status, st, prof);
  if (md.D == 384) return embed_impl<384>(md, w, cand, rows, act_a, status, st, prof);
  return cudaErrorInvalidValue;
}

cudaError_t launch_adaln(const ModelDims& md, const DevWeights& w, int rows, const __nv_bfloat16* act_a,
                         __nv_bfloat16* mod, uint32_t* status, cudaStream_t st, Prof* prof) {
  if (md.D == 192) return adaln_impl<192>(md, w, rows, act_a, mod, status, st, prof);
  if (md.D == 384) return adaln_impl<384>(md, w, rows, act_a, mod, status, st, prof);
  return cudaErrorInvalidValue;
}

cudaError_t launch_call(const ModelDims& md, const DevWeights& w, const CallGeom& g, const RolloutBufs& b,
                        uint32_t* status, cudaStream_t st, Prof* prof) {
  if (md.D == 192) return call_impl<192>(md, w, g, b, status, st, prof);
  if (md.D == 384) return call_impl<384>(md, w, g, b, status, st, prof);
  return cudaErrorInvalidValue;
}

}  // namespace lewm
