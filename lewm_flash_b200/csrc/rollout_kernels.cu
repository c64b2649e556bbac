// LeWM predictor rollout kernels for sm_100a.
//
// One model-cost evaluation (reference JEPA.get_cost_from_embeddings,
// lewm/jepa.py:302-317) is:
//   k_embed_hidden, k_embed_out
//             Embedder (lewm/module.py:205-214) + SiLU for every (candidate, time)
//   k_adaln   AdaLN modulation Linear (lewm/module.py:98-100) for every layer at once;
//             it depends only on the actions, so it is hoisted out of the
//             autoregressive chain and computed once per candidate and time step
//   k_prep0   first predictor call: layer-0 residual rows (history + position)
//   per predictor call (lewm/jepa.py:284-298), per layer (lewm/module.py:105-111):
//     k_qkv_attn   LN1 -> modulate -> attn.norm of the residual rows, QKV GEMM (one
//                  head per CTA), causal attention over the window (lewm/module.py:75-85)
//     k_partial_gemm  out-proj GEMM, two K halves written as partial sums
//     k_fc1        residual update r + gate_msa * (out-proj + bias), then LN2 -> modulate
//                  -> FFN LayerNorm, FC1 GEMM + bias -> GELU
//     k_partial_gemm  FC2 GEMM partial sums; its residual update is applied by the next
//                  layer's k_qkv_attn (or by k_final after the last layer)
//   k_final   final LayerNorm (lewm/module.py:183) on each window's last token,
//             then score against the goal (cost_from_rollout, lewm/jepa.py:246-260)
//             or append to the history and write the next call's layer-0 rows
//
// GEMMs run on tcgen05 (bf16 in, fp32 accumulate in TMEM); weight operands arrive in
// shared memory by bulk copy of pre-swizzled blocks; LayerNorm, modulation, bias,
// GELU, gates, residuals and the cost are fp32.
//
// Latency structure (a single-env plan is a chain of thousands of small
// dependent kernels, so every global-memory round trip on a kernel's critical
// path counts):
//   * every kernel is launched with programmatic stream serialization; before
//     griddep_wait() it only initialises barriers, allocates TMEM and starts
//     bulk copies of weights and per-layer vectors into shared memory, which
//     overlaps the previous kernel;
//   * the LayerNorms of a GEMM operand run in that GEMM's kernel, four threads per
//     row reducing through shuffles, straight into the swizzled shared-memory tile:
//     the residual GEMMs need no cross-CTA exchange;
//   * accumulator columns are split over the four warps that share a TMEM lane
//     quadrant;
//   * copies are issued one per lane of one warp instruction, and streamed-K GEMMs
//     move their K blocks in as few instruction rounds as shared memory allows.
#include <algorithm>

#include <cuda.h>  // CUtensorMap (tiled TMA store of the AdaLN output)

#include "lewm_common.cuh"
#include "lewm_internal.h"

// Phase-timing hook for diagnostic builds (no code in the product build).
#ifndef LEWM_STAMP
#define LEWM_STAMP(kind, phase)
#endif

namespace lewm {
namespace {

constexpr int kBlk = 16384;           // bytes of one [128 x 64] bf16 block
constexpr int kBlkElems = 128 * 64;   // elements of one [128 x 64] block
constexpr int kMaxWindow = 8;
constexpr int kKVStride = 132;        // floats per row of the k|v scratch: 16-byte rows, and
                                       // float4 accesses of 8 consecutive rows hit distinct banks
constexpr int kThreads = 512;         // 16 warps: 4 per TMEM lane quadrant
constexpr int kFc1N = 32;             // hidden columns per FC1 CTA (N of its MMA)

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
  // K blocks per copy group of the streamed-K GEMMs (two groups in flight).
  static constexpr int KG = (D == 192) ? 4 : 3;
};

struct RowMap {
  bool valid;
  int cand, pos, tok;  // tok = cand*T + history index
};
__device__ __forceinline__ RowMap map_row(const CallGeom& g, int tile, int r) {
  RowMap m;
  const int cl = r / g.rpc;  // g.rpc rows per candidate, window positions pos0 ..
  m.pos = g.pos0 + (r - cl * g.rpc);
  m.cand = tile * g.cpt + cl;
  m.valid = (cl < g.cpt) && (m.cand < g.n_cand);
  m.tok = m.cand * g.T + g.start + m.pos;
  return m;
}

// ---------------------------------------------------------------- streamed-K operand pipeline
// K blocks travel in groups of G. All copies of a group are issued by the lanes of
// one warp in a single instruction: 1-D bulk copies issued by separate instructions
// complete one after another, those issued together overlap. When every K block fits
// in shared memory at once (G >= nkb) there is one group and no refill; otherwise two
// groups are in flight (slots [2G]) and group g + 2 is issued as soon as the MMAs of
// group g retire. A slots are `as` bytes apart: the tile's used rows (packed) or a
// full block; the MMA reads 128 rows from each slot, so the A region keeps a tail of
// (kBlk - as) bytes after its last slot.
template <int B_BLK>
struct KStream {
  uint8_t* sA;
  uint8_t* sB;                // slots of B_BLK bytes
  uint64_t* full;             // [2] one per slot half
  uint64_t* empty;            // [2]
  const __nv_bfloat16* tA;    // A block kb at tA + kb * a_step
  size_t a_step;
  const __nv_bfloat16* tB;    // B block kb at tB + kb * b_step
  size_t b_step;
  uint32_t ab;                // A bytes per block (the tile's used rows)
  uint32_t as;                // A slot stride, a multiple of 1024
  int nkb;
  int G;                      // K blocks per group (<= 16)
  __device__ __forceinline__ int groups() const { return (nkb + G - 1) / G; }
  __device__ __forceinline__ int blocks(int g) const { return min(G, nkb - g * G); }
  __device__ __forceinline__ uint32_t bytes(int g) const { return (uint32_t)blocks(g) * (ab + B_BLK); }
  // Lanes 0 .. 2G-1: block (lane % G) of group lane / G (groups 0 and 1); A or B.
  __device__ __forceinline__ void issue_first(int lane, bool a_side) const {
    if (lane >= 2 * G) return;
    const int g = lane / G, j = lane - g * G;
    if (g >= groups() || j >= blocks(g)) return;
    const int kb = g * G + j;
    if (a_side)
      bulk_g2s(sA + (size_t)lane * as, tA + (size_t)kb * a_step, ab, &full[g]);
    else
      bulk_g2s(sB + (size_t)lane * B_BLK, tB + (size_t)kb * b_step, B_BLK, &full[g]);
  }
  // Lanes 0 .. G-1: A blocks of group g, lanes G .. 2G-1: its B blocks.
  __device__ __forceinline__ void issue_group(int g, int lane) const {
    if (lane >= 2 * G) return;
    const int j = lane < G ? lane : lane - G;
    if (j >= blocks(g)) return;
    const int kb = g * G + j, slot = (g & 1) * G + j;
    if (lane < G)
      bulk_g2s(sA + (size_t)slot * as, tA + (size_t)kb * a_step, ab, &full[g & 1]);
    else
      bulk_g2s(sB + (size_t)slot * B_BLK, tB + (size_t)kb * b_step, B_BLK, &full[g & 1]);
  }
  // Warp 0: wait for each group, issue its MMAs (lane 0), release its slots.
  __device__ __forceinline__ bool mma(uint32_t tmem, uint32_t idesc, int lane, uint32_t* status) const {
    bool ok = true;
    for (int g = 0; g < groups(); ++g) {
      if (!__all_sync(0xffffffffu, mbar_wait(&full[g & 1], (g >> 1) & 1, status))) {
        ok = false;
        break;
      }
      tc_fence_after();
      if (lane == 0) {
        // Descriptors are built once and stepped: the start-address field (bits 0-13,
        // address >> 4) advances by 2 per 32-byte K step and by the slot stride per block
        // (shared addresses stay below 256 KB, so the field never carries).
        const int slot0 = (g & 1) * G;
        uint64_t ad = sdesc_sw128(smem_u32(sA) + slot0 * as);
        uint64_t bd = sdesc_sw128(smem_u32(sB) + slot0 * B_BLK);
        const uint64_t astep = as >> 4, bstep = B_BLK >> 4;
        const int nb = blocks(g);
        for (int j = 0; j < nb; ++j) {
          umma_bf16(tmem, ad, bd, idesc, (g | j) ? 1u : 0u);
          umma_bf16(tmem, ad + 2, bd + 2, idesc, 1u);
          umma_bf16(tmem, ad + 4, bd + 4, idesc, 1u);
          umma_bf16(tmem, ad + 6, bd + 6, idesc, 1u);
          ad += astep;
          bd += bstep;
        }
        umma_commit(&empty[g & 1]);
      }
      __syncwarp();
    }
    return ok;
  }
  // Warp 1: refill a slot half once the MMAs of the group before it retired.
  __device__ __forceinline__ void produce(int lane, uint32_t* status) const {
    for (int g = 2; g < groups(); ++g) {
      if (!__all_sync(0xffffffffu, mbar_wait(&empty[g & 1], ((g >> 1) - 1) & 1, status))) break;
      if (lane == 0) mbar_arrive_expect_tx(&full[g & 1], bytes(g));
      __syncwarp();
      issue_group(g, lane);
      __syncwarp();
    }
  }
};

// Shared-memory layout of a residual-GEMM launch: one group holding every K block when
// it fits in the 227 KB a CTA may use, else two groups of kg blocks; A slots packed
// at the tile's used rows. The host sizes the launch with the same function.
struct ResidLayout {
  int G;          // K blocks per group
  int a_stride;   // bytes between A slots
  int b_off;      // offset of the B slots
  int v_off;      // offset of the vectors / reduction scratch / barriers
  int bytes;      // dynamic shared memory to request (includes 1024 alignment slack)
};
__host__ __device__ inline ResidLayout resid_layout(int rows8, int nkb, int b_blk, int kg, int extra) {
  ResidLayout L{};
  L.a_stride = rows8 * 128;
  for (int pass = 0; pass < 2; ++pass) {
    L.G = pass == 0 ? nkb : kg;
    const int slots = L.G >= nkb ? nkb : 2 * L.G;
    const int a_bytes = ((slots * L.a_stride + (kBlk - L.a_stride)) + 1023) & ~1023;
    L.b_off = a_bytes;
    L.v_off = (a_bytes + slots * b_blk + 1023) & ~1023;
    L.bytes = 1024 + L.v_off + extra;
    if (L.G <= 16 && L.bytes <= 232448) break;
  }
  return L;
}

// ---------------------------------------------------------------- Embedder + SiLU
// act_a[row] = bf16(SiLU(Linear2(SiLU(Linear1(Conv1x1(a)))))), rows = candidate*T + t,
// in two kernels so the hidden layer is spread over many SMs:
//   k_embed_hidden  one CTA per (128-row tile, 64 hidden units): Conv1x1 and Linear1 in
//                   fp32, SiLU, bf16 into a pre-swizzled [128 x 64] block of `eh`
//   k_embed_out     Linear2 on tcgen05 (K = embed_hidden streamed, one CTA per N/4
//                   columns), + bias, SiLU, bf16 into act_a.
template <int D>
__global__ void __launch_bounds__(256) k_embed_hidden(DevWeights w, ModelDims md, const float* __restrict__ cand,
                                                      int rows, __nv_bfloat16* __restrict__ eh) {
  __shared__ float actc[128 * 16];
  __shared__ __align__(1024) uint8_t sO[kBlk];
  griddep_wait();
  griddep_launch();
  const int tid = threadIdx.x;
  const int row0 = blockIdx.x * 128, hc = blockIdx.y;
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
  __syncthreads();
  const int k = tid & 63;
  const int hk = hc * 64 + k;
  float wv[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) wv[i] = (i < md.As) ? w.e1_w[hk * md.As + i] : 0.f;
  const float bias = w.e1_b[hk];
  for (int r = tid >> 6; r < 128; r += 4) {
    float acc = bias;
#pragma unroll
    for (int i = 0; i < 16; ++i) acc += wv[i] * actc[r * 16 + i];
    *reinterpret_cast<__nv_bfloat16*>(sO + sw128_off(r, k)) = __float2bfloat16_rn(silu_f(acc));
  }
  fence_async_smem();
  __syncthreads();
  if (tid == 0) {
    bulk_s2g(eh + ((size_t)blockIdx.x * (md.eh / 64) + hc) * kBlkElems, sO, kBlk);
    bulk_commit();
    bulk_wait_read();
  }
}

template <int D>
__global__ void __launch_bounds__(kThreads) k_embed_out(DevWeights w, ModelDims md, int rows,
                                                        const __nv_bfloat16* __restrict__ eh,
                                                        __nv_bfloat16* __restrict__ act_a, uint32_t* status) {
  using C = Cfg<D>;
  constexpr int NT = C::NT_OUT;  // D / 4 columns per CTA
  constexpr int CW = NT / 4;
  constexpr int G = C::KG;
  constexpr int B_BLK = NT * 128;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* sA = smem;
  uint8_t* sB = smem + 2 * G * kBlk;
  float* sbias = reinterpret_cast<float*>(sB + 2 * G * B_BLK);  // [NT]
  uint64_t* full = reinterpret_cast<uint64_t*>(sbias + NT);
  uint64_t* empty = full + 2;
  uint64_t* bar_mma = empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_mma + 1);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int tile = blockIdx.x, nt = blockIdx.y;
  const int nkb = md.eh / 64;
  // we2 K block kb holds all D rows: this CTA's N tile is rows [nt * NT, nt * NT + NT).
  const KStream<B_BLK> ks{sA, sB, full, empty, eh + (size_t)tile * nkb * kBlkElems, (size_t)kBlkElems,
                          w.we2 + (size_t)nt * NT * 64, (size_t)D * 64, (uint32_t)kBlk, (uint32_t)kBlk, nkb, G};
  if (tid == 0) {
    for (int h = 0; h < 2; ++h) {
      mbar_init(&full[h], 1);
      mbar_init(&empty[h], 1);
    }
    mbar_init(bar_mma, 1);
    fence_mbar_init();
    mbar_arrive_expect_tx(&full[0], ks.bytes(0) + NT * 4);
    if (ks.groups() > 1) mbar_arrive_expect_tx(&full[1], ks.bytes(1));
  }
  __syncwarp();
  if (warp == 0) {  // weights and bias before the wait, one instruction
    if (lane < 2 * G)
      ks.issue_first(lane, false);
    else if (lane == 2 * G)
      bulk_g2s(sbias, w.e2_b + nt * NT, NT * 4, &full[0]);
  }
  __syncwarp();
  if (warp == 0) {
    tmem_alloc(tmem_slot, C::TMEM_OUT);
    tmem_relinquish();
  }
  griddep_wait();
  griddep_launch();
  if (warp == 0) ks.issue_first(lane, true);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (warp == 0) {  // MMA issuer
    ks.mma(tmem, idesc_bf16(128, NT), lane, status);
    if (lane == 0) umma_commit(bar_mma);
    __syncwarp();
  } else if (warp == 1) {
    ks.produce(lane, status);
  }
  const bool ok = cta_wait_mma(bar_mma, status, tmem_slot + 1);
  __syncwarp();
  tc_fence_after();
  const int quad = warp & 3, slice = warp >> 2;
  const int r = quad * 32 + lane;
  const bool valid = ok && (tile * 128 + r < rows);
  const uint32_t taddr = tmem + ((uint32_t)(quad * 32) << 16) + slice * CW;
  float v[CW];
  tmem_ld_cols<CW>(taddr, v);
  const int c0 = nt * NT + slice * CW;
  uint8_t* at = reinterpret_cast<uint8_t*>(act_a + (size_t)tile * (D / 64) * kBlkElems);
#pragma unroll
  for (int i = 0; i < CW; i += 4) {
    const int c = c0 + i;
    const float* bs = sbias + slice * CW + i;
    uint2 pk = make_uint2(0u, 0u);
    if (valid) {
      pk.x = pack_bf16x2(silu_f(v[i] + bs[0]), silu_f(v[i + 1] + bs[1]));
      pk.y = pack_bf16x2(silu_f(v[i + 2] + bs[2]), silu_f(v[i + 3] + bs[3]));
    }
    *reinterpret_cast<uint2*>(at + (c >> 6) * kBlk + sw128_off(r, c & 63)) = pk;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, C::TMEM_OUT);
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
  float* sbias = reinterpret_cast<float*>(sB + C::KB * NT * 128);  // NT floats
  uint64_t* bars = reinterpret_cast<uint64_t*>(sbias + NT);      // [0] weights, [1] mma, [2] act
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 3);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int tile = blockIdx.x, nt = blockIdx.y;
  LEWM_STAMP(1, 0);
  if (tid == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    mbar_init(&bars[2], 1);
    fence_mbar_init();
    mbar_arrive_expect_tx(&bars[0], C::KB * NT * 128 + NT * 4);
  }
  __syncwarp();
  // One copy per lane: copies issued by one thread complete one after another.
  if (warp == 0) {
    if (lane < C::KB)
      bulk_g2s(sB + lane * NT * 128, w.wada + ((size_t)nt * C::KB + lane) * NT * 64, NT * 128, &bars[0]);
    else if (lane == C::KB)
      bulk_g2s(sbias, w.ada_b + nt * NT, NT * 4, &bars[0]);
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, 256);
    tmem_relinquish();
  }
  LEWM_STAMP(1, 1);
  griddep_wait();
  LEWM_STAMP(1, 2);
  griddep_launch();
  if (warp == 0) {
    if (lane == 0) mbar_arrive_expect_tx(&bars[2], C::KB * kBlk);
    __syncwarp();
    if (lane < C::KB) bulk_g2s(sA + lane * kBlk, act_a + ((size_t)tile * C::KB + lane) * kBlkElems, kBlk, &bars[2]);
  }
  LEWM_STAMP(1, 5);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (warp == 0) {
    const bool got = __all_sync(0xffffffffu, mbar_wait(&bars[0], 0, status) && mbar_wait(&bars[2], 0, status));
    if (lane == 0) {
      if (got) {
        tc_fence_after();
        umma_tile(tmem, smem_u32(sA), kBlk, smem_u32(sB), NT * 128, 0, C::KB, idesc_bf16(128, NT), false);
      }
      LEWM_STAMP(1, 3);
      umma_commit(&bars[1]);
    }
    __syncwarp();
  }
  const bool ok = cta_wait_mma(&bars[1], status, tmem_slot + 1);
  LEWM_STAMP(1, 4);
  __syncwarp();
  tc_fence_after();
  const int quad = warp & 3, slice = warp >> 2;
  const int row = tile * 128 + quad * 32 + lane;
  const int ncols = md.L * 6 * D;
  const uint32_t taddr = tmem + ((uint32_t)(quad * 32) << 16) + slice * CW;
  float v[CW];
  tmem_ld_cols<CW>(taddr, v);
  // The tile's rows staged as bf16 in the operand / weight slots (dead once the MMAs
  // retired; rows padded to SROW bytes, so 8 consecutive rows' 16-byte stores hit distinct
  // banks), then one bulk copy per row: the NT columns of a row are contiguous in mod
  // (row-per-thread global stores would touch 32 lines per warp instruction).
  constexpr int SROW = NT * 2 + 16;
  static_assert(128 * SROW <= C::KB * (kBlk + NT * 128), "staging fits the operand slots");
  uint8_t* stg = smem;
  const int r = quad * 32 + lane;
  if (ok) {
    const float* bs = sbias + slice * CW;
    uint4* sr = reinterpret_cast<uint4*>(stg + r * SROW + slice * CW * 2);
#pragma unroll
    for (int i = 0; i < CW / 8; ++i) {
      uint32_t pk[4];
#pragma unroll
      for (int k = 0; k < 4; ++k)
        pk[k] = pack_bf16x2(v[8 * i + 2 * k] + bs[8 * i + 2 * k], v[8 * i + 2 * k + 1] + bs[8 * i + 2 * k + 1]);
      sr[i] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
    }
  }
  fence_async_smem();
  __syncthreads();
  if (warp < 4 && ok) {  // lane of warp q copies row 32 q + lane and waits for its own copy's reads
    if (row < rows) bulk_s2g(mod + (size_t)row * ncols + nt * NT, stg + r * SROW, NT * 2);
    bulk_commit();
    bulk_wait_read();
  }
  LEWM_STAMP(1, 6);
  tc_fence_before();
  __syncthreads();
  __syncwarp();
  if (warp == 0) tmem_dealloc(tmem, 256);
}

// ---------------------------------------------------------------- AdaLN modulation, persistent
// The same product as k_adaln for calls with many row tiles (width 192): one CTA per
// (192-column N tile, row-tile group) keeps its weight slice in shared memory and runs its
// row tiles through a pipeline, so the tensor pipe works on tile i + 1 while the epilogue
// drains tile i. Warp 0 streams the tiles' operands into two buffers, warp 1 issues each
// tile's 12 MMAs into one of two TMEM accumulators, warps 4-15 apply the bias, convert to
// bf16 and stage the tile as three 128-byte-swizzled [128 x 64] blocks, which one thread
// writes to mod with three tiled TMA stores (the tensor map clips rows past the end; 384-byte
// bulk copies per row cost ~2x more per tile). Hand-offs are mbarriers: full_a (operand
// landed), empty_a and mma_done (the tile's MMAs retired), tmem_empty (the epilogue read the
// accumulator). Every wait is bounded; after a timeout every role stops at its next wait,
// and the epilogue's decisions come from one thread through shared memory, so its named
// barriers are always reached by all 384 threads. Per tile the MMAs and the epilogue
// arithmetic are those of k_adaln: the same bits.
constexpr int kAdaGroups = 4;  // row-tile groups per N tile (36 N tiles x 4 = 144 CTAs at width 192)
template <int D>
constexpr int smem_adaln_ps() {
  constexpr int NT = Cfg<D>::NT_ADA;
  return 1024 + Cfg<D>::KB * NT * 128 + 2 * Cfg<D>::KB * kBlk + (NT / 64) * kBlk + NT * 4 + 8 * 9 + 16;
}

template <int D>
__global__ void __launch_bounds__(kThreads) k_adaln_ps(DevWeights w, ModelDims md, int rows,
                                                       const __nv_bfloat16* __restrict__ act_a,
                                                       const __grid_constant__ CUtensorMap mod_map,
                                                       uint32_t* status) {
  using C = Cfg<D>;
  constexpr int NT = C::NT_ADA;
  constexpr int KB = C::KB;
  constexpr int CWE = NT / 3;        // columns per epilogue warp (3 warps per TMEM lane quadrant)
  static_assert(NT == 192 && CWE == 64, "width 192: one staged 64-column block per epilogue warp");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* sB = smem;                                  // weights of this N tile, [KB][NT x 64]
  uint8_t* sA = sB + KB * NT * 128;                    // two operand buffers, [2][KB][128 x 64]
  uint8_t* stg = sA + 2 * KB * kBlk;                   // staged output tile, [NT/64][128 x 64] SW128
  float* sbias = reinterpret_cast<float*>(stg + (NT / 64) * kBlk);
  uint64_t* bar_w = reinterpret_cast<uint64_t*>(sbias + NT);
  uint64_t* full_a = bar_w + 1;      // [2]
  uint64_t* empty_a = full_a + 2;    // [2]
  uint64_t* mma_done = empty_a + 2;  // [2]
  uint64_t* tmem_empty = mma_done + 2;  // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tmem_empty + 2);
  volatile uint32_t* eflag = tmem_slot + 1;  // epilogue leader's verdict
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nt = blockIdx.x, grp = blockIdx.y, ngrp = gridDim.y;
  const int ntile_rows = (rows + 127) / 128;
  if (tid == 0) {
    mbar_init(bar_w, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&full_a[i], 1);
      mbar_init(&empty_a[i], 1);
      mbar_init(&mma_done[i], 1);
      mbar_init(&tmem_empty[i], 1);
    }
    fence_mbar_init();
    mbar_arrive_expect_tx(bar_w, KB * NT * 128 + NT * 4);
  }
  __syncwarp();
  if (warp == 0) {  // weights and bias before the wait, one copy per lane
    if (lane < KB)
      bulk_g2s(sB + lane * NT * 128, w.wada + ((size_t)nt * KB + lane) * NT * 64, NT * 128, bar_w);
    else if (lane == KB)
      bulk_g2s(sbias, w.ada_b + nt * NT, NT * 4, bar_w);
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  griddep_wait();
  griddep_launch();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (warp == 0) {  // producer: operand of tile i into buffer i & 1
    for (int i = 0;; ++i) {
      const int t = grp + i * ngrp;
      if (t >= ntile_rows) break;
      const int bi = i & 1;
      if (i >= 2 && !__all_sync(0xffffffffu, mbar_wait(&empty_a[bi], ((i >> 1) - 1) & 1, status))) break;
      if (lane == 0) mbar_arrive_expect_tx(&full_a[bi], KB * kBlk);
      __syncwarp();
      if (lane < KB)
        bulk_g2s(sA + (bi * KB + lane) * kBlk, act_a + ((size_t)t * KB + lane) * kBlkElems, kBlk, &full_a[bi]);
      __syncwarp();
    }
  } else if (warp == 1) {  // MMA issuer: tile i into accumulator i & 1 (TMEM columns 256 (i & 1) ..)
    const uint32_t idesc = idesc_bf16(128, NT);
    bool ok = __all_sync(0xffffffffu, mbar_wait(bar_w, 0, status));
    for (int i = 0; ok; ++i) {
      const int t = grp + i * ngrp;
      if (t >= ntile_rows) break;
      const int bi = i & 1;
      if (i >= 2 && !__all_sync(0xffffffffu, mbar_wait(&tmem_empty[bi], ((i >> 1) - 1) & 1, status))) break;
      if (!__all_sync(0xffffffffu, mbar_wait(&full_a[bi], (i >> 1) & 1, status))) break;
      tc_fence_after();
      if (lane == 0) {
        umma_tile(tmem + bi * 256, smem_u32(sA + bi * KB * kBlk), kBlk, smem_u32(sB), NT * 128, 0, KB, idesc, false);
        umma_commit(&mma_done[bi]);
        umma_commit(&empty_a[bi]);
      }
      __syncwarp();
    }
  } else if (warp >= 4) {  // epilogue: 12 warps, warp (quad, slice) = 32 rows x CWE columns
    const int e = tid - 128;
    const int quad = warp & 3, slice = (warp - 4) >> 2;
    const int r = quad * 32 + lane;
    for (int i = 0;; ++i) {
      const int t = grp + i * ngrp;
      if (t >= ntile_rows) break;
      const int bi = i & 1;
      if (e == 0) {
        const bool ok = (i > 0 || mbar_wait(bar_w, 0, status)) && mbar_wait(&mma_done[bi], (i >> 1) & 1, status);
        *eflag = ok ? 1u : 0u;
      }
      if (e == 0) bulk_wait_read();  // the previous tile's stores have read the staged blocks
      named_bar(1, 384);
      if (*eflag == 0u) break;
      tc_fence_after();
      float v[CWE];
      tmem_ld_cols<CWE>(tmem + bi * 256 + ((uint32_t)(quad * 32) << 16) + slice * CWE, v);
      tc_fence_before();
      const float* bs = sbias + slice * CWE;
      uint8_t* blk = stg + slice * kBlk;  // this warp's 64 columns: one swizzled block
#pragma unroll
      for (int k = 0; k < CWE / 8; ++k) {
        uint32_t pk[4];
#pragma unroll
        for (int m = 0; m < 4; ++m)
          pk[m] = pack_bf16x2(v[8 * k + 2 * m] + bs[8 * k + 2 * m], v[8 * k + 2 * m + 1] + bs[8 * k + 2 * m + 1]);
        *reinterpret_cast<uint4*>(blk + sw128_off(r, 8 * k)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
      }
      fence_async_smem();
      named_bar(1, 384);
      if (e == 0) {
        mbar_arrive(&tmem_empty[bi]);  // every thread's loads of accumulator bi completed
#pragma unroll
        for (int j = 0; j < NT / 64; ++j)  // x: column (a multiple of 64), y: first row of the tile
          asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                           reinterpret_cast<uint64_t>(&mod_map)),
                       "r"(nt * NT + 64 * j), "r"(t * 128), "r"(smem_u32(stg + j * kBlk))
                       : "memory");
        bulk_commit();
      }
    }
    if (e == 0) bulk_wait_read();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 512);
}

// ---------------------------------------------------------------- GEMM operand from the residual
// A operand of the QKV / FC1 GEMM, built in shared memory from the fp32 residual rows:
// bf16(LN_{g,b}(LN(x) * (1 + scale) + shift)) with the first LayerNorm at eps 1e-6 and
// no affine (AdaLN modulate, lewm/module.py:105-111) and the second the attention /
// feed-forward block's own LayerNorm at eps 1e-5. TPR consecutive threads share a row
// (a warp covers 32 / TPR rows), D / TPR columns each in 4-column chunks; the row
// moments reduce through shuffles among them. Rows at or past rows8 are skipped (whole
// warps: the row range bounds are multiples of 8 >= 32 / TPR); window slots without a candidate get
// zeros.
// A residual update still pending when a GEMM operand is built: the residual-branch GEMM
// wrote partial sums P0 .. P(n-1) (two K halves, or four hidden quarters of a fused
// FFN), and the residual is r = src + gate * (sum + bias), the sum taken as (P0 + P1)
// or ((P0 + P1) + (P2 + P3)). With bias == nullptr the rows of src are used as they are.
struct ResidUpdate {
  const float* src;     // [tile rows][D] residual before the update (or the final rows)
  const float* part;    // partial sums of the tile, partial i at + i * part_stride
  size_t part_stride;
  int nparts;           // 2 or 4
  const float* bias;    // [D] bias of that GEMM, or null: no pending update
  int gate_off;         // mod column of its gate (layer * 6D + chunk * D)
  float* dst;           // [tile rows][D] where the updated rows are written, or null
};

// Partial sums of a residual-branch GEMM (out-projection, FC2): a tile's block of
// 128 x D floats holds one slab of 128 rows x D/4 floats per N piece (the columns one
// CTA computes), so each piece leaves its CTA as a single bulk copy. Within a slab row
// the 4-float chunks are rotated by part_rot(r): the row-per-thread staging stores in
// shared memory then hit distinct banks (D/16 chunks a row).
template <int D>
__device__ __forceinline__ int part_rot(int r) {
  return ((D / 16) % 8 == 4) ? (r >> 1) : r;
}
// Offset in floats of (row r, column c) inside a tile's partial block.
template <int D>
__device__ __forceinline__ int part_off(int r, int c) {
  constexpr int NT = D / 4, NCH = D / 16;
  const int piece = c / NT, ch = (c - piece * NT) >> 2;
  return (piece * 128 + r) * NT + ((ch + part_rot<D>(r)) % NCH) * 4 + (c & 3);
}
// Stage a row's chunks [chunk0, chunk0 + N/4) of N piece-local columns into a slab of
// shared memory laid out like a global partial slab.
template <int D, int N>
__device__ __forceinline__ void stage_part_row(float* slab, int r, int chunk0, const float* v) {
  constexpr int NT = D / 4, NCH = D / 16;
  const int rot = part_rot<D>(r);
#pragma unroll
  for (int i = 0; i < N / 4; ++i)
    *reinterpret_cast<float4*>(slab + r * NT + ((chunk0 + i + rot) % NCH) * 4) =
        make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
}

// Loads of one builder row (D / TPR columns of this thread, in 4-column chunks) that
// come from kernels at least two launches back: the modulation rows (written by k_adaln
// at the start of the rollout) and — where the caller says so — the residual rows. A
// kernel's CTAs start only after every CTA of the kernel before it passed
// griddepcontrol.wait (each kernel waits before it triggers its dependents), so by then
// the kernel two back has completed: these loads may be issued before this kernel's own
// wait. They bypass L1 (ld.global.cg) and read the coherent L2.
template <int D, int TPR>
struct LnEarly {
  static constexpr int NCH = D / TPR / 4;
  float4 src[NCH];
  uint2 shift[NCH], scale[NCH], gate[NCH];
  bool src_loaded;
};

template <int D, int TPR>
__device__ __forceinline__ void ln_row_early(LnEarly<D, TPR>& E, const ResidUpdate& u, const RowMap& m, int r,
                                             int part, const __nv_bfloat16* __restrict__ mod, int mod_cols,
                                             int shift_col, bool with_src) {
  constexpr int NCH = LnEarly<D, TPR>::NCH;
  const size_t mbase = m.valid ? (size_t)m.tok * mod_cols : 0;
  const __nv_bfloat16* mrow = mod + mbase + shift_col;
  E.src_loaded = with_src;
#pragma unroll
  for (int k = 0; k < NCH; ++k) {
    const int c = 4 * (part + TPR * k);
    E.src[k] = make_float4(0.f, 0.f, 0.f, 0.f);
    E.shift[k] = E.scale[k] = E.gate[k] = make_uint2(0u, 0u);
    if (m.valid) {
      E.shift[k] = __ldcg(reinterpret_cast<const uint2*>(mrow + c));
      E.scale[k] = __ldcg(reinterpret_cast<const uint2*>(mrow + D + c));
      if (u.bias) E.gate[k] = __ldcg(reinterpret_cast<const uint2*>(mod + mbase + u.gate_off + c));
      if (with_src) E.src[k] = __ldcg(reinterpret_cast<const float4*>(u.src + (size_t)r * D + c));
    }
  }
}

// Early loads of this thread's first-pass row, issued before griddepcontrol.wait.
template <int D>
__device__ __forceinline__ void prefetch_ln_operand(LnEarly<D, D / 12>& pf, const ResidUpdate& u, const CallGeom& g,
                                                    int tile, const __nv_bfloat16* __restrict__ mod, int mod_cols,
                                                    int shift_col, int tid, int r_begin, int r_end, bool with_src) {
  constexpr int TPR = D / 12;
  const int r = r_begin + tid / TPR;
  const RowMap m = map_row(g, tile, r);  // rows at or past rows8 map to no candidate
  ln_row_early<D, TPR>(pf, u, m, r, tid % TPR, mod, mod_cols, shift_col, with_src && r < r_end);
}

template <int D, int TPR, int SK = 0>
__device__ __forceinline__ void build_ln_operand_t(const ResidUpdate& u, const CallGeom& g, int tile,
                                                   const __nv_bfloat16* __restrict__ mod, int mod_cols, int shift_col,
                                                   const float* __restrict__ lg, const float* __restrict__ lb,
                                                   uint8_t* sA, int tid, int r_begin, int r_end,
                                                   const LnEarly<D, TPR>* pre = nullptr) {
  constexpr int NPER = D / TPR;   // columns per thread, a multiple of 4
  constexpr int NCH = NPER / 4;   // 4-column chunks per thread
  static_assert(NPER % 4 == 0, "4-column chunks");
  const int part = tid % TPR;
  const int r_first = r_begin + tid / TPR;
  for (int r = r_first; r < r_end; r += kThreads / TPR) {
    const RowMap m = map_row(g, tile, r);
    LnEarly<D, TPR> E;
    if (pre && r == r_first)
      E = *pre;
    else
      ln_row_early<D, TPR>(E, u, m, r, part, mod, mod_cols, shift_col, false);
    // The loads that depend on the kernel just before this one (the residual rows
    // unless prefetched, the partial sums) and the bias, through the read-only path (none of these buffers is written by this kernel: the updated rows
    // go to u.dst, never u.src), all issued before the update and its write-back.
    float xv[NPER];
    float4 pa[NCH], pb[NCH], bb[NCH];
    const bool four = u.nparts == 4;
    LEWM_STAMP(SK, 1);
#pragma unroll
    for (int k = 0; k < NCH; ++k) {
      const int c = 4 * (part + TPR * k);
      float4 t = E.src[k];
      pa[k] = pb[k] = bb[k] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (m.valid) {
        if (!E.src_loaded) t = __ldg(reinterpret_cast<const float4*>(u.src + (size_t)r * D + c));
        if (u.bias) {
          const int o = part_off<D>(r, c);
          pa[k] = __ldg(reinterpret_cast<const float4*>(u.part + o));
          pb[k] = __ldg(reinterpret_cast<const float4*>(u.part + u.part_stride + o));
          if (four) {  // (P0 + P1) + (P2 + P3), kept in pa / pb
            const float4 pc = __ldg(reinterpret_cast<const float4*>(u.part + 2 * u.part_stride + o));
            const float4 pd = __ldg(reinterpret_cast<const float4*>(u.part + 3 * u.part_stride + o));
            pa[k] = make_float4(pa[k].x + pb[k].x, pa[k].y + pb[k].y, pa[k].z + pb[k].z, pa[k].w + pb[k].w);
            pb[k] = make_float4(pc.x + pd.x, pc.y + pd.y, pc.z + pd.z, pc.w + pd.w);
          }
          bb[k] = __ldg(reinterpret_cast<const float4*>(u.bias + c));
        }
      }
      xv[4 * k] = t.x;
      xv[4 * k + 1] = t.y;
      xv[4 * k + 2] = t.z;
      xv[4 * k + 3] = t.w;
    }
    if (u.bias && m.valid) {
#pragma unroll
      for (int k = 0; k < NCH; ++k) {
        const float2 g01 = unpack_bf16x2(E.gate[k].x), g23 = unpack_bf16x2(E.gate[k].y);
        float* t = xv + 4 * k;
        t[0] += g01.x * ((pa[k].x + pb[k].x) + bb[k].x);
        t[1] += g01.y * ((pa[k].y + pb[k].y) + bb[k].y);
        t[2] += g23.x * ((pa[k].z + pb[k].z) + bb[k].z);
        t[3] += g23.y * ((pa[k].w + pb[k].w) + bb[k].w);
      }
      if (u.dst) {
#pragma unroll
        for (int k = 0; k < NCH; ++k) {
          const int c = 4 * (part + TPR * k);
          *reinterpret_cast<float4*>(u.dst + (size_t)r * D + c) =
              make_float4(xv[4 * k], xv[4 * k + 1], xv[4 * k + 2], xv[4 * k + 3]);
        }
      }
    }
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < NPER; ++i) s += xv[i];
    LEWM_STAMP(SK, 2);
#pragma unroll
    for (int o = 1; o < TPR; o <<= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const float mean = s * (1.0f / D);
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < NPER; ++i) q += (xv[i] - mean) * (xv[i] - mean);
#pragma unroll
    for (int o = 1; o < TPR; o <<= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
    const float rstd = rsqrtf(q * (1.0f / D) + 1e-6f);
    LEWM_STAMP(SK, 3);
    float s2 = 0.f;
#pragma unroll
    for (int k = 0; k < NCH; ++k) {
      const float2 h01 = unpack_bf16x2(E.shift[k].x), h23 = unpack_bf16x2(E.shift[k].y);
      const float2 a01 = unpack_bf16x2(E.scale[k].x), a23 = unpack_bf16x2(E.scale[k].y);
      float* y = xv + 4 * k;
      y[0] = (y[0] - mean) * rstd * (1.0f + a01.x) + h01.x;
      y[1] = (y[1] - mean) * rstd * (1.0f + a01.y) + h01.y;
      y[2] = (y[2] - mean) * rstd * (1.0f + a23.x) + h23.x;
      y[3] = (y[3] - mean) * rstd * (1.0f + a23.y) + h23.y;
      s2 += (y[0] + y[1]) + (y[2] + y[3]);
    }
#pragma unroll
    for (int o = 1; o < TPR; o <<= 1) s2 += __shfl_xor_sync(0xffffffffu, s2, o);
    const float mean2 = s2 * (1.0f / D);
    float q2 = 0.f;
#pragma unroll
    for (int i = 0; i < NPER; ++i) q2 += (xv[i] - mean2) * (xv[i] - mean2);
#pragma unroll
    for (int o = 1; o < TPR; o <<= 1) q2 += __shfl_xor_sync(0xffffffffu, q2, o);
    const float rstd2 = rsqrtf(q2 * (1.0f / D) + 1e-5f);
    LEWM_STAMP(SK, 4);
#pragma unroll
    for (int k = 0; k < NCH; ++k) {
      const int c = 4 * (part + TPR * k);
      const float4 g4 = __ldg(reinterpret_cast<const float4*>(lg + c));
      const float4 b4 = __ldg(reinterpret_cast<const float4*>(lb + c));
      const float* y = xv + 4 * k;
      uint2 pk = make_uint2(0u, 0u);
      if (m.valid) {
        pk.x = pack_bf16x2((y[0] - mean2) * rstd2 * g4.x + b4.x, (y[1] - mean2) * rstd2 * g4.y + b4.y);
        pk.y = pack_bf16x2((y[2] - mean2) * rstd2 * g4.z + b4.z, (y[3] - mean2) * rstd2 * g4.w + b4.w);
      }
      *reinterpret_cast<uint2*>(sA + (c >> 6) * kBlk + sw128_off(r, c & 63)) = pk;
    }
    LEWM_STAMP(SK, 5);
  }
}

// D / 12 threads per row (12 columns each: 16 threads at width 192, 32 at 384) for every
// tile size: all 16 warps work on the first rows, and larger tiles loop over further
// passes. The reduction order of the row moments is then the same for every tile
// geometry, so an env's results do not depend on how many candidates share its call.
template <int D, int SK = 0>
__device__ __forceinline__ void build_ln_operand(const ResidUpdate& u, const CallGeom& g, int tile,
                                                 const __nv_bfloat16* __restrict__ mod, int mod_cols, int shift_col,
                                                 const float* __restrict__ lg, const float* __restrict__ lb,
                                                 uint8_t* sA, int tid, const LnEarly<D, D / 12>* pre = nullptr) {
  build_ln_operand_t<D, D / 12, SK>(u, g, tile, mod, mod_cols, shift_col, lg, lb, sA, tid, 0, g.rows8, pre);
}

// Layer-0 residual row x0 = history row + position embedding of window position p.
template <int D>
__device__ __forceinline__ void prep_layer0_row(const DevWeights& w, const float* __restrict__ src, int p,
                                                float* __restrict__ xdst, int lane) {
  constexpr int NP = D / 64;
#pragma unroll
  for (int i = 0; i < NP; ++i) {
    const int c = 64 * i + 2 * lane;
    const float2 a = *reinterpret_cast<const float2*>(src + c);
    const float2 pe = *reinterpret_cast<const float2*>(w.pos + p * D + c);
    *reinterpret_cast<float2*>(xdst + c) = make_float2(a.x + pe.x, a.y + pe.y);
  }
}

// ---------------------------------------------------------------- GEMM operand, one CTA per 32 rows
// For tiles of more than 32 used rows the operand of a QKV / FC1 GEMM is built once per
// tile by this kernel (grid: tiles x 32-row groups) into the pre-swizzled global
// [tile][D/64][128 x 64] layout, which the GEMM's CTAs then bulk-copy; building it in
// each of the GEMM's 16-24 CTAs per tile would repeat several passes per CTA. Same
// device code as the in-kernel build, so the results are identical either way; every
// CTA writes back the updated residual rows it owns.
// src_early: the residual rows come from a kernel at least two launches back and are
// loaded with the modulation before griddepcontrol.wait.
template <int D>
__global__ void __launch_bounds__(kThreads) k_ln_operand(ResidUpdate u, CallGeom g, const __nv_bfloat16* mod,
                                                         int mod_cols, int shift_col, const float* lg, const float* lb,
                                                         __nv_bfloat16* a_op, int src_early) {
  const int tile = blockIdx.x;
  const int r0 = blockIdx.y * (kThreads / (D / 12));
  const int r1 = min(r0 + kThreads / (D / 12), g.rows8);
  const size_t t0 = (size_t)tile * 128 * D;
  ResidUpdate ut = u;
  ut.src += t0;
  if (ut.part) ut.part += t0;
  if (ut.dst) ut.dst += t0;
  LnEarly<D, D / 12> pf;
  prefetch_ln_operand<D>(pf, ut, g, tile, mod, mod_cols, shift_col, threadIdx.x, r0, r1, src_early != 0);
  griddep_wait();
  griddep_launch();
  build_ln_operand_t<D, D / 12>(ut, g, tile, mod, mod_cols, shift_col, lg, lb,
                                reinterpret_cast<uint8_t*>(a_op + (size_t)tile * (D / 64) * kBlkElems), threadIdx.x,
                                r0, r1, &pf);
}

// ---------------------------------------------------------------- first-call layer-0 inputs
// Warp per window row of the first predictor call (its history rows are all
// observation embeddings).
template <int D>
__global__ void __launch_bounds__(128) k_prep0(DevWeights w, ModelDims md, CallGeom g, RolloutBufs b) {
  griddep_wait();
  griddep_launch();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * 4 + warp;
  if (row >= g.n_cand * g.w) return;
  const int cand = row / g.w, p = row - cand * g.w;
  const int j = g.start + p;  // < H for the first call
  const int e = b.emb_per_cand ? cand : cand / g.S;
  const int tile = cand / g.cpt;
  const int r = (cand - tile * g.cpt) * g.w + p;
  prep_layer0_row<D>(w, b.emb + ((size_t)e * g.H + j) * D, p, b.x + ((size_t)tile * 128 + r) * D, lane);
}

// ---------------------------------------------------------------- QKV + attention
// Attention epilogue of one (row tile, head) of k_qkv_attn / k_qkv_attn_ps: q, k, v in TMEM
// columns [0, 192) of `tmem`; the head's output block is staged in sO and bulk-stored to
// b.attn (thread 0 waits until the copy has read sO). `kv` / `spart` / `sO` are shared scratch.
// Every thread calls `mid()` once the tile's TMEM reads are done (after the partial scores'
// CTA barrier): the persistent kernel issues the next tile's MMAs there.
template <int D, typename Mid>
__device__ __forceinline__ void qkv_attn_epilogue(const ModelDims& md, const CallGeom& g, const RolloutBufs& b,
                                                  int layer, int head, int tile, uint32_t tmem, bool ok,
                                                  float* kv, float* spart, uint8_t* sO, const Mid& mid) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // Causal softmax(q k^T / 8) v within the candidate's window. Thread (warp w, lane l)
  // owns window row r = 32 (w & 3) + l, its TMEM lane, and head-dim part p = w >> 2:
  // dims [8p, 8p + 8) and [32 + 8p, 40 + 8p) of q, k and v, read straight from TMEM.
  // Only k and v of the other rows of a window go through shared memory (row stride
  // kKVStride = 132 floats, float4 accesses conflict-free), and the four parts of
  // a row combine their partial scores through `spart`.
  {
    const int quad = warp & 3, part = warp >> 2;
    const int r = quad * 32 + lane;
    const RowMap m = map_row(g, tile, r);
    const bool valid = ok && m.valid;
    const int base = r - (m.pos - g.pos0);  // tile row of window position pos0 of the candidate
    const uint32_t trow = tmem + ((uint32_t)(quad * 32) << 16) + part * 8;
    float q[16], kk[16], vv[16];
    tmem_ld8(trow, q);
    tmem_ld8(trow + 32, q + 8);
    tmem_ld8(trow + 64, kk);
    tmem_ld8(trow + 96, kk + 8);
    tmem_ld8(trow + 128, vv);
    tmem_ld8(trow + 160, vv + 8);
    float4* kvr = reinterpret_cast<float4*>(kv + r * kKVStride + part * 8);
    // dims [8p, 8p + 8) at float4 0-1, [32 + 8p, 40 + 8p) at 8-9; v 16 float4 further
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const int o = (t & 1) + (t >> 1) * 8;
      kvr[o] = make_float4(kk[4 * t], kk[4 * t + 1], kk[4 * t + 2], kk[4 * t + 3]);
      kvr[16 + o] = make_float4(vv[4 * t], vv[4 * t + 1], vv[4 * t + 2], vv[4 * t + 3]);
    }
    // Key / value rows of the growing-window positions a later call reads instead of
    // recomputing them (same row format, row stride heads x 128 floats).
    const size_t kv_cand = ((size_t)layer * g.n_cand + m.cand) * b.kvc_pos;
    if (g.kv_write && valid && m.pos < b.kvc_pos) {
      float4* cw = reinterpret_cast<float4*>(b.kvc + ((kv_cand + m.pos) * md.heads + head) * 128 + part * 8);
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const int o = (t & 1) + (t >> 1) * 8;
        cw[o] = make_float4(kk[4 * t], kk[4 * t + 1], kk[4 * t + 2], kk[4 * t + 3]);
        cw[16 + o] = make_float4(vv[4 * t], vv[4 * t + 1], vv[4 * t + 2], vv[4 * t + 3]);
      }
    }
    // Rows of the earlier window positions: this tile's rows in shared memory, or, on a
    // call that runs only the new position, the cache (positions 0 .. pos - 1).
    const float* kvb = g.kv_read ? b.kvc + (kv_cand * md.heads + head) * 128 + part * 8
                                 : kv + (size_t)base * kKVStride + part * 8;
    const int kvs = g.kv_read ? md.heads * 128 : kKVStride;  // floats between window positions
    __syncthreads();
    LEWM_STAMP(2, 7);
    // Loops over the window stay rolled: each CTA runs this code once, so compact code
    // (fewer cold instruction fetches) beats unrolling.
    const int npos = valid ? m.pos : -1;
#pragma unroll 1
    for (int j = 0; j < npos; ++j) {
      const float4* kr = reinterpret_cast<const float4*>(kvb + (size_t)j * kvs);
      float d = 0.f;
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const float4 k4 = kr[(t & 1) + (t >> 1) * 8];
        d += q[4 * t] * k4.x;
        d += q[4 * t + 1] * k4.y;
        d += q[4 * t + 2] * k4.z;
        d += q[4 * t + 3] * k4.w;
      }
      spart[(part * kMaxWindow + j) * 128 + r] = d;
    }
    if (valid) {
      float d = 0.f;
#pragma unroll
      for (int t = 0; t < 16; ++t) d += q[t] * kk[t];
      spart[(part * kMaxWindow + m.pos) * 128 + r] = d;
    }
    __syncthreads();
    LEWM_STAMP(2, 9);
    mid();
    // One pass of online softmax over the window: running max, denominator and output
    // (exponentials on the special-function unit, __expf: ~2^-21 relative).
    // Window rows before this one come from shared memory, this row from registers.
    float mx = -INFINITY, den = 0.f;
    float o[16];
#pragma unroll
    for (int t = 0; t < 16; ++t) o[t] = 0.f;
#pragma unroll 1
    for (int j = 0; j < npos; ++j) {
      const float sj = (spart[(0 * kMaxWindow + j) * 128 + r] + spart[(1 * kMaxWindow + j) * 128 + r] +
                        spart[(2 * kMaxWindow + j) * 128 + r] + spart[(3 * kMaxWindow + j) * 128 + r]) *
                       0.125f;
      const float mnew = fmaxf(mx, sj);
      const float scale = __expf(mx - mnew);  // 0 on the first step (mx = -inf)
      const float pj = __expf(sj - mnew);
      den = den * scale + pj;
      mx = mnew;
      const float4* vr = reinterpret_cast<const float4*>(kvb + (size_t)j * kvs + 64);
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const float4 v4 = vr[(t & 1) + (t >> 1) * 8];
        o[4 * t] = o[4 * t] * scale + pj * v4.x;
        o[4 * t + 1] = o[4 * t + 1] * scale + pj * v4.y;
        o[4 * t + 2] = o[4 * t + 2] * scale + pj * v4.z;
        o[4 * t + 3] = o[4 * t + 3] * scale + pj * v4.w;
      }
    }
    float inv = 0.f;
    if (valid) {
      const int j = npos;
      const float sj = (spart[(0 * kMaxWindow + j) * 128 + r] + spart[(1 * kMaxWindow + j) * 128 + r] +
                        spart[(2 * kMaxWindow + j) * 128 + r] + spart[(3 * kMaxWindow + j) * 128 + r]) *
                       0.125f;
      const float mnew = fmaxf(mx, sj);
      const float scale = __expf(mx - mnew);
      const float pj = __expf(sj - mnew);
      den = den * scale + pj;
#pragma unroll
      for (int t = 0; t < 16; ++t) o[t] = o[t] * scale + pj * vv[t];
      inv = 1.0f / den;
    }
    LEWM_STAMP(2, 0);
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
    *reinterpret_cast<uint4*>(sO + sw128_off(r, part * 8)) = lo;
    *reinterpret_cast<uint4*>(sO + sw128_off(r, 32 + part * 8)) = hi;
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  LEWM_STAMP(2, 8);
  if (tid == 0) {
    bulk_s2g(b.attn + ((size_t)tile * md.heads + head) * kBlkElems, sO, g.rows8 * 128);
    bulk_commit();
    bulk_wait_read();
  }
}

template <int D>
__global__ void __launch_bounds__(kThreads) k_qkv_attn(DevWeights w, ModelDims md, CallGeom g, RolloutBufs b,
                                                       int layer, uint32_t* status) {
  using C = Cfg<D>;
  constexpr int KB = C::KB;
  constexpr int ST = C::QKV_ST;
  constexpr int B_BLK = 192 * 128;
  constexpr int R1 = KB * kBlk + ST * B_BLK;
  constexpr int SCR = 128 * kKVStride * 4 + 4 * kMaxWindow * 128 * 4;
  constexpr int R1S = ((R1 > SCR ? R1 : SCR) + 1023) & ~1023;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* sA = smem;
  uint8_t* sB = smem + KB * kBlk;
  float* kv = reinterpret_cast<float*>(smem);   // [128][kKVStride], aliases sA/sB after the MMA
  float* spart = kv + 128 * kKVStride;           // [4 parts][kMaxWindow][128] partial scores
  // The output block also lives in the operand region when it fits after the scratch.
  constexpr int SO_OFF = (((SCR + 1023) & ~1023) + kBlk <= R1) ? ((SCR + 1023) & ~1023) : R1S;
  constexpr int BAR_OFF = (SO_OFF + kBlk > R1S) ? SO_OFF + kBlk : R1S;
  uint8_t* sO = smem + SO_OFF;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + BAR_OFF);
  uint64_t* empty = full + ST;
  uint64_t* bar_mma = empty + ST;
  uint64_t* bar_a = bar_mma + 1;  // [KB], operand bulk copies when prebuilt
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_a + KB);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int tile = blockIdx.x, head = blockIdx.y;
  const __nv_bfloat16* wq = w.qkv + (size_t)((layer * md.heads + head) * KB) * (192 * 64);

  if (tid == 0) {
    for (int s = 0; s < ST; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(bar_mma, 1);
    for (int kb = 0; kb < KB; ++kb) mbar_init(&bar_a[kb], 1);
    fence_mbar_init();
  }
  __syncwarp();
  if (warp == 0 && lane < ST) {  // one copy per lane
    mbar_arrive_expect_tx(&full[lane], B_BLK);
    bulk_g2s(sB + lane * B_BLK, wq + (size_t)lane * 192 * 64, B_BLK, &full[lane]);
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, 256);
    tmem_relinquish();
  }
  // A operand: LN1 -> modulate (shift/scale_msa of this layer) -> attn.norm of the residual
  // rows. After layer 0 the previous layer's FC2 update is still pending: r = s + gate_mlp *
  // (sum of the FC2 partials + b2); the head-0 CTAs write r back for this layer's FC1. The
  // modulation rows are loaded before the wait (the residual rows come from the kernel
  // just before this one).
  const size_t t0 = (size_t)tile * 128 * D;
  ResidUpdate u{b.x + t0, nullptr, 0, 2, nullptr, 0, nullptr};
  if (layer > 0)
    u = ResidUpdate{b.xs + t0, b.part_b + t0, b.part_stride, g.fc2_parts, w.b2 + (layer - 1) * D,
                    (layer - 1) * 6 * D + 5 * D, head == 0 ? b.x + t0 : nullptr};
  LnEarly<D, D / 12> pf;
  if (!g.ln_prebuilt)
    prefetch_ln_operand<D>(pf, u, g, tile, b.mod, md.L * 6 * D, layer * 6 * D, tid, 0, g.rows8, false);
  LEWM_STAMP(2, 1);
  griddep_wait();
  LEWM_STAMP(2, 2);
  griddep_launch();
  if (g.ln_prebuilt) {  // built once per tile by k_ln_operand: one copy per lane
    if (warp == 0 && lane < KB) {
      mbar_arrive_expect_tx(&bar_a[lane], g.rows8 * 128);
      bulk_g2s(sA + lane * kBlk, b.a_op + ((size_t)tile * KB + lane) * kBlkElems, g.rows8 * 128, &bar_a[lane]);
    }
  } else {
    build_ln_operand<D, 6>(u, g, tile, b.mod, md.L * 6 * D, layer * 6 * D, w.attn_ln_w + layer * D,
                           w.attn_ln_b + layer * D, sA, tid, &pf);
  }
  fence_async_smem();
  LEWM_STAMP(2, 5);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (warp == 0) {  // whole warp waits, lane 0 issues
    const uint32_t idesc = idesc_bf16(128, 192);
    for (int kb = 0; kb < KB; ++kb) {
      const int s = kb % ST;
      if (!__all_sync(0xffffffffu, (!g.ln_prebuilt || mbar_wait(&bar_a[kb], 0, status)) &&
                                       mbar_wait(&full[s], (kb / ST) & 1, status)))
        break;
      tc_fence_after();
      if (lane == 0) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint64_t ad = sdesc_sw128(smem_u32(sA) + kb * kBlk + j * 32);
          const uint64_t bd = sdesc_sw128(smem_u32(sB) + s * B_BLK + j * 32);
          umma_bf16(tmem, ad, bd, idesc, (kb | j) ? 1u : 0u);
        }
        umma_commit(&empty[s]);
      }
      __syncwarp();
      if (kb + ST < KB) {
        if (!__all_sync(0xffffffffu, mbar_wait(&empty[s], (kb / ST) & 1, status))) break;
        if (lane == 0) {
          mbar_arrive_expect_tx(&full[s], B_BLK);
          bulk_g2s(sB + s * B_BLK, wq + (size_t)(kb + ST) * 192 * 64, B_BLK, &full[s]);
        }
        __syncwarp();
      }
    }
    LEWM_STAMP(2, 3);
    if (lane == 0) umma_commit(bar_mma);
    __syncwarp();
  }
  const bool ok = cta_wait_mma(bar_mma, status, tmem_slot + 1);
  LEWM_STAMP(2, 4);
  __syncwarp();
  tc_fence_after();
  qkv_attn_epilogue<D>(md, g, b, layer, head, tile, tmem, ok, kv, spart, sO, [] {});
  LEWM_STAMP(2, 6);
  __syncwarp();
  if (warp == 0) tmem_dealloc(tmem, 256);
}

// ---------------------------------------------------------------- QKV + attention, persistent
// k_qkv_attn for calls with many row tiles whose operands k_ln_operand prebuilt (width
// 192): one CTA per (head, tile group) keeps the head's QKV weights in shared memory for
// the whole launch (the one-tile kernel reloads 72 KB per tile) and loops over its tiles;
// as soon as a tile's MMAs retire it issues the next tile's operand copy, which lands
// during the attention epilogue, and part-way through that epilogue thread 0 issues the
// next tile's MMAs into the second of two TMEM accumulators, so the tensor pipe works
// while the epilogue runs. The k / v scratch has its own space instead of aliasing
// the operand and weights. Per tile the MMAs and the epilogue are those of k_qkv_attn: the
// same bits. A timed-out wait ends the CTA's loop (the flag comes from one warp through
// shared memory, so every thread leaves at the same tile).
template <int D>
constexpr int smem_qkv_ps() {
  constexpr int SCR = 128 * kKVStride * 4 + 4 * kMaxWindow * 128 * 4;
  constexpr int W = Cfg<D>::KB * 192 * 128, A = Cfg<D>::KB * kBlk;
  return 1024 + W + A + ((SCR + 1023) & ~1023) + kBlk + 8 * 8 + 16;
}

template <int D>
__global__ void __launch_bounds__(kThreads) k_qkv_attn_ps(DevWeights w, ModelDims md, CallGeom g, RolloutBufs b,
                                                          int layer, uint32_t* status) {
  constexpr int KB = Cfg<D>::KB;
  constexpr int B_BLK = 192 * 128;
  constexpr int SCR = 128 * kKVStride * 4 + 4 * kMaxWindow * 128 * 4;
  static_assert(Cfg<D>::QKV_ST == KB, "every weight block resident");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* sB = smem;                      // the head's QKV weights, [KB][192 x 64]
  uint8_t* sA = sB + KB * B_BLK;           // operand of the current tile, [KB][128 x 64]
  float* kv = reinterpret_cast<float*>(sA + KB * kBlk);  // [128][kKVStride] k | v of the tile's rows
  float* spart = kv + 128 * kKVStride;                    // [4 parts][kMaxWindow][128] partial scores
  uint8_t* sO = reinterpret_cast<uint8_t*>(kv) + ((SCR + 1023) & ~1023);  // output block [128 x 64]
  uint64_t* bar_w = reinterpret_cast<uint64_t*>(sO + kBlk);  // [KB] weights
  uint64_t* bar_a = bar_w + KB;                               // operand of a tile (one phase per tile)
  uint64_t* bar_mma = bar_a + 1;                              // MMAs of a tile retired (one phase per tile)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_mma + 1);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int head = blockIdx.x, grp = blockIdx.y, ngrp = gridDim.y;
  const __nv_bfloat16* wq = w.qkv + (size_t)((layer * md.heads + head) * KB) * (192 * 64);
  if (tid == 0) {
    for (int kb = 0; kb < KB; ++kb) mbar_init(&bar_w[kb], 1);
    mbar_init(bar_a, 1);
    mbar_init(bar_mma, 1);
    fence_mbar_init();
  }
  __syncwarp();
  if (warp == 0) {
    if (lane < KB) {  // weights before the wait, one copy per lane
      mbar_arrive_expect_tx(&bar_w[lane], B_BLK);
      bulk_g2s(sB + lane * B_BLK, wq + (size_t)lane * 192 * 64, B_BLK, &bar_w[lane]);
    }
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  griddep_wait();
  griddep_launch();
  auto issue_operand = [&](int t) {  // warp 0: the prebuilt operand of tile t, one copy per lane
    if (lane == 0) mbar_arrive_expect_tx(bar_a, KB * g.rows8 * 128);
    __syncwarp();
    if (lane < KB)
      bulk_g2s(sA + lane * kBlk, b.a_op + ((size_t)t * KB + lane) * kBlkElems, g.rows8 * 128, bar_a);
    __syncwarp();
  };
  if (warp == 0 && grp < g.n_tiles) issue_operand(grp);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t idesc = idesc_bf16(128, 192);
  // Thread 0: the MMAs of the i-th tile of this CTA into accumulator i & 1 (TMEM columns
  // 256 (i & 1) ..), once its operand landed; commits bar_mma even when a wait gave up.
  auto issue_mma = [&](int i) {
    bool got = mbar_wait(bar_a, i & 1, status);
    for (int kb = 0; kb < KB; ++kb) got = got && mbar_wait(&bar_w[kb], 0, status);
    tc_fence_after();
    if (got) umma_tile(tmem + (i & 1) * 256, smem_u32(sA), kBlk, smem_u32(sB), B_BLK, 0, KB, idesc, false);
    umma_commit(bar_mma);
  };
  if (tid == 0 && grp < g.n_tiles) issue_mma(0);
  for (int i = 0, t = grp; t < g.n_tiles; ++i, t += ngrp) {
    const bool ok = cta_wait_mma(bar_mma, status, tmem_slot + 1, i & 1);
    if (!ok) break;  // the same verdict in every thread
    tc_fence_after();
    const bool more = t + ngrp < g.n_tiles;
    if (warp == 0 && more) issue_operand(t + ngrp);  // sA is free: the MMAs retired
    qkv_attn_epilogue<D>(md, g, b, layer, head, t, tmem + (i & 1) * 256, ok, kv, spart, sO, [&] {
      if (tid == 0 && more) issue_mma(i + 1);  // accumulator (i + 1) & 1 was drained last iteration
    });
    tc_fence_before();
    __syncthreads();  // every TMEM read and shared-scratch use of tile t done before the next MMAs
    tc_fence_after();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 512);
}

// ---------------------------------------------------------------- K-split residual-branch GEMM
// Bytes after the operand slots: 5 barriers, the TMEM slot and a flag.
constexpr int kKSplit = 2;  // K halves of the out-projection GEMM (FC2: CallGeom::fc2_parts)
template <int D>
__host__ __device__ constexpr int resid_extra() { return 8 * 5 + 16; }
// K blocks per copy group: the N = D/4 pieces stream KG blocks; the N = D (192) tile's
// 24 KB weight blocks stream two at a time (2 groups x 2 x (A + B) in shared memory).
template <int D, int NT>
__host__ __device__ constexpr int partial_kg() { return NT == Cfg<D>::NT_OUT ? Cfg<D>::KG : 2; }

// part[kh][rows][n-tile] = A[:, K part kh] . B[n-tile, K part kh]^T for the out-projection
// or FC2 of a layer. Grid (tiles, 4 N tiles, K parts): each CTA issues 1 / gridDim.z of
// the MMAs and all its operand blocks fit one copy round. The bias, gate and residual
// add are applied by the consumer of the sum (the next GEMM's operand builder, or
// k_final), which adds the parts in a fixed order. Warp 0 issues MMAs, warp 1 refills the
// operand slots when they do not all fit.
template <int D, int NT>
__global__ void __launch_bounds__(kThreads) k_partial_gemm(const __nv_bfloat16* __restrict__ gA, int nkb,
                                                           const __nv_bfloat16* __restrict__ gB, CallGeom g,
                                                           float* __restrict__ part, size_t part_stride, int skind,
                                                           uint32_t* status) {
  using C = Cfg<D>;
  constexpr int CW = NT / 4;          // columns per warp slice
  constexpr int B_BLK = NT * 128;
  constexpr int PW = D / 4;           // columns of one partial-sum piece
  constexpr int NLP = NT / PW;        // pieces this CTA writes (1, or 4 when N = D)
  constexpr int TMEM_COLS = NT <= 64 ? 64 : (NT <= 128 ? 128 : 256);
  static_assert(NT % PW == 0 && NT <= 256, "N tile");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  const int tile = blockIdx.x, nt = blockIdx.y, kh = blockIdx.z;
  const int kcount = nkb / (int)gridDim.z, kb0 = kh * kcount;
  const ResidLayout lay = resid_layout(g.rows8, kcount, B_BLK, partial_kg<D, NT>(), resid_extra<D>());
  uint8_t* sA = smem;
  uint8_t* sB = smem + lay.b_off;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + lay.v_off);
  uint64_t* empty = full + 2;
  uint64_t* bar_mma = empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_mma + 1);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  (void)skind;  // diagnostic stamp stream
  const KStream<B_BLK> ks{sA, sB, full, empty, gA + ((size_t)tile * nkb + kb0) * kBlkElems, (size_t)kBlkElems,
                          gB + ((size_t)nt * nkb + kb0) * NT * 64, (size_t)NT * 64, (uint32_t)g.rows8 * 128,
                          (uint32_t)lay.a_stride, kcount, lay.G};
  if (tid == 0) {
    for (int h = 0; h < 2; ++h) {
      mbar_init(&full[h], 1);
      mbar_init(&empty[h], 1);
    }
    mbar_init(bar_mma, 1);
    fence_mbar_init();
    mbar_arrive_expect_tx(&full[0], ks.bytes(0));
    if (ks.groups() > 1) mbar_arrive_expect_tx(&full[1], ks.bytes(1));
  }
  __syncwarp();
  if (warp == 0) ks.issue_first(lane, false);  // weights before the wait, one instruction
  __syncwarp();
  if (warp == 0) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  LEWM_STAMP(skind, 1);
  griddep_wait();
  LEWM_STAMP(skind, 2);
  griddep_launch();
  if (warp == 0) ks.issue_first(lane, true);
  LEWM_STAMP(skind, 5);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (warp == 0) {  // MMA issuer
    ks.mma(tmem, idesc_bf16(128, NT), lane, status);
    LEWM_STAMP(skind, 3);
    if (lane == 0) umma_commit(bar_mma);
    __syncwarp();
  } else if (warp == 1) {
    ks.produce(lane, status);
  }
  const bool ok = cta_wait_mma(bar_mma, status, tmem_slot + 1);
  LEWM_STAMP(skind, 4);
  __syncwarp();
  tc_fence_after();
  const int quad = warp & 3, slice = warp >> 2;
  const int r = quad * 32 + lane;
  const uint32_t taddr = tmem + ((uint32_t)(quad * 32) << 16) + slice * CW;
  float v[CW];
  tmem_ld_cols<CW>(taddr, v);
  LEWM_STAMP(skind, 7);
  // The CTA's pieces staged as slabs in the operand slots (dead once the MMAs retired),
  // then one bulk copy per piece. The slabs (rows8 x NT floats) fit below the barriers
  // (checked; the A slots alone hold rows8 x 128 bytes per K block plus a 16 KB tail).
  float* slab = reinterpret_cast<float*>(smem);
  const bool fits = g.rows8 * NT * 4 <= lay.v_off;
  const int col0 = slice * CW;  // CTA-local first column of this warp slice
  if (fits && r < g.rows8)
    stage_part_row<D, CW>(slab + (col0 / PW) * g.rows8 * PW, r, (col0 % PW) / 4, v);
  fence_async_smem();
  __syncthreads();
  LEWM_STAMP(skind, 9);
  if (warp == 0 && lane < NLP) {  // each issuing lane waits for its own copy's reads
    if (ok && fits)
      bulk_s2g(part + kh * part_stride + ((size_t)tile * 4 + nt * NLP + lane) * 128 * PW,
               slab + lane * g.rows8 * PW, g.rows8 * PW * 4);
    bulk_commit();
    bulk_wait_read();
  }
  if (tid == 0 && !fits) atomicOr(status, LEWM_DEV_BADARG);
  LEWM_STAMP(skind, 6);
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, TMEM_COLS);
}

// ---------------------------------------------------------------- FC1 + GELU
// One CTA per (row tile, 32 hidden columns): h[:, 32 nt .. 32 nt + 32) = GELU(A . W1^T + b1).
// The weight operand of an N tile is one quarter (4 KB, 32 rows) of a pre-swizzled
// [128 x 64] block; the swizzle repeats every 8 rows, so the quarter is itself a
// valid SW128 operand. Each A K-block has its own barrier so the first MMA
// starts when the first block lands. The 32 columns are half of a swizzled h
// block, so the epilogue stores them directly (16 bytes per thread).
template <int D, int NT>
__global__ void __launch_bounds__(kThreads) k_fc1(DevWeights w, ModelDims md, CallGeom g, RolloutBufs b, int layer,
                                                  uint32_t* status) {
  using C = Cfg<D>;
  constexpr int KB = C::KB;
  constexpr int ST = C::QKV_ST;
  constexpr int CW = NT / 4;     // columns per warp slice
  constexpr int PER128 = 128 / NT;  // N tiles per packed 128-row weight block
  constexpr int PER64 = 64 / NT;    // N tiles per 64-column h block
  constexpr int B_BLK = NT * 128;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* sA = smem;
  uint8_t* sB = smem + KB * kBlk;
  float* svec = reinterpret_cast<float*>(sB + ST * B_BLK);  // [b1 NT]
  uint64_t* full = reinterpret_cast<uint64_t*>(svec + NT);
  uint64_t* empty = full + ST;
  uint64_t* bar_mma = empty + ST;
  uint64_t* bar_a = bar_mma + 1;  // [KB], operand bulk copies when prebuilt
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_a + KB);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  LEWM_STAMP(4, 0);
  const int tile = blockIdx.x, nt = blockIdx.y;
  const int nmlp = md.mlp / 128;
  const __nv_bfloat16* wb =
      w.w1 + (size_t)((layer * nmlp + nt / PER128) * KB) * kBlkElems + (size_t)(nt % PER128) * (NT * 64);
  if (tid == 0) {
    for (int s = 0; s < ST; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(bar_mma, 1);
    for (int kb = 0; kb < KB; ++kb) mbar_init(&bar_a[kb], 1);
    fence_mbar_init();
    mbar_arrive_expect_tx(&full[0], B_BLK + NT * 4);
    for (int s = 1; s < ST; ++s) mbar_arrive_expect_tx(&full[s], B_BLK);
  }
  __syncwarp();
  if (warp == 0) {  // one copy per lane
    if (lane < ST)
      bulk_g2s(sB + lane * B_BLK, wb + (size_t)lane * kBlkElems, B_BLK, &full[lane]);
    else if (lane == ST)
      bulk_g2s(svec, w.b1 + layer * md.mlp + nt * NT, NT * 4, &full[0]);
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, NT);
    tmem_relinquish();
  }
  // A operand: LN2 -> modulate (shift/scale_mlp of this layer) -> ffn.norm of s = r +
  // gate_msa * (P0 + P1 + out_b), the out-projection update; the N-tile-0 CTAs write s back.
  // The residual rows r (written by k_qkv_attn, two launches back) and the modulation are
  // loaded before the wait.
  const size_t t0 = (size_t)tile * 128 * D;
  const ResidUpdate u{b.x + t0, b.part_a + t0, b.part_stride, 2, w.out_b + layer * D, layer * 6 * D + 2 * D,
                      nt == 0 ? b.xs + t0 : nullptr};
  LnEarly<D, D / 12> pf;
  if (!g.ln_prebuilt)
    prefetch_ln_operand<D>(pf, u, g, tile, b.mod, md.L * 6 * D, layer * 6 * D + 3 * D, tid, 0, g.rows8, true);
  LEWM_STAMP(4, 1);
  griddep_wait();
  LEWM_STAMP(4, 2);
  griddep_launch();
  if (g.ln_prebuilt) {  // built once per tile by k_ln_operand: one copy per lane
    if (warp == 0 && lane < KB) {
      mbar_arrive_expect_tx(&bar_a[lane], g.rows8 * 128);
      bulk_g2s(sA + lane * kBlk, b.a_op + ((size_t)tile * KB + lane) * kBlkElems, g.rows8 * 128, &bar_a[lane]);
    }
  } else {
    build_ln_operand<D>(u, g, tile, b.mod, md.L * 6 * D, layer * 6 * D + 3 * D, w.ffn_ln_w + layer * D,
                        w.ffn_ln_b + layer * D, sA, tid, &pf);
  }
  fence_async_smem();
  LEWM_STAMP(4, 5);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (warp == 0) {  // whole warp waits, lane 0 issues
    const uint32_t idesc = idesc_bf16(128, NT);
    for (int kb = 0; kb < KB; ++kb) {
      const int s = kb % ST;
      if (!__all_sync(0xffffffffu, (!g.ln_prebuilt || mbar_wait(&bar_a[kb], 0, status)) &&
                                       mbar_wait(&full[s], (kb / ST) & 1, status)))
        break;
      tc_fence_after();
      if (lane == 0) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint64_t ad = sdesc_sw128(smem_u32(sA) + kb * kBlk + j * 32);
          const uint64_t bd = sdesc_sw128(smem_u32(sB) + s * B_BLK + j * 32);
          umma_bf16(tmem, ad, bd, idesc, (kb | j) ? 1u : 0u);
        }
        umma_commit(&empty[s]);
      }
      __syncwarp();
      if (kb + ST < KB) {
        if (!__all_sync(0xffffffffu, mbar_wait(&empty[s], (kb / ST) & 1, status))) break;
        if (lane == 0) {
          mbar_arrive_expect_tx(&full[s], B_BLK);
          bulk_g2s(sB + s * B_BLK, wb + (size_t)(kb + ST) * kBlkElems, B_BLK, &full[s]);
        }
        __syncwarp();
      }
    }
    LEWM_STAMP(4, 3);
    if (lane == 0) umma_commit(bar_mma);
    __syncwarp();
  }
  const bool ok = cta_wait_mma(bar_mma, status, tmem_slot + 1);
  LEWM_STAMP(4, 4);
  __syncwarp();
  tc_fence_after();
  {  // warp slice s owns hidden columns [CW s, CW s + CW) of this NT-wide tile
    const int quad = warp & 3, slice = warp >> 2;
    const int r = quad * 32 + lane;
    const RowMap m = map_row(g, tile, r);
    const bool valid = ok && m.valid;
    const uint32_t taddr = tmem + ((uint32_t)(quad * 32) << 16) + slice * CW;
    const float* bs = svec + slice * CW;
    float v[CW];
    tmem_ld_cols<CW>(taddr, v);
    LEWM_STAMP(4, 8);
    const int nkm = md.mlp / 64;
    uint8_t* hb = reinterpret_cast<uint8_t*>(b.h + ((size_t)tile * nkm + nt / PER64) * kBlkElems);
#pragma unroll
    for (int i = 0; i < CW; i += 8) {
      uint4 pk = make_uint4(0u, 0u, 0u, 0u);
      if (valid) {
        pk.x = pack_bf16x2(gelu_f(v[i] + bs[i]), gelu_f(v[i + 1] + bs[i + 1]));
        pk.y = pack_bf16x2(gelu_f(v[i + 2] + bs[i + 2]), gelu_f(v[i + 3] + bs[i + 3]));
        pk.z = pack_bf16x2(gelu_f(v[i + 4] + bs[i + 4]), gelu_f(v[i + 5] + bs[i + 5]));
        pk.w = pack_bf16x2(gelu_f(v[i + 6] + bs[i + 6]), gelu_f(v[i + 7] + bs[i + 7]));
      }
      if (r < g.rows8) *reinterpret_cast<uint4*>(hb + sw128_off(r, (nt % PER64) * NT + slice * CW + i)) = pk;
    }
    LEWM_STAMP(4, 9);
  }
  LEWM_STAMP(4, 7);
  tc_fence_before();
  __syncthreads();
  LEWM_STAMP(4, 6);
  if (warp == 0) tmem_dealloc(tmem, NT);
}

// ---------------------------------------------------------------- fused feed-forward (small tiles)
// One CTA per (row tile, hidden quarter q of 192 units), for tiles whose operand is built
// in-kernel (at most 32 rows) at width 192: the FC1 operand (s = r + gate_msa *
// (out-proj + bias), LN2 -> modulate -> ffn.norm; the q == 0 CTAs write s back), FC1 on
// the quarter's 192 hidden units (N = 192, K = D) + bias -> GELU into shared memory, then
// the quarter's FC2 contribution to all D outputs (N = 192, K = 192) as the fp32 partial
// P_q. The consumer adds the four quarters in a fixed order. Replaces k_fc1 and the FC2
// k_partial_gemm: one kernel boundary and the global round trip of h fewer per layer.
// The FC1 accumulator is staged through shared memory so all 16 warps share the GELUs
// (TMEM lanes 0-31, the tile's rows, belong to 4 warps).
constexpr int kFfnQ = 192;  // hidden units per fused-FFN CTA
template <int D>
constexpr int smem_ffn() {
  return 1024 + (D / 64) * kBlk + (D / 64) * kFfnQ * 128 + (kFfnQ / 64) * D * 128 + kFfnQ * 4 + 8 * 5 + 16;
}

template <int D>
__global__ void __launch_bounds__(kThreads) k_ffn(DevWeights w, ModelDims md, CallGeom g, RolloutBufs b, int layer,
                                                  uint32_t* status) {
  constexpr int KB = D / 64;          // K blocks of FC1
  constexpr int HB = kFfnQ / 64;      // K blocks of FC2 (this quarter's hidden units)
  constexpr int W1_BLK = kFfnQ * 128; // [192 hidden x 64] bf16
  constexpr int W2_BLK = D * 128;     // [D x 64] bf16
  constexpr int NT2 = Cfg<D>::NT_OUT; // rows of one packed FC2 weight piece (N tile)
  constexpr int kStage = kFfnQ + 4;   // floats per staged row: 16-byte rows, float4 accesses conflict-free
  static_assert(HB == KB, "h reuses the operand blocks");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* sA = smem;                                  // FC1 operand, then h (FC2 operand)
  uint8_t* sW1 = smem + KB * kBlk;                     // FC1 weights, then the staged accumulator
  uint8_t* sW2 = sW1 + KB * W1_BLK;
  float* sb1 = reinterpret_cast<float*>(sW2 + HB * W2_BLK);
  // [0] W1+b1, [1] W2, [2] FC1 done, [3] FC2 done, [4] prebuilt operand
  uint64_t* bars = reinterpret_cast<uint64_t*>(sb1 + kFfnQ);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 5);
  float* stage = reinterpret_cast<float*>(sW1);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int tile = blockIdx.x, q = blockIdx.y;
  const int nmlp = md.mlp / 128, nkm = md.mlp / 64;
  if (tid == 0) {
    for (int i = 0; i < 5; ++i) mbar_init(&bars[i], 1);
    fence_mbar_init();
    mbar_arrive_expect_tx(&bars[0], KB * W1_BLK + kFfnQ * 4);
    mbar_arrive_expect_tx(&bars[1], HB * W2_BLK);
  }
  __syncwarp();
  if (warp == 0) {  // weights before the wait: 2 x KB + 4 x HB + 1 copies in one instruction
    const int h0 = kFfnQ * q;                 // first hidden unit
    const int hb0 = h0 / 128, r0 = h0 % 128;  // its packed 128-row block and row (0 or 64)
    if (lane < 2 * KB) {
      // FC1 block kb: rows [r0, 128) of block hb0, then rows [0, 64 + r0) of block hb0 + 1
      const int kb = lane >> 1, second = lane & 1;
      const __nv_bfloat16* src =
          w.w1 + ((size_t)(layer * nmlp + hb0 + second) * KB + kb) * kBlkElems + (second ? 0 : (size_t)r0 * 64);
      const uint32_t bytes = second ? (64 + r0) * 128 : (128 - r0) * 128;
      bulk_g2s(sW1 + kb * W1_BLK + (second ? (128 - r0) * 128 : 0), src, bytes, &bars[0]);
    } else if (lane < 2 * KB + 4 * HB) {
      // FC2 block j: the four packed N-tile pieces [NT2 x 64] of hidden K block 3q + j
      const int i = lane - 2 * KB, j = i >> 2, nt = i & 3;
      const __nv_bfloat16* src =
          w.w2 + (((size_t)layer * 4 + nt) * nkm + HB * q + j) * NT2 * 64;
      bulk_g2s(sW2 + j * W2_BLK + nt * NT2 * 128, src, NT2 * 128, &bars[1]);
    } else if (lane == 2 * KB + 4 * HB) {
      bulk_g2s(sb1, w.b1 + layer * md.mlp + kFfnQ * q, kFfnQ * 4, &bars[0]);
    }
  }
  __syncwarp();
  if (warp == 0) {
    tmem_alloc(tmem_slot, 256);
    tmem_relinquish();
  }
  // FC1 operand: on tiles of more than 32 rows built once per tile by k_ln_operand and
  // bulk-copied (one copy per lane); otherwise built here from the residual rows with the
  // out-projection update pending (rows written by k_qkv_attn two launches back and the
  // modulation are loaded before the wait; the q == 0 CTAs write the updated rows back).
  const size_t t0 = (size_t)tile * 128 * D;
  const ResidUpdate u{b.x + t0, b.part_a + t0, b.part_stride, 2, w.out_b + layer * D, layer * 6 * D + 2 * D,
                      q == 0 ? b.xs + t0 : nullptr};
  LnEarly<D, D / 12> pf;
  if (!g.ln_prebuilt)
    prefetch_ln_operand<D>(pf, u, g, tile, b.mod, md.L * 6 * D, layer * 6 * D + 3 * D, tid, 0, g.rows8, true);
  LEWM_STAMP(4, 1);
  griddep_wait();
  LEWM_STAMP(4, 2);
  griddep_launch();
  if (g.ln_prebuilt) {
    if (warp == 0) {
      if (lane == 0) mbar_arrive_expect_tx(&bars[4], KB * g.rows8 * 128);
      __syncwarp();
      if (lane < KB)
        bulk_g2s(sA + lane * kBlk, b.a_op + ((size_t)tile * KB + lane) * kBlkElems, g.rows8 * 128, &bars[4]);
    }
  } else {
    build_ln_operand<D, 7>(u, g, tile, b.mod, md.L * 6 * D, layer * 6 * D + 3 * D, w.ffn_ln_w + layer * D,
                           w.ffn_ln_b + layer * D, sA, tid, &pf);
  }
  fence_async_smem();
  LEWM_STAMP(4, 5);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t idesc = idesc_bf16(128, 192);
  if (warp == 0) {  // FC1: D[0, 192) = A . W1^T
    const bool got = __all_sync(0xffffffffu, mbar_wait(&bars[0], 0, status) &&
                                                 (!g.ln_prebuilt || mbar_wait(&bars[4], 0, status)));
    tc_fence_after();
    if (lane == 0) {
      if (got) {
        uint64_t ad = sdesc_sw128(smem_u32(sA)), bd = sdesc_sw128(smem_u32(sW1));
        for (int kb = 0; kb < KB; ++kb) {
#pragma unroll
          for (int j = 0; j < 4; ++j) umma_bf16(tmem, ad + 2 * j, bd + 2 * j, idesc, (kb | j) ? 1u : 0u);
          ad += kBlk >> 4;
          bd += W1_BLK >> 4;
        }
      }
      umma_commit(&bars[2]);
    }
    __syncwarp();
  }
  const bool ok1 = cta_wait_mma(&bars[2], status, tmem_slot + 1);
  LEWM_STAMP(4, 3);
  tc_fence_after();
  const int quad = warp & 3, slice = warp >> 2;
  const int r = quad * 32 + lane;
  if (g.rows8 > 64) {
    // Every TMEM lane quadrant holds rows: each warp applies bias + GELU to its 32 rows x
    // 48 hidden columns straight from TMEM, 16 at a time, into h (the FC2 operand, in sA).
    if (quad * 32 < g.rows8) {
      const bool valid = ok1 && r < g.rows8 && map_row(g, tile, r).valid;  // empty window slots stay zero
      LEWM_STAMP(4, 0);
#pragma unroll 1
      for (int cc = 0; cc < 48; cc += 16) {
        float v[16];
        tmem_ld_cols<16>(tmem + ((uint32_t)(quad * 32) << 16) + slice * 48 + cc, v);
        const int c0 = slice * 48 + cc;  // multiple of 16: two 8-column chunks of one 64-column block
        uint32_t pk[8];
#pragma unroll
        for (int i = 0; i < 8; ++i)
          pk[i] = valid ? pack_bf16x2(gelu_f(v[2 * i] + sb1[c0 + 2 * i]), gelu_f(v[2 * i + 1] + sb1[c0 + 2 * i + 1]))
                        : 0u;
        if (r < g.rows8) {
          uint8_t* blk = sA + (c0 >> 6) * kBlk;
          *reinterpret_cast<uint4*>(blk + sw128_off(r, c0 & 63)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
          *reinterpret_cast<uint4*>(blk + sw128_off(r, (c0 & 63) + 8)) = make_uint4(pk[4], pk[5], pk[6], pk[7]);
        }
      }
    }
  } else {
    // At most two quadrants hold rows: stage the accumulator through the dead W1 slots
    // so all 16 warps share the GELUs.
    if (quad * 32 < g.rows8) {  // stage the accumulator rows of the tile (whole warps load)
      float v[48];
      tmem_ld_cols<48>(tmem + ((uint32_t)(quad * 32) << 16) + slice * 48, v);
      if (r < g.rows8) {
        float4* sr = reinterpret_cast<float4*>(stage + r * kStage + slice * 48);
#pragma unroll
        for (int i = 0; i < 12; ++i) sr[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
      }
    }
    __syncthreads();
    LEWM_STAMP(4, 0);
    // bias + GELU over all threads into h (the FC2 operand, in sA): 12 columns of one row
    // per item, loaded first so the 12 GELUs overlap (one item per thread at 32 rows).
    constexpr int kCpi = 12;
    static_assert(kFfnQ == 16 * kCpi, "16 items per row");
    for (int it = tid; it < g.rows8 * 16; it += kThreads) {
      const int rr = it >> 4, c = (it & 15) * kCpi;
      const float4* sr = reinterpret_cast<const float4*>(stage + rr * kStage + c);
      const float4* sb = reinterpret_cast<const float4*>(sb1 + c);
      float hv[kCpi];
#pragma unroll
      for (int i = 0; i < kCpi / 4; ++i) {
        const float4 a = sr[i], bq = sb[i];
        hv[4 * i] = a.x + bq.x;
        hv[4 * i + 1] = a.y + bq.y;
        hv[4 * i + 2] = a.z + bq.z;
        hv[4 * i + 3] = a.w + bq.w;
      }
      const bool valid = ok1 && map_row(g, tile, rr).valid;  // window slots without a candidate stay zero
#pragma unroll
      for (int i = 0; i < kCpi; i += 4) {
        uint2 pk = make_uint2(0u, 0u);
        if (valid) {
          pk.x = pack_bf16x2(gelu_f(hv[i]), gelu_f(hv[i + 1]));
          pk.y = pack_bf16x2(gelu_f(hv[i + 2]), gelu_f(hv[i + 3]));
        }
        *reinterpret_cast<uint2*>(sA + ((c + i) >> 6) * kBlk + sw128_off(rr, (c + i) & 63)) = pk;
      }
    }
  }
  fence_async_smem();
  LEWM_STAMP(4, 9);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) {  // FC2 partial: D[0, 192) = h . W2^T over this quarter's hidden units (FC1's
                    // columns: every thread's loads of them completed before the barrier)
    const bool got = __all_sync(0xffffffffu, mbar_wait(&bars[1], 0, status));
    tc_fence_after();
    if (lane == 0) {
      if (got) {
        uint64_t ad = sdesc_sw128(smem_u32(sA)), bd = sdesc_sw128(smem_u32(sW2));
        for (int kb = 0; kb < HB; ++kb) {
#pragma unroll
          for (int j = 0; j < 4; ++j) umma_bf16(tmem, ad + 2 * j, bd + 2 * j, idesc, (kb | j) ? 1u : 0u);
          ad += kBlk >> 4;
          bd += W2_BLK >> 4;
        }
      }
      umma_commit(&bars[3]);
    }
    __syncwarp();
  }
  const bool ok2 = cta_wait_mma(&bars[3], status, tmem_slot + 1);
  LEWM_STAMP(4, 4);
  tc_fence_after();
  // Warp slice s holds N piece s (D/4 = 48 columns): staged as four slabs of rows8 x 48
  // floats (up to 96 KB) in the W1 + W2 region (free since FC2 retired; the staged FC1
  // rows were read before the barrier above), then one bulk copy per piece.
  static_assert(D / 4 == 48, "one N piece per warp slice");
  float* slabs = stage;
  if (quad * 32 < g.rows8) {
    float v[48];
    tmem_ld_cols<48>(tmem + ((uint32_t)(quad * 32) << 16) + slice * 48, v);
    LEWM_STAMP(4, 8);
    if (r < g.rows8) stage_part_row<D, 48>(slabs + slice * g.rows8 * 48, r, 0, v);
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  LEWM_STAMP(4, 7);
  if (warp == 0 && lane < 4) {  // each issuing lane waits for its own copy's reads
    if (ok1 && ok2)
      bulk_s2g(b.part_b + q * b.part_stride + ((size_t)tile * 4 + lane) * 128 * 48, slabs + lane * g.rows8 * 48,
               g.rows8 * 48 * 4);
    bulk_commit();
    bulk_wait_read();
  }
  LEWM_STAMP(4, 6);
  if (warp == 0) tmem_dealloc(tmem, 256);
}

// ---------------------------------------------------------------- final LayerNorm + history / cost
// The last call: warp per candidate, final LayerNorm of the window's last token and its
// squared distance to the goal. Earlier calls: warp per (candidate, row p of the next
// call's window). The warp of the last row, the new prediction, computes the final
// LayerNorm of this call's last token, appends it to the history and prepares its row;
// the other warps prepare their rows from the history (observation embeddings or
// earlier predictions), which this call does not change.
// With a pred_proj head the step runs in two launches around the head's GEMMs: mode 1, a
// warp per candidate, writes the final-LayerNorm row of the new prediction as bf16 into the
// head's operand (b.pp_in); mode 2 is the step above with the new prediction read from the
// head's output rows (b.pp_out). Mode 0: no head (Identity).
template <int D>
__global__ void __launch_bounds__(128) k_final(DevWeights w, ModelDims md, CallGeom g, RolloutBufs b, int mode) {
  griddep_wait();
  griddep_launch();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // rows the next call processes per candidate (one warp per candidate in mode 1)
  const int rows_per_cand = (g.last || mode == 1) ? 1 : g.next_rpc;
  const int item = blockIdx.x * 4 + warp;
  if (item >= g.n_cand * rows_per_cand) return;
  const int cand = item / rows_per_cand, pi = item - cand * rows_per_cand;
  const int p = g.last ? pi : g.next_pos0 + pi;  // window position in the next call
  constexpr int NP = D / 64;
  const int NPred = g.T - g.H + 1;
  float* pcand = b.pred + (size_t)cand * NPred * D;
  const int j = g.next_start + p;  // history index of this row (unused when last)
  const bool new_pred = mode == 1 || g.last || (j - g.H == g.call);
  float2 v[NP];
  if (new_pred && mode == 2) {  // the head's output row
    const float* pr = b.pp_out + (size_t)cand * D;
#pragma unroll
    for (int i = 0; i < NP; ++i) v[i] = *reinterpret_cast<const float2*>(pr + 64 * i + 2 * lane);
  } else if (new_pred) {
    // Output of the last layer for the window's last token: s + gate_mlp * ((P0 + P1) + b2),
    // the FC2 update of the last layer still pending.
    const int tile = cand / g.cpt;
    const int r = (cand - tile * g.cpt) * g.rpc + (g.rpc - 1);  // window position w - 1
    const size_t o = ((size_t)tile * 128 + r) * D;
    const float* pt = b.part_b + (size_t)tile * 128 * D;  // the tile's partial block
    const int tok = cand * g.T + g.start + g.w - 1;
    const __nv_bfloat16* gate = b.mod + (size_t)tok * (md.L * 6 * D) + (md.L - 1) * 6 * D + 5 * D;
    const float* b2 = w.b2 + (md.L - 1) * D;
    float2 fw[NP], fb[NP];
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < NP; ++i) {
      const int c = 64 * i + 2 * lane;
      const float2 xs = *reinterpret_cast<const float2*>(b.xs + o + c);
      const int po = part_off<D>(r, c);
      float2 p0 = *reinterpret_cast<const float2*>(pt + po);
      float2 p1 = *reinterpret_cast<const float2*>(pt + b.part_stride + po);
      if (g.fc2_parts == 4) {  // four hidden-quarter partials: (P0 + P1) + (P2 + P3)
        const float2 p2 = *reinterpret_cast<const float2*>(pt + 2 * b.part_stride + po);
        const float2 p3 = *reinterpret_cast<const float2*>(pt + 3 * b.part_stride + po);
        p0 = make_float2(p0.x + p1.x, p0.y + p1.y);
        p1 = make_float2(p2.x + p3.x, p2.y + p3.y);
      }
      const float2 bb = *reinterpret_cast<const float2*>(b2 + c);
      const float2 gg = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(gate + c));
      v[i] = make_float2(xs.x + gg.x * ((p0.x + p1.x) + bb.x), xs.y + gg.y * ((p0.y + p1.y) + bb.y));
      fw[i] = *reinterpret_cast<const float2*>(w.fin_w + c);
      fb[i] = *reinterpret_cast<const float2*>(w.fin_b + c);
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
      v[i].x = (v[i].x - mean) * rstd * fw[i].x + fb[i].x;
      v[i].y = (v[i].y - mean) * rstd * fw[i].y + fb[i].y;
    }
    if (mode == 1) {  // row `cand` of the head's operand blocks
      uint8_t* blk = reinterpret_cast<uint8_t*>(b.pp_in) + (size_t)(cand / 128) * NP * kBlk;
#pragma unroll
      for (int i = 0; i < NP; ++i)
        *reinterpret_cast<uint32_t*>(blk + i * kBlk + sw128_off(cand % 128, 2 * lane)) =
            pack_bf16x2(v[i].x, v[i].y);
      return;
    }
  }
  if (new_pred) {
    if (g.last) {
      const int e = b.goal_per_cand ? cand : cand / g.S;
      const float* gr = b.goal + (size_t)e * D;
      float acc = 0.f;
#pragma unroll
      for (int i = 0; i < NP; ++i) {
        const float2 gv = *reinterpret_cast<const float2*>(gr + 64 * i + 2 * lane);
        const float dx = v[i].x - gv.x, dy = v[i].y - gv.y;
        acc += dx * dx + dy * dy;
      }
      acc = warp_sum(acc);
      if (lane == 0) b.costs[cand] = acc;
      return;
    }
#pragma unroll
    for (int i = 0; i < NP; ++i) *reinterpret_cast<float2*>(pcand + g.call * D + 64 * i + 2 * lane) = v[i];
  }
  // Row p of the candidate's next window (each lane reads back only its own columns).
  const int ntile = cand / g.next_cpt;
  const int e2 = b.emb_per_cand ? cand : cand / g.S;
  const float* src = new_pred ? pcand + (size_t)g.call * D
                              : ((j < g.H) ? b.emb + ((size_t)e2 * g.H + j) * D : pcand + (size_t)(j - g.H) * D);
  const int nr = (cand - ntile * g.next_cpt) * g.next_rpc + pi;
  prep_layer0_row<D>(w, src, p, b.xn + ((size_t)ntile * 128 + nr) * D, lane);
}

// ---------------------------------------------------------------- shared-memory sizes
template <int D>
constexpr int smem_embed_out() {
  return 1024 + 2 * Cfg<D>::KG * (kBlk + Cfg<D>::NT_OUT * 128) + Cfg<D>::NT_OUT * 4 + 8 * 5 + 16;
}
template <int D>
constexpr int smem_adaln() { return 1024 + Cfg<D>::KB * (kBlk + Cfg<D>::NT_ADA * 128) + Cfg<D>::NT_ADA * 4 + 64; }
template <int D>
constexpr int smem_qkv() {
  constexpr int R1 = Cfg<D>::KB * kBlk + Cfg<D>::QKV_ST * 192 * 128;
  constexpr int SCR = 128 * kKVStride * 4 + 4 * kMaxWindow * 128 * 4;
  constexpr int R1S = ((R1 > SCR ? R1 : SCR) + 1023) & ~1023;
  constexpr int SO_OFF = (((SCR + 1023) & ~1023) + kBlk <= R1) ? ((SCR + 1023) & ~1023) : R1S;
  constexpr int BAR_OFF = (SO_OFF + kBlk > R1S) ? SO_OFF + kBlk : R1S;
  return 1024 + BAR_OFF + 128;
}
template <int D>
constexpr int smem_resid() { return 232448; }  // per launch: resid_layout(...).bytes
template <int D, int NT>
constexpr int smem_fc1() { return 1024 + Cfg<D>::KB * kBlk + Cfg<D>::QKV_ST * NT * 128 + NT * 4 + 8 * (2 * Cfg<D>::QKV_ST + 1 + Cfg<D>::KB) + 16; }

static_assert(smem_qkv<192>() <= 232448 && smem_qkv<384>() <= 232448, "qkv smem");
static_assert(smem_embed_out<384>() <= 232448 && smem_adaln<384>() <= 232448, "embed/adaln smem");
static_assert(smem_fc1<384, kFc1N>() <= 232448 && smem_resid<384>() <= 232448, "fc smem");
static_assert(smem_ffn<192>() <= 232448, "ffn smem");
static_assert(smem_adaln_ps<192>() <= 232448, "persistent adaln smem");
static_assert(smem_qkv_ps<192>() <= 232448, "persistent qkv smem");

template <int D>
cudaError_t set_smem_attrs() {
  static bool done = false;  // per process; attributes are per device function
  if (done) return cudaSuccess;
  cudaError_t e;
  if ((e = cudaFuncSetAttribute(k_embed_out<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_embed_out<D>())))
    return e;
  if ((e = cudaFuncSetAttribute(k_adaln<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_adaln<D>()))) return e;
  if ((e = cudaFuncSetAttribute(k_qkv_attn<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_qkv<D>()))) return e;
  if constexpr (D == 192) {
    if ((e = cudaFuncSetAttribute(k_ffn<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_ffn<D>()))) return e;
    if ((e = cudaFuncSetAttribute(k_adaln_ps<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_adaln_ps<D>())))
      return e;
    if ((e = cudaFuncSetAttribute(k_qkv_attn_ps<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_qkv_ps<D>())))
      return e;
  }
  if constexpr (D == 192)
    if ((e = cudaFuncSetAttribute(k_partial_gemm<D, D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  smem_resid<D>())))
      return e;
  if ((e = cudaFuncSetAttribute(k_partial_gemm<D, Cfg<D>::NT_OUT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                smem_resid<D>())))
    return e;
  if ((e = cudaFuncSetAttribute(k_fc1<D, kFc1N>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_fc1<D, kFc1N>())))
    return e;
  done = true;
  return cudaSuccess;
}

template <int D>
cudaError_t embed_impl(const ModelDims& md, const DevWeights& w, const float* cand, int rows, __nv_bfloat16* eh,
                       __nv_bfloat16* act_a, uint32_t* status, cudaStream_t st, Prof* prof) {
  cudaError_t e = set_smem_attrs<D>();
  if (e) return e;
  const int tiles = (rows + 127) / 128;
  if (prof) prof->begin(st);
  e = launch_k(k_embed_hidden<D>, dim3(tiles, md.eh / 64), dim3(256), 0, st, w, md, cand, rows, eh);
  if (prof) prof->end(KC_EMBED, 2.0 * rows * ((double)md.A * md.As + (double)md.As * md.eh), st);
  if (e) return e;
  if (prof) prof->begin(st);
  e = launch_k(k_embed_out<D>, dim3(tiles, 4), dim3(kThreads), smem_embed_out<D>(), st, w, md, rows, eh, act_a, status);
  if (prof) prof->end(KC_EMBED, 2.0 * rows * (double)md.eh * D, st);
  return e;
}

// Tensor map of mod ([rows][ncols] bf16, row-major) for 128-byte-swizzled [128 x 64] TMA
// stores. cuTensorMapEncodeTiled comes from the driver through the runtime's entry-point
// query (no link against libcuda). False when it is unavailable or rejects the map: the
// caller then uses the one-tile kernel.
bool mod_tensor_map(CUtensorMap* map, void* mod, int rows, int ncols) {
  using Encode = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
  static Encode encode = [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      fn = nullptr;
    return reinterpret_cast<Encode>(fn);
  }();
  if (!encode || rows <= 0) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)ncols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)ncols * 2};
  const cuuint32_t box[2] = {64, 128};
  const cuuint32_t estr[2] = {1, 1};
  return encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, mod, dims, strides, box, estr,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int D>
cudaError_t adaln_impl(const ModelDims& md, const DevWeights& w, int rows, const __nv_bfloat16* act_a,
                       __nv_bfloat16* mod, uint32_t* status, cudaStream_t st, Prof* prof) {
  cudaError_t e = set_smem_attrs<D>();
  if (e) return e;
  const int tiles = (rows + 127) / 128;
  const int ntiles = md.L * 6 * D / Cfg<D>::NT_ADA;
  if (prof) prof->begin(st);
  // Calls with at least 4 row tiles per CTA group run the persistent pipeline (the same bits).
  static const int ps_env = [] {
    const char* v = std::getenv("LEWM_ADALN_PERSISTENT");
    return v ? std::atoi(v) : 1;
  }();
  bool ps = false;
  if constexpr (D == 192) {
    CUtensorMap map;
    ps = ps_env != 0 && tiles >= 4 * kAdaGroups && mod_tensor_map(&map, mod, rows, md.L * 6 * D);
    if (ps)
      e = launch_k(k_adaln_ps<D>, dim3(ntiles, kAdaGroups), dim3(kThreads), smem_adaln_ps<D>(), st, w, md, rows,
                   act_a, map, status);
  }
  if (!ps)
    e = launch_k(k_adaln<D>, dim3(tiles, ntiles), dim3(kThreads), smem_adaln<D>(), st, w, md, rows, act_a, mod,
                 status);
  if (prof) prof->end(KC_ADALN, 2.0 * rows * (double)D * md.L * 6 * D, st);
  return e;
}

template <int D>
cudaError_t prep0_impl(const ModelDims& md, const DevWeights& w, const CallGeom& g, const RolloutBufs& b,
                       cudaStream_t st, Prof* prof) {
  if (prof) prof->begin(st);
  const cudaError_t e = launch_k(k_prep0<D>, dim3((g.n_cand * g.w + 3) / 4), dim3(128), 0, st, w, md, g, b);
  if (prof) prof->end(KC_PREP0, 0.0, st);
  return e;
}

template <int D>
cudaError_t call_impl(const ModelDims& md, const DevWeights& w, const CallGeom& g, const RolloutBufs& b,
                      uint32_t* status, cudaStream_t st, Prof* prof) {
  cudaError_t e = set_smem_attrs<D>();
  if (e) return e;
  const int nkb_inner = md.inner / 64, nkb_mlp = md.mlp / 64;
  const double rows = (double)g.n_cand * g.rpc;  // valid rows this call processes
#define LEWM_TRY(x)                         \
  do {                                      \
    if ((e = (x)) != cudaSuccess) return e; \
  } while (0)
  const int op_rows = kThreads / (D / 12);  // rows per k_ln_operand CTA
  const dim3 op_grid(g.n_tiles, (g.rows8 + op_rows - 1) / op_rows);
  const int mcols = md.L * 6 * D;
  for (int l = 0; l < md.L; ++l) {
    if (g.ln_prebuilt) {  // QKV operand of every tile: LN1 -> modulate -> attn.norm (+ pending FC2 update)
      ResidUpdate u{b.x, nullptr, 0, 2, nullptr, 0, nullptr};
      if (l > 0)
        u = ResidUpdate{b.xs, b.part_b, b.part_stride, g.fc2_parts, w.b2 + (l - 1) * D,
                        (l - 1) * 6 * D + 5 * D, b.x};
      if (prof) prof->begin(st);
      LEWM_TRY(launch_k(k_ln_operand<D>, op_grid, dim3(kThreads), 0, st, u, g, (const __nv_bfloat16*)b.mod, mcols,
                        l * 6 * D, w.attn_ln_w + l * D, w.attn_ln_b + l * D, b.a_op, l > 0 ? 1 : 0));
      if (prof) prof->end(KC_LN_OP, 0.0, st);
    }
    if (prof) prof->begin(st);
    bool qkv_done = false;
    if constexpr (D == 192) {
      if (g.qkv_persistent) {
        LEWM_TRY(launch_k(k_qkv_attn_ps<D>, dim3(md.heads, kQkvGroups), dim3(kThreads), smem_qkv_ps<D>(), st, w, md,
                          g, b, l, status));
        qkv_done = true;
      }
    }
    if (!qkv_done)
      LEWM_TRY(launch_k(k_qkv_attn<D>, dim3(g.n_tiles, md.heads), dim3(kThreads), smem_qkv<D>(), st, w, md, g, b, l,
                        status));
    if (prof) prof->end(KC_QKV_ATTN, 2.0 * rows * D * 3 * md.inner + 4.0 * rows * g.w * md.inner, st);
    // out-projection partial sums (bias, gate_msa and residual applied by FC1's operand builder)
    if (prof) prof->begin(st);
    if constexpr (D == 192) {
      if (g.outproj_wide)
        LEWM_TRY(launch_k(k_partial_gemm<D, D>, dim3(g.n_tiles, 1, kKSplit), dim3(kThreads),
                          resid_layout(g.rows8, nkb_inner / kKSplit, D * 128, partial_kg<D, D>(), resid_extra<D>())
                              .bytes,
                          st, (const __nv_bfloat16*)b.attn, nkb_inner,
                          (const __nv_bfloat16*)(w.wout_wide + (size_t)l * nkb_inner * D * 64), g, b.part_a,
                          b.part_stride, 5, status));
    }
    if (!g.outproj_wide)
      LEWM_TRY(launch_k(k_partial_gemm<D, Cfg<D>::NT_OUT>, dim3(g.n_tiles, 4, kKSplit), dim3(kThreads),
                        resid_layout(g.rows8, nkb_inner / kKSplit, Cfg<D>::NT_OUT * 128, Cfg<D>::KG,
                                     resid_extra<D>())
                            .bytes,
                        st, (const __nv_bfloat16*)b.attn, nkb_inner,
                        (const __nv_bfloat16*)(w.wout + (size_t)l * 4 * nkb_inner * Cfg<D>::NT_OUT * 64), g,
                        b.part_a, b.part_stride, 5, status));
    if (prof) prof->end(KC_OUT, 2.0 * rows * md.inner * D, st);
    if (g.ln_prebuilt) {  // FC1 operand: s = r + gate_msa * (out-proj + bias), LN2 -> modulate -> ffn.norm
      const ResidUpdate u{b.x, b.part_a, b.part_stride, 2, w.out_b + l * D, l * 6 * D + 2 * D, b.xs};
      if (prof) prof->begin(st);
      LEWM_TRY(launch_k(k_ln_operand<D>, op_grid, dim3(kThreads), 0, st, u, g, (const __nv_bfloat16*)b.mod, mcols,
                        l * 6 * D + 3 * D, w.ffn_ln_w + l * D, w.ffn_ln_b + l * D, b.a_op, 1));
      if (prof) prof->end(KC_LN_OP, 0.0, st);
    }
    if (g.ffn_fused) {  // FC1 + GELU + FC2 quarter partials in one kernel
      if constexpr (D == 192) {
        if (prof) prof->begin(st);
        LEWM_TRY(launch_k(k_ffn<D>, dim3(g.n_tiles, md.mlp / kFfnQ), dim3(kThreads), smem_ffn<D>(), st, w, md, g, b,
                          l, status));
        if (prof) prof->end(KC_FFN, 4.0 * rows * D * md.mlp, st);
        continue;
      }
      return cudaErrorInvalidValue;
    }
    if (prof) prof->begin(st);
    LEWM_TRY(launch_k(k_fc1<D, kFc1N>, dim3(g.n_tiles, md.mlp / kFc1N), dim3(kThreads), smem_fc1<D, kFc1N>(), st, w,
                      md, g, b, l,
                      status));
    if (prof) prof->end(KC_FC1, 2.0 * rows * D * md.mlp, st);
    // FC2 partial sums over fc2_parts K parts (bias, gate_mlp and residual applied by the
    // next QKV operand builder or, after the last layer, by k_final)
    if (prof) prof->begin(st);
    LEWM_TRY(launch_k(k_partial_gemm<D, Cfg<D>::NT_OUT>, dim3(g.n_tiles, 4, g.fc2_parts), dim3(kThreads),
                      resid_layout(g.rows8, nkb_mlp / g.fc2_parts, Cfg<D>::NT_OUT * 128, Cfg<D>::KG, resid_extra<D>())
                          .bytes,
                      st, (const __nv_bfloat16*)b.h, nkb_mlp,
                      (const __nv_bfloat16*)(w.w2 + (size_t)l * 4 * nkb_mlp * Cfg<D>::NT_OUT * 64), g, b.part_b,
                      b.part_stride, 3, status));
    if (prof) prof->end(KC_FC2, 2.0 * rows * md.mlp * D, st);
  }
  if (prof) prof->begin(st);
  const int final_mode = b.pp_in ? 1 : 0;
  const int final_items = g.n_cand * ((g.last || final_mode == 1) ? 1 : g.next_rpc);
  LEWM_TRY(launch_k(k_final<D>, dim3((final_items + 3) / 4), dim3(128), 0, st, w, md, g, b, final_mode));
  if (prof) prof->end(KC_FINAL, 0.0, st);
#undef LEWM_TRY
  return cudaSuccess;
}

}  // namespace

cudaError_t launch_embed(const ModelDims& md, const DevWeights& w, const float* cand, int rows, __nv_bfloat16* eh,
                         __nv_bfloat16* act_a, uint32_t* status, cudaStream_t st, Prof* prof) {
  if (md.D == 192) return embed_impl<192>(md, w, cand, rows, eh, act_a, status, st, prof);
  if (md.D == 384) return embed_impl<384>(md, w, cand, rows, eh, act_a, status, st, prof);
  return cudaErrorInvalidValue;
}

cudaError_t launch_adaln(const ModelDims& md, const DevWeights& w, int rows, const __nv_bfloat16* act_a,
                         __nv_bfloat16* mod, uint32_t* status, cudaStream_t st, Prof* prof) {
  if (md.D == 192) return adaln_impl<192>(md, w, rows, act_a, mod, status, st, prof);
  if (md.D == 384) return adaln_impl<384>(md, w, rows, act_a, mod, status, st, prof);
  return cudaErrorInvalidValue;
}

cudaError_t launch_prep0(const ModelDims& md, const DevWeights& w, const CallGeom& g, const RolloutBufs& b,
                         cudaStream_t st, Prof* prof) {
  if (md.D == 192) return prep0_impl<192>(md, w, g, b, st, prof);
  if (md.D == 384) return prep0_impl<384>(md, w, g, b, st, prof);
  return cudaErrorInvalidValue;
}

cudaError_t launch_final_post(const ModelDims& md, const DevWeights& w, const CallGeom& g, const RolloutBufs& b,
                              cudaStream_t st, Prof* prof) {
  if (md.D != 192 || !b.pp_out) return cudaErrorInvalidValue;  // the head is built for width 192
  const int items = g.n_cand * (g.last ? 1 : g.next_rpc);
  if (prof) prof->begin(st);
  const cudaError_t e = launch_k(k_final<192>, dim3((items + 3) / 4), dim3(128), 0, st, w, md, g, b, 2);
  if (prof) prof->end(KC_FINAL, 0.0, st);
  return e;
}

cudaError_t launch_call(const ModelDims& md, const DevWeights& w, const CallGeom& g, const RolloutBufs& b,
                        uint32_t* status, cudaStream_t st, Prof* prof) {
  if (md.D == 192) return call_impl<192>(md, w, g, b, status, st, prof);
  if (md.D == 384) return call_impl<384>(md, w, g, b, status, st, prof);
  return cudaErrorInvalidValue;
}

}  // namespace lewm
