// ViT observation encoder + projector on sm_100a: the observation / goal embedding
// step in front of LeWM planning (reference lewm/jepa.py:88-104, JEPA.encode).
//
// The reference encoder is a transformers ViTModel built by stable-pretraining 0.1.7
// `vit_hf` (reference tools/benchmarks/stage_lewm_weights.py:72-78): patch embedding
// (Conv2d, stride = kernel = patch), CLS token, learned position embedding, pre-norm
// encoder layers (LayerNorm eps 1e-12, QKV with bias, softmax attention over all
// tokens, output dense, GELU MLP), final LayerNorm. JEPA.encode keeps the CLS row of
// last_hidden_state and applies the projector MLP (reference lewm/module.py:217-240:
// Linear, LayerNorm / BatchNorm1d / none, GELU, Linear).
//
// Rows are (image, token) pairs, 128 to a tile. Every GEMM runs on tcgen05 from
// K-major SW128 operand blocks and fuses its elementwise tail:
//   k_vit_patch_op   pixels -> patch operand (CLS rows and K padding are zeros)
//   k_vit_gemm       C = A . W^T over a ring of K blocks with one of five epilogues:
//                    PATCH   + bias, CLS / position embedding -> fp32 residual rows
//                    QKV     + bias, scattered to per-head Q rows, K rows and V^T blocks
//                    RESID   + bias, added into the fp32 residual rows
//                    GELU_OP GELU(acc * scale + shift) -> bf16 operand of the next GEMM
//                    F32     + bias -> fp32 rows
//   k_vit_ln_op      LayerNorm (+ optional GELU) of fp32 rows -> bf16 operand blocks
//   k_vit_attn       one CTA per (query tile, head, image): S = Q K^T into TMEM, softmax in
//                    registers, P V on the tensor core, written as the out-proj operand
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "lewm_b200.h"
#include "lewm_common.cuh"
#include "lewm_internal.h"

namespace lewm {
namespace vit {

constexpr int kD = 192;                // hidden width the kernels are built for (ViT-tiny)
constexpr int kHB = kD / 64;           // heads (dim_head 64) = K blocks of one hidden row
constexpr int kMaxTok = 272;           // tokens one attention CTA holds (S in 272 TMEM columns)
constexpr int kBlk = 128 * 64;         // elements of a [128 x 64] operand block
constexpr int kBlkBytes = kBlk * 2;
constexpr int kMaxStages = 4;
constexpr int kGemmThreads = 256;      // two warpgroups: each reads half of the accumulator columns

enum Epi { EPI_PATCH = 0, EPI_QKV = 1, EPI_RESID = 2, EPI_GELU_OP = 3, EPI_F32 = 4 };

struct EpiArgs {
  float* x;             // PATCH / RESID: fp32 residual rows [rows][kD]; F32: output rows [rows][n_total]
  const float* bias;    // per output column over all N chunks
  const float* scale;   // GELU_OP: per-column multiplier (null = 1)
  const float* pos;     // PATCH: position embedding [tokens][kD]
  const float* cls;     // PATCH: CLS token [kD]
  __nv_bfloat16* op;    // GELU_OP: operand blocks [tiles][n_total / 64][128 x 64]
  __nv_bfloat16* q;     // QKV: [image][head][q_rows x 64] swizzled rows
  __nv_bfloat16* k;     // QKV: [image][head][kv_rows x 64]
  __nv_bfloat16* vt;    // QKV: [image][head][kv_rows / 64][64 x 64], row = d, column = key
  const float* ln_g;    // PATCH / RESID: LayerNorm of the updated rows for the next GEMM
  const float* ln_b;    //   (affine), written as bf16 operand blocks to ln_out (null = none)
  __nv_bfloat16* ln_out;
  float ln_eps;
  int rows;             // valid rows
  int tokens;           // tokens per image
  int n_total;          // output columns over all chunks (GELU_OP, F32)
  int q_rows, kv_rows;
};

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

__device__ __forceinline__ uint4 pack8(const float* v) {
  return make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]), pack_bf16x2(v[4], v[5]),
                    pack_bf16x2(v[6], v[7]));
}

template <int NC>
constexpr int gemm_stage_bytes() { return kBlkBytes + NC * 128; }
constexpr bool staged_epi(int epi) { return epi == EPI_PATCH || epi == EPI_RESID || epi == EPI_F32; }

// Operand slots; the row-wise (staged) epilogues reuse them after the MMAs retire as the
// fp32 staging tile [128][NC + 4]. The mbarriers sit after the larger of the two.
template <int NC, int EPI>
__host__ __device__ constexpr int gemm_area(int stages) {
  return !staged_epi(EPI) || stages * gemm_stage_bytes<NC>() > 128 * (NC + 4) * 4 ? stages * gemm_stage_bytes<NC>()
                                                                                  : 128 * (NC + 4) * 4;
}
template <int NC, int EPI>
size_t gemm_smem(int stages) { return 1024 + (size_t)gemm_area<NC, EPI>(stages) + 128; }

// Row-wise epilogues from the staging tile, consecutive threads on consecutive float4s of
// a row (coalesced, and no thread re-reads a sector it has just written): PATCH writes
// acc + bias + position (CLS + position on token 0) into the residual rows, RESID adds
// acc + bias into them, F32 writes acc + bias. With ln_out set (PATCH / RESID, whose
// tile holds whole rows) the new residual rows go back into the staging tile and are
// layer-normalized into the next GEMM's operand, the same arithmetic as k_vit_ln_op<kD>.
template <int NC, int EPI>
__device__ __forceinline__ void staged_epilogue(const EpiArgs& ea, int tile, int chunk, float* __restrict__ stage) {
  constexpr int NV = NC / 4, SROW = NC + 4;
  const float* __restrict__ bias = ea.bias;
  float* __restrict__ x = ea.x;
  if constexpr (EPI == EPI_RESID) {
    // All of this thread's residual float4s are loaded before any is written back, so
    // the loads overlap instead of forming a chain of memory round trips.
    constexpr int PER = 128 * NV / kGemmThreads;
    static_assert(128 * NV % kGemmThreads == 0, "residual float4s per thread");
    float4 xa[PER];
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int idx = threadIdx.x + i * kGemmThreads, row = idx / NV, q = idx % NV;
      const int grow = tile * 128 + row;
      xa[i] = grow < ea.rows ? *reinterpret_cast<const float4*>(x + (size_t)grow * kD + chunk * NC + q * 4)
                             : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int idx = threadIdx.x + i * kGemmThreads, row = idx / NV, q = idx % NV;
      const int grow = tile * 128 + row;
      if (grow >= ea.rows) continue;
      const float4 a = *reinterpret_cast<const float4*>(stage + row * SROW + q * 4);
      const int col = chunk * NC + q * 4;
      const float4 b = *reinterpret_cast<const float4*>(bias + col);
      float4 o = xa[i];
      o.x += a.x + b.x;
      o.y += a.y + b.y;
      o.z += a.z + b.z;
      o.w += a.w + b.w;
      *reinterpret_cast<float4*>(x + (size_t)grow * kD + col) = o;
      if (ea.ln_out) *reinterpret_cast<float4*>(stage + row * SROW + q * 4) = o;
    }
  } else
#pragma unroll 4
  for (int idx = threadIdx.x; idx < 128 * NV; idx += kGemmThreads) {
    const int row = idx / NV, q = idx % NV;
    const int grow = tile * 128 + row;
    if (grow >= ea.rows) continue;
    const float4 a = *reinterpret_cast<const float4*>(stage + row * SROW + q * 4);
    const int col = chunk * NC + q * 4;
    if constexpr (EPI == EPI_PATCH) {
      const int tok = grow % ea.tokens;
      const float4 p = *reinterpret_cast<const float4*>(ea.pos + (size_t)tok * kD + q * 4);
      float4 o;
      if (tok == 0) {
        const float4 c = *reinterpret_cast<const float4*>(ea.cls + q * 4);
        o = make_float4(c.x + p.x, c.y + p.y, c.z + p.z, c.w + p.w);
      } else {
        const float4 b = *reinterpret_cast<const float4*>(bias + q * 4);
        o = make_float4(a.x + b.x + p.x, a.y + b.y + p.y, a.z + b.z + p.z, a.w + b.w + p.w);
      }
      *reinterpret_cast<float4*>(x + (size_t)grow * kD + q * 4) = o;
      if (ea.ln_out) *reinterpret_cast<float4*>(stage + row * SROW + q * 4) = o;
    } else {
      const float4 b = *reinterpret_cast<const float4*>(bias + col);
      *reinterpret_cast<float4*>(x + (size_t)grow * ea.n_total + col) =
          make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w);
    }
  }
  if constexpr (EPI == EPI_PATCH || EPI == EPI_RESID) {
    static_assert(NC == kD, "row LayerNorm needs whole rows");
    if (!ea.ln_out) return;
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    constexpr int WARPS = kGemmThreads / 32, U = 4;  // rows in flight per warp
    for (int r0 = warp; r0 < 128; r0 += WARPS * U) {
      float v[U][8], mean[U], rstd[U], s[U], ss[U];
      bool live[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int row = r0 + u * WARPS;
        live[u] = row < 128 && tile * 128 + row < ea.rows;  // rows past the last stay zero
        s[u] = 0.f;
        if (live[u] && lane < kD / 8) {
          const float4 lo = *reinterpret_cast<const float4*>(stage + row * SROW + lane * 8);
          const float4 hi = *reinterpret_cast<const float4*>(stage + row * SROW + lane * 8 + 4);
          v[u][0] = lo.x; v[u][1] = lo.y; v[u][2] = lo.z; v[u][3] = lo.w;
          v[u][4] = hi.x; v[u][5] = hi.y; v[u][6] = hi.z; v[u][7] = hi.w;
#pragma unroll
          for (int e = 0; e < 8; ++e) s[u] += v[u][e];
        } else {
#pragma unroll
          for (int e = 0; e < 8; ++e) v[u][e] = 0.f;
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) mean[u] = warp_sum(s[u]) * (1.0f / kD);
#pragma unroll
      for (int u = 0; u < U; ++u) {
        ss[u] = 0.f;
        if (lane < kD / 8) {
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const float d = v[u][e] - mean[u];
            ss[u] += d * d;
          }
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) rstd[u] = rsqrtf(warp_sum(ss[u]) * (1.0f / kD) + ea.ln_eps);
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int row = r0 + u * WARPS;
        if (!live[u] || lane >= kD / 8) continue;
        float y[8];
#pragma unroll
        for (int e = 0; e < 8; ++e)
          y[e] = fmaf((v[u][e] - mean[u]) * rstd[u], ea.ln_g[lane * 8 + e], ea.ln_b[lane * 8 + e]);
        uint8_t* blk = reinterpret_cast<uint8_t*>(ea.ln_out) + ((size_t)tile * kHB + lane / 8) * kBlkBytes;
        *reinterpret_cast<uint4*>(blk + sw128_off(row, (lane % 8) * 8)) = pack8(y);
      }
    }
  }
}

// Per-thread epilogue of 16 accumulator columns [c0, c0 + 16) of tile row r, for the
// epilogues that write bf16 operands (GELU_OP, QKV); the fp32 row-wise ones are staged.
template <int NC, int EPI>
__device__ __forceinline__ void gemm_epilogue(const EpiArgs& ea, int tile, int chunk, int r, int c0, float* v) {
  static_assert(EPI == EPI_GELU_OP || EPI == EPI_QKV, "fp32 row epilogues go through staged_epilogue");
  const int grow = tile * 128 + r;
  if (grow >= ea.rows) return;
  const int col = chunk * NC + c0;  // first output column over all chunks
  if constexpr (EPI == EPI_GELU_OP) {
    float bb[16], sc[16];
#pragma unroll
    for (int i = 0; i < 16; i += 4) {
      const float4 b4 = *reinterpret_cast<const float4*>(ea.bias + col + i);
      const float4 s4 = ea.scale ? *reinterpret_cast<const float4*>(ea.scale + col + i) : make_float4(1.f, 1.f, 1.f, 1.f);
      bb[i] = b4.x; bb[i + 1] = b4.y; bb[i + 2] = b4.z; bb[i + 3] = b4.w;
      sc[i] = s4.x; sc[i + 1] = s4.y; sc[i + 2] = s4.z; sc[i + 3] = s4.w;
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = gelu_f(fmaf(v[i], sc[i], bb[i]));
    uint8_t* blk = reinterpret_cast<uint8_t*>(ea.op) + ((size_t)tile * (ea.n_total / 64) + col / 64) * kBlkBytes;
    *reinterpret_cast<uint4*>(blk + sw128_off(r, col % 64)) = pack8(v);
    *reinterpret_cast<uint4*>(blk + sw128_off(r, col % 64 + 8)) = pack8(v + 8);
  } else {  // EPI_QKV: chunk 0 = Q, 1 = K, 2 = V; NC == kD
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] += ea.bias[col + i];
    const int img = grow / ea.tokens, tok = grow % ea.tokens;
    const int head = c0 / 64, d0 = c0 % 64;
    const size_t hi = (size_t)img * kHB + head;
    if (chunk < 2) {
      const int nrow = chunk == 0 ? ea.q_rows : ea.kv_rows;
      uint8_t* base = reinterpret_cast<uint8_t*>(chunk == 0 ? ea.q : ea.k) + hi * nrow * 128;
      *reinterpret_cast<uint4*>(base + sw128_off(tok, d0)) = pack8(v);
      *reinterpret_cast<uint4*>(base + sw128_off(tok, d0 + 8)) = pack8(v + 8);
    } else {
      uint8_t* base = reinterpret_cast<uint8_t*>(ea.vt) + (hi * (ea.kv_rows / 64) + tok / 64) * 8192;
#pragma unroll
      for (int i = 0; i < 16; ++i)
        *reinterpret_cast<__nv_bfloat16*>(base + sw128_off(d0 + i, tok % 64)) = __float2bfloat16_rn(v[i]);
    }
  }
}

// C[tile, chunk] = A[tile] . W[chunk]^T, K = 64 * kb_n, streamed through `stages`
// shared-memory slots (A block + W block each). Thread 0 issues the copies and the
// MMAs; all eight warps run the epilogue: warp w reads the TMEM lanes of rows
// 32 (w % 4) .. + 31 and the accumulator columns of half w / 4.
template <int NC, int EPI>
__global__ void __launch_bounds__(kGemmThreads) k_vit_gemm(const __nv_bfloat16* __restrict__ A, int kb_n,
                                                  const __nv_bfloat16* __restrict__ W, int stages, EpiArgs ea,
                                                  uint32_t* status) {
  constexpr int STG = gemm_stage_bytes<NC>();
  constexpr int TCOLS = NC <= 128 ? 128 : 256;
  static_assert(NC % 64 == 0 && NC <= 256, "N chunk");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + gemm_area<NC, EPI>(stages));
  uint64_t* freed = full + kMaxStages;
  uint64_t* done = freed + kMaxStages;
  uint32_t* slot = reinterpret_cast<uint32_t*>(done + 1);  // [0] TMEM base, [1] wait flag
  const int tid = threadIdx.x, warp = tid >> 5;
  const int tile = blockIdx.x, chunk = blockIdx.y;
  const __nv_bfloat16* a_src = A + (size_t)tile * kb_n * kBlk;
  const __nv_bfloat16* w_src = W + (size_t)chunk * kb_n * NC * 64;
  if (tid == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&freed[s], 1);
    }
    mbar_init(done, 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(slot, TCOLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = slot[0];
  if (tid == 0) {
    int loaded = 0, used = 0;
    auto load = [&](int kb) {
      const int s = kb % stages;
      mbar_arrive_expect_tx(&full[s], STG);
      bulk_g2s(smem + s * STG, a_src + (size_t)kb * kBlk, kBlkBytes, &full[s]);
      bulk_g2s(smem + s * STG + kBlkBytes, w_src + (size_t)kb * NC * 64, NC * 128, &full[s]);
    };
    for (; loaded < stages && loaded < kb_n; ++loaded) load(loaded);
    const uint32_t idesc = idesc_bf16(128, NC);
    for (int kb = 0; kb < kb_n; ++kb) {
      const int s = kb % stages;
      const uint32_t ph = (uint32_t)(kb / stages) & 1u;
      if (!mbar_wait(&full[s], ph, status)) break;
      used = kb + 1;
      tc_fence_after();
      umma_tile(tmem, smem_u32(smem + s * STG), kBlkBytes, smem_u32(smem + s * STG + kBlkBytes), NC * 128, 0, 1,
                idesc, kb > 0);
      umma_commit(&freed[s]);
      if (loaded < kb_n) {  // loaded == kb + stages: refill this slot once its MMAs retired
        if (!mbar_wait(&freed[s], ph, status)) break;
        load(loaded++);
      }
    }
    umma_commit(done);
    // After an expired wait, let the copies still in flight land before the CTA exits.
    for (int kb = used; kb < loaded; ++kb) mbar_wait(&full[kb % stages], (uint32_t)(kb / stages) & 1u, status);
  }
  const bool ok = cta_wait_mma(done, status, slot + 1);
  tc_fence_after();
  const uint32_t trow = tmem + ((uint32_t)((warp & 3) * 32) << 16);
  const int row = tid & 127, cbeg = (tid >> 7) * (NC / 2), cend = cbeg + NC / 2;
  if constexpr (staged_epi(EPI)) {
    float* stage = reinterpret_cast<float*>(smem);  // operand slots are dead once the MMAs retired
    if (ok) {
#pragma unroll 1
      for (int c0 = cbeg; c0 < cend; c0 += 16) {
        float v[16];
        tmem_ld16(trow + c0, v);
        float* dst = stage + row * (NC + 4) + c0;
#pragma unroll
        for (int i = 0; i < 16; i += 4) *reinterpret_cast<float4*>(dst + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
      }
    }
    __syncthreads();
    if (ok) staged_epilogue<NC, EPI>(ea, tile, chunk, stage);
  } else if (ok) {
#pragma unroll 1
    for (int c0 = cbeg; c0 < cend; c0 += 16) {
      float v[16];
      tmem_ld16(trow + c0, v);
      gemm_epilogue<NC, EPI>(ea, tile, chunk, row, c0, v);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, TCOLS);
}

// LayerNorm over C columns of fp32 rows (row r reads src + r * src_stride * C), optional
// affine and GELU, written as bf16 operand blocks [out_rows / 128][C / 64][128 x 64].
// Rows at or past n_valid are written as zeros. One warp per row.
template <int C>
__global__ void __launch_bounds__(256) k_vit_ln_op(const float* __restrict__ src, int src_stride, int n_valid,
                                                   int out_rows, float eps, const float* __restrict__ gamma,
                                                   const float* __restrict__ beta, int gelu,
                                                   __nv_bfloat16* __restrict__ out) {
  constexpr int NCH = C / 8;             // 16-byte output chunks per row
  constexpr int PER = (NCH + 31) / 32;   // chunks per lane
  constexpr int KB = C / 64;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = blockIdx.x * 8 + warp;
  if (r >= out_rows) return;
  uint8_t* ob = reinterpret_cast<uint8_t*>(out) + (size_t)(r / 128) * KB * kBlkBytes;
  const int rr = r % 128;
  if (r >= n_valid) {
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      const int q = lane + 32 * j;
      if (q < NCH) *reinterpret_cast<uint4*>(ob + (q / 8) * kBlkBytes + sw128_off(rr, (q % 8) * 8)) = make_uint4(0, 0, 0, 0);
    }
    return;
  }
  const float* row = src + (size_t)r * src_stride * C;
  float v[PER][8];
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    const int q = lane + 32 * j;
    if (q < NCH) {
      const float4 a = *reinterpret_cast<const float4*>(row + q * 8);
      const float4 b = *reinterpret_cast<const float4*>(row + q * 8 + 4);
      v[j][0] = a.x; v[j][1] = a.y; v[j][2] = a.z; v[j][3] = a.w;
      v[j][4] = b.x; v[j][5] = b.y; v[j][6] = b.z; v[j][7] = b.w;
#pragma unroll
      for (int e = 0; e < 8; ++e) s += v[j][e];
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) v[j][e] = 0.f;
    }
  }
  const float mean = warp_sum(s) * (1.0f / C);
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    if (lane + 32 * j < NCH) {
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float d = v[j][e] - mean;
        ss += d * d;
      }
    }
  }
  const float rstd = rsqrtf(warp_sum(ss) * (1.0f / C) + eps);
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    const int q = lane + 32 * j;
    if (q >= NCH) continue;
    float y[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int k = q * 8 + e;
      float t = (v[j][e] - mean) * rstd;
      if (gamma) t = fmaf(t, gamma[k], beta[k]);
      y[e] = gelu ? gelu_f(t) : t;
    }
    *reinterpret_cast<uint4*>(ob + (q / 8) * kBlkBytes + sw128_off(rr, (q % 8) * 8)) = pack8(y);
  }
}

// LayerNorm (+ optional GELU) over a runtime width C (a multiple of 64) of fp32 rows
// [n][C], written as bf16 operand blocks [out_rows / 128][C / 64][128 x 64]: the
// projector hidden, a few rows per batch. Three passes over the row (mean, variance,
// output); rows at or past n_valid are written as zeros. One warp per row.
__global__ void __launch_bounds__(256) k_vit_ln_wide(const float* __restrict__ src, int C, int n_valid,
                                                     int out_rows, float eps, const float* __restrict__ gamma,
                                                     const float* __restrict__ beta, int gelu,
                                                     __nv_bfloat16* __restrict__ out) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = blockIdx.x * 8 + warp;
  if (r >= out_rows) return;
  const int nch = C / 8, kb_n = C / 64;
  uint8_t* ob = reinterpret_cast<uint8_t*>(out) + (size_t)(r / 128) * kb_n * kBlkBytes;
  const int rr = r % 128;
  if (r >= n_valid) {
    for (int q = lane; q < nch; q += 32)
      *reinterpret_cast<uint4*>(ob + (q / 8) * kBlkBytes + sw128_off(rr, (q % 8) * 8)) = make_uint4(0, 0, 0, 0);
    return;
  }
  const float* row = src + (size_t)r * C;
  float s = 0.f;
  for (int q = lane; q < nch; q += 32)
    for (int e = 0; e < 8; ++e) s += row[q * 8 + e];
  const float mean = warp_sum(s) / (float)C;
  float ss = 0.f;
  for (int q = lane; q < nch; q += 32)
    for (int e = 0; e < 8; ++e) {
      const float d = row[q * 8 + e] - mean;
      ss += d * d;
    }
  const float rstd = rsqrtf(warp_sum(ss) / (float)C + eps);
  for (int q = lane; q < nch; q += 32) {
    float y[8];
    for (int e = 0; e < 8; ++e) {
      const int k = q * 8 + e;
      float t = (row[k] - mean) * rstd;
      if (gamma) t = fmaf(t, gamma[k], beta[k]);
      y[e] = gelu ? gelu_f(t) : t;
    }
    *reinterpret_cast<uint4*>(ob + (q / 8) * kBlkBytes + sw128_off(rr, (q % 8) * 8)) = pack8(y);
  }
}

// Patch operand: row (image, token) holds the token's C x p x p pixels in Conv2d weight
// order (channel, ky, kx), zero-padded to kbp * 64; CLS rows and rows past the last image
// are zeros. One thread per 16-byte chunk.
__global__ void __launch_bounds__(256) k_vit_patch_op(const float* __restrict__ pix, int n_img, int img, int p,
                                                      int ch, int tokens, int kbp, int total_rows,
                                                      __nv_bfloat16* __restrict__ out) {
  const int nchunk = kbp * 8;
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long long)total_rows * nchunk) return;
  const int r = (int)(idx / nchunk), q = (int)(idx % nchunk);
  const int gw = img / p, pp2 = p * p, K = ch * pp2;
  const int im = r / tokens, tok = r % tokens;
  const bool valid = im < n_img && tok > 0;
  const int py = valid ? (tok - 1) / gw : 0, px = valid ? (tok - 1) % gw : 0;
  float v[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const int k = q * 8 + e;
    float x = 0.f;
    if (valid && k < K) {
      const int c = k / pp2, rem = k % pp2, ky = rem / p, kx = rem % p;
      x = pix[(((size_t)im * ch + c) * img + (size_t)(py * p + ky)) * img + px * p + kx];
    }
    v[e] = x;
  }
  uint8_t* blk = reinterpret_cast<uint8_t*>(out) + ((size_t)(r / 128) * kbp + q / 8) * kBlkBytes;
  *reinterpret_cast<uint4*>(blk + sw128_off(r % 128, (q % 8) * 8)) = pack8(v);
}

// Per-channel normalization of uint8 frames (at most 4 channels).
struct FrameNorm {
  float mean[4];
  float stdv[4];
};

// Patch operand straight from uint8 frames [n][img][img][ch] (height, width, channel):
// each sample becomes (u * float32(1/255) - mean[c]) / std[c], rounded after every
// step (no contraction), the arithmetic of the policy's image transform ToDtype(float32,
// scale=True) + Normalize (reference lewm/eval.py:17-26, torchvision v2), so this equals
// k_vit_patch_op on the transformed float pixels bit for bit. Same row / chunk layout.
__global__ void __launch_bounds__(256) k_vit_patch_op_u8(const uint8_t* __restrict__ frames, FrameNorm nm,
                                                         int n_img, int img, int p, int ch, int tokens, int kbp,
                                                         int total_rows, __nv_bfloat16* __restrict__ out) {
  const int nchunk = kbp * 8;
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long long)total_rows * nchunk) return;
  const int r = (int)(idx / nchunk), q = (int)(idx % nchunk);
  const int gw = img / p, pp2 = p * p, K = ch * pp2;
  const int im = r / tokens, tok = r % tokens;
  const bool valid = im < n_img && tok > 0;
  const int py = valid ? (tok - 1) / gw : 0, px = valid ? (tok - 1) % gw : 0;
  const float inv255 = __int_as_float(0x3b808081);  // float32 nearest to 1/255
  float v[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const int k = q * 8 + e;
    float x = 0.f;
    if (valid && k < K) {
      const int c = k / pp2, rem = k % pp2, ky = rem / p, kx = rem % p;
      const float u = (float)frames[(((size_t)im * img + (size_t)(py * p + ky)) * img + px * p + kx) * ch + c];
      const float mu = c == 0 ? nm.mean[0] : c == 1 ? nm.mean[1] : c == 2 ? nm.mean[2] : nm.mean[3];
      const float sd = c == 0 ? nm.stdv[0] : c == 1 ? nm.stdv[1] : c == 2 ? nm.stdv[2] : nm.stdv[3];
      x = __fdiv_rn(__fsub_rn(__fmul_rn(u, inv255), mu), sd);
    }
    v[e] = x;
  }
  uint8_t* blk = reinterpret_cast<uint8_t*>(out) + ((size_t)(r / 128) * kbp + q / 8) * kBlkBytes;
  *reinterpret_cast<uint4*>(blk + sw128_off(r % 128, (q % 8) * 8)) = pack8(v);
}

struct AttnGeom {
  int tokens;    // keys = queries per image
  int ns;        // tokens rounded up to 16: S columns
  int q_tiles;   // 128-row query tiles
  int kv_rows;   // key rows held (kvb * 64)
  int kvb;       // 64-key blocks of P and V^T
};

constexpr int kAttnThreads = 256;  // two warpgroups split each row's key columns
constexpr int kAttnSplit = 144;    // first key column of the second warpgroup (multiple of 16)

inline size_t attn_smem(const AttnGeom& g) {
  return 1024 + (size_t)kBlkBytes + (size_t)g.kv_rows * 128 + (size_t)g.kvb * 8192 + (size_t)g.kvb * kBlkBytes +
         4 * 128 * 4 + 64;
}

// Softmax attention of one (query tile, head, image): the Q tile, K and V^T are loaded
// once; S = Q K^T (M 128, N <= 256 + a 16-column remainder) lands in TMEM. Warpgroup g
// (warps 4g .. 4g + 3, TMEM lanes by warp % 4) owns key columns [0, 144) or [144, end):
// each finds its part of the row maximum, the two parts are exchanged through shared
// memory, and each writes its keys' bf16 probabilities into P (masked past the last
// token) and a partial row sum. O = P V (N 64, K over the key blocks) lands in TMEM
// columns 384..447; each warpgroup scales 32 of its columns by 1 / (sum0 + sum1) and
// writes them into the out-projection operand block of the row. Warps without a valid
// query row (the tail tile holds one token) skip the softmax: their P rows only feed
// their own O rows, which are never written.
__global__ void __launch_bounds__(kAttnThreads) k_vit_attn(const __nv_bfloat16* __restrict__ q,
                                                           const __nv_bfloat16* __restrict__ k,
                                                           const __nv_bfloat16* __restrict__ vt, AttnGeom ag,
                                                           __nv_bfloat16* __restrict__ attn_op, uint32_t* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  const int head = blockIdx.x / ag.q_tiles, qt = blockIdx.x % ag.q_tiles, img = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, wg = warp >> 2, row = tid & 127;
  const uint32_t qb = (uint32_t)ag.q_tiles * kBlkBytes, kbytes = (uint32_t)ag.kv_rows * 128,
                 vb = (uint32_t)ag.kvb * 8192, pb = (uint32_t)ag.kvb * kBlkBytes;
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + kBlkBytes;
  uint8_t* sV = sK + kbytes;
  uint8_t* sP = sV + vb;
  float* red = reinterpret_cast<float*>(sP + pb);  // [0..1][128] partial max, [2..3][128] partial sum
  uint64_t* bar = reinterpret_cast<uint64_t*>(red + 4 * 128);  // [0] loads, [1] S, [2] O
  uint32_t* slot = reinterpret_cast<uint32_t*>(bar + 3);        // [0] TMEM base, [1] wait flag
  const size_t hi = (size_t)img * kHB + head;
  if (tid == 0) {
    for (int i = 0; i < 3; ++i) mbar_init(&bar[i], 1);
    fence_mbar_init();
    mbar_arrive_expect_tx(&bar[0], kBlkBytes + kbytes + vb);
    bulk_g2s(sQ, reinterpret_cast<const uint8_t*>(q) + hi * qb + (size_t)qt * kBlkBytes, kBlkBytes, &bar[0]);
    bulk_g2s(sK, reinterpret_cast<const uint8_t*>(k) + hi * kbytes, kbytes, &bar[0]);
    bulk_g2s(sV, reinterpret_cast<const uint8_t*>(vt) + hi * vb, vb, &bar[0]);
  }
  if (warp == 0) {
    tmem_alloc(slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = slot[0];
  const uint32_t trow = tmem + ((uint32_t)((warp & 3) * 32) << 16);
  bool ok = cta_wait_mma(&bar[0], status, slot + 1);
  const int n1 = ag.ns < 256 ? ag.ns : 256, n2 = ag.ns - n1;
  const float c = 0.125f * 1.44269504088896341f;  // dim_head^-1/2 * log2(e)
  if (ok) {
    if (tid == 0) {
      tc_fence_after();
      const uint32_t a = smem_u32(sQ);
      umma_tile(tmem, a, kBlkBytes, smem_u32(sK), 0, 0, 1, idesc_bf16(128, n1), false);
      if (n2 > 0) umma_tile(tmem + 256, a, kBlkBytes, smem_u32(sK + 256 * 128), 0, 0, 1, idesc_bf16(128, n2), false);
      umma_commit(&bar[1]);
    }
    ok = cta_wait_mma(&bar[1], status, slot + 1);
  }
  const int qi = qt * 128 + row;
  const bool valid = qi < ag.tokens;
  const bool warp_rows = qt * 128 + (warp & 3) * 32 < ag.tokens;  // warp-uniform
  // This warpgroup's S columns [s_beg, s_end) and P key columns [p_beg, p_end).
  const int s_beg = wg == 0 ? 0 : kAttnSplit, s_end = wg == 0 ? min(kAttnSplit, ag.ns) : ag.ns;
  const int p_beg = s_beg, p_end = wg == 0 ? min(kAttnSplit, ag.kvb * 64) : ag.kvb * 64;
  if (ok) {
    tc_fence_after();
    float m = -INFINITY;
    if (warp_rows) {
#pragma unroll 1
      for (int j0 = s_beg; j0 < s_end; j0 += 16) {
        float v[16];
        tmem_ld16(trow + j0, v);
#pragma unroll
        for (int i = 0; i < 16; ++i)
          if (j0 + i < ag.tokens) m = fmaxf(m, v[i]);
      }
    }
    red[wg * 128 + row] = m;
    __syncthreads();
    m = fmaxf(red[row], red[128 + row]);
    const float mc = m * c;
    float sum = 0.f;
    if (warp_rows) {
#pragma unroll 1
      for (int j0 = p_beg; j0 < p_end; j0 += 16) {
        float v[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = 0.f;
        if (j0 < s_end) tmem_ld16(trow + j0, v);
        float pr[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float e = (valid && j0 + i < ag.tokens) ? exp2f(fmaf(v[i], c, -mc)) : 0.f;
          pr[i] = __bfloat162float(__float2bfloat16_rn(e));  // the value the P V MMA sees
          sum += pr[i];
        }
        uint8_t* blk = sP + (j0 / 64) * kBlkBytes;
        *reinterpret_cast<uint4*>(blk + sw128_off(row, j0 % 64)) = pack8(pr);
        *reinterpret_cast<uint4*>(blk + sw128_off(row, j0 % 64 + 8)) = pack8(pr + 8);
      }
    }
    red[256 + wg * 128 + row] = sum;
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      umma_tile(tmem + 384, smem_u32(sP), kBlkBytes, smem_u32(sV), 8192, 0, ag.kvb, idesc_bf16(128, 64), false);
      umma_commit(&bar[2]);
    }
    ok = cta_wait_mma(&bar[2], status, slot + 1);
  }
  if (ok) {
    tc_fence_after();
    float o[32];
    tmem_ld_cols<32>(trow + 384 + wg * 32, o);
    if (valid) {
      const float inv = 1.0f / (red[256 + row] + red[384 + row]);
#pragma unroll
      for (int d = 0; d < 32; ++d) o[d] *= inv;
      const int grow = img * ag.tokens + qi;
      uint8_t* dst = reinterpret_cast<uint8_t*>(attn_op) + ((size_t)(grow / 128) * kHB + head) * kBlkBytes;
#pragma unroll
      for (int d0 = 0; d0 < 32; d0 += 8)
        *reinterpret_cast<uint4*>(dst + sw128_off(grow % 128, wg * 32 + d0)) = pack8(o + d0);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 512);
}

// ----------------------------------------------------------------- host side

uint16_t bf16_bits(float f) {  // round to nearest even; NaN stays NaN
  uint32_t u;
  std::memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return 0x7fc0;
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

// W [N x K] row-major -> [N / nc chunks][ceil(K / 64)][nc x 64] swizzled blocks, K zero-padded.
void pack_blocks(const float* w, int N, int K, int nc, std::vector<uint16_t>& out, size_t at) {
  const int kb_n = (K + 63) / 64;
  for (int n = 0; n < N; ++n)
    for (int kk = 0; kk < kb_n * 64; ++kk) {
      const float val = kk < K ? w[(size_t)n * K + kk] : 0.f;
      const int chunk = n / nc, nn = n % nc, kb = kk / 64;
      const size_t blk = at + ((size_t)chunk * kb_n + kb) * nc * 64;
      out[blk + sw128_off(nn, kk % 64) / 2] = bf16_bits(val);
    }
}

struct Geo {
  int tokens, kbp, fc1_nc, q_tiles, kv_rows, kvb, ns;
};

Geo geo_of(const lewm_encoder_desc& d) {
  Geo g{};
  const int gw = d.image_size / d.patch_size;
  g.tokens = gw * gw + 1;
  g.kbp = (d.channels * d.patch_size * d.patch_size + 63) / 64;
  g.fc1_nc = d.mlp_dim % 256 == 0 ? 256 : 192;
  g.ns = (g.tokens + 15) / 16 * 16;
  g.q_tiles = (g.tokens + 127) / 128;
  g.kvb = (g.ns + 63) / 64;
  g.kv_rows = g.kvb * 64;
  return g;
}

}  // namespace vit
}  // namespace lewm

using namespace lewm;
using namespace lewm::vit;

namespace {
std::string g_enc_create_error;
}

struct lewm_encoder {
  int device = 0;
  lewm_encoder_desc desc{};
  Geo geo{};
  std::string err;
  void* d_w = nullptr;       // bf16 blocks then fp32 vectors
  uint32_t* d_status = nullptr;
  // weight views
  const __nv_bfloat16 *w_patch = nullptr, *w_p1 = nullptr, *w_p2 = nullptr;
  std::vector<const __nv_bfloat16*> w_qkv, w_out, w_fc1, w_fc2;
  const float *b_patch = nullptr, *cls = nullptr, *pos = nullptr, *lnf_g = nullptr, *lnf_b = nullptr;
  const float *p1_scale = nullptr, *p1_shift = nullptr, *pn_g = nullptr, *pn_b = nullptr, *b_p2 = nullptr;
  std::vector<const float*> ln1_g, ln1_b, b_qkv, b_out, ln2_g, ln2_b, b_fc1, b_fc2;
  // workspace
  void* d_ws = nullptr;
  size_t ws_bytes = 0;
  int ws_images = 0;
  __nv_bfloat16 *patch_a = nullptr, *ln_a = nullptr, *attn_a = nullptr, *h_a = nullptr, *cls_a = nullptr,
                *ph_a = nullptr, *q = nullptr, *k = nullptr, *vt = nullptr;
  float *x = nullptr, *ph32 = nullptr;
};

namespace {

lewm_status efail(lewm_encoder* e, lewm_status s, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  if (e)
    e->err = buf;
  else
    g_enc_create_error = buf;
  return s;
}

#define ENC_CK(enc, call)                                                                                \
  do {                                                                                                   \
    cudaError_t e_ = (call);                                                                             \
    if (e_ != cudaSuccess)                                                                               \
      return efail(enc, e_ == cudaErrorMemoryAllocation ? LEWM_OUT_OF_MEMORY : LEWM_CUDA_ERROR, "%s: %s", \
                   #call, cudaGetErrorString(e_));                                                       \
  } while (0)

struct EncDeviceGuard {
  int prev = -1;
  explicit EncDeviceGuard(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    cudaSetDevice(dev);
  }
  ~EncDeviceGuard() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

lewm_status check_enc_desc(const lewm_encoder_desc* d) {
  if (!d) return efail(nullptr, LEWM_INVALID_ARG, "desc is NULL");
  if (d->image_size <= 0 || d->patch_size <= 0 || d->channels <= 0 || d->depth <= 0 || d->heads <= 0 ||
      d->mlp_dim <= 0 || d->proj_hidden < 0 || d->proj_out <= 0 || !(d->ln_eps > 0.f) || !(d->proj_eps > 0.f))
    return efail(nullptr, LEWM_INVALID_ARG, "encoder desc has a non-positive size or eps");
  if (d->proj_norm < 0 || d->proj_norm > 2) return efail(nullptr, LEWM_INVALID_ARG, "proj_norm must be 0, 1 or 2");
  if (d->hidden != kD || d->heads * 64 != d->hidden)
    return efail(nullptr, LEWM_UNSUPPORTED_SHAPE, "encoder kernels are built for hidden %d with dim_head 64", kD);
  if (d->image_size % d->patch_size != 0)
    return efail(nullptr, LEWM_UNSUPPORTED_SHAPE, "image_size must be a multiple of patch_size");
  const Geo g = geo_of(*d);
  if (g.tokens > kMaxTok)
    return efail(nullptr, LEWM_UNSUPPORTED_SHAPE, "%d tokens per image; at most %d", g.tokens, kMaxTok);
  if (g.kbp > 32) return efail(nullptr, LEWM_UNSUPPORTED_SHAPE, "channels x patch^2 above 2048");
  if (d->mlp_dim % 256 != 0 && d->mlp_dim % 192 != 0)
    return efail(nullptr, LEWM_UNSUPPORTED_SHAPE, "mlp_dim must be a multiple of 192 or 256");
  if (d->proj_hidden == 0 || d->proj_hidden % 256 != 0)
    return efail(nullptr, LEWM_UNSUPPORTED_SHAPE, "proj_hidden must be a positive multiple of 256");
  if (d->proj_out != kD) return efail(nullptr, LEWM_UNSUPPORTED_SHAPE, "proj_out must be %d", kD);
  return LEWM_OK;
}

size_t weight_count(const lewm_encoder_desc& d) {
  const Geo g = geo_of(d);
  const size_t D = d.hidden, M = d.mlp_dim, P = d.proj_hidden;
  size_t n = D + (size_t)g.tokens * D + D * d.channels * d.patch_size * d.patch_size + D;
  n += (size_t)d.depth * (2 * D + 3 * (D * D + D) + D * D + D + 2 * D + M * D + M + D * M + D);
  n += 2 * D;
  n += P * D + P + (d.proj_norm == 1 ? 2 * P : d.proj_norm == 2 ? 4 * P : 0) + (size_t)d.proj_out * P + d.proj_out;
  return n;
}

template <int NC, int EPI>
cudaError_t set_gemm_smem() {
  return cudaFuncSetAttribute(k_vit_gemm<NC, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              (int)gemm_smem<NC, EPI>(kMaxStages));
}

template <int NC, int EPI>
void launch_gemm(const __nv_bfloat16* A, int kb_n, const __nv_bfloat16* W, int tiles, int chunks, const EpiArgs& ea,
                 uint32_t* status, cudaStream_t st) {
  // Per-thread epilogues need no staging tile: two operand slots keep two CTAs (and
  // 2 x 256 TMEM columns) on an SM, so one CTA's epilogue overlaps the other's loads.
  const int cap = staged_epi(EPI) ? kMaxStages : 2;
  const int stages = kb_n < cap ? kb_n : cap;
  k_vit_gemm<NC, EPI><<<dim3(tiles, chunks), kGemmThreads, gemm_smem<NC, EPI>(stages), st>>>(A, kb_n, W, stages, ea,
                                                                                      status);
}

template <int C>
void launch_ln(const float* src, int src_stride, int n_valid, int out_rows, float eps, const float* g,
               const float* b, int gelu, __nv_bfloat16* out, cudaStream_t st) {
  k_vit_ln_op<C><<<(out_rows + 7) / 8, 256, 0, st>>>(src, src_stride, n_valid, out_rows, eps, g, b, gelu, out);
}

lewm_status ensure_enc_ws(lewm_encoder* e, int n_img, cudaStream_t st) {
  if (e->d_ws && n_img <= e->ws_images) return LEWM_OK;
  const lewm_encoder_desc& d = e->desc;
  const Geo& g = e->geo;
  const size_t rows = (size_t)n_img * g.tokens, mt = (rows + 127) / 128, mi = ((size_t)n_img + 127) / 128;
  size_t off = 0;
  auto carve = [&](size_t bytes) {
    const size_t at = off;
    off += (bytes + 1023) / 1024 * 1024;
    return at;
  };
  const size_t o_patch = carve(mt * g.kbp * kBlkBytes);
  const size_t o_x = carve(mt * 128 * kD * 4);
  const size_t o_ln = carve(mt * kHB * kBlkBytes);
  const size_t o_attn = carve(mt * kHB * kBlkBytes);
  const size_t o_h = carve(mt * (d.mlp_dim / 64) * kBlkBytes);
  const size_t o_q = carve((size_t)n_img * kHB * g.q_tiles * kBlkBytes);
  const size_t o_k = carve((size_t)n_img * kHB * g.kv_rows * 128);
  const size_t o_vt = carve((size_t)n_img * kHB * g.kvb * 8192);
  const size_t o_cls = carve(mi * kHB * kBlkBytes);
  const size_t o_ph = carve(mi * (d.proj_hidden / 64) * kBlkBytes);
  const size_t o_ph32 = carve(d.proj_norm == 1 ? mi * 128 * d.proj_hidden * 4 : 0);
  if (e->d_ws) {
    cudaFree(e->d_ws);
    e->d_ws = nullptr;
    e->ws_images = 0;
  }
  ENC_CK(e, cudaMalloc(&e->d_ws, off));
  // Padding rows and key slots are never written by the kernels and must read as zero.
  ENC_CK(e, cudaMemsetAsync(e->d_ws, 0, off, st));
  uint8_t* base = static_cast<uint8_t*>(e->d_ws);
  e->patch_a = reinterpret_cast<__nv_bfloat16*>(base + o_patch);
  e->x = reinterpret_cast<float*>(base + o_x);
  e->ln_a = reinterpret_cast<__nv_bfloat16*>(base + o_ln);
  e->attn_a = reinterpret_cast<__nv_bfloat16*>(base + o_attn);
  e->h_a = reinterpret_cast<__nv_bfloat16*>(base + o_h);
  e->q = reinterpret_cast<__nv_bfloat16*>(base + o_q);
  e->k = reinterpret_cast<__nv_bfloat16*>(base + o_k);
  e->vt = reinterpret_cast<__nv_bfloat16*>(base + o_vt);
  e->cls_a = reinterpret_cast<__nv_bfloat16*>(base + o_cls);
  e->ph_a = reinterpret_cast<__nv_bfloat16*>(base + o_ph);
  e->ph32 = reinterpret_cast<float*>(base + o_ph32);
  e->ws_bytes = off;
  e->ws_images = n_img;
  return LEWM_OK;
}

}  // namespace

extern "C" {

size_t lewm_encoder_weight_count(const lewm_encoder_desc* desc) {
  if (check_enc_desc(desc) != LEWM_OK) return 0;
  return weight_count(*desc);
}

lewm_status lewm_encoder_create(lewm_encoder** out, const lewm_encoder_desc* desc, const float* weights,
                                size_t n_floats, int device) {
  if (!out) return efail(nullptr, LEWM_INVALID_ARG, "out is NULL");
  *out = nullptr;
  lewm_status s = check_enc_desc(desc);
  if (s != LEWM_OK) return s;
  if (!weights) return efail(nullptr, LEWM_INVALID_ARG, "weights is NULL");
  const lewm_encoder_desc d = *desc;
  if (n_floats != weight_count(d))
    return efail(nullptr, LEWM_INVALID_ARG, "expected %zu weight floats, got %zu", weight_count(d), n_floats);
  const Geo g = geo_of(d);
  const int D = kD, M = d.mlp_dim, P = d.proj_hidden, L = d.depth;
  const int KP = d.channels * d.patch_size * d.patch_size;

  // Layout of the device weight buffer: bf16 blocks first, then fp32 vectors.
  std::vector<size_t> bf_at;
  size_t bf = 0;
  auto bf_take = [&](size_t elems) {
    bf_at.push_back(bf);
    bf += (elems + 511) / 512 * 512;  // 1 KB granules keep every block base 1024-byte aligned
    return bf_at.back();
  };
  const size_t a_patch = bf_take((size_t)D * g.kbp * 64);
  std::vector<size_t> a_qkv(L), a_out(L), a_fc1(L), a_fc2(L);
  for (int l = 0; l < L; ++l) {
    a_qkv[l] = bf_take((size_t)3 * D * D);
    a_out[l] = bf_take((size_t)D * D);
    a_fc1[l] = bf_take((size_t)M * D);
    a_fc2[l] = bf_take((size_t)D * M);
  }
  const size_t a_p1 = bf_take((size_t)P * D);
  const size_t a_p2 = bf_take((size_t)d.proj_out * P);
  std::vector<uint16_t> hb(bf, 0);
  std::vector<float> fv;
  auto f_take = [&](const float* src, size_t n) {
    const size_t at = fv.size();
    fv.insert(fv.end(), src, src + n);
    fv.resize((fv.size() + 3) / 4 * 4, 0.f);  // 16-byte alignment of every vector
    return at;
  };
  const float* w = weights;
  const size_t f_cls = f_take(w, D);
  w += D;
  const size_t f_pos = f_take(w, (size_t)g.tokens * D);
  w += (size_t)g.tokens * D;
  pack_blocks(w, D, KP, D, hb, a_patch);
  w += (size_t)D * KP;
  const size_t f_bpatch = f_take(w, D);
  w += D;
  std::vector<size_t> f_ln1g(L), f_ln1b(L), f_bqkv(L), f_bout(L), f_ln2g(L), f_ln2b(L), f_bfc1(L), f_bfc2(L);
  for (int l = 0; l < L; ++l) {
    f_ln1g[l] = f_take(w, D);
    w += D;
    f_ln1b[l] = f_take(w, D);
    w += D;
    std::vector<float> qkv_w((size_t)3 * D * D), qkv_b((size_t)3 * D);
    for (int t = 0; t < 3; ++t) {  // query, key, value: weight then bias
      std::memcpy(qkv_w.data() + (size_t)t * D * D, w, sizeof(float) * D * D);
      w += (size_t)D * D;
      std::memcpy(qkv_b.data() + (size_t)t * D, w, sizeof(float) * D);
      w += D;
    }
    pack_blocks(qkv_w.data(), 3 * D, D, D, hb, a_qkv[l]);
    f_bqkv[l] = f_take(qkv_b.data(), 3 * D);
    pack_blocks(w, D, D, D, hb, a_out[l]);
    w += (size_t)D * D;
    f_bout[l] = f_take(w, D);
    w += D;
    f_ln2g[l] = f_take(w, D);
    w += D;
    f_ln2b[l] = f_take(w, D);
    w += D;
    pack_blocks(w, M, D, g.fc1_nc, hb, a_fc1[l]);
    w += (size_t)M * D;
    f_bfc1[l] = f_take(w, M);
    w += M;
    pack_blocks(w, D, M, D, hb, a_fc2[l]);
    w += (size_t)D * M;
    f_bfc2[l] = f_take(w, D);
    w += D;
  }
  const size_t f_lnfg = f_take(w, D);
  w += D;
  const size_t f_lnfb = f_take(w, D);
  w += D;
  pack_blocks(w, P, D, 256, hb, a_p1);
  w += (size_t)P * D;
  const float* p1_bias = w;
  w += P;
  // Projector hidden: BatchNorm1d (eval) folds into a per-column scale and shift of the
  // first Linear's accumulator; LayerNorm runs as its own row pass after the bias.
  std::vector<float> scale(P, 1.f), shift(p1_bias, p1_bias + P);
  size_t f_png = 0, f_pnb = 0;
  if (d.proj_norm == 1) {
    f_png = f_take(w, P);
    w += P;
    f_pnb = f_take(w, P);
    w += P;
  } else if (d.proj_norm == 2) {
    const float *gam = w, *bet = w + P, *rm = w + 2 * P, *rv = w + 3 * P;
    for (int i = 0; i < P; ++i) {
      const double sc = (double)gam[i] / std::sqrt((double)rv[i] + (double)d.proj_eps);
      scale[i] = (float)sc;
      shift[i] = (float)(((double)p1_bias[i] - (double)rm[i]) * sc + (double)bet[i]);
    }
    w += 4 * P;
  }
  const size_t f_scale = f_take(scale.data(), P);
  const size_t f_shift = f_take(shift.data(), P);
  pack_blocks(w, d.proj_out, P, d.proj_out, hb, a_p2);
  w += (size_t)d.proj_out * P;
  const size_t f_bp2 = f_take(w, d.proj_out);
  w += d.proj_out;

  lewm_encoder* e = new lewm_encoder();
  e->device = device;
  e->desc = d;
  e->geo = g;
  {
    EncDeviceGuard guard(device);
    const size_t bf_bytes = bf * 2, total = bf_bytes + fv.size() * 4;
    cudaError_t ce = cudaMalloc(&e->d_w, total);
    if (ce == cudaSuccess) ce = cudaMemcpy(e->d_w, hb.data(), bf_bytes, cudaMemcpyHostToDevice);
    if (ce == cudaSuccess)
      ce = cudaMemcpy(static_cast<uint8_t*>(e->d_w) + bf_bytes, fv.data(), fv.size() * 4, cudaMemcpyHostToDevice);
    if (ce == cudaSuccess) ce = cudaMalloc(&e->d_status, kStatusBytes);  // status word + wait limit
    if (ce == cudaSuccess) ce = cudaMemset(e->d_status, 0, kStatusBytes);
    if (ce == cudaSuccess) ce = set_gemm_smem<192, EPI_PATCH>();
    if (ce == cudaSuccess) ce = set_gemm_smem<192, EPI_QKV>();
    if (ce == cudaSuccess) ce = set_gemm_smem<192, EPI_RESID>();
    if (ce == cudaSuccess) ce = set_gemm_smem<192, EPI_GELU_OP>();
    if (ce == cudaSuccess) ce = set_gemm_smem<256, EPI_GELU_OP>();
    if (ce == cudaSuccess) ce = set_gemm_smem<256, EPI_F32>();
    if (ce == cudaSuccess) ce = set_gemm_smem<192, EPI_F32>();
    if (ce == cudaSuccess) {
      // The attribute is per function: size it for the largest supported geometry so an
      // encoder created later with fewer tokens does not lower it under this one.
      const int ns_max = (kMaxTok + 15) / 16 * 16, kvb_max = (ns_max + 63) / 64;
      const AttnGeom big{kMaxTok, ns_max, (kMaxTok + 127) / 128, kvb_max * 64, kvb_max};
      ce = cudaFuncSetAttribute(k_vit_attn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)attn_smem(big));
    }
    if (ce != cudaSuccess) {
      efail(nullptr, ce == cudaErrorMemoryAllocation ? LEWM_OUT_OF_MEMORY : LEWM_CUDA_ERROR, "encoder create: %s",
            cudaGetErrorString(ce));
      if (e->d_w) cudaFree(e->d_w);
      if (e->d_status) cudaFree(e->d_status);
      delete e;
      return ce == cudaErrorMemoryAllocation ? LEWM_OUT_OF_MEMORY : LEWM_CUDA_ERROR;
    }
  }
  const __nv_bfloat16* wb = static_cast<const __nv_bfloat16*>(e->d_w);
  const float* wf = reinterpret_cast<const float*>(static_cast<const uint8_t*>(e->d_w) + bf * 2);
  e->w_patch = wb + a_patch;
  e->w_p1 = wb + a_p1;
  e->w_p2 = wb + a_p2;
  e->b_patch = wf + f_bpatch;
  e->cls = wf + f_cls;
  e->pos = wf + f_pos;
  e->lnf_g = wf + f_lnfg;
  e->lnf_b = wf + f_lnfb;
  e->p1_scale = wf + f_scale;
  e->p1_shift = wf + f_shift;
  e->pn_g = d.proj_norm == 1 ? wf + f_png : nullptr;
  e->pn_b = d.proj_norm == 1 ? wf + f_pnb : nullptr;
  e->b_p2 = wf + f_bp2;
  for (int l = 0; l < L; ++l) {
    e->w_qkv.push_back(wb + a_qkv[l]);
    e->w_out.push_back(wb + a_out[l]);
    e->w_fc1.push_back(wb + a_fc1[l]);
    e->w_fc2.push_back(wb + a_fc2[l]);
    e->ln1_g.push_back(wf + f_ln1g[l]);
    e->ln1_b.push_back(wf + f_ln1b[l]);
    e->b_qkv.push_back(wf + f_bqkv[l]);
    e->b_out.push_back(wf + f_bout[l]);
    e->ln2_g.push_back(wf + f_ln2g[l]);
    e->ln2_b.push_back(wf + f_ln2b[l]);
    e->b_fc1.push_back(wf + f_bfc1[l]);
    e->b_fc2.push_back(wf + f_bfc2[l]);
  }
  *out = e;
  return LEWM_OK;
}

}  // extern "C"

namespace {

// Float pixels (pixels != null) or uint8 frames with their per-channel normalization.
lewm_status encode_impl(lewm_encoder* e, const float* pixels, const uint8_t* frames, const FrameNorm& nm,
                        int32_t n_images, float* emb_out, void* stream) {
  if (!e) return efail(nullptr, LEWM_INVALID_ARG, "encoder is NULL");
  if (n_images < 0) return efail(e, LEWM_INVALID_ARG, "n_images < 0");
  if (n_images == 0) return LEWM_OK;
  if ((!pixels && !frames) || !emb_out) return efail(e, LEWM_INVALID_ARG, "pixels / emb_out is NULL");
  if (n_images > 65535)  // images are the attention grid's y dimension
    return efail(e, LEWM_UNSUPPORTED_SHAPE, "at most 65535 images per call, got %d", n_images);
  if ((reinterpret_cast<uintptr_t>(emb_out) & 15u) != 0)
    return efail(e, LEWM_INVALID_ARG, "emb_out must be 16-byte aligned");
  EncDeviceGuard guard(e->device);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  lewm_status s = ensure_enc_ws(e, n_images, st);
  if (s != LEWM_OK) return s;
  const lewm_encoder_desc& d = e->desc;
  const Geo& g = e->geo;
  const int rows = n_images * g.tokens, mt = (rows + 127) / 128, mi = (n_images + 127) / 128;
  const float eps = d.ln_eps;
  {
    const long long total = (long long)mt * 128 * g.kbp * 8;
    const unsigned blocks = (unsigned)((total + 255) / 256);
    if (pixels)
      k_vit_patch_op<<<blocks, 256, 0, st>>>(pixels, n_images, d.image_size, d.patch_size, d.channels, g.tokens,
                                             g.kbp, mt * 128, e->patch_a);
    else
      k_vit_patch_op_u8<<<blocks, 256, 0, st>>>(frames, nm, n_images, d.image_size, d.patch_size, d.channels,
                                                g.tokens, g.kbp, mt * 128, e->patch_a);
  }
  EpiArgs ea{};
  ea.rows = rows;
  ea.tokens = g.tokens;
  ea.q_rows = g.q_tiles * 128;
  ea.kv_rows = g.kv_rows;
  ea.x = e->x;
  ea.ln_eps = eps;
  EpiArgs pe = ea;
  pe.bias = e->b_patch;
  pe.pos = e->pos;
  pe.cls = e->cls;
  pe.ln_g = e->ln1_g[0];  // layer 0's first LayerNorm, fused
  pe.ln_b = e->ln1_b[0];
  pe.ln_out = e->ln_a;
  launch_gemm<192, EPI_PATCH>(e->patch_a, g.kbp, e->w_patch, mt, 1, pe, e->d_status, st);
  const AttnGeom ag{g.tokens, g.ns, g.q_tiles, g.kv_rows, g.kvb};
  const size_t asm_bytes = attn_smem(ag);
  for (int l = 0; l < d.depth; ++l) {
    // ln_a holds LN_before(x) of layer l, written by the previous residual epilogue.
    EpiArgs qa = ea;
    qa.bias = e->b_qkv[l];
    qa.q = e->q;
    qa.k = e->k;
    qa.vt = e->vt;
    launch_gemm<192, EPI_QKV>(e->ln_a, kHB, e->w_qkv[l], mt, 3, qa, e->d_status, st);
    k_vit_attn<<<dim3(g.q_tiles * kHB, n_images), kAttnThreads, asm_bytes, st>>>(e->q, e->k, e->vt, ag,
                                                                                 e->attn_a, e->d_status);
    EpiArgs ra = ea;
    ra.bias = e->b_out[l];
    ra.ln_g = e->ln2_g[l];  // LN_after of this layer, fused
    ra.ln_b = e->ln2_b[l];
    ra.ln_out = e->ln_a;
    launch_gemm<192, EPI_RESID>(e->attn_a, kHB, e->w_out[l], mt, 1, ra, e->d_status, st);
    EpiArgs ha = ea;
    ha.bias = e->b_fc1[l];
    ha.scale = nullptr;
    ha.op = e->h_a;
    ha.n_total = d.mlp_dim;
    if (g.fc1_nc == 256)
      launch_gemm<256, EPI_GELU_OP>(e->ln_a, kHB, e->w_fc1[l], mt, d.mlp_dim / 256, ha, e->d_status, st);
    else
      launch_gemm<192, EPI_GELU_OP>(e->ln_a, kHB, e->w_fc1[l], mt, d.mlp_dim / 192, ha, e->d_status, st);
    EpiArgs fa = ea;
    fa.bias = e->b_fc2[l];
    if (l + 1 < d.depth) {  // LN_before of the next layer, fused
      fa.ln_g = e->ln1_g[l + 1];
      fa.ln_b = e->ln1_b[l + 1];
      fa.ln_out = e->ln_a;
    }
    launch_gemm<192, EPI_RESID>(e->h_a, d.mlp_dim / 64, e->w_fc2[l], mt, 1, fa, e->d_status, st);
  }
  // Final LayerNorm of the CLS rows only (row image * tokens), then the projector.
  launch_ln<kD>(e->x, g.tokens, n_images, mi * 128, eps, e->lnf_g, e->lnf_b, 0, e->cls_a, st);
  EpiArgs pa{};
  pa.rows = n_images;
  pa.n_total = d.proj_hidden;
  if (d.proj_norm == 1) {
    pa.x = e->ph32;
    pa.bias = e->p1_shift;  // the Linear bias (scale is 1 without BatchNorm)
    launch_gemm<256, EPI_F32>(e->cls_a, kHB, e->w_p1, mi, d.proj_hidden / 256, pa, e->d_status, st);
    k_vit_ln_wide<<<mi * 16, 256, 0, st>>>(e->ph32, d.proj_hidden, n_images, mi * 128, d.proj_eps, e->pn_g, e->pn_b,
                                           1, e->ph_a);
  } else {
    pa.op = e->ph_a;
    pa.scale = e->p1_scale;
    pa.bias = e->p1_shift;
    launch_gemm<256, EPI_GELU_OP>(e->cls_a, kHB, e->w_p1, mi, d.proj_hidden / 256, pa, e->d_status, st);
  }
  EpiArgs oa{};
  oa.rows = n_images;
  oa.n_total = d.proj_out;
  oa.x = emb_out;
  oa.bias = e->b_p2;
  launch_gemm<192, EPI_F32>(e->ph_a, d.proj_hidden / 64, e->w_p2, mi, 1, oa, e->d_status, st);
  ENC_CK(e, cudaGetLastError());
  return LEWM_OK;
}

}  // namespace

extern "C" {

lewm_status lewm_encode(lewm_encoder* e, const float* pixels, int32_t n_images, float* emb_out, void* stream) {
  if (!pixels && n_images > 0) return efail(e, LEWM_INVALID_ARG, "pixels is NULL");
  return encode_impl(e, pixels, nullptr, FrameNorm{}, n_images, emb_out, stream);
}

lewm_status lewm_encode_u8(lewm_encoder* e, const uint8_t* frames, int32_t n_images, const float* mean,
                           const float* stdv, float* emb_out, void* stream) {
  if (!e) return efail(nullptr, LEWM_INVALID_ARG, "encoder is NULL");
  if (e->desc.channels > 4) return efail(e, LEWM_UNSUPPORTED_SHAPE, "uint8 frames support at most 4 channels");
  if (!mean || !stdv) return efail(e, LEWM_INVALID_ARG, "mean / std is NULL");
  if (!frames && n_images > 0) return efail(e, LEWM_INVALID_ARG, "frames is NULL");
  FrameNorm nm{};
  for (int c = 0; c < e->desc.channels; ++c) {
    if (!(stdv[c] != 0.f)) return efail(e, LEWM_INVALID_ARG, "std[%d] is zero", c);
    nm.mean[c] = mean[c];
    nm.stdv[c] = stdv[c];
  }
  return encode_impl(e, nullptr, frames, nm, n_images, emb_out, stream);
}

lewm_status lewm_encoder_sync_status(lewm_encoder* e, void* stream) {
  if (!e) return efail(nullptr, LEWM_INVALID_ARG, "encoder is NULL");
  EncDeviceGuard guard(e->device);
  ENC_CK(e, cudaStreamSynchronize(static_cast<cudaStream_t>(stream)));
  ENC_CK(e, cudaGetLastError());
  uint32_t v = 0;
  ENC_CK(e, cudaMemcpy(&v, e->d_status, 4, cudaMemcpyDeviceToHost));
  if (v) {
    ENC_CK(e, cudaMemset(e->d_status, 0, 4));
    return efail(e, LEWM_DEVICE_TIMEOUT, "device status 0x%x: a bounded device wait expired", v);
  }
  return LEWM_OK;
}

const char* lewm_encoder_last_error(const lewm_encoder* e) { return e ? e->err.c_str() : g_enc_create_error.c_str(); }

void lewm_encoder_destroy(lewm_encoder* e) {
  if (!e) return;
  {
    EncDeviceGuard guard(e->device);
    if (e->d_ws) cudaFree(e->d_ws);
    if (e->d_w) cudaFree(e->d_w);
    if (e->d_status) cudaFree(e->d_status);
  }
  delete e;
}

}  // extern "C"

// ---------------------------------------------------------------- MLP head (predictor pred_proj)
// The reference MLP (lewm/module.py:217-240) at input and output width 192: Linear(192 -> P),
// LayerNorm(P) / BatchNorm1d(P) in eval / no norm, GELU, Linear(P -> 192). The predictor's
// pred_proj head (JEPA.predict, lewm/jepa.py:106-114) runs on the projector kernels of the
// encoder: BatchNorm folds into a per-column scale / shift of the first GEMM's accumulator,
// LayerNorm runs as a row pass over the fp32 hidden (eps 1e-5, nn.LayerNorm's default).
namespace lewm {

size_t mlp_head_floats(int P, int norm) {
  return (size_t)P * kD + P + (norm == 1 ? 2 * (size_t)P : norm == 2 ? 4 * (size_t)P : 0) + (size_t)kD * P + kD;
}

cudaError_t mlp_head_create(MlpHead* h, const float* w, int P, int norm, float eps) {
  *h = MlpHead{};
  h->P = P;
  h->norm = norm;
  h->eps = eps;
  // bf16 blocks: W1 as 256-column chunks [P / 256][3][256 x 64], W2 [1][P / 64][192 x 64].
  const size_t n1 = (size_t)P * kD, n2 = (size_t)kD * P;
  std::vector<uint16_t> hb(n1 + n2);
  pack_blocks(w, P, kD, 256, hb, 0);
  const float* b1 = w + n1;
  const float* np = b1 + P;
  std::vector<float> scale(P, 1.f), shift(b1, b1 + P), lng, lnb;
  const float* w2 = np;
  if (norm == 1) {
    lng.assign(np, np + P);
    lnb.assign(np + P, np + 2 * P);
    w2 = np + 2 * P;
  } else if (norm == 2) {
    const float *gam = np, *bet = np + P, *rm = np + 2 * P, *rv = np + 3 * P;
    for (int i = 0; i < P; ++i) {
      const double sc = (double)gam[i] / std::sqrt((double)rv[i] + (double)eps);
      scale[i] = (float)sc;
      shift[i] = (float)(((double)b1[i] - (double)rm[i]) * sc + (double)bet[i]);
    }
    w2 = np + 4 * P;
  }
  pack_blocks(w2, kD, P, kD, hb, n1);
  const float* b2 = w2 + n2;
  std::vector<float> fv;
  auto take = [&](const float* src, size_t n) {
    const size_t o = fv.size();
    fv.insert(fv.end(), src, src + n);
    while (fv.size() % 64) fv.push_back(0.f);  // 256-byte aligned vectors
    return o;
  };
  const size_t o_scale = take(scale.data(), P), o_shift = take(shift.data(), P), o_b2 = take(b2, kD);
  const size_t o_lng = norm == 1 ? take(lng.data(), P) : 0, o_lnb = norm == 1 ? take(lnb.data(), P) : 0;
  const size_t bf_bytes = (hb.size() * 2 + 1023) / 1024 * 1024;
  cudaError_t ce = cudaMalloc(&h->d_w, bf_bytes + fv.size() * 4);
  if (ce == cudaSuccess) ce = cudaMemcpy(h->d_w, hb.data(), hb.size() * 2, cudaMemcpyHostToDevice);
  if (ce == cudaSuccess)
    ce = cudaMemcpy(static_cast<uint8_t*>(h->d_w) + bf_bytes, fv.data(), fv.size() * 4, cudaMemcpyHostToDevice);
  if (ce == cudaSuccess) ce = set_gemm_smem<256, EPI_GELU_OP>();
  if (ce == cudaSuccess) ce = set_gemm_smem<256, EPI_F32>();
  if (ce == cudaSuccess) ce = set_gemm_smem<192, EPI_F32>();
  if (ce != cudaSuccess) {
    mlp_head_destroy(h);
    return ce;
  }
  const auto* wb = static_cast<const __nv_bfloat16*>(h->d_w);
  const auto* wf = reinterpret_cast<const float*>(static_cast<const uint8_t*>(h->d_w) + bf_bytes);
  h->w1 = wb;
  h->w2 = wb + n1;
  h->scale = wf + o_scale;
  h->shift = wf + o_shift;
  h->b2 = wf + o_b2;
  h->ln_g = norm == 1 ? wf + o_lng : nullptr;
  h->ln_b = norm == 1 ? wf + o_lnb : nullptr;
  return cudaSuccess;
}

void mlp_head_destroy(MlpHead* h) {
  if (h->d_w) cudaFree(h->d_w);
  *h = MlpHead{};
}

cudaError_t mlp_head_run(const MlpHead& h, const __nv_bfloat16* in_op, int n_rows, __nv_bfloat16* hid_op,
                         float* hid32, float* out, uint32_t* status, cudaStream_t st) {
  const int tiles = (n_rows + 127) / 128;
  EpiArgs pa{};
  pa.rows = n_rows;
  pa.n_total = h.P;
  if (h.norm == 1) {
    pa.x = hid32;
    pa.bias = h.shift;  // the Linear bias (scale 1 without BatchNorm)
    launch_gemm<256, EPI_F32>(in_op, kHB, h.w1, tiles, h.P / 256, pa, status, st);
    k_vit_ln_wide<<<tiles * 16, 256, 0, st>>>(hid32, h.P, n_rows, tiles * 128, h.eps, h.ln_g, h.ln_b, 1, hid_op);
  } else {
    pa.op = hid_op;
    pa.scale = h.scale;
    pa.bias = h.shift;
    launch_gemm<256, EPI_GELU_OP>(in_op, kHB, h.w1, tiles, h.P / 256, pa, status, st);
  }
  EpiArgs oa{};
  oa.rows = n_rows;
  oa.n_total = kD;
  oa.x = out;
  oa.bias = h.b2;
  launch_gemm<192, EPI_F32>(hid_op, h.P / 64, h.w2, tiles, 1, oa, status, st);
  return cudaGetLastError();
}

}  // namespace lewm
