// Mixture-of-experts kernels for sm_100a ("K3"/"K4"/"K5"/"K6"):
//
//   * route_topk       router logits -> top-k experts + weights. gpt-oss: top-k
//                      on the logits, softmax over the k (rlx-models-core
//                      src/standard_decoder.rs:1063-1093); qwen3-moe: softmax
//                      over all experts, top-k, optional renormalisation.
//   * moe_align        per-expert counts, offsets, the permutation
//                      (token, slot) -> row of the expert-sorted activation
//                      matrix, its inverse, and the list of token tiles per
//                      expert - all on the device (no host sync, graph safe).
//   * gather_rows      builds the expert-sorted activation matrix.
//   * moe_gemm         grouped GEMM over experts with MXFP4 weights (E2M1
//                      codes, one E8M0 scale per 32 along K - the gpt-oss
//                      checkpoint layout), weights as the M = 128 operand and
//                      a 32..128-token tile as N. Warp roles: producer (TMA
//                      token tile + bulk copy of a pre-tiled weight block), MMA
//                      issuer (tcgen05 kind::f16, A from TMEM), 8 converter
//                      warps that expand E2M1 codes to f16 (hardware cvt + one
//                      f16x2 scale multiply) straight into TMEM, 4 epilogue warps.
//                      Epilogues: clamped SwiGLU with bias (gate/up) and
//                      bias x router weight (down).
//   * combine          out[t] = sum over its k rows (fixed slot order).
//
// The reference runs the grouped MXFP4 matmul as a SIMT kernel per expert slot
// (rlx-models-core src/standard_decoder.rs:1120-1190; external
// dequant_matmul_mlx.cu, crates/rlx-kimi-k3/docs/MOE_EXPERT_OPTIMIZATION.md:68-105).
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <cstdlib>
#include <stdexcept>

#include "../common/b200.cuh"
#include "../common/launch.h"
#include "../common/pdl_launch.h"
#include "../common/tma_host.h"

namespace b200 {
namespace moe {

// ---------------------------------------------------------------------------
// Routing
// ---------------------------------------------------------------------------
// One warp per token; E <= 256 logits (E / 32 per lane), k <= 8.
__global__ void route_topk_kernel(const float* __restrict__ logits, int64_t ld, int T, int E, int k,
                                  int softmax_first, int renorm, int32_t* __restrict__ experts,
                                  float* __restrict__ weights) {
  pdl_wait();
  pdl_trigger();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= T) return;
  const float* x = logits + (int64_t)warp * ld;
  constexpr int MAXV = 8;
  float v[MAXV];
  const int per = (E + 31) / 32;
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int e = lane + i * 32;
    v[i] = (i < per && e < E) ? x[e] : -INFINITY;
    mx = fmaxf(mx, v[i]);
  }
  if (softmax_first) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      v[i] = (v[i] == -INFINITY) ? 0.f : __expf(v[i] - mx);
      s += v[i];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
#pragma unroll
    for (int i = 0; i < MAXV; ++i) v[i] = (lane + i * 32 < E && i < per) ? v[i] / s : -INFINITY;
  }
  float sel_v[8];
  int sel_e[8];
  for (int j = 0; j < k; ++j) {
    // warp argmax (ties -> lowest expert id)
    float bv = -INFINITY;
    int be = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const int e = lane + i * 32;
      if (v[i] > bv || (v[i] == bv && e < be)) {
        bv = v[i];
        be = e;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oe = __shfl_xor_sync(0xffffffffu, be, o);
      if (ov > bv || (ov == bv && oe < be)) {
        bv = ov;
        be = oe;
      }
    }
    sel_v[j] = bv;
    sel_e[j] = be;
#pragma unroll
    for (int i = 0; i < MAXV; ++i)
      if (lane + i * 32 == be) v[i] = -INFINITY;
  }
  if (lane == 0) {
    float w[8];
    if (!softmax_first) {  // softmax over the selected logits (gpt-oss)
      float m = sel_v[0], s = 0.f;
      for (int j = 0; j < k; ++j) {
        w[j] = __expf(sel_v[j] - m);
        s += w[j];
      }
      for (int j = 0; j < k; ++j) w[j] /= s;
    } else {
      float s = 0.f;
      for (int j = 0; j < k; ++j) {
        w[j] = sel_v[j];
        s += w[j];
      }
      if (renorm)
        for (int j = 0; j < k; ++j) w[j] /= s;
    }
    for (int j = 0; j < k; ++j) {
      experts[(int64_t)warp * k + j] = sel_e[j];
      weights[(int64_t)warp * k + j] = w[j];
    }
  }
}

// Single CTA: counts, exclusive offsets, list of bt-row token tiles, permutation.
// meta layout (int32): [0] total tiles, [1 .. E] counts, [E+1 .. 2E+1] offsets.
// tiles: int4 per tile {expert, tile index within the expert, first sorted row, valid rows}.
__global__ void moe_align_kernel(const int32_t* __restrict__ experts, int n_assign, int E, int e_lo, int e_cnt,
                                 int bt, int32_t* __restrict__ meta, int32_t* __restrict__ tiles, int max_tiles,
                                 int32_t* __restrict__ perm, int32_t* __restrict__ inv, int32_t* __restrict__ cursor) {
  pdl_wait();
  pdl_trigger();
  int32_t* counts = meta + 1;
  int32_t* offs = meta + 1 + E;
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    counts[e] = 0;
    cursor[e] = 0;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < n_assign; i += blockDim.x) {
    const int e = experts[i] - e_lo;
    if (e >= 0 && e < e_cnt) atomicAdd(&counts[e], 1);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int off = 0, nt = 0;
    for (int e = 0; e < E; ++e) {
      offs[e] = off;
      const int c = (e < e_cnt) ? counts[e] : 0;
      const int mt = (c + bt - 1) / bt;
      for (int m = 0; m < mt && nt < max_tiles; ++m, ++nt)  // tile info {expert, m, first row, rows}
        reinterpret_cast<int4*>(tiles)[nt] = make_int4(e, m, off + m * bt, min(bt, c - m * bt));
      off += c;
    }
    offs[E] = off;
    meta[0] = nt;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < n_assign; i += blockDim.x) {
    const int e = experts[i] - e_lo;
    if (e >= 0 && e < e_cnt) {
      const int pos = offs[e] + atomicAdd(&cursor[e], 1);
      perm[pos] = i;  // assignment index = token * k + slot
      inv[i] = pos;
    } else {
      inv[i] = -1;
    }
  }
}

// A_perm[pos] = x[perm[pos] / k]   (16-byte vectors)
// TO_F16: bf16 rows -> f16 (the grouped GEMM's operand type).
template <bool TO_F16>
__global__ void gather_rows_kernel(const uint4* __restrict__ x, int64_t H8, const int32_t* __restrict__ perm,
                                   const int32_t* __restrict__ meta, int E, int k, uint4* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  const int total = meta[1 + E + E];
  for (int pos = blockIdx.x; pos < total; pos += gridDim.x) {
    const int t = perm[pos] / k;
    for (int64_t i = threadIdx.x; i < H8; i += blockDim.x) {
      uint4 v = __ldg(x + (int64_t)t * H8 + i);
      if (TO_F16) {
        uint32_t* w = reinterpret_cast<uint32_t*>(&v);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const __half2 h = __floats2half2_rn(bf16_lo(w[j]), bf16_hi(w[j]));
          w[j] = *reinterpret_cast<const uint32_t*>(&h);
        }
      }
      out[(int64_t)pos * H8 + i] = v;
    }
  }
}

// out[t] = sum_s rows[inv[t*k + s]]  (fixed slot order; missing slots skipped)
__global__ void combine_kernel(const __nv_bfloat16* __restrict__ rows, const int32_t* __restrict__ inv, int k,
                               int64_t H, __nv_bfloat16* __restrict__ out, int accumulate) {
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x;
  for (int64_t c = threadIdx.x * 8; c < H; c += blockDim.x * 8) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if (accumulate) {
      const uint4 o = *reinterpret_cast<const uint4*>(out + (int64_t)t * H + c);
      const uint32_t ow[4] = {o.x, o.y, o.z, o.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        acc[2 * q] = bf16_lo(ow[q]);
        acc[2 * q + 1] = bf16_hi(ow[q]);
      }
    }
    for (int s = 0; s < k; ++s) {
      const int pos = inv[(int64_t)t * k + s];
      if (pos < 0) continue;
      const uint4 r = *reinterpret_cast<const uint4*>(rows + (int64_t)pos * H + c);
      const uint32_t rw[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        acc[2 * q] += bf16_lo(rw[q]);
        acc[2 * q + 1] += bf16_hi(rw[q]);
      }
    }
    *reinterpret_cast<uint4*>(out + (int64_t)t * H + c) =
        make_uint4(pack_bf16x2(acc[0], acc[1]), pack_bf16x2(acc[2], acc[3]), pack_bf16x2(acc[4], acc[5]),
                   pack_bf16x2(acc[6], acc[7]));
  }
}

// ---------------------------------------------------------------------------
// Grouped MXFP4 GEMM, weights x tokens^T ("swap-AB")
// ---------------------------------------------------------------------------
// The accumulator tile is [128 weight rows (output features)] x [BT tokens]:
// the expert's weight tile is the tcgen05 A operand (M = 128) and its tokens
// are B (N = BT). A decode step routes a handful of tokens to each expert, so
// BT = 32 keeps the token tile small while every weight byte is read once;
// prefill uses BT = 128.
//
// The dequantised weight tile never touches shared memory: converter warps
// write it straight into TMEM (tcgen05.st) and the MMA reads A from TMEM.
// Expanding 4-bit codes to a 16-bit tile in shared memory would cost ~8 bytes
// of shared-memory traffic per weight (write + MMA read) against 0.5 byte from
// HBM, which caps a weight-streaming decode step near a third of HBM
// bandwidth; through TMEM, shared memory only carries the packed codes and the
// token tile.
//
// Weights are re-laid out at load time (quant/mxfp4.py `tile_mxfp4`) into one
// contiguous block per (expert, 128-row n-tile, 64-wide k-tile): 4096 bytes of
// E2M1 codes ([2 k-halves][128 rows][16 bytes], low nibble = even k) followed
// by 256 bytes of scale offsets ([2][128 rows]): each group's E8M0 exponent stored as
// d = row_exp - s, where row_exp (a separate [E, rows] byte array) is the
// largest exponent of the weight row. One cp.async.bulk moves a block;
// converter warps expand it with the hardware E2M1x2 -> f16x2 conversion and
// one f16x2 multiply by 2^-d (at most 1, so nothing overflows) into the
// TMEM A tile that the MMA reads; the epilogue multiplies
// each accumulator row by 2^(row_exp - 127) in fp32. Operands are f16 (tokens
// are converted when gathered): f16 has three more mantissa bits than bf16 and
// the expert inputs (RMS-normalised activations, clamped SwiGLU outputs) sit
// far inside its range.
//
// Warps: 0 producer (TMA token tile + bulk weight block), 1 MMA issuer,
// 2-5 epilogue (TMEM lane quadrant = warp % 4), 6-13 converters.
constexpr int kBK = 64;
constexpr uint32_t kWBlock = 4096 + 256;
constexpr int kConvWarps = 8;
constexpr int kThreads = (6 + kConvWarps) * 32;
constexpr int kNC = 8;                 // TMEM A ring: 8 x [128 lanes x 32 columns] at columns 256..511
constexpr uint32_t kTmemCols = 512;    // accumulators at [0, 2 BT), A ring at [256, 512)

template <int BT>
struct MoeCfg {
  static_assert(BT == 32 || BT == 64 || BT == 128, "token tile");
  static constexpr uint32_t kTok = BT * kBK * 2;
  static constexpr uint32_t kPStage = (kTok + kWBlock + 1023) / 1024 * 1024;
  static constexpr uint32_t kXchg = 64 * 33 * 4;
  static constexpr int kNP = (200 * 1024) / kPStage;  // 21 / 15 / 9 stages
  static constexpr uint32_t kSmem = 1024 + kNP * kPStage + kXchg + 512;
  static_assert(kSmem <= 232448, "shared memory");
};

enum MoeEpi : int { MOE_SWIGLU_CLAMP = 0, MOE_DOWN = 1 };

struct MoeParams {
  const int32_t* meta;    // [0] tiles, counts[E], offsets[E + 1]
  const int4* tiles;      // {expert, token-tile index, first sorted row, valid rows}
  int E;                  // local experts
  int N, NT, KT;          // weight rows (output features), 128-row tiles, 64-wide k tiles
  const uint8_t* w;       // tiled blocks [E, NT, KT, kWBlock]
  const uint8_t* row_exp; // [E, NT * 128] largest E8M0 exponent of each weight row
  const __nv_bfloat16* bias;  // [E, N] or null
  const float* row_weight;    // [n_assign] router weight per assignment (down) or null
  const int32_t* perm;        // sorted row -> assignment
  void* out;                  // [rows, N] bf16 (down) or [rows, N / 2] f16 (gate/up)
  float limit, alpha;         // clamped SwiGLU
  float up_offset;            // act = (up + up_offset) * g * sigmoid(alpha g): gpt-oss 1, plain SwiGLU 0
  int* status;
  int debug;                  // B200_MOE_DEBUG (timing experiments only): bit 0 skips the dequant,
                              // bit 1 the MMAs, bit 2 the token-tile loads, bit 3 runs the copy
                              // stream alone (no consumers)
};

__device__ __forceinline__ uint32_t f16x2_mul(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// Eight E2M1 codes (one packed word, low nibble first) -> four f16x2 words
// scaled by fac (f16x2).
__device__ __forceinline__ void e2m1x8_to_f16(uint32_t w, uint32_t fac, uint32_t (&o)[4]) {
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "mov.b32 {b0, b1, b2, b3}, %4;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t"
      "cvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %2, b2;\n\t"
      "cvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
      : "=r"(o[0]), "=r"(o[1]), "=r"(o[2]), "=r"(o[3])
      : "r"(w));
#pragma unroll
  for (int j = 0; j < 4; ++j) o[j] = f16x2_mul(o[j], fac);
}

// f16 bits of 2^-d (d >= 0): normal down to 2^-14, subnormal to 2^-24, then 0.
__device__ __forceinline__ uint32_t f16_pow2_neg(uint32_t d) {
  return d <= 14u ? (15u - d) << 10 : (d <= 24u ? 1u << (24u - d) : 0u);
}

// 2^(e - 127) as f32 (E8M0 value); e = 0 -> 0.
__device__ __forceinline__ float e8m0_f32(uint32_t e) { return e ? __uint_as_float(e << 23) : 0.f; }

template <int BT, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    moe_gemm_kernel(const __grid_constant__ CUtensorMap tmX, const MoeParams p) {
  using Cfg = MoeCfg<BT>;
  constexpr int NP = Cfg::kNP, NC = kNC;
  extern __shared__ uint8_t smem_dyn[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~uintptr_t(1023));
  float* xchg = reinterpret_cast<float*>(smem + NP * Cfg::kPStage);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + NP * Cfg::kPStage + Cfg::kXchg);
  uint64_t* fullP = bars;
  uint64_t* emptyP = fullP + NP;
  uint64_t* fullC = emptyP + NP;
  uint64_t* emptyC = fullC + NC;
  uint64_t* accf = emptyC + NC;
  uint64_t* acce = accf + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acce + 2);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tmX);
    for (int s = 0; s < NP; ++s) {
      mbar_init(&fullP[s], 1);
      mbar_init(&emptyP[s], 1);
    }
    for (int c = 0; c < NC; ++c) {
      mbar_init(&fullC[c], kConvWarps);
      mbar_init(&emptyC[c], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&accf[a], 1);
      mbar_init(&acce[a], 4);
    }
    fence_mbarrier_init();
  }
  if (warp == 2) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_wait();  // routing metadata and activations come from the previous kernels
  pdl_trigger();
  const int units = p.meta[0] * p.NT;
  // each CTA takes a contiguous run of units: consecutive n-tiles of one expert
  // are adjacent weight blocks and share the token tile
  const int u_begin = (int)(((int64_t)blockIdx.x * units) / gridDim.x);
  const int u_end = (int)(((int64_t)(blockIdx.x + 1) * units) / gridDim.x);

  if (warp == 0) {
    if (elect_one_sync()) {
      int s = 0;
      uint32_t ph = 0;
      int4 cur = u_begin < u_end ? p.tiles[u_begin / p.NT] : make_int4(0, 0, 0, 0);
      for (int u = u_begin; u < u_end; ++u) {
        const int un = u + 1;  // next unit's tile info: load now, use next iteration
        const int4 nxt = un < u_end ? p.tiles[un / p.NT] : cur;
        const int e = cur.x, nt = u % p.NT;
        const int row0 = cur.z;
        const uint8_t* wblk = p.w + ((int64_t)e * p.NT + nt) * p.KT * kWBlock;
        for (int kt = 0; kt < p.KT; ++kt) {
          if (p.debug & 8) {  // copy-engine streaming only: wait for this stage's previous copy to land
            if (!mbar_wait(&fullP[s], ph ^ 1, p.status, kErrTimeoutEmpty)) goto prod_done;
          } else if (!mbar_wait(&emptyP[s], ph ^ 1, p.status, kErrTimeoutEmpty)) {
            goto prod_done;
          }
          uint8_t* st = smem + s * Cfg::kPStage;
          mbar_arrive_expect_tx(&fullP[s], ((p.debug & 4) ? 0u : Cfg::kTok) + kWBlock);
          if (!(p.debug & 4)) tma_load_2d(st, &tmX, &fullP[s], kt * kBK, row0);
          bulk_load(st + Cfg::kTok, wblk + (int64_t)kt * kWBlock, kWBlock, &fullP[s]);
          if (++s == NP) {
            s = 0;
            ph ^= 1;
          }
        }
        cur = nxt;
      }
      if (p.debug & 8) {  // drain: every stage's last copy has landed
        for (int i = 0; i < NP; ++i) {
          if (!mbar_wait(&fullP[s], ph ^ 1, p.status, kErrTimeoutDrain)) break;
          if (++s == NP) {
            s = 0;
            ph ^= 1;
          }
        }
      }
    prod_done:;
    }
  } else if (p.debug & 8) {
    // streaming experiment: other roles idle
  } else if (warp == 1) {
    if (elect_one_sync()) {
      constexpr uint32_t idesc = umma_idesc_f16(128, BT, false, false);
      int s = 0, c = 0, it = 0;
      uint32_t ph = 0, phc = 0;
      for (int u = u_begin; u < u_end; ++u, ++it) {
        const int acc = it & 1;
        if (!mbar_wait(&acce[acc], ((it >> 1) & 1) ^ 1, p.status, kErrTimeoutAccEmpty)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + acc * BT;
        for (int kt = 0; kt < p.KT; ++kt) {
          if (!mbar_wait(&fullP[s], ph, p.status, kErrTimeoutFull)) goto mma_done;
          if (!mbar_wait(&fullC[c], phc, p.status, kErrTimeoutFull)) goto mma_done;
          tc_fence_after();
          const uint32_t a_tm = tmem_base + 256 + c * 32;
          const uint32_t b_addr = smem_u32(smem + s * Cfg::kPStage);
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)
            if (!(p.debug & 2)) umma_f16_ts(d, a_tm + kk * 8, umma_desc_sw128(b_addr + kk * 32, 16, 1024), idesc,
                        (kt > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&emptyP[s]);
          umma_commit(&emptyC[c]);
          if (++s == NP) {
            s = 0;
            ph ^= 1;
          }
          if (++c == NC) {
            c = 0;
            phc ^= 1;
          }
        }
        umma_commit(&accf[acc]);
      }
    mma_done:;
    }
  } else if (warp >= 6) {
    // converters: warp -> (TMEM lane quadrant, k half); thread -> weight row. 16 packed
    // bytes = 32 codes sharing one scale -> 16 TMEM columns of f16x2.
    const int qd = warp & 3;
    const int half = (warp - 6) >> 2;
    const int r = qd * 32 + lane;
    const uint32_t t_row = tmem_base + ((uint32_t)(qd * 32) << 16) + 256 + half * 16;
    int s = 0, c = 0;
    uint32_t ph = 0, phc = 0;
    for (int u = u_begin; u < u_end; ++u) {
      for (int kt = 0; kt < p.KT; ++kt) {
        if (!mbar_wait(&fullP[s], ph, p.status, kErrTimeoutFull)) return;
        if (!mbar_wait(&emptyC[c], phc ^ 1, p.status, kErrTimeoutEmpty)) return;
        const uint8_t* blk = smem + s * Cfg::kPStage + Cfg::kTok;
        if (!(p.debug & 1)) {
          const uint4 q = *reinterpret_cast<const uint4*>(blk + half * 2048 + r * 16);
          const uint32_t f = f16_pow2_neg(blk[4096 + half * 128 + r]);
          const uint32_t fac = f | (f << 16);
          uint32_t o[16];
          e2m1x8_to_f16(q.x, fac, *reinterpret_cast<uint32_t(*)[4]>(&o[0]));
          e2m1x8_to_f16(q.y, fac, *reinterpret_cast<uint32_t(*)[4]>(&o[4]));
          e2m1x8_to_f16(q.z, fac, *reinterpret_cast<uint32_t(*)[4]>(&o[8]));
          e2m1x8_to_f16(q.w, fac, *reinterpret_cast<uint32_t(*)[4]>(&o[12]));
          tmem_st_32x32b_x16(t_row + c * 32, o);
          tmem_wait_st();
        }
        tc_fence_before();  // TMEM stores -> visible to the MMA issued after the barrier
        __syncwarp();
        if (lane == 0) mbar_arrive(&fullC[c]);
        if (++s == NP) {
          s = 0;
          ph ^= 1;
        }
        if (++c == NC) {
          c = 0;
          phc ^= 1;
        }
      }
    }
  } else {
    // epilogue warps 2..5: TMEM lanes (weight rows) q*32 .. q*32 + 31, columns = tokens
    const int q = warp & 3;
    int it = 0;
    int4 cur = u_begin < u_end ? p.tiles[u_begin / p.NT] : make_int4(0, 0, 0, 0);
    for (int u = u_begin; u < u_end; ++u, ++it) {
      const int acc = it & 1;
      const int un = u + 1;
      const int4 nxt = un < u_end ? p.tiles[un / p.NT] : cur;
      const int e = cur.x, nt = u % p.NT;
      const int rows_valid = cur.w;
      const int row0 = cur.z;
      cur = nxt;
      if (!mbar_wait(&accf[acc], (it >> 1) & 1, p.status, kErrTimeoutAccFull)) break;
      tc_fence_after();
      const uint32_t t_lane = tmem_base + ((uint32_t)(q * 32) << 16) + acc * BT;
      const float rf = e8m0_f32(p.row_exp[((int64_t)e * p.NT + nt) * 128 + q * 32 + lane]);
      if (EPI == MOE_SWIGLU_CLAMP) {
        // rows [0, 64) gate, [64, 128) up of features nt * 64 + [0, 64)
        const int fl = (q & 1) * 32 + lane;
        const int Nh = p.N / 2;
        const int f = nt * 64 + fl;
        float bg = 0.f, bu = 0.f;
        if (p.bias != nullptr) {
          bg = __bfloat162float(p.bias[(int64_t)e * p.N + nt * 128 + fl]);
          bu = __bfloat162float(p.bias[(int64_t)e * p.N + nt * 128 + 64 + fl]);
        }
#pragma unroll 1
        for (int cc = 0; cc < BT / 32; ++cc) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(t_lane + cc * 32, v);
          tmem_wait_ld();
          if (q >= 2) {
#pragma unroll
            for (int j = 0; j < 32; ++j) xchg[fl * 33 + j] = __uint_as_float(v[j]) * rf + bu;
          }
          named_bar_sync(1, 128);
          if (q < 2) {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const int col = cc * 32 + j;
              if (col < rows_valid) {
                float g = __uint_as_float(v[j]) * rf + bg;
                float uu = xchg[fl * 33 + j];
                g = fminf(g, p.limit);
                uu = fmaxf(fminf(uu, p.limit), -p.limit);
                const float a = (uu + p.up_offset) * g / (1.f + __expf(-p.alpha * g));
                reinterpret_cast<__half*>(p.out)[(int64_t)(row0 + col) * Nh + f] = __float2half_rn(a);
              }
            }
          }
          named_bar_sync(1, 128);
        }
      } else {
        const int f = nt * 128 + q * 32 + lane;
        const bool fvalid = f < p.N;
        const float bd = (p.bias != nullptr && fvalid) ? __bfloat162float(p.bias[(int64_t)e * p.N + f]) : 0.f;
#pragma unroll 1
        for (int cc = 0; cc < BT / 32; ++cc) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(t_lane + cc * 32, v);
          tmem_wait_ld();
          const int mycol = cc * 32 + lane;
          float rwl = 1.f;
          if (p.row_weight != nullptr && mycol < rows_valid) rwl = p.row_weight[p.perm[row0 + mycol]];
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const float rw = __shfl_sync(0xffffffffu, rwl, j);
            const int col = cc * 32 + j;
            if (fvalid && col < rows_valid)
              reinterpret_cast<__nv_bfloat16*>(p.out)[(int64_t)(row0 + col) * p.N + f] =
                  __float2bfloat16((__uint_as_float(v[j]) * rf + bd) * rw);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acce[acc]);
    }
  }
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

}  // namespace moe

void moe_route_launch(const float* logits, int64_t ld, int T, int E, int k, int softmax_first, int renorm,
                      int32_t* experts, float* weights, cudaStream_t st) {
  if (T == 0) return;
  if (E > 256 || k > 8) throw std::runtime_error("b200.moe_route: E <= 256, k <= 8");
  launch_pdl(moe::route_topk_kernel, dim3((T * 32 + 255) / 256), dim3(256), 0, st, logits, ld, T, E, k,
             softmax_first, renorm, experts, weights);
}

void moe_align_launch(const int32_t* experts, int n_assign, int E, int e_lo, int e_cnt, int bt, int32_t* meta,
                      int32_t* tiles, int max_tiles, int32_t* perm, int32_t* inv, int32_t* cursor, cudaStream_t st) {
  launch_pdl(moe::moe_align_kernel, dim3(1), dim3(1024), 0, st, experts, n_assign, E, e_lo, e_cnt, bt, meta, tiles,
             max_tiles, perm, inv, cursor);
}

void moe_gather_launch(const void* x, int64_t H, const int32_t* perm, const int32_t* meta, int E, int k,
                       int max_rows, void* out, int to_f16, cudaStream_t st) {
  if (max_rows == 0) return;
  if (to_f16)
    launch_pdl(moe::gather_rows_kernel<true>, dim3(std::min(max_rows, 148 * 8)), dim3(128), 0, st,
               reinterpret_cast<const uint4*>(x), H / 8, perm, meta, E, k, reinterpret_cast<uint4*>(out));
  else
    launch_pdl(moe::gather_rows_kernel<false>, dim3(std::min(max_rows, 148 * 8)), dim3(128), 0, st,
               reinterpret_cast<const uint4*>(x), H / 8, perm, meta, E, k, reinterpret_cast<uint4*>(out));
}

void moe_combine_launch(const void* rows, const int32_t* inv, int T, int k, int64_t H, void* out, int accumulate,
                        cudaStream_t st) {
  if (T == 0) return;
  launch_pdl(moe::combine_kernel, dim3(T), dim3(128), 0, st, reinterpret_cast<const __nv_bfloat16*>(rows), inv, k, H,
             reinterpret_cast<__nv_bfloat16*>(out), accumulate);
}

template <int BT, int EPI>
static void moe_gemm_go(const MoeGemmArgs& a, const moe::MoeParams& p, int grid, cudaStream_t st) {
  using namespace moe;
  CUtensorMap tx = make_tmap_2d(a.x, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, a.rows, a.K, a.K, BT, kBK);
  auto k = moe_gemm_kernel<BT, EPI>;
  ensure_smem(k, MoeCfg<BT>::kSmem);
  launch_pdl(k, dim3(grid), dim3(kThreads), MoeCfg<BT>::kSmem, st, tx, p);
}

template <int EPI>
static void moe_gemm_bt(const MoeGemmArgs& a, const moe::MoeParams& p, int grid, cudaStream_t st) {
  switch (a.bt) {
    case 32: return moe_gemm_go<32, EPI>(a, p, grid, st);
    case 64: return moe_gemm_go<64, EPI>(a, p, grid, st);
    case 128: return moe_gemm_go<128, EPI>(a, p, grid, st);
    default: throw std::runtime_error("b200.moe_gemm: token tile must be 32, 64 or 128");
  }
}

void moe_gemm_launch(const MoeGemmArgs& a, cudaStream_t st) {
  using namespace moe;
  if (a.K % kBK != 0 || a.N % 32 != 0 || (a.swiglu && a.N % 128 != 0))
    throw std::runtime_error("b200.moe_gemm: K % 64, N % 32 (N % 128 for gate/up) required");
  if (a.rows == 0 || a.max_tiles == 0) return;
  MoeParams p{};
  p.meta = a.meta;
  p.tiles = reinterpret_cast<const int4*>(a.tiles);
  p.E = a.E;
  p.N = a.N;
  p.NT = (a.N + 127) / 128;
  p.KT = a.K / kBK;
  p.w = reinterpret_cast<const uint8_t*>(a.w);
  p.row_exp = reinterpret_cast<const uint8_t*>(a.row_exp);
  p.bias = reinterpret_cast<const __nv_bfloat16*>(a.bias);
  p.row_weight = a.row_weight;
  p.perm = a.perm;
  p.out = a.out;
  p.limit = a.limit;
  p.alpha = a.alpha;
  p.up_offset = a.up_offset;
  p.status = a.status;
  static const int dbg = [] {
    const char* e = std::getenv("B200_MOE_DEBUG");
    return e ? std::atoi(e) : 0;
  }();
  p.debug = dbg;
  const int grid = (int)std::min<int64_t>(num_sms(a.device), (int64_t)a.max_tiles * p.NT);
  if (a.swiglu)
    moe_gemm_bt<MOE_SWIGLU_CLAMP>(a, p, grid, st);
  else
    moe_gemm_bt<MOE_DOWN>(a, p, grid, st);
}

}  // namespace b200
