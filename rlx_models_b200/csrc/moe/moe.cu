// Mixture-of-experts kernels for sm_100a ("K3"/"K4"/"K5"/"K6"):
//
//   * route_topk       router logits -> top-k experts + weights. gpt-oss: top-k
//                      on the logits, softmax over the k (rlx-models-core
//                      src/standard_decoder.rs:1063-1093); qwen3-moe: softmax
//                      over all experts, top-k, optional renormalisation.
//   * moe_align        per-expert counts, offsets, the permutation
//                      (token, slot) -> row of the expert-sorted activation
//                      matrix, its inverse, and the list of 128-row tiles per
//                      expert - all on the device (no host sync, graph safe).
//   * gather_rows      builds the expert-sorted activation matrix.
//   * moe_gemm         grouped GEMM over experts with MXFP4 weights (E2M1
//                      codes, one E8M0 scale per 32 along K - the gpt-oss
//                      checkpoint layout). Warp roles: TMA producer (activation
//                      tile + packed weight bytes), MMA issuer (tcgen05 kind::f16
//                      into TMEM), 4 converter warps that expand the packed
//                      weights to bf16 straight into the 128-byte-swizzled UMMA
//                      layout, 4 epilogue warps. Epilogues: clamped SwiGLU with
//                      bias (gate/up) and bias + router weight (down).
//   * combine          out[t] = sum over its k rows (fixed slot order).
//
// The reference runs the grouped MXFP4 matmul as a SIMT kernel per expert slot
// (rlx-models-core src/standard_decoder.rs:1120-1190; external
// dequant_matmul_mlx.cu, crates/rlx-kimi-k3/docs/MOE_EXPERT_OPTIMIZATION.md:68-105).
#include <cuda_bf16.h>

#include <algorithm>
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

// Single CTA: counts, exclusive offsets, 128-row tile list, permutation.
// meta layout (int32): [0] total tiles, [1 .. E] counts, [E+1 .. 2E+1] offsets.
__global__ void moe_align_kernel(const int32_t* __restrict__ experts, int n_assign, int E, int e_lo, int e_cnt,
                                 int32_t* __restrict__ meta, int32_t* __restrict__ tiles, int max_tiles,
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
      const int mt = (c + 127) / 128;
      for (int m = 0; m < mt && nt < max_tiles; ++m) tiles[nt++] = (e << 16) | m;
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
__global__ void gather_rows_kernel(const uint4* __restrict__ x, int64_t H8, const int32_t* __restrict__ perm,
                                   const int32_t* __restrict__ meta, int E, int k, uint4* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  const int total = meta[1 + E + E];
  for (int pos = blockIdx.x; pos < total; pos += gridDim.x) {
    const int t = perm[pos] / k;
    for (int64_t i = threadIdx.x; i < H8; i += blockDim.x) out[(int64_t)pos * H8 + i] = __ldg(x + (int64_t)t * H8 + i);
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
// Grouped MXFP4 GEMM
// ---------------------------------------------------------------------------
constexpr int kBM = 128, kBK = 64, kBN = 128;
constexpr int kStages = 5;
constexpr int kThreads = 320;  // 10 warps
constexpr uint32_t kA = kBM * kBK * 2;       // 16 KB bf16 activations
constexpr uint32_t kB = kBN * kBK * 2;       // 16 KB bf16 weights (converted)
constexpr uint32_t kP = kBN * kBK / 2;       // 4 KB packed E2M1
constexpr uint32_t kStage = kA + kB + kP;
constexpr uint32_t kSmem = 1024 + kStages * kStage + 32 * 132 * 4 + 512;

enum MoeEpi : int { MOE_SWIGLU_CLAMP = 0, MOE_DOWN = 1 };

struct MoeParams {
  const int32_t* meta;    // [0] tiles, counts, offsets
  const int32_t* tiles;   // (expert << 16) | m_tile
  int E;                  // local experts
  int N, K;               // weight rows (output features) / reduction dim
  const uint8_t* scales;  // [E, N, K/32]
  const __nv_bfloat16* bias;  // [E, N] or null
  const float* row_weight;    // [n_assign] router weight per assignment (down epilogue) or null
  const int32_t* perm;        // row -> assignment (for row_weight)
  __nv_bfloat16* out;         // [rows, N] (down) or [rows, N/2] (swiglu)
  float limit, alpha;         // clamped SwiGLU
  int* status;
};

__device__ __forceinline__ float e2m1(uint32_t nib) {
  const float mag[8] = {0.f, 0.5f, 1.f, 1.5f, 2.f, 3.f, 4.f, 6.f};
  const float v = mag[nib & 7u];
  return (nib & 8u) ? -v : v;
}

template <int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    moe_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmP,
                    const MoeParams p) {
  extern __shared__ uint8_t smem_dyn[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~uintptr_t(1023));
  float* xchg = reinterpret_cast<float*>(smem + kStages * kStage);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kStages * kStage + 32 * 132 * 4);
  uint64_t* full = bars;
  uint64_t* conv = bars + kStages;
  uint64_t* empty = bars + 2 * kStages;
  uint64_t* accf = bars + 3 * kStages;
  uint64_t* acce = accf + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acce + 2);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmP);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&conv[s], 4);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&accf[a], 1);
      mbar_init(&acce[a], 4);
    }
    fence_mbarrier_init();
  }
  if (warp == 2) {
    tmem_alloc(tmem_slot, 2 * kBN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_wait();  // routing metadata and activations come from the previous kernels
  pdl_trigger();
  const int n_tiles_m = p.meta[0];
  const int32_t* offs = p.meta + 1 + p.E;
  const int n_n = (p.N + kBN - 1) / kBN;
  const int units = n_tiles_m * n_n;
  const int k_tiles = p.K / kBK;

  if (warp == 0) {
    if (elect_one_sync()) {
      int s = 0;
      uint32_t ph = 0;
      for (int u = blockIdx.x; u < units; u += gridDim.x) {
        const int tv = p.tiles[u / n_n];
        const int e = tv >> 16, mt = tv & 0xffff;
        const int nt = u % n_n;
        const int row0 = offs[e] + mt * kBM;
        const int wrow = e * p.N + nt * kBN;
        for (int kt = 0; kt < k_tiles; ++kt) {
          if (!mbar_wait(&empty[s], ph ^ 1, p.status, kErrTimeoutEmpty)) goto prod_done;
          uint8_t* st = smem + s * kStage;
          mbar_arrive_expect_tx(&full[s], kA + kP);
          tma_load_2d(st, &tmA, &full[s], kt * kBK, row0);
          tma_load_2d(st + kA + kB, &tmP, &full[s], kt * (kBK / 2), wrow);
          if (++s == kStages) {
            s = 0;
            ph ^= 1;
          }
        }
      }
    prod_done:;
    }
  } else if (warp == 1) {
    if (elect_one_sync()) {
      constexpr uint32_t idesc = umma_idesc_bf16(kBM, kBN, false, false);
      int s = 0;
      uint32_t ph = 0;
      int it = 0;
      for (int u = blockIdx.x; u < units; u += gridDim.x, ++it) {
        const int acc = it & 1;
        if (!mbar_wait(&acce[acc], ((it >> 1) & 1) ^ 1, p.status, kErrTimeoutAccEmpty)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + acc * kBN;
        for (int kt = 0; kt < k_tiles; ++kt) {
          if (!mbar_wait(&conv[s], ph, p.status, kErrTimeoutFull)) goto mma_done;
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + s * kStage);
          const uint32_t b_addr = a_addr + kA;
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)
            umma_f16(d, umma_desc_sw128(a_addr + kk * 32, 16, 1024), umma_desc_sw128(b_addr + kk * 32, 16, 1024),
                     idesc, (kt > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&empty[s]);
          if (++s == kStages) {
            s = 0;
            ph ^= 1;
          }
        }
        umma_commit(&accf[acc]);
      }
    mma_done:;
    }
  } else if (warp >= 6) {
    // converters: packed E2M1 + E8M0 scale -> bf16 in the 128B-swizzled K-major layout
    const int r = threadIdx.x - 192;  // weight row within the tile, 0..127
    int s = 0;
    uint32_t ph = 0;
    for (int u = blockIdx.x; u < units; u += gridDim.x) {
      const int tv = p.tiles[u / n_n];
      const int e = tv >> 16;
      const int nt = u % n_n;
      const bool rvalid = nt * kBN + r < p.N;  // partial last n-tile: rows past N are never stored
      const uint8_t* srow = p.scales + ((int64_t)e * p.N + (rvalid ? nt * kBN + r : 0)) * (p.K / 32);
      for (int kt = 0; kt < k_tiles; ++kt) {
        if (!mbar_wait(&full[s], ph, p.status, kErrTimeoutFull)) return;
        uint8_t* st = smem + s * kStage;
        const uint4* pk = reinterpret_cast<const uint4*>(st + kA + kB + r * 32);
        const uint4 q0 = pk[0], q1 = pk[1];
        const uint32_t words[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
        const uint32_t s0 = rvalid ? srow[kt * 2] : 127u, s1 = rvalid ? srow[kt * 2 + 1] : 127u;
        const float f0 = __uint_as_float(s0 << 23), f1 = __uint_as_float(s1 << 23);  // 2^(s-127)
        uint8_t* brow = st + kA + (r >> 3) * 1024 + (r & 7) * 128;
#pragma unroll
        for (int c = 0; c < 8; ++c) {  // 8 chunks of 8 values (4 packed bytes each)
          const uint32_t w = words[c];
          const float f = c < 4 ? f0 : f1;
          uint32_t o[4];
#pragma unroll
          for (int b = 0; b < 4; ++b) {
            const uint32_t byte = (w >> (8 * b)) & 0xffu;
            o[b] = pack_bf16x2(e2m1(byte & 0xfu) * f, e2m1(byte >> 4) * f);
          }
          *reinterpret_cast<uint4*>(brow + ((c ^ (r & 7)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
        }
        fence_proxy_async_smem();  // generic-proxy writes -> visible to tcgen05.mma (async proxy)
        __syncwarp();
        if (lane == 0) mbar_arrive(&conv[s]);
        if (++s == kStages) {
          s = 0;
          ph ^= 1;
        }
      }
    }
  } else {
    // epilogue warps 2..5
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    int it = 0;
    for (int u = blockIdx.x; u < units; u += gridDim.x, ++it) {
      const int acc = it & 1;
      if (!mbar_wait(&accf[acc], (it >> 1) & 1, p.status, kErrTimeoutAccFull)) break;
      tc_fence_after();
      const int tv = p.tiles[u / n_n];
      const int e = tv >> 16, mt = tv & 0xffff;
      const int nt = u % n_n;
      const int cnt = p.meta[1 + e];
      const int rows_valid = min(kBM, cnt - mt * kBM);
      const int prow = offs[e] + mt * kBM + row;  // row of the expert-sorted matrix
      const uint32_t t_row = tmem_base + ((uint32_t)(quad * 32) << 16) + acc * kBN;
      if (EPI == MOE_SWIGLU_CLAMP) {
        // columns: [0,64) gate, [64,128) up of features nt*64 + [0,64)
#pragma unroll 1
        for (int h = 0; h < 2; ++h) {
          uint32_t rg[32], ru[32];
          tmem_ld_32x32b_x32(t_row + h * 32, rg);
          tmem_ld_32x32b_x32(t_row + 64 + h * 32, ru);
          tmem_wait_ld();
          if (row < rows_valid) {
            const int f0 = nt * 64 + h * 32;
            __nv_bfloat16* dst = p.out + (int64_t)prow * (p.N / 2) + f0;
            uint32_t packed[16];
#pragma unroll
            for (int t = 0; t < 32; t += 2) {
              float g[2], uu[2];
#pragma unroll
              for (int q = 0; q < 2; ++q) {
                const int col = nt * kBN + h * 32 + t + q;  // gate column index in the interleaved layout
                g[q] = __uint_as_float(rg[t + q]);
                uu[q] = __uint_as_float(ru[t + q]);
                if (p.bias != nullptr) {
                  g[q] += __bfloat162float(p.bias[(int64_t)e * p.N + col]);
                  uu[q] += __bfloat162float(p.bias[(int64_t)e * p.N + col + 64]);
                }
                g[q] = fminf(g[q], p.limit);
                uu[q] = fmaxf(fminf(uu[q], p.limit), -p.limit);
                g[q] = (uu[q] + 1.f) * g[q] / (1.f + __expf(-p.alpha * g[q]));
              }
              packed[t / 2] = pack_bf16x2(g[0], g[1]);
            }
#pragma unroll
            for (int q = 0; q < 4; ++q)
              *reinterpret_cast<uint4*>(dst + q * 8) =
                  make_uint4(packed[q * 4], packed[q * 4 + 1], packed[q * 4 + 2], packed[q * 4 + 3]);
          }
        }
      } else {
        const float rw = (row < rows_valid && p.row_weight != nullptr) ? p.row_weight[p.perm[prow]] : 1.f;
#pragma unroll 1
        for (int c = 0; c < kBN / 32; ++c) {
          uint32_t rr[32];
          tmem_ld_32x32b_x32(t_row + c * 32, rr);
          tmem_wait_ld();
          const int f0 = nt * kBN + c * 32;
          if (row < rows_valid && f0 < p.N) {
            __nv_bfloat16* dst = p.out + (int64_t)prow * p.N + f0;
            uint32_t packed[16];
#pragma unroll
            for (int t = 0; t < 32; t += 2) {
              float a = __uint_as_float(rr[t]), b = __uint_as_float(rr[t + 1]);
              if (p.bias != nullptr) {
                a += __bfloat162float(p.bias[(int64_t)e * p.N + f0 + t]);
                b += __bfloat162float(p.bias[(int64_t)e * p.N + f0 + t + 1]);
              }
              packed[t / 2] = pack_bf16x2(a * rw, b * rw);
            }
#pragma unroll
            for (int q = 0; q < 4; ++q)
              *reinterpret_cast<uint4*>(dst + q * 8) =
                  make_uint4(packed[q * 4], packed[q * 4 + 1], packed[q * 4 + 2], packed[q * 4 + 3]);
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
    tmem_dealloc(tmem_base, 2 * kBN);
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

void moe_align_launch(const int32_t* experts, int n_assign, int E, int e_lo, int e_cnt, int32_t* meta,
                      int32_t* tiles, int max_tiles, int32_t* perm, int32_t* inv, int32_t* cursor, cudaStream_t st) {
  launch_pdl(moe::moe_align_kernel, dim3(1), dim3(1024), 0, st, experts, n_assign, E, e_lo, e_cnt, meta, tiles,
             max_tiles, perm, inv, cursor);
}

void moe_gather_launch(const void* x, int64_t H, const int32_t* perm, const int32_t* meta, int E, int k,
                       int max_rows, void* out, cudaStream_t st) {
  if (max_rows == 0) return;
  launch_pdl(moe::gather_rows_kernel, dim3(std::min(max_rows, 148 * 8)), dim3(128), 0, st,
             reinterpret_cast<const uint4*>(x), H / 8, perm, meta, E, k, reinterpret_cast<uint4*>(out));
}

void moe_combine_launch(const void* rows, const int32_t* inv, int T, int k, int64_t H, void* out, int accumulate,
                        cudaStream_t st) {
  if (T == 0) return;
  launch_pdl(moe::combine_kernel, dim3(T), dim3(128), 0, st, reinterpret_cast<const __nv_bfloat16*>(rows), inv, k, H,
             reinterpret_cast<__nv_bfloat16*>(out), accumulate);
}

void moe_gemm_launch(const MoeGemmArgs& a, cudaStream_t st) {
  using namespace moe;
  if (a.K % kBK != 0 || a.N % 32 != 0 || (a.swiglu && a.N % kBN != 0))
    throw std::runtime_error("b200.moe_gemm: K % 64, N % 32 (N % 128 for gate/up) required");
  CUtensorMap ta = make_tmap_2d(a.x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.rows, a.K, a.K, kBM, kBK);
  // packed weights viewed as bytes [E * N, K / 2], box [128 rows][32 bytes], no swizzle
  CUtensorMap tp = make_tmap_2d(a.blocks, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)a.E * a.N, a.K / 2, a.K / 2,
                                kBN, kBK / 2, CU_TENSOR_MAP_SWIZZLE_NONE);
  MoeParams p{};
  p.meta = a.meta;
  p.tiles = a.tiles;
  p.E = a.E;
  p.N = a.N;
  p.K = a.K;
  p.scales = reinterpret_cast<const uint8_t*>(a.scales);
  p.bias = reinterpret_cast<const __nv_bfloat16*>(a.bias);
  p.row_weight = a.row_weight;
  p.perm = a.perm;
  p.out = reinterpret_cast<__nv_bfloat16*>(a.out);
  p.limit = a.limit;
  p.alpha = a.alpha;
  p.status = a.status;
  const int grid = num_sms(a.device);
  if (a.swiglu) {
    auto k = moe_gemm_kernel<MOE_SWIGLU_CLAMP>;
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
    launch_pdl(k, dim3(grid), dim3(kThreads), kSmem, st, ta, tp, p);
  } else {
    auto k = moe_gemm_kernel<MOE_DOWN>;
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
    launch_pdl(k, dim3(grid), dim3(kThreads), kSmem, st, ta, tp, p);
  }
}

}  // namespace b200
