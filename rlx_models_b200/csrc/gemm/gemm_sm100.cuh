// Persistent, warp-specialized tcgen05 BF16 GEMM for sm_100a.
//
//   D[i, j] = alpha * sum_k A[i, k] * B[j, k]      (A: [MA, K], B: [NB, K], both K-major)
//
// followed by a fused epilogue (bias, residual add, SwiGLU pairing, bf16/f32
// store, split-K reduction). This is the dense-linear kernel ("K1") behind every
// projection of the decoder families; the reference emits the same op as a
// graph MatMul lowered to a library GEMM (rlx-models-core
// src/standard_decoder.rs:727 `emit_proj`).
//
// Roles (192 threads, one CTA per SM, grid = min(work units, #SMs)):
//   warp 0      TMA producer: one elected lane streams A/B k-tiles into a
//               STAGES-deep shared-memory ring (128-byte swizzle) using
//               cp.async.bulk.tensor (no multicast) + mbarrier complete_tx.
//   warp 1      MMA issuer: one elected lane issues tcgen05.mma (M=128, N=BN,
//               K=16) into a double-buffered TMEM accumulator and releases each
//               smem stage with tcgen05.commit.
//   warps 2..5  epilogue: tcgen05.ld 32x32b from TMEM -> registers -> fused
//               epilogue -> global, overlapping the next tile's MMAs.
//
// Split-K (used for skinny GEMMs so that all SMs stream weights): each split
// stores its fp32 partial tile into its own workspace slice (L2); the last
// split of a tile (per-tile semaphore) sums the slices in split order, runs the
// real epilogue and resets the semaphore. The fixed order keeps the result
// independent of which split finished first (eager and graph-replayed runs,
// and repeated runs, give the same bits).
#pragma once

#include "../common/b200.cuh"

namespace b200 {
namespace gemm {

// EPI_ACC (swap-AB only): accumulate-only split-K. Every unit adds its fp32
// partial into the caller's [tokens][features] buffer with vector red.add and
// leaves; there is no semaphore and no last-CTA tail. The consumer kernel
// (add+RMSNorm, QK-norm/RoPE, SwiGLU) reads the sum and writes zeros back.
enum Epi : int { EPI_BF16 = 0, EPI_F32 = 1, EPI_SWIGLU = 2, EPI_ACC = 3 };

struct Params {
  int MA, NB, K;
  int k_tiles, splits, kt_per_split;
  int num_m, num_n, num_units;
  void* C;
  int64_t ldc_i, ldc_j;
  const __nv_bfloat16* R;
  int64_t ldr_i, ldr_j;
  const __nv_bfloat16* bias;
  int bias_on_i;
  float alpha;
  int swiglu_on_i;
  int w_is_a;  // 1: A is the weight operand (swap-AB), 0: B is
  int accumulate;  // EPI_F32: C += result (gradient accumulation)
  int prefetch_w;  // 1: the weight operand may be loaded before griddepcontrol.wait
  float* ws;
  int* sem;
  int* status;
  // Reduce-scatter push mode (tensor parallel). When peer_out != nullptr,
  // output row `t` (a token) is written to rank owner = t / rpr, into slot
  // `my_rank` of that rank's receive buffer: peer_out[owner] + my_rank *
  // slot_elems + (t % rpr) * ldc. After the last tile, the last CTA writes
  // epoch+1 into peer_flags[q][my_rank] of every rank q (release, system
  // scope), so owners know when all partials for this op have landed.
  void* const* peer_out;
  int rpr;
  int64_t slot_elems;
  int my_rank, world;
  const unsigned* epoch;
  unsigned* done_ctr;
  unsigned* const* peer_flags;
  int bcast;  // push every output row to all ranks (one-shot all-reduce slots) instead of its owner
  unsigned long long* trace;  // optional per-CTA timeline ([grid][16] globaltimer ns), debug only
  // Normal orientation only (adaLN DiT blocks):
  //   act = 1: GELU (tanh form), 2: ReLU, on output columns j >= act_from, after the bias;
  //   gate != null: y = gate[batch(i)][j] * y before the residual is added, with
  //   batch(i) = g < gate_split ? g / gate_r1 : (g - gate_split) / gate_r2 with g = i + gate_off.
  int act, act_from;
  int glu_act;  // EPI_SWIGLU gate activation: 0 SiLU (SwiGLU), 1 GELU tanh form (GeGLU)
  const __nv_bfloat16* gate;
  int64_t gate_ld;
  int gate_split, gate_r1, gate_r2, gate_off;
  // FSDP gradient reduce-scatter push (EPI_F32, normal orientation). When
  // shard_peer != nullptr, output element (i, j) is the gradient of flat
  // parameter shard_base + i * ldc_i + j; it is added (red.add, fp32) into
  // the owning rank's gradient shard shard_peer[idx / shard_n] at idx %
  // shard_n, over NVLink for remote owners. C is not written.
  float* const* shard_peer;
  int64_t shard_base, shard_n;
};

__device__ __forceinline__ float gelu_tanh(float x) {
  // 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))), tanh from the SFU
  const float u = 0.7978845608028654f * (x + 0.044715f * x * x * x);
  float t;
  asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(u));
  return 0.5f * x * (1.f + t);
}

// Base pointer of output row `t` (a token index), local or pushed to its owner.
template <typename T>
__device__ __forceinline__ T* out_row(const Params& p, int t, int64_t ld) {
  if (p.peer_out == nullptr) return reinterpret_cast<T*>(p.C) + (int64_t)t * ld;
  const int owner = t / p.rpr;
  return reinterpret_cast<T*>(p.peer_out[owner]) + (int64_t)p.my_rank * p.slot_elems + (int64_t)(t - owner * p.rpr) * ld;
}

#define B200_GEMM_TRACE(i) \
  if (p.trace != nullptr) p.trace[blockIdx.x * 16 + (i)] = globaltimer_ns();

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kGroupM = 8;
constexpr int kThreads = 192;

template <int BN>
struct Cfg {
  static constexpr uint32_t A_BYTES = kBM * kBK * 2;
  static constexpr uint32_t B_BYTES = BN * kBK * 2;
  static constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (BN >= 256) ? 4 : (BN >= 128 ? 6 : 8);
  static constexpr uint32_t TMEM_COLS = (2 * BN < 32) ? 32 : 2 * BN;
  static constexpr uint32_t XCHG_BYTES = 32 * 132 * 4;  // swap-AB transpose stage [32 tok][128 feat]
  static constexpr uint32_t SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + XCHG_BYTES + 256;
};

__device__ __forceinline__ void unit_to_tile(const Params& p, int u, int& m_tile, int& n_tile, int& ks, int& tile) {
  ks = u % p.splits;
  tile = u / p.splits;
  const int group_size = kGroupM * p.num_n;
  const int g = tile / group_size;
  const int first_m = g * kGroupM;
  const int gm = min(p.num_m - first_m, kGroupM);
  const int r = tile % group_size;
  m_tile = first_m + r % gm;
  n_tile = r / gm;
}

template <int BN, int EPI>
__device__ __forceinline__ void store_chunk(const Params& p, int i, int j0, float (&v)[32]) {
  if (i >= p.MA) return;
  // scalar-or-vector epilogue for one row i and 32 consecutive j
  float bi = 0.f;
  if (p.bias != nullptr && p.bias_on_i) bi = __bfloat162float(p.bias[i]);
#pragma unroll
  for (int t = 0; t < 32; ++t) {
    float x = v[t] * p.alpha + bi;
    v[t] = x;
  }
  if (p.bias != nullptr && !p.bias_on_i) {
#pragma unroll
    for (int t = 0; t < 32; ++t)
      if (j0 + t < p.NB) v[t] += __bfloat162float(p.bias[j0 + t]);
  }
  const bool full = (j0 + 32 <= p.NB);
  if (p.act != 0 && j0 + 32 > p.act_from) {
#pragma unroll
    for (int t = 0; t < 32; ++t)
      if (j0 + t >= p.act_from) v[t] = p.act == 1 ? gelu_tanh(v[t]) : fmaxf(v[t], 0.f);
  }
  if (p.gate != nullptr) {
    const int gi = i + p.gate_off;
    const int gb = gi < p.gate_split ? gi / p.gate_r1 : (gi - p.gate_split) / p.gate_r2;
    const __nv_bfloat16* g = p.gate + (int64_t)gb * p.gate_ld;
    if (full && ((reinterpret_cast<uintptr_t>(g + j0) & 15u) == 0)) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint4 w = *reinterpret_cast<const uint4*>(g + j0 + q * 8);
        const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          v[q * 8 + 2 * h] *= bf16_lo(ww[h]);
          v[q * 8 + 2 * h + 1] *= bf16_hi(ww[h]);
        }
      }
    } else {
#pragma unroll
      for (int t = 0; t < 32; ++t)
        if (j0 + t < p.NB) v[t] *= __bfloat162float(g[j0 + t]);
    }
  }
  if (p.R != nullptr) {
    const __nv_bfloat16* r = p.R + (int64_t)i * p.ldr_i;
    if (p.ldr_j == 1 && full && ((reinterpret_cast<uintptr_t>(r + j0) & 15u) == 0)) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint4 w = *reinterpret_cast<const uint4*>(r + j0 + q * 8);
        uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          v[q * 8 + 2 * h] += bf16_lo(ww[h]);
          v[q * 8 + 2 * h + 1] += bf16_hi(ww[h]);
        }
      }
    } else {
#pragma unroll
      for (int t = 0; t < 32; ++t)
        if (j0 + t < p.NB) v[t] += __bfloat162float(r[(int64_t)(j0 + t) * p.ldr_j]);
    }
  }
  if (EPI == EPI_F32 && p.shard_peer != nullptr) {
    const int64_t base = p.shard_base + (int64_t)i * p.ldc_i + j0;
    const int64_t own0 = base / p.shard_n;
    if (full && (base & 3) == 0 && base + 31 < (own0 + 1) * p.shard_n) {
      float* d = p.shard_peer[own0] + (base - own0 * p.shard_n);  // one owner for the whole chunk
#pragma unroll
      for (int q = 0; q < 8; ++q) red_add_v4(d + q * 4, v[q * 4], v[q * 4 + 1], v[q * 4 + 2], v[q * 4 + 3]);
    } else {
#pragma unroll
      for (int t = 0; t < 32; ++t)
        if (j0 + t < p.NB) {
          const int64_t idx = base + t;
          const int64_t own = idx / p.shard_n;
          atomicAdd(p.shard_peer[own] + (idx - own * p.shard_n), v[t]);
        }
    }
    return;
  }
  if (EPI == EPI_F32) {
    float* c = out_row<float>(p, i, p.ldc_i);
    if (p.ldc_j == 1 && full && ((reinterpret_cast<uintptr_t>(c + j0) & 15u) == 0)) {
      if (p.accumulate) {
        float4 o[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) o[q] = *reinterpret_cast<const float4*>(c + j0 + q * 4);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          v[q * 4] += o[q].x;
          v[q * 4 + 1] += o[q].y;
          v[q * 4 + 2] += o[q].z;
          v[q * 4 + 3] += o[q].w;
        }
      }
#pragma unroll
      for (int q = 0; q < 8; ++q)
        *reinterpret_cast<float4*>(c + j0 + q * 4) = make_float4(v[q * 4], v[q * 4 + 1], v[q * 4 + 2], v[q * 4 + 3]);
    } else {
#pragma unroll
      for (int t = 0; t < 32; ++t)
        if (j0 + t < p.NB) {
          float* cc = c + (int64_t)(j0 + t) * p.ldc_j;
          *cc = p.accumulate ? *cc + v[t] : v[t];
        }
    }
  } else {
    __nv_bfloat16* c = out_row<__nv_bfloat16>(p, i, p.ldc_i);
    if (p.ldc_j == 1 && full && ((reinterpret_cast<uintptr_t>(c + j0) & 15u) == 0)) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint4 w;
        w.x = pack_bf16x2(v[q * 8 + 0], v[q * 8 + 1]);
        w.y = pack_bf16x2(v[q * 8 + 2], v[q * 8 + 3]);
        w.z = pack_bf16x2(v[q * 8 + 4], v[q * 8 + 5]);
        w.w = pack_bf16x2(v[q * 8 + 6], v[q * 8 + 7]);
        *reinterpret_cast<uint4*>(c + j0 + q * 8) = w;
      }
    } else {
#pragma unroll
      for (int t = 0; t < 32; ++t)
        if (j0 + t < p.NB) c[(int64_t)(j0 + t) * p.ldc_j] = __float2bfloat16(v[t]);
    }
  }
}

__device__ __forceinline__ float silu_mul(float g, float u) { return g / (1.f + __expf(-g)) * u; }
__device__ __forceinline__ float glu_mul(float g, float u, int act) { return act ? gelu_tanh(g) * u : silu_mul(g, u); }

// Swap-AB output: token j, NV consecutive features [fo, fo + NV) of one lane
// (the lanes of a warp cover one token's features contiguously).
template <int EPI, int NV>
__device__ __forceinline__ void store_vec(const Params& p, int j, int fo, int nfeat, float (&o)[4]) {
  if (fo >= nfeat) return;
  const bool full = fo + NV <= nfeat;
  if (p.bias != nullptr) {
#pragma unroll
    for (int t = 0; t < NV; ++t)
      if (fo + t < nfeat) o[t] += __bfloat162float(p.bias[fo + t]);
  }
  if (p.act != 0) {
#pragma unroll
    for (int t = 0; t < NV; ++t)
      if (fo + t >= p.act_from) o[t] = p.act == 1 ? gelu_tanh(o[t]) : fmaxf(o[t], 0.f);
  }
  if (p.gate != nullptr) {
    const int gj = j + p.gate_off;
    const int gb = gj < p.gate_split ? gj / p.gate_r1 : (gj - p.gate_split) / p.gate_r2;
#pragma unroll
    for (int t = 0; t < NV; ++t)
      if (fo + t < nfeat) o[t] *= __bfloat162float(p.gate[(int64_t)gb * p.gate_ld + fo + t]);
  }
  if (p.R != nullptr) {
    const __nv_bfloat16* r = p.R + (int64_t)j * p.ldr_j + fo;
    if (NV == 4 && full && ((reinterpret_cast<uintptr_t>(r) & 7u) == 0)) {
      const uint2 w = *reinterpret_cast<const uint2*>(r);
      o[0] += bf16_lo(w.x);
      o[1] += bf16_hi(w.x);
      o[2] += bf16_lo(w.y);
      o[3] += bf16_hi(w.y);
    } else {
#pragma unroll
      for (int t = 0; t < NV; ++t)
        if (fo + t < nfeat) o[t] += __bfloat162float(r[t]);
    }
  }
  if (EPI == EPI_F32) {
    float* c = out_row<float>(p, j, p.ldc_j) + fo;
    if (NV == 4 && full && ((reinterpret_cast<uintptr_t>(c) & 15u) == 0)) {
      *reinterpret_cast<float4*>(c) = make_float4(o[0], o[1], o[2], o[3]);
    } else {
#pragma unroll
      for (int t = 0; t < NV; ++t)
        if (fo + t < nfeat) c[t] = o[t];
    }
  } else {
    const int nq = p.bcast ? p.world : 1;
    for (int q = 0; q < nq; ++q) {
      __nv_bfloat16* c =
          (p.bcast ? reinterpret_cast<__nv_bfloat16*>(p.peer_out[q]) + (int64_t)p.my_rank * p.slot_elems +
                         (int64_t)j * p.ldc_j
                   : out_row<__nv_bfloat16>(p, j, p.ldc_j)) +
          fo;
      if (full && NV == 4 && ((reinterpret_cast<uintptr_t>(c) & 7u) == 0)) {
        *reinterpret_cast<uint2*>(c) = make_uint2(pack_bf16x2(o[0], o[1]), pack_bf16x2(o[2], o[3]));
      } else if (full && NV == 2 && ((reinterpret_cast<uintptr_t>(c) & 3u) == 0)) {
        *reinterpret_cast<uint32_t*>(c) = pack_bf16x2(o[0], o[1]);
      } else {
#pragma unroll
        for (int t = 0; t < NV; ++t)
          if (fo + t < nfeat) c[t] = __float2bfloat16(o[t]);
      }
    }
  }
}

// Operand tiles: K-major -> one TMA box [rows][64 k] (128-byte rows);
// MN-major (the matrix is stored [K][rows], rows contiguous) -> rows/64 boxes
// of [64 k][64 rows], each 8 KB, whose UMMA descriptor strides are LBO = 8 KB
// (next 64 rows) and SBO = 1 KB (next 8 k), advancing 2 KB per K=16 step.
template <bool MN, int ROWS>
__device__ __forceinline__ void load_operand(uint8_t* dst, const CUtensorMap* tm, uint64_t* bar, int kt, int row0) {
  if (!MN) {
    tma_load_2d(dst, tm, bar, kt * kBK, row0);
  } else {
#pragma unroll
    for (int c = 0; c < ROWS / 64; ++c) tma_load_2d(dst + c * 8192, tm, bar, row0 + c * 64, kt * kBK);
  }
}

template <bool MN>
__device__ __forceinline__ uint64_t operand_desc(uint32_t base, int kk) {
  return MN ? umma_desc_sw128(base + kk * 2048, 8192, 1024) : umma_desc_sw128(base + kk * 32, 16, 1024);
}

template <int BN, int EPI, bool A_MN = false, bool B_MN = false>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_bf16_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const Params p) {
  using C = Cfg<BN>;
  constexpr int STAGES = C::STAGES;
  extern __shared__ uint8_t smem_dyn[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = smem;
  float* xchg = reinterpret_cast<float*>(smem + STAGES * C::STAGE_BYTES);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * C::STAGE_BYTES + C::XCHG_BYTES);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* accf = bars + 2 * STAGES;
  uint64_t* acce = bars + 2 * STAGES + 2;
  uint64_t* drain = bars + 2 * STAGES + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 5);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* s_last = reinterpret_cast<int*>(tmem_slot + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) B200_GEMM_TRACE(0);

  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&accf[a], 1);
      mbar_init(&acce[a], 4);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == 2) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_trigger();
  if (threadIdx.x == 0) B200_GEMM_TRACE(1);

  if (warp == 0) {
    if (elect_one_sync()) {
      // ---------------- TMA producer ----------------
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued = 0;
      bool ok = true;
      // PDL prologue: the weight operand does not depend on the previous
      // kernel, so the first ring's worth of weight tiles is requested before
      // griddepcontrol.wait; the activation halves of those stages follow it.
      int npre = 0;
      if (p.prefetch_w && (int)blockIdx.x < p.num_units) {
        int m_tile, n_tile, ks, tile;
        unit_to_tile(p, blockIdx.x, m_tile, n_tile, ks, tile);
        const int kb = ks * p.kt_per_split;
        npre = min(STAGES, min(p.k_tiles, kb + p.kt_per_split) - kb);
        for (int q = 0; q < npre; ++q) {
          uint8_t* sa = ring + q * C::STAGE_BYTES;
          mbar_arrive_expect_tx(&full[q], C::STAGE_BYTES);
          if (p.w_is_a) load_operand<A_MN, kBM>(sa, &tmA, &full[q], kb + q, m_tile * kBM);
          else load_operand<B_MN, BN>(sa + C::A_BYTES, &tmB, &full[q], kb + q, n_tile * BN);
        }
      }
      B200_GEMM_TRACE(2);
      pdl_wait();
      B200_GEMM_TRACE(3);
      bool first = true;
      for (int u = blockIdx.x; u < p.num_units && ok; u += gridDim.x) {
        int m_tile, n_tile, ks, tile;
        unit_to_tile(p, u, m_tile, n_tile, ks, tile);
        const int kb = ks * p.kt_per_split;
        const int ke = min(p.k_tiles, kb + p.kt_per_split);
        for (int kt = kb; kt < ke; ++kt) {
          uint8_t* sa = ring + stage * C::STAGE_BYTES;
          uint8_t* sb = sa + C::A_BYTES;
          if (first && kt - kb < npre) {
            // weight half already in flight; issue the activation half
            if (p.w_is_a) load_operand<B_MN, BN>(sb, &tmB, &full[stage], kt, n_tile * BN);
            else load_operand<A_MN, kBM>(sa, &tmA, &full[stage], kt, m_tile * kBM);
          } else {
            if (!mbar_wait(&empty[stage], phase ^ 1, p.status, kErrTimeoutEmpty) || *abort_flag) {
              *abort_flag = 1;
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&full[stage], C::STAGE_BYTES);
            load_operand<A_MN, kBM>(sa, &tmA, &full[stage], kt, m_tile * kBM);
            load_operand<B_MN, BN>(sb, &tmB, &full[stage], kt, n_tile * BN);
          }
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        first = false;
      }
      if (!ok) {
        // Error path: wait (bounded) for the loads this thread put in flight.
        int s = stage;
        uint32_t ph = phase;
        const uint32_t n = issued < (uint32_t)STAGES ? issued : (uint32_t)STAGES;
        for (uint32_t q = 0; q < n; ++q) {
          if (--s < 0) {
            s = STAGES - 1;
            ph ^= 1;
          }
          mbar_wait(&full[s], ph, p.status, kErrTimeoutDrain);
        }
      }
    }
  } else if (warp == 1) {
    if (elect_one_sync()) {
      // ---------------- MMA issuer ----------------
      constexpr uint32_t idesc = umma_idesc_bf16(kBM, BN, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < p.num_units && ok; u += gridDim.x, ++it) {
        int m_tile, n_tile, ks, tile;
        unit_to_tile(p, u, m_tile, n_tile, ks, tile);
        const int kb = ks * p.kt_per_split;
        const int ke = min(p.k_tiles, kb + p.kt_per_split);
        const int acc = it & 1;
        const uint32_t acc_phase = (it >> 1) & 1;
        if (!mbar_wait(&acce[acc], acc_phase ^ 1, p.status, kErrTimeoutAccEmpty) || *abort_flag) {
          *abort_flag = 1;
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kt = kb; kt < ke; ++kt) {
          if (!mbar_wait(&full[stage], phase, p.status, kErrTimeoutFull) || *abort_flag) {
            *abort_flag = 1;
            ok = false;
            break;
          }
          if (it == 0 && kt == kb) B200_GEMM_TRACE(4);
          tc_fence_after();
          const uint32_t a_addr = smem_u32(ring + stage * C::STAGE_BYTES);
          const uint32_t b_addr = a_addr + C::A_BYTES;
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            const uint64_t ad = operand_desc<A_MN>(a_addr, kk);
            const uint64_t bd = operand_desc<B_MN>(b_addr, kk);
            umma_f16(d_tmem, ad, bd, idesc, (kt > kb || kk > 0) ? 1u : 0u);
          }
          umma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (ok) umma_commit(&accf[acc]);
      }
      B200_GEMM_TRACE(5);
      if (!ok) {
        umma_commit(drain);
        mbar_wait(drain, 0, p.status, kErrTimeoutDrain);
      }
    }
  } else {
    // ---------------- Epilogue (warps 2..5) ----------------
    const int quad = warp & 3;  // TMEM lane quadrant this warp may access
    const int row = quad * 32 + lane;
    const int ew = warp - 2;
    const int et = ew * 32 + lane;  // 0..127 epilogue thread id
    pdl_wait();  // residual / workspace / outputs may belong to the previous kernel
    const bool swap_out = (p.ldc_i == 1);
    int it = 0;
    for (int u = blockIdx.x; u < p.num_units; u += gridDim.x, ++it) {
      int m_tile, n_tile, ks, tile;
      unit_to_tile(p, u, m_tile, n_tile, ks, tile);
      const int acc = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      if (!mbar_wait(&accf[acc], acc_phase, p.status, kErrTimeoutAccFull) || *abort_flag) {
        *abort_flag = 1;
        break;
      }
      if (et == 0 && it == 0) B200_GEMM_TRACE(6);
      tc_fence_after();
      const uint32_t t_row = tmem_base + ((uint32_t)(quad * 32) << 16) + acc * BN;
      const int i = m_tile * kBM + row;
      const int jt = n_tile * BN;
      // split-K: each split's fp32 partial of this tile in its own workspace slice
      // [split][tile][kBM][BN]; the last split to arrive sums the slices in split
      // order, so the result does not depend on which split finished first
      const int64_t slice = (int64_t)(p.num_m * p.num_n) * (kBM * BN);
      float* acc_row = p.ws + (int64_t)tile * (kBM * BN) + (int64_t)row * BN;

      if (EPI == EPI_ACC) {
        float* dst = reinterpret_cast<float*>(p.C);
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(t_row + c * 32, r);
          tmem_wait_ld();
#pragma unroll
          for (int t = 0; t < 32; ++t) xchg[t * 132 + row] = __uint_as_float(r[t]);
          named_bar_sync(2, 128);
          // one token per warp-instruction: lane l adds features [4l, 4l+4) -> 512 B contiguous
          const float4* xs = reinterpret_cast<const float4*>(xchg);
          for (int tt = ew; tt < 32; tt += 4) {
            const int j = jt + c * 32 + tt;
            const int f = m_tile * kBM + lane * 4;
            if (j < p.NB && f < p.MA) {
              // local accumulator, or (tensor parallel) the row owner's over NVLink
              float* drow = (p.peer_out != nullptr ? out_row<float>(p, j, p.ldc_j) : dst + (int64_t)j * p.ldc_j) + f;
              const float4 v4 = xs[tt * 33 + lane];
              if (f + 4 <= p.MA) {
                red_add_v4(drow, v4.x * p.alpha, v4.y * p.alpha, v4.z * p.alpha, v4.w * p.alpha);
              } else {
                const float vv[4] = {v4.x, v4.y, v4.z, v4.w};
                for (int t = 0; f + t < p.MA; ++t) atomicAdd(drow + t, vv[t] * p.alpha);
              }
            }
          }
          named_bar_sync(2, 128);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acce[acc]);
        continue;
      }

      if (p.splits > 1) {
        // Store this split's partial into its slice (L2), release TMEM, then
        // count arrivals.
        float* my_row = acc_row + ks * slice;
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(t_row + c * 32, r);
          tmem_wait_ld();
#pragma unroll
          for (int q = 0; q < 8; ++q)
            __stcg(reinterpret_cast<float4*>(my_row + c * 32) + q,
                   make_float4(__uint_as_float(r[q * 4]), __uint_as_float(r[q * 4 + 1]),
                               __uint_as_float(r[q * 4 + 2]), __uint_as_float(r[q * 4 + 3])));
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acce[acc]);
        __threadfence();
        named_bar_sync(1, 128);
        if (et == 0) {
          const int old = atomicAdd(&p.sem[tile], 1);
          *s_last = (old == p.splits - 1) ? 1 : 0;
        }
        named_bar_sync(1, 128);
        if (et == 0 && it == 0) B200_GEMM_TRACE(7);
        if (*s_last == 0) continue;
        __threadfence();
      }

      // Fetch 32 accumulator columns [c*32, c*32+32) of this thread's row.
      auto fetch = [&](int c, float (&v)[32]) {
        if (p.splits > 1) {
#pragma unroll
          for (int t = 0; t < 32; ++t) v[t] = 0.f;
#pragma unroll 1
          for (int sp = 0; sp < p.splits; ++sp) {
            float4 w[8];
#pragma unroll
            for (int q = 0; q < 8; ++q) w[q] = __ldcg(reinterpret_cast<const float4*>(acc_row + sp * slice + c * 32) + q);
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              v[q * 4] += w[q].x;
              v[q * 4 + 1] += w[q].y;
              v[q * 4 + 2] += w[q].z;
              v[q * 4 + 3] += w[q].w;
            }
          }
        } else {
          uint32_t r[32];
          tmem_ld_32x32b_x32(t_row + c * 32, r);
          tmem_wait_ld();
#pragma unroll
          for (int t = 0; t < 32; ++t) v[t] = __uint_as_float(r[t]);
        }
      };

      if (swap_out) {
        // A rows are output features, B rows are tokens: stage [32 tokens][128
        // features] in smem, then write each token's features as 16B vectors.
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          float v[32];
          fetch(c, v);
#pragma unroll
          for (int t = 0; t < 32; ++t) xchg[t * 132 + row] = v[t];
          named_bar_sync(2, 128);
          const int nfeat = (EPI == EPI_SWIGLU) ? p.MA / 2 : p.MA;
          // one token per warp-instruction, contiguous features across the lanes
          for (int tt = ew; tt < 32; tt += 4) {
            const int j = jt + c * 32 + tt;
            if (j >= p.NB) continue;
            if (EPI == EPI_SWIGLU) {
              const int fl = lane * 2;  // 64 outputs per tile: 2 per lane
              const int fo = m_tile * 64 + fl;
              float o[4] = {glu_mul(xchg[tt * 132 + fl] * p.alpha, xchg[tt * 132 + 64 + fl] * p.alpha, p.glu_act),
                            glu_mul(xchg[tt * 132 + fl + 1] * p.alpha, xchg[tt * 132 + 64 + fl + 1] * p.alpha,
                                    p.glu_act),
                            0.f, 0.f};
              store_vec<EPI, 2>(p, j, fo, nfeat, o);
            } else {
              const int fl = lane * 4;
              const int fo = m_tile * kBM + fl;
              const float4 v4 = reinterpret_cast<const float4*>(xchg)[tt * 33 + lane];
              float o[4] = {v4.x * p.alpha, v4.y * p.alpha, v4.z * p.alpha, v4.w * p.alpha};
              store_vec<EPI, 4>(p, j, fo, nfeat, o);
            }
          }
          named_bar_sync(2, 128);
        }
      } else if (EPI == EPI_SWIGLU) {
        // gate/up interleaved along j in groups of 64 columns: [g*128, g*128+64) gate, +64 up.
#pragma unroll 1
        for (int g = 0; g < BN / 128; ++g) {
#pragma unroll 1
          for (int h = 0; h < 2; ++h) {
            float vg[32], vu[32];
            fetch(g * 4 + h, vg);
            fetch(g * 4 + h + 2, vu);
#pragma unroll
            for (int t = 0; t < 32; ++t) vg[t] = glu_mul(vg[t] * p.alpha, vu[t] * p.alpha, p.glu_act);
            Params q = p;
            q.alpha = 1.f;
            q.NB = p.NB / 2;
            q.bias = nullptr;
            store_chunk<BN, EPI_BF16>(q, i, (jt + g * 128) / 2 + h * 32, vg);
          }
        }
      } else if (EPI == EPI_BF16 && p.peer_out != nullptr) {
        // Reduce-scatter push (remote rows): stage the [128 x 32] chunk in smem
        // so that each store is a 64-byte row segment instead of one 16-byte
        // piece per lane, then write 8 rows per warp instruction.
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          float v[32];
          fetch(c, v);
          const int j0 = jt + c * 32;
#pragma unroll
          for (int t = 0; t < 32; ++t) {
            float x = v[t] * p.alpha;
            if (p.bias != nullptr && j0 + t < p.NB) x += __bfloat162float(p.bias[j0 + t]);
            xchg[row * 33 + t] = x;
          }
          named_bar_sync(2, 128);
#pragma unroll
          for (int st = 0; st < 4; ++st) {
            const int rr = ew * 32 + st * 8 + (lane >> 2);
            const int q = lane & 3;
            const int ii = m_tile * kBM + rr;
            const int jj = j0 + q * 8;
            if (ii < p.MA && jj < p.NB) {
              __nv_bfloat16* cptr = out_row<__nv_bfloat16>(p, ii, p.ldc_i) + jj;
              const float* src = xchg + rr * 33 + q * 8;
              if (jj + 8 <= p.NB && ((reinterpret_cast<uintptr_t>(cptr) & 15u) == 0)) {
                *reinterpret_cast<uint4*>(cptr) = make_uint4(pack_bf16x2(src[0], src[1]), pack_bf16x2(src[2], src[3]),
                                                             pack_bf16x2(src[4], src[5]), pack_bf16x2(src[6], src[7]));
              } else {
                for (int t = 0; t < 8 && jj + t < p.NB; ++t) cptr[t] = __float2bfloat16(src[t]);
              }
            }
          }
          named_bar_sync(2, 128);
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          float v[32];
          fetch(c, v);
          store_chunk<BN, EPI>(p, i, jt + c * 32, v);
        }
      }

      if (p.splits > 1) {
        if (et == 0) p.sem[tile] = 0;
      } else {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acce[acc]);
      }
    }
    if (et == 0) B200_GEMM_TRACE(8);
    if (p.peer_out != nullptr) {
      // Reduce-scatter completion: this CTA's pushes are issued; make them
      // visible at system scope, count CTAs, and let the last one signal
      // every rank (itself included) with this op's epoch.
      __threadfence_system();
      named_bar_sync(1, 128);
      if (et == 0) {
        const unsigned old = atomicAdd(p.done_ctr, 1u);
        if (old == gridDim.x - 1) {
          __threadfence_system();
          const unsigned e = *reinterpret_cast<const volatile unsigned*>(p.epoch) + 1u;
          for (int q = 0; q < p.world; ++q) st_release_sys_u32(p.peer_flags[q] + p.my_rank, e);
          *p.done_ctr = 0;
        }
      }
    }
  }

  __syncthreads();
  if (threadIdx.x == 0) B200_GEMM_TRACE(9);
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

}  // namespace gemm
}  // namespace b200
