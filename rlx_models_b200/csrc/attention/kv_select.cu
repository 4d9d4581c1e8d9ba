// KV-block retrieval selection for long-context decode: one CTA per sequence
// scores every block of the sequence's table against the step's query
// (sum over each KV head's query heads of q . block-key-summary), keeps the
// sink and recent-window blocks, picks the top-k older blocks by an exact
// radix select on the score bits, and writes the selected block ids in block
// order plus the matching context length for the paged decode kernel.
//
// Two launches: kv_score_kernel spreads the block scores over many CTAs
// (a GEMV-like pass over the summaries at HBM bandwidth), kv_select_kernel
// (one CTA per sequence) stages them in shared memory (4 W bytes, W <= 49152
// blocks, i.e. 786k tokens) for the selection.
#include <cuda_bf16.h>

#include <cstdint>
#include <stdexcept>

#include "../common/b200.cuh"
#include "../common/launch.h"
#include "../common/pdl_launch.h"

namespace b200 {
namespace kvsel {

constexpr int kThreads = 256;
constexpr int kMaxQ = 4096;  // Hkv * D

__device__ __forceinline__ uint32_t order_key(float f) {
  // monotone map float -> uint32 (larger float -> larger key)
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// exclusive prefix sum of one flag per thread; returns the total in *tot
__device__ __forceinline__ int block_scan(int v, int* tot, int* warp_sums) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_sums[w] = x;
  __syncthreads();
  if (w == 0) {
    int s = lane < kThreads / 32 ? warp_sums[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, s, o);
      if (lane >= o) s += y;
    }
    if (lane < kThreads / 32) warp_sums[lane] = s;  // inclusive per warp
  }
  __syncthreads();
  const int before = (w > 0 ? warp_sums[w - 1] : 0) + x - v;
  *tot = warp_sums[kThreads / 32 - 1];
  __syncthreads();
  return before;
}

// Block scores: grid (B, ceil(W / kBlocksPerCta)); each warp scores blocks of
// the table (its query-sum vector staged in shared memory); blocks past the
// context get -inf.
constexpr int kBlocksPerCta = 32;

__global__ void __launch_bounds__(kThreads) kv_score_kernel(KvSelectArgs a) {
  __shared__ float qs[kMaxQ];
  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.x, t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int HD = a.Hkv * a.D, G = a.Hq / a.Hkv;
  const __nv_bfloat16* q = a.q + (int64_t)b * a.Hq * a.D;
  for (int i = t; i < HD; i += kThreads) {
    const int h = i / a.D, d = i % a.D;
    float s = 0.f;
    for (int g = 0; g < G; ++g) s += __bfloat162float(q[(h * G + g) * a.D + d]);
    qs[i] = s;
  }
  __syncthreads();
  const int nblk = (a.ctx[b] + 15) / 16;
  const int32_t* tab = a.tables + (int64_t)b * a.W;
  const int w0 = blockIdx.y * kBlocksPerCta;
  for (int w = w0 + warp; w < min(a.W, w0 + kBlocksPerCta); w += kThreads / 32) {
    float s = -INFINITY;
    if (w < nblk) {
      s = 0.f;
      const __nv_bfloat16* sm = a.summ + (int64_t)tab[w] * HD;
      for (int i = lane * 8; i < HD; i += 256) {
        const uint4 v = *reinterpret_cast<const uint4*>(sm + i);
        const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = __bfloat1622float2(p[j]);
          s += f.x * qs[i + 2 * j] + f.y * qs[i + 2 * j + 1];
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    }
    if (lane == 0) a.scores[(int64_t)b * a.W + w] = s;
  }
}

// Block key summaries of the blocks written this step: summ[blk] = mean of
// the block's 16 key rows per KV head (grid: one CTA per token of the step;
// tokens of the same block write the same values).
__global__ void kv_summary_kernel(const __nv_bfloat16* __restrict__ k_cache, const int64_t* __restrict__ slots,
                                  __nv_bfloat16* __restrict__ summ, int Hkv, int D) {
  pdl_wait();
  pdl_trigger();
  const int64_t blk = slots[blockIdx.x] >> 4;
  const __nv_bfloat16* src = k_cache + blk * Hkv * 16 * D;
  __nv_bfloat16* dst = summ + blk * Hkv * D;
  for (int i = threadIdx.x; i < Hkv * D; i += blockDim.x) {
    const int h = i / D, d = i % D;
    float s = 0.f;
#pragma unroll
    for (int r = 0; r < 16; ++r) s += __bfloat162float(src[(int64_t)(h * 16 + r) * D + d]);
    dst[i] = __float2bfloat16(s * (1.f / 16.f));
  }
}

__global__ void __launch_bounds__(kThreads) kv_select_kernel(KvSelectArgs a) {
  extern __shared__ float sc[];  // [W] scores
  __shared__ unsigned hist[256];
  __shared__ int warp_sums[kThreads / 32];
  __shared__ uint32_t s_prefix;
  __shared__ int s_need;
  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.x, t = threadIdx.x;
  const int ctx = a.ctx[b];
  const int nblk = (ctx + 15) / 16;
  const int32_t* tab = a.tables + (int64_t)b * a.W;
  // 1. the scores from kv_score_kernel
  for (int w = t; w < nblk; w += kThreads) sc[w] = a.scores[(int64_t)b * a.W + w];
  __syncthreads();
  auto kept = [&](int w) { return w < nblk && (w < a.sink || w >= nblk - a.window); };
  auto cand = [&](int w) { return w < nblk && !(w < a.sink || w >= nblk - a.window); };
  const int lo_end = min(a.sink, nblk), hi_start = max(nblk - a.window, lo_end);
  const int n_keep = lo_end + (nblk - hi_start);
  const int n_cand = nblk - n_keep;
  const int k = min(a.topk, n_cand);
  // 2. radix select: the k-th largest candidate key (all candidates when k == n_cand)
  uint32_t thr = 0;  // take candidates with key > thr, plus `need` of those equal to thr (in block order)
  int need = 0;
  if (k > 0 && k < n_cand) {
    if (t == 0) {
      s_prefix = 0;
      s_need = k;
    }
    __syncthreads();
    for (int shift = 24; shift >= 0; shift -= 8) {
      for (int i = t; i < 256; i += kThreads) hist[i] = 0;
      __syncthreads();
      const uint32_t pre = s_prefix;
      const uint32_t mask_hi = shift == 24 ? 0u : (0xffffffffu << (shift + 8));
      for (int w = t; w < nblk; w += kThreads) {
        if (!cand(w)) continue;
        const uint32_t key = order_key(sc[w]);
        if ((key & mask_hi) == (pre & mask_hi)) atomicAdd(&hist[(key >> shift) & 255u], 1u);
      }
      __syncthreads();
      if (t == 0) {
        int rem = s_need;
        int bin = 255;
        for (; bin > 0; --bin) {
          if ((int)hist[bin] >= rem) break;
          rem -= (int)hist[bin];
        }
        s_prefix = pre | ((uint32_t)bin << shift);
        s_need = rem;
      }
      __syncthreads();
    }
    thr = s_prefix;
    need = s_need;  // ties at thr to take
  }
  // 3. ordered output: kept blocks, candidates above the threshold, the first `need` ties
  int taken = 0, ties_taken = 0;
  for (int base = 0; base < nblk; base += kThreads) {
    const int w = base + t;
    int take = 0, tie = 0;
    if (w < nblk) {
      if (kept(w)) {
        take = 1;
      } else if (k > 0) {
        if (k == n_cand) {
          take = 1;
        } else {
          const uint32_t key = order_key(sc[w]);
          if (key > thr) take = 1;
          else if (key == thr) tie = 1;
        }
      }
    }
    int tot_tie;
    const int tie_rank = block_scan(tie, &tot_tie, warp_sums);
    if (tie && ties_taken + tie_rank < need) take = 1;
    ties_taken += tot_tie;
    int tot;
    const int pos = block_scan(take, &tot, warp_sums);
    if (take && taken + pos < a.budget) a.sel[(int64_t)b * a.budget + taken + pos] = tab[w];
    taken += tot;
  }
  for (int i = taken + t; i < a.budget; i += kThreads) a.sel[(int64_t)b * a.budget + i] = 0;  // beyond sel_ctx
  if (t == 0) a.sel_ctx[b] = nblk == 0 ? 0 : (min(taken, a.budget) - 1) * 16 + (ctx - (nblk - 1) * 16);
}

}  // namespace kvsel

void kv_select_launch(const KvSelectArgs& a, cudaStream_t st) {
  if (a.B == 0) return;
  if (a.Hkv * a.D > kvsel::kMaxQ || (a.Hkv * a.D) % 8 != 0)
    throw std::runtime_error("b200.kv_select: Hkv * head_dim must be a multiple of 8 and <= 4096");
  if (a.window < 1) throw std::runtime_error("b200.kv_select: the recent window must hold at least one block");
  const size_t smem = (size_t)a.W * sizeof(float);
  if (smem > 196608) throw std::runtime_error("b200.kv_select: block table too wide (W > 49152)");
  ensure_smem(kvsel::kv_select_kernel, 196608);
  launch_pdl(kvsel::kv_score_kernel, dim3(a.B, (a.W + kvsel::kBlocksPerCta - 1) / kvsel::kBlocksPerCta),
             dim3(kvsel::kThreads), 0, st, a);
  launch_pdl(kvsel::kv_select_kernel, dim3(a.B), dim3(kvsel::kThreads), smem, st, a);
}

void kv_summary_launch(const void* k_cache, const int64_t* slots, int64_t T, void* summ, int Hkv, int D,
                       cudaStream_t st) {
  if (T == 0) return;
  launch_pdl(kvsel::kv_summary_kernel, dim3((unsigned)T), dim3(128), 0, st,
             reinterpret_cast<const __nv_bfloat16*>(k_cache), slots, reinterpret_cast<__nv_bfloat16*>(summ), Hkv,
             D);
}

}  // namespace b200
