// Vocab-parallel greedy token choice over NVLink peer memory (no NCCL).
//
// Under tensor parallelism every rank holds the logits of its vocabulary shard
// [R, V / world]. One kernel per rank: CTA r takes the (value, index) argmax
// of row r over its shard and stores it, packed into one 64-bit key, into this
// rank's pair buffer (parity = epoch & 1); the last CTA to finish announces the
// epoch in every rank's flag[rank] (release, system scope); every CTA then
// waits for all ranks' flags, reads row r's key from every rank's buffer over
// NVLink and keeps the largest. All ranks compute the same winner, so every
// rank samples identical tokens. Ties resolve to the smallest global index,
// like a single argmax over the full vocabulary.
//
// Key: (order-preserving bits of the fp32 value) << 32 | (0xFFFFFFFF - index),
// so one unsigned max compares values first and prefers lower indices.
// Double buffering by epoch parity: a rank overwrites a parity's pairs two
// steps later, after every peer passed the intervening step's flag wait, i.e.
// after every peer finished reading them. Waits are bounded (status word).
#include <cfloat>
#include <cstdint>
#include <stdexcept>

#include "../common/b200.cuh"
#include "../common/launch.h"
#include "../common/pdl_launch.h"

namespace b200 {
namespace tps {

constexpr int kThreads = 512;

__device__ __forceinline__ uint32_t ord_f32(float v) {
  const uint32_t u = __float_as_uint(v);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__global__ void __launch_bounds__(kThreads) tp_argmax_kernel(TpArgmaxArgs a) {
  __shared__ unsigned long long red[kThreads / 32];
  pdl_wait();
  pdl_trigger();
  const unsigned e = *reinterpret_cast<volatile unsigned*>(a.epoch) + 1u;
  const int row = blockIdx.x;
  const float* x = a.logits + (int64_t)row * a.ld;
  unsigned long long best = 0ull;
  auto consider = [&](float v, int i) {
    if (v != v) return;  // NaN never wins
    const unsigned long long k =
        ((unsigned long long)ord_f32(v) << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)(a.v_offset + i));
    best = k > best ? k : best;
  };
  if ((a.ld & 3) == 0 && (reinterpret_cast<uintptr_t>(a.logits) & 15) == 0) {
    // 16-byte loads, kUnroll of them in flight per thread before any compare
    constexpr int kUnroll = 4;
    const int nv = a.V_local >> 2;
    const float4* x4 = reinterpret_cast<const float4*>(x);
    for (int base = threadIdx.x; base < nv; base += kThreads * kUnroll) {
      float4 v[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u)
        if (base + u * kThreads < nv) v[u] = __ldg(x4 + base + u * kThreads);
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int j = base + u * kThreads;
        if (j < nv) {
          consider(v[u].x, 4 * j);
          consider(v[u].y, 4 * j + 1);
          consider(v[u].z, 4 * j + 2);
          consider(v[u].w, 4 * j + 3);
        }
      }
    }
    for (int i = (nv << 2) + threadIdx.x; i < a.V_local; i += kThreads) consider(x[i], i);
  } else {
    for (int i = threadIdx.x; i < a.V_local; i += kThreads) consider(x[i], i);
  }
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long ob = __shfl_xor_sync(0xffffffffu, best, o);
    best = ob > best ? ob : best;
  }
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
  __syncthreads();
  const int par = e & 1;
  if (threadIdx.x == 0) {
    unsigned long long b = 0ull;
    for (int w = 0; w < kThreads / 32; ++w) b = red[w] > b ? red[w] : b;
    a.own_pairs[(int64_t)par * a.max_rows + row] = b;
    __threadfence_system();
    // the last CTA to store announces this rank's pairs to every peer
    if (atomicAdd(a.cta_ctr, 1u) == gridDim.x - 1) {
      __threadfence_system();  // one system fence covers every rank's flag store below
      for (int q = 0; q < a.world; ++q) st_relaxed_sys_u32(a.peer_flags[q] + a.rank, e);
    }
  }
  if (threadIdx.x < (unsigned)a.world) wait_flag_geq(a.flags + threadIdx.x, e, a.status, 600 + threadIdx.x);
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long kq[8], b = 0ull;
#pragma unroll
    for (int q = 0; q < 8; ++q)  // every rank's key requested before any is compared
      if (q < a.world) kq[q] = __ldcg(a.peer_pairs[q] + (int64_t)par * a.max_rows + row);
#pragma unroll
    for (int q = 0; q < 8; ++q)
      if (q < a.world) b = kq[q] > b ? kq[q] : b;
    a.out[row] = (int32_t)(0xFFFFFFFFu - (uint32_t)(b & 0xFFFFFFFFull));
    __threadfence();
    // the last CTA to finish resets the arrival counter and publishes the epoch
    if (atomicAdd(a.cta_ctr + 1, 1u) == gridDim.x - 1) {
      a.cta_ctr[0] = 0;
      a.cta_ctr[1] = 0;
      __threadfence();
      *reinterpret_cast<volatile unsigned*>(a.epoch) = e;
    }
  }
}

}  // namespace tps

void tp_argmax_launch(const TpArgmaxArgs& a, cudaStream_t st) {
  if (a.R <= 0) return;
  if (a.R > a.max_rows) throw std::runtime_error("b200.tp_argmax: more rows than the pair buffers hold");
  if (a.world > 8) throw std::runtime_error("b200.tp_argmax: at most 8 ranks");
  launch_pdl(tps::tp_argmax_kernel, dim3((unsigned)a.R), dim3(tps::kThreads), 0, st, a);
}

}  // namespace b200
