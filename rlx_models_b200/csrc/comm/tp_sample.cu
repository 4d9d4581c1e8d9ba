// Vocab-parallel greedy token choice over NVLink peer memory (no NCCL, no
// flags, no fences).
//
// Under tensor parallelism every rank holds the logits of its vocabulary shard
// [R, V / world]. One kernel per rank, CTA r on row r: the (value, index) argmax
// of the row over the shard is packed into one self-validating 64-bit key and
// stored into slot [parity][r][rank] of EVERY rank's key buffer (relaxed
// system-scope stores over NVLink); then lanes q < world poll this rank's own
// slots [parity][r][q] until each carries this op's tag, take the largest key,
// and clear the slots. All ranks compute the same winner, so every rank samples
// identical tokens; ties resolve to the smallest global index, like a single
// argmax over the full vocabulary.
//
// Key bits: [63:32] order-preserving bits of the fp32 value, [31:13]
// (kIdxMask - global index), [12:0] tag = 1 + epoch % 8191 (never 0). A key is
// written with one aligned 8-byte store, so a reader sees either the old word
// or the whole new key: the tag is the "data ready" flag, and no flag store,
// fence or second barrier is needed. Slots are double-buffered by epoch parity
// and cleared by their reader: a rank writes parity p again two ops later, after
// it received every peer's key of the op in between, which each peer pushed
// only after its previous op (and its reads and clears of parity p) completed.
// Waits are bounded (status word). Vocabulary: global ids < 2^19.
#include <cfloat>
#include <cstdint>
#include <stdexcept>

#include "../common/b200.cuh"
#include "../common/launch.h"
#include "../common/pdl_launch.h"

namespace b200 {
namespace tps {

constexpr int kThreads = 512;
constexpr uint32_t kIdxBits = 19, kTagBits = 13;
constexpr uint32_t kIdxMask = (1u << kIdxBits) - 1u, kTagMask = (1u << kTagBits) - 1u;

__device__ __forceinline__ uint32_t ord_f32(float v) {
  const uint32_t u = __float_as_uint(v);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ void st_relaxed_sys_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(kThreads) tp_argmax_kernel(TpArgmaxArgs a) {
  __shared__ unsigned long long red[kThreads / 32];
  pdl_wait();
  pdl_trigger();
  const unsigned e = *reinterpret_cast<volatile unsigned*>(a.epoch) + 1u;
  const uint32_t tag = 1u + e % kTagMask;
  const int row = blockIdx.x;
  const float* x = a.logits + (int64_t)row * a.ld;
  // best (value, smallest index) as ord(value) << 32 | (kIdxMask - local index)
  unsigned long long best = 0ull;
  auto consider = [&](float v, int i) {
    if (v != v) return;  // NaN never wins
    const unsigned long long k = ((unsigned long long)ord_f32(v) << 32) | (unsigned long long)(kIdxMask - (uint32_t)i);
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
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    unsigned long long b = lane < kThreads / 32 ? red[lane] : 0ull;
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long ob = __shfl_xor_sync(0xffffffffu, b, o);
      b = ob > b ? ob : b;
    }
    // local index -> global index, then the packed key with this op's tag
    const uint32_t li = kIdxMask - (uint32_t)(b & kIdxMask);
    const uint32_t gi = b ? (uint32_t)a.v_offset + li : kIdxMask;  // an all-NaN shard never wins
    const unsigned long long key =
        (b & 0xFFFFFFFF00000000ull) | ((unsigned long long)((kIdxMask - gi) & kIdxMask) << kTagBits) | tag;
    const int64_t slot = ((int64_t)(e & 1) * a.max_rows + row) * a.world;
    if (lane < a.world) st_relaxed_sys_u64(a.peer_pairs[lane] + slot + a.rank, key);
    unsigned long long got = 0ull;
    bool ok = true;
    if (lane < a.world) {
      const unsigned long long* mine = a.own_pairs + slot + lane;
      got = ld_relaxed_sys_u64(mine);
      if ((uint32_t)(got & kTagMask) != tag) {
        const unsigned long long t0 = globaltimer_ns();
        for (uint32_t i = 0;; ++i) {
          got = ld_relaxed_sys_u64(mine);
          if ((uint32_t)(got & kTagMask) == tag) break;
          if ((i & 63u) == 63u) {
            __nanosleep(64);
            if (globaltimer_ns() - t0 > kWaitTimeoutNs) {
              report_error(a.status, kErrTimeoutPeer, 600 + lane);
              ok = false;
              got = 0ull;
              break;
            }
          }
        }
      }
      if (ok) a.own_pairs[slot + lane] = 0ull;  // consumed: tag 0 never matches
    }
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long ob = __shfl_xor_sync(0xffffffffu, got, o);
      got = ob > got ? ob : got;
    }
    if (lane == 0) {
      a.out[row] = (int32_t)(kIdxMask - (uint32_t)((got >> kTagBits) & kIdxMask));
      __threadfence();
      // the last CTA to finish publishes the epoch for the next op
      if (atomicAdd(a.cta_ctr, 1u) == gridDim.x - 1) {
        a.cta_ctr[0] = 0;
        __threadfence();
        *reinterpret_cast<volatile unsigned*>(a.epoch) = e;
      }
    }
  }
}

}  // namespace tps

void tp_argmax_launch(const TpArgmaxArgs& a, cudaStream_t st) {
  if (a.R <= 0) return;
  if (a.R > a.max_rows) throw std::runtime_error("b200.tp_argmax: more rows than the key buffers hold");
  if (a.world > 8) throw std::runtime_error("b200.tp_argmax: at most 8 ranks");
  if ((int64_t)a.v_offset + a.V_local > (int64_t)tps::kIdxMask)
    throw std::runtime_error("b200.tp_argmax: vocabulary ids must stay below 2^19 - 1");
  launch_pdl(tps::tp_argmax_kernel, dim3((unsigned)a.R), dim3(tps::kThreads), 0, st, a);
}

}  // namespace b200
