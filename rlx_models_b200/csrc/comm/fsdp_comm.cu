// FSDP gradient reduce-scatter by push over NVLink peer memory.
//
// Every rank's gradient shard (fp32, shard_n elements of a parameter group's
// flat buffer) lives in a symmetric IPC heap. Instead of materialising the
// full gradient and calling a collective, each rank ADDS its contribution to
// flat element idx straight into the owner's shard: rank idx / shard_n, offset
// idx % shard_n (red.global.add, fp32, over NVLink for remote owners).
//
//   * weight matrices: the wgrad GEMM's epilogue does the push itself
//     (gemm::Params::shard_peer), tile by tile while the backward pass runs;
//   * everything else (norm weights, embedding / lm_head gradients):
//     shard_push_add below, from the dense gradient autograd produced;
//   * before the optimizer reads its shard, peer_barrier: announce this
//     step's epoch to every rank and wait (bounded) for all of them, so every
//     rank's pushes of this step have landed.
//
// Atomic adds make the sum order run-dependent across ranks (not bitwise
// reproducible at world > 1); with one rank the order is the stream order.
//
// Reference: the reference's ZeRO-1 reduce-scatter is an all-reduce + slice
// over host TCP (crates/rlx-tune/src/distributed.rs:106-123, trainer.rs:1063).
#include <cuda_bf16.h>

#include <algorithm>
#include <stdexcept>

#include "../common/b200.cuh"
#include "../common/launch.h"
#include "../common/pdl_launch.h"

namespace b200 {
namespace fsdpc {

template <typename T>
__device__ __forceinline__ float ld_f(const T* p, int64_t i);
template <>
__device__ __forceinline__ float ld_f<float>(const float* p, int64_t i) { return p[i]; }
template <>
__device__ __forceinline__ float ld_f<__nv_bfloat16>(const __nv_bfloat16* p, int64_t i) {
  return __bfloat162float(p[i]);
}

// dst(flat idx) += src[i] for idx = base + i; vector path when every 4-group
// of flat indices starts on a multiple of 4 (shard_n is a multiple of 4, so a
// group never straddles two owners).
template <typename T>
__global__ void shard_push_add_kernel(const T* __restrict__ src, int64_t n, int64_t base, float* const* peers,
                                      int64_t shard_n, float scale) {
  pdl_wait();
  pdl_trigger();
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  if ((base & 3) == 0) {
    const int64_t n4 = n / 4;
    for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < n4; v += stride) {
      const int64_t idx = base + v * 4;
      const int64_t own = idx / shard_n;
      red_add_v4(peers[own] + (idx - own * shard_n), ld_f(src, v * 4) * scale, ld_f(src, v * 4 + 1) * scale,
                 ld_f(src, v * 4 + 2) * scale, ld_f(src, v * 4 + 3) * scale);
    }
    for (int64_t i = n4 * 4 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
      const int64_t idx = base + i;
      const int64_t own = idx / shard_n;
      atomicAdd(peers[own] + (idx - own * shard_n), ld_f(src, i) * scale);
    }
  } else {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
      const int64_t idx = base + i;
      const int64_t own = idx / shard_n;
      atomicAdd(peers[own] + (idx - own * shard_n), ld_f(src, i) * scale);
    }
  }
}

// One CTA: raise this op's epoch in flags[rank] of every rank, wait until all
// ranks raised it here (bounded; kErrTimeoutPeer on expiry), advance the epoch.
__global__ void peer_barrier_kernel(unsigned* const* peer_flags, const unsigned* flags, unsigned* epoch, int rank,
                                    int world, int* status) {
  pdl_wait();
  pdl_trigger();
  const unsigned e = *reinterpret_cast<volatile unsigned*>(epoch) + 1u;
  __threadfence_system();
  if (threadIdx.x < (unsigned)world) st_release_sys_u32(peer_flags[threadIdx.x] + rank, e);
  if (threadIdx.x < (unsigned)world) wait_flag_geq(flags + threadIdx.x, e, status, 800 + threadIdx.x);
  __syncthreads();
  if (threadIdx.x == 0) *epoch = e;
}

}  // namespace fsdpc

void shard_push_add_launch(const void* src, bool f32, int64_t n, int64_t base, float* const* peers, int64_t shard_n,
                           float scale, cudaStream_t st) {
  if (n == 0) return;
  if (shard_n <= 0 || shard_n % 4 != 0) throw std::runtime_error("b200.shard_push_add: shard_n % 4 required");
  const int threads = 256;
  const int blocks = (int)std::min<int64_t>((n / 4 + threads - 1) / threads + 1, 148 * 8);
  if (f32)
    launch_pdl(fsdpc::shard_push_add_kernel<float>, dim3(blocks), dim3(threads), 0, st,
               reinterpret_cast<const float*>(src), n, base, peers, shard_n, scale);
  else
    launch_pdl(fsdpc::shard_push_add_kernel<__nv_bfloat16>, dim3(blocks), dim3(threads), 0, st,
               reinterpret_cast<const __nv_bfloat16*>(src), n, base, peers, shard_n, scale);
}

void peer_barrier_launch(unsigned* const* peer_flags, const unsigned* flags, unsigned* epoch, int rank, int world,
                         int* status, cudaStream_t st) {
  if (world < 1 || world > 32) throw std::runtime_error("b200.peer_barrier: 1 <= world <= 32");
  launch_pdl(fsdpc::peer_barrier_kernel, dim3(1), dim3(32), 0, st, peer_flags, flags, epoch, rank, world, status);
}

}  // namespace b200
