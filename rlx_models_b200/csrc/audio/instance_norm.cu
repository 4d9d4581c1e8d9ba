// Instance normalisation over the time axis with an "active" prefix ("K18"):
// x [N, C, T] -> y = (x - mean) * rsqrt(var + eps) * gamma[c] + beta[c], with
// mean and (biased) variance taken over the first `active` steps of each
// (n, c) row and applied to all T steps (padding after the active prefix does
// not move the statistics). One CTA per row; fp32 statistics; fp32 or bf16 data.
//
// Reference: the Kitten TTS generator's instance norm
// (crates/kitten_tts_mini_rlx/src/gpu_kernels.rs:1188-1290, one block per row,
// statistics over the active window applied to the whole axis).
#include <cuda_bf16.h>

#include <stdexcept>

#include "../common/b200.cuh"
#include "../common/launch.h"
#include "../common/pdl_launch.h"

namespace b200 {
namespace inorm {

constexpr int kThreads = 256;

template <typename T>
__device__ __forceinline__ float ld(const T* p) { return (float)p[0]; }
template <>
__device__ __forceinline__ float ld<__nv_bfloat16>(const __nv_bfloat16* p) { return __bfloat162float(*p); }
template <typename T>
__device__ __forceinline__ void st(T* p, float v) { *p = (T)v; }
template <>
__device__ __forceinline__ void st<__nv_bfloat16>(__nv_bfloat16* p, float v) { *p = __float2bfloat16(v); }

__device__ __forceinline__ float block_sum(float v, float* sh) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = v;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < kThreads / 32 ? sh[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (threadIdx.x == 0) sh[0] = t;
  }
  __syncthreads();
  return sh[0];
}

template <typename T>
__global__ void __launch_bounds__(kThreads) instance_norm_kernel(const T* __restrict__ x, const float* __restrict__ gamma,
                                                                 const float* __restrict__ beta, T* __restrict__ y,
                                                                 int C, int64_t Tlen, int64_t active, float eps) {
  __shared__ float sh[kThreads / 32];
  pdl_wait();
  pdl_trigger();
  const int64_t row = blockIdx.x;
  const int c = (int)(row % C);
  const T* xr = x + row * Tlen;
  T* yr = y + row * Tlen;
  float s = 0.f;
  for (int64_t j = threadIdx.x; j < active; j += kThreads) s += ld(xr + j);
  const float mean = block_sum(s, sh) / (float)active;
  float v = 0.f;
  for (int64_t j = threadIdx.x; j < active; j += kThreads) {
    const float d = ld(xr + j) - mean;
    v += d * d;
  }
  const float inv = rsqrtf(block_sum(v, sh) / (float)active + eps);
  const float g = gamma != nullptr ? gamma[c] : 1.f, b = beta != nullptr ? beta[c] : 0.f;
  for (int64_t j = threadIdx.x; j < Tlen; j += kThreads) st(yr + j, (ld(xr + j) - mean) * inv * g + b);
}

}  // namespace inorm

void instance_norm_launch(const void* x, const float* gamma, const float* beta, void* y, int64_t N, int C,
                          int64_t T, int64_t active, float eps, bool bf16, cudaStream_t st) {
  if (N * C == 0 || T == 0) return;
  if (active <= 0 || active > T) active = T;
  if (bf16)
    launch_pdl(inorm::instance_norm_kernel<__nv_bfloat16>, dim3((unsigned)(N * C)), dim3(inorm::kThreads), 0, st,
               reinterpret_cast<const __nv_bfloat16*>(x), gamma, beta, reinterpret_cast<__nv_bfloat16*>(y), C, T,
               active, eps);
  else
    launch_pdl(inorm::instance_norm_kernel<float>, dim3((unsigned)(N * C)), dim3(inorm::kThreads), 0, st,
               reinterpret_cast<const float*>(x), gamma, beta, reinterpret_cast<float*>(y), C, T, active, eps);
}

}  // namespace b200
