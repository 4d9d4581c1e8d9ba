// Training kernels: fused AdamW on flat fp32 shards ("K16"), gradient
// sum-of-squares for global-norm clipping ("K17"), and softmax
// cross-entropy forward + backward on a logits chunk ("K15").
//
// AdamW follows the decoupled-weight-decay update the reference trainer
// applies (rlx-tune src/trainer.rs:26-130 Adam, :273-320 AdamConfig):
//   m = b1 m + (1 - b1) g,  v = b2 v + (1 - b2) g^2,
//   p -= lr * (m / (1 - b1^t) / (sqrt(v / (1 - b2^t)) + eps) + wd * p)
// with g = grad * grad_scale (grad_scale folds in the clipping coefficient and
// any 1/accumulation factor). It reads the bf16 or fp32 gradient shard once,
// updates the fp32 master and both moments in place and writes the bf16
// parameter shard that the next FSDP all-gather sends (cast fused).
#include <cuda_bf16.h>

#include <algorithm>
#include <stdexcept>

#include "../common/b200.cuh"
#include "../common/launch.h"
#include "../common/pdl_launch.h"

namespace b200 {

template <typename G>
__device__ __forceinline__ float gload(const G* g, int64_t i);
template <>
__device__ __forceinline__ float gload<float>(const float* g, int64_t i) {
  return g[i];
}
template <>
__device__ __forceinline__ float gload<__nv_bfloat16>(const __nv_bfloat16* g, int64_t i) {
  return __bfloat162float(g[i]);
}

template <typename G>
__global__ void adamw_kernel(float* __restrict__ master, const G* __restrict__ grad, float* __restrict__ m,
                             float* __restrict__ v, __nv_bfloat16* __restrict__ param_out, int64_t n, float lr,
                             float b1, float b2, float eps, float wd, float bc1, float bc2, const float* scale_ptr,
                             float scale) {
  pdl_wait();
  pdl_trigger();
  const float gs = scale * (scale_ptr ? *scale_ptr : 1.f);
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    const float g = gload<G>(grad, i) * gs;
    float mi = m[i], vi = v[i], p = master[i];
    mi = b1 * mi + (1.f - b1) * g;
    vi = b2 * vi + (1.f - b2) * g * g;
    const float mh = mi / bc1;
    const float vh = vi / bc2;
    p -= lr * (mh / (sqrtf(vh) + eps) + wd * p);
    m[i] = mi;
    v[i] = vi;
    master[i] = p;
    if (param_out != nullptr) param_out[i] = __float2bfloat16(p);
  }
}

void adamw_launch(float* master, const void* grad, bool grad_f32, float* m, float* v, void* param_out, int64_t n,
                  float lr, float b1, float b2, float eps, float wd, int64_t step, const float* scale_ptr,
                  float scale, cudaStream_t st) {
  if (n == 0) return;
  const float bc1 = 1.f - powf(b1, (float)step);
  const float bc2 = 1.f - powf(b2, (float)step);
  const int threads = 256;
  const int blocks = (int)std::min<int64_t>((n + threads - 1) / threads, 148 * 16);
  auto po = reinterpret_cast<__nv_bfloat16*>(param_out);
  if (grad_f32)
    launch_pdl(adamw_kernel<float>, dim3(blocks), dim3(threads), 0, st, master,
               reinterpret_cast<const float*>(grad), m, v, po, n, lr, b1, b2, eps, wd, bc1, bc2, scale_ptr, scale);
  else
    launch_pdl(adamw_kernel<__nv_bfloat16>, dim3(blocks), dim3(threads), 0, st, master,
               reinterpret_cast<const __nv_bfloat16*>(grad), m, v, po, n, lr, b1, b2, eps, wd, bc1, bc2, scale_ptr,
               scale);
}

template <typename G>
__global__ void sumsq_kernel(const G* __restrict__ g, int64_t n, float* __restrict__ out) {
  __shared__ float red[32];
  pdl_wait();
  pdl_trigger();
  float s = 0.f;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    const float x = gload<G>(g, i);
    s += x * x;
  }
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (threadIdx.x == 0) atomicAdd(out, t);
  }
}

void sumsq_launch(const void* g, bool f32, int64_t n, float* out, cudaStream_t st) {
  if (n == 0) return;
  const int threads = 512;
  const int blocks = (int)std::min<int64_t>((n + threads - 1) / threads, 148 * 4);
  if (f32)
    launch_pdl(sumsq_kernel<float>, dim3(blocks), dim3(threads), 0, st, reinterpret_cast<const float*>(g), n, out);
  else
    launch_pdl(sumsq_kernel<__nv_bfloat16>, dim3(blocks), dim3(threads), 0, st,
               reinterpret_cast<const __nv_bfloat16*>(g), n, out);
}

// One CTA per row of a [T, V] fp32 logits chunk: loss[t] = lse - x[target],
// dlogits[t] = (softmax(x) - onehot(target)) * grad_scale (bf16, may alias
// nothing); rows whose target is < 0 (ignore index) get zero loss and grad.
__global__ void __launch_bounds__(1024) ce_fwd_bwd_kernel(const float* __restrict__ logits, int64_t ld, int64_t V,
                                                          const int64_t* __restrict__ targets,
                                                          float* __restrict__ loss, __nv_bfloat16* __restrict__ dlogits,
                                                          int64_t ldd, float grad_scale) {
  __shared__ float red[32];
  pdl_wait();
  pdl_trigger();
  const int64_t row = blockIdx.x;
  const float* x = logits + row * ld;
  const int64_t tgt = targets[row];
  float mx = -INFINITY;
  for (int64_t i = threadIdx.x; i < V; i += blockDim.x) mx = fmaxf(mx, x[i]);
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : -INFINITY;
    for (int o = 16; o > 0; o >>= 1) t = fmaxf(t, __shfl_xor_sync(0xffffffffu, t, o));
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  mx = red[0];
  __syncthreads();
  float s = 0.f;
  for (int64_t i = threadIdx.x; i < V; i += blockDim.x) s += __expf(x[i] - mx);
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  const float sum = red[0];
  const float lse = mx + logf(sum);
  const bool valid = tgt >= 0 && tgt < V;
  if (threadIdx.x == 0) loss[row] = valid ? (lse - x[tgt]) : 0.f;
  if (dlogits != nullptr) {
    __nv_bfloat16* d = dlogits + row * ldd;
    const float inv = 1.f / sum;
    for (int64_t i = threadIdx.x; i < V; i += blockDim.x) {
      float gval = valid ? (__expf(x[i] - mx) * inv - (i == tgt ? 1.f : 0.f)) * grad_scale : 0.f;
      d[i] = __float2bfloat16(gval);
    }
  }
}

void ce_fwd_bwd_launch(const float* logits, int64_t ld, int64_t T, int64_t V, const int64_t* targets, float* loss,
                       void* dlogits, int64_t ldd, float grad_scale, cudaStream_t st) {
  if (T == 0) return;
  launch_pdl(ce_fwd_bwd_kernel, dim3((unsigned)T), dim3(1024), 0, st, logits, ld, V, targets, loss,
             reinterpret_cast<__nv_bfloat16*>(dlogits), ldd, grad_scale);
}

}  // namespace b200
