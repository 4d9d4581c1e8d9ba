// Training-path elementwise kernels, forward and backward (bf16 activations,
// fp32 math and weight-gradient accumulation):
//
//   rmsnorm_fwd / rmsnorm_bwd          y = w * bf16(x * rstd), rstd saved per row;
//                                      dx = rstd * (g - xhat * mean(g * xhat)),
//                                      g = dy * w; dw += sum_rows dy * bf16(xhat)
//   qk_norm_rope_fwd / _bwd            on the fused q|k|v GEMM output: per-head
//                                      RMSNorm of q and k (optional) and the
//                                      half-split rotary embedding, written as
//                                      [T, H, D] q / k / v; backward un-rotates,
//                                      runs the per-head norm backward and
//                                      assembles the q|k|v gradient
//   swiglu_fwd / swiglu_bwd            h = silu(g) * u over [gate | up] halves;
//                                      dg = dh * u * silu'(g), du = dh * silu(g)
//   scale_by                           t *= g for a device scalar g
//
// The weight gradients of the norms are reduced per CTA in registers and added
// to fp32 buffers with one atomic per column per CTA (grid-stride over rows).
// HF semantics: norms normalise in fp32 and round to bf16 before the weight;
// the rounding is treated as identity in backward.
//
// Reference: rlx-tune differentiates the same decoder graph with its autodiff
// crate (rlx-tune src/lm.rs:77-115); these are the B200 kernels of that graph.
#include <cuda_bf16.h>

#include <algorithm>
#include <stdexcept>

#include "../common/b200.cuh"
#include "../common/launch.h"
#include "../common/pdl_launch.h"
#include "../common/tma_host.h"

namespace b200 {
namespace trf {

constexpr int kThreads = 256;

__device__ __forceinline__ float rbf(float v) { return __bfloat162float(__float2bfloat16(v)); }

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

// Each thread owns 8 consecutive columns of every row it visits (H <= 256 * 8 * kMaxChunks).
constexpr int kMaxChunks = 4;

__global__ void __launch_bounds__(kThreads) rmsnorm_fwd_kernel(const __nv_bfloat16* __restrict__ x,
                                                               const __nv_bfloat16* __restrict__ w,
                                                               __nv_bfloat16* __restrict__ y, float* __restrict__ rstd,
                                                               int rows, int H, float eps) {
  __shared__ float sh[kThreads / 32];
  pdl_wait();
  pdl_trigger();
  const int nch = H / (kThreads * 8);
  for (int r = blockIdx.x; r < rows; r += gridDim.x) {
    float v[kMaxChunks][8];
    float ss = 0.f;
#pragma unroll
    for (int c = 0; c < kMaxChunks; ++c) {
      if (c >= nch) break;
      const int col = (c * kThreads + threadIdx.x) * 8;
      const uint4 u = *reinterpret_cast<const uint4*>(x + (int64_t)r * H + col);
      const uint32_t p[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        v[c][2 * k] = bf16_lo(p[k]);
        v[c][2 * k + 1] = bf16_hi(p[k]);
        ss += v[c][2 * k] * v[c][2 * k] + v[c][2 * k + 1] * v[c][2 * k + 1];
      }
    }
    const float inv = rsqrtf(block_sum(ss, sh) / (float)H + eps);
    if (threadIdx.x == 0) rstd[r] = inv;
#pragma unroll
    for (int c = 0; c < kMaxChunks; ++c) {
      if (c >= nch) break;
      const int col = (c * kThreads + threadIdx.x) * 8;
      const uint4 wu = *reinterpret_cast<const uint4*>(w + col);
      const uint32_t wp[4] = {wu.x, wu.y, wu.z, wu.w};
      uint32_t o[4];
#pragma unroll
      for (int k = 0; k < 4; ++k)
        o[k] = pack_bf16x2(rbf(v[c][2 * k] * inv) * bf16_lo(wp[k]), rbf(v[c][2 * k + 1] * inv) * bf16_hi(wp[k]));
      *reinterpret_cast<uint4*>(y + (int64_t)r * H + col) = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

__global__ void __launch_bounds__(kThreads) rmsnorm_bwd_kernel(const __nv_bfloat16* __restrict__ dy,
                                                               const __nv_bfloat16* __restrict__ x,
                                                               const __nv_bfloat16* __restrict__ w,
                                                               const float* __restrict__ rstd,
                                                               __nv_bfloat16* __restrict__ dx, float* __restrict__ dw,
                                                               int rows, int H) {
  __shared__ float sh[kThreads / 32];
  pdl_wait();
  pdl_trigger();
  const int nch = H / (kThreads * 8);
  float dwacc[kMaxChunks][8];
  float wv[kMaxChunks][8];
#pragma unroll
  for (int c = 0; c < kMaxChunks; ++c) {
    if (c >= nch) break;
    const int col = (c * kThreads + threadIdx.x) * 8;
    const uint4 wu = *reinterpret_cast<const uint4*>(w + col);
    const uint32_t wp[4] = {wu.x, wu.y, wu.z, wu.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      wv[c][2 * k] = bf16_lo(wp[k]);
      wv[c][2 * k + 1] = bf16_hi(wp[k]);
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) dwacc[c][k] = 0.f;
  }
  for (int r = blockIdx.x; r < rows; r += gridDim.x) {
    const float inv = rstd[r];
    float xh[kMaxChunks][8], g[kMaxChunks][8];
    float dot = 0.f;
#pragma unroll
    for (int c = 0; c < kMaxChunks; ++c) {
      if (c >= nch) break;
      const int col = (c * kThreads + threadIdx.x) * 8;
      const uint4 xu = *reinterpret_cast<const uint4*>(x + (int64_t)r * H + col);
      const uint4 du = *reinterpret_cast<const uint4*>(dy + (int64_t)r * H + col);
      const uint32_t xp[4] = {xu.x, xu.y, xu.z, xu.w};
      const uint32_t dp[4] = {du.x, du.y, du.z, du.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        xh[c][2 * k] = bf16_lo(xp[k]) * inv;
        xh[c][2 * k + 1] = bf16_hi(xp[k]) * inv;
        const float d0 = bf16_lo(dp[k]), d1 = bf16_hi(dp[k]);
        g[c][2 * k] = d0 * wv[c][2 * k];
        g[c][2 * k + 1] = d1 * wv[c][2 * k + 1];
        dwacc[c][2 * k] += d0 * rbf(xh[c][2 * k]);
        dwacc[c][2 * k + 1] += d1 * rbf(xh[c][2 * k + 1]);
        dot += g[c][2 * k] * xh[c][2 * k] + g[c][2 * k + 1] * xh[c][2 * k + 1];
      }
    }
    const float mean = block_sum(dot, sh) / (float)H;
#pragma unroll
    for (int c = 0; c < kMaxChunks; ++c) {
      if (c >= nch) break;
      const int col = (c * kThreads + threadIdx.x) * 8;
      uint32_t o[4];
#pragma unroll
      for (int k = 0; k < 4; ++k)
        o[k] = pack_bf16x2(inv * (g[c][2 * k] - xh[c][2 * k] * mean),
                           inv * (g[c][2 * k + 1] - xh[c][2 * k + 1] * mean));
      *reinterpret_cast<uint4*>(dx + (int64_t)r * H + col) = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
#pragma unroll
  for (int c = 0; c < kMaxChunks; ++c) {
    if (c >= nch) break;
    const int col = (c * kThreads + threadIdx.x) * 8;
#pragma unroll
    for (int k = 0; k < 8; ++k) atomicAdd(dw + col + k, dwacc[c][k]);
  }
}

// ---------------------------------------------------------------------------
// Per-head RMSNorm + rotary embedding on the q|k|v GEMM output.
// One warp per (token, head); head_dim 128: lane l holds dims 4l..4l+3, and
// the rotary partner of dim d < 64 is d + 64, held by lane l + 16.
// Heads [0, Hq) are q, [Hq, Hq + Hkv) k, [Hq + Hkv, Hq + 2 Hkv) v (copied).
// ---------------------------------------------------------------------------
constexpr int kD = 128;

__device__ __forceinline__ void load4(const __nv_bfloat16* p, float (&v)[4]) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  v[0] = bf16_lo(u.x);
  v[1] = bf16_hi(u.x);
  v[2] = bf16_lo(u.y);
  v[3] = bf16_hi(u.y);
}
__device__ __forceinline__ void store4(__nv_bfloat16* p, const float (&v)[4]) {
  *reinterpret_cast<uint2*>(p) = make_uint2(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]));
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__global__ void __launch_bounds__(kThreads) qk_norm_rope_fwd_kernel(QKNormRopeArgs a) {
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int heads = a.Hq + 2 * a.Hkv;
  const int64_t item = (int64_t)blockIdx.x * (kThreads / 32) + (threadIdx.x >> 5);
  if (item >= (int64_t)a.T * heads) return;
  const int t = (int)(item / heads), hh = (int)(item % heads);
  const __nv_bfloat16* src = reinterpret_cast<const __nv_bfloat16*>(a.qkv) + (int64_t)t * heads * kD + hh * kD;
  float v[4];
  load4(src + lane * 4, v);
  if (hh >= a.Hq + a.Hkv) {  // v: copy
    store4(reinterpret_cast<__nv_bfloat16*>(a.v) + ((int64_t)t * a.Hkv + (hh - a.Hq - a.Hkv)) * kD + lane * 4, v);
    return;
  }
  const bool isq = hh < a.Hq;
  const __nv_bfloat16* nw = reinterpret_cast<const __nv_bfloat16*>(isq ? a.q_norm : a.k_norm);
  if (nw != nullptr) {
    const float inv = rsqrtf(warp_sum(v[0] * v[0] + v[1] * v[1] + v[2] * v[2] + v[3] * v[3]) / kD + a.eps);
    float wv[4];
    load4(nw + lane * 4, wv);
#pragma unroll
    for (int k = 0; k < 4; ++k) v[k] = rbf(rbf(v[k] * inv) * wv[k]);
    if (lane == 0) (isq ? a.rstd_q : a.rstd_k)[(int64_t)t * (isq ? a.Hq : a.Hkv) + (isq ? hh : hh - a.Hq)] = inv;
  }
  // rotary: out[d] = x[d] c - x[d+64] s (d < 64); out[d+64] = x[d+64] c + x[d] s
  const int pos = a.positions != nullptr ? a.positions[t] : t % a.S;
  float c[4], s[4], o[4];
  load4(reinterpret_cast<const __nv_bfloat16*>(a.cos) + (int64_t)pos * kD + lane * 4, c);
  load4(reinterpret_cast<const __nv_bfloat16*>(a.sin) + (int64_t)pos * kD + lane * 4, s);
  const bool lo = lane < 16;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float partner = __shfl_xor_sync(0xffffffffu, v[k], 16);
    // HF: x * cos + rotate_half(x) * sin in bf16 ops (each product rounded, then the sum)
    o[k] = rbf(rbf(v[k] * c[k]) + rbf((lo ? -partner : partner) * s[k]));
  }
  __nv_bfloat16* dst = isq ? reinterpret_cast<__nv_bfloat16*>(a.q) + ((int64_t)t * a.Hq + hh) * kD
                           : reinterpret_cast<__nv_bfloat16*>(a.k) + ((int64_t)t * a.Hkv + hh - a.Hq) * kD;
  store4(dst + lane * 4, o);
}

__global__ void __launch_bounds__(kThreads) qk_norm_rope_bwd_kernel(QKNormRopeArgs a) {
  __shared__ float red[2][kThreads / 32][kD];
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int heads = a.Hq + 2 * a.Hkv;
  // weight-gradient partials of this warp's items (q and k norms): 4 dims per lane
  float dwq[4] = {0.f, 0.f, 0.f, 0.f}, dwk[4] = {0.f, 0.f, 0.f, 0.f};
  const int64_t n_items = (int64_t)a.T * heads;
  const int64_t wstride = (int64_t)gridDim.x * (kThreads / 32);
  for (int64_t item = (int64_t)blockIdx.x * (kThreads / 32) + (threadIdx.x >> 5); item < n_items; item += wstride) {
    const int t = (int)(item / heads), hh = (int)(item % heads);
    __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(a.dqkv) + (int64_t)t * heads * kD + hh * kD + lane * 4;
    float g[4];
    if (hh >= a.Hq + a.Hkv) {
      load4(reinterpret_cast<const __nv_bfloat16*>(a.dv) + ((int64_t)t * a.Hkv + hh - a.Hq - a.Hkv) * kD + lane * 4,
            g);
      store4(dst, g);
      continue;
    }
    const bool isq = hh < a.Hq;
    load4(isq ? reinterpret_cast<const __nv_bfloat16*>(a.dq) + ((int64_t)t * a.Hq + hh) * kD + lane * 4
              : reinterpret_cast<const __nv_bfloat16*>(a.dk) + ((int64_t)t * a.Hkv + hh - a.Hq) * kD + lane * 4,
          g);
    // un-rotate: dn[d] = g[d] c + g[d+64] s ; dn[d+64] = g[d+64] c - g[d] s
    const int pos = a.positions != nullptr ? a.positions[t] : t % a.S;
    float c[4], s[4], dn[4];
    load4(reinterpret_cast<const __nv_bfloat16*>(a.cos) + (int64_t)pos * kD + lane * 4, c);
    load4(reinterpret_cast<const __nv_bfloat16*>(a.sin) + (int64_t)pos * kD + lane * 4, s);
    const bool lo = lane < 16;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float partner = __shfl_xor_sync(0xffffffffu, g[k], 16);
      const float ps = __shfl_xor_sync(0xffffffffu, s[k], 16);
      dn[k] = g[k] * c[k] + (lo ? partner * ps : -partner * ps);
    }
    const __nv_bfloat16* nw = reinterpret_cast<const __nv_bfloat16*>(isq ? a.q_norm : a.k_norm);
    if (nw == nullptr) {
      store4(dst, dn);
      continue;
    }
    float x[4], wv[4];
    load4(reinterpret_cast<const __nv_bfloat16*>(a.qkv) + (int64_t)t * heads * kD + hh * kD + lane * 4, x);
    load4(nw + lane * 4, wv);
    const float inv = (isq ? a.rstd_q : a.rstd_k)[(int64_t)t * (isq ? a.Hq : a.Hkv) + (isq ? hh : hh - a.Hq)];
    float xh[4], gg[4], dot = 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      xh[k] = x[k] * inv;
      gg[k] = dn[k] * wv[k];
      dot += gg[k] * xh[k];
      if (isq)
        dwq[k] += dn[k] * rbf(xh[k]);
      else
        dwk[k] += dn[k] * rbf(xh[k]);
    }
    const float mean = warp_sum(dot) / kD;
    float o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) o[k] = inv * (gg[k] - xh[k] * mean);
    store4(dst, o);
  }
  if (a.dw_q != nullptr) {
    // per-CTA reduction of the warps' partials, then one atomic per dim
    const int w = threadIdx.x >> 5;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      red[0][w][lane * 4 + k] = dwq[k];
      red[1][w][lane * 4 + k] = dwk[k];
    }
    __syncthreads();
    for (int i = threadIdx.x; i < 2 * kD; i += kThreads) {
      const int which = i / kD, d = i % kD;
      float sum = 0.f;
#pragma unroll
      for (int ww = 0; ww < kThreads / 32; ++ww) sum += red[which][ww][d];
      atomicAdd((which ? a.dw_k : a.dw_q) + d, sum);
    }
  }
}

// ---------------------------------------------------------------------------
// SwiGLU over [T, 2I] = [gate | up] rows.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float sigmoid(float x) { return 1.f / (1.f + __expf(-x)); }

__global__ void __launch_bounds__(kThreads) swiglu_fwd_kernel(const __nv_bfloat16* __restrict__ gu,
                                                              __nv_bfloat16* __restrict__ h, int64_t T, int I) {
  pdl_wait();
  pdl_trigger();
  const int64_t n8 = T * (int64_t)(I / 8);
  for (int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x; i < n8; i += (int64_t)gridDim.x * kThreads) {
    const int64_t t = i / (I / 8);
    const int col = (int)(i % (I / 8)) * 8;
    const uint4 gv = *reinterpret_cast<const uint4*>(gu + t * 2 * I + col);
    const uint4 uv = *reinterpret_cast<const uint4*>(gu + t * 2 * I + I + col);
    const uint32_t gp[4] = {gv.x, gv.y, gv.z, gv.w}, up[4] = {uv.x, uv.y, uv.z, uv.w};
    uint32_t o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float g0 = bf16_lo(gp[k]), g1 = bf16_hi(gp[k]);
      // HF: silu(g) rounded to bf16, then times u (bf16 product)
      o[k] = pack_bf16x2(rbf(g0 * sigmoid(g0)) * bf16_lo(up[k]), rbf(g1 * sigmoid(g1)) * bf16_hi(up[k]));
    }
    *reinterpret_cast<uint4*>(h + t * I + col) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

__global__ void __launch_bounds__(kThreads) swiglu_bwd_kernel(const __nv_bfloat16* __restrict__ dh,
                                                              const __nv_bfloat16* __restrict__ gu,
                                                              __nv_bfloat16* __restrict__ dgu, int64_t T, int I) {
  pdl_wait();
  pdl_trigger();
  const int64_t n8 = T * (int64_t)(I / 8);
  for (int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x; i < n8; i += (int64_t)gridDim.x * kThreads) {
    const int64_t t = i / (I / 8);
    const int col = (int)(i % (I / 8)) * 8;
    const uint4 gv = *reinterpret_cast<const uint4*>(gu + t * 2 * I + col);
    const uint4 uv = *reinterpret_cast<const uint4*>(gu + t * 2 * I + I + col);
    const uint4 dv = *reinterpret_cast<const uint4*>(dh + t * I + col);
    const uint32_t gp[4] = {gv.x, gv.y, gv.z, gv.w}, up[4] = {uv.x, uv.y, uv.z, uv.w},
                   dp[4] = {dv.x, dv.y, dv.z, dv.w};
    uint32_t og[4], ou[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float g[2] = {bf16_lo(gp[k]), bf16_hi(gp[k])}, u[2] = {bf16_lo(up[k]), bf16_hi(up[k])},
                  d[2] = {bf16_lo(dp[k]), bf16_hi(dp[k])};
      float rg[2], ru[2];
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const float sg = sigmoid(g[j]);
        ru[j] = d[j] * rbf(g[j] * sg);
        rg[j] = d[j] * u[j] * sg * (1.f + g[j] * (1.f - sg));
      }
      og[k] = pack_bf16x2(rg[0], rg[1]);
      ou[k] = pack_bf16x2(ru[0], ru[1]);
    }
    *reinterpret_cast<uint4*>(dgu + t * 2 * I + col) = make_uint4(og[0], og[1], og[2], og[3]);
    *reinterpret_cast<uint4*>(dgu + t * 2 * I + I + col) = make_uint4(ou[0], ou[1], ou[2], ou[3]);
  }
}

// t *= *g for a device scalar g (the loss gradient of a fused loss whose
// parameter gradients were formed in forward): fp32 or bf16 tensors.
__global__ void __launch_bounds__(kThreads) scale_f32_kernel(float* __restrict__ t, int64_t n,
                                                             const float* __restrict__ g) {
  pdl_wait();
  pdl_trigger();
  const float s = *g;
  if (s == 1.f) return;
  for (int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x; i < n; i += (int64_t)gridDim.x * kThreads)
    t[i] *= s;
}
__global__ void __launch_bounds__(kThreads) scale_bf16_kernel(__nv_bfloat16* __restrict__ t, int64_t n,
                                                              const float* __restrict__ g) {
  pdl_wait();
  pdl_trigger();
  const float s = *g;
  if (s == 1.f) return;
  for (int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x; i < n; i += (int64_t)gridDim.x * kThreads)
    t[i] = __float2bfloat16(__bfloat162float(t[i]) * s);
}

static int grid_for(int64_t work, int per_cta, int device) {
  const int64_t need = (work + per_cta - 1) / per_cta;
  const int64_t cap = (int64_t)num_sms(device) * 8;
  return (int)std::max<int64_t>(1, std::min(need, cap));
}

}  // namespace trf

void rmsnorm_train_fwd_launch(const void* x, const void* w, void* y, float* rstd, int rows, int H, float eps,
                              int device, cudaStream_t st) {
  if (H % (trf::kThreads * 8) != 0 || H > trf::kThreads * 8 * trf::kMaxChunks)
    throw std::runtime_error("b200.rmsnorm_train: hidden must be a multiple of 2048 and <= 8192");
  if (rows == 0) return;
  launch_pdl(trf::rmsnorm_fwd_kernel, dim3(trf::grid_for(rows, 1, device)), dim3(trf::kThreads), 0, st,
             reinterpret_cast<const __nv_bfloat16*>(x), reinterpret_cast<const __nv_bfloat16*>(w),
             reinterpret_cast<__nv_bfloat16*>(y), rstd, rows, H, eps);
}

void rmsnorm_train_bwd_launch(const void* dy, const void* x, const void* w, const float* rstd, void* dx, float* dw,
                              int rows, int H, int device, cudaStream_t st) {
  if (H % (trf::kThreads * 8) != 0 || H > trf::kThreads * 8 * trf::kMaxChunks)
    throw std::runtime_error("b200.rmsnorm_train: hidden must be a multiple of 2048 and <= 8192");
  if (rows == 0) return;
  // fewer CTAs than rows: each CTA keeps its weight-gradient partial in registers
  launch_pdl(trf::rmsnorm_bwd_kernel, dim3(std::min(rows, num_sms(device) * 2)), dim3(trf::kThreads), 0, st,
             reinterpret_cast<const __nv_bfloat16*>(dy), reinterpret_cast<const __nv_bfloat16*>(x),
             reinterpret_cast<const __nv_bfloat16*>(w), rstd, reinterpret_cast<__nv_bfloat16*>(dx), dw, rows, H);
}

void qk_norm_rope_fwd_launch(const QKNormRopeArgs& a, int device, cudaStream_t st) {
  (void)device;
  if (a.D != trf::kD) throw std::runtime_error("b200.qk_norm_rope: head_dim must be 128");
  const int64_t items = (int64_t)a.T * (a.Hq + 2 * a.Hkv);
  if (items == 0) return;
  launch_pdl(trf::qk_norm_rope_fwd_kernel, dim3((unsigned)((items + 7) / 8)), dim3(trf::kThreads), 0, st, a);
}

void qk_norm_rope_bwd_launch(const QKNormRopeArgs& a, int device, cudaStream_t st) {
  if (a.D != trf::kD) throw std::runtime_error("b200.qk_norm_rope: head_dim must be 128");
  const int64_t items = (int64_t)a.T * (a.Hq + 2 * a.Hkv);
  if (items == 0) return;
  launch_pdl(trf::qk_norm_rope_bwd_kernel, dim3(trf::grid_for(items, 64, device)), dim3(trf::kThreads), 0, st, a);
}

void swiglu_train_fwd_launch(const void* gu, void* h, int64_t T, int I, int device, cudaStream_t st) {
  if (I % 8 != 0) throw std::runtime_error("b200.swiglu_train: width must be a multiple of 8");
  if (T == 0) return;
  launch_pdl(trf::swiglu_fwd_kernel, dim3(trf::grid_for(T * (I / 8), trf::kThreads * 4, device)),
             dim3(trf::kThreads), 0, st, reinterpret_cast<const __nv_bfloat16*>(gu),
             reinterpret_cast<__nv_bfloat16*>(h), T, I);
}

void swiglu_train_bwd_launch(const void* dh, const void* gu, void* dgu, int64_t T, int I, int device,
                             cudaStream_t st) {
  if (I % 8 != 0) throw std::runtime_error("b200.swiglu_train: width must be a multiple of 8");
  if (T == 0) return;
  launch_pdl(trf::swiglu_bwd_kernel, dim3(trf::grid_for(T * (I / 8), trf::kThreads * 4, device)),
             dim3(trf::kThreads), 0, st, reinterpret_cast<const __nv_bfloat16*>(dh),
             reinterpret_cast<const __nv_bfloat16*>(gu), reinterpret_cast<__nv_bfloat16*>(dgu), T, I);
}

void scale_by_launch(void* t, bool is_f32, int64_t n, const float* g, int device, cudaStream_t st) {
  if (n == 0) return;
  const dim3 grid(trf::grid_for(n, trf::kThreads * 8, device));
  if (is_f32)
    launch_pdl(trf::scale_f32_kernel, grid, dim3(trf::kThreads), 0, st, reinterpret_cast<float*>(t), n, g);
  else
    launch_pdl(trf::scale_bf16_kernel, grid, dim3(trf::kThreads), 0, st, reinterpret_cast<__nv_bfloat16*>(t), n, g);
}

}  // namespace b200
