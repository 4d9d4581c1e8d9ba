// Memory-bound per-token kernels of the decoder block ("K7", "K8", "K11", "K12"):
//   * embedding gather,
//   * RMSNorm with an optional fused residual add (residual stream update +
//     normalisation in one pass over HBM),
//   * the QKV post-processing epilogue: per-head QK RMSNorm (Qwen3 style),
//     rotary embedding (half-split / NeoX layout, cos/sin computed in-kernel
//     from an inv_freq table so every RoPE scaling variant is one table), and
//     the paged KV-cache write (block size 16).
//
// Semantics follow the HF modules the reference mirrors: Qwen3 RMSNorm
// normalises in fp32, casts to the activation dtype, then multiplies by the
// weight (rlx-models-core src/standard_decoder.rs:370-410 `load_norm`,
// `per_head_rms`); RoPE rotates (x[i], x[i+half]) pairs
// (standard_decoder.rs:411,705; rlx-qwen3 src/generator.rs:4486).
#include <cuda_bf16.h>
#include <cuda_fp8.h>

#include "../common/b200.cuh"
#include "../common/launch.h"
#include "../common/pdl_launch.h"

#include <algorithm>
#include <stdexcept>

namespace b200 {

__global__ void embedding_kernel(const int32_t* __restrict__ ids, const uint4* __restrict__ table,
                                 uint4* __restrict__ out, int64_t H8, int64_t V) {
  pdl_wait();
  pdl_trigger();
  const int64_t t = blockIdx.x;
  int64_t id = ids[t];
  if (id < 0 || id >= V) id = 0;  // out-of-range ids read row 0 rather than faulting
  const uint4* src = table + id * H8;
  uint4* dst = out + t * H8;
  for (int64_t i = threadIdx.x; i < H8; i += blockDim.x) dst[i] = __ldg(src + i);
}

void embedding_launch(const int32_t* ids, const void* table, void* out, int64_t T, int64_t H, int64_t V,
                      cudaStream_t st) {
  if (T == 0) return;
  launch_pdl(embedding_kernel, dim3((unsigned)T), dim3(256), 0, st, ids, reinterpret_cast<const uint4*>(table),
             reinterpret_cast<uint4*>(out), H / 8, V);
}

// One CTA per row, one 8-element vector (16 B) per thread and pass; the row
// stays in registers between the sum-of-squares and the scaling pass.
template <int VPT>
__global__ void rmsnorm_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx,
                               const __nv_bfloat16* __restrict__ res_in, __nv_bfloat16* __restrict__ res_out,
                               const __nv_bfloat16* __restrict__ w, __nv_bfloat16* __restrict__ out, int64_t ldo,
                               int H, float eps) {
  __shared__ float red[32];
  pdl_wait();
  pdl_trigger();
  const int64_t row = blockIdx.x;
  const int nv = H / 8;
  float v[VPT][8];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int vi = threadIdx.x + k * blockDim.x;
    if (vi >= nv) break;
    const uint4 xv = *reinterpret_cast<const uint4*>(x + row * ldx + vi * 8);
    uint32_t a[4] = {xv.x, xv.y, xv.z, xv.w};
    if (res_in != nullptr) {
      const uint4 r = *reinterpret_cast<const uint4*>(res_in + row * (int64_t)H + vi * 8);
      const uint32_t b[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
      for (int h = 0; h < 4; ++h)  // residual stream stays bf16 (HF): round the sum once
        a[h] = pack_bf16x2(bf16_lo(a[h]) + bf16_lo(b[h]), bf16_hi(a[h]) + bf16_hi(b[h]));
      if (res_out != nullptr)
        *reinterpret_cast<uint4*>(res_out + row * (int64_t)H + vi * 8) = make_uint4(a[0], a[1], a[2], a[3]);
    }
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      v[k][2 * h] = bf16_lo(a[h]);
      v[k][2 * h + 1] = bf16_hi(a[h]);
      ss += v[k][2 * h] * v[k][2 * h] + v[k][2 * h + 1] * v[k][2 * h + 1];
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  const float inv = rsqrtf(red[0] / (float)H + eps);
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int vi = threadIdx.x + k * blockDim.x;
    if (vi >= nv) break;
    const uint4 wv = *reinterpret_cast<const uint4*>(w + vi * 8);
    const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
    uint32_t o[4];
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      // normalise in fp32, round to bf16, then scale by the bf16 weight
      const float lo = __bfloat162float(__float2bfloat16(v[k][2 * h] * inv)) * bf16_lo(ww[h]);
      const float hi = __bfloat162float(__float2bfloat16(v[k][2 * h + 1] * inv)) * bf16_hi(ww[h]);
      o[h] = pack_bf16x2(lo, hi);
    }
    *reinterpret_cast<uint4*>(out + row * ldo + vi * 8) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

void rmsnorm_launch(const void* x, int64_t ldx, const void* residual_in, void* residual_out, const void* w,
                    void* out, int64_t ldo, int64_t T, int64_t H, float eps, cudaStream_t st) {
  if (T == 0) return;
  const int nv = (int)(H / 8);
  int threads = std::min(1024, (nv + 31) / 32 * 32);
  const int vpt = (nv + threads - 1) / threads;
  auto xb = reinterpret_cast<const __nv_bfloat16*>(x);
  auto rb = reinterpret_cast<const __nv_bfloat16*>(residual_in);
  auto ro = reinterpret_cast<__nv_bfloat16*>(residual_out);
  auto wb = reinterpret_cast<const __nv_bfloat16*>(w);
  auto ob = reinterpret_cast<__nv_bfloat16*>(out);
  if (vpt <= 1) launch_pdl(rmsnorm_kernel<1>, dim3((unsigned)T), dim3(threads), 0, st, xb, ldx, rb, ro, wb, ob, ldo, (int)H, eps);
  else if (vpt <= 2) launch_pdl(rmsnorm_kernel<2>, dim3((unsigned)T), dim3(threads), 0, st, xb, ldx, rb, ro, wb, ob, ldo, (int)H, eps);
  else if (vpt <= 4) launch_pdl(rmsnorm_kernel<4>, dim3((unsigned)T), dim3(threads), 0, st, xb, ldx, rb, ro, wb, ob, ldo, (int)H, eps);
  else throw std::runtime_error("b200.rmsnorm: hidden size too large (max 32768)");
}

// One warp per (token, head) over q heads, k heads and v heads.
// E = D / 32 elements per lane (D in {64, 128}); the rotation partner of
// element d (< D/2) is d + D/2, held by lane (lane ^ 16).
template <int E>
__global__ void qkv_rope_kernel(QkvRopeArgs a) {
  pdl_wait();
  pdl_trigger();
  const int nh = a.Hq + 2 * a.Hkv;
  const int64_t gw = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (gw >= a.T * nh) return;
  const int64_t t = gw / nh;
  const int h = (int)(gw % nh);
  const int D = 32 * E;
  float x[E];
  if (a.qkv_f32 != nullptr) {
    // accumulate-only GEMM output: round the fp32 sum to bf16 (as the bf16
    // GEMM epilogue would) and zero it for the next use
    float* src = a.qkv_f32 + t * a.ld_qkv + (int64_t)h * D;
    const __nv_bfloat16* bb =
        a.bias != nullptr ? reinterpret_cast<const __nv_bfloat16*>(a.bias) + (int64_t)h * D + lane * E : nullptr;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const float bv = bb != nullptr ? __bfloat162float(bb[e]) : 0.f;  // the bf16 epilogue adds the bias
      x[e] = __bfloat162float(__float2bfloat16(__ldcg(src + lane * E + e) + bv));
      __stcg(src + lane * E + e, 0.f);
    }
  } else {
    const __nv_bfloat16* src = reinterpret_cast<const __nv_bfloat16*>(a.qkv) + t * a.ld_qkv + (int64_t)h * D;
#pragma unroll
    for (int e = 0; e < E; ++e) x[e] = __bfloat162float(src[lane * E + e]);
  }

  const bool is_q = h < a.Hq;
  const bool is_k = !is_q && h < a.Hq + a.Hkv;
  const bool is_v = !is_q && !is_k;
  if (!is_v) {
    const __nv_bfloat16* nw = reinterpret_cast<const __nv_bfloat16*>(is_q ? a.q_norm : a.k_norm);
    if (nw != nullptr) {
      float ss = 0.f;
#pragma unroll
      for (int e = 0; e < E; ++e) ss += x[e] * x[e];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      const float inv = rsqrtf(ss / (float)D + a.eps);
#pragma unroll
      for (int e = 0; e < E; ++e)
        x[e] = __bfloat162float(__float2bfloat16(x[e] * inv)) * __bfloat162float(nw[lane * E + e]);
#pragma unroll
      for (int e = 0; e < E; ++e) x[e] = __bfloat162float(__float2bfloat16(x[e]));
    }
    // rotary embedding over the first rot_dim dims (half-split layout: dim d
    // pairs with d + rot_dim/2); dims >= rot_dim pass through (partial RoPE)
    const float pos = (float)a.positions[t];
    const int rh = a.rot_dim / 2;
    const int base = lane * E;
    const int off = rh / E;  // lanes between the two halves of a pair
    const int src = base < rh ? lane + off : (base < a.rot_dim ? lane - off : lane);
    float y[E];
#pragma unroll
    for (int e = 0; e < E; ++e) y[e] = __shfl_sync(0xffffffffu, x[e], src);
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const int d = base + e;
      if (d < a.rot_dim) {
        const int fi = d < rh ? d : d - rh;
        float s, c;
        sincosf(pos * a.inv_freq[fi], &s, &c);
        c *= a.rope_scale;
        s *= a.rope_scale;
        x[e] = d < rh ? (x[e] * c - y[e] * s) : (x[e] * c + y[e] * s);
      }
    }
  }
  if (is_q) {
    __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(a.q_out) + (t * a.Hq + h) * D;
#pragma unroll
    for (int e = 0; e < E; ++e) dst[lane * E + e] = __float2bfloat16(x[e]);
    return;
  }
  const int kh = is_k ? h - a.Hq : h - a.Hq - a.Hkv;
  void* kvo = is_k ? a.k_out : a.v_out;
  if (kvo != nullptr) {
    __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(kvo) + (t * a.Hkv + kh) * D;
#pragma unroll
    for (int e = 0; e < E; ++e) dst[lane * E + e] = __float2bfloat16(x[e]);
  }
  if (a.slots != nullptr) {
    const int64_t slot = a.slots[t];
    if (slot >= 0) {
      const int64_t blk = slot >> 4, off = slot & 15;
      const int64_t at = ((blk * a.Hkv + kh) * 16 + off) * D;
      if (a.kv_fp8) {
        // the bf16-rounded value, scaled, to e4m3 with saturation (what the bf16 cache would hold)
        __nv_fp8_e4m3* dst = reinterpret_cast<__nv_fp8_e4m3*>(is_k ? a.k_cache : a.v_cache) + at;
        const float inv = is_k ? a.k_inv_scale : a.v_inv_scale;
#pragma unroll
        for (int e = 0; e < E; ++e) dst[lane * E + e] = __nv_fp8_e4m3(__bfloat162float(__float2bfloat16(x[e])) * inv);
      } else {
        __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(is_k ? a.k_cache : a.v_cache) + at;
#pragma unroll
        for (int e = 0; e < E; ++e) dst[lane * E + e] = __float2bfloat16(x[e]);
      }
    }
  }
}

void qkv_rope_launch(const QkvRopeArgs& a, cudaStream_t st) {
  if (a.T == 0) return;
  const int64_t warps = a.T * (a.Hq + 2 * a.Hkv);
  const int wpb = 8;
  const unsigned grid = (unsigned)((warps + wpb - 1) / wpb);
  if (a.D == 256) launch_pdl(qkv_rope_kernel<8>, dim3(grid), dim3(wpb * 32), 0, st, a);
  else if (a.D == 128) launch_pdl(qkv_rope_kernel<4>, dim3(grid), dim3(wpb * 32), 0, st, a);
  else launch_pdl(qkv_rope_kernel<2>, dim3(grid), dim3(wpb * 32), 0, st, a);
}

// ---------------------------------------------------------------------------
// Consumers of the accumulate-only GEMM (fp32 [T, N] sums, zeroed after use).
// ---------------------------------------------------------------------------

// h = bf16(h + bf16(acc)); out = rmsnorm(h) * w; acc = 0.   One CTA per row.
template <int VPT>
__global__ void add_rmsnorm_acc_kernel(float* __restrict__ acc, __nv_bfloat16* __restrict__ h,
                                       const __nv_bfloat16* __restrict__ w, __nv_bfloat16* __restrict__ out,
                                       int64_t ldo, int H, float eps, const __nv_bfloat16* __restrict__ bias) {
  __shared__ float red[32];
  pdl_wait();
  pdl_trigger();
  const int64_t row = blockIdx.x;
  const int nv = H / 8;
  float v[VPT][8];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int vi = threadIdx.x + k * blockDim.x;
    if (vi >= nv) break;
    float4* ap = reinterpret_cast<float4*>(acc + row * (int64_t)H + vi * 8);
    const float4 a0 = __ldcg(ap), a1 = __ldcg(ap + 1);
    __stcg(ap, make_float4(0.f, 0.f, 0.f, 0.f));
    __stcg(ap + 1, make_float4(0.f, 0.f, 0.f, 0.f));
    float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
    if (bias != nullptr) {
      const uint4 bv = *reinterpret_cast<const uint4*>(bias + vi * 8);
      const uint32_t bw[4] = {bv.x, bv.y, bv.z, bv.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        av[2 * q] += bf16_lo(bw[q]);
        av[2 * q + 1] += bf16_hi(bw[q]);
      }
    }
    uint4* hp = reinterpret_cast<uint4*>(h + row * (int64_t)H + vi * 8);
    const uint4 hv = *hp;
    const uint32_t hw[4] = {hv.x, hv.y, hv.z, hv.w};
    uint32_t o[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float lo = __bfloat162float(__float2bfloat16(av[2 * q]));
      const float hi = __bfloat162float(__float2bfloat16(av[2 * q + 1]));
      o[q] = pack_bf16x2(bf16_lo(hw[q]) + lo, bf16_hi(hw[q]) + hi);
      v[k][2 * q] = bf16_lo(o[q]);
      v[k][2 * q + 1] = bf16_hi(o[q]);
      ss += v[k][2 * q] * v[k][2 * q] + v[k][2 * q + 1] * v[k][2 * q + 1];
    }
    *hp = make_uint4(o[0], o[1], o[2], o[3]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  const float inv = rsqrtf(red[0] / (float)H + eps);
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int vi = threadIdx.x + k * blockDim.x;
    if (vi >= nv) break;
    const uint4 wv = *reinterpret_cast<const uint4*>(w + vi * 8);
    const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
    uint32_t o[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float lo = __bfloat162float(__float2bfloat16(v[k][2 * q] * inv)) * bf16_lo(ww[q]);
      const float hi = __bfloat162float(__float2bfloat16(v[k][2 * q + 1] * inv)) * bf16_hi(ww[q]);
      o[q] = pack_bf16x2(lo, hi);
    }
    *reinterpret_cast<uint4*>(out + row * ldo + vi * 8) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

void add_rmsnorm_acc_launch(float* acc, void* h, const void* w, void* out, int64_t ldo, int64_t T, int64_t H,
                            float eps, cudaStream_t st, const void* bias) {
  if (T == 0) return;
  const int nv = (int)(H / 8);
  const int threads = std::min(1024, (nv + 31) / 32 * 32);
  const int vpt = (nv + threads - 1) / threads;
  auto hb = reinterpret_cast<__nv_bfloat16*>(h);
  auto wb = reinterpret_cast<const __nv_bfloat16*>(w);
  auto ob = reinterpret_cast<__nv_bfloat16*>(out);
  if (vpt <= 1) launch_pdl(add_rmsnorm_acc_kernel<1>, dim3((unsigned)T), dim3(threads), 0, st, acc, hb, wb, ob, ldo, (int)H, eps,
                                    reinterpret_cast<const __nv_bfloat16*>(bias));
  else if (vpt <= 2) launch_pdl(add_rmsnorm_acc_kernel<2>, dim3((unsigned)T), dim3(threads), 0, st, acc, hb, wb, ob, ldo, (int)H, eps,
                                    reinterpret_cast<const __nv_bfloat16*>(bias));
  else if (vpt <= 4) launch_pdl(add_rmsnorm_acc_kernel<4>, dim3((unsigned)T), dim3(threads), 0, st, acc, hb, wb, ob, ldo, (int)H, eps,
                                    reinterpret_cast<const __nv_bfloat16*>(bias));
  else throw std::runtime_error("b200.add_rmsnorm_acc: hidden size too large");
}

// out[t, f] = silu(acc[t, g(f)]) * acc[t, g(f) + 64], g(f) = (f / 64) * 128 + f % 64
// (gate/up interleaved in groups of 64 features); the consumed sums are zeroed.
// act = 1: GELU (tanh form) on the gate instead of SiLU (GeGLU).
__device__ __forceinline__ float glu_gate(float g, int act) {
  if (act) {
    const float u = 0.7978845608028654f * (g + 0.044715f * g * g * g);
    float t;
    asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(u));
    return 0.5f * g * (1.f + t);
  }
  return g / (1.f + __expf(-g));
}

__global__ void swiglu_acc_kernel(float* __restrict__ acc, __nv_bfloat16* __restrict__ out, int64_t I, int64_t T,
                                  int act) {
  pdl_wait();
  pdl_trigger();
  const int64_t idx = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 8;  // 8 outputs per thread
  if (idx >= T * I) return;
  const int64_t t = idx / I, f = idx % I;
  float* row = acc + t * 2 * I;
  const int64_t g = (f / 64) * 128 + (f % 64);
  float4* gp = reinterpret_cast<float4*>(row + g);
  float4* up = reinterpret_cast<float4*>(row + g + 64);
  const float4 g0 = __ldcg(gp), g1 = __ldcg(gp + 1), u0 = __ldcg(up), u1 = __ldcg(up + 1);
  const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
  __stcg(gp, z);
  __stcg(gp + 1, z);
  __stcg(up, z);
  __stcg(up + 1, z);
  const float gv[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
  const float uv[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
  uint32_t o[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float a = glu_gate(gv[2 * q], act) * uv[2 * q];
    const float b = glu_gate(gv[2 * q + 1], act) * uv[2 * q + 1];
    o[q] = pack_bf16x2(a, b);
  }
  *reinterpret_cast<uint4*>(out + t * I + f) = make_uint4(o[0], o[1], o[2], o[3]);
}

void swiglu_acc_launch(float* acc, void* out, int64_t T, int64_t I, int act, cudaStream_t st) {
  if (T == 0) return;
  const int64_t n = T * I / 8;
  launch_pdl(swiglu_acc_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, st, acc,
             reinterpret_cast<__nv_bfloat16*>(out), I, T, act);
}

}  // namespace b200
