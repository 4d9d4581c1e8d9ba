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

#include "../common/b200.cuh"
#include "../common/launch.h"

namespace b200 {

__global__ void embedding_kernel(const int32_t* __restrict__ ids, const uint4* __restrict__ table,
                                 uint4* __restrict__ out, int64_t H8, int64_t V) {
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
  embedding_kernel<<<(unsigned)T, 256, 0, st>>>(ids, reinterpret_cast<const uint4*>(table),
                                                 reinterpret_cast<uint4*>(out), H / 8, V);
}

// One warp per row. H % 256 == 0 (8 bf16 per lane per step).
__global__ void rmsnorm_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx,
                               const __nv_bfloat16* __restrict__ res_in, __nv_bfloat16* __restrict__ res_out,
                               const __nv_bfloat16* __restrict__ w, __nv_bfloat16* __restrict__ out, int64_t ldo,
                               int64_t T, int H, float eps) {
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (row >= T) return;
  const __nv_bfloat16* xr = x + row * ldx;
  float ss = 0.f;
  for (int c = lane * 8; c < H; c += 256) {
    uint4 v = *reinterpret_cast<const uint4*>(xr + c);
    uint32_t a[4] = {v.x, v.y, v.z, v.w};
    if (res_in != nullptr) {
      uint4 r = *reinterpret_cast<const uint4*>(res_in + row * (int64_t)H + c);
      uint32_t b[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        // residual stream is kept in bf16 (HF semantics): round the sum once
        a[h] = pack_bf16x2(bf16_lo(a[h]) + bf16_lo(b[h]), bf16_hi(a[h]) + bf16_hi(b[h]));
      }
      if (res_out != nullptr)
        *reinterpret_cast<uint4*>(res_out + row * (int64_t)H + c) = make_uint4(a[0], a[1], a[2], a[3]);
    }
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      const float lo = bf16_lo(a[h]), hi = bf16_hi(a[h]);
      ss += lo * lo + hi * hi;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float inv = rsqrtf(ss / (float)H + eps);
  const __nv_bfloat16* src = (res_in != nullptr && res_out != nullptr) ? res_out + row * (int64_t)H : xr;
  for (int c = lane * 8; c < H; c += 256) {
    uint4 v;
    if (res_in != nullptr && res_out == nullptr) {
      uint4 xv = *reinterpret_cast<const uint4*>(xr + c);
      uint4 r = *reinterpret_cast<const uint4*>(res_in + row * (int64_t)H + c);
      uint32_t a[4] = {xv.x, xv.y, xv.z, xv.w}, b[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
      for (int h = 0; h < 4; ++h)
        a[h] = pack_bf16x2(bf16_lo(a[h]) + bf16_lo(b[h]), bf16_hi(a[h]) + bf16_hi(b[h]));
      v = make_uint4(a[0], a[1], a[2], a[3]);
    } else {
      v = *reinterpret_cast<const uint4*>(src + c);
    }
    const uint4 wv = *reinterpret_cast<const uint4*>(w + c);
    uint32_t a[4] = {v.x, v.y, v.z, v.w}, ww[4] = {wv.x, wv.y, wv.z, wv.w}, o[4];
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      // normalise in fp32, round to bf16, then scale by the bf16 weight
      const float lo = __bfloat162float(__float2bfloat16(bf16_lo(a[h]) * inv)) * bf16_lo(ww[h]);
      const float hi = __bfloat162float(__float2bfloat16(bf16_hi(a[h]) * inv)) * bf16_hi(ww[h]);
      o[h] = pack_bf16x2(lo, hi);
    }
    *reinterpret_cast<uint4*>(out + row * ldo + c) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

void rmsnorm_launch(const void* x, int64_t ldx, const void* residual_in, void* residual_out, const void* w,
                    void* out, int64_t ldo, int64_t T, int64_t H, float eps, cudaStream_t st) {
  if (T == 0) return;
  const int rows_per_block = 8;
  const unsigned grid = (unsigned)((T + rows_per_block - 1) / rows_per_block);
  rmsnorm_kernel<<<grid, rows_per_block * 32, 0, st>>>(
      reinterpret_cast<const __nv_bfloat16*>(x), ldx, reinterpret_cast<const __nv_bfloat16*>(residual_in),
      reinterpret_cast<__nv_bfloat16*>(residual_out), reinterpret_cast<const __nv_bfloat16*>(w),
      reinterpret_cast<__nv_bfloat16*>(out), ldo, T, (int)H, eps);
}

// One warp per (token, head) over q heads, k heads and v heads.
// E = D / 32 elements per lane (D in {64, 128}); the rotation partner of
// element d (< D/2) is d + D/2, held by lane (lane ^ 16).
template <int E>
__global__ void qkv_rope_kernel(QkvRopeArgs a) {
  const int nh = a.Hq + 2 * a.Hkv;
  const int64_t gw = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (gw >= a.T * nh) return;
  const int64_t t = gw / nh;
  const int h = (int)(gw % nh);
  const int D = 32 * E;
  const __nv_bfloat16* src = reinterpret_cast<const __nv_bfloat16*>(a.qkv) + t * a.ld_qkv + (int64_t)h * D;
  float x[E];
#pragma unroll
  for (int e = 0; e < E; ++e) x[e] = __bfloat162float(src[lane * E + e]);

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
    // rotary embedding (full rotary dim, half-split layout)
    const float pos = (float)a.positions[t];
    float y[E];
#pragma unroll
    for (int e = 0; e < E; ++e) y[e] = __shfl_xor_sync(0xffffffffu, x[e], 16);
    const int half = D / 2;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const int d = lane * E + e;
      const int fi = d < half ? d : d - half;
      float s, c;
      sincosf(pos * a.inv_freq[fi], &s, &c);
      c *= a.rope_scale;
      s *= a.rope_scale;
      x[e] = d < half ? (x[e] * c - y[e] * s) : (x[e] * c + y[e] * s);
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
      __nv_bfloat16* cache = reinterpret_cast<__nv_bfloat16*>(is_k ? a.k_cache : a.v_cache);
      __nv_bfloat16* dst = cache + ((blk * a.Hkv + kh) * 16 + off) * D;
#pragma unroll
      for (int e = 0; e < E; ++e) dst[lane * E + e] = __float2bfloat16(x[e]);
    }
  }
}

void qkv_rope_launch(const QkvRopeArgs& a, cudaStream_t st) {
  if (a.T == 0) return;
  const int64_t warps = a.T * (a.Hq + 2 * a.Hkv);
  const int wpb = 8;
  const unsigned grid = (unsigned)((warps + wpb - 1) / wpb);
  if (a.D == 128) qkv_rope_kernel<4><<<grid, wpb * 32, 0, st>>>(a);
  else qkv_rope_kernel<2><<<grid, wpb * 32, 0, st>>>(a);
}

}  // namespace b200
