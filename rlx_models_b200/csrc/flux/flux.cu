// FLUX.1 DiT kernels for sm_100a ("K14" adaLN pieces + the DiT QK-norm/RoPE):
//
//   * ln_modulate      LayerNorm without affine (fp32 statistics) followed by
//                      the adaLN modulation (1 + scale[b]) * x + shift[b]; one
//                      CTA per row, the row held in registers (H / 8 threads x
//                      8 values). Reference: rlx-flux1 src/transformer.rs:262-305.
//   * dit_qk_rope      per (row, head): RMSNorm of q and k with learned scales,
//                      half-split RoPE from cos/sin tables indexed by the row's
//                      position in its joint (txt, img) sequence, q written
//                      row-major, k and v into [rows/16, heads, 16, D] pages
//                      that the attention kernel reads with TMA. Query/key rows
//                      are de-interleaved at load so the BFL interleaved-pair
//                      rotation becomes this half split (rlx-flux1
//                      src/weights.rs:202, src/rope.rs:20-78). One warp per
//                      (row, head), D = 128: 4 dims per lane; the partner dim
//                      d +- 64 lives in lane ^ 16.
//
// Rows are "stream-major": all text rows of the batch first (B * Lt), then all
// image rows (B * Li); batch(row) = row < split ? row / r1 : (row - split) / r2
// and the joint position of a row is row % Lt (text) or Lt + (row - split) % Li.
#include <cuda_bf16.h>

#include <algorithm>
#include <stdexcept>

#include "../common/b200.cuh"
#include "../common/launch.h"
#include "../common/pdl_launch.h"

namespace b200 {
namespace flux {

__device__ __forceinline__ int batch_of(int row, int split, int r1, int r2) {
  return row < split ? row / r1 : (row - split) / r2;
}

__device__ __forceinline__ float block_sum(float s, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();  // red[] is reused by consecutive reductions
  if (lane == 0) red[warp] = s;
  __syncthreads();
  float t = 0.f;
  const int nw = (blockDim.x + 31) >> 5;
  for (int i = 0; i < nw; ++i) t += red[i];
  return t;
}

__global__ void ln_modulate_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx, __nv_bfloat16* __restrict__ out,
                                   int64_t ldo, const __nv_bfloat16* __restrict__ mod, int64_t ld_mod, int shift_off,
                                   int scale_off, int H, float eps, int split, int r1, int r2, int row_off) {
  pdl_wait();
  pdl_trigger();
  __shared__ float red[32];
  const int row = blockIdx.x;
  const int c0 = threadIdx.x * 8;
  const bool active = c0 < H;
  float v[8];
  if (active) {
    const uint4 w = *reinterpret_cast<const uint4*>(x + (int64_t)row * ldx + c0);
    const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      v[2 * h] = bf16_lo(ww[h]);
      v[2 * h + 1] = bf16_hi(ww[h]);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = 0.f;
  }
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) s += v[i];
  const float mean = block_sum(s, red) / H;
  float q = 0.f;
  if (active) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float d = v[i] - mean;
      q += d * d;
    }
  }
  const float rstd = rsqrtf(block_sum(q, red) / H + eps);
  if (!active) return;
  const int b = batch_of(row + row_off, split, r1, r2);
  const __nv_bfloat16* m = mod + (int64_t)b * ld_mod;
  const uint4 sh = *reinterpret_cast<const uint4*>(m + shift_off + c0);
  const uint4 sc = *reinterpret_cast<const uint4*>(m + scale_off + c0);
  const uint32_t shw[4] = {sh.x, sh.y, sh.z, sh.w}, scw[4] = {sc.x, sc.y, sc.z, sc.w};
  uint32_t o[4];
#pragma unroll
  for (int h = 0; h < 4; ++h) {
    const float a0 = (v[2 * h] - mean) * rstd * (1.f + bf16_lo(scw[h])) + bf16_lo(shw[h]);
    const float a1 = (v[2 * h + 1] - mean) * rstd * (1.f + bf16_hi(scw[h])) + bf16_hi(shw[h]);
    o[h] = pack_bf16x2(a0, a1);
  }
  *reinterpret_cast<uint4*>(out + (int64_t)row * ldo + c0) = make_uint4(o[0], o[1], o[2], o[3]);
}

// qkv: [rows, 3 * heads * 128] (row stride ld). Scales: [2][128] bf16 per stream
// (q then k), text scales for rows < split, image scales above.
__global__ void dit_qk_rope_kernel(const __nv_bfloat16* __restrict__ qkv, int64_t ld, int rows, int heads,
                                   const __nv_bfloat16* __restrict__ scales_txt,
                                   const __nv_bfloat16* __restrict__ scales_img, const float* __restrict__ cos_t,
                                   const float* __restrict__ sin_t, int split, int Lt, int Li, float eps,
                                   __nv_bfloat16* __restrict__ q_out, __nv_bfloat16* __restrict__ k_pages,
                                   __nv_bfloat16* __restrict__ v_pages, int row_off, int kv_groups) {
  pdl_wait();
  pdl_trigger();
  constexpr int D = 128;
  const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (gw >= (int64_t)rows * heads) return;
  const int row = (int)(gw / heads), head = (int)(gw % heads);
  const int grow = row + row_off;  // row in the global stream-major order
  const int pos = grow < split ? grow % Lt : Lt + (grow - split) % Li;
  const __nv_bfloat16* sc = grow < split ? scales_txt : scales_img;
  const int d0 = lane * 4;
  // rope: dims d < 64 pair with d + 64 (lane ^ 16); angle index d % 64
  const float4 cs = *reinterpret_cast<const float4*>(cos_t + (int64_t)pos * (D / 2) + (d0 & 63));
  const float4 sn = *reinterpret_cast<const float4*>(sin_t + (int64_t)pos * (D / 2) + (d0 & 63));
  const float cc[4] = {cs.x, cs.y, cs.z, cs.w}, ss[4] = {sn.x, sn.y, sn.z, sn.w};
  const bool lo = lane < 16;
  const __nv_bfloat16* src = qkv + (int64_t)row * ld + head * D + d0;
  const int H = heads * D;
  int64_t page, qoff;
  if (kv_groups > 0) {  // [groups][rows][heads per group][D]
    const int hpg = heads / kv_groups;
    page = ((int64_t)(head / hpg) * rows + row) * hpg + head % hpg;
    qoff = page;
  } else {
    page = ((int64_t)(row >> 4) * heads + head) * 16 + (row & 15);
    qoff = (int64_t)row * heads + head;
  }
#pragma unroll
  for (int which = 0; which < 2; ++which) {  // q, k
    const uint2 w = *reinterpret_cast<const uint2*>(src + which * H);
    float x[4] = {bf16_lo(w.x), bf16_hi(w.x), bf16_lo(w.y), bf16_hi(w.y)};
    float ssq = x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ssq += __shfl_xor_sync(0xffffffffu, ssq, o);
    const float r = rsqrtf(ssq / D + eps);
    const uint2 g2 = *reinterpret_cast<const uint2*>(sc + which * D + d0);
    const float g[4] = {bf16_lo(g2.x), bf16_hi(g2.x), bf16_lo(g2.y), bf16_hi(g2.y)};
#pragma unroll
    for (int i = 0; i < 4; ++i) x[i] = x[i] * r * g[i];
    float y[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float partner = __shfl_xor_sync(0xffffffffu, x[i], 16);
      // half split: out[d] = x[d] cos - x[d+64] sin (d < 64); out[d+64] = x[d+64] cos + x[d] sin
      y[i] = lo ? x[i] * cc[i] - partner * ss[i] : x[i] * cc[i] + partner * ss[i];
    }
    const uint2 o = make_uint2(pack_bf16x2(y[0], y[1]), pack_bf16x2(y[2], y[3]));
    if (which == 0)
      *reinterpret_cast<uint2*>(q_out + qoff * D + d0) = o;
    else
      *reinterpret_cast<uint2*>(k_pages + page * D + d0) = o;
  }
  *reinterpret_cast<uint2*>(v_pages + page * D + d0) = *reinterpret_cast<const uint2*>(src + 2 * H);
}

}  // namespace flux

void ln_modulate_launch(const void* x, int64_t ldx, void* out, int64_t ldo, const void* mod, int64_t ld_mod,
                        int shift_off, int scale_off, int rows, int H, float eps, int split, int r1, int r2,
                        int row_off, cudaStream_t st) {
  if (rows == 0) return;
  if (H % 8 != 0 || H / 8 > 1024) throw std::runtime_error("b200.ln_modulate: H % 8 == 0 and H <= 8192");
  const int threads = ((H / 8 + 31) / 32) * 32;
  launch_pdl(flux::ln_modulate_kernel, dim3(rows), dim3(threads), 0, st, reinterpret_cast<const __nv_bfloat16*>(x),
             ldx, reinterpret_cast<__nv_bfloat16*>(out), ldo, reinterpret_cast<const __nv_bfloat16*>(mod), ld_mod,
             shift_off, scale_off, H, eps, split, std::max(1, r1), std::max(1, r2), row_off);
}

void dit_qk_rope_launch(const void* qkv, int64_t ld, int rows, int heads, const void* scales_txt,
                        const void* scales_img, const float* cos_t, const float* sin_t, int split, int Lt, int Li,
                        float eps, void* q_out, void* k_pages, void* v_pages, int row_off, int kv_groups,
                        cudaStream_t st) {
  if (rows == 0) return;
  const int64_t warps = (int64_t)rows * heads;
  launch_pdl(flux::dit_qk_rope_kernel, dim3((unsigned)((warps * 32 + 255) / 256)), dim3(256), 0, st,
             reinterpret_cast<const __nv_bfloat16*>(qkv), ld, rows, heads,
             reinterpret_cast<const __nv_bfloat16*>(scales_txt), reinterpret_cast<const __nv_bfloat16*>(scales_img),
             cos_t, sin_t, split, std::max(1, Lt), std::max(1, Li), eps, reinterpret_cast<__nv_bfloat16*>(q_out),
             reinterpret_cast<__nv_bfloat16*>(k_pages), reinterpret_cast<__nv_bfloat16*>(v_pages), row_off,
             kv_groups);
}

}  // namespace b200
