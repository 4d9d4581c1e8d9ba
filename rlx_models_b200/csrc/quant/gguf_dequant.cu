// GGUF block dequantisation on the device: ggml legacy quants (Q4_0, Q4_1,
// Q5_0, Q5_1, Q8_0) and K-quants (Q2_K, Q3_K, Q4_K, Q5_K, Q6_K, Q8_K) ->
// bf16 or fp32, one thread per output element (adjacent threads write
// adjacent elements; a block's scale bytes are re-read from L1). Used when a
// GGUF checkpoint is loaded onto the GPU: the quantised bytes cross PCIe and
// expand in HBM, after which the tcgen05 GEMMs run on bf16 weights.
//
// The block layouts are the GGUF file format's (weights/gguf.py documents and
// tests them against an independent implementation); every formula here
// matches weights/gguf.py `dequantize_blocks`, which the GPU test compares
// bit for bit.
//
// Reference: the reference's GGUF K-quant dequant matmul is an external
// NVRTC kernel (README.md:1266, RLX_CUDA_Q4K_GEMV_COOP); its GGUF type table
// is rlx-models-core src/weight_loader.rs:497-554.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <stdexcept>
#include <string>

#include "../common/b200.cuh"
#include "../common/launch.h"
#include "../common/pdl_launch.h"

namespace b200 {
namespace gguf {

enum Kind : int { Q4_0 = 2, Q4_1 = 3, Q5_0 = 6, Q5_1 = 7, Q8_0 = 8, Q2_K = 10, Q3_K = 11, Q4_K = 12, Q5_K = 13,
                  Q6_K = 14, Q8_K = 15 };

__device__ __forceinline__ float h16(const uint8_t* p) {
  return __half2float(__ushort_as_half((unsigned short)(p[0] | (p[1] << 8))));
}

// six-bit (scale, min) pair `j` of the 12 packed bytes of a Q4_K / Q5_K block
__device__ __forceinline__ void k4_scale_min(const uint8_t* s, int j, float& sc, float& mn) {
  if (j < 4) {
    sc = (float)(s[j] & 63);
    mn = (float)(s[j + 4] & 63);
  } else {
    sc = (float)((s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4));
    mn = (float)((s[j + 4] >> 4) | ((s[j] >> 6) << 4));
  }
}

// six-bit scale `i` (0..15) of a Q3_K block, minus 32
__device__ __forceinline__ float q3k_scale(const uint8_t* s, int i) {
  const int k = i & 3;
  const int hi = (s[8 + k] >> (2 * (i >> 2))) & 3;
  const int lo = (i < 8) ? (s[i] & 0xF) : (s[i - 8] >> 4);
  return (float)((lo | (hi << 4)) - 32);
}

template <int KIND>
__device__ __forceinline__ float deq(const uint8_t* b, int j) {
  if constexpr (KIND == Q4_0 || KIND == Q4_1) {
    const int off = KIND == Q4_0 ? 2 : 4;
    const int q = j < 16 ? (b[off + j] & 0xF) : (b[off + j - 16] >> 4);
    return KIND == Q4_0 ? (float)(q - 8) * h16(b) : (float)q * h16(b) + h16(b + 2);
  } else if constexpr (KIND == Q5_0 || KIND == Q5_1) {
    const int off = KIND == Q5_0 ? 2 : 4;
    const uint32_t qh = (uint32_t)b[off] | ((uint32_t)b[off + 1] << 8) | ((uint32_t)b[off + 2] << 16) |
                        ((uint32_t)b[off + 3] << 24);
    const int nib = j < 16 ? (b[off + 4 + j] & 0xF) : (b[off + 4 + j - 16] >> 4);
    const int q = nib | (((qh >> j) & 1) << 4);
    return KIND == Q5_0 ? (float)(q - 16) * h16(b) : (float)q * h16(b) + h16(b + 2);
  } else if constexpr (KIND == Q8_0) {
    return (float)(int8_t)b[2 + j] * h16(b);
  } else if constexpr (KIND == Q8_K) {
    return (float)(int8_t)b[4 + j] * *reinterpret_cast<const float*>(b);
  } else if constexpr (KIND == Q2_K || KIND == Q3_K) {
    const int n = j >> 7, r = j & 127, s = r >> 5, h = (r >> 4) & 1, l = r & 15;
    const int is = n * 8 + s * 2 + h;
    if constexpr (KIND == Q2_K) {
      const int q = (b[16 + n * 32 + h * 16 + l] >> (2 * s)) & 3;
      const int sc = b[is];
      return h16(b + 80) * (float)(sc & 0xF) * (float)q - h16(b + 82) * (float)(sc >> 4);
    } else {
      const int q = (b[32 + n * 32 + h * 16 + l] >> (2 * s)) & 3;
      const int hb = (b[h * 16 + l] >> (4 * n + s)) & 1;
      return h16(b + 108) * q3k_scale(b + 96, is) * (float)(q - (hb ? 0 : 4));
    }
  } else if constexpr (KIND == Q4_K || KIND == Q5_K) {
    const int p = j >> 6, hi = (j >> 5) & 1, l = j & 31;
    float sc, mn;
    k4_scale_min(b + 4, 2 * p + hi, sc, mn);
    int q;
    if constexpr (KIND == Q4_K) {
      const int byte = b[16 + p * 32 + l];
      q = hi ? (byte >> 4) : (byte & 0xF);
    } else {
      const int byte = b[48 + p * 32 + l];
      q = (hi ? (byte >> 4) : (byte & 0xF)) + (((b[16 + l] >> (2 * p + hi)) & 1) << 4);
    }
    return h16(b) * sc * (float)q - h16(b + 2) * mn;
  } else {  // Q6_K
    const int n = j >> 7, r = j & 127, qq = r >> 5, l = r & 31;
    const uint8_t* ql = b + n * 64;
    const int qh = b[128 + n * 32 + l];
    const int lo = (qq & 1) ? ql[l + 32] : ql[l];
    const int nib = (qq & 2) ? (lo >> 4) : (lo & 0xF);
    const int q = (nib | (((qh >> (2 * qq)) & 3) << 4)) - 32;
    const float sc = (float)(int8_t)b[192 + n * 8 + (l >> 4) + 2 * qq];
    return h16(b + 208) * sc * (float)q;
  }
}

template <int KIND, int BE, int BB, typename T>
__global__ void dequant_kernel(const uint8_t* __restrict__ raw, int64_t n, T* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    const float v = deq<KIND>(raw + (i / BE) * BB, (int)(i % BE));
    if constexpr (sizeof(T) == 2) out[i] = __float2bfloat16(v);
    else out[i] = v;
  }
}

template <int KIND, int BE, int BB>
void go(const void* raw, int64_t n, void* out, bool f32, cudaStream_t st) {
  const int threads = 256;
  const int blocks = (int)std::min<int64_t>((n + threads - 1) / threads, 148 * 32);
  const auto* r = reinterpret_cast<const uint8_t*>(raw);
  if (f32)
    launch_pdl(dequant_kernel<KIND, BE, BB, float>, dim3(blocks), dim3(threads), 0, st, r, n,
               reinterpret_cast<float*>(out));
  else
    launch_pdl(dequant_kernel<KIND, BE, BB, __nv_bfloat16>, dim3(blocks), dim3(threads), 0, st, r, n,
               reinterpret_cast<__nv_bfloat16*>(out));
}

}  // namespace gguf

void gguf_dequant_launch(const void* raw, int ggml_type, int64_t n, void* out, bool out_f32, cudaStream_t st) {
  using namespace gguf;
  if (n == 0) return;
  switch (ggml_type) {
    case Q4_0: return go<Q4_0, 32, 18>(raw, n, out, out_f32, st);
    case Q4_1: return go<Q4_1, 32, 20>(raw, n, out, out_f32, st);
    case Q5_0: return go<Q5_0, 32, 22>(raw, n, out, out_f32, st);
    case Q5_1: return go<Q5_1, 32, 24>(raw, n, out, out_f32, st);
    case Q8_0: return go<Q8_0, 32, 34>(raw, n, out, out_f32, st);
    case Q2_K: return go<Q2_K, 256, 84>(raw, n, out, out_f32, st);
    case Q3_K: return go<Q3_K, 256, 110>(raw, n, out, out_f32, st);
    case Q4_K: return go<Q4_K, 256, 144>(raw, n, out, out_f32, st);
    case Q5_K: return go<Q5_K, 256, 176>(raw, n, out, out_f32, st);
    case Q6_K: return go<Q6_K, 256, 210>(raw, n, out, out_f32, st);
    case Q8_K: return go<Q8_K, 256, 292>(raw, n, out, out_f32, st);
    default: throw std::runtime_error("b200.gguf_dequant: unsupported ggml type " + std::to_string(ggml_type));
  }
}

}  // namespace b200
