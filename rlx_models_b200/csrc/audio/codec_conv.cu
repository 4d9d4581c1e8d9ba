// Channels-last 1-D convolutions of the neural audio codecs (DAC, EnCodec) and
// audio front ends (wav2vec 2.0) as
// GEMMs on the tcgen05 linear, with the elementwise work fused into the operand
// producers, plus the LSTM cell of EnCodec's recurrent layers.
//
// act_im2col: x [B, T, C] bf16 -> cols [B * T_out, Kp] bf16,
//     cols[(b, t), j * C + c] = act(x[b, idx(t * stride - pad_l + j * dil), c])
//     act: none | snake(v) = v + sin(alpha[c] v)^2 / (alpha[c] + 1e-9) | elu(v) = v > 0 ? v : exp(v) - 1
//          | gelu(v) = v / 2 (1 + erf(v / sqrt 2))
//     idx(s) = s inside [0, T); outside, zero padding (the column is 0) or
//              reflection (-s on the left, 2 (T - 1) - s on the right)
//   and zeros in columns [k * C, Kp) (Kp = k * C rounded up to 8, the GEMM's
//   16-byte row rule). A convolution is then cols @ W'^T with
//   W'[o, j * C + c] = W[o, c, j]; the activation that precedes every codec
//   conv costs no extra pass over the activations.
//
// convt_fold: the transposed convolution (kernel k = m * stride) as a GEMM
//   Y = x @ W'' ([B * T_in, k * C_out] fp32, W''[j * C_out + o, c] = W[c, o, j])
//   followed by this overlap-add, fused with the bias and the output crop:
//     y[b, u, o] = bias[o] + sum_{q < m} Y[b, t - q, (q * stride + r) * C_out + o]
//     with v = u + pad_l, t = v / stride, r = v % stride, over 0 <= t - q < T_in.
//
// lstm_cell: one time step of an LSTM layer whose gate pre-activations
//   G = x W_ih^T + b_ih + b_hh + h W_hh^T (fp32 [B, 4H], PyTorch gate order
//   i, f, g, o) were accumulated by the GEMMs: c = sig(f) c + sig(i) tanh(g),
//   h = sig(o) tanh(c); h is written in bf16 twice (the next step's GEMM
//   operand and the layer output row).
//
// Reference: the reference's codec layers (crates/rlx-dac/src/ops.rs:3-40 snake,
// ops.rs:159-220 transposed convolution as one sgemm plus a scatter,
// crates/rlx-dac/src/layers.rs:7-60 weight-normalised convolutions;
// crates/rlx-encodec for the SEANet / LSTM codec).
#include <cuda_bf16.h>

#include <cstdint>
#include <stdexcept>

#include "../common/b200.cuh"
#include "../common/launch.h"
#include "../common/pdl_launch.h"

namespace b200 {
namespace codec {

constexpr int kThreads = 256;

enum Act { kNone = 0, kSnake = 1, kElu = 2, kGelu = 3 };

__device__ __forceinline__ float act_f(float v, int act, const float* alpha, int c) {
  if (act == kSnake) {
    const float a = alpha[c];
    const float s = sinf(a * v);
    return v + s * s / (a + 1e-9f);
  }
  if (act == kElu) return v > 0.f ? v : expm1f(v);
  if (act == kGelu) return 0.5f * v * (1.f + erff(v * 0.70710678118654752f));
  return v;
}

// Source time index of a padded position, or -1 for a zero column.
__device__ __forceinline__ int src_t(int ts, int T, bool reflect) {
  if (ts >= 0 && ts < T) return ts;
  if (!reflect) return -1;
  const int r = ts < 0 ? -ts : 2 * (T - 1) - ts;
  return (r >= 0 && r < T) ? r : -1;
}

// C % 8 == 0: one thread per 8 channels of one (row, tap), 16-byte loads and stores.
__global__ void __launch_bounds__(kThreads) im2col_vec_kernel(const __nv_bfloat16* __restrict__ x,
                                                              const float* __restrict__ alpha,
                                                              __nv_bfloat16* __restrict__ cols, int64_t rows,
                                                              int T, int T_out, int C, int k, int stride, int pad,
                                                              int dil, int act, bool reflect) {
  pdl_wait();
  pdl_trigger();
  const int cv = C / 8;
  const int64_t n = rows * k * cv;
  for (int64_t i = blockIdx.x * (int64_t)kThreads + threadIdx.x; i < n; i += (int64_t)gridDim.x * kThreads) {
    const int c8 = (int)(i % cv);
    const int64_t rj = i / cv;
    const int j = (int)(rj % k);
    const int64_t row = rj / k;
    const int b = (int)(row / T_out), t = (int)(row % T_out);
    const int ts = src_t(t * stride - pad + j * dil, T, reflect);
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (ts >= 0) {
      v = *reinterpret_cast<const uint4*>(x + ((int64_t)b * T + ts) * C + c8 * 8);
      if (act != kNone) {
        __nv_bfloat16* e = reinterpret_cast<__nv_bfloat16*>(&v);
#pragma unroll
        for (int q = 0; q < 8; ++q) e[q] = __float2bfloat16(act_f(__bfloat162float(e[q]), act, alpha, c8 * 8 + q));
      }
    }
    *reinterpret_cast<uint4*>(cols + row * (int64_t)k * C + (int64_t)j * C + c8 * 8) = v;
  }
}

// Any C (the stems' single input channel): one thread per output element,
// including the zero padding columns.
__global__ void __launch_bounds__(kThreads) im2col_scalar_kernel(const __nv_bfloat16* __restrict__ x,
                                                                 const float* __restrict__ alpha,
                                                                 __nv_bfloat16* __restrict__ cols, int64_t rows,
                                                                 int Kp, int T, int T_out, int C, int k, int stride,
                                                                 int pad, int dil, int act, bool reflect) {
  pdl_wait();
  pdl_trigger();
  const int64_t n = rows * Kp;
  for (int64_t i = blockIdx.x * (int64_t)kThreads + threadIdx.x; i < n; i += (int64_t)gridDim.x * kThreads) {
    const int col = (int)(i % Kp);
    const int64_t row = i / Kp;
    float v = 0.f;
    if (col < k * C) {
      const int j = col / C, c = col % C;
      const int b = (int)(row / T_out), t = (int)(row % T_out);
      const int ts = src_t(t * stride - pad + j * dil, T, reflect);
      if (ts >= 0) v = act_f(__bfloat162float(x[((int64_t)b * T + ts) * C + c]), act, alpha, c);
    }
    cols[i] = __float2bfloat16(v);
  }
}

__global__ void __launch_bounds__(kThreads) convt_fold_kernel(const float* __restrict__ Y, const float* __restrict__ bias,
                                                              __nv_bfloat16* __restrict__ y, int64_t n, int T_in,
                                                              int T_out, int C_out, int stride, int m, int pad) {
  pdl_wait();
  pdl_trigger();
  const int64_t ycols = (int64_t)m * stride * C_out;
  for (int64_t i = blockIdx.x * (int64_t)kThreads + threadIdx.x; i < n; i += (int64_t)gridDim.x * kThreads) {
    const int o = (int)(i % C_out);
    const int64_t bu = i / C_out;
    const int u = (int)(bu % T_out), b = (int)(bu / T_out);
    const int v = u + pad, t = v / stride, r = v % stride;
    float acc = bias != nullptr ? bias[o] : 0.f;
    for (int q = 0; q < m; ++q) {
      const int ti = t - q;
      if (ti >= 0 && ti < T_in) acc += Y[((int64_t)b * T_in + ti) * ycols + (int64_t)(q * stride + r) * C_out + o];
    }
    y[i] = __float2bfloat16(acc);
  }
}

__global__ void __launch_bounds__(kThreads) lstm_cell_kernel(const float* __restrict__ G, float* __restrict__ c,
                                                             __nv_bfloat16* __restrict__ h, __nv_bfloat16* __restrict__ y,
                                                             int B, int H) {
  pdl_wait();
  pdl_trigger();
  const int64_t n = (int64_t)B * H;
  for (int64_t i = blockIdx.x * (int64_t)kThreads + threadIdx.x; i < n; i += (int64_t)gridDim.x * kThreads) {
    const int b = (int)(i / H), j = (int)(i % H);
    const float* g = G + (int64_t)b * 4 * H;
    const float ig = 1.f / (1.f + expf(-g[j]));
    const float fg = 1.f / (1.f + expf(-g[H + j]));
    const float gg = tanhf(g[2 * H + j]);
    const float og = 1.f / (1.f + expf(-g[3 * H + j]));
    const float cn = fg * c[i] + ig * gg;
    c[i] = cn;
    const __nv_bfloat16 hv = __float2bfloat16(og * tanhf(cn));
    h[i] = hv;
    y[i] = hv;
  }
}

inline unsigned grid_for(int64_t n) {
  const int64_t want = (n + kThreads - 1) / kThreads;
  return (unsigned)(want < 148 * 16 ? (want > 0 ? want : 1) : 148 * 16);
}

}  // namespace codec

void act_im2col_launch(const void* x, const float* alpha, void* cols, int B, int T, int T_out, int C, int Kp, int k,
                       int stride, int pad_l, int dil, int act, bool reflect, cudaStream_t st) {
  const int64_t rows = (int64_t)B * T_out;
  if (rows == 0) return;
  auto* xp = reinterpret_cast<const __nv_bfloat16*>(x);
  auto* cp = reinterpret_cast<__nv_bfloat16*>(cols);
  const bool aligned = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(cols)) & 15u) == 0;
  if (C % 8 == 0 && Kp == k * C && aligned) {
    launch_pdl(codec::im2col_vec_kernel, dim3(codec::grid_for(rows * k * (C / 8))), dim3(codec::kThreads), 0, st, xp,
               alpha, cp, rows, T, T_out, C, k, stride, pad_l, dil, act, reflect);
  } else {
    launch_pdl(codec::im2col_scalar_kernel, dim3(codec::grid_for(rows * Kp)), dim3(codec::kThreads), 0, st, xp, alpha,
               cp, rows, Kp, T, T_out, C, k, stride, pad_l, dil, act, reflect);
  }
}

void convt_fold_launch(const float* Y, const float* bias, void* y, int B, int T_in, int T_out, int C_out, int stride,
                       int m, int pad, cudaStream_t st) {
  const int64_t n = (int64_t)B * T_out * C_out;
  if (n == 0) return;
  launch_pdl(codec::convt_fold_kernel, dim3(codec::grid_for(n)), dim3(codec::kThreads), 0, st, Y, bias,
             reinterpret_cast<__nv_bfloat16*>(y), n, T_in, T_out, C_out, stride, m, pad);
}

void lstm_cell_launch(const float* G, float* c, void* h, void* y, int B, int H, cudaStream_t st) {
  const int64_t n = (int64_t)B * H;
  if (n == 0) return;
  launch_pdl(codec::lstm_cell_kernel, dim3(codec::grid_for(n)), dim3(codec::kThreads), 0, st, G, c,
             reinterpret_cast<__nv_bfloat16*>(h), reinterpret_cast<__nv_bfloat16*>(y), B, H);
}

}  // namespace b200
