// Gated DeltaNet decode step (Qwen3.5 linear-attention layers), one fused
// kernel per layer and step:
//
//   conv1d step over the q / k / v channels (window of K-1 inputs per
//   channel, double-buffered by position parity), SiLU, l2norm of q and k,
//   q *= dk^-1/2, log decay g = -exp(A_log) * softplus(a + dt_bias),
//   beta = sigmoid(b), the delta-rule update of the fp32 state
//   S <- exp(g) S + k u^T with u = beta (v - exp(g) S^T k), o = S^T q, and the
//   gated RMSNorm rmsnorm(o) * w * silu(z) that feeds out_proj.
//
// Grid (B, Hv), one CTA per (sequence, value head), DV threads: thread t owns
// state column t (DK fp32 values kept in registers across the update), so the
// state streams through HBM once per step (read + write of DK x DV fp32).
// Value heads that share a key head compute the same q / k conv outputs; only
// the first of them advances the q / k conv windows, and it writes them to the
// other parity buffer, so the readers of this step never see a half-updated
// window.
//
// Reference behaviour: transformers qwen3_5 Qwen3_5GatedDeltaNet (recurrent
// path) and the family in crates/rlx-qwen35.
//
// The KDA instantiation (Kimi Delta Attention: Kimi-Linear, Ling 3) differs in
// two places: the log decay is per key channel, g_i = -exp(A_log) *
// softplus(a_i + dt_bias_i) with a the Hv*D logits at the end of the row, so
// the state update scales row i of S by exp(g_i); and the output gate is
// sigmoid(z) instead of silu(z). Key and value heads are the same heads.
// Reference behaviour: crates/rlx-models-core/src/standard_decoder.rs
// build_kimi_kda (lines 11527-11680).
#include <cuda_bf16.h>

#include <cstdint>
#include <stdexcept>

#include "../common/b200.cuh"
#include "../common/launch.h"
#include "../common/pdl_launch.h"

namespace b200 {
namespace gdn {

constexpr int kMaxK = 8;

template <int NT>
__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();  // red reuse across calls
  if (l == 0) red[w] = v;
  __syncthreads();
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < NT / 32; ++i) s += red[i];
  return s;
}

__device__ __forceinline__ float bf(const __nv_bfloat16 x) { return __bfloat162float(x); }
__device__ __forceinline__ float rbf(float x) { return __bfloat162float(__float2bfloat16(x)); }
__device__ __forceinline__ float silu(float x) { return x / (1.f + __expf(-x)); }

// One conv1d step of channel c: window (K-1 previous inputs) + the new input.
__device__ __forceinline__ float conv_step(const GdnDecodeArgs& a, const __nv_bfloat16* row, int64_t slot, int par,
                                           int c, bool advance) {
  const int W = a.K - 1;
  const __nv_bfloat16* win = a.conv_state + ((slot * 2 + par) * a.conv_dim + c) * W;
  __nv_bfloat16* nxt = a.conv_state + ((slot * 2 + (par ^ 1)) * a.conv_dim + c) * W;
  float xs[kMaxK];
#pragma unroll
  for (int i = 0; i < kMaxK; ++i) xs[i] = 0.f;
  for (int i = 0; i < W; ++i) xs[i] = bf(win[i]);
  xs[W] = bf(row[c]);
  float acc = 0.f;
  for (int i = 0; i <= W; ++i) acc += a.conv_w[(int64_t)c * a.K + i] * xs[i];
  if (advance)
    for (int i = 0; i < W; ++i) nxt[i] = __float2bfloat16(xs[i + 1]);
  return rbf(silu(acc));  // the conv output is a bf16 activation
}

template <int D, bool KDA>
__global__ void __launch_bounds__(D) gdn_decode_kernel(GdnDecodeArgs a) {
  __shared__ float qs[D], ks[D], gs[KDA ? D : 1];
  __shared__ float red[D / 32];
  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.x, hv = blockIdx.y, t = threadIdx.x;
  const int64_t slot = a.seq_slots[b];
  __nv_bfloat16* out = a.out + ((int64_t)b * a.Hv + hv) * D + t;
  if (slot < 0 || slot >= a.num_slots) {  // a padding row without a state slot
    *out = __float2bfloat16(0.f);
    return;
  }
  const int par = a.positions[b] & 1;
  const int rep = a.Hv / a.Hk;
  const int kh = hv / rep;
  const bool owner = (hv % rep) == 0;
  const __nv_bfloat16* row = a.proj + (int64_t)b * a.ld;

  float q = conv_step(a, row, slot, par, kh * D + t, owner);
  float k = conv_step(a, row, slot, par, a.key_dim + kh * D + t, owner);
  const float v = conv_step(a, row, slot, par, 2 * a.key_dim + hv * D + t, true);
  const float qn = rsqrtf(block_sum<D>(q * q, red) + 1e-6f);
  const float kn = rsqrtf(block_sum<D>(k * k, red) + 1e-6f);
  qs[t] = q * qn * rsqrtf((float)D);
  ks[t] = k * kn;
  const float zb = bf(row[a.conv_dim + hv * D + t]);
  const float bb = bf(row[a.conv_dim + a.value_dim + hv]);
  float decay;
  if constexpr (KDA) {  // per key channel: this thread computes channel t's decay for the whole CTA
    const float ab = bf(row[a.conv_dim + a.value_dim + a.Hv + hv * D + t]);
    const float xa = ab + a.dt_bias[hv * D + t];
    const float softplus = xa > 20.f ? xa : log1pf(__expf(xa));
    gs[t] = __expf(-__expf(a.A_log[hv]) * softplus);
    decay = 1.f;
  } else {
    const float ab = bf(row[a.conv_dim + a.value_dim + a.Hv + hv]);
    const float xa = ab + a.dt_bias[hv];
    const float softplus = xa > 20.f ? xa : log1pf(__expf(xa));
    decay = __expf(-__expf(a.A_log[hv]) * softplus);
  }
  const float beta = 1.f / (1.f + __expf(-bb));
  __syncthreads();

  float* S = a.rec_state + ((slot * a.Hv + hv) * (int64_t)D) * D + t;  // column t of [D, D]
  float s[D];
  float kv = 0.f;
#pragma unroll
  for (int i = 0; i < D; ++i) {
    s[i] = S[(int64_t)i * D] * (KDA ? gs[i] : decay);
    kv += s[i] * ks[i];
  }
  const float u = beta * (v - kv);
  float o = 0.f;
#pragma unroll
  for (int i = 0; i < D; ++i) {
    s[i] += ks[i] * u;
    o += s[i] * qs[i];
    S[(int64_t)i * D] = s[i];
  }
  o = rbf(o);
  const float inv = rsqrtf(block_sum<D>(o * o, red) / (float)D + a.eps);
  const float gate = KDA ? 1.f / (1.f + __expf(-zb)) : silu(zb);
  *out = __float2bfloat16(rbf(o * inv) * a.norm_w[t] * gate);
}

}  // namespace gdn

void gdn_decode_launch(const GdnDecodeArgs& a, cudaStream_t st) {
  if (a.B == 0) return;
  if (a.K < 2 || a.K > gdn::kMaxK) throw std::runtime_error("b200.gdn_decode: conv kernel 2..8");
  if (a.Hv % a.Hk != 0) throw std::runtime_error("b200.gdn_decode: value heads must be a multiple of key heads");
  dim3 grid(a.B, a.Hv);
  if (a.kda && a.Hk != a.Hv) throw std::runtime_error("b200.kda_decode: key heads == value heads");
  if (a.D == 128 && a.kda) launch_pdl(gdn::gdn_decode_kernel<128, true>, grid, dim3(128), 0, st, a);
  else if (a.D == 64 && a.kda) launch_pdl(gdn::gdn_decode_kernel<64, true>, grid, dim3(64), 0, st, a);
  else if (a.D == 128) launch_pdl(gdn::gdn_decode_kernel<128, false>, grid, dim3(128), 0, st, a);
  else if (a.D == 64) launch_pdl(gdn::gdn_decode_kernel<64, false>, grid, dim3(64), 0, st, a);
  else throw std::runtime_error("b200.gdn_decode: head dims 64 or 128 (key == value)");
}

}  // namespace b200

// ---------------------------------------------------------------------------
// LFM2 short-convolution decode step: per (row, channel c)
//   bx = B[c] * x[c];  y = C[c] * (sum_i w[c][i] * [window | bx][i] (+ bias[c]))
// with the window (K-1 previous bx values) read from parity pos & 1 and the
// advanced window written to the other parity (no activation).
// ---------------------------------------------------------------------------
namespace b200 {
namespace shortconv {

__global__ void shortconv_decode_kernel(ShortConvArgs a) {
  pdl_wait();
  pdl_trigger();
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (int64_t)a.B * a.H) return;
  const int b = (int)(idx / a.H), c = (int)(idx % a.H);
  const int64_t slot = a.seq_slots[b];
  __nv_bfloat16* out = a.out + (int64_t)b * a.H + c;
  if (slot < 0 || slot >= a.num_slots) {
    *out = __float2bfloat16(0.f);
    return;
  }
  const __nv_bfloat16* row = a.proj + (int64_t)b * a.ld;
  const float bv = __bfloat162float(row[c]), cv = __bfloat162float(row[a.H + c]),
              xv = __bfloat162float(row[2 * a.H + c]);
  const float bx = __bfloat162float(__float2bfloat16(bv * xv));  // B * x is a bf16 activation
  const int W = a.K - 1, par = a.positions[b] & 1;
  const __nv_bfloat16* win = a.conv_state + ((slot * 2 + par) * a.H + c) * W;
  __nv_bfloat16* nxt = a.conv_state + ((slot * 2 + (par ^ 1)) * a.H + c) * W;
  float acc = a.bias != nullptr ? a.bias[c] : 0.f;
  float prev[8];
  for (int i = 0; i < W; ++i) {
    prev[i] = __bfloat162float(win[i]);
    acc += a.w[(int64_t)c * a.K + i] * prev[i];
  }
  acc += a.w[(int64_t)c * a.K + W] * bx;
  for (int i = 0; i + 1 < W; ++i) nxt[i] = __float2bfloat16(prev[i + 1]);
  nxt[W - 1] = __float2bfloat16(bx);
  *out = __float2bfloat16(cv * __bfloat162float(__float2bfloat16(acc)));
}

}  // namespace shortconv

void shortconv_decode_launch(const ShortConvArgs& a, cudaStream_t st) {
  if (a.B == 0) return;
  if (a.K < 2 || a.K > 9) throw std::runtime_error("b200.shortconv_decode: kernel size 2..9");
  const int64_t n = (int64_t)a.B * a.H;
  launch_pdl(shortconv::shortconv_decode_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, st, a);
}

}  // namespace b200

// ---------------------------------------------------------------------------
// Mamba-2 (SSD) decode step: per (sequence, head h of group g = h / (H / G)):
//   conv1d step (+ bias, SiLU) over the head's P x channels and the group's
//   N B and N C channels; dt = clamp(softplus(dt_raw + dt_bias)); dA = exp(dt A)
//   S[n, p] <- dA S[n, p] + dt x[p] B[n];  y[p] = sum_n S[n, p] C[n] + D x[p]
// One CTA of P threads per (sequence, head); thread p keeps state column p
// (N fp32 values) in registers. The first head of a group advances the
// group's B / C conv windows (written to the other parity buffer).
// ---------------------------------------------------------------------------
namespace b200 {
namespace ssd {

__device__ __forceinline__ float conv_ch(const SsdDecodeArgs& a, const __nv_bfloat16* row, int64_t slot, int par,
                                         int c, bool advance) {
  const int W = a.K - 1;
  const __nv_bfloat16* win = a.conv_state + ((slot * 2 + par) * a.conv_dim + c) * W;
  __nv_bfloat16* nxt = a.conv_state + ((slot * 2 + (par ^ 1)) * a.conv_dim + c) * W;
  const float xin = __bfloat162float(row[a.xbc_off + c]);
  float acc = a.conv_b != nullptr ? a.conv_b[c] : 0.f;
  float prev[8];
  for (int i = 0; i < W; ++i) {
    prev[i] = __bfloat162float(win[i]);
    acc += a.conv_w[(int64_t)c * a.K + i] * prev[i];
  }
  acc += a.conv_w[(int64_t)c * a.K + W] * xin;
  if (advance) {
    for (int i = 0; i + 1 < W; ++i) nxt[i] = __float2bfloat16(prev[i + 1]);
    nxt[W - 1] = __float2bfloat16(xin);
  }
  return __bfloat162float(__float2bfloat16(acc / (1.f + __expf(-acc))));
}

template <int N, int P>
__global__ void __launch_bounds__(P) ssd_decode_kernel(SsdDecodeArgs a) {
  __shared__ float Bs[N], Cs[N];
  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.x, h = blockIdx.y, t = threadIdx.x;
  const int64_t slot = a.seq_slots[b];
  __nv_bfloat16* out = a.out + ((int64_t)b * a.H + h) * P + t;
  if (slot < 0 || slot >= a.num_slots) {
    *out = __float2bfloat16(0.f);
    return;
  }
  const int par = a.positions[b] & 1;
  const int hpg = a.H / a.G, g = h / hpg;
  const bool owner = (h % hpg) == 0;
  const __nv_bfloat16* row = a.proj + (int64_t)b * a.ld;
  const int I = a.H * P;
  const float x = conv_ch(a, row, slot, par, h * P + t, true);
  for (int n = t; n < N; n += P) {
    Bs[n] = conv_ch(a, row, slot, par, I + g * N + n, owner);
    Cs[n] = conv_ch(a, row, slot, par, I + a.G * N + g * N + n, owner);
  }
  const float dr = __bfloat162float(row[a.dt_off + h]) + a.dt_bias[h];
  float dt = dr > 20.f ? dr : log1pf(__expf(dr));
  dt = fminf(fmaxf(dt, a.dt_min), a.dt_max);
  const float dA = __expf(-__expf(a.A_log[h]) * dt);
  __syncthreads();
  float* S = a.ssm_state + ((slot * a.H + h) * (int64_t)N) * P + t;  // column t of [N, P]
  const float dx = dt * x;
  float y = 0.f;
#pragma unroll
  for (int n = 0; n < N; ++n) {
    const float s = S[(int64_t)n * P] * dA + dx * Bs[n];
    S[(int64_t)n * P] = s;
    y += s * Cs[n];
  }
  *out = __float2bfloat16(y + a.D[h] * x);
}

}  // namespace ssd

void ssd_decode_launch(const SsdDecodeArgs& a, cudaStream_t st) {
  if (a.B == 0) return;
  if (a.K < 2 || a.K > 9) throw std::runtime_error("b200.ssd_decode: conv kernel 2..9");
  if (a.H % a.G != 0) throw std::runtime_error("b200.ssd_decode: heads must be a multiple of groups");
  dim3 grid(a.B, a.H);
  if (a.N == 128 && a.P == 64) launch_pdl(ssd::ssd_decode_kernel<128, 64>, grid, dim3(64), 0, st, a);
  else if (a.N == 64 && a.P == 64) launch_pdl(ssd::ssd_decode_kernel<64, 64>, grid, dim3(64), 0, st, a);
  else if (a.N == 128 && a.P == 128) launch_pdl(ssd::ssd_decode_kernel<128, 128>, grid, dim3(128), 0, st, a);
  else if (a.N == 16 && a.P == 32) launch_pdl(ssd::ssd_decode_kernel<16, 32>, grid, dim3(32), 0, st, a);
  else throw std::runtime_error("b200.ssd_decode: (state, head_dim) in {(128, 64), (64, 64), (128, 128), (16, 32)}");
}

}  // namespace b200

// ---------------------------------------------------------------------------
// Mamba-1 (selective scan), prefill and decode in the same two kernels. The
// step's tokens are grouped by sequence (cu offsets, decode sequences hold one
// token); a sequence whose first token sits at position 0 starts from zero
// state, otherwise from its slot's saved state. One thread per channel walks
// its sequence in time order, so a channel's conv window and SSM state stay in
// registers across the sequence and each slot row has exactly one writer.
//   conv:  x = silu(conv1d(x_raw) + bias)          (window of K-1 raw inputs)
//   scan:  dt = softplus(dt_raw + dt_bias); h[n] = exp(dt A[n]) h[n] + dt B[n] x
//          y = (sum_n h[n] C[n] + D x) * silu(z)
// ---------------------------------------------------------------------------
namespace b200 {
namespace mamba1 {

__global__ void mamba_conv_kernel(MambaScanArgs a) {
  pdl_wait();
  pdl_trigger();
  const int s = blockIdx.x;
  const int d = blockIdx.y * blockDim.x + threadIdx.x;
  if (d >= a.Di) return;
  const int t0 = a.cu[s], t1 = a.cu[s + 1];
  if (t1 <= t0) return;
  const int64_t slot = a.slots[s];
  const bool fresh = a.positions[t0] == 0;
  const int W = a.K - 1;
  const bool has_slot = slot >= 0 && slot < a.num_slots;
  __nv_bfloat16* win = has_slot ? a.conv_state + (slot * a.Di + d) * W : nullptr;
  float w[8], prev[8];
  for (int i = 0; i < a.K; ++i) w[i] = a.conv_w[(int64_t)d * a.K + i];
  for (int i = 0; i < W; ++i) prev[i] = (fresh || !has_slot) ? 0.f : __bfloat162float(win[i]);
  const float bias = a.conv_b != nullptr ? a.conv_b[d] : 0.f;
  for (int t = t0; t < t1; ++t) {
    const float xin = __bfloat162float(a.x_raw[(int64_t)t * a.ld_raw + d]);
    float acc = bias + w[W] * xin;
    for (int i = 0; i < W; ++i) acc += w[i] * prev[i];
    for (int i = 0; i + 1 < W; ++i) prev[i] = prev[i + 1];
    prev[W - 1] = xin;
    a.x_out[(int64_t)t * a.Di + d] = __float2bfloat16(acc / (1.f + __expf(-acc)));
  }
  if (has_slot)
    for (int i = 0; i < W; ++i) win[i] = __float2bfloat16(prev[i]);
}

template <int N>
__global__ void mamba_scan_kernel(MambaScanArgs a) {
  pdl_wait();
  pdl_trigger();
  const int s = blockIdx.x;
  const int d = blockIdx.y * blockDim.x + threadIdx.x;
  if (d >= a.Di) return;
  const int t0 = a.cu[s], t1 = a.cu[s + 1];
  if (t1 <= t0) return;
  const int64_t slot = a.slots[s];
  const bool has_slot = slot >= 0 && slot < a.num_slots;
  const bool fresh = a.positions[t0] == 0 || !has_slot;
  float* st = has_slot ? a.ssm_state + (slot * a.Di + d) * N : nullptr;
  float h[N], A[N];
#pragma unroll
  for (int n = 0; n < N; ++n) {
    h[n] = fresh ? 0.f : st[n];
    A[n] = -__expf(a.A_log[(int64_t)d * N + n]);
  }
  const float Dd = a.D[d], db = a.dt_bias[d];
  for (int t = t0; t < t1; ++t) {
    const float x = __bfloat162float(a.x_out[(int64_t)t * a.Di + d]);
    const float r = __bfloat162float(a.dt[(int64_t)t * a.ld_dt + d]) + db;
    const float dt = r > 20.f ? r : log1pf(__expf(r));
    const __nv_bfloat16* Bt = a.Bc + (int64_t)t * a.ld_bc;
    const __nv_bfloat16* Ct = Bt + a.c_off;
    float y = 0.f;
#pragma unroll
    for (int n = 0; n < N; ++n) {
      h[n] = __expf(dt * A[n]) * h[n] + dt * __bfloat162float(Bt[n]) * x;
      y += h[n] * __bfloat162float(Ct[n]);
    }
    const float z = __bfloat162float(a.z[(int64_t)t * a.ld_z + d]);
    a.y[(int64_t)t * a.Di + d] = __float2bfloat16((y + Dd * x) * (z / (1.f + __expf(-z))));
  }
  if (has_slot)
#pragma unroll
    for (int n = 0; n < N; ++n) st[n] = h[n];
}

}  // namespace mamba1

void mamba_conv_launch(const MambaScanArgs& a, cudaStream_t st) {
  if (a.nseq == 0) return;
  if (a.K < 2 || a.K > 8) throw std::runtime_error("b200.mamba_conv: conv kernel 2..8");
  launch_pdl(mamba1::mamba_conv_kernel, dim3(a.nseq, (a.Di + 127) / 128), dim3(128), 0, st, a);
}

void mamba_scan_launch(const MambaScanArgs& a, cudaStream_t st) {
  if (a.nseq == 0) return;
  dim3 grid(a.nseq, (a.Di + 127) / 128);
  if (a.N == 16) launch_pdl(mamba1::mamba_scan_kernel<16>, grid, dim3(128), 0, st, a);
  else if (a.N == 8) launch_pdl(mamba1::mamba_scan_kernel<8>, grid, dim3(128), 0, st, a);
  else throw std::runtime_error("b200.mamba_scan: state size 8 or 16");
}

}  // namespace b200
