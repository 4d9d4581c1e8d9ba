// On-GPU token selection ("K13"): greedy argmax and temperature / top-k /
// top-p / min-p sampling over a [B, V] fp32 logits matrix, one CTA per row.
//
// Sampling uses the Gumbel-max identity: argmax_i(x_i / T + G_i) with i.i.d.
// standard Gumbel noise G_i is an exact draw from softmax(x / T), and
// restricting the argmax to a candidate set is an exact draw from the
// renormalised distribution over that set. Candidate sets are thresholds in
// logit space:
//   * top-k: the k-th largest logit, found by an MSB-first 8-bit radix select
//     over order-preserving uint32 keys (4 passes over the L2-resident row);
//   * top-p: the largest threshold whose retained probability mass (within the
//     top-k set, as HF applies top-k before top-p) reaches p, found by the same
//     radix walk with per-bin probability mass instead of counts;
//   * min-p: x / T >= max / T + log(min_p).
// Noise comes from SplitMix64 (Steele, Lea, Flood 2014) of (seed, counter,
// token), so a (seed, counter) pair replays the same draw.
//
// The reference samples on the host (rlx-qwen3 src/sampling.rs:41-400).
#include <cuda_runtime.h>

#include <cfloat>
#include <cstdint>

#include "../common/b200.cuh"
#include "../common/launch.h"
#include "../common/pdl_launch.h"

namespace b200 {
namespace smp {

constexpr int kThreads = 1024;

__device__ __forceinline__ uint32_t fkey(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float kfloat(uint32_t k) {
  const uint32_t u = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
  return __uint_as_float(u);
}

__device__ __forceinline__ uint64_t splitmix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

__device__ __forceinline__ float gumbel(uint64_t seed, uint64_t ctr, uint64_t i) {
  const uint64_t h = splitmix64(seed ^ splitmix64(ctr * 0x632BE59BD9B4E019ull + i));
  const float u = ((float)(h >> 40) + 0.5f) * (1.0f / 16777216.0f);  // (0, 1)
  return -logf(-logf(u));
}

// block-wide reductions (kThreads threads)
__device__ __forceinline__ float block_max(float v, float* sh) {
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) sh[w] = v;
  __syncthreads();
  v = (threadIdx.x < kThreads / 32) ? sh[threadIdx.x] : -FLT_MAX;
  if (w == 0)
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  if (threadIdx.x == 0) sh[0] = v;
  __syncthreads();
  return sh[0];
}
__device__ __forceinline__ float block_sum(float v, float* sh) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) sh[w] = v;
  __syncthreads();
  v = (threadIdx.x < kThreads / 32) ? sh[threadIdx.x] : 0.f;
  if (w == 0)
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if (threadIdx.x == 0) sh[0] = v;
  __syncthreads();
  return sh[0];
}
// (value, index) argmax; ties -> smallest index
__device__ __forceinline__ void block_argmax(float& v, int& idx, float* shv, int* shi) {
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
    if (ov > v || (ov == v && oi < idx)) {
      v = ov;
      idx = oi;
    }
  }
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) {
    shv[w] = v;
    shi[w] = idx;
  }
  __syncthreads();
  if (w == 0) {
    v = (l < kThreads / 32) ? shv[l] : -FLT_MAX;
    idx = (l < kThreads / 32) ? shi[l] : 0x7fffffff;
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, v, o);
      const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
      if (ov > v || (ov == v && oi < idx)) {
        v = ov;
        idx = oi;
      }
    }
    if (l == 0) {
      shv[0] = v;
      shi[0] = idx;
    }
  }
  __syncthreads();
  v = shv[0];
  idx = shi[0];
}

__global__ void __launch_bounds__(kThreads) argmax_kernel(const float* __restrict__ logits, int64_t ld, int64_t V,
                                                          int32_t* __restrict__ out) {
  __shared__ float shv[32];
  __shared__ int shi[32];
  pdl_wait();
  pdl_trigger();
  const float* x = logits + (int64_t)blockIdx.x * ld;
  float best = -FLT_MAX;
  int bi = 0x7fffffff;
  for (int64_t i = threadIdx.x; i < V; i += kThreads) {
    const float v = x[i];
    if (v > best) {
      best = v;
      bi = (int)i;
    }
  }
  block_argmax(best, bi, shv, shi);
  if (threadIdx.x == 0) out[blockIdx.x] = bi == 0x7fffffff ? 0 : bi;
}

// Radix walk over keys >= lo_key (MSB first). mode 0: find the key of the
// `target`-th largest element (counts); mode 1: find the largest threshold key
// whose retained mass sum(exp(x/T - mx)) over keys >= threshold reaches target.
__device__ uint32_t radix_select(const float* x, int64_t V, uint32_t lo_key, float target, int mode, float inv_t,
                                 float mx, float* hist) {
  uint32_t prefix = 0, mask = 0;
  float remaining = target;
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = threadIdx.x; i < 256; i += kThreads) hist[i] = 0.f;
    __syncthreads();
    for (int64_t i = threadIdx.x; i < V; i += kThreads) {
      const float v = x[i];
      const uint32_t k = fkey(v);
      if (k >= lo_key && (k & mask) == prefix) {
        const float w = mode == 0 ? 1.f : __expf(v * inv_t - mx);
        atomicAdd(&hist[(k >> shift) & 255u], w);
      }
    }
    __syncthreads();
    // scan bins from the top (single thread: 256 bins)
    __shared__ uint32_t s_bin;
    __shared__ float s_rem;
    if (threadIdx.x == 0) {
      float acc = 0.f;
      int bin = 0;
      for (int bb = 255; bb >= 0; --bb) {
        if (acc + hist[bb] >= remaining) {
          bin = bb;
          break;
        }
        acc += hist[bb];
        bin = bb;
      }
      s_bin = (uint32_t)bin;
      s_rem = remaining - acc;
    }
    __syncthreads();
    prefix |= s_bin << shift;
    mask |= 255u << shift;
    remaining = s_rem;
    __syncthreads();
  }
  return prefix;
}

__global__ void __launch_bounds__(kThreads) sample_kernel(SampleArgs a) {
  __shared__ float sh[32];
  __shared__ int shi[32];
  __shared__ float hist[256];
  pdl_wait();
  pdl_trigger();
  const int64_t row = blockIdx.x;
  const float* x = a.logits + row * a.ld;
  const float temp = a.temperature ? a.temperature[row] : 0.f;
  if (!(temp > 0.f)) {  // greedy
    float best = -FLT_MAX;
    int bi = 0x7fffffff;
    for (int64_t i = threadIdx.x; i < a.V; i += kThreads) {
      const float v = x[i];
      if (v > best) {
        best = v;
        bi = (int)i;
      }
    }
    block_argmax(best, bi, sh, shi);
    if (bi == 0x7fffffff) bi = 0;
    if (a.out_logprob) {
      float s = 0.f;
      for (int64_t i = threadIdx.x; i < a.V; i += kThreads) s += __expf(x[i] - best);
      s = block_sum(s, sh);
      if (threadIdx.x == 0) a.out_logprob[row] = -logf(s);
    }
    if (threadIdx.x == 0) a.out[row] = bi;
    return;
  }
  const float inv_t = 1.f / temp;
  float mx = -FLT_MAX;
  for (int64_t i = threadIdx.x; i < a.V; i += kThreads) mx = fmaxf(mx, x[i]);
  mx = block_max(mx, sh) * inv_t;
  float tot = 0.f;
  for (int64_t i = threadIdx.x; i < a.V; i += kThreads) tot += __expf(x[i] * inv_t - mx);
  tot = block_sum(tot, sh);

  uint32_t thr = 0;
  const int k = a.top_k ? a.top_k[row] : 0;
  const float p = a.top_p ? a.top_p[row] : 1.f;
  const float mp = a.min_p ? a.min_p[row] : 0.f;
  float kept = tot;
  if (k > 0 && k < a.V) {
    thr = radix_select(x, a.V, 0u, (float)k, 0, inv_t, mx, hist);
    float s = 0.f;
    for (int64_t i = threadIdx.x; i < a.V; i += kThreads)
      if (fkey(x[i]) >= thr) s += __expf(x[i] * inv_t - mx);
    kept = block_sum(s, sh);
  }
  if (p < 1.f && p > 0.f) {
    const uint32_t t2 = radix_select(x, a.V, thr, p * kept, 1, inv_t, mx, hist);
    thr = t2 > thr ? t2 : thr;
  }
  if (mp > 0.f) {
    const float lim = (mx + logf(mp)) * temp;  // x >= temp * (mx + log(min_p))
    const uint32_t t3 = fkey(lim);
    thr = t3 > thr ? t3 : thr;
  }
  const uint64_t seed = a.seeds ? a.seeds[row] : 0x1234ull;
  const uint64_t ctr = a.offsets ? (uint64_t)a.offsets[row] : 0ull;
  float best = -FLT_MAX;
  int bi = 0x7fffffff;
  for (int64_t i = threadIdx.x; i < a.V; i += kThreads) {
    const float v = x[i];
    if (fkey(v) < thr) continue;
    const float sc = v * inv_t + gumbel(seed, ctr, (uint64_t)i);
    if (sc > best) {
      best = sc;
      bi = (int)i;
    }
  }
  block_argmax(best, bi, sh, shi);
  if (bi == 0x7fffffff) bi = 0;
  if (threadIdx.x == 0) {
    a.out[row] = bi;
    if (a.out_logprob) a.out_logprob[row] = x[bi] * inv_t - mx - logf(tot);
  }
}

// Penalties and logit bias, in place on fp32 logits before token selection.
// Row r's distinct previously seen tokens are ids[off[r] .. off[r + 1]) with
// their counts; its biases are bias_ids / bias_vals[boff[r] .. boff[r + 1]).
//   repetition (CTRL, Keskar et al. 2019, as HF applies it): x / rep if x > 0
//   else x * rep, for every listed token (prompt and output); frequency:
//   x -= freq * count; presence: x -= pres, for tokens generated (count > 0).
// Each (row, token) pair appears once, so threads never collide.
__global__ void penalties_kernel(float* __restrict__ logits, int64_t ld, const int32_t* __restrict__ off,
                                 const int32_t* __restrict__ ids, const int32_t* __restrict__ counts,
                                 const float* __restrict__ rep, const float* __restrict__ freq,
                                 const float* __restrict__ pres, const int32_t* __restrict__ boff,
                                 const int32_t* __restrict__ bias_ids, const float* __restrict__ bias_vals,
                                 int64_t V) {
  pdl_wait();
  pdl_trigger();
  const int row = blockIdx.x;
  float* x = logits + (int64_t)row * ld;
  const float rp = rep[row], fq = freq[row], pr = pres[row];
  for (int i = off[row] + threadIdx.x; i < off[row + 1]; i += blockDim.x) {
    const int t = ids[i];
    if (t < 0 || t >= V) continue;
    float v = x[t];
    if (rp != 1.f) v = v > 0.f ? v / rp : v * rp;
    const int n = counts[i];  // 0: seen in the prompt only (repetition penalty applies, the others do not)
    if (n > 0) v -= fq * (float)n + pr;
    x[t] = v;
  }
  __syncthreads();
  for (int i = boff[row] + threadIdx.x; i < boff[row + 1]; i += blockDim.x) {
    const int t = bias_ids[i];
    if (t >= 0 && t < V) x[t] += bias_vals[i];
  }
}

}  // namespace smp

void penalties_launch(float* logits, int64_t ld, int64_t B, int64_t V, const int32_t* off, const int32_t* ids,
                      const int32_t* counts, const float* rep, const float* freq, const float* pres,
                      const int32_t* boff, const int32_t* bias_ids, const float* bias_vals, cudaStream_t st) {
  if (B == 0) return;
  launch_pdl(smp::penalties_kernel, dim3((unsigned)B), dim3(128), 0, st, logits, ld, off, ids, counts, rep, freq,
             pres, boff, bias_ids, bias_vals, V);
}

void argmax_launch(const float* logits, int64_t ld, int64_t B, int64_t V, int32_t* out, cudaStream_t st) {
  if (B == 0) return;
  launch_pdl(smp::argmax_kernel, dim3((unsigned)B), dim3(smp::kThreads), 0, st, logits, ld, V, out);
}

namespace smp {
// Overlapped scheduling: a decode row whose input token was still being
// sampled when its step was scheduled names the logit row of the previous
// step (src >= 0); copy that row's sampled id from the previous step's output.
__global__ void forward_tokens_kernel(int32_t* __restrict__ ids, const int32_t* __restrict__ src,
                                      const int32_t* __restrict__ prev, int n) {
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t < n) {
    const int r = src[t];
    if (r >= 0) ids[t] = prev[r];
  }
}
}  // namespace smp

void forward_tokens_launch(int32_t* ids, const int32_t* src, const int32_t* prev, int n, cudaStream_t st) {
  if (n == 0) return;
  launch_pdl(smp::forward_tokens_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, st, ids, src, prev, n);
}

void sample_launch(const SampleArgs& a, cudaStream_t st) {
  if (a.B == 0) return;
  launch_pdl(smp::sample_kernel, dim3((unsigned)a.B), dim3(smp::kThreads), 0, st, a);
}

}  // namespace b200
