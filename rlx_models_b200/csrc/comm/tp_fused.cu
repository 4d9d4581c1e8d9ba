// Tensor-parallel residual-stream collective fused with RMSNorm, over NVLink
// peer memory (no NCCL, no multicast loads).
//
// One row-parallel op of the sequence-parallel TP decoder is two kernels:
//   1. the tcgen05 GEMM in push mode: every output row (token) of this rank's
//      partial product is stored straight into slot `rank` of the row
//      owner's receive buffer over NVLink, tile by tile as the MMAs finish
//      (reduce-scatter fused into the GEMM epilogue); the GEMM's last CTA
//      raises this op's epoch in every rank's rs_flags[rank];
//   2. rs_norm_ag (this file): each rank waits for all rs flags, sums the
//      `world` partial slots of the rows it owns, adds its residual-stream
//      shard (h = h + sum, bf16 like HF), computes RMSNorm(h) * w and writes the
//      normalised row into every rank's gather buffer (all-gather by P2P
//      stores). The last CTA raises ag flags on every rank and waits for all
//      ranks' ag flags, then advances the local epoch.
// After (2) every rank holds the full normalised activation [M, H] locally, the
// input of the next column-parallel GEMM; the residual stream itself stays
// sharded by rows (sequence parallel).
//
// Ordering: a rank reuses its receive / gather buffers only after an epoch
// barrier that every peer passes after its last read of them (see
// parallel/fused_tp.py). All waits are bounded (kWaitTimeoutNs) and report
// kErrTimeoutPeer in the status word instead of hanging.
#include <cuda_bf16.h>

#include <algorithm>
#include <stdexcept>

#include "../common/b200.cuh"
#include "../common/launch.h"
#include "../common/pdl_launch.h"

namespace b200 {


constexpr int kRsThreads = 256;
constexpr int kRsMaxChunks = 4;  // H <= 256 * 8 * 4 = 8192

__global__ void __launch_bounds__(kRsThreads) rs_norm_ag_kernel(RsNormAgArgs a) {
  __shared__ float red[kRsThreads / 32];
  pdl_wait();
  pdl_trigger();
  const unsigned e = *reinterpret_cast<volatile unsigned*>(a.epoch) + 1u;
  const __nv_bfloat16* recv = reinterpret_cast<const __nv_bfloat16*>(a.recv);
  __nv_bfloat16* hbuf = reinterpret_cast<__nv_bfloat16*>(a.h);
  const __nv_bfloat16* nw = reinterpret_cast<const __nv_bfloat16*>(a.norm_w);
  __nv_bfloat16* const* pg = reinterpret_cast<__nv_bfloat16* const*>(a.peer_gath);
  const int n_my = max(0, min(a.rpr, a.M - a.rank * a.rpr));
  if (a.do_reduce) {
    if (threadIdx.x < (unsigned)a.world) wait_flag_geq(a.rs_flags + threadIdx.x, e, a.status, 100 + threadIdx.x);
    __syncthreads();
  }
  const int r = blockIdx.x;
  if (r < n_my) {
    const int nch = a.H / (kRsThreads * 8);
    float v[kRsMaxChunks][8];
#pragma unroll
    for (int c = 0; c < kRsMaxChunks; ++c) {
      if (c >= nch) break;
      const int col = (c * kRsThreads + threadIdx.x) * 8;
      const uint4 hv = *reinterpret_cast<const uint4*>(hbuf + (int64_t)r * a.H + col);
      const uint32_t hw[4] = {hv.x, hv.y, hv.z, hv.w};
      float s[8];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        s[2 * k] = 0.f;
        s[2 * k + 1] = 0.f;
      }
      if (a.do_reduce == 2) {
        // fp32 sums that every rank's accumulate-mode GEMM added in place
        float4* ap = reinterpret_cast<float4*>(a.racc + (int64_t)r * a.H + col);
        const float4 a0 = __ldcg(ap), a1 = __ldcg(ap + 1);
        __stcg(ap, make_float4(0.f, 0.f, 0.f, 0.f));
        __stcg(ap + 1, make_float4(0.f, 0.f, 0.f, 0.f));
        s[0] = a0.x; s[1] = a0.y; s[2] = a0.z; s[3] = a0.w;
        s[4] = a1.x; s[5] = a1.y; s[6] = a1.z; s[7] = a1.w;
      }
      if (a.do_reduce == 1) {
        for (int q = 0; q < a.world; ++q) {
          const uint4 pv = __ldcg(reinterpret_cast<const uint4*>(recv + q * a.slot_elems + (int64_t)r * a.H + col));
          const uint32_t pw[4] = {pv.x, pv.y, pv.z, pv.w};
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            s[2 * k] += bf16_lo(pw[k]);
            s[2 * k + 1] += bf16_hi(pw[k]);
          }
        }
      }
      if (a.do_reduce) {
        // residual stream in bf16: h = bf16(h + bf16(sum))
        uint32_t o[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float lo = __bfloat162float(__float2bfloat16(s[2 * k]));
          const float hi = __bfloat162float(__float2bfloat16(s[2 * k + 1]));
          o[k] = pack_bf16x2(bf16_lo(hw[k]) + lo, bf16_hi(hw[k]) + hi);
          v[c][2 * k] = bf16_lo(o[k]);
          v[c][2 * k + 1] = bf16_hi(o[k]);
        }
        *reinterpret_cast<uint4*>(hbuf + (int64_t)r * a.H + col) = make_uint4(o[0], o[1], o[2], o[3]);
      } else {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          v[c][2 * k] = bf16_lo(hw[k]);
          v[c][2 * k + 1] = bf16_hi(hw[k]);
        }
      }
    }
    float ss = 0.f;
#pragma unroll
    for (int c = 0; c < kRsMaxChunks; ++c) {
      if (c >= nch) break;
#pragma unroll
      for (int k = 0; k < 8; ++k) ss += v[c][k] * v[c][k];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x < 32) {
      float t = threadIdx.x < kRsThreads / 32 ? red[threadIdx.x] : 0.f;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
      if (threadIdx.x == 0) red[0] = t;
    }
    __syncthreads();
    const float inv = rsqrtf(red[0] / (float)a.H + a.eps);
    const int64_t grow = (int64_t)(a.rank * a.rpr + r) * a.H;
#pragma unroll
    for (int c = 0; c < kRsMaxChunks; ++c) {
      if (c >= nch) break;
      const int col = (c * kRsThreads + threadIdx.x) * 8;
      const uint4 wv = *reinterpret_cast<const uint4*>(nw + col);
      const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
      uint32_t o[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float lo = __bfloat162float(__float2bfloat16(v[c][2 * k] * inv)) * bf16_lo(ww[k]);
        const float hi = __bfloat162float(__float2bfloat16(v[c][2 * k + 1] * inv)) * bf16_hi(ww[k]);
        o[k] = pack_bf16x2(lo, hi);
      }
      const uint4 ov = make_uint4(o[0], o[1], o[2], o[3]);
      // all-gather: the same normalised row into every rank's gather buffer
      for (int q = 0; q < a.world; ++q) *reinterpret_cast<uint4*>(pg[q] + grow + col) = ov;
    }
  }
  __syncthreads();  // the CTA's gather stores, then one system fence (cumulative) per CTA
  if (threadIdx.x == 0) {
    __threadfence_system();
    const unsigned old = atomicAdd(a.cta_ctr, 1u);
    if (old == gridDim.x - 1) {
      __threadfence_system();
      for (int q = 0; q < a.world; ++q) st_release_sys_u32(a.peer_ag_flags[q] + a.rank, e);
      for (int q = 0; q < a.world; ++q) wait_flag_geq(a.ag_flags + q, e, a.status, 200 + q);
      *a.cta_ctr = 0;
      __threadfence();
      *reinterpret_cast<volatile unsigned*>(a.epoch) = e;
    }
  }
}

void rs_norm_ag_launch(const RsNormAgArgs& a, cudaStream_t st) {
  if (a.H % (kRsThreads * 8) != 0 || a.H > kRsThreads * 8 * kRsMaxChunks)
    throw std::runtime_error("b200.rs_norm_ag: hidden must be a multiple of 2048 and <= 8192");
  const int n_my = std::max(0, std::min(a.rpr, a.M - a.rank * a.rpr));
  launch_pdl(rs_norm_ag_kernel, dim3(std::max(1, n_my)), dim3(kRsThreads), 0, st, a);
}

// ---------------------------------------------------------------------------
// One-shot variant for decode-sized steps: the GEMM broadcast its bf16 partial
// into slot `rank` of every rank; every rank sums all slots for all rows.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kRsThreads) os_reduce_norm_kernel(OsReduceArgs a) {
  __shared__ float red[kRsThreads / 32];
  pdl_wait();
  pdl_trigger();
  const unsigned e = *reinterpret_cast<volatile unsigned*>(a.epoch) + 1u;
  if (threadIdx.x < (unsigned)a.world) wait_flag_geq(a.flags + threadIdx.x, e, a.status, 300 + threadIdx.x);
  __syncthreads();
  const __nv_bfloat16* slots = reinterpret_cast<const __nv_bfloat16*>(a.slots);
  __nv_bfloat16* hbuf = reinterpret_cast<__nv_bfloat16*>(a.h);
  const __nv_bfloat16* nw = reinterpret_cast<const __nv_bfloat16*>(a.norm_w);
  __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(a.out);
  const int r = blockIdx.x;
  const int nch = a.H / (kRsThreads * 8);
  float v[kRsMaxChunks][8];
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < kRsMaxChunks; ++c) {
    if (c >= nch) break;
    const int col = (c * kRsThreads + threadIdx.x) * 8;
    float s[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int q = 0; q < a.world; ++q) {
      const uint4 pv = __ldcg(reinterpret_cast<const uint4*>(slots + q * a.slot_elems + (int64_t)r * a.H + col));
      const uint32_t pw[4] = {pv.x, pv.y, pv.z, pv.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        s[2 * k] += bf16_lo(pw[k]);
        s[2 * k + 1] += bf16_hi(pw[k]);
      }
    }
    const uint4 hv = *reinterpret_cast<const uint4*>(hbuf + (int64_t)r * a.H + col);
    const uint32_t hw[4] = {hv.x, hv.y, hv.z, hv.w};
    uint32_t o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      o[k] = pack_bf16x2(bf16_lo(hw[k]) + __bfloat162float(__float2bfloat16(s[2 * k])),
                         bf16_hi(hw[k]) + __bfloat162float(__float2bfloat16(s[2 * k + 1])));
      v[c][2 * k] = bf16_lo(o[k]);
      v[c][2 * k + 1] = bf16_hi(o[k]);
      ss += v[c][2 * k] * v[c][2 * k] + v[c][2 * k + 1] * v[c][2 * k + 1];
    }
    *reinterpret_cast<uint4*>(hbuf + (int64_t)r * a.H + col) = make_uint4(o[0], o[1], o[2], o[3]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < kRsThreads / 32 ? red[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  const float inv = rsqrtf(red[0] / (float)a.H + a.eps);
#pragma unroll
  for (int c = 0; c < kRsMaxChunks; ++c) {
    if (c >= nch) break;
    const int col = (c * kRsThreads + threadIdx.x) * 8;
    const uint4 wv = *reinterpret_cast<const uint4*>(nw + col);
    const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
    uint32_t o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      o[k] = pack_bf16x2(__bfloat162float(__float2bfloat16(v[c][2 * k] * inv)) * bf16_lo(ww[k]),
                         __bfloat162float(__float2bfloat16(v[c][2 * k + 1] * inv)) * bf16_hi(ww[k]));
    }
    *reinterpret_cast<uint4*>(out + (int64_t)r * a.H + col) = make_uint4(o[0], o[1], o[2], o[3]);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned old = atomicAdd(a.cta_ctr, 1u);
    if (old == gridDim.x - 1) {
      *a.cta_ctr = 0;
      __threadfence();
      *reinterpret_cast<volatile unsigned*>(a.epoch) = e;
    }
  }
}

void os_reduce_norm_launch(const OsReduceArgs& a, cudaStream_t st) {
  if (a.H % (kRsThreads * 8) != 0 || a.H > kRsThreads * 8 * kRsMaxChunks)
    throw std::runtime_error("b200.os_reduce_norm: hidden must be a multiple of 2048 and <= 8192");
  launch_pdl(os_reduce_norm_kernel, dim3(std::max(1, a.M)), dim3(kRsThreads), 0, st, a);
}

}  // namespace b200

namespace b200 {
namespace {
// Failure-path probe: one bounded wait on a flag. A flag that nothing sets
// makes the wait run out (kWaitTimeoutNs), record kErrTimeoutPeer with
// detail kErrTimeoutTest in the status word and return, leaving the context
// usable; tests use it to check the host-side error reporting.
__global__ void flag_wait_probe_kernel(const unsigned* flag, unsigned target, int* status, int* ok) {
  if (threadIdx.x == 0 && blockIdx.x == 0) *ok = wait_flag_geq(flag, target, status, kErrTimeoutTest) ? 1 : 0;
}
}  // namespace

void flag_wait_probe_launch(const unsigned* flag, unsigned target, int* status, int* ok, cudaStream_t st) {
  flag_wait_probe_kernel<<<1, 32, 0, st>>>(flag, target, status, ok);
}
}  // namespace b200

namespace b200 {
namespace tpc {
// Pull all-reduce + residual add + RMSNorm for decode-sized steps (M <= 128).
//
// Every rank's row-parallel GEMM accumulates its fp32 partial into its own
// slot of the symmetric heap (local red.add, no NVLink traffic in the GEMM).
// This kernel: CTA 0 announces "partial ready" by writing this op's epoch into
// every rank's flag[my rank] (release, system scope); every CTA waits until all
// ranks announced, then row r is reduced by reading the world partials
// straight from peer memory (P2P loads over NVLink), the residual is added and
// the row normalised. Finally the CTA zeroes row r of its own *previous*
// parity accumulator, which every rank has finished reading (they all passed
// this op's barrier, hence finished the previous op), so the next GEMM can
// accumulate into it. One barrier per op; no NCCL call.
// Threads per CTA: one 8-column chunk of the row per thread up to 512 threads
// (H = 4096: every peer load of a thread is issued in one round), 512 threads
// with 2-4 chunks above that.
constexpr int kPullThreads = 512;
__host__ __device__ constexpr int pull_threads(int H) { return H / 8 < kPullThreads ? H / 8 : kPullThreads; }
constexpr int kMaxWorld = 8;

// s[0..8) = sum over the world ranks of the 8 fp32 values at element offset
// `off` of each rank's partial (peer memory). Every rank's two 16-byte loads
// are issued before any is consumed, so the NVLink round trips overlap
// instead of running one after another. Plain L2 (.cg) loads: the data was
// published before the flag this kernel acquired, and is never cached in L1.
__device__ __forceinline__ void sum_peer_rows(const float* const* peer, int world, int64_t off, float (&s)[8]) {
  float4 x[kMaxWorld][2];
#pragma unroll
  for (int q = 0; q < kMaxWorld; ++q) {
    if (q < world) {
      const float4* src = reinterpret_cast<const float4*>(peer[q] + off);
      x[q][0] = __ldcg(src);
      x[q][1] = __ldcg(src + 1);
    }
  }
#pragma unroll
  for (int k = 0; k < 8; ++k) s[k] = 0.f;
#pragma unroll
  for (int q = 0; q < kMaxWorld; ++q) {
    if (q < world) {
      s[0] += x[q][0].x; s[1] += x[q][0].y; s[2] += x[q][0].z; s[3] += x[q][0].w;
      s[4] += x[q][1].x; s[5] += x[q][1].y; s[6] += x[q][1].z; s[7] += x[q][1].w;
    }
  }
}

__global__ void __launch_bounds__(kPullThreads) ar_pull_norm_kernel(PullNormArgs a) {
  __shared__ float red[kPullThreads / 32];
  pdl_wait();
  pdl_trigger();
  const unsigned e = *reinterpret_cast<volatile unsigned*>(a.epoch) + 1u;
  if (blockIdx.x == 0 && threadIdx.x < (unsigned)a.world)
    st_release_sys_u32(a.peer_flags[threadIdx.x] + a.rank, e);
  if (threadIdx.x < (unsigned)a.world) wait_flag_geq(a.flags + threadIdx.x, e, a.status, 500 + threadIdx.x);
  __syncthreads();
  const int r = blockIdx.x;
  const int H = a.H;
  if (r < a.M) {
    __nv_bfloat16* hbuf = reinterpret_cast<__nv_bfloat16*>(a.h);
    const __nv_bfloat16* nw = reinterpret_cast<const __nv_bfloat16*>(a.norm_w);
    __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(a.out);
    constexpr int kMaxChunks = 4;  // H <= 512 * 8 * 4
    const int nch = H / ((int)blockDim.x * 8);
    float v[kMaxChunks][8];
    float ss = 0.f;
#pragma unroll
    for (int c = 0; c < kMaxChunks; ++c) {
      if (c >= nch) break;
      const int col = (c * (int)blockDim.x + threadIdx.x) * 8;
      float s[8];
      sum_peer_rows(a.peer_acc, a.world, (int64_t)r * H + col, s);
      const uint4 hv = *reinterpret_cast<const uint4*>(hbuf + (int64_t)r * H + col);
      const uint32_t hw[4] = {hv.x, hv.y, hv.z, hv.w};
      uint32_t o[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        o[k] = pack_bf16x2(bf16_lo(hw[k]) + __bfloat162float(__float2bfloat16(s[2 * k])),
                           bf16_hi(hw[k]) + __bfloat162float(__float2bfloat16(s[2 * k + 1])));
        v[c][2 * k] = bf16_lo(o[k]);
        v[c][2 * k + 1] = bf16_hi(o[k]);
        ss += v[c][2 * k] * v[c][2 * k] + v[c][2 * k + 1] * v[c][2 * k + 1];
      }
      *reinterpret_cast<uint4*>(hbuf + (int64_t)r * H + col) = make_uint4(o[0], o[1], o[2], o[3]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x < 32) {
      float t = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : 0.f;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
      if (threadIdx.x == 0) red[0] = t;
    }
    __syncthreads();
    const float inv = rsqrtf(red[0] / (float)H + a.eps);
#pragma unroll
    for (int c = 0; c < kMaxChunks; ++c) {
      if (c >= nch) break;
      const int col = (c * (int)blockDim.x + threadIdx.x) * 8;
      const uint4 wv = *reinterpret_cast<const uint4*>(nw + col);
      const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
      uint32_t o[4];
#pragma unroll
      for (int k = 0; k < 4; ++k)
        o[k] = pack_bf16x2(v[c][2 * k] * inv * bf16_lo(ww[k]), v[c][2 * k + 1] * inv * bf16_hi(ww[k]));
      *reinterpret_cast<uint4*>(out + (int64_t)r * H + col) = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
  if (r < a.zero_rows) {
    float4* z = reinterpret_cast<float4*>(a.zero_buf + (int64_t)r * H);
    for (int i = threadIdx.x; i < H / 4; i += blockDim.x) z[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  // the last CTA publishes this op's epoch for the next op
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(a.cta_ctr, 1u) == gridDim.x - 1) {
      *a.cta_ctr = 0;
      *a.epoch = e;
    }
  }
}
}  // namespace tpc

void ar_pull_norm_launch(const PullNormArgs& a, cudaStream_t st) {
  if (a.world > tpc::kMaxWorld) throw std::runtime_error("b200.ar_pull_norm: at most 8 ranks");
  const int nt = tpc::pull_threads(a.H);
  if (a.H % 256 != 0 || a.H % (nt * 8) != 0 || a.H > nt * 8 * 4)
    throw std::runtime_error("b200.ar_pull_norm: hidden must be a multiple of 256 and <= 16384");
  launch_pdl(tpc::ar_pull_norm_kernel, dim3(std::max(std::max(1, a.M), a.zero_rows)), dim3(nt), 0, st, a);
}
}  // namespace b200

namespace b200 {
namespace tpc {
// Two-shot all-reduce + residual add + RMSNorm for decode-sized steps.
//
// Same inputs as ar_pull_norm (every rank's fp32 partial in its symmetric
// slot, a replicated bf16 residual stream), but each rank reduces only the
// rows it owns (row i belongs to rank i / rpr) and the others fetch the
// finished rows:
//   barrier 1  CTA 0 announces "partial ready" to every rank; the phase-A CTAs
//              wait for all ranks' announcements;
//   phase A    work item = (owned row, 512-column slice), spread over the CTAs so
//              the remote reads of the owned rows use many SMs: sum the
//              world partials of the slice over NVLink (fp32), add the
//              residual, store the new residual slice (bf16) and the slice's
//              sum of squares in this rank's result slot; the last item
//              announces "rows ready" to every rank (barrier 2);
//   phase B    every CTA waits for barrier 2, copies row i's new residual and
//              its per-slice sums of squares from the owner, and applies the
//              RMSNorm itself (the owner never writes a normalised row).
// Per rank, each op moves M*H*4/world bytes of partials and M*H*2 bytes of
// residual rows in over NVLink, against M*H*4*(world-1) bytes of partials for
// the one-shot pull. Result slots are reused without double buffering: a rank
// rewrites its slot in op k+1 only after every rank announced op k+1's
// partial, which each does after its op-k kernel (and its phase-B reads)
// completed. One system fence per phase-A CTA (after a CTA barrier, so it
// covers every thread's stores) and one before the barrier-2 flags.
constexpr int kSliceCols = 512;              // phase-A item width
constexpr int kSliceThreads = kSliceCols / 8;  // 64 threads, 8 columns each

__global__ void __launch_bounds__(kPullThreads) ar2_norm_kernel(TwoShotNormArgs a) {
  __shared__ float red[kPullThreads / 32];
  pdl_wait();
  pdl_trigger();
  const unsigned e = *reinterpret_cast<volatile unsigned*>(a.epoch) + 1u;
  const int H = a.H;
  const int i = blockIdx.x;
  const int S = H / kSliceCols;
  const int n_my = max(0, min(a.rpr, a.M - a.rank * a.rpr));
  const int n_items = n_my * S;
  __nv_bfloat16* hbuf = reinterpret_cast<__nv_bfloat16*>(a.h);
  __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(a.out);
  __nv_bfloat16* res = reinterpret_cast<__nv_bfloat16*>(a.own_res);  // [rpr_max][H] new residual rows
  float* ssq = reinterpret_cast<float*>(res + (int64_t)a.rpr_max * H);  // [rpr_max][S] slice sums of squares
  if (i == 0 && threadIdx.x < (unsigned)a.world) st_release_sys_u32(a.peer_flags[threadIdx.x] + a.rank, e);
  if (i < n_items) {
    if (threadIdx.x < (unsigned)a.world) wait_flag_geq(a.flags + threadIdx.x, e, a.status, 700 + threadIdx.x);
    __syncthreads();
    // items i, i + grid, ...: the grid stays within one CTA per SM, so every CTA
    // (all of which wait at barrier 2 below) is resident at once
    for (int item = i; item < n_items; item += gridDim.x) {
      const int li = item / S, sl = item % S;
      const int r = a.rank * a.rpr + li;
      float ss = 0.f;
      if (threadIdx.x < (unsigned)kSliceThreads) {
        const int col = sl * kSliceCols + threadIdx.x * 8;
        float sm[8];
        sum_peer_rows(a.peer_acc, a.world, (int64_t)r * H + col, sm);
        const uint4 hv = *reinterpret_cast<const uint4*>(hbuf + (int64_t)r * H + col);
        const uint32_t hw[4] = {hv.x, hv.y, hv.z, hv.w};
        uint32_t o[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          o[k] = pack_bf16x2(bf16_lo(hw[k]) + __bfloat162float(__float2bfloat16(sm[2 * k])),
                             bf16_hi(hw[k]) + __bfloat162float(__float2bfloat16(sm[2 * k + 1])));
          const float lo = bf16_lo(o[k]), hi = bf16_hi(o[k]);
          ss += lo * lo + hi * hi;
        }
        *reinterpret_cast<uint4*>(res + (int64_t)li * H + col) = make_uint4(o[0], o[1], o[2], o[3]);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      if ((threadIdx.x & 31) == 0 && threadIdx.x < (unsigned)kSliceThreads) red[threadIdx.x >> 5] = ss;
      __syncthreads();
      if (threadIdx.x == 0) {
        float t = 0.f;
#pragma unroll
        for (int w = 0; w < kSliceThreads / 32; ++w) t += red[w];
        ssq[li * S + sl] = t;
        // every thread's stores are ordered before this fence by the barrier above
        // (fence cumulativity): one system fence per item publishes the slice
        __threadfence_system();
        if (atomicAdd(a.cta_ctr, 1u) == (unsigned)n_items - 1) {
          __threadfence_system();  // one system fence covers every rank's flag store below
          for (int q = 0; q < a.world; ++q) st_relaxed_sys_u32(a.peer_flags[q] + a.world + a.rank, e);
        }
      }
      __syncthreads();  // red[] is reused by the next item
    }
  } else if (n_my == 0 && i == 0 && threadIdx.x == 0) {
    for (int q = 0; q < a.world; ++q) st_release_sys_u32(a.peer_flags[q] + a.world + a.rank, e);
  }
  // every CTA passes barrier 2 (it also orders the accumulator clearing below after
  // every rank's phase-A reads of the previous op's partials)
  if (threadIdx.x < (unsigned)a.world) wait_flag_geq(a.flags + a.world + threadIdx.x, e, a.status, 800 + threadIdx.x);
  __syncthreads();
  if (i < a.M) {
    const int owner = i / a.rpr, j = i % a.rpr;
    const __nv_bfloat16* src = reinterpret_cast<const __nv_bfloat16*>(a.peer_res[owner]);
    const uint4* sh = reinterpret_cast<const uint4*>(src + (int64_t)j * H);
    const float* sq = reinterpret_cast<const float*>(src + (int64_t)a.rpr_max * H) + j * S;
    constexpr int kMaxIt = 4;  // H <= 512 * 8 * 4: every load of the row is issued before any store
    uint4 vh[kMaxIt];
#pragma unroll
    for (int it = 0; it < kMaxIt; ++it) {
      const int c = it * (int)blockDim.x + threadIdx.x;
      if (c < H / 8) vh[it] = __ldcg(sh + c);
    }
    if (threadIdx.x < 32) {
      float t = threadIdx.x < (unsigned)S ? __ldcg(sq + threadIdx.x) : 0.f;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
      if (threadIdx.x == 0) red[0] = t;
    }
    __syncthreads();
    const float inv = rsqrtf(red[0] / (float)H + a.eps);
    const __nv_bfloat16* nw = reinterpret_cast<const __nv_bfloat16*>(a.norm_w);
    uint4* dh = reinterpret_cast<uint4*>(hbuf + (int64_t)i * H);
    uint4* dout = reinterpret_cast<uint4*>(out + (int64_t)i * H);
#pragma unroll
    for (int it = 0; it < kMaxIt; ++it) {
      const int c = it * (int)blockDim.x + threadIdx.x;
      if (c < H / 8) {
        dh[c] = vh[it];
        const uint4 wv = *reinterpret_cast<const uint4*>(nw + c * 8);
        const uint32_t hw[4] = {vh[it].x, vh[it].y, vh[it].z, vh[it].w};
        const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
        uint32_t o[4];
#pragma unroll
        for (int k = 0; k < 4; ++k)
          o[k] = pack_bf16x2(bf16_lo(hw[k]) * inv * bf16_lo(ww[k]), bf16_hi(hw[k]) * inv * bf16_hi(ww[k]));
        dout[c] = make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
  }
  if (i < a.zero_rows) {
    float4* z = reinterpret_cast<float4*>(a.zero_buf + (int64_t)i * H);
    for (int c = threadIdx.x; c < H / 4; c += blockDim.x) z[c] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(a.cta_ctr + 1, 1u) == gridDim.x - 1) {
      a.cta_ctr[0] = 0;
      a.cta_ctr[1] = 0;
      __threadfence();
      *reinterpret_cast<volatile unsigned*>(a.epoch) = e;
    }
  }
}
}  // namespace tpc

void ar2_norm_launch(const TwoShotNormArgs& a, cudaStream_t st) {
  if (a.world > tpc::kMaxWorld) throw std::runtime_error("b200.ar2_norm: at most 8 ranks");
  const int nt = tpc::pull_threads(a.H);
  if (a.H % tpc::kSliceCols != 0 || a.H % (nt * 8) != 0 || a.H > nt * 8 * 4 || a.H / tpc::kSliceCols > 32)
    throw std::runtime_error("b200.ar2_norm: hidden must be a multiple of 512 and <= 16384");
  if (a.rpr <= 0 || a.rpr > a.rpr_max || (int64_t)a.rpr * a.world < a.M)
    throw std::runtime_error("b200.ar2_norm: row split does not cover the rows");
  // every CTA waits at barrier 2, which the phase-A CTAs release: the grid (at most
  // 128 CTAs, one per SM at this block size) must be resident at once
  const int grid = std::max(std::max(1, a.M), a.zero_rows);
  if (grid > 128) throw std::runtime_error("b200.ar2_norm: at most 128 rows per op");
  launch_pdl(tpc::ar2_norm_kernel, dim3(grid), dim3(nt), 0, st, a);
}
}  // namespace b200

