// Expert-parallel MoE combine over NVLink peer memory, fused with the residual
// add and the next RMSNorm (one kernel, no NCCL, no multicast loads).
//
// Expert parallelism here keeps attention replicated: every rank holds the
// whole step's tokens, routes all of them identically, and runs the grouped
// MXFP4 GEMMs only for the experts it owns ([rank * e_local, (rank + 1) *
// e_local)). The down GEMM's epilogue already scales each expert row by its
// router weight and writes it into this rank's slot of a symmetric (IPC) heap,
// together with the step's inverse permutation (token, slot) -> row.
//
// This kernel then, per token t (one CTA):
//   1. barrier: announce this op's epoch to every rank, wait (bounded) until
//      every rank has announced it - so every rank's rows and inverse
//      permutation for this op are complete and visible;
//   2. for each slot s in fixed order: owner q = experts[t, s] / e_local,
//      row = inv_q[t * k + s] (a peer load), then the 16-byte vectors of that
//      row straight from rank q's HBM over NVLink;
//   3. moe = bf16(sum_s rows) (fp32 sum in slot order), h = bf16(h + moe),
//      out = rmsnorm(h) * w.
// Each rank reads only the k rows its tokens need: T * k * H * 2 bytes per op
// (7/8 of them remote at EP 8), against 2 * T * H * 2 * (world - 1) / world
// for a ring all-reduce of the combined partials plus the separate combine,
// add and norm kernels it replaces. The sum has the single-GPU kernels' order,
// so EP = N reproduces EP = 1 bit for bit.
//
// Slots are double-buffered by op parity on the host: a rank writes parity p
// again only two ops later, after it passed the barrier of the op in between,
// which every peer enters only after finishing its reads of parity p.
//
// Reference: the reference dispatches expert rows to workers over host TCP and
// sums the returned partials on the orchestrator
// (crates/rlx-kimi-k3/src/dist_experts.rs:666-757, `dispatch_experts` :712).
#include <cuda_bf16.h>

#include <algorithm>
#include <stdexcept>

#include "../common/b200.cuh"
#include "../common/launch.h"
#include "../common/pdl_launch.h"

namespace b200 {
namespace epc {

constexpr int kMaxK = 8;

template <int VPT>
__global__ void ep_combine_norm_kernel(EpCombineArgs a) {
  __shared__ float red[32];
  __shared__ const uint4* s_row[kMaxK];
  pdl_wait();
  pdl_trigger();
  const unsigned e = *reinterpret_cast<volatile unsigned*>(a.epoch) + 1u;
  if (blockIdx.x == 0 && threadIdx.x < (unsigned)a.world)
    st_release_sys_u32(a.peer_flags[threadIdx.x] + a.rank, e);
  if (threadIdx.x < (unsigned)a.world) wait_flag_geq(a.flags + threadIdx.x, e, a.status, 700 + threadIdx.x);
  __syncthreads();
  const int t = blockIdx.x;
  const int H = a.H;
  const int nv = H / 8;
  if (t < a.T) {
    if (threadIdx.x < (unsigned)a.k) {
      const int s = threadIdx.x;
      const int ex = a.experts[(int64_t)t * a.k + s];
      const int q = ex / a.e_local;
      const uint4* row = nullptr;
      if (ex >= 0 && q < a.world) {
        const int pos = __ldcg(a.peer_inv[q] + (int64_t)t * a.k + s);  // peer memory through L2 only
        if (pos >= 0)
          row = reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(a.peer_rows[q]) +
                                               (int64_t)pos * H);
      }
      s_row[s] = row;
    }
    __syncthreads();
    __nv_bfloat16* hrow = reinterpret_cast<__nv_bfloat16*>(a.h) + (int64_t)t * H;
    float v[VPT][8];
    float ss = 0.f;
#pragma unroll
    for (int c = 0; c < VPT; ++c) {
      const int vi = threadIdx.x + c * blockDim.x;
      if (vi >= nv) break;
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      uint4 rv[kMaxK];
#pragma unroll
      for (int s = 0; s < kMaxK; ++s)  // issue every slot's load before summing
        if (s < a.k && s_row[s] != nullptr) rv[s] = __ldcg(s_row[s] + vi);
#pragma unroll
      for (int s = 0; s < kMaxK; ++s) {
        if (s >= a.k || s_row[s] == nullptr) continue;
        const uint32_t w[4] = {rv[s].x, rv[s].y, rv[s].z, rv[s].w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          acc[2 * j] += bf16_lo(w[j]);
          acc[2 * j + 1] += bf16_hi(w[j]);
        }
      }
      const uint4 hv = *reinterpret_cast<const uint4*>(hrow + vi * 8);
      const uint32_t hw[4] = {hv.x, hv.y, hv.z, hv.w};
      uint32_t o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t m = pack_bf16x2(acc[2 * j], acc[2 * j + 1]);  // the combine's bf16 output
        o[j] = pack_bf16x2(bf16_lo(m) + bf16_lo(hw[j]), bf16_hi(m) + bf16_hi(hw[j]));
        v[c][2 * j] = bf16_lo(o[j]);
        v[c][2 * j + 1] = bf16_hi(o[j]);
        ss += v[c][2 * j] * v[c][2 * j] + v[c][2 * j + 1] * v[c][2 * j + 1];
      }
      *reinterpret_cast<uint4*>(hrow + vi * 8) = make_uint4(o[0], o[1], o[2], o[3]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x < 32) {
      float x = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
      if (threadIdx.x == 0) red[0] = x;
    }
    __syncthreads();
    const float inv = rsqrtf(red[0] / (float)H + a.eps);
    const __nv_bfloat16* nw = reinterpret_cast<const __nv_bfloat16*>(a.norm_w);
    __nv_bfloat16* orow = reinterpret_cast<__nv_bfloat16*>(a.out) + (int64_t)t * H;
#pragma unroll
    for (int c = 0; c < VPT; ++c) {
      const int vi = threadIdx.x + c * blockDim.x;
      if (vi >= nv) break;
      const uint4 wv = *reinterpret_cast<const uint4*>(nw + vi * 8);
      const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
      uint32_t o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float lo = __bfloat162float(__float2bfloat16(v[c][2 * j] * inv)) * bf16_lo(ww[j]);
        const float hi = __bfloat162float(__float2bfloat16(v[c][2 * j + 1] * inv)) * bf16_hi(ww[j]);
        o[j] = pack_bf16x2(lo, hi);
      }
      *reinterpret_cast<uint4*>(orow + vi * 8) = make_uint4(o[0], o[1], o[2], o[3]);
    }
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

}  // namespace epc

void ep_combine_norm_launch(const EpCombineArgs& a, cudaStream_t st) {
  using namespace epc;
  if (a.H % 8 != 0 || a.k < 1 || a.k > kMaxK || a.e_local < 1 || a.world < 1 || a.world > 32)
    throw std::runtime_error("b200.ep_combine_norm: hidden % 8, 1 <= k <= 8, world <= 32 required");
  const int nv = a.H / 8;
  const int threads = std::min(512, (nv + 31) / 32 * 32);
  const int vpt = (nv + threads - 1) / threads;
  const dim3 grid(std::max(1, a.T));
  if (vpt <= 1) launch_pdl(ep_combine_norm_kernel<1>, grid, dim3(threads), 0, st, a);
  else if (vpt <= 2) launch_pdl(ep_combine_norm_kernel<2>, grid, dim3(threads), 0, st, a);
  else if (vpt <= 4) launch_pdl(ep_combine_norm_kernel<4>, grid, dim3(threads), 0, st, a);
  else throw std::runtime_error("b200.ep_combine_norm: hidden size too large (max 16384)");
}

}  // namespace b200
