// Causal attention backward for training (head_dim 128, GQA, bf16 in, fp32
// accumulation), paired with the tcgen05 forward kernel (attention/fmha_sm100.cu)
// which saves the per-row log2-sum-exp2 of the scaled scores.
//
// Flash-attention style, no S x S matrix in memory:
//   prep      delta[t, h] = sum_d dO * O (fp32); dq_acc = 0
//   main      one CTA per (key tile of 64, kv head, sequence); for every query
//             head of the GQA group and every query tile of 64 at or after the
//             key tile (causal):
//               S  = Q K^T,          P  = exp2(S * scale * log2e - lse)
//               dP = dO V^T,         dS = P * (dP - delta)
//               dV += P^T dO,        dK += scale * dS^T Q    (registers, per warp 16 keys)
//               dQ += scale * dS K   (fp32 atomics into dq_acc, per warp 16 queries)
//             4 warps; the q / dO / K / V tiles and the bf16 P and dS tiles sit in
//             shared memory in the 128-byte swizzled layout the ldmatrix loads
//             read conflict-free; products run on mma.sync m16n8k16.
//   finish    dq = bf16(dq_acc)
// dK / dV of a kv head sum over its query heads inside the CTA (no atomics).
//
// Reference: rlx-tune gets these gradients from its autodiff crate over the
// same attention graph (rlx-tune src/lm.rs:77-115).
#include <cuda_bf16.h>

#include <algorithm>
#include <stdexcept>

#include "../common/b200.cuh"
#include "../common/launch.h"
#include "../common/pdl_launch.h"
#include "../common/tma_host.h"

namespace b200 {
namespace abw {

constexpr int kD = 128;
constexpr int kBM = 64;  // queries per tile
constexpr int kBN = 64;  // keys per CTA
constexpr int kThreads = 128;
constexpr float kLog2e = 1.4426950408889634f;
// shared memory: K, V, Q, dO tiles [64][128] (two 64-column boxes each), P and dS [64][64]
constexpr int kTile = 64 * 128 * 2;
constexpr int kPS = 64 * 64 * 2;
constexpr int kSmem = 4 * kTile + 2 * kPS + 2 * 64 * 4 + 1024;

// copy a [64][128] bf16 tile (row stride ld elements) into the swizzled smem layout
__device__ __forceinline__ void load_tile(uint8_t* dst, const __nv_bfloat16* src, int64_t ld, int rows_valid) {
  for (int i = threadIdx.x; i < 64 * 16; i += kThreads) {
    const int r = i >> 4, c = (i & 15) * 8;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (r < rows_valid) v = *reinterpret_cast<const uint4*>(src + (int64_t)r * ld + c);
    *reinterpret_cast<uint4*>(dst + sw128_off(r, c, 64)) = v;
  }
}

__device__ __forceinline__ void red_add_v2(float* p, float a, float b) {
  asm volatile("red.global.add.v2.f32 [%0], {%1, %2};" ::"l"(p), "f"(a), "f"(b) : "memory");
}

__global__ void __launch_bounds__(256) attn_bwd_prep_kernel(AttnBwdArgs a) {
  pdl_wait();
  pdl_trigger();
  // one warp per (token, head): delta = sum_d dO * O, and clear dq_acc
  const int64_t item = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const int64_t n = (int64_t)a.B * a.S * a.Hq;
  if (item >= n) return;
  const __nv_bfloat16* o = reinterpret_cast<const __nv_bfloat16*>(a.o) + item * kD + lane * 4;
  const __nv_bfloat16* d = reinterpret_cast<const __nv_bfloat16*>(a.dout) + item * kD + lane * 4;
  const uint2 ov = *reinterpret_cast<const uint2*>(o), dv = *reinterpret_cast<const uint2*>(d);
  float s = bf16_lo(ov.x) * bf16_lo(dv.x) + bf16_hi(ov.x) * bf16_hi(dv.x) + bf16_lo(ov.y) * bf16_lo(dv.y) +
            bf16_hi(ov.y) * bf16_hi(dv.y);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  if (lane == 0) a.delta[item] = s;
  *reinterpret_cast<float4*>(a.dq_acc + item * kD + lane * 4) = make_float4(0.f, 0.f, 0.f, 0.f);
}

__global__ void __launch_bounds__(kThreads) attn_bwd_kernel(AttnBwdArgs a) {
  extern __shared__ uint8_t smem_dyn[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = smem;
  uint8_t* sV = sK + kTile;
  uint8_t* sQ = sV + kTile;
  uint8_t* sO = sQ + kTile;  // dO
  uint8_t* sP = sO + kTile;
  uint8_t* sS = sP + kPS;  // dS
  float* sL = reinterpret_cast<float*>(sS + kPS);  // lse of the query tile
  float* sDl = sL + 64;                            // delta of the query tile
  pdl_wait();
  pdl_trigger();

  const int G = a.Hq / a.Hkv;
  const int n_kt = a.S / kBN;
  const int kt = blockIdx.x;  // heavy (early) key tiles first
  const int hkv = blockIdx.y, b = blockIdx.z;
  const int k0 = kt * kBN;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g8 = lane >> 2, t4 = lane & 3;
  const int mi = lane >> 3, rr = lane & 7;
  const int64_t tok0 = (int64_t)b * a.S;
  const float sl2 = a.scale * kLog2e;
  (void)n_kt;

  load_tile(sK, reinterpret_cast<const __nv_bfloat16*>(a.k) + ((tok0 + k0) * a.Hkv + hkv) * kD,
            (int64_t)a.Hkv * kD, 64);
  load_tile(sV, reinterpret_cast<const __nv_bfloat16*>(a.v) + ((tok0 + k0) * a.Hkv + hkv) * kD,
            (int64_t)a.Hkv * kD, 64);

  // dV / dK accumulators: warp w owns keys [16w, 16w + 16) x 128 dims (16 n-tiles of 8)
  float dv[16][4], dk[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) dv[i][j] = dk[i][j] = 0.f;

  const uint32_t uK = smem_u32(sK), uV = smem_u32(sV), uQ = smem_u32(sQ), uO = smem_u32(sO), uP = smem_u32(sP),
                 uS = smem_u32(sS);

  for (int gq = 0; gq < G; ++gq) {
    const int h = hkv * G + gq;
    for (int q0 = k0; q0 < a.S; q0 += kBM) {
      __syncthreads();  // previous tile's readers are done with Q / dO / P / dS
      load_tile(sQ, reinterpret_cast<const __nv_bfloat16*>(a.q) + ((tok0 + q0) * a.Hq + h) * kD, (int64_t)a.Hq * kD,
                64);
      load_tile(sO, reinterpret_cast<const __nv_bfloat16*>(a.dout) + ((tok0 + q0) * a.Hq + h) * kD,
                (int64_t)a.Hq * kD, 64);
      if (threadIdx.x < 64) {
        sL[threadIdx.x] = a.lse[(tok0 + q0 + threadIdx.x) * a.Hq + h];
        sDl[threadIdx.x] = a.delta[(tok0 + q0 + threadIdx.x) * a.Hq + h];
      }
      __syncthreads();

      // ---- S = Q K^T and dP = dO V^T for this warp's 16 query rows x 64 keys ----
      float s[8][4], dp[8][4];
#pragma unroll
      for (int n = 0; n < 8; ++n)
#pragma unroll
        for (int j = 0; j < 4; ++j) s[n][j] = dp[n][j] = 0.f;
#pragma unroll
      for (int ks = 0; ks < kD / 16; ++ks) {
        uint32_t qa[4], oa[4];
        const int ar = warp * 16 + (mi & 1) * 8 + rr, ac = ks * 16 + (mi >> 1) * 8;
        ldmatrix_x4(uQ + sw128_off(ar, ac, 64), qa[0], qa[1], qa[2], qa[3]);
        ldmatrix_x4(uO + sw128_off(ar, ac, 64), oa[0], oa[1], oa[2], oa[3]);
#pragma unroll
        for (int np = 0; np < 4; ++np) {  // pairs of 8-key n-tiles
          const int key = np * 16 + (mi >> 1) * 8 + rr, d0 = ks * 16 + (mi & 1) * 8;
          uint32_t b0, b1, b2, b3;
          ldmatrix_x4(uK + sw128_off(key, d0, 64), b0, b1, b2, b3);
          mma_bf16_16816(s[np * 2], qa, b0, b1);
          mma_bf16_16816(s[np * 2 + 1], qa, b2, b3);
          ldmatrix_x4(uV + sw128_off(key, d0, 64), b0, b1, b2, b3);
          mma_bf16_16816(dp[np * 2], oa, b0, b1);
          mma_bf16_16816(dp[np * 2 + 1], oa, b2, b3);
        }
      }
      // ---- P, dS (masked) -> shared memory as bf16 [q][key] ----
      const int rq0 = warp * 16 + g8, rq1 = rq0 + 8;  // tile-local query rows of this thread
      const float lse0 = sL[rq0], lse1 = sL[rq1], dl0 = sDl[rq0], dl1 = sDl[rq1];
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        const int kc = n * 8 + 2 * t4;  // tile-local key column
        float p[4], ds[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int qr = (j < 2) ? rq0 : rq1;
          const int kk = kc + (j & 1);
          const bool ok = (k0 + kk) <= (q0 + qr);
          p[j] = ok ? exp2f(s[n][j] * sl2 - ((j < 2) ? lse0 : lse1)) : 0.f;
          ds[j] = p[j] * (dp[n][j] - ((j < 2) ? dl0 : dl1));
        }
        *reinterpret_cast<uint32_t*>(sP + sw128_off(rq0, kc, 64)) = pack_bf16x2(p[0], p[1]);
        *reinterpret_cast<uint32_t*>(sP + sw128_off(rq1, kc, 64)) = pack_bf16x2(p[2], p[3]);
        *reinterpret_cast<uint32_t*>(sS + sw128_off(rq0, kc, 64)) = pack_bf16x2(ds[0], ds[1]);
        *reinterpret_cast<uint32_t*>(sS + sw128_off(rq1, kc, 64)) = pack_bf16x2(ds[2], ds[3]);
      }
      __syncthreads();

      // ---- dV += P^T dO, dK += dS^T Q for this warp's 16 keys x 128 dims ----
#pragma unroll
      for (int ks = 0; ks < kBM / 16; ++ks) {  // contraction over 16 queries at a time
        uint32_t pa[4], sa[4];
        // A = P^T: rows = keys (warp * 16 ..), cols = queries; stored [q][key] -> transposed load
        const int sq = ks * 16 + (mi >> 1) * 8 + rr, sk = warp * 16 + (mi & 1) * 8;
        ldmatrix_x4_trans(uP + sw128_off(sq, sk, 64), pa[0], pa[1], pa[2], pa[3]);
        ldmatrix_x4_trans(uS + sw128_off(sq, sk, 64), sa[0], sa[1], sa[2], sa[3]);
#pragma unroll
        for (int dp2 = 0; dp2 < 8; ++dp2) {  // pairs of 8-dim n-tiles; B = dO / Q [q][d] (N-major)
          const int qrow = ks * 16 + (mi & 1) * 8 + rr, d0 = (dp2 * 2 + (mi >> 1)) * 8;
          uint32_t b0, b1, b2, b3;
          ldmatrix_x4_trans(uO + sw128_off(qrow, d0, 64), b0, b1, b2, b3);
          mma_bf16_16816(dv[dp2 * 2], pa, b0, b1);
          mma_bf16_16816(dv[dp2 * 2 + 1], pa, b2, b3);
          ldmatrix_x4_trans(uQ + sw128_off(qrow, d0, 64), b0, b1, b2, b3);
          mma_bf16_16816(dk[dp2 * 2], sa, b0, b1);
          mma_bf16_16816(dk[dp2 * 2 + 1], sa, b2, b3);
        }
      }

      // ---- dQ += scale * dS K for this warp's 16 queries, two 64-dim halves ----
      float* dqg = a.dq_acc + ((tok0 + q0) * a.Hq + h) * kD;
      const int64_t dq_ld = (int64_t)a.Hq * kD;
#pragma unroll 1
      for (int half = 0; half < 2; ++half) {
        float dq[8][4];
#pragma unroll
        for (int n = 0; n < 8; ++n)
#pragma unroll
          for (int j = 0; j < 4; ++j) dq[n][j] = 0.f;
#pragma unroll
        for (int ks = 0; ks < kBN / 16; ++ks) {  // contraction over keys
          uint32_t sa[4];
          const int ar = warp * 16 + (mi & 1) * 8 + rr, ac = ks * 16 + (mi >> 1) * 8;
          ldmatrix_x4(uS + sw128_off(ar, ac, 64), sa[0], sa[1], sa[2], sa[3]);
#pragma unroll
          for (int dp2 = 0; dp2 < 4; ++dp2) {  // B = K [key][d] (N-major)
            const int key = ks * 16 + (mi & 1) * 8 + rr, d0 = half * 64 + (dp2 * 2 + (mi >> 1)) * 8;
            uint32_t b0, b1, b2, b3;
            ldmatrix_x4_trans(uK + sw128_off(key, d0, 64), b0, b1, b2, b3);
            mma_bf16_16816(dq[dp2 * 2], sa, b0, b1);
            mma_bf16_16816(dq[dp2 * 2 + 1], sa, b2, b3);
          }
        }
#pragma unroll
        for (int n = 0; n < 8; ++n) {
          const int d = half * 64 + n * 8 + 2 * t4;
          float* r0 = dqg + (int64_t)rq0 * dq_ld + d;
          float* r1 = dqg + (int64_t)rq1 * dq_ld + d;
          red_add_v2(r0, dq[n][0] * a.scale, dq[n][1] * a.scale);
          red_add_v2(r1, dq[n][2] * a.scale, dq[n][3] * a.scale);
        }
      }
    }
  }

  // ---- write dK (scaled) and dV for this warp's 16 keys ----
  __nv_bfloat16* dkg = reinterpret_cast<__nv_bfloat16*>(a.dk) + ((tok0 + k0) * a.Hkv + hkv) * kD;
  __nv_bfloat16* dvg = reinterpret_cast<__nv_bfloat16*>(a.dv) + ((tok0 + k0) * a.Hkv + hkv) * kD;
  const int64_t kv_ld = (int64_t)a.Hkv * kD;
  const int kr0 = warp * 16 + g8, kr1 = kr0 + 8;
#pragma unroll
  for (int n = 0; n < 16; ++n) {
    const int d = n * 8 + 2 * t4;
    *reinterpret_cast<uint32_t*>(dkg + kr0 * kv_ld + d) = pack_bf16x2(dk[n][0] * a.scale, dk[n][1] * a.scale);
    *reinterpret_cast<uint32_t*>(dkg + kr1 * kv_ld + d) = pack_bf16x2(dk[n][2] * a.scale, dk[n][3] * a.scale);
    *reinterpret_cast<uint32_t*>(dvg + kr0 * kv_ld + d) = pack_bf16x2(dv[n][0], dv[n][1]);
    *reinterpret_cast<uint32_t*>(dvg + kr1 * kv_ld + d) = pack_bf16x2(dv[n][2], dv[n][3]);
  }
}

__global__ void __launch_bounds__(256) attn_bwd_finish_kernel(const float* __restrict__ acc,
                                                              __nv_bfloat16* __restrict__ out, int64_t n) {
  pdl_wait();
  pdl_trigger();
  for (int64_t i = (int64_t)blockIdx.x * 256 + threadIdx.x; i < n / 4; i += (int64_t)gridDim.x * 256) {
    const float4 v = reinterpret_cast<const float4*>(acc)[i];
    reinterpret_cast<uint2*>(out)[i] = make_uint2(pack_bf16x2(v.x, v.y), pack_bf16x2(v.z, v.w));
  }
}

}  // namespace abw

void attn_bwd_launch(const AttnBwdArgs& a, int device, cudaStream_t st) {
  using namespace abw;
  if (a.S % kBN != 0) throw std::runtime_error("b200.attn_bwd: sequence length must be a multiple of 64");
  if (a.Hq % a.Hkv != 0) throw std::runtime_error("b200.attn_bwd: query heads must be a multiple of kv heads");
  const int64_t items = (int64_t)a.B * a.S * a.Hq;
  if (items == 0) return;
  launch_pdl(attn_bwd_prep_kernel, dim3((unsigned)((items + 7) / 8)), dim3(256), 0, st, a);
  ensure_smem(attn_bwd_kernel, kSmem);
  launch_pdl(attn_bwd_kernel, dim3(a.S / kBN, a.Hkv, a.B), dim3(kThreads), kSmem, st, a);
  const int64_t n = items * kD;
  const int grid = (int)std::min<int64_t>((n / 4 + 255) / 256, (int64_t)num_sms(device) * 8);
  launch_pdl(attn_bwd_finish_kernel, dim3(grid), dim3(256), 0, st, a.dq_acc,
             reinterpret_cast<__nv_bfloat16*>(a.dq), n);
}

}  // namespace b200
