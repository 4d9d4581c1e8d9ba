// Causal attention backward for training (head_dim 128, GQA, bf16 in, fp32
// accumulation), paired with the tcgen05 forward kernel (attention/fmha_sm100.cu)
// which saves the per-row log2-sum-exp2 of the scaled scores.
//
// Flash-attention style, no S x S matrix in memory:
//   prep      delta[t, h] = sum_d dO * O (fp32); dq_acc = 0
//   main      one CTA (8 warps) per (key tile of 128, kv head, sequence); for
//             every query head of the GQA group and every query tile of 64 at or
//             after the key tile (causal):
//               S  = Q K^T,          P  = exp2(S * scale * log2e - lse)
//               dP = dO V^T,         dS = P * (dP - delta)
//               dV += P^T dO,        dK += scale * dS^T Q    (registers, 16 keys per warp)
//               dQ  = scale * dS K   (64 x 128 fp32 tile staged in shared memory and
//                                     added to dq_acc by bulk async reductions, one
//                                     512-byte row per operation)
//             The next query tile's Q / dO are fetched with cp.async into a second
//             buffer while the current one is processed; K / V / Q / dO and the
//             bf16 P / dS tiles use the 128-byte swizzled layout the ldmatrix loads
//             read conflict-free; products run on mma.sync m16n8k16. Grid order puts
//             the key tiles with the most query tiles (the first ones) first.
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
constexpr int kBM = 64;   // queries per tile
constexpr int kBN = 128;  // keys per CTA
constexpr int kThreads = 256;
constexpr float kLog2e = 1.4426950408889634f;
constexpr int kQTile = kBM * kD * 2;              // Q or dO tile [64][128] bf16 (two 64-column boxes)
constexpr int kKTile = kBN * kD * 2;              // K or V tile [128][128] bf16
constexpr int kPTile = kBM * kBN * 2;             // P or dS [64 q][128 keys] bf16
constexpr int kDqRow = kD * 4 + 16;               // fp32 dQ stage row, padded by 16 bytes
constexpr int kSmem = 2 * kKTile + 4 * kQTile + 2 * kPTile + kBM * kDqRow + 128;

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ void bulk_reduce_add_f32(float* gdst, uint32_t ssrc, uint32_t bytes) {
  asm volatile("cp.reduce.async.bulk.global.shared::cta.bulk_group.add.f32 [%0], [%1], %2;" ::"l"(gdst), "r"(ssrc),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// [rows][128] bf16 tile (row stride ld elements) -> swizzled smem (boxes of [rows][64]) by cp.async;
// rows at or past rows_valid are zero-filled
template <int ROWS>
__device__ __forceinline__ void async_tile(uint32_t dst, const __nv_bfloat16* src, int64_t ld, int rows_valid) {
#pragma unroll
  for (int i = threadIdx.x; i < ROWS * 16; i += kThreads) {
    const int r = i >> 4, c = (i & 15) * 8;
    const bool ok = r < rows_valid;
    cp_async16(dst + sw128_off(r, c, ROWS), src + (ok ? (int64_t)r * ld + c : 0), ok);
  }
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

__global__ void __launch_bounds__(kThreads, 1) attn_bwd_kernel(AttnBwdArgs a) {
  extern __shared__ uint8_t smem_dyn[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_dyn) + 127) & ~uintptr_t(127));
  uint8_t* sK = smem;
  uint8_t* sV = sK + kKTile;
  uint8_t* sQ = sV + kKTile;       // two buffers
  uint8_t* sO = sQ + 2 * kQTile;   // dO, two buffers
  uint8_t* sP = sO + 2 * kQTile;
  uint8_t* sS = sP + kPTile;       // dS
  uint8_t* sDq = sS + kPTile;      // fp32 dQ stage [64][kDqRow bytes]
  pdl_wait();
  pdl_trigger();

  const int G = a.Hq / a.Hkv;
  const int hkv = blockIdx.x, b = blockIdx.y;
  const int kt = blockIdx.z;  // the first key tiles have the most query tiles: they start first
  const int k0 = kt * kBN;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g8 = lane >> 2, t4 = lane & 3;
  const int mi = lane >> 3, rr = lane & 7;
  const int64_t tok0 = (int64_t)b * a.S;
  const float sl2 = a.scale * kLog2e;
  const int nq = (a.S - k0) / kBM;  // query tiles at or after the key tile
  const int n_it = G * nq;
  const int64_t q_ld = (int64_t)a.Hq * kD;
  const int64_t kv_ld = (int64_t)a.Hkv * kD;
  const __nv_bfloat16* qg = reinterpret_cast<const __nv_bfloat16*>(a.q);
  const __nv_bfloat16* og = reinterpret_cast<const __nv_bfloat16*>(a.dout);

  const uint32_t uK = smem_u32(sK), uV = smem_u32(sV), uQ0 = smem_u32(sQ), uO0 = smem_u32(sO), uP = smem_u32(sP),
                 uS = smem_u32(sS), uDq = smem_u32(sDq);
  const int keys_valid = min(kBN, a.S - k0);
  async_tile<kBN>(uK, reinterpret_cast<const __nv_bfloat16*>(a.k) + ((tok0 + k0) * a.Hkv + hkv) * kD, kv_ld,
                  keys_valid);
  async_tile<kBN>(uV, reinterpret_cast<const __nv_bfloat16*>(a.v) + ((tok0 + k0) * a.Hkv + hkv) * kD, kv_ld,
                  keys_valid);
  auto issue_q = [&](int it, int buf) {
    const int h = hkv * G + it / nq, q0 = k0 + (it % nq) * kBM;
    async_tile<kBM>(uQ0 + buf * kQTile, qg + ((tok0 + q0) * a.Hq + h) * kD, q_ld, kBM);
    async_tile<kBM>(uO0 + buf * kQTile, og + ((tok0 + q0) * a.Hq + h) * kD, q_ld, kBM);
  };
  if (n_it > 0) issue_q(0, 0);
  cp_async_commit();

  // dV / dK accumulators: warp w owns keys [16w, 16w + 16) x 128 dims (16 n-tiles of 8)
  float dv[16][4], dk[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) dv[i][j] = dk[i][j] = 0.f;

  const int qw = (warp & 3) * 16;   // phase 1 / 3: this warp's 16 query rows of the tile
  const int kh = (warp >> 2) * 64;  // phase 1: this warp's 64 keys; phase 3: its 64 dQ dims
  const int rq0 = qw + g8, rq1 = rq0 + 8;

  for (int it = 0; it < n_it; ++it) {
    const int buf = it & 1;
    const int h = hkv * G + it / nq, q0 = k0 + (it % nq) * kBM;
    // this thread's two query rows: log2-sum-exp and delta (latency overlaps the products below)
    const int64_t r0 = (tok0 + q0 + rq0) * a.Hq + h, r1 = (tok0 + q0 + rq1) * a.Hq + h;
    const float lse0 = __ldg(a.lse + r0), lse1 = __ldg(a.lse + r1);
    const float dl0 = __ldg(a.delta + r0), dl1 = __ldg(a.delta + r1);
    cp_async_wait_all();
    __syncthreads();  // tile `it` landed; every thread is past iteration it-1 (buffer buf^1 and P / dS free)
    if (it + 1 < n_it) issue_q(it + 1, buf ^ 1);
    cp_async_commit();
    const uint32_t uQ = uQ0 + buf * kQTile, uO = uO0 + buf * kQTile;

    // ---- S = Q K^T and dP = dO V^T: 16 query rows x 64 keys per warp ----
    float s[8][4], dp[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int j = 0; j < 4; ++j) s[n][j] = dp[n][j] = 0.f;
#pragma unroll
    for (int ks = 0; ks < kD / 16; ++ks) {
      uint32_t qa[4], oa[4];
      const int ar = qw + (mi & 1) * 8 + rr, ac = ks * 16 + (mi >> 1) * 8;
      ldmatrix_x4(uQ + sw128_off(ar, ac, kBM), qa[0], qa[1], qa[2], qa[3]);
      ldmatrix_x4(uO + sw128_off(ar, ac, kBM), oa[0], oa[1], oa[2], oa[3]);
#pragma unroll
      for (int np = 0; np < 4; ++np) {  // pairs of 8-key n-tiles
        const int key = kh + np * 16 + (mi >> 1) * 8 + rr, d0 = ks * 16 + (mi & 1) * 8;
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4(uK + sw128_off(key, d0, kBN), b0, b1, b2, b3);
        mma_bf16_16816(s[np * 2], qa, b0, b1);
        mma_bf16_16816(s[np * 2 + 1], qa, b2, b3);
        ldmatrix_x4(uV + sw128_off(key, d0, kBN), b0, b1, b2, b3);
        mma_bf16_16816(dp[np * 2], oa, b0, b1);
        mma_bf16_16816(dp[np * 2 + 1], oa, b2, b3);
      }
    }
    // ---- P, dS (masked) -> shared memory as bf16 [q][key] ----
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      const int kc = kh + n * 8 + 2 * t4;  // tile-local key column
      float p[4], ds[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int qr = (j < 2) ? rq0 : rq1;
        const int kk = kc + (j & 1);
        const bool ok = (k0 + kk) <= (q0 + qr);
        p[j] = ok ? exp2f(s[n][j] * sl2 - ((j < 2) ? lse0 : lse1)) : 0.f;
        ds[j] = ok ? p[j] * (dp[n][j] - ((j < 2) ? dl0 : dl1)) : 0.f;
      }
      *reinterpret_cast<uint32_t*>(sP + sw128_off(rq0, kc, kBM)) = pack_bf16x2(p[0], p[1]);
      *reinterpret_cast<uint32_t*>(sP + sw128_off(rq1, kc, kBM)) = pack_bf16x2(p[2], p[3]);
      *reinterpret_cast<uint32_t*>(sS + sw128_off(rq0, kc, kBM)) = pack_bf16x2(ds[0], ds[1]);
      *reinterpret_cast<uint32_t*>(sS + sw128_off(rq1, kc, kBM)) = pack_bf16x2(ds[2], ds[3]);
    }
    // the dQ stage is rewritten below: the previous tile's bulk reductions must have read it
    if (threadIdx.x < kBM) bulk_wait_read();
    __syncthreads();

    // ---- dV += P^T dO, dK += dS^T Q for this warp's 16 keys x 128 dims ----
#pragma unroll
    for (int ks = 0; ks < kBM / 16; ++ks) {  // contraction over 16 queries at a time
      uint32_t pa[4], sa[4];
      // A = P^T: rows = keys (warp * 16 ..), cols = queries; stored [q][key] -> transposed load
      const int sq = ks * 16 + (mi >> 1) * 8 + rr, sk = warp * 16 + (mi & 1) * 8;
      ldmatrix_x4_trans(uP + sw128_off(sq, sk, kBM), pa[0], pa[1], pa[2], pa[3]);
      ldmatrix_x4_trans(uS + sw128_off(sq, sk, kBM), sa[0], sa[1], sa[2], sa[3]);
#pragma unroll
      for (int dp2 = 0; dp2 < 8; ++dp2) {  // pairs of 8-dim n-tiles; B = dO / Q [q][d] (N-major)
        const int qrow = ks * 16 + (mi & 1) * 8 + rr, d0 = (dp2 * 2 + (mi >> 1)) * 8;
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4_trans(uO + sw128_off(qrow, d0, kBM), b0, b1, b2, b3);
        mma_bf16_16816(dv[dp2 * 2], pa, b0, b1);
        mma_bf16_16816(dv[dp2 * 2 + 1], pa, b2, b3);
        ldmatrix_x4_trans(uQ + sw128_off(qrow, d0, kBM), b0, b1, b2, b3);
        mma_bf16_16816(dk[dp2 * 2], sa, b0, b1);
        mma_bf16_16816(dk[dp2 * 2 + 1], sa, b2, b3);
      }
    }

    // ---- dQ = scale * dS K: 16 queries x 64 dims per warp, contraction over 128 keys ----
    {
      float dq[8][4];
#pragma unroll
      for (int n = 0; n < 8; ++n)
#pragma unroll
        for (int j = 0; j < 4; ++j) dq[n][j] = 0.f;
#pragma unroll
      for (int ks = 0; ks < kBN / 16; ++ks) {
        uint32_t sa[4];
        const int ar = qw + (mi & 1) * 8 + rr, ac = ks * 16 + (mi >> 1) * 8;
        ldmatrix_x4(uS + sw128_off(ar, ac, kBM), sa[0], sa[1], sa[2], sa[3]);
#pragma unroll
        for (int dp2 = 0; dp2 < 4; ++dp2) {  // B = K [key][d] (N-major)
          const int key = ks * 16 + (mi & 1) * 8 + rr, d0 = kh + (dp2 * 2 + (mi >> 1)) * 8;
          uint32_t b0, b1, b2, b3;
          ldmatrix_x4_trans(uK + sw128_off(key, d0, kBN), b0, b1, b2, b3);
          mma_bf16_16816(dq[dp2 * 2], sa, b0, b1);
          mma_bf16_16816(dq[dp2 * 2 + 1], sa, b2, b3);
        }
      }
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        const int d = kh + n * 8 + 2 * t4;
        *reinterpret_cast<float2*>(sDq + rq0 * kDqRow + d * 4) = make_float2(dq[n][0] * a.scale, dq[n][1] * a.scale);
        *reinterpret_cast<float2*>(sDq + rq1 * kDqRow + d * 4) = make_float2(dq[n][2] * a.scale, dq[n][3] * a.scale);
      }
    }
    fence_proxy_async_smem();  // the stage's generic-proxy writes, before the async-proxy reads
    __syncthreads();
    if (threadIdx.x < kBM) {  // one 512-byte row per thread: dq_acc[row] += stage[row]
      const int r = threadIdx.x;
      bulk_reduce_add_f32(a.dq_acc + ((tok0 + q0 + r) * a.Hq + h) * kD, uDq + r * kDqRow, kD * 4);
      bulk_commit();
    }
  }
  if (threadIdx.x < kBM) bulk_wait_all();

  // ---- write dK (scaled) and dV for this warp's 16 keys ----
  __nv_bfloat16* dkg = reinterpret_cast<__nv_bfloat16*>(a.dk) + ((tok0 + k0) * a.Hkv + hkv) * kD;
  __nv_bfloat16* dvg = reinterpret_cast<__nv_bfloat16*>(a.dv) + ((tok0 + k0) * a.Hkv + hkv) * kD;
  const int kr0 = warp * 16 + g8, kr1 = kr0 + 8;
#pragma unroll
  for (int n = 0; n < 16; ++n) {
    const int d = n * 8 + 2 * t4;
    if (kr0 < keys_valid) {
      *reinterpret_cast<uint32_t*>(dkg + kr0 * kv_ld + d) = pack_bf16x2(dk[n][0] * a.scale, dk[n][1] * a.scale);
      *reinterpret_cast<uint32_t*>(dvg + kr0 * kv_ld + d) = pack_bf16x2(dv[n][0], dv[n][1]);
    }
    if (kr1 < keys_valid) {
      *reinterpret_cast<uint32_t*>(dkg + kr1 * kv_ld + d) = pack_bf16x2(dk[n][2] * a.scale, dk[n][3] * a.scale);
      *reinterpret_cast<uint32_t*>(dvg + kr1 * kv_ld + d) = pack_bf16x2(dv[n][2], dv[n][3]);
    }
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
  if (a.S % kBM != 0) throw std::runtime_error("b200.attn_bwd: sequence length must be a multiple of 64");
  if (a.Hq % a.Hkv != 0) throw std::runtime_error("b200.attn_bwd: query heads must be a multiple of kv heads");
  const int64_t items = (int64_t)a.B * a.S * a.Hq;
  if (items == 0) return;
  launch_pdl(attn_bwd_prep_kernel, dim3((unsigned)((items + 7) / 8)), dim3(256), 0, st, a);
  ensure_smem(attn_bwd_kernel, kSmem);
  launch_pdl(attn_bwd_kernel, dim3(a.Hkv, a.B, (a.S + kBN - 1) / kBN), dim3(kThreads), kSmem, st, a);
  const int64_t n = items * kD;
  const int grid = (int)std::min<int64_t>((n / 4 + 255) / 256, (int64_t)num_sms(device) * 8);
  launch_pdl(attn_bwd_finish_kernel, dim3(grid), dim3(256), 0, st, a.dq_acc,
             reinterpret_cast<__nv_bfloat16*>(a.dq), n);
}

}  // namespace b200
