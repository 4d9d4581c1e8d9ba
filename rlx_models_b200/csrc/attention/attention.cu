// Paged attention for sm_100a ("K9" prefill, "K10" decode).
//
// KV cache layout: [num_blocks, Hkv, 16, D] bf16 (block size 16). One page of
// one kv head is a contiguous [16, D] tile, which a TMA 2-D map over the cache
// viewed as [num_blocks * Hkv * 16, D] fetches as D/64 boxes of [16, 64] with
// 128-byte swizzle (conflict-free ldmatrix reads).
//
// GQA packing: all G = Hq / Hkv query heads that share a kv head are rows of
// the same MMA tile, so each K/V page is read from HBM once per kv head.
// Supports causal prefill over cached pages (chunked prefill), decode with
// split-KV ("flash decoding"), sliding windows and learned per-head sink
// logits (gpt-oss: an extra softmax column that is dropped after softmax).
//
// Reference behaviour: fused SDPA with causal / sliding-window / sink masks
// (rlx-models-core src/standard_decoder.rs:11946-12079
// `build_gpt_oss_attention_with_sinks`; rlx-qwen3 src/builder.rs:450 ragged
// decode). The reference re-uploads host KV per step; here the KV is always
// device resident in pages.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>

#include <algorithm>
#include <cstdlib>
#include <stdexcept>
#include <type_traits>

#include "../common/b200.cuh"
#include "../common/launch.h"
#include "../common/pdl_launch.h"
#include "../common/tma_host.h"

namespace b200 {
namespace attn {

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kNegInf = -INFINITY;

// Scaled score in log2 units; with logit softcapping, cap * tanh(scale * s / cap).
__device__ __forceinline__ float score_log2(float s, const AttnArgs& a, float scale_log2) {
  return a.softcap > 0.f ? a.softcap * tanhf(s * a.scale / a.softcap) * kLog2e : s * scale_log2;
}

// ---------------------------------------------------------------------------
// Decode: grid (B * Hkv, splits), 4 compute warps + 1 TMA producer warp.
// Warp w consumes pages w, w+4, ... of this split from an NST-deep ring.
// ---------------------------------------------------------------------------
// F8: pages hold float8 e4m3 ([16, D] bytes, one unswizzled TMA box); each
// compute warp widens its page into a private f16 staging tile in the 128-byte
// swizzled layout the bf16 path reads, then releases the ring slot at once.
template <int D, int NST, bool F8 = false>
struct DecCfg {
  static constexpr int PAGE_BYTES = 16 * D * (F8 ? 1 : 2);
  static constexpr int STAGE_BYTES = 2 * PAGE_BYTES;  // K page + V page
  static constexpr int MERGE_BYTES = 4 * 16 * (D + 2) * 4;
  static constexpr int RING_BYTES = NST * STAGE_BYTES;
  static constexpr int RING_OR_MERGE = RING_BYTES > MERGE_BYTES ? RING_BYTES : MERGE_BYTES;
  static constexpr int BF16_PAGE = 16 * D * 2;
  static constexpr int STAGING_BYTES = F8 ? 4 * 2 * BF16_PAGE : 0;  // per compute warp: K and V in bf16
  static constexpr int SMEM = 1024 + RING_OR_MERGE + STAGING_BYTES + 2 * NST * 8 + 64;
};

// fp8 pages are widened to f16 (one cvt per two values; e4m3 is exact in f16)
// and the F8 kernel runs its MMAs in f16 (Q converted once, P packed as f16).
__device__ __forceinline__ void mma_f16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <bool F8>
__device__ __forceinline__ void mma16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  if constexpr (F8) mma_f16_16816(d, a, b0, b1);
  else mma_bf16_16816(d, a, b0, b1);
}

template <bool F8>
__device__ __forceinline__ uint32_t pack16(float a, float b) {
  if constexpr (F8) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
  } else {
    return pack_bf16x2(a, b);
  }
}

// 16 e4m3 values -> 16 f16.
__device__ __forceinline__ void fp8x16_to_f16(const uint4 raw, uint4& lo, uint4& hi) {
  const __nv_fp8x2_storage_t* p = reinterpret_cast<const __nv_fp8x2_storage_t*>(&raw);
  uint32_t w[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const __half2_raw hr = __nv_cvt_fp8x2_to_halfraw2(p[i], __NV_E4M3);
    w[i] = *reinterpret_cast<const uint32_t*>(&hr);
  }
  lo = make_uint4(w[0], w[1], w[2], w[3]);
  hi = make_uint4(w[4], w[5], w[6], w[7]);
}

// 16 e4m3 values -> 16 bf16 (exact: e4m3 values are representable in bf16).
__device__ __forceinline__ void fp8x16_to_bf16(const uint4 raw, uint4& lo, uint4& hi) {
  const __nv_fp8x2_storage_t* p = reinterpret_cast<const __nv_fp8x2_storage_t*>(&raw);
  uint32_t w[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const __half2_raw hr = __nv_cvt_fp8x2_to_halfraw2(p[i], __NV_E4M3);
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&hr));
    const __nv_bfloat162 b = __floats2bfloat162_rn(f.x, f.y);
    w[i] = *reinterpret_cast<const uint32_t*>(&b);
  }
  lo = make_uint4(w[0], w[1], w[2], w[3]);
  hi = make_uint4(w[4], w[5], w[6], w[7]);
}

// One [16, D] e4m3 page (row-major bytes) -> f16 in the swizzled page layout.
// Work item = (row, 64-column box), 4 lanes of 16 values each; the two items
// of an 8-lane group are rows r and r + 1 with boxes of opposite parity (D >=
// 128; for D = 64 the rows alternate 64-byte halves), so each group's 16-byte
// reads cover all 32 banks and its swizzled writes land on disjoint chunks.
template <int D>
__device__ __forceinline__ void widen_page(const uint8_t* src, uint8_t* dst, int lane) {
  constexpr int NB = D / 64;
  const int h = (lane >> 2) & 1, cq = lane & 3, g = lane >> 3;
#pragma unroll
  for (int it = 0; it < 2 * NB; ++it) {
    const int P = it * 4 + g;                 // pair of items, 0 .. 8 * NB - 1
    const int r = 2 * (P & 7) + h;
    const int bx = NB >= 2 ? ((P >> 3) ^ h) : 0;
    const int col = bx * 64 + cq * 16;
    uint4 lo, hi;
    fp8x16_to_f16(*reinterpret_cast<const uint4*>(src + r * D + col), lo, hi);
    *reinterpret_cast<uint4*>(dst + sw128_off(r, col, 16)) = lo;
    *reinterpret_cast<uint4*>(dst + sw128_off(r, col + 8, 16)) = hi;
  }
}

template <int D, int NST, bool F8 = false>
__global__ void __launch_bounds__(160) decode_attn_kernel(const __grid_constant__ CUtensorMap tmK,
                                                          const __grid_constant__ CUtensorMap tmV, AttnArgs a) {
  using Cf = DecCfg<D, NST, F8>;
  extern __shared__ uint8_t smem_dyn[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~uintptr_t(1023));
  const int ring_or_merge = Cf::RING_OR_MERGE;
  uint8_t* staging = smem + ring_or_merge;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + ring_or_merge + Cf::STAGING_BYTES);
  uint64_t* empty = full + NST;

  pdl_wait();
  const int G = a.Hq / a.Hkv;
  const int bh = blockIdx.x;
  const int b = bh / a.Hkv;
  const int hkv = bh % a.Hkv;
  const int split = blockIdx.y;
  const int nsplit = gridDim.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  const int ctx = a.ctx_lens[b];
  int first_tok = 0;
  if (a.window > 0) first_tok = max(0, ctx - a.window);
  const int first_page = first_tok >> 4;
  int last_page = (ctx + 15) >> 4;  // exclusive
  if (last_page > a.max_blocks) {  // ctx_lens[b] > 16 * max_blocks: never read past the table row
    if (threadIdx.x == 0 && blockIdx.y == 0) report_error(a.status, kErrBounds, b);
    last_page = a.max_blocks;
  }
  const int npages = max(0, last_page - first_page);
  const int pps = a.chunk_pages > 0 ? a.chunk_pages : (npages + nsplit - 1) / nsplit;
  const int p0 = first_page + split * pps;
  const int p1 = min(last_page, p0 + pps);
  const int my_pages = max(0, p1 - p0);
  const int32_t* btab = a.block_tables + (int64_t)b * a.max_blocks;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NST; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    fence_mbarrier_init();
  }
  __syncthreads();
  pdl_wait();
  pdl_trigger();

  const float scale_log2 = a.scale * kLog2e;
  float m_r[2] = {kNegInf, kNegInf}, l_r[2] = {0.f, 0.f};
  float o[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;

  if (warp == 4) {
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      for (int j = 0; j < my_pages; ++j) {
        if (!mbar_wait(&empty[s], ph ^ 1, a.status, kErrTimeoutEmpty)) break;
        const int blk = btab[p0 + j];
        const int row = (blk * a.Hkv + hkv) * 16;
        uint8_t* st = smem + s * Cf::STAGE_BYTES;
        mbar_arrive_expect_tx(&full[s], Cf::STAGE_BYTES);
        if constexpr (F8) {
          tma_load_2d(st, &tmK, &full[s], 0, row);
          tma_load_2d(st + Cf::PAGE_BYTES, &tmV, &full[s], 0, row);
        } else {
#pragma unroll
          for (int bx = 0; bx < D / 64; ++bx) {
            tma_load_2d(st + bx * 2048, &tmK, &full[s], bx * 64, row);
            tma_load_2d(st + Cf::PAGE_BYTES + bx * 2048, &tmV, &full[s], bx * 64, row);
          }
        }
        if (++s == NST) {
          s = 0;
          ph ^= 1;
        }
      }
    }
  } else {
    // Q fragments: rows = heads of this kv group (row r < G valid), k = dims.
    const int g = lane >> 2, t4 = lane & 3;
    uint32_t qa[D / 16][4];
    const __nv_bfloat16* qb = reinterpret_cast<const __nv_bfloat16*>(a.q) + ((int64_t)b * a.Hq + hkv * G) * D;
#pragma unroll
    for (int ks = 0; ks < D / 16; ++ks) {
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const int r = g + ((h & 1) ? 8 : 0);
        const int c = ks * 16 + 2 * t4 + ((h & 2) ? 8 : 0);
        uint32_t v = (r < G) ? *reinterpret_cast<const uint32_t*>(qb + (int64_t)r * D + c) : 0u;
        if constexpr (F8) {  // the F8 kernel multiplies in f16
          const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&v));
          v = pack16<true>(f.x, f.y);
        }
        qa[ks][h] = v;
      }
    }
    int s = warp % NST;
    uint32_t ph = 0;
    // pages j = warp, warp+4, ...; stage of page j is j % NST, phase (j / NST) & 1
    for (int j = warp; j < my_pages; j += 4) {
      s = j % NST;
      ph = (j / NST) & 1;
      if (!mbar_wait(&full[s], ph, a.status, kErrTimeoutFull)) break;
      uint32_t kb, vb;
      if constexpr (F8) {
        uint8_t* mine = staging + warp * 2 * Cf::BF16_PAGE;
        widen_page<D>(smem + s * Cf::STAGE_BYTES, mine, lane);
        widen_page<D>(smem + s * Cf::STAGE_BYTES + Cf::PAGE_BYTES, mine + Cf::BF16_PAGE, lane);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);  // the ring slot is free once widened
        kb = smem_u32(mine);
        vb = kb + Cf::BF16_PAGE;
      } else {
        kb = smem_u32(smem + s * Cf::STAGE_BYTES);
        vb = kb + Cf::PAGE_BYTES;
      }
      float sc[2][4];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
      const int mi = lane >> 3, rr = lane & 7;
#pragma unroll
      for (int ks = 0; ks < D / 16; ++ks) {
        const int tok = (mi >> 1) * 8 + rr;
        const int d0 = ks * 16 + (mi & 1) * 8;
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4(kb + sw128_off(tok, d0, 16), b0, b1, b2, b3);
        mma16<F8>(sc[0], qa[ks], b0, b1);
        mma16<F8>(sc[1], qa[ks], b2, b3);
      }
      // mask + online softmax (rows g and g+8)
      const int base_tok = (p0 + j) * 16;
      float mx[2] = {kNegInf, kNegInf};
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          const int tk = base_tok + nt * 8 + 2 * t4 + (h & 1);
          const bool ok = tk < ctx && tk >= first_tok;
          const float raw = F8 ? sc[nt][h] * a.k_scale : sc[nt][h];
          sc[nt][h] = ok ? score_log2(raw, a, scale_log2) : kNegInf;
          mx[h >> 1] = fmaxf(mx[h >> 1], sc[nt][h]);
        }
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
        mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
      }
      float corr[2];
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const float mn = fmaxf(m_r[r], mx[r]);
        corr[r] = (mn == kNegInf) ? 1.f : exp2f(m_r[r] - mn);
        m_r[r] = mn;
        l_r[r] *= corr[r];
      }
      uint32_t pa[4];
      {
        float p[2][4];
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int h = 0; h < 4; ++h) {
            const float mm = m_r[h >> 1];
            p[nt][h] = (mm == kNegInf) ? 0.f : exp2f(sc[nt][h] - mm);
            l_r[h >> 1] += p[nt][h];
          }
        pa[0] = pack16<F8>(p[0][0], p[0][1]);
        pa[1] = pack16<F8>(p[0][2], p[0][3]);
        pa[2] = pack16<F8>(p[1][0], p[1][1]);
        pa[3] = pack16<F8>(p[1][2], p[1][3]);
      }
#pragma unroll
      for (int dn = 0; dn < D / 8; ++dn) {
        o[dn][0] *= corr[0];
        o[dn][1] *= corr[0];
        o[dn][2] *= corr[1];
        o[dn][3] *= corr[1];
      }
#pragma unroll
      for (int dp = 0; dp < D / 16; ++dp) {
        const int tok = (mi & 1) * 8 + rr;
        const int d0 = (dp * 2 + (mi >> 1)) * 8;
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4_trans(vb + sw128_off(tok, d0, 16), b0, b1, b2, b3);
        mma16<F8>(o[dp * 2], pa, b0, b1);
        mma16<F8>(o[dp * 2 + 1], pa, b2, b3);
      }
      __syncwarp();
      if (!F8 && lane == 0) mbar_arrive(&empty[s]);
    }
    // finish row sums inside the quad
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      l_r[r] += __shfl_xor_sync(0xffffffffu, l_r[r], 1);
      l_r[r] += __shfl_xor_sync(0xffffffffu, l_r[r], 2);
    }
  }
  __syncthreads();  // ring no longer needed: reuse it for the cross-warp merge

  float* sm_o = reinterpret_cast<float*>(smem);       // [4][16][D]
  float* sm_ml = sm_o + 4 * 16 * D;                   // [4][16][2]
  if (warp < 4) {
    const int g = lane >> 2, t4 = lane & 3;
#pragma unroll
    for (int dn = 0; dn < D / 8; ++dn) {
      const int c = dn * 8 + 2 * t4;
      sm_o[(warp * 16 + g) * D + c] = o[dn][0];
      sm_o[(warp * 16 + g) * D + c + 1] = o[dn][1];
      sm_o[(warp * 16 + g + 8) * D + c] = o[dn][2];
      sm_o[(warp * 16 + g + 8) * D + c + 1] = o[dn][3];
    }
    if (t4 == 0) {
      sm_ml[(warp * 16 + g) * 2] = m_r[0];
      sm_ml[(warp * 16 + g) * 2 + 1] = l_r[0];
      sm_ml[(warp * 16 + g + 8) * 2] = m_r[1];
      sm_ml[(warp * 16 + g + 8) * 2 + 1] = l_r[1];
    }
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < G * D; idx += blockDim.x) {
    const int r = idx / D, d = idx % D;
    float M = kNegInf;
#pragma unroll
    for (int w = 0; w < 4; ++w) M = fmaxf(M, sm_ml[(w * 16 + r) * 2]);
    float L = 0.f, O = 0.f;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const float mw = sm_ml[(w * 16 + r) * 2];
      const float f = (mw == kNegInf) ? 0.f : exp2f(mw - M);
      L += sm_ml[(w * 16 + r) * 2 + 1] * f;
      O += sm_o[(w * 16 + r) * D + d] * f;
    }
    if (F8) O *= a.v_scale;
    const int head = hkv * G + r;
    if (nsplit == 1) {
      if (a.sinks != nullptr) {
        const float sk = a.sinks[head] * kLog2e;
        const float Mx = fmaxf(M, sk);
        const float f = (M == kNegInf) ? 0.f : exp2f(M - Mx);
        L = L * f + exp2f(sk - Mx);
        O *= f;
      }
      const float inv = L > 0.f ? 1.f / L : 0.f;
      reinterpret_cast<__nv_bfloat16*>(a.out)[((int64_t)b * a.Hq + head) * D + d] = __float2bfloat16(O * inv);
    } else {
      // workspace: [B, Hq, splits, D] partial O  followed by [B, Hq, splits, 2] (M, L)
      const int64_t slot = ((int64_t)b * a.Hq + head) * nsplit + split;
      a.ws[slot * D + d] = O;
      if (d == 0) {
        float* ml = a.ws + (int64_t)a.B * a.Hq * nsplit * D;
        ml[slot * 2] = M;
        ml[slot * 2 + 1] = L;
      }
    }
  }
}

template <int D>
__global__ void decode_merge_kernel(AttnArgs a, int nsplit) {
  pdl_wait();
  pdl_trigger();
  const int bh = blockIdx.x;  // b * Hq + head
  const int head = bh % a.Hq;
  const float* ml = a.ws + (int64_t)a.B * a.Hq * nsplit * D;
  float M = kNegInf;
  for (int s = 0; s < nsplit; ++s) M = fmaxf(M, ml[((int64_t)bh * nsplit + s) * 2]);
  float sk = kNegInf;
  if (a.sinks != nullptr) {
    sk = a.sinks[head] * kLog2e;
  }
  const float Mx = fmaxf(M, sk);
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float L = (sk == kNegInf) ? 0.f : exp2f(sk - Mx), O = 0.f;
    for (int s = 0; s < nsplit; ++s) {
      const float ms = ml[((int64_t)bh * nsplit + s) * 2];
      const float f = (ms == kNegInf) ? 0.f : exp2f(ms - Mx);
      L += ml[((int64_t)bh * nsplit + s) * 2 + 1] * f;
      O += a.ws[((int64_t)bh * nsplit + s) * D + d] * f;
    }
    reinterpret_cast<__nv_bfloat16*>(a.out)[(int64_t)bh * D + d] = __float2bfloat16(L > 0.f ? O / L : 0.f);
  }
}

// ---------------------------------------------------------------------------
// Prefill (causal over cached pages, or non-causal joint attention with
// paged query rows for the DiT): grid (B * q_tiles, Hkv), 8 compute
// warps (16 MMA rows each; row = token * G + head) + 1 TMA producer warp.
// K/V tiles of 64 keys (4 pages) in an NST-deep ring.
// ---------------------------------------------------------------------------
template <int D, int NST>
struct PreCfg {
  static constexpr int TILE_KEYS = 64;
  static constexpr int HALF = TILE_KEYS * D * 2;  // K (or V) bytes per stage
  static constexpr int STAGE_BYTES = 2 * HALF;
  static constexpr int SMEM = 1024 + NST * STAGE_BYTES + 2 * NST * 8 + 64;
};

template <int D, int NST>
__global__ void __launch_bounds__(288) prefill_attn_kernel(const __grid_constant__ CUtensorMap tmK,
                                                           const __grid_constant__ CUtensorMap tmV, AttnArgs a,
                                                           int q_tiles, int rows_tok) {
  using Cf = PreCfg<D, NST>;
  extern __shared__ uint8_t smem_dyn[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + NST * Cf::STAGE_BYTES);
  uint64_t* empty = full + NST;

  pdl_wait();
  pdl_trigger();
  const int G = a.Hq / a.Hkv;
  const int b = blockIdx.x / q_tiles;
  const int qt = blockIdx.x % q_tiles;
  const int hkv = blockIdx.y;
  const int q0 = a.cu_q[b];
  const int q_len = a.cu_q[b + 1] - q0;
  const int tok0 = qt * rows_tok;  // first query (within this sequence) of the tile
  if (tok0 >= q_len) return;
  const int ntok = min(rows_tok, q_len - tok0);
  const int ctx = a.ctx_lens[b];
  const int pos_base = ctx - q_len;  // position of query 0
  const int pos_lo = pos_base + tok0, pos_hi = pos_base + tok0 + ntok - 1;
  const bool causal = a.causal != 0;
  int k_begin = 0;
  if (causal && a.window > 0) k_begin = max(0, pos_lo - a.window + 1);
  k_begin &= ~(Cf::TILE_KEYS - 1);
  const int k_end = causal ? pos_hi + 1 : ctx;
  const int ntiles = (k_end - k_begin + Cf::TILE_KEYS - 1) / Cf::TILE_KEYS;
  const int32_t* btab = a.block_tables + (int64_t)b * a.max_blocks;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NST; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 8);
    }
    fence_mbarrier_init();
  }
  __syncthreads();

  if (warp == 8) {
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      const int max_page = (ctx + 15) >> 4;
      for (int it = 0; it < ntiles; ++it) {
        if (!mbar_wait(&empty[s], ph ^ 1, a.status, kErrTimeoutEmpty)) break;
        uint8_t* st = smem + s * Cf::STAGE_BYTES;
        mbar_arrive_expect_tx(&full[s], Cf::STAGE_BYTES);
        const int page0 = (k_begin >> 4) + it * 4;
        for (int pg = 0; pg < 4; ++pg) {
          const int page = page0 + pg;
          // pages beyond the context reuse a valid page; their keys are masked
          const int blk = btab[min(page, max_page - 1)];
          const int row = (blk * a.Hkv + hkv) * 16;
#pragma unroll
          for (int bx = 0; bx < D / 64; ++bx) {
            // box bx holds dims [64 bx, 64 bx + 64) of all 64 keys: [64 rows][128 B]
            tma_load_2d(st + bx * (Cf::TILE_KEYS * 128) + pg * 16 * 128, &tmK, &full[s], bx * 64, row);
            tma_load_2d(st + Cf::HALF + bx * (Cf::TILE_KEYS * 128) + pg * 16 * 128, &tmV, &full[s], bx * 64, row);
          }
        }
        if (++s == NST) {
          s = 0;
          ph ^= 1;
        }
      }
    }
    return;
  }

  const int g = lane >> 2, t4 = lane & 3;
  const float scale_log2 = a.scale * kLog2e;
  // rows of this warp: warp*16 + {g, g+8}; row -> (token, head)
  int r_tok[2], r_head[2], r_pos[2];
  bool r_ok[2];
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int row = warp * 16 + g + r * 8;
    r_tok[r] = row / G;
    r_head[r] = row % G;
    r_ok[r] = r_tok[r] < ntok;
    r_pos[r] = pos_base + tok0 + r_tok[r];
  }
  // query / output row of the sequence's token t
  auto q_row = [&](int t) -> int64_t {
    return a.q_paged ? (int64_t)btab[t >> 4] * 16 + (t & 15) : (int64_t)(q0 + t);
  };
  uint32_t qa[D / 16][4];
  {
    const __nv_bfloat16* qb = reinterpret_cast<const __nv_bfloat16*>(a.q);
#pragma unroll
    for (int ks = 0; ks < D / 16; ++ks)
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const int r = h & 1;
        const int c = ks * 16 + 2 * t4 + ((h & 2) ? 8 : 0);
        qa[ks][h] = r_ok[r] ? *reinterpret_cast<const uint32_t*>(
                                  qb + (q_row(tok0 + r_tok[r]) * a.Hq + hkv * G + r_head[r]) * D + c)
                            : 0u;
      }
  }
  float m_r[2] = {kNegInf, kNegInf}, l_r[2] = {0.f, 0.f};
  float o[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;

  const int mi = lane >> 3, rr = lane & 7;
  int s = 0;
  uint32_t ph = 0;
  for (int it = 0; it < ntiles; ++it) {
    if (!mbar_wait(&full[s], ph, a.status, kErrTimeoutFull)) break;
    const uint32_t kb = smem_u32(smem + s * Cf::STAGE_BYTES);
    const uint32_t vb = kb + Cf::HALF;
    const int key0 = k_begin + it * Cf::TILE_KEYS;
    float sc[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < D / 16; ++ks) {
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        const int tok = np * 16 + (mi >> 1) * 8 + rr;
        const int d0 = ks * 16 + (mi & 1) * 8;
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4(kb + sw128_off(tok, d0, Cf::TILE_KEYS), b0, b1, b2, b3);
        mma_bf16_16816(sc[np * 2], qa[ks], b0, b1);
        mma_bf16_16816(sc[np * 2 + 1], qa[ks], b2, b3);
      }
    }
    float mx[2] = {kNegInf, kNegInf};
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const int r = h >> 1;
        const int kp = key0 + nt * 8 + 2 * t4 + (h & 1);
        const bool ok = r_ok[r] && kp < ctx &&
                        (!causal || (kp <= r_pos[r] && (a.window <= 0 || kp > r_pos[r] - a.window)));
        sc[nt][h] = ok ? score_log2(sc[nt][h], a, scale_log2) : kNegInf;
        mx[r] = fmaxf(mx[r], sc[nt][h]);
      }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
    }
    float corr[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const float mn = fmaxf(m_r[r], mx[r]);
      corr[r] = (mn == kNegInf) ? 1.f : exp2f(m_r[r] - mn);
      m_r[r] = mn;
      l_r[r] *= corr[r];
    }
#pragma unroll
    for (int dn = 0; dn < D / 8; ++dn) {
      o[dn][0] *= corr[0];
      o[dn][1] *= corr[0];
      o[dn][2] *= corr[1];
      o[dn][3] *= corr[1];
    }
#pragma unroll
    for (int kc = 0; kc < 4; ++kc) {  // 16 keys per P fragment
      uint32_t pa[4];
      float p[2][4];
#pragma unroll
      for (int q = 0; q < 2; ++q)
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          const float mm = m_r[h >> 1];
          p[q][h] = (mm == kNegInf) ? 0.f : exp2f(sc[kc * 2 + q][h] - mm);
          l_r[h >> 1] += p[q][h];
        }
      pa[0] = pack_bf16x2(p[0][0], p[0][1]);
      pa[1] = pack_bf16x2(p[0][2], p[0][3]);
      pa[2] = pack_bf16x2(p[1][0], p[1][1]);
      pa[3] = pack_bf16x2(p[1][2], p[1][3]);
#pragma unroll
      for (int dp = 0; dp < D / 16; ++dp) {
        const int tok = kc * 16 + (mi & 1) * 8 + rr;
        const int d0 = (dp * 2 + (mi >> 1)) * 8;
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4_trans(vb + sw128_off(tok, d0, Cf::TILE_KEYS), b0, b1, b2, b3);
        mma_bf16_16816(o[dp * 2], pa, b0, b1);
        mma_bf16_16816(o[dp * 2 + 1], pa, b2, b3);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
    if (++s == NST) {
      s = 0;
      ph ^= 1;
    }
  }
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    l_r[r] += __shfl_xor_sync(0xffffffffu, l_r[r], 1);
    l_r[r] += __shfl_xor_sync(0xffffffffu, l_r[r], 2);
  }
  __nv_bfloat16* ob = reinterpret_cast<__nv_bfloat16*>(a.out);
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    if (!r_ok[r]) continue;
    const int head = hkv * G + r_head[r];
    float L = l_r[r], M = m_r[r], f = 1.f;
    if (a.sinks != nullptr) {
      const float sk = a.sinks[head] * kLog2e;
      const float Mx = fmaxf(M, sk);
      f = (M == kNegInf) ? 0.f : exp2f(M - Mx);
      L = L * f + exp2f(sk - Mx);
    }
    const float inv = L > 0.f ? f / L : 0.f;
    __nv_bfloat16* dst = ob + q_row(tok0 + r_tok[r]) * (a.out_ld ? a.out_ld : (int64_t)a.Hq * D) + (int64_t)head * D;
#pragma unroll
    for (int dn = 0; dn < D / 8; ++dn) {
      const int c = dn * 8 + 2 * t4;
      *reinterpret_cast<uint32_t*>(dst + c) = pack_bf16x2(o[dn][r * 2] * inv, o[dn][r * 2 + 1] * inv);
    }
  }
}


}  // namespace attn

int decode_attention_launch(const AttnArgs& a, cudaStream_t st) {
  using namespace attn;
  if (a.B == 0) return 0;
  const int G = a.Hq / a.Hkv;
  if (G > 16 || a.Hq % a.Hkv != 0) throw std::runtime_error("b200.decode_attention: G must divide and be <= 16");
  if (a.D != 256 && a.D != 128 && a.D != 64) throw std::runtime_error("b200.decode_attention: D must be 64, 128 or 256");
  const int64_t rows = a.num_blocks * a.Hkv * 16;
  const bool f8 = a.kv_fp8 != 0;
  // e4m3 pages: one unswizzled [16, D]-byte box per page (D <= 256 bytes per row)
  CUtensorMap tk = f8 ? make_tmap_2d(a.k_cache, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, rows, a.D, a.D, 16, a.D,
                                     CU_TENSOR_MAP_SWIZZLE_NONE)
                      : make_tmap_2d(a.k_cache, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, rows, a.D, a.D, 16, 64);
  CUtensorMap tv = f8 ? make_tmap_2d(a.v_cache, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, rows, a.D, a.D, 16, a.D,
                                     CU_TENSOR_MAP_SWIZZLE_NONE)
                      : make_tmap_2d(a.v_cache, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, rows, a.D, a.D, 16, 64);
  int splits = a.splits;
  const int sms = num_sms(a.device);
  AttnArgs args = a;
  if (splits <= 0) {
    const int ctas = a.B * a.Hkv;
    // split the KV range only when (sequence, kv-head) pairs leave SMs idle: measured on B200 at Hkv 8,
    // ctx 1400, one split beats two at 256 pairs (42.4 vs 48.3 us) and at 512 (79.4 vs 90.8 us); fixed
    // 32-page chunks per CTA (B200_DECODE_CHUNK) measured slower still (6.87 vs 6.23 ms per Qwen3-8B
    // decode step at batch 64): the extra partials and the merge cost more than the shorter tail saves
    splits = std::max(1, std::min(16, (3 * sms + ctas - 1) / ctas));
    if (ctas >= sms) splits = 1;
    if (const char* e = std::getenv("B200_DECODE_CHUNK")) {
      int chunk = std::max(1, std::atoi(e));
      while (chunk < a.max_blocks &&
             (int64_t)a.B * a.Hq * ((a.max_blocks + chunk - 1) / chunk) * (a.D + 2) > a.ws_elems)
        chunk *= 2;
      splits = (a.max_blocks + chunk - 1) / chunk;
      args.chunk_pages = splits > 1 ? chunk : 0;
    }
  }
  if (splits > 1 && a.ws_elems < (int64_t)a.B * a.Hq * splits * (a.D + 2))
    throw std::runtime_error("b200.decode_attention: split workspace too small");
  dim3 grid(a.B * a.Hkv, splits);
  auto run = [&](auto dtag, auto ntag, auto ftag) {
    constexpr int Dv = decltype(dtag)::value, NST = decltype(ntag)::value;
    constexpr bool F8 = decltype(ftag)::value;
    auto k = decode_attn_kernel<Dv, NST, F8>;
    ensure_smem(k, DecCfg<Dv, NST, F8>::SMEM);
    launch_pdl(k, grid, dim3(160), DecCfg<Dv, NST, F8>::SMEM, st, tk, tv, args);
    if (splits > 1) launch_pdl(decode_merge_kernel<Dv>, dim3(a.B * a.Hq), dim3(Dv), 0, st, args, splits);
  };
  using I256 = std::integral_constant<int, 256>;
  using I128 = std::integral_constant<int, 128>;
  using I64 = std::integral_constant<int, 64>;
  using N4 = std::integral_constant<int, 4>;
  using N8 = std::integral_constant<int, 8>;
  if (a.D == 256) {
    if (f8) run(I256{}, N4{}, std::true_type{}); else run(I256{}, N4{}, std::false_type{});
  } else if (a.D == 128) {
    if (f8) run(I128{}, N8{}, std::true_type{}); else run(I128{}, N8{}, std::false_type{});
  } else {
    if (f8) run(I64{}, N8{}, std::true_type{}); else run(I64{}, N8{}, std::false_type{});
  }
  return splits > 1 ? 2 : 1;
}

namespace attn {
// One CTA per (sequence, page): all kv heads of the page, K and V, e4m3 -> bf16.
__global__ void __launch_bounds__(256) kv_dequant_pages_kernel(const uint8_t* __restrict__ k8,
                                                               const uint8_t* __restrict__ v8,
                                                               const int32_t* __restrict__ tables,
                                                               const int32_t* __restrict__ ctx_lens, int max_blocks,
                                                               int64_t page_bytes, float ks, float vs,
                                                               __nv_bfloat16* __restrict__ k_out,
                                                               __nv_bfloat16* __restrict__ v_out) {
  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.x / max_blocks, p = blockIdx.x % max_blocks;
  if (p * 16 >= ctx_lens[b]) return;
  const int64_t src = (int64_t)tables[(int64_t)b * max_blocks + p] * page_bytes;
  const int64_t dst = (int64_t)blockIdx.x * page_bytes;
  for (int64_t i = threadIdx.x * 16; i < page_bytes; i += 256 * 16) {
    uint4 lo, hi;
    fp8x16_to_bf16(*reinterpret_cast<const uint4*>(k8 + src + i), lo, hi);
    if (ks != 1.f) {
      __nv_bfloat16* e = reinterpret_cast<__nv_bfloat16*>(&lo);
      __nv_bfloat16* f = reinterpret_cast<__nv_bfloat16*>(&hi);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        e[q] = __float2bfloat16(__bfloat162float(e[q]) * ks);
        f[q] = __float2bfloat16(__bfloat162float(f[q]) * ks);
      }
    }
    *reinterpret_cast<uint4*>(k_out + dst + i) = lo;
    *reinterpret_cast<uint4*>(k_out + dst + i + 8) = hi;
    fp8x16_to_bf16(*reinterpret_cast<const uint4*>(v8 + src + i), lo, hi);
    if (vs != 1.f) {
      __nv_bfloat16* e = reinterpret_cast<__nv_bfloat16*>(&lo);
      __nv_bfloat16* f = reinterpret_cast<__nv_bfloat16*>(&hi);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        e[q] = __float2bfloat16(__bfloat162float(e[q]) * vs);
        f[q] = __float2bfloat16(__bfloat162float(f[q]) * vs);
      }
    }
    *reinterpret_cast<uint4*>(v_out + dst + i) = lo;
    *reinterpret_cast<uint4*>(v_out + dst + i + 8) = hi;
  }
}
}  // namespace attn

void kv_dequant_pages_launch(const void* k8, const void* v8, const int32_t* block_tables, const int32_t* ctx_lens,
                             int B, int max_blocks, int Hkv, int D, float k_scale, float v_scale, void* k_out,
                             void* v_out, cudaStream_t st) {
  if (B == 0 || max_blocks == 0) return;
  launch_pdl(attn::kv_dequant_pages_kernel, dim3((unsigned)(B * max_blocks)), dim3(256), 0, st,
             reinterpret_cast<const uint8_t*>(k8), reinterpret_cast<const uint8_t*>(v8), block_tables, ctx_lens,
             max_blocks, (int64_t)Hkv * 16 * D, k_scale, v_scale, reinterpret_cast<__nv_bfloat16*>(k_out),
             reinterpret_cast<__nv_bfloat16*>(v_out));
}

void prefill_attention_launch(const AttnArgs& a, cudaStream_t st) {
  using namespace attn;
  if (a.B == 0) return;
  if (fmha_supported(a)) {
    fmha_launch(a, st);
    return;
  }
  if (a.kv_dense) throw std::runtime_error("b200.prefill_attention: row-major K/V needs the tcgen05 kernel (D 128)");
  const int G = a.Hq / a.Hkv;
  if (a.Hq % a.Hkv != 0 || 128 % G != 0) throw std::runtime_error("b200.prefill_attention: G must divide 128");
  if (a.D != 256 && a.D != 128 && a.D != 64)
    throw std::runtime_error("b200.prefill_attention: D must be 64, 128 or 256");
  const int64_t rows = a.num_blocks * a.Hkv * 16;
  CUtensorMap tk = make_tmap_2d(a.k_cache, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, rows, a.D, a.D, 16, 64);
  CUtensorMap tv = make_tmap_2d(a.v_cache, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, rows, a.D, a.D, 16, 64);
  const int rows_tok = 128 / G;
  const int q_tiles = (a.max_q_len + rows_tok - 1) / rows_tok;
  dim3 grid(a.B * q_tiles, a.Hkv);
  if (a.D == 256) {
    constexpr int NST = 2;
    auto k = prefill_attn_kernel<256, NST>;
    ensure_smem(k, PreCfg<256, NST>::SMEM);
    launch_pdl(k, grid, dim3(288), PreCfg<256, NST>::SMEM, st, tk, tv, a, q_tiles, rows_tok);
  } else if (a.D == 128) {
    constexpr int NST = 2;
    auto k = prefill_attn_kernel<128, NST>;
    ensure_smem(k, PreCfg<128, NST>::SMEM);
    launch_pdl(k, grid, dim3(288), PreCfg<128, NST>::SMEM, st, tk, tv, a, q_tiles, rows_tok);
  } else {
    constexpr int NST = 3;
    auto k = prefill_attn_kernel<64, NST>;
    ensure_smem(k, PreCfg<64, NST>::SMEM);
    launch_pdl(k, grid, dim3(288), PreCfg<64, NST>::SMEM, st, tk, tv, a, q_tiles, rows_tok);
  }
}

}  // namespace b200

// ---------------------------------------------------------------------------
// Allocation-free variant of decode attention (see decode_attention_noalloc.h).
// Launches the same split-KV and merge kernels as decode_attention_launch, but
// the split partials go to a file-scope device array instead of a caller- or
// torch-allocated workspace.
// ---------------------------------------------------------------------------
#include <mutex>

#include "decode_attention_noalloc.h"

namespace b200 {
namespace attn_noalloc {

// Per-split partial outputs and (max, sum) pairs of every call on this device.
static __device__ __align__(256) float g_decode_scratch[B200_NOALLOC_SCRATCH_FLOATS];

constexpr int kMaxDevices = 64;
static float* g_scratch_ptr[kMaxDevices] = {nullptr};
static bool g_attr_done[kMaxDevices] = {false};
static std::mutex g_setup_mu;

// Once per device, with that device current: resolve the array's device
// address (host code must not use the symbol itself) and raise the kernels'
// dynamic shared-memory limit.
static int setup(int dev, float** ptr) {
  if (dev < 0 || dev >= kMaxDevices) return B200_NOALLOC_ERR_SETUP;
  std::lock_guard<std::mutex> lk(g_setup_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_decode_scratch) != cudaSuccess || p == nullptr) return B200_NOALLOC_ERR_SETUP;
    g_scratch_ptr[dev] = static_cast<float*>(p);
  }
  if (!g_attr_done[dev]) {
    using namespace attn;
    if (cudaFuncSetAttribute(decode_attn_kernel<128, 8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             DecCfg<128, 8>::SMEM) != cudaSuccess ||
        cudaFuncSetAttribute(decode_attn_kernel<64, 8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             DecCfg<64, 8>::SMEM) != cudaSuccess)
      return B200_NOALLOC_ERR_SETUP;
    g_attr_done[dev] = true;
  }
  *ptr = g_scratch_ptr[dev];
  return B200_NOALLOC_OK;
}

}  // namespace attn_noalloc
}  // namespace b200

extern "C" int b200_decode_attention_noalloc(const void* q, const void* k_cache, const void* v_cache,
                                             int64_t num_blocks, const int32_t* block_tables, int max_blocks,
                                             const int32_t* ctx_lens, void* out, const float* sinks, int window,
                                             int B, int Hq, int Hkv, int D, float scale, int splits, int* status,
                                             void* stream) {
  using namespace b200;
  using namespace b200::attn;
  if (q == nullptr || k_cache == nullptr || v_cache == nullptr || block_tables == nullptr || ctx_lens == nullptr ||
      out == nullptr || B <= 0 || Hq <= 0 || Hkv <= 0 || num_blocks <= 0 || max_blocks <= 0 || splits < 1)
    return B200_NOALLOC_ERR_ARGS;
  if (Hq % Hkv != 0 || Hq / Hkv > 16 || (D != 64 && D != 128)) return B200_NOALLOC_ERR_ARGS;
  if ((int64_t)B * Hq * splits * (D + 2) > (int64_t)B200_NOALLOC_SCRATCH_FLOATS) return B200_NOALLOC_ERR_SCRATCH;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return B200_NOALLOC_ERR_SETUP;
  float* scratch = nullptr;
  const int rc = attn_noalloc::setup(dev, &scratch);
  if (rc != B200_NOALLOC_OK) return rc;

  AttnArgs a{};
  a.q = q;
  a.k_cache = k_cache;
  a.v_cache = v_cache;
  a.num_blocks = num_blocks;
  a.block_tables = block_tables;
  a.max_blocks = max_blocks;
  a.ctx_lens = ctx_lens;
  a.cu_q = nullptr;
  a.out = out;
  a.sinks = sinks;
  a.window = window;
  a.B = B;
  a.Hq = Hq;
  a.Hkv = Hkv;
  a.D = D;
  a.scale = scale;
  a.splits = splits;
  a.ws = scratch;
  a.ws_elems = B200_NOALLOC_SCRATCH_FLOATS;
  a.status = status;
  a.device = dev;
  CUtensorMap tk, tv;
  try {
    const int64_t rows = num_blocks * Hkv * 16;
    tk = make_tmap_2d(k_cache, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, rows, D, D, 16, 64);
    tv = make_tmap_2d(v_cache, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, rows, D, D, 16, 64);
  } catch (...) {
    return B200_NOALLOC_ERR_TMA;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // cudaLaunchKernelEx returns this launch's own error; an error left pending
  // by unrelated earlier work on the thread is neither reported nor cleared here
  auto launch = [&](auto kern, dim3 grid, int threads, size_t smem, auto... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    return cudaLaunchKernelEx(&cfg, kern, args...) == cudaSuccess;
  };
  const dim3 grid(B * Hkv, splits);
  bool ok;
  if (D == 128) {
    ok = launch(decode_attn_kernel<128, 8>, grid, 160, DecCfg<128, 8>::SMEM, tk, tv, a);
    if (ok && splits > 1) ok = launch(decode_merge_kernel<128>, dim3(B * Hq), 128, 0, a, splits);
  } else {
    ok = launch(decode_attn_kernel<64, 8>, grid, 160, DecCfg<64, 8>::SMEM, tk, tv, a);
    if (ok && splits > 1) ok = launch(decode_merge_kernel<64>, dim3(B * Hq), 64, 0, a, splits);
  }
  return ok ? B200_NOALLOC_OK : B200_NOALLOC_ERR_LAUNCH;
}
