// Flash attention forward on the 5th-generation tensor cores (head_dim 128).
//
// One CTA per (sequence, tile of 128 query rows, kv head); rows are
// (token, query head) pairs of one GQA group (row = token * G + g), so every
// K/V page is read once per kv head. Warp roles:
//   warp 0     TMA producer: the Q tile once (3-D boxes [16 tokens][G heads]
//              [64 dims]), then K and V tiles of 128 keys (eight 16-key pages)
//              into a 3-deep ring, K and V on separate barriers;
//   warp 1     MMA issuer (one thread): S_j = Q K_j^T into a double-buffered
//              TMEM tile, then O += P_j V_j with P_j read from TMEM (A operand)
//              and V_j from shared memory as an MN-major B operand;
//   warps 2-5  softmax, one query row per thread (TMEM lane quadrant =
//              warp % 4): row max over the masked S tile, P = exp2(S*scale -
//              m) written back over the consumed S columns as bf16, row sums
//              in fp32. The running max is rescaled lazily: O (in TMEM) is
//              corrected only when the max grows by more than 2^8, so most
//              tiles never touch O. At the end they normalise O (learned sink
//              logits join the denominator) and store the rows.
// TMEM: S0 [0,128), S1 [128,256), O [256,384) of 512 allocated columns.
// The MMA for S_{j+1} overlaps the softmax of tile j; S_{j+1} reuses the S
// buffer of tile j-1 only after P_{j-1} V_{j-1} has completed.
//
// Masks: causal over absolute positions (queries are the last q_len of ctx
// positions), sliding window, context length; the DiT joint attention runs
// non-causally with query rows placed through the key block table.
//
// Reference behaviour: the fused SDPA of rlx-models-core
// src/standard_decoder.rs:11946-12079 (sinks, sliding window) and rlx-flux1
// src/transformer.rs:327-340 (joint, unmasked attention).
#include <cuda_bf16.h>

#include <algorithm>
#include <cstdlib>
#include <stdexcept>

#include "../common/b200.cuh"
#include "../common/launch.h"
#include "../common/pdl_launch.h"
#include "../common/tma_host.h"

namespace b200 {
namespace fmha {

constexpr int kD = 128;
constexpr int kBN = 128;                   // keys per tile
constexpr int kNST = 3;                    // K/V ring depth
constexpr uint32_t kHalf = 128 * 64 * 2;   // [128 rows][64 dims] bf16, 128B-swizzled
constexpr uint32_t kQ = 2 * kHalf;
constexpr uint32_t kKV = 2 * kHalf;        // one K (or V) tile
constexpr uint32_t kStage = 2 * kKV;
constexpr uint32_t kSmem = 1024 + kQ + kNST * kStage + 256;
constexpr int kThreads = 192;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kOCol = 256;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescale = 8.f;            // lazy rescale threshold (log2 units)

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void tma_load_3d_q(void* dst, const CUtensorMap* m, uint64_t* bar, int x, int y, int z) {
  tma_load_3d(dst, m, bar, x, y, z);
}

__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]),
      "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]),
      "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

__global__ void __launch_bounds__(kThreads, 1)
    fmha_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const AttnArgs a, int q_tiles, int rows_tok) {
  extern __shared__ uint8_t smem_dyn[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~uintptr_t(1023));
  uint8_t* Qs = smem;
  uint8_t* KVs = smem + kQ;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kQ + kNST * kStage);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* v_full = k_full + kNST;
  uint64_t* kv_empty = v_full + kNST;
  uint64_t* s_full = kv_empty + kNST;
  uint64_t* p_full = s_full + 2;
  uint64_t* o_done = p_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_done + 2);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  pdl_wait();
  pdl_trigger();
  const int G = a.Hq / a.Hkv;
  const int b = blockIdx.x / q_tiles, qt = blockIdx.x % q_tiles, hkv = blockIdx.y;
  const int q0 = a.cu_q[b];
  const int q_len = a.cu_q[b + 1] - q0;
  const int tok0 = qt * rows_tok;
  if (tok0 >= q_len) return;  // uniform for the CTA, before any barrier or TMEM use
  const int ntok = min(rows_tok, q_len - tok0);
  const int ctx = a.ctx_lens[b];
  const int pos_base = ctx - q_len;
  const bool causal = a.causal != 0;
  const int pos_lo = pos_base + tok0, pos_hi = pos_base + tok0 + ntok - 1;
  int k_begin = 0;
  if (causal && a.window > 0) k_begin = max(0, pos_lo - a.window + 1);
  k_begin &= ~(kBN - 1);
  const int k_end = causal ? min(ctx, pos_hi + 1) : ctx;
  const int n_tiles = max(1, (k_end - k_begin + kBN - 1) / kBN);
  const int32_t* btab = a.block_tables + (int64_t)b * a.max_blocks;
  const int max_page = max(1, (ctx + 15) >> 4);

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < kNST; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 4);
      mbar_init(&o_done[i], 1);
    }
    fence_mbarrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (elect_one_sync()) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      mbar_arrive_expect_tx(q_full, kQ);
      for (int c = 0; c < rows_tok / 16; ++c) {
        const int t = tok0 + 16 * c;
        const int row = a.q_paged ? btab[min(t >> 4, max_page - 1)] * 16 : q0 + t;
#pragma unroll
        for (int h = 0; h < 2; ++h)
          tma_load_3d_q(Qs + h * kHalf + c * (16 * G * 128), &tmQ, q_full, h * 64, hkv * G, row);
      }
      int s = 0;
      uint32_t ph = 0;
      for (int j = 0; j < n_tiles; ++j) {
        if (!mbar_wait(&kv_empty[s], ph ^ 1, a.status, kErrTimeoutEmpty)) break;
        uint8_t* st = KVs + s * kStage;
        const int page0 = (k_begin >> 4) + j * (kBN / 16);
        mbar_arrive_expect_tx(&k_full[s], kKV);
        for (int pg = 0; pg < kBN / 16; ++pg) {
          const int blk = btab[min(page0 + pg, max_page - 1)];  // pages past the context are masked
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            if (a.kv_dense)
              tma_load_3d(st + h * kHalf + pg * 2048, &tmK, &k_full[s], h * 64, hkv, blk * 16);
            else
              tma_load_2d(st + h * kHalf + pg * 2048, &tmK, &k_full[s], h * 64, (blk * a.Hkv + hkv) * 16);
          }
        }
        mbar_arrive_expect_tx(&v_full[s], kKV);
        for (int pg = 0; pg < kBN / 16; ++pg) {
          const int blk = btab[min(page0 + pg, max_page - 1)];
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            if (a.kv_dense)
              tma_load_3d(st + kKV + h * kHalf + pg * 2048, &tmV, &v_full[s], h * 64, hkv, blk * 16);
            else
              tma_load_2d(st + kKV + h * kHalf + pg * 2048, &tmV, &v_full[s], h * 64, (blk * a.Hkv + hkv) * 16);
          }
        }
        if (++s == kNST) {
          s = 0;
          ph ^= 1;
        }
      }
    }
  } else if (warp == 1) {
    if (elect_one_sync()) {
      constexpr uint32_t idS = umma_idesc_bf16(128, kBN, false, false);
      constexpr uint32_t idO = umma_idesc_bf16(128, kD, false, true);  // V: MN-major B
      const uint32_t qa = smem_u32(Qs);
      bool ok = mbar_wait(q_full, 0, a.status, kErrTimeoutFull);
      auto stage_of = [](int j) { return j % kNST; };
      auto phase_of = [](int j) { return (uint32_t)((j / kNST) & 1); };
      if (ok) ok = mbar_wait(&k_full[0], 0, a.status, kErrTimeoutFull);
      if (ok) {
        tc_fence_after();
        const uint32_t kb = smem_u32(KVs);
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk) {
          const uint32_t off = (kk >> 2) * kHalf + (kk & 3) * 32;
          umma_f16(tmem, umma_desc_sw128(qa + off, 16, 1024), umma_desc_sw128(kb + off, 16, 1024), idS,
                   kk > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[0]);
      }
      for (int j = 0; ok && j < n_tiles; ++j) {
        if (j + 1 < n_tiles) {
          // S buffer (j+1)&1 held P_{j-1}: wait until P_{j-1} V_{j-1} has completed
          if (j >= 1 && !mbar_wait(&o_done[(j - 1) & 1], ((j - 1) >> 1) & 1, a.status, kErrTimeoutAccEmpty)) break;
          if (!mbar_wait(&k_full[stage_of(j + 1)], phase_of(j + 1), a.status, kErrTimeoutFull)) break;
          tc_fence_after();
          const uint32_t kb = smem_u32(KVs + stage_of(j + 1) * kStage);
          const uint32_t d = tmem + ((j + 1) & 1) * kBN;
#pragma unroll
          for (int kk = 0; kk < kD / 16; ++kk) {
            const uint32_t off = (kk >> 2) * kHalf + (kk & 3) * 32;
            umma_f16(d, umma_desc_sw128(qa + off, 16, 1024), umma_desc_sw128(kb + off, 16, 1024), idS,
                     kk > 0 ? 1u : 0u);
          }
          umma_commit(&s_full[(j + 1) & 1]);
        }
        if (!mbar_wait(&p_full[j & 1], (j >> 1) & 1, a.status, kErrTimeoutFull)) break;
        if (!mbar_wait(&v_full[stage_of(j)], phase_of(j), a.status, kErrTimeoutFull)) break;
        tc_fence_after();
        const uint32_t pa = tmem + (j & 1) * kBN;  // P_j: bf16 pairs in columns [0, 64) of its S buffer
        const uint32_t vb = smem_u32(KVs + stage_of(j) * kStage + kKV);
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk)
          umma_f16_ts(tmem + kOCol, pa + kk * 8, umma_desc_sw128(vb + kk * 2048, kHalf, 1024), idO,
                      (j > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&o_done[j & 1]);
        umma_commit(&kv_empty[stage_of(j)]);
      }
    }
  } else {
    // softmax / correction / epilogue: one query row per thread
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const int tok = row / G, g = row % G;
    const bool row_ok = tok < ntok;
    const int qpos = pos_base + tok0 + tok;
    const float sl2 = a.scale * kLog2e;
    const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16);
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    // tcgen05.ld / st / wait are warp-collective (.sync.aligned): every branch
    // around them below is warp-uniform; per-row choices only pick values.
    for (int j = 0; j < n_tiles; ++j) {
      if (!__all_sync(0xffffffffu, mbar_wait(&s_full[j & 1], (j >> 1) & 1, a.status, kErrTimeoutAccFull))) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t sb = lane_base + (j & 1) * kBN;
      const int key0 = k_begin + j * kBN;
      // keys of this tile visible to the row: [lo, hi)
      int lo = 0, hi = 0;
      if (row_ok) {
        int kmin = 0, kmax = ctx;  // absolute positions
        if (causal) {
          kmax = min(kmax, qpos + 1);
          if (a.window > 0) kmin = max(kmin, qpos - a.window + 1);
        }
        lo = max(0, kmin - key0);
        hi = min(kBN, kmax - key0);
      }
      float mx = -INFINITY;
#pragma unroll 1
      for (int c = 0; c < kBN / 32; ++c) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(sb + c * 32, v);
        tmem_wait_ld();
#pragma unroll
        for (int t = 0; t < 32; ++t)
          if (c * 32 + t >= lo && c * 32 + t < hi) mx = fmaxf(mx, __uint_as_float(v[t]));
      }
      const float m_tile = mx * sl2;
      const bool grow = m_tile > m_used + kRescale;  // this row's max moved by more than 2^8
      if (__any_sync(0xffffffffu, grow) && j > 0) {
        // O holds P V of earlier tiles: wait for the last one, then rescale the rows that grew
        if (!__all_sync(0xffffffffu,
                        mbar_wait(&o_done[(j - 1) & 1], ((j - 1) >> 1) & 1, a.status, kErrTimeoutAccFull))) {
          ok = false;
          break;
        }
        tc_fence_after();
        // rows whose max was still -inf have an all-zero O row: any factor works
        const float f = grow ? (m_used == -INFINITY ? 0.f : ex2(m_used - m_tile)) : 1.f;
#pragma unroll 1
        for (int c = 0; c < kD / 32; ++c) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(lane_base + kOCol + c * 32, v);
          tmem_wait_ld();
#pragma unroll
          for (int t = 0; t < 32; ++t) v[t] = __float_as_uint(__uint_as_float(v[t]) * f);
          tmem_st_32x32b_x32(lane_base + kOCol + c * 32, v);
        }
        tmem_wait_st();
        l *= f;
      }
      if (grow) m_used = m_tile;
#pragma unroll 1
      for (int c = 0; c < kBN / 32; ++c) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(sb + c * 32, v);
        tmem_wait_ld();
        uint32_t pk[16];
#pragma unroll
        for (int t = 0; t < 32; t += 2) {
          const int k0 = c * 32 + t;
          const float p0 = (k0 >= lo && k0 < hi) ? ex2(__uint_as_float(v[t]) * sl2 - m_used) : 0.f;
          const float p1 = (k0 + 1 >= lo && k0 + 1 < hi) ? ex2(__uint_as_float(v[t + 1]) * sl2 - m_used) : 0.f;
          l += p0 + p1;
          pk[t / 2] = pack_bf16x2(p0, p1);
        }
        tmem_st_32x32b_x16(sb + c * 16, pk);  // over S columns already consumed
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[j & 1]);
    }
    if (ok && __all_sync(0xffffffffu, mbar_wait(&o_done[(n_tiles - 1) & 1], ((n_tiles - 1) >> 1) & 1, a.status,
                                                kErrTimeoutAccFull))) {
      tc_fence_after();
      const int head = hkv * G + g;
      float L = l, f = 1.f;
      if (a.sinks != nullptr) {
        const float sk = a.sinks[head] * kLog2e;
        const float Mx = fmaxf(m_used, sk);
        f = (m_used == -INFINITY) ? 0.f : ex2(m_used - Mx);
        L = L * f + ex2(sk - Mx);
      }
      const float inv = L > 0.f ? f / L : 0.f;
      const int t = tok0 + tok;
      if (a.lse != nullptr && a.sinks == nullptr && row_ok && !a.q_paged)  // training: log2-sum-exp2 of the scaled row
        a.lse[(int64_t)(q0 + t) * a.Hq + head] = L > 0.f ? m_used + __log2f(L) : -INFINITY;
      const int64_t orow = a.q_paged ? (int64_t)btab[min(t >> 4, max_page - 1)] * 16 + (t & 15) : (int64_t)(q0 + t);
      __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(a.out) +
                           orow * (a.out_ld ? a.out_ld : (int64_t)a.Hq * kD) + (int64_t)head * kD;
#pragma unroll 1
      for (int c = 0; c < kD / 32; ++c) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(lane_base + kOCol + c * 32, v);
        tmem_wait_ld();
        if (row_ok) {
#pragma unroll
          for (int qd = 0; qd < 4; ++qd) {
            uint4 w;
            w.x = pack_bf16x2(__uint_as_float(v[qd * 8 + 0]) * inv, __uint_as_float(v[qd * 8 + 1]) * inv);
            w.y = pack_bf16x2(__uint_as_float(v[qd * 8 + 2]) * inv, __uint_as_float(v[qd * 8 + 3]) * inv);
            w.z = pack_bf16x2(__uint_as_float(v[qd * 8 + 4]) * inv, __uint_as_float(v[qd * 8 + 5]) * inv);
            w.w = pack_bf16x2(__uint_as_float(v[qd * 8 + 6]) * inv, __uint_as_float(v[qd * 8 + 7]) * inv);
            *reinterpret_cast<uint4*>(dst + c * 32 + qd * 8) = w;
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace fmha

bool fmha_supported(const AttnArgs& a) {
  static const bool legacy = [] {
    const char* e = std::getenv("B200_ATTN_LEGACY");
    return e != nullptr && e[0] == '1';
  }();
  const int G = a.Hq / a.Hkv;
  // logit softcapping runs on the mma.sync kernel
  return !legacy && a.D == 128 && a.softcap <= 0.f && a.Hq % a.Hkv == 0 && G >= 1 && G <= 8 &&
         (G & (G - 1)) == 0 && a.q_rows > 0;
}

void fmha_launch(const AttnArgs& a, cudaStream_t st) {
  using namespace fmha;
  const int G = a.Hq / a.Hkv;
  const int rows_tok = 128 / G;
  CUtensorMap tq = make_tmap_3d(a.q, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, kD, a.Hq, a.q_rows, kD,
                                (uint64_t)a.Hq * kD, 64, G, 16);
  CUtensorMap tk, tv;
  if (a.kv_dense) {  // [rows, Hkv, D]: one 16-row page of one head = box [16][1][64]
    tk = make_tmap_3d(a.k_cache, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, kD, a.Hkv, a.kv_rows, kD,
                      (uint64_t)a.Hkv * kD, 64, 1, 16);
    tv = make_tmap_3d(a.v_cache, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, kD, a.Hkv, a.kv_rows, kD,
                      (uint64_t)a.Hkv * kD, 64, 1, 16);
  } else {
    const int64_t kv_rows = a.num_blocks * a.Hkv * 16;
    tk = make_tmap_2d(a.k_cache, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, kv_rows, kD, kD, 16, 64);
    tv = make_tmap_2d(a.v_cache, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, kv_rows, kD, kD, 16, 64);
  }
  const int q_tiles = (a.max_q_len + rows_tok - 1) / rows_tok;
  ensure_smem(fmha_fwd_kernel, kSmem);
  launch_pdl(fmha_fwd_kernel, dim3(a.B * q_tiles, a.Hkv), dim3(kThreads), kSmem, st, tq, tk, tv, a, q_tiles,
             rows_tok);
}

}  // namespace b200
