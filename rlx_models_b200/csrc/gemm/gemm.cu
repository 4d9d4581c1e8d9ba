// Host launcher for the tcgen05 BF16 GEMM (see gemm_sm100.cuh).
//
// linear(x[M,K], w[N,K]) -> out: picks the orientation, tile width and split-K
// factor for the shape, builds the two TMA maps and launches the persistent
// kernel on the current stream.
//   * prefill / training shapes (M > 128): A = x, B = w, BN = 256.
//   * decode shapes (M <= 128): "swap-AB" - A = w (weights fill the 128-row MMA
//     M dimension), B = x (the few tokens are the MMA N dimension), and split-K
//     so that every SM streams a slice of the weights.
#include <algorithm>
#include <stdexcept>
#include <string>

#include "../common/pdl_launch.h"
#include "../common/tma_host.h"
#include "gemm_sm100.cuh"

namespace b200 {
namespace gemm {

template <int BN, int EPI, bool A_MN = false, bool B_MN = false>
static void launch_t(const CUtensorMap& ta, const CUtensorMap& tb, const Params& p, int grid, cudaStream_t st,
                     int device) {
  auto kern = gemm_bf16_kernel<BN, EPI, A_MN, B_MN>;
  (void)device;
  ensure_smem(kern, Cfg<BN>::SMEM_BYTES);
  launch_pdl(kern, dim3(grid), dim3(kThreads), Cfg<BN>::SMEM_BYTES, st, ta, tb, p);
}

template <int EPI>
static void launch_bn(int BN, const CUtensorMap& ta, const CUtensorMap& tb, const Params& p, int grid,
                      cudaStream_t st, int device) {
  switch (BN) {
    case 32: launch_t<32, EPI>(ta, tb, p, grid, st, device); break;
    case 64: launch_t<64, EPI>(ta, tb, p, grid, st, device); break;
    case 128: launch_t<128, EPI>(ta, tb, p, grid, st, device); break;
    case 256: launch_t<256, EPI>(ta, tb, p, grid, st, device); break;
    default: throw std::runtime_error("b200.linear: unsupported BN " + std::to_string(BN));
  }
}

}  // namespace gemm
}  // namespace b200

#include "../common/launch.h"

namespace b200 {

// Raw-pointer GEMM entry used by the torch bindings and by the fused kernels'
// host code. All tensors are row-major with unit inner stride.
void linear_launch(const LinearArgs& a, cudaStream_t st) {
  const int64_t M = a.M, K = a.K, N = a.N;
  const int epi = a.mode;
  if (M == 0 || N == 0) return;
  const int sms = num_sms(a.device);
  const bool dit_epi = a.act != 0 || a.gate != nullptr;
  const bool sw = a.swap < 0 ? (M <= 128 && N >= 256) : (a.swap == 1);

  gemm::Params p{};
  const void* A = sw ? a.w : a.x;
  const void* B = sw ? a.x : a.w;
  const int64_t lda = sw ? a.ldw : a.ldx;
  const int64_t ldb = sw ? a.ldx : a.ldw;
  p.MA = (int)(sw ? N : M);
  p.NB = (int)(sw ? M : N);
  p.K = (int)K;
  int BN = a.bn;
  if (BN == 0) {
    if (sw) BN = p.NB <= 32 ? 32 : (p.NB <= 64 ? 64 : 128);
    else BN = p.NB >= 256 ? 256 : (p.NB > 64 ? 128 : (p.NB > 32 ? 64 : 32));
    if (epi == gemm::EPI_SWIGLU && !sw && BN < 128) BN = 128;
  }
  p.k_tiles = (int)((K + gemm::kBK - 1) / gemm::kBK);
  p.num_m = (p.MA + gemm::kBM - 1) / gemm::kBM;
  p.num_n = (p.NB + BN - 1) / BN;
  const int tiles = p.num_m * p.num_n;
  int sp = a.splits;
  if (sp <= 0) {
    // Split-K only to fill the machine: pick the factor minimising
    // waves * k-tiles-per-unit plus a per-split reduction cost (in k-tiles).
    sp = 1;
    double best = 1e30;
    // large tile counts already fill the machine; their partial tiles would
    // also outgrow the accumulator
    // non-accumulating split-K pays a partial-tile round trip through the workspace
    // and a semaphore tail per tile: only worth it when the tiles leave most SMs idle
    const int max_sp = (tiles >= (epi == gemm::EPI_ACC ? 2 * sms : sms)) ? 1
                                                                         : std::max(1, std::min(16, p.k_tiles / 4));
    for (int s = 1; s <= max_sp; ++s) {
      const int kts = (p.k_tiles + s - 1) / s;
      const int waves = (tiles * s + sms - 1) / sms;
      // a handful of output tiles (a router, a small head) would otherwise stream the whole K
      // on a few SMs: there the partial-tile round trip is cheap next to the serial k loop
      const double per_split = epi == gemm::EPI_ACC ? 0.5 : (tiles <= 8 ? 1.0 : 6.0);
      const double cost = (double)waves * kts + (s > 1 ? per_split * s : 0.0);
      if (cost < best - 1e-9) {
        best = cost;
        sp = s;
      }
    }
  }
  sp = std::max(1, std::min(sp, p.k_tiles));
  if (sp > 1 && epi != gemm::EPI_ACC)  // one fp32 partial slice per split must fit the workspace
    sp = (int)std::max<int64_t>(1, std::min<int64_t>(sp, a.ws_elems / ((int64_t)tiles * gemm::kBM * BN)));
  if (dit_epi) sp = 1;  // the activation / gate must see the full sum
  p.kt_per_split = (p.k_tiles + sp - 1) / sp;
  p.splits = (p.k_tiles + p.kt_per_split - 1) / p.kt_per_split;
  p.num_units = tiles * p.splits;
  if (epi == gemm::EPI_ACC && !sw) throw std::runtime_error("b200.linear: accumulate mode needs swap-AB (M <= 128)");
  if (p.splits > 1 && epi != gemm::EPI_ACC) {
    if (a.ws_elems < (int64_t)p.splits * tiles * gemm::kBM * BN || a.ws == nullptr)
      throw std::runtime_error("b200.linear: split-K accumulator too small");
    if (a.sem_elems < tiles || a.sem == nullptr) throw std::runtime_error("b200.linear: semaphore buffer too small");
  }
  p.C = a.out;
  p.ldc_i = sw ? 1 : a.ldo;
  p.ldc_j = sw ? a.ldo : 1;
  p.R = reinterpret_cast<const __nv_bfloat16*>(a.residual);
  p.ldr_i = sw ? 1 : a.ldr;
  p.ldr_j = sw ? a.ldr : 1;
  p.bias = reinterpret_cast<const __nv_bfloat16*>(a.bias);
  p.bias_on_i = sw ? 1 : 0;
  p.alpha = a.alpha;
  p.swiglu_on_i = sw ? 1 : 0;
  p.w_is_a = sw ? 1 : 0;
  p.prefetch_w = 1;
  p.ws = a.ws;
  p.sem = a.sem;
  p.status = a.status;
  p.peer_out = a.peer_out;
  p.rpr = a.rpr;
  p.slot_elems = a.slot_elems;
  p.my_rank = a.my_rank;
  p.world = a.world;
  p.epoch = a.epoch;
  p.done_ctr = a.done_ctr;
  p.peer_flags = a.peer_flags;
  p.bcast = a.bcast;
  if (p.bcast && !sw) throw std::runtime_error("b200.linear: broadcast push needs the swap-AB (decode) path");
  p.trace = a.trace;
  p.act = a.act;
  p.glu_act = a.glu_act;
  p.act_from = a.act_from;
  p.gate = reinterpret_cast<const __nv_bfloat16*>(a.gate);
  p.gate_ld = a.gate_ld;
  p.gate_split = a.gate_split;
  p.gate_r1 = std::max(1, a.gate_r1);
  p.gate_r2 = std::max(1, a.gate_r2);
  p.gate_off = a.gate_off;
  if (dit_epi && (epi != gemm::EPI_BF16 || p.splits > 1))
    throw std::runtime_error("b200.linear: GELU / gate epilogues need bf16 output without split-K");
  if (p.peer_out != nullptr && (p.rpr <= 0 || p.done_ctr == nullptr || p.peer_flags == nullptr || p.epoch == nullptr))
    throw std::runtime_error("b200.linear: incomplete push-mode arguments");

  CUtensorMap ta = make_tmap_2d(A, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, p.MA, K, lda, gemm::kBM, gemm::kBK);
  CUtensorMap tb = make_tmap_2d(B, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, p.NB, K, ldb, BN, gemm::kBK);
  const int grid = std::min(p.num_units, sms);
  switch (epi) {
    case gemm::EPI_BF16: gemm::launch_bn<gemm::EPI_BF16>(BN, ta, tb, p, grid, st, a.device); break;
    case gemm::EPI_F32: gemm::launch_bn<gemm::EPI_F32>(BN, ta, tb, p, grid, st, a.device); break;
    case gemm::EPI_SWIGLU: gemm::launch_bn<gemm::EPI_SWIGLU>(BN, ta, tb, p, grid, st, a.device); break;
    case gemm::EPI_ACC: gemm::launch_bn<gemm::EPI_ACC>(BN, ta, tb, p, grid, st, a.device); break;
    default: throw std::runtime_error("b200.linear: bad mode");
  }
}

}  // namespace b200

namespace b200 {

// General GEMM for training: D[i, j] = alpha * sum_k A[i, k] * B[j, k] with
// either operand K-major or MN-major; bf16 or f32 (optionally accumulated)
// output, optional residual / bias. No orientation swap, no TP push.
void gemm_launch(const GemmArgs& a, cudaStream_t st) {
  if (a.MA == 0 || a.NB == 0) return;
  const int sms = num_sms(a.device);
  const int epi = a.out_f32 ? gemm::EPI_F32 : gemm::EPI_BF16;
  gemm::Params p{};
  p.MA = (int)a.MA;
  p.NB = (int)a.NB;
  p.K = (int)a.K;
  int BN = a.bn ? a.bn : (a.NB > 128 ? 256 : 128);
  if (BN != 128 && BN != 256) throw std::runtime_error("b200.gemm: BN must be 128 or 256");
  p.k_tiles = (int)((a.K + gemm::kBK - 1) / gemm::kBK);
  p.num_m = (p.MA + gemm::kBM - 1) / gemm::kBM;
  p.num_n = (p.NB + BN - 1) / BN;
  const int tiles = p.num_m * p.num_n;
  int sp = a.splits;
  if (sp <= 0) {
    sp = 1;
    double best = 1e30;
    // non-accumulating split-K pays a partial-tile round trip through the workspace
    // and a semaphore tail per tile: only worth it when the tiles leave most SMs idle
    const int max_sp = (tiles >= (epi == gemm::EPI_ACC ? 2 * sms : sms)) ? 1
                                                                         : std::max(1, std::min(16, p.k_tiles / 4));
    for (int s = 1; s <= max_sp; ++s) {
      const int kts = (p.k_tiles + s - 1) / s;
      const int waves = (tiles * s + sms - 1) / sms;
      const double cost = (double)waves * kts + (s > 1 ? 2.0 * s : 0.0);
      if (cost < best - 1e-9) {
        best = cost;
        sp = s;
      }
    }
  }
  sp = std::max(1, std::min(sp, p.k_tiles));
  if (sp > 1) sp = (int)std::max<int64_t>(1, std::min<int64_t>(sp, a.ws_elems / ((int64_t)tiles * gemm::kBM * BN)));
  p.kt_per_split = (p.k_tiles + sp - 1) / sp;
  p.splits = (p.k_tiles + p.kt_per_split - 1) / p.kt_per_split;
  p.num_units = tiles * p.splits;
  if (p.splits > 1 && (a.ws == nullptr || a.sem == nullptr || a.sem_elems < tiles ||
                       a.ws_elems < (int64_t)p.splits * tiles * gemm::kBM * BN))
    throw std::runtime_error("b200.gemm: split-K buffers too small");
  p.C = a.c;
  p.ldc_i = a.ldc;
  p.ldc_j = 1;
  p.R = reinterpret_cast<const __nv_bfloat16*>(a.residual);
  p.ldr_i = a.ldr;
  p.ldr_j = 1;
  p.bias = reinterpret_cast<const __nv_bfloat16*>(a.bias);
  p.bias_on_i = 0;
  p.alpha = a.alpha;
  p.swiglu_on_i = 0;
  p.w_is_a = 0;
  p.accumulate = a.accumulate;
  p.prefetch_w = a.prefetch_b;
  p.shard_peer = a.shard_peer;
  p.shard_base = a.shard_base;
  p.shard_n = a.shard_n;
  if (a.shard_peer != nullptr && (!a.out_f32 || a.accumulate || a.residual != nullptr || a.bias != nullptr ||
                                  a.shard_n <= 0))
    throw std::runtime_error("b200.gemm: shard push needs f32 output, no accumulate / residual / bias");
  p.ws = a.ws;
  p.sem = a.sem;
  p.status = a.status;
  // K-major operand: [rows, K] (ld = row stride); MN-major: stored [K, rows] (ld = stride of k)
  CUtensorMap ta = a.a_mn ? make_tmap_2d(a.a, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.K, a.MA, a.lda, 64, 64)
                          : make_tmap_2d(a.a, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.MA, a.K, a.lda, gemm::kBM, 64);
  CUtensorMap tb = a.b_mn ? make_tmap_2d(a.b, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.K, a.NB, a.ldb, 64, 64)
                          : make_tmap_2d(a.b, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.NB, a.K, a.ldb, BN, 64);
  const int grid = std::min(p.num_units, sms);
  const int code = (a.a_mn ? 2 : 0) + (a.b_mn ? 1 : 0);
#define B200_GEMM_CASE(BNV, EPIV)                                                                      \
  switch (code) {                                                                                      \
    case 0: gemm::launch_t<BNV, EPIV, false, false>(ta, tb, p, grid, st, a.device); break;             \
    case 1: gemm::launch_t<BNV, EPIV, false, true>(ta, tb, p, grid, st, a.device); break;              \
    case 3: gemm::launch_t<BNV, EPIV, true, true>(ta, tb, p, grid, st, a.device); break;               \
    default: throw std::runtime_error("b200.gemm: A MN-major with B K-major is not instantiated");     \
  }
  if (BN == 256) {
    if (epi == gemm::EPI_F32) { B200_GEMM_CASE(256, gemm::EPI_F32) } else { B200_GEMM_CASE(256, gemm::EPI_BF16) }
  } else {
    if (epi == gemm::EPI_F32) { B200_GEMM_CASE(128, gemm::EPI_F32) } else { B200_GEMM_CASE(128, gemm::EPI_BF16) }
  }
#undef B200_GEMM_CASE
}

}  // namespace b200
