// Plain-C++ launch interfaces of the CUDA kernels. The .cu files implement
// them without any torch headers (so they compile quickly with nvcc); the
// torch bindings in bindings.cpp validate tensors and fill these structs.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace b200 {

// ---------------- GEMM ----------------
struct LinearArgs {
  const void* x;
  int64_t ldx;  // [M, K]
  const void* w;
  int64_t ldw;  // [N, K]
  void* out;
  int64_t ldo;  // [M, N] or [M, N/2] for SwiGLU
  const void* residual;
  int64_t ldr;  // optional [M, N] bf16 added in the epilogue
  const void* bias;  // optional [N] bf16
  int64_t M, N, K;
  int mode;  // 0 bf16, 1 f32, 2 SwiGLU (interleaved gate/up groups of 64)
  float alpha;
  int swap, bn, splits;  // -1/0 = auto
  float* ws;
  int64_t ws_elems;
  int* sem;
  int64_t sem_elems;
  int* status;
  int device;
  // tensor-parallel reduce-scatter push mode (see gemm_sm100.cuh); null = off
  void* const* peer_out = nullptr;
  int rpr = 0;
  int64_t slot_elems = 0;
  int my_rank = 0, world = 1;
  const unsigned* epoch = nullptr;
  unsigned* done_ctr = nullptr;
  unsigned* const* peer_flags = nullptr;
  int bcast = 0;  // one-shot: push rows to every rank's slot `my_rank`
  unsigned long long* trace = nullptr;  // debug timeline
  // adaLN DiT epilogues (normal orientation): GELU-tanh on columns >= act_from;
  // y *= gate[batch(row)][col] before the residual (batch(row) as in gemm::Params)
  int act = 0, act_from = 0;
  int glu_act = 0;  // mode 2: 0 SwiGLU, 1 GeGLU (GELU tanh form)
  const void* gate = nullptr;
  int64_t gate_ld = 0;
  int gate_split = 0, gate_r1 = 1, gate_r2 = 1, gate_off = 0;
};
void linear_launch(const LinearArgs& a, cudaStream_t st);

// General (training) GEMM: D[MA, NB] = alpha * A[MA, K] . B[NB, K]^T with
// per-operand major (K-major rows, or MN-major = stored [K, rows]).
struct GemmArgs {
  const void* a;
  int64_t lda;
  int a_mn;
  const void* b;
  int64_t ldb;
  int b_mn;
  void* c;
  int64_t ldc;
  int64_t MA, NB, K;
  int out_f32, accumulate;
  float alpha;
  const void* residual;
  int64_t ldr;
  const void* bias;
  int prefetch_b;  // B may be read before the previous kernel finishes (static weights)
  int bn, splits;
  float* ws;
  int64_t ws_elems;
  int* sem;
  int64_t sem_elems;
  int* status;
  int device;
  float* const* shard_peer = nullptr;  // FSDP gradient push (see gemm::Params::shard_peer)
  int64_t shard_base = 0, shard_n = 0;
};
void gemm_launch(const GemmArgs& a, cudaStream_t st);

// ---------------- tensor-parallel fused collective ----------------
struct RsNormAgArgs {
  const void* recv;           // local [world][rpr][H] (reduce inputs), unused if !do_reduce
  void* h;                    // local residual shard [rpr][H]
  const void* norm_w;         // [H]
  void* const* peer_gath;     // [world] gather buffers [M][H]
  const unsigned* rs_flags;            // local [world]
  const unsigned* ag_flags;            // local [world]
  unsigned* const* peer_ag_flags;      // [world] -> each rank's ag_flags
  unsigned* epoch;                     // local op counter
  unsigned* cta_ctr;                   // local arrival counter (self-resetting)
  float* racc;                         // local fp32 [rpr][H] accumulator (do_reduce == 2)
  int M, H, rpr, world, rank, do_reduce;  // do_reduce: 0 none, 1 bf16 slots, 2 fp32 accumulator
  int64_t slot_elems;                  // rpr_max * H
  float eps;
  int* status;
};
void rs_norm_ag_launch(const RsNormAgArgs& a, cudaStream_t st);

// One-shot all-reduce consumer: wait for every rank's epoch flag, then per row
// h = bf16(h + bf16(sum_q slots[q][row])) (fixed rank order: identical on all
// ranks), out = rmsnorm(h) * w; the last CTA advances the local epoch.
struct OsReduceArgs {
  const void* slots;        // local [world][M][H] bf16 (this op's parity buffer)
  int64_t slot_elems;       // elements per slot
  void* h;                  // [M][H] bf16 replicated residual stream (in/out)
  const void* norm_w;
  void* out;                // [M][H] bf16
  const unsigned* flags;    // local [world]
  unsigned* epoch;
  unsigned* cta_ctr;
  int M, H, world;
  float eps;
  int* status;
};
void os_reduce_norm_launch(const OsReduceArgs& a, cudaStream_t st);

// pull all-reduce + residual add + RMSNorm (decode steps): see tp_fused.cu
struct PullNormArgs {
  const float* const* peer_acc;  // [world] each rank's fp32 [rows][H] partial (this op's parity)
  unsigned* const* peer_flags;   // [world] each rank's flag array [world]
  const unsigned* flags;         // local flags [world]
  float* zero_buf;               // own previous-parity accumulator
  int zero_rows;
  void* h;                       // [M][H] bf16 replicated residual (in/out)
  const void* norm_w;
  void* out;                     // [M][H] bf16
  unsigned* epoch;
  unsigned* cta_ctr;
  int M, H, world, rank;
  float eps;
  int* status;
};
void ar_pull_norm_launch(const PullNormArgs& a, cudaStream_t st);

// Two-shot variant (each rank reduces the rows it owns, the others fetch them):
// see comm/tp_fused.cu ar2_norm_kernel.
struct TwoShotNormArgs {
  const float* const* peer_acc;  // [world] each rank's fp32 [rows][H] partial (this op's parity)
  const void* const* peer_res;   // [world] each rank's result slot: bf16 [rpr_max][H] new residual rows,
                                 // then fp32 [rpr_max][H / 512] slice sums of squares (within 2*rpr_max*H bf16)
  void* own_res;                 // this rank's result slot
  unsigned* const* peer_flags;   // [world] each rank's flag array [2][world]
  const unsigned* flags;         // local flags [2][world]
  float* zero_buf;               // own previous-parity accumulator
  int zero_rows;
  void* h;                       // [M][H] bf16 replicated residual (in/out)
  const void* norm_w;
  void* out;                     // [M][H] bf16
  unsigned* epoch;
  unsigned* cta_ctr;             // [2]
  int M, H, world, rank, rpr, rpr_max;
  float eps;
  int* status;
};
void ar2_norm_launch(const TwoShotNormArgs& a, cudaStream_t st);

// Training-path elementwise kernels (forward + backward): see train/train_fused.cu.
struct QKNormRopeArgs {
  const void* qkv;           // [T][(Hq + 2 Hkv) * D] bf16 GEMM output
  const void* q_norm;        // [D] bf16 or null (no QK-norm)
  const void* k_norm;
  const void* cos;           // [S][D] bf16 rotary tables (halves duplicated)
  const void* sin;
  const int32_t* positions;  // [T] or null: position = t % S
  void* q;                   // [T][Hq][D]  forward outputs
  void* k;                   // [T][Hkv][D]
  void* v;                   // [T][Hkv][D]
  float* rstd_q;             // [T][Hq] saved for backward
  float* rstd_k;             // [T][Hkv]
  const void* dq;            // backward inputs [T][H][D]
  const void* dk;
  const void* dv;
  void* dqkv;                // backward output, layout of qkv
  float* dw_q;               // [D] fp32 weight-gradient accumulators (or null)
  float* dw_k;
  int T, S, Hq, Hkv, D;
  float eps;
};
void rmsnorm_train_fwd_launch(const void* x, const void* w, void* y, float* rstd, int rows, int H, float eps,
                              int device, cudaStream_t st);
void rmsnorm_train_bwd_launch(const void* dy, const void* x, const void* w, const float* rstd, void* dx, float* dw,
                              int rows, int H, int device, cudaStream_t st);
void qk_norm_rope_fwd_launch(const QKNormRopeArgs& a, int device, cudaStream_t st);
void qk_norm_rope_bwd_launch(const QKNormRopeArgs& a, int device, cudaStream_t st);
void swiglu_train_fwd_launch(const void* gu, void* h, int64_t T, int I, int device, cudaStream_t st);
void swiglu_train_bwd_launch(const void* dh, const void* gu, void* dgu, int64_t T, int I, int device,
                             cudaStream_t st);
void scale_by_launch(void* t, bool is_f32, int64_t n, const float* g, int device, cudaStream_t st);

// Instance norm over time with an active prefix (Kitten TTS): see audio/instance_norm.cu.
void instance_norm_launch(const void* x, const float* gamma, const float* beta, void* y, int64_t N, int C,
                          int64_t T, int64_t active, float eps, bool bf16, cudaStream_t st);

// Channels-last convolutions of the audio codecs (activation-fused im2col, transposed-conv overlap-add) and the
// LSTM cell: see audio/codec_conv.cu. act: 0 none, 1 snake (alpha [C]), 2 ELU, 3 GELU (erf).
void act_im2col_launch(const void* x, const float* alpha, void* cols, int B, int T, int T_out, int C, int Kp, int k,
                       int stride, int pad_l, int dil, int act, bool reflect, cudaStream_t st);
void convt_fold_launch(const float* Y, const float* bias, void* y, int B, int T_in, int T_out, int C_out, int stride,
                       int m, int pad_l, cudaStream_t st);
void lstm_cell_launch(const float* G, float* c, void* h, void* y, int B, int H, cudaStream_t st);

// Vocab-parallel greedy argmax over NVLink peer memory: see comm/tp_sample.cu.
struct TpArgmaxArgs {
  const float* logits;                    // [R][ld] fp32, this rank's vocab shard
  int64_t ld;
  int V_local, v_offset;                  // shard width, first global id of the shard
  unsigned long long* own_pairs;          // this rank's [2][max_rows][world] tagged keys
  unsigned long long* const* peer_pairs;  // [world] every rank's key buffer
  unsigned* epoch;
  unsigned* cta_ctr;                      // [1] departure counter
  int32_t* out;                           // [R] global token ids
  int R, max_rows, world, rank;
  int* status;
};
void tp_argmax_launch(const TpArgmaxArgs& a, cudaStream_t st);

// Expert-parallel combine over NVLink + residual add + RMSNorm: see
// comm/ep_combine.cu. Every rank routed the same tokens; token t's slot s went
// to expert experts[t, s], held by rank experts[t, s] / e_local, whose down
// GEMM wrote the router-weighted row at position inv_q[t * k + s] of its rows.
struct EpCombineArgs {
  const void* const* peer_rows;     // [world] each rank's bf16 [rows][H] expert outputs (this op's slot)
  const int32_t* const* peer_inv;   // [world] each rank's inverse permutation [T * k] (-1: not its expert)
  unsigned* const* peer_flags;      // [world] each rank's flag array [world]
  const unsigned* flags;            // local flags [world]
  const int32_t* experts;           // [T][k] global expert ids (identical on every rank)
  void* h;                          // [T][H] bf16 replicated residual stream (in/out)
  const void* norm_w;               // [H] bf16
  void* out;                        // [T][H] bf16 = rmsnorm(h + moe) * w
  unsigned* epoch;
  unsigned* cta_ctr;
  int T, k, H, e_local, world, rank;
  float eps;
  int* status;
};
void ep_combine_norm_launch(const EpCombineArgs& a, cudaStream_t st);

// FSDP gradient push into the owners' fp32 shards + cross-rank barrier: see
// comm/fsdp_comm.cu.
void shard_push_add_launch(const void* src, bool f32, int64_t n, int64_t base, float* const* peers, int64_t shard_n,
                           float scale, cudaStream_t st);
// GGUF block dequantisation (quant/gguf_dequant.cu): n output elements of
// ggml type `ggml_type` from its raw blocks into bf16 (or fp32).
void gguf_dequant_launch(const void* raw, int ggml_type, int64_t n, void* out, bool out_f32, cudaStream_t st);
void peer_barrier_launch(unsigned* const* peer_flags, const unsigned* flags, unsigned* epoch, int rank, int world,
                         int* status, cudaStream_t st);

// ---------------- norms / rope / embedding ----------------
void embedding_launch(const int32_t* ids, const void* table, void* out, int64_t T, int64_t H, int64_t V,
                      cudaStream_t st);
// out = rmsnorm(x (+ residual_in)) * w ; if residual_out: residual_out = x (+ residual_in)
void rmsnorm_launch(const void* x, int64_t ldx, const void* residual_in, void* residual_out, const void* w,
                    void* out, int64_t ldo, int64_t T, int64_t H, float eps, cudaStream_t st);

struct QkvRopeArgs {
  const void* qkv;  // [T, (Hq + 2 Hkv) * D] bf16
  float* qkv_f32 = nullptr;  // or: fp32 sums from the accumulate-only GEMM (zeroed after use)
  int64_t ld_qkv;
  const void* q_norm;  // [D] or null
  const void* k_norm;  // [D] or null
  const int32_t* positions;  // [T]
  const int64_t* slots;      // [T] cache slot (block * 16 + offset), -1 = skip
  const float* inv_freq;     // [rot_dim / 2]
  float rope_scale;          // multiplier on cos/sin (YaRN mscale), 1 otherwise
  int rot_dim;               // rotary dims (<= D), half-split (NeoX) layout
  void* q_out;               // [T, Hq, D]
  void* k_cache;             // [NB, Hkv, 16, D]
  void* v_cache;
  void* k_out;               // optional [T, Hkv, D] (training / no cache)
  void* v_out;
  int64_t T;
  int Hq, Hkv, D;
  float eps;
  const void* bias = nullptr;  // [(Hq + 2 Hkv) * D] bf16 added to the fp32 sums (accumulate-mode input only)
  int kv_fp8 = 0;              // caches hold float8 e4m3: stored value = saturate(x / scale)
  float k_inv_scale = 1.f, v_inv_scale = 1.f;
};
void qkv_rope_launch(const QkvRopeArgs& a, cudaStream_t st);
// bias ([H] bf16, may be null) is added to the fp32 sums before the residual add
void add_rmsnorm_acc_launch(float* acc, void* h, const void* w, void* out, int64_t ldo, int64_t T, int64_t H,
                            float eps, cudaStream_t st, const void* bias = nullptr);
void swiglu_acc_launch(float* acc, void* out, int64_t T, int64_t I, int act, cudaStream_t st);

// ---------------- attention ----------------
struct AttnArgs {
  const void* q;  // [Tq, Hq, D] bf16
  const void* k_cache;
  const void* v_cache;  // [NB, Hkv, 16, D]
  int64_t num_blocks;
  const int32_t* block_tables;  // [B, max_blocks]
  int max_blocks;
  const int32_t* ctx_lens;   // [B] kv length incl. the new tokens
  const int32_t* cu_q;       // [B+1] query offsets (prefill); null for decode (1 query / seq)
  void* out;                 // [Tq, Hq, D] bf16
  const float* sinks;        // [Hq] or null (learned sink logits)
  int window;                // sliding window (0 = full)
  int B, Hq, Hkv, D;
  float scale;
  float softcap = 0.f;       // > 0: scores = softcap * tanh(scale * q.k / softcap) (Gemma-2)
  int max_q_len;             // prefill: max query length per sequence
  int splits;                // decode: KV splits (0 = auto)
  int chunk_pages = 0;       // decode: > 0 cuts every sequence's pages into chunks of this many pages
                             // (split s takes chunk s; empty chunks write an empty partial), 0 = splits
                             // equal parts of each sequence
  int causal = 1;            // prefill: 0 = every query sees the whole context (DiT joint attention)
  int q_paged = 0;           // prefill: query / output row of token t = block_tables[b][t / 16] * 16 + t % 16
  int64_t out_ld = 0;        // prefill: output row stride in elements (0 = Hq * D)
  int64_t q_rows = 0;        // prefill: rows of q (bounds of its TMA map)
  int kv_dense = 0;          // prefill: k/v row-major [kv_rows, Hkv, D] (pages = 16 consecutive rows)
  int64_t kv_rows = 0;
  float* lse = nullptr;      // prefill (tcgen05 kernel, no sinks): per (row, head) log2-sum-exp2 of the
                             // scaled scores, [q_rows][Hq], for the attention backward
  float* ws;                 // decode split workspace
  int64_t ws_elems;
  int* status;
  int device;
  int kv_fp8 = 0;            // decode: pages hold float8 e4m3 (K = k_scale * stored, V = v_scale * stored)
  float k_scale = 1.f, v_scale = 1.f;
};
int decode_attention_launch(const AttnArgs& a, cudaStream_t st);  // returns #launches
// float8 e4m3 pages of the sequences in a prefill batch -> bf16 pages at block b * max_blocks + p
// (pages at or past ceil(ctx_lens[b] / 16) are skipped): see attention/attention.cu.
void kv_dequant_pages_launch(const void* k8, const void* v8, const int32_t* block_tables, const int32_t* ctx_lens,
                             int B, int max_blocks, int Hkv, int D, float k_scale, float v_scale, void* k_out,
                             void* v_out, cudaStream_t st);
void prefill_attention_launch(const AttnArgs& a, cudaStream_t st);
// tcgen05 flash attention (head_dim 128, G <= 8 query heads per kv head); used by
// prefill_attention_launch when supported (B200_ATTN_LEGACY=1 forces the mma.sync kernel)
bool fmha_supported(const AttnArgs& a);
void fmha_launch(const AttnArgs& a, cudaStream_t st);

// Attention backward for training (causal, dense [T, H, D] rows, head_dim 128):
// see train/attn_bwd.cu.
struct AttnBwdArgs {
  const void* q;      // [T][Hq][D] bf16
  const void* k;      // [T][Hkv][D]
  const void* v;
  const void* o;      // forward output [T][Hq][D]
  const void* dout;   // [T][Hq][D]
  const float* lse;   // [T][Hq] log2 units (forward)
  float* delta;       // [T][Hq] scratch: rowsum(dO * O)
  float* dq_acc;      // [T][Hq][D] fp32 scratch (zeroed by the prep kernel)
  void* dq;           // [T][Hq][D] bf16
  void* dk;           // [T][Hkv][D]
  void* dv;
  int B, S, Hq, Hkv;
  float scale;
};
void attn_bwd_launch(const AttnBwdArgs& a, int device, cudaStream_t st);

// ---------------- linear attention (Gated DeltaNet) ----------------
struct GdnDecodeArgs {
  const __nv_bfloat16* proj;  // [B, ld]: [q k v conv inputs (conv_dim) | z (Hv*D) | b (Hv) | a (Hv)]
  int64_t ld;
  const float* conv_w;        // [conv_dim, K]
  const float* A_log;         // [Hv]
  const float* dt_bias;       // [Hv]
  const float* norm_w;        // [D]
  __nv_bfloat16* conv_state;  // [num_slots, 2, conv_dim, K-1] (window before the token, by position parity)
  float* rec_state;           // [num_slots, Hv, D, D]
  const int32_t* seq_slots;   // [B] state slot per row (out of range: padding row)
  const int32_t* positions;   // [B]
  __nv_bfloat16* out;         // [B, Hv*D]
  int B, Hk, Hv, D, K;
  int conv_dim, key_dim, value_dim;
  int64_t num_slots;
  float eps;
  int kda;  // 1: per-channel decay (a: Hv*D logits, dt_bias [Hv*D]) and a sigmoid output gate
};
void gdn_decode_launch(const GdnDecodeArgs& a, cudaStream_t st);

// LFM2 short convolution, decode step (see gdn.cu)
struct ShortConvArgs {
  const __nv_bfloat16* proj;  // [B, ld]: [B gate (H) | C gate (H) | x (H)]
  int64_t ld;
  const float* w;             // [H, K]
  const float* bias;          // [H] or null
  __nv_bfloat16* conv_state;  // [num_slots, 2, H, K-1] (window of B*x before the token, by position parity)
  const int32_t* seq_slots;   // [B]
  const int32_t* positions;   // [B]
  __nv_bfloat16* out;         // [B, H]
  int B, H, K;
  int64_t num_slots;
};
void shortconv_decode_launch(const ShortConvArgs& a, cudaStream_t st);

// Mamba-2 SSD decode step (see gdn.cu)
struct SsdDecodeArgs {
  const __nv_bfloat16* proj;  // [B, ld]: x/B/C conv inputs at xbc_off (conv_dim), dt at dt_off (H)
  int64_t ld;
  int xbc_off, dt_off;
  const float* conv_w;        // [conv_dim, K]
  const float* conv_b;        // [conv_dim] or null
  const float* A_log;         // [H]
  const float* dt_bias;       // [H]
  const float* D;             // [H]
  float dt_min, dt_max;
  __nv_bfloat16* conv_state;  // [num_slots, 2, conv_dim, K-1]
  float* ssm_state;           // [num_slots, H, N, P]
  const int32_t* seq_slots;   // [B]
  const int32_t* positions;   // [B]
  __nv_bfloat16* out;         // [B, H*P]: y + D x (before the gated norm)
  int B, H, G, N, P, K, conv_dim;
  int64_t num_slots;
};
void ssd_decode_launch(const SsdDecodeArgs& a, cudaStream_t st);

// Mamba-1 selective scan (see linear_attn/gdn.cu): conv kernel then scan kernel
struct MambaScanArgs {
  const int32_t* cu;          // [nseq + 1] token offsets of each sequence of the step
  const int64_t* slots;       // [nseq] state slot (out of range: no state kept)
  const int32_t* positions;   // [T]: a sequence starting at position 0 starts from zero state
  const __nv_bfloat16* x_raw; // [T, ld_raw] conv input (channels 0..Di)
  int64_t ld_raw;
  const float* conv_w;        // [Di, K]
  const float* conv_b;        // [Di] or null
  __nv_bfloat16* conv_state;  // [num_slots, Di, K-1]
  __nv_bfloat16* x_out;       // [T, Di] silu(conv)
  const __nv_bfloat16* dt;    // [T, ld_dt] dt_proj output without its bias
  int64_t ld_dt;
  const float* dt_bias;       // [Di]
  const __nv_bfloat16* Bc;    // [T, ld_bc]: B at 0, C at c_off
  int64_t ld_bc;
  int c_off;
  const float* A_log;         // [Di, N]
  const float* D;             // [Di]
  const __nv_bfloat16* z;     // [T, ld_z] gate
  int64_t ld_z;
  float* ssm_state;           // [num_slots, Di, N]
  __nv_bfloat16* y;           // [T, Di]
  int nseq, Di, N, K;
  int64_t num_slots;
};
void mamba_conv_launch(const MambaScanArgs& a, cudaStream_t st);
void mamba_scan_launch(const MambaScanArgs& a, cudaStream_t st);

// KV-block retrieval selection (attention/kv_select.cu)
struct KvSelectArgs {
  const __nv_bfloat16* q;     // [B, Hq, D]
  const __nv_bfloat16* summ;  // [num_blocks, Hkv, D] block key summaries of the layer
  const int32_t* tables;      // [B, W]
  const int32_t* ctx;         // [B]
  float* scores;              // [B, W] workspace
  int32_t* sel;               // [B, budget] selected block ids in block order
  int32_t* sel_ctx;           // [B]
  int B, W, Hq, Hkv, D;
  int topk, window, sink, budget;
};
void kv_select_launch(const KvSelectArgs& a, cudaStream_t st);
void kv_summary_launch(const void* k_cache, const int64_t* slots, int64_t T, void* summ, int Hkv, int D,
                       cudaStream_t st);

// ---------------- training ----------------
void adamw_launch(float* master, const void* grad, bool grad_f32, float* m, float* v, void* param_out, int64_t n,
                  float lr, float b1, float b2, float eps, float wd, int64_t step, const float* scale_ptr,
                  float scale, cudaStream_t st);
void sumsq_launch(const void* g, bool f32, int64_t n, float* out, cudaStream_t st);
void ce_fwd_bwd_launch(const float* logits, int64_t ld, int64_t T, int64_t V, const int64_t* targets, float* loss,
                       void* dlogits, int64_t ldd, float grad_scale, cudaStream_t st);

// ---------------- mixture of experts ----------------
void moe_route_launch(const float* logits, int64_t ld, int T, int E, int k, int softmax_first, int renorm,
                      int32_t* experts, float* weights, cudaStream_t st);
void moe_align_launch(const int32_t* experts, int n_assign, int E, int e_lo, int e_cnt, int bt, int32_t* meta,
                      int32_t* tiles, int max_tiles, int32_t* perm, int32_t* inv, int32_t* cursor, cudaStream_t st);
void moe_gather_launch(const void* x, int64_t H, const int32_t* perm, const int32_t* meta, int E, int k,
                       int max_rows, void* out, int to_f16, cudaStream_t st);
void moe_combine_launch(const void* rows, const int32_t* inv, int T, int k, int64_t H, void* out, int accumulate,
                        cudaStream_t st);
struct MoeGemmArgs {
  const void* x;          // expert-sorted activations [rows, K] f16
  int64_t rows;
  const void* w;          // tiled MXFP4 blocks [E, ceil(N/128), K/64, 4096 codes + 256 scales]
                          // (gate/up rows interleaved in groups of 64); scales as offsets from row_exp
  const void* row_exp;    // [E, ceil(N/128) * 128] uint8 largest E8M0 exponent per weight row
  const void* bias;       // [E, N] bf16 or null
  const float* row_weight;  // router weights per assignment (down) or null
  const int32_t* perm;
  const int32_t* meta;
  const int32_t* tiles;
  void* out;
  int E, N, K;
  int bt;                 // token tile (32, 64, 128, 256)
  int max_tiles;          // capacity of the tile list (grid bound)
  int swiglu;
  float limit, alpha;
  float up_offset;        // (up + up_offset): gpt-oss 1, plain SwiGLU 0
  int* status;
  int device;
};
void moe_gemm_launch(const MoeGemmArgs& a, cudaStream_t st);

// bounded flag wait that reports a timeout in the status word (failure-path tests)
void flag_wait_probe_launch(const unsigned* flag, unsigned target, int* status, int* ok, cudaStream_t st);

// ---------------- DiT (FLUX) ----------------
void ln_modulate_launch(const void* x, int64_t ldx, void* out, int64_t ldo, const void* mod, int64_t ld_mod,
                        int shift_off, int scale_off, int rows, int H, float eps, int split, int r1, int r2,
                        int row_off, cudaStream_t st);
// kv_groups == 0: q row-major [rows, heads, 128], k/v in 16-row pages [rows/16, heads, 16, 128];
// kv_groups  > 0: q, k, v all in head-group-major [groups][rows][heads/groups][128] (all-to-all ready)
void dit_qk_rope_launch(const void* qkv, int64_t ld, int rows, int heads, const void* scales_txt,
                        const void* scales_img, const float* cos_t, const float* sin_t, int split, int Lt, int Li,
                        float eps, void* q_out, void* k_pages, void* v_pages, int row_off, int kv_groups,
                        cudaStream_t st);

// ---------------- sampling ----------------
void argmax_launch(const float* logits, int64_t ld, int64_t B, int64_t V, int32_t* out, cudaStream_t st);
void forward_tokens_launch(int32_t* ids, const int32_t* src, const int32_t* prev, int n, cudaStream_t st);

struct SampleArgs {
  const float* logits;  // [B, V]
  int64_t ld;
  int64_t B, V;
  const float* temperature;  // [B] (<= 0 -> greedy)
  const int32_t* top_k;      // [B] (0 -> disabled)
  const float* top_p;        // [B] (1 -> disabled)
  const float* min_p;        // [B] (0 -> disabled)
  const uint64_t* seeds;     // [B] per-row RNG seed
  const int64_t* offsets;    // [B] per-row RNG counter
  int32_t* out;              // [B]
  float* out_logprob;        // [B] or null
  float* ws;                 // candidate workspace
  int64_t ws_elems;
};
void sample_launch(const SampleArgs& a, cudaStream_t st);
// repetition / frequency / presence penalties + logit bias, in place (CSR per row)
void penalties_launch(float* logits, int64_t ld, int64_t B, int64_t V, const int32_t* off, const int32_t* ids,
                      const int32_t* counts, const float* rep, const float* freq, const float* pres,
                      const int32_t* boff, const int32_t* bias_ids, const float* bias_vals, cudaStream_t st);

}  // namespace b200
