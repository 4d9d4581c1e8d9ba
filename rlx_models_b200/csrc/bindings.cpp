// torch bindings of the sm_100a kernels: tensor validation, then a call into
// the plain-C++ launchers declared in common/launch.h on the current stream.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common/launch.h"

using at::Tensor;
using c10::optional;

namespace {

inline const void* opt_ptr(const optional<Tensor>& t) {
  return (t.has_value() && t->defined()) ? t->data_ptr() : nullptr;
}

inline cudaStream_t cur_stream(const Tensor& t) { return at::cuda::getCurrentCUDAStream(t.get_device()); }

void check_cuda(const Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), "b200: ", name, " must be a CUDA tensor");
}

}  // namespace

void linear(const Tensor& x, const Tensor& w, Tensor& out, int64_t mode, const optional<Tensor>& residual,
            const optional<Tensor>& bias, double alpha, Tensor& ws, Tensor& sem, Tensor& status, int64_t swap,
            int64_t bn, int64_t splits, const optional<Tensor>& trace, int64_t act_from, const optional<Tensor>& gate,
            int64_t gate_split, int64_t gate_r1, int64_t gate_r2, int64_t gate_off, int64_t glu_act) {
  check_cuda(x, "x");
  check_cuda(w, "w");
  check_cuda(out, "out");
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16, "b200.linear: bf16 inputs");
  TORCH_CHECK(x.dim() == 2 && w.dim() == 2 && out.dim() == 2, "b200.linear: 2-D tensors");
  TORCH_CHECK(x.stride(1) == 1 && w.stride(1) == 1 && out.stride(1) == 1, "b200.linear: inner dim contiguous");
  const int64_t M = x.size(0), K = x.size(1), N = w.size(0);
  TORCH_CHECK(w.size(1) == K, "b200.linear: K mismatch ", w.size(1), " vs ", K);
  TORCH_CHECK(K % 8 == 0 && x.stride(0) % 8 == 0 && w.stride(0) % 8 == 0, "b200.linear: K and row strides % 8");
  if (mode == 2) {
    TORCH_CHECK(N % 128 == 0 && out.size(0) == M && out.size(1) == N / 2, "b200.linear(swiglu): shapes");
  } else {
    TORCH_CHECK(out.size(0) == M && out.size(1) == N, "b200.linear: out shape");
  }
  TORCH_CHECK((mode == 1 || mode == 3) == (out.scalar_type() == at::kFloat), "b200.linear: out dtype");
  TORCH_CHECK(mode != 3 || (M <= 128 && out.is_contiguous() && N % 4 == 0), "b200.linear(acc): M <= 128, N % 4");
  c10::cuda::CUDAGuard g(x.device());
  b200::LinearArgs a{};
  a.x = x.data_ptr();
  a.ldx = x.stride(0);
  a.w = w.data_ptr();
  a.ldw = w.stride(0);
  a.out = out.data_ptr();
  a.ldo = out.stride(0);
  a.residual = nullptr;
  if (residual.has_value() && residual->defined()) {
    TORCH_CHECK(residual->scalar_type() == at::kBFloat16 && residual->stride(1) == 1 && residual->size(0) == M &&
                    residual->size(1) == out.size(1),
                "b200.linear: residual");
    a.residual = residual->data_ptr();
    a.ldr = residual->stride(0);
  }
  if (bias.has_value() && bias->defined())
    TORCH_CHECK(bias->scalar_type() == at::kBFloat16 && bias->numel() == N, "b200.linear: bias");
  a.bias = opt_ptr(bias);
  a.M = M;
  a.N = N;
  a.K = K;
  a.mode = (int)mode;
  a.alpha = (float)alpha;
  a.swap = (int)swap;
  a.bn = (int)bn;
  a.splits = (int)splits;
  a.ws = ws.numel() ? ws.data_ptr<float>() : nullptr;
  a.ws_elems = ws.numel();
  a.sem = sem.numel() ? sem.data_ptr<int>() : nullptr;
  a.sem_elems = sem.numel();
  a.status = status.data_ptr<int>();
  a.device = x.get_device();
  if (trace.has_value() && trace->defined())
    a.trace = reinterpret_cast<unsigned long long*>(trace->data_ptr<int64_t>());
  if (act_from >= 0) {  // act_from >= (1 << 30): ReLU from column act_from - (1 << 30)
    a.act = act_from >= (1LL << 30) ? 2 : 1;
    a.act_from = (int)(act_from >= (1LL << 30) ? act_from - (1LL << 30) : act_from);
  }
  if (gate.has_value() && gate->defined()) {
    TORCH_CHECK(gate->scalar_type() == at::kBFloat16 && gate->dim() == 2 && gate->stride(1) == 1 &&
                    gate->size(1) == N,
                "b200.linear: gate [batches, N] bf16 with unit inner stride");
    a.gate = gate->data_ptr();
    a.gate_ld = gate->stride(0);
    a.gate_split = (int)gate_split;
    a.gate_r1 = (int)gate_r1;
    a.gate_r2 = (int)gate_r2;
    a.gate_off = (int)gate_off;
  }
  TORCH_CHECK(glu_act == 0 || mode == 2, "b200.linear: glu_act needs the gated (mode 2) epilogue");
  a.glu_act = (int)glu_act;
  b200::linear_launch(a, cur_stream(x));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

static void gdn_decode_impl(const Tensor& proj, const Tensor& conv_w, const Tensor& A_log, const Tensor& dt_bias,
                            const Tensor& norm_w, Tensor& conv_state, Tensor& rec_state, const Tensor& seq_slots,
                            const Tensor& positions, Tensor& out, int64_t Hk, int64_t Hv, int64_t D, double eps,
                            bool kda) {
  const int64_t n_gate = kda ? Hv * D : Hv;  // decay logits per head (GDN) or per key channel (KDA)
  check_cuda(proj, "proj");
  const int64_t B = proj.size(0);
  TORCH_CHECK(proj.scalar_type() == at::kBFloat16 && proj.dim() == 2 && proj.stride(1) == 1, "b200.gdn_decode: proj");
  TORCH_CHECK(conv_w.scalar_type() == at::kFloat && conv_w.is_contiguous() && conv_w.dim() == 2, "b200.gdn_decode: conv_w");
  const int64_t conv_dim = conv_w.size(0), K = conv_w.size(1);
  const int64_t key_dim = Hk * D, value_dim = Hv * D;
  TORCH_CHECK(conv_dim == 2 * key_dim + value_dim, "b200.gdn_decode: conv_dim != 2 key_dim + value_dim");
  TORCH_CHECK(!kda || Hk == Hv, "b200.kda_decode: key heads == value heads");
  TORCH_CHECK(proj.size(1) >= conv_dim + value_dim + Hv + n_gate, "b200.gdn_decode: proj width");
  TORCH_CHECK(A_log.scalar_type() == at::kFloat && A_log.numel() == Hv && dt_bias.scalar_type() == at::kFloat &&
                  dt_bias.numel() == n_gate && norm_w.scalar_type() == at::kFloat && norm_w.numel() == D,
              "b200.gdn_decode: A_log / dt_bias / norm_w fp32");
  TORCH_CHECK(conv_state.scalar_type() == at::kBFloat16 && conv_state.is_contiguous() && conv_state.dim() == 4 &&
                  conv_state.size(1) == 2 && conv_state.size(2) == conv_dim && conv_state.size(3) == K - 1,
              "b200.gdn_decode: conv_state [slots, 2, conv_dim, K-1] bf16");
  TORCH_CHECK(rec_state.scalar_type() == at::kFloat && rec_state.is_contiguous() && rec_state.dim() == 4 &&
                  rec_state.size(0) == conv_state.size(0) && rec_state.size(1) == Hv && rec_state.size(2) == D &&
                  rec_state.size(3) == D,
              "b200.gdn_decode: rec_state [slots, Hv, D, D] fp32");
  TORCH_CHECK(seq_slots.scalar_type() == at::kInt && seq_slots.numel() == B && positions.scalar_type() == at::kInt &&
                  positions.numel() == B,
              "b200.gdn_decode: seq_slots / positions int32 [B]");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.is_contiguous() && out.numel() == B * value_dim,
              "b200.gdn_decode: out [B, Hv*D] bf16");
  c10::cuda::CUDAGuard g(proj.device());
  b200::GdnDecodeArgs a{};
  a.proj = reinterpret_cast<const __nv_bfloat16*>(proj.data_ptr());
  a.ld = proj.stride(0);
  a.conv_w = conv_w.data_ptr<float>();
  a.A_log = A_log.data_ptr<float>();
  a.dt_bias = dt_bias.data_ptr<float>();
  a.norm_w = norm_w.data_ptr<float>();
  a.conv_state = reinterpret_cast<__nv_bfloat16*>(conv_state.data_ptr());
  a.rec_state = rec_state.data_ptr<float>();
  a.seq_slots = seq_slots.data_ptr<int32_t>();
  a.positions = positions.data_ptr<int32_t>();
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.B = (int)B;
  a.Hk = (int)Hk;
  a.Hv = (int)Hv;
  a.D = (int)D;
  a.K = (int)K;
  a.conv_dim = (int)conv_dim;
  a.key_dim = (int)key_dim;
  a.value_dim = (int)value_dim;
  a.num_slots = conv_state.size(0);
  a.eps = (float)eps;
  a.kda = kda ? 1 : 0;
  b200::gdn_decode_launch(a, cur_stream(proj));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void gdn_decode(const Tensor& proj, const Tensor& conv_w, const Tensor& A_log, const Tensor& dt_bias,
                const Tensor& norm_w, Tensor& conv_state, Tensor& rec_state, const Tensor& seq_slots,
                const Tensor& positions, Tensor& out, int64_t Hk, int64_t Hv, int64_t D, double eps) {
  gdn_decode_impl(proj, conv_w, A_log, dt_bias, norm_w, conv_state, rec_state, seq_slots, positions, out, Hk, Hv, D,
                  eps, false);
}

// Kimi Delta Attention decode step: proj rows [q k v (3 Hv D) | z (Hv D) | b (Hv) | a (Hv D)], dt_bias [Hv D].
void kda_decode(const Tensor& proj, const Tensor& conv_w, const Tensor& A_log, const Tensor& dt_bias,
                const Tensor& norm_w, Tensor& conv_state, Tensor& rec_state, const Tensor& seq_slots,
                const Tensor& positions, Tensor& out, int64_t H, int64_t D, double eps) {
  gdn_decode_impl(proj, conv_w, A_log, dt_bias, norm_w, conv_state, rec_state, seq_slots, positions, out, H, H, D,
                  eps, true);
}

void shortconv_decode(const Tensor& proj, const Tensor& w, const optional<Tensor>& bias, Tensor& conv_state,
                      const Tensor& seq_slots, const Tensor& positions, Tensor& out) {
  check_cuda(proj, "proj");
  const int64_t B = proj.size(0), H = w.size(0), K = w.size(1);
  TORCH_CHECK(proj.scalar_type() == at::kBFloat16 && proj.dim() == 2 && proj.stride(1) == 1 && proj.size(1) >= 3 * H,
              "b200.shortconv_decode: proj [B, >= 3H] bf16");
  TORCH_CHECK(w.scalar_type() == at::kFloat && w.is_contiguous() && w.dim() == 2, "b200.shortconv_decode: w [H, K]");
  if (bias.has_value() && bias->defined())
    TORCH_CHECK(bias->scalar_type() == at::kFloat && bias->numel() == H, "b200.shortconv_decode: bias [H] fp32");
  TORCH_CHECK(conv_state.scalar_type() == at::kBFloat16 && conv_state.is_contiguous() && conv_state.dim() == 4 &&
                  conv_state.size(1) == 2 && conv_state.size(2) == H && conv_state.size(3) == K - 1,
              "b200.shortconv_decode: conv_state [slots, 2, H, K-1] bf16");
  TORCH_CHECK(seq_slots.scalar_type() == at::kInt && seq_slots.numel() == B && positions.scalar_type() == at::kInt &&
                  positions.numel() == B,
              "b200.shortconv_decode: seq_slots / positions int32 [B]");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.is_contiguous() && out.numel() == B * H,
              "b200.shortconv_decode: out [B, H] bf16");
  c10::cuda::CUDAGuard g(proj.device());
  b200::ShortConvArgs a{};
  a.proj = reinterpret_cast<const __nv_bfloat16*>(proj.data_ptr());
  a.ld = proj.stride(0);
  a.w = w.data_ptr<float>();
  a.bias = (bias.has_value() && bias->defined()) ? bias->data_ptr<float>() : nullptr;
  a.conv_state = reinterpret_cast<__nv_bfloat16*>(conv_state.data_ptr());
  a.seq_slots = seq_slots.data_ptr<int32_t>();
  a.positions = positions.data_ptr<int32_t>();
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.B = (int)B;
  a.H = (int)H;
  a.K = (int)K;
  a.num_slots = conv_state.size(0);
  b200::shortconv_decode_launch(a, cur_stream(proj));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void ssd_decode(const Tensor& proj, int64_t xbc_off, int64_t dt_off, const Tensor& conv_w,
                const optional<Tensor>& conv_b, const Tensor& A_log, const Tensor& dt_bias, const Tensor& D,
                double dt_min, double dt_max, Tensor& conv_state, Tensor& ssm_state, const Tensor& seq_slots,
                const Tensor& positions, Tensor& out, int64_t G) {
  check_cuda(proj, "proj");
  const int64_t B = proj.size(0), H = A_log.numel();
  TORCH_CHECK(proj.scalar_type() == at::kBFloat16 && proj.dim() == 2 && proj.stride(1) == 1, "b200.ssd_decode: proj");
  TORCH_CHECK(conv_w.scalar_type() == at::kFloat && conv_w.is_contiguous() && conv_w.dim() == 2, "b200.ssd_decode: conv_w");
  const int64_t conv_dim = conv_w.size(0), K = conv_w.size(1);
  TORCH_CHECK(ssm_state.scalar_type() == at::kFloat && ssm_state.is_contiguous() && ssm_state.dim() == 4 &&
                  ssm_state.size(1) == H,
              "b200.ssd_decode: ssm_state [slots, H, N, P] fp32");
  const int64_t N = ssm_state.size(2), P = ssm_state.size(3);
  TORCH_CHECK(conv_dim == H * P + 2 * G * N, "b200.ssd_decode: conv_dim != H P + 2 G N");
  TORCH_CHECK(xbc_off + conv_dim <= proj.size(1) && dt_off + H <= proj.size(1), "b200.ssd_decode: proj offsets");
  if (conv_b.has_value() && conv_b->defined())
    TORCH_CHECK(conv_b->scalar_type() == at::kFloat && conv_b->numel() == conv_dim, "b200.ssd_decode: conv_b");
  TORCH_CHECK(A_log.scalar_type() == at::kFloat && dt_bias.scalar_type() == at::kFloat && dt_bias.numel() == H &&
                  D.scalar_type() == at::kFloat && D.numel() == H,
              "b200.ssd_decode: A_log / dt_bias / D fp32 [H]");
  TORCH_CHECK(conv_state.scalar_type() == at::kBFloat16 && conv_state.is_contiguous() && conv_state.dim() == 4 &&
                  conv_state.size(0) == ssm_state.size(0) && conv_state.size(1) == 2 &&
                  conv_state.size(2) == conv_dim && conv_state.size(3) == K - 1,
              "b200.ssd_decode: conv_state [slots, 2, conv_dim, K-1] bf16");
  TORCH_CHECK(seq_slots.scalar_type() == at::kInt && seq_slots.numel() == B && positions.scalar_type() == at::kInt &&
                  positions.numel() == B,
              "b200.ssd_decode: seq_slots / positions int32 [B]");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.is_contiguous() && out.numel() == B * H * P,
              "b200.ssd_decode: out [B, H*P] bf16");
  c10::cuda::CUDAGuard g(proj.device());
  b200::SsdDecodeArgs a{};
  a.proj = reinterpret_cast<const __nv_bfloat16*>(proj.data_ptr());
  a.ld = proj.stride(0);
  a.xbc_off = (int)xbc_off;
  a.dt_off = (int)dt_off;
  a.conv_w = conv_w.data_ptr<float>();
  a.conv_b = (conv_b.has_value() && conv_b->defined()) ? conv_b->data_ptr<float>() : nullptr;
  a.A_log = A_log.data_ptr<float>();
  a.dt_bias = dt_bias.data_ptr<float>();
  a.D = D.data_ptr<float>();
  a.dt_min = (float)dt_min;
  a.dt_max = (float)dt_max;
  a.conv_state = reinterpret_cast<__nv_bfloat16*>(conv_state.data_ptr());
  a.ssm_state = ssm_state.data_ptr<float>();
  a.seq_slots = seq_slots.data_ptr<int32_t>();
  a.positions = positions.data_ptr<int32_t>();
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.B = (int)B;
  a.H = (int)H;
  a.G = (int)G;
  a.N = (int)N;
  a.P = (int)P;
  a.K = (int)K;
  a.conv_dim = (int)conv_dim;
  a.num_slots = ssm_state.size(0);
  b200::ssd_decode_launch(a, cur_stream(proj));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void kv_summary(const Tensor& k_cache, const Tensor& slots, Tensor& summ) {
  check_cuda(k_cache, "k_cache");
  TORCH_CHECK(k_cache.scalar_type() == at::kBFloat16 && k_cache.is_contiguous() && k_cache.dim() == 4 &&
                  k_cache.size(2) == 16,
              "b200.kv_summary: k_cache [blocks, Hkv, 16, D] bf16");
  TORCH_CHECK(summ.scalar_type() == at::kBFloat16 && summ.is_contiguous() && summ.size(0) >= k_cache.size(0) &&
                  summ.size(1) == k_cache.size(1) && summ.size(2) == k_cache.size(3),
              "b200.kv_summary: summ [blocks, Hkv, D] bf16");
  TORCH_CHECK(slots.scalar_type() == at::kLong && slots.is_contiguous(), "b200.kv_summary: slots int64");
  c10::cuda::CUDAGuard g(k_cache.device());
  b200::kv_summary_launch(k_cache.data_ptr(), slots.data_ptr<int64_t>(), slots.numel(), summ.data_ptr(),
                          (int)k_cache.size(1), (int)k_cache.size(3), cur_stream(k_cache));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void kv_select(const Tensor& q, const Tensor& summ, const Tensor& tables, const Tensor& ctx, Tensor& scores,
               Tensor& sel, Tensor& sel_ctx, int64_t topk, int64_t window, int64_t sink) {
  check_cuda(q, "q");
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && q.is_contiguous() && q.dim() == 3, "b200.kv_select: q [B, Hq, D]");
  TORCH_CHECK(summ.scalar_type() == at::kBFloat16 && summ.is_contiguous() && summ.dim() == 3 &&
                  summ.size(2) == q.size(2),
              "b200.kv_select: summ [blocks, Hkv, D] bf16");
  TORCH_CHECK(tables.scalar_type() == at::kInt && tables.dim() == 2 && tables.is_contiguous() &&
                  tables.size(0) == q.size(0),
              "b200.kv_select: tables [B, W] int32");
  TORCH_CHECK(ctx.scalar_type() == at::kInt && ctx.numel() == q.size(0), "b200.kv_select: ctx [B] int32");
  const int64_t budget = topk + window + sink;
  TORCH_CHECK(sel.scalar_type() == at::kInt && sel.is_contiguous() && sel.size(0) == q.size(0) &&
                  sel.size(1) == budget && sel_ctx.scalar_type() == at::kInt && sel_ctx.numel() == q.size(0),
              "b200.kv_select: sel [B, budget] / sel_ctx [B] int32");
  TORCH_CHECK(q.size(1) % summ.size(1) == 0, "b200.kv_select: Hq must be a multiple of Hkv");
  c10::cuda::CUDAGuard g(q.device());
  b200::KvSelectArgs a{};
  a.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  a.summ = reinterpret_cast<const __nv_bfloat16*>(summ.data_ptr());
  a.tables = tables.data_ptr<int32_t>();
  a.ctx = ctx.data_ptr<int32_t>();
  TORCH_CHECK(scores.scalar_type() == at::kFloat && scores.is_contiguous() && scores.numel() >= tables.numel(),
              "b200.kv_select: scores workspace [B, W] fp32");
  a.scores = scores.data_ptr<float>();
  a.sel = sel.data_ptr<int32_t>();
  a.sel_ctx = sel_ctx.data_ptr<int32_t>();
  a.B = (int)q.size(0);
  a.W = (int)tables.size(1);
  a.Hq = (int)q.size(1);
  a.Hkv = (int)summ.size(1);
  a.D = (int)q.size(2);
  a.topk = (int)topk;
  a.window = (int)window;
  a.sink = (int)sink;
  a.budget = (int)budget;
  b200::kv_select_launch(a, cur_stream(q));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

static b200::MambaScanArgs mamba_args(const Tensor& cu, const Tensor& slots, const Tensor& positions, int64_t Di,
                                      int64_t num_slots) {
  TORCH_CHECK(cu.scalar_type() == at::kInt && cu.is_contiguous() && cu.dim() == 1 && cu.numel() >= 1,
              "b200.mamba: cu int32 [nseq + 1]");
  TORCH_CHECK(slots.scalar_type() == at::kLong && slots.is_contiguous() && slots.numel() == cu.numel() - 1,
              "b200.mamba: slots int64 [nseq]");
  TORCH_CHECK(positions.scalar_type() == at::kInt && positions.is_contiguous(), "b200.mamba: positions int32");
  b200::MambaScanArgs a{};
  a.cu = cu.data_ptr<int32_t>();
  a.slots = slots.data_ptr<int64_t>();
  a.positions = positions.data_ptr<int32_t>();
  a.nseq = (int)(cu.numel() - 1);
  a.Di = (int)Di;
  a.num_slots = num_slots;
  return a;
}

void mamba_conv(const Tensor& cu, const Tensor& slots, const Tensor& positions, const Tensor& x_raw,
                const Tensor& conv_w, const optional<Tensor>& conv_b, Tensor& conv_state, Tensor& x_out) {
  check_cuda(x_raw, "x_raw");
  const int64_t Di = conv_w.size(0), K = conv_w.size(1);
  TORCH_CHECK(x_raw.scalar_type() == at::kBFloat16 && x_raw.dim() == 2 && x_raw.stride(1) == 1 &&
                  x_raw.size(1) >= Di && x_raw.size(0) == positions.numel(),
              "b200.mamba_conv: x_raw [T, >= Di] bf16");
  TORCH_CHECK(conv_w.scalar_type() == at::kFloat && conv_w.is_contiguous(), "b200.mamba_conv: conv_w [Di, K] fp32");
  if (conv_b.has_value() && conv_b->defined())
    TORCH_CHECK(conv_b->scalar_type() == at::kFloat && conv_b->numel() == Di, "b200.mamba_conv: conv_b");
  TORCH_CHECK(conv_state.scalar_type() == at::kBFloat16 && conv_state.is_contiguous() && conv_state.dim() == 3 &&
                  conv_state.size(1) == Di && conv_state.size(2) == K - 1,
              "b200.mamba_conv: conv_state [slots, Di, K-1] bf16");
  TORCH_CHECK(x_out.scalar_type() == at::kBFloat16 && x_out.is_contiguous() && x_out.size(0) == x_raw.size(0) &&
                  x_out.size(1) == Di,
              "b200.mamba_conv: x_out [T, Di] bf16");
  c10::cuda::CUDAGuard g(x_raw.device());
  auto a = mamba_args(cu, slots, positions, Di, conv_state.size(0));
  a.x_raw = reinterpret_cast<const __nv_bfloat16*>(x_raw.data_ptr());
  a.ld_raw = x_raw.stride(0);
  a.conv_w = conv_w.data_ptr<float>();
  a.conv_b = (conv_b.has_value() && conv_b->defined()) ? conv_b->data_ptr<float>() : nullptr;
  a.conv_state = reinterpret_cast<__nv_bfloat16*>(conv_state.data_ptr());
  a.x_out = reinterpret_cast<__nv_bfloat16*>(x_out.data_ptr());
  a.K = (int)K;
  b200::mamba_conv_launch(a, cur_stream(x_raw));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void mamba_scan(const Tensor& cu, const Tensor& slots, const Tensor& positions, const Tensor& x, const Tensor& dt,
                const Tensor& dt_bias, const Tensor& Bc, int64_t c_off, const Tensor& A_log, const Tensor& D,
                const Tensor& z, Tensor& ssm_state, Tensor& y) {
  check_cuda(x, "x");
  const int64_t T = x.size(0), Di = x.size(1), N = A_log.size(1);
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.is_contiguous(), "b200.mamba_scan: x [T, Di] bf16");
  for (const Tensor* t : {&dt, &Bc, &z})
    TORCH_CHECK(t->scalar_type() == at::kBFloat16 && t->dim() == 2 && t->stride(1) == 1 && t->size(0) == T,
                "b200.mamba_scan: dt / Bc / z [T, *] bf16 with unit inner stride");
  TORCH_CHECK(dt.size(1) >= Di && z.size(1) >= Di && Bc.size(1) >= c_off + N, "b200.mamba_scan: widths");
  TORCH_CHECK(A_log.scalar_type() == at::kFloat && A_log.is_contiguous() && A_log.size(0) == Di &&
                  dt_bias.scalar_type() == at::kFloat && dt_bias.numel() == Di && D.scalar_type() == at::kFloat &&
                  D.numel() == Di,
              "b200.mamba_scan: A_log [Di, N] / dt_bias / D fp32");
  TORCH_CHECK(ssm_state.scalar_type() == at::kFloat && ssm_state.is_contiguous() && ssm_state.dim() == 3 &&
                  ssm_state.size(1) == Di && ssm_state.size(2) == N,
              "b200.mamba_scan: ssm_state [slots, Di, N] fp32");
  TORCH_CHECK(y.scalar_type() == at::kBFloat16 && y.is_contiguous() && y.sizes() == x.sizes(), "b200.mamba_scan: y");
  c10::cuda::CUDAGuard g(x.device());
  auto a = mamba_args(cu, slots, positions, Di, ssm_state.size(0));
  a.x_out = reinterpret_cast<__nv_bfloat16*>(const_cast<void*>(x.data_ptr()));
  a.dt = reinterpret_cast<const __nv_bfloat16*>(dt.data_ptr());
  a.ld_dt = dt.stride(0);
  a.dt_bias = dt_bias.data_ptr<float>();
  a.Bc = reinterpret_cast<const __nv_bfloat16*>(Bc.data_ptr());
  a.ld_bc = Bc.stride(0);
  a.c_off = (int)c_off;
  a.A_log = A_log.data_ptr<float>();
  a.D = D.data_ptr<float>();
  a.z = reinterpret_cast<const __nv_bfloat16*>(z.data_ptr());
  a.ld_z = z.stride(0);
  a.ssm_state = ssm_state.data_ptr<float>();
  a.y = reinterpret_cast<__nv_bfloat16*>(y.data_ptr());
  a.N = (int)N;
  b200::mamba_scan_launch(a, cur_stream(x));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void embedding(const Tensor& ids, const Tensor& table, Tensor& out) {
  check_cuda(ids, "ids");
  TORCH_CHECK(ids.scalar_type() == at::kInt && ids.is_contiguous(), "b200.embedding: int32 ids");
  TORCH_CHECK(table.scalar_type() == at::kBFloat16 && table.is_contiguous() && table.size(1) % 8 == 0,
              "b200.embedding: table");
  TORCH_CHECK(out.is_contiguous() && out.size(0) == ids.numel() && out.size(1) == table.size(1), "b200.embedding: out");
  c10::cuda::CUDAGuard g(ids.device());
  b200::embedding_launch(ids.data_ptr<int32_t>(), table.data_ptr(), out.data_ptr(), ids.numel(), table.size(1),
                         table.size(0), cur_stream(ids));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void rmsnorm(const Tensor& x, const Tensor& w, Tensor& out, double eps, const optional<Tensor>& residual_in,
             const optional<Tensor>& residual_out) {
  check_cuda(x, "x");
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.dim() == 2 && x.stride(1) == 1, "b200.rmsnorm: x");
  const int64_t T = x.size(0), H = x.size(1);
  TORCH_CHECK(H % 8 == 0, "b200.rmsnorm: hidden % 8");
  TORCH_CHECK(w.numel() == H && w.scalar_type() == at::kBFloat16, "b200.rmsnorm: weight");
  TORCH_CHECK(out.size(0) == T && out.size(1) == H && out.stride(1) == 1, "b200.rmsnorm: out");
  if (residual_in.has_value() && residual_in->defined())
    TORCH_CHECK(residual_in->is_contiguous() && residual_in->numel() == T * H, "b200.rmsnorm: residual_in");
  if (residual_out.has_value() && residual_out->defined())
    TORCH_CHECK(residual_out->is_contiguous() && residual_out->numel() == T * H, "b200.rmsnorm: residual_out");
  c10::cuda::CUDAGuard g(x.device());
  b200::rmsnorm_launch(x.data_ptr(), x.stride(0), opt_ptr(residual_in),
                       const_cast<void*>(opt_ptr(residual_out)), w.data_ptr(), out.data_ptr(), out.stride(0), T, H,
                       (float)eps, cur_stream(x));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void qkv_rope(const Tensor& qkv, const optional<Tensor>& q_norm, const optional<Tensor>& k_norm,
              const Tensor& positions, const optional<Tensor>& slots, const Tensor& inv_freq, double rope_scale,
              Tensor& q_out, const optional<Tensor>& k_cache, const optional<Tensor>& v_cache,
              const optional<Tensor>& k_out, const optional<Tensor>& v_out, int64_t Hq, int64_t Hkv, int64_t D,
              double eps, int64_t rot_dim, const optional<Tensor>& bias, double k_scale, double v_scale) {
  check_cuda(qkv, "qkv");
  if (rot_dim <= 0) rot_dim = D;
  TORCH_CHECK(rot_dim <= D && rot_dim % (2 * (D / 32)) == 0, "b200.qkv_rope: rot_dim must be <= head_dim and a "
              "multiple of 2 * head_dim / 32");
  TORCH_CHECK((qkv.scalar_type() == at::kBFloat16 || qkv.scalar_type() == at::kFloat) && qkv.dim() == 2 &&
                  qkv.stride(1) == 1,
              "b200.qkv_rope: qkv");
  TORCH_CHECK(qkv.size(1) == (Hq + 2 * Hkv) * D, "b200.qkv_rope: qkv width");
  TORCH_CHECK(D == 64 || D == 128 || D == 256, "b200.qkv_rope: head_dim 64, 128 or 256");
  TORCH_CHECK(positions.scalar_type() == at::kInt && positions.numel() == qkv.size(0), "b200.qkv_rope: positions");
  TORCH_CHECK(inv_freq.scalar_type() == at::kFloat && inv_freq.numel() == rot_dim / 2, "b200.qkv_rope: inv_freq");
  TORCH_CHECK(q_out.is_contiguous() && q_out.numel() == qkv.size(0) * Hq * D, "b200.qkv_rope: q_out");
  if (slots.has_value() && slots->defined()) {
    TORCH_CHECK(slots->scalar_type() == at::kLong && slots->numel() == qkv.size(0), "b200.qkv_rope: slots");
    TORCH_CHECK(k_cache.has_value() && v_cache.has_value(), "b200.qkv_rope: caches");
  }
  c10::cuda::CUDAGuard g(qkv.device());
  b200::QkvRopeArgs a{};
  a.qkv = qkv.data_ptr();
  if (qkv.scalar_type() == at::kFloat) a.qkv_f32 = qkv.data_ptr<float>();
  if (bias.has_value() && bias->defined()) {
    TORCH_CHECK(qkv.scalar_type() == at::kFloat && bias->scalar_type() == at::kBFloat16 &&
                    bias->numel() == qkv.size(1),
                "b200.qkv_rope: bias applies to the fp32 accumulate input, bf16 [(Hq + 2 Hkv) * D]");
    a.bias = bias->data_ptr();
  }
  a.ld_qkv = qkv.stride(0);
  a.q_norm = opt_ptr(q_norm);
  a.k_norm = opt_ptr(k_norm);
  a.positions = positions.data_ptr<int32_t>();
  a.slots = (slots.has_value() && slots->defined()) ? slots->data_ptr<int64_t>() : nullptr;
  a.inv_freq = inv_freq.data_ptr<float>();
  a.rope_scale = (float)rope_scale;
  a.rot_dim = (int)rot_dim;
  a.q_out = q_out.data_ptr();
  a.k_cache = const_cast<void*>(opt_ptr(k_cache));
  a.v_cache = const_cast<void*>(opt_ptr(v_cache));
  if (k_cache.has_value() && k_cache->defined()) {
    const auto kt = k_cache->scalar_type();
    TORCH_CHECK((kt == at::kBFloat16 || kt == at::kFloat8_e4m3fn) && v_cache.has_value() &&
                    v_cache->scalar_type() == kt,
                "b200.qkv_rope: caches bf16 or float8_e4m3fn, both the same");
    if (kt == at::kFloat8_e4m3fn) {
      TORCH_CHECK(k_scale > 0 && v_scale > 0, "b200.qkv_rope: fp8 cache scales must be > 0");
      a.kv_fp8 = 1;
      a.k_inv_scale = (float)(1.0 / k_scale);
      a.v_inv_scale = (float)(1.0 / v_scale);
    }
  }
  a.k_out = const_cast<void*>(opt_ptr(k_out));
  a.v_out = const_cast<void*>(opt_ptr(v_out));
  a.T = qkv.size(0);
  a.Hq = (int)Hq;
  a.Hkv = (int)Hkv;
  a.D = (int)D;
  a.eps = (float)eps;
  b200::qkv_rope_launch(a, cur_stream(qkv));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

static b200::AttnArgs attn_args(const Tensor& q, const Tensor& k_cache, const Tensor& v_cache,
                                const Tensor& block_tables, const Tensor& ctx_lens, Tensor& out,
                                const optional<Tensor>& sinks, int64_t window, double scale, Tensor& status) {
  check_cuda(q, "q");
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && q.dim() == 3 && q.is_contiguous(), "b200.attention: q [T,Hq,D]");
  const bool dense = k_cache.dim() == 3;  // prefill only: row-major [rows, Hkv, D] (pages of 16 rows)
  TORCH_CHECK((k_cache.dim() == 4 || dense) && v_cache.dim() == k_cache.dim() && k_cache.is_contiguous() &&
                  v_cache.is_contiguous(),
              "b200.attention: caches [NB,Hkv,16,D] (or [rows,Hkv,D] for prefill)");
  TORCH_CHECK(dense ? (k_cache.size(0) % 16 == 0 && k_cache.size(2) == q.size(2))
                    : (k_cache.size(2) == 16 && k_cache.size(3) == q.size(2)),
              "b200.attention: cache block/head dim");
  TORCH_CHECK(block_tables.scalar_type() == at::kInt && block_tables.dim() == 2 && block_tables.is_contiguous(),
              "b200.attention: block_tables int32 [B, max_blocks]");
  TORCH_CHECK(ctx_lens.scalar_type() == at::kInt && ctx_lens.numel() == block_tables.size(0),
              "b200.attention: ctx_lens");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 &&
                  ((out.is_contiguous() && out.sizes() == q.sizes()) ||
                   (out.dim() == 2 && out.size(0) == q.size(0) && out.stride(1) == 1)),
              "b200.attention: out [Tq, Hq, D] (or a row-strided [Tq, Hq * D] view for prefill)");
  if (sinks.has_value() && sinks->defined())
    TORCH_CHECK(sinks->scalar_type() == at::kFloat && sinks->numel() == q.size(1), "b200.attention: sinks f32 [Hq]");
  TORCH_CHECK((k_cache.scalar_type() == at::kBFloat16 || k_cache.scalar_type() == at::kFloat8_e4m3fn) &&
                  v_cache.scalar_type() == k_cache.scalar_type(),
              "b200.attention: caches bf16 or float8_e4m3fn, both the same");
  b200::AttnArgs a{};
  a.kv_fp8 = k_cache.scalar_type() == at::kFloat8_e4m3fn ? 1 : 0;
  a.q = q.data_ptr();
  a.k_cache = k_cache.data_ptr();
  a.v_cache = v_cache.data_ptr();
  a.num_blocks = dense ? k_cache.size(0) / 16 : k_cache.size(0);
  a.block_tables = block_tables.data_ptr<int32_t>();
  a.max_blocks = (int)block_tables.size(1);
  a.ctx_lens = ctx_lens.data_ptr<int32_t>();
  a.out = out.data_ptr();
  a.sinks = (sinks.has_value() && sinks->defined()) ? sinks->data_ptr<float>() : nullptr;
  a.window = (int)window;
  a.B = (int)block_tables.size(0);
  a.Hq = (int)q.size(1);
  a.Hkv = (int)k_cache.size(1);
  a.D = (int)q.size(2);
  a.scale = (float)scale;
  a.status = status.data_ptr<int>();
  a.device = q.get_device();
  return a;
}

int64_t decode_attention(const Tensor& q, const Tensor& k_cache, const Tensor& v_cache, const Tensor& block_tables,
                         const Tensor& ctx_lens, Tensor& out, const optional<Tensor>& sinks, int64_t window,
                         double scale, int64_t splits, Tensor& ws, Tensor& status, double softcap, double k_scale,
                         double v_scale) {
  c10::cuda::CUDAGuard g(q.device());
  auto a = attn_args(q, k_cache, v_cache, block_tables, ctx_lens, out, sinks, window, scale, status);
  a.softcap = (float)softcap;
  a.k_scale = (float)k_scale;
  a.v_scale = (float)v_scale;
  TORCH_CHECK(q.size(0) == block_tables.size(0), "b200.decode_attention: one query per sequence");
  a.cu_q = nullptr;
  a.splits = (int)splits;
  a.ws = ws.numel() ? ws.data_ptr<float>() : nullptr;
  a.ws_elems = ws.numel();
  const int n = b200::decode_attention_launch(a, cur_stream(q));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return n;
}

void prefill_attention(const Tensor& q, const Tensor& k_cache, const Tensor& v_cache, const Tensor& block_tables,
                       const Tensor& ctx_lens, const Tensor& cu_q, Tensor& out, const optional<Tensor>& sinks,
                       int64_t window, double scale, int64_t max_q_len, Tensor& status, bool causal, bool q_paged,
                       double softcap) {
  c10::cuda::CUDAGuard g(q.device());
  auto a = attn_args(q, k_cache, v_cache, block_tables, ctx_lens, out, sinks, window, scale, status);
  TORCH_CHECK(!a.kv_fp8, "b200.prefill: fp8 pages are read through kv_dequant_pages (bf16 copies)");
  a.softcap = (float)softcap;
  TORCH_CHECK(cu_q.scalar_type() == at::kInt && cu_q.numel() == block_tables.size(0) + 1, "b200.prefill: cu_q");
  a.cu_q = cu_q.data_ptr<int32_t>();
  a.max_q_len = (int)max_q_len;
  a.causal = causal ? 1 : 0;
  a.q_paged = q_paged ? 1 : 0;
  a.q_rows = q.size(0);
  if (k_cache.dim() == 3) {  // row-major [rows, Hkv, D] keys / values
    a.kv_dense = 1;
    a.kv_rows = k_cache.size(0);
  }
  if (out.dim() == 2) {  // [rows, Hq * D] view with a row stride (DiT: a column slice of a wider buffer)
    TORCH_CHECK(out.stride(1) == 1 && out.size(1) == a.Hq * a.D && out.stride(0) % 8 == 0,
                "b200.prefill: 2-D out must be [rows, Hq * D] with unit inner stride");
    a.out_ld = out.stride(0);
  }
  b200::prefill_attention_launch(a, cur_stream(q));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void kv_dequant_pages(const Tensor& k8, const Tensor& v8, const Tensor& block_tables, const Tensor& ctx_lens,
                      double k_scale, double v_scale, Tensor& k_out, Tensor& v_out) {
  check_cuda(k8, "k8");
  TORCH_CHECK(k8.scalar_type() == at::kFloat8_e4m3fn && v8.scalar_type() == at::kFloat8_e4m3fn && k8.dim() == 4 &&
                  k8.is_contiguous() && v8.is_contiguous() && v8.sizes() == k8.sizes() && k8.size(2) == 16,
              "b200.kv_dequant_pages: float8_e4m3fn pages [NB, Hkv, 16, D]");
  TORCH_CHECK(block_tables.scalar_type() == at::kInt && block_tables.dim() == 2 && block_tables.is_contiguous() &&
                  ctx_lens.scalar_type() == at::kInt && ctx_lens.numel() == block_tables.size(0),
              "b200.kv_dequant_pages: int32 tables [B, max_blocks] and ctx_lens [B]");
  const int64_t B = block_tables.size(0), mb = block_tables.size(1), Hkv = k8.size(1), D = k8.size(3);
  TORCH_CHECK(D % 16 == 0, "b200.kv_dequant_pages: D % 16");
  for (const Tensor* t : {&k_out, &v_out})
    TORCH_CHECK(t->scalar_type() == at::kBFloat16 && t->is_contiguous() && t->dim() == 4 && t->size(0) >= B * mb &&
                    t->size(1) == Hkv && t->size(2) == 16 && t->size(3) == D && t->device() == k8.device(),
                "b200.kv_dequant_pages: bf16 outputs [>= B * max_blocks, Hkv, 16, D]");
  c10::cuda::CUDAGuard g(k8.device());
  b200::kv_dequant_pages_launch(k8.data_ptr(), v8.data_ptr(), block_tables.data_ptr<int32_t>(),
                                ctx_lens.data_ptr<int32_t>(), (int)B, (int)mb, (int)Hkv, (int)D, (float)k_scale,
                                (float)v_scale, k_out.data_ptr(), v_out.data_ptr(), cur_stream(k8));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void argmax(const Tensor& logits, Tensor& out) {
  check_cuda(logits, "logits");
  TORCH_CHECK(logits.scalar_type() == at::kFloat && logits.dim() == 2 && logits.stride(1) == 1, "b200.argmax");
  TORCH_CHECK(out.scalar_type() == at::kInt && out.numel() == logits.size(0), "b200.argmax: out");
  c10::cuda::CUDAGuard g(logits.device());
  b200::argmax_launch(logits.data_ptr<float>(), logits.stride(0), logits.size(0), logits.size(1),
                      out.data_ptr<int32_t>(), cur_stream(logits));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void forward_tokens(Tensor& ids, const Tensor& src, const Tensor& prev) {
  check_cuda(ids, "ids");
  TORCH_CHECK(ids.scalar_type() == at::kInt && src.scalar_type() == at::kInt && prev.scalar_type() == at::kInt &&
                  ids.is_contiguous() && src.is_contiguous() && prev.is_contiguous() && src.numel() >= ids.numel(),
              "b200.forward_tokens: int32 ids / src / prev");
  c10::cuda::CUDAGuard g(ids.device());
  b200::forward_tokens_launch(ids.data_ptr<int32_t>(), src.data_ptr<int32_t>(), prev.data_ptr<int32_t>(),
                              (int)ids.numel(), cur_stream(ids));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void sample(const Tensor& logits, const Tensor& temperature, const Tensor& top_k, const Tensor& top_p,
            const Tensor& min_p, const Tensor& seeds, const Tensor& offsets, Tensor& out,
            const optional<Tensor>& logprob) {
  check_cuda(logits, "logits");
  TORCH_CHECK(logits.scalar_type() == at::kFloat && logits.dim() == 2 && logits.stride(1) == 1, "b200.sample");
  const int64_t B = logits.size(0);
  TORCH_CHECK(temperature.numel() == B && top_k.numel() == B && top_p.numel() == B && min_p.numel() == B &&
                  seeds.numel() == B && offsets.numel() == B && out.numel() == B,
              "b200.sample: per-row parameter sizes");
  TORCH_CHECK(temperature.scalar_type() == at::kFloat && top_k.scalar_type() == at::kInt &&
                  top_p.scalar_type() == at::kFloat && min_p.scalar_type() == at::kFloat &&
                  seeds.scalar_type() == at::kLong && offsets.scalar_type() == at::kLong &&
                  out.scalar_type() == at::kInt,
              "b200.sample: parameter dtypes");
  c10::cuda::CUDAGuard g(logits.device());
  b200::SampleArgs a{};
  a.logits = logits.data_ptr<float>();
  a.ld = logits.stride(0);
  a.B = B;
  a.V = logits.size(1);
  a.temperature = temperature.data_ptr<float>();
  a.top_k = top_k.data_ptr<int32_t>();
  a.top_p = top_p.data_ptr<float>();
  a.min_p = min_p.data_ptr<float>();
  a.seeds = reinterpret_cast<const uint64_t*>(seeds.data_ptr<int64_t>());
  a.offsets = offsets.data_ptr<int64_t>();
  a.out = out.data_ptr<int32_t>();
  a.out_logprob = (logprob.has_value() && logprob->defined()) ? logprob->data_ptr<float>() : nullptr;
  b200::sample_launch(a, cur_stream(logits));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ---------------------------------------------------------------------------
// Symmetric memory: raw device buffers shared between ranks by CUDA IPC.
// ---------------------------------------------------------------------------
int64_t symm_malloc(int64_t bytes, int64_t device) {
  c10::cuda::CUDAGuard g((c10::DeviceIndex)device);
  void* p = nullptr;
  C10_CUDA_CHECK(cudaMalloc(&p, (size_t)bytes));
  C10_CUDA_CHECK(cudaMemset(p, 0, (size_t)bytes));
  return reinterpret_cast<int64_t>(p);
}

void symm_free(int64_t ptr, int64_t device) {
  c10::cuda::CUDAGuard g((c10::DeviceIndex)device);
  C10_CUDA_CHECK(cudaFree(reinterpret_cast<void*>(ptr)));
}

py::bytes ipc_handle(int64_t ptr, int64_t device) {
  c10::cuda::CUDAGuard g((c10::DeviceIndex)device);
  cudaIpcMemHandle_t h;
  C10_CUDA_CHECK(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(ptr)));
  return py::bytes(reinterpret_cast<const char*>(&h), sizeof(h));
}

int64_t ipc_open(py::bytes handle, int64_t device) {
  c10::cuda::CUDAGuard g((c10::DeviceIndex)device);
  std::string s = handle;
  TORCH_CHECK(s.size() == sizeof(cudaIpcMemHandle_t), "b200.ipc_open: bad handle size");
  cudaIpcMemHandle_t h;
  memcpy(&h, s.data(), sizeof(h));
  void* p = nullptr;
  C10_CUDA_CHECK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  return reinterpret_cast<int64_t>(p);
}

void ipc_close(int64_t ptr, int64_t device) {
  c10::cuda::CUDAGuard g((c10::DeviceIndex)device);
  C10_CUDA_CHECK(cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr)));
}

Tensor tensor_from_ptr(int64_t ptr, std::vector<int64_t> sizes, at::ScalarType dtype, int64_t device) {
  auto opts = at::TensorOptions().dtype(dtype).device(at::kCUDA, (c10::DeviceIndex)device);
  return torch::from_blob(reinterpret_cast<void*>(ptr), sizes, opts);
}

// GEMM in reduce-scatter push mode (see gemm_sm100.cuh). peer_out / peer_flags
// are device int64 arrays of peer pointers; epoch / done_ctr are local uint32.
void linear_push(const Tensor& x, const Tensor& w, const optional<Tensor>& bias, int64_t mode, bool bcast, int64_t rpr,
                 int64_t ld_out, int64_t slot_elems, int64_t my_rank, int64_t world, const Tensor& peer_out,
                 const Tensor& peer_flags, const Tensor& epoch, const Tensor& done_ctr, Tensor& ws, Tensor& sem,
                 Tensor& status) {
  check_cuda(x, "x");
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16 && x.dim() == 2 && w.dim() == 2,
              "b200.linear_push: bf16 2-D");
  TORCH_CHECK(x.stride(1) == 1 && w.stride(1) == 1 && x.size(1) == w.size(1), "b200.linear_push: shapes");
  TORCH_CHECK(peer_out.scalar_type() == at::kLong && peer_out.numel() == world && peer_flags.numel() == world,
              "b200.linear_push: peer arrays");
  c10::cuda::CUDAGuard g(x.device());
  b200::LinearArgs a{};
  a.x = x.data_ptr();
  a.ldx = x.stride(0);
  a.w = w.data_ptr();
  a.ldw = w.stride(0);
  a.out = nullptr;
  a.ldo = ld_out;
  a.residual = nullptr;
  a.bias = opt_ptr(bias);
  a.M = x.size(0);
  a.N = w.size(0);
  a.K = x.size(1);
  TORCH_CHECK(mode == 0 || (mode == 3 && x.size(0) <= 128 && !(bias.has_value() && bias->defined())),
              "b200.linear_push: mode 0 (bf16 slots) or 3 (fp32 accumulate, M <= 128, no bias)");
  a.mode = (int)mode;
  a.alpha = 1.f;
  a.swap = -1;
  a.bn = 0;
  a.splits = 0;
  a.ws = ws.data_ptr<float>();
  a.ws_elems = ws.numel();
  a.sem = sem.data_ptr<int>();
  a.sem_elems = sem.numel();
  a.status = status.data_ptr<int>();
  a.device = x.get_device();
  a.peer_out = reinterpret_cast<void* const*>(peer_out.data_ptr<int64_t>());
  a.rpr = (int)rpr;
  a.slot_elems = slot_elems;
  a.my_rank = (int)my_rank;
  a.world = (int)world;
  a.epoch = reinterpret_cast<const unsigned*>(epoch.data_ptr<int>());
  a.done_ctr = reinterpret_cast<unsigned*>(done_ctr.data_ptr<int>());
  a.peer_flags = reinterpret_cast<unsigned* const*>(peer_flags.data_ptr<int64_t>());
  a.bcast = bcast ? 1 : 0;
  b200::linear_launch(a, cur_stream(x));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void rs_norm_ag(const optional<Tensor>& recv, const optional<Tensor>& racc, Tensor& h, const Tensor& norm_w, const Tensor& peer_gath,
                const Tensor& rs_flags, const Tensor& ag_flags, const Tensor& peer_ag_flags, Tensor& epoch,
                Tensor& cta_ctr, int64_t M, int64_t rpr, int64_t world, int64_t rank, int64_t slot_elems,
                double eps, Tensor& status) {
  check_cuda(h, "h");
  TORCH_CHECK(h.scalar_type() == at::kBFloat16 && h.is_contiguous(), "b200.rs_norm_ag: h");
  c10::cuda::CUDAGuard g(h.device());
  b200::RsNormAgArgs a{};
  a.recv = opt_ptr(recv);
  a.h = h.data_ptr();
  a.norm_w = norm_w.data_ptr();
  a.peer_gath = reinterpret_cast<void* const*>(peer_gath.data_ptr<int64_t>());
  a.rs_flags = reinterpret_cast<const unsigned*>(rs_flags.data_ptr<int>());
  a.ag_flags = reinterpret_cast<const unsigned*>(ag_flags.data_ptr<int>());
  a.peer_ag_flags = reinterpret_cast<unsigned* const*>(peer_ag_flags.data_ptr<int64_t>());
  a.epoch = reinterpret_cast<unsigned*>(epoch.data_ptr<int>());
  a.cta_ctr = reinterpret_cast<unsigned*>(cta_ctr.data_ptr<int>());
  a.M = (int)M;
  a.H = (int)h.size(1);
  a.rpr = (int)rpr;
  a.world = (int)world;
  a.rank = (int)rank;
  a.racc = (racc.has_value() && racc->defined()) ? racc->data_ptr<float>() : nullptr;
  a.do_reduce = a.racc != nullptr ? 2 : (a.recv != nullptr ? 1 : 0);
  a.slot_elems = slot_elems;
  a.eps = (float)eps;
  a.status = status.data_ptr<int>();
  b200::rs_norm_ag_launch(a, cur_stream(h));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void add_rmsnorm_acc(Tensor& acc, Tensor& h, const Tensor& w, Tensor& out, double eps,
                     const optional<Tensor>& bias) {
  check_cuda(acc, "acc");
  TORCH_CHECK(acc.scalar_type() == at::kFloat && acc.is_contiguous() && h.is_contiguous() &&
                  h.scalar_type() == at::kBFloat16 && acc.sizes() == h.sizes() && h.size(1) % 8 == 0,
              "b200.add_rmsnorm_acc: shapes");
  c10::cuda::CUDAGuard g(acc.device());
  b200::add_rmsnorm_acc_launch(acc.data_ptr<float>(), h.data_ptr(), w.data_ptr(), out.data_ptr(), out.stride(0),
                               h.size(0), h.size(1), (float)eps, cur_stream(acc), opt_ptr(bias));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void swiglu_acc(Tensor& acc, Tensor& out, int64_t act) {
  check_cuda(acc, "acc");
  TORCH_CHECK(acc.scalar_type() == at::kFloat && acc.is_contiguous() && out.is_contiguous() &&
                  acc.size(1) == 2 * out.size(1) && out.size(1) % 64 == 0 && acc.size(0) == out.size(0),
              "b200.swiglu_acc: shapes");
  c10::cuda::CUDAGuard g(acc.device());
  b200::swiglu_acc_launch(acc.data_ptr<float>(), out.data_ptr(), out.size(0), out.size(1), (int)act, cur_stream(acc));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// out[M, N] = alpha * a[M, K] @ b[K, N] for any mix of row-major / transposed
// views (the operand majors are read from the strides); bf16 inputs.
// Operand layouts of the training GEMM: A [M, K] and B [K, N], each row-major
// or a transposed view.
static void gemm_operands(const Tensor& a, const Tensor& b, b200::GemmArgs& g) {
  check_cuda(a, "a");
  TORCH_CHECK(a.scalar_type() == at::kBFloat16 && b.scalar_type() == at::kBFloat16 && a.dim() == 2 && b.dim() == 2,
              "b200.gemm: bf16 2-D operands");
  TORCH_CHECK(b.size(0) == a.size(1), "b200.gemm: inner dims");
  if (a.stride(1) == 1) { g.a_mn = 0; g.lda = a.stride(0); }
  else { TORCH_CHECK(a.stride(0) == 1, "b200.gemm: a must be row-major or a transposed view"); g.a_mn = 1; g.lda = a.stride(1); }
  if (b.stride(0) == 1) { g.b_mn = 0; g.ldb = b.stride(1); }
  else { TORCH_CHECK(b.stride(1) == 1, "b200.gemm: b must be row-major or a transposed view"); g.b_mn = 1; g.ldb = b.stride(0); }
  TORCH_CHECK(!(g.a_mn && !g.b_mn), "b200.gemm: transposed a needs row-major b");
  TORCH_CHECK(g.lda % 8 == 0 && g.ldb % 8 == 0, "b200.gemm: strides % 8");
  g.a = a.data_ptr();
  g.b = b.data_ptr();
  g.MA = a.size(0);
  g.NB = b.size(1);
  g.K = a.size(1);
}

// FSDP weight gradient pushed into the owners' gradient shards: element
// (i, j) of a @ b is added to flat parameter base + i * N + j of the group
// whose shard_n-element shards live at peer_shards[rank] (an int64 table of
// device addresses, this GPU's own shard included).
void gemm_push_shards(const Tensor& a, const Tensor& b, const Tensor& peer_shards, int64_t base, int64_t shard_n,
                      double alpha, Tensor& ws, Tensor& sem, Tensor& status) {
  b200::GemmArgs g{};
  gemm_operands(a, b, g);
  TORCH_CHECK(peer_shards.scalar_type() == at::kLong && peer_shards.is_cuda() && shard_n > 0 && base >= 0,
              "b200.gemm_push_shards: peer table / shard size");
  g.c = nullptr;
  g.ldc = g.NB;
  g.out_f32 = 1;
  g.alpha = (float)alpha;
  g.ws = ws.data_ptr<float>();
  g.ws_elems = ws.numel();
  g.sem = sem.data_ptr<int>();
  g.sem_elems = sem.numel();
  g.status = status.data_ptr<int>();
  g.device = a.get_device();
  g.shard_peer = reinterpret_cast<float* const*>(peer_shards.data_ptr<int64_t>());
  g.shard_base = base;
  g.shard_n = shard_n;
  c10::cuda::CUDAGuard gd(a.device());
  b200::gemm_launch(g, cur_stream(a));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void gemm(const Tensor& a, const Tensor& b, Tensor& out, bool accumulate, double alpha,
          const optional<Tensor>& residual, const optional<Tensor>& bias, bool prefetch_b, Tensor& ws, Tensor& sem,
          Tensor& status) {
  check_cuda(a, "a");
  TORCH_CHECK(a.scalar_type() == at::kBFloat16 && b.scalar_type() == at::kBFloat16 && a.dim() == 2 && b.dim() == 2,
              "b200.gemm: bf16 2-D operands");
  const int64_t M = a.size(0), K = a.size(1), N = b.size(1);
  TORCH_CHECK(b.size(0) == K, "b200.gemm: inner dims");
  TORCH_CHECK(out.dim() == 2 && out.size(0) == M && out.size(1) == N && out.stride(1) == 1, "b200.gemm: out");
  b200::GemmArgs g{};
  // A[i=m, k]: K-major if a is row-major, MN-major if a is a transposed view
  if (a.stride(1) == 1) { g.a_mn = 0; g.lda = a.stride(0); }
  else { TORCH_CHECK(a.stride(0) == 1, "b200.gemm: a must be row-major or a transposed view"); g.a_mn = 1; g.lda = a.stride(1); }
  // B[j=n, k]: K-major if b is a transposed view of [N, K], MN-major if b is row-major [K, N]
  if (b.stride(0) == 1) { g.b_mn = 0; g.ldb = b.stride(1); }
  else { TORCH_CHECK(b.stride(1) == 1, "b200.gemm: b must be row-major or a transposed view"); g.b_mn = 1; g.ldb = b.stride(0); }
  TORCH_CHECK(!(g.a_mn && !g.b_mn), "b200.gemm: transposed a needs row-major b");
  TORCH_CHECK(g.lda % 8 == 0 && g.ldb % 8 == 0, "b200.gemm: strides % 8");
  g.a = a.data_ptr();
  g.b = b.data_ptr();
  g.c = out.data_ptr();
  g.ldc = out.stride(0);
  g.MA = M;
  g.NB = N;
  g.K = K;
  g.out_f32 = out.scalar_type() == at::kFloat;
  TORCH_CHECK(g.out_f32 || out.scalar_type() == at::kBFloat16, "b200.gemm: out dtype");
  TORCH_CHECK(!accumulate || g.out_f32, "b200.gemm: accumulate needs f32 out");
  g.accumulate = accumulate;
  g.alpha = (float)alpha;
  g.residual = opt_ptr(residual);
  g.ldr = (residual.has_value() && residual->defined()) ? residual->stride(0) : 0;
  g.bias = opt_ptr(bias);
  g.prefetch_b = prefetch_b;
  g.ws = ws.data_ptr<float>();
  g.ws_elems = ws.numel();
  g.sem = sem.data_ptr<int>();
  g.sem_elems = sem.numel();
  g.status = status.data_ptr<int>();
  g.device = a.get_device();
  c10::cuda::CUDAGuard gd(a.device());
  b200::gemm_launch(g, cur_stream(a));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void adamw(Tensor& master, const Tensor& grad, Tensor& m, Tensor& v, const optional<Tensor>& param_out, double lr,
           double b1, double b2, double eps, double wd, int64_t step, const optional<Tensor>& scale_t,
           double scale) {
  check_cuda(master, "master");
  const int64_t n = master.numel();
  TORCH_CHECK(master.scalar_type() == at::kFloat && m.scalar_type() == at::kFloat && v.scalar_type() == at::kFloat &&
                  master.is_contiguous() && m.is_contiguous() && v.is_contiguous() && grad.is_contiguous() &&
                  m.numel() == n && v.numel() == n && grad.numel() == n,
              "b200.adamw: fp32 contiguous master/moments, matching grad");
  TORCH_CHECK(grad.scalar_type() == at::kFloat || grad.scalar_type() == at::kBFloat16, "b200.adamw: grad dtype");
  if (param_out.has_value() && param_out->defined())
    TORCH_CHECK(param_out->scalar_type() == at::kBFloat16 && param_out->numel() == n && param_out->is_contiguous(),
                "b200.adamw: param_out");
  c10::cuda::CUDAGuard g(master.device());
  b200::adamw_launch(master.data_ptr<float>(), grad.data_ptr(), grad.scalar_type() == at::kFloat,
                     m.data_ptr<float>(), v.data_ptr<float>(), const_cast<void*>(opt_ptr(param_out)), n, (float)lr,
                     (float)b1, (float)b2, (float)eps, (float)wd, step,
                     (scale_t.has_value() && scale_t->defined()) ? scale_t->data_ptr<float>() : nullptr,
                     (float)scale, cur_stream(master));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void sumsq(const Tensor& g, Tensor& out) {
  check_cuda(g, "g");
  TORCH_CHECK(g.is_contiguous() && (g.scalar_type() == at::kFloat || g.scalar_type() == at::kBFloat16) &&
                  out.scalar_type() == at::kFloat,
              "b200.sumsq");
  c10::cuda::CUDAGuard gd(g.device());
  b200::sumsq_launch(g.data_ptr(), g.scalar_type() == at::kFloat, g.numel(), out.data_ptr<float>(), cur_stream(g));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void ce_fwd_bwd(const Tensor& logits, const Tensor& targets, Tensor& loss, const optional<Tensor>& dlogits,
                double grad_scale) {
  check_cuda(logits, "logits");
  TORCH_CHECK(logits.scalar_type() == at::kFloat && logits.dim() == 2 && logits.stride(1) == 1, "b200.ce: logits");
  TORCH_CHECK(targets.scalar_type() == at::kLong && targets.numel() == logits.size(0), "b200.ce: targets int64");
  if (dlogits.has_value() && dlogits->defined())
    TORCH_CHECK(dlogits->scalar_type() == at::kBFloat16 && dlogits->stride(1) == 1 &&
                    dlogits->size(0) == logits.size(0) && dlogits->size(1) == logits.size(1),
                "b200.ce: dlogits");
  c10::cuda::CUDAGuard g(logits.device());
  b200::ce_fwd_bwd_launch(logits.data_ptr<float>(), logits.stride(0), logits.size(0), logits.size(1),
                          targets.data_ptr<int64_t>(), loss.data_ptr<float>(), const_cast<void*>(opt_ptr(dlogits)),
                          (dlogits.has_value() && dlogits->defined()) ? dlogits->stride(0) : 0, (float)grad_scale,
                          cur_stream(logits));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void os_reduce_norm(const Tensor& slots, int64_t slot_elems, Tensor& h, const Tensor& norm_w, Tensor& out,
                    const Tensor& flags, Tensor& epoch, Tensor& cta_ctr, int64_t M, int64_t world, double eps,
                    Tensor& status) {
  check_cuda(h, "h");
  TORCH_CHECK(h.scalar_type() == at::kBFloat16 && h.is_contiguous() && out.is_contiguous(), "b200.os_reduce_norm");
  c10::cuda::CUDAGuard g(h.device());
  b200::OsReduceArgs a{};
  a.slots = slots.data_ptr();
  a.slot_elems = slot_elems;
  a.h = h.data_ptr();
  a.norm_w = norm_w.data_ptr();
  a.out = out.data_ptr();
  a.flags = reinterpret_cast<const unsigned*>(flags.data_ptr<int>());
  a.epoch = reinterpret_cast<unsigned*>(epoch.data_ptr<int>());
  a.cta_ctr = reinterpret_cast<unsigned*>(cta_ctr.data_ptr<int>());
  a.M = (int)M;
  a.H = (int)h.size(1);
  a.world = (int)world;
  a.eps = (float)eps;
  a.status = status.data_ptr<int>();
  b200::os_reduce_norm_launch(a, cur_stream(h));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void moe_route(const Tensor& logits, int64_t k, bool softmax_first, bool renorm, Tensor& experts, Tensor& weights) {
  check_cuda(logits, "logits");
  TORCH_CHECK(logits.scalar_type() == at::kFloat && logits.stride(1) == 1, "b200.moe_route: f32 logits");
  c10::cuda::CUDAGuard g(logits.device());
  b200::moe_route_launch(logits.data_ptr<float>(), logits.stride(0), (int)logits.size(0), (int)logits.size(1),
                         (int)k, softmax_first, renorm, experts.data_ptr<int32_t>(), weights.data_ptr<float>(),
                         cur_stream(logits));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void moe_align(const Tensor& experts, int64_t E, int64_t e_lo, int64_t e_cnt, int64_t bt, Tensor& meta,
               Tensor& tiles, Tensor& perm, Tensor& inv, Tensor& cursor) {
  check_cuda(experts, "experts");
  TORCH_CHECK(meta.numel() >= 2 * E + 2 && cursor.numel() >= E, "b200.moe_align: buffers");
  c10::cuda::CUDAGuard g(experts.device());
  TORCH_CHECK(bt >= 1 && tiles.numel() >= 4 * (experts.numel() / bt + E + 1), "b200.moe_align: tile list too small");
  b200::moe_align_launch(experts.data_ptr<int32_t>(), (int)experts.numel(), (int)E, (int)e_lo, (int)e_cnt, (int)bt,
                         meta.data_ptr<int32_t>(), tiles.data_ptr<int32_t>(), (int)(tiles.numel() / 4),
                         perm.data_ptr<int32_t>(), inv.data_ptr<int32_t>(), cursor.data_ptr<int32_t>(),
                         cur_stream(experts));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void moe_gather(const Tensor& x, const Tensor& perm, const Tensor& meta, int64_t E, int64_t k, Tensor& out) {
  check_cuda(x, "x");
  TORCH_CHECK(x.is_contiguous() && out.is_contiguous() && x.size(1) % 8 == 0, "b200.moe_gather");
  c10::cuda::CUDAGuard g(x.device());
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 &&
                  (out.scalar_type() == at::kBFloat16 || out.scalar_type() == at::kHalf),
              "b200.moe_gather: bf16 -> bf16/f16");
  b200::moe_gather_launch(x.data_ptr(), x.size(1), perm.data_ptr<int32_t>(), meta.data_ptr<int32_t>(), (int)E,
                          (int)k, (int)out.size(0), out.data_ptr(), out.scalar_type() == at::kHalf, cur_stream(x));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void moe_combine(const Tensor& rows, const Tensor& inv, int64_t k, Tensor& out, bool accumulate) {
  check_cuda(rows, "rows");
  TORCH_CHECK(out.is_contiguous() && rows.is_contiguous() && out.size(1) % 8 == 0, "b200.moe_combine");
  c10::cuda::CUDAGuard g(rows.device());
  b200::moe_combine_launch(rows.data_ptr(), inv.data_ptr<int32_t>(), (int)out.size(0), (int)k, out.size(1),
                           out.data_ptr(), accumulate, cur_stream(rows));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// w, row_exp: tiled MXFP4 weights [E, ceil(N/128), K/64, 4352] and per-row exponents [E, ceil(N/128)*128]
// (quant.mxfp4.tile_mxfp4); N: logical weight rows. x f16; out f16 (gate/up) or bf16 (down).
void moe_gemm(const Tensor& x, const Tensor& w, const Tensor& row_exp, int64_t N, const optional<Tensor>& bias,
              const optional<Tensor>& row_weight, const Tensor& perm, const Tensor& meta, const Tensor& tiles,
              Tensor& out, bool swiglu, double limit, double alpha, int64_t bt, Tensor& status,
              double up_offset) {
  check_cuda(x, "x");
  TORCH_CHECK(x.scalar_type() == at::kHalf && x.is_contiguous(), "b200.moe_gemm: x must be f16");
  TORCH_CHECK(out.scalar_type() == (swiglu ? at::kHalf : at::kBFloat16), "b200.moe_gemm: out f16 (gate/up) / bf16");
  TORCH_CHECK(w.scalar_type() == at::kByte && w.is_contiguous() && w.dim() == 4 && w.size(3) == 4352,
              "b200.moe_gemm: tiled uint8 weights [E, NT, KT, 4352]");
  const int64_t E = w.size(0);
  const int64_t K = w.size(2) * 64;
  TORCH_CHECK(w.size(1) == (N + 127) / 128, "b200.moe_gemm: weight n-tiles do not match N");
  TORCH_CHECK(row_exp.scalar_type() == at::kByte && row_exp.numel() == E * w.size(1) * 128, "b200.moe_gemm: row_exp");
  TORCH_CHECK(x.size(1) == K, "b200.moe_gemm: K mismatch");
  TORCH_CHECK(out.is_contiguous() && out.size(1) == (swiglu ? N / 2 : N), "b200.moe_gemm: out");
  TORCH_CHECK(!bias.has_value() || !bias->defined() || bias->numel() == E * N, "b200.moe_gemm: bias [E, N]");
  c10::cuda::CUDAGuard g(x.device());
  b200::MoeGemmArgs a{};
  a.x = x.data_ptr();
  a.rows = x.size(0);
  a.w = w.data_ptr();
  a.row_exp = row_exp.data_ptr();
  a.bias = opt_ptr(bias);
  a.row_weight = (row_weight.has_value() && row_weight->defined()) ? row_weight->data_ptr<float>() : nullptr;
  a.perm = perm.data_ptr<int32_t>();
  a.meta = meta.data_ptr<int32_t>();
  a.tiles = tiles.data_ptr<int32_t>();
  a.out = out.data_ptr();
  a.E = (int)E;
  a.N = (int)N;
  a.K = (int)K;
  a.bt = (int)bt;
  a.max_tiles = (int)(tiles.numel() / 4);
  a.swiglu = swiglu;
  a.limit = (float)limit;
  a.alpha = (float)alpha;
  a.up_offset = (float)up_offset;
  a.status = status.data_ptr<int>();
  a.device = x.get_device();
  b200::moe_gemm_launch(a, cur_stream(x));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// x [rows, H] (row stride), mod [B, *] bf16: out = LN(x) * (1 + mod[b][scale_off:]) + mod[b][shift_off:]
void ln_modulate(const Tensor& x, Tensor& out, const Tensor& mod, int64_t shift_off, int64_t scale_off, double eps,
                 int64_t split, int64_t r1, int64_t r2, int64_t row_off) {
  check_cuda(x, "x");
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && out.scalar_type() == at::kBFloat16 &&
                  mod.scalar_type() == at::kBFloat16 && x.dim() == 2 && x.stride(1) == 1 && out.stride(1) == 1 &&
                  mod.stride(1) == 1,
              "b200.ln_modulate: bf16, unit inner stride");
  const int64_t H = x.size(1);
  TORCH_CHECK(out.size(0) == x.size(0) && out.size(1) == H && x.stride(0) % 8 == 0 && out.stride(0) % 8 == 0 &&
                  mod.stride(0) % 8 == 0 && shift_off % 8 == 0 && scale_off % 8 == 0 &&
                  shift_off + H <= mod.size(1) && scale_off + H <= mod.size(1),
              "b200.ln_modulate: shapes / 16-byte alignment");
  c10::cuda::CUDAGuard g(x.device());
  b200::ln_modulate_launch(x.data_ptr(), x.stride(0), out.data_ptr(), out.stride(0), mod.data_ptr(), mod.stride(0),
                           (int)shift_off, (int)scale_off, (int)x.size(0), (int)H, (float)eps, (int)split, (int)r1,
                           (int)r2, (int)row_off, cur_stream(x));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// qkv [rows, 3 H] (row stride) -> q [rows, heads, 128], k/v pages [rows/16, heads, 16, 128]
void dit_qk_rope(const Tensor& qkv, int64_t heads, const Tensor& scales_txt, const Tensor& scales_img,
                 const Tensor& cos_t, const Tensor& sin_t, int64_t split, int64_t Lt, int64_t Li, double eps,
                 Tensor& q_out, Tensor& k_pages, Tensor& v_pages, int64_t row_off, int64_t kv_groups) {
  check_cuda(qkv, "qkv");
  const int64_t rows = qkv.size(0);
  TORCH_CHECK(qkv.scalar_type() == at::kBFloat16 && qkv.stride(1) == 1 && qkv.size(1) >= 3 * heads * 128 &&
                  qkv.stride(0) % 4 == 0,
              "b200.dit_qk_rope: qkv [rows, 3 * heads * 128]");
  TORCH_CHECK((rows % 16 == 0 || kv_groups > 0) && (kv_groups == 0 || heads % kv_groups == 0) && q_out.is_contiguous() && k_pages.is_contiguous() && v_pages.is_contiguous() &&
                  q_out.numel() == rows * heads * 128 && k_pages.numel() == rows * heads * 128 &&
                  v_pages.numel() == rows * heads * 128,
              "b200.dit_qk_rope: outputs");
  TORCH_CHECK(cos_t.scalar_type() == at::kFloat && sin_t.scalar_type() == at::kFloat && cos_t.is_contiguous() &&
                  sin_t.is_contiguous() && cos_t.size(1) == 64 && cos_t.size(0) >= Lt + Li,
              "b200.dit_qk_rope: f32 tables [Lt + Li, 64]");
  TORCH_CHECK(scales_txt.numel() == 256 && scales_img.numel() == 256 && scales_txt.scalar_type() == at::kBFloat16 &&
                  scales_img.scalar_type() == at::kBFloat16,
              "b200.dit_qk_rope: scales [2, 128] bf16 (q, k)");
  c10::cuda::CUDAGuard g(qkv.device());
  b200::dit_qk_rope_launch(qkv.data_ptr(), qkv.stride(0), (int)rows, (int)heads, scales_txt.data_ptr(),
                           scales_img.data_ptr(), cos_t.data_ptr<float>(), sin_t.data_ptr<float>(), (int)split,
                           (int)Lt, (int)Li, (float)eps, q_out.data_ptr(), k_pages.data_ptr(), v_pages.data_ptr(),
                           (int)row_off, (int)kv_groups, cur_stream(qkv));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void flag_wait_probe(const Tensor& flag, int64_t target, Tensor& status, Tensor& ok) {
  check_cuda(flag, "flag");
  TORCH_CHECK(flag.scalar_type() == at::kInt && ok.scalar_type() == at::kInt, "b200.flag_wait_probe: int32");
  c10::cuda::CUDAGuard g(flag.device());
  b200::flag_wait_probe_launch(reinterpret_cast<const unsigned*>(flag.data_ptr<int32_t>()), (unsigned)target,
                               status.data_ptr<int>(), ok.data_ptr<int32_t>(), cur_stream(flag));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// -- training elementwise kernels (train/train_fused.cu) ---------------------
static void check_bf16_contig(const Tensor& t, const char* what) {
  check_cuda(t, what);
  TORCH_CHECK(t.scalar_type() == at::kBFloat16 && t.is_contiguous(), "b200: ", what, " must be contiguous bf16");
}

void rmsnorm_train_fwd(const Tensor& x, const Tensor& w, Tensor& y, Tensor& rstd, double eps) {
  check_bf16_contig(x, "x");
  check_bf16_contig(w, "w");
  const int64_t H = x.size(-1), rows = x.numel() / H;
  TORCH_CHECK(y.numel() == x.numel() && y.is_contiguous() && rstd.scalar_type() == at::kFloat && rstd.numel() >= rows,
              "b200.rmsnorm_train_fwd: outputs");
  c10::cuda::CUDAGuard g(x.device());
  b200::rmsnorm_train_fwd_launch(x.data_ptr(), w.data_ptr(), y.data_ptr(), rstd.data_ptr<float>(), (int)rows, (int)H,
                                 (float)eps, x.get_device(), cur_stream(x));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void rmsnorm_train_bwd(const Tensor& dy, const Tensor& x, const Tensor& w, const Tensor& rstd, Tensor& dx,
                       Tensor& dw) {
  check_bf16_contig(dy, "dy");
  check_bf16_contig(x, "x");
  check_bf16_contig(w, "w");
  const int64_t H = x.size(-1), rows = x.numel() / H;
  TORCH_CHECK(dw.scalar_type() == at::kFloat && dw.numel() == H && dx.numel() == x.numel() && dx.is_contiguous() &&
                  dy.numel() == x.numel(),
              "b200.rmsnorm_train_bwd: fp32 dw [H], dx like x");
  c10::cuda::CUDAGuard g(x.device());
  b200::rmsnorm_train_bwd_launch(dy.data_ptr(), x.data_ptr(), w.data_ptr(), rstd.data_ptr<float>(), dx.data_ptr(),
                                 dw.data_ptr<float>(), (int)rows, (int)H, x.get_device(), cur_stream(x));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

static b200::QKNormRopeArgs qknr_args(const Tensor& qkv, const optional<Tensor>& qn, const optional<Tensor>& kn,
                                      const Tensor& cos, const Tensor& sin, int64_t S, int64_t Hq, int64_t Hkv,
                                      double eps) {
  check_bf16_contig(qkv, "qkv");
  TORCH_CHECK(cos.scalar_type() == at::kBFloat16 && sin.scalar_type() == at::kBFloat16 && cos.size(-1) == 128 &&
                  cos.is_contiguous() && sin.is_contiguous() && cos.size(0) >= S,
              "b200.qk_norm_rope: bf16 [S, 128] tables");
  TORCH_CHECK(qkv.size(-1) == (Hq + 2 * Hkv) * 128, "b200.qk_norm_rope: qkv width");
  b200::QKNormRopeArgs a{};
  a.qkv = qkv.data_ptr();
  a.q_norm = opt_ptr(qn);
  a.k_norm = opt_ptr(kn);
  a.cos = cos.data_ptr();
  a.sin = sin.data_ptr();
  a.positions = nullptr;
  a.D = 128;
  a.Hq = (int)Hq;
  a.Hkv = (int)Hkv;
  a.T = (int)(qkv.numel() / ((Hq + 2 * Hkv) * 128));
  a.S = (int)S;
  a.eps = (float)eps;
  return a;
}

void qk_norm_rope_fwd(const Tensor& qkv, const optional<Tensor>& qn, const optional<Tensor>& kn, const Tensor& cos,
                      const Tensor& sin, int64_t S, int64_t Hq, int64_t Hkv, double eps, Tensor& q, Tensor& k,
                      Tensor& v, Tensor& rstd_q, Tensor& rstd_k) {
  auto a = qknr_args(qkv, qn, kn, cos, sin, S, Hq, Hkv, eps);
  TORCH_CHECK(q.is_contiguous() && k.is_contiguous() && v.is_contiguous() && q.numel() == (int64_t)a.T * Hq * 128 &&
                  k.numel() == (int64_t)a.T * Hkv * 128 && v.numel() == k.numel() && rstd_q.numel() >= a.T * Hq &&
                  rstd_k.numel() >= a.T * Hkv,
              "b200.qk_norm_rope_fwd: outputs");
  a.q = q.data_ptr();
  a.k = k.data_ptr();
  a.v = v.data_ptr();
  a.rstd_q = rstd_q.data_ptr<float>();
  a.rstd_k = rstd_k.data_ptr<float>();
  c10::cuda::CUDAGuard g(qkv.device());
  b200::qk_norm_rope_fwd_launch(a, qkv.get_device(), cur_stream(qkv));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void qk_norm_rope_bwd(const Tensor& qkv, const optional<Tensor>& qn, const optional<Tensor>& kn, const Tensor& cos,
                      const Tensor& sin, int64_t S, int64_t Hq, int64_t Hkv, const Tensor& rstd_q,
                      const Tensor& rstd_k, const Tensor& dq, const Tensor& dk, const Tensor& dv, Tensor& dqkv,
                      const optional<Tensor>& dw_q, const optional<Tensor>& dw_k) {
  auto a = qknr_args(qkv, qn, kn, cos, sin, S, Hq, Hkv, 1e-6);
  TORCH_CHECK(dq.is_contiguous() && dk.is_contiguous() && dv.is_contiguous() && dqkv.is_contiguous() &&
                  dqkv.numel() == qkv.numel() && dq.numel() == (int64_t)a.T * Hq * 128,
              "b200.qk_norm_rope_bwd: contiguous gradients");
  a.rstd_q = const_cast<float*>(rstd_q.data_ptr<float>());
  a.rstd_k = const_cast<float*>(rstd_k.data_ptr<float>());
  a.dq = dq.data_ptr();
  a.dk = dk.data_ptr();
  a.dv = dv.data_ptr();
  a.dqkv = dqkv.data_ptr();
  a.dw_q = dw_q.has_value() && dw_q->defined() ? dw_q->data_ptr<float>() : nullptr;
  a.dw_k = dw_k.has_value() && dw_k->defined() ? dw_k->data_ptr<float>() : nullptr;
  c10::cuda::CUDAGuard g(qkv.device());
  b200::qk_norm_rope_bwd_launch(a, qkv.get_device(), cur_stream(qkv));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void swiglu_train_fwd(const Tensor& gu, Tensor& h) {
  check_bf16_contig(gu, "gate_up");
  const int64_t I = gu.size(-1) / 2, T = gu.numel() / gu.size(-1);
  TORCH_CHECK(h.numel() == T * I && h.is_contiguous(), "b200.swiglu_train_fwd: h");
  c10::cuda::CUDAGuard g(gu.device());
  b200::swiglu_train_fwd_launch(gu.data_ptr(), h.data_ptr(), T, (int)I, gu.get_device(), cur_stream(gu));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void swiglu_train_bwd(const Tensor& dh, const Tensor& gu, Tensor& dgu) {
  check_bf16_contig(gu, "gate_up");
  check_bf16_contig(dh, "dh");
  const int64_t I = gu.size(-1) / 2, T = gu.numel() / gu.size(-1);
  TORCH_CHECK(dgu.numel() == gu.numel() && dgu.is_contiguous() && dh.numel() == T * I,
              "b200.swiglu_train_bwd: shapes");
  c10::cuda::CUDAGuard g(gu.device());
  b200::swiglu_train_bwd_launch(dh.data_ptr(), gu.data_ptr(), dgu.data_ptr(), T, (int)I, gu.get_device(),
                                cur_stream(gu));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Causal training attention over dense [B * S, H, D] rows: forward on the tcgen05
// kernel with the per-row log2-sum-exp2 saved, backward in train/attn_bwd.cu.
void attn_train_fwd(const Tensor& q, const Tensor& k, const Tensor& v, const Tensor& block_tables,
                    const Tensor& ctx_lens, const Tensor& cu_q, int64_t S, double scale, Tensor& out, Tensor& lse,
                    Tensor& status) {
  c10::cuda::CUDAGuard g(q.device());
  auto a = attn_args(q, k, v, block_tables, ctx_lens, out, c10::nullopt, 0, scale, status);
  TORCH_CHECK(k.dim() == 3 && lse.scalar_type() == at::kFloat && lse.numel() == q.size(0) * q.size(1),
              "b200.attn_train_fwd: dense k/v [T, Hkv, D], fp32 lse [T, Hq]");
  a.cu_q = cu_q.data_ptr<int32_t>();
  a.max_q_len = (int)S;
  a.causal = 1;
  a.q_rows = q.size(0);
  a.kv_dense = 1;
  a.kv_rows = k.size(0);
  a.lse = lse.data_ptr<float>();
  TORCH_CHECK(b200::fmha_supported(a), "b200.attn_train_fwd: needs the tcgen05 attention (head_dim 128, G <= 8)");
  b200::prefill_attention_launch(a, cur_stream(q));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void attn_train_bwd(const Tensor& q, const Tensor& k, const Tensor& v, const Tensor& o, const Tensor& dout,
                    const Tensor& lse, Tensor& delta, Tensor& dq_acc, Tensor& dq, Tensor& dk, Tensor& dv, int64_t B,
                    int64_t S, double scale) {
  for (const Tensor* t : std::initializer_list<const Tensor*>{&q, &k, &v, &o, &dout, &dq, &dk, &dv})
    check_bf16_contig(*t, "attention tensor");
  TORCH_CHECK(q.dim() == 3 && q.size(2) == 128 && k.size(2) == 128 && q.size(0) == B * S && k.size(0) == B * S &&
                  o.sizes() == q.sizes() && dout.sizes() == q.sizes() && dq.sizes() == q.sizes() &&
                  dk.sizes() == k.sizes() && dv.sizes() == k.sizes(),
              "b200.attn_train_bwd: shapes");
  TORCH_CHECK(lse.numel() == q.size(0) * q.size(1) && delta.numel() == lse.numel() &&
                  dq_acc.numel() == q.numel() && dq_acc.scalar_type() == at::kFloat,
              "b200.attn_train_bwd: fp32 lse / delta / dq accumulator");
  c10::cuda::CUDAGuard g(q.device());
  b200::AttnBwdArgs a{};
  a.q = q.data_ptr();
  a.k = k.data_ptr();
  a.v = v.data_ptr();
  a.o = o.data_ptr();
  a.dout = dout.data_ptr();
  a.lse = lse.data_ptr<float>();
  a.delta = delta.data_ptr<float>();
  a.dq_acc = dq_acc.data_ptr<float>();
  a.dq = dq.data_ptr();
  a.dk = dk.data_ptr();
  a.dv = dv.data_ptr();
  a.B = (int)B;
  a.S = (int)S;
  a.Hq = (int)q.size(1);
  a.Hkv = (int)k.size(1);
  a.scale = (float)scale;
  b200::attn_bwd_launch(a, q.get_device(), cur_stream(q));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void instance_norm(const Tensor& x, const optional<Tensor>& gamma, const optional<Tensor>& beta, Tensor& y,
                   int64_t active, double eps) {
  check_cuda(x, "x");
  TORCH_CHECK(x.dim() == 3 && x.is_contiguous() && y.is_contiguous() && y.sizes() == x.sizes() &&
                  y.scalar_type() == x.scalar_type() &&
                  (x.scalar_type() == at::kFloat || x.scalar_type() == at::kBFloat16),
              "b200.instance_norm: contiguous fp32 / bf16 [N, C, T]");
  for (const optional<Tensor>* t : {&gamma, &beta})
    if (t->has_value() && (*t)->defined())
      TORCH_CHECK((*t)->scalar_type() == at::kFloat && (*t)->numel() == x.size(1), "b200.instance_norm: fp32 [C]");
  c10::cuda::CUDAGuard g(x.device());
  b200::instance_norm_launch(x.data_ptr(), static_cast<const float*>(opt_ptr(gamma)),
                             static_cast<const float*>(opt_ptr(beta)), y.data_ptr(), x.size(0), (int)x.size(1),
                             x.size(2), active, (float)eps, x.scalar_type() == at::kBFloat16, cur_stream(x));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void act_im2col(const Tensor& x, const optional<Tensor>& alpha, Tensor& cols, int64_t k, int64_t stride, int64_t pad_l,
                int64_t pad_r, int64_t dil, int64_t act, bool reflect) {
  check_cuda(x, "x");
  TORCH_CHECK(x.dim() == 3 && x.is_contiguous() && x.scalar_type() == at::kBFloat16,
              "b200.act_im2col: contiguous bf16 x [B, T, C]");
  const int64_t B = x.size(0), T = x.size(1), C = x.size(2);
  TORCH_CHECK(k >= 1 && stride >= 1 && dil >= 1 && pad_l >= 0 && pad_r >= 0 && act >= 0 && act <= 3,
              "b200.act_im2col: bad geometry");
  TORCH_CHECK(!reflect || (pad_l < T && pad_r < T), "b200.act_im2col: reflection needs padding < T");
  const int64_t T_out = (T + pad_l + pad_r - dil * (k - 1) - 1) / stride + 1;
  const int64_t Kp = (k * C + 7) / 8 * 8;
  TORCH_CHECK(T_out >= 1 && cols.is_contiguous() && cols.scalar_type() == at::kBFloat16 && cols.dim() == 2 &&
                  cols.size(0) == B * T_out && cols.size(1) == Kp,
              "b200.act_im2col: cols must be contiguous bf16 [B * T_out, round_up(k * C, 8)]");
  TORCH_CHECK(B * T <= INT32_MAX && B * T_out <= INT32_MAX && Kp <= INT32_MAX, "b200.act_im2col: too large");
  TORCH_CHECK(act != 1 || (alpha.has_value() && alpha->defined()), "b200.act_im2col: snake needs alpha");
  if (alpha.has_value() && alpha->defined())
    TORCH_CHECK(alpha->scalar_type() == at::kFloat && alpha->is_contiguous() && alpha->numel() == C &&
                    alpha->device() == x.device(),
                "b200.act_im2col: alpha fp32 [C] on the device of x");
  c10::cuda::CUDAGuard g(x.device());
  b200::act_im2col_launch(x.data_ptr(), static_cast<const float*>(opt_ptr(alpha)), cols.data_ptr(), (int)B, (int)T,
                          (int)T_out, (int)C, (int)Kp, (int)k, (int)stride, (int)pad_l, (int)dil, (int)act, reflect,
                          cur_stream(x));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void convt_fold(const Tensor& Y, const optional<Tensor>& bias, Tensor& y, int64_t stride, int64_t pad_l, int64_t pad_r) {
  check_cuda(Y, "Y");
  TORCH_CHECK(Y.dim() == 3 && Y.is_contiguous() && Y.scalar_type() == at::kFloat,
              "b200.convt_fold: contiguous fp32 Y [B, T_in, k * C_out]");
  TORCH_CHECK(y.dim() == 3 && y.is_contiguous() && y.scalar_type() == at::kBFloat16 && y.size(0) == Y.size(0),
              "b200.convt_fold: contiguous bf16 y [B, T_out, C_out]");
  const int64_t C_out = y.size(2);
  TORCH_CHECK(stride >= 1 && pad_l >= 0 && pad_r >= 0 && C_out > 0 && Y.size(2) % (stride * C_out) == 0,
              "b200.convt_fold: kernel size must be a multiple of the stride");
  const int64_t m = Y.size(2) / (stride * C_out);
  TORCH_CHECK(y.size(1) == (Y.size(1) - 1) * stride + m * stride - pad_l - pad_r, "b200.convt_fold: T_out mismatch");
  if (bias.has_value() && bias->defined())
    TORCH_CHECK(bias->scalar_type() == at::kFloat && bias->is_contiguous() && bias->numel() == C_out &&
                    bias->device() == Y.device(),
                "b200.convt_fold: bias fp32 [C_out] on the device of Y");
  c10::cuda::CUDAGuard g(Y.device());
  b200::convt_fold_launch(Y.data_ptr<float>(), static_cast<const float*>(opt_ptr(bias)), y.data_ptr(),
                          (int)Y.size(0), (int)Y.size(1), (int)y.size(1), (int)C_out, (int)stride, (int)m, (int)pad_l,
                          cur_stream(Y));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void lstm_cell(const Tensor& G, Tensor& c, Tensor& h, Tensor& y) {
  check_cuda(G, "G");
  TORCH_CHECK(G.dim() == 2 && G.is_contiguous() && G.scalar_type() == at::kFloat && G.size(1) % 4 == 0,
              "b200.lstm_cell: contiguous fp32 G [B, 4H]");
  const int64_t B = G.size(0), H = G.size(1) / 4;
  TORCH_CHECK(c.is_contiguous() && c.scalar_type() == at::kFloat && c.numel() == B * H && c.device() == G.device(),
              "b200.lstm_cell: fp32 c [B, H]");
  for (const Tensor* t : {&h, &y})
    TORCH_CHECK(t->is_contiguous() && t->scalar_type() == at::kBFloat16 && t->numel() == B * H &&
                    t->device() == G.device(),
                "b200.lstm_cell: bf16 h / y [B, H]");
  c10::cuda::CUDAGuard g(G.device());
  b200::lstm_cell_launch(G.data_ptr<float>(), c.data_ptr<float>(), h.data_ptr(), y.data_ptr(), (int)B, (int)H,
                         cur_stream(G));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void scale_by(Tensor& t, const Tensor& g) {
  check_cuda(t, "t");
  TORCH_CHECK(t.is_contiguous() && (t.scalar_type() == at::kFloat || t.scalar_type() == at::kBFloat16) &&
                  g.scalar_type() == at::kFloat && g.numel() == 1 && g.is_cuda(),
              "b200.scale_by: contiguous fp32/bf16 tensor, fp32 device scalar");
  c10::cuda::CUDAGuard gd(t.device());
  b200::scale_by_launch(t.data_ptr(), t.scalar_type() == at::kFloat, t.numel(), g.data_ptr<float>(), t.get_device(),
                        cur_stream(t));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void tp_argmax(const Tensor& logits, int64_t v_offset, Tensor& own_pairs, const Tensor& peer_pairs, Tensor& epoch,
               Tensor& cta_ctr, Tensor& out, int64_t max_rows, int64_t rank, int64_t world, Tensor& status) {
  check_cuda(logits, "logits");
  TORCH_CHECK(logits.scalar_type() == at::kFloat && logits.dim() == 2 && logits.stride(1) == 1,
              "b200.tp_argmax: fp32 [R, V/world] logits");
  TORCH_CHECK(out.scalar_type() == at::kInt && out.numel() >= logits.size(0), "b200.tp_argmax: out");
  TORCH_CHECK(peer_pairs.scalar_type() == at::kLong && peer_pairs.numel() == world && cta_ctr.numel() >= 1 &&
                  own_pairs.numel() >= 2 * max_rows * world,
              "b200.tp_argmax: key buffers / peer table / counter");
  c10::cuda::CUDAGuard g(logits.device());
  b200::TpArgmaxArgs a{};
  a.logits = logits.data_ptr<float>();
  a.ld = logits.stride(0);
  a.V_local = (int)logits.size(1);
  a.v_offset = (int)v_offset;
  a.own_pairs = reinterpret_cast<unsigned long long*>(own_pairs.data_ptr());
  a.peer_pairs = reinterpret_cast<unsigned long long* const*>(peer_pairs.data_ptr<int64_t>());
  a.epoch = reinterpret_cast<unsigned*>(epoch.data_ptr<int32_t>());
  a.cta_ctr = reinterpret_cast<unsigned*>(cta_ctr.data_ptr<int32_t>());
  a.out = out.data_ptr<int32_t>();
  a.R = (int)logits.size(0);
  a.max_rows = (int)max_rows;
  a.world = (int)world;
  a.rank = (int)rank;
  a.status = status.data_ptr<int>();
  b200::tp_argmax_launch(a, cur_stream(logits));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void ar2_norm(const Tensor& peer_acc, const Tensor& peer_res, Tensor& own_res, const Tensor& peer_flags,
              const Tensor& flags, Tensor& zero_buf, int64_t zero_rows, Tensor& h, const Tensor& norm_w, Tensor& out,
              Tensor& epoch, Tensor& cta_ctr, int64_t rank, int64_t world, int64_t rpr, int64_t rpr_max, double eps,
              Tensor& status) {
  check_cuda(h, "h");
  TORCH_CHECK(peer_acc.scalar_type() == at::kLong && peer_acc.numel() == world && peer_res.numel() == world &&
                  peer_flags.numel() == world && flags.numel() >= 2 * world && cta_ctr.numel() >= 2,
              "b200.ar2_norm: peer tables");
  TORCH_CHECK(h.scalar_type() == at::kBFloat16 && h.is_contiguous() && out.is_contiguous() &&
                  zero_buf.scalar_type() == at::kFloat && zero_buf.size(0) >= zero_rows &&
                  own_res.numel() >= 2 * rpr_max * h.size(1),
              "b200.ar2_norm: buffers");
  c10::cuda::CUDAGuard g(h.device());
  b200::TwoShotNormArgs a{};
  a.peer_acc = reinterpret_cast<const float* const*>(peer_acc.data_ptr<int64_t>());
  a.peer_res = reinterpret_cast<const void* const*>(peer_res.data_ptr<int64_t>());
  a.own_res = own_res.data_ptr();
  a.peer_flags = reinterpret_cast<unsigned* const*>(peer_flags.data_ptr<int64_t>());
  a.flags = reinterpret_cast<const unsigned*>(flags.data_ptr<int32_t>());
  a.zero_buf = zero_buf.data_ptr<float>();
  a.zero_rows = (int)zero_rows;
  a.h = h.data_ptr();
  a.norm_w = norm_w.data_ptr();
  a.out = out.data_ptr();
  a.epoch = reinterpret_cast<unsigned*>(epoch.data_ptr<int32_t>());
  a.cta_ctr = reinterpret_cast<unsigned*>(cta_ctr.data_ptr<int32_t>());
  a.M = (int)h.size(0);
  a.H = (int)h.size(1);
  a.world = (int)world;
  a.rank = (int)rank;
  a.rpr = (int)rpr;
  a.rpr_max = (int)rpr_max;
  a.eps = (float)eps;
  a.status = status.data_ptr<int>();
  b200::ar2_norm_launch(a, cur_stream(h));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void ar_pull_norm(const Tensor& peer_acc, const Tensor& peer_flags, const Tensor& flags, Tensor& zero_buf,
                  int64_t zero_rows, Tensor& h, const Tensor& norm_w, Tensor& out, Tensor& epoch, Tensor& cta_ctr,
                  int64_t rank, int64_t world, double eps, Tensor& status) {
  check_cuda(h, "h");
  TORCH_CHECK(peer_acc.scalar_type() == at::kLong && peer_acc.numel() == world && peer_flags.numel() == world,
              "b200.ar_pull_norm: peer tables");
  TORCH_CHECK(h.scalar_type() == at::kBFloat16 && h.is_contiguous() && out.is_contiguous() &&
                  zero_buf.scalar_type() == at::kFloat && zero_buf.size(0) >= zero_rows,
              "b200.ar_pull_norm: buffers");
  c10::cuda::CUDAGuard g(h.device());
  b200::PullNormArgs a{};
  a.peer_acc = reinterpret_cast<const float* const*>(peer_acc.data_ptr<int64_t>());
  a.peer_flags = reinterpret_cast<unsigned* const*>(peer_flags.data_ptr<int64_t>());
  a.flags = reinterpret_cast<const unsigned*>(flags.data_ptr<int32_t>());
  a.zero_buf = zero_buf.data_ptr<float>();
  a.zero_rows = (int)zero_rows;
  a.h = h.data_ptr();
  a.norm_w = norm_w.data_ptr();
  a.out = out.data_ptr();
  a.epoch = reinterpret_cast<unsigned*>(epoch.data_ptr<int32_t>());
  a.cta_ctr = reinterpret_cast<unsigned*>(cta_ctr.data_ptr<int32_t>());
  a.M = (int)h.size(0);
  a.H = (int)h.size(1);
  a.world = (int)world;
  a.rank = (int)rank;
  a.eps = (float)eps;
  a.status = status.data_ptr<int>();
  b200::ar_pull_norm_launch(a, cur_stream(h));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void ep_combine_norm(const Tensor& peer_rows, const Tensor& peer_inv, const Tensor& peer_flags, const Tensor& flags,
                     const Tensor& experts, int64_t e_local, Tensor& h, const Tensor& norm_w, Tensor& out,
                     Tensor& epoch, Tensor& cta_ctr, int64_t rank, int64_t world, double eps, Tensor& status) {
  check_cuda(h, "h");
  TORCH_CHECK(peer_rows.scalar_type() == at::kLong && peer_rows.numel() == world && peer_inv.numel() == world &&
                  peer_flags.numel() == world && flags.numel() >= world,
              "b200.ep_combine_norm: peer tables");
  TORCH_CHECK(h.scalar_type() == at::kBFloat16 && h.is_contiguous() && out.is_contiguous() &&
                  out.sizes() == h.sizes() && norm_w.numel() == h.size(1),
              "b200.ep_combine_norm: h / out / norm_w");
  TORCH_CHECK(experts.scalar_type() == at::kInt && experts.is_contiguous() && experts.dim() == 2 &&
                  experts.size(0) == h.size(0),
              "b200.ep_combine_norm: experts [T, k] int32");
  c10::cuda::CUDAGuard g(h.device());
  b200::EpCombineArgs a{};
  a.peer_rows = reinterpret_cast<const void* const*>(peer_rows.data_ptr<int64_t>());
  a.peer_inv = reinterpret_cast<const int32_t* const*>(peer_inv.data_ptr<int64_t>());
  a.peer_flags = reinterpret_cast<unsigned* const*>(peer_flags.data_ptr<int64_t>());
  a.flags = reinterpret_cast<const unsigned*>(flags.data_ptr<int32_t>());
  a.experts = experts.data_ptr<int32_t>();
  a.h = h.data_ptr();
  a.norm_w = norm_w.data_ptr();
  a.out = out.data_ptr();
  a.epoch = reinterpret_cast<unsigned*>(epoch.data_ptr<int32_t>());
  a.cta_ctr = reinterpret_cast<unsigned*>(cta_ctr.data_ptr<int32_t>());
  a.T = (int)h.size(0);
  a.k = (int)experts.size(1);
  a.H = (int)h.size(1);
  a.e_local = (int)e_local;
  a.world = (int)world;
  a.rank = (int)rank;
  a.eps = (float)eps;
  a.status = status.data_ptr<int>();
  b200::ep_combine_norm_launch(a, cur_stream(h));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void shard_push_add(const Tensor& src, const Tensor& peer_shards, int64_t base, int64_t shard_n, double scale) {
  check_cuda(src, "src");
  TORCH_CHECK(src.is_contiguous() && (src.scalar_type() == at::kFloat || src.scalar_type() == at::kBFloat16),
              "b200.shard_push_add: contiguous fp32 / bf16 source");
  TORCH_CHECK(peer_shards.scalar_type() == at::kLong && peer_shards.is_cuda() && base >= 0,
              "b200.shard_push_add: peer table");
  c10::cuda::CUDAGuard g(src.device());
  b200::shard_push_add_launch(src.data_ptr(), src.scalar_type() == at::kFloat, src.numel(), base,
                              reinterpret_cast<float* const*>(peer_shards.data_ptr<int64_t>()), shard_n, (float)scale,
                              cur_stream(src));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void peer_barrier(const Tensor& peer_flags, const Tensor& flags, Tensor& epoch, int64_t rank, int64_t world,
                  Tensor& status) {
  check_cuda(flags, "flags");
  TORCH_CHECK(peer_flags.scalar_type() == at::kLong && peer_flags.numel() == world && flags.numel() >= world,
              "b200.peer_barrier: tables");
  c10::cuda::CUDAGuard g(flags.device());
  b200::peer_barrier_launch(reinterpret_cast<unsigned* const*>(peer_flags.data_ptr<int64_t>()),
                            reinterpret_cast<const unsigned*>(flags.data_ptr<int32_t>()),
                            reinterpret_cast<unsigned*>(epoch.data_ptr<int32_t>()), (int)rank, (int)world,
                            status.data_ptr<int>(), cur_stream(flags));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void gguf_dequant(const Tensor& raw, int64_t ggml_type, Tensor& out) {
  check_cuda(raw, "raw");
  TORCH_CHECK(raw.scalar_type() == at::kByte && raw.is_contiguous() && out.is_contiguous() &&
                  (out.scalar_type() == at::kBFloat16 || out.scalar_type() == at::kFloat),
              "b200.gguf_dequant: contiguous uint8 blocks -> bf16 / fp32");
  c10::cuda::CUDAGuard g(raw.device());
  b200::gguf_dequant_launch(raw.data_ptr(), (int)ggml_type, out.numel(), out.data_ptr(),
                            out.scalar_type() == at::kFloat, cur_stream(raw));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void apply_penalties(Tensor& logits, const Tensor& off, const Tensor& ids, const Tensor& counts, const Tensor& rep,
                     const Tensor& freq, const Tensor& pres, const Tensor& boff, const Tensor& bias_ids,
                     const Tensor& bias_vals) {
  check_cuda(logits, "logits");
  TORCH_CHECK(logits.scalar_type() == at::kFloat && logits.dim() == 2 && logits.stride(1) == 1,
              "b200.apply_penalties: fp32 [B, V] logits with unit column stride");
  const int64_t B = logits.size(0);
  TORCH_CHECK(off.numel() == B + 1 && boff.numel() == B + 1 && rep.numel() >= B && freq.numel() >= B &&
                  pres.numel() >= B && ids.numel() == counts.numel() && bias_ids.numel() == bias_vals.numel(),
              "b200.apply_penalties: table sizes");
  TORCH_CHECK(off.scalar_type() == at::kInt && ids.scalar_type() == at::kInt && counts.scalar_type() == at::kInt &&
                  boff.scalar_type() == at::kInt && bias_ids.scalar_type() == at::kInt &&
                  rep.scalar_type() == at::kFloat && freq.scalar_type() == at::kFloat &&
                  pres.scalar_type() == at::kFloat && bias_vals.scalar_type() == at::kFloat,
              "b200.apply_penalties: dtypes");
  c10::cuda::CUDAGuard g(logits.device());
  b200::penalties_launch(logits.data_ptr<float>(), logits.stride(0), B, logits.size(1), off.data_ptr<int32_t>(),
                         ids.data_ptr<int32_t>(), counts.data_ptr<int32_t>(), rep.data_ptr<float>(),
                         freq.data_ptr<float>(), pres.data_ptr<float>(), boff.data_ptr<int32_t>(),
                         bias_ids.data_ptr<int32_t>(), bias_vals.data_ptr<float>(), cur_stream(logits));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "rlx_models_b200 sm_100a kernels";
  m.def("linear", &linear, "tcgen05 bf16 GEMM with fused epilogues", py::arg("x"), py::arg("w"), py::arg("out"), py::arg("mode"), py::arg("residual"), py::arg("bias"), py::arg("alpha"), py::arg("ws"), py::arg("sem"), py::arg("status"), py::arg("swap"), py::arg("bn"), py::arg("splits"), py::arg("trace") = py::none(),
        py::arg("act_from") = -1, py::arg("gate") = py::none(), py::arg("gate_split") = 0, py::arg("gate_r1") = 1,
        py::arg("gate_r2") = 1, py::arg("gate_off") = 0, py::arg("glu_act") = 0);
  m.def("gemm", &gemm);
  m.def("gdn_decode", &gdn_decode);
  m.def("kda_decode", &kda_decode);
  m.def("shortconv_decode", &shortconv_decode);
  m.def("ssd_decode", &ssd_decode);
  m.def("kv_select", &kv_select);
  m.def("kv_summary", &kv_summary);
  m.def("mamba_conv", &mamba_conv);
  m.def("mamba_scan", &mamba_scan);
  m.def("gemm_push_shards", &gemm_push_shards);
  m.def("shard_push_add", &shard_push_add);
  m.def("peer_barrier", &peer_barrier);
  m.def("gguf_dequant", &gguf_dequant);
  m.def("apply_penalties", &apply_penalties);
  m.def("flag_wait_probe", &flag_wait_probe);
  m.def("ar_pull_norm", &ar_pull_norm);
  m.def("ep_combine_norm", &ep_combine_norm);
  m.def("ln_modulate", &ln_modulate, py::arg("x"), py::arg("out"), py::arg("mod"), py::arg("shift_off"),
        py::arg("scale_off"), py::arg("eps"), py::arg("split"), py::arg("r1"), py::arg("r2"), py::arg("row_off") = 0);
  m.def("dit_qk_rope", &dit_qk_rope, py::arg("qkv"), py::arg("heads"), py::arg("scales_txt"), py::arg("scales_img"),
        py::arg("cos_t"), py::arg("sin_t"), py::arg("split"), py::arg("Lt"), py::arg("Li"), py::arg("eps"),
        py::arg("q_out"), py::arg("k_pages"), py::arg("v_pages"), py::arg("row_off") = 0, py::arg("kv_groups") = 0);
  m.def("moe_route", &moe_route);
  m.def("moe_align", &moe_align);
  m.def("moe_gather", &moe_gather);
  m.def("moe_combine", &moe_combine);
  m.def("moe_gemm", &moe_gemm, py::arg("x"), py::arg("w"), py::arg("row_exp"), py::arg("N"), py::arg("bias"),
        py::arg("row_weight"), py::arg("perm"), py::arg("meta"), py::arg("tiles"), py::arg("out"), py::arg("swiglu"),
        py::arg("limit"), py::arg("alpha"), py::arg("bt"), py::arg("status"), py::arg("up_offset") = 1.0);
  m.def("adamw", &adamw);
  m.def("sumsq", &sumsq);
  m.def("ce_fwd_bwd", &ce_fwd_bwd);
  m.def("embedding", &embedding);
  m.def("rmsnorm", &rmsnorm);
  m.def("qkv_rope", &qkv_rope);
  m.def("decode_attention", &decode_attention, py::arg("q"), py::arg("k_cache"), py::arg("v_cache"),
        py::arg("block_tables"), py::arg("ctx_lens"), py::arg("out"), py::arg("sinks"), py::arg("window"),
        py::arg("scale"), py::arg("splits"), py::arg("ws"), py::arg("status"), py::arg("softcap") = 0.0,
        py::arg("k_scale") = 1.0, py::arg("v_scale") = 1.0);
  m.def("prefill_attention", &prefill_attention, py::arg("q"), py::arg("k_cache"), py::arg("v_cache"),
        py::arg("block_tables"), py::arg("ctx_lens"), py::arg("cu_q"), py::arg("out"), py::arg("sinks"),
        py::arg("window"), py::arg("scale"), py::arg("max_q_len"), py::arg("status"), py::arg("causal"),
        py::arg("q_paged"), py::arg("softcap") = 0.0);
  m.def("argmax", &argmax);
  m.def("forward_tokens", &forward_tokens);
  m.def("tp_argmax", &tp_argmax);
  m.def("ar2_norm", &ar2_norm);
  m.def("rmsnorm_train_fwd", &rmsnorm_train_fwd);
  m.def("rmsnorm_train_bwd", &rmsnorm_train_bwd);
  m.def("qk_norm_rope_fwd", &qk_norm_rope_fwd);
  m.def("qk_norm_rope_bwd", &qk_norm_rope_bwd);
  m.def("swiglu_train_fwd", &swiglu_train_fwd);
  m.def("swiglu_train_bwd", &swiglu_train_bwd);
  m.def("scale_by", &scale_by);
  m.def("instance_norm", &instance_norm);
  m.def("kv_dequant_pages", &kv_dequant_pages);
  m.def("act_im2col", &act_im2col);
  m.def("lstm_cell", &lstm_cell);
  m.def("convt_fold", &convt_fold);
  m.def("attn_train_fwd", &attn_train_fwd);
  m.def("attn_train_bwd", &attn_train_bwd);
  m.def("sample", &sample);
  m.def("symm_malloc", &symm_malloc);
  m.def("symm_free", &symm_free);
  m.def("ipc_handle", &ipc_handle);
  m.def("ipc_open", &ipc_open);
  m.def("ipc_close", &ipc_close);
  m.def("tensor_from_ptr", &tensor_from_ptr);
  m.def("linear_push", &linear_push);
  m.def("rs_norm_ag", &rs_norm_ag);
  m.def("os_reduce_norm", &os_reduce_norm);
  m.def("add_rmsnorm_acc", &add_rmsnorm_acc);
  m.def("swiglu_acc", &swiglu_acc, py::arg("acc"), py::arg("out"), py::arg("act") = 0);
}
