// Python bindings of the avgen_b200 CUDA extension (module `avgen_b200._C`).
//
// The only translation unit that sees torch: it validates tensors (device,
// dtype, shape, strides, alignment) and fills the torch-free launch descriptors
// of include/launchers.h. Kernels run on torch's current CUDA stream.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "include/host_utils.h"
#include "include/launchers.h"

namespace avgen {
bool install_crash_backtrace();  // crash_trace.cpp
}

namespace avgen {
namespace {

using OptT = c10::optional<at::Tensor>;

cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream(); }

bool has(const OptT& t) { return t.has_value() && t->defined(); }

void check_cuda(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
}
void check_bf16(const at::Tensor& t, const char* name) {
  check_cuda(t, name);
  TORCH_CHECK(t.scalar_type() == at::kBFloat16, name, " must be bf16, got ", t.scalar_type());
}
void check_f32(const at::Tensor& t, const char* name) {
  check_cuda(t, name);
  TORCH_CHECK(t.scalar_type() == at::kFloat, name, " must be fp32, got ", t.scalar_type());
}
void check_rows(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.dim() == 2 && t.stride(1) == 1, name, " must be 2-D with a contiguous last dim");
  TORCH_CHECK((t.stride(0) * t.element_size()) % 16 == 0, name, " row stride must be 16-byte aligned");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0, name, " must be 16-byte aligned");
}
const float* f32_or_null(const OptT& t, const char* name) {
  if (!has(t)) return nullptr;
  check_f32(*t, name);
  TORCH_CHECK(t->is_contiguous(), name, " must be contiguous");
  return t->data_ptr<float>();
}

// Optional per-row modulation group index: contiguous int32 with one entry per row.
const int* groups_or_null(const OptT& g, long rows, const char* what) {
  if (!has(g)) return nullptr;
  TORCH_CHECK(g->scalar_type() == at::kInt && g->is_cuda() && g->is_contiguous() && g->numel() >= rows, what,
              ": groups must be a contiguous int32 device tensor with one entry per row");
  return g->data_ptr<int>();
}

// --------------------------------------------------------------------- GEMM
void gemm(const at::Tensor& a, const at::Tensor& b, at::Tensor& out, bool a_mn, bool b_mn, int64_t epilogue,
          const OptT& bias, const OptT& resid, const OptT& gate, int64_t rows_per_batch, const OptT& aux,
          int64_t k_splits, const OptT& groups, const OptT& a2, const OptT& b2, const OptT& gate_flags,
          int64_t gate_epoch, int64_t gate_operand, int64_t gate_chunk, int64_t gate_rank) {
  check_bf16(a, "a");
  check_bf16(b, "b");
  check_cuda(out, "out");
  check_rows(a, "a");
  check_rows(b, "b");
  check_rows(out, "out");
  c10::cuda::CUDAGuard guard(a.device());
  GemmDesc d;
  d.device = a.device().index();
  d.M = static_cast<int>(a_mn ? a.size(1) : a.size(0));
  d.K = static_cast<int>(a_mn ? a.size(0) : a.size(1));
  d.N = static_cast<int>(b_mn ? b.size(1) : b.size(0));
  const int kb = static_cast<int>(b_mn ? b.size(0) : b.size(1));
  TORCH_CHECK(d.K == kb, "gemm: reduction sizes differ (", d.K, " vs ", kb, ")");
  d.a = a.data_ptr();
  d.lda = a.stride(0);
  d.a_mn = a_mn;
  d.b = b.data_ptr();
  d.ldb = b.stride(0);
  d.b_mn = b_mn;
  d.out = out.data_ptr();
  d.ldo = out.stride(0);
  d.out_f32 = out.scalar_type() == at::kFloat;
  TORCH_CHECK(d.out_f32 || out.scalar_type() == at::kBFloat16, "gemm: out must be bf16 or fp32");
  d.epilogue = static_cast<int>(epilogue);
  if (d.epilogue == kEpiSwiGLU) {
    TORCH_CHECK(out.size(0) == d.M && out.size(1) * 2 == d.N, "gemm: swiglu out must be [M, N/2]");
  } else {
    TORCH_CHECK(out.size(0) == d.M && out.size(1) == d.N, "gemm: out must be [M, N] = [", d.M, ", ", d.N, "]");
  }
  if (d.epilogue == kEpiAtomicF32) TORCH_CHECK(d.out_f32, "gemm: atomic epilogue needs fp32 out");
  if (has(bias)) {
    check_f32(*bias, "bias");
    TORCH_CHECK(bias->numel() == d.N && bias->is_contiguous(), "gemm: bias must be fp32 [N]");
    d.bias = bias->data_ptr<float>();
  }
  d.rows_per_batch = static_cast<int>(std::max<int64_t>(1, rows_per_batch));
  if (d.epilogue == kEpiGateResid) {
    TORCH_CHECK(has(resid), "gemm: gate_resid needs resid");
    check_bf16(*resid, "resid");
    check_rows(*resid, "resid");
    TORCH_CHECK(resid->size(0) == d.M && resid->size(1) == d.N, "gemm: resid must be [M, N]");
    TORCH_CHECK(!d.out_f32, "gemm: gate_resid writes bf16");
    d.resid = resid->data_ptr();
    d.ldr = resid->stride(0);
    if (has(gate)) {
      check_f32(*gate, "gate");
      TORCH_CHECK(gate->dim() == 2 && gate->size(1) == d.N && gate->stride(1) == 1, "gemm: gate must be fp32 [B, N]");
      d.groups = groups_or_null(groups, d.M, "gemm");
      d.num_groups = static_cast<int>(gate->size(0));
      TORCH_CHECK(d.groups != nullptr || gate->size(0) * d.rows_per_batch >= d.M, "gemm: gate rows do not cover M");
      d.gate = gate->data_ptr<float>();
      d.gate_stride = gate->stride(0);
    }
  }
  if (has(aux)) {
    check_bf16(*aux, "aux");
    check_rows(*aux, "aux");
    TORCH_CHECK(aux->size(0) == d.M && aux->size(1) == d.N, "gemm: aux must be bf16 [M, N]");
    d.aux = aux->data_ptr();
    d.ldaux = aux->stride(0);
  }
  if (has(a2) || has(b2)) {
    // Appended reduction pair with the majorness of (a, b): D = [a | a2] . [b | b2]^T.
    TORCH_CHECK(has(a2) && has(b2), "gemm: a2 and b2 go together");
    check_bf16(*a2, "a2");
    check_bf16(*b2, "b2");
    check_rows(*a2, "a2");
    check_rows(*b2, "b2");
    const long m2 = a_mn ? a2->size(1) : a2->size(0);
    const long k2a = a_mn ? a2->size(0) : a2->size(1);
    const long n2 = b_mn ? b2->size(1) : b2->size(0);
    const long k2b = b_mn ? b2->size(0) : b2->size(1);
    TORCH_CHECK(m2 == d.M && n2 == d.N && k2a == k2b && k2a > 0, "gemm: appended pair must be a2 [M, K2] and b2 [N, K2]",
                " in the majorness of a and b; got M=", m2, " N=", n2, " K2=", k2a, "/", k2b);
    d.a2 = a2->data_ptr();
    d.lda2 = a2->stride(0);
    d.b2 = b2->data_ptr();
    d.ldb2 = b2->stride(0);
    d.K2 = static_cast<int>(k2a);
  }
  if (has(gate_flags)) {
    TORCH_CHECK(gate_flags->scalar_type() == at::kInt && gate_flags->is_cuda() && gate_flags->is_contiguous() &&
                    gate_flags->device() == a.device(),
                "gemm: gate_flags must be a contiguous int32 tensor on the GEMM's device");
    const long extent = gate_operand == 1 ? d.M : d.N;
    TORCH_CHECK(gate_chunk > 0 && gate_flags->numel() * gate_chunk >= extent,
                "gemm: gate_flags needs one word per chunk of ", gate_chunk, " rows");
    d.gate_flags = reinterpret_cast<const unsigned*>(gate_flags->data_ptr<int>());
    d.gate_epoch = static_cast<unsigned>(gate_epoch);
    d.gate_operand = static_cast<int>(gate_operand);
    d.gate_chunk = static_cast<int>(gate_chunk);
    d.gate_rank = static_cast<int>(gate_rank);
  }
  d.k_splits = static_cast<int>(std::max<int64_t>(1, k_splits));
  d.err = error_word(d.device);
  gemm_launch(d, cur_stream());
}

// --------------------------------------------------------------------- norms
NormDesc norm_common(const at::Tensor& x, int64_t rows_per_batch, double eps, const OptT& w, const OptT& scale,
                     const OptT& shift, const OptT& groups) {
  check_bf16(x, "x");
  check_rows(x, "x");
  NormDesc d;
  d.device = x.device().index();
  d.rows = x.size(0);
  d.W = static_cast<int>(x.size(1));
  d.rows_per_batch = std::max<int64_t>(1, rows_per_batch);
  d.eps = static_cast<float>(eps);
  d.x = x.data_ptr();
  d.ldx = x.stride(0);
  d.w = f32_or_null(w, "weight");
  if (has(scale) || has(shift)) {
    const at::Tensor& ref = has(scale) ? *scale : *shift;
    TORCH_CHECK(ref.dim() == 2 && ref.size(1) >= d.W && ref.stride(1) == 1, "norm: modulation must be [B, >=W]");
    d.groups = groups_or_null(groups, d.rows, "norm");
    d.num_groups = static_cast<int>(ref.size(0));
    TORCH_CHECK(d.groups != nullptr || ref.size(0) * d.rows_per_batch >= d.rows, "norm: modulation rows do not cover x");
    d.mod_stride = ref.stride(0);
    if (has(scale)) {
      check_f32(*scale, "scale");
      TORCH_CHECK(scale->stride(0) == d.mod_stride, "norm: scale/shift strides differ");
      d.scale = scale->data_ptr<float>();
    }
    if (has(shift)) {
      check_f32(*shift, "shift");
      TORCH_CHECK(shift->stride(0) == d.mod_stride, "norm: scale/shift strides differ");
      d.shift = shift->data_ptr<float>();
    }
  }
  return d;
}

void rmsnorm_mod_fwd(const at::Tensor& x, at::Tensor& y, const OptT& rstd, const OptT& w, const OptT& scale,
                     const OptT& shift, int64_t rows_per_batch, double eps, const OptT& groups) {
  c10::cuda::CUDAGuard guard(x.device());
  NormDesc d = norm_common(x, rows_per_batch, eps, w, scale, shift, groups);
  check_bf16(y, "y");
  check_rows(y, "y");
  TORCH_CHECK(y.size(0) == d.rows && y.size(1) == d.W, "norm: y shape");
  d.y = y.data_ptr();
  d.ldy = y.stride(0);
  if (has(rstd)) {
    check_f32(*rstd, "rstd");
    TORCH_CHECK(rstd->numel() == d.rows, "norm: rstd must be [rows]");
    d.rstd = rstd->data_ptr<float>();
  }
  rmsnorm_mod_fwd_launch(d, cur_stream());
}

void rmsnorm_mod_bwd(const at::Tensor& x, const at::Tensor& rstd, const at::Tensor& dy, const OptT& dx,
                     const OptT& dres, const OptT& w, const OptT& scale, const OptT& shift, const OptT& dw,
                     const OptT& dscale, const OptT& dshift, int64_t rows_per_batch, const OptT& groups) {
  c10::cuda::CUDAGuard guard(x.device());
  NormDesc d = norm_common(x, rows_per_batch, 0.0, w, scale, shift, groups);
  TORCH_CHECK(d.groups != nullptr || !has(groups), "norm bwd: groups need scale or shift");
  check_f32(rstd, "rstd");
  TORCH_CHECK(rstd.numel() == d.rows, "norm bwd: rstd must be [rows]");
  d.rstd = rstd.data_ptr<float>();
  check_bf16(dy, "dy");
  check_rows(dy, "dy");
  d.dy = dy.data_ptr();
  d.lddy = dy.stride(0);
  if (has(dx)) {
    check_bf16(*dx, "dx");
    check_rows(*dx, "dx");
    d.dx = dx->data_ptr();
    d.lddx = dx->stride(0);
  }
  if (has(dres)) {
    check_bf16(*dres, "dres");
    check_rows(*dres, "dres");
    d.dres = dres->data_ptr();
    d.lddres = dres->stride(0);
  }
  d.dw = has(dw) ? dw->data_ptr<float>() : nullptr;
  if (has(dscale) || has(dshift)) {
    const at::Tensor& ref = has(dscale) ? *dscale : *dshift;
    d.dmod_stride = ref.stride(0);
    d.dscale = has(dscale) ? dscale->data_ptr<float>() : nullptr;
    d.dshift = has(dshift) ? dshift->data_ptr<float>() : nullptr;
  }
  rmsnorm_mod_bwd_launch(d, cur_stream());
}

void gate_bwd(const at::Tensor& dx, const at::Tensor& a, const at::Tensor& gate, at::Tensor& da, at::Tensor& dgate,
              int64_t rows_per_batch, const OptT& groups) {
  c10::cuda::CUDAGuard guard(dx.device());
  check_bf16(dx, "dx");
  check_bf16(a, "a");
  check_bf16(da, "da");
  check_f32(gate, "gate");
  check_f32(dgate, "dgate");
  GateBwdDesc d;
  d.device = dx.device().index();
  d.rows = dx.size(0);
  d.W = static_cast<int>(dx.size(1));
  d.rows_per_batch = std::max<int64_t>(1, rows_per_batch);
  d.groups = groups_or_null(groups, d.rows, "gate_bwd");
  d.num_groups = static_cast<int>(gate.size(0));
  d.dx = dx.data_ptr();
  d.lddx = dx.stride(0);
  d.a = a.data_ptr();
  d.lda = a.stride(0);
  d.gate = gate.data_ptr<float>();
  d.gate_stride = gate.stride(0);
  d.da = da.data_ptr();
  d.ldda = da.stride(0);
  d.dgate = dgate.data_ptr<float>();
  d.dgate_stride = dgate.stride(0);
  gate_bwd_launch(d, cur_stream());
}

// --------------------------------------------------------------------- qk-norm + rope
QkvRopeDesc rope_common(const at::Tensor& qkv, int64_t B, int64_t L, int64_t H, int64_t Hk, int64_t D, double eps,
                        const OptT& q_w, const OptT& k_w, const OptT& coords, const OptT& freq, const OptT& axis) {
  check_bf16(qkv, "qkv");
  check_rows(qkv, "qkv");
  TORCH_CHECK(qkv.size(0) == B * L && qkv.size(1) == (H + 2 * Hk) * D, "qkv_rope: qkv must be [B*L, (H+2Hk)*D]");
  QkvRopeDesc d;
  d.device = qkv.device().index();
  d.B = static_cast<int>(B);
  d.L = static_cast<int>(L);
  d.H = static_cast<int>(H);
  d.Hk = static_cast<int>(Hk);
  d.D = static_cast<int>(D);
  d.eps = static_cast<float>(eps);
  d.qkv = qkv.data_ptr();
  d.ldqkv = qkv.stride(0);
  d.q_w = f32_or_null(q_w, "q_w");
  d.k_w = f32_or_null(k_w, "k_w");
  if (has(coords)) {
    check_f32(*coords, "coords");
    TORCH_CHECK(coords->is_contiguous() && coords->numel() == B * L * 3, "qkv_rope: coords must be [B, L, 3]");
    TORCH_CHECK(has(freq) && has(axis), "qkv_rope: freq and axis required with coords");
    check_f32(*freq, "freq");
    TORCH_CHECK(freq->numel() == D / 2 && axis->numel() == D / 2, "qkv_rope: freq/axis must be [D/2]");
    TORCH_CHECK(axis->scalar_type() == at::kInt && axis->is_cuda(), "qkv_rope: axis must be int32 CUDA");
    d.coords = coords->data_ptr<float>();
    d.freq = freq->data_ptr<float>();
    d.axis = axis->data_ptr<int>();
  }
  return d;
}

void qkv_rope_fwd(const at::Tensor& qkv, int64_t B, int64_t L, int64_t H, int64_t Hk, int64_t D, double eps,
                  const OptT& q_w, const OptT& k_w, const OptT& coords, const OptT& freq, const OptT& axis,
                  const OptT& q, const OptT& k, const OptT& v) {
  c10::cuda::CUDAGuard guard(qkv.device());
  QkvRopeDesc d = rope_common(qkv, B, L, H, Hk, D, eps, q_w, k_w, coords, freq, axis);
  if (H > 0) {
    TORCH_CHECK(has(q) && q->is_contiguous() && q->numel() == B * H * L * D, "qkv_rope: q must be [B, H, L, D]");
    check_bf16(*q, "q");
    d.q = q->data_ptr();
  }
  if (Hk > 0) {
    TORCH_CHECK(has(k) && has(v) && k->is_contiguous() && v->is_contiguous(), "qkv_rope: k, v required");
    TORCH_CHECK(k->numel() == B * Hk * L * D && v->numel() == B * Hk * L * D, "qkv_rope: k, v must be [B, Hk, L, D]");
    check_bf16(*k, "k");
    check_bf16(*v, "v");
    d.k = k->data_ptr();
    d.v = v->data_ptr();
  }
  qkv_rope_fwd_launch(d, cur_stream());
}

void qkv_rope_bwd(const at::Tensor& qkv, at::Tensor& dqkv, int64_t B, int64_t L, int64_t H, int64_t Hk, int64_t D,
                  double eps, const OptT& q_w, const OptT& k_w, const OptT& coords, const OptT& freq,
                  const OptT& axis, const OptT& dq, const OptT& dk, const OptT& dv, const OptT& dq_w,
                  const OptT& dk_w) {
  c10::cuda::CUDAGuard guard(qkv.device());
  QkvRopeDesc d = rope_common(qkv, B, L, H, Hk, D, eps, q_w, k_w, coords, freq, axis);
  if (H > 0) {
    TORCH_CHECK(has(dq) && dq->is_contiguous() && dq->numel() == B * H * L * D, "qkv_rope bwd: dq");
    check_bf16(*dq, "dq");
    d.dq = dq->data_ptr();
  }
  if (Hk > 0) {
    TORCH_CHECK(has(dk) && has(dv) && dk->is_contiguous() && dv->is_contiguous(), "qkv_rope bwd: dk, dv");
    check_bf16(*dk, "dk");
    check_bf16(*dv, "dv");
    d.dk = dk->data_ptr();
    d.dv = dv->data_ptr();
  }
  check_bf16(dqkv, "dqkv");
  check_rows(dqkv, "dqkv");
  TORCH_CHECK(dqkv.sizes() == qkv.sizes(), "qkv_rope bwd: dqkv must match qkv");
  d.dqkv = dqkv.data_ptr();
  d.lddqkv = dqkv.stride(0);
  d.dq_w = has(dq_w) ? dq_w->data_ptr<float>() : nullptr;
  d.dk_w = has(dk_w) ? dk_w->data_ptr<float>() : nullptr;
  qkv_rope_bwd_launch(d, cur_stream());
}

// --------------------------------------------------------------------- activations
void swiglu_bwd(const at::Tensor& dh, const at::Tensor& gu, at::Tensor& dgu) {
  c10::cuda::CUDAGuard guard(dh.device());
  check_bf16(dh, "dh");
  check_bf16(gu, "gu");
  check_bf16(dgu, "dgu");
  TORCH_CHECK(gu.size(0) == dh.size(0) && gu.size(1) == 2 * dh.size(1), "swiglu_bwd: gu must be [M, 2F]");
  TORCH_CHECK(dgu.sizes() == gu.sizes(), "swiglu_bwd: dgu must match gu");
  swiglu_bwd_launch(dh.device().index(), dh.size(0), static_cast<int>(dh.size(1)), dh.data_ptr(), dh.stride(0),
                    gu.data_ptr(), gu.stride(0), dgu.data_ptr(), dgu.stride(0), cur_stream());
}

void gelu_bwd(const at::Tensor& dh, const at::Tensor& pre, at::Tensor& dpre) {
  c10::cuda::CUDAGuard guard(dh.device());
  check_bf16(dh, "dh");
  check_bf16(pre, "pre");
  check_bf16(dpre, "dpre");
  TORCH_CHECK(pre.sizes() == dh.sizes() && dpre.sizes() == dh.sizes(), "gelu_bwd: shapes differ");
  gelu_bwd_launch(dh.device().index(), dh.size(0), static_cast<int>(dh.size(1)), dh.data_ptr(), dh.stride(0),
                  pre.data_ptr(), pre.stride(0), dpre.data_ptr(), dpre.stride(0), cur_stream());
}

// --------------------------------------------------------------------- loss / noise
FlowLossDesc loss_common(const at::Tensor& pred, const at::Tensor& target, const at::Tensor& mask, const OptT& weight,
                         int64_t rows_per_batch) {
  check_cuda(pred, "pred");
  check_cuda(target, "target");
  TORCH_CHECK(pred.is_contiguous() && target.is_contiguous() && mask.is_contiguous(), "loss: contiguous inputs");
  TORCH_CHECK(pred.sizes() == target.sizes(), "loss: pred/target shapes differ");
  TORCH_CHECK(mask.scalar_type() == at::kBool && mask.numel() * pred.size(-1) == pred.numel(), "loss: mask [rows]");
  FlowLossDesc d;
  d.device = pred.device().index();
  d.P = static_cast<int>(pred.size(-1));
  d.rows = pred.numel() / d.P;
  d.rows_per_batch = std::max<int64_t>(1, rows_per_batch);
  d.pred = pred.data_ptr();
  d.pred_f32 = pred.scalar_type() == at::kFloat;
  d.target = target.data_ptr();
  d.target_f32 = target.scalar_type() == at::kFloat;
  d.mask = reinterpret_cast<const uint8_t*>(mask.data_ptr());
  d.weight = f32_or_null(weight, "weight");
  return d;
}

void flow_loss_fwd(const at::Tensor& pred, const at::Tensor& target, const at::Tensor& mask, const OptT& weight,
                   int64_t rows_per_batch, at::Tensor& stats) {
  c10::cuda::CUDAGuard guard(pred.device());
  FlowLossDesc d = loss_common(pred, target, mask, weight, rows_per_batch);
  check_f32(stats, "stats");
  TORCH_CHECK(stats.numel() >= 3, "loss: stats must hold 3 floats");
  d.stats = stats.data_ptr<float>();
  flow_loss_fwd_launch(d, cur_stream());
}

void flow_loss_bwd(const at::Tensor& pred, const at::Tensor& target, const at::Tensor& mask, const OptT& weight,
                   int64_t rows_per_batch, const at::Tensor& scale, at::Tensor& dpred) {
  c10::cuda::CUDAGuard guard(pred.device());
  FlowLossDesc d = loss_common(pred, target, mask, weight, rows_per_batch);
  check_f32(scale, "scale");
  TORCH_CHECK(dpred.sizes() == pred.sizes() && dpred.is_contiguous(), "loss: dpred shape");
  d.scale = scale.data_ptr<float>();
  d.dpred = dpred.data_ptr();
  d.dpred_f32 = dpred.scalar_type() == at::kFloat;
  flow_loss_bwd_launch(d, cur_stream());
}

void noise_interp(const at::Tensor& clean, const at::Tensor& t, int64_t seed, int64_t offset, int64_t row_base,
                  int64_t rows_per_sample, int64_t global_rows_per_sample, at::Tensor& noisy, at::Tensor& target,
                  const OptT& noise) {
  c10::cuda::CUDAGuard guard(clean.device());
  check_cuda(clean, "clean");
  check_f32(t, "t");
  check_f32(noisy, "noisy");
  check_f32(target, "target");
  TORCH_CHECK(clean.is_contiguous() && t.is_contiguous() && noisy.is_contiguous() && target.is_contiguous(),
              "noise: contiguous tensors required");
  NoiseDesc d;
  d.device = clean.device().index();
  d.P = static_cast<int>(clean.size(-1));
  d.rows = clean.numel() / d.P;
  TORCH_CHECK(t.numel() == d.rows, "noise: t must be [rows]");
  d.seed = static_cast<uint64_t>(seed);
  d.offset = static_cast<uint64_t>(offset);
  d.row_base = row_base;
  d.rows_per_sample = std::max<int64_t>(1, rows_per_sample);
  d.global_rows_per_sample = std::max<int64_t>(1, global_rows_per_sample);
  d.clean = clean.data_ptr();
  d.clean_f32 = clean.scalar_type() == at::kFloat;
  d.t = t.data_ptr<float>();
  d.noisy = noisy.data_ptr();
  d.target = target.data_ptr();
  if (has(noise)) {
    check_f32(*noise, "noise");
    d.noise = noise->data_ptr();
  }
  noise_interp_launch(d, cur_stream());
}

// --------------------------------------------------------------------- sampling
void guided_euler(const at::Tensor& cond, const OptT& uncond, const at::Tensor& x, const at::Tensor& sigma,
                  const at::Tensor& sigma_next, double scale, at::Tensor& out) {
  c10::cuda::CUDAGuard guard(x.device());
  check_cuda(cond, "cond");
  check_cuda(x, "x");
  check_f32(sigma, "sigma");
  check_f32(sigma_next, "sigma_next");
  TORCH_CHECK(cond.is_contiguous() && x.is_contiguous() && out.is_contiguous(), "guided_euler: contiguous tensors");
  TORCH_CHECK(cond.numel() == x.numel() && out.numel() == x.numel(), "guided_euler: shape mismatch");
  GuidedEulerDesc d;
  d.device = x.device().index();
  d.batch = static_cast<int>(x.size(0));
  d.per_sample = x.numel() / std::max<int64_t>(1, x.size(0));
  TORCH_CHECK(sigma.numel() == d.batch && sigma_next.numel() == d.batch, "guided_euler: sigma must be [batch]");
  d.cond = cond.data_ptr();
  d.vel_f32 = cond.scalar_type() == at::kFloat;
  if (has(uncond)) {
    TORCH_CHECK(uncond->is_contiguous() && uncond->numel() == x.numel() &&
                uncond->scalar_type() == cond.scalar_type(), "guided_euler: uncond must match cond");
    d.uncond = uncond->data_ptr();
  }
  d.x = x.data_ptr();
  d.x_f32 = x.scalar_type() == at::kFloat;
  d.out = out.data_ptr();
  d.out_f32 = out.scalar_type() == at::kFloat;
  d.sigma = sigma.data_ptr<float>();
  d.sigma_next = sigma_next.data_ptr<float>();
  d.scale = static_cast<float>(scale);
  guided_euler_launch(d, cur_stream());
}

void sde_step(const at::Tensor& v, const at::Tensor& x, const at::Tensor& sigma, const at::Tensor& sigma_next,
              const at::Tensor& g, double floor, at::Tensor& mean, at::Tensor& log_prob, const OptT& noise,
              const OptT& prev, const OptT& mask, const OptT& sample) {
  c10::cuda::CUDAGuard guard(x.device());
  check_cuda(v, "v");
  check_f32(x, "x");
  check_f32(sigma, "sigma");
  check_f32(sigma_next, "sigma_next");
  check_f32(g, "g");
  check_f32(mean, "mean");
  check_f32(log_prob, "log_prob");
  TORCH_CHECK(v.is_contiguous() && x.is_contiguous() && mean.is_contiguous(), "sde_step: contiguous tensors");
  SDEStepDesc d;
  d.device = x.device().index();
  d.batch = static_cast<int>(x.size(0));
  d.per_sample = x.numel() / std::max<int64_t>(1, x.size(0));
  TORCH_CHECK(v.numel() == x.numel() && mean.numel() == x.numel(), "sde_step: shape mismatch");
  TORCH_CHECK(sigma.numel() == d.batch && sigma_next.numel() == d.batch && g.numel() == d.batch &&
              log_prob.numel() == d.batch, "sde_step: per-sample tensors must be [batch]");
  TORCH_CHECK(has(noise) != has(prev), "sde_step: give exactly one of noise (rollout) or prev (update)");
  d.v = v.data_ptr();
  d.v_f32 = v.scalar_type() == at::kFloat;
  d.x = x.data_ptr<float>();
  d.sigma = sigma.data_ptr<float>();
  d.sigma_next = sigma_next.data_ptr<float>();
  d.g = g.data_ptr<float>();
  d.floor = static_cast<float>(floor);
  if (has(noise)) {
    check_f32(*noise, "noise");
    TORCH_CHECK(noise->is_contiguous() && noise->numel() == x.numel(), "sde_step: noise shape");
    TORCH_CHECK(has(sample), "sde_step: rollout needs a sample output");
    check_f32(*sample, "sample");
    TORCH_CHECK(sample->is_contiguous() && sample->numel() == x.numel(), "sde_step: sample shape");
    d.noise = noise->data_ptr<float>();
    d.sample = sample->data_ptr<float>();
  } else {
    check_f32(*prev, "prev");
    TORCH_CHECK(prev->is_contiguous() && prev->numel() == x.numel(), "sde_step: prev shape");
    d.prev = prev->data_ptr<float>();
  }
  if (has(mask)) {
    TORCH_CHECK(mask->scalar_type() == at::kBool && mask->is_contiguous() && mask->numel() == x.numel(),
                "sde_step: mask must be a contiguous bool tensor shaped like x");
    d.mask = mask->data_ptr<bool>();
  }
  d.mean = mean.data_ptr<float>();
  d.log_prob = log_prob.data_ptr<float>();
  sde_step_launch(d, cur_stream());
}

// --------------------------------------------------------------------- optimizer
void adamw(at::Tensor& param, const at::Tensor& grad, at::Tensor& exp_avg, at::Tensor& exp_avg_sq, double lr,
           double beta1, double beta2, double eps, double weight_decay, int64_t step, const OptT& param_bf16,
           const OptT& grad_scale, const OptT& skip) {
  c10::cuda::CUDAGuard guard(param.device());
  for (at::Tensor* t : {&param, &exp_avg, &exp_avg_sq}) {
    check_f32(*t, "adamw state");
    TORCH_CHECK(t->is_contiguous() && t->numel() == param.numel(), "adamw: state must match param");
  }
  check_f32(grad, "grad");
  TORCH_CHECK(grad.is_contiguous() && grad.numel() == param.numel(), "adamw: grad must match param");
  AdamWDesc d;
  d.device = param.device().index();
  d.n = param.numel();
  d.param = param.data_ptr<float>();
  d.grad = grad.data_ptr<float>();
  d.exp_avg = exp_avg.data_ptr<float>();
  d.exp_avg_sq = exp_avg_sq.data_ptr<float>();
  if (has(param_bf16)) {
    check_bf16(*param_bf16, "param_bf16");
    TORCH_CHECK(param_bf16->is_contiguous() && param_bf16->numel() == d.n, "adamw: bf16 copy must match");
    d.param_bf16 = param_bf16->data_ptr();
  }
  d.lr = static_cast<float>(lr);
  d.beta1 = static_cast<float>(beta1);
  d.beta2 = static_cast<float>(beta2);
  d.eps = static_cast<float>(eps);
  d.weight_decay = static_cast<float>(weight_decay);
  TORCH_CHECK(step >= 1, "adamw: step must be >= 1");
  d.bias_correction1 = static_cast<float>(1.0 - std::pow(beta1, static_cast<double>(step)));
  d.bias_correction2_sqrt = static_cast<float>(std::sqrt(1.0 - std::pow(beta2, static_cast<double>(step))));
  d.grad_scale = f32_or_null(grad_scale, "grad_scale");
  if (has(skip)) {
    TORCH_CHECK(skip->scalar_type() == at::kInt && skip->is_cuda(), "adamw: skip must be int32 CUDA");
    d.skip = skip->data_ptr<int>();
  }
  adamw_launch(d, cur_stream());
}

void sq_norm(const at::Tensor& x, at::Tensor& out) {
  c10::cuda::CUDAGuard guard(x.device());
  check_f32(x, "x");
  check_f32(out, "out");
  TORCH_CHECK(x.is_contiguous(), "sq_norm: contiguous input");
  sq_norm_launch(x.device().index(), x.data_ptr<float>(), x.numel(), out.data_ptr<float>(), cur_stream());
}

void ema(const at::Tensor& param, at::Tensor& shadow, double decay) {
  c10::cuda::CUDAGuard guard(param.device());
  check_f32(param, "param");
  check_cuda(shadow, "shadow");
  TORCH_CHECK(param.is_contiguous() && shadow.is_contiguous() && shadow.numel() == param.numel(), "ema: shapes");
  const bool bf = shadow.scalar_type() == at::kBFloat16;
  TORCH_CHECK(bf || shadow.scalar_type() == at::kFloat, "ema: shadow must be bf16 or fp32");
  ema_launch(param.device().index(), param.numel(), param.data_ptr<float>(), shadow.data_ptr(), bf,
             static_cast<float>(decay), cur_stream());
}

// --------------------------------------------------------------------- attention
// Row stride (in floats) of a [B, H, Lq] row-statistics tensor whose (b, h) rows
// may be padded: the backward reads them with TMA, which needs 16-byte rows.
long stat_row_stride(const at::Tensor& t, int B, int H, int Lq, const char* what) {
  TORCH_CHECK(t.dim() == 3 && t.size(0) == B && t.size(1) == H && t.size(2) == Lq && t.stride(2) == 1 &&
                  t.stride(1) >= Lq && t.stride(0) == t.stride(1) * H,
              what, " must be [B, H, Lq] with unit last stride and (b, h) rows laid out densely");
  return t.stride(1);
}

// k, v: [B, Hk, Lk, D], or the context-parallel ring layout [world, B, Hk, L, D]
// (keys of rank r in slab r; Lk = world * L) together with ring_flags.
void attn_fwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, at::Tensor& out, const OptT& lse,
              const OptT& kmask, double scale, const OptT& trace, int64_t ring_rank, const OptT& ring_flags,
              int64_t ring_epoch, const OptT& ring_wait) {
  c10::cuda::CUDAGuard guard(q.device());
  check_bf16(q, "q");
  check_bf16(k, "k");
  check_bf16(v, "v");
  check_bf16(out, "out");
  const bool ring = k.dim() == 5;
  TORCH_CHECK(q.dim() == 4 && (k.dim() == 4 || ring) && v.dim() == k.dim(),
              "attention: q must be [B, H, L, D]; k, v [B, Hk, L, D] or [world, B, Hk, L, D]");
  TORCH_CHECK(q.is_contiguous() && k.is_contiguous() && v.is_contiguous(), "attention: dense q, k, v");
  TORCH_CHECK(k.sizes() == v.sizes(), "attention: k and v shapes differ");
  const int o5 = ring ? 1 : 0;
  AttnFwdDesc d;
  d.device = q.device().index();
  d.B = static_cast<int>(q.size(0));
  d.H = static_cast<int>(q.size(1));
  d.Lq = static_cast<int>(q.size(2));
  d.D = static_cast<int>(q.size(3));
  d.Hk = static_cast<int>(k.size(1 + o5));
  d.Lk = static_cast<int>(k.size(2 + o5) * (ring ? k.size(0) : 1));
  TORCH_CHECK(k.size(o5) == d.B && k.size(3 + o5) == d.D, "attention: k batch/dim mismatch");
  if (ring) {
    TORCH_CHECK(has(ring_flags) && ring_flags->scalar_type() == at::kInt && ring_flags->is_cuda() &&
                    ring_flags->numel() >= k.size(0),
                "attention ring: ring_flags must be an int32 device tensor with one word per rank");
    d.ring_world = static_cast<int>(k.size(0));
    d.ring_rank = static_cast<int>(ring_rank);
    d.ring_len = static_cast<int>(k.size(3));
    d.ring_flags = reinterpret_cast<const unsigned*>(ring_flags->data_ptr<int>());
    d.ring_epoch = static_cast<unsigned>(ring_epoch);
    if (has(ring_wait)) {
      TORCH_CHECK(ring_wait->scalar_type() == at::kLong && ring_wait->is_cuda() && ring_wait->numel() >= 1,
                  "attention ring: ring_wait must be an int64 device tensor");
      d.wait_cycles = reinterpret_cast<unsigned long long*>(ring_wait->data_ptr<int64_t>());
    }
  }
  // out: token-major [B, Lq, H, D] (any strides with a contiguous last dim)
  TORCH_CHECK(out.dim() == 4 && out.size(0) == d.B && out.size(1) == d.Lq && out.size(2) == d.H &&
                  out.size(3) == d.D && out.stride(3) == 1,
              "attention: out must be [B, Lq, H, D]");
  TORCH_CHECK(out.stride(2) % 8 == 0 && out.stride(1) % 8 == 0, "attention: out strides must be 16-byte aligned");
  d.q = q.data_ptr();
  d.k = k.data_ptr();
  d.v = v.data_ptr();
  d.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  d.o_sb = out.stride(0);
  d.o_sl = out.stride(1);
  d.o_sh = out.stride(2);
  if (has(lse)) {
    check_f32(*lse, "lse");
    d.stat_ld = stat_row_stride(*lse, d.B, d.H, d.Lq, "attention: lse");
    d.lse = lse->data_ptr<float>();
  }
  if (has(kmask)) {
    TORCH_CHECK(kmask->scalar_type() == at::kInt && kmask->is_cuda() && kmask->dim() == 2 && kmask->size(0) == d.B,
                "attention: kmask must be packed int32 [B, words]");
    d.kmask = reinterpret_cast<const uint32_t*>(kmask->data_ptr<int>());
    d.kmask_words = static_cast<int>(kmask->stride(0));
  }
  d.scale_log2 = static_cast<float>(scale * 1.4426950408889634);
  d.err = error_word(d.device);
  if (has(trace)) {
    TORCH_CHECK(trace->scalar_type() == at::kLong && trace->is_cuda() && trace->numel() >= 64 * 24,
                "attention fwd: trace must be an int64 device tensor of at least 1536 entries");
    d.trace = reinterpret_cast<long long*>(trace->data_ptr<int64_t>());
  }
  attn_fwd_launch(d, cur_stream());
}

void attn_bwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& o,
              const at::Tensor& dout, const at::Tensor& lse, at::Tensor& delta, at::Tensor& dq, at::Tensor& dk,
              at::Tensor& dv, const OptT& kmask, double scale, const OptT& dq_acc, const OptT& trace,
              int64_t kt_begin, int64_t kt_count, bool skip_prologue, bool skip_epilogue) {
  c10::cuda::CUDAGuard guard(q.device());
  for (const at::Tensor* t : {&q, &k, &v, &o, &dout, static_cast<const at::Tensor*>(&dk), static_cast<const at::Tensor*>(&dv)}) check_bf16(*t, "attention bwd tensor");
  check_f32(lse, "lse");
  check_f32(delta, "delta");
  check_bf16(dq, "dq");
  AttnBwdDesc d;
  d.device = q.device().index();
  d.B = static_cast<int>(q.size(0));
  d.H = static_cast<int>(q.size(1));
  d.Lq = static_cast<int>(q.size(2));
  d.D = static_cast<int>(q.size(3));
  const bool ring = k.dim() == 5;  // [world, B, Hk, L, D] (dk, dv likewise)
  const int o5 = ring ? 1 : 0;
  d.Hk = static_cast<int>(k.size(1 + o5));
  d.Lk = static_cast<int>(k.size(2 + o5) * (ring ? k.size(0) : 1));
  if (ring) {
    d.ring_world = static_cast<int>(k.size(0));
    d.ring_len = static_cast<int>(k.size(3));
  }
  TORCH_CHECK(q.is_contiguous() && k.is_contiguous() && v.is_contiguous(), "attention bwd: dense q, k, v");
  TORCH_CHECK(o.is_contiguous() && dout.is_contiguous() && o.dim() == 4 && o.size(1) == d.Lq && o.size(2) == d.H,
              "attention bwd: o / dout must be dense [B, Lq, H, D]");
  TORCH_CHECK(dout.sizes() == o.sizes(), "attention bwd: dout must match o");
  TORCH_CHECK(dq.is_contiguous() && dq.sizes() == q.sizes(), "attention bwd: dq must match q");
  TORCH_CHECK(dk.is_contiguous() && dv.is_contiguous() && dk.sizes() == k.sizes() && dv.sizes() == v.sizes(),
              "attention bwd: dk/dv must match k/v");
  d.stat_ld = stat_row_stride(lse, d.B, d.H, d.Lq, "attention bwd: lse");
  TORCH_CHECK(delta.strides() == lse.strides() && delta.sizes() == lse.sizes(),
              "attention bwd: delta must have the shape and strides of lse");
  d.q = q.data_ptr();
  d.k = k.data_ptr();
  d.v = v.data_ptr();
  d.o = o.data_ptr();
  d.dout = dout.data_ptr();
  d.o_sb = o.stride(0);
  d.o_sl = o.stride(1);
  d.o_sh = o.stride(2);
  d.lse = lse.data_ptr<float>();
  d.delta = delta.data_ptr<float>();
  d.dq = reinterpret_cast<__nv_bfloat16*>(dq.data_ptr());
  d.dk = reinterpret_cast<__nv_bfloat16*>(dk.data_ptr());
  d.dv = reinterpret_cast<__nv_bfloat16*>(dv.data_ptr());
  if (has(dq_acc)) {
    check_f32(*dq_acc, "dq_acc");
    TORCH_CHECK(dq_acc->numel() >= static_cast<long>(d.B) * d.H * ((d.Lq + 3) / 4 * 4) * d.D && dq_acc->is_contiguous(),
                "attention bwd: dq_acc must be contiguous fp32 with B*H*128*ceil4(Lq) elements");
    d.dq_acc = dq_acc->data_ptr<float>();
  }
  if (has(trace)) {
    TORCH_CHECK(trace->scalar_type() == at::kLong && trace->is_cuda() && trace->numel() >= 64 * 24,
                "attention bwd: trace must be an int64 device tensor of at least 1536 entries");
    d.trace = reinterpret_cast<long long*>(trace->data_ptr<int64_t>());
  }
  if (has(kmask)) {
    TORCH_CHECK(kmask->scalar_type() == at::kInt && kmask->is_cuda() && kmask->dim() == 2 && kmask->size(0) == d.B,
                "attention bwd: kmask must be packed int32 [B, words]");
    d.kmask = reinterpret_cast<const uint32_t*>(kmask->data_ptr<int>());
    d.kmask_words = static_cast<int>(kmask->stride(0));
  }
  d.scale = static_cast<float>(scale);
  d.scale_log2 = static_cast<float>(scale * 1.4426950408889634);
  d.err = error_word(d.device);
  d.kt_begin = static_cast<int>(kt_begin);
  d.kt_count = static_cast<int>(kt_count);
  d.skip_prologue = skip_prologue;
  d.skip_epilogue = skip_epilogue;
  attn_bwd_launch(d, cur_stream());
}

// --------------------------------------------------------------------- sharded AdamW
std::vector<const float*> addr_list(const std::vector<int64_t>& addrs) {
  std::vector<const float*> out;
  out.reserve(addrs.size());
  for (int64_t a : addrs) out.push_back(reinterpret_cast<const float*>(a));
  return out;
}

void shard_reduce(const std::vector<int64_t>& grads, int64_t lo, at::Tensor& out, at::Tensor& sq_acc) {
  c10::cuda::CUDAGuard guard(out.device());
  check_f32(out, "out");
  check_f32(sq_acc, "sq_acc");
  TORCH_CHECK(out.is_contiguous(), "shard_reduce: out must be contiguous");
  const auto p = addr_list(grads);
  shard_reduce_launch(p.data(), static_cast<int>(p.size()), lo, out.numel(), out.data_ptr<float>(),
                      sq_acc.data_ptr<float>(), out.device().index(), cur_stream());
}

void shard_adamw_push(const std::vector<int64_t>& params, int64_t rank, int64_t lo, const at::Tensor& grad,
                      at::Tensor& exp_avg, at::Tensor& exp_avg_sq, double lr, double beta1, double beta2, double eps,
                      double weight_decay, int64_t step, const OptT& grad_scale, const OptT& skip) {
  c10::cuda::CUDAGuard guard(grad.device());
  check_f32(grad, "grad");
  check_f32(exp_avg, "exp_avg");
  check_f32(exp_avg_sq, "exp_avg_sq");
  TORCH_CHECK(grad.numel() == exp_avg.numel() && grad.numel() == exp_avg_sq.numel() && grad.numel() % 4 == 0,
              "shard_adamw_push: shard tensors must match and hold a multiple of 4 elements");
  ShardAdamWDesc d;
  d.device = grad.device().index();
  d.rank = static_cast<int>(rank);
  d.world = static_cast<int>(params.size());
  TORCH_CHECK(d.rank >= 0 && d.rank < d.world, "shard_adamw_push: rank outside the parameter list");
  d.lo = lo;
  d.n4 = grad.numel() / 4;
  d.grad = grad.data_ptr<float>();
  d.exp_avg = exp_avg.data_ptr<float>();
  d.exp_avg_sq = exp_avg_sq.data_ptr<float>();
  d.lr = static_cast<float>(lr);
  d.beta1 = static_cast<float>(beta1);
  d.beta2 = static_cast<float>(beta2);
  d.eps = static_cast<float>(eps);
  d.weight_decay = static_cast<float>(weight_decay);
  d.bias_correction1 = static_cast<float>(1.0 - std::pow(beta1, static_cast<double>(step)));
  d.bias_correction2_sqrt = static_cast<float>(std::sqrt(1.0 - std::pow(beta2, static_cast<double>(step))));
  d.grad_scale = f32_or_null(grad_scale, "grad_scale");
  if (has(skip)) {
    TORCH_CHECK(skip->scalar_type() == at::kInt && skip->is_cuda(), "shard_adamw_push: skip must be int32 on device");
    d.skip = skip->data_ptr<int>();
  }
  const auto p = addr_list(params);
  shard_adamw_push_launch(d, p.data(), cur_stream());
}

// --------------------------------------------------------------------- sharded data parallelism
void peer_reduce(const std::vector<int64_t>& srcs, int64_t rank, int64_t offset, at::Tensor& out, bool src_bf16,
                 double scale, const OptT& sq_acc) {
  c10::cuda::CUDAGuard guard(out.device());
  check_f32(out, "out");
  TORCH_CHECK(out.is_contiguous(), "peer_reduce: out must be contiguous");
  std::vector<const void*> p;
  p.reserve(srcs.size());
  for (int64_t a : srcs) p.push_back(reinterpret_cast<const void*>(a));
  peer_reduce_launch(p.data(), static_cast<int>(p.size()), static_cast<int>(rank), offset, out.numel(), src_bf16,
                     static_cast<float>(scale), out.data_ptr<float>(), const_cast<float*>(f32_or_null(sq_acc, "sq_acc")),
                     out.device().index(), cur_stream());
}

// `table`: int64 device tensor [T, 4] of (param, grad, exp_avg, exp_avg_sq) addresses;
// `chunks`: int64 device tensor [C, 3] of (row, start, length).
const MTTensor* mt_rows(const at::Tensor& table) {
  TORCH_CHECK(table.is_cuda() && table.scalar_type() == at::kLong && table.is_contiguous() && table.dim() == 2 &&
                  table.size(1) == 4,
              "multi-tensor: the table must be a contiguous int64 [T, 4] device tensor");
  static_assert(sizeof(MTTensor) == 4 * sizeof(int64_t), "MTTensor layout");
  return reinterpret_cast<const MTTensor*>(table.data_ptr<int64_t>());
}
const MTChunk* mt_chunks(const at::Tensor& chunks) {
  TORCH_CHECK(chunks.is_cuda() && chunks.scalar_type() == at::kLong && chunks.is_contiguous() && chunks.dim() == 2 &&
                  chunks.size(1) == 3,
              "multi-tensor: chunks must be a contiguous int64 [C, 3] device tensor");
  static_assert(sizeof(MTChunk) == 3 * sizeof(int64_t), "MTChunk layout");
  return reinterpret_cast<const MTChunk*>(chunks.data_ptr<int64_t>());
}

void mt_sq_norm(const at::Tensor& table, const at::Tensor& chunks, at::Tensor& acc) {
  c10::cuda::CUDAGuard guard(acc.device());
  check_f32(acc, "acc");
  mt_sq_norm_launch(mt_chunks(chunks), static_cast<int>(chunks.size(0)), mt_rows(table), acc.data_ptr<float>(),
                    cur_stream());
}

void mt_adamw(const at::Tensor& table, const at::Tensor& chunks, double lr, double beta1, double beta2, double eps,
              double weight_decay, int64_t step, const OptT& grad_scale, const OptT& skip) {
  c10::cuda::CUDAGuard guard(table.device());
  MTAdamWArgs a;
  a.lr = static_cast<float>(lr);
  a.beta1 = static_cast<float>(beta1);
  a.beta2 = static_cast<float>(beta2);
  a.eps = static_cast<float>(eps);
  a.weight_decay = static_cast<float>(weight_decay);
  a.bias_correction1 = static_cast<float>(1.0 - std::pow(beta1, static_cast<double>(step)));
  a.bias_correction2_sqrt = static_cast<float>(std::sqrt(1.0 - std::pow(beta2, static_cast<double>(step))));
  a.grad_scale = f32_or_null(grad_scale, "grad_scale");
  if (has(skip)) {
    TORCH_CHECK(skip->scalar_type() == at::kInt && skip->is_cuda(), "mt_adamw: skip must be int32 on device");
    a.skip = skip->data_ptr<int>();
  }
  mt_adamw_launch(mt_chunks(chunks), static_cast<int>(chunks.size(0)), mt_rows(table), a, cur_stream());
}

// --------------------------------------------------------------------- peer memory
int64_t p2p_alloc_py(int64_t bytes, int64_t device) {
  return reinterpret_cast<int64_t>(p2p_alloc(static_cast<size_t>(bytes), static_cast<int>(device)));
}
void p2p_free_py(int64_t ptr) { p2p_free(reinterpret_cast<void*>(ptr)); }
py::bytes p2p_export_py(int64_t ptr) {
  char h[64];
  p2p_export(reinterpret_cast<void*>(ptr), h);
  return py::bytes(h, 64);
}
int64_t p2p_open_py(const py::bytes& handle, int64_t device) {
  const std::string h = handle;
  TORCH_CHECK(h.size() == 64, "p2p_open: a CUDA IPC handle is 64 bytes");
  return reinterpret_cast<int64_t>(p2p_open(h.data(), static_cast<int>(device)));
}
void p2p_close_py(int64_t ptr) { p2p_close(reinterpret_cast<void*>(ptr)); }
// A tensor viewing device memory this library manages (no ownership, no deleter).
at::Tensor tensor_at(int64_t ptr, const std::vector<int64_t>& sizes, at::ScalarType dtype, int64_t device) {
  auto opts = at::TensorOptions().dtype(dtype).device(at::kCUDA, static_cast<int>(device));
  return at::from_blob(reinterpret_cast<void*>(ptr), sizes, opts);
}
void stream_write_py(int64_t flag, int64_t value) {
  stream_write(cur_stream(), reinterpret_cast<void*>(flag), static_cast<unsigned>(value));
}
// dst = sum of the bf16 tensors whose device addresses `srcs` (int64 device tensor) holds,
// each with dst's element count.
void slab_sum(const at::Tensor& srcs, at::Tensor& dst) {
  c10::cuda::CUDAGuard guard(dst.device());
  check_bf16(dst, "slab_sum dst");
  TORCH_CHECK(dst.is_contiguous(), "slab_sum: dst must be contiguous");
  TORCH_CHECK(srcs.is_cuda() && srcs.scalar_type() == at::kLong && srcs.is_contiguous() && srcs.numel() > 0,
              "slab_sum: srcs must be a non-empty int64 device tensor of addresses");
  slab_sum_launch(reinterpret_cast<const void* const*>(srcs.data_ptr<int64_t>()), static_cast<int>(srcs.numel()),
                  dst.data_ptr(), dst.numel(), dst.device().index(), cur_stream());
}

void p2p_copy_py(int64_t dst, int64_t src, int64_t bytes) {
  p2p_copy(reinterpret_cast<void*>(dst), reinterpret_cast<const void*>(src), static_cast<size_t>(bytes), cur_stream());
}

int64_t read_error(int64_t device) {
  int v = 0;
  AVGEN_CUDA_CHECK(cudaMemcpy(&v, error_word(static_cast<int>(device)), sizeof(int), cudaMemcpyDeviceToHost));
  return v;
}

void clear_error(int64_t device) {
  AVGEN_CUDA_CHECK(cudaMemset(error_word(static_cast<int>(device)), 0, sizeof(int)));
}

}  // namespace

}  // namespace avgen

PYBIND11_MODULE(_C, m) {
  namespace a = avgen;
  using py::arg;
  auto none = py::none();
  m.doc() = "avgen_b200 sm_100a kernels";
  m.def("gemm", &a::gemm, arg("a"), arg("b"), arg("out"), arg("a_mn"), arg("b_mn"), arg("epilogue"),
        arg("bias") = none, arg("resid") = none, arg("gate") = none, arg("rows_per_batch") = 1, arg("aux") = none,
        arg("k_splits") = 1, arg("groups") = none, arg("a2") = none, arg("b2") = none, arg("gate_flags") = none,
        arg("gate_epoch") = 0, arg("gate_operand") = 0, arg("gate_chunk") = 0, arg("gate_rank") = 0);
  m.def("rmsnorm_mod_fwd", &a::rmsnorm_mod_fwd, arg("x"), arg("y"), arg("rstd") = none, arg("w") = none,
        arg("scale") = none, arg("shift") = none, arg("rows_per_batch") = 1, arg("eps") = 1e-6,
        arg("groups") = none);
  m.def("rmsnorm_mod_bwd", &a::rmsnorm_mod_bwd, arg("x"), arg("rstd"), arg("dy"), arg("dx") = none,
        arg("dres") = none, arg("w") = none, arg("scale") = none, arg("shift") = none, arg("dw") = none,
        arg("dscale") = none, arg("dshift") = none, arg("rows_per_batch") = 1, arg("groups") = none);
  m.def("gate_bwd", &a::gate_bwd, arg("dx"), arg("a"), arg("gate"), arg("da"), arg("dgate"), arg("rows_per_batch"),
        arg("groups") = none);
  m.def("qkv_rope_fwd", &a::qkv_rope_fwd, arg("qkv"), arg("B"), arg("L"), arg("H"), arg("Hk"), arg("D"), arg("eps"),
        arg("q_w") = none, arg("k_w") = none, arg("coords") = none, arg("freq") = none, arg("axis") = none,
        arg("q") = none, arg("k") = none, arg("v") = none);
  m.def("qkv_rope_bwd", &a::qkv_rope_bwd, arg("qkv"), arg("dqkv"), arg("B"), arg("L"), arg("H"), arg("Hk"), arg("D"),
        arg("eps"), arg("q_w") = none, arg("k_w") = none, arg("coords") = none, arg("freq") = none,
        arg("axis") = none, arg("dq") = none, arg("dk") = none, arg("dv") = none, arg("dq_w") = none,
        arg("dk_w") = none);
  m.def("swiglu_bwd", &a::swiglu_bwd);
  m.def("gelu_bwd", &a::gelu_bwd);
  m.def("flow_loss_fwd", &a::flow_loss_fwd);
  m.def("flow_loss_bwd", &a::flow_loss_bwd);
  m.def("noise_interp", &a::noise_interp, arg("clean"), arg("t"), arg("seed"), arg("offset"), arg("row_base"),
        arg("rows_per_sample"), arg("global_rows_per_sample"), arg("noisy"), arg("target"), arg("noise") = none);
  m.def("guided_euler", &a::guided_euler, arg("cond"), arg("uncond"), arg("x"), arg("sigma"), arg("sigma_next"),
        arg("scale"), arg("out"));
  m.def("sde_step", &a::sde_step, arg("v"), arg("x"), arg("sigma"), arg("sigma_next"), arg("g"), arg("floor"),
        arg("mean"), arg("log_prob"), arg("noise") = none, arg("prev") = none, arg("mask") = none,
        arg("sample") = none);
  m.def("adamw", &a::adamw, arg("param"), arg("grad"), arg("exp_avg"), arg("exp_avg_sq"), arg("lr"), arg("beta1"),
        arg("beta2"), arg("eps"), arg("weight_decay"), arg("step"), arg("param_bf16") = none,
        arg("grad_scale") = none, arg("skip") = none);
  m.def("sq_norm", &a::sq_norm);
  m.def("ema", &a::ema);
  m.def("attn_fwd", &a::attn_fwd, arg("q"), arg("k"), arg("v"), arg("out"), arg("lse") = none, arg("kmask") = none,
        arg("scale") = 0.0, arg("trace") = none, arg("ring_rank") = 0, arg("ring_flags") = none,
        arg("ring_epoch") = 0, arg("ring_wait") = none);
  m.def("shard_reduce", &a::shard_reduce, arg("grads"), arg("lo"), arg("out"), arg("sq_acc"));
  m.def("shard_adamw_push", &a::shard_adamw_push, arg("params"), arg("rank"), arg("lo"), arg("grad"),
        arg("exp_avg"), arg("exp_avg_sq"), arg("lr"), arg("beta1"), arg("beta2"), arg("eps"), arg("weight_decay"),
        arg("step"), arg("grad_scale") = none, arg("skip") = none);
  m.def("peer_reduce", &a::peer_reduce, arg("srcs"), arg("rank"), arg("offset"), arg("out"), arg("src_bf16"),
        arg("scale"), arg("sq_acc") = none);
  m.def("mt_sq_norm", &a::mt_sq_norm, arg("table"), arg("chunks"), arg("acc"));
  m.def("mt_adamw", &a::mt_adamw, arg("table"), arg("chunks"), arg("lr"), arg("beta1"), arg("beta2"), arg("eps"),
        arg("weight_decay"), arg("step"), arg("grad_scale") = none, arg("skip") = none);
  m.def("p2p_alloc", &a::p2p_alloc_py, arg("bytes"), arg("device"));
  m.def("p2p_free", &a::p2p_free_py);
  m.def("p2p_export", &a::p2p_export_py);
  m.def("p2p_open", &a::p2p_open_py, arg("handle"), arg("device"));
  m.def("p2p_close", &a::p2p_close_py);
  m.def("tensor_at", &a::tensor_at, arg("ptr"), arg("sizes"), arg("dtype"), arg("device"));
  m.def("stream_write", &a::stream_write_py, arg("flag"), arg("value"));
  m.def("p2p_copy", &a::p2p_copy_py, arg("dst"), arg("src"), arg("bytes"));
  m.def("attn_bwd", &a::attn_bwd, arg("q"), arg("k"), arg("v"), arg("o"), arg("dout"), arg("lse"), arg("delta"),
        arg("dq"), arg("dk"), arg("dv"), arg("kmask") = none, arg("scale") = 0.0, arg("dq_acc") = none,
        arg("trace") = none, arg("kt_begin") = 0, arg("kt_count") = 0, arg("skip_prologue") = false,
        arg("skip_epilogue") = false);
  m.def("slab_sum", &a::slab_sum, arg("srcs"), arg("dst"));
  m.def("install_crash_backtrace", &avgen::install_crash_backtrace,
        "print native frames on SIGSEGV/SIGBUS/SIGFPE/SIGILL/SIGABRT, then chain to the previous handler");
  m.def("read_error", &a::read_error);
  m.def("clear_error", &a::clear_error);
}
