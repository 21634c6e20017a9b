// Python binding: turns torch tensors into the plain-C descriptors of api.h and launches on the
// current CUDA stream.  Allocation of outputs happens here (through the torch caching allocator),
// never inside the .cu files.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "api.h"

namespace {

using torch::Tensor;

Tensor g_status;   // one int32 word per device, lazily created

uint32_t* status_ptr(const Tensor& like) {
  if (!g_status.defined() || g_status.device() != like.device())
    g_status = torch::zeros({1}, torch::dtype(torch::kInt32).device(like.device()));
  return reinterpret_cast<uint32_t*>(g_status.data_ptr<int32_t>());
}

void* cur_stream() { return at::cuda::getCurrentCUDAStream().stream(); }

int dtype_code(const Tensor& t) {
  if (t.scalar_type() == torch::kBFloat16) return MNG_BF16;
  if (t.scalar_type() == torch::kFloat8_e4m3fn) return MNG_E4M3;
  if (t.scalar_type() == torch::kFloat8_e5m2) return MNG_E5M2;
  TORCH_CHECK(false, "gemm operands must be bf16, float8_e4m3fn or float8_e5m2");
}

const float* fptr(const c10::optional<Tensor>& t) {
  if (!t.has_value() || !t->defined()) return nullptr;
  TORCH_CHECK(t->scalar_type() == torch::kFloat32 && t->is_cuda() && t->is_contiguous());
  return t->data_ptr<float>();
}

void check(int rc, const char* what) { TORCH_CHECK(rc == 0, what, " failed with code ", rc); }

// D = epi(A * B^T).  a: [b?, M, K] (or [b?, K, M] when a_mn); b: [b?, N, K] (or [b?, K, N] when b_mn).
void gemm(const Tensor& a, const Tensor& b, Tensor& out, bool a_mn, bool b_mn, int64_t epilogue, int64_t bn, double alpha,
          double beta, const c10::optional<Tensor>& cin, const c10::optional<Tensor>& alpha_t,
          const c10::optional<Tensor>& row_scale, const c10::optional<Tensor>& col_scale, const c10::optional<Tensor>& out8,
          const c10::optional<Tensor>& act_scale, const c10::optional<Tensor>& amax_bits, int64_t max_ctas) {
  TORCH_CHECK(a.is_cuda() && b.is_cuda() && out.is_cuda());
  TORCH_CHECK(a.dim() == b.dim() && (a.dim() == 2 || a.dim() == 3) && out.dim() == a.dim());
  TORCH_CHECK(a.stride(-1) == 1 && b.stride(-1) == 1 && out.stride(-1) == 1, "innermost dims must be contiguous");
  c10::cuda::CUDAGuard guard(a.device());
  const bool batched = a.dim() == 3;
  GemmDesc g{};
  g.a = a.data_ptr();
  g.b = b.data_ptr();
  g.batch = batched ? (int)a.size(0) : 1;
  g.M = (int)(a_mn ? a.size(-1) : a.size(-2));
  g.K = (int)(a_mn ? a.size(-2) : a.size(-1));
  g.N = (int)(b_mn ? b.size(-1) : b.size(-2));
  TORCH_CHECK((b_mn ? b.size(-2) : b.size(-1)) == g.K, "K mismatch");
  TORCH_CHECK(out.size(-2) == g.M && out.size(-1) == g.N, "output shape mismatch");
  g.dtype_a = dtype_code(a);
  g.dtype_b = dtype_code(b);
  g.a_mn = a_mn;
  g.b_mn = b_mn;
  g.lda = a.stride(-2);
  g.ldb = b.stride(-2);
  g.a_bstride = batched ? a.stride(0) : 0;
  g.b_bstride = batched ? b.stride(0) : 0;
  g.epilogue = (int)epilogue;
  g.bn = (int)bn;
  g.out_f32 = out.scalar_type() == torch::kFloat32;
  TORCH_CHECK(g.out_f32 || out.scalar_type() == torch::kBFloat16);
  g.out = out.data_ptr();
  g.ldc = out.stride(-2);
  g.c_bstride = batched ? out.stride(0) : 0;
  if (cin.has_value() && cin->defined()) {
    TORCH_CHECK(cin->stride(-2) == out.stride(-2) && cin->stride(-1) == 1, "cin must share the output layout");
    TORCH_CHECK(epilogue == MNG_EPI_DPRE || cin->scalar_type() == out.scalar_type());
    if (batched) TORCH_CHECK(cin->stride(0) == out.stride(0));
    g.cin = cin->data_ptr();
  } else {
    TORCH_CHECK(beta == 0.0 && epilogue != MNG_EPI_DPRE, "beta / dpre need cin");
  }
  g.alpha = (float)alpha;
  g.beta = (float)beta;
  g.alpha_ptr = fptr(alpha_t);
  g.row_scale = fptr(row_scale);
  g.col_scale = fptr(col_scale);
  if (out8.has_value() && out8->defined()) {
    TORCH_CHECK(out8->scalar_type() == torch::kFloat8_e4m3fn && out8->stride(-2) == out.stride(-2));
    g.out8 = out8->data_ptr();
    TORCH_CHECK(act_scale.has_value() && amax_bits.has_value());
    g.amax_bits = reinterpret_cast<unsigned int*>(amax_bits->data_ptr());
  }
  g.act_scale = fptr(act_scale);
  g.max_ctas = (int)max_ctas;
  g.stream = cur_stream();
  g.status = status_ptr(a);
  check(mng_gemm(&g), "mng_gemm");
}

std::vector<Tensor> rmsnorm_fwd(const Tensor& x, bool want_y, bool want_fp8, bool want_rstd) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == torch::kBFloat16 && x.is_contiguous());
  c10::cuda::CUDAGuard guard(x.device());
  const int cols = (int)x.size(-1);
  const int64_t rows = x.numel() / cols;
  Tensor y, y8, scale, rstd;
  if (want_y) y = torch::empty_like(x);
  if (want_fp8) {
    y8 = torch::empty(x.sizes(), x.options().dtype(torch::kFloat8_e4m3fn));
    scale = torch::empty({rows}, x.options().dtype(torch::kFloat32));
  }
  if (want_rstd) rstd = torch::empty({rows}, x.options().dtype(torch::kFloat32));
  check(mng_rmsnorm_fwd(x.data_ptr(), want_y ? y.data_ptr() : nullptr, want_fp8 ? y8.data_ptr() : nullptr,
                        want_fp8 ? scale.data_ptr<float>() : nullptr, want_rstd ? rstd.data_ptr<float>() : nullptr, rows, cols,
                        cur_stream()),
        "mng_rmsnorm_fwd");
  return {y, y8, scale, rstd};
}

Tensor rmsnorm_bwd(const Tensor& x, const Tensor& dy, const c10::optional<Tensor>& rstd, const c10::optional<Tensor>& accum_into) {
  TORCH_CHECK(x.is_contiguous() && dy.is_contiguous() && x.scalar_type() == torch::kBFloat16 && dy.scalar_type() == torch::kBFloat16);
  c10::cuda::CUDAGuard guard(x.device());
  const int cols = (int)x.size(-1);
  const int64_t rows = x.numel() / cols;
  Tensor dx = (accum_into.has_value() && accum_into->defined()) ? *accum_into : torch::empty_like(x);
  TORCH_CHECK(dx.is_contiguous());
  check(mng_rmsnorm_bwd(x.data_ptr(), dy.data_ptr(), fptr(rstd), dx.data_ptr(), rows, cols,
                        (accum_into.has_value() && accum_into->defined()) ? 1 : 0, cur_stream()),
        "mng_rmsnorm_bwd");
  return dx;
}

std::vector<Tensor> quant_rows(const Tensor& x) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == torch::kBFloat16 && x.is_contiguous());
  c10::cuda::CUDAGuard guard(x.device());
  const int cols = (int)x.size(-1);
  const int64_t rows = x.numel() / cols;
  Tensor q = torch::empty(x.sizes(), x.options().dtype(torch::kFloat8_e4m3fn));
  Tensor s = torch::empty({rows}, x.options().dtype(torch::kFloat32));
  check(mng_quant_rows_e4m3(x.data_ptr(), q.data_ptr(), s.data_ptr<float>(), rows, cols, cur_stream()), "mng_quant_rows_e4m3");
  return {q, s};
}

void transpose(const Tensor& src, Tensor& dst, bool accumulate) {
  TORCH_CHECK(src.dim() == 2 && dst.dim() == 2 && src.is_contiguous() && dst.is_contiguous());
  TORCH_CHECK(src.scalar_type() == torch::kBFloat16 && dst.scalar_type() == torch::kBFloat16);
  TORCH_CHECK(dst.size(0) == src.size(1) && dst.size(1) == src.size(0));
  c10::cuda::CUDAGuard guard(src.device());
  check(mng_transpose_bf16(src.data_ptr(), dst.data_ptr(), src.size(0), src.size(1), accumulate, cur_stream()), "mng_transpose_bf16");
}

// q [cols, rows] e4m3 and scale [cols] of the transpose of src [rows, cols]; `scratch` is cols int32 words.
void quant_transpose(const Tensor& src, Tensor& q, Tensor& scale, Tensor& scratch) {
  TORCH_CHECK(src.dim() == 2 && src.is_contiguous() && src.scalar_type() == torch::kBFloat16);
  TORCH_CHECK(q.is_contiguous() && q.numel() == src.numel() && scale.numel() == src.size(1) && scratch.numel() >= src.size(1));
  c10::cuda::CUDAGuard guard(src.device());
  check(mng_quant_transpose_e4m3(src.data_ptr(), q.data_ptr(), scale.data_ptr<float>(),
                                 reinterpret_cast<unsigned int*>(scratch.data_ptr()), src.size(0), src.size(1), cur_stream()),
        "mng_quant_transpose_e4m3");
}

std::vector<Tensor> softcap_ce(const Tensor& logits, const Tensor& targets, const Tensor& mtp_weights,
                               const c10::optional<Tensor>& prefix_targets, const c10::optional<Tensor>& prefix_weight,
                               bool dlogits_e5m2, double A, double B, double C, double grad_mul) {
  TORCH_CHECK(logits.dim() == 2 && logits.scalar_type() == torch::kBFloat16 && logits.stride(1) == 1);
  TORCH_CHECK(targets.scalar_type() == torch::kInt64 && targets.is_contiguous() && mtp_weights.scalar_type() == torch::kFloat32);
  c10::cuda::CUDAGuard guard(logits.device());
  const int64_t rows = logits.size(0);
  const int vocab = (int)logits.size(1);
  TORCH_CHECK(logits.stride(0) == vocab, "logits must be dense");
  Tensor losses = torch::empty({rows}, logits.options().dtype(torch::kFloat32));
  Tensor dl = torch::empty({rows, vocab}, logits.options().dtype(dlogits_e5m2 ? torch::kFloat8_e5m2 : torch::kBFloat16));
  const long long* pt = nullptr;
  if (prefix_targets.has_value() && prefix_targets->defined()) {
    TORCH_CHECK(prefix_targets->scalar_type() == torch::kInt64 && prefix_targets->is_contiguous());
    pt = reinterpret_cast<const long long*>(prefix_targets->data_ptr<int64_t>());
  }
  check(mng_softcap_ce(logits.data_ptr(), reinterpret_cast<const long long*>(targets.data_ptr<int64_t>()),
                       mtp_weights.data_ptr<float>(), (int)mtp_weights.numel(), pt, fptr(prefix_weight),
                       losses.data_ptr<float>(), dl.data_ptr(), dlogits_e5m2, rows, vocab, vocab, (float)A, (float)B, (float)C,
                       (float)grad_mul, cur_stream()),
        "mng_softcap_ce");
  return {losses, dl};
}

PeerPtrs peers_from(const std::vector<int64_t>& ptrs, int64_t self) {
  PeerPtrs p{};
  TORCH_CHECK(ptrs.size() >= 1 && ptrs.size() <= MNG_MAX_RANKS && self >= 0 && self < (int64_t)ptrs.size());
  p.n = (int)ptrs.size();
  p.self = (int)self;
  for (size_t i = 0; i < ptrs.size(); ++i) p.p[i] = reinterpret_cast<void*>(ptrs[i]);
  return p;
}

// Adam on elements [off, off+n) of the flat parameter.  grad_ptrs / param_ptrs: addresses of the whole
// gradient / parameter buffers on each rank (length 1 = local only).
void adam(const std::vector<int64_t>& grad_ptrs, const std::vector<int64_t>& param_ptrs, int64_t self, int64_t off, Tensor& exp_avg,
          Tensor& exp_avg_sq, int64_t n, bool p_is_f32, double beta1, double beta2, double eps, double step_size, double eff_wd,
          double grad_mul) {
  c10::cuda::CUDAGuard guard(exp_avg.device());
  AdamDesc d{};
  d.grads = peers_from(grad_ptrs, grad_ptrs.size() == 1 ? 0 : self);
  d.params = peers_from(param_ptrs, param_ptrs.size() == 1 ? 0 : self);
  d.off = off;
  d.exp_avg = exp_avg.data_ptr<float>();
  d.exp_avg_sq = exp_avg_sq.data_ptr<float>();
  d.n = n;
  d.p_is_f32 = p_is_f32;
  d.beta1 = (float)beta1; d.beta2 = (float)beta2; d.eps = (float)eps;
  d.step_size = (float)step_size; d.eff_wd = (float)eff_wd; d.grad_mul = (float)grad_mul;
  TORCH_CHECK(exp_avg.numel() >= n && exp_avg_sq.numel() >= n);
  check(mng_adam(&d, cur_stream()), "mng_adam");
}

void nesterov(const std::vector<int64_t>& grad_ptrs, int64_t self, int64_t off, Tensor& buf, Tensor& out, Tensor& sumsq,
              double momentum, double grad_mul) {
  TORCH_CHECK(buf.dim() == 3 && out.sizes() == buf.sizes() && buf.scalar_type() == torch::kFloat32 &&
              out.scalar_type() == torch::kBFloat16 && buf.is_contiguous() && out.is_contiguous() && sumsq.numel() == buf.size(0));
  c10::cuda::CUDAGuard guard(buf.device());
  PeerPtrs g = peers_from(grad_ptrs, grad_ptrs.size() == 1 ? 0 : self);
  check(mng_nesterov(&g, off, buf.data_ptr<float>(), out.data_ptr(), sumsq.data_ptr<float>(), buf.size(0),
                     buf.size(1) * buf.size(2), (float)momentum, (float)grad_mul, cur_stream()),
        "mng_nesterov");
}

void scale_by_norm(Tensor& x, const Tensor& sumsq) {
  TORCH_CHECK(x.dim() == 3 && x.is_contiguous() && x.scalar_type() == torch::kBFloat16 && sumsq.numel() == x.size(0));
  c10::cuda::CUDAGuard guard(x.device());
  check(mng_scale_by_norm(x.data_ptr(), sumsq.data_ptr<float>(), x.size(0), x.size(1) * x.size(2), cur_stream()), "mng_scale_by_norm");
}

void normuon_apply(const std::vector<int64_t>& param_ptrs, int64_t self, int64_t off, Tensor& mantissa, const Tensor& v,
                   Tensor& second_mom, Tensor& scratch, bool red_rows, double beta2, double eff_wd, const Tensor& eff_lr_per_mat) {
  TORCH_CHECK(v.dim() == 3 && v.is_contiguous() && v.scalar_type() == torch::kBFloat16 && mantissa.is_contiguous());
  TORCH_CHECK(mantissa.numel() == v.numel() && eff_lr_per_mat.numel() == v.size(0));
  const int rows = (int)v.size(1), cols = (int)v.size(2);
  TORCH_CHECK(second_mom.numel() == v.size(0) * (red_rows ? rows : cols) && scratch.numel() >= second_mom.numel());
  c10::cuda::CUDAGuard guard(v.device());
  PeerPtrs p = peers_from(param_ptrs, param_ptrs.size() == 1 ? 0 : self);
  check(mng_normuon_apply(&p, off, mantissa.data_ptr(), v.data_ptr(), second_mom.data_ptr<float>(), scratch.data_ptr<float>(),
                          v.size(0), rows, cols, red_rows, (float)beta2, (float)eff_wd, eff_lr_per_mat.data_ptr<float>(),
                          cur_stream()),
        "mng_normuon_apply");
}

void peer_barrier(const std::vector<int64_t>& pad_ptrs, int64_t rank, int64_t epoch, const Tensor& like) {
  c10::cuda::CUDAGuard guard(like.device());
  PeerPtrs p = peers_from(pad_ptrs, rank);
  check(mng_peer_barrier(&p, (int)rank, (uint32_t)epoch, status_ptr(like), cur_stream()), "mng_peer_barrier");
}

Tensor status_tensor(const Tensor& like) {
  status_ptr(like);
  return g_status;
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("gemm", &gemm);
  m.def("rmsnorm_fwd", &rmsnorm_fwd);
  m.def("rmsnorm_bwd", &rmsnorm_bwd);
  m.def("quant_rows", &quant_rows);
  m.def("transpose", &transpose);
  m.def("quant_transpose", &quant_transpose);
  m.def("softcap_ce", &softcap_ce);
  m.def("adam", &adam);
  m.def("nesterov", &nesterov);
  m.def("scale_by_norm", &scale_by_norm);
  m.def("normuon_apply", &normuon_apply);
  m.def("peer_barrier", &peer_barrier);
  m.def("status_tensor", &status_tensor);
}
