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
int64_t g_launches = 0;   // kernels launched by this extension since import
int64_t launch_count() { return g_launches; }

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
          const c10::optional<Tensor>& act_scale, const c10::optional<Tensor>& amax_bits, int64_t max_ctas,
          const c10::optional<Tensor>& alpha2_t, const c10::optional<Tensor>& beta_t, const c10::optional<Tensor>& dot_out,
          bool symmetric) {
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
  g.alpha2_ptr = fptr(alpha2_t);
  g.beta_ptr = fptr(beta_t);
  g.dot_out = const_cast<float*>(fptr(dot_out));
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
  g.symmetric = symmetric;
  TORCH_CHECK(!symmetric || (epilogue == MNG_EPI_STORE && g.M == g.N && g.M % 128 == 0 && !g.row_scale && !g.col_scale),
              "symmetric: plain store epilogue, square output, a multiple of 128");
  g.stream = cur_stream();
  g.status = status_ptr(a);
  check(mng_gemm(&g), "mng_gemm");
  g_launches += 1;
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
  g_launches += 1;
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
  g_launches += 1;
  return dx;
}

// dx = rmsnorm backward(x, dy) + scale * addend in one pass; dot (fp32, one element) += sum(addend * x)
Tensor rmsnorm_bwd_add_scaled(const Tensor& x, const Tensor& dy, const c10::optional<Tensor>& rstd, const Tensor& addend,
                              const Tensor& scale, Tensor& dot) {
  TORCH_CHECK(x.is_contiguous() && dy.is_contiguous() && addend.is_contiguous() && x.scalar_type() == torch::kBFloat16 &&
              dy.scalar_type() == torch::kBFloat16 && addend.scalar_type() == torch::kBFloat16 && addend.numel() == x.numel());
  TORCH_CHECK(scale.scalar_type() == torch::kFloat32 && scale.numel() == 1 && dot.scalar_type() == torch::kFloat32 && dot.numel() >= 1);
  c10::cuda::CUDAGuard guard(x.device());
  const int cols = (int)x.size(-1);
  Tensor dx = torch::empty_like(x);
  check(mng_rmsnorm_bwd_add_scaled(x.data_ptr(), dy.data_ptr(), fptr(rstd), addend.data_ptr(), scale.data_ptr<float>(),
                                   dot.data_ptr<float>(), dx.data_ptr(), x.numel() / cols, cols, cur_stream()),
        "mng_rmsnorm_bwd_add_scaled");
  g_launches += 1;
  return dx;
}

// dx = rmsnorm backward(x, dy) + addend, in one pass
Tensor rmsnorm_bwd_add(const Tensor& x, const Tensor& dy, const c10::optional<Tensor>& rstd, const Tensor& addend) {
  TORCH_CHECK(x.is_contiguous() && dy.is_contiguous() && addend.is_contiguous() && x.scalar_type() == torch::kBFloat16 &&
              dy.scalar_type() == torch::kBFloat16 && addend.scalar_type() == torch::kBFloat16 && addend.numel() == x.numel());
  c10::cuda::CUDAGuard guard(x.device());
  const int cols = (int)x.size(-1);
  const int64_t rows = x.numel() / cols;
  Tensor dx = torch::empty_like(x);
  check(mng_rmsnorm_bwd_add(x.data_ptr(), dy.data_ptr(), fptr(rstd), addend.data_ptr(), dx.data_ptr(), rows, cols, cur_stream()),
        "mng_rmsnorm_bwd_add");
  g_launches += 1;
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
  g_launches += 1;
  return {q, s};
}

void transpose(const Tensor& src, Tensor& dst, bool accumulate) {
  TORCH_CHECK(src.dim() == 2 && dst.dim() == 2 && src.is_contiguous() && dst.is_contiguous());
  TORCH_CHECK(src.scalar_type() == torch::kBFloat16 && dst.scalar_type() == torch::kBFloat16);
  TORCH_CHECK(dst.size(0) == src.size(1) && dst.size(1) == src.size(0));
  c10::cuda::CUDAGuard guard(src.device());
  check(mng_transpose_bf16(src.data_ptr(), dst.data_ptr(), src.size(0), src.size(1), accumulate, cur_stream()), "mng_transpose_bf16");
  g_launches += 1;
}

Tensor transpose_u8(const Tensor& src) {
  TORCH_CHECK(src.is_cuda() && src.dim() == 2 && src.is_contiguous() && src.element_size() == 1);
  c10::cuda::CUDAGuard guard(src.device());
  Tensor dst = torch::empty({src.size(1), src.size(0)}, src.options());
  check(mng_transpose_u8(src.data_ptr(), dst.data_ptr(), src.size(0), src.size(1), cur_stream()), "mng_transpose_u8");
  g_launches += 1;
  return dst;
}

// q [cols, rows] e4m3 and scale [cols] of the transpose of src [rows, cols]; `scratch` is cols int32 words.
void quant_transpose(const Tensor& src, Tensor& q, Tensor& scale, Tensor& scratch) {
  TORCH_CHECK(src.dim() == 2 && src.is_contiguous() && src.scalar_type() == torch::kBFloat16);
  TORCH_CHECK(q.is_contiguous() && q.numel() == src.numel() && scale.numel() == src.size(1) && scratch.numel() >= src.size(1));
  c10::cuda::CUDAGuard guard(src.device());
  check(mng_quant_transpose_e4m3(src.data_ptr(), q.data_ptr(), scale.data_ptr<float>(),
                                 reinterpret_cast<unsigned int*>(scratch.data_ptr()), src.size(0), src.size(1), cur_stream()),
        "mng_quant_transpose_e4m3");
  g_launches += 2;
}

void mlp_weight_refresh(const Tensor& bank, Tensor& fc8, Tensor& fc_scale, Tensor& projT8, Tensor& projT_scale, Tensor& scratch,
                        Tensor& act_scale, Tensor& amax_bits, Tensor& used, Tensor& next, bool bootstrap) {
  TORCH_CHECK(bank.is_cuda() && bank.dim() == 4 && bank.size(1) == 2 && bank.is_contiguous() && bank.scalar_type() == torch::kBFloat16);
  const int64_t L = bank.size(0), hid = bank.size(2), dim = bank.size(3);
  TORCH_CHECK(fc8.is_contiguous() && fc8.numel() == L * hid * dim && fc8.element_size() == 1);
  TORCH_CHECK(projT8.is_contiguous() && projT8.numel() == L * hid * dim && projT8.element_size() == 1);
  TORCH_CHECK(fc_scale.is_contiguous() && fc_scale.numel() == L * hid && fc_scale.scalar_type() == torch::kFloat32);
  TORCH_CHECK(projT_scale.is_contiguous() && projT_scale.numel() == L * dim && projT_scale.scalar_type() == torch::kFloat32);
  TORCH_CHECK(scratch.is_contiguous() && scratch.numel() >= L * dim && scratch.element_size() == 4);
  TORCH_CHECK(act_scale.numel() == L && amax_bits.numel() == L && used.numel() >= L && next.numel() >= L);
  TORCH_CHECK(act_scale.is_contiguous() && amax_bits.is_contiguous() && used.is_contiguous() && next.is_contiguous());
  TORCH_CHECK(used.scalar_type() == torch::kFloat32 && next.scalar_type() == torch::kFloat32 && act_scale.scalar_type() == torch::kFloat32);
  c10::cuda::CUDAGuard guard(bank.device());
  check(mng_mlp_weight_refresh(bank.data_ptr(), (int)L, (int)hid, (int)dim, fc8.data_ptr(), fc_scale.data_ptr<float>(), projT8.data_ptr(),
                               projT_scale.data_ptr<float>(), reinterpret_cast<unsigned int*>(scratch.data_ptr()),
                               act_scale.data_ptr<float>(), reinterpret_cast<unsigned int*>(amax_bits.data_ptr()),
                               used.data_ptr<float>(), next.data_ptr<float>(), bootstrap ? 1 : 0, cur_stream()),
        "mng_mlp_weight_refresh");
  g_launches += 4;
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
  g_launches += 1;
  return {losses, dl};
}

// (q [rows, cols], qT [cols, rows]) saturating e4m3 of src / scale; either output on request
std::vector<Tensor> quant_static_dual(const Tensor& src, double scale, bool want_plain, bool want_t) {
  TORCH_CHECK(src.is_cuda() && src.dim() == 2 && src.is_contiguous() && src.scalar_type() == torch::kBFloat16);
  c10::cuda::CUDAGuard guard(src.device());
  Tensor q, qT;
  if (want_plain) q = torch::empty(src.sizes(), src.options().dtype(torch::kFloat8_e4m3fn));
  if (want_t) qT = torch::empty({src.size(1), src.size(0)}, src.options().dtype(torch::kFloat8_e4m3fn));
  check(mng_quant_static_dual(src.data_ptr(), want_plain ? q.data_ptr() : nullptr, want_t ? qT.data_ptr() : nullptr, src.size(0),
                              src.size(1), (float)scale, cur_stream()),
        "mng_quant_static_dual");
  g_launches += 1;
  return {q, qT};
}

// losses [T] fp32, dlogits [T, V] e5m2 from x8 [T, K] and wT8 [V, K] (e4m3, logit = acc * alpha)
std::vector<Tensor> lmhead_ce_fused(const Tensor& x8, const Tensor& wT8, double alpha, const Tensor& targets, const Tensor& mtp_weights,
                                    const c10::optional<Tensor>& prefix_targets, const c10::optional<Tensor>& prefix_weight,
                                    double A, double B, double C, double grad_mul) {
  TORCH_CHECK(x8.is_cuda() && x8.dim() == 2 && x8.is_contiguous() && x8.scalar_type() == torch::kFloat8_e4m3fn);
  TORCH_CHECK(wT8.dim() == 2 && wT8.is_contiguous() && wT8.scalar_type() == torch::kFloat8_e4m3fn && wT8.size(1) == x8.size(1));
  TORCH_CHECK(targets.scalar_type() == torch::kInt64 && targets.is_contiguous() && targets.numel() == x8.size(0));
  TORCH_CHECK(mtp_weights.scalar_type() == torch::kFloat32 && mtp_weights.is_contiguous());
  c10::cuda::CUDAGuard guard(x8.device());
  const int64_t T = x8.size(0), V = wT8.size(0), K = x8.size(1);
  const long long* pt = nullptr;
  if (prefix_targets.has_value() && prefix_targets->defined()) {
    TORCH_CHECK(prefix_targets->scalar_type() == torch::kInt64 && prefix_targets->is_contiguous() && prefix_targets->numel() == T);
    pt = reinterpret_cast<const long long*>(prefix_targets->data_ptr<int64_t>());
  }
  auto f32 = x8.options().dtype(torch::kFloat32);
  Tensor losses = torch::empty({T}, f32);
  Tensor dl = torch::empty({T, V}, x8.options().dtype(torch::kFloat8_e5m2));
  const int64_t slabs = (V + 127) / 128;
  Tensor slab = torch::empty({T * slabs}, f32), ztgt = torch::zeros({T * 4}, f32), rowc = torch::empty({T}, f32);
  check(mng_lmhead_ce_fused(x8.data_ptr(), wT8.data_ptr(), (int)T, (int)V, (int)K, (float)alpha,
                            reinterpret_cast<const long long*>(targets.data_ptr<int64_t>()), mtp_weights.data_ptr<float>(),
                            (int)mtp_weights.numel(), pt, fptr(prefix_weight), (float)A, (float)B, (float)C, (float)grad_mul,
                            losses.data_ptr<float>(), dl.data_ptr(), slab.data_ptr<float>(), ztgt.data_ptr<float>(),
                            rowc.data_ptr<float>(), cur_stream(), status_ptr(x8)),
        "mng_lmhead_ce_fused");
  g_launches += 3;
  return {losses, dl};
}

PeerPtrs peers_from(const std::vector<int64_t>& ptrs, int64_t self, int64_t mc = 0) {
  PeerPtrs p{};
  p.mc = reinterpret_cast<void*>(mc);
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
          double grad_mul, const c10::optional<Tensor>& row_mask, int64_t row_elems, int64_t grad_mc, int64_t param_mc) {
  c10::cuda::CUDAGuard guard(exp_avg.device());
  AdamDesc d{};
  if (row_mask.has_value() && row_mask->defined()) {        // [ranks, rows] uint8 in local memory
    TORCH_CHECK(row_mask->dim() == 2 && row_mask->is_contiguous() && row_mask->scalar_type() == torch::kUInt8 &&
                row_mask->size(0) == (int64_t)grad_ptrs.size() && row_mask->is_cuda());
    TORCH_CHECK(row_elems > 0 && (off + n + row_elems - 1) / row_elems <= row_mask->size(1));
    d.row_mask = row_mask->data_ptr<uint8_t>();
    d.mask_stride = row_mask->size(1);
    d.row_elems = (int)row_elems;
  }
  d.grads = peers_from(grad_ptrs, grad_ptrs.size() == 1 ? 0 : self, grad_mc);
  d.params = peers_from(param_ptrs, param_ptrs.size() == 1 ? 0 : self, param_mc);
  d.off = off;
  d.exp_avg = exp_avg.data_ptr<float>();
  d.exp_avg_sq = exp_avg_sq.data_ptr<float>();
  d.n = n;
  d.p_is_f32 = p_is_f32;
  d.beta1 = (float)beta1; d.beta2 = (float)beta2; d.eps = (float)eps;
  d.step_size = (float)step_size; d.eff_wd = (float)eff_wd; d.grad_mul = (float)grad_mul;
  TORCH_CHECK(exp_avg.numel() >= n && exp_avg_sq.numel() >= n);
  check(mng_adam(&d, cur_stream()), "mng_adam");
  g_launches += 1;
}

// A batch of small replicated parameters in one launch.  base_ptrs: the address of the buffer holding them on every rank
// (p_offs / g_offs are byte offsets from it), or [0] with absolute addresses as offsets.  hyper: beta1, beta2, eps,
// step_size, eff_wd per entry.
void adam_small(const std::vector<int64_t>& base_ptrs, int64_t self, const std::vector<int64_t>& p_offs,
                const std::vector<int64_t>& g_offs, std::vector<Tensor>& ms, std::vector<Tensor>& vs, const std::vector<int64_t>& ns,
                const std::vector<int64_t>& is_f32, const std::vector<double>& hyper, double grad_mul) {
  const size_t k = p_offs.size();
  TORCH_CHECK(k >= 1 && g_offs.size() == k && ms.size() == k && vs.size() == k && ns.size() == k && is_f32.size() == k &&
              hyper.size() == 5 * k);
  c10::cuda::CUDAGuard guard(ms[0].device());
  for (size_t lo = 0; lo < k; lo += MNG_SMALL_ADAM_MAX) {
    SmallAdamTable t{};
    t.base = peers_from(base_ptrs, base_ptrs.size() == 1 ? 0 : self);
    t.gmul = (float)grad_mul;
    t.count = (int)std::min<size_t>(MNG_SMALL_ADAM_MAX, k - lo);
    for (int i = 0; i < t.count; ++i) {
      const size_t j = lo + i;
      TORCH_CHECK(ms[j].is_cuda() && ms[j].scalar_type() == torch::kFloat32 && ms[j].is_contiguous() && ms[j].numel() >= ns[j]);
      TORCH_CHECK(vs[j].is_cuda() && vs[j].scalar_type() == torch::kFloat32 && vs[j].is_contiguous() && vs[j].numel() >= ns[j]);
      t.e[i] = SmallAdamEntry{p_offs[j], g_offs[j], ms[j].data_ptr<float>(), vs[j].data_ptr<float>(), ns[j], (int)is_f32[j],
                              (float)hyper[5 * j], (float)hyper[5 * j + 1], (float)hyper[5 * j + 2], (float)hyper[5 * j + 3],
                              (float)hyper[5 * j + 4]};
    }
    check(mng_adam_small(&t, cur_stream()), "mng_adam_small");
    g_launches += 1;
  }
}

void fill_zero(Tensor& t) {
  TORCH_CHECK(t.is_cuda() && t.is_contiguous());
  c10::cuda::CUDAGuard guard(t.device());
  check(mng_fill_zero(t.data_ptr(), (long long)t.numel() * t.element_size(), cur_stream()), "mng_fill_zero");
}

void nesterov(const std::vector<int64_t>& grad_ptrs, int64_t self, int64_t off, Tensor& buf, Tensor& out, Tensor& sumsq,
              double momentum, double grad_mul, int64_t grad_mc) {
  TORCH_CHECK(buf.dim() == 3 && out.sizes() == buf.sizes() && buf.scalar_type() == torch::kFloat32 &&
              out.scalar_type() == torch::kBFloat16 && buf.is_contiguous() && out.is_contiguous() && sumsq.numel() == buf.size(0));
  c10::cuda::CUDAGuard guard(buf.device());
  PeerPtrs g = peers_from(grad_ptrs, grad_ptrs.size() == 1 ? 0 : self, grad_mc);
  check(mng_nesterov(&g, off, buf.data_ptr<float>(), out.data_ptr(), sumsq.data_ptr<float>(), buf.size(0),
                     buf.size(1) * buf.size(2), (float)momentum, (float)grad_mul, cur_stream()),
        "mng_nesterov");
  g_launches += 1;
}

void scale_by_norm(Tensor& x, const Tensor& sumsq) {
  TORCH_CHECK(x.dim() == 3 && x.is_contiguous() && x.scalar_type() == torch::kBFloat16 && sumsq.numel() == x.size(0));
  c10::cuda::CUDAGuard guard(x.device());
  check(mng_scale_by_norm(x.data_ptr(), sumsq.data_ptr<float>(), x.size(0), x.size(1) * x.size(2), cur_stream()), "mng_scale_by_norm");
  g_launches += 1;
}

void normuon_apply(const std::vector<int64_t>& param_ptrs, int64_t self, int64_t off, Tensor& mantissa, const Tensor& v,
                   Tensor& second_mom, Tensor& scratch, bool red_rows, double beta2, double eff_wd, double lr_base,
                   const Tensor& lr_mul_per_mat, int64_t param_mc) {
  TORCH_CHECK(v.dim() == 3 && v.is_contiguous() && v.scalar_type() == torch::kBFloat16 && mantissa.is_contiguous());
  TORCH_CHECK(mantissa.numel() == v.numel() && lr_mul_per_mat.numel() == v.size(0) && lr_mul_per_mat.is_cuda() &&
              lr_mul_per_mat.scalar_type() == torch::kFloat32);
  const int rows = (int)v.size(1), cols = (int)v.size(2);
  TORCH_CHECK(second_mom.numel() == v.size(0) * (red_rows ? rows : cols));
  TORCH_CHECK(scratch.scalar_type() == torch::kFloat32 && scratch.is_contiguous() &&
              scratch.numel() >= v.size(0) * ((red_rows ? rows : cols) + 65), "scratch: mats * (max(rows, cols) + 65) zeroed floats");
  c10::cuda::CUDAGuard guard(v.device());
  PeerPtrs p = peers_from(param_ptrs, param_ptrs.size() == 1 ? 0 : self, param_mc);
  check(mng_normuon_apply(&p, off, mantissa.data_ptr(), v.data_ptr(), second_mom.data_ptr<float>(), scratch.data_ptr<float>(),
                          v.size(0), rows, cols, red_rows, (float)beta2, (float)eff_wd, (float)lr_base,
                          lr_mul_per_mat.data_ptr<float>(), cur_stream()),
        "mng_normuon_apply");
  g_launches += 2;
}

void peer_barrier(const std::vector<int64_t>& pad_ptrs, int64_t rank, int64_t epoch, const Tensor& like) {
  c10::cuda::CUDAGuard guard(like.device());
  PeerPtrs p = peers_from(pad_ptrs, rank);
  check(mng_peer_barrier(&p, (int)rank, (uint32_t)epoch, status_ptr(like), cur_stream()), "mng_peer_barrier");
  g_launches += 1;
}

using OptT = c10::optional<Tensor>;

LinCombArgs make_lincomb(const std::vector<Tensor>& xs, const std::vector<OptT>& scalars, const std::vector<OptT>& gates,
                         const std::vector<int64_t>& cols, const std::vector<double>& addc) {
  const size_t k = xs.size();
  TORCH_CHECK(k >= 1 && k <= LC_MAX_TERMS && scalars.size() == k && gates.size() == k && cols.size() == k && addc.size() == k);
  LinCombArgs a{};
  a.k = (int)k;
  for (size_t j = 0; j < k; ++j) {
    TORCH_CHECK(xs[j].is_contiguous() && xs[j].scalar_type() == torch::kBFloat16 && xs[j].sizes() == xs[0].sizes());
    a.t[j].x = xs[j].data_ptr();
    if (scalars[j].has_value() && scalars[j]->defined()) {
      TORCH_CHECK(scalars[j]->scalar_type() == torch::kFloat32 && scalars[j]->numel() == 1);
      a.t[j].scalar = scalars[j]->data_ptr<float>();
    }
    if (gates[j].has_value() && gates[j]->defined()) {
      const Tensor& g = *gates[j];
      TORCH_CHECK(g.dim() == 2 && g.stride(1) == 1 && g.size(0) == xs[0].size(0) && cols[j] < g.size(1));
      TORCH_CHECK(g.scalar_type() == torch::kBFloat16 || g.scalar_type() == torch::kFloat32);
      a.t[j].gate = g.data_ptr();
      a.t[j].gate_stride = g.stride(0);
      a.t[j].gate_col = (int)cols[j];
      a.t[j].gate_bf16 = g.scalar_type() == torch::kBFloat16;
    }
    a.t[j].addc = (float)addc[j];
  }
  return a;
}

Tensor lincomb_fwd(const std::vector<Tensor>& xs, const std::vector<OptT>& scalars, const std::vector<OptT>& gates,
                   const std::vector<int64_t>& cols, const std::vector<double>& addc) {
  c10::cuda::CUDAGuard guard(xs[0].device());
  LinCombArgs a = make_lincomb(xs, scalars, gates, cols, addc);
  Tensor out = torch::empty_like(xs[0]);
  const int ncols = (int)xs[0].size(-1);
  check(mng_lincomb_fwd(&a, out.data_ptr(), xs[0].numel() / ncols, ncols, cur_stream()), "mng_lincomb_fwd");
  g_launches += 1;
  return out;
}

// need_dx[j]: allocate and return dx_j; dx_into[j] (optional): use that tensor for this term's gradient instead, adding
// to what it holds where dx_acc[j] (terms run in order, so a later term may add to what an earlier one of the same call wrote).
// dgates[j]: bf16 [rows, C] buffer (zeroed by the caller; may be shared between
// terms) written at column cols[j].  dscalars[j]: fp32 one-element accumulator (zeroed by the caller).
std::vector<Tensor> lincomb_bwd(const std::vector<Tensor>& xs, const std::vector<OptT>& scalars, const std::vector<OptT>& gates,
                                const std::vector<int64_t>& cols, const std::vector<double>& addc, const Tensor& gout,
                                const std::vector<bool>& need_dx, const std::vector<OptT>& dgates, const std::vector<OptT>& dscalars,
                                const std::vector<OptT>& dx_into, const std::vector<bool>& dx_acc) {
  c10::cuda::CUDAGuard guard(xs[0].device());
  LinCombArgs a = make_lincomb(xs, scalars, gates, cols, addc);
  TORCH_CHECK(gout.is_contiguous() && gout.scalar_type() == torch::kBFloat16 && gout.numel() == xs[0].numel());
  LinCombGrads g{};
  std::vector<Tensor> dxs;
  for (int j = 0; j < a.k; ++j) {
    Tensor dx;
    if (j < (int)dx_into.size() && dx_into[j].has_value() && dx_into[j]->defined()) {
      const Tensor& acc = *dx_into[j];
      TORCH_CHECK(acc.is_contiguous() && acc.scalar_type() == torch::kBFloat16 && acc.numel() == xs[j].numel());
      g.t[j].dx = acc.data_ptr();
      g.t[j].dx_accumulate = (j < (int)dx_acc.size() && dx_acc[j]) ? 1 : 0;
    } else if (need_dx[j]) {
      dx = torch::empty_like(xs[j]);
      g.t[j].dx = dx.data_ptr();
    }
    dxs.push_back(dx);
    if (dgates[j].has_value() && dgates[j]->defined()) {
      TORCH_CHECK(dgates[j]->scalar_type() == torch::kBFloat16 && dgates[j]->stride(1) == 1);
      g.t[j].dgate = dgates[j]->data_ptr();
      g.t[j].dgate_stride = dgates[j]->stride(0);
      g.t[j].dgate_col = (int)cols[j];
    }
    if (dscalars[j].has_value() && dscalars[j]->defined()) g.t[j].dscalar = dscalars[j]->data_ptr<float>();
  }
  const int ncols = (int)xs[0].size(-1);
  check(mng_lincomb_bwd(&a, &g, gout.data_ptr(), xs[0].numel() / ncols, ncols, cur_stream()), "mng_lincomb_bwd");
  g_launches += 1;
  return dxs;
}

const void* optr(const OptT& t) { return (t.has_value() && t->defined()) ? t->data_ptr() : nullptr; }

// qkv [T, 3*H*128] bf16 -> q, k, v [T, H, 128] (+ rstd_q, rstd_k [T*H]).  cos/sin fp32 [positions, 32].
std::vector<Tensor> qkv_post_fwd(const Tensor& qkv, const Tensor& cos_t, const Tensor& sin_t, const OptT& ve, const OptT& vgate,
                                 const OptT& vadd, int64_t H, bool paired, bool key_offset, bool split) {
  TORCH_CHECK(qkv.dim() == 2 && qkv.is_contiguous() && qkv.scalar_type() == torch::kBFloat16 && qkv.size(1) == 3 * H * 128);
  TORCH_CHECK(cos_t.scalar_type() == torch::kFloat32 && cos_t.is_contiguous() && cos_t.size(1) == 32 && sin_t.sizes() == cos_t.sizes());
  const int64_t T = qkv.size(0);
  TORCH_CHECK(cos_t.size(0) >= (paired ? 2 * T : T));
  c10::cuda::CUDAGuard guard(qkv.device());
  auto o = qkv.options();
  Tensor q = torch::empty({T, H, 128}, o), k = torch::empty({T, H, 128}, o), v = torch::empty({T, H, 128}, o);
  Tensor rq = torch::empty({T * H}, o.dtype(torch::kFloat32)), rk = torch::empty({T * H}, o.dtype(torch::kFloat32));
  int vstride = 0;
  if (vgate.has_value() && vgate->defined()) {
    TORCH_CHECK(vgate->scalar_type() == torch::kBFloat16 && vgate->stride(1) == 1 && vgate->size(1) >= H);
    vstride = (int)vgate->stride(0);
  }
  if (ve.has_value() && ve->defined()) TORCH_CHECK(ve->is_contiguous() && ve->numel() == T * H * 128 && ve->scalar_type() == torch::kBFloat16);
  if (vadd.has_value() && vadd->defined()) TORCH_CHECK(vadd->is_contiguous() && vadd->numel() == T * H * 128 && vadd->scalar_type() == torch::kBFloat16);
  check(mng_qkv_post_fwd(qkv.data_ptr(), cos_t.data_ptr<float>(), sin_t.data_ptr<float>(), optr(ve), optr(vgate), vstride,
                         optr(vadd), q.data_ptr(), k.data_ptr(), v.data_ptr(), rq.data_ptr<float>(), rk.data_ptr<float>(), T,
                         (int)H, paired, key_offset, split, cur_stream()),
        "mng_qkv_post_fwd");
  g_launches += 1;
  return {q, k, v, rq, rk};
}

// Returns d_qkv, d_ve (or undefined), d_vgate [T, H] bf16 (or undefined).
std::vector<Tensor> qkv_post_bwd(const Tensor& qkv, const Tensor& cos_t, const Tensor& sin_t, const Tensor& rq, const Tensor& rk,
                                 const Tensor& dq, const Tensor& dk, const Tensor& dv, const OptT& ve, const OptT& vgate,
                                 int64_t H, bool paired, bool key_offset, bool need_dve, bool need_dvgate, bool split) {
  const int64_t T = qkv.size(0);
  TORCH_CHECK(dq.is_contiguous() && dk.is_contiguous() && dv.is_contiguous());
  c10::cuda::CUDAGuard guard(qkv.device());
  Tensor dqkv = torch::empty_like(qkv), dve, dvg;
  const bool has_ve = ve.has_value() && ve->defined();
  if (has_ve && need_dve) dve = torch::empty({T, H * 128}, qkv.options());
  if (has_ve && need_dvgate) dvg = torch::empty({T, H}, qkv.options());
  int vstride = (vgate.has_value() && vgate->defined()) ? (int)vgate->stride(0) : 0;
  check(mng_qkv_post_bwd(qkv.data_ptr(), cos_t.data_ptr<float>(), sin_t.data_ptr<float>(), rq.data_ptr<float>(),
                         rk.data_ptr<float>(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), optr(ve), optr(vgate), vstride,
                         dqkv.data_ptr(), dve.defined() ? dve.data_ptr() : nullptr, dvg.defined() ? dvg.data_ptr() : nullptr,
                         (int)H, T, (int)H, paired, key_offset, split, cur_stream()),
        "mng_qkv_post_bwd");
  g_launches += 1;
  return {dqkv, dve, dvg};
}

// QKV projection with norm / rotary / key offset / value-embedding add in the GEMM epilogue.
// Returns q, k, v [T, H, 128], rstd_q, rstd_k [T*H], k_last [H, 64].
std::vector<Tensor> qkv_proj(const Tensor& x, const Tensor& w, const Tensor& lam, const Tensor& cos_t, const Tensor& sin_t,
                             const OptT& ve, const OptT& vgate, int64_t H, bool paired, bool key_offset) {
  TORCH_CHECK(x.is_cuda() && x.dim() == 2 && x.is_contiguous() && x.scalar_type() == torch::kBFloat16);
  TORCH_CHECK(w.dim() == 2 && w.is_contiguous() && w.scalar_type() == torch::kBFloat16 && w.size(0) == 3 * H * 128 && w.size(1) == x.size(1));
  TORCH_CHECK(cos_t.scalar_type() == torch::kFloat32 && cos_t.is_contiguous() && cos_t.size(1) == 32 && sin_t.sizes() == cos_t.sizes());
  const int64_t T = x.size(0);
  TORCH_CHECK(cos_t.size(0) >= (paired ? 2 * T : T));
  c10::cuda::CUDAGuard guard(x.device());
  auto o = x.options();
  Tensor q = torch::empty({T, H, 128}, o), k = torch::empty({T, H, 128}, o), v = torch::empty({T, H, 128}, o);
  Tensor rq = torch::empty({T * H}, o.dtype(torch::kFloat32)), rk = torch::empty({T * H}, o.dtype(torch::kFloat32));
  Tensor k_last = torch::zeros({H, 64}, o);
  int vstride = 0;
  if (vgate.has_value() && vgate->defined()) {
    TORCH_CHECK(vgate->scalar_type() == torch::kBFloat16 && vgate->stride(1) == 1 && vgate->size(1) >= H);
    vstride = (int)vgate->stride(0);
  }
  if (ve.has_value() && ve->defined()) TORCH_CHECK(ve->is_contiguous() && ve->numel() == T * H * 128 && ve->scalar_type() == torch::kBFloat16);
  check(mng_qkv_proj(x.data_ptr(), w.data_ptr(), (int)T, (int)x.size(1), (int)H, fptr(lam), cos_t.data_ptr<float>(),
                     sin_t.data_ptr<float>(), optr(ve), optr(vgate), vstride, q.data_ptr(), k.data_ptr(), v.data_ptr(),
                     rq.data_ptr<float>(), rk.data_ptr<float>(), k_last.data_ptr(), paired, key_offset, cur_stream(), status_ptr(x)),
        "mng_qkv_proj");
  g_launches += 1;
  return {q, k, v, rq, rk, k_last};
}

// d_qkv [T, 3*H*128], d_ve, d_vgate from the outputs of qkv_proj and the gradients of q, k, v.
std::vector<Tensor> qkv_post_bwd_from_out(const Tensor& q, const Tensor& k, const Tensor& k_last, const Tensor& cos_t,
                                          const Tensor& sin_t, const Tensor& rq, const Tensor& rk, const Tensor& dq,
                                          const Tensor& dk, const Tensor& dv, const OptT& ve, const OptT& vgate, int64_t H,
                                          bool paired, bool key_offset, bool need_dve, bool need_dvgate) {
  const int64_t T = q.size(0);
  TORCH_CHECK(q.is_contiguous() && k.is_contiguous() && dq.is_contiguous() && dk.is_contiguous() && dv.is_contiguous());
  c10::cuda::CUDAGuard guard(q.device());
  Tensor dqkv = torch::empty({T, 3 * H * 128}, q.options()), dve, dvg;
  const bool has_ve = ve.has_value() && ve->defined();
  if (has_ve && need_dve) dve = torch::empty({T, H * 128}, q.options());
  if (has_ve && need_dvgate) dvg = torch::empty({T, H}, q.options());
  int vstride = (vgate.has_value() && vgate->defined()) ? (int)vgate->stride(0) : 0;
  check(mng_qkv_post_bwd_from_out(q.data_ptr(), k.data_ptr(), k_last.data_ptr(), cos_t.data_ptr<float>(), sin_t.data_ptr<float>(),
                                  rq.data_ptr<float>(), rk.data_ptr<float>(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), optr(ve),
                                  optr(vgate), vstride, dqkv.data_ptr(), dve.defined() ? dve.data_ptr() : nullptr,
                                  dvg.defined() ? dvg.data_ptr() : nullptr, (int)H, T, (int)H, paired, key_offset, cur_stream()),
        "mng_qkv_post_bwd_from_out");
  g_launches += 1;
  return {dqkv, dve, dvg};
}

// alpha / gate: bf16 [T, >=H] views (row stride arbitrary, unit column stride) or None.
Tensor xsa_gate_fwd(const Tensor& y, const Tensor& v, const OptT& alpha, const OptT& gate) {
  TORCH_CHECK(y.dim() == 3 && y.size(2) == 128 && y.is_contiguous() && v.is_contiguous() && y.scalar_type() == torch::kBFloat16);
  c10::cuda::CUDAGuard guard(y.device());
  Tensor out = torch::empty_like(y);
  auto st = [](const OptT& t) { return (t.has_value() && t->defined()) ? (int)t->stride(0) : 0; };
  if (alpha.has_value() && alpha->defined()) TORCH_CHECK(alpha->scalar_type() == torch::kBFloat16 && alpha->stride(1) == 1);
  if (gate.has_value() && gate->defined()) TORCH_CHECK(gate->scalar_type() == torch::kBFloat16 && gate->stride(1) == 1);
  check(mng_xsa_gate_fwd(y.data_ptr(), v.data_ptr(), optr(alpha), st(alpha), optr(gate), st(gate), out.data_ptr(), y.size(0),
                         (int)y.size(1), cur_stream()),
        "mng_xsa_gate_fwd");
  g_launches += 1;
  return out;
}

// Returns dy, dv (undefined without alpha), dalpha [T,H], dgate [T,H] (undefined when absent).  da_into / dg_into
// (optional): [T,H] views with unit column stride, e.g. columns of a wider shared gradient buffer, written instead.
std::vector<Tensor> xsa_gate_bwd(const Tensor& y, const Tensor& v, const OptT& alpha, const OptT& gate, const Tensor& dout,
                                 const OptT& da_into, const OptT& dg_into) {
  c10::cuda::CUDAGuard guard(y.device());
  TORCH_CHECK(dout.is_contiguous());
  const int64_t T = y.size(0), H = y.size(1);
  const bool ha = alpha.has_value() && alpha->defined(), hg = gate.has_value() && gate->defined();
  Tensor dy = torch::empty_like(y), dv, da, dg;
  auto view_ok = [&](const Tensor& t) {
    return t.dim() == 2 && t.size(0) == T && t.size(1) == H && t.stride(1) == 1 && t.scalar_type() == torch::kBFloat16;
  };
  if (ha) {
    dv = torch::empty_like(v);
    if (da_into.has_value() && da_into->defined()) {
      TORCH_CHECK(view_ok(*da_into));
      da = *da_into;
    } else {
      da = torch::empty({T, H}, y.options());
    }
  }
  if (hg) {
    if (dg_into.has_value() && dg_into->defined()) {
      TORCH_CHECK(view_ok(*dg_into));
      dg = *dg_into;
    } else {
      dg = torch::empty({T, H}, y.options());
    }
  }
  auto st = [](const OptT& t) { return (t.has_value() && t->defined()) ? (int)t->stride(0) : 0; };
  check(mng_xsa_gate_bwd(y.data_ptr(), v.data_ptr(), optr(alpha), st(alpha), optr(gate), st(gate), dout.data_ptr(), dy.data_ptr(),
                         ha ? dv.data_ptr() : nullptr, ha ? da.data_ptr() : nullptr, ha ? (int)da.stride(0) : 0,
                         hg ? dg.data_ptr() : nullptr, hg ? (int)dg.stride(0) : 0,
                         T, (int)H, cur_stream()),
        "mng_xsa_gate_bwd");
  g_launches += 1;
  return {dy, dv, da, dg};
}

// S [H, T/128, 128, 256] fp32 -> P (same shape, bf16), a [T/128, 128, 256] bf16
std::vector<Tensor> dc_mix_fwd(const Tensor& S, const Tensor& w1, const Tensor& doc_start, int64_t window) {
  TORCH_CHECK(S.dim() == 4 && S.is_contiguous() && S.scalar_type() == torch::kFloat32 && S.size(2) == 128 && S.size(3) == 256);
  const int64_t H = S.size(0), T = S.size(1) * 128;
  TORCH_CHECK(w1.is_contiguous() && w1.scalar_type() == torch::kBFloat16 && w1.numel() == T * H);
  TORCH_CHECK(doc_start.is_contiguous() && doc_start.scalar_type() == torch::kInt32 && doc_start.numel() == T);
  c10::cuda::CUDAGuard guard(S.device());
  Tensor P = torch::empty(S.sizes(), S.options().dtype(torch::kBFloat16));
  Tensor a = torch::empty({S.size(1), 128, 256}, S.options().dtype(torch::kBFloat16));
  check(mng_dc_mix_fwd(S.data_ptr<float>(), w1.data_ptr(), doc_start.data_ptr<int>(), P.data_ptr(), a.data_ptr(), T, (int)H,
                       (int)window, cur_stream()),
        "mng_dc_mix_fwd");
  g_launches += 1;
  return {P, a};
}

// returns dS [H, T/128, 128, 256] bf16, g_w1, g_w2 [T, H] fp32
std::vector<Tensor> dc_mix_bwd(const Tensor& dM, const Tensor& P, const Tensor& a, const Tensor& w1, const Tensor& w2, double scale) {
  TORCH_CHECK(dM.is_contiguous() && dM.scalar_type() == torch::kFloat32 && P.is_contiguous() && a.is_contiguous());
  TORCH_CHECK(w1.is_contiguous() && w2.is_contiguous() && w2.scalar_type() == torch::kBFloat16);
  const int64_t H = dM.size(0), T = dM.size(1) * 128;
  c10::cuda::CUDAGuard guard(dM.device());
  Tensor dS = torch::empty(dM.sizes(), dM.options().dtype(torch::kBFloat16));
  Tensor g1 = torch::empty({T, H}, dM.options()), g2 = torch::empty({T, H}, dM.options());
  check(mng_dc_mix_bwd(dM.data_ptr<float>(), P.data_ptr(), a.data_ptr(), w1.data_ptr(), w2.data_ptr(), dS.data_ptr(),
                       g1.data_ptr<float>(), g2.data_ptr<float>(), T, (int)H, (float)scale, cur_stream()),
        "mng_dc_mix_bwd");
  g_launches += 1;
  return {dS, g1, g2};
}

// part [H, T/128, 256, 128] bf16 (windowed gradients) -> [T, H, 128]: own rows of a block plus the next block's look-back rows
Tensor dc_fold(const Tensor& part) {
  TORCH_CHECK(part.dim() == 4 && part.is_contiguous() && part.scalar_type() == torch::kBFloat16 && part.size(2) == 256 &&
              part.size(3) == 128);
  const int64_t H = part.size(0), T = part.size(1) * 128;
  c10::cuda::CUDAGuard guard(part.device());
  Tensor out = torch::empty({T, H, 128}, part.options());
  check(mng_dc_fold(part.data_ptr(), out.data_ptr(), T, (int)H, cur_stream()), "mng_dc_fold");
  g_launches += 1;
  return out;
}

// grad[sorted_ids[j], :] += g[perm[j], :]   (grad: bf16 [V, D] updated in place)
void embed_bwd(const Tensor& g, const Tensor& sorted_ids, const Tensor& perm, Tensor& grad) {
  TORCH_CHECK(g.dim() == 2 && g.is_contiguous() && g.scalar_type() == torch::kBFloat16);
  TORCH_CHECK(grad.dim() == 2 && grad.is_contiguous() && grad.scalar_type() == torch::kBFloat16 && grad.size(1) == g.size(1));
  TORCH_CHECK(sorted_ids.scalar_type() == torch::kInt64 && perm.scalar_type() == torch::kInt64 && sorted_ids.is_contiguous() &&
              perm.is_contiguous() && sorted_ids.numel() == g.size(0) && perm.numel() == g.size(0));
  c10::cuda::CUDAGuard guard(g.device());
  check(mng_embed_bwd(g.data_ptr(), reinterpret_cast<const long long*>(sorted_ids.data_ptr<int64_t>()),
                      reinterpret_cast<const long long*>(perm.data_ptr<int64_t>()), grad.data_ptr(), g.size(0), (int)g.size(1),
                      grad.size(0), cur_stream()),
        "mng_embed_bwd");
  g_launches += 1;
}

std::vector<Tensor> attn_fwd(const Tensor& q, const Tensor& k, const Tensor& v, const Tensor& doc_start, int64_t window,
                             double scale) {
  TORCH_CHECK(q.is_cuda() && q.dim() == 3 && q.size(2) == 128 && q.scalar_type() == torch::kBFloat16);
  TORCH_CHECK(k.sizes() == q.sizes() && v.sizes() == q.sizes() && k.scalar_type() == q.scalar_type() && v.scalar_type() == q.scalar_type());
  for (const Tensor* t : {&q, &k, &v}) TORCH_CHECK(t->stride(2) == 1 && t->stride(1) == 128 && t->stride(0) == q.stride(0));
  TORCH_CHECK(doc_start.scalar_type() == torch::kInt32 && doc_start.is_contiguous() && doc_start.numel() == q.size(0));
  c10::cuda::CUDAGuard guard(q.device());
  const int64_t T = q.size(0), H = q.size(1);
  Tensor out = torch::empty({T, H, 128}, q.options());
  Tensor lse = torch::empty({H, T}, q.options().dtype(torch::kFloat32));
  check(mng_attn_fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), doc_start.data_ptr<int>(), out.data_ptr(), lse.data_ptr<float>(),
                     (int)T, (int)H, q.stride(0), (int)window, (float)scale, cur_stream(), status_ptr(q)),
        "mng_attn_fwd");
  g_launches += 1;
  return {out, lse};
}

std::vector<Tensor> attn_bwd(const Tensor& dout, const Tensor& q, const Tensor& k, const Tensor& v, const Tensor& out,
                             const Tensor& lse, const Tensor& doc_start, const Tensor& doc_end, int64_t window, double scale) {
  TORCH_CHECK(q.is_cuda() && q.dim() == 3 && q.size(2) == 128 && q.scalar_type() == torch::kBFloat16);
  for (const Tensor* t : {&q, &k, &v})
    TORCH_CHECK(t->sizes() == q.sizes() && t->stride(2) == 1 && t->stride(1) == 128 && t->stride(0) == q.stride(0));
  TORCH_CHECK(out.is_contiguous() && dout.is_contiguous() && out.sizes() == q.sizes() && dout.sizes() == q.sizes());
  TORCH_CHECK(dout.scalar_type() == torch::kBFloat16 && out.scalar_type() == torch::kBFloat16);
  const int64_t T = q.size(0), H = q.size(1);
  TORCH_CHECK(lse.scalar_type() == torch::kFloat32 && lse.is_contiguous() && lse.size(0) == H && lse.size(1) == T);
  TORCH_CHECK(doc_start.scalar_type() == torch::kInt32 && doc_start.is_contiguous() && doc_start.numel() == T);
  TORCH_CHECK(doc_end.scalar_type() == torch::kInt32 && doc_end.is_contiguous() && doc_end.numel() == T);
  c10::cuda::CUDAGuard guard(q.device());
  Tensor dq = torch::empty({T, H, 128}, q.options()), dk = torch::empty({T, H, 128}, q.options()),
         dv = torch::empty({T, H, 128}, q.options());
  Tensor scratch = torch::empty({2, H, T}, q.options().dtype(torch::kFloat32));
  check(mng_attn_bwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), dout.data_ptr(), lse.data_ptr<float>(),
                     doc_start.data_ptr<int>(), doc_end.data_ptr<int>(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(),
                     scratch.data_ptr<float>(), scratch.data_ptr<float>() + H * T, (int)T, (int)H, q.stride(0), (int)window,
                     (float)scale, cur_stream(), status_ptr(q)),
        "mng_attn_bwd");
  g_launches += 3;
  return {dq, dk, dv};
}

// Folds the split-K partial products of a bank-backed linear layer's weight gradient: grad slices += lam * dW,
// returns dlam = <dW, W> as a 0-dim fp32 tensor.
Tensor g_bank_counter;   // one zero word per device, left at zero by every launch
Tensor bank_grad_acc(const Tensor& parts, const Tensor& W, const Tensor& lam, Tensor& g0, const c10::optional<Tensor>& g1) {
  TORCH_CHECK(parts.is_cuda() && parts.scalar_type() == torch::kFloat32 && parts.is_contiguous() && parts.dim() == 3);
  TORCH_CHECK(W.scalar_type() == torch::kBFloat16 && W.is_contiguous() && W.numel() == parts.size(1) * parts.size(2));
  TORCH_CHECK(lam.scalar_type() == torch::kFloat32 && lam.numel() == 1 && lam.is_cuda());
  TORCH_CHECK(g0.scalar_type() == torch::kBFloat16 && g0.is_contiguous());
  c10::cuda::CUDAGuard guard(parts.device());
  const int64_t n = W.numel(), n0 = g0.numel();
  void* p1 = nullptr;
  if (g1.has_value() && g1->defined()) {
    TORCH_CHECK(g1->scalar_type() == torch::kBFloat16 && g1->is_contiguous() && n0 + g1->numel() == n);
    p1 = g1->data_ptr();
  } else {
    TORCH_CHECK(n0 == n, "gradient slices do not cover the weight");
  }
  if (!g_bank_counter.defined() || g_bank_counter.device() != parts.device())
    g_bank_counter = torch::zeros({1}, torch::dtype(torch::kInt32).device(parts.device()));
  Tensor partials = torch::empty({MNG_BANK_GRAD_BLOCKS}, parts.options());
  Tensor dlam = torch::empty({}, parts.options());
  check(mng_bank_grad_acc(parts.data_ptr<float>(), (int)parts.size(0), n, W.data_ptr(), lam.data_ptr<float>(), g0.data_ptr(), n0,
                          p1, partials.data_ptr<float>(), reinterpret_cast<unsigned int*>(g_bank_counter.data_ptr<int32_t>()),
                          dlam.data_ptr<float>(), cur_stream()),
        "mng_bank_grad_acc");
  g_launches += 1;
  return dlam;
}

// Tail of the gate / MUDD MLPs (gatemlp.cu): out = (gelu(pre) W2^T + b2) * scale.
Tensor gate_tail_fwd(const Tensor& pre, const Tensor& W2, const Tensor& b2, const c10::optional<Tensor>& scale_t, double scale_c) {
  TORCH_CHECK(pre.is_cuda() && pre.scalar_type() == torch::kBFloat16 && pre.is_contiguous() && pre.dim() == 2 && pre.size(1) == 64);
  TORCH_CHECK(W2.scalar_type() == torch::kBFloat16 && W2.dim() == 2 && W2.size(1) == 64 && W2.stride(1) == 1 && W2.size(0) <= 48);
  TORCH_CHECK(b2.scalar_type() == torch::kBFloat16 && b2.is_contiguous() && b2.numel() == W2.size(0));
  c10::cuda::CUDAGuard guard(pre.device());
  const int n = (int)W2.size(0);
  Tensor out = torch::empty({pre.size(0), n}, pre.options());
  check(mng_gate_tail_fwd(pre.data_ptr(), W2.data_ptr(), W2.stride(0), b2.data_ptr(), fptr(scale_t), (float)scale_c, out.data_ptr(),
                          pre.size(0), n, cur_stream()),
        "mng_gate_tail_fwd");
  g_launches += 1;
  return out;
}

std::vector<Tensor> gate_tail_bwd(const Tensor& pre, const Tensor& W2, const Tensor& b2, const c10::optional<Tensor>& scale_t,
                                  double scale_c, const Tensor& dout) {
  TORCH_CHECK(pre.is_cuda() && pre.scalar_type() == torch::kBFloat16 && pre.is_contiguous() && pre.dim() == 2 && pre.size(1) == 64);
  TORCH_CHECK(W2.scalar_type() == torch::kBFloat16 && W2.dim() == 2 && W2.size(1) == 64 && W2.stride(1) == 1 && W2.size(0) <= 48);
  TORCH_CHECK(b2.scalar_type() == torch::kBFloat16 && b2.is_contiguous() && b2.numel() == W2.size(0));
  const int n = (int)W2.size(0);
  TORCH_CHECK(dout.scalar_type() == torch::kBFloat16 && dout.dim() == 2 && dout.size(0) == pre.size(0) && dout.size(1) == n &&
              dout.stride(1) == 1);
  c10::cuda::CUDAGuard guard(pre.device());
  Tensor dpre = torch::empty_like(pre);
  Tensor dW2 = torch::empty({n, 64}, pre.options());
  Tensor db2 = torch::empty({n}, pre.options());
  Tensor dscale = torch::empty({}, pre.options().dtype(torch::kFloat32));
  Tensor partials = torch::empty({(int64_t)MNG_GATE_TAIL_BLOCKS * (n * 64 + n + 1)}, pre.options().dtype(torch::kFloat32));
  check(mng_gate_tail_bwd(pre.data_ptr(), W2.data_ptr(), W2.stride(0), b2.data_ptr(), fptr(scale_t), (float)scale_c, dout.data_ptr(),
                          dout.stride(0), dpre.data_ptr(), partials.data_ptr<float>(), dW2.data_ptr(), 64, db2.data_ptr(),
                          dscale.data_ptr<float>(), pre.size(0), n, cur_stream()),
        "mng_gate_tail_bwd");
  g_launches += 2;
  return {dpre, dW2, db2, dscale};
}

// Debug build only: the largest source line at which a kernel saw an out-of-range index since the last call (0 = none).
int64_t bounds_status() {
  cudaDeviceSynchronize();
  unsigned int v = 0;
  for (unsigned int w : {mng_bounds_embed(), mng_bounds_glue(), mng_bounds_dc(), mng_bounds_optim()}) v = w > v ? w : v;
  return (int64_t)v;
}
bool bounds_checked_build() {
#ifdef MNG_BOUNDS_CHECK
  return true;
#else
  return false;
#endif
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
  m.def("rmsnorm_bwd_add", &rmsnorm_bwd_add);
  m.def("rmsnorm_bwd_add_scaled", &rmsnorm_bwd_add_scaled);
  m.def("quant_rows", &quant_rows);
  m.def("transpose", &transpose);
  m.def("quant_transpose", &quant_transpose);
  m.def("transpose_u8", &transpose_u8);
  m.def("softcap_ce", &softcap_ce);
  m.def("quant_static_dual", &quant_static_dual);
  m.def("lmhead_ce_fused", &lmhead_ce_fused);
  m.def("adam", &adam);
  m.def("adam_small", &adam_small);
  m.def("fill_zero", &fill_zero);
  m.def("nesterov", &nesterov);
  m.def("scale_by_norm", &scale_by_norm);
  m.def("normuon_apply", &normuon_apply);
  m.def("peer_barrier", &peer_barrier);
  m.def("lincomb_fwd", &lincomb_fwd);
  m.def("lincomb_bwd", &lincomb_bwd);
  m.def("qkv_post_fwd", &qkv_post_fwd);
  m.def("qkv_post_bwd", &qkv_post_bwd);
  m.def("qkv_proj", &qkv_proj);
  m.def("qkv_post_bwd_from_out", &qkv_post_bwd_from_out);
  m.def("xsa_gate_fwd", &xsa_gate_fwd);
  m.def("xsa_gate_bwd", &xsa_gate_bwd);
  m.def("embed_bwd", &embed_bwd);
  m.def("dc_mix_fwd", &dc_mix_fwd);
  m.def("dc_mix_bwd", &dc_mix_bwd);
  m.def("dc_fold", &dc_fold);
  m.def("attn_fwd", &attn_fwd);
  m.def("attn_bwd", &attn_bwd);
  m.def("mlp_weight_refresh", &mlp_weight_refresh);
  m.def("bank_grad_acc", &bank_grad_acc);
  m.def("gate_tail_fwd", &gate_tail_fwd);
  m.def("gate_tail_bwd", &gate_tail_bwd);
  m.def("status_tensor", &status_tensor);
  m.def("bounds_status", &bounds_status);
  m.def("bounds_checked_build", &bounds_checked_build);
  m.def("launch_count", &launch_count);
}
