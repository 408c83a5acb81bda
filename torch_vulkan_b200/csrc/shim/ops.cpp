// ATen operator shim: registers the hot-path operators for CUDA tensors and forwards them to the
// C ABI of libb2rt.so (include/b2rt.h). This is the B200 counterpart of the reference's
// TORCH_LIBRARY_IMPL(aten, PrivateUse1, ...) blocks:
//   mm/bmm/addmm/baddbmm            csrc/ops_mm.cpp:177-221
//   SDPA overrideable fwd/bwd       csrc/ops_attn.cpp:166-310 (+ the _fused_sdp_choice stub, 97-101)
//   _softmax/_safe_softmax/_softmax_backward_data, native_layer_norm[_backward]
//                                   csrc/ops_rows.cpp:59-181, 336-341
//   addcmul(_)/addcdiv(_)/lerp(_).Scalar   csrc/ops_ew.cpp:405-455, 537-542
//   b2::dequant_int8                csrc/shim.cpp:420-423 (torch_vulkan_C.dequant_int8)
// The wrappers only validate, compute strides and allocate outputs (at::empty on the current
// allocator); every launch is on the current CUDA stream. Registration is dynamic: set_enabled(false)
// destroys the registration object and PyTorch's own CUDA kernels come back (the A/B switch the
// reference offers per kernel family through set_coop_enabled / set_fused_attention).
// Cases a kernel does not cover (dtype outside f32/bf16/f16[/f64], > 8 broadcast dims) run the stock
// CUDA implementation through composite ATen ops and are counted as fallbacks; nothing runs on the CPU.
#include <ATen/ATen.h>
#include <ATen/Functions.h>
#include <ATen/SDPBackend.h>
#include <ATen/cuda/CUDAContext.h>
#include <ATen/native/transformers/attention.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

#include <atomic>
#include <cmath>
#include <cstdlib>
#include <memory>
#include <mutex>
#include <optional>
#include <string>
#include <vector>

#include "../../../include/b2rt.h"

namespace {

std::string b2_error() {
  char buf[1024];
  b2rt_last_error(buf, sizeof(buf));
  return std::string(buf);
}

void b2_check(int rc, const char* what) { TORCH_CHECK(rc == 0, "b200 ", what, " failed: ", b2_error()); }

void count(const char* name) { b2rt_count_op(name); }
void count_fallback(const std::string& name) { b2rt_count_op(("fallback:" + name).c_str()); }

b2_stream_t cur_stream() { return (b2_stream_t)at::cuda::getCurrentCUDAStream().stream(); }

int dtype_code(at::ScalarType t) {
  switch (t) {
    case at::kFloat: return B2_F32;
    case at::kBFloat16: return B2_BF16;
    case at::kHalf: return B2_F16;
    case at::kDouble: return B2_F64;
    default: return -1;
  }
}
bool is_row_dtype(at::ScalarType t) { return t == at::kFloat || t == at::kBFloat16 || t == at::kHalf; }

std::atomic<int> g_force_simt{0};     // bit0: gemm, bit1: attention
std::atomic<int> g_attn_policy{-1};  // 0 off, 1 on, 2 auto (-1: read the environment)

int attn_policy() {
  int p = g_attn_policy.load();
  if (p < 0) {
    p = 2;
    const char* n = std::getenv("B2_NO_FUSED_ATTN");
    const char* e = std::getenv("B2_FUSED_ATTN");
    if (n && n[0] && n[0] != '0') p = 0;
    else if (e && e[0]) p = e[0] == '0' ? 0 : 1;
    g_attn_policy.store(p);
  }
  return p;
}

// =============================== GEMM ==============================================================

// Strides of `bias` broadcast to `full` (batch?, M, N); false if not broadcastable.
bool bias_strides(const at::Tensor& bias, c10::IntArrayRef full, std::vector<int64_t>& st) {
  if (bias.dim() > (int64_t)full.size()) return false;
  st.assign(full.size(), 0);
  for (size_t i = 0; i < full.size(); ++i) {
    int64_t j = (int64_t)i - ((int64_t)full.size() - bias.dim());
    if (j < 0) continue;
    if (bias.size(j) == full[i]) st[i] = bias.stride(j);
    else if (bias.size(j) == 1) st[i] = 0;
    else return false;
  }
  return true;
}

// C = alpha * A @ B + beta * bias. Follows try_gemm (csrc/ops_mm.cpp:61-175).
at::Tensor run_gemm(const at::Tensor& a, const at::Tensor& b, const at::Tensor* bias, double alpha, double beta,
                    const char* name) {
  TORCH_CHECK(a.scalar_type() == b.scalar_type(), name, ": expected mat1 and mat2 to have the same dtype, but got: ",
              a.scalar_type(), " != ", b.scalar_type());
  const bool batched = a.dim() == 3;
  TORCH_CHECK(a.dim() == b.dim() && (a.dim() == 2 || batched), name, ": expected 2-D (or 3-D batched) tensors");
  const int64_t batch = batched ? a.size(0) : 1;
  const int off = batched ? 1 : 0;
  const int64_t M = a.size(off), K = a.size(off + 1), N = b.size(off + 1);
  TORCH_CHECK(b.size(off) == K, name, ": mat1 and mat2 shapes cannot be multiplied (", a.sizes(), " and ", b.sizes(), ")");
  if (batched) TORCH_CHECK(b.size(0) == batch, name, ": batch sizes differ");
  const int dt = dtype_code(a.scalar_type());
  at::Tensor out = batched ? at::empty({batch, M, N}, a.options()) : at::empty({M, N}, a.options());
  bool use_bias = bias != nullptr && beta != 0.0;
  std::vector<int64_t> bst;
  if (use_bias) {
    TORCH_CHECK(bias->scalar_type() == a.scalar_type(), name, ": bias dtype must match");
    TORCH_CHECK(bias_strides(*bias, out.sizes(), bst), name, ": bias of shape ", bias->sizes(),
                " is not broadcastable to ", out.sizes());
  }
  TORCH_CHECK(dt >= 0, name, " (b200): dtype ", a.scalar_type(), " is not supported");
  if (out.numel() == 0) return out;
  b2_gemm_args g{};
  g.a = a.data_ptr();
  g.b = b.data_ptr();
  g.c = out.data_ptr();
  g.M = M, g.N = N, g.K = K, g.batch = batch;
  g.a_sb = batched ? a.stride(0) : 0, g.a_sm = a.stride(off), g.a_sk = a.stride(off + 1);
  g.b_sb = batched ? b.stride(0) : 0, g.b_sk = b.stride(off), g.b_sn = b.stride(off + 1);
  g.c_sb = M * N, g.c_sm = N, g.c_sn = 1;
  // size-1 dims may carry arbitrary strides; normalise so the kernel sees a canonical layout
  if (M == 1) g.a_sm = K;
  if (K == 1) g.a_sk = 1, g.b_sk = N;
  if (N == 1) g.b_sn = 1;
  g.alpha = (float)alpha, g.beta = (float)beta;
  g.dtype = dt;
  g.has_bias = use_bias ? 1 : 0;
  if (use_bias) {
    g.bias = bias->data_ptr();
    g.bias_sb = batched ? bst[0] : 0;
    g.bias_sm = bst[off];
    g.bias_sn = bst[off + 1];
  }
  g.force_simt = (g_force_simt.load() & 1) ? 1 : 0;
  if (K == 0) {
    // empty reduction: C = beta * bias (or 0)
    if (use_bias) out.copy_(bias->expand(out.sizes()) * beta);
    else out.zero_();
    count(name);
    return out;
  }
  // split-K scratch (few output tiles, long K: the LoRA projections) from the caching allocator
  at::Tensor ws;
  if (const uint64_t wsb = b2_gemm_workspace_bytes(&g)) {
    ws = at::empty({(int64_t)wsb}, a.options().dtype(at::kByte));
    g.workspace = ws.data_ptr(), g.workspace_bytes = (int64_t)wsb;
  }
  b2_check(b2_gemm(&g, cur_stream()), name);
  count(name);
  return out;
}

bool gemm_supported(const at::Tensor& a, const at::Tensor& b) {
  return a.is_cuda() && b.is_cuda() && dtype_code(a.scalar_type()) >= 0 && a.scalar_type() == b.scalar_type() &&
         a.layout() == at::kStrided && b.layout() == at::kStrided;
}

at::Tensor k_mm(const at::Tensor& a, const at::Tensor& b) {
  c10::cuda::CUDAGuard guard(a.device());
  TORCH_CHECK(gemm_supported(a, b), "aten::mm (b200): unsupported operands ", a.scalar_type(), "/", b.scalar_type());
  return run_gemm(a, b, nullptr, 1.0, 0.0, "aten::mm");
}
at::Tensor k_bmm(const at::Tensor& a, const at::Tensor& b) {
  c10::cuda::CUDAGuard guard(a.device());
  TORCH_CHECK(gemm_supported(a, b), "aten::bmm (b200): unsupported operands ", a.scalar_type(), "/", b.scalar_type());
  return run_gemm(a, b, nullptr, 1.0, 0.0, "aten::bmm");
}
at::Tensor k_addmm(const at::Tensor& self, const at::Tensor& a, const at::Tensor& b, const at::Scalar& beta,
                   const at::Scalar& alpha) {
  c10::cuda::CUDAGuard guard(a.device());
  TORCH_CHECK(gemm_supported(a, b) && a.dim() == 2, "aten::addmm (b200): unsupported operands");
  return run_gemm(a, b, &self, alpha.toDouble(), beta.toDouble(), "aten::addmm");
}
at::Tensor k_baddbmm(const at::Tensor& self, const at::Tensor& a, const at::Tensor& b, const at::Scalar& beta,
                     const at::Scalar& alpha) {
  c10::cuda::CUDAGuard guard(a.device());
  TORCH_CHECK(gemm_supported(a, b) && a.dim() == 3, "aten::baddbmm (b200): unsupported operands");
  return run_gemm(a, b, &self, alpha.toDouble(), beta.toDouble(), "aten::baddbmm");
}

// =============================== softmax ===========================================================

void softmax_dims(const at::Tensor& t, int64_t dim, int64_t& outer, int64_t& R, int64_t& inner) {
  if (t.dim() == 0) {
    outer = R = inner = 1;
    return;
  }
  dim = c10::maybe_wrap_dim(dim, t.dim());
  outer = 1, inner = 1;
  for (int64_t d = 0; d < dim; ++d) outer *= t.size(d);
  for (int64_t d = dim + 1; d < t.dim(); ++d) inner *= t.size(d);
  R = t.size(dim);
}

at::Tensor softmax_impl(const at::Tensor& self, int64_t dim, at::ScalarType out_dt, bool safe, const char* name) {
  c10::cuda::CUDAGuard guard(self.device());
  if (!is_row_dtype(self.scalar_type()) || !is_row_dtype(out_dt)) {
    count_fallback(name);
    at::Tensor x = self.to(at::kDouble);
    at::Tensor y = (x - std::get<0>(x.max(dim, true))).exp();
    y = y / y.sum(dim, true);
    if (safe) y = at::where(self.isneginf().all(dim, true), at::zeros_like(y), y);
    return y.to(out_dt);
  }
  at::Tensor x = self.is_contiguous() ? self : self.contiguous();
  at::Tensor out = at::empty(x.sizes(), x.options().dtype(out_dt));
  if (x.numel() == 0) return out;
  b2_softmax_args s{};
  s.x = x.data_ptr();
  s.out = out.data_ptr();
  softmax_dims(x, dim, s.outer, s.R, s.inner);
  s.in_dtype = dtype_code(x.scalar_type());
  s.out_dtype = dtype_code(out_dt);
  s.safe = safe ? 1 : 0;
  b2_check(b2_softmax_fwd(&s, cur_stream()), name);
  count(name);
  return out;
}

at::Tensor k_softmax(const at::Tensor& self, int64_t dim, bool half_to_float) {
  at::ScalarType dt = half_to_float ? at::kFloat : self.scalar_type();
  return softmax_impl(self, dim, dt, false, "aten::_softmax");
}
at::Tensor k_safe_softmax(const at::Tensor& self, int64_t dim, std::optional<at::ScalarType> dtype) {
  return softmax_impl(self, dim, dtype.value_or(self.scalar_type()), true, "aten::_safe_softmax");
}
at::Tensor k_softmax_backward(const at::Tensor& g, const at::Tensor& y, int64_t dim, at::ScalarType input_dtype) {
  c10::cuda::CUDAGuard guard(y.device());
  const char* name = "aten::_softmax_backward_data";
  if (!is_row_dtype(y.scalar_type()) || !is_row_dtype(input_dtype) || !is_row_dtype(g.scalar_type())) {
    count_fallback(name);
    at::Tensor yd = y.to(at::kDouble), gd = g.to(at::kDouble);
    return (yd * (gd - (gd * yd).sum(dim, true))).to(input_dtype);
  }
  TORCH_CHECK(g.sizes() == y.sizes(), name, ": grad and output shapes differ");
  at::Tensor yc = y.is_contiguous() ? y : y.contiguous();
  at::Tensor gc = g.scalar_type() == y.scalar_type() ? g : g.to(y.scalar_type());
  if (!gc.is_contiguous()) gc = gc.contiguous();
  at::Tensor dx = at::empty(yc.sizes(), yc.options().dtype(input_dtype));
  if (yc.numel() == 0) return dx;
  b2_softmax_args s{};
  s.y = yc.data_ptr();
  s.g = gc.data_ptr();
  s.out = dx.data_ptr();
  softmax_dims(yc, dim, s.outer, s.R, s.inner);
  s.in_dtype = dtype_code(yc.scalar_type());
  s.out_dtype = dtype_code(input_dtype);
  b2_check(b2_softmax_bwd(&s, cur_stream()), name);
  count(name);
  return dx;
}

// =============================== layer norm ========================================================

int64_t prod(c10::IntArrayRef s) {
  int64_t n = 1;
  for (auto v : s) n *= v;
  return n;
}

std::tuple<at::Tensor, at::Tensor, at::Tensor> k_native_layer_norm(const at::Tensor& input,
                                                                   c10::SymIntArrayRef normalized_shape_sym,
                                                                   const std::optional<at::Tensor>& weight,
                                                                   const std::optional<at::Tensor>& bias, double eps) {
  c10::cuda::CUDAGuard guard(input.device());
  const char* name = "aten::native_layer_norm";
  auto normalized_shape = C10_AS_INTARRAYREF_SLOW(normalized_shape_sym);
  const int64_t D = prod(normalized_shape);
  const bool has_w = weight.has_value() && weight->defined();
  const bool has_b = bias.has_value() && bias->defined();
  const int nd = (int)normalized_shape.size();
  TORCH_CHECK(nd <= input.dim(), name, ": normalized_shape longer than input");
  for (int i = 0; i < nd; ++i)
    TORCH_CHECK(input.size(input.dim() - nd + i) == normalized_shape[i], name, ": input shape ", input.sizes(),
                " does not end with normalized_shape ", normalized_shape);
  bool ok = is_row_dtype(input.scalar_type()) && (!has_w || (weight->scalar_type() == input.scalar_type() && weight->numel() == D)) &&
            (!has_b || (bias->scalar_type() == input.scalar_type() && bias->numel() == D));
  if (!ok) {
    count_fallback(name);
    return at::native::layer_norm_cuda(input, normalized_shape, weight, bias, eps);
  }
  at::Tensor x = input.is_contiguous() ? input : input.contiguous();
  std::vector<int64_t> stat_shape(x.sizes().begin(), x.sizes().end() - nd);
  for (int i = 0; i < nd; ++i) stat_shape.push_back(1);
  at::Tensor y = at::empty(x.sizes(), x.options());
  at::Tensor mean = at::empty(stat_shape, x.options().dtype(at::kFloat));
  at::Tensor rstd = at::empty(stat_shape, x.options().dtype(at::kFloat));
  if (x.numel() == 0 || D == 0) return {y, mean, rstd};
  at::Tensor w = has_w ? weight->contiguous() : at::Tensor();
  at::Tensor b = has_b ? bias->contiguous() : at::Tensor();
  b2_layernorm_args l{};
  l.x = x.data_ptr();
  l.w = has_w ? w.data_ptr() : nullptr;
  l.b = has_b ? b.data_ptr() : nullptr;
  l.y = y.data_ptr();
  l.mean = mean.data_ptr<float>();
  l.rstd = rstd.data_ptr<float>();
  l.rows = x.numel() / D;
  l.D = D;
  l.eps = (float)eps;
  l.dtype = dtype_code(x.scalar_type());
  b2_check(b2_layernorm_fwd(&l, cur_stream()), name);
  count(name);
  return {y, mean, rstd};
}

std::tuple<at::Tensor, at::Tensor, at::Tensor> k_native_layer_norm_backward(
    const at::Tensor& grad_out, const at::Tensor& input, c10::SymIntArrayRef normalized_shape_sym, const at::Tensor& mean,
    const at::Tensor& rstd, const std::optional<at::Tensor>& weight, const std::optional<at::Tensor>& bias,
    std::array<bool, 3> output_mask) {
  c10::cuda::CUDAGuard guard(input.device());
  const char* name = "aten::native_layer_norm_backward";
  auto normalized_shape = C10_AS_INTARRAYREF_SLOW(normalized_shape_sym);
  const int64_t D = prod(normalized_shape);
  const bool has_w = weight.has_value() && weight->defined();
  const bool has_b = bias.has_value() && bias->defined();
  bool ok = is_row_dtype(input.scalar_type()) && grad_out.scalar_type() == input.scalar_type() &&
            grad_out.sizes() == input.sizes() && mean.scalar_type() == at::kFloat && rstd.scalar_type() == at::kFloat &&
            (!has_w || (weight->scalar_type() == input.scalar_type() && weight->numel() == D));
  if (!ok) {
    count_fallback(name);
    return at::native::layer_norm_backward_cuda(grad_out, input, normalized_shape, mean, rstd, weight, bias, output_mask);
  }
  at::Tensor g = grad_out.is_contiguous() ? grad_out : grad_out.contiguous();
  at::Tensor x = input.is_contiguous() ? input : input.contiguous();
  at::Tensor mu = mean.contiguous(), rs = rstd.contiguous();
  at::Tensor w = has_w ? weight->contiguous() : at::Tensor();
  at::Tensor dx, dw, db;
  if (output_mask[0]) dx = at::empty(x.sizes(), x.options());
  const bool want_dw = output_mask[1] && has_w;
  const bool want_db = output_mask[2] && has_b;
  if (want_dw) dw = at::empty(weight->sizes(), weight->options());
  if (want_db) db = at::empty(bias->sizes(), bias->options());
  if (x.numel() == 0 || D == 0) {
    if (want_dw) dw.zero_();
    if (want_db) db.zero_();
    return {dx, dw, db};
  }
  b2_layernorm_args l{};
  l.x = x.data_ptr();
  l.w = has_w ? w.data_ptr() : nullptr;
  l.mean = mu.data_ptr<float>();
  l.rstd = rs.data_ptr<float>();
  l.g = g.data_ptr();
  l.dx = output_mask[0] ? dx.data_ptr() : nullptr;
  l.dw = want_dw ? dw.data_ptr() : nullptr;
  l.db = want_db ? db.data_ptr() : nullptr;
  l.rows = x.numel() / D;
  l.D = D;
  l.dtype = dtype_code(x.scalar_type());
  at::Tensor ws;
  if (want_dw || want_db) {
    uint64_t bytes = b2_layernorm_bwd_workspace_bytes(&l);
    ws = at::empty({(int64_t)((bytes + 3) / 4)}, x.options().dtype(at::kFloat));
    l.workspace = ws.data_ptr();
  }
  if (l.dx || l.dw || l.db) b2_check(b2_layernorm_bwd(&l, cur_stream()), name);
  count(name);
  return {dx, dw, db};
}

// =============================== optimizer ternaries ===============================================

bool fill_ew(b2_ew_args& e, c10::IntArrayRef sizes, const at::Tensor& out, const at::Tensor& x, const at::Tensor& t1,
             const at::Tensor* t2) {
  if ((int)sizes.size() > B2_EW_MAX_DIMS) return false;
  e.ndim = (int)sizes.size();
  auto ex = [&](const at::Tensor& t, int64_t* s) {
    at::Tensor v = t.expand(sizes);
    for (int d = 0; d < e.ndim; ++d) s[d] = v.stride(d);
  };
  for (int d = 0; d < e.ndim; ++d) e.sizes[d] = sizes[d];
  ex(out, e.out_s);
  ex(x, e.x_s);
  ex(t1, e.t1_s);
  if (t2) ex(*t2, e.t2_s);
  e.out = out.data_ptr();
  e.x = x.data_ptr();
  e.t1 = t1.data_ptr();
  e.t2 = t2 ? t2->data_ptr() : nullptr;
  return true;
}

// op: 0 addcmul, 1 addcdiv, 2 lerp. Returns false when the case needs the stock path.
bool ternary(int op, const at::Tensor& self, const at::Tensor& t1, const at::Tensor* t2, double value, at::Tensor& out,
             bool inplace, const char* name) {
  if (!is_row_dtype(self.scalar_type()) || t1.scalar_type() != self.scalar_type() ||
      (t2 && t2->scalar_type() != self.scalar_type()) || !t1.is_cuda() || (t2 && !t2->is_cuda()))
    return false;
  std::vector<int64_t> sizes = at::infer_size(self.sizes(), t1.sizes());
  if (t2) sizes = at::infer_size(sizes, t2->sizes());
  if (inplace) {
    TORCH_CHECK(std::vector<int64_t>(self.sizes().begin(), self.sizes().end()) == sizes, name,
                ": output with shape ", self.sizes(), " doesn't match the broadcast shape ", c10::IntArrayRef(sizes));
    out = self;
  } else {
    out = at::empty(sizes, self.options());
  }
  if (out.numel() == 0) return true;
  b2_ew_args e{};
  if (!fill_ew(e, sizes, out, self, t1, t2)) return false;
  e.op = op;
  e.dtype = dtype_code(self.scalar_type());
  e.value = (float)value;
  b2_check(b2_ew_ternary(&e, cur_stream()), name);
  count(name);
  return true;
}

at::Tensor& k_addcmul_(at::Tensor& self, const at::Tensor& t1, const at::Tensor& t2, const at::Scalar& v) {
  c10::cuda::CUDAGuard guard(self.device());
  at::Tensor out;
  if (ternary(0, self, t1, &t2, v.toDouble(), out, true, "aten::addcmul_")) return self;
  count_fallback("aten::addcmul_");
  return self.add_(t1 * t2 * v);
}
at::Tensor k_addcmul(const at::Tensor& self, const at::Tensor& t1, const at::Tensor& t2, const at::Scalar& v) {
  c10::cuda::CUDAGuard guard(self.device());
  at::Tensor out;
  if (ternary(0, self, t1, &t2, v.toDouble(), out, false, "aten::addcmul")) return out;
  count_fallback("aten::addcmul");
  return self + t1 * t2 * v;
}
at::Tensor& k_addcdiv_(at::Tensor& self, const at::Tensor& t1, const at::Tensor& t2, const at::Scalar& v) {
  c10::cuda::CUDAGuard guard(self.device());
  at::Tensor out;
  if (ternary(1, self, t1, &t2, v.toDouble(), out, true, "aten::addcdiv_")) return self;
  count_fallback("aten::addcdiv_");
  return self.add_(t1 * v / t2);
}
at::Tensor k_addcdiv(const at::Tensor& self, const at::Tensor& t1, const at::Tensor& t2, const at::Scalar& v) {
  c10::cuda::CUDAGuard guard(self.device());
  at::Tensor out;
  if (ternary(1, self, t1, &t2, v.toDouble(), out, false, "aten::addcdiv")) return out;
  count_fallback("aten::addcdiv");
  return self + t1 * v / t2;
}
at::Tensor& k_lerp__Scalar(at::Tensor& self, const at::Tensor& end, const at::Scalar& w) {
  c10::cuda::CUDAGuard guard(self.device());
  at::Tensor out;
  if (ternary(2, self, end, nullptr, w.toDouble(), out, true, "aten::lerp_.Scalar")) return self;
  count_fallback("aten::lerp_.Scalar");
  return self.add_((end - self) * w);
}
at::Tensor k_lerp_Scalar(const at::Tensor& self, const at::Tensor& end, const at::Scalar& w) {
  c10::cuda::CUDAGuard guard(self.device());
  at::Tensor out;
  if (ternary(2, self, end, nullptr, w.toDouble(), out, false, "aten::lerp.Scalar")) return out;
  count_fallback("aten::lerp.Scalar");
  return self + (end - self) * w;
}

// =============================== attention =========================================================

bool attn_dtype(at::ScalarType t) { return is_row_dtype(t); }

// Eligibility of the fused kernels, attn_supported (csrc/ops_attn.cpp:80-95).
bool attn_supported(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const std::optional<at::Tensor>& mask,
                    double dropout_p, bool is_causal, bool enable_gqa) {
  if (mask.has_value() && mask->defined()) return false;
  if (dropout_p != 0.0 || is_causal) return false;
  if (!q.is_cuda() || !k.is_cuda() || !v.is_cuda()) return false;
  if (q.dim() != 4 || k.dim() != 4 || v.dim() != 4) return false;
  if (!attn_dtype(q.scalar_type()) || k.scalar_type() != q.scalar_type() || v.scalar_type() != q.scalar_type()) return false;
  const int64_t D = q.size(3);
  if (D < 1 || D > 128 || k.size(3) != D || v.size(3) != D) return false;
  if (q.size(0) != k.size(0) || q.size(0) != v.size(0) || q.size(1) != k.size(1) || q.size(1) != v.size(1)) return false;
  if (k.size(2) != v.size(2) || k.size(2) < 1 || q.size(2) < 1 || q.size(0) < 1 || q.size(1) < 1) return false;
  (void)enable_gqa;  // equal head counts are required above, so GQA never reaches here
  return true;
}

// auto: half types always; fp32 when the score matrix would be >= 256 MiB (fused_wanted, ops_attn.cpp:70-77)
bool fused_wanted(const at::Tensor& q, const at::Tensor& k) {
  int p = attn_policy();
  if (p == 0) return false;
  if (p == 1) return true;
  if (q.scalar_type() != at::kFloat) return true;
  double score_bytes = 4.0 * (double)q.size(0) * q.size(1) * q.size(2) * k.size(2);
  return score_bytes >= 256.0 * 1024 * 1024;
}

at::native::fused_sdp_choice_fn g_stock_choice = nullptr;

int64_t fused_sdp_choice_b2(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                            const std::optional<at::Tensor>& mask, double dropout_p, bool is_causal,
                            std::optional<double> scale, bool enable_gqa) {
  if (attn_supported(q, k, v, mask, dropout_p, is_causal, enable_gqa) && fused_wanted(q, k))
    return static_cast<int64_t>(at::SDPBackend::overrideable);
  if (g_stock_choice) return g_stock_choice(q, k, v, mask, dropout_p, is_causal, scale, enable_gqa);
  return static_cast<int64_t>(at::SDPBackend::math);
}

void fill_strides(int64_t* dst, const at::Tensor& t) {
  dst[0] = t.stride(0), dst[1] = t.stride(1), dst[2] = t.stride(2);
}

// [B,S,H,D] contiguous storage returned as a [B,H,S,D] view (alloc_bshd, ops_attn.cpp:160-162)
at::Tensor alloc_bshd(int64_t B, int64_t H, int64_t S, int64_t D, const at::TensorOptions& o) {
  return at::empty({B, S, H, D}, o).permute({0, 2, 1, 3});
}

at::Tensor unit_d(const at::Tensor& t) { return t.stride(3) == 1 ? t : t.contiguous(); }

using FwdRet = std::tuple<at::Tensor, at::Tensor, at::Tensor, at::Tensor, c10::SymInt, c10::SymInt, at::Tensor, at::Tensor,
                          at::Tensor>;

FwdRet k_sdpa_fwd(const at::Tensor& query, const at::Tensor& key, const at::Tensor& value,
                  const std::optional<at::Tensor>& attn_bias, double dropout_p, bool is_causal, bool /*debug_mask*/,
                  std::optional<double> scale) {
  const char* name = "aten::_scaled_dot_product_fused_attention_overrideable";
  TORCH_CHECK(attn_supported(query, key, value, attn_bias, dropout_p, is_causal, false),
              "b200: this attention case is not supported by the fused kernel");
  c10::cuda::CUDAGuard guard(query.device());
  at::Tensor q = unit_d(query), k = unit_d(key), v = unit_d(value);
  const int64_t B = q.size(0), H = q.size(1), Sq = q.size(2), Sk = k.size(2), D = q.size(3);
  at::Tensor out = alloc_bshd(B, H, Sq, D, q.options());
  at::Tensor lse = at::empty({B, H, Sq}, q.options().dtype(at::kFloat));
  b2_attn_args a{};
  a.q = q.data_ptr(), a.k = k.data_ptr(), a.v = v.data_ptr(), a.o = out.data_ptr(), a.lse = lse.data_ptr<float>();
  a.B = B, a.H = H, a.Sq = Sq, a.Sk = Sk, a.D = D;
  fill_strides(a.q_s, q), fill_strides(a.k_s, k), fill_strides(a.v_s, v), fill_strides(a.o_s, out);
  a.scale = (float)scale.value_or(1.0 / std::sqrt((double)D));
  a.dtype = dtype_code(q.scalar_type());
  a.force_simt = (g_force_simt.load() & 2) ? 1 : 0;
  b2_check(b2_attn_fwd(&a, cur_stream()), name);
  count(name);
  at::Tensor el = at::empty({0}, q.options().dtype(at::kLong));
  return FwdRet{out, lse, el, el, c10::SymInt(Sq), c10::SymInt(Sk), el, el, at::empty({0}, q.options())};
}

using BwdRet = std::tuple<at::Tensor, at::Tensor, at::Tensor, at::Tensor>;

BwdRet k_sdpa_bwd(const at::Tensor& grad_out, const at::Tensor& query, const at::Tensor& key, const at::Tensor& value,
                  const at::Tensor& attn_bias, std::array<bool, 4> mask, const at::Tensor& out, const at::Tensor& lse,
                  const at::Tensor&, const at::Tensor&, c10::SymInt, c10::SymInt, double dropout_p, bool is_causal,
                  const at::Tensor&, const at::Tensor&, std::optional<double> scale) {
  const char* name = "aten::_scaled_dot_product_fused_attention_overrideable_backward";
  TORCH_CHECK(attn_supported(query, key, value,
                             attn_bias.defined() ? std::optional<at::Tensor>(attn_bias) : std::nullopt, dropout_p,
                             is_causal, false),
              "b200: this attention backward case is not supported by the fused kernel");
  c10::cuda::CUDAGuard guard(query.device());
  at::Tensor q = unit_d(query), k = unit_d(key), v = unit_d(value);
  const int64_t B = q.size(0), H = q.size(1), Sq = q.size(2), Sk = k.size(2), D = q.size(3);
  at::Tensor dO = grad_out.scalar_type() == q.scalar_type() ? grad_out : grad_out.to(q.scalar_type());
  dO = unit_d(dO);
  at::Tensor o = unit_d(out.scalar_type() == q.scalar_type() ? out : out.to(q.scalar_type()));
  at::Tensor lse_c = lse.contiguous();
  at::Tensor delta = at::empty({B, H, Sq}, q.options().dtype(at::kFloat));
  at::Tensor dq, dk, dv;
  if (mask[0]) dq = alloc_bshd(B, H, Sq, D, q.options());
  if (mask[1]) dk = alloc_bshd(B, H, Sk, D, q.options());
  if (mask[2]) dv = alloc_bshd(B, H, Sk, D, q.options());
  if (!mask[0] && !mask[1] && !mask[2]) return BwdRet{dq, dk, dv, at::Tensor()};
  b2_attn_args a{};
  a.q = q.data_ptr(), a.k = k.data_ptr(), a.v = v.data_ptr(), a.o = o.data_ptr(), a.lse = lse_c.data_ptr<float>();
  a.d_o = dO.data_ptr(), a.delta = delta.data_ptr<float>();
  a.dq = mask[0] ? dq.data_ptr() : nullptr;
  a.dk = mask[1] ? dk.data_ptr() : nullptr;
  a.dv = mask[2] ? dv.data_ptr() : nullptr;
  a.B = B, a.H = H, a.Sq = Sq, a.Sk = Sk, a.D = D;
  fill_strides(a.q_s, q), fill_strides(a.k_s, k), fill_strides(a.v_s, v), fill_strides(a.o_s, o);
  fill_strides(a.do_s, dO);
  if (mask[0]) fill_strides(a.dq_s, dq);
  if (mask[1]) fill_strides(a.dk_s, dk);
  if (mask[2]) fill_strides(a.dv_s, dv);
  a.scale = (float)scale.value_or(1.0 / std::sqrt((double)D));
  a.dtype = dtype_code(q.scalar_type());
  a.force_simt = (g_force_simt.load() & 2) ? 1 : 0;
  at::Tensor ws;
  uint64_t wsb = b2_attn_bwd_workspace_bytes(&a);
  if (wsb) {
    ws = at::empty({(int64_t)((wsb + 3) / 4)}, q.options().dtype(at::kFloat));
    a.workspace = ws.data_ptr();
  }
  b2_check(b2_attn_bwd(&a, cur_stream()), name);
  count(name);
  return BwdRet{dq, dk, dv, at::Tensor()};
}

// The fused attention backward writing dq, dk, dv into caller-provided [B,H,S,D] views (unit stride along
// D; e.g. column slices of one stacked q/k/v gradient buffer, so the caller needs no concatenation
// afterwards). Same kernel and arguments as the ATen backward above; scale 0 means 1/sqrt(D).
void b2_sdpa_bwd_into(const at::Tensor& grad_out, const at::Tensor& query, const at::Tensor& key, const at::Tensor& value,
                      const at::Tensor& out, const at::Tensor& lse, double scale, const at::Tensor& dq,
                      const at::Tensor& dk, const at::Tensor& dv) {
  const char* name = "b2::sdpa_bwd_into";
  TORCH_CHECK(attn_supported(query, key, value, std::nullopt, 0.0, false, false),
              "sdpa_bwd_into: this attention case is not supported by the fused kernel");
  c10::cuda::CUDAGuard guard(query.device());
  at::Tensor q = unit_d(query), k = unit_d(key), v = unit_d(value);
  const int64_t B = q.size(0), H = q.size(1), Sq = q.size(2), Sk = k.size(2), D = q.size(3);
  for (const at::Tensor* t : {&dq, &dk, &dv}) {
    TORCH_CHECK(t->dim() == 4 && t->stride(3) == 1 && t->scalar_type() == q.scalar_type() && t->device() == q.device(),
                "sdpa_bwd_into: gradients must be [B,H,S,D] views with unit stride along D, in q's dtype and device");
  }
  TORCH_CHECK(dq.sizes() == q.sizes() && dk.sizes() == k.sizes() && dv.sizes() == value.sizes(),
              "sdpa_bwd_into: gradient shapes must match q, k, v");
  at::Tensor dO = unit_d(grad_out.scalar_type() == q.scalar_type() ? grad_out : grad_out.to(q.scalar_type()));
  at::Tensor o = unit_d(out.scalar_type() == q.scalar_type() ? out : out.to(q.scalar_type()));
  at::Tensor lse_c = lse.contiguous();
  at::Tensor delta = at::empty({B, H, Sq}, q.options().dtype(at::kFloat));
  b2_attn_args a{};
  a.q = q.data_ptr(), a.k = k.data_ptr(), a.v = v.data_ptr(), a.o = o.data_ptr(), a.lse = lse_c.data_ptr<float>();
  a.d_o = dO.data_ptr(), a.delta = delta.data_ptr<float>();
  a.dq = dq.data_ptr(), a.dk = dk.data_ptr(), a.dv = dv.data_ptr();
  a.B = B, a.H = H, a.Sq = Sq, a.Sk = Sk, a.D = D;
  fill_strides(a.q_s, q), fill_strides(a.k_s, k), fill_strides(a.v_s, v), fill_strides(a.o_s, o);
  fill_strides(a.do_s, dO);
  fill_strides(a.dq_s, dq), fill_strides(a.dk_s, dk), fill_strides(a.dv_s, dv);
  a.scale = (float)(scale > 0 ? scale : 1.0 / std::sqrt((double)D));
  a.dtype = dtype_code(q.scalar_type());
  a.force_simt = (g_force_simt.load() & 2) ? 1 : 0;
  at::Tensor ws;
  if (uint64_t wsb = b2_attn_bwd_workspace_bytes(&a)) {
    ws = at::empty({(int64_t)((wsb + 3) / 4)}, q.options().dtype(at::kFloat));
    a.workspace = ws.data_ptr();
  }
  b2_check(b2_attn_bwd(&a, cur_stream()), name);
  count(name);
}

// =============================== int8 ==============================================================

int scale_layout_of(const at::Tensor& q, const at::Tensor& scale) {
  const int64_t rows = q.size(0), cols = q.size(1);
  if (scale.scalar_type() == at::kBFloat16 && scale.dim() == 2 && scale.size(0) == rows &&
      scale.size(1) == (cols + 63) / 64)
    return 0;
  if (scale.scalar_type() == at::kFloat && scale.numel() == rows && (scale.dim() == 1 || scale.size(-1) == 1)) return 1;
  TORCH_CHECK(false, "b200 int8: scale must be bf16 [rows, ceil(cols/64)] or fp32 [rows]; got ", scale.scalar_type(), " ",
              scale.sizes());
}

at::Tensor b2_dequant_int8_op(const at::Tensor& q0, const at::Tensor& scale0, at::ScalarType out_dtype) {
  TORCH_CHECK(q0.is_cuda() && scale0.is_cuda(), "dequant_int8: q and scale must be CUDA tensors");
  TORCH_CHECK(q0.scalar_type() == at::kChar && q0.dim() == 2, "dequant_int8: q must be a 2-D int8 tensor");
  TORCH_CHECK(out_dtype == at::kFloat || out_dtype == at::kBFloat16 || out_dtype == at::kHalf,
              "dequant_int8: out_dtype must be float32, bfloat16 or float16");
  c10::cuda::CUDAGuard guard(q0.device());
  at::Tensor q = q0.stride(1) == 1 && q0.stride(0) >= q0.size(1) ? q0 : q0.contiguous();
  at::Tensor scale = scale0.contiguous();
  const int layout = scale_layout_of(q, scale);
  at::Tensor out = at::empty({q.size(0), q.size(1)}, q.options().dtype(out_dtype));
  if (out.numel() == 0) return out;
  b2_dequant_args d{};
  d.q = (const int8_t*)q.data_ptr();
  d.scale = scale.data_ptr();
  d.out = out.data_ptr();
  d.rows = q.size(0), d.cols = q.size(1), d.q_ld = q.stride(0);
  d.scale_layout = layout;
  d.out_dtype = dtype_code(out_dtype);
  b2_check(b2_dequant_int8(&d, cur_stream()), "dequant_int8");
  count("b2::dequant_int8");
  return out;
}

// =============================== MSE loss ==========================================================

int mse_dtype(const at::Tensor& x, const at::Tensor& t, const char* what) {
  TORCH_CHECK(x.is_cuda() && t.is_cuda(), what, ": CUDA tensors expected");
  TORCH_CHECK(x.scalar_type() == t.scalar_type(), what, ": input and target must share a dtype");
  TORCH_CHECK(x.sizes() == t.sizes(), what, ": input and target must have the same shape");
  const auto st = x.scalar_type();
  TORCH_CHECK(st == at::kFloat || st == at::kBFloat16 || st == at::kHalf, what, ": float32, bfloat16 or float16");
  return dtype_code(st);
}

// mean((x - t)^2) in fp32 from the inputs' own dtype (F.mse_loss(x.float(), t.float())), deterministic
at::Tensor b2_mse_loss_fwd_op(const at::Tensor& x0, const at::Tensor& t0) {
  const int dt = mse_dtype(x0, t0, "mse_loss");
  c10::cuda::CUDAGuard guard(x0.device());
  at::Tensor x = x0.contiguous(), t = t0.contiguous();
  at::Tensor loss = at::empty({}, x.options().dtype(at::kFloat));
  const uint64_t wsb = b2_mse_loss_workspace_bytes(x.numel());
  at::Tensor ws = at::empty({(int64_t)std::max<uint64_t>(wsb / 4, 1)}, x.options().dtype(at::kFloat));
  b2_mse_args a{};
  a.x = x.data_ptr(), a.t = t.data_ptr(), a.loss = loss.data_ptr<float>(), a.partial = ws.data_ptr<float>();
  a.n = x.numel(), a.dtype = dt;
  b2_check(b2_mse_loss_fwd(&a, cur_stream()), "mse_loss");
  count("b2::mse_loss_fwd");
  return loss;
}

// d loss / d x = 2 (x - t) * grad / n, in x's dtype
at::Tensor b2_mse_loss_bwd_op(const at::Tensor& grad0, const at::Tensor& x0, const at::Tensor& t0) {
  const int dt = mse_dtype(x0, t0, "mse_loss_backward");
  c10::cuda::CUDAGuard guard(x0.device());
  at::Tensor x = x0.contiguous(), t = t0.contiguous();
  at::Tensor grad = grad0.to(at::kFloat).contiguous();
  TORCH_CHECK(grad.numel() == 1, "mse_loss_backward: a scalar upstream gradient is expected");
  at::Tensor gx = at::empty_like(x);
  b2_mse_args a{};
  a.x = x.data_ptr(), a.t = t.data_ptr(), a.grad_x = gx.data_ptr(), a.grad_loss = grad.data_ptr<float>();
  a.n = x.numel(), a.dtype = dt;
  b2_check(b2_mse_loss_bwd(&a, cur_stream()), "mse_loss_backward");
  count("b2::mse_loss_bwd");
  return gx;
}

// split-K scratch for the int8 GEMM (GEMMs with too few output tiles to fill the GPU) from the
// caching allocator; the returned tensor keeps it alive for the call
at::Tensor int8_workspace(b2_int8_gemm_args& g, const at::Tensor& like) {
  at::Tensor ws;
  if (const uint64_t wsb = b2_int8_gemm_workspace_bytes(&g)) {
    ws = at::empty({(int64_t)wsb}, like.options().dtype(at::kByte));
    g.workspace = ws.data_ptr(), g.workspace_bytes = (int64_t)wsb;
  }
  return ws;
}

// y[..., N] = x[..., K] @ (q * scale)^T + bias; with `gelu_out` the GEMM's epilogue also writes
// gelu_tanh(y) there (the DiT MLP's fc1: y is the pre-activation the backward needs)
// LoRA side operands of one int8 GEMM: h [rows, r] and the weight-side matrix, both bf16; returns r.
int64_t lora_operands(b2_int8_gemm_args& g, const at::Tensor* h, const at::Tensor* w, at::Tensor& hc, at::Tensor& wc,
                      int64_t rows, bool transposed) {
  if (!h) return 0;
  TORCH_CHECK(h->scalar_type() == at::kBFloat16 && w->scalar_type() == at::kBFloat16, "int8 LoRA: bf16 operands required");
  hc = h->reshape({-1, h->size(-1)});
  if (!hc.is_contiguous()) hc = hc.contiguous();
  wc = w->contiguous();
  const int64_t r = hc.size(1);
  TORCH_CHECK(hc.size(0) == rows && r >= 8 && r <= 64 && r % 8 == 0, "int8 LoRA: h must be [rows, r] with 8 <= r <= 64, r % 8 == 0");
  TORCH_CHECK(transposed ? (wc.dim() == 2 && wc.size(0) == r) : (wc.dim() == 2 && wc.size(1) == r),
              "int8 LoRA: the weight-side operand must be [N, r] (forward) or [r, K] (dX)");
  g.lora_h = hc.data_ptr(), g.lora_b = wc.data_ptr();
  g.lora_h_ld = r, g.lora_b_ld = wc.size(1), g.lora_r = (int32_t)r;
  return r;
}

at::Tensor int8_fwd_impl(const at::Tensor& x0, const at::Tensor& q, const at::Tensor& scale0,
                         const std::optional<at::Tensor>& bias0, at::Tensor* gelu_out,
                         const at::Tensor* lora_h = nullptr, const at::Tensor* lora_b = nullptr) {
  TORCH_CHECK(x0.is_cuda() && q.is_cuda(), "int8_linear: CUDA tensors required");
  TORCH_CHECK(x0.scalar_type() == at::kBFloat16, "int8_linear: x must be bfloat16");
  TORCH_CHECK(q.scalar_type() == at::kChar && q.dim() == 2 && q.is_contiguous(), "int8_linear: q must be contiguous int8 [N,K]");
  c10::cuda::CUDAGuard guard(x0.device());
  const int64_t N = q.size(0), K = q.size(1);
  TORCH_CHECK(x0.size(-1) == K, "int8_linear: x last dim ", x0.size(-1), " != K ", K);
  at::Tensor scale = scale0.contiguous();
  const int layout = scale_layout_of(q, scale);
  at::Tensor x = x0.reshape({-1, K});
  if (!x.is_contiguous()) x = x.contiguous();
  std::vector<int64_t> osz(x0.sizes().begin(), x0.sizes().end());
  osz.back() = N;
  at::Tensor out = at::empty({x.size(0), N}, x.options());
  if (gelu_out) *gelu_out = at::empty({x.size(0), N}, x.options());
  if (out.numel() == 0) {
    if (gelu_out) *gelu_out = gelu_out->view(osz);
    return out.view(osz);
  }
  at::Tensor bias;
  if (bias0.has_value() && bias0->defined()) {
    bias = bias0->contiguous();
    TORCH_CHECK(bias.scalar_type() == at::kBFloat16 && bias.numel() == N, "int8_linear: bias must be bf16 [N]");
  }
  b2_int8_gemm_args g{};
  g.x = x.data_ptr(), g.q = (const int8_t*)q.data_ptr(), g.scale = scale.data_ptr();
  g.bias = bias.defined() ? bias.data_ptr() : nullptr;
  g.out = out.data_ptr();
  g.M = x.size(0), g.N = N, g.K = K, g.x_ld = K, g.out_ld = N;
  g.scale_layout = layout;
  g.transpose_w = 0;
  if (gelu_out) g.epilogue = 1, g.aux = gelu_out->data_ptr(), g.aux_ld = N;
  at::Tensor lh, lb;
  if (lora_h) TORCH_CHECK(lora_b->size(0) == N, "int8_lora_fwd: b must be [N, r]");
  lora_operands(g, lora_h, lora_b, lh, lb, g.M, false);
  at::Tensor ws = int8_workspace(g, x);
  b2_check(b2_int8_gemm(&g, cur_stream()), gelu_out ? "int8_linear_gelu_fwd" : "int8_linear_fwd");
  count(gelu_out ? "b2::int8_linear_gelu" : "b2::int8_linear");
  if (gelu_out) *gelu_out = gelu_out->view(osz);
  return out.view(osz);
}

at::Tensor b2_int8_linear_fwd(const at::Tensor& x0, const at::Tensor& q, const at::Tensor& scale0,
                              const std::optional<at::Tensor>& bias0) {
  return int8_fwd_impl(x0, q, scale0, bias0, nullptr);
}

// (gelu_tanh(h), h) with h = x @ (q * scale)^T + bias, from one GEMM
std::tuple<at::Tensor, at::Tensor> b2_int8_linear_gelu_fwd(const at::Tensor& x0, const at::Tensor& q,
                                                           const at::Tensor& scale0,
                                                           const std::optional<at::Tensor>& bias0) {
  at::Tensor act;
  at::Tensor h = int8_fwd_impl(x0, q, scale0, bias0, &act);
  return {act, h};
}

// dx[..., K] = dy[..., N] @ (q * scale); with `h` (the pre-activation of a GELU that follows this
// linear's input) the epilogue returns dx * gelu_tanh'(h) instead
at::Tensor int8_dx_impl(const at::Tensor& dy0, const at::Tensor& q, const at::Tensor& scale0, const at::Tensor* h,
                        const at::Tensor* lora_h = nullptr, const at::Tensor* lora_a = nullptr) {
  TORCH_CHECK(dy0.is_cuda() && q.is_cuda() && dy0.scalar_type() == at::kBFloat16, "int8_linear_dx: bf16 CUDA dy required");
  c10::cuda::CUDAGuard guard(dy0.device());
  const int64_t N = q.size(0), K = q.size(1);
  at::Tensor scale = scale0.contiguous();
  const int layout = scale_layout_of(q, scale);
  at::Tensor dy = dy0.reshape({-1, N});
  if (!dy.is_contiguous()) dy = dy.contiguous();
  std::vector<int64_t> osz(dy0.sizes().begin(), dy0.sizes().end());
  osz.back() = K;
  at::Tensor dx = at::empty({dy.size(0), K}, dy.options());
  if (dx.numel() == 0) return dx.view(osz);
  at::Tensor hh;
  if (h) {
    TORCH_CHECK(h->scalar_type() == at::kBFloat16 && h->numel() == dx.numel() && h->size(-1) == K,
                "int8_linear_dx_gelu: h must be bf16 with the shape of dx");
    hh = h->reshape({-1, K});
    if (!hh.is_contiguous()) hh = hh.contiguous();
  }
  b2_int8_gemm_args g{};
  g.x = dy.data_ptr(), g.q = (const int8_t*)q.data_ptr(), g.scale = scale.data_ptr();
  g.out = dx.data_ptr();
  g.M = dy.size(0), g.N = N, g.K = K, g.x_ld = N, g.out_ld = K;
  g.scale_layout = layout;
  g.transpose_w = 1;
  if (h) g.epilogue = 2, g.aux = hh.data_ptr(), g.aux_ld = K;
  at::Tensor lh, la;
  if (lora_h) TORCH_CHECK(lora_a->dim() == 2 && lora_a->size(1) == K, "int8_lora_dx: a must be [r, K]");
  lora_operands(g, lora_h, lora_a, lh, la, g.M, true);
  at::Tensor ws = int8_workspace(g, dy);
  b2_check(b2_int8_gemm(&g, cur_stream()), h ? "int8_linear_dx_gelu" : "int8_linear_dx");
  count(h ? "b2::int8_linear_dx_gelu" : "b2::int8_linear_dx");
  return dx.view(osz);
}

at::Tensor b2_int8_linear_dx(const at::Tensor& dy0, const at::Tensor& q, const at::Tensor& scale0) {
  return int8_dx_impl(dy0, q, scale0, nullptr);
}

at::Tensor b2_int8_linear_dx_gelu(const at::Tensor& dy0, const at::Tensor& q, const at::Tensor& scale0,
                                  const at::Tensor& h) {
  return int8_dx_impl(dy0, q, scale0, &h);
}

// y = x @ (q * scale)^T + bias + h @ b^T: the LoRA up-projection (b = B * alpha / r, h = x @ A^T) added by
// the int8 GEMM itself as one more reduction block
at::Tensor b2_int8_lora_fwd(const at::Tensor& x0, const at::Tensor& q, const at::Tensor& scale0,
                            const std::optional<at::Tensor>& bias0, const at::Tensor& h, const at::Tensor& b) {
  at::Tensor y = int8_fwd_impl(x0, q, scale0, bias0, nullptr, &h, &b);
  count("b2::int8_lora_fwd");
  return y;
}

// dx = dy @ (q * scale) + dh @ a: the LoRA input gradient (dh = dy @ B * alpha / r, a = A) in the same GEMM
at::Tensor b2_int8_lora_dx(const at::Tensor& dy0, const at::Tensor& q, const at::Tensor& scale0, const at::Tensor& dh,
                           const at::Tensor& a) {
  at::Tensor dx = int8_dx_impl(dy0, q, scale0, nullptr, &dh, &a);
  count("b2::int8_lora_dx");
  return dx;
}

// One AdamW step for a list of parameters (the arithmetic and roundings of torch.optim.AdamW with
// foreach=False, csrc/ops_ew.cpp:432-451), one launch per 48 tensors instead of ~6 per tensor.
void b2_adamw_step_op(at::TensorList params, at::TensorList grads, at::TensorList exp_avgs, at::TensorList exp_avg_sqs,
                      double lr, double beta1, double beta2, double eps, double weight_decay, int64_t step) {
  const size_t n = params.size();
  TORCH_CHECK(grads.size() == n && exp_avgs.size() == n && exp_avg_sqs.size() == n, "adamw_step_: list lengths differ");
  TORCH_CHECK(step >= 1, "adamw_step_: step must be >= 1");
  if (n == 0) return;
  c10::cuda::CUDAGuard guard(params[0].device());
  const auto dt = params[0].scalar_type();
  TORCH_CHECK(dt == at::kFloat || dt == at::kBFloat16, "adamw_step_: parameters must be float32 or bfloat16");
  std::vector<void*> P(n), M(n), V(n);
  std::vector<const void*> G(n);
  std::vector<int64_t> N(n);
  for (size_t i = 0; i < n; ++i) {
    for (const at::Tensor* t : {&params[i], &grads[i], &exp_avgs[i], &exp_avg_sqs[i]}) {
      TORCH_CHECK(t->is_cuda() && t->scalar_type() == dt && t->is_contiguous() && t->device() == params[0].device(),
                  "adamw_step_: every tensor must be a contiguous CUDA tensor of the parameters' dtype and device");
      TORCH_CHECK(t->numel() == params[i].numel(), "adamw_step_: shape mismatch");
    }
    P[i] = params[i].data_ptr(), G[i] = grads[i].data_ptr(), M[i] = exp_avgs[i].data_ptr(), V[i] = exp_avg_sqs[i].data_ptr();
    N[i] = params[i].numel();
  }
  b2_adamw_args a{};
  a.param = P.data(), a.grad = G.data(), a.exp_avg = M.data(), a.exp_avg_sq = V.data(), a.numel = N.data();
  a.n = (int32_t)n;
  a.dtype = dt == at::kFloat ? B2_F32 : B2_BF16;
  a.lr = (float)lr, a.beta1 = (float)beta1, a.beta2 = (float)beta2, a.eps = (float)eps, a.weight_decay = (float)weight_decay;
  a.bias_correction1 = (float)(1.0 - std::pow(beta1, (double)step));
  a.bias_correction2 = (float)(1.0 - std::pow(beta2, (double)step));
  b2_check(b2_adamw_step(&a, cur_stream()), "adamw_step_");
  count("b2::adamw_step_");
}

// =============================== registration ======================================================

std::mutex g_reg_mu;
std::unique_ptr<torch::Library> g_lib;

void register_all(torch::Library& m) {
  m.impl("mm", &k_mm);
  m.impl("bmm", &k_bmm);
  m.impl("addmm", &k_addmm);
  m.impl("baddbmm", &k_baddbmm);
  m.impl("_softmax", &k_softmax);
  m.impl("_safe_softmax", &k_safe_softmax);
  m.impl("_softmax_backward_data", &k_softmax_backward);
  m.impl("native_layer_norm", &k_native_layer_norm);
  m.impl("native_layer_norm_backward", &k_native_layer_norm_backward);
  m.impl("addcmul", &k_addcmul);
  m.impl("addcmul_", &k_addcmul_);
  m.impl("addcdiv", &k_addcdiv);
  m.impl("addcdiv_", &k_addcdiv_);
  m.impl("lerp.Scalar", &k_lerp_Scalar);
  m.impl("lerp_.Scalar", &k_lerp__Scalar);
  m.impl("_scaled_dot_product_fused_attention_overrideable", &k_sdpa_fwd);
  m.impl("_scaled_dot_product_fused_attention_overrideable_backward", &k_sdpa_bwd);
}

void set_enabled(bool on) {
  std::lock_guard<std::mutex> g(g_reg_mu);
  if (on && !g_lib) {
    g_lib = std::make_unique<torch::Library>(torch::Library::IMPL, "aten", c10::DispatchKey::CUDA, __FILE__, __LINE__);
    register_all(*g_lib);
    auto& stub = at::native::_fused_sdp_choice_stub;
    // DispatchStub's only data member is its DispatchStubImpl (public struct); read the stock CUDA
    // entry through it so set_enabled(false) can put it back.
    if (!g_stock_choice)
      g_stock_choice = reinterpret_cast<at::native::fused_sdp_choice_fn>(
          reinterpret_cast<at::native::DispatchStubImpl*>(&stub)->cuda_dispatch_ptr);
    stub.set_cuda_dispatch_ptr(&fused_sdp_choice_b2);
  } else if (!on && g_lib) {
    g_lib.reset();
    if (g_stock_choice) at::native::_fused_sdp_choice_stub.set_cuda_dispatch_ptr(g_stock_choice);
  }
}

bool is_enabled() {
  std::lock_guard<std::mutex> g(g_reg_mu);
  return g_lib != nullptr;
}

void op_set_enabled(bool on) { set_enabled(on); }
bool op_is_enabled() { return is_enabled(); }
void op_set_fused_attention(int64_t mode) { g_attn_policy.store((int)mode); }
int64_t op_fused_attention() { return attn_policy(); }
void op_set_force_simt(int64_t mask) { g_force_simt.store((int)mask); }
int64_t op_gemm_path(const at::Tensor& a, const at::Tensor& b) {
  // 1 when b2_gemm would take the tensor-core kernel for mm(a, b)
  b2_gemm_args g{};
  g.a = a.data_ptr(), g.b = b.data_ptr();
  g.M = a.size(0), g.K = a.size(1), g.N = b.size(1), g.batch = 1;
  g.a_sm = a.stride(0), g.a_sk = a.stride(1), g.b_sk = b.stride(0), g.b_sn = b.stride(1);
  g.dtype = dtype_code(a.scalar_type());
  g.force_simt = (g_force_simt.load() & 1) ? 1 : 0;
  return b2_gemm_path(&g);
}

}  // namespace

TORCH_LIBRARY(b2, m) {
  m.def("dequant_int8(Tensor q, Tensor scale, ScalarType out_dtype) -> Tensor");
  m.def("int8_linear_fwd(Tensor x, Tensor q, Tensor scale, Tensor? bias) -> Tensor");
  m.def("int8_linear_dx(Tensor dy, Tensor q, Tensor scale) -> Tensor");
  m.def("int8_linear_gelu_fwd(Tensor x, Tensor q, Tensor scale, Tensor? bias) -> (Tensor, Tensor)");
  m.def("int8_linear_dx_gelu(Tensor dy, Tensor q, Tensor scale, Tensor h) -> Tensor");
  m.def("int8_lora_fwd(Tensor x, Tensor q, Tensor scale, Tensor? bias, Tensor h, Tensor b) -> Tensor");
  m.def("int8_lora_dx(Tensor dy, Tensor q, Tensor scale, Tensor dh, Tensor a) -> Tensor");
  m.def("mse_loss_fwd(Tensor x, Tensor t) -> Tensor");
  m.def("mse_loss_bwd(Tensor grad, Tensor x, Tensor t) -> Tensor");
  m.def("sdpa_bwd_into(Tensor grad_out, Tensor q, Tensor k, Tensor v, Tensor out, Tensor lse, float scale, "
        "Tensor(a!) dq, Tensor(b!) dk, Tensor(c!) dv) -> ()");
  m.def("adamw_step_(Tensor(a!)[] params, Tensor[] grads, Tensor(b!)[] exp_avgs, Tensor(c!)[] exp_avg_sqs, float lr, "
        "float beta1, float beta2, float eps, float weight_decay, int step) -> ()");
  m.def("set_enabled(bool on) -> ()", &op_set_enabled);
  m.def("is_enabled() -> bool", &op_is_enabled);
  m.def("set_fused_attention(int mode) -> ()", &op_set_fused_attention);
  m.def("fused_attention() -> int", &op_fused_attention);
  m.def("set_force_simt(int mask) -> ()", &op_set_force_simt);
  m.def("gemm_path(Tensor a, Tensor b) -> int", &op_gemm_path);
}

TORCH_LIBRARY_IMPL(b2, CUDA, m) {
  m.impl("dequant_int8", &b2_dequant_int8_op);
  m.impl("int8_linear_fwd", &b2_int8_linear_fwd);
  m.impl("int8_linear_dx", &b2_int8_linear_dx);
  m.impl("int8_linear_gelu_fwd", &b2_int8_linear_gelu_fwd);
  m.impl("int8_linear_dx_gelu", &b2_int8_linear_dx_gelu);
  m.impl("int8_lora_fwd", &b2_int8_lora_fwd);
  m.impl("int8_lora_dx", &b2_int8_lora_dx);
  m.impl("mse_loss_fwd", &b2_mse_loss_fwd_op);
  m.impl("mse_loss_bwd", &b2_mse_loss_bwd_op);
  m.impl("sdpa_bwd_into", &b2_sdpa_bwd_into);
  m.impl("adamw_step_", &b2_adamw_step_op);
}
