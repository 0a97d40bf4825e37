// Tensor-level bindings of the memory-bound, loss, optimiser and routing
// kernels.  Shapes, dtypes and alignment are checked here; the kernels assume
// them.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "attention.h"
#include "kernels.h"

namespace omni {

namespace {
cudaStream_t stream() { return at::cuda::getCurrentCUDAStream().stream(); }

void check_bf16(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16 && t.is_contiguous(), name,
              " must be a contiguous CUDA bf16 tensor");
}
void check_f32(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kFloat && t.is_contiguous(), name,
              " must be a contiguous CUDA fp32 tensor");
}
void check_i32(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kInt && t.is_contiguous(), name,
              " must be a contiguous CUDA int32 tensor");
}
template <typename T>
T* opt_ptr(const c10::optional<at::Tensor>& t) {
  return t.has_value() ? reinterpret_cast<T*>(t->data_ptr()) : nullptr;
}
}  // namespace

// ---- norms -----------------------------------------------------------------
std::vector<at::Tensor> rmsnorm_fwd_t(const at::Tensor& x, const c10::optional<at::Tensor>& res, const at::Tensor& w,
                                      double eps) {
  check_bf16(x, "x");
  check_bf16(w, "w");
  const c10::cuda::CUDAGuard g(x.device());
  const int64_t dim = x.size(-1), rows = x.numel() / dim;
  TORCH_CHECK(dim % 8 == 0 && w.numel() == dim, "rmsnorm: dim must be a multiple of 8 and match w");
  auto y = at::empty_like(x);
  auto rstd = at::empty({rows}, x.options().dtype(at::kFloat));
  at::Tensor h;
  if (res.has_value()) {
    check_bf16(*res, "res");
    TORCH_CHECK(res->sizes() == x.sizes(), "rmsnorm: residual shape");
    h = at::empty_like(x);
  }
  rmsnorm_fwd(x.data_ptr(), res.has_value() ? res->data_ptr() : nullptr, res.has_value() ? h.data_ptr() : nullptr,
              w.data_ptr(), y.data_ptr(), rstd.data_ptr<float>(), (int)rows, (int)dim, (float)eps, stream());
  if (res.has_value()) return {y, rstd, h};
  return {y, rstd};
}

std::vector<at::Tensor> rmsnorm_bwd_t(const at::Tensor& x, const at::Tensor& w, const at::Tensor& rstd,
                                      const at::Tensor& dy, const c10::optional<at::Tensor>& dres) {
  check_bf16(x, "x");
  check_bf16(dy, "dy");
  check_f32(rstd, "rstd");
  const c10::cuda::CUDAGuard g(x.device());
  const int64_t dim = x.size(-1), rows = x.numel() / dim;
  auto dx = at::empty_like(x);
  auto dw = at::zeros({dim}, x.options().dtype(at::kFloat));
  if (dres.has_value()) check_bf16(*dres, "dres");
  rmsnorm_bwd(x.data_ptr(), w.data_ptr(), rstd.data_ptr<float>(), dy.data_ptr(), opt_ptr<void>(dres), dx.data_ptr(),
              dw.data_ptr<float>(), (int)rows, (int)dim, stream());
  return {dx, dw};
}

std::vector<at::Tensor> layernorm_fwd_t(const at::Tensor& x, const at::Tensor& w, const at::Tensor& b, double eps) {
  check_bf16(x, "x");
  const c10::cuda::CUDAGuard g(x.device());
  const int64_t dim = x.size(-1), rows = x.numel() / dim;
  TORCH_CHECK(dim % 8 == 0, "layernorm: dim must be a multiple of 8");
  auto y = at::empty_like(x);
  auto mean = at::empty({rows}, x.options().dtype(at::kFloat));
  auto rstd = at::empty({rows}, x.options().dtype(at::kFloat));
  layernorm_fwd(x.data_ptr(), w.data_ptr(), b.data_ptr(), y.data_ptr(), mean.data_ptr<float>(),
                rstd.data_ptr<float>(), (int)rows, (int)dim, (float)eps, stream());
  return {y, mean, rstd};
}

std::vector<at::Tensor> layernorm_bwd_t(const at::Tensor& x, const at::Tensor& w, const at::Tensor& mean,
                                        const at::Tensor& rstd, const at::Tensor& dy) {
  const c10::cuda::CUDAGuard g(x.device());
  const int64_t dim = x.size(-1), rows = x.numel() / dim;
  auto dx = at::empty_like(x);
  auto dw = at::zeros({dim}, x.options().dtype(at::kFloat));
  auto db = at::zeros({dim}, x.options().dtype(at::kFloat));
  layernorm_bwd(x.data_ptr(), w.data_ptr(), mean.data_ptr<float>(), rstd.data_ptr<float>(), dy.data_ptr(),
                dx.data_ptr(), dw.data_ptr<float>(), db.data_ptr<float>(), (int)rows, (int)dim, stream());
  return {dx, dw, db};
}

// ---- rope (in place) ---------------------------------------------------------
void rope_t(at::Tensor& x, const at::Tensor& cs, const c10::optional<at::Tensor>& pos, int64_t pos0, int64_t seq,
            int64_t tokens, int64_t heads, int64_t row_stride, int64_t head_stride, int64_t off, int64_t rot,
            bool interleaved, double sign) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16, "rope: x must be CUDA bf16");
  check_f32(cs, "cs");
  TORCH_CHECK(cs.dim() == 3 && cs.size(0) == 2 && cs.size(2) == rot / 2, "rope: cs must be [2, max_pos, rot/2]");
  const c10::cuda::CUDAGuard g(x.device());
  if (pos.has_value()) check_i32(*pos, "pos");
  rope_apply(x.data_ptr(), cs.data_ptr<float>(), (int)cs.size(1), opt_ptr<int>(pos), (int)pos0, (int)seq,
             (int)tokens, (int)heads, row_stride, head_stride, (int)off, (int)rot, interleaved, (float)sign, stream());
}

// ---- embedding ---------------------------------------------------------------
at::Tensor embedding_fwd_t(const at::Tensor& ids, const at::Tensor& w) {
  TORCH_CHECK(ids.scalar_type() == at::kLong && ids.is_contiguous(), "embedding: ids must be contiguous int64");
  check_bf16(w, "w");
  const c10::cuda::CUDAGuard g(w.device());
  const int64_t dim = w.size(1);
  TORCH_CHECK(dim % 8 == 0, "embedding: dim must be a multiple of 8");
  auto sizes = ids.sizes().vec();
  sizes.push_back(dim);
  auto out = at::empty(sizes, w.options());
  embedding_fwd(ids.data_ptr<int64_t>(), w.data_ptr(), out.data_ptr(), (int)ids.numel(), (int)dim, (int)w.size(0),
                stream());
  return out;
}

void embedding_bwd_t(const at::Tensor& ids, const at::Tensor& dout, at::Tensor& dw) {
  check_bf16(dout, "dout");
  check_f32(dw, "dw");
  const c10::cuda::CUDAGuard g(dw.device());
  embedding_bwd(ids.data_ptr<int64_t>(), dout.data_ptr(), dw.data_ptr<float>(), (int)ids.numel(), (int)dw.size(1),
                (int)dw.size(0), stream());
}

// ---- cross entropy -----------------------------------------------------------
std::vector<at::Tensor> cross_entropy_t(const at::Tensor& logits, const at::Tensor& labels,
                                        const c10::optional<at::Tensor>& dlogits, double grad_scale, double z_loss) {
  TORCH_CHECK(logits.is_cuda() && logits.scalar_type() == at::kBFloat16 && logits.dim() == 2 &&
                  logits.stride(1) == 1 && logits.stride(0) % 8 == 0,
              "cross_entropy: logits must be 2-D bf16 with row stride multiple of 8");
  TORCH_CHECK(labels.scalar_type() == at::kLong && labels.is_contiguous() && labels.numel() == logits.size(0),
              "cross_entropy: labels must be int64 [rows]");
  const c10::cuda::CUDAGuard g(logits.device());
  const int64_t rows = logits.size(0);
  auto loss = at::empty({rows}, logits.options().dtype(at::kFloat));
  auto lse = at::empty({rows}, logits.options().dtype(at::kFloat));
  void* d = nullptr;
  if (dlogits.has_value()) {
    TORCH_CHECK(dlogits->strides() == logits.strides() && dlogits->sizes() == logits.sizes(),
                "cross_entropy: dlogits layout must match logits");
    d = dlogits->data_ptr();
  }
  cross_entropy_fwd_bwd(logits.data_ptr(), logits.stride(0), labels.data_ptr<int64_t>(), loss.data_ptr<float>(),
                        lse.data_ptr<float>(), d, (int)rows, (int)logits.size(1), (float)grad_scale, (float)z_loss,
                        stream());
  return {loss, lse};
}

// ---- optimiser ---------------------------------------------------------------
void adamw_t(at::Tensor& p, at::Tensor& m, at::Tensor& v, const at::Tensor& g, const c10::optional<at::Tensor>& pb,
             double lr, double b1, double b2, double eps, double wd, int64_t step, double grad_scale,
             const c10::optional<at::Tensor>& norm_sq, double max_norm) {
  check_f32(p, "p");
  check_f32(m, "m");
  check_f32(v, "v");
  check_bf16(g, "g");
  TORCH_CHECK(p.numel() == g.numel() && m.numel() == p.numel() && v.numel() == p.numel(), "adamw: sizes");
  const c10::cuda::CUDAGuard gd(p.device());
  const double bc1 = 1.0 - std::pow(b1, (double)step);
  const double bc2 = 1.0 - std::pow(b2, (double)step);
  if (pb.has_value()) check_bf16(*pb, "p_bf16");
  adamw_step(p.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(), g.data_ptr(), opt_ptr<void>(pb),
             p.numel(), (float)lr, (float)b1, (float)b2, (float)eps, (float)wd, (float)bc1, (float)bc2,
             (float)grad_scale, opt_ptr<float>(norm_sq), (float)max_norm, stream());
}

// Lists of small tensors: one launch per kMultiItems tensors.
void adamw_multi_t(const std::vector<at::Tensor>& p, const std::vector<at::Tensor>& m, const std::vector<at::Tensor>& v,
                   const std::vector<at::Tensor>& g, const std::vector<c10::optional<at::Tensor>>& pb,
                   const std::vector<double>& wd, double lr, double b1, double b2, double eps, int64_t step,
                   double grad_scale, const c10::optional<at::Tensor>& norm_sq, double max_norm) {
  const size_t n = p.size();
  TORCH_CHECK(m.size() == n && v.size() == n && g.size() == n && pb.size() == n && wd.size() == n,
              "adamw_multi: list lengths");
  if (n == 0) return;
  const c10::cuda::CUDAGuard gd(p[0].device());
  const double bc1 = 1.0 - std::pow(b1, (double)step);
  const double bc2 = 1.0 - std::pow(b2, (double)step);
  AdamwMulti t;
  t.count = 0;
  for (size_t i = 0; i < n; ++i) {
    check_f32(p[i], "p");
    check_f32(m[i], "m");
    check_f32(v[i], "v");
    check_bf16(g[i], "g");
    TORCH_CHECK(p[i].is_contiguous() && m[i].is_contiguous() && v[i].is_contiguous() && g[i].is_contiguous() &&
                    g[i].numel() == p[i].numel() && m[i].numel() == p[i].numel() && v[i].numel() == p[i].numel(),
                "adamw_multi: contiguous tensors of one size per item");
    if (pb[i].has_value()) check_bf16(*pb[i], "p_bf16");
    AdamwItem& it = t.item[t.count++];
    it.p = p[i].data_ptr<float>();
    it.m = m[i].data_ptr<float>();
    it.v = v[i].data_ptr<float>();
    it.g = g[i].data_ptr();
    it.pb = pb[i].has_value() ? pb[i]->data_ptr() : nullptr;
    it.n = p[i].numel();
    it.wd = (float)wd[i];
    if (t.count == kMultiItems || i + 1 == n) {
      adamw_multi(t, (float)lr, (float)b1, (float)b2, (float)eps, (float)bc1, (float)bc2, (float)grad_scale,
                  opt_ptr<float>(norm_sq), (float)max_norm, stream());
      t.count = 0;
    }
  }
}

void sq_norm_multi_t(const std::vector<at::Tensor>& g, double scale, at::Tensor& out) {
  if (g.empty()) return;
  check_f32(out, "out");
  const c10::cuda::CUDAGuard gd(out.device());
  AdamwMulti t;
  t.count = 0;
  for (size_t i = 0; i < g.size(); ++i) {
    check_bf16(g[i], "g");
    TORCH_CHECK(g[i].is_contiguous(), "sq_norm_multi: contiguous gradients");
    AdamwItem& it = t.item[t.count++];
    it = AdamwItem{nullptr, nullptr, nullptr, g[i].data_ptr(), nullptr, g[i].numel(), 0.f};
    if (t.count == kMultiItems || i + 1 == g.size()) {
      sq_norm_multi(t, (float)scale, out.data_ptr<float>(), stream());
      t.count = 0;
    }
  }
}

void sq_norm_t(const at::Tensor& g, double scale, at::Tensor& out) {
  check_bf16(g, "g");
  check_f32(out, "out");
  const c10::cuda::CUDAGuard gd(g.device());
  sq_norm_accum(g.data_ptr(), g.numel(), (float)scale, out.data_ptr<float>(), stream());
}

// ---- MoE routing -------------------------------------------------------------
std::vector<at::Tensor> router_topk_t(const at::Tensor& logits, int64_t k, bool renorm) {
  check_f32(logits, "logits");
  const c10::cuda::CUDAGuard g(logits.device());
  const int64_t T = logits.size(0), E = logits.size(1);
  TORCH_CHECK(E <= 256 && k <= 16 && k <= E, "router: E <= 256, k <= 16");
  auto idx = at::empty({T, k}, logits.options().dtype(at::kInt));
  auto w = at::empty({T, k}, logits.options());
  auto probs = at::empty({T, E}, logits.options());
  router_topk(logits.data_ptr<float>(), idx.data_ptr<int>(), w.data_ptr<float>(), probs.data_ptr<float>(), (int)T,
              (int)E, (int)k, renorm, stream());
  return {idx, w, probs};
}

// Returns counts[E], offsets[E+1], pos[T*K], src[cap_rows].
std::vector<at::Tensor> moe_plan_t(const at::Tensor& idx, int64_t E, int64_t capacity, int64_t cap_rows,
                                   int64_t align) {
  check_i32(idx, "idx");
  const c10::cuda::CUDAGuard g(idx.device());
  const int64_t T = idx.size(0), K = idx.size(1);
  TORCH_CHECK(E <= 256, "moe_plan: E <= 256");
  TORCH_CHECK(align >= 1, "moe_plan: align >= 1");
  auto o = idx.options();
  auto counts = at::empty({E}, o);
  auto offsets = at::empty({E + 1}, o);
  auto pos = at::empty({T, K}, o);
  auto src = at::empty({cap_rows}, o);
  const int64_t nblocks = (T * K + 1023) / 1024;
  auto ws = at::empty({std::max<int64_t>(1, 2 * nblocks * E)}, o);
  moe_permute_plan(idx.data_ptr<int>(), (int)T, (int)K, (int)E, (int)capacity, counts.data_ptr<int>(),
                   offsets.data_ptr<int>(), pos.data_ptr<int>(), src.data_ptr<int>(), (int)cap_rows,
                   ws.data_ptr<int>(), stream(), (int)align);
  return {counts, offsets, pos, src};
}

void moe_gather_t(const at::Tensor& x, const at::Tensor& src, at::Tensor& x_perm, int64_t K, const at::Tensor& offsets) {
  check_bf16(x, "x");
  check_bf16(x_perm, "x_perm");
  const c10::cuda::CUDAGuard g(x.device());
  TORCH_CHECK(x.size(-1) % 8 == 0, "moe_gather: dim % 8");
  moe_gather(x.data_ptr(), src.data_ptr<int>(), x_perm.data_ptr(), (int)x_perm.size(0), (int)K, (int)x.size(-1),
             offsets.data_ptr<int>(), (int)offsets.numel() - 1, stream());
}

at::Tensor moe_combine_t(const at::Tensor& y_perm, const at::Tensor& pos, const at::Tensor& w,
                         const c10::optional<at::Tensor>& add) {
  check_bf16(y_perm, "y_perm");
  check_f32(w, "w");
  const c10::cuda::CUDAGuard g(y_perm.device());
  const int64_t T = pos.size(0), K = pos.size(1), dim = y_perm.size(1);
  TORCH_CHECK(dim % 8 == 0, "moe_combine: dim % 8");
  auto out = at::empty({T, dim}, y_perm.options());
  if (add.has_value()) check_bf16(*add, "add");
  moe_combine(y_perm.data_ptr(), pos.data_ptr<int>(), w.data_ptr<float>(), opt_ptr<void>(add), out.data_ptr(),
              (int)T, (int)K, (int)dim, stream());
  return out;
}

std::vector<at::Tensor> moe_combine_bwd_t(const at::Tensor& dout, const at::Tensor& y_perm, const at::Tensor& src,
                                          const at::Tensor& w, const at::Tensor& offsets, int64_t K) {
  check_bf16(dout, "dout");
  const c10::cuda::CUDAGuard g(dout.device());
  auto dy = at::empty_like(y_perm);
  auto dw = at::zeros_like(w);
  moe_combine_bwd(dout.data_ptr(), y_perm.data_ptr(), src.data_ptr<int>(), w.data_ptr<float>(), dy.data_ptr(),
                  dw.data_ptr<float>(), (int)y_perm.size(0), (int)K, (int)y_perm.size(1), offsets.data_ptr<int>(),
                  (int)offsets.numel() - 1, stream());
  return {dy, dw};
}

at::Tensor moe_scatter_add_t(const at::Tensor& dx_perm, const at::Tensor& pos, const c10::optional<at::Tensor>& add) {
  check_bf16(dx_perm, "dx_perm");
  const c10::cuda::CUDAGuard g(dx_perm.device());
  const int64_t T = pos.size(0), K = pos.size(1), dim = dx_perm.size(1);
  auto dx = at::empty({T, dim}, dx_perm.options());
  moe_scatter_add(dx_perm.data_ptr(), pos.data_ptr<int>(), opt_ptr<void>(add), dx.data_ptr(), (int)T, (int)K,
                  (int)dim, stream());
  return dx;
}

std::vector<at::Tensor> router_bwd_t(const at::Tensor& logits, const at::Tensor& probs, const at::Tensor& idx,
                                     const at::Tensor& dw, const at::Tensor& counts, bool renorm, double aux_alpha,
                                     double z_beta) {
  const c10::cuda::CUDAGuard g(logits.device());
  const int64_t T = logits.size(0), E = logits.size(1), K = idx.size(1);
  auto dlogits = at::empty({T, E}, logits.options().dtype(at::kBFloat16));
  auto aux = at::zeros({2}, logits.options());
  router_bwd(logits.data_ptr<float>(), probs.data_ptr<float>(), idx.data_ptr<int>(), dw.data_ptr<float>(),
             counts.data_ptr<int>(), dlogits.data_ptr(), (int)T, (int)E, (int)K, renorm, (float)aux_alpha,
             (float)z_beta, aux.data_ptr<float>(), stream());
  return {dlogits, aux};
}


// ---- attention -----------------------------------------------------------------
namespace {
AttnTensors attn_desc(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                      const c10::optional<at::Tensor>& kr, int64_t seq, bool causal, int64_t window, double scale) {
  TORCH_CHECK(q.dim() == 3 && k.dim() == 3 && v.dim() == 3, "attention: q/k/v must be [T, heads, dim]");
  for (const at::Tensor* t : {&q, &k, &v}) {
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kBFloat16 && t->stride(2) == 1,
                "attention: q/k/v must be CUDA bf16 with a contiguous last dim");
  }
  AttnTensors a{};
  a.q = q.data_ptr(); a.q_row = q.stride(0); a.q_head = q.stride(1);
  a.k = k.data_ptr(); a.k_row = k.stride(0); a.k_head = k.stride(1);
  a.v = v.data_ptr(); a.v_row = v.stride(0); a.v_head = v.stride(1);
  a.T = (int)q.size(0); a.S = (int)seq; a.H = (int)q.size(1); a.Hk = (int)k.size(1);
  a.DQ = (int)q.size(2); a.DV = (int)v.size(2);
  a.DR = 0;
  if (kr.has_value()) {
    TORCH_CHECK(kr->dim() == 2 && kr->stride(1) == 1 && kr->scalar_type() == at::kBFloat16, "attention: k_rope [T, 64]");
    a.kr = kr->data_ptr(); a.kr_row = kr->stride(0); a.DR = (int)kr->size(1);
  }
  TORCH_CHECK(a.DQ == k.size(2) + a.DR, "attention: q dim must equal k dim (+ rope dim)");
  TORCH_CHECK(v.size(1) == k.size(1) && k.size(0) == q.size(0), "attention: k/v heads or tokens differ");
  a.causal = causal ? 1 : 0; a.window = (int)window; a.scale = (float)scale;
  return a;
}
}  // namespace

std::vector<at::Tensor> attn_fwd_t(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                                   const c10::optional<at::Tensor>& kr, int64_t seq, bool causal, int64_t window,
                                   double scale) {
  const c10::cuda::CUDAGuard g(q.device());
  AttnTensors a = attn_desc(q, k, v, kr, seq, causal, window, scale);
  auto o = at::empty({q.size(0), q.size(1), v.size(2)}, q.options());
  auto lse = at::empty({q.size(1), q.size(0)}, q.options().dtype(at::kFloat));
  attention_fwd(a, o.data_ptr(), lse.data_ptr<float>(), status_ptr(), stream());
  return {o, lse};
}

// Returns [dq, dk, dv] (+ dk_rope summed over heads).  Optional output buffers
// (which may be strided views into one gradient tensor) avoid extra copies.
std::vector<at::Tensor> attn_bwd_t(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                                   const c10::optional<at::Tensor>& kr, const at::Tensor& o, const at::Tensor& lse,
                                   const at::Tensor& dO, int64_t seq, bool causal, int64_t window, double scale,
                                   const c10::optional<at::Tensor>& dq_out, const c10::optional<at::Tensor>& dk_out,
                                   const c10::optional<at::Tensor>& dv_out) {
  const c10::cuda::CUDAGuard g(q.device());
  AttnTensors a = attn_desc(q, k, v, kr, seq, causal, window, scale);
  TORCH_CHECK(dO.is_contiguous() && o.is_contiguous(), "attention bwd: o and dO must be contiguous");
  auto dq = dq_out.has_value() ? *dq_out : at::empty(q.sizes(), q.options());
  auto dk = dk_out.has_value() ? *dk_out : at::empty(k.sizes(), k.options());
  auto dv = dv_out.has_value() ? *dv_out : at::empty(v.sizes(), v.options());
  TORCH_CHECK(dq.stride(2) == 1 && dk.stride(2) == 1 && dv.stride(2) == 1, "attention bwd: outputs need unit last stride");
  at::Tensor dkr_heads;
  if (kr.has_value()) dkr_heads = at::empty({q.size(0), k.size(1), kr->size(1)}, q.options());
  auto delta = at::empty({q.size(1), q.size(0)}, q.options().dtype(at::kFloat));
  attention_bwd(a, o.data_ptr(), lse.data_ptr<float>(), dO.data_ptr(), delta.data_ptr<float>(), dq.data_ptr(),
                dq.stride(0), dq.stride(1), dk.data_ptr(), dk.stride(0), dk.stride(1),
                kr.has_value() ? dkr_heads.data_ptr() : nullptr, kr.has_value() ? dkr_heads.stride(0) : 0,
                kr.has_value() ? dkr_heads.stride(1) : 0, dv.data_ptr(), dv.stride(0), dv.stride(1), status_ptr(),
                stream());
  if (kr.has_value()) return {dq, dk, dv, dkr_heads.sum(1)};
  return {dq, dk, dv};
}

// ---- decode attention --------------------------------------------------------
at::Tensor attn_decode_t(const at::Tensor& q, const at::Tensor& k, const c10::optional<at::Tensor>& v,
                         const c10::optional<at::Tensor>& ks, const c10::optional<at::Tensor>& vs,
                         const at::Tensor& q_pos, const at::Tensor& kv_len, int64_t window, double scale,
                         int64_t latent_v_dim, int64_t sink_rows, int64_t n_sink) {
  check_bf16(q, "q");
  check_i32(q_pos, "q_pos");
  check_i32(kv_len, "kv_len");
  TORCH_CHECK(q.dim() == 4, "attn_decode: q must be [B, Tn, H, D]");
  const c10::cuda::CUDAGuard g(q.device());
  const int64_t B = q.size(0), Tn = q.size(1), H = q.size(2), DQ = q.size(3);
  const bool int8_kv = k.scalar_type() == at::kChar;
  TORCH_CHECK(int8_kv || k.scalar_type() == at::kBFloat16, "attn_decode: cache must be bf16 or int8");
  TORCH_CHECK(k.is_cuda() && k.stride(-1) == 1, "attn_decode: cache rows must be contiguous");
  int64_t Hk, DV, L = k.size(1);
  long long v_b = 0, v_l = 0;
  if (!v.has_value()) {
    TORCH_CHECK(k.dim() == 3 && k.size(2) == DQ && latent_v_dim > 0 && latent_v_dim <= DQ,
                "attn_decode: latent cache [B, L, DQ] with 0 < latent_v_dim <= DQ");
    Hk = 1;
    DV = latent_v_dim;
  } else {
    TORCH_CHECK(k.dim() == 4 && k.size(3) == DQ && k.stride(2) == DQ, "attn_decode: k [B, L, Hk, D]");
    TORCH_CHECK(v->dim() == 4 && v->scalar_type() == k.scalar_type() && v->stride(-1) == 1 &&
                    v->stride(2) == v->size(3) && v->size(2) == k.size(2),
                "attn_decode: v [B, L, Hk, Dv]");
    Hk = k.size(2);
    DV = v->size(3);
    v_b = v->stride(0);
    v_l = v->stride(1);
  }
  TORCH_CHECK(H % Hk == 0, "attn_decode: heads must be a multiple of kv heads");
  TORCH_CHECK(0 <= n_sink && n_sink <= sink_rows && sink_rows <= L, "attn_decode: memory rows");
  long long s_b = 0, s_l = 0;
  if (int8_kv) {
    TORCH_CHECK(ks.has_value() && ks->scalar_type() == at::kFloat && ks->is_cuda(), "attn_decode: int8 needs k scales");
    s_b = ks->stride(0);
    s_l = ks->stride(1);
    if (v.has_value()) {
      TORCH_CHECK(vs.has_value() && vs->stride(0) == s_b && vs->stride(1) == s_l, "attn_decode: v scales");
    }
  }
  const DecodePlan pl = decode_plan((int)B, (int)Tn, (int)H, (int)Hk, (int)L, (int)DQ, (int)DV, !v.has_value(),
                                    (int)window, (int)sink_rows, int8_kv ? 1 : 2);
  auto ws = at::empty({(int64_t)pl.ws_floats}, q.options().dtype(at::kFloat));
  auto out = at::empty({B, Tn, H, DV}, q.options());
  attn_decode(q.data_ptr(), k.data_ptr(), v.has_value() ? v->data_ptr() : nullptr,
              int8_kv ? ks->data_ptr<float>() : nullptr,
              (int8_kv && vs.has_value()) ? vs->data_ptr<float>() : nullptr, int8_kv, q_pos.data_ptr<int>(),
              kv_len.data_ptr<int>(), out.data_ptr(), ws.data_ptr<float>(), (int)B, (int)Tn, (int)H, (int)Hk, (int)L,
              (int)DQ, (int)DV, k.stride(0), k.stride(1), v_b, v_l, s_b, s_l, (int)window, (float)scale, pl,
              (int)sink_rows, (int)n_sink, status_ptr(), stream());
  return out;
}

// ---- KV-cache append ---------------------------------------------------------------
void kv_cache_write_t(const at::Tensor& src, const at::Tensor& pos, at::Tensor& dst,
                      const c10::optional<at::Tensor>& scale, int64_t row_offset) {
  check_bf16(src, "src");
  TORCH_CHECK(src.dim() == 4 && src.is_contiguous(), "kv_cache_write: src must be a contiguous [B, T, G, D]");
  TORCH_CHECK(pos.scalar_type() == at::kLong && pos.is_contiguous() && pos.dim() == 2, "kv_cache_write: pos int64 [B, T]");
  const int64_t B = src.size(0), T = src.size(1), G = src.size(2), D = src.size(3);
  TORCH_CHECK(pos.size(0) == B && pos.size(1) == T, "kv_cache_write: pos shape");
  TORCH_CHECK(D <= 1024, "kv_cache_write: D <= 1024");
  TORCH_CHECK(dst.is_cuda() && dst.size(0) == B && dst.numel() == B * dst.size(1) * G * D && dst.stride(-1) == 1,
              "kv_cache_write: dst [B, L, G, D] with contiguous rows");
  const int64_t d_b = dst.stride(0), d_l = dst.stride(1);
  TORCH_CHECK(d_l >= G * D, "kv_cache_write: dst row stride");
  const bool int8 = dst.scalar_type() == at::kChar;
  int64_t s_b = 0, s_l = 0;
  if (int8) {
    TORCH_CHECK(scale.has_value() && scale->scalar_type() == at::kFloat && scale->stride(-1) == 1,
                "kv_cache_write: int8 cache needs fp32 scales");
    s_b = scale->stride(0);
    s_l = scale->stride(1);
  } else {
    TORCH_CHECK(dst.scalar_type() == at::kBFloat16 && D % 8 == 0, "kv_cache_write: bf16 cache with D % 8 == 0");
  }
  const c10::cuda::CUDAGuard g(src.device());
  kv_cache_write(src.data_ptr(), reinterpret_cast<const long long*>(pos.data_ptr<int64_t>()), dst.data_ptr(), int8 ? scale->data_ptr<float>() : nullptr,
                 int8, (int)B, (int)T, (int)G, (int)D, d_b, d_l, s_b, s_l, (int)row_offset, (int)dst.size(1),
                 stream());
}

// ---- int4 weight-only linear ----------------------------------------------------
at::Tensor int4_gemv_t(const at::Tensor& x, const at::Tensor& w, const at::Tensor& scale, double offset) {
  check_bf16(x, "x");
  check_f32(scale, "scale");
  TORCH_CHECK(w.is_cuda() && w.scalar_type() == at::kByte && w.is_contiguous() && w.dim() == 2, "int4: packed uint8 [N, ldw]");
  const c10::cuda::CUDAGuard g(x.device());
  const int64_t M = x.size(0), K = x.size(1), N = w.size(0), ldw = w.size(1);
  TORCH_CHECK(M <= 8, "int4_gemv: at most 8 rows (use int4_dequant + gemm)");
  TORCH_CHECK(K % 8 == 0 && 2 * ldw >= K && ldw % 16 == 0, "int4_gemv: K % 8 == 0, rows padded to 32 bytes");
  TORCH_CHECK(scale.numel() == N, "int4_gemv: one scale per row");
  auto y = at::empty({M, N}, x.options());
  int4_gemv(x.data_ptr(), w.data_ptr<uint8_t>(), scale.data_ptr<float>(), y.data_ptr(), (int)M, (int)N, (int)K, (int)ldw,
            (float)offset, stream());
  return y;
}

at::Tensor int4_dequant_t(const at::Tensor& w, const at::Tensor& scale, int64_t K, double offset) {
  check_f32(scale, "scale");
  TORCH_CHECK(w.is_cuda() && w.scalar_type() == at::kByte && w.is_contiguous() && w.dim() == 2, "int4: packed uint8 [N, ldw]");
  TORCH_CHECK(K % 8 == 0 && 2 * w.size(1) >= K && w.size(1) % 4 == 0, "int4_dequant: K % 8 == 0");
  const c10::cuda::CUDAGuard g(w.device());
  auto out = at::empty({w.size(0), K}, w.options().dtype(at::kBFloat16));
  int4_dequant(w.data_ptr<uint8_t>(), scale.data_ptr<float>(), out.data_ptr(), (int)w.size(0), (int)K, (int)w.size(1),
               (float)offset, stream());
  return out;
}

// ---- Gaussian splatting ------------------------------------------------------
std::vector<at::Tensor> gsplat_forward_t(const at::Tensor& u, const at::Tensor& v, const at::Tensor& sx,
                                         const at::Tensor& sy, const at::Tensor& opa, const at::Tensor& rgb,
                                         const c10::optional<at::Tensor>& z, int64_t H, int64_t W, int64_t k) {
  for (const at::Tensor* t : {&u, &v, &sx, &sy, &opa, &rgb}) check_f32(*t, "gsplat input");
  const c10::cuda::CUDAGuard g(u.device());
  const int64_t B = u.size(0), N = u.size(1);
  TORCH_CHECK(rgb.numel() == B * N * 3 && opa.numel() == B * N, "gsplat: shapes");
  auto acc = at::empty({B, 5, H, W}, u.options());
  auto out = at::empty({B, 3, H, W}, u.options());
  at::Tensor depth;
  if (z.has_value()) {
    check_f32(*z, "z");
    depth = at::empty({B, 1, H, W}, u.options());
  }
  gsplat_forward(u.data_ptr<float>(), v.data_ptr<float>(), sx.data_ptr<float>(), sy.data_ptr<float>(),
                 opa.data_ptr<float>(), rgb.data_ptr<float>(), z.has_value() ? z->data_ptr<float>() : nullptr,
                 acc.data_ptr<float>(), out.data_ptr<float>(), z.has_value() ? depth.data_ptr<float>() : nullptr,
                 (int)B, (int)N, (int)H, (int)W, (int)k, stream());
  if (z.has_value()) return {out, depth};
  return {out};
}

// ---- speculative verify ------------------------------------------------------
// -> (n_acc [B] int32, next [B] (draft dtype), new_len [B] (base_len dtype))
std::vector<at::Tensor> spec_verify_t(const at::Tensor& logits, const c10::optional<at::Tensor>& pdraft,
                                      const at::Tensor& draft, const c10::optional<at::Tensor>& u,
                                      const at::Tensor& base_len, double temperature) {
  check_f32(logits, "logits");
  TORCH_CHECK(logits.dim() == 3, "spec_verify: logits [B, K+1, V]");
  const int64_t B = logits.size(0), K = logits.size(1) - 1, V = logits.size(2);
  TORCH_CHECK(draft.is_cuda() && draft.is_contiguous() && draft.dim() == 2 && draft.size(0) == B &&
                  draft.size(1) == K && (draft.scalar_type() == at::kLong || draft.scalar_type() == at::kInt),
              "spec_verify: draft tokens [B, K] int32/int64");
  TORCH_CHECK(base_len.is_cuda() && base_len.is_contiguous() && base_len.numel() == B &&
                  (base_len.scalar_type() == at::kLong || base_len.scalar_type() == at::kInt),
              "spec_verify: base_len [B] int32/int64");
  TORCH_CHECK(K >= 0 && V > 0 && V < (1 << 30), "spec_verify: sizes");
  const bool sample = temperature > 0;
  if (sample) {
    TORCH_CHECK(pdraft.has_value() && u.has_value(), "spec_verify: sampling needs draft probabilities and uniforms");
    check_f32(*pdraft, "pdraft");
    check_f32(*u, "u");
    TORCH_CHECK(pdraft->numel() == B * K * V && u->numel() == B * (K + 1), "spec_verify: pdraft [B, K, V], u [B, K+1]");
  }
  const c10::cuda::CUDAGuard g(logits.device());
  auto n_acc = at::empty({B}, logits.options().dtype(at::kInt));
  auto next = at::empty({B}, draft.options());
  auto new_len = at::empty_like(base_len);
  spec_verify(logits.data_ptr<float>(), sample ? pdraft->data_ptr<float>() : nullptr, draft.data_ptr(),
              draft.scalar_type() == at::kLong, sample ? u->data_ptr<float>() : nullptr, base_len.data_ptr(),
              base_len.scalar_type() == at::kLong, (int)B, (int)K, (int)V, (float)temperature, n_acc.data_ptr<int>(),
              next.data_ptr(), new_len.data_ptr(), stream());
  return {n_acc, next, new_len};
}

void register_kernels(pybind11::module_& m) {
  m.def("rmsnorm_fwd", &rmsnorm_fwd_t, py::arg("x"), py::arg("res"), py::arg("w"), py::arg("eps"));
  m.def("rmsnorm_bwd", &rmsnorm_bwd_t, py::arg("x"), py::arg("w"), py::arg("rstd"), py::arg("dy"), py::arg("dres"));
  m.def("layernorm_fwd", &layernorm_fwd_t);
  m.def("layernorm_bwd", &layernorm_bwd_t);
  m.def("rope", &rope_t, py::arg("x"), py::arg("cs"), py::arg("pos"), py::arg("pos0"), py::arg("seq"),
        py::arg("tokens"), py::arg("heads"), py::arg("row_stride"), py::arg("head_stride"), py::arg("off"),
        py::arg("rot"), py::arg("interleaved"), py::arg("sign"));
  m.def("embedding_fwd", &embedding_fwd_t);
  m.def("embedding_bwd", &embedding_bwd_t);
  m.def("cross_entropy", &cross_entropy_t, py::arg("logits"), py::arg("labels"), py::arg("dlogits"),
        py::arg("grad_scale"), py::arg("z_loss"));
  m.def("adamw", &adamw_t, py::arg("p"), py::arg("m"), py::arg("v"), py::arg("g"), py::arg("p_bf16"), py::arg("lr"),
        py::arg("beta1"), py::arg("beta2"), py::arg("eps"), py::arg("wd"), py::arg("step"), py::arg("grad_scale"),
        py::arg("norm_sq"), py::arg("max_norm"));
  m.def("sq_norm", &sq_norm_t);
  m.def("adamw_multi", &adamw_multi_t, py::arg("p"), py::arg("m"), py::arg("v"), py::arg("g"), py::arg("p_bf16"),
        py::arg("wd"), py::arg("lr"), py::arg("b1"), py::arg("b2"), py::arg("eps"), py::arg("step"),
        py::arg("grad_scale"), py::arg("norm_sq") = py::none(), py::arg("max_norm") = 0.0);
  m.def("sq_norm_multi", &sq_norm_multi_t);
  m.def("router_topk", &router_topk_t);
  m.def("kv_cache_write", &kv_cache_write_t, py::arg("src"), py::arg("pos"), py::arg("dst"), py::arg("scale"),
        py::arg("row_offset"));
  m.def("spec_verify", &spec_verify_t, py::arg("logits"), py::arg("pdraft"), py::arg("draft"), py::arg("u"),
        py::arg("base_len"), py::arg("temperature"));
  m.def("moe_plan", &moe_plan_t, py::arg("idx"), py::arg("E"), py::arg("capacity"), py::arg("cap_rows"),
        py::arg("align") = 128);
  m.def("moe_gather", &moe_gather_t);
  m.def("moe_combine", &moe_combine_t);
  m.def("moe_combine_bwd", &moe_combine_bwd_t);
  m.def("moe_scatter_add", &moe_scatter_add_t);
  m.def("router_bwd", &router_bwd_t);
  m.def("gsplat_forward", &gsplat_forward_t);
  m.def("int4_gemv", &int4_gemv_t, py::arg("x"), py::arg("w"), py::arg("scale"), py::arg("offset"));
  m.def("int4_dequant", &int4_dequant_t, py::arg("w"), py::arg("scale"), py::arg("K"), py::arg("offset"));
  m.def("decode_rows_limit", [](int64_t DQ, int64_t DV, bool latent, int64_t Hk) -> int64_t {
    return (latent && Hk == 1 && decode_plan(1, 1, 1, 1, 1, (int)DQ, (int)DV, true, 0, 0, 2).tc) ? (1 << 20) : 64;
  }, "query rows (tokens x heads per kv group) one decode call takes");
  m.def("attn_decode", &attn_decode_t, py::arg("q"), py::arg("k"), py::arg("v"), py::arg("k_scale"),
        py::arg("v_scale"), py::arg("q_pos"), py::arg("kv_len"), py::arg("window"), py::arg("scale"),
        py::arg("latent_v_dim"), py::arg("sink_rows") = 0, py::arg("n_sink") = 0);
  m.def("attn_fwd", &attn_fwd_t, py::arg("q"), py::arg("k"), py::arg("v"), py::arg("k_rope"), py::arg("seq"),
        py::arg("causal"), py::arg("window"), py::arg("scale"));
  m.def("attn_bwd", &attn_bwd_t, py::arg("q"), py::arg("k"), py::arg("v"), py::arg("k_rope"), py::arg("o"),
        py::arg("lse"), py::arg("dO"), py::arg("seq"), py::arg("causal"), py::arg("window"), py::arg("scale"),
        py::arg("dq_out") = py::none(), py::arg("dk_out") = py::none(), py::arg("dv_out") = py::none());
}

}  // namespace omni
