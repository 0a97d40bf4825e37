// torch.ops.omnicoder: the reference's native operator namespace
// (src/omnicoder/modeling/kernels/dml_fused_attention.cpp:1-97, registered for
// DirectML there) as dispatcher operators with CUDA kernels for sm_100a and
// ATen CPU implementations.
//
//   omnicoder::mla(q, k, v, mask=None, is_causal=False) -> Tensor
//       q [BH, Tq, D], k [BH, Tk, D], v [BH, Tk, Dv]; softmax(q k^T / sqrt(D)) v
//       with an optional additive / boolean mask.  CUDA, bf16, no mask,
//       Tq == Tk a multiple of 128, D and Dv in {64, 128}: the tcgen05 flash
//       attention kernel, reading the [BH, T, D] tensors in place as
//       [T, BH, D] views.  Other CUDA cases run ATen's scaled_dot_product_attention.
//   omnicoder::matmul_int4(x, packed, scale, zero=None, offset=8.0) -> Tensor
//       y = x @ W^T with W[n, k] = (nibble[n, k] - z[n]) * scale[n], nibbles
//       packed two per byte, element 2i in the low nibble; z = zero when given,
//       else the constant offset (zero may hold one value or one per row).
//       CUDA: at most 8 rows of bf16 x run the int4 GEMV kernel, otherwise the
//       weight is dequantised to bf16 once by a kernel and multiplied.  With a
//       zero tensor the kernels run centred at 8 and (8 - z[n]) * scale[n] *
//       sum_k x[k] is added in fp32, which stays small for zero points near the
//       middle of the nibble range.
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

#include <cmath>
#include <vector>

namespace omni {

std::vector<at::Tensor> attn_fwd_t(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                                   const c10::optional<at::Tensor>& kr, int64_t seq, bool causal, int64_t window,
                                   double scale);
at::Tensor int4_gemv_t(const at::Tensor& x, const at::Tensor& w, const at::Tensor& scale, double offset);
at::Tensor int4_dequant_t(const at::Tensor& w, const at::Tensor& scale, int64_t K, double offset);

namespace {

at::Tensor mla_cpu(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const c10::optional<at::Tensor>& mask,
                   bool is_causal) {
  return at::scaled_dot_product_attention(q, k, v, mask, 0.0, is_causal);
}

bool mla_kernel_ok(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                   const c10::optional<at::Tensor>& mask) {
  if (mask.has_value() || q.dim() != 3 || k.dim() != 3 || v.dim() != 3) return false;
  for (const at::Tensor* t : {&q, &k, &v})
    if (t->scalar_type() != at::kBFloat16 || t->stride(2) != 1 || t->stride(1) % 8 != 0 || t->stride(0) % 8 != 0 ||
        reinterpret_cast<uintptr_t>(t->data_ptr()) % 16 != 0)
      return false;
  const int64_t T = q.size(1), D = q.size(2), Dv = v.size(2);
  return k.size(1) == T && v.size(1) == T && T % 128 == 0 && k.size(2) == D && (D == 64 || D == 128) &&
         (Dv == 64 || Dv == 128) && k.size(0) == q.size(0) && v.size(0) == q.size(0);
}

at::Tensor mla_cuda(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                    const c10::optional<at::Tensor>& mask, bool is_causal) {
  if (!mla_kernel_ok(q, k, v, mask)) return at::scaled_dot_product_attention(q, k, v, mask, 0.0, is_causal);
  const int64_t T = q.size(1);
  auto r = attn_fwd_t(q.transpose(0, 1), k.transpose(0, 1), v.transpose(0, 1), c10::nullopt, T, is_causal, 0,
                      1.0 / std::sqrt((double)q.size(2)));
  return r[0].transpose(0, 1).contiguous();
}

at::Tensor zero_or_offset(const at::Tensor& scale, const c10::optional<at::Tensor>& zero, double offset) {
  return zero.has_value() ? zero->to(at::kFloat).reshape({-1}) : at::full({scale.numel()}, offset, scale.options().dtype(at::kFloat));
}

at::Tensor matmul_int4_cpu(const at::Tensor& x, const at::Tensor& packed, const at::Tensor& scale,
                           const c10::optional<at::Tensor>& zero, double offset) {
  const int64_t K = x.size(-1), N = packed.size(0);
  auto lo = at::bitwise_and(packed, 0x0F);
  auto hi = at::bitwise_and(at::bitwise_right_shift(packed, 4), 0x0F);
  auto q = at::stack({lo, hi}, -1).reshape({N, -1}).slice(1, 0, K).to(at::kFloat);
  auto w = (q - zero_or_offset(scale, zero, offset).unsqueeze(1)) * scale.to(at::kFloat).reshape({-1, 1});
  return at::matmul(x.to(at::kFloat), w.t()).to(x.scalar_type());
}

at::Tensor matmul_int4_cuda(const at::Tensor& x, const at::Tensor& packed, const at::Tensor& scale,
                            const c10::optional<at::Tensor>& zero, double offset) {
  const c10::cuda::CUDAGuard g(x.device());
  const int64_t K = x.size(-1), N = packed.size(0);
  TORCH_CHECK(packed.scalar_type() == at::kByte && packed.dim() == 2 && 2 * packed.size(1) >= K,
              "matmul_int4: packed must be uint8 [N, >= K/2]");
  if (K % 8 != 0) return matmul_int4_cpu(x, packed, scale, zero, offset);
  auto x2 = x.reshape({-1, K}).to(at::kBFloat16).contiguous();
  auto sc = scale.to(at::kFloat).reshape({-1}).contiguous();
  auto pk = packed.contiguous();
  const double base = zero.has_value() ? 8.0 : offset;
  at::Tensor y;
  if (x2.size(0) <= 8 && pk.size(1) % 16 == 0) {
    y = int4_gemv_t(x2, pk, sc, base);
  } else {
    y = at::matmul(x2, int4_dequant_t(pk, sc, K, base).t());
  }
  if (zero.has_value()) {
    auto shift = (8.0 - zero->to(at::kFloat).reshape({1, -1})) * sc.reshape({1, -1});
    y = (y.to(at::kFloat) + x2.to(at::kFloat).sum(1, true) * shift).to(at::kBFloat16);
  }
  std::vector<int64_t> shape(x.sizes().begin(), x.sizes().end());
  shape.back() = N;
  return y.view(shape).to(x.scalar_type());
}

}  // namespace
}  // namespace omni

TORCH_LIBRARY(omnicoder, m) {
  m.def("mla(Tensor q, Tensor k, Tensor v, Tensor? mask=None, bool is_causal=False) -> Tensor");
  m.def("matmul_int4(Tensor x, Tensor packed, Tensor scale, Tensor? zero=None, float offset=8.0) -> Tensor");
}

TORCH_LIBRARY_IMPL(omnicoder, CPU, m) {
  m.impl("mla", &omni::mla_cpu);
  m.impl("matmul_int4", &omni::matmul_int4_cpu);
}

TORCH_LIBRARY_IMPL(omnicoder, CUDA, m) {
  m.impl("mla", &omni::mla_cuda);
  m.impl("matmul_int4", &omni::matmul_int4_cuda);
}
