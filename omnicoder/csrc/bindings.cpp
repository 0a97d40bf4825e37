// Python bindings of the omnicoder sm_100a kernels (module omnicoder._C).
//
// Every entry point validates devices, dtypes, shapes and alignment on the
// host and launches on the current PyTorch CUDA stream.  Kernels report
// device-side failures (bounded waits that ran out, failed bounds checks) in a
// per-device status block that `status()` reads.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <algorithm>
#include <cstdlib>
#include <mutex>
#include <vector>

#include "gemm_sm100.h"
#include "kernels.h"

namespace omni {

// ---------------------------------------------------------------------------
// Status block (one per device, allocated on first use, never freed)
// ---------------------------------------------------------------------------
static std::mutex g_status_mu;
static std::vector<void*> g_status(64, nullptr);

void* status_ptr() {
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lk(g_status_mu);
  if (g_status[dev] == nullptr) {
    void* p = nullptr;
    C10_CUDA_CHECK(cudaMalloc(&p, 16));
    C10_CUDA_CHECK(cudaMemset(p, 0, 16));
    g_status[dev] = p;
  }
  return g_status[dev];
}

std::vector<int64_t> status_read() {
  int h[4] = {0, 0, 0, 0};
  C10_CUDA_CHECK(cudaMemcpy(h, status_ptr(), 16, cudaMemcpyDeviceToHost));
  return {h[0], h[1], h[2]};
}

void status_reset() { C10_CUDA_CHECK(cudaMemset(status_ptr(), 0, 16)); }

#define CHECK_CUDA_T(x) TORCH_CHECK((x).is_cuda(), #x " must be a CUDA tensor")
#define CHECK_BF16(x) TORCH_CHECK((x).scalar_type() == at::kBFloat16, #x " must be bfloat16")
#define CHECK_ROWMAJOR(x) TORCH_CHECK((x).dim() >= 2 && (x).stride(-1) == 1, #x " must have a contiguous last dim")

static cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream().stream(); }

// ---------------------------------------------------------------------------
// GEMM
// ---------------------------------------------------------------------------
// Row count up to which dense GEMMs with K-major operands take the few-row
// (swap-AB) kernel; OMNI_SKINNY_MAX_ROWS overrides it (0 disables).
static int g_skinny_rows = -1;
static int skinny_rows() {
  if (g_skinny_rows < 0) {
    const char* e = std::getenv("OMNI_SKINNY_MAX_ROWS");
    g_skinny_rows = e ? std::max(0, std::min(std::atoi(e), kSkinnyMaxRows)) : 128;
  }
  return g_skinny_rows;
}
void set_skinny_rows(int64_t n) { g_skinny_rows = (int)std::max<int64_t>(0, std::min<int64_t>(n, kSkinnyMaxRows)); }

static void run_skinny(const at::Tensor& A, const at::Tensor& B, const int* offsets, int G, int rows, int N, int K,
                       long long w_group_stride, at::Tensor& C, int epilogue, double alpha,
                       const c10::optional<at::Tensor>& R) {
  SkinnyDesc sd;
  sd.M = rows;
  sd.N = N;
  sd.K = K;
  sd.G = G;
  sd.offsets = offsets;
  sd.X = A.data_ptr();
  sd.ldx = A.stride(0);
  sd.W = B.data_ptr();
  sd.ldw = B.stride(-2);
  sd.w_group_stride = w_group_stride;
  sd.status = status_ptr();
  if ((epilogue == EPI_STORE_BF16 || epilogue == EPI_SWIGLU) && C.scalar_type() == at::kBFloat16 &&
      skinny_ksplit(sd) == 1) {
    // every output tile is computed by one CTA: the epilogue writes C itself
    sd.out = C.data_ptr();
    sd.ldo = C.stride(0);
    sd.epilogue = epilogue;
    sd.alpha = (float)alpha;
    skinny_gemm_launch(sd, cur_stream());
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return;
  }
  auto acc = at::empty({(int64_t)rows, (int64_t)N}, A.options().dtype(at::kFloat));
  C10_CUDA_CHECK(cudaMemsetAsync(acc.data_ptr<float>(), 0, (size_t)rows * N * sizeof(float), cur_stream()));
  sd.acc = acc.data_ptr<float>();
  skinny_gemm_launch(sd, cur_stream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  skinny_finalize(acc.data_ptr<float>(), rows, N, epilogue, (float)alpha, C.data_ptr(), C.stride(0),
                  R.has_value() ? R->data_ptr() : nullptr, R.has_value() ? R->stride(0) : 0, cur_stream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
// Dense: C = alpha * op(A) op(B)^T.
//   a_mn=false: A [M,K]; a_mn=true: A [K,M].  b_mn=false: B [N,K]; b_mn=true: B [K,N].
void gemm(const at::Tensor& A, const at::Tensor& B, at::Tensor& C, bool a_mn, bool b_mn, int64_t epilogue,
          double alpha, const c10::optional<at::Tensor>& R, const c10::optional<at::Tensor>& H, int64_t block_n) {
  CHECK_CUDA_T(A);
  CHECK_CUDA_T(B);
  CHECK_CUDA_T(C);
  CHECK_BF16(A);
  CHECK_BF16(B);
  TORCH_CHECK(A.dim() == 2 && B.dim() == 2 && C.dim() == 2, "gemm: 2-D operands expected");
  CHECK_ROWMAJOR(A);
  CHECK_ROWMAJOR(B);
  CHECK_ROWMAJOR(C);
  const c10::cuda::CUDAGuard guard(A.device());
  GemmDesc d;
  d.mode = GEMM_DENSE;
  d.epilogue = (int)epilogue;
  d.block_n = (int)block_n;
  d.a_mn_major = a_mn;
  d.b_mn_major = b_mn;
  const int64_t M = a_mn ? A.size(1) : A.size(0);
  const int64_t K = a_mn ? A.size(0) : A.size(1);
  const int64_t N = b_mn ? B.size(1) : B.size(0);
  const int64_t Kb = b_mn ? B.size(0) : B.size(1);
  TORCH_CHECK(K == Kb, "gemm: reduction dims differ (", K, " vs ", Kb, ")");
  TORCH_CHECK(K % 8 == 0 && M > 0 && N > 0 && K > 0, "gemm: K must be a positive multiple of 8");
  d.M = (int)M;
  d.N = (int)N;
  d.K = (int)K;
  d.A = A.data_ptr();
  d.lda = A.stride(0);
  d.rows_a = A.size(0);
  d.K_extent_a = K;
  d.B = B.data_ptr();
  d.ldb = B.stride(0);
  d.K_extent_b = K;
  d.C = C.data_ptr();
  d.ldc = C.stride(0);
  d.alpha = (float)alpha;
  const int64_t out_cols = epilogue == EPI_SWIGLU ? N / 2 : (epilogue == EPI_SWIGLU_BWD ? 2 * N : N);
  TORCH_CHECK(C.size(0) == M && C.size(1) == out_cols, "gemm: output shape mismatch");
  if (epilogue == EPI_STORE_F32 || epilogue == EPI_ACCUM_F32) {
    TORCH_CHECK(C.scalar_type() == at::kFloat, "gemm: fp32 output expected");
  } else {
    CHECK_BF16(C);
  }
  if (epilogue == EPI_ADD_BF16 || epilogue == EPI_SWIGLU_BWD) {
    TORCH_CHECK(R.has_value(), "gemm: epilogue needs R");
    CHECK_BF16(R.value());
    CHECK_ROWMAJOR(R.value());
    d.R = R->data_ptr();
    d.ldr = R->stride(0);
  }
  if (epilogue == EPI_SWIGLU) {
    TORCH_CHECK(N % 64 == 0, "gemm swiglu: N must be a multiple of 64");
    if (H.has_value()) {
      CHECK_BF16(H.value());
      TORCH_CHECK(H->size(0) == M && H->size(1) == N, "gemm swiglu: H shape");
      d.H = H->data_ptr();
      d.ldh = H->stride(0);
    }
  }
  if (epilogue == EPI_SWIGLU_BWD) TORCH_CHECK(N % 32 == 0, "gemm swiglu bwd: N must be a multiple of 32");
  const bool skinny_epi = epilogue == EPI_STORE_BF16 || epilogue == EPI_STORE_F32 || epilogue == EPI_ADD_BF16 ||
                          (epilogue == EPI_SWIGLU && !H.has_value());
  if (!a_mn && !b_mn && skinny_epi && M <= skinny_rows()) {
    run_skinny(A, B, nullptr, 1, (int)M, (int)N, (int)K, 0, C, (int)epilogue, alpha, R);
    return;
  }
  d.status = status_ptr();
  gemm_sm100_launch(d, cur_stream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Few-row grouped GEMM: group g owns rows [offsets[g], offsets[g+1]) of A (at most
// `rows` rows in all, any alignment); B is [G, N, K].  Epilogues: bf16 store or
// SwiGLU (C then has N/2 columns).
void gemm_skinny_grouped(const at::Tensor& A, const at::Tensor& B, const at::Tensor& offsets, at::Tensor& C,
                         int64_t epilogue, double alpha, int64_t rows) {
  CHECK_CUDA_T(A);
  CHECK_BF16(A);
  CHECK_BF16(B);
  CHECK_BF16(C);
  CHECK_ROWMAJOR(A);
  CHECK_ROWMAJOR(C);
  TORCH_CHECK(B.dim() == 3 && B.is_contiguous(), "gemm_skinny_grouped: B must be a contiguous [G, N, K] stack");
  TORCH_CHECK(offsets.scalar_type() == at::kInt && offsets.is_cuda() && offsets.numel() == B.size(0) + 1,
              "gemm_skinny_grouped: offsets must be int32 [G+1] on the device");
  TORCH_CHECK(epilogue == EPI_STORE_BF16 || epilogue == EPI_SWIGLU, "gemm_skinny_grouped: bf16 or swiglu epilogue");
  const int64_t K = A.size(1), N = B.size(1);
  TORCH_CHECK(B.size(2) == K && K % 8 == 0, "gemm_skinny_grouped: reduction dims");
  TORCH_CHECK(rows >= 0 && rows <= A.size(0) && rows <= C.size(0), "gemm_skinny_grouped: rows");
  TORCH_CHECK(C.size(1) == (epilogue == EPI_SWIGLU ? N / 2 : N), "gemm_skinny_grouped: output columns");
  if (epilogue == EPI_SWIGLU) TORCH_CHECK(N % 64 == 0, "gemm_skinny_grouped: swiglu needs N % 64 == 0");
  const c10::cuda::CUDAGuard guard(A.device());
  if (rows == 0) return;
  run_skinny(A, B, offsets.data_ptr<int>(), (int)B.size(0), (int)rows, (int)N, (int)K, B.stride(0), C,
             (int)epilogue, alpha, c10::nullopt);
}

// Grouped-M: rows of A ([rows, K], K-major) segmented by offsets [G+1];
// B is [G, N, K] (b_mn=false) or [G, K, N] (b_mn=true).
void gemm_grouped_m(const at::Tensor& A, const at::Tensor& B, const at::Tensor& offsets, at::Tensor& C,
                    bool b_mn, int64_t epilogue, double alpha, const c10::optional<at::Tensor>& R,
                    const c10::optional<at::Tensor>& H, int64_t block_n, int64_t max_rows_hint,
                    int64_t ready_ptr, const c10::optional<at::Tensor>& ready_epoch,
                    const c10::optional<at::Tensor>& src_pref, int64_t nsrc, int64_t me) {
  CHECK_CUDA_T(A);
  CHECK_BF16(A);
  CHECK_BF16(B);
  CHECK_ROWMAJOR(A);
  TORCH_CHECK(B.dim() == 3 && B.is_contiguous(), "gemm_grouped_m: B must be a contiguous [G, ., .] stack");
  TORCH_CHECK(offsets.scalar_type() == at::kInt && offsets.is_cuda() && offsets.numel() == B.size(0) + 1,
              "gemm_grouped_m: offsets must be int32 [G+1] on the device");
  const c10::cuda::CUDAGuard guard(A.device());
  GemmDesc d;
  d.mode = GEMM_GROUPED_M;
  d.epilogue = (int)epilogue;
  d.block_n = (int)block_n;
  d.a_mn_major = false;
  d.b_mn_major = b_mn;
  const int64_t G = B.size(0);
  const int64_t K = A.size(1);
  const int64_t N = b_mn ? B.size(2) : B.size(1);
  TORCH_CHECK((b_mn ? B.size(1) : B.size(2)) == K, "gemm_grouped_m: reduction dims differ");
  TORCH_CHECK(K % 8 == 0, "gemm_grouped_m: K must be a multiple of 8");
  d.M = (int)A.size(0);
  d.N = (int)N;
  d.K = (int)K;
  d.A = A.data_ptr();
  d.lda = A.stride(0);
  d.rows_a = A.size(0);
  d.K_extent_a = K;
  d.B = B.data_ptr();
  d.ldb = B.stride(1);
  d.b_group_stride = B.stride(0);
  d.K_extent_b = K;
  d.num_groups = (int)G;
  d.group_offsets = offsets.data_ptr<int>();
  d.max_rows_hint = (int)max_rows_hint;
  d.C = C.data_ptr();
  d.ldc = C.stride(0);
  d.rows_c = C.size(0);
  d.alpha = (float)alpha;
  CHECK_BF16(C);
  CHECK_ROWMAJOR(C);
  if (epilogue == EPI_SWIGLU_BWD) {
    TORCH_CHECK(R.has_value(), "gemm_grouped_m: swiglu bwd needs R");
    d.R = R->data_ptr();
    d.ldr = R->stride(0);
  }
  if (epilogue == EPI_SWIGLU && H.has_value()) {
    d.H = H->data_ptr();
    d.ldh = H->stride(0);
  }
  if (ready_ptr != 0) {
    TORCH_CHECK(ready_epoch.has_value() && src_pref.has_value() && ready_epoch->is_cuda() &&
                    src_pref->scalar_type() == at::kInt && src_pref->numel() == B.size(0) * (nsrc + 1),
                "gemm_grouped_m: readiness gating needs the epoch counter and src_pref [G, ranks + 1]");
    d.ready = reinterpret_cast<const unsigned*>(ready_ptr);
    d.ready_epoch = reinterpret_cast<const unsigned*>(ready_epoch->data_ptr());
    d.src_pref = src_pref->data_ptr<int>();
    d.nsrc = (int)nsrc;
    d.me = (int)me;
  }
  d.status = status_ptr();
  gemm_sm100_launch(d, cur_stream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Expert-parallel combine from the GEMM epilogue: per-expert products of A's row groups, each output
// row r stored to its origin: peer_ptrs[s] + i * D (bf16) with (-, s, i, -) = meta[r] (int4 rows;
// s < 0 marks padding).  dest_rows bounds i.  B [G, N, K] (b_mn: [G, K, N]).
void gemm_grouped_m_push(const at::Tensor& A, const at::Tensor& B, const at::Tensor& offsets, const at::Tensor& meta,
                         const std::vector<int64_t>& peer_ptrs, int64_t dest_rows, bool b_mn, int64_t max_rows_hint) {
  CHECK_CUDA_T(A);
  CHECK_BF16(A);
  CHECK_BF16(B);
  CHECK_ROWMAJOR(A);
  TORCH_CHECK(B.dim() == 3 && B.is_contiguous(), "gemm_grouped_m_push: B must be a contiguous [G, ., .] stack");
  TORCH_CHECK(offsets.scalar_type() == at::kInt && offsets.is_cuda() && offsets.numel() == B.size(0) + 1,
              "gemm_grouped_m_push: offsets must be int32 [G+1] on the device");
  TORCH_CHECK(meta.scalar_type() == at::kInt && meta.is_cuda() && meta.is_contiguous() && meta.dim() == 2 &&
                  meta.size(1) == 4 && meta.size(0) >= A.size(0), "gemm_grouped_m_push: meta int32 [rows, 4]");
  TORCH_CHECK(!peer_ptrs.empty() && peer_ptrs.size() <= (size_t)GEMM_MAX_PEERS, "gemm_grouped_m_push: 1..8 ranks");
  const c10::cuda::CUDAGuard guard(A.device());
  GemmDesc d;
  d.mode = GEMM_GROUPED_M;
  d.epilogue = EPI_EP_PUSH;
  d.block_n = 256;
  d.b_mn_major = b_mn;
  const int64_t K = A.size(1);
  const int64_t N = b_mn ? B.size(2) : B.size(1);
  TORCH_CHECK((b_mn ? B.size(1) : B.size(2)) == K && K % 8 == 0 && N % 8 == 0, "gemm_grouped_m_push: dims");
  d.M = (int)A.size(0);
  d.N = (int)N;
  d.K = (int)K;
  d.A = A.data_ptr();
  d.lda = A.stride(0);
  d.rows_a = A.size(0);
  d.K_extent_a = K;
  d.B = B.data_ptr();
  d.ldb = B.stride(1);
  d.b_group_stride = B.stride(0);
  d.K_extent_b = K;
  d.num_groups = (int)B.size(0);
  d.group_offsets = offsets.data_ptr<int>();
  d.max_rows_hint = (int)max_rows_hint;
  d.ldc = N;
  d.rows_c = A.size(0);
  d.nsrc = (int)peer_ptrs.size();
  d.src_rows = (int)dest_rows;
  for (size_t r = 0; r < peer_ptrs.size(); ++r) d.peer_c[r] = reinterpret_cast<void*>(peer_ptrs[r]);
  d.row_meta = meta.data_ptr();
  d.status = status_ptr();
  gemm_sm100_launch(d, cur_stream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ---------------------------------------------------------------------------
// Block-scaled fp8 (1 x 128 activation scales, 128 x 128 weight scales)
// ---------------------------------------------------------------------------
std::vector<at::Tensor> fp8_quant_act_t(const at::Tensor& x, bool pow2, const c10::optional<at::Tensor>& offsets) {
  CHECK_CUDA_T(x);
  CHECK_BF16(x);
  CHECK_ROWMAJOR(x);
  TORCH_CHECK(x.dim() == 2 && x.size(1) % 128 == 0, "fp8_quant_act: x [M, K] with K % 128 == 0");
  const c10::cuda::CUDAGuard guard(x.device());
  const int64_t M = x.size(0), K = x.size(1), Mp = (M + 127) / 128 * 128;
  auto xq = at::empty({M, K}, x.options().dtype(at::kFloat8_e4m3fn));
  auto sx = at::empty({K / 128, Mp}, x.options().dtype(at::kFloat));
  const int* limit = nullptr;
  if (offsets.has_value()) {
    TORCH_CHECK(offsets->scalar_type() == at::kInt && offsets->is_cuda() && offsets->numel() >= 1,
                "fp8_quant_act: offsets int32 on the device");
    limit = offsets->data_ptr<int>() + (offsets->numel() - 1);
  }
  fp8_quant_act(x.data_ptr(), x.stride(0), (int)M, (int)K, xq.data_ptr(), sx.data_ptr<float>(), Mp, pow2, cur_stream(),
                limit);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {xq, sx};
}

std::vector<at::Tensor> fp8_quant_weight_t(const at::Tensor& w, bool pow2) {
  CHECK_CUDA_T(w);
  CHECK_BF16(w);
  TORCH_CHECK(w.is_contiguous() && (w.dim() == 2 || w.dim() == 3), "fp8_quant_weight: contiguous [N, K] or [G, N, K]");
  const c10::cuda::CUDAGuard guard(w.device());
  const int64_t G = w.dim() == 3 ? w.size(0) : 1, N = w.size(-2), K = w.size(-1);
  TORCH_CHECK(K % 128 == 0, "fp8_quant_weight: K % 128 == 0");
  auto wq = at::empty_like(w, w.options().dtype(at::kFloat8_e4m3fn));
  auto sw = at::empty({G, (N + 127) / 128, K / 128}, w.options().dtype(at::kFloat));
  fp8_quant_weight(w.data_ptr(), (int)G, (int)N, (int)K, wq.data_ptr(), sw.data_ptr<float>(), pow2, cur_stream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {wq, sw};
}

std::vector<at::Tensor> fp8_quant_t_t(const at::Tensor& x) {
  CHECK_CUDA_T(x);
  CHECK_BF16(x);
  CHECK_ROWMAJOR(x);
  TORCH_CHECK(x.dim() == 2 && x.size(0) % 128 == 0 && x.size(1) % 8 == 0,
              "fp8_quant_t: x [T, C] with T % 128 == 0 and C % 8 == 0");
  const c10::cuda::CUDAGuard guard(x.device());
  const int64_t T = x.size(0), Cn = x.size(1), Cp = (Cn + 255) / 256 * 256;  // A or per-row B scales
  auto xt = at::empty({Cn, T}, x.options().dtype(at::kFloat8_e4m3fn));
  auto st = at::ones({T / 128, Cp}, x.options().dtype(at::kFloat));
  fp8_quant_t(x.data_ptr(), x.stride(0), (int)T, (int)Cn, xt.data_ptr(), T, st.data_ptr<float>(), Cp, cur_stream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {xt, st};
}

// C [M, N] bf16 = fp8 GEMM; grouped when offsets is given (wq [G, N, K], offsets int32 [G+1],
// multiples of 128, rows = allocated rows of xq).
void fp8_gemm_t(const at::Tensor& xq, const at::Tensor& sx, const at::Tensor& wq, const at::Tensor& sw, at::Tensor& C,
                const c10::optional<at::Tensor>& offsets, int64_t max_rows, bool scaled_mma, bool sw_rows) {
  CHECK_CUDA_T(xq);
  TORCH_CHECK(xq.scalar_type() == at::kFloat8_e4m3fn && wq.scalar_type() == at::kFloat8_e4m3fn,
              "fp8_gemm: e4m3 operands");
  TORCH_CHECK(sx.scalar_type() == at::kFloat && sw.scalar_type() == at::kFloat && sx.is_contiguous() &&
                  sw.is_contiguous(), "fp8_gemm: fp32 contiguous scales");
  CHECK_BF16(C);
  CHECK_ROWMAJOR(C);
  CHECK_ROWMAJOR(xq);
  TORCH_CHECK(wq.is_contiguous(), "fp8_gemm: contiguous weights");
  const c10::cuda::CUDAGuard guard(xq.device());
  Fp8GemmDesc d;
  d.M = (int)xq.size(0);
  d.K = (int)xq.size(1);
  d.N = (int)wq.size(-2);
  TORCH_CHECK(wq.size(-1) == d.K && d.K % 128 == 0, "fp8_gemm: K mismatch or K % 128 != 0");
  TORCH_CHECK(sx.dim() == 2 && sx.size(0) == d.K / 128 && sx.size(1) >= (d.M + 127) / 128 * 128,
              "fp8_gemm: sx [K/128, >= M rounded up to 128]");
  TORCH_CHECK(C.size(0) == d.M && C.size(1) == d.N && C.stride(0) % 8 == 0, "fp8_gemm: C [M, N], row stride % 8");
  d.X = xq.data_ptr();
  d.ldx = xq.stride(0);
  d.sx = sx.data_ptr<float>();
  d.ldsx = sx.size(1);
  d.W = wq.data_ptr();
  d.ldw = d.K;
  d.sw = sw.data_ptr<float>();
  d.C = C.data_ptr();
  d.ldc = C.stride(0);
  if (offsets.has_value()) {
    TORCH_CHECK(wq.dim() == 3 && offsets->scalar_type() == at::kInt && offsets->numel() == wq.size(0) + 1,
                "fp8_gemm: grouped needs wq [G, N, K] and int32 offsets [G+1]");
    d.G = (int)wq.size(0);
    d.offsets = offsets->data_ptr<int>();
    d.w_group_stride = (long long)d.N * d.K;
    d.max_rows_hint = (int)max_rows;
    TORCH_CHECK(sw.numel() == (long long)d.G * ((d.N + 127) / 128) * (d.K / 128), "fp8_gemm: sw shape");
  } else if (sw_rows) {
    TORCH_CHECK(sw.dim() == 2 && sw.size(0) == d.K / 128 && sw.size(1) >= (d.N + 255) / 256 * 256,
                "fp8_gemm: per-row sw [K/128, >= N rounded up to 256]");
    d.ldsw = sw.size(1);
  } else {
    TORCH_CHECK(sw.numel() == (long long)((d.N + 127) / 128) * (d.K / 128), "fp8_gemm: sw shape");
  }
  d.status = status_ptr();
  d.scaled_mma = scaled_mma;
  fp8_gemm_launch(d, cur_stream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Block-scaled fp8 gate|up GEMM with the SwiGLU + requantisation epilogue: H [rows, N] bf16
// pre-activation, act [rows, N/2] bf16 (optional), actq [rows, N/2] e4m3 and act_scale fp32
// [N/256, rows padded to 128] for the down GEMM.  Grouped when offsets is given.
void fp8_gemm_swiglu_q_t(const at::Tensor& xq, const at::Tensor& sx, const at::Tensor& wq, const at::Tensor& sw,
                         const c10::optional<at::Tensor>& H, const c10::optional<at::Tensor>& act, at::Tensor& actq,
                         at::Tensor& act_scale, const c10::optional<at::Tensor>& offsets, int64_t max_rows) {
  CHECK_CUDA_T(xq);
  TORCH_CHECK(xq.scalar_type() == at::kFloat8_e4m3fn && wq.scalar_type() == at::kFloat8_e4m3fn &&
                  actq.scalar_type() == at::kFloat8_e4m3fn, "fp8_gemm_swiglu_q: e4m3 operands / output");
  TORCH_CHECK(sx.scalar_type() == at::kFloat && sw.scalar_type() == at::kFloat && act_scale.scalar_type() == at::kFloat &&
                  sx.is_contiguous() && sw.is_contiguous() && act_scale.is_contiguous(), "fp8_gemm_swiglu_q: fp32 scales");
  CHECK_ROWMAJOR(xq);
  CHECK_ROWMAJOR(actq);
  TORCH_CHECK(wq.is_contiguous(), "fp8_gemm_swiglu_q: contiguous weights");
  const c10::cuda::CUDAGuard guard(xq.device());
  Fp8GemmDesc d;
  d.M = (int)xq.size(0);
  d.K = (int)xq.size(1);
  d.N = (int)wq.size(-2);
  TORCH_CHECK(wq.size(-1) == d.K && d.K % 128 == 0 && d.N % 256 == 0, "fp8_gemm_swiglu_q: K % 128, N % 256");
  TORCH_CHECK(sx.dim() == 2 && sx.size(0) == d.K / 128 && sx.size(1) >= (d.M + 127) / 128 * 128, "fp8_gemm_swiglu_q: sx");
  TORCH_CHECK(actq.size(0) == d.M && actq.size(1) == d.N / 2 && actq.stride(0) % 16 == 0, "fp8_gemm_swiglu_q: actq");
  TORCH_CHECK(act_scale.dim() == 2 && act_scale.size(0) == d.N / 256 && act_scale.size(1) >= (d.M + 127) / 128 * 128,
              "fp8_gemm_swiglu_q: act_scale [N/256, rows padded to 128]");
  d.X = xq.data_ptr();
  d.ldx = xq.stride(0);
  d.sx = sx.data_ptr<float>();
  d.ldsx = sx.size(1);
  d.W = wq.data_ptr();
  d.ldw = d.K;
  d.sw = sw.data_ptr<float>();
  if (H.has_value()) {
    CHECK_BF16(*H);
    CHECK_ROWMAJOR(*H);
    TORCH_CHECK(H->size(0) == d.M && H->size(1) == d.N && H->stride(0) % 8 == 0, "fp8_gemm_swiglu_q: H");
    d.C = H->data_ptr();
    d.ldc = H->stride(0);
  }
  if (act.has_value()) {
    CHECK_BF16(*act);
    CHECK_ROWMAJOR(*act);
    TORCH_CHECK(act->size(0) == d.M && act->size(1) == d.N / 2 && act->stride(0) % 8 == 0, "fp8_gemm_swiglu_q: act");
    d.act = act->data_ptr();
    d.ld_act = act->stride(0);
  }
  d.actq = actq.data_ptr();
  d.ld_actq = actq.stride(0);
  d.act_scale = act_scale.data_ptr<float>();
  d.ld_as = act_scale.size(1);
  if (offsets.has_value()) {
    TORCH_CHECK(wq.dim() == 3 && offsets->scalar_type() == at::kInt && offsets->numel() == wq.size(0) + 1,
                "fp8_gemm_swiglu_q: grouped needs wq [G, N, K] and int32 offsets [G+1]");
    d.G = (int)wq.size(0);
    d.offsets = offsets->data_ptr<int>();
    d.w_group_stride = (long long)d.N * d.K;
    d.max_rows_hint = (int)max_rows;
  }
  d.status = status_ptr();
  d.scaled_mma = true;
  fp8_gemm_launch(d, cur_stream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ---------------------------------------------------------------------------
// Tensor-parallel fused collectives over peer memory
// ---------------------------------------------------------------------------
// C [nsrc * src_rows, N] = gather_r(A_r) . B^T: rank r's row block A_r ([src_rows, K] bf16, row stride of
// a_local) is read straight from its buffer (peer_a[r], mapped in this process) by the GEMM's loads.
void gemm_ag(const at::Tensor& a_local, const std::vector<int64_t>& peer_a, int64_t me, const at::Tensor& B,
             at::Tensor& C, bool b_mn, int64_t epilogue, double alpha, const c10::optional<at::Tensor>& H,
             int64_t block_n) {
  CHECK_BF16(a_local);
  CHECK_BF16(B);
  CHECK_BF16(C);
  CHECK_ROWMAJOR(a_local);
  CHECK_ROWMAJOR(B);
  CHECK_ROWMAJOR(C);
  const int64_t nsrc = (int64_t)peer_a.size(), src_rows = a_local.size(0), K = a_local.size(1);
  TORCH_CHECK(nsrc >= 1 && nsrc <= GEMM_MAX_PEERS && me >= 0 && me < nsrc, "gemm_ag: ranks");
  const int64_t N = b_mn ? B.size(1) : B.size(0);
  TORCH_CHECK((b_mn ? B.size(0) : B.size(1)) == K, "gemm_ag: reduction dims differ");
  TORCH_CHECK(C.size(0) == nsrc * src_rows && C.size(1) == (epilogue == EPI_SWIGLU ? N / 2 : N), "gemm_ag: C shape");
  const c10::cuda::CUDAGuard guard(a_local.device());
  GemmDesc d;
  d.mode = GEMM_AG;
  d.epilogue = (int)epilogue;
  d.block_n = (int)block_n;
  d.b_mn_major = b_mn;
  d.M = (int)(nsrc * src_rows);
  d.N = (int)N;
  d.K = (int)K;
  d.lda = a_local.stride(0);
  d.K_extent_a = K;
  d.rows_a = src_rows;
  d.B = B.data_ptr();
  d.ldb = B.stride(0);
  d.K_extent_b = K;
  d.C = C.data_ptr();
  d.ldc = C.stride(0);
  d.alpha = (float)alpha;
  d.nsrc = (int)nsrc;
  d.me = (int)me;
  d.src_rows = (int)src_rows;
  for (int r = 0; r < nsrc; ++r) d.peer_a[r] = reinterpret_cast<const void*>(peer_a[r]);
  if (epilogue == EPI_SWIGLU && H.has_value()) {
    CHECK_BF16(H.value());
    TORCH_CHECK(H->size(0) == d.M && H->size(1) == N, "gemm_ag swiglu: H shape");
    d.H = H->data_ptr();
    d.ldh = H->stride(0);
  }
  d.status = status_ptr();
  gemm_sm100_launch(d, cur_stream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Partial products A . B^T (A [nsrc * src_rows, K]) stored tile by tile into the row owners' staging
// buffers: rows of rank r go to peer_c[r] + (me * src_rows + local row) * ldc (bf16).
void gemm_rs(const at::Tensor& A, const at::Tensor& B, const std::vector<int64_t>& peer_c, int64_t src_rows,
             int64_t ldc, int64_t me, bool b_mn, int64_t block_n) {
  CHECK_BF16(A);
  CHECK_BF16(B);
  CHECK_ROWMAJOR(A);
  CHECK_ROWMAJOR(B);
  const int64_t nsrc = (int64_t)peer_c.size(), M = A.size(0), K = A.size(1);
  const int64_t N = b_mn ? B.size(1) : B.size(0);
  TORCH_CHECK(nsrc >= 1 && nsrc <= GEMM_MAX_PEERS && M == nsrc * src_rows && me >= 0 && me < nsrc, "gemm_rs: rows");
  TORCH_CHECK((b_mn ? B.size(0) : B.size(1)) == K && ldc >= N && ldc % 8 == 0, "gemm_rs: dims");
  const c10::cuda::CUDAGuard guard(A.device());
  GemmDesc d;
  d.mode = GEMM_DENSE;
  d.epilogue = EPI_PEER_BF16;
  d.block_n = (int)block_n;
  d.b_mn_major = b_mn;
  d.M = (int)M;
  d.N = (int)N;
  d.K = (int)K;
  d.A = A.data_ptr();
  d.lda = A.stride(0);
  d.rows_a = M;
  d.K_extent_a = K;
  d.B = B.data_ptr();
  d.ldb = B.stride(0);
  d.K_extent_b = K;
  d.ldc = ldc;
  d.nsrc = (int)nsrc;
  d.me = (int)me;
  d.src_rows = (int)src_rows;
  for (int r = 0; r < nsrc; ++r) d.peer_c[r] = reinterpret_cast<void*>(peer_c[r]);
  d.status = status_ptr();
  gemm_sm100_launch(d, cur_stream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// dst (contiguous bytes) <- nbytes at device address src (a peer's buffer mapped in this process), on the
// current stream (copy engine over NVLink).
void peer_copy(at::Tensor& dst, int64_t src, int64_t nbytes) {
  TORCH_CHECK(dst.is_cuda() && dst.is_contiguous() && dst.numel() * dst.element_size() >= nbytes, "peer_copy: dst");
  const c10::cuda::CUDAGuard guard(dst.device());
  C10_CUDA_CHECK(cudaMemcpyAsync(dst.data_ptr(), reinterpret_cast<const void*>(src), (size_t)nbytes,
                                 cudaMemcpyDeviceToDevice, cur_stream()));
}

void tp_reduce(const at::Tensor& staging, at::Tensor& out, const c10::optional<at::Tensor>& residual) {
  CHECK_BF16(staging);
  CHECK_BF16(out);
  TORCH_CHECK(staging.dim() == 3 && staging.stride(-1) == 1, "tp_reduce: staging [nsrc, rows, D]");
  const int64_t nsrc = staging.size(0), rows = staging.size(1), D = staging.size(2);
  TORCH_CHECK(staging.stride(0) == rows * staging.stride(1), "tp_reduce: slots must be packed");
  TORCH_CHECK(out.size(0) == rows && out.size(1) == D && out.stride(-1) == 1, "tp_reduce: out [rows, D]");
  if (residual.has_value()) {
    CHECK_BF16(residual.value());
    TORCH_CHECK(residual->size(0) == rows && residual->size(1) == D && residual->stride(-1) == 1, "tp_reduce: residual");
  }
  const c10::cuda::CUDAGuard guard(staging.device());
  tp_reduce_slots(staging.data_ptr(), (int)nsrc, (int)rows, (int)D, staging.stride(1),
                  residual.has_value() ? residual->data_ptr() : nullptr, residual.has_value() ? residual->stride(0) : 0,
                  out.data_ptr(), out.stride(0), cur_stream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Grouped-K: C[g] (M x N) = alpha * A[rows_g]^T B[rows_g] with A [rows, M], B [rows, N].
void gemm_grouped_k(const at::Tensor& A, const at::Tensor& B, const at::Tensor& offsets, at::Tensor& C,
                    int64_t epilogue, double alpha, int64_t block_n) {
  CHECK_BF16(A);
  CHECK_BF16(B);
  CHECK_ROWMAJOR(A);
  CHECK_ROWMAJOR(B);
  TORCH_CHECK(C.dim() == 3 && C.is_contiguous(), "gemm_grouped_k: C must be a contiguous [G, M, N] stack");
  TORCH_CHECK(offsets.scalar_type() == at::kInt && offsets.numel() == C.size(0) + 1, "gemm_grouped_k: offsets");
  const c10::cuda::CUDAGuard guard(A.device());
  GemmDesc d;
  d.mode = GEMM_GROUPED_K;
  d.epilogue = (int)epilogue;
  d.block_n = (int)block_n;
  d.a_mn_major = true;
  d.b_mn_major = true;
  d.M = (int)A.size(1);
  d.N = (int)B.size(1);
  d.K = 0;
  TORCH_CHECK(C.size(1) == d.M && C.size(2) == d.N, "gemm_grouped_k: output shape");
  d.A = A.data_ptr();
  d.lda = A.stride(0);
  d.rows_a = A.size(0);
  d.K_extent_a = A.size(0);
  d.B = B.data_ptr();
  d.ldb = B.stride(0);
  d.K_extent_b = B.size(0);
  d.num_groups = (int)C.size(0);
  d.group_offsets = offsets.data_ptr<int>();
  d.C = C.data_ptr();
  d.ldc = C.stride(1);
  d.c_group_stride = C.stride(0);
  d.alpha = (float)alpha;
  if (epilogue == EPI_STORE_F32 || epilogue == EPI_ACCUM_F32) {
    TORCH_CHECK(C.scalar_type() == at::kFloat, "gemm_grouped_k: fp32 output expected");
  } else {
    CHECK_BF16(C);
  }
  d.status = status_ptr();
  gemm_sm100_launch(d, cur_stream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace omni

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "omnicoder sm_100a kernels (tcgen05/TMEM/TMA)";
  m.def("status", &omni::status_read, "Read the device status block: [code, info, count]");
  m.def("status_reset", &omni::status_reset);
  m.def("gemm", &omni::gemm, "tcgen05 GEMM", py::arg("A"), py::arg("B"), py::arg("C"), py::arg("a_mn"),
        py::arg("b_mn"), py::arg("epilogue"), py::arg("alpha") = 1.0, py::arg("R") = py::none(),
        py::arg("H") = py::none(), py::arg("block_n") = 256);
  m.def("gemm_ag", &omni::gemm_ag, py::arg("a_local"), py::arg("peer_a"), py::arg("me"), py::arg("B"), py::arg("C"),
        py::arg("b_mn"), py::arg("epilogue"), py::arg("alpha") = 1.0, py::arg("H") = py::none(),
        py::arg("block_n") = 256);
  m.def("gemm_rs", &omni::gemm_rs, py::arg("A"), py::arg("B"), py::arg("peer_c"), py::arg("src_rows"), py::arg("ldc"),
        py::arg("me"), py::arg("b_mn"), py::arg("block_n") = 256);
  m.def("peer_copy", &omni::peer_copy, py::arg("dst"), py::arg("src"), py::arg("nbytes"));
  m.def("tp_reduce", &omni::tp_reduce, py::arg("staging"), py::arg("out"), py::arg("residual") = py::none());
  m.def("fp8_quant_act", &omni::fp8_quant_act_t, "bf16 [M, K] -> (e4m3 [M, K], fp32 scales [K/128, M padded to 128])",
        py::arg("x"), py::arg("pow2") = true, py::arg("offsets") = py::none());
  m.def("fp8_quant_weight", &omni::fp8_quant_weight_t, "bf16 [(G,) N, K] -> (e4m3, fp32 scales [G, N/128, K/128])",
        py::arg("w"), py::arg("pow2") = true);
  m.def("fp8_gemm", &omni::fp8_gemm_t, py::arg("xq"), py::arg("sx"), py::arg("wq"), py::arg("sw"), py::arg("C"),
        py::arg("offsets") = py::none(), py::arg("max_rows") = 0, py::arg("scaled_mma") = true,
        py::arg("sw_rows") = false);
  m.def("fp8_quant_t", &omni::fp8_quant_t_t, "bf16 [T, C] -> (e4m3 [C, T], fp32 scales [T/128, C padded to 256])");
  m.def("gemm_grouped_m_push", &omni::gemm_grouped_m_push, py::arg("A"), py::arg("B"), py::arg("offsets"),
        py::arg("meta"), py::arg("peer_ptrs"), py::arg("dest_rows"), py::arg("b_mn"), py::arg("max_rows") = 0);
  m.def("fp8_gemm_swiglu_q", &omni::fp8_gemm_swiglu_q_t, py::arg("xq"), py::arg("sx"), py::arg("wq"), py::arg("sw"),
        py::arg("H"), py::arg("act"), py::arg("actq"), py::arg("act_scale"), py::arg("offsets") = py::none(),
        py::arg("max_rows") = 0);
  m.def("gemm_skinny_grouped", &omni::gemm_skinny_grouped, py::arg("A"), py::arg("B"), py::arg("offsets"),
        py::arg("C"), py::arg("epilogue"), py::arg("alpha") = 1.0, py::arg("rows") = 0);
  m.def("set_skinny_rows", &omni::set_skinny_rows, "rows up to which dense GEMMs use the few-row kernel (0: off)");
  m.def("set_gemm_pair", &omni::set_gemm_pair, "use CTA-pair (cta_group::2) 256-row tiles for large dense / grouped-K GEMMs");
  m.def("gemm_pair_enabled", &omni::gemm_pair_enabled);
  m.def("gemm_grouped_m", &omni::gemm_grouped_m, py::arg("A"), py::arg("B"), py::arg("offsets"), py::arg("C"),
        py::arg("b_mn"), py::arg("epilogue"), py::arg("alpha") = 1.0, py::arg("R") = py::none(),
        py::arg("H") = py::none(), py::arg("block_n") = 256, py::arg("max_rows_hint") = 0,
        py::arg("ready_ptr") = 0, py::arg("ready_epoch") = py::none(), py::arg("src_pref") = py::none(),
        py::arg("nsrc") = 0, py::arg("me") = 0);
  m.def("gemm_grouped_k", &omni::gemm_grouped_k, py::arg("A"), py::arg("B"), py::arg("offsets"), py::arg("C"),
        py::arg("epilogue"), py::arg("alpha") = 1.0, py::arg("block_n") = 256);
  omni::register_kernels(m);
  omni::register_ep(m);
}
