// Host interface of the tcgen05 GEMM (see gemm_sm100.cu).
#pragma once
#include <cuda_runtime.h>

namespace omni {

enum GemmMode : int { GEMM_DENSE = 0, GEMM_GROUPED_M = 1, GEMM_GROUPED_K = 2 };

enum GemmEpi : int {
  EPI_STORE_BF16 = 0,  // C(bf16) = alpha * acc
  EPI_STORE_F32 = 1,   // C(f32)  = alpha * acc
  EPI_ACCUM_F32 = 2,   // C(f32) += alpha * acc
  EPI_ADD_BF16 = 3,    // C(bf16) = alpha * acc + R(bf16)   (R may alias C)
  EPI_SWIGLU = 4,      // acc = [gate|up] interleaved by 32; C = silu(gate)*up (bf16, N/2 cols); H = acc (bf16)
  EPI_SWIGLU_BWD = 5,  // acc = dAct; R = saved H; C = dH (bf16, 2N cols, interleaved by 32)
};

constexpr int GEMM_MAX_GROUPS = 256;

struct GemmDesc {
  int mode = GEMM_DENSE;
  int epilogue = EPI_STORE_BF16;
  int block_n = 256;  // 128 or 256
  bool a_mn_major = false;
  bool b_mn_major = false;
  int M = 0, N = 0, K = 0;
  // A: K-major -> stored [rows_a, K_extent_a]; MN-major -> stored [K_extent_a, M]
  const void* A = nullptr;
  long long lda = 0;
  long long rows_a = 0;
  long long K_extent_a = 0;
  // B: K-major -> stored [N, K_extent_b] (or [G, N, K]); MN-major -> stored [K_extent_b, N] (or [G, K, N])
  const void* B = nullptr;
  long long ldb = 0;
  long long b_group_stride = 0;
  long long K_extent_b = 0;
  int num_groups = 1;
  const int* group_offsets = nullptr;  // device [G+1], multiples of 128
  int max_rows_hint = 0;               // grouped-M: upper bound on total rows (0 = unknown)
  void* C = nullptr;
  long long ldc = 0;
  long long c_group_stride = 0;
  const void* R = nullptr;
  long long ldr = 0;
  void* H = nullptr;
  long long ldh = 0;
  float alpha = 1.0f;
  void* status = nullptr;  // omni::StatusBlock*
};

// Launch on `stream`.  Throws std::runtime_error on an invalid description.
void gemm_sm100_launch(const GemmDesc& d, cudaStream_t stream);

}  // namespace omni
