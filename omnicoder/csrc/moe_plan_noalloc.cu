// Allocation-free variant of the MoE permutation plan (see moe_plan_noalloc.h
// for who needs it, its limits and its concurrency rules).  It launches the
// same three kernels as omni::moe_permute_plan (moe_route.cu) but takes their
// workspace from a file-scope device array instead of from an allocator.  No counterpart in the reference.
// Out-of-range expert ids are skipped without a status report (the kernels
// accept a null status block).
#include <cuda_runtime.h>

#include <mutex>

#include "common.cuh"
#include "moe_plan_noalloc.h"

namespace omni {
// Kernels defined in moe_route.cu (same launch geometry is used below).
__global__ void plan_count_kernel(const int* idx, int N, int E, int* blk_cnt, StatusBlock* st);
__global__ void plan_scan_kernel(int nblocks, int E, int capacity, const int* blk_cnt, int* blk_base, int* counts,
                                 int* offsets, int* src, int cap_rows, int align);
__global__ void plan_assign_kernel(const int* idx, int N, int E, int capacity, const int* blk_base,
                                   const int* offsets, int* pos, int* src, int cap_rows, StatusBlock* st);
}  // namespace omni

namespace {

constexpr int kPairsPerBlock = 1024;  // matches moe_route.cu
constexpr int kThreads = 256;         // matches moe_route.cu
constexpr int kMaxDevices = 64;

// The scratch: per-block expert counts followed by their exclusive prefix sums.
static __device__ __align__(256) int g_plan_scratch[OMNI_PLAN_NOALLOC_MAX_INTS];

std::mutex g_mu;
int* g_scratch_addr[kMaxDevices] = {nullptr};

// Device address of g_plan_scratch for the current device (looked up once).
int* scratch_for_current_device(int* err) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    *err = OMNI_NOALLOC_SETUP_FAILED;
    return nullptr;
  }
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_plan_scratch);
    if (e != cudaSuccess || p == nullptr) {
      *err = OMNI_NOALLOC_SETUP_FAILED;
      return nullptr;
    }
    g_scratch_addr[dev] = static_cast<int*>(p);
  }
  return g_scratch_addr[dev];
}

// Scratch integers the plan needs: a count and a base per (block, expert).
long long scratch_ints(int T, int K, int E) {
  const long long n = (long long)T * K;
  const long long nblocks = (n + kPairsPerBlock - 1) / kPairsPerBlock;
  return 2 * nblocks * (long long)E;
}

}  // namespace

extern "C" int omni_moe_permute_plan_noalloc(const int* idx, int T, int K, int E, int capacity, int* counts,
                                             int* offsets, int* pos, int* src, int cap_rows, void* stream) {
  if (T < 0 || K <= 0 || K > 16 || E <= 0 || E > 256 || cap_rows < 0 || counts == nullptr || offsets == nullptr ||
      (T > 0 && (idx == nullptr || pos == nullptr)) || (cap_rows > 0 && src == nullptr))
    return OMNI_NOALLOC_BAD_ARGUMENT;
  if ((long long)T * K > (1ll << 30)) return OMNI_NOALLOC_TOO_LARGE;
  const long long need = scratch_ints(T, K, E);
  if (need > OMNI_PLAN_NOALLOC_MAX_INTS) return OMNI_NOALLOC_TOO_LARGE;
  // an error left by unrelated earlier work is not ours to consume: report it and launch nothing
  if (cudaPeekAtLastError() != cudaSuccess) return OMNI_NOALLOC_PENDING_ERROR;
  int err = OMNI_NOALLOC_OK;
  int* base = scratch_for_current_device(&err);
  if (base == nullptr) return err;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int* blk_cnt = base;
  const int N = T * K;
  const int nblocks = (N + kPairsPerBlock - 1) / kPairsPerBlock;
  int* blk_base = blk_cnt + nblocks * E;
  if (nblocks == 0) {
    if (cudaMemsetAsync(counts, 0, E * sizeof(int), s) != cudaSuccess) return OMNI_NOALLOC_LAUNCH_FAILED;
    if (cudaMemsetAsync(offsets, 0, (E + 1) * sizeof(int), s) != cudaSuccess) return OMNI_NOALLOC_LAUNCH_FAILED;
    return OMNI_NOALLOC_OK;
  }
  // no error was pending above, so an error read after a launch belongs to that launch
  omni::plan_count_kernel<<<nblocks, kThreads, 0, s>>>(idx, N, E, blk_cnt, nullptr);
  if (cudaGetLastError() != cudaSuccess) return OMNI_NOALLOC_LAUNCH_FAILED;
  omni::plan_scan_kernel<<<1, 256, 0, s>>>(nblocks, E, capacity, blk_cnt, blk_base, counts, offsets, src, cap_rows,
                                           128);
  if (cudaGetLastError() != cudaSuccess) return OMNI_NOALLOC_LAUNCH_FAILED;
  omni::plan_assign_kernel<<<nblocks, kThreads, 0, s>>>(idx, N, E, capacity, blk_base, offsets, pos, src, cap_rows,
                                                        nullptr);
  if (cudaGetLastError() != cudaSuccess) return OMNI_NOALLOC_LAUNCH_FAILED;
  return OMNI_NOALLOC_OK;
}
