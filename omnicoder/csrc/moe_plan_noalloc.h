// Allocation-free C entry point for the MoE permutation plan.
//
// This entry point has no counterpart in the reference project; it exists for
// callers of this library that cannot allocate device memory on their own
// path: for example a plugin running inside another inference runtime that
// owns every byte of device memory and forbids cudaMalloc during execution,
// or a latency-critical serving loop where a cudaMalloc could implicitly
// synchronise the device.  The regular binding (omnicoder._C.moe_plan) asks
// PyTorch's allocator for its scratch workspace; this one uses a fixed,
// file-scope device array instead and allocates nothing.
//
// Limits and behaviour:
//   * Scratch is a static __device__ array of OMNI_PLAN_NOALLOC_MAX_INTS
//     32-bit integers (256 KiB).  Every GPU that loads this library holds it
//     until the process exits.  The plan needs 2 * ceil(T*K/1024) * E
//     integers; larger problems are rejected with OMNI_NOALLOC_TOO_LARGE.
//   * The first call on a device looks up the array's device address with
//     cudaGetSymbolAddress (with that device current) and caches it; make
//     that first call before any stream capture.
//   * All calls share the one array, which keeps the contents of the last
//     call.  The plan kernels overwrite every scratch entry before reading it,
//     so nothing in the array needs clearing between calls.  Calls whose
//     executions overlap on the GPU (different streams, or different host
//     threads) race on the shared array and produce wrong plans: serialise
//     them.
//   * Expert ids outside [0, E) are skipped (their pos is -1); unlike the
//     regular binding this variant does not record them in a status block.
//   * The caller passes every input and output buffer (device pointers):
//       idx     [T*K] int32 expert ids (row-major [T, K])
//       counts  [E]   int32 routed pairs per expert (before capacity)
//       offsets [E+1] int32 start row of each expert segment (multiples of 128)
//       pos     [T*K] int32 permuted row of each pair, -1 if dropped
//       src     [cap_rows] int32 pair index of each permuted row, -1 for padding
//     Outputs are identical to omnicoder._C.moe_plan for the same inputs.
#pragma once

#ifdef __cplusplus
extern "C" {
#endif

#define OMNI_PLAN_NOALLOC_MAX_INTS 65536

enum {
  OMNI_NOALLOC_OK = 0,
  OMNI_NOALLOC_TOO_LARGE = 1,    // problem needs more scratch than the static array holds
  OMNI_NOALLOC_BAD_ARGUMENT = 2, // null pointer or size outside the supported range
  OMNI_NOALLOC_SETUP_FAILED = 3, // cudaGetSymbolAddress failed on this device
  OMNI_NOALLOC_LAUNCH_FAILED = 4, // a kernel launch of this call reported an error
  OMNI_NOALLOC_PENDING_ERROR = 5  // an earlier CUDA error was pending on this thread; nothing was
                                  // launched and the error is left for its owner to read
};

// Enqueue the permutation plan on `stream` (a cudaStream_t, may be null for the
// legacy default stream).  Returns one of the OMNI_NOALLOC_* codes; on success
// the outputs are ready when the stream reaches this point.
int omni_moe_permute_plan_noalloc(const int* idx, int T, int K, int E, int capacity, int* counts, int* offsets,
                                  int* pos, int* src, int cap_rows, void* stream);

#ifdef __cplusplus
}
#endif
