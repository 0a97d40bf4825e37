// Speculative-decoding verify step (sm_100a): per-sequence acceptance of k draft
// tokens against the target's logits of the k + 1 verified positions, the next
// token, and the KV-cache lengths after rollback -- one CTA per sequence, no
// host round trip.
//
//   greedy (temperature <= 0): draft token j is accepted while it equals the
//     target's argmax at position j (first index among equal maxima); the next
//     token is the target's argmax at the first rejected position (or at k).
//   sampling (temperature > 0): p_t = softmax(logits / T) per position, p_d the
//     draft's distribution; token j is accepted while u_j < min(1, p_t(d_j) /
//     p_d(d_j)); at the first rejection j the next token is drawn from
//     normalize(max(0, p_t(j) - p_d(j))), after k acceptances from p_t(k).
//     The draw is an inverse-CDF lookup with the caller's uniform u_k, so a
//     given set of uniforms gives one answer (the torch restatement in
//     omnicoder/ops/spec.py computes the same).
//   new_len[b] = base_len[b] + n_acc[b] + 1: the tokens kept in the cache (the
//     verified input token and the accepted drafts).
//
// The reference accepts drafts by a verifier-probability threshold and feeds
// accepted tokens back one at a time (src/omnicoder/inference/generate.py:
// 2925-3048); exact rejection sampling keeps the target's output distribution.
#include <cuda_runtime.h>

#include <cfloat>
#include <cstdint>

#include "common.cuh"
#include "kernels.h"

namespace omni {

namespace {

constexpr int kThreads = 1024;
constexpr int kWarps = kThreads / 32;

struct ArgMax {
  float v;
  int i;
};

__device__ __forceinline__ ArgMax better(ArgMax a, ArgMax b) {
  // larger value wins; equal values: the lower index (torch.argmax returns the first maximum)
  if (b.v > a.v || (b.v == a.v && b.i < a.i)) return b;
  return a;
}

__device__ ArgMax block_argmax(const float* __restrict__ x, int V, ArgMax* sh) {
  ArgMax m{-FLT_MAX, 0x7fffffff};
  for (int v = threadIdx.x; v < V; v += kThreads) m = better(m, ArgMax{x[v], v});
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    ArgMax t{__shfl_xor_sync(0xffffffffu, m.v, o), __shfl_xor_sync(0xffffffffu, m.i, o)};
    m = better(m, t);
  }
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) sh[w] = m;
  __syncthreads();
  if (w == 0) {
    m = lane < kWarps ? sh[lane] : ArgMax{-FLT_MAX, 0x7fffffff};
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      ArgMax t{__shfl_xor_sync(0xffffffffu, m.v, o), __shfl_xor_sync(0xffffffffu, m.i, o)};
      m = better(m, t);
    }
    if (lane == 0) sh[0] = m;
  }
  __syncthreads();
  const ArgMax r = sh[0];
  __syncthreads();
  return r;
}

__device__ float block_sum(float v, float* sh) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) sh[w] = v;
  __syncthreads();
  if (w == 0) {
    v = lane < kWarps ? sh[lane] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) sh[0] = v;
  }
  __syncthreads();
  const float r = sh[0];
  __syncthreads();
  return r;
}

// Inverse-CDF draw from the unnormalised weights w(v) >= 0 that `weight(v)` returns:
// the smallest v whose inclusive prefix sum exceeds u * total.  Each thread owns one
// contiguous range of the vocabulary; the ranges' sums are scanned across the block.
template <typename W>
__device__ int block_sample(int V, float u, W weight, float* shf, int* shi) {
  const int per = (V + kThreads - 1) / kThreads;
  const int v0 = threadIdx.x * per, v1 = min(V, v0 + per);
  float local = 0.f;
  for (int v = v0; v < v1; ++v) local += weight(v);
  // exclusive scan of `local` over the block
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float incl = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  __syncthreads();
  if (lane == 31) shf[w] = incl;
  __syncthreads();
  if (w == 0) {
    float s = lane < kWarps ? shf[lane] : 0.f;
    float si = s;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float t = __shfl_up_sync(0xffffffffu, si, o);
      if (lane >= o) si += t;
    }
    if (lane < kWarps) shf[32 + lane] = si - s;   // exclusive prefix of warp sums
    if (lane == kWarps - 1) shf[64] = si;         // total
  }
  if (threadIdx.x == 0) *shi = -1;
  __syncthreads();
  const float total = shf[64];
  const float target = u * total;
  const float start = shf[32 + w] + (incl - local);
  if (total > 0.f && local > 0.f && target >= start && target < start + local) {
    float c = start;
    int pick = v1 - 1;
    for (int v = v0; v < v1; ++v) {
      c += weight(v);
      if (c > target) {
        pick = v;
        break;
      }
    }
    atomicMax(shi, pick);  // one thread matches; max() keeps the result defined at rounding ties
  }
  __syncthreads();
  int r = *shi;
  if (r < 0) {
    // u * total fell beyond the last positive weight by rounding (or total == 0): take the last
    // positive-weight index
    if (threadIdx.x == 0) *shi = -1;
    __syncthreads();
    for (int v = v1 - 1; v >= v0; --v)
      if (weight(v) > 0.f) {
        atomicMax(shi, v);
        break;
      }
    __syncthreads();
    r = max(*shi, 0);
  }
  __syncthreads();
  return r;
}

template <typename TokT, typename LenT>
__global__ void __launch_bounds__(kThreads) spec_verify_kernel(const float* __restrict__ logits,
                                                               const float* __restrict__ pdraft,
                                                               const TokT* __restrict__ draft, const float* __restrict__ u,
                                                               const LenT* __restrict__ base_len, int K, int V,
                                                               float inv_t, int* __restrict__ n_acc_out,
                                                               TokT* __restrict__ next_out, LenT* __restrict__ new_len) {
  __shared__ ArgMax sh_am[kWarps];
  __shared__ float shf[80];
  __shared__ int shi;
  const int b = blockIdx.x;
  const float* lg = logits + (long long)b * (K + 1) * V;
  int n_acc = K, next = 0;
  if (inv_t <= 0.f) {
    for (int j = 0; j <= K; ++j) {
      const ArgMax m = block_argmax(lg + (long long)j * V, V, sh_am);
      if (j == K || m.i != (int)draft[(long long)b * K + j]) {
        n_acc = j;
        next = m.i;
        break;
      }
    }
  } else {
    const float* pd = pdraft + (long long)b * K * V;
    int j = 0;
    float mx = 0.f, z = 1.f;
    for (; j <= K; ++j) {
      const float* x = lg + (long long)j * V;
      mx = block_argmax(x, V, sh_am).v;
      float part = 0.f;
      for (int v = threadIdx.x; v < V; v += kThreads) part += __expf((x[v] - mx) * inv_t);
      z = block_sum(part, shf);
      if (j == K) break;
      const int d = (int)draft[(long long)b * K + j];
      const float pt = __expf((x[d] - mx) * inv_t) / z;
      const float pdd = fmaxf(pd[(long long)j * V + d], 1e-20f);
      if (!(u[(long long)b * (K + 1) + j] < fminf(1.f, pt / pdd))) break;
    }
    n_acc = j;
    const float* x = lg + (long long)j * V;
    const float uk = u[(long long)b * (K + 1) + K];
    const float m = mx, zz = z;
    if (j < K) {
      const float* q = pd + (long long)j * V;
      next = block_sample(V, uk, [&](int v) { return fmaxf(0.f, __expf((x[v] - m) * inv_t) / zz - q[v]); }, shf,
                          &shi);
    } else {
      next = block_sample(V, uk, [&](int v) { return __expf((x[v] - m) * inv_t) / zz; }, shf, &shi);
    }
  }
  if (threadIdx.x == 0) {
    n_acc_out[b] = n_acc;
    next_out[b] = (TokT)next;
    new_len[b] = base_len[b] + (LenT)(n_acc + 1);
  }
}

}  // namespace

void spec_verify(const float* logits, const float* pdraft, const void* draft, bool draft_i64, const float* u,
                 const void* base_len, bool len_i64, int B, int K, int V, float temperature, int* n_acc, void* next,
                 void* new_len, cudaStream_t s) {
  if (B == 0) return;
  const float inv_t = temperature > 0.f ? 1.f / temperature : 0.f;
  if (draft_i64 && len_i64)
    spec_verify_kernel<long long, long long><<<B, kThreads, 0, s>>>(
        logits, pdraft, (const long long*)draft, u, (const long long*)base_len, K, V, inv_t, n_acc, (long long*)next,
        (long long*)new_len);
  else if (draft_i64)
    spec_verify_kernel<long long, int><<<B, kThreads, 0, s>>>(logits, pdraft, (const long long*)draft, u,
                                                              (const int*)base_len, K, V, inv_t, n_acc,
                                                              (long long*)next, (int*)new_len);
  else if (len_i64)
    spec_verify_kernel<int, long long><<<B, kThreads, 0, s>>>(logits, pdraft, (const int*)draft, u,
                                                              (const long long*)base_len, K, V, inv_t, n_acc,
                                                              (int*)next, (long long*)new_len);
  else
    spec_verify_kernel<int, int><<<B, kThreads, 0, s>>>(logits, pdraft, (const int*)draft, u, (const int*)base_len, K,
                                                        V, inv_t, n_acc, (int*)next, (int*)new_len);
}

}  // namespace omni
