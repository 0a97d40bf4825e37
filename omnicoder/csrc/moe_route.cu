// MoE routing kernels (sm_100a): softmax top-k router, deterministic
// expert-major permutation with segments padded to 128 rows (the layout the
// grouped tile GEMM consumes; align = 1 packs them for the few-row GEMM of a
// decode step), gather, weighted combine and their backward passes.
//
// Behaviour of the reference being replaced: moe_scatter.fused_dispatch
// (src/omnicoder/modeling/kernels/moe_scatter.py:315-912) stable-sorts the N*K
// expert ids to get each pair's rank inside its expert (:480), keeps
// rank < capacity (:553), packs rows per expert (:726), runs the expert GEMMs
// and sums the gated outputs back per token (:828).  Here the rank comes from
// a per-block count + scan + in-order warp match, which gives the same
// token-order ranks as a stable sort without sorting, and routers/experts
// receive gradients (the reference detaches them, moe_scatter.py:344-345).
#include "common.cuh"
#include "kernels.h"

namespace omni {

using bf16 = __nv_bfloat16;

constexpr int kRouteMaxE = 256;
constexpr int kRouteMaxK = 16;
constexpr int kPlanPairsPerBlock = 1024;
constexpr int kPlanThreads = 256;

// ---------------------------------------------------------------------------
// Router: softmax over E logits, top-k, optional renormalisation (one warp per token)
// ---------------------------------------------------------------------------
// p[j] = logit of expert lane + 32 j on entry (-inf where e >= E); softmax over the E logits,
// then the top K by repeated warp argmax (ties -> lowest expert id), optionally renormalised.
__device__ __forceinline__ void router_select(float (&p)[kRouteMaxE / 32], int t, int lane, int E, int K,
                                              bool renorm, int* __restrict__ idx, float* __restrict__ wts,
                                              float* __restrict__ probs) {
  const int per = (E + 31) / 32;
  float m = -INFINITY;
#pragma unroll
  for (int j = 0; j < kRouteMaxE / 32; ++j) m = fmaxf(m, p[j]);
  m = warp_max(m);
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < kRouteMaxE / 32; ++j) {
    p[j] = (p[j] == -INFINITY) ? 0.f : __expf(p[j] - m);
    s += p[j];
  }
  s = warp_sum(s);
  const float inv = 1.f / s;
#pragma unroll
  for (int j = 0; j < kRouteMaxE / 32; ++j) {
    p[j] *= inv;
    const int e = lane + 32 * j;
    if (probs != nullptr && j < per && e < E) probs[(long long)t * E + e] = p[j];
  }
  float sel_w[kRouteMaxK];
  int sel_e[kRouteMaxK];
  float wsum = 0.f;
  for (int k = 0; k < K; ++k) {
    float bv = -1.f;
    int be = 0x7fffffff;
#pragma unroll
    for (int j = 0; j < kRouteMaxE / 32; ++j) {
      const int e = lane + 32 * j;
      if (j < per && e < E && (p[j] > bv || (p[j] == bv && e < be))) {
        bv = p[j];
        be = e;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oe = __shfl_xor_sync(0xffffffffu, be, o);
      if (ov > bv || (ov == bv && oe < be)) {
        bv = ov;
        be = oe;
      }
    }
    sel_w[k] = bv;
    sel_e[k] = be;
    wsum += bv;
#pragma unroll
    for (int j = 0; j < kRouteMaxE / 32; ++j)
      if (lane + 32 * j == be) p[j] = -2.f;  // taken
  }
  if (lane == 0) {
    const float r = renorm ? 1.f / wsum : 1.f;
    for (int k = 0; k < K; ++k) {
      idx[(long long)t * K + k] = sel_e[k];
      wts[(long long)t * K + k] = sel_w[k] * r;
    }
  }
}

__global__ void router_topk_kernel(const float* __restrict__ logits, int* __restrict__ idx, float* __restrict__ wts,
                                   float* __restrict__ probs, int T, int E, int K, bool renorm) {
  const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (t >= T) return;
  float p[kRouteMaxE / 32];
  const int per = (E + 31) / 32;
#pragma unroll
  for (int j = 0; j < kRouteMaxE / 32; ++j) {
    const int e = lane + 32 * j;
    p[j] = (j < per && e < E) ? logits[(long long)t * E + e] : -INFINITY;
  }
  router_select(p, t, lane, E, K, renorm, idx, wts, probs);
}

void router_topk(const float* logits, int* idx, float* wts, float* probs, int T, int E, int K, bool renorm,
                 cudaStream_t s) {
  const int warps = 8;
  router_topk_kernel<<<(T + warps - 1) / warps, warps * 32, 0, s>>>(logits, idx, wts, probs, T, E, K, renorm);
}

// ---------------------------------------------------------------------------
// Permutation plan
// ---------------------------------------------------------------------------
__global__ void plan_count_kernel(const int* __restrict__ idx, int N, int E, int* __restrict__ blk_cnt,
                                  StatusBlock* st) {
  __shared__ int cnt[kRouteMaxE];
  for (int e = threadIdx.x; e < E; e += blockDim.x) cnt[e] = 0;
  __syncthreads();
  const int b = blockIdx.x;
  for (int i = b * kPlanPairsPerBlock + threadIdx.x; i < min(N, (b + 1) * kPlanPairsPerBlock); i += blockDim.x) {
    const int e = idx[i];
    if (e >= 0 && e < E)
      atomicAdd(&cnt[e], 1);
    else
      report_error(st, STATUS_BAD_INDEX, e);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) blk_cnt[b * E + e] = cnt[e];
}

__global__ void plan_scan_kernel(int nblocks, int E, int capacity, const int* __restrict__ blk_cnt,
                                 int* __restrict__ blk_base, int* __restrict__ counts, int* __restrict__ offsets,
                                 int* __restrict__ src, int cap_rows, int align) {
  __shared__ int kept[kRouteMaxE];
  __shared__ int off[kRouteMaxE + 1];
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int base = 0;
    for (int b = 0; b < nblocks; ++b) {
      blk_base[b * E + e] = base;
      base += blk_cnt[b * E + e];
    }
    counts[e] = base;
    kept[e] = capacity > 0 ? min(base, capacity) : base;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int o = 0;
    for (int e = 0; e < E; ++e) {
      off[e] = o;
      offsets[e] = o;
      o += (kept[e] + align - 1) / align * align;
    }
    off[E] = o;
    offsets[E] = o;
  }
  __syncthreads();
  // mark the padding rows of every segment
  for (int e = 0; e < E; ++e)
    for (int r = off[e] + kept[e] + threadIdx.x; r < min(off[e + 1], cap_rows); r += blockDim.x) src[r] = -1;
}

__global__ void plan_assign_kernel(const int* __restrict__ idx, int N, int E, int capacity,
                                   const int* __restrict__ blk_base, const int* __restrict__ offsets,
                                   int* __restrict__ pos, int* __restrict__ src, int cap_rows, StatusBlock* st) {
  __shared__ int running[kRouteMaxE];
  __shared__ int wcnt[kPlanThreads / 32][kRouteMaxE];
  const int b = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int e = threadIdx.x; e < E; e += blockDim.x) running[e] = blk_base[b * E + e];
  for (int round = 0; round < kPlanPairsPerBlock / kPlanThreads; ++round) {
    for (int i = threadIdx.x; i < (kPlanThreads / 32) * E; i += blockDim.x) (&wcnt[0][0])[(i / E) * kRouteMaxE + i % E] = 0;
    __syncthreads();
    const int i = b * kPlanPairsPerBlock + round * kPlanThreads + threadIdx.x;
    const bool active = i < N;
    int e = active ? idx[i] : -1;
    if (e >= E) e = -1;
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    const int rank_w = __popc(peers & ((1u << lane) - 1u));
    if (e >= 0 && rank_w == 0) wcnt[warp][e] = __popc(peers);
    __syncthreads();
    if (active) {
      if (e < 0) {
        pos[i] = -1;
      } else {
        int r = running[e] + rank_w;
        for (int w = 0; w < warp; ++w) r += wcnt[w][e];
        const int limit = capacity > 0 ? capacity : 0x7fffffff;
        if (r < limit) {
          const int row = offsets[e] + r;
          if (row < cap_rows) {
            pos[i] = row;
            src[row] = i;
          } else {
            pos[i] = -1;
            report_error(st, STATUS_BAD_INDEX, row);
          }
        } else {
          pos[i] = -1;
        }
      }
    }
    __syncthreads();
    for (int ee = threadIdx.x; ee < E; ee += blockDim.x) {
      int add = 0;
      for (int w = 0; w < kPlanThreads / 32; ++w) add += wcnt[w][ee];
      running[ee] += add;
    }
    __syncthreads();
  }
}

// The whole plan in one CTA when every pair fits one block (decode steps): the same
// token-order ranks as count -> scan -> assign, in one launch.
__global__ void __launch_bounds__(kPlanPairsPerBlock) plan_small_kernel(
    const int* __restrict__ idx, int N, int E, int capacity, int* __restrict__ counts, int* __restrict__ offsets,
    int* __restrict__ pos, int* __restrict__ src, int cap_rows, int align, StatusBlock* st) {
  __shared__ int wcnt[kPlanPairsPerBlock / 32][kRouteMaxE];
  __shared__ int kept[kRouteMaxE];
  __shared__ int off[kRouteMaxE + 1];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int kWarps = kPlanPairsPerBlock / 32;
  for (int i = threadIdx.x; i < kWarps * kRouteMaxE; i += blockDim.x) (&wcnt[0][0])[i] = 0;
  __syncthreads();
  const int i = threadIdx.x;
  const bool active = i < N;
  int e = active ? idx[i] : -1;
  if (active && (e < 0 || e >= E)) {
    report_error(st, STATUS_BAD_INDEX, e);
    e = -1;
  }
  const unsigned peers = __match_any_sync(0xffffffffu, e);
  const int rank_w = __popc(peers & ((1u << lane) - 1u));
  if (e >= 0 && rank_w == 0) wcnt[warp][e] = __popc(peers);
  __syncthreads();
  for (int x = threadIdx.x; x < E; x += blockDim.x) {
    int tot = 0;
    for (int w = 0; w < kWarps; ++w) tot += wcnt[w][x];
    counts[x] = tot;
    kept[x] = capacity > 0 ? min(tot, capacity) : tot;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int o = 0;
    for (int x = 0; x < E; ++x) {
      off[x] = o;
      offsets[x] = o;
      o += (kept[x] + align - 1) / align * align;
    }
    off[E] = o;
    offsets[E] = o;
  }
  __syncthreads();
  for (int x = 0; x < E; ++x)
    for (int r = off[x] + kept[x] + threadIdx.x; r < min(off[x + 1], cap_rows); r += blockDim.x) src[r] = -1;
  if (active) {
    if (e < 0) {
      pos[i] = -1;
    } else {
      int r = rank_w;
      for (int w = 0; w < warp; ++w) r += wcnt[w][e];
      if (r < kept[e]) {
        const int row = off[e] + r;
        if (row < cap_rows) {
          pos[i] = row;
          src[row] = i;
        } else {
          pos[i] = -1;
          report_error(st, STATUS_BAD_INDEX, row);
        }
      } else {
        pos[i] = -1;
      }
    }
  }
}

void moe_permute_plan(const int* idx, int T, int K, int E, int capacity, int* counts, int* offsets, int* pos,
                      int* src, int cap_rows, int* workspace, cudaStream_t s, int align) {
  const int N = T * K;
  const int nblocks = (N + kPlanPairsPerBlock - 1) / kPlanPairsPerBlock;
  if (nblocks == 0) {
    cudaMemsetAsync(counts, 0, E * sizeof(int), s);
    cudaMemsetAsync(offsets, 0, (E + 1) * sizeof(int), s);
    return;
  }
  if (nblocks == 1) {
    plan_small_kernel<<<1, kPlanPairsPerBlock, 0, s>>>(idx, N, E, capacity, counts, offsets, pos, src, cap_rows,
                                                       align, (StatusBlock*)status_ptr());
    return;
  }
  StatusBlock* st = (StatusBlock*)status_ptr();
  int* blk_cnt = workspace;
  int* blk_base = workspace + nblocks * E;
  plan_count_kernel<<<nblocks, kPlanThreads, 0, s>>>(idx, N, E, blk_cnt, st);
  plan_scan_kernel<<<1, 256, 0, s>>>(nblocks, E, capacity, blk_cnt, blk_base, counts, offsets, src, cap_rows, align);
  plan_assign_kernel<<<nblocks, kPlanThreads, 0, s>>>(idx, N, E, capacity, blk_base, offsets, pos, src, cap_rows, st);
}

// ---------------------------------------------------------------------------
// Gather / combine
// ---------------------------------------------------------------------------
__global__ void moe_gather_kernel(const bf16* __restrict__ x, const int* __restrict__ src, bf16* __restrict__ xp,
                                  int cap_rows, int K, int dim, const int* __restrict__ offsets, int E) {
  const int total = min(cap_rows, offsets[E]);
  const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
  for (int r = blockIdx.x * warps + (threadIdx.x >> 5); r < total; r += gridDim.x * warps) {
    const int s = src[r];
    bf16* o = xp + (long long)r * dim;
    if (s < 0) {
      for (int c = lane * 8; c < dim; c += 256) *reinterpret_cast<uint4*>(o + c) = make_uint4(0, 0, 0, 0);
    } else {
      const bf16* i = x + (long long)(s / K) * dim;
      for (int c = lane * 8; c < dim; c += 256)
        *reinterpret_cast<uint4*>(o + c) = *reinterpret_cast<const uint4*>(i + c);
    }
  }
}

void moe_gather(const void* x, const int* src, void* x_perm, int cap_rows, int K, int dim, const int* offsets, int E,
                cudaStream_t s) {
  moe_gather_kernel<<<148 * 8, 256, 0, s>>>((const bf16*)x, src, (bf16*)x_perm, cap_rows, K, dim, offsets, E);
}

// One thread per (token, 8 columns): every load is independent, so even a
// decode batch of a few tokens spreads over many SMs.
__global__ void moe_combine_kernel(const bf16* __restrict__ y, const int* __restrict__ pos,
                                   const float* __restrict__ w, const bf16* __restrict__ add, bf16* __restrict__ out,
                                   int T, int K, int dim) {
  const int chunks = dim / 8;
  const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  if (i >= (long long)T * chunks) return;
  const int t = (int)(i / chunks);
  const int c = (int)(i - (long long)t * chunks) * 8;
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  if (add != nullptr) {
    uint4 v = *reinterpret_cast<const uint4*>(add + (long long)t * dim + c);
    const uint32_t* q = reinterpret_cast<const uint32_t*>(&v);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      acc[2 * j] = bf16_lo(q[j]);
      acc[2 * j + 1] = bf16_hi(q[j]);
    }
  }
  for (int k = 0; k < K; ++k) {
    const int p = __ldg(pos + (long long)t * K + k);
    if (p < 0) continue;
    const float wk = __ldg(w + (long long)t * K + k);
    uint4 v = *reinterpret_cast<const uint4*>(y + (long long)p * dim + c);
    const uint32_t* q = reinterpret_cast<const uint32_t*>(&v);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      acc[2 * j] += wk * bf16_lo(q[j]);
      acc[2 * j + 1] += wk * bf16_hi(q[j]);
    }
  }
  uint4 o;
  o.x = pack_bf16x2(acc[0], acc[1]);
  o.y = pack_bf16x2(acc[2], acc[3]);
  o.z = pack_bf16x2(acc[4], acc[5]);
  o.w = pack_bf16x2(acc[6], acc[7]);
  *reinterpret_cast<uint4*>(out + (long long)t * dim + c) = o;
}

void moe_combine(const void* y_perm, const int* pos, const float* w, const void* add, void* out, int T, int K,
                 int dim, cudaStream_t s) {
  const long long work = (long long)T * (dim / 8);
  if (work == 0) return;
  moe_combine_kernel<<<(unsigned)((work + 255) / 256), 256, 0, s>>>((const bf16*)y_perm, pos, w, (const bf16*)add,
                                                                  (bf16*)out, T, K, dim);
}

__global__ void moe_combine_bwd_kernel(const bf16* __restrict__ dout, const bf16* __restrict__ y,
                                       const int* __restrict__ src, const float* __restrict__ w,
                                       bf16* __restrict__ dy, float* __restrict__ dw, int cap_rows, int K, int dim,
                                       const int* __restrict__ offsets, int E) {
  const int total = min(cap_rows, offsets[E]);
  const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
  for (int r = blockIdx.x * warps + (threadIdx.x >> 5); r < total; r += gridDim.x * warps) {
    const int s = src[r];
    bf16* o = dy + (long long)r * dim;
    if (s < 0) {
      for (int c = lane * 8; c < dim; c += 256) *reinterpret_cast<uint4*>(o + c) = make_uint4(0, 0, 0, 0);
      continue;
    }
    const int t = s / K;
    const float wk = w[s];
    const bf16* d = dout + (long long)t * dim;
    const bf16* yr = y + (long long)r * dim;
    float dot = 0.f;
    for (int c = lane * 8; c < dim; c += 256) {
      uint4 dv = *reinterpret_cast<const uint4*>(d + c);
      uint4 yv = *reinterpret_cast<const uint4*>(yr + c);
      const uint32_t* dq = reinterpret_cast<const uint32_t*>(&dv);
      const uint32_t* yq = reinterpret_cast<const uint32_t*>(&yv);
      uint4 ov;
      uint32_t* oq = reinterpret_cast<uint32_t*>(&ov);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float d0 = bf16_lo(dq[j]), d1 = bf16_hi(dq[j]);
        dot += d0 * bf16_lo(yq[j]) + d1 * bf16_hi(yq[j]);
        oq[j] = pack_bf16x2(d0 * wk, d1 * wk);
      }
      *reinterpret_cast<uint4*>(o + c) = ov;
    }
    dot = warp_sum(dot);
    if (lane == 0) dw[s] = dot;
  }
}

void moe_combine_bwd(const void* dout, const void* y_perm, const int* src, const float* w, void* dy_perm, float* dw,
                     int cap_rows, int K, int dim, const int* offsets, int E, cudaStream_t s) {
  moe_combine_bwd_kernel<<<148 * 8, 256, 0, s>>>((const bf16*)dout, (const bf16*)y_perm, src, w, (bf16*)dy_perm, dw,
                                                 cap_rows, K, dim, offsets, E);
}

__global__ void moe_scatter_add_kernel(const bf16* __restrict__ dxp, const int* __restrict__ pos,
                                       const bf16* __restrict__ dx_add, bf16* __restrict__ dx, int T, int K, int dim) {
  const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (t >= T) return;
  for (int c = lane * 8; c < dim; c += 256) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if (dx_add != nullptr) {
      uint4 v = *reinterpret_cast<const uint4*>(dx_add + (long long)t * dim + c);
      const uint32_t* q = reinterpret_cast<const uint32_t*>(&v);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        acc[2 * j] = bf16_lo(q[j]);
        acc[2 * j + 1] = bf16_hi(q[j]);
      }
    }
    for (int k = 0; k < K; ++k) {
      const int p = pos[(long long)t * K + k];
      if (p < 0) continue;
      uint4 v = *reinterpret_cast<const uint4*>(dxp + (long long)p * dim + c);
      const uint32_t* q = reinterpret_cast<const uint32_t*>(&v);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        acc[2 * j] += bf16_lo(q[j]);
        acc[2 * j + 1] += bf16_hi(q[j]);
      }
    }
    uint4 o;
    o.x = pack_bf16x2(acc[0], acc[1]);
    o.y = pack_bf16x2(acc[2], acc[3]);
    o.z = pack_bf16x2(acc[4], acc[5]);
    o.w = pack_bf16x2(acc[6], acc[7]);
    *reinterpret_cast<uint4*>(dx + (long long)t * dim + c) = o;
  }
}

void moe_scatter_add(const void* dx_perm, const int* pos, const void* dx_add, void* dx, int T, int K, int dim,
                     cudaStream_t s) {
  const int warps = 8;
  moe_scatter_add_kernel<<<(T + warps - 1) / warps, warps * 32, 0, s>>>((const bf16*)dx_perm, pos,
                                                                        (const bf16*)dx_add, (bf16*)dx, T, K, dim);
}

// ---------------------------------------------------------------------------
// Router backward
// ---------------------------------------------------------------------------
__global__ void router_bwd_kernel(const float* __restrict__ logits, const float* __restrict__ probs,
                                  const int* __restrict__ idx, const float* __restrict__ dw,
                                  const int* __restrict__ counts, bf16* __restrict__ dlogits, int T, int E, int K,
                                  bool renorm, float aux_alpha, float z_beta, float* __restrict__ aux_out) {
  const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (t >= T) return;
  const int per = (E + 31) / 32;
  float p[kRouteMaxE / 32], dp[kRouteMaxE / 32];
  float lmax = -INFINITY;
#pragma unroll
  for (int j = 0; j < kRouteMaxE / 32; ++j) {
    const int e = lane + 32 * j;
    const bool ok = j < per && e < E;
    p[j] = ok ? probs[(long long)t * E + e] : 0.f;
    dp[j] = 0.f;
    if (ok) lmax = fmaxf(lmax, logits[(long long)t * E + e]);
  }
  // gradient w.r.t. the kept probabilities
  float S = 0.f, sdw = 0.f;
  // gather p of the selected experts (each lane reads from global; E*T probs are small)
  float psel[kRouteMaxK];
  for (int k = 0; k < K; ++k) {
    const int e = idx[(long long)t * K + k];
    psel[k] = probs[(long long)t * E + e];
    S += psel[k];
  }
  if (renorm) {
    for (int k = 0; k < K; ++k) sdw += dw[(long long)t * K + k] * (psel[k] / S);
  }
  for (int k = 0; k < K; ++k) {
    const int e = idx[(long long)t * K + k];
    const float g = renorm ? (dw[(long long)t * K + k] - sdw) / S : dw[(long long)t * K + k];
#pragma unroll
    for (int j = 0; j < kRouteMaxE / 32; ++j)
      if (lane + 32 * j == e) dp[j] += g;
  }
  // load-balance loss: alpha * E * sum_e f_e * mean_t p_te  with f_e = counts/(T*K)
  float aux = 0.f;
  if (aux_alpha > 0.f) {
#pragma unroll
    for (int j = 0; j < kRouteMaxE / 32; ++j) {
      const int e = lane + 32 * j;
      if (j < per && e < E) {
        const float f = (float)counts[e] / (float)(T * K);
        dp[j] += aux_alpha * (float)E * f / (float)T;
        aux += aux_alpha * (float)E * f * p[j] / (float)T;
      }
    }
  }
  // softmax backward
  float dot = 0.f;
#pragma unroll
  for (int j = 0; j < kRouteMaxE / 32; ++j) dot += p[j] * dp[j];
  dot = warp_sum(dot);
  // z-loss: beta * mean_t lse^2
  const float lmax_all = warp_max(lmax);
  float zsum = 0.f;
#pragma unroll
  for (int j = 0; j < kRouteMaxE / 32; ++j) {
    const int e = lane + 32 * j;
    if (j < per && e < E) zsum += __expf(logits[(long long)t * E + e] - lmax_all);
  }
  const float lse = lmax_all + __logf(warp_sum(zsum));
#pragma unroll
  for (int j = 0; j < kRouteMaxE / 32; ++j) {
    const int e = lane + 32 * j;
    if (j < per && e < E) {
      float g = p[j] * (dp[j] - dot);
      if (z_beta > 0.f) g += z_beta * 2.f * lse * p[j] / (float)T;
      dlogits[(long long)t * E + e] = __float2bfloat16(g);
    }
  }
  aux = warp_sum(aux);
  if (lane == 0 && aux_out != nullptr) {
    atomicAdd(&aux_out[0], aux);
    atomicAdd(&aux_out[1], z_beta * lse * lse / (float)T);
  }
}

void router_bwd(const float* logits, const float* probs, const int* idx, const float* dw, const int* counts,
                void* dlogits, int T, int E, int K, bool renorm, float aux_alpha, float z_beta, float* aux_out,
                cudaStream_t s) {
  const int warps = 8;
  router_bwd_kernel<<<(T + warps - 1) / warps, warps * 32, 0, s>>>(logits, probs, idx, dw, counts, (bf16*)dlogits, T,
                                                                   E, K, renorm, aux_alpha, z_beta, aux_out);
}

}  // namespace omni
