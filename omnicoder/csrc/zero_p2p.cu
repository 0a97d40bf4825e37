// ZeRO-1 data-parallel optimiser step over NVLink peer memory (sm_100a).
//
// Every rank's flat gradient bucket and flat bf16 parameter bucket are
// peer-mapped (symmetric memory).  Rank `me` owns elements [lo, lo + n) of the
// bucket:
//   zero_rs          reduce-scatter fused with the bucket's scaling and the
//                    squared-norm partial of gradient clipping: this rank's shard
//                    is summed in fp32 straight from every rank's gradient bucket
//                    (peer loads) into an fp32 shard gradient
//   zero_adamw_push  the partitioned AdamW update of the shard (fp32 master,
//                    moments) fused with the all-gather of the new weights: the
//                    bf16 result is stored into every rank's parameter bucket
//                    (peer stores)
// A device barrier over the group (bounded waits) precedes zero_rs (every
// rank's bucket gradient is complete) and follows the last zero_adamw_push
// (every rank's parameters are complete).  Plain loads and stores only: no TMA,
// no multicast.  Replaces NCCL reduce-scatter + separate norm / AdamW kernels
// + NCCL all-gather; the reference has no data-parallel optimiser
// (src/omnicoder/tools/torchrun_ep.py:13-18 defines an unused all_reduce).
#include <algorithm>
#include <cmath>

#include "common.cuh"
#include "ep_comm.h"

namespace omni {

namespace {

using bf16 = __nv_bfloat16;

__device__ __forceinline__ void block_add(float v, float* out) {
  __shared__ float sh[32];
  v = warp_sum(v);
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = v;
  __syncthreads();
  if (threadIdx.x < 32) {
    v = threadIdx.x < (blockDim.x >> 5) ? sh[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) atomicAdd(out, v);
  }
}

__global__ void zero_rs_kernel(EpPeers g, int world, long long lo, long long n, float scale, float* __restrict__ out,
                               float* __restrict__ norm_sq) {
  float sq = 0.f;
  const long long n8 = n / 8;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n8; i += (long long)gridDim.x * blockDim.x) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int r = 0; r < world; ++r) {
      const uint4 v = *reinterpret_cast<const uint4*>(reinterpret_cast<const bf16*>(g.ptr[r]) + lo + i * 8);
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        acc[2 * k] += bf16_lo(w[k]);
        acc[2 * k + 1] += bf16_hi(w[k]);
      }
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      acc[k] *= scale;
      sq += acc[k] * acc[k];
    }
    float4* o = reinterpret_cast<float4*>(out + i * 8);
    o[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
    o[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
  }
  for (long long i = n8 * 8 + blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    float a = 0.f;
    for (int r = 0; r < world; ++r) a += __bfloat162float(reinterpret_cast<const bf16*>(g.ptr[r])[lo + i]);
    a *= scale;
    sq += a * a;
    out[i] = a;
  }
  if (norm_sq != nullptr) block_add(sq, norm_sq);
}

__global__ void zero_adamw_push_kernel(float* __restrict__ p, float* __restrict__ m, float* __restrict__ v,
                                       const float* __restrict__ g, EpPeers dst, int world, long long lo, long long n,
                                       float lr, float b1, float b2, float eps, float wd, float bc1, float bc2,
                                       const float* __restrict__ norm_sq, float max_norm) {
  float clip = 1.f;
  if (max_norm > 0.f && norm_sq != nullptr) clip = fminf(1.f, max_norm / (sqrtf(*norm_sq) + 1e-6f));
  const float step = lr / bc1;
  const float inv_sqrt_bc2 = rsqrtf(bc2);
  const float decay = 1.f - lr * wd;
  const long long n4 = n / 4;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n4; i += (long long)gridDim.x * blockDim.x) {
    float4 pp = reinterpret_cast<float4*>(p)[i];
    float4 mm = reinterpret_cast<float4*>(m)[i];
    float4 vv = reinterpret_cast<float4*>(v)[i];
    const float4 gg = reinterpret_cast<const float4*>(g)[i];
    const float gf[4] = {gg.x * clip, gg.y * clip, gg.z * clip, gg.w * clip};
    float* pa = &pp.x;
    float* ma = &mm.x;
    float* va = &vv.x;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      ma[k] = b1 * ma[k] + (1.f - b1) * gf[k];
      va[k] = b2 * va[k] + (1.f - b2) * gf[k] * gf[k];
      pa[k] = pa[k] * decay - step * ma[k] / (sqrtf(va[k]) * inv_sqrt_bc2 + eps);
    }
    reinterpret_cast<float4*>(p)[i] = pp;
    reinterpret_cast<float4*>(m)[i] = mm;
    reinterpret_cast<float4*>(v)[i] = vv;
    const uint2 packed = make_uint2(pack_bf16x2(pa[0], pa[1]), pack_bf16x2(pa[2], pa[3]));
    for (int r = 0; r < world; ++r)
      *reinterpret_cast<uint2*>(reinterpret_cast<bf16*>(dst.ptr[r]) + lo + i * 4) = packed;
  }
  for (long long i = n4 * 4 + blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const float gf = g[i] * clip;
    m[i] = b1 * m[i] + (1.f - b1) * gf;
    v[i] = b2 * v[i] + (1.f - b2) * gf * gf;
    p[i] = p[i] * decay - step * m[i] / (sqrtf(v[i]) * inv_sqrt_bc2 + eps);
    const bf16 b = __float2bfloat16(p[i]);
    for (int r = 0; r < world; ++r) reinterpret_cast<bf16*>(dst.ptr[r])[lo + i] = b;
  }
}

int grid_for(long long n, int per_thread) {
  const long long b = (n / per_thread + 255) / 256;
  return (int)std::max(1ll, std::min(b, 148ll * 8));
}

}  // namespace

void zero_rs(const EpPeers& g, int world, long long lo, long long n, float scale, float* out, float* norm_sq,
             cudaStream_t s) {
  if (n <= 0) return;
  zero_rs_kernel<<<grid_for(n, 8), 256, 0, s>>>(g, world, lo, n, scale, out, norm_sq);
}

void zero_adamw_push(float* p, float* m, float* v, const float* g, const EpPeers& dst, int world, long long lo,
                     long long n, float lr, float b1, float b2, float eps, float wd, int step, const float* norm_sq,
                     float max_norm, cudaStream_t s) {
  if (n <= 0) return;
  const float bc1 = (float)(1.0 - std::pow((double)b1, (double)step));
  const float bc2 = (float)(1.0 - std::pow((double)b2, (double)step));
  zero_adamw_push_kernel<<<grid_for(n, 4), 256, 0, s>>>(p, m, v, g, dst, world, lo, n, lr, b1, b2, eps, wd, bc1, bc2,
                                                        norm_sq, max_norm);
}

}  // namespace omni
