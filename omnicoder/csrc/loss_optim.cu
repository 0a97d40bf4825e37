// Cross-entropy and AdamW kernels (sm_100a).
//
// Cross entropy follows the reference trainer's token loss
// (src/omnicoder/training/pretrain.py:727, F.cross_entropy over the vocabulary)
// and adds the optional z-loss of the spec family.  AdamW follows
// torch.optim.AdamW's decoupled update, which the reference uses
// (src/omnicoder/training/pretrain.py:582).
#include "common.cuh"
#include "kernels.h"

namespace omni {

using bf16 = __nv_bfloat16;

template <int THREADS>
__device__ __forceinline__ void block_max_sum(float& m, float& s, float* sh_m, float* sh_s) {
  // combine (max, sum-of-exp relative to max) pairs
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
    const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
    const float mm = fmaxf(m, m2);
    s = (m == -INFINITY ? 0.f : s * __expf(m - mm)) + (m2 == -INFINITY ? 0.f : s2 * __expf(m2 - mm));
    m = mm;
  }
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) {
    sh_m[w] = m;
    sh_s[w] = s;
  }
  __syncthreads();
  if (w == 0) {
    m = l < THREADS / 32 ? sh_m[l] : -INFINITY;
    s = l < THREADS / 32 ? sh_s[l] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
      const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
      const float mm = fmaxf(m, m2);
      s = (m == -INFINITY ? 0.f : s * __expf(m - mm)) + (m2 == -INFINITY ? 0.f : s2 * __expf(m2 - mm));
      m = mm;
    }
    if (l == 0) {
      sh_m[0] = m;
      sh_s[0] = s;
    }
  }
  __syncthreads();
  m = sh_m[0];
  s = sh_s[0];
}

template <int THREADS>
__global__ void __launch_bounds__(THREADS) ce_kernel(const bf16* __restrict__ logits, long long ld,
                                                     const int64_t* __restrict__ labels, float* __restrict__ loss,
                                                     float* __restrict__ lse_out, bf16* dlogits, int vocab,
                                                     float grad_scale, float z_loss) {
  __shared__ float sh_m[32], sh_s[32];
  const int row = blockIdx.x;
  const bf16* x = logits + (long long)row * ld;
  const int vec_end = (vocab / 8) * 8;
  float m = -INFINITY, s = 0.f;
  for (int c = threadIdx.x * 8; c < vec_end; c += THREADS * 8) {
    uint4 v = *reinterpret_cast<const uint4*>(x + c);
    const uint32_t* w = reinterpret_cast<const uint32_t*>(&v);
    float f[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      f[2 * i] = bf16_lo(w[i]);
      f[2 * i + 1] = bf16_hi(w[i]);
    }
    float lm = f[0];
#pragma unroll
    for (int i = 1; i < 8; ++i) lm = fmaxf(lm, f[i]);
    const float nm = fmaxf(m, lm);
    float acc = (m == -INFINITY) ? 0.f : s * __expf(m - nm);
#pragma unroll
    for (int i = 0; i < 8; ++i) acc += __expf(f[i] - nm);
    s = acc;
    m = nm;
  }
  for (int c = vec_end + threadIdx.x; c < vocab; c += THREADS) {
    const float f = __bfloat162float(x[c]);
    const float nm = fmaxf(m, f);
    s = ((m == -INFINITY) ? 0.f : s * __expf(m - nm)) + __expf(f - nm);
    m = nm;
  }
  block_max_sum<THREADS>(m, s, sh_m, sh_s);
  const float lse = m + __logf(s);
  const int64_t lab = labels[row];
  const bool valid = lab >= 0 && lab < vocab;
  if (threadIdx.x == 0) {
    lse_out[row] = lse;
    loss[row] = valid ? (lse - __bfloat162float(x[lab]) + z_loss * lse * lse) : 0.f;
  }
  if (dlogits == nullptr) return;
  // All reads of this row above precede the in-place writes below.
  __syncthreads();
  bf16* d = dlogits + (long long)row * ld;
  const float sc = valid ? grad_scale : 0.f;
  const float zf = 1.f + 2.f * z_loss * lse;
  for (int c = threadIdx.x * 8; c < vec_end; c += THREADS * 8) {
    uint4 v = *reinterpret_cast<const uint4*>(x + c);
    const uint32_t* w = reinterpret_cast<const uint32_t*>(&v);
    float f[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      f[2 * i] = bf16_lo(w[i]);
      f[2 * i + 1] = bf16_hi(w[i]);
    }
    float g[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) g[i] = (__expf(f[i] - lse) * zf - ((c + i) == lab ? 1.f : 0.f)) * sc;
    uint4 o;
    o.x = pack_bf16x2(g[0], g[1]);
    o.y = pack_bf16x2(g[2], g[3]);
    o.z = pack_bf16x2(g[4], g[5]);
    o.w = pack_bf16x2(g[6], g[7]);
    *reinterpret_cast<uint4*>(d + c) = o;
  }
  for (int c = vec_end + threadIdx.x; c < vocab; c += THREADS) {
    const float f = __bfloat162float(x[c]);
    d[c] = __float2bfloat16((__expf(f - lse) * zf - (c == lab ? 1.f : 0.f)) * sc);
  }
}

void cross_entropy_fwd_bwd(const void* logits, long long ld, const int64_t* labels, float* loss, float* lse,
                           void* dlogits, int rows, int vocab, float grad_scale, float z_loss, cudaStream_t s) {
  if (rows <= 0) return;
  ce_kernel<512><<<rows, 512, 0, s>>>((const bf16*)logits, ld, labels, loss, lse, (bf16*)dlogits, vocab,
                                      grad_scale, z_loss);
}

// ---------------------------------------------------------------------------
// AdamW over flat buffers
// ---------------------------------------------------------------------------
__global__ void adamw_kernel(float* __restrict__ p, float* __restrict__ m, float* __restrict__ v,
                             const bf16* __restrict__ g, bf16* __restrict__ pb, long long n, float lr, float b1,
                             float b2, float eps, float wd, float bc1, float bc2, float grad_scale,
                             const float* __restrict__ norm_sq, float max_norm) {
  float clip = 1.f;
  if (max_norm > 0.f && norm_sq != nullptr) {
    const float nrm = sqrtf(*norm_sq);
    clip = fminf(1.f, max_norm / (nrm + 1e-6f));
  }
  const float gs = grad_scale * clip;
  const float step = lr / bc1;
  const float inv_sqrt_bc2 = rsqrtf(bc2);
  const float decay = 1.f - lr * wd;
  const long long n4 = n / 4;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n4; i += (long long)gridDim.x * blockDim.x) {
    float4 pp = reinterpret_cast<float4*>(p)[i];
    float4 mm = reinterpret_cast<float4*>(m)[i];
    float4 vv = reinterpret_cast<float4*>(v)[i];
    uint2 gg = reinterpret_cast<const uint2*>(g)[i];
    float gf[4] = {bf16_lo(gg.x) * gs, bf16_hi(gg.x) * gs, bf16_lo(gg.y) * gs, bf16_hi(gg.y) * gs};
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
    if (pb != nullptr) reinterpret_cast<uint2*>(pb)[i] = make_uint2(pack_bf16x2(pa[0], pa[1]), pack_bf16x2(pa[2], pa[3]));
  }
  // tail
  for (long long i = n4 * 4 + blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const float gf = __bfloat162float(g[i]) * gs;
    m[i] = b1 * m[i] + (1.f - b1) * gf;
    v[i] = b2 * v[i] + (1.f - b2) * gf * gf;
    p[i] = p[i] * decay - step * m[i] / (sqrtf(v[i]) * inv_sqrt_bc2 + eps);
    if (pb != nullptr) pb[i] = __float2bfloat16(p[i]);
  }
}

void adamw_step(float* p, float* m, float* v, const void* g, void* p_bf16, long long n, float lr, float beta1,
                float beta2, float eps, float wd, float bc1, float bc2, float grad_scale, const float* norm_sq,
                float max_norm, cudaStream_t s) {
  if (n <= 0) return;
  long long blocks = (n / 4 + 255) / 256;
  if (blocks > 148 * 8) blocks = 148 * 8;
  if (blocks < 1) blocks = 1;
  adamw_kernel<<<(int)blocks, 256, 0, s>>>(p, m, v, (const bf16*)g, (bf16*)p_bf16, n, lr, beta1, beta2, eps, wd,
                                           bc1, bc2, grad_scale, norm_sq, max_norm);
}

__global__ void sq_norm_kernel(const bf16* __restrict__ g, long long n, float scale, float* out) {
  __shared__ float sh[32];
  float acc = 0.f;
  const long long n8 = n / 8;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n8; i += (long long)gridDim.x * blockDim.x) {
    uint4 v = reinterpret_cast<const uint4*>(g)[i];
    const uint32_t* w = reinterpret_cast<const uint32_t*>(&v);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float a = bf16_lo(w[k]), b = bf16_hi(w[k]);
      acc += a * a + b * b;
    }
  }
  for (long long i = n8 * 8 + blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const float a = __bfloat162float(g[i]);
    acc += a * a;
  }
  acc = warp_sum(acc);
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x < 32) {
    acc = threadIdx.x < (blockDim.x >> 5) ? sh[threadIdx.x] : 0.f;
    acc = warp_sum(acc);
    if (threadIdx.x == 0) atomicAdd(out, acc * scale * scale);
  }
}

void sq_norm_accum(const void* g, long long n, float scale, float* out, cudaStream_t s) {
  if (n <= 0) return;
  long long blocks = (n / 8 + 255) / 256;
  if (blocks > 148 * 4) blocks = 148 * 4;
  if (blocks < 1) blocks = 1;
  sq_norm_kernel<<<(int)blocks, 256, 0, s>>>((const bf16*)g, n, scale, out);
}

// ---------------------------------------------------------------------------
// Multi-tensor forms for many small parameters (norm weights, routers): one block
// per tensor, up to kMultiItems tensors per launch, the table passed by value.
// Same arithmetic as adamw_kernel / sq_norm_kernel (scalar loop, fp32).
// ---------------------------------------------------------------------------
__global__ void adamw_multi_kernel(AdamwMulti t, float lr, float b1, float b2, float eps, float bc1, float bc2,
                                   float grad_scale, const float* __restrict__ norm_sq, float max_norm) {
  if ((int)blockIdx.x >= t.count) return;
  const AdamwItem it = t.item[blockIdx.x];
  float clip = 1.f;
  if (max_norm > 0.f && norm_sq != nullptr) clip = fminf(1.f, max_norm / (sqrtf(*norm_sq) + 1e-6f));
  const float gs = grad_scale * clip;
  const float step = lr / bc1;
  const float inv_sqrt_bc2 = rsqrtf(bc2);
  const float decay = 1.f - lr * it.wd;
  const bf16* g = reinterpret_cast<const bf16*>(it.g);
  bf16* pb = reinterpret_cast<bf16*>(it.pb);
  for (long long i = threadIdx.x; i < it.n; i += blockDim.x) {
    const float gf = __bfloat162float(g[i]) * gs;
    it.m[i] = b1 * it.m[i] + (1.f - b1) * gf;
    it.v[i] = b2 * it.v[i] + (1.f - b2) * gf * gf;
    it.p[i] = it.p[i] * decay - step * it.m[i] / (sqrtf(it.v[i]) * inv_sqrt_bc2 + eps);
    if (pb != nullptr) pb[i] = __float2bfloat16(it.p[i]);
  }
}

__global__ void sq_norm_multi_kernel(AdamwMulti t, float scale, float* out) {
  __shared__ float sh[32];
  if ((int)blockIdx.x >= t.count) return;
  const AdamwItem it = t.item[blockIdx.x];
  const bf16* g = reinterpret_cast<const bf16*>(it.g);
  float acc = 0.f;
  for (long long i = threadIdx.x; i < it.n; i += blockDim.x) {
    const float a = __bfloat162float(g[i]);
    acc += a * a;
  }
  acc = warp_sum(acc);
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x < 32) {
    acc = threadIdx.x < (blockDim.x >> 5) ? sh[threadIdx.x] : 0.f;
    acc = warp_sum(acc);
    if (threadIdx.x == 0) atomicAdd(out, acc * scale * scale);
  }
}

void adamw_multi(const AdamwMulti& t, float lr, float b1, float b2, float eps, float bc1, float bc2, float grad_scale,
                 const float* norm_sq, float max_norm, cudaStream_t s) {
  if (t.count <= 0) return;
  adamw_multi_kernel<<<t.count, 256, 0, s>>>(t, lr, b1, b2, eps, bc1, bc2, grad_scale, norm_sq, max_norm);
}

void sq_norm_multi(const AdamwMulti& t, float scale, float* out, cudaStream_t s) {
  if (t.count <= 0) return;
  sq_norm_multi_kernel<<<t.count, 256, 0, s>>>(t, scale, out);
}

}  // namespace omni
