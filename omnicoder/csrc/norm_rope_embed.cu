// Normalisation, rotary embedding and embedding-table kernels (sm_100a).
//
// All kernels are bandwidth bound: one warp per row, 16-byte vector accesses,
// fp32 arithmetic, bf16 storage.  Reference behaviour:
//   * RMSNorm replaces the reference's nn.LayerNorm in the spec family; the
//     compat family keeps LayerNorm (src/omnicoder/modeling/transformer_moe.py:809).
//   * RoPE rotates pairs (x0, x1) -> (x0 cos - x1 sin, x1 cos + x0 sin)
//     (src/omnicoder/modeling/attention.py:115-320); the interleaved pairing is
//     the reference's, the half-split pairing is the spec family's.
#include "common.cuh"
#include "kernels.h"

namespace omni {

using bf16 = __nv_bfloat16;

__device__ __forceinline__ void load8(const bf16* p, float* f) {
  uint4 v = *reinterpret_cast<const uint4*>(p);
  const uint32_t* w = reinterpret_cast<const uint32_t*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = bf16_lo(w[i]);
    f[2 * i + 1] = bf16_hi(w[i]);
  }
}

__device__ __forceinline__ void store8(bf16* p, const float* f) {
  uint4 v;
  v.x = pack_bf16x2(f[0], f[1]);
  v.y = pack_bf16x2(f[2], f[3]);
  v.z = pack_bf16x2(f[4], f[5]);
  v.w = pack_bf16x2(f[6], f[7]);
  *reinterpret_cast<uint4*>(p) = v;
}

// Round-trip through bf16 (the value that is stored).
__device__ __forceinline__ float rt_bf16(float x) { return __bfloat162float(__float2bfloat16(x)); }

// ---------------------------------------------------------------------------
// RMSNorm
// ---------------------------------------------------------------------------
template <bool RES>
__global__ void rmsnorm_fwd_kernel(const bf16* __restrict__ x, const bf16* __restrict__ r, bf16* __restrict__ h,
                                   const bf16* __restrict__ w, bf16* __restrict__ y, float* __restrict__ rstd,
                                   int rows, int dim, float eps) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const long long base = (long long)row * dim;
  float ss = 0.f;
  for (int c = lane * 8; c < dim; c += 256) {
    float a[8];
    load8(x + base + c, a);
    if (RES) {
      float b[8];
      load8(r + base + c, b);
#pragma unroll
      for (int i = 0; i < 8; ++i) a[i] = rt_bf16(a[i] + b[i]);
      store8(h + base + c, a);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) ss += a[i] * a[i];
  }
  ss = warp_sum(ss);
  const float rs = rsqrtf(ss / (float)dim + eps);
  if (lane == 0) rstd[row] = rs;
  const bf16* src = RES ? h : x;
  for (int c = lane * 8; c < dim; c += 256) {
    float a[8], g[8];
    load8(src + base + c, a);
    load8(w + c, g);
#pragma unroll
    for (int i = 0; i < 8; ++i) a[i] = a[i] * rs * g[i];
    store8(y + base + c, a);
  }
}

void rmsnorm_fwd(const void* x, const void* r, void* h, const void* w, void* y, float* rstd, int rows, int dim,
                 float eps, cudaStream_t s) {
  const int warps = 8;
  dim3 grid((rows + warps - 1) / warps);
  if (r != nullptr)
    rmsnorm_fwd_kernel<true><<<grid, warps * 32, 0, s>>>((const bf16*)x, (const bf16*)r, (bf16*)h, (const bf16*)w,
                                                          (bf16*)y, rstd, rows, dim, eps);
  else
    rmsnorm_fwd_kernel<false><<<grid, warps * 32, 0, s>>>((const bf16*)x, nullptr, nullptr, (const bf16*)w,
                                                           (bf16*)y, rstd, rows, dim, eps);
}

// dx = rstd * (w*dy - xhat * mean(xhat * w * dy)) (+ dres);  dw += sum_rows dy * xhat
__global__ void rmsnorm_bwd_kernel(const bf16* __restrict__ x, const bf16* __restrict__ w,
                                   const float* __restrict__ rstd, const bf16* __restrict__ dy,
                                   const bf16* __restrict__ dres, bf16* __restrict__ dx, float* __restrict__ dw,
                                   int rows, int dim) {
  extern __shared__ float s_dw[];
  for (int i = threadIdx.x; i < dim; i += blockDim.x) s_dw[i] = 0.f;
  __syncthreads();
  const int warps = blockDim.x >> 5;
  const int lane = threadIdx.x & 31;
  for (int row = blockIdx.x * warps + (threadIdx.x >> 5); row < rows; row += gridDim.x * warps) {
    const long long base = (long long)row * dim;
    const float rs = rstd[row];
    float dot = 0.f;
    for (int c = lane * 8; c < dim; c += 256) {
      float a[8], g[8], d[8];
      load8(x + base + c, a);
      load8(w + c, g);
      load8(dy + base + c, d);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float xh = a[i] * rs;
        dot += xh * g[i] * d[i];
        atomicAdd(&s_dw[c + i], d[i] * xh);
      }
    }
    dot = warp_sum(dot) / (float)dim;
    for (int c = lane * 8; c < dim; c += 256) {
      float a[8], g[8], d[8], o[8];
      load8(x + base + c, a);
      load8(w + c, g);
      load8(dy + base + c, d);
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = rs * (g[i] * d[i] - a[i] * rs * dot);
      if (dres != nullptr) {
        float e[8];
        load8(dres + base + c, e);
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] += e[i];
      }
      store8(dx + base + c, o);
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < dim; i += blockDim.x) atomicAdd(&dw[i], s_dw[i]);
}

// Same, for dim = NC * 256 <= 2048: each warp accumulates dw for its rows in its own
// shared-memory row (lane owns columns lane*8 + 256k, so no atomics), and the block sums its
// warps' rows once at the end (the general kernel above does a shared-memory atomic per
// element).
template <int NC>
__global__ void __launch_bounds__(128) rmsnorm_bwd_warp_kernel(const bf16* __restrict__ x, const bf16* __restrict__ w,
                                                               const float* __restrict__ rstd, const bf16* __restrict__ dy,
                                                               const bf16* __restrict__ dres, bf16* __restrict__ dx,
                                                               float* __restrict__ dw, int rows) {
  constexpr int dim = NC * 256;
  constexpr int kWarps = 4;
  __shared__ __align__(16) float s_acc[kWarps][dim];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  for (int i = lane * 4; i < dim; i += 128) *reinterpret_cast<float4*>(&s_acc[warp][i]) = make_float4(0.f, 0.f, 0.f, 0.f);
  __syncwarp();
  for (int row = blockIdx.x * kWarps + warp; row < rows; row += gridDim.x * kWarps) {
    const long long base = (long long)row * dim + lane * 8;
    const float rs = rstd[row];
    float dot = 0.f;
#pragma unroll 2
    for (int k = 0; k < NC; ++k) {
      float wv[8], xh[8], g[8];
      load8(w + k * 256 + lane * 8, wv);
      load8(x + base + k * 256, xh);
      load8(dy + base + k * 256, g);
      float4* a = reinterpret_cast<float4*>(&s_acc[warp][k * 256 + lane * 8]);
      float4 a0 = a[0], a1 = a[1];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        xh[i] *= rs;
        dot += xh[i] * wv[i] * g[i];
      }
      a0.x += g[0] * xh[0]; a0.y += g[1] * xh[1]; a0.z += g[2] * xh[2]; a0.w += g[3] * xh[3];
      a1.x += g[4] * xh[4]; a1.y += g[5] * xh[5]; a1.z += g[6] * xh[6]; a1.w += g[7] * xh[7];
      a[0] = a0;
      a[1] = a1;
    }
    dot = warp_sum(dot) / (float)dim;
#pragma unroll 2
    for (int k = 0; k < NC; ++k) {  // second pass over the row: its 4 KB are still in L1
      float wv[8], xh[8], g[8], o[8];
      load8(w + k * 256 + lane * 8, wv);
      load8(x + base + k * 256, xh);
      load8(dy + base + k * 256, g);
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = rs * (wv[i] * g[i] - xh[i] * rs * dot);
      if (dres != nullptr) {
        float e[8];
        load8(dres + base + k * 256, e);
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] += e[i];
      }
      store8(dx + base + k * 256, o);
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < dim; i += blockDim.x) {
    float t = 0.f;
#pragma unroll
    for (int v = 0; v < kWarps; ++v) t += s_acc[v][i];
    atomicAdd(&dw[i], t);
  }
}

void rmsnorm_bwd(const void* x, const void* w, const float* rstd, const void* dy, const void* dres, void* dx,
                 float* dw, int rows, int dim, cudaStream_t s) {
  if (dim == 512 || dim == 1024 || dim == 2048) {
    int grid = (rows + 3) / 4;
    if (grid > 148 * 6) grid = 148 * 6;
    auto launch = [&](auto kern) {
      kern<<<grid, 128, 0, s>>>((const bf16*)x, (const bf16*)w, rstd, (const bf16*)dy, (const bf16*)dres, (bf16*)dx,
                                dw, rows);
    };
    if (dim == 512) launch(rmsnorm_bwd_warp_kernel<2>);
    else if (dim == 1024) launch(rmsnorm_bwd_warp_kernel<4>);
    else launch(rmsnorm_bwd_warp_kernel<8>);
    return;
  }
  const int warps = 8;
  int grid = (rows + warps - 1) / warps;
  if (grid > 148 * 4) grid = 148 * 4;
  rmsnorm_bwd_kernel<<<grid, warps * 32, dim * sizeof(float), s>>>((const bf16*)x, (const bf16*)w, rstd,
                                                                   (const bf16*)dy, (const bf16*)dres, (bf16*)dx,
                                                                   dw, rows, dim);
}

// ---------------------------------------------------------------------------
// LayerNorm (affine), compat family
// ---------------------------------------------------------------------------
__global__ void layernorm_fwd_kernel(const bf16* __restrict__ x, const bf16* __restrict__ w,
                                     const bf16* __restrict__ b, bf16* __restrict__ y, float* __restrict__ mean_out,
                                     float* __restrict__ rstd_out, int rows, int dim, float eps) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const long long base = (long long)row * dim;
  float s1 = 0.f;
  for (int c = lane * 8; c < dim; c += 256) {
    float a[8];
    load8(x + base + c, a);
#pragma unroll
    for (int i = 0; i < 8; ++i) s1 += a[i];
  }
  const float mu = warp_sum(s1) / (float)dim;
  float s2 = 0.f;
  for (int c = lane * 8; c < dim; c += 256) {
    float a[8];
    load8(x + base + c, a);
#pragma unroll
    for (int i = 0; i < 8; ++i) s2 += (a[i] - mu) * (a[i] - mu);
  }
  const float rs = rsqrtf(warp_sum(s2) / (float)dim + eps);
  if (lane == 0) {
    mean_out[row] = mu;
    rstd_out[row] = rs;
  }
  for (int c = lane * 8; c < dim; c += 256) {
    float a[8], g[8], bb[8];
    load8(x + base + c, a);
    load8(w + c, g);
    load8(b + c, bb);
#pragma unroll
    for (int i = 0; i < 8; ++i) a[i] = (a[i] - mu) * rs * g[i] + bb[i];
    store8(y + base + c, a);
  }
}

void layernorm_fwd(const void* x, const void* w, const void* b, void* y, float* mean, float* rstd, int rows,
                   int dim, float eps, cudaStream_t s) {
  const int warps = 8;
  layernorm_fwd_kernel<<<(rows + warps - 1) / warps, warps * 32, 0, s>>>(
      (const bf16*)x, (const bf16*)w, (const bf16*)b, (bf16*)y, mean, rstd, rows, dim, eps);
}

__global__ void layernorm_bwd_kernel(const bf16* __restrict__ x, const bf16* __restrict__ w,
                                     const float* __restrict__ mean, const float* __restrict__ rstd,
                                     const bf16* __restrict__ dy, bf16* __restrict__ dx, float* __restrict__ dw,
                                     float* __restrict__ db, int rows, int dim) {
  extern __shared__ float s_acc[];  // [2*dim]: dw, db
  for (int i = threadIdx.x; i < 2 * dim; i += blockDim.x) s_acc[i] = 0.f;
  __syncthreads();
  const int warps = blockDim.x >> 5;
  const int lane = threadIdx.x & 31;
  for (int row = blockIdx.x * warps + (threadIdx.x >> 5); row < rows; row += gridDim.x * warps) {
    const long long base = (long long)row * dim;
    const float mu = mean[row], rs = rstd[row];
    float s_g = 0.f, s_gx = 0.f;
    for (int c = lane * 8; c < dim; c += 256) {
      float a[8], g[8], d[8];
      load8(x + base + c, a);
      load8(w + c, g);
      load8(dy + base + c, d);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float xh = (a[i] - mu) * rs;
        const float gd = g[i] * d[i];
        s_g += gd;
        s_gx += gd * xh;
        atomicAdd(&s_acc[c + i], d[i] * xh);
        atomicAdd(&s_acc[dim + c + i], d[i]);
      }
    }
    s_g = warp_sum(s_g) / (float)dim;
    s_gx = warp_sum(s_gx) / (float)dim;
    for (int c = lane * 8; c < dim; c += 256) {
      float a[8], g[8], d[8], o[8];
      load8(x + base + c, a);
      load8(w + c, g);
      load8(dy + base + c, d);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float xh = (a[i] - mu) * rs;
        o[i] = rs * (g[i] * d[i] - s_g - xh * s_gx);
      }
      store8(dx + base + c, o);
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < dim; i += blockDim.x) {
    atomicAdd(&dw[i], s_acc[i]);
    atomicAdd(&db[i], s_acc[dim + i]);
  }
}

void layernorm_bwd(const void* x, const void* w, const float* mean, const float* rstd, const void* dy, void* dx,
                   float* dw, float* db, int rows, int dim, cudaStream_t s) {
  const int warps = 8;
  int grid = (rows + warps - 1) / warps;
  if (grid > 148 * 4) grid = 148 * 4;
  layernorm_bwd_kernel<<<grid, warps * 32, 2 * dim * sizeof(float), s>>>(
      (const bf16*)x, (const bf16*)w, mean, rstd, (const bf16*)dy, (bf16*)dx, dw, db, rows, dim);
}

// ---------------------------------------------------------------------------
// RoPE
// ---------------------------------------------------------------------------
__global__ void rope_kernel(bf16* __restrict__ x, const float* __restrict__ cs, int max_pos,
                            const int* __restrict__ pos, int pos0, int seq, int tokens, int heads,
                            long long row_stride, long long head_stride, int off, int rot, bool interleaved,
                            float sign, StatusBlock* st) {
  const int half = rot >> 1;
  const long long total = (long long)tokens * heads * half;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int j = (int)(i % half);
    const long long th = i / half;
    const int h = (int)(th % heads);
    const int t = (int)(th / heads);
    int p = pos != nullptr ? pos[t] : pos0 + (t % seq);
    if (p < 0 || p >= max_pos) {
      report_error(st, STATUS_BAD_INDEX, p);
      continue;
    }
    const float c = cs[(long long)p * half + j];
    const float s = sign * cs[(long long)max_pos * half + (long long)p * half + j];
    bf16* b = x + (long long)t * row_stride + (long long)h * head_stride + off;
    const int i0 = interleaved ? 2 * j : j;
    const int i1 = interleaved ? 2 * j + 1 : j + half;
    const float a0 = __bfloat162float(b[i0]);
    const float a1 = __bfloat162float(b[i1]);
    b[i0] = __float2bfloat16(a0 * c - a1 * s);
    b[i1] = __float2bfloat16(a1 * c + a0 * s);
  }
}

void rope_apply(void* x, const float* cs, int max_pos, const int* pos, int pos0, int seq, int tokens, int heads,
                long long row_stride, long long head_stride, int off, int rot, bool interleaved, float sign,
                cudaStream_t s) {
  const long long total = (long long)tokens * heads * (rot / 2);
  long long blocks = (total + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  if (blocks < 1) blocks = 1;
  rope_kernel<<<(int)blocks, 256, 0, s>>>((bf16*)x, cs, max_pos, pos, pos0, seq > 0 ? seq : 1, tokens, heads,
                                          row_stride, head_stride, off, rot, interleaved, sign,
                                          (StatusBlock*)status_ptr());
}

// ---------------------------------------------------------------------------
// Embedding
// ---------------------------------------------------------------------------
__global__ void embedding_fwd_kernel(const int64_t* __restrict__ ids, const bf16* __restrict__ w,
                                     bf16* __restrict__ out, int tokens, int dim, int vocab, StatusBlock* st) {
  const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (t >= tokens) return;
  const int64_t id = ids[t];
  bf16* o = out + (long long)t * dim;
  if (id < 0 || id >= vocab) {
    if (lane == 0) report_error(st, STATUS_BAD_INDEX, (int)id);
    for (int c = lane * 8; c < dim; c += 256) *reinterpret_cast<uint4*>(o + c) = make_uint4(0, 0, 0, 0);
    return;
  }
  const bf16* src = w + id * (long long)dim;
  for (int c = lane * 8; c < dim; c += 256)
    *reinterpret_cast<uint4*>(o + c) = *reinterpret_cast<const uint4*>(src + c);
}

void embedding_fwd(const int64_t* ids, const void* w, void* out, int tokens, int dim, int vocab, cudaStream_t s) {
  const int warps = 8;
  embedding_fwd_kernel<<<(tokens + warps - 1) / warps, warps * 32, 0, s>>>(
      ids, (const bf16*)w, (bf16*)out, tokens, dim, vocab, (StatusBlock*)status_ptr());
}

__global__ void embedding_bwd_kernel(const int64_t* __restrict__ ids, const bf16* __restrict__ dout,
                                     float* __restrict__ dw, int tokens, int dim, int vocab) {
  const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (t >= tokens) return;
  const int64_t id = ids[t];
  if (id < 0 || id >= vocab) return;
  const bf16* d = dout + (long long)t * dim;
  float* g = dw + id * (long long)dim;
  for (int c = lane * 8; c < dim; c += 256) {
    float a[8];
    load8(d + c, a);
#pragma unroll
    for (int i = 0; i < 8; ++i) atomicAdd(&g[c + i], a[i]);
  }
}

void embedding_bwd(const int64_t* ids, const void* dout, float* dw, int tokens, int dim, int vocab,
                   cudaStream_t s) {
  const int warps = 8;
  embedding_bwd_kernel<<<(tokens + warps - 1) / warps, warps * 32, 0, s>>>(ids, (const bf16*)dout, dw, tokens,
                                                                           dim, vocab);
}

}  // namespace omni
