// Weight-only int4 linear layer for sm_100a.
//
// Weights: per output row n, K values quantised to unsigned nibbles q in
// [0, 15] with value (q - offset) * scale[n]; two per byte, element 2i in the
// low nibble, 2i+1 in the high nibble; rows padded to a multiple of 64 elements
// (the reference packer's format, src/omnicoder/modeling/quant/int4_linear.py:20-80;
// its packer stores q + 7, its dequantiser subtracts 7, its kernel registry 8
// (int4_kernels.py:33-60): the offset is an argument here).
//
// int4_gemv: y[m, n] = scale[n] * (sum_k x[m,k] q[n,k] - offset * sum_k x[m,k])
//   for small M (decode: the number of sequences in flight).  Weight bytes are
//   read once, 16 bytes per lane per row; each warp owns two output rows, each
//   CTA eight warps; the activation rows come from L1/L2 (they are shared by all
//   rows).  Memory-bound by design: N*K/2 bytes per call.
// int4_dequant: unpacks to bf16 for large M, where the tcgen05 GEMM takes over.
#include "common.cuh"
#include "kernels.h"

namespace omni {

using bf16 = __nv_bfloat16;

namespace {

constexpr int kRowsPerWarp = 2;
constexpr int kWarps = 8;

template <int MT>
__global__ void __launch_bounds__(kWarps * 32) int4_gemv_kernel(const bf16* __restrict__ x, const uint8_t* __restrict__ w,
                                                               const float* __restrict__ scale, bf16* __restrict__ y,
                                                               int M, int N, int K, int ldw, float offset) {
  const int lane = threadIdx.x & 31;
  const int n0 = (blockIdx.x * kWarps + (threadIdx.x >> 5)) * kRowsPerWarp;
  if (n0 >= N) return;
  float acc[kRowsPerWarp][MT];
  float xs[MT];
#pragma unroll
  for (int m = 0; m < MT; ++m) {
    xs[m] = 0.f;
#pragma unroll
    for (int r = 0; r < kRowsPerWarp; ++r) acc[r][m] = 0.f;
  }
  // each lane: 32 consecutive k per step (16 weight bytes per row); warp: 1024 k per step
  for (int k0 = lane * 32; k0 < K; k0 += 32 * 32) {
    uint4 wv[kRowsPerWarp];
#pragma unroll
    for (int r = 0; r < kRowsPerWarp; ++r) {
      const int n = n0 + r;
      wv[r] = n < N ? *reinterpret_cast<const uint4*>(w + (long long)n * ldw + k0 / 2) : make_uint4(0, 0, 0, 0);
    }
    const int kvalid = min(32, K - k0);
#pragma unroll
    for (int sub = 0; sub < 4; ++sub) {
      if (sub * 8 >= kvalid) break;
      float xv[MT][8];
#pragma unroll
      for (int m = 0; m < MT; ++m) {
        if (m < M) {
          const uint4 v = *reinterpret_cast<const uint4*>(x + (long long)m * K + k0 + sub * 8);
          const uint32_t* q = reinterpret_cast<const uint32_t*>(&v);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            xv[m][2 * j] = bf16_lo(q[j]);
            xv[m][2 * j + 1] = bf16_hi(q[j]);
          }
        } else {
#pragma unroll
          for (int j = 0; j < 8; ++j) xv[m][j] = 0.f;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) xs[m] += xv[m][j];
      }
#pragma unroll
      for (int r = 0; r < kRowsPerWarp; ++r) {
        const uint32_t word = reinterpret_cast<const uint32_t*>(&wv[r])[sub];  // 8 nibbles
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float qv = (float)((word >> (4 * j)) & 0xFu);
#pragma unroll
          for (int m = 0; m < MT; ++m) acc[r][m] += qv * xv[m][j];
        }
      }
    }
  }
  // sum(x) is identical for every row: reduce once
#pragma unroll
  for (int m = 0; m < MT; ++m) xs[m] = warp_sum(xs[m]);
#pragma unroll
  for (int r = 0; r < kRowsPerWarp; ++r) {
#pragma unroll
    for (int m = 0; m < MT; ++m) acc[r][m] = warp_sum(acc[r][m]);
  }
  if (lane == 0) {
#pragma unroll
    for (int r = 0; r < kRowsPerWarp; ++r) {
      const int n = n0 + r;
      if (n >= N) continue;
      const float s = scale[n];
#pragma unroll
      for (int m = 0; m < MT; ++m)
        if (m < M) y[(long long)m * N + n] = __float2bfloat16(s * (acc[r][m] - offset * xs[m]));
    }
  }
}

__global__ void int4_dequant_kernel(const uint8_t* __restrict__ w, const float* __restrict__ scale,
                                    bf16* __restrict__ out, int N, int K, int ldw, float offset) {
  const long long total = (long long)N * (K / 8);
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const int n = (int)(i / (K / 8));
    const int c = (int)(i % (K / 8));
    const uint32_t word = *reinterpret_cast<const uint32_t*>(w + (long long)n * ldw + c * 4);
    const float s = scale[n];
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = ((float)((word >> (4 * j)) & 0xFu) - offset) * s;
    uint4 o;
    o.x = pack_bf16x2(v[0], v[1]);
    o.y = pack_bf16x2(v[2], v[3]);
    o.z = pack_bf16x2(v[4], v[5]);
    o.w = pack_bf16x2(v[6], v[7]);
    *reinterpret_cast<uint4*>(out + (long long)n * K + c * 8) = o;
  }
}

}  // namespace

void int4_gemv(const void* x, const uint8_t* w, const float* scale, void* y, int M, int N, int K, int ldw,
               float offset, cudaStream_t s) {
  const int grid = (N + kWarps * kRowsPerWarp - 1) / (kWarps * kRowsPerWarp);
  const bf16* xb = (const bf16*)x;
  bf16* yb = (bf16*)y;
  if (M <= 1)
    int4_gemv_kernel<1><<<grid, kWarps * 32, 0, s>>>(xb, w, scale, yb, M, N, K, ldw, offset);
  else if (M <= 2)
    int4_gemv_kernel<2><<<grid, kWarps * 32, 0, s>>>(xb, w, scale, yb, M, N, K, ldw, offset);
  else if (M <= 4)
    int4_gemv_kernel<4><<<grid, kWarps * 32, 0, s>>>(xb, w, scale, yb, M, N, K, ldw, offset);
  else
    int4_gemv_kernel<8><<<grid, kWarps * 32, 0, s>>>(xb, w, scale, yb, M, N, K, ldw, offset);
}

void int4_dequant(const uint8_t* w, const float* scale, void* out, int N, int K, int ldw, float offset,
                  cudaStream_t s) {
  const long long total = (long long)N * (K / 8);
  const int grid = (int)std::min<long long>((total + 255) / 256, 148ll * 32);
  int4_dequant_kernel<<<grid, 256, 0, s>>>(w, scale, (bf16*)out, N, K, ldw, offset);
}

}  // namespace omni
