// KV-cache append (sm_100a): new keys / values / MLA latents of a decode or
// prefill step written into their cache rows in one launch, quantised on the
// way for int8 caches.
//
//   src    [B, T, G, D] bf16      (G groups per row: kv heads, or 1 for a latent)
//   dst    [B, L, G, D] bf16 / int8 with row = row_offset + pos[b, t]
//   scale  [B, L, G] fp32         (int8 only): q = rint(x / s), s = max|x| * (1/127)
//                                  (max clamped to 1e-8), q clamped to [-127, 127]
// One warp per (b, t, g); the group's max comes from a warp reduction.  This is
// the quantiser of omnicoder.inference.kv_cache.quantize_int8 in one kernel
// instead of the seven element-wise launches plus two index_put scatters of the
// PyTorch form.
#include "common.cuh"
#include "kernels.h"

namespace omni {

using bf16 = __nv_bfloat16;

namespace {

constexpr int kKvMaxPerLane = 32;  // D <= 1024

template <bool I8>
__global__ void kv_write_kernel(const bf16* __restrict__ src, const long long* __restrict__ pos, void* dst,
                                float* __restrict__ scale, int B, int T, int G, int D, long long d_b, long long d_l,
                                long long s_b, long long s_l, int row_offset, int L) {
  const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
  const long long item = (long long)blockIdx.x * warps + (threadIdx.x >> 5);
  if (item >= (long long)B * T * G) return;
  const int g = (int)(item % G);
  const long long bt = item / G;
  const int b = (int)(bt / T);
  const long long row = pos[bt] + row_offset;
  if (row < 0 || row >= L) return;
  const bf16* s = src + item * D;
  if (!I8) {
    bf16* o = reinterpret_cast<bf16*>(dst) + b * d_b + row * d_l + (long long)g * D;
    for (int c = lane * 8; c < D; c += 256) *reinterpret_cast<uint4*>(o + c) = *reinterpret_cast<const uint4*>(s + c);
    return;
  }
  float v[kKvMaxPerLane];
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < kKvMaxPerLane; ++i) {
    const int c = lane + 32 * i;
    v[i] = c < D ? __bfloat162float(s[c]) : 0.f;
    amax = fmaxf(amax, fabsf(v[i]));
  }
  amax = warp_max(amax);
  const float sc = fmaxf(amax, 1e-8f) * (1.0f / 127.0f);  // the scale PyTorch computes for amax / 127.0
  int8_t* o = reinterpret_cast<int8_t*>(dst) + b * d_b + row * d_l + (long long)g * D;
#pragma unroll
  for (int i = 0; i < kKvMaxPerLane; ++i) {
    const int c = lane + 32 * i;
    if (c < D) o[c] = (int8_t)fminf(fmaxf(rintf(v[i] / sc), -127.f), 127.f);
  }
  if (lane == 0) scale[b * s_b + row * s_l + g] = sc;
}

}  // namespace

void kv_cache_write(const void* src, const long long* pos, void* dst, float* scale, bool int8, int B, int T, int G,
                    int D, long long d_b, long long d_l, long long s_b, long long s_l, int row_offset, int L,
                    cudaStream_t s) {
  const long long items = (long long)B * T * G;
  if (items == 0) return;
  const int warps = 8;
  const unsigned blocks = (unsigned)((items + warps - 1) / warps);
  if (int8)
    kv_write_kernel<true><<<blocks, warps * 32, 0, s>>>((const bf16*)src, pos, dst, scale, B, T, G, D, d_b, d_l, s_b,
                                                        s_l, row_offset, L);
  else
    kv_write_kernel<false><<<blocks, warps * 32, 0, s>>>((const bf16*)src, pos, dst, scale, B, T, G, D, d_b, d_l, s_b,
                                                         s_l, row_offset, L);
}

}  // namespace omni
