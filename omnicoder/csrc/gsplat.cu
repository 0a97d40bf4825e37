// Gaussian splatting forward (sm_100a): every (Gaussian, footprint tap) pair
// adds alpha * colour, alpha and alpha * depth into per-pixel accumulators
// with fire-and-forget float reductions (red.global.add via atomicAdd with the
// result unused); a second kernel divides by the accumulated alpha.
//
// Per Gaussian (already projected on the host side): centre (u, v) in pixels,
// footprint scales (sx, sy) in pixels, opacity, colour, depth.  Tap (ox, oy),
// ox, oy in [-k/2, k/2]: pixel (rint(u + ox*sx), rint(v + oy*sy)), weight
// exp(-0.5 ((ox/sx)^2 + (oy/sy)^2)), skipped when outside the image -- the
// formulation of the reference renderer (src/omnicoder/modeling/gaussian/
// renderer.py:12-235), whose sum is order independent, so no depth sort is
// needed for the accumulation.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace omni {

namespace {

__global__ void gsplat_accum_kernel(const float* __restrict__ u, const float* __restrict__ v,
                                    const float* __restrict__ sx, const float* __restrict__ sy,
                                    const float* __restrict__ opa, const float* __restrict__ rgb,
                                    const float* __restrict__ z, float* __restrict__ acc, int B, int N, int H, int W,
                                    int k, bool with_depth) {
  const long long k2 = (long long)k * k;
  const long long total = (long long)B * N * k2;
  const int half = k / 2;
  const long long plane = (long long)H * W;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long g = i / k2;  // b * N + n
    const int tap = (int)(i - g * k2);
    const int oy = tap / k - half, ox = tap % k - half;
    const float sxg = fmaxf(sx[g], 1e-6f), syg = fmaxf(sy[g], 1e-6f);
    const float px = rintf(u[g] + (float)ox * sx[g]);
    const float py = rintf(v[g] + (float)oy * sy[g]);
    if (!(px >= 0.f && px <= (float)(W - 1) && py >= 0.f && py <= (float)(H - 1))) continue;
    const float gx = (float)ox / sxg, gy = (float)oy / syg;
    const float a = opa[g] * __expf(-0.5f * (gx * gx + gy * gy));
    const int b = (int)(g / N);
    float* base = acc + (long long)b * 5 * plane + (long long)py * W + (long long)px;
    atomicAdd(base + 0 * plane, a * rgb[g * 3 + 0]);
    atomicAdd(base + 1 * plane, a * rgb[g * 3 + 1]);
    atomicAdd(base + 2 * plane, a * rgb[g * 3 + 2]);
    atomicAdd(base + 3 * plane, a);
    if (with_depth) atomicAdd(base + 4 * plane, a * z[g]);
  }
}

__global__ void gsplat_norm_kernel(const float* __restrict__ acc, float* __restrict__ rgb, float* __restrict__ depth,
                                   int B, int H, int W) {
  const long long plane = (long long)H * W;
  const long long total = (long long)B * plane;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long b = i / plane, p = i - b * plane;
    const float* a = acc + b * 5 * plane + p;
    const float inv = 1.f / fmaxf(a[3 * plane], 1e-6f);
    rgb[b * 3 * plane + p] = a[0] * inv;
    rgb[b * 3 * plane + plane + p] = a[plane] * inv;
    rgb[b * 3 * plane + 2 * plane + p] = a[2 * plane] * inv;
    if (depth != nullptr) depth[b * plane + p] = a[4 * plane] * inv;
  }
}

}  // namespace

void gsplat_forward(const float* u, const float* v, const float* sx, const float* sy, const float* opa,
                    const float* rgb, const float* z, float* acc, float* out_rgb, float* out_depth, int B, int N,
                    int H, int W, int k, cudaStream_t s) {
  cudaMemsetAsync(acc, 0, sizeof(float) * 5 * (size_t)B * H * W, s);
  const long long total = (long long)B * N * k * k;
  if (total > 0) {
    const int grid = (int)std::min<long long>((total + 255) / 256, 148ll * 64);
    gsplat_accum_kernel<<<grid, 256, 0, s>>>(u, v, sx, sy, opa, rgb, z, acc, B, N, H, W, k, z != nullptr);
  }
  const long long pix = (long long)B * H * W;
  gsplat_norm_kernel<<<(int)std::min<long long>((pix + 255) / 256, 148ll * 32), 256, 0, s>>>(acc, out_rgb, out_depth,
                                                                                              B, H, W);
}

}  // namespace omni
