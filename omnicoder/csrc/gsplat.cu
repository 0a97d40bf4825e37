// Gaussian splatting forward (sm_100a): every (Gaussian, footprint tap) pair
// adds (alpha * colour, alpha) and alpha * depth into per-pixel accumulators
// with fire-and-forget float reductions (atomicAdd with the result unused); a
// second kernel divides by the accumulated alpha.
//
// Per Gaussian (already projected on the host side): centre (u, v) in pixels,
// footprint scales (sx, sy) in pixels, opacity, colour, depth.  Tap (ox, oy),
// ox, oy in [-k/2, k/2]: pixel (rint(u + ox*sx), rint(v + oy*sy)), weight
// exp(-0.5 ((ox/sx)^2 + (oy/sy)^2)), skipped when outside the image -- the
// formulation of the reference renderer (src/omnicoder/modeling/gaussian/
// renderer.py:12-235), whose sum is order independent, so no depth sort is
// needed for the accumulation.
//
// Layout and mapping: one warp per Gaussian (its parameters are read once per
// lane from the same addresses, a broadcast), the lanes stride over the k*k
// taps, so the index arithmetic per tap is one 32-bit division by k.  Colour
// and alpha accumulate interleaved as one float4 per pixel ([B, H, W, 4]) and
// are added with one 16-byte vector reduction per tap; depth has its own
// [B, H, W] plane.  Two reductions per tap instead of five scalar ones into
// five planes.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace omni {

namespace {

constexpr int kSplatThreads = 256;

__global__ void __launch_bounds__(kSplatThreads)
gsplat_accum_kernel(const float* __restrict__ u, const float* __restrict__ v, const float* __restrict__ sx,
                    const float* __restrict__ sy, const float* __restrict__ opa, const float* __restrict__ rgb,
                    const float* __restrict__ z, float4* __restrict__ acc4, float* __restrict__ accd, int B, int N,
                    int H, int W, int k, bool with_depth) {
  const int lane = threadIdx.x & 31;
  const long long total = (long long)B * N;
  const long long warps = ((long long)gridDim.x * blockDim.x) >> 5;
  const int k2 = k * k, half = k / 2;
  const long long plane = (long long)H * W;
  for (long long g = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5; g < total; g += warps) {
    const float ug = u[g], vg = v[g], sxr = sx[g], syr = sy[g], op = opa[g];
    const float sxg = fmaxf(sxr, 1e-6f), syg = fmaxf(syr, 1e-6f);
    const float cr = rgb[g * 3 + 0], cg = rgb[g * 3 + 1], cb = rgb[g * 3 + 2];
    const float zg = with_depth ? z[g] : 0.f;
    const long long img = (g / N) * plane;
    for (int t = lane; t < k2; t += 32) {
      const int row = t / k;
      const int oy = row - half, ox = t - row * k - half;
      const float px = rintf(ug + (float)ox * sxr);
      const float py = rintf(vg + (float)oy * syr);
      if (!(px >= 0.f && px <= (float)(W - 1) && py >= 0.f && py <= (float)(H - 1))) continue;
      const float gx = (float)ox / sxg, gy = (float)oy / syg;
      const float a = op * __expf(-0.5f * (gx * gx + gy * gy));
      const long long p = img + (long long)py * W + (long long)px;
      atomicAdd(acc4 + p, make_float4(a * cr, a * cg, a * cb, a));
      if (with_depth) atomicAdd(accd + p, a * zg);
    }
  }
}

__global__ void gsplat_norm_kernel(const float4* __restrict__ acc4, const float* __restrict__ accd,
                                   float* __restrict__ rgb, float* __restrict__ depth, int B, int H, int W) {
  const long long plane = (long long)H * W;
  const long long total = (long long)B * plane;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long b = i / plane, p = i - b * plane;
    const float4 a = acc4[i];
    const float inv = 1.f / fmaxf(a.w, 1e-6f);
    rgb[b * 3 * plane + p] = a.x * inv;
    rgb[b * 3 * plane + plane + p] = a.y * inv;
    rgb[b * 3 * plane + 2 * plane + p] = a.z * inv;
    if (depth != nullptr) depth[i] = accd[i] * inv;
  }
}

}  // namespace

void gsplat_forward(const float* u, const float* v, const float* sx, const float* sy, const float* opa,
                    const float* rgb, const float* z, float* acc, float* out_rgb, float* out_depth, int B, int N,
                    int H, int W, int k, cudaStream_t s) {
  const long long pix = (long long)B * H * W;
  cudaMemsetAsync(acc, 0, sizeof(float) * 5 * (size_t)pix, s);
  float4* acc4 = reinterpret_cast<float4*>(acc);   // [B, H, W, 4], then the [B, H, W] depth plane
  float* accd = acc + 4 * pix;
  const long long gaussians = (long long)B * N;
  if (gaussians > 0 && k > 0) {
    const long long blocks = (gaussians + kSplatThreads / 32 - 1) / (kSplatThreads / 32);
    const int grid = (int)std::min<long long>(blocks, 148ll * 16);
    gsplat_accum_kernel<<<grid, kSplatThreads, 0, s>>>(u, v, sx, sy, opa, rgb, z, acc4, accd, B, N, H, W, k,
                                                       z != nullptr);
  }
  gsplat_norm_kernel<<<(int)std::min<long long>((pix + 255) / 256, 148ll * 32), 256, 0, s>>>(acc4, accd, out_rgb,
                                                                                              out_depth, B, H, W);
}

}  // namespace omni
