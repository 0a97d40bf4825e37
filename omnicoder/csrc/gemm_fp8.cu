// Block-scaled fp8 GEMM for sm_100a (tcgen05 kind::f8f6f4, e4m3 x e4m3 -> fp32).
//
//   C[m, n] = sum_kb  sx[kb][m] * sw[g][n/128][kb] * sum_{k in kb} Xq[m, k] Wq[n, k]
//
// The scaling is the 1 x 128 (activations) / 128 x 128 (weights) block scheme of
// the block-scaled fp8 training recipes: every 128-wide K block of a row of X
// and every 128 x 128 block of W has its own fp32 scale.  Because the scale
// changes at every K block, the tensor core cannot accumulate across blocks;
// instead each K block's partial product goes to one of four tensor-memory
// buffers and the epilogue warps fold it into fp32 registers with its scale
// product while the tensor core computes the next blocks into the others.
//
// Tile 128 x 128, K block 128 (four K=32 MMAs), 6-stage TMA ring of 16 KB + 16 KB,
// four partial-product buffers in tensor memory, persistent grid of one CTA per
// SM.  Roles: warp 0 lane 0 TMA producer, warp 1 lane 0 MMA issuer + TMEM owner,
// warps 2..17 epilogue (four warps per TMEM lane quadrant, 32 columns each: one
// FMA per element per K block, spread over enough warps to hide the TMEM loads).
// Dense and grouped-M (per-expert weights, row offsets of the groups on the
// device, multiples of 128).  Every wait is bounded and reports through the
// status block.
#include <cuda_fp8.h>
#include <cudaTypedefs.h>

#include <stdexcept>

#include "common.cuh"
#include "gemm_sm100.h"

namespace omni {

namespace {

using bf16 = __nv_bfloat16;

constexpr int kF8BM = 128, kF8BN = 128, kF8BK = 128;
constexpr int kF8Stages = 6;
constexpr int kF8StageA = kF8BM * kF8BK;  // 16 KB
constexpr int kF8StageB = kF8BN * kF8BK;  // 16 KB
constexpr int kF8Stage = kF8StageA + kF8StageB;
constexpr int kF8EpiWarps = 16;  // four per TMEM lane quadrant, 32 columns each
constexpr int kF8Bufs = 4;       // partial-product buffers in tensor memory (4 x 128 columns)
constexpr int kF8Threads = 64 + 32 * kF8EpiWarps;
constexpr int kF8Smem = kF8Stages * kF8Stage + 1024 + 256;
constexpr int kF8MaxGroups = 256;

// Instruction descriptor, kind::f8f6f4: D f32 [4,6) = 1; A, B e4m3 (format 0); both K-major;
// N >> 3 at [17,23); M >> 4 at [24,29).
__host__ __device__ constexpr uint32_t umma_idesc_e4m3(int M, int N) {
  return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void tc_mma_f8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

struct F8Args {
  int M, N, K, G;
  const int* offsets;
  const float* sx;
  long long ldsx;
  const float* sw;
  bf16* C;
  long long ldc;
  StatusBlock* status;
};

struct F8Tile {
  int m0, n0, g, m_limit;
};

template <bool GROUPED>
__device__ __forceinline__ int f8_tiles(const F8Args& p, const int* s_off) {
  const int nn = (p.N + kF8BN - 1) / kF8BN;
  if (GROUPED) return (s_off[p.G] / kF8BM) * nn;
  return ((p.M + kF8BM - 1) / kF8BM) * nn;
}

template <bool GROUPED>
__device__ __forceinline__ F8Tile f8_tile(const F8Args& p, int t, const int* s_off) {
  F8Tile ti;
  const int nn = (p.N + kF8BN - 1) / kF8BN;
  if (GROUPED) {
    const int mt = t / nn;
    ti.m0 = mt * kF8BM;
    ti.n0 = (t - mt * nn) * kF8BN;
    int g = 0;
    while (g + 1 < p.G && s_off[g + 1] <= ti.m0) ++g;
    ti.g = g;
    ti.m_limit = s_off[g + 1];
  } else {
    // 8 M tiles share a sweep over N so the B tiles stay in L2
    const int nm = (p.M + kF8BM - 1) / kF8BM;
    constexpr int GM = 8;
    const int grp = t / (GM * nn);
    const int first = grp * GM;
    const int gsize = min(nm - first, GM);
    const int r = t - grp * GM * nn;
    ti.m0 = (first + r % gsize) * kF8BM;
    ti.n0 = (r / gsize) * kF8BN;
    ti.g = 0;
    ti.m_limit = p.M;
  }
  return ti;
}

template <bool GROUPED>
__global__ void __launch_bounds__(kF8Threads, 1)
    fp8_gemm_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW, F8Args p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kF8Stages * kF8Stage);
  uint64_t* empty = full + kF8Stages;
  uint64_t* tfull = empty + kF8Stages;  // [kF8Bufs] partial product of one K block ready
  uint64_t* tempty = tfull + kF8Bufs;   // [kF8Bufs] read by every epilogue warp
  uint64_t* drain = tempty + kF8Bufs;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  __shared__ int s_off[kF8MaxGroups + 1];
  const int warp = warp_id(), lane = lane_id();
  if (GROUPED)
    for (int i = threadIdx.x; i <= p.G; i += kF8Threads) s_off[i] = p.offsets[i];
  if (threadIdx.x == 0) {
    for (int s = 0; s < kF8Stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < kF8Bufs; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], kF8EpiWarps);
    }
    mbar_init(drain, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kF8Bufs * kF8BN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int ntiles = f8_tiles<GROUPED>(p, s_off);
  const int nkb = p.K / kF8BK;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------ TMA producer ------------------------------
      tma_prefetch_desc(&tmX);
      tma_prefetch_desc(&tmW);
      int it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
        const F8Tile ti = f8_tile<GROUPED>(p, t, s_off);
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int s = it % kF8Stages;
          if (!mbar_wait(&empty[s], ((it / kF8Stages) & 1) ^ 1, p.status, STATUS_TIMEOUT_TMA_EMPTY)) { ok = false; break; }
          uint8_t* sa = smem + s * kF8Stage;
          mbar_arrive_expect_tx(&full[s], kF8Stage);
          tma_load_2d(sa, &tmX, &full[s], kb * kF8BK, ti.m0);
          if (GROUPED)
            tma_load_3d(sa + kF8StageA, &tmW, &full[s], kb * kF8BK, ti.n0, ti.g);
          else
            tma_load_2d(sa + kF8StageA, &tmW, &full[s], kb * kF8BK, ti.n0);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------- MMA issuer -------------------------------
      constexpr uint32_t idesc = umma_idesc_e4m3(kF8BM, kF8BN);
      int it = 0, kc = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
        for (int kb = 0; kb < nkb; ++kb, ++it, ++kc) {
          const int b = kc % kF8Bufs;
          if (!mbar_wait(&tempty[b], ((kc / kF8Bufs) & 1) ^ 1, p.status, STATUS_TIMEOUT_TMEM_EMPTY)) { ok = false; break; }
          const int s = it % kF8Stages;
          if (!mbar_wait(&full[s], (it / kF8Stages) & 1, p.status, STATUS_TIMEOUT_TMA_FULL)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + s * kF8Stage);
          const uint64_t da = umma_desc_sw128(sa, 16, 1024), db = umma_desc_sw128(sa + kF8StageA, 16, 1024);
#pragma unroll
          for (int k4 = 0; k4 < 4; ++k4)  // K = 32 bytes per MMA
            tc_mma_f8(tmem + b * kF8BN, da + ((k4 * 32) >> 4), db + ((k4 * 32) >> 4), idesc, k4 > 0 ? 1u : 0u);
          tc_commit(&empty[s]);
          tc_commit(&tfull[b]);
        }
      }
      tc_commit(drain);
      mbar_wait(drain, 0, p.status, STATUS_TIMEOUT_DRAIN);
    }
  } else {
    // ------------------- epilogue: scale, accumulate, store ---------------------
    const int q = warp & 3;
    const int h = (warp - 2) >> 2;  // columns [32 h, 32 h + 32) of the tile
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    const int nb_per_g = (p.N + 127) / 128;
    int kc = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
      const F8Tile ti = f8_tile<GROUPED>(p, t, s_off);
      const int row = ti.m0 + q * 32 + lane;
      const float* swp = p.sw + ((long long)ti.g * nb_per_g + ti.n0 / 128) * nkb;
      float acc[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) acc[j] = 0.f;
      float sxn = p.sx[row];  // kb = 0 (sx is padded to whole 128-row tiles)
      for (int kb = 0; kb < nkb; ++kb, ++kc) {
        const int b = kc % kF8Bufs;
        const float sc = sxn * __ldg(swp + kb);
        if (kb + 1 < nkb) sxn = p.sx[(long long)(kb + 1) * p.ldsx + row];
        bool got = mbar_wait(&tfull[b], (kc / kF8Bufs) & 1, p.status, STATUS_TIMEOUT_TMEM_FULL);
        got = __all_sync(0xffffffffu, got);  // tcgen05.ld is warp-collective
        if (!got) { ok = false; break; }
        tc_fence_after();
        float v[32];
        tmem_ld32(tmem + b * kF8BN + h * 32 + lane_off, v);
        tc_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[b]);
#pragma unroll
        for (int j = 0; j < 32; ++j) acc[j] = fmaf(v[j], sc, acc[j]);
      }
      if (!ok) break;
      if (row < ti.m_limit) {
        bf16* dst = p.C + (long long)row * p.ldc + ti.n0 + h * 32;
        const int ncol = min(32, p.N - (ti.n0 + h * 32));
        if (ncol == 32) {
#pragma unroll
          for (int j = 0; j < 32; j += 8) {
            uint4 w = make_uint4(pack_bf16x2(acc[j], acc[j + 1]), pack_bf16x2(acc[j + 2], acc[j + 3]),
                                 pack_bf16x2(acc[j + 4], acc[j + 5]), pack_bf16x2(acc[j + 6], acc[j + 7]));
            *reinterpret_cast<uint4*>(dst + j) = w;
          }
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (j < ncol) dst[j] = __float2bfloat16(acc[j]);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kF8Bufs * kF8BN);
  }
}

// ---- quantisers ---------------------------------------------------------------------
constexpr float kE4M3Max = 448.f;

__device__ __forceinline__ uint16_t f32x2_to_e4m3x2(float a, float b) {
  return (uint16_t)__nv_cvt_float2_to_fp8x2(make_float2(a, b), __NV_SATFINITE, __NV_E4M3);
}

// one warp per (row, 128-column block): 4 elements per lane
__global__ void fp8_quant_act_kernel(const bf16* __restrict__ x, long long ldx, int M, int K, uint8_t* __restrict__ xq,
                                     float* __restrict__ sx, long long ldsx) {
  const int kbn = K / 128;
  const long long w = blockIdx.x * (long long)(blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (w >= (long long)ldsx * kbn) return;
  const int row = (int)(w / kbn), kb = (int)(w % kbn);
  if (row >= M) {
    if (lane == 0) sx[(long long)kb * ldsx + row] = 0.f;
    return;
  }
  const bf16* src = x + (long long)row * ldx + kb * 128 + lane * 4;
  const uint2 raw = *reinterpret_cast<const uint2*>(src);
  float v[4] = {bf16_lo(raw.x), bf16_hi(raw.x), bf16_lo(raw.y), bf16_hi(raw.y)};
  float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
  amax = warp_max(amax);
  const float scale = amax > 0.f ? amax * (1.0f / kE4M3Max) : 1.f;
  const uint32_t packed = (uint32_t)f32x2_to_e4m3x2(v[0] / scale, v[1] / scale) |
                          ((uint32_t)f32x2_to_e4m3x2(v[2] / scale, v[3] / scale) << 16);
  *reinterpret_cast<uint32_t*>(xq + (long long)row * K + kb * 128 + lane * 4) = packed;
  if (lane == 0) sx[(long long)kb * ldsx + row] = scale;
}

// one CTA (256 threads) per 128 x 128 weight block: 64 elements per thread
__global__ void fp8_quant_weight_kernel(const bf16* __restrict__ w, int N, int K, uint8_t* __restrict__ wq,
                                        float* __restrict__ sw) {
  const int nbn = (N + 127) / 128, kbn = K / 128;
  const int g = blockIdx.z, nb = blockIdx.y, kb = blockIdx.x;
  const bf16* base = w + (long long)g * N * K;
  uint8_t* qbase = wq + (long long)g * N * K;
  __shared__ float red[8];
  const int tid = threadIdx.x;
  // thread -> (row r = tid / 2, half = tid % 2 covering 64 columns)
  const int r = nb * 128 + (tid >> 1), c0 = kb * 128 + (tid & 1) * 64;
  float amax = 0.f;
  if (r < N) {
    for (int c = 0; c < 64; c += 8) {
      const uint4 raw = *reinterpret_cast<const uint4*>(base + (long long)r * K + c0 + c);
      const uint32_t* u = reinterpret_cast<const uint32_t*>(&raw);
#pragma unroll
      for (int j = 0; j < 4; ++j) amax = fmaxf(amax, fmaxf(fabsf(bf16_lo(u[j])), fabsf(bf16_hi(u[j]))));
    }
  }
  amax = warp_max(amax);
  if ((tid & 31) == 0) red[tid >> 5] = amax;
  __syncthreads();
  float bmax = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) bmax = fmaxf(bmax, red[i]);
  const float scale = bmax > 0.f ? bmax * (1.0f / kE4M3Max) : 1.f;
  if (r < N) {
    for (int c = 0; c < 64; c += 8) {
      const uint4 raw = *reinterpret_cast<const uint4*>(base + (long long)r * K + c0 + c);
      const uint32_t* u = reinterpret_cast<const uint32_t*>(&raw);
      uint2 o;
      o.x = (uint32_t)f32x2_to_e4m3x2(bf16_lo(u[0]) / scale, bf16_hi(u[0]) / scale) |
            ((uint32_t)f32x2_to_e4m3x2(bf16_lo(u[1]) / scale, bf16_hi(u[1]) / scale) << 16);
      o.y = (uint32_t)f32x2_to_e4m3x2(bf16_lo(u[2]) / scale, bf16_hi(u[2]) / scale) |
            ((uint32_t)f32x2_to_e4m3x2(bf16_lo(u[3]) / scale, bf16_hi(u[3]) / scale) << 16);
      *reinterpret_cast<uint2*>(qbase + (long long)r * K + c0 + c) = o;
    }
  }
  if (tid == 0) sw[((long long)g * nbn + nb) * kbn + kb] = scale;
}

}  // namespace

void fp8_gemm_launch(const Fp8GemmDesc& d, cudaStream_t stream) {
  if (d.K % kF8BK != 0 || d.K <= 0) throw std::runtime_error("fp8 gemm: K must be a positive multiple of 128");
  if (d.N <= 0 || d.M <= 0) return;
  const bool grouped = d.offsets != nullptr;
  if (grouped && d.G > kF8MaxGroups) throw std::runtime_error("fp8 gemm: too many groups");
  CUtensorMap tmX, tmW;
  {
    uint64_t dims[2] = {(uint64_t)d.K, (uint64_t)d.M};
    uint64_t str[1] = {(uint64_t)d.ldx};
    uint32_t box[2] = {kF8BK, kF8BM};
    tmX = make_tmap_u8_sw128(d.X, 2, dims, str, box);
  }
  if (grouped) {
    uint64_t dims[3] = {(uint64_t)d.K, (uint64_t)d.N, (uint64_t)d.G};
    uint64_t str[2] = {(uint64_t)d.ldw, (uint64_t)d.w_group_stride};
    uint32_t box[3] = {kF8BK, kF8BN, 1};
    tmW = make_tmap_u8_sw128(d.W, 3, dims, str, box);
  } else {
    uint64_t dims[2] = {(uint64_t)d.K, (uint64_t)d.N};
    uint64_t str[1] = {(uint64_t)d.ldw};
    uint32_t box[2] = {kF8BK, kF8BN};
    tmW = make_tmap_u8_sw128(d.W, 2, dims, str, box);
  }
  F8Args p;
  p.M = d.M;
  p.N = d.N;
  p.K = d.K;
  p.G = grouped ? d.G : 1;
  p.offsets = d.offsets;
  p.sx = d.sx;
  p.ldsx = d.ldsx;
  p.sw = d.sw;
  p.C = reinterpret_cast<bf16*>(d.C);
  p.ldc = d.ldc;
  p.status = reinterpret_cast<StatusBlock*>(d.status);
  const int nn = (d.N + kF8BN - 1) / kF8BN;
  int tiles = grouped ? (d.max_rows_hint > 0 ? d.max_rows_hint / kF8BM : (d.M + kF8BM - 1) / kF8BM) * nn
                      : ((d.M + kF8BM - 1) / kF8BM) * nn;
  const int grid = std::max(1, std::min(tiles, num_sms()));
  if (grouped) {
    auto kern = fp8_gemm_kernel<true>;
    ensure_smem_attr(reinterpret_cast<const void*>(kern), kF8Smem);
    kern<<<grid, kF8Threads, kF8Smem, stream>>>(tmX, tmW, p);
  } else {
    auto kern = fp8_gemm_kernel<false>;
    ensure_smem_attr(reinterpret_cast<const void*>(kern), kF8Smem);
    kern<<<grid, kF8Threads, kF8Smem, stream>>>(tmX, tmW, p);
  }
}

void fp8_quant_act(const void* x, long long ldx, int M, int K, void* xq, float* sx, long long ldsx, cudaStream_t s) {
  if (K % 128 != 0) throw std::runtime_error("fp8 quant: K must be a multiple of 128");
  const long long warps = ldsx * (K / 128);
  if (warps == 0) return;
  fp8_quant_act_kernel<<<(unsigned)((warps + 7) / 8), 256, 0, s>>>((const bf16*)x, ldx, M, K, (uint8_t*)xq, sx, ldsx);
}

void fp8_quant_weight(const void* w, int G, int N, int K, void* wq, float* sw, cudaStream_t s) {
  if (K % 128 != 0) throw std::runtime_error("fp8 quant: K must be a multiple of 128");
  const dim3 grid(K / 128, (N + 127) / 128, G);
  fp8_quant_weight_kernel<<<grid, 256, 0, s>>>((const bf16*)w, N, K, (uint8_t*)wq, sw);
}

}  // namespace omni
