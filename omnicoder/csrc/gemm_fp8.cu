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
  long long ldsw;  // > 0: per-row B scales sw[kb][n] (row stride ldsw) instead of 128 x 128 blocks
  bf16* C;
  long long ldc;
  StatusBlock* status;
  // SwiGLU + requantisation epilogue (block-scaled MMA kernel): C receives the gate|up
  // pre-activation, act (optional) silu(g) * u in bf16, actq / act_scale the same product
  // quantised per 1 x 128 block (power-of-two scales) for the next fp8 GEMM
  int swiglu_q;
  bf16* act;
  long long ld_act;
  uint8_t* actq;
  long long ld_actq;
  float* act_scale;
  long long ld_as;
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

constexpr float kE4M3Max = 448.f;

// max|block| / 448, rounded up to a power of two when pow2 (an exact UE8M0 exponent; the
// division by it is then exact); an all-zero block gets scale 1.
__device__ __forceinline__ float block_scale(float amax, bool pow2) {
  if (!(amax > 0.f)) return 1.f;
  const float s = amax * (1.0f / kE4M3Max);
  if (!pow2) return s;
  const uint32_t bits = __float_as_uint(s);
  uint32_t e = ((bits >> 23) & 0xffu) + ((bits & 0x7fffffu) != 0u);
  e = max(e, 1u);
  return __uint_as_float(e << 23);
}

__device__ __forceinline__ uint16_t f32x2_to_e4m3x2(float a, float b) {
  return (uint16_t)__nv_cvt_float2_to_fp8x2(make_float2(a, b), __NV_SATFINITE, __NV_E4M3);
}

// ---- block-scaled MMA variant (power-of-two scales) ----------------------------------
// When every scale is a power of two (the quantisers' default), the scale of a K block is
// an 8-bit exponent (UE8M0) and the tensor core applies it itself: tcgen05.mma
// kind::mxf8f6f4.block_scale.scale_vec::1X multiplies each 32-wide K slice of a row of A
// (column of B) by its scale factor read from tensor memory, so the product accumulates
// across all K blocks in the tensor-memory accumulator and the epilogue only converts.
// The 1 x 128 / 128 x 128 scheme maps onto it by repeating each scale over the four
// 32-wide slices of its 128 block (and over the 128 rows of a weight block).
//
// Tile 128 x 256, K block 128 (four K = 32 MMAs), 4-stage TMA ring of 16 KB + 32 KB.
// Tensor memory (512 columns): accumulator [0, 256); per stage s a scale-factor slot for A
// at 256 + 16 s (4 columns) and for B at 320 + 16 s (8 columns).  Scale-factor layout (the
// one a 32-lane x 128-bit copy replicated into the four lane quadrants produces): lane
// 32 q + r, column j, byte b holds the scale of row 32 j + r (A: M row; B: N row, columns
// 4..7 for rows 128..255) for the 32-wide K slice b; the same in every quadrant q.
// Roles: warp 0 TMA producer, warp 1 MMA issuer + tensor-memory owner, warps 2..5 write the
// scale factors of each stage (one per lane quadrant), warps 6..21 epilogue (quadrant
// warp % 4, 64 columns each).  The accumulator is released as soon as the epilogue has
// loaded it, so the next tile's MMAs overlap the conversion and stores.
constexpr int kMxBM = 128, kMxBN = 256, kMxBK = 128;
constexpr int kMxStages = 4;
constexpr int kMxStageA = kMxBM * kMxBK;  // 16 KB
constexpr int kMxStageB = kMxBN * kMxBK;  // 32 KB
constexpr int kMxStage = kMxStageA + kMxStageB;
constexpr int kMxSfWarps = 4, kMxEpiWarps = 16;
constexpr int kMxThreads = 64 + 32 * (kMxSfWarps + kMxEpiWarps);
constexpr int kMxSmem = kMxStages * kMxStage + 1024 + 256;
constexpr int kMxSfaCol = 256, kMxSfbCol = 320;

// Instruction descriptor, kind::mxf8f6f4 block-scaled: B scale-factor byte [4,6); A, B e4m3
// (format 0) K-major; N >> 3 at [17,23); scale type UE8M0 at bit 23; M >> 4 at [24,29);
// A scale-factor byte [29,31).
__host__ __device__ constexpr uint32_t umma_idesc_mxf8(int M, int N, int sf_id) {
  return ((uint32_t)sf_id << 4) | ((uint32_t)(N >> 3) << 17) | (1u << 23) | ((uint32_t)(M >> 4) << 24) |
         ((uint32_t)sf_id << 29);
}

__device__ __forceinline__ void tc_mma_mxf8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                            uint32_t tmem_sfa, uint32_t tmem_sfb, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %6, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale.scale_vec::1X [%0], %1, %2, %3, [%4], [%5], p;\n\t}" ::"r"(
          tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(tmem_sfa), "r"(tmem_sfb), "r"(accumulate)
      : "memory");
}

// fp32 power of two -> its UE8M0 byte repeated in the four bytes of a word
__device__ __forceinline__ uint32_t ue8m0_x4(float s) { return ((__float_as_uint(s) >> 23) & 0xffu) * 0x01010101u; }

template <bool GROUPED>
__device__ __forceinline__ int mx_tiles(const F8Args& p, const int* s_off) {
  const int nn = (p.N + kMxBN - 1) / kMxBN;
  if (GROUPED) return (s_off[p.G] / kMxBM) * nn;
  return ((p.M + kMxBM - 1) / kMxBM) * nn;
}

template <bool GROUPED>
__device__ __forceinline__ F8Tile mx_tile(const F8Args& p, int t, const int* s_off) {
  F8Tile ti;
  const int nn = (p.N + kMxBN - 1) / kMxBN;
  if (GROUPED) {
    const int mt = t / nn;
    ti.m0 = mt * kMxBM;
    ti.n0 = (t - mt * nn) * kMxBN;
    int g = 0;
    while (g + 1 < p.G && s_off[g + 1] <= ti.m0) ++g;
    ti.g = g;
    ti.m_limit = s_off[g + 1];
  } else {
    const int nm = (p.M + kMxBM - 1) / kMxBM;
    constexpr int GM = 8;
    const int grp = t / (GM * nn);
    const int first = grp * GM;
    const int gsize = min(nm - first, GM);
    const int r = t - grp * GM * nn;
    ti.m0 = (first + r % gsize) * kMxBM;
    ti.n0 = (r / gsize) * kMxBN;
    ti.g = 0;
    ti.m_limit = p.M;
  }
  return ti;
}

// named barriers over the epilogue warps only: 1 plain, 2 with an AND of a predicate (so that
// a wait that gave up in one warp makes every epilogue warp leave the loop together)
__device__ __forceinline__ void mx_epi_bar() { asm volatile("bar.sync 1, %0;" ::"n"(32 * kMxEpiWarps) : "memory"); }
__device__ __forceinline__ bool mx_epi_all(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, 2, %2, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)v), "n"(32 * kMxEpiWarps)
      : "memory");
  return r != 0;
}

template <bool GROUPED, bool SWIGLU>
__global__ void __launch_bounds__(kMxThreads, 1)
    fp8mx_gemm_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW, F8Args p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kMxStages * kMxStage);
  uint64_t* empty = full + kMxStages;
  uint64_t* sf_full = empty + kMxStages;   // scale factors of the stage in tensor memory
  uint64_t* acc_full = sf_full + kMxStages;
  uint64_t* acc_empty = acc_full + 1;
  uint64_t* drain = acc_empty + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  __shared__ int s_off[kF8MaxGroups + 1];
  __shared__ float s_amax[4 * 128];  // SwiGLU epilogue: per-row partial amax of each 32-column act slice
  const int warp = warp_id(), lane = lane_id();
  if (GROUPED)
    for (int i = threadIdx.x; i <= p.G; i += kMxThreads) s_off[i] = p.offsets[i];
  if (threadIdx.x == 0) {
    for (int s = 0; s < kMxStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      mbar_init(&sf_full[s], kMxSfWarps);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, kMxEpiWarps);
    mbar_init(drain, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int ntiles = mx_tiles<GROUPED>(p, s_off);
  const int nkb = p.K / kMxBK;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------ TMA producer ------------------------------
      tma_prefetch_desc(&tmX);
      tma_prefetch_desc(&tmW);
      int it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
        const F8Tile ti = mx_tile<GROUPED>(p, t, s_off);
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int s = it % kMxStages;
          if (!mbar_wait(&empty[s], ((it / kMxStages) & 1) ^ 1, p.status, STATUS_TIMEOUT_TMA_EMPTY)) { ok = false; break; }
          uint8_t* sa = smem + s * kMxStage;
          mbar_arrive_expect_tx(&full[s], kMxStage);
          tma_load_2d(sa, &tmX, &full[s], kb * kMxBK, ti.m0);
          if (GROUPED)
            tma_load_3d(sa + kMxStageA, &tmW, &full[s], kb * kMxBK, ti.n0, ti.g);
          else
            tma_load_2d(sa + kMxStageA, &tmW, &full[s], kb * kMxBK, ti.n0);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------- MMA issuer -------------------------------
      int it = 0, tc = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x, ++tc) {
        if (!mbar_wait(acc_empty, (tc & 1) ^ 1, p.status, STATUS_TIMEOUT_TMEM_EMPTY)) { ok = false; break; }
        tc_fence_after();
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int s = it % kMxStages;
          const uint32_t ph = (it / kMxStages) & 1;
          if (!mbar_wait(&full[s], ph, p.status, STATUS_TIMEOUT_TMA_FULL) ||
              !mbar_wait(&sf_full[s], ph, p.status, STATUS_TIMEOUT_TMA_FULL)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + s * kMxStage);
          const uint64_t da = umma_desc_sw128(sa, 16, 1024), db = umma_desc_sw128(sa + kMxStageA, 16, 1024);
#pragma unroll
          for (int k4 = 0; k4 < 4; ++k4)  // K = 32 bytes per MMA, scale-factor byte k4
            tc_mma_mxf8(tmem, da + ((k4 * 32) >> 4), db + ((k4 * 32) >> 4), umma_idesc_mxf8(kMxBM, kMxBN, k4),
                        tmem + kMxSfaCol + 16 * s, tmem + kMxSfbCol + 16 * s, (kb | k4) ? 1u : 0u);
          tc_commit(&empty[s]);
        }
        if (!ok) break;
        tc_commit(acc_full);
      }
      tc_commit(drain);
      mbar_wait(drain, 0, p.status, STATUS_TIMEOUT_DRAIN);
    }
  } else if (warp < 2 + kMxSfWarps) {
    // ------------------ scale factors of each stage -> tensor memory ------------------
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    const int nb_per_g = (p.N + 127) / 128;
    int it = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
      const F8Tile ti = mx_tile<GROUPED>(p, t, s_off);
      const float* swp = p.sw + (long long)ti.g * nb_per_g * nkb;
      const int nb0 = ti.n0 / 128, nb1 = min(nb0 + 1, nb_per_g - 1);
      for (int kb = 0; kb < nkb; ++kb, ++it) {
        const int s = it % kMxStages;
        uint32_t a[16], b[16];
        const float* sxk = p.sx + (long long)kb * p.ldsx + ti.m0 + lane;
#pragma unroll
        for (int j = 0; j < 4; ++j) a[j] = ue8m0_x4(__ldg(sxk + 32 * j));
        if (p.ldsw > 0) {
          // per-row B scales (both operands quantised per row and 128-wide K block)
          const float* swk = p.sw + (long long)kb * p.ldsw + ti.n0 + lane;
#pragma unroll
          for (int j = 0; j < 8; ++j) b[j] = ue8m0_x4(__ldg(swk + 32 * j));
        } else {
          const uint32_t w0 = ue8m0_x4(__ldg(swp + (long long)nb0 * nkb + kb));
          const uint32_t w1 = ue8m0_x4(__ldg(swp + (long long)nb1 * nkb + kb));
#pragma unroll
          for (int j = 0; j < 8; ++j) b[j] = j < 4 ? w0 : w1;
        }
#pragma unroll
        for (int j = 4; j < 16; ++j) a[j] = 0u;
#pragma unroll
        for (int j = 8; j < 16; ++j) b[j] = 0u;
        bool got = mbar_wait(&empty[s], ((it / kMxStages) & 1) ^ 1, p.status, STATUS_TIMEOUT_TMA_EMPTY);
        got = __all_sync(0xffffffffu, got);  // tcgen05.st is warp-collective
        if (!got) { ok = false; break; }
        tc_fence_after();
        tmem_st16_u32(tmem + kMxSfaCol + 16 * s + lane_off, a);
        tmem_st16_u32(tmem + kMxSfbCol + 16 * s + lane_off, b);
        tc_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sf_full[s]);
      }
    }
  } else {
    // ------------------------- epilogue: convert and store -------------------------
    const int q = warp & 3;
    const int h = (warp - 2 - kMxSfWarps) >> 2;  // columns [64 h, 64 h + 64) of the tile
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    int tc = 0;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++tc) {
      const F8Tile ti = mx_tile<GROUPED>(p, t, s_off);
      bool got = mbar_wait(acc_full, tc & 1, p.status, STATUS_TIMEOUT_TMEM_FULL);
      got = __all_sync(0xffffffffu, got);
      if (SWIGLU) got = mx_epi_all(got);        // the epilogue barriers below need every warp
      if (!got) break;
      tc_fence_after();
      float v[64];
      tmem_ld32(tmem + h * 64 + lane_off, v);
      tmem_ld32(tmem + h * 64 + 32 + lane_off, v + 32);
      tc_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acc_empty);
      const int row = ti.m0 + q * 32 + lane;
      if (row < ti.m_limit && p.C != nullptr) {
        bf16* dst = p.C + (long long)row * p.ldc + ti.n0 + h * 64;
        const int ncol = min(64, p.N - (ti.n0 + h * 64));
        if (ncol == 64) {
#pragma unroll
          for (int j = 0; j < 64; j += 8) {
            uint4 w = make_uint4(pack_bf16x2(v[j], v[j + 1]), pack_bf16x2(v[j + 2], v[j + 3]),
                                 pack_bf16x2(v[j + 4], v[j + 5]), pack_bf16x2(v[j + 6], v[j + 7]));
            *reinterpret_cast<uint4*>(dst + j) = w;
          }
        } else {
#pragma unroll
          for (int j = 0; j < 64; ++j)
            if (j < ncol) dst[j] = __float2bfloat16(v[j]);
        }
      }
      if (SWIGLU) {
        // columns [64 h, 64 h + 32) are gate, [64 h + 32, 64 h + 64) up (32-interleaved layout):
        // act columns n0 / 2 + 32 h + j; one 128-wide act block per row per tile (four warps)
        float amax = 0.f;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          v[j] = silu_f(v[j]) * v[32 + j];
          amax = fmaxf(amax, fabsf(v[j]));
        }
        s_amax[h * 128 + q * 32 + lane] = amax;
        mx_epi_bar();
        const int r = q * 32 + lane;
        const float bmax = fmaxf(fmaxf(s_amax[r], s_amax[128 + r]), fmaxf(s_amax[256 + r], s_amax[384 + r]));
        mx_epi_bar();                                   // partials read before the next tile writes them
        const float sc = block_scale(bmax, true);
        const long long acol = ti.n0 / 2 + h * 32;
        if (h == 0) p.act_scale[(long long)(ti.n0 / 256) * p.ld_as + row] = sc;
        if (row < ti.m_limit) {
          if (p.act != nullptr) {
            bf16* da = p.act + (long long)row * p.ld_act + acol;
#pragma unroll
            for (int j = 0; j < 32; j += 8)
              *reinterpret_cast<uint4*>(da + j) =
                  make_uint4(pack_bf16x2(v[j], v[j + 1]), pack_bf16x2(v[j + 2], v[j + 3]),
                             pack_bf16x2(v[j + 4], v[j + 5]), pack_bf16x2(v[j + 6], v[j + 7]));
          }
          uint4* dq = reinterpret_cast<uint4*>(p.actq + (long long)row * p.ld_actq + acol);
#pragma unroll
          for (int j = 0; j < 32; j += 16) {
            uint32_t w8[4];
#pragma unroll
            for (int i = 0; i < 4; ++i)
              w8[i] = (uint32_t)f32x2_to_e4m3x2(v[j + 4 * i] / sc, v[j + 4 * i + 1] / sc) |
                      ((uint32_t)f32x2_to_e4m3x2(v[j + 4 * i + 2] / sc, v[j + 4 * i + 3] / sc) << 16);
            dq[j / 16] = make_uint4(w8[0], w8[1], w8[2], w8[3]);
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ---- quantisers ---------------------------------------------------------------------

// one warp per (row, 128-column block): 4 elements per lane
__global__ void fp8_quant_act_kernel(const bf16* __restrict__ x, long long ldx, int M, int K, uint8_t* __restrict__ xq,
                                     float* __restrict__ sx, long long ldsx, bool pow2,
                                     const int* __restrict__ row_limit) {
  const int kbn = K / 128;
  const long long w = blockIdx.x * (long long)(blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (w >= (long long)ldsx * kbn) return;
  const int row = (int)(w / kbn), kb = (int)(w % kbn);
  if (row_limit != nullptr && row >= __ldg(row_limit)) return;  // rows no GEMM tile reads
  if (row >= M) {
    if (lane == 0) sx[(long long)kb * ldsx + row] = 0.f;
    return;
  }
  const bf16* src = x + (long long)row * ldx + kb * 128 + lane * 4;
  const uint2 raw = *reinterpret_cast<const uint2*>(src);
  float v[4] = {bf16_lo(raw.x), bf16_hi(raw.x), bf16_lo(raw.y), bf16_hi(raw.y)};
  float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
  amax = warp_max(amax);
  const float scale = block_scale(amax, pow2);
  const uint32_t packed = (uint32_t)f32x2_to_e4m3x2(v[0] / scale, v[1] / scale) |
                          ((uint32_t)f32x2_to_e4m3x2(v[2] / scale, v[3] / scale) << 16);
  *reinterpret_cast<uint32_t*>(xq + (long long)row * K + kb * 128 + lane * 4) = packed;
  if (lane == 0) sx[(long long)kb * ldsx + row] = scale;
}

// one CTA (256 threads) per 128 x 128 weight block: 64 elements per thread
__global__ void fp8_quant_weight_kernel(const bf16* __restrict__ w, int N, int K, uint8_t* __restrict__ wq,
                                        float* __restrict__ sw, bool pow2) {
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
  const float scale = block_scale(bmax, pow2);
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

// x [T, C] bf16 -> xt [C, T] e4m3 with a power-of-two scale per column and 128-token block,
// st [T/128][ldst] (ldst >= C): the operand of a GEMM that reduces over tokens (weight gradients).
// One CTA (256 threads) per 128 tokens x 64 columns: four threads per column, 32 tokens each.
__global__ void fp8_quant_t_kernel(const bf16* __restrict__ x, long long ldx, int T, int Cn, uint8_t* __restrict__ xt,
                                   long long ldxt, float* __restrict__ st, long long ldst) {
  __shared__ bf16 tile[128][66];
  const int t0 = blockIdx.x * 128, c0 = blockIdx.y * 64;
  const int tid = threadIdx.x;
  for (int i = tid; i < 128 * 32; i += 256) {  // bf16 pairs
    const int r = i >> 5, cp = (i & 31) * 2;
    const int t = t0 + r, c = c0 + cp;
    uint32_t v = 0u;
    if (t < T && c + 1 < Cn) v = *reinterpret_cast<const uint32_t*>(x + (long long)t * ldx + c);
    else if (t < T && c < Cn) v = (uint32_t)__bfloat16_as_ushort(x[(long long)t * ldx + c]);
    *reinterpret_cast<uint32_t*>(&tile[r][cp]) = v;
  }
  __syncthreads();
  const int col = tid >> 2, sub = tid & 3;
  float v[32], amax = 0.f;
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    v[j] = __bfloat162float(tile[sub * 32 + j][col]);
    amax = fmaxf(amax, fabsf(v[j]));
  }
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
  const float sc = block_scale(amax, true);
  const int c = c0 + col;
  if (c >= Cn) return;
  if (sub == 0) st[(long long)blockIdx.x * ldst + c] = sc;
  uint32_t w[8];
#pragma unroll
  for (int j = 0; j < 32; j += 4)
    w[j / 4] = (uint32_t)f32x2_to_e4m3x2(v[j] / sc, v[j + 1] / sc) |
               ((uint32_t)f32x2_to_e4m3x2(v[j + 2] / sc, v[j + 3] / sc) << 16);
  uint8_t* dst = xt + (long long)c * ldxt + t0 + sub * 32;
  reinterpret_cast<uint4*>(dst)[0] = make_uint4(w[0], w[1], w[2], w[3]);
  reinterpret_cast<uint4*>(dst)[1] = make_uint4(w[4], w[5], w[6], w[7]);
}

}  // namespace

void fp8_quant_t(const void* x, long long ldx, int T, int Cn, void* xt, long long ldxt, float* st, long long ldst,
                 cudaStream_t s) {
  if (T % 128 != 0) throw std::runtime_error("fp8 quant_t: the token count must be a multiple of 128");
  if (T == 0 || Cn == 0) return;
  const dim3 grid(T / 128, (Cn + 63) / 64);
  fp8_quant_t_kernel<<<grid, 256, 0, s>>>((const bf16*)x, ldx, T, Cn, (uint8_t*)xt, ldxt, st, ldst);
}

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
  p.ldsw = d.ldsw;
  if (d.ldsw > 0 && (!d.scaled_mma || grouped))
    throw std::runtime_error("fp8 gemm: per-row B scales need scaled_mma and a dense problem");
  p.C = reinterpret_cast<bf16*>(d.C);
  p.ldc = d.ldc;
  p.status = reinterpret_cast<StatusBlock*>(d.status);
  p.swiglu_q = d.actq != nullptr;
  p.act = reinterpret_cast<bf16*>(d.act);
  p.ld_act = d.ld_act;
  p.actq = reinterpret_cast<uint8_t*>(d.actq);
  p.ld_actq = d.ld_actq;
  p.act_scale = d.act_scale;
  p.ld_as = d.ld_as;
  if (p.swiglu_q && (!d.scaled_mma || d.N % 256 != 0))
    throw std::runtime_error("fp8 gemm: the SwiGLU requantisation epilogue needs scaled_mma and N % 256 == 0");
  if (d.scaled_mma) {
    // B tiles of 256 rows
    uint32_t boxw[3] = {kMxBK, kMxBN, 1};
    if (grouped) {
      uint64_t dims[3] = {(uint64_t)d.K, (uint64_t)d.N, (uint64_t)d.G};
      uint64_t str[2] = {(uint64_t)d.ldw, (uint64_t)d.w_group_stride};
      tmW = make_tmap_u8_sw128(d.W, 3, dims, str, boxw);
    } else {
      uint64_t dims[2] = {(uint64_t)d.K, (uint64_t)d.N};
      uint64_t str[1] = {(uint64_t)d.ldw};
      tmW = make_tmap_u8_sw128(d.W, 2, dims, str, boxw);
    }
    const int nnm = (d.N + kMxBN - 1) / kMxBN;
    const int tiles = grouped ? (d.max_rows_hint > 0 ? d.max_rows_hint / kMxBM : (d.M + kMxBM - 1) / kMxBM) * nnm
                              : ((d.M + kMxBM - 1) / kMxBM) * nnm;
    const int grid = std::max(1, std::min(tiles, num_sms()));
    auto kern = grouped ? (p.swiglu_q ? fp8mx_gemm_kernel<true, true> : fp8mx_gemm_kernel<true, false>)
                        : (p.swiglu_q ? fp8mx_gemm_kernel<false, true> : fp8mx_gemm_kernel<false, false>);
    ensure_smem_attr(reinterpret_cast<const void*>(kern), kMxSmem);
    kern<<<grid, kMxThreads, kMxSmem, stream>>>(tmX, tmW, p);
    return;
  }
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

void fp8_quant_act(const void* x, long long ldx, int M, int K, void* xq, float* sx, long long ldsx, bool pow2,
                   cudaStream_t s, const int* row_limit) {
  if (K % 128 != 0) throw std::runtime_error("fp8 quant: K must be a multiple of 128");
  const long long warps = ldsx * (K / 128);
  if (warps == 0) return;
  fp8_quant_act_kernel<<<(unsigned)((warps + 7) / 8), 256, 0, s>>>((const bf16*)x, ldx, M, K, (uint8_t*)xq, sx, ldsx, pow2,
                                                                          row_limit);
}

void fp8_quant_weight(const void* w, int G, int N, int K, void* wq, float* sw, bool pow2, cudaStream_t s) {
  if (K % 128 != 0) throw std::runtime_error("fp8 quant: K must be a multiple of 128");
  const dim3 grid(K / 128, (N + 127) / 128, G);
  fp8_quant_weight_kernel<<<grid, 256, 0, s>>>((const bf16*)w, N, K, (uint8_t*)wq, sw, pow2);
}

}  // namespace omni
