// Few-row GEMM for sm_100a: Y[rows, N] = X[rows, K] W[N, K]^T with rows <= 256
// per weight (batched decode, speculative verification, the expert GEMMs of a
// decode step where each expert sees a handful of tokens).
//
// Such GEMMs are bound by streaming W from HBM.  The tile GEMM (128 rows of X x
// 256 columns of W per tile) would pad the few token rows to 128 and launch only
// N/256 tiles, far fewer than there are SMs for most decode shapes.  Here the
// operands are swapped on the tensor core:
//     D^T[128 weight rows, tokens] = W_tile . X^T
// (tcgen05 M = 128 weight rows, N = the group's token count rounded up to 16,
// K = 64 per pipeline stage), so every CTA streams a 128-row slab of W through
// an 8-stage TMA ring while the token rows ride along as the small operand.
// Work units are (group, 128-row slab, K split); the split count is the largest
// that keeps the units within one wave of the persistent grid.  Each unit adds its fp32 partial sums
// into acc[rows, N] (red.global.add, one warp writes 32 consecutive columns of
// one row per instruction); skinny_finalize applies the epilogue (bf16 / fp32 /
// + residual / SwiGLU of the 32-interleaved gate|up columns).
//
// Roles (192 threads, one CTA per SM): warp 0 lane 0 TMA producer, warp 1 lane
// 0 MMA issuer + TMEM owner, warps 2-5 epilogue (warp w reads TMEM lanes
// 32*(w%4)..+31 = weight rows).  The accumulator is double buffered in tensor
// memory.  Every wait is bounded and reports through the status block.
#include <cudaTypedefs.h>

#include <cstdlib>
#include <stdexcept>

#include "common.cuh"
#include "gemm_sm100.h"

namespace omni {

namespace {

using bf16 = __nv_bfloat16;

constexpr int kSkThreads = 192;
constexpr int kSkRows = 64;                 // token rows per accumulator tile (MMA N <= 64)
constexpr int kSkStages = 8;
constexpr int kSkW = 128 * 64 * 2;          // 16 KB weight slab per stage
constexpr int kSkX = kSkRows * 64 * 2;      // 8 KB token rows per stage
constexpr int kSkStage = kSkW + kSkX;
constexpr int kSkSmem = kSkStages * kSkStage + 1024 + 256;

struct SkArgs {
  int M, N, K, G;
  int nt, ksplit, kb_per;
  const int* offsets;
  float* acc;
  StatusBlock* status;
  // direct epilogue (no K split): bf16 out = alpha * acc, or SwiGLU of the gate|up rows
  int direct, epi;
  float alpha;
  bf16* out;
  long long ldo;
};

// AND of `v` over the 128 epilogue threads (named barrier 1), so that they all take the
// same branch afterwards and none is left waiting at the barrier.
__device__ __forceinline__ bool all_epilogue(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, 1, 128, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)v)
      : "memory");
  return r != 0;
}

__device__ __forceinline__ void epilogue_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

struct SkWork {
  int g, rt, kb0, kb1, row0, rows;
};

__device__ __forceinline__ bool sk_unit(const SkArgs& p, int u, SkWork& w) {
  const int per_g = p.nt * p.ksplit;
  w.g = u / per_g;
  const int r = u - w.g * per_g;
  w.rt = r / p.ksplit;
  const int ks = r - w.rt * p.ksplit;
  const int nkb = (p.K + 63) / 64;
  w.kb0 = ks * p.kb_per;
  w.kb1 = min(nkb, w.kb0 + p.kb_per);
  if (p.offsets != nullptr) {
    w.row0 = p.offsets[w.g];
    w.rows = min(p.offsets[w.g + 1], p.M) - w.row0;
  } else {
    w.row0 = 0;
    w.rows = p.M;
  }
  return w.rows > 0 && w.kb1 > w.kb0;
}

template <bool GROUPED>
__global__ void __launch_bounds__(kSkThreads, 1)
    skinny_gemm_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX, SkArgs p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kSkStages * kSkStage);
  uint64_t* empty = full + kSkStages;
  uint64_t* tfull = empty + kSkStages;  // [2] accumulator ready
  uint64_t* tempty = tfull + 2;         // [2] accumulator drained by the epilogue
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  const int warp = warp_id(), lane = lane_id();
  if (threadIdx.x == 0) {
    for (int s = 0; s < kSkStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 128);
    }
    mbar_init(drain, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 2 * kSkRows);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int units = p.G * p.nt * p.ksplit;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------ TMA producer ------------------------------
      tma_prefetch_desc(&tmW);
      tma_prefetch_desc(&tmX);
      int it = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
        SkWork w;
        if (!sk_unit(p, u, w)) continue;
        for (int c0 = 0; c0 < w.rows && ok; c0 += kSkRows) {
          const int nx = (min(kSkRows, w.rows - c0) + 15) / 16;
          for (int kb = w.kb0; kb < w.kb1; ++kb, ++it) {
            const int s = it % kSkStages;
            const uint32_t ph = (it / kSkStages) & 1;
            if (!mbar_wait(&empty[s], ph ^ 1, p.status, STATUS_TIMEOUT_TMA_EMPTY)) { ok = false; break; }
            uint8_t* sw = smem + s * kSkStage;
            uint8_t* sx = sw + kSkW;
            mbar_arrive_expect_tx(&full[s], kSkW + nx * 2048);
            if (GROUPED)
              tma_load_3d(sw, &tmW, &full[s], kb * 64, w.rt * 128, w.g);
            else
              tma_load_2d(sw, &tmW, &full[s], kb * 64, w.rt * 128);
            for (int j = 0; j < nx; ++j) tma_load_2d(sx + j * 2048, &tmX, &full[s], kb * 64, w.row0 + c0 + 16 * j);
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------- MMA issuer -------------------------------
      int it = 0, tile = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
        SkWork w;
        if (!sk_unit(p, u, w)) continue;
        for (int c0 = 0; c0 < w.rows && ok; c0 += kSkRows, ++tile) {
          const int nx = (min(kSkRows, w.rows - c0) + 15) / 16;
          const int a = tile & 1;
          if (!mbar_wait(&tempty[a], ((tile >> 1) & 1) ^ 1, p.status, STATUS_TIMEOUT_TMEM_EMPTY)) { ok = false; break; }
          tc_fence_after();
          const uint32_t d = tmem + a * kSkRows;
          const uint32_t idesc = umma_idesc_f16(128, nx * 16, false, false, true);
          for (int kb = w.kb0; kb < w.kb1; ++kb, ++it) {
            const int s = it % kSkStages;
            if (!mbar_wait(&full[s], (it / kSkStages) & 1, p.status, STATUS_TIMEOUT_TMA_FULL)) { ok = false; break; }
            tc_fence_after();
            const uint32_t wa = smem_u32(smem + s * kSkStage), xa = wa + kSkW;
#pragma unroll
            for (int k4 = 0; k4 < 4; ++k4)
              tc_mma_f16(d, umma_desc_sw128(wa + k4 * 32, 16, 1024), umma_desc_sw128(xa + k4 * 32, 16, 1024), idesc,
                         (kb > w.kb0 || k4 > 0) ? 1u : 0u);
            tc_commit(&empty[s]);
          }
          if (!ok) break;
          tc_commit(&tfull[a]);
        }
      }
      tc_commit(drain);
      mbar_wait(drain, 0, p.status, STATUS_TIMEOUT_DRAIN);
    }
  } else {
    // --------------------------------- epilogue ---------------------------------
    const int q = warp & 3;
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    __shared__ float s_up[2][16][32];  // SwiGLU: up values of the current 16 tokens, per 64-row block
    int tile = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
      SkWork w;
      if (!sk_unit(p, u, w)) continue;
      const int n = w.rt * 128 + q * 32 + lane;
      for (int c0 = 0; c0 < w.rows; c0 += kSkRows, ++tile) {
        const int nx = (min(kSkRows, w.rows - c0) + 15) / 16;
        const int a = tile & 1;
        bool got = mbar_wait(&tfull[a], (tile >> 1) & 1, p.status, STATUS_TIMEOUT_TMEM_FULL);
        got = all_epilogue(got);  // tcgen05.ld is warp-collective; the direct epilogue syncs all 4 warps
        if (!got) { ok = false; break; }
        tc_fence_after();
        if (p.direct) {
          for (int j = 0; j < nx; ++j) {
            float v[16];
            tmem_ld16(tmem + a * kSkRows + j * 16 + lane_off, v);
            tc_wait_ld();
            const int t0 = c0 + j * 16;
            if (p.epi == EPI_SWIGLU) {
              // weight rows of the tile: [gate 32 | up 32] x 2; warp q holds block q >> 1, gate if q even
              if (q & 1) {
#pragma unroll
                for (int i = 0; i < 16; ++i) s_up[q >> 1][i][lane] = v[i] * p.alpha;
              }
              epilogue_bar();
              if (!(q & 1)) {
                const int col = w.rt * 64 + (q >> 1) * 32 + lane;
                if (col < p.N / 2) {
#pragma unroll
                  for (int i = 0; i < 16; ++i)
                    if (t0 + i < w.rows)
                      p.out[(long long)(w.row0 + t0 + i) * p.ldo + col] =
                          __float2bfloat16(silu_f(v[i] * p.alpha) * s_up[q >> 1][i][lane]);
                }
              }
              epilogue_bar();
            } else if (n < p.N) {
#pragma unroll
              for (int i = 0; i < 16; ++i)
                if (t0 + i < w.rows) p.out[(long long)(w.row0 + t0 + i) * p.ldo + n] = __float2bfloat16(v[i] * p.alpha);
            }
          }
          tc_fence_before();
          mbar_arrive(&tempty[a]);
          continue;
        }
        for (int j = 0; j < nx; ++j) {
          float v[16];
          tmem_ld16(tmem + a * kSkRows + j * 16 + lane_off, v);
          tc_wait_ld();
          if (n < p.N) {
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const int t = c0 + j * 16 + i;
              if (t < w.rows) atomicAdd(p.acc + (long long)(w.row0 + t) * p.N + n, v[i]);
            }
          }
        }
        tc_fence_before();
        mbar_arrive(&tempty[a]);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 2 * kSkRows);
  }
}

template <int EPI>
__global__ void skinny_finalize_kernel(const float* __restrict__ acc, int rows, int N, float alpha, void* out,
                                       long long ldo, const bf16* __restrict__ R, long long ldr) {
  const int outN = EPI == EPI_SWIGLU ? N / 2 : N;
  const long long total = (long long)rows * outN;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const int r = (int)(i / outN), c = (int)(i - (long long)r * outN);
    const float* row = acc + (long long)r * N;
    float v;
    if (EPI == EPI_SWIGLU) {
      const int base = (c >> 5) * 64 + (c & 31);
      v = silu_f(row[base] * alpha) * (row[base + 32] * alpha);
    } else {
      v = row[c] * alpha;
    }
    if (EPI == EPI_STORE_F32) {
      reinterpret_cast<float*>(out)[(long long)r * ldo + c] = v;
    } else {
      if (EPI == EPI_ADD_BF16) v += __bfloat162float(R[(long long)r * ldr + c]);
      reinterpret_cast<bf16*>(out)[(long long)r * ldo + c] = __float2bfloat16(v);
    }
  }
}

}  // namespace

int skinny_ksplit(const SkinnyDesc& d) {
  const int nt = (d.N + 127) / 128;
  const int nkb = (d.K + 63) / 64;
  const int base = (d.offsets != nullptr ? d.G : 1) * nt;
  const int sms = num_sms();
  // At most one wave of units: a slab streams fast enough that ~40 % of the SMs saturate HBM, so
  // extra K splits only add fp32 partial-sum traffic (red.global), the workspace clear and the
  // finalize launch.  From 40 % of an SM's worth of slabs on there is no split (direct bf16
  // epilogue, no workspace): 9216 x 2048 at 64 rows takes 20.5 us unsplit against 28.7 us in
  // two splits.
  int ks = base * 5 >= sms * 2 ? 1 : std::max(1, sms / base);
  static const int forced = [] {
    const char* e = getenv("OMNI_SKINNY_SPLIT");  // fixed split count (measurements)
    return e != nullptr ? std::max(0, atoi(e)) : 0;
  }();
  if (forced > 0) ks = forced;
  ks = std::max(1, std::min(ks, std::max(1, nkb / 4)));
  const int kb_per = (nkb + ks - 1) / ks;
  return (nkb + kb_per - 1) / kb_per;
}

void skinny_gemm_launch(const SkinnyDesc& d, cudaStream_t stream) {
  if (d.M <= 0 || d.N <= 0) return;
  if (d.K <= 0 || d.K % 8 != 0) throw std::runtime_error("skinny gemm: K must be a positive multiple of 8");
  const bool grouped = d.offsets != nullptr;
  CUtensorMap tmW, tmX;
  if (grouped) {
    uint64_t dims[3] = {(uint64_t)d.K, (uint64_t)d.N, (uint64_t)d.G};
    uint64_t str[2] = {(uint64_t)d.ldw * 2, (uint64_t)d.w_group_stride * 2};
    uint32_t box[3] = {64, 128, 1};
    tmW = make_tmap_bf16_sw128(d.W, 3, dims, str, box);
  } else {
    uint64_t dims[2] = {(uint64_t)d.K, (uint64_t)d.N};
    uint64_t str[1] = {(uint64_t)d.ldw * 2};
    uint32_t box[2] = {64, 128};
    tmW = make_tmap_bf16_sw128(d.W, 2, dims, str, box);
  }
  {
    uint64_t dims[2] = {(uint64_t)d.K, (uint64_t)d.M};
    uint64_t str[1] = {(uint64_t)d.ldx * 2};
    uint32_t box[2] = {64, 16};
    tmX = make_tmap_bf16_sw128(d.X, 2, dims, str, box);
  }
  SkArgs p;
  p.direct = 0;
  p.epi = d.epilogue;
  p.alpha = d.alpha;
  p.out = reinterpret_cast<bf16*>(d.out);
  p.ldo = d.ldo;
  p.M = d.M;
  p.N = d.N;
  p.K = d.K;
  p.G = grouped ? d.G : 1;
  p.offsets = d.offsets;
  p.acc = d.acc;
  p.status = reinterpret_cast<StatusBlock*>(d.status);
  p.nt = (d.N + 127) / 128;
  const int nkb = (d.K + 63) / 64;
  const int sms = num_sms();
  const int base = p.G * p.nt;
  const int ks = skinny_ksplit(d);
  p.kb_per = (nkb + ks - 1) / ks;
  p.ksplit = (nkb + p.kb_per - 1) / p.kb_per;
  if (d.out != nullptr) {
    if (p.ksplit != 1 || !(d.epilogue == EPI_STORE_BF16 || d.epilogue == EPI_SWIGLU))
      throw std::runtime_error("skinny gemm: direct output needs an unsplit K and a bf16 / SwiGLU epilogue");
    p.direct = 1;
  }
  const int units = base * p.ksplit;
  const int grid = std::min(units, sms);
  if (grouped) {
    auto kern = skinny_gemm_kernel<true>;
    ensure_smem_attr(reinterpret_cast<const void*>(kern), kSkSmem);
    kern<<<grid, kSkThreads, kSkSmem, stream>>>(tmW, tmX, p);
  } else {
    auto kern = skinny_gemm_kernel<false>;
    ensure_smem_attr(reinterpret_cast<const void*>(kern), kSkSmem);
    kern<<<grid, kSkThreads, kSkSmem, stream>>>(tmW, tmX, p);
  }
}

void skinny_finalize(const float* acc, int rows, int N, int epilogue, float alpha, void* out, long long ldo,
                     const void* R, long long ldr, cudaStream_t stream) {
  if (rows <= 0) return;
  const long long total = (long long)rows * (epilogue == EPI_SWIGLU ? N / 2 : N);
  const int threads = 256;
  const int blocks = (int)std::min<long long>((total + threads - 1) / threads, 4L * num_sms());
  const bf16* r = reinterpret_cast<const bf16*>(R);
  switch (epilogue) {
    case EPI_STORE_BF16: skinny_finalize_kernel<EPI_STORE_BF16><<<blocks, threads, 0, stream>>>(acc, rows, N, alpha, out, ldo, r, ldr); break;
    case EPI_STORE_F32: skinny_finalize_kernel<EPI_STORE_F32><<<blocks, threads, 0, stream>>>(acc, rows, N, alpha, out, ldo, r, ldr); break;
    case EPI_ADD_BF16: skinny_finalize_kernel<EPI_ADD_BF16><<<blocks, threads, 0, stream>>>(acc, rows, N, alpha, out, ldo, r, ldr); break;
    case EPI_SWIGLU: skinny_finalize_kernel<EPI_SWIGLU><<<blocks, threads, 0, stream>>>(acc, rows, N, alpha, out, ldo, r, ldr); break;
    default: throw std::runtime_error("skinny gemm: unsupported epilogue");
  }
}

}  // namespace omni
