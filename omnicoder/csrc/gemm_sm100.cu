// tcgen05 / TMEM / TMA GEMM for sm_100a.
//
// C[M,N] = alpha * sum_k A[M,k] * B[N,k]   (fp32 accumulation in tensor memory)
//
// Operand storage (bf16, row-major in global memory):
//   A K-major  : A stored [M, K]          A MN-major : A stored [K, M]
//   B K-major  : B stored [N, K]          B MN-major : B stored [K, N]
// This covers every linear-layer GEMM of training: Y = X W^T (K,K),
// dX = dY W (K,MN) and dW = dY^T X (MN,MN).
//
// Modes:
//   dense     : one problem.
//   grouped-M : rows of A are segmented into groups (experts) by a device
//               offset table whose entries are multiples of 128; group g uses
//               B[g] (a [G, N, K] or [G, K, N] weight stack).  The row count is
//               read on the device, so no host synchronisation is needed.
//   grouped-K : the reduction runs over the rows of group g only and the
//               output is C[g] (expert weight gradients).
//
// Kernel structure (one persistent CTA per SM, 192 threads):
//   warp 0     : TMA producer (one lane), 4-6 stage shared-memory ring
//   warp 1     : TMEM allocator + tcgen05.mma issuer (one lane)
//   warps 2..5 : epilogue; each warp owns the 32 TMEM lanes (rows) that its
//                warp index selects, reads 32 fp32 columns per tcgen05.ld,
//                applies the fused epilogue and stores to global memory.
// The accumulator is double buffered in TMEM so the epilogue of tile i
// overlaps the main loop of tile i+1.
//
// The epilogue fusions cover what the reference's linear layers and expert FFN
// do around their GEMMs (src/omnicoder/modeling/kernels/moe_scatter.py:738-753
// applies bias + GELU between the two batched expert GEMMs; the spec family
// uses SwiGLU instead).
#include <cudaTypedefs.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <stdexcept>
#include <string>

#include "common.cuh"
#include "gemm_sm100.h"

namespace omni {

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kThreads = 192;
constexpr int kSwizzleChunk = 8192;  // bytes of one 64(MN) x 64(K) bf16 swizzled box

struct GemmArgs {
  int M, N, K;
  int num_groups;
  const int* group_offsets;  // [G+1], multiples of 128 (grouped modes)
  void* C;
  long long ldc;
  long long c_group_stride;  // elements between C[g] and C[g+1] (grouped-K)
  const void* R;             // residual (EPI_ADD_BF16) or pre-activation H (EPI_SWIGLU_BWD)
  long long ldr;
  void* H;                   // pre-activation store (EPI_SWIGLU)
  long long ldh;
  float alpha;
  StatusBlock* status;
  int nsrc, me, src_rows;
  int mt_rot;                      // dense raster: rotate the M tiles so a rank starts on its own rows
  void* peer_c[GEMM_MAX_PEERS];
  const int4* row_meta;            // EPI_EP_PUSH: (weight, source rank, pair index, -) per row
  const unsigned* ready;           // grouped-M: per-source readiness flags (nullptr: no gating)
  const unsigned* ready_epoch;
  const int* src_pref;             // [G][nsrc + 1]
  int tma_c;                       // bf16 / SwiGLU outputs leave through shared memory + TMA stores
  int rows_c;                      // rows of C (per group in grouped-K mode)
};

// Per-source tensor maps of A (GEMM_AG mode; unused otherwise).
struct AgMaps {
  CUtensorMap m[GEMM_MAX_PEERS];
};

// PAIR: a cluster of two CTAs computes one (2*128) x BN tile with cta_group::2 MMAs;
// each CTA stages its 128 rows of A and BN/2 rows of B, so per SM the shared-memory
// operand traffic per FLOP drops by a third against the one-CTA 128 x BN tile.
template <int BN, bool PAIR = false>
struct Cfg {
  static constexpr int kTM = PAIR ? 2 * kBM : kBM;  // rows of C per tile
  static constexpr int kBNc = PAIR ? BN / 2 : BN;  // rows of B staged by one CTA
  static constexpr int kStageA = kBM * kBK * 2;    // 16 KB
  static constexpr int kStageB = kBNc * kBK * 2;   // 32 KB at BN=256 (16 KB per CTA of a pair)
  static constexpr int kStageBytes = kStageA + kStageB;
  static constexpr int kStages = PAIR ? 6 : (BN >= 256 ? 4 : 6);
  static constexpr int kTmemCols = 2 * BN;         // double-buffered accumulator
  // epilogue staging: two [32 rows x 128 B] swizzled boxes per epilogue warp
  static constexpr int kEpiBox = 4096;
  static constexpr int kEpiBytes = 4 * 2 * kEpiBox;
  static constexpr int kSmemBytes = kStages * kStageBytes + kEpiBytes + 1024 /*align*/ + 256 /*barriers*/;
};

// Epilogue staging of one warp: its 32 accumulator rows, 64 bf16 columns at a time, are
// written into a 128B-swizzled [32 x 128 B] box in shared memory (conflict-free: lane r
// writes 16-byte chunk q of its row at chunk q ^ (r & 7)) and leave with one TMA store,
// so global memory sees whole 128-byte row segments instead of one 16-byte piece per row.
struct EpiStage {
  uint8_t* base;  // two 4 KB boxes, 1024-byte aligned
  int cur;
  // Next free box (the store issued two boxes ago has finished reading it).
  __device__ __forceinline__ uint8_t* acquire(int lane) {
    if (lane == 0) bulk_wait_group_read<1>();
    __syncwarp();
    return base + cur * 4096;
  }
  // Row `lane` of the box: 8 chunks of 8 bf16 (packed pairs).
  __device__ __forceinline__ static void put_row(uint8_t* box, int lane, const uint32_t* w) {
#pragma unroll
    for (int q = 0; q < 8; ++q)
      *reinterpret_cast<uint4*>(box + lane * 128 + ((q ^ (lane & 7)) << 4)) =
          make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
  }
  __device__ __forceinline__ void issue_2d(int lane, const CUtensorMap* m, int x, int y) {
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      tma_store_2d(m, base + cur * 4096, x, y);
      bulk_commit_group();
    }
    cur ^= 1;
  }
  __device__ __forceinline__ void issue_3d(int lane, const CUtensorMap* m, int x, int y, int z) {
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      tma_store_3d(m, base + cur * 4096, x, y, z);
      bulk_commit_group();
    }
    cur ^= 1;
  }
};

struct TileInfo {
  int m0, n0, g, k0, num_kb;
  int m_limit;  // rows >= m_limit are not stored
};

template <int BN, int MODE, int TM = kBM>
__device__ __forceinline__ int total_tiles(const GemmArgs& p, const int* s_off) {
  const int num_n = (p.N + BN - 1) / BN;
  if (MODE == GEMM_DENSE || MODE == GEMM_AG) return ((p.M + TM - 1) / TM) * num_n;
  if (MODE == GEMM_GROUPED_M) return (s_off[p.num_groups] / kBM) * num_n;
  return p.num_groups * ((p.M + TM - 1) / TM) * num_n;
}

template <int BN, int MODE, int TM = kBM>
__device__ __forceinline__ TileInfo tile_info(const GemmArgs& p, int t, const int* s_off) {
  TileInfo ti;
  const int num_n = (p.N + BN - 1) / BN;
  if (MODE == GEMM_DENSE || MODE == GEMM_AG) {
    // Grouped raster: 8 M-tiles share each sweep over N for L2 reuse of B.
    const int num_m = (p.M + TM - 1) / TM;
    constexpr int GM = 8;
    const int per_group = GM * num_n;
    const int grp = t / per_group;
    const int first_m = grp * GM;
    const int gsize = min(num_m - first_m, GM);
    const int r = t - grp * per_group;
    ti.m0 = ((first_m + r % gsize + p.mt_rot) % num_m) * TM;
    ti.n0 = (r / gsize) * BN;
    ti.g = 0;
    ti.k0 = 0;
    ti.num_kb = (p.K + kBK - 1) / kBK;
    ti.m_limit = p.M;
  } else if (MODE == GEMM_GROUPED_M) {
    const int mt = t / num_n;
    ti.m0 = mt * kBM;
    ti.n0 = (t - mt * num_n) * BN;
    int g = 0;
    while (g + 1 < p.num_groups && s_off[g + 1] <= ti.m0) ++g;
    ti.g = g;
    ti.k0 = 0;
    ti.num_kb = (p.K + kBK - 1) / kBK;
    ti.m_limit = s_off[g + 1];
  } else {
    const int num_m = (p.M + TM - 1) / TM;
    const int per_g = num_m * num_n;
    const int g = t / per_g;
    const int r = t - g * per_g;
    ti.g = g;
    ti.m0 = (r / num_n) * TM;
    ti.n0 = (r % num_n) * BN;
    ti.k0 = s_off[g];
    ti.num_kb = (s_off[g + 1] - s_off[g]) / kBK;
    ti.m_limit = p.M;
  }
  return ti;
}

// ---------------------------------------------------------------------------
// Epilogue: 32 accumulator columns of one row -> global memory
// ---------------------------------------------------------------------------
template <int EPI>
__device__ __forceinline__ void store_chunk(const GemmArgs& p, int row, int col, int g, const float* v,
                                            bool row_ok) {
  if (!row_ok) return;
  const int ncols = min(32, p.N - col);
  if (ncols <= 0) return;
  if (EPI == EPI_STORE_BF16 || EPI == EPI_ADD_BF16) {
    __nv_bfloat16* C = reinterpret_cast<__nv_bfloat16*>(p.C) + (long long)g * p.c_group_stride +
                       (long long)row * p.ldc + col;
    float o[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) o[j] = v[j] * p.alpha;
    if (EPI == EPI_ADD_BF16) {
      const __nv_bfloat16* R = reinterpret_cast<const __nv_bfloat16*>(p.R) + (long long)row * p.ldr + col;
      if (ncols == 32) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint4 r = *reinterpret_cast<const uint4*>(R + q * 8);
          const uint32_t* rw = reinterpret_cast<const uint32_t*>(&r);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            o[q * 8 + 2 * j] += bf16_lo(rw[j]);
            o[q * 8 + 2 * j + 1] += bf16_hi(rw[j]);
          }
        }
      } else {
        for (int j = 0; j < ncols; ++j) o[j] += __bfloat162float(R[j]);
      }
    }
    if (ncols == 32) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint4 w;
        w.x = pack_bf16x2(o[q * 8 + 0], o[q * 8 + 1]);
        w.y = pack_bf16x2(o[q * 8 + 2], o[q * 8 + 3]);
        w.z = pack_bf16x2(o[q * 8 + 4], o[q * 8 + 5]);
        w.w = pack_bf16x2(o[q * 8 + 6], o[q * 8 + 7]);
        *reinterpret_cast<uint4*>(C + q * 8) = w;
      }
    } else {
      for (int j = 0; j < ncols; ++j) C[j] = __float2bfloat16(o[j]);
    }
  } else if (EPI == EPI_PEER_BF16) {
    // partial sums of a row owned by rank `owner` go to slot `me` of that rank's staging buffer
    const int owner = row / p.src_rows;
    __nv_bfloat16* C = reinterpret_cast<__nv_bfloat16*>(p.peer_c[owner]) +
                       ((long long)p.me * p.src_rows + (row - owner * p.src_rows)) * p.ldc + col;
    if (ncols == 32) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint4 w;
        w.x = pack_bf16x2(v[q * 8 + 0] * p.alpha, v[q * 8 + 1] * p.alpha);
        w.y = pack_bf16x2(v[q * 8 + 2] * p.alpha, v[q * 8 + 3] * p.alpha);
        w.z = pack_bf16x2(v[q * 8 + 4] * p.alpha, v[q * 8 + 5] * p.alpha);
        w.w = pack_bf16x2(v[q * 8 + 6] * p.alpha, v[q * 8 + 7] * p.alpha);
        *reinterpret_cast<uint4*>(C + q * 8) = w;
      }
    } else {
      for (int j = 0; j < ncols; ++j) C[j] = __float2bfloat16(v[j] * p.alpha);
    }
  } else if (EPI == EPI_STORE_F32 || EPI == EPI_ACCUM_F32) {
    float* C = reinterpret_cast<float*>(p.C) + (long long)g * p.c_group_stride + (long long)row * p.ldc + col;
    if (ncols == 32) {
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        float4 w = make_float4(v[4 * q] * p.alpha, v[4 * q + 1] * p.alpha, v[4 * q + 2] * p.alpha,
                               v[4 * q + 3] * p.alpha);
        if (EPI == EPI_ACCUM_F32) {
          float4 c = *reinterpret_cast<const float4*>(C + 4 * q);
          w.x += c.x;
          w.y += c.y;
          w.z += c.z;
          w.w += c.w;
        }
        *reinterpret_cast<float4*>(C + 4 * q) = w;
      }
    } else {
      for (int j = 0; j < ncols; ++j) C[j] = v[j] * p.alpha + (EPI == EPI_ACCUM_F32 ? C[j] : 0.f);
    }
  }
}

// SwiGLU forward epilogue.  The gate/up weight rows are interleaved in blocks
// of 32: accumulator columns [64j, 64j+32) are gate rows 32j.., columns
// [64j+32, 64j+64) the matching up rows.  Output column 32j+i of the
// activation is silu(gate_i) * up_i.  The raw (gate, up) pair is also stored
// (interleaved, as computed) for the backward pass.
__device__ __forceinline__ void store_swiglu(const GemmArgs& p, int row, int col /*acc col of gate chunk*/,
                                             const float* gt, const float* up, bool row_ok) {
  if (!row_ok || col >= p.N) return;
  const int ocol = col >> 1;
  __nv_bfloat16* C = reinterpret_cast<__nv_bfloat16*>(p.C) + (long long)row * p.ldc + ocol;
  uint32_t packed[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const float a0 = silu_f(gt[2 * j]) * up[2 * j];
    const float a1 = silu_f(gt[2 * j + 1]) * up[2 * j + 1];
    packed[j] = pack_bf16x2(a0, a1);
  }
#pragma unroll
  for (int q = 0; q < 4; ++q)
    *reinterpret_cast<uint4*>(C + q * 8) =
        make_uint4(packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]);
  if (p.H != nullptr) {
    __nv_bfloat16* H = reinterpret_cast<__nv_bfloat16*>(p.H) + (long long)row * p.ldh + col;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      *reinterpret_cast<uint4*>(H + q * 8) =
          make_uint4(pack_bf16x2(gt[8 * q], gt[8 * q + 1]), pack_bf16x2(gt[8 * q + 2], gt[8 * q + 3]),
                     pack_bf16x2(gt[8 * q + 4], gt[8 * q + 5]), pack_bf16x2(gt[8 * q + 6], gt[8 * q + 7]));
      *reinterpret_cast<uint4*>(H + 32 + q * 8) =
          make_uint4(pack_bf16x2(up[8 * q], up[8 * q + 1]), pack_bf16x2(up[8 * q + 2], up[8 * q + 3]),
                     pack_bf16x2(up[8 * q + 4], up[8 * q + 5]), pack_bf16x2(up[8 * q + 6], up[8 * q + 7]));
    }
  }
}

// SwiGLU backward epilogue: the accumulator holds dA (gradient of the
// activation, 32 columns starting at activation column `col`).  R points at
// the saved interleaved pre-activation H; the output C is dH in the same
// interleaved layout (ldc counts dH columns = 2 * activation columns).
__device__ __forceinline__ void store_swiglu_bwd(const GemmArgs& p, int row, int col, const float* da,
                                                 bool row_ok) {
  if (!row_ok || col >= p.N) return;
  const __nv_bfloat16* H = reinterpret_cast<const __nv_bfloat16*>(p.R) + (long long)row * p.ldr + 2 * col;
  __nv_bfloat16* D = reinterpret_cast<__nv_bfloat16*>(p.C) + (long long)row * p.ldc + 2 * col;
  float gt[32], up[32];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint4 a = *reinterpret_cast<const uint4*>(H + q * 8);
    uint4 b = *reinterpret_cast<const uint4*>(H + 32 + q * 8);
    const uint32_t* aw = reinterpret_cast<const uint32_t*>(&a);
    const uint32_t* bw = reinterpret_cast<const uint32_t*>(&b);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      gt[q * 8 + 2 * j] = bf16_lo(aw[j]);
      gt[q * 8 + 2 * j + 1] = bf16_hi(aw[j]);
      up[q * 8 + 2 * j] = bf16_lo(bw[j]);
      up[q * 8 + 2 * j + 1] = bf16_hi(bw[j]);
    }
  }
  uint32_t dg[16], du[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    float r[2], s[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const float g = gt[2 * j + h], u = up[2 * j + h], d = da[2 * j + h] * p.alpha;
      const float sg = 1.0f / (1.0f + __expf(-g));
      const float si = g * sg;
      s[h] = d * si;                                // d/du
      r[h] = d * u * (sg * (1.0f + g * (1.0f - sg)));  // d/dg
    }
    dg[j] = pack_bf16x2(r[0], r[1]);
    du[j] = pack_bf16x2(s[0], s[1]);
  }
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    *reinterpret_cast<uint4*>(D + q * 8) = make_uint4(dg[4 * q], dg[4 * q + 1], dg[4 * q + 2], dg[4 * q + 3]);
    *reinterpret_cast<uint4*>(D + 32 + q * 8) =
        make_uint4(du[4 * q], du[4 * q + 1], du[4 * q + 2], du[4 * q + 3]);
  }
}

// ---------------------------------------------------------------------------
// The kernel
// ---------------------------------------------------------------------------
template <int BN, bool A_MN, bool B_MN, int EPI, int MODE, bool PAIR = false>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_sm100_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                      const __grid_constant__ AgMaps ag, const __grid_constant__ CUtensorMap tmC,
                      const __grid_constant__ CUtensorMap tmH, GemmArgs p) {
  using C_ = Cfg<BN, PAIR>;
  constexpr int S = C_::kStages;
  constexpr int TM = C_::kTM;
  constexpr bool kTmaEpi = EPI == EPI_STORE_BF16 || EPI == EPI_SWIGLU;
  // epilogues with a bf16 side input (residual R, or the saved SwiGLU pre-activation H)
  constexpr bool kTmaIn = EPI == EPI_ADD_BF16 || EPI == EPI_SWIGLU_BWD;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* epi_smem = smem + S * C_::kStageBytes;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(epi_smem + C_::kEpiBytes);
  uint64_t* empty_bar = full_bar + S;
  uint64_t* tfull_bar = empty_bar + S;   // [2]
  uint64_t* tempty_bar = tfull_bar + 2;  // [2]
  uint64_t* drain_bar = tempty_bar + 2;  // [1]
  uint64_t* in_bar = drain_bar + 1;      // [4 warps x 2 boxes] side-input (residual / H) box loads
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(in_bar + 8);
  __shared__ int s_off[GEMM_MAX_GROUPS + 1];

  const int warp = warp_id();
  const int lane = lane_id();
  // A pair is two consecutive CTAs of one cluster; rank 0 (the leader) issues the MMAs
  // and owns the barriers that the MMAs wait on.
  const uint32_t crank = PAIR ? cluster_ctarank() : 0u;
  const bool leader = crank == 0u;
  const int tile0 = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
  const int tile_step = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;

  if (MODE != GEMM_DENSE) {
    for (int i = threadIdx.x; i <= p.num_groups; i += kThreads) s_off[i] = p.group_offsets[i];
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull_bar[b], 1);
      mbar_init(&tempty_bar[b], PAIR ? 8 : 4);  // every epilogue warp of the tile's CTAs
    }
    mbar_init(drain_bar, 1);
    for (int i = 0; i < 8; ++i) mbar_init(&in_bar[i], 1);
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    if (MODE == GEMM_AG) {
      for (int r = 0; r < p.nsrc; ++r) tma_prefetch_desc(&ag.m[r]);
    } else {
      tma_prefetch_desc(&tmA);
    }
    tma_prefetch_desc(&tmB);
    if ((kTmaEpi || kTmaIn) && p.tma_c) {
      tma_prefetch_desc(&tmC);
      if ((EPI == EPI_SWIGLU && p.H != nullptr) || kTmaIn) tma_prefetch_desc(&tmH);
    }
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc_pair(tmem_slot, C_::kTmemCols);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, C_::kTmemCols);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  if constexpr (PAIR) cluster_sync_all(); else __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int ntiles = total_tiles<BN, MODE, TM>(p, s_off);

  if (warp == 0) {
    // ------------------------------ TMA producer ------------------------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      // expert-parallel receive rows: sources whose rows this CTA has seen ready
      uint32_t seen = 0;
      const unsigned epoch = (MODE == GEMM_GROUPED_M && p.ready != nullptr) ? *p.ready_epoch : 0u;
      for (int t = tile0; t < ntiles && ok; t += tile_step) {
        const TileInfo ti = tile_info<BN, MODE, TM>(p, t, s_off);
        const int am0 = ti.m0 + (int)crank * kBM;         // this CTA's rows of A
        const int bn0 = ti.n0 + (int)crank * C_::kBNc;    // this CTA's rows of B
        if (MODE == GEMM_GROUPED_M && p.ready != nullptr) {
          // wait (bounded) for every other source rank with rows in [m0, m0 + 128) of this group
          const int r0 = ti.m0 - s_off[ti.g];
          const int* pref = p.src_pref + ti.g * (p.nsrc + 1);
          bool waited = false;
          for (int s = 0; s < p.nsrc && ok; ++s) {
            if (s == p.me || ((seen >> s) & 1u) || !(pref[s] < r0 + kBM && pref[s + 1] > r0)) continue;
            const uint64_t t0 = globaltimer_ns();
            uint32_t spins = 0;
            while (true) {
              unsigned v;
              asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p.ready + s) : "memory");
              if ((int)(v - epoch) >= 0) break;
              if ((++spins & 63u) == 0u && globaltimer_ns() - t0 > kWaitBudgetNs) {
                report_error(p.status, STATUS_TIMEOUT_PEER_FLAG, s);
                ok = false;
                break;
              }
            }
            seen |= 1u << s;
            waited = true;
          }
          if (!ok) break;
          if (waited) fence_proxy_async_global();  // the rows acquired above, then TMA reads them
        }
        for (int kb = 0; kb < ti.num_kb; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1, p.status, STATUS_TIMEOUT_TMA_EMPTY)) {
            ok = false;
            break;
          }
          uint8_t* sA = smem + stage * C_::kStageBytes;
          uint8_t* sB = sA + C_::kStageA;
          const int k = ti.k0 + kb * kBK;
          if constexpr (PAIR) {
            // both CTAs' bytes complete on the leader's barrier
            const uint32_t bar = mapa_shared(smem_u32(&full_bar[stage]), 0);
            if (leader) mbar_arrive_expect_tx(&full_bar[stage], 2 * C_::kStageBytes);
            if (!A_MN) {
              tma_load_2d_pair(sA, &tmA, bar, k, am0);
            } else {
#pragma unroll
              for (int i = 0; i < kBM / 64; ++i) tma_load_2d_pair(sA + i * kSwizzleChunk, &tmA, bar, am0 + 64 * i, k);
            }
            if (!B_MN) {
              tma_load_2d_pair(sB, &tmB, bar, k, bn0);
            } else {
#pragma unroll
              for (int i = 0; i < C_::kBNc / 64; ++i)
                tma_load_2d_pair(sB + i * kSwizzleChunk, &tmB, bar, bn0 + 64 * i, k);
            }
          } else {
            mbar_arrive_expect_tx(&full_bar[stage], C_::kStageBytes);
            if (MODE == GEMM_AG) {
              // rows of source rank `src`, read from its buffer (over NVLink for a peer)
              const int src = ti.m0 / p.src_rows;
              tma_load_2d(sA, &ag.m[src], &full_bar[stage], k, ti.m0 - src * p.src_rows);
            } else if (!A_MN) {
              tma_load_2d(sA, &tmA, &full_bar[stage], k, ti.m0);
            } else {
#pragma unroll
              for (int i = 0; i < kBM / 64; ++i)
                tma_load_2d(sA + i * kSwizzleChunk, &tmA, &full_bar[stage], ti.m0 + 64 * i, k);
            }
            if (!B_MN) {
              if (MODE == GEMM_GROUPED_M)
                tma_load_3d(sB, &tmB, &full_bar[stage], k, ti.n0, ti.g);
              else
                tma_load_2d(sB, &tmB, &full_bar[stage], k, ti.n0);
            } else {
#pragma unroll
              for (int i = 0; i < BN / 64; ++i) {
                if (MODE == GEMM_GROUPED_M)
                  tma_load_3d(sB + i * kSwizzleChunk, &tmB, &full_bar[stage], ti.n0 + 64 * i, k, ti.g);
                else
                  tma_load_2d(sB + i * kSwizzleChunk, &tmB, &full_bar[stage], ti.n0 + 64 * i, k);
              }
            }
          }
          if (++stage == S) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------ MMA issuer --------------------------------
    if (lane == 0 && leader) {
      constexpr uint32_t idesc = umma_idesc_f16(TM, BN, A_MN, B_MN, true);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int t = tile0; t < ntiles && ok; t += tile_step) {
        const TileInfo ti = tile_info<BN, MODE, TM>(p, t, s_off);
        if (!mbar_wait(&tempty_bar[acc], acc_phase ^ 1, p.status, STATUS_TIMEOUT_TMEM_EMPTY)) break;
        tc_fence_after();
        const uint32_t tmem_d = tmem_base + acc * BN;
        for (int kb = 0; kb < ti.num_kb; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase, p.status, STATUS_TIMEOUT_TMA_FULL)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + stage * C_::kStageBytes);
          const uint32_t b_addr = a_addr + C_::kStageA;
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            const uint64_t adesc = A_MN ? umma_desc_sw128(a_addr + kk * 2048, kSwizzleChunk, 1024)
                                        : umma_desc_sw128(a_addr + kk * 32, 16, 1024);
            const uint64_t bdesc = B_MN ? umma_desc_sw128(b_addr + kk * 2048, kSwizzleChunk, 1024)
                                        : umma_desc_sw128(b_addr + kk * 32, 16, 1024);
            if constexpr (PAIR)
              tc_mma_f16_pair(tmem_d, adesc, bdesc, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
            else
              tc_mma_f16(tmem_d, adesc, bdesc, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
          }
          if constexpr (PAIR) tc_commit_pair(&empty_bar[stage], 0x3); else tc_commit(&empty_bar[stage]);
          if (++stage == S) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        if constexpr (PAIR) tc_commit_pair(&tfull_bar[acc], 0x3); else tc_commit(&tfull_bar[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
      // Drain: wait for every MMA this thread issued before TMEM is released.
      if constexpr (PAIR) tc_commit_pair(drain_bar, 0x1); else tc_commit(drain_bar);
      mbar_wait(drain_bar, 0, p.status, STATUS_TIMEOUT_DRAIN);
    }
  } else {
    // ------------------------------ Epilogue ----------------------------------
    const int quarter = warp & 3;  // TMEM lane quarter this warp may access
    const int row_in_tile = (int)crank * kBM + quarter * 32 + lane;
    EpiStage stg{epi_smem + (warp - 2) * 2 * C_::kEpiBox, 0};
    uint64_t* wbar = in_bar + (warp - 2) * 2;  // this warp's two box-load barriers
    uint32_t in_phase = 0;                     // bit b: parity of box b's next load completion
    int in_box = 0;                            // box of the next side-input chunk
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = tile0; t < ntiles; t += tile_step) {
      const TileInfo ti = tile_info<BN, MODE, TM>(p, t, s_off);
      const int y0 = ti.m0 + (int)crank * kBM + quarter * 32;  // first row of this warp's 32
      // Side-input epilogue, one box (32 rows x 64 bf16 columns) per chunk: the box of R (or
      // H) is loaded by TMA into shared memory one chunk ahead, combined with the
      // accumulator in place and stored back out with TMA.  The residual chunk is 64
      // accumulator columns; the SwiGLU-backward chunk is 32 dAct columns, whose H / dH
      // columns (gate 32 | up 32) fill one box.  The whole tile's side input is requested
      // into L2, and the first box into shared memory, before the accumulator is ready.
      constexpr int kChunk = EPI == EPI_SWIGLU_BWD ? 32 : 64;
      int nvalid = 0;
      if (kTmaIn && p.tma_c && y0 < p.rows_c && y0 < ti.m_limit && ti.n0 < p.N)
        nvalid = min(BN / kChunk, (p.N - ti.n0 + kChunk - 1) / kChunk);
      auto box_x = [&](int c) { return EPI == EPI_SWIGLU_BWD ? 2 * (ti.n0 + c * kChunk) : ti.n0 + c * kChunk; };
      auto load_box = [&](int c, int b) {
        if (lane == 0) {
          bulk_wait_group_read<0>();  // the store that last used this box has read it
          mbar_arrive_expect_tx(&wbar[b], C_::kEpiBox);
          tma_load_2d(stg.base + b * C_::kEpiBox, &tmH, &wbar[b], box_x(c), y0);
        }
        __syncwarp();
      };
      if (kTmaIn && nvalid > 0) {
        if (lane == 0)
          for (int c = 1; c < nvalid; ++c) tma_prefetch_l2_2d(&tmH, box_x(c), y0);
        load_box(0, in_box);
      }
      if (!mbar_wait(&tfull_bar[acc], acc_phase, p.status, STATUS_TIMEOUT_TMEM_FULL)) break;
      tc_fence_after();
      const int row = ti.m0 + row_in_tile;
      const bool row_ok = row < ti.m_limit;
      const uint32_t tbase = tmem_base + acc * BN + ((uint32_t)(quarter * 32) << 16);
      const bool zero = ti.num_kb == 0;
      if (kTmaIn && p.tma_c) {
#pragma unroll 1
        for (int c = 0; c < nvalid; ++c) {
          const int b = (in_box + c) & 1;
          if (c + 1 < nvalid) load_box(c + 1, b ^ 1);
          float v[kChunk];
          tmem_ld32(tbase + c * kChunk, v);
          if constexpr (kChunk == 64) tmem_ld32(tbase + c * kChunk + 32, v + 32);
          tc_wait_ld();
          if (!mbar_wait(&wbar[b], (in_phase >> b) & 1u, p.status, STATUS_TIMEOUT_TMA_FULL)) break;
          in_phase ^= 1u << b;
          uint8_t* box = stg.base + b * C_::kEpiBox + lane * 128;
          uint32_t w[32];
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const uint4 r4 = *reinterpret_cast<const uint4*>(box + ((q ^ (lane & 7)) << 4));
            w[4 * q] = r4.x;
            w[4 * q + 1] = r4.y;
            w[4 * q + 2] = r4.z;
            w[4 * q + 3] = r4.w;
          }
          if (EPI == EPI_ADD_BF16) {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const float a0 = zero ? 0.f : v[2 * j] * p.alpha, a1 = zero ? 0.f : v[2 * j + 1] * p.alpha;
              w[j] = pack_bf16x2(a0 + bf16_lo(w[j]), a1 + bf16_hi(w[j]));
            }
          } else {
            // w[0..16) = gate (32 values), w[16..32) = up; out: dgate | dup
            uint32_t o[32];
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              float r[2], sgl[2];
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                const float g = h ? bf16_hi(w[j]) : bf16_lo(w[j]);
                const float u = h ? bf16_hi(w[16 + j]) : bf16_lo(w[16 + j]);
                const float d = zero ? 0.f : v[2 * j + h] * p.alpha;
                const float sg = __fdividef(1.0f, 1.0f + __expf(-g));
                sgl[h] = d * g * sg;                              // d/du
                r[h] = d * u * (sg * (1.0f + g * (1.0f - sg)));  // d/dg
              }
              o[j] = pack_bf16x2(r[0], r[1]);
              o[16 + j] = pack_bf16x2(sgl[0], sgl[1]);
            }
#pragma unroll
            for (int j = 0; j < 32; ++j) w[j] = o[j];
          }
#pragma unroll
          for (int q = 0; q < 8; ++q)
            *reinterpret_cast<uint4*>(box + ((q ^ (lane & 7)) << 4)) =
                make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tmC, stg.base + b * C_::kEpiBox, box_x(c), y0);
            bulk_commit_group();
          }
        }
        in_box = (in_box + nvalid) & 1;
      } else if (kTmaEpi && p.tma_c) {
        // whole-box stores; a box that starts past the last row or column is skipped, one
        // that overhangs is clipped by the tensor map
        const bool rows_ok = y0 < p.rows_c && y0 < ti.m_limit;
        if (EPI == EPI_STORE_BF16) {
#pragma unroll 1
          for (int c = 0; c < BN / 64; ++c) {
            float v[64];
            tmem_ld32(tbase + c * 64, v);
            tmem_ld32(tbase + c * 64 + 32, v + 32);
            tc_wait_ld();
            const int x = ti.n0 + c * 64;
            if (!rows_ok || x >= p.N) continue;
            uint32_t w[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) w[j] = zero ? 0u : pack_bf16x2(v[2 * j] * p.alpha, v[2 * j + 1] * p.alpha);
            uint8_t* box = stg.acquire(lane);
            EpiStage::put_row(box, lane, w);
            if (MODE == GEMM_GROUPED_K)
              stg.issue_3d(lane, &tmC, x, y0, ti.g);
            else
              stg.issue_2d(lane, &tmC, x, y0);
          }
        } else {
          // SwiGLU: two 64-column accumulator blocks (gate 32 | up 32 each) make 64 activation
          // columns; the raw blocks are the saved pre-activation H
#pragma unroll 1
          for (int c = 0; c < BN / 64; c += 2) {
            uint32_t act[32];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              float gt[32], up[32];
              tmem_ld32(tbase + (c + h) * 64, gt);
              tmem_ld32(tbase + (c + h) * 64 + 32, up);
              tc_wait_ld();
#pragma unroll
              for (int j = 0; j < 16; ++j)
                act[16 * h + j] = pack_bf16x2(silu_f(gt[2 * j]) * up[2 * j], silu_f(gt[2 * j + 1]) * up[2 * j + 1]);
              const int xh = ti.n0 + (c + h) * 64;
              if (p.H != nullptr && rows_ok && xh < p.N) {
                uint32_t w[32];
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                  w[j] = pack_bf16x2(gt[2 * j], gt[2 * j + 1]);
                  w[16 + j] = pack_bf16x2(up[2 * j], up[2 * j + 1]);
                }
                uint8_t* box = stg.acquire(lane);
                EpiStage::put_row(box, lane, w);
                stg.issue_2d(lane, &tmH, xh, y0);
              }
            }
            const int xa = (ti.n0 + c * 64) >> 1;
            if (rows_ok && 2 * xa < p.N) {
              uint8_t* box = stg.acquire(lane);
              EpiStage::put_row(box, lane, act);
              stg.issue_2d(lane, &tmC, xa, y0);
            }
          }
        }
      } else if (EPI == EPI_SWIGLU) {
#pragma unroll 1
        for (int c = 0; c < BN / 64; ++c) {
          float gt[32], up[32];
          tmem_ld32(tbase + c * 64, gt);
          tmem_ld32(tbase + c * 64 + 32, up);
          tc_wait_ld();
          store_swiglu(p, row, ti.n0 + c * 64, gt, up, row_ok);
        }
      } else if (EPI == EPI_EP_PUSH) {
        // Rows go to different ranks' slots: each 32 x 64 chunk is transposed through this warp's
        // shared-memory box so that every store instruction writes four whole 128-byte row
        // segments (eight lanes per row) instead of 32 scattered 16-byte pieces (small writes
        // waste most of an NVLink packet).
        int4 m = make_int4(0, -1, 0, 0);
        if (row_ok) m = p.row_meta[row];
        const bool valid = m.y >= 0 && m.y < p.nsrc && m.z >= 0 && m.z < p.src_rows;
        if (row_ok && m.y >= 0 && !valid) report_error(p.status, STATUS_BAD_INDEX, m.z);
        const unsigned long long rp =
            valid ? reinterpret_cast<unsigned long long>(reinterpret_cast<__nv_bfloat16*>(p.peer_c[m.y]) +
                                                         (long long)m.z * p.ldc)
                  : 0ull;
        uint8_t* box = stg.base;
#pragma unroll 1
        for (int c = 0; c < BN / 64; ++c) {
          float a[32], b[32];
          tmem_ld32(tbase + c * 64, a);
          tmem_ld32(tbase + c * 64 + 32, b);
          tc_wait_ld();
          uint32_t w[32];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            w[j] = zero ? 0u : pack_bf16x2(a[2 * j] * p.alpha, a[2 * j + 1] * p.alpha);
            w[16 + j] = zero ? 0u : pack_bf16x2(b[2 * j] * p.alpha, b[2 * j + 1] * p.alpha);
          }
          __syncwarp();                       // the previous chunk's reads of the box are done
          EpiStage::put_row(box, lane, w);
          __syncwarp();
          const int col0 = ti.n0 + c * 64;
#pragma unroll
          for (int pass = 0; pass < 8; ++pass) {
            const int r = pass * 4 + (lane >> 3), q = lane & 7;
            const unsigned long long dst = __shfl_sync(0xffffffffu, rp, r);
            const int colq = col0 + q * 8;
            if (dst != 0ull && colq < p.N) {
              const uint4 v = *reinterpret_cast<const uint4*>(box + r * 128 + ((q ^ (r & 7)) << 4));
              *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(dst) + colq) = v;
            }
          }
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          float v[32];
          tmem_ld32(tbase + c * 32, v);
          tc_wait_ld();
          if (zero) {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = 0.f;
          }
          if (EPI == EPI_SWIGLU_BWD)
            store_swiglu_bwd(p, row, ti.n0 + c * 32, v, row_ok);
          else
            store_chunk<EPI>(p, row, ti.n0 + c * 32, ti.g, v, row_ok);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (PAIR && !leader)
          mbar_arrive_cluster(mapa_shared(smem_u32(&tempty_bar[acc]), 0));
        else
          mbar_arrive(&tempty_bar[acc]);
      }
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
    if ((kTmaEpi || kTmaIn) && p.tma_c && lane == 0) bulk_wait_group_all();
  }

  __syncwarp();
  tc_fence_before();
  // A pair stays resident until the leader's MMAs (which read the peer's shared memory
  // and write its tensor memory) have drained.
  if constexpr (PAIR) cluster_sync_all(); else __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    if constexpr (PAIR) tmem_dealloc_pair(tmem_base, C_::kTmemCols); else tmem_dealloc(tmem_base, C_::kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (fn == nullptr) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || ptr == nullptr)
      throw std::runtime_error("omnicoder: cuTensorMapEncodeTiled entry point not available");
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

// rank-2 or rank-3 bf16 tensor map with 128-byte swizzle.  dims[0] is the
// contiguous dimension; strides are in bytes for dims 1.. .
static CUtensorMap make_tmap_sw128(const void* base, CUtensorMapDataType dtype, int rank, const uint64_t* dims,
                                   const uint64_t* strides_bytes, const uint32_t* box);

CUtensorMap make_tmap_bf16_sw128(const void* base, int rank, const uint64_t* dims, const uint64_t* strides_bytes,
                                 const uint32_t* box) {
  return make_tmap_sw128(base, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, dims, strides_bytes, box);
}

CUtensorMap make_tmap_u8_sw128(const void* base, int rank, const uint64_t* dims, const uint64_t* strides_bytes,
                               const uint32_t* box) {
  return make_tmap_sw128(base, CU_TENSOR_MAP_DATA_TYPE_UINT8, rank, dims, strides_bytes, box);
}

static CUtensorMap make_tmap_sw128(const void* base, CUtensorMapDataType dtype, int rank, const uint64_t* dims,
                                   const uint64_t* strides_bytes, const uint32_t* box) {
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0)
    throw std::runtime_error("omnicoder gemm: operand base address must be 16-byte aligned");
  for (int i = 0; i + 1 < rank; ++i)
    if (strides_bytes[i] % 16 != 0)
      throw std::runtime_error("omnicoder gemm: operand row stride must be a multiple of 16 bytes");
  CUtensorMap m;
  cuuint64_t d[3], s[2];
  cuuint32_t b[3], es[3] = {1, 1, 1};
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
  }
  for (int i = 0; i + 1 < rank; ++i) s[i] = strides_bytes[i];
  CUresult r = encode_fn()(&m, dtype, rank, const_cast<void*>(base), d, s, b, es,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("omnicoder gemm: cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
  return m;
}

int num_sms() {
  static int n = 0;
  if (n == 0) {
    int dev;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

template <int BN, bool A_MN, bool B_MN, int EPI, int MODE, bool PAIR = false>
static void launch_impl(const GemmDesc& d, cudaStream_t stream) {
  using C_ = Cfg<BN, PAIR>;
  auto kern = gemm_sm100_kernel<BN, A_MN, B_MN, EPI, MODE, PAIR>;
  ensure_smem_attr(reinterpret_cast<const void*>(kern), C_::kSmemBytes);
  // A operand tensor map(s).
  CUtensorMap tmA, tmB;
  AgMaps ag;
  memset(&ag, 0, sizeof(ag));
  memset(&tmA, 0, sizeof(tmA));
  if (MODE == GEMM_AG) {
    for (int r = 0; r < d.nsrc; ++r) {
      uint64_t dims[2] = {(uint64_t)d.K_extent_a, (uint64_t)d.src_rows};
      uint64_t str[1] = {(uint64_t)d.lda * 2};
      uint32_t box[2] = {64, 128};
      ag.m[r] = make_tmap_bf16_sw128(d.peer_a[r], 2, dims, str, box);
    }
  } else {
    if (!A_MN) {  // A stored [rowsA, K] with row stride lda
      uint64_t dims[2] = {(uint64_t)d.K_extent_a, (uint64_t)d.rows_a};
      uint64_t str[1] = {(uint64_t)d.lda * 2};
      uint32_t box[2] = {64, 128};
      tmA = make_tmap_bf16_sw128(d.A, 2, dims, str, box);
    } else {      // A stored [K, M] with row stride lda
      uint64_t dims[2] = {(uint64_t)d.M, (uint64_t)d.K_extent_a};
      uint64_t str[1] = {(uint64_t)d.lda * 2};
      uint32_t box[2] = {64, 64};
      tmA = make_tmap_bf16_sw128(d.A, 2, dims, str, box);
    }
  }
  {
    if (!B_MN) {  // B stored [N, K] (per group when grouped-M)
      if (MODE == GEMM_GROUPED_M) {
        uint64_t dims[3] = {(uint64_t)d.K, (uint64_t)d.N, (uint64_t)d.num_groups};
        uint64_t str[2] = {(uint64_t)d.ldb * 2, (uint64_t)d.b_group_stride * 2};
        uint32_t box[3] = {64, (uint32_t)BN, 1};
        tmB = make_tmap_bf16_sw128(d.B, 3, dims, str, box);
      } else {
        uint64_t dims[2] = {(uint64_t)d.K_extent_b, (uint64_t)d.N};
        uint64_t str[1] = {(uint64_t)d.ldb * 2};
        uint32_t box[2] = {64, (uint32_t)C_::kBNc};
        tmB = make_tmap_bf16_sw128(d.B, 2, dims, str, box);
      }
    } else {      // B stored [K, N]
      if (MODE == GEMM_GROUPED_M) {
        uint64_t dims[3] = {(uint64_t)d.N, (uint64_t)d.K, (uint64_t)d.num_groups};
        uint64_t str[2] = {(uint64_t)d.ldb * 2, (uint64_t)d.b_group_stride * 2};
        uint32_t box[3] = {64, 64, 1};
        tmB = make_tmap_bf16_sw128(d.B, 3, dims, str, box);
      } else {
        uint64_t dims[2] = {(uint64_t)d.N, (uint64_t)d.K_extent_b};
        uint64_t str[1] = {(uint64_t)d.ldb * 2};
        uint32_t box[2] = {64, 64};
        tmB = make_tmap_bf16_sw128(d.B, 2, dims, str, box);
      }
    }
  }
  // Output tensor maps for the shared-memory + TMA-store epilogue (bf16 outputs whose base
  // and row stride are 16-byte aligned; otherwise the epilogue stores rows directly).
  constexpr bool kTmaEpi = EPI == EPI_STORE_BF16 || EPI == EPI_SWIGLU;
  constexpr bool kTmaIn = EPI == EPI_ADD_BF16 || EPI == EPI_SWIGLU_BWD;
  CUtensorMap tmC, tmH;
  memset(&tmC, 0, sizeof(tmC));
  memset(&tmH, 0, sizeof(tmH));
  const long long rows_c = d.rows_c > 0 ? d.rows_c : d.M;
  int tma_c = 0;
  static const bool tma_epi_on = [] {
    const char* e = getenv("OMNI_GEMM_TMA_EPI");  // "0": rows stored directly from registers
    return !(e != nullptr && e[0] == '0');
  }();
  if (kTmaIn && tma_epi_on && MODE != GEMM_GROUPED_K && d.R != nullptr) {
    // side-input epilogues: R / H read and C written as [rows, cols] bf16 boxes
    const long long cols = EPI == EPI_SWIGLU_BWD ? 2LL * d.N : d.N;
    uint32_t box[2] = {64, 32};
    uint64_t cd[2] = {(uint64_t)cols, (uint64_t)rows_c};
    uint64_t cs[1] = {(uint64_t)d.ldc * 2};
    uint64_t rs[1] = {(uint64_t)d.ldr * 2};
    tmC = make_tmap_bf16_sw128(d.C, 2, cd, cs, box);
    tmH = make_tmap_bf16_sw128(d.R, 2, cd, rs, box);
    tma_c = 1;
  }
  if (kTmaEpi && tma_epi_on) {
    auto al16 = [](const void* ptr, long long ld) {
      return ptr != nullptr && (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0 && (ld * 2) % 16 == 0;
    };
    const long long cols_c = EPI == EPI_SWIGLU ? d.N / 2 : d.N;
    bool ok = al16(d.C, d.ldc) && (MODE != GEMM_GROUPED_K || (d.c_group_stride * 2) % 16 == 0);
    if (EPI == EPI_SWIGLU && d.H != nullptr) ok = ok && al16(d.H, d.ldh);
    if (ok) {
      uint32_t box[3] = {64, 32, 1};
      if (MODE == GEMM_GROUPED_K) {
        uint64_t dims[3] = {(uint64_t)cols_c, (uint64_t)rows_c, (uint64_t)d.num_groups};
        uint64_t str[2] = {(uint64_t)d.ldc * 2, (uint64_t)d.c_group_stride * 2};
        tmC = make_tmap_bf16_sw128(d.C, 3, dims, str, box);
      } else {
        uint64_t dims[2] = {(uint64_t)cols_c, (uint64_t)rows_c};
        uint64_t str[1] = {(uint64_t)d.ldc * 2};
        tmC = make_tmap_bf16_sw128(d.C, 2, dims, str, box);
        if (EPI == EPI_SWIGLU && d.H != nullptr) {
          uint64_t hd[2] = {(uint64_t)d.N, (uint64_t)rows_c};
          uint64_t hs[1] = {(uint64_t)d.ldh * 2};
          tmH = make_tmap_bf16_sw128(d.H, 2, hd, hs, box);
        }
      }
      tma_c = 1;
    }
  }
  GemmArgs p;
  p.tma_c = tma_c;
  p.rows_c = (int)rows_c;
  p.M = d.M;
  p.N = d.N;
  p.K = d.K;
  p.num_groups = d.num_groups;
  p.group_offsets = d.group_offsets;
  p.C = d.C;
  p.ldc = d.ldc;
  p.c_group_stride = d.c_group_stride;
  p.R = d.R;
  p.ldr = d.ldr;
  p.H = d.H;
  p.ldh = d.ldh;
  p.alpha = d.alpha;
  p.status = reinterpret_cast<StatusBlock*>(d.status);
  p.nsrc = d.nsrc;
  p.me = d.me;
  p.src_rows = d.src_rows > 0 ? d.src_rows : 1;
  p.mt_rot = 0;
  for (int r = 0; r < GEMM_MAX_PEERS; ++r) p.peer_c[r] = d.peer_c[r];
  p.row_meta = reinterpret_cast<const int4*>(d.row_meta);
  p.ready = d.ready;
  p.ready_epoch = d.ready_epoch;
  p.src_pref = d.src_pref;
  if (MODE == GEMM_AG) {
    p.mt_rot = d.me * (d.src_rows / kBM);               // start on this rank's own rows
  } else if (EPI == EPI_PEER_BF16) {
    p.mt_rot = ((d.me + 1) % d.nsrc) * (d.src_rows / kBM);  // peers' rows first, own rows last
  }
  constexpr int TM = C_::kTM;
  // persistent grid: one CTA (pair) per SM (pair of SMs), no more than there are tiles
  int grid = num_sms();
  if constexpr (PAIR) {
    static int max_pairs = 0;  // co-resident clusters of two for this kernel
    if (max_pairs == 0) {
      cudaLaunchConfig_t q = {};
      q.gridDim = dim3(2 * num_sms());
      q.blockDim = dim3(kThreads);
      q.dynamicSmemBytes = C_::kSmemBytes;
      cudaLaunchAttribute qa[1];
      qa[0].id = cudaLaunchAttributeClusterDimension;
      qa[0].val.clusterDim.x = 2;
      qa[0].val.clusterDim.y = 1;
      qa[0].val.clusterDim.z = 1;
      q.attrs = qa;
      q.numAttrs = 1;
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, kern, &q) != cudaSuccess || n < 1) {
        (void)cudaGetLastError();
        n = num_sms() / 2;
      }
      max_pairs = n;
    }
    grid = max_pairs;
  }
  if (MODE == GEMM_DENSE || MODE == GEMM_AG) {
    const int tiles = ((d.M + TM - 1) / TM) * ((d.N + BN - 1) / BN);
    grid = tiles < grid ? tiles : grid;
  } else if (MODE == GEMM_GROUPED_K) {
    const int tiles = d.num_groups * ((d.M + TM - 1) / TM) * ((d.N + BN - 1) / BN);
    grid = tiles < grid ? tiles : grid;
  } else if (d.max_rows_hint > 0) {
    const int tiles = (d.max_rows_hint / kBM) * ((d.N + BN - 1) / BN);
    grid = tiles < grid ? tiles : grid;
  }
  if (grid < 1) grid = 1;
  if constexpr (PAIR) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = C_::kSmemBytes;
    cfg.stream = stream;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = 2;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, tmA, tmB, ag, tmC, tmH, p);
    if (e != cudaSuccess) throw std::runtime_error(std::string("omnicoder gemm: pair launch failed: ") + cudaGetErrorString(e));
  } else {
    kern<<<grid, kThreads, C_::kSmemBytes, stream>>>(tmA, tmB, ag, tmC, tmH, p);
  }
}

// CTA-pair tiles are used for large dense and grouped-K problems (and can be switched off
// with set_gemm_pair(false), or OMNI_GEMM_PAIR=0, for comparisons).
static int g_pair_mode = -1;  // -1: read the environment on first use
void set_gemm_pair(bool on) { g_pair_mode = on ? 1 : 0; }
bool gemm_pair_enabled() {
  if (g_pair_mode < 0) {
    const char* e = getenv("OMNI_GEMM_PAIR");
    g_pair_mode = (e != nullptr && e[0] == '0') ? 0 : 1;
  }
  return g_pair_mode == 1;
}

template <int EPI, int MODE>
constexpr bool pair_supported() {
  return (MODE == GEMM_DENSE || MODE == GEMM_GROUPED_K) && EPI != EPI_PEER_BF16;
}

template <bool A_MN, bool B_MN, int EPI, int MODE>
static void dispatch_bn(const GemmDesc& d, cudaStream_t s) {
  if (d.block_n == 128) {
    launch_impl<128, A_MN, B_MN, EPI, MODE>(d, s);
    return;
  }
  if constexpr (pair_supported<EPI, MODE>()) {
    const bool pair = d.pair == 1 || (d.pair < 0 && gemm_pair_enabled() && d.M > kBM);
    if (pair) {
      launch_impl<256, A_MN, B_MN, EPI, MODE, true>(d, s);
      return;
    }
  }
  launch_impl<256, A_MN, B_MN, EPI, MODE>(d, s);
}

// Epilogue / layout combinations that training actually uses; others are
// rejected so the number of kernel instantiations stays small.
template <bool A_MN, bool B_MN, int EPI, int MODE>
constexpr bool combo_supported() {
  if (MODE == GEMM_AG) return !A_MN && (EPI == EPI_STORE_BF16 || (EPI == EPI_SWIGLU && !B_MN));
  if (EPI == EPI_PEER_BF16) return !A_MN && MODE == GEMM_DENSE;
  if (EPI == EPI_EP_PUSH) return !A_MN && MODE == GEMM_GROUPED_M;
  if (EPI == EPI_SWIGLU) return !A_MN && !B_MN && MODE != GEMM_GROUPED_K;
  if (EPI == EPI_SWIGLU_BWD) return !A_MN && B_MN && MODE != GEMM_GROUPED_K;
  if (EPI == EPI_ADD_BF16) return !A_MN && MODE == GEMM_DENSE;
  if (EPI == EPI_STORE_F32) return (A_MN && B_MN) || (!A_MN && !B_MN && MODE == GEMM_DENSE);
  if (EPI == EPI_ACCUM_F32) return A_MN && B_MN;
  return true;
}

template <bool A_MN, bool B_MN, int EPI, int MODE>
static void dispatch_checked(const GemmDesc& d, cudaStream_t s) {
  if constexpr (combo_supported<A_MN, B_MN, EPI, MODE>()) {
    dispatch_bn<A_MN, B_MN, EPI, MODE>(d, s);
  } else {
    throw std::runtime_error("omnicoder gemm: unsupported epilogue/layout/mode combination");
  }
}

template <bool A_MN, bool B_MN, int MODE>
static void dispatch_epi(const GemmDesc& d, cudaStream_t s) {
  switch (d.epilogue) {
    case EPI_STORE_BF16: dispatch_checked<A_MN, B_MN, EPI_STORE_BF16, MODE>(d, s); break;
    case EPI_STORE_F32: dispatch_checked<A_MN, B_MN, EPI_STORE_F32, MODE>(d, s); break;
    case EPI_ACCUM_F32: dispatch_checked<A_MN, B_MN, EPI_ACCUM_F32, MODE>(d, s); break;
    case EPI_ADD_BF16: dispatch_checked<A_MN, B_MN, EPI_ADD_BF16, MODE>(d, s); break;
    case EPI_SWIGLU: dispatch_checked<A_MN, B_MN, EPI_SWIGLU, MODE>(d, s); break;
    case EPI_SWIGLU_BWD: dispatch_checked<A_MN, B_MN, EPI_SWIGLU_BWD, MODE>(d, s); break;
    case EPI_PEER_BF16: dispatch_checked<A_MN, B_MN, EPI_PEER_BF16, MODE>(d, s); break;
    case EPI_EP_PUSH: dispatch_checked<A_MN, B_MN, EPI_EP_PUSH, MODE>(d, s); break;
    default: throw std::runtime_error("omnicoder gemm: unknown epilogue");
  }
}

// out[r, :] = sum over slots s of staging[s, r, :] (+ residual[r, :]), fp32 sums, bf16 out; one thread per
// 8 columns.  The second half of a fused GEMM -> reduce-scatter: every rank stored its partial rows here.
__global__ void tp_reduce_kernel(const __nv_bfloat16* __restrict__ st, int nsrc, int rows, int D, long long ld,
                                 const __nv_bfloat16* __restrict__ res, long long ldr, __nv_bfloat16* __restrict__ out,
                                 long long ldo) {
  const int chunks = D / 8;
  const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  if (i >= (long long)rows * chunks) return;
  const int r = (int)(i / chunks), c = (int)(i - (long long)r * chunks) * 8;
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  for (int s = 0; s < nsrc; ++s) {
    const uint4 v = *reinterpret_cast<const uint4*>(st + ((long long)s * rows + r) * ld + c);
    const uint32_t* w = reinterpret_cast<const uint32_t*>(&v);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      acc[2 * j] += bf16_lo(w[j]);
      acc[2 * j + 1] += bf16_hi(w[j]);
    }
  }
  if (res != nullptr) {
    const uint4 v = *reinterpret_cast<const uint4*>(res + (long long)r * ldr + c);
    const uint32_t* w = reinterpret_cast<const uint32_t*>(&v);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      acc[2 * j] += bf16_lo(w[j]);
      acc[2 * j + 1] += bf16_hi(w[j]);
    }
  }
  *reinterpret_cast<uint4*>(out + (long long)r * ldo + c) =
      make_uint4(pack_bf16x2(acc[0], acc[1]), pack_bf16x2(acc[2], acc[3]), pack_bf16x2(acc[4], acc[5]),
                 pack_bf16x2(acc[6], acc[7]));
}

void tp_reduce_slots(const void* staging, int nsrc, int rows, int D, long long ld, const void* residual,
                     long long ldr, void* out, long long ldo, cudaStream_t s) {
  if (D % 8 != 0) throw std::runtime_error("tp reduce: D % 8");
  const long long work = (long long)rows * (D / 8);
  if (work == 0) return;
  tp_reduce_kernel<<<(unsigned)((work + 255) / 256), 256, 0, s>>>(
      (const __nv_bfloat16*)staging, nsrc, rows, D, ld, (const __nv_bfloat16*)residual, ldr, (__nv_bfloat16*)out, ldo);
}

void gemm_sm100_launch(const GemmDesc& d, cudaStream_t stream) {
  // The epilogues move 16-byte vectors (or 16-byte-aligned TMA boxes): every output / residual
  // row must start on a 16-byte boundary.
  {
    const int c_elem = (d.epilogue == EPI_STORE_F32 || d.epilogue == EPI_ACCUM_F32) ? 4 : 2;
    auto aligned = [](const void* ptr, long long ld, int elem) {
      return ptr == nullptr || ((reinterpret_cast<uintptr_t>(ptr) & 15u) == 0 && (ld * elem) % 16 == 0);
    };
    if (d.epilogue != EPI_PEER_BF16 && d.epilogue != EPI_EP_PUSH && !aligned(d.C, d.ldc, c_elem))
      throw std::runtime_error("omnicoder gemm: output base and row stride must be 16-byte aligned");
    if (d.mode == GEMM_GROUPED_K && (d.c_group_stride * c_elem) % 16 != 0)
      throw std::runtime_error("omnicoder gemm: output group stride must be 16-byte aligned");
    if (!aligned(d.R, d.ldr, 2) || !aligned(d.H, d.ldh, 2))
      throw std::runtime_error("omnicoder gemm: residual / pre-activation rows must be 16-byte aligned");
  }
  if (d.epilogue == EPI_PEER_BF16 &&
      (d.nsrc < 1 || d.nsrc > GEMM_MAX_PEERS || d.src_rows <= 0 || d.src_rows % kBM != 0 || d.M != d.nsrc * d.src_rows))
    throw std::runtime_error("omnicoder gemm: peer-store epilogue needs M = ranks x src_rows, src_rows % 128 == 0");
  if (d.ready != nullptr && (d.mode != GEMM_GROUPED_M || d.a_mn_major || d.ready_epoch == nullptr ||
                            d.src_pref == nullptr || d.nsrc < 1 || d.nsrc > 32))
    throw std::runtime_error("omnicoder gemm: readiness gating needs grouped-M, K-major A, an epoch and prefixes");
  if (d.epilogue == EPI_EP_PUSH &&
      (d.row_meta == nullptr || d.nsrc < 1 || d.nsrc > GEMM_MAX_PEERS || d.src_rows <= 0 || d.ldc % 8 != 0))
    throw std::runtime_error("omnicoder gemm: expert push epilogue needs row metadata, 1..8 ranks, rows and ldc % 8");
  if (d.num_groups > GEMM_MAX_GROUPS) throw std::runtime_error("omnicoder gemm: too many groups");
  if (d.K % 8 != 0 && !(d.mode == GEMM_GROUPED_K)) throw std::runtime_error("omnicoder gemm: K must be a multiple of 8");
  const int combo = (d.a_mn_major ? 2 : 0) | (d.b_mn_major ? 1 : 0);
  switch (d.mode) {
    case GEMM_DENSE:
      if (combo == 0) dispatch_epi<false, false, GEMM_DENSE>(d, stream);
      else if (combo == 1) dispatch_epi<false, true, GEMM_DENSE>(d, stream);
      else if (combo == 3) dispatch_epi<true, true, GEMM_DENSE>(d, stream);
      else throw std::runtime_error("omnicoder gemm: unsupported major combination");
      break;
    case GEMM_GROUPED_M:
      if (combo == 0) dispatch_epi<false, false, GEMM_GROUPED_M>(d, stream);
      else if (combo == 1) dispatch_epi<false, true, GEMM_GROUPED_M>(d, stream);
      else throw std::runtime_error("omnicoder gemm: unsupported major combination (grouped-M)");
      break;
    case GEMM_AG:
      if (d.nsrc < 1 || d.nsrc > GEMM_MAX_PEERS || d.src_rows <= 0 || d.src_rows % kBM != 0 ||
          d.M != d.nsrc * d.src_rows)
        throw std::runtime_error("omnicoder gemm: all-gather mode needs M = ranks x src_rows, src_rows % 128 == 0");
      if (combo == 0) dispatch_epi<false, false, GEMM_AG>(d, stream);
      else if (combo == 1) dispatch_epi<false, true, GEMM_AG>(d, stream);
      else throw std::runtime_error("omnicoder gemm: unsupported major combination (all-gather)");
      break;
    case GEMM_GROUPED_K:
      if (combo == 3) dispatch_epi<true, true, GEMM_GROUPED_K>(d, stream);
      else throw std::runtime_error("omnicoder gemm: grouped-K needs MN-major A and B");
      break;
    default:
      throw std::runtime_error("omnicoder gemm: unknown mode");
  }
}

}  // namespace omni
