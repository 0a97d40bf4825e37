// Split-KV decode attention (sm_100a): new query tokens against a KV cache.
//
//   q      [B, Tn, H, DQ]  bf16 (rotated)
//   k      [B, L, Hk, DQ]  bf16 or int8 (+ fp32 scale per (b, pos, kv head))
//   v      [B, L, Hk, DV]  bf16 or int8 (+ scale); MLA latent cache: v == nullptr,
//                          the value is the first DV dims of each key row
//   q_pos  [B, Tn] absolute positions; kv_len [B] number of cached tokens.
// Token position p lives in cache row sink_rows + p and is visible to query
// (b, t) when p < kv_len[b], p <= q_pos[b, t] and, with a window,
// p > q_pos[b, t] - window.  Rows [0, n_sink) hold compressed memory of tokens
// that left the window and are visible to every query.
//
// Kernel 1 (grid = B x Hk x splits, 256 threads): the CTA keeps the R = Tn * G
// query rows of one KV group (G = H / Hk heads; MLA: all heads share the
// latent) in shared memory and streams its share of the keys in tiles of 32
// through a cp.async double buffer.  Each key tile is read from HBM once for
// all R rows.  Scores: thread = (key, row group), the dot product walks the
// head dimension in 16-byte chunks starting at a key-dependent chunk so that
// the 8 threads of a quarter warp hit distinct shared-memory banks.  int8
// caches stay int8 in shared memory; the per-key scale multiplies the score
// (keys) or the probability (values).  Online softmax per row, O accumulates
// in registers (thread = 4 value columns x up to 32 rows).
// Kernel 2 merges the splits (log-sum-exp weights) and writes bf16.
//
// The reference decodes one token of one sequence at a time over a 16-slot
// latent window with ATen bmm + softmax (src/omnicoder/modeling/
// attention.py:1265-1612) and dequantises a u8/nf4 cache into a fresh tensor
// before every step (src/omnicoder/inference/generate.py:1630-1660).
#include <algorithm>
#include <stdexcept>
#include <type_traits>

#include <cuda_fp16.h>

#include "common.cuh"
#include "kernels.h"

namespace omni {

using bf16 = __nv_bfloat16;

namespace {

constexpr int kDecThreads = 256;
constexpr int kKT = 32;        // keys per tile
constexpr int kMaxRows = 64;   // Tn * heads-per-group
constexpr int kPvRows = 32;    // rows per thread in the P.V phase (upper bound)

struct DecArgs {
  const bf16* q;
  const void* k;
  const void* v;
  const float* ks;
  const float* vs;
  const int* q_pos;
  const int* kv_len;
  float* part_o;  // [B, Hk, splits, R, DV]
  float* part_ml;  // [B, Hk, splits, R, 2]
  int B, Tn, H, Hk, L, DQ, DV, window, splits;
  int sink_rows, n_sink;          // cache rows reserved before the tokens / how many of them are valid
  long long k_b, k_l, v_b, v_l;  // element strides of the caches (batch, position); head stride = DQ / DV
  long long s_b, s_l;            // scale strides (batch, position); head stride 1
  float scale;
};

template <typename KV>
struct KVTraits;
template <>
struct KVTraits<bf16> {
  static constexpr int kPerChunk = 8;  // elements per 16-byte chunk
  __device__ static void load4(const bf16* p, float* out) {
    const uint2 w = *reinterpret_cast<const uint2*>(p);
    out[0] = bf16_lo(w.x);
    out[1] = bf16_hi(w.x);
    out[2] = bf16_lo(w.y);
    out[3] = bf16_hi(w.y);
  }
};
template <>
struct KVTraits<int8_t> {
  static constexpr int kPerChunk = 16;
  __device__ static void load4(const int8_t* p, float* out) {
    const int w = *reinterpret_cast<const int*>(p);
    out[0] = (float)(signed char)(w & 0xff);
    out[1] = (float)(signed char)((w >> 8) & 0xff);
    out[2] = (float)(signed char)((w >> 16) & 0xff);
    out[3] = (float)(signed char)((w >> 24) & 0xff);
  }
};

// dot(q chunk (bf16, kPerChunk elems), k chunk (KV, 16 bytes))
__device__ __forceinline__ float dot_chunk(const bf16* q, const bf16* k) {
  const uint4 a = *reinterpret_cast<const uint4*>(q);
  const uint4 b = *reinterpret_cast<const uint4*>(k);
  const uint32_t* x = reinterpret_cast<const uint32_t*>(&a);
  const uint32_t* y = reinterpret_cast<const uint32_t*>(&b);
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) s += bf16_lo(x[j]) * bf16_lo(y[j]) + bf16_hi(x[j]) * bf16_hi(y[j]);
  return s;
}
__device__ __forceinline__ float dot_chunk(const bf16* q, const int8_t* k) {
  const uint4 a0 = *reinterpret_cast<const uint4*>(q);
  const uint4 a1 = *reinterpret_cast<const uint4*>(q + 8);
  const int4 b = *reinterpret_cast<const int4*>(k);
  const uint32_t* x0 = reinterpret_cast<const uint32_t*>(&a0);
  const uint32_t* x1 = reinterpret_cast<const uint32_t*>(&a1);
  const int* y = reinterpret_cast<const int*>(&b);
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int w = y[j];
    s += bf16_lo(x0[2 * j]) * (float)(signed char)(w & 0xff) + bf16_hi(x0[2 * j]) * (float)(signed char)((w >> 8) & 0xff) +
         bf16_lo(x0[2 * j + 1]) * (float)(signed char)((w >> 16) & 0xff) +
         bf16_hi(x0[2 * j + 1]) * (float)(signed char)((w >> 24) & 0xff);
  }
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int w = y[2 + j];
    s += bf16_lo(x1[2 * j]) * (float)(signed char)(w & 0xff) + bf16_hi(x1[2 * j]) * (float)(signed char)((w >> 8) & 0xff) +
         bf16_lo(x1[2 * j + 1]) * (float)(signed char)((w >> 16) & 0xff) +
         bf16_hi(x1[2 * j + 1]) * (float)(signed char)((w >> 24) & 0xff);
  }
  return s;
}

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem)), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_one() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

template <typename KV, bool LATENT>
__global__ void __launch_bounds__(kDecThreads, 1) decode_split_kernel(DecArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int b = blockIdx.x, g = blockIdx.y, split = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = a.H / a.Hk;
  const int R = a.Tn * G;
  const int DQ = a.DQ, DV = a.DV;
  constexpr int PC = KVTraits<KV>::kPerChunk;
  const int nchunk = DQ / PC;

  bf16* sQ = reinterpret_cast<bf16*>(smem);                                   // [R][DQ]
  KV* sK = reinterpret_cast<KV*>(smem + kMaxRows * DQ * 2);                    // 2 x [kKT][DQ]
  const int kTileBytes = kKT * DQ * (int)sizeof(KV);
  KV* sV = reinterpret_cast<KV*>(smem + kMaxRows * DQ * 2 + 2 * kTileBytes);   // 2 x [kKT][DV] (non-latent)
  const int vTileBytes = LATENT ? 0 : kKT * DV * (int)sizeof(KV);
  float* sP = reinterpret_cast<float*>(smem + kMaxRows * DQ * 2 + 2 * kTileBytes + 2 * vTileBytes);  // [R][kKT]
  float* sM = sP + kMaxRows * kKT;
  float* sL = sM + kMaxRows;
  float* sA = sL + kMaxRows;
  int* sPos = reinterpret_cast<int*>(sA + kMaxRows);

  // ---- queries of this group ----------------------------------------------
  for (int i = tid; i < R * (DQ / 8); i += kDecThreads) {
    const int r = i / (DQ / 8), c = i % (DQ / 8);
    const int t = r / G, h = g * G + r % G;
    const bf16* src = a.q + (((long long)b * a.Tn + t) * a.H + h) * DQ + c * 8;
    *reinterpret_cast<uint4*>(sQ + r * DQ + c * 8) = *reinterpret_cast<const uint4*>(src);
  }
  int pmin = 0x7fffffff, pmax = -1;
  for (int t = 0; t < a.Tn; ++t) {
    const int p = a.q_pos[b * a.Tn + t];
    pmin = min(pmin, p);
    pmax = max(pmax, p);
  }
  if (tid < R) {
    sPos[tid] = a.q_pos[b * a.Tn + tid / G];
    sM[tid] = -INFINITY;
    sL[tid] = 0.f;
  }
  // ---- key range of this split ----------------------------------------------
  // key tiles: first the always-visible memory rows [0, n_sink), then the token rows
  // sink_rows + [lo, hi) that the window and causality allow
  const int len = a.kv_len[b];
  const int hi = min(len, pmax + 1);
  const int lo = a.window > 0 ? max(0, pmin - a.window + 1) : 0;
  const int nsk = (a.n_sink + kKT - 1) / kKT;
  const int ntiles_all = nsk + (hi > lo ? (hi - lo + kKT - 1) / kKT : 0);
  const int per = (ntiles_all + a.splits - 1) / a.splits;
  const int t0 = split * per, t1 = min(ntiles_all, t0 + per);

  // P.V thread mapping
  const int colt = min(kDecThreads, DV / 4);
  const int rgroups = kDecThreads / colt;
  const int c4 = tid % colt, rg = tid / colt;
  const bool pv_active = rg < rgroups && c4 * 4 < DV;
  float acc[kPvRows][4];
#pragma unroll
  for (int i = 0; i < kPvRows; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;

  auto row_of = [&](int tile) { return tile < nsk ? tile * kKT : a.sink_rows + lo + (tile - nsk) * kKT; };
  auto issue = [&](int tile, int buf) {
    const int p0 = row_of(tile);
    KV* dk = sK + buf * (kKT * DQ);
    const int kchunks = DQ * (int)sizeof(KV) / 16;
    for (int i = tid; i < kKT * kchunks; i += kDecThreads) {
      const int kk = i / kchunks, c = i % kchunks;
      const int p = min(p0 + kk, a.L - 1);
      const KV* src = reinterpret_cast<const KV*>(a.k) + (long long)b * a.k_b + (long long)p * a.k_l + (long long)g * DQ;
      cp_async16(reinterpret_cast<uint8_t*>(dk + kk * DQ) + c * 16, reinterpret_cast<const uint8_t*>(src) + c * 16);
    }
    if (!LATENT) {
      KV* dv = sV + buf * (kKT * DV);
      const int vchunks = DV * (int)sizeof(KV) / 16;
      for (int i = tid; i < kKT * vchunks; i += kDecThreads) {
        const int kk = i / vchunks, c = i % vchunks;
        const int p = min(p0 + kk, a.L - 1);
        const KV* src = reinterpret_cast<const KV*>(a.v) + (long long)b * a.v_b + (long long)p * a.v_l + (long long)g * DV;
        cp_async16(reinterpret_cast<uint8_t*>(dv + kk * DV) + c * 16, reinterpret_cast<const uint8_t*>(src) + c * 16);
      }
    }
    cp_async_commit();
  };

  __syncthreads();
  if (t0 < t1) issue(t0, 0);
  for (int tile = t0; tile < t1; ++tile) {
    const int buf = (tile - t0) & 1;
    if (tile + 1 < t1) {
      issue(tile + 1, buf ^ 1);
      cp_async_wait_one();
    } else {
      cp_async_wait_all();
    }
    __syncthreads();
    const int p0 = row_of(tile);
    const bool sink_tile = tile < nsk;
    const KV* tK = sK + buf * (kKT * DQ);
    // ---- scores: thread = (key kk, rows rgs, rgs+8, ...) ---------------------
    {
      const int kk = lane, rgs = warp;
      const int p = p0 + kk;
      float s[kMaxRows / 8];
#pragma unroll
      for (int i = 0; i < kMaxRows / 8; ++i) s[i] = 0.f;
      const KV* krow = tK + kk * DQ;
      for (int st = 0; st < nchunk; ++st) {
        int c = st + kk;
        c = c >= nchunk ? c - nchunk : c;
        c = c >= nchunk ? c % nchunk : c;
#pragma unroll
        for (int i = 0; i < kMaxRows / 8; ++i) {
          const int r = rgs + 8 * i;
          if (r < R) s[i] += dot_chunk(sQ + r * DQ + c * PC, krow + c * PC);
        }
      }
      const float ksc = (a.ks != nullptr && p < a.L) ? a.ks[(long long)b * a.s_b + (long long)p * a.s_l + g] : 1.f;
#pragma unroll
      for (int i = 0; i < kMaxRows / 8; ++i) {
        const int r = rgs + 8 * i;
        if (r < R) {
          const int qp = sPos[r];
          const int tp = p - a.sink_rows;
          const bool ok = sink_tile ? (p < a.n_sink)
                                    : (tp < len && tp <= qp && (a.window <= 0 || tp > qp - a.window));
          sP[r * kKT + kk] = ok ? s[i] * ksc * a.scale : -INFINITY;
        }
      }
    }
    __syncthreads();
    // ---- online softmax (warp w: rows w, w+8, ...) ------------------------------
    {
      const int kk = lane;
      const int p = p0 + kk;
      const float vsc = (!LATENT && a.vs != nullptr && p < a.L)
                            ? a.vs[(long long)b * a.s_b + (long long)p * a.s_l + g]
                            : ((LATENT && a.ks != nullptr && p < a.L) ? a.ks[(long long)b * a.s_b + (long long)p * a.s_l + g]
                                                                    : 1.f);
      for (int r = warp; r < R; r += 8) {
        const float x = sP[r * kKT + kk];
        const float mold = sM[r];
        const float mt = warp_max(x);
        const float mnew = fmaxf(mold, mt);
        const float e = mnew == -INFINITY ? 0.f : __expf(x - mnew);
        const float sum = warp_sum(e);
        sP[r * kKT + kk] = e * vsc;
        if (kk == 0) {
          const float alpha = mold == -INFINITY ? 0.f : __expf(mold - mnew);
          sA[r] = alpha;
          sL[r] = sL[r] * alpha + sum;
          sM[r] = mnew;
        }
      }
    }
    __syncthreads();
    // ---- O = O * alpha + P V ------------------------------------------------
    if (pv_active) {
      const KV* tV = LATENT ? tK : sV + buf * (kKT * DV);
      const int vstride = LATENT ? DQ : DV;
#pragma unroll
      for (int i = 0; i < kPvRows; ++i) {
        const int r = rg + i * rgroups;
        if (r < R) {
          const float al = sA[r];
          acc[i][0] *= al;
          acc[i][1] *= al;
          acc[i][2] *= al;
          acc[i][3] *= al;
        }
      }
      for (int kk = 0; kk < kKT; ++kk) {
        float vv[4];
        KVTraits<KV>::load4(tV + kk * vstride + c4 * 4, vv);
#pragma unroll
        for (int i = 0; i < kPvRows; ++i) {
          const int r = rg + i * rgroups;
          if (r < R) {
            const float pr = sP[r * kKT + kk];
            acc[i][0] += pr * vv[0];
            acc[i][1] += pr * vv[1];
            acc[i][2] += pr * vv[2];
            acc[i][3] += pr * vv[3];
          }
        }
      }
    }
    __syncthreads();
  }
  // ---- partial results ----------------------------------------------------------
  const long long base = (((long long)b * a.Hk + g) * a.splits + split) * kMaxRows;
  if (pv_active) {
#pragma unroll
    for (int i = 0; i < kPvRows; ++i) {
      const int r = rg + i * rgroups;
      if (r < R) {
        float4 o = make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
        *reinterpret_cast<float4*>(a.part_o + (base + r) * DV + c4 * 4) = o;
      }
    }
  }
  if (tid < R) {
    a.part_ml[(base + tid) * 2] = sM[tid];
    a.part_ml[(base + tid) * 2 + 1] = sL[tid];
  }
}

__global__ void decode_combine_kernel(const float* __restrict__ part_o, const float* __restrict__ part_ml,
                                      bf16* __restrict__ out, int B, int Tn, int H, int Hk, int DV, int splits,
                                      int rstride) {
  const int G = H / Hk;
  const int R = Tn * G;
  const int row = blockIdx.x;  // b * Hk * R + g * R + r
  const int r = row % R;
  const int g = (row / R) % Hk;
  const int b = row / (R * Hk);
  const long long base = ((long long)b * Hk + g) * splits * rstride;
  float M = -INFINITY;
  for (int s = 0; s < splits; ++s) M = fmaxf(M, part_ml[(base + (long long)s * rstride + r) * 2]);
  float Lsum = 0.f;
  for (int s = 0; s < splits; ++s) {
    const float m = part_ml[(base + (long long)s * rstride + r) * 2];
    if (m != -INFINITY) Lsum += part_ml[(base + (long long)s * rstride + r) * 2 + 1] * __expf(m - M);
  }
  const float inv = Lsum > 0.f ? 1.f / Lsum : 0.f;
  const int t = r / G, h = g * G + r % G;
  bf16* o = out + (((long long)b * Tn + t) * H + h) * DV;
  for (int c = threadIdx.x; c < DV; c += blockDim.x) {
    float acc = 0.f;
    for (int s = 0; s < splits; ++s) {
      const float m = part_ml[(base + (long long)s * rstride + r) * 2];
      if (m == -INFINITY) continue;
      acc += part_o[(base + (long long)s * rstride + r) * DV + c] * __expf(m - M);
    }
    o[c] = __float2bfloat16(acc * inv);
  }
}


// ===========================================================================
// Tensor-core path: MLA latent cache (one KV group, value = first DV dims of
// each key row).
//
// CTA = (row group of RG query rows, split, sequence), one CTA per SM, three
// warp roles over tiles of 128 keys:
//   * converters (warps 0-7, thread pair = one 32-byte sector of one key row):
//     the next tile is always in flight in registers (streaming 16-byte loads);
//     each 64-dim chunk is written to shared memory as fp16 (int8 cache: the
//     integers are exact in fp16) or bf16, 128-byte swizzled
//     [chunk][128 keys][128 B], as soon as the tensor core has released that
//     chunk of the previous tile, and announced on chunk_full[c].  The rope
//     chunks go first (free once the scores are computed), then the value
//     chunks in value-block order (free once that block of P.V is done).
//   * MMA (lane 0 of warp 8): S^T[key, row] = K . Q^T chunk by chunk as the
//     chunks land (M = 128 keys, N = RG rows, 4 interleaved accumulators so
//     consecutive MMAs are independent), then, after the softmax,
//     O^T[dim, row] += V^T . P'^T per 128-dim value block (the same shared
//     tile read MN-major), each block's commit releasing its two chunks.
//   * softmax (warps 8-11, thread = key = TMEM lane): scale, mask, row maxima
//     (butterflies + shared memory across the four warps), P' = exp2(s - m_ref)
//     * k_scale into shared memory.  m_ref moves only when a row max grows by
//     more than 2^8 (then O and l are rescaled in place), so O normally stays
//     in tensor memory untouched.
// Converting tile t+1 overlaps P.V of tile t and the scores of t+1 overlap
// the conversion; the tensor core idles only during the softmax.  Every
// mbarrier wait is bounded and reports through the status block.
// ===========================================================================
constexpr int kTcKeys = 128;
constexpr int kTcConvWarps = 8;
constexpr int kTcSmWarp0 = 8;   // softmax warps 8..11 (TMEM lane quadrants 0..3); lane 0 of warp 8 issues the MMAs
constexpr int kTcThreads = 12 * 32;  // 3 warps per SM sub-partition: up to 168 registers each

// Phase timestamps of CTA (0, 0, 0) for profiling builds (-DOMNI_DEC_TRACE): slot
// [tile][role][phase], role 0 = converter thread 0, 1 = MMA thread, 2 = softmax thread 0.
#ifdef OMNI_DEC_TRACE
__device__ long long g_dec_trace[64][3][8];
#define DEC_TRACE(role, it, ph)                                                            \
  do {                                                                                     \
    if (blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0 && (it) < 64)               \
      g_dec_trace[(it)][(role)][(ph)] = clock64();                                         \
  } while (0)
#else
#define DEC_TRACE(role, it, ph) \
  do {                          \
  } while (0)
#endif

template <int DQ, int RG>
struct TcSmem {
  static constexpr int NQC = DQ / 64;
  static constexpr int kK = NQC * kTcKeys * 128;
  static constexpr int kQ = NQC * RG * 128;
  static constexpr int kP = 2 * RG * 128;
  static constexpr int kOffK = 0;
  static constexpr int kOffQ = kOffK + kK;
  static constexpr int kOffP = kOffQ + kQ;
  static constexpr int kOffRed = kOffP + kP;                 // float [2][4][RG]
  static constexpr int kOffScale = kOffRed + 8 * RG * 4;     // float [2][128]
  static constexpr int kOffPos = kOffScale + 2 * kTcKeys * 4;  // int [RG]
  static constexpr int kOffBar = kOffPos + RG * 4;           // mbarriers + TMEM slot
  static constexpr int kBars = 2 * NQC + 8;
  static constexpr int kBytes = kOffBar + kBars * 8 + 16 + 1024;  // + alignment slack
};

__device__ __forceinline__ uint4 ld_stream16(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// 4 int8 (one word) -> 2 x fp16x2, exact: bias to unsigned, place each byte in
// the mantissa of 1024.0 (0x64XX), subtract 1024 + 128.
__device__ __forceinline__ void i8x4_to_f16x4(uint32_t w, uint32_t& lo, uint32_t& hi) {
  const uint32_t x = w ^ 0x80808080u;
  uint32_t a, b;
  asm("prmt.b32 %0, %1, %2, 0x7170;" : "=r"(a) : "r"(x), "r"(0x64646464u));
  asm("prmt.b32 %0, %1, %2, 0x7372;" : "=r"(b) : "r"(x), "r"(0x64646464u));
  const __half2 bias = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));
  const __half2 ha = __hsub2(*reinterpret_cast<const __half2*>(&a), bias);
  const __half2 hb = __hsub2(*reinterpret_cast<const __half2*>(&b), bias);
  lo = *reinterpret_cast<const uint32_t*>(&ha);
  hi = *reinterpret_cast<const uint32_t*>(&hb);
}

__device__ __forceinline__ uint32_t bf16x2_to_f16x2(uint32_t w) {
  const __half2 h = __floats2half2_rn(bf16_lo(w), bf16_hi(w));
  return *reinterpret_cast<const uint32_t*>(&h);
}

__device__ __forceinline__ void named_bar_softmax() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// AND of `v` over the 128 softmax threads (named barrier 1): every one of them
// takes the same branch afterwards, so none is left waiting on the barrier.
__device__ __forceinline__ bool all_softmax(bool v) {
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

// Reduce-scatter over the 32 lanes of 16 per-lane values: afterwards lane l holds
// the max (or sum) over all lanes of value ((l >> 1) & 15) with the bits of l
// reversed into the row index: row = 8*b4 + 4*b3 + 2*b2 + b1 (b_i = bit i of l).
template <bool MAX>
__device__ __forceinline__ float lanes_reduce16(float (&v)[16]) {
  const int lane = threadIdx.x & 31;
  auto op = [](float x, float y) { return MAX ? fmaxf(x, y) : x + y; };
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const bool up = lane & 16;
    const float send = up ? v[i] : v[i + 8], keep = up ? v[i + 8] : v[i];
    v[i] = op(keep, __shfl_xor_sync(0xffffffffu, send, 16));
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const bool up = lane & 8;
    const float send = up ? v[i] : v[i + 4], keep = up ? v[i + 4] : v[i];
    v[i] = op(keep, __shfl_xor_sync(0xffffffffu, send, 8));
  }
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const bool up = lane & 4;
    const float send = up ? v[i] : v[i + 2], keep = up ? v[i + 2] : v[i];
    v[i] = op(keep, __shfl_xor_sync(0xffffffffu, send, 4));
  }
  {
    const bool up = lane & 2;
    const float send = up ? v[0] : v[1], keep = up ? v[1] : v[0];
    v[0] = op(keep, __shfl_xor_sync(0xffffffffu, send, 2));
  }
  return op(v[0], __shfl_xor_sync(0xffffffffu, v[0], 1));
}
__device__ __forceinline__ int reduce16_row(int lane) {
  return ((lane >> 4) & 1) * 8 + ((lane >> 3) & 1) * 4 + ((lane >> 2) & 1) * 2 + ((lane >> 1) & 1);
}

template <int N>
__device__ __forceinline__ void tmem_ld_n(uint32_t taddr, float* v) {
#pragma unroll
  for (int c = 0; c < N / 16; ++c) tmem_ld16(taddr + c * 16, v + c * 16);
}
template <int N>
__device__ __forceinline__ void tmem_st_n(uint32_t taddr, const float* v) {
#pragma unroll
  for (int c = 0; c < N / 16; ++c) tmem_st16(taddr + c * 16, v + c * 16);
}

template <typename KV, int DQ, int DV, int RG>
__global__ void __launch_bounds__(kTcThreads, 1) decode_mla_tc_kernel(DecArgs a, StatusBlock* status) {
  using Lay = TcSmem<DQ, RG>;
  constexpr bool I8 = std::is_same<KV, int8_t>::value;
  constexpr int NQC = DQ / 64;                  // 64-dim chunks of a key row
  constexpr int NVB = DV / 128;                 // 128-dim value blocks (2 chunks each)
  constexpr int NROPE = NQC - 2 * NVB;          // chunks used only by the scores
  constexpr int PPC = 64 * (int)sizeof(KV) / 32;  // 32-byte sectors per chunk per key
  constexpr int NJ = NQC * PPC;                 // sectors per key row
  constexpr int SACC = 4;                       // interleaved score accumulators
  static_assert(DQ % 64 == 0 && DV % 128 == 0 && DV <= DQ, "tile shape");
  static_assert(SACC * RG + NVB * RG <= 128, "tensor memory columns");
  static_assert(RG == 16, "the row reductions assume 16 rows per CTA");
  constexpr float kLog2e = 1.4426950408889634f;
  constexpr float kLn2 = 0.6931471805599453f;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = smem + Lay::kOffK;
  uint8_t* sQ = smem + Lay::kOffQ;
  uint8_t* sP = smem + Lay::kOffP;
  float* sRed = reinterpret_cast<float*>(smem + Lay::kOffRed);
  float* sScale = reinterpret_cast<float*>(smem + Lay::kOffScale);
  int* sPos = reinterpret_cast<int*>(smem + Lay::kOffPos);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Lay::kOffBar);
  uint64_t* chunk_full = bars;            // [NQC]  converters -> MMA (256 arrivals)
  uint64_t* chunk_free = bars + NQC;      // [NQC]  MMA commit -> converters
  uint64_t* s_full = bars + 2 * NQC;      // scores ready (commit)
  uint64_t* p_full = s_full + 1;          // P' written (128 arrivals)
  uint64_t* o_done = s_full + 2;          // last P.V complete (commit)
  uint64_t* drain = s_full + 3;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(s_full + 4);

  const int grp = blockIdx.x, split = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = a.H;  // one KV group
  const int R = a.Tn * G;
  const int r0 = grp * RG;

  if (tid == 0) {
    for (int c = 0; c < NQC; ++c) {
      mbar_init(&chunk_full[c], kTcConvWarps * 32);
      mbar_init(&chunk_free[c], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(p_full, 128);
    mbar_init(o_done, 1);
    mbar_init(drain, 1);
    fence_barrier_init();
  }
  if (warp == kTcSmWarp0) {
    tmem_alloc(tmem_slot, 128);
    tmem_relinquish();
  }
  // ---- query rows (zero beyond R) ------------------------------------------------
  for (int i = tid; i < RG * (DQ / 8); i += kTcThreads) {
    const int r = i / (DQ / 8), c8 = i % (DQ / 8);
    uint4 w = make_uint4(0u, 0u, 0u, 0u);
    if (r0 + r < R) {
      const int t = (r0 + r) / G, h = (r0 + r) % G;
      w = *reinterpret_cast<const uint4*>(a.q + (((long long)b * a.Tn + t) * a.H + h) * DQ + c8 * 8);
      if (I8) w = make_uint4(bf16x2_to_f16x2(w.x), bf16x2_to_f16x2(w.y), bf16x2_to_f16x2(w.z), bf16x2_to_f16x2(w.w));
    }
    *reinterpret_cast<uint4*>(sQ + (c8 >> 3) * (RG * 128) + r * 128 + (((c8 & 7) ^ (r & 7)) << 4)) = w;
  }
  int pmin = 0x7fffffff, pmax = -1;
  for (int t = 0; t < a.Tn; ++t) {
    const int p = a.q_pos[b * a.Tn + t];
    pmin = min(pmin, p);
    pmax = max(pmax, p);
  }
  if (tid < RG) sPos[tid] = (r0 + tid < R) ? a.q_pos[b * a.Tn + (r0 + tid) / G] : pmax;
  const int len = a.kv_len[b];
  const int hi = min(len, pmax + 1);
  const int lo = a.window > 0 ? max(0, pmin - a.window + 1) : 0;
  const int nsk = (a.n_sink + kTcKeys - 1) / kTcKeys;
  const int ntiles = nsk + (hi > lo ? (hi - lo + kTcKeys - 1) / kTcKeys : 0);
  const int per = (ntiles + a.splits - 1) / a.splits;
  const int t0 = min(ntiles, split * per), t1 = min(ntiles, t0 + per);
  const int nt = t1 - t0;
  auto row_of = [&](int tile) { return tile < nsk ? tile * kTcKeys : a.sink_rows + lo + (tile - nsk) * kTcKeys; };
  // chunk processing order: rope chunks first, then the value chunks block by block
  auto chunk_at = [&](int i) { return i < NROPE ? 2 * NVB + i : i - NROPE; };

  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS = tmem, tO = tmem + SACC * RG;
  bool ok = true;

  if (warp < kTcConvWarps) {
    // =============================== converters ===============================
    const int key = 16 * warp + (lane >> 1);
    const int half = lane & 1;
    const uint8_t* kbase = reinterpret_cast<const uint8_t*>(a.k) + (long long)b * a.k_b * (long long)sizeof(KV);
    const int sw = key & 7;
    uint8_t* rowb = sK + key * 128;
    uint4 pre[NJ];
    float kpre = 1.f;
    auto src_of = [&](int tile) {
      const int p = min(row_of(tile) + key, a.L - 1);
      return kbase + (long long)p * a.k_l * (long long)sizeof(KV) + half * 16;
    };
    auto scale_of = [&](int tile) {
      return (I8 && a.ks != nullptr)
                 ? __ldg(a.ks + (long long)b * a.s_b + (long long)min(row_of(tile) + tid, a.L - 1) * a.s_l)
                 : 1.f;
    };
    if (nt > 0) {
      const uint8_t* src = src_of(t0);
#pragma unroll
      for (int j = 0; j < NJ; ++j) pre[j] = ld_stream16(src + j * 32);
      if (tid < kTcKeys) kpre = scale_of(t0);
    }
    for (int it = 0; it < nt && ok; ++it) {
      const int tile = t0 + it;
      const bool more = it + 1 < nt;
      const uint8_t* nsrc = src_of(more ? tile + 1 : tile);
      if (tid < kTcKeys) {
        sScale[(it & 1) * kTcKeys + tid] = kpre;
        if (more) kpre = scale_of(tile + 1);
      }
      if (tid == 0) DEC_TRACE(0, it, 0);
#pragma unroll
      for (int i = 0; i < NQC; ++i) {
        const int c = chunk_at(i);
        if (it > 0 && !mbar_wait(&chunk_free[c], (it - 1) & 1, status, STATUS_TIMEOUT_TMA_EMPTY)) { ok = false; break; }
        if (tid == 0 && i == NROPE) DEC_TRACE(0, it, 2);
        if (tid == 0 && i == NQC - 1) DEC_TRACE(0, it, 3);
        uint8_t* cb = rowb + c * (kTcKeys * 128);
#pragma unroll
        for (int q = 0; q < PPC; ++q) {
          const int j = c * PPC + q;        // sector of the row: dims 32j/sizeof(KV)...
          const uint4 v = pre[j];
          if (more) pre[j] = ld_stream16(nsrc + j * 32);
          if (I8) {
            const int u = ((j * 32 + half * 16) & 63) >> 3;  // first 16-byte fp16 unit (even)
            uint4 x, y;
            i8x4_to_f16x4(v.x, x.x, x.y);
            i8x4_to_f16x4(v.y, x.z, x.w);
            i8x4_to_f16x4(v.z, y.x, y.y);
            i8x4_to_f16x4(v.w, y.z, y.w);
            *reinterpret_cast<uint4*>(cb + ((u ^ sw) << 4)) = x;
            *reinterpret_cast<uint4*>(cb + (((u + 1) ^ sw) << 4)) = y;
          } else {
            const int u = (((j * 32 + half * 16) >> 1) & 63) >> 3;
            *reinterpret_cast<uint4*>(cb + ((u ^ sw) << 4)) = v;
          }
        }
        fence_proxy_async_smem();
        mbar_arrive(&chunk_full[c]);
      }
      if (tid == 0) DEC_TRACE(0, it, 1);
    }
  } else {
    // ================================ softmax =================================
    const int sq = warp - kTcSmWarp0;       // TMEM lane quadrant
    const int key = sq * 32 + lane;
    const uint32_t lane_off = (uint32_t)(sq * 32) << 16;
    float m_ref[RG], l_part[RG];
#pragma unroll
    for (int r = 0; r < RG; ++r) {
      m_ref[r] = -INFINITY;
      l_part[r] = 0.f;
    }
    const bool issuer = warp == kTcSmWarp0 && lane == 0;
    // rows of this group that all belong to one query token share one visibility test
    const bool one_token = (r0 / G) == (min(r0 + RG, R) - 1) / G;
    const int qp0 = sPos[0];
    constexpr uint32_t idesc_s = umma_idesc_f16(128, RG, false, false, !I8);
    constexpr uint32_t idesc_o = umma_idesc_f16(128, RG, true, false, !I8);
    const uint32_t ka = smem_u32(sK), qa = smem_u32(sQ), pa = smem_u32(sP);
    // base descriptors; an operand at byte offset `off` is base + (off >> 4) (the 14-bit
    // start-address field cannot carry for shared-memory addresses)
    const uint64_t dK = umma_desc_sw128(ka, 16, 1024), dQ = umma_desc_sw128(qa, 16, 1024);
    const uint64_t dV = umma_desc_sw128(ka, kTcKeys * 128, 1024), dP = umma_desc_sw128(pa, 16, 1024);
    for (int it = 0; it < nt; ++it) {
      const int tile = t0 + it;
      if (issuer && ok) {
        // S^T = K . Q^T, chunk by chunk as the converters publish them
        DEC_TRACE(1, it, 0);
#pragma unroll
        for (int i = 0; i < NQC; ++i) {
          const int c = chunk_at(i);
          if (!mbar_wait(&chunk_full[c], it & 1, status, STATUS_TIMEOUT_TMA_FULL)) { ok = false; break; }
          tc_fence_after();
#pragma unroll
          for (int k4 = 0; k4 < 4; ++k4) {
            const uint32_t koff = c * (kTcKeys * 128) + k4 * 32;
            const uint32_t qoff = c * (RG * 128) + k4 * 32;
            tc_mma_f16(tS + k4 * RG, dK + (koff >> 4), dQ + (qoff >> 4),
                       idesc_s, i > 0 ? 1u : 0u);
          }
          if (i < NROPE) tc_commit(&chunk_free[c]);  // rope chunks: free once the scores are done
        }
        if (ok) tc_commit(s_full);
        DEC_TRACE(1, it, 1);
      }
      // scores of this tile (their commit also covers the previous P.V: O and P are free);
      // the last value chunk's arrival publishes this tile's key scales
      if (ok && !mbar_wait(s_full, it & 1, status, STATUS_TIMEOUT_TMEM_FULL)) ok = false;
      if (ok && !mbar_wait(&chunk_full[2 * NVB - 1], it & 1, status, STATUS_TIMEOUT_TMA_FULL)) ok = false;
      ok = all_softmax(ok);  // the only exit point of the loop: uniform over the four warps
      if (!ok) break;
      tc_fence_after();
      if (tid == kTcSmWarp0 * 32) DEC_TRACE(2, it, 0);
      float s[RG];
      tmem_ld_n<RG>(tS + lane_off, s);
#pragma unroll
      for (int q = 1; q < SACC; ++q) {
        float s2[RG];
        tmem_ld_n<RG>(tS + q * RG + lane_off, s2);
        tc_wait_ld();
#pragma unroll
        for (int r = 0; r < RG; ++r) s[r] += s2[r];
      }
      tc_wait_ld();
      const int p0 = row_of(tile);
      const int prow = p0 + key;
      const bool sink_tile = tile < nsk;
      const int tp = prow - a.sink_rows;
      const float ksc = sScale[(it & 1) * kTcKeys + key];
      const float mul = ksc * a.scale * kLog2e;
      float wm[RG];
      if (one_token) {
        const bool vis = sink_tile ? (prow < a.n_sink) : (tp < len && tp <= qp0 && (a.window <= 0 || tp > qp0 - a.window));
#pragma unroll
        for (int r = 0; r < RG; ++r) {
          s[r] = vis ? s[r] * mul : -INFINITY;
          wm[r] = s[r];
        }
      } else {
#pragma unroll
        for (int r = 0; r < RG; ++r) {
          const int qp = sPos[r];
          const bool vis = sink_tile ? (prow < a.n_sink) : (tp < len && tp <= qp && (a.window <= 0 || tp > qp - a.window));
          s[r] = vis ? s[r] * mul : -INFINITY;
          wm[r] = s[r];
        }
      }
      const float rmax = lanes_reduce16<true>(wm);
      float* red = sRed + (it & 1) * 4 * RG;
      if ((lane & 1) == 0) red[sq * RG + reduce16_row(lane)] = rmax;
      named_bar_softmax();
      float alpha[RG];
      bool any = false;
#pragma unroll
      for (int r = 0; r < RG; ++r) {
        const float tmax = fmaxf(fmaxf(red[r], red[RG + r]), fmaxf(red[2 * RG + r], red[3 * RG + r]));
        alpha[r] = 1.f;
        if (tmax > m_ref[r] + 8.f) {
          alpha[r] = (m_ref[r] == -INFINITY) ? 0.f : fast_exp2(m_ref[r] - tmax);
          m_ref[r] = tmax;
          l_part[r] *= alpha[r];
          any = true;
        }
      }
      if (any && it > 0) {
#pragma unroll
        for (int j = 0; j < NVB; ++j) {
          float o[RG];
          tmem_ld_n<RG>(tO + j * RG + lane_off, o);
          tc_wait_ld();
#pragma unroll
          for (int r = 0; r < RG; ++r) o[r] *= alpha[r];
          tmem_st_n<RG>(tO + j * RG + lane_off, o);
        }
        tc_wait_st();
      }
      uint8_t* pcol = sP + (key >> 6) * (RG * 128) + (key & 7) * 2;
      const int ku = (key & 63) >> 3;
#pragma unroll
      for (int r = 0; r < RG; ++r) {
        const float e = (m_ref[r] == -INFINITY) ? 0.f : fast_exp2(s[r] - m_ref[r]);
        l_part[r] += e;
        const float pv = e * ksc;
        unsigned short bits;
        if (I8) bits = __half_as_ushort(__float2half_rn(pv));
        else bits = __bfloat16_as_ushort(__float2bfloat16_rn(pv));
        *reinterpret_cast<unsigned short*>(pcol + r * 128 + ((ku ^ (r & 7)) << 4)) = bits;
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(p_full);
      if (tid == kTcSmWarp0 * 32) DEC_TRACE(2, it, 1);
      if (issuer) {
        // O^T += V^T . P'^T per value block; each block's commit frees its two chunks
        if (!mbar_wait(p_full, it & 1, status, STATUS_TIMEOUT_TMEM_FULL)) ok = false;
        tc_fence_after();
        DEC_TRACE(1, it, 2);
        if (ok) {
#pragma unroll
          for (int j = 0; j < NVB; ++j) {
#pragma unroll
            for (int kk = 0; kk < kTcKeys / 16; ++kk) {
              const uint32_t aoff = (2 * j) * (kTcKeys * 128) + kk * 2048;
              const uint32_t poff = (kk >> 2) * (RG * 128) + (kk & 3) * 32;
              tc_mma_f16(tO + j * RG, dV + (aoff >> 4), dP + (poff >> 4), idesc_o, (it > 0 || kk > 0) ? 1u : 0u);
            }
            tc_commit(&chunk_free[2 * j]);
            tc_commit(&chunk_free[2 * j + 1]);
          }
        }
        DEC_TRACE(1, it, 3);
      }
    }
    if (issuer) tc_commit(o_done);
    // ---- epilogue: partial (O, m, l) of this split ----------------------------------
    if (ok && nt > 0 && !mbar_wait(o_done, 0, status, STATUS_TIMEOUT_TMEM_FULL)) ok = false;
    ok = all_softmax(ok);  // tcgen05.ld below is warp-collective: decide once for all four warps
    const bool have = ok && nt > 0;
    tc_fence_after();
    const long long obase = ((long long)b * a.splits + split) * R;
    const float lsum = lanes_reduce16<false>(l_part);
    float* red = sRed + (nt & 1) * 4 * RG;
    if ((lane & 1) == 0) red[sq * RG + reduce16_row(lane)] = lsum;
    named_bar_softmax();
    const int st = tid - kTcSmWarp0 * 32;
    if (st < RG && r0 + st < R) {
      float mm = -INFINITY;
#pragma unroll
      for (int r = 0; r < RG; ++r)
        if (r == st) mm = m_ref[r];
      const float l = red[st] + red[RG + st] + red[2 * RG + st] + red[3 * RG + st];
      a.part_ml[(obase + r0 + st) * 2] = (ok && have && mm != -INFINITY) ? mm * kLn2 : -INFINITY;
      a.part_ml[(obase + r0 + st) * 2 + 1] = l;
    }
    if (ok && have) {
#pragma unroll
      for (int j = 0; j < NVB; ++j) {
        float o[RG];
        tmem_ld_n<RG>(tO + j * RG + lane_off, o);
        tc_wait_ld();
        const int dim = j * 128 + sq * 32 + lane;
#pragma unroll
        for (int r = 0; r < RG; ++r)
          if (r0 + r < R) a.part_o[(obase + r0 + r) * DV + dim] = o[r];
      }
    }
  }
  // drain whatever the tensor core still has in flight before the columns are released
  if (warp == kTcSmWarp0 && lane == 0) {
    tc_commit(drain);
    mbar_wait(drain, 0, status, STATUS_TIMEOUT_DRAIN);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kTcSmWarp0) {
    tc_fence_after();
    tmem_dealloc(tmem, 128);
  }
}

template <typename KV, int DQ, int DV, int RG>
void launch_tc(const DecArgs& a, int groups, StatusBlock* st, cudaStream_t s) {
  auto kern = decode_mla_tc_kernel<KV, DQ, DV, RG>;
  constexpr int smem = TcSmem<DQ, RG>::kBytes;
  ensure_smem_attr(reinterpret_cast<const void*>(kern), smem);
  kern<<<dim3(groups, a.splits, a.B), kTcThreads, smem, s>>>(a, st);
}

template <typename KV, int RG>
bool dispatch_tc_dims(const DecArgs& a, int groups, StatusBlock* st, cudaStream_t s) {
  if (a.DQ == 576 && a.DV == 512) { launch_tc<KV, 576, 512, RG>(a, groups, st, s); return true; }
  if (a.DQ == 320 && a.DV == 256) { launch_tc<KV, 320, 256, RG>(a, groups, st, s); return true; }
  return false;
}

bool tc_dims_supported(int DQ, int DV) { return (DQ == 576 && DV == 512) || (DQ == 320 && DV == 256); }

// ===========================================================================
// Few-row path (MHA / GQA caches with at most 16 query rows per KV head, e.g.
// one decode token of an MHA model): the op is a pair of GEMVs over the cache
// and must run at HBM bandwidth, so every thread works on keys in both phases.
// CTA = (sequence, kv head, split), 256 threads, tiles of 64 keys staged by
// cp.async (double buffered, rows padded by 16 bytes):
//   scores : 4 threads per key, each a quarter of the head dim for all rows,
//            combined by two shuffles;
//   softmax: one warp per row (online max / sum in shared memory);
//   P.V    : thread = (2 value dims, key group); the groups are summed once at
//            the end.
// ===========================================================================
constexpr int kGvThreads = 256;
constexpr int kGvKeys = 64;
constexpr int kGvMaxRows = 16;

struct GvLayout {
  int kRow, vRow, offQ, offK, offV, offS, offKs, offVs, offM, offL, offA, offPos, bytes;
};

__host__ __device__ inline GvLayout gv_layout(int DQ, int DV, int kv_bytes) {
  GvLayout L;
  L.kRow = DQ * kv_bytes + 16;
  L.vRow = DV * kv_bytes + 16;
  L.offQ = 0;                                                   // float [16][DQ]
  L.offK = L.offQ + kGvMaxRows * DQ * 4;                        // [2][64][kRow]
  L.offV = L.offK + 2 * kGvKeys * L.kRow;                       // [2][64][vRow]
  L.offS = L.offV + 2 * kGvKeys * L.vRow;                       // float [16][64]
  L.offKs = L.offS + kGvMaxRows * kGvKeys * 4;                  // float [2][64]
  L.offVs = L.offKs + 2 * kGvKeys * 4;                          // float [2][64]
  L.offM = L.offVs + 2 * kGvKeys * 4;
  L.offL = L.offM + kGvMaxRows * 4;
  L.offA = L.offL + kGvMaxRows * 4;
  L.offPos = L.offA + kGvMaxRows * 4;
  L.bytes = L.offPos + kGvMaxRows * 4;
  return L;
}

__device__ __forceinline__ void cp_async4(void* smem, const void* gmem) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(smem)), "l"(gmem) : "memory");
}

// 16 bytes of cache elements -> floats (8 for bf16, 16 for int8)
__device__ __forceinline__ void unpack16(const bf16*, const uint4 w, float* f) {
  const uint32_t* x = reinterpret_cast<const uint32_t*>(&w);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    f[2 * j] = bf16_lo(x[j]);
    f[2 * j + 1] = bf16_hi(x[j]);
  }
}
__device__ __forceinline__ void unpack16(const int8_t*, const uint4 w, float* f) {
  const uint32_t* x = reinterpret_cast<const uint32_t*>(&w);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    f[4 * j] = (float)(signed char)(x[j] & 0xff);
    f[4 * j + 1] = (float)(signed char)((x[j] >> 8) & 0xff);
    f[4 * j + 2] = (float)(signed char)((x[j] >> 16) & 0xff);
    f[4 * j + 3] = (float)(signed char)((x[j] >> 24) & 0xff);
  }
}

template <typename KV, int RMAX>
__global__ void __launch_bounds__(kGvThreads) decode_gemv_kernel(DecArgs a) {
  extern __shared__ __align__(16) uint8_t smem[];
  constexpr int PC = 16 / (int)sizeof(KV);  // elements per 16-byte chunk
  constexpr float kLog2e = 1.4426950408889634f;
  constexpr float kLn2 = 0.6931471805599453f;
  const int b = blockIdx.x, g = blockIdx.y, split = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = a.H / a.Hk, R = a.Tn * G;
  const int DQ = a.DQ, DV = a.DV;
  const GvLayout Ly = gv_layout(DQ, DV, (int)sizeof(KV));
  float* sQ = reinterpret_cast<float*>(smem + Ly.offQ);
  uint8_t* sK = smem + Ly.offK;
  uint8_t* sV = smem + Ly.offV;
  float* sS = reinterpret_cast<float*>(smem + Ly.offS);
  float* sKs = reinterpret_cast<float*>(smem + Ly.offKs);
  float* sVs = reinterpret_cast<float*>(smem + Ly.offVs);
  float* sM = reinterpret_cast<float*>(smem + Ly.offM);
  float* sL = reinterpret_cast<float*>(smem + Ly.offL);
  float* sA = reinterpret_cast<float*>(smem + Ly.offA);
  int* sPos = reinterpret_cast<int*>(smem + Ly.offPos);

  for (int i = tid; i < R * DQ; i += kGvThreads) {
    const int r = i / DQ, d = i % DQ;
    const int t = r / G, h = g * G + r % G;
    sQ[r * DQ + d] = __bfloat162float(a.q[(((long long)b * a.Tn + t) * a.H + h) * DQ + d]);
  }
  int pmin = 0x7fffffff, pmax = -1;
  for (int t = 0; t < a.Tn; ++t) {
    const int p = a.q_pos[b * a.Tn + t];
    pmin = min(pmin, p);
    pmax = max(pmax, p);
  }
  if (tid < R) {
    sPos[tid] = a.q_pos[b * a.Tn + tid / G];
    sM[tid] = -INFINITY;
    sL[tid] = 0.f;
  }
  const int len = a.kv_len[b];
  const int hi = min(len, pmax + 1);
  const int lo = a.window > 0 ? max(0, pmin - a.window + 1) : 0;
  const int nsk = (a.n_sink + kGvKeys - 1) / kGvKeys;
  const int ntiles = nsk + (hi > lo ? (hi - lo + kGvKeys - 1) / kGvKeys : 0);
  const int per = (ntiles + a.splits - 1) / a.splits;
  const int t0 = min(ntiles, split * per), t1 = min(ntiles, t0 + per);
  auto row_of = [&](int tile) { return tile < nsk ? tile * kGvKeys : a.sink_rows + lo + (tile - nsk) * kGvKeys; };

  // copy assignment (fixed for the whole loop): thread -> (key kk, 16-byte chunk c) pairs
  const int kch = DQ * (int)sizeof(KV) / 16, vch = DV * (int)sizeof(KV) / 16;
  const int k_per = kGvKeys * kch / kGvThreads, v_per = kGvKeys * vch / kGvThreads;  // exact (dims checked)
  const int k_kk0 = tid / kch, k_c = tid % kch, k_step = kGvThreads / kch;
  const int v_kk0 = tid / vch, v_c = tid % vch, v_step = kGvThreads / vch;
  const uint8_t* kbase = reinterpret_cast<const uint8_t*>(a.k) +
                         ((long long)b * a.k_b + (long long)g * DQ) * (long long)sizeof(KV) + k_c * 16;
  const uint8_t* vbase = reinterpret_cast<const uint8_t*>(a.v) +
                         ((long long)b * a.v_b + (long long)g * DV) * (long long)sizeof(KV) + v_c * 16;
  auto issue = [&](int tile, int buf) {
    const int p0 = row_of(tile);
    for (int j = 0; j < k_per; ++j) {
      const int kk = k_kk0 + j * k_step;
      const int p = min(p0 + kk, a.L - 1);
      cp_async16(sK + (buf * kGvKeys + kk) * Ly.kRow + k_c * 16, kbase + (long long)p * a.k_l * (long long)sizeof(KV));
    }
    for (int j = 0; j < v_per; ++j) {
      const int kk = v_kk0 + j * v_step;
      const int p = min(p0 + kk, a.L - 1);
      cp_async16(sV + (buf * kGvKeys + kk) * Ly.vRow + v_c * 16, vbase + (long long)p * a.v_l * (long long)sizeof(KV));
    }
    if (a.ks != nullptr && tid < kGvKeys) {
      const int p = min(p0 + tid, a.L - 1);
      cp_async4(sKs + buf * kGvKeys + tid, a.ks + (long long)b * a.s_b + (long long)p * a.s_l + g);
      cp_async4(sVs + buf * kGvKeys + tid, a.vs + (long long)b * a.s_b + (long long)p * a.s_l + g);
    }
    cp_async_commit();
  };

  // P.V mapping: thread = (value dims 2*d2, 2*d2+1; key group kg)
  const int nd2 = DV / 2;
  const int nkg = kGvThreads / nd2;
  const int d2 = tid % nd2, kg = tid / nd2;
  const int kpg = kGvKeys / nkg;
  float acc[RMAX][2];
#pragma unroll
  for (int r = 0; r < RMAX; ++r) acc[r][0] = acc[r][1] = 0.f;

  __syncthreads();
  if (t0 < t1) issue(t0, 0);
  for (int tile = t0; tile < t1; ++tile) {
    const int buf = (tile - t0) & 1;
    if (tile + 1 < t1) {
      issue(tile + 1, buf ^ 1);
      cp_async_wait_one();
    } else {
      cp_async_wait_all();
    }
    __syncthreads();
    const int p0 = row_of(tile);
    const bool sink_tile = tile < nsk;
    // ---- scores -------------------------------------------------------------------
    {
      const int key = tid >> 2, part = tid & 3;
      const int n_el = DQ / 4;
      const KV* krow = reinterpret_cast<const KV*>(sK + (buf * kGvKeys + key) * Ly.kRow) + part * n_el;
      float sc[RMAX];
#pragma unroll
      for (int r = 0; r < RMAX; ++r) sc[r] = 0.f;
      for (int c = 0; c < n_el; c += PC) {
        float kf[PC];
        unpack16(krow, *reinterpret_cast<const uint4*>(krow + c), kf);
        const float* qb = sQ + part * n_el + c;
#pragma unroll
        for (int r = 0; r < RMAX; ++r) {
          if (r < R) {
            float acc_r = 0.f;
#pragma unroll
            for (int e = 0; e < PC; e += 4) {
              const float4 qv = *reinterpret_cast<const float4*>(qb + r * DQ + e);
              acc_r += kf[e] * qv.x + kf[e + 1] * qv.y + kf[e + 2] * qv.z + kf[e + 3] * qv.w;
            }
            sc[r] += acc_r;
          }
        }
      }
      const int p = p0 + key;
      const int tp = p - a.sink_rows;
      const float mul = a.scale * kLog2e * (a.ks != nullptr ? sKs[buf * kGvKeys + key] : 1.f);
#pragma unroll
      for (int r = 0; r < RMAX; ++r) {
        if (r < R) {
          float v = sc[r];
          v += __shfl_xor_sync(0xffffffffu, v, 1);
          v += __shfl_xor_sync(0xffffffffu, v, 2);
          const int qp = sPos[r];
          const bool vis = sink_tile ? (p < a.n_sink) : (tp < len && tp <= qp && (a.window <= 0 || tp > qp - a.window));
          if (part == 0) sS[r * kGvKeys + key] = vis ? v * mul : -INFINITY;
        }
      }
    }
    __syncthreads();
    // ---- online softmax, one warp per row ----------------------------------------------
    for (int r = warp; r < R; r += kGvThreads / 32) {
      const float x0 = sS[r * kGvKeys + lane], x1 = sS[r * kGvKeys + lane + 32];
      const float mold = sM[r];
      const float mnew = fmaxf(mold, warp_max(fmaxf(x0, x1)));
      const float e0 = mnew == -INFINITY ? 0.f : fast_exp2(x0 - mnew);
      const float e1 = mnew == -INFINITY ? 0.f : fast_exp2(x1 - mnew);
      const float sum = warp_sum(e0 + e1);
      const float vs0 = a.vs != nullptr ? sVs[buf * kGvKeys + lane] : 1.f;
      const float vs1 = a.vs != nullptr ? sVs[buf * kGvKeys + lane + 32] : 1.f;
      sS[r * kGvKeys + lane] = e0 * vs0;
      sS[r * kGvKeys + lane + 32] = e1 * vs1;
      if (lane == 0) {
        const float alpha = mold == -INFINITY ? 0.f : fast_exp2(mold - mnew);
        sA[r] = alpha;
        sL[r] = sL[r] * alpha + sum;
        sM[r] = mnew;
      }
    }
    __syncthreads();
    // ---- O = O * alpha + P V ---------------------------------------------------------
#pragma unroll
    for (int r = 0; r < RMAX; ++r) {
      if (r < R) {
        const float al = sA[r];
        acc[r][0] *= al;
        acc[r][1] *= al;
      }
    }
    for (int j = 0; j < kpg; ++j) {
      const int key = kg * kpg + j;
      const KV* vrow = reinterpret_cast<const KV*>(sV + (buf * kGvKeys + key) * Ly.vRow);
      float v0, v1;
      if (sizeof(KV) == 2) {
        const uint32_t w = *reinterpret_cast<const uint32_t*>(vrow + 2 * d2);
        v0 = bf16_lo(w);
        v1 = bf16_hi(w);
      } else {
        const uint16_t w = *reinterpret_cast<const uint16_t*>(vrow + 2 * d2);
        v0 = (float)(signed char)(w & 0xff);
        v1 = (float)(signed char)(w >> 8);
      }
#pragma unroll
      for (int r = 0; r < RMAX; ++r) {
        if (r < R) {
          const float pr = sS[r * kGvKeys + key];
          acc[r][0] += pr * v0;
          acc[r][1] += pr * v1;
        }
      }
    }
    __syncthreads();
  }
  // ---- sum the key groups (shared memory reused), write the split's partials ----------
  float* red = reinterpret_cast<float*>(smem + Ly.offK);  // [nkg][R][DV] <= 8 * 16 * 256 floats
#pragma unroll
  for (int r = 0; r < RMAX; ++r) {
    if (r < R) {
      red[(kg * R + r) * DV + 2 * d2] = acc[r][0];
      red[(kg * R + r) * DV + 2 * d2 + 1] = acc[r][1];
    }
  }
  __syncthreads();
  const long long base = (((long long)b * a.Hk + g) * a.splits + split) * R;
  for (int i = tid; i < R * DV; i += kGvThreads) {
    const int r = i / DV, d = i % DV;
    float o = 0.f;
    for (int q = 0; q < nkg; ++q) o += red[(q * R + r) * DV + d];
    a.part_o[(base + r) * DV + d] = o;
  }
  if (tid < R) {
    a.part_ml[(base + tid) * 2] = sM[tid] == -INFINITY ? -INFINITY : sM[tid] * kLn2;
    a.part_ml[(base + tid) * 2 + 1] = sL[tid];
  }
}

template <typename KV, int RMAX>
void launch_gemv_r(const DecArgs& a, int smem, cudaStream_t s) {
  auto kern = decode_gemv_kernel<KV, RMAX>;
  ensure_smem_attr(reinterpret_cast<const void*>(kern), smem);
  kern<<<dim3(a.B, a.Hk, a.splits), kGvThreads, smem, s>>>(a);
}
template <typename KV>
void launch_gemv(const DecArgs& a, int smem, cudaStream_t s) {
  const int R = a.Tn * (a.H / a.Hk);
  if (R <= 1) launch_gemv_r<KV, 1>(a, smem, s);
  else if (R <= 2) launch_gemv_r<KV, 2>(a, smem, s);
  else if (R <= 4) launch_gemv_r<KV, 4>(a, smem, s);
  else if (R <= 8) launch_gemv_r<KV, 8>(a, smem, s);
  else launch_gemv_r<KV, 16>(a, smem, s);
}

bool gemv_dims_supported(int DQ, int DV, int kv_bytes) {
  if (DQ % 32 != 0 || DV % 64 != 0 || DQ > 256 || DV > 256) return false;
  if ((DQ / 4) % (16 / kv_bytes) != 0) return false;        // whole 16-byte chunks per quarter row
  if (kGvKeys % (kGvThreads / (DV / 2)) != 0) return false;   // key groups divide the tile
  const int kch = DQ * kv_bytes / 16, vch = DV * kv_bytes / 16;
  if (kGvThreads % kch != 0 || kGvThreads % vch != 0) return false;  // whole keys per copy pass
  const GvLayout L = gv_layout(DQ, DV, kv_bytes);
  return L.bytes <= 227 * 1024 && (kGvThreads / (DV / 2)) * kGvMaxRows * DV * 4 <= 2 * kGvKeys * L.kRow +
                                                                                      2 * kGvKeys * L.vRow;
}

int decode_smem_bytes(int DQ, int DV, int kv_bytes, bool latent) {
  return kMaxRows * DQ * 2 + 2 * kKT * DQ * kv_bytes + (latent ? 0 : 2 * kKT * DV * kv_bytes) +
         (kMaxRows * kKT + 3 * kMaxRows) * 4 + kMaxRows * 4 + 128;
}

template <typename KV, bool LATENT>
void launch_split(const DecArgs& a, dim3 grid, int smem, cudaStream_t s) {
  auto kern = decode_split_kernel<KV, LATENT>;
  ensure_smem_attr(reinterpret_cast<const void*>(kern), smem);
  kern<<<grid, kDecThreads, smem, s>>>(a);
}

}  // namespace

DecodePlan decode_plan(int B, int Tn, int H, int Hk, int L, int DQ, int DV, bool latent, int window, int sink_rows,
                       int kv_bytes) {
  DecodePlan pl;
  const int R = Tn * (H / Hk);
  pl.tc = latent && Hk == 1 && tc_dims_supported(DQ, DV);
  pl.gemv = !pl.tc && !latent && R <= kGvMaxRows && gemv_dims_supported(DQ, DV, kv_bytes);
  if (pl.gemv) {
    pl.rg = R;
    pl.groups = 1;
    pl.rstride = R;
    const int tokens = window > 0 ? std::min(L - sink_rows, window + Tn) : L - sink_rows;
    const int tiles = (sink_rows + kGvKeys - 1) / kGvKeys + std::max(1, (tokens + kGvKeys - 1) / kGvKeys);
    const int per_sm = std::max(1, std::min(8, (227 * 1024) / gv_layout(DQ, DV, kv_bytes).bytes));
    const int slots = 148 * per_sm;
    const int ctas = B * Hk;
    long best = -1;
    pl.splits = 1;
    for (int sp = 1; sp <= std::min(64, tiles); ++sp) {
      const long waves = ((long)ctas * sp + slots - 1) / slots;
      const long cost = waves * ((tiles + sp - 1) / sp + 2);
      if (best < 0 || cost < best) { best = cost; pl.splits = sp; }
    }
  } else if (pl.tc) {
    pl.rg = 16;  // 16 query rows per CTA keep the prefetch registers and softmax state spill-free
    pl.groups = (R + pl.rg - 1) / pl.rg;
    pl.rstride = R;
    const int tokens = window > 0 ? std::min(L - sink_rows, window + Tn) : L - sink_rows;
    const int tiles = (sink_rows + kTcKeys - 1) / kTcKeys + std::max(1, (tokens + kTcKeys - 1) / kTcKeys);
    // one CTA per SM: pick the split count with the fewest (waves x tiles per CTA), counting
    // one tile of fixed cost per CTA
    const int ctas = B * pl.groups;
    long best = -1;
    pl.splits = 1;
    for (int sp = 1; sp <= std::min(64, tiles); ++sp) {
      const long waves = ((long)ctas * sp + 147) / 148;
      const long cost = waves * ((tiles + sp - 1) / sp + 1);
      if (best < 0 || cost < best) { best = cost; pl.splits = sp; }
    }
  } else {
    pl.rg = 0;
    pl.groups = 1;
    pl.rstride = kMaxRows;
    const int ctas = B * Hk;
    int splits = std::max(1, (2 * 148 + ctas - 1) / ctas);
    splits = std::min(splits, std::max(1, (L + kKT - 1) / kKT));
    pl.splits = std::min(splits, 64);
  }
  pl.ws_floats = (size_t)B * Hk * pl.splits * pl.rstride * (DV + 2);
  return pl;
}

void attn_decode(const void* q, const void* k, const void* v, const float* ks, const float* vs, bool int8_kv,
                 const int* q_pos, const int* kv_len, void* out, float* workspace, int B, int Tn, int H, int Hk,
                 int L, int DQ, int DV, long long k_b, long long k_l, long long v_b, long long v_l, long long s_b,
                 long long s_l, int window, float scale, const DecodePlan& pl, int sink_rows, int n_sink,
                 void* status, cudaStream_t s) {
  const bool latent = v == nullptr;
  const int G = H / Hk;
  if (!pl.tc && !pl.gemv) {
    if (Tn * G > kMaxRows) throw std::runtime_error("attn_decode: Tn * heads-per-kv-group must be <= 64");
    if (DQ % 16 != 0 || DV % 4 != 0 || DV > 4 * kDecThreads) throw std::runtime_error("attn_decode: head dims");
    if ((DV / 4 < kDecThreads) && (kDecThreads % (DV / 4) != 0))
      throw std::runtime_error("attn_decode: DV/4 must divide 256");
    const int colt = std::min(kDecThreads, DV / 4);
    const int rgroups = kDecThreads / colt;
    if ((Tn * G + rgroups - 1) / rgroups > kPvRows) throw std::runtime_error("attn_decode: too many rows per thread");
  }
  DecArgs a;
  a.q = (const bf16*)q;
  a.k = k;
  a.v = v;
  a.ks = ks;
  a.vs = vs;
  a.q_pos = q_pos;
  a.kv_len = kv_len;
  a.part_o = workspace;
  a.part_ml = workspace + (size_t)B * Hk * pl.splits * pl.rstride * DV;
  a.B = B;
  a.Tn = Tn;
  a.H = H;
  a.Hk = Hk;
  a.L = L;
  a.DQ = DQ;
  a.DV = DV;
  a.window = window;
  a.splits = pl.splits;
  a.sink_rows = sink_rows;
  a.n_sink = n_sink;
  a.k_b = k_b;
  a.k_l = k_l;
  a.v_b = v_b;
  a.v_l = v_l;
  a.s_b = s_b;
  a.s_l = s_l;
  a.scale = scale;
  StatusBlock* st = reinterpret_cast<StatusBlock*>(status);
  if (pl.tc) {
    bool done;
    done = int8_kv ? dispatch_tc_dims<int8_t, 16>(a, pl.groups, st, s) : dispatch_tc_dims<bf16, 16>(a, pl.groups, st, s);
    if (!done) throw std::runtime_error("attn_decode: no tensor-core kernel for these dims");
  } else if (pl.gemv) {
    const int smem = gv_layout(DQ, DV, int8_kv ? 1 : 2).bytes;
    if (int8_kv)
      launch_gemv<int8_t>(a, smem, s);
    else
      launch_gemv<bf16>(a, smem, s);
  } else {
    const dim3 grid(B, Hk, pl.splits);
    const int smem = decode_smem_bytes(DQ, DV, int8_kv ? 1 : 2, latent);
    if (smem > 227 * 1024) throw std::runtime_error("attn_decode: head dims too large for shared memory");
    if (int8_kv) {
      if (latent)
        launch_split<int8_t, true>(a, grid, smem, s);
      else
        launch_split<int8_t, false>(a, grid, smem, s);
    } else {
      if (latent)
        launch_split<bf16, true>(a, grid, smem, s);
      else
        launch_split<bf16, false>(a, grid, smem, s);
    }
  }
  decode_combine_kernel<<<B * Hk * Tn * G, 128, 0, s>>>(a.part_o, a.part_ml, (bf16*)out, B, Tn, H, Hk, DV, pl.splits,
                                                         pl.rstride);
}

}  // namespace omni
