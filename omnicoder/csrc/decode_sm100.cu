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

__device__ __forceinline__ float bf16f(const bf16 x) { return __bfloat162float(x); }

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
                                      bf16* __restrict__ out, int B, int Tn, int H, int Hk, int DV, int splits) {
  const int G = H / Hk;
  const int R = Tn * G;
  const int row = blockIdx.x;  // b * Hk * R + g * R + r
  const int r = row % R;
  const int g = (row / R) % Hk;
  const int b = row / (R * Hk);
  const long long base = ((long long)b * Hk + g) * splits * kMaxRows;
  float M = -INFINITY;
  for (int s = 0; s < splits; ++s) M = fmaxf(M, part_ml[(base + (long long)s * kMaxRows + r) * 2]);
  float Lsum = 0.f;
  for (int s = 0; s < splits; ++s) {
    const float m = part_ml[(base + (long long)s * kMaxRows + r) * 2];
    if (m != -INFINITY) Lsum += part_ml[(base + (long long)s * kMaxRows + r) * 2 + 1] * __expf(m - M);
  }
  const float inv = Lsum > 0.f ? 1.f / Lsum : 0.f;
  const int t = r / G, h = g * G + r % G;
  bf16* o = out + (((long long)b * Tn + t) * H + h) * DV;
  for (int c = threadIdx.x; c < DV; c += blockDim.x) {
    float acc = 0.f;
    for (int s = 0; s < splits; ++s) {
      const float m = part_ml[(base + (long long)s * kMaxRows + r) * 2];
      if (m == -INFINITY) continue;
      acc += part_o[(base + (long long)s * kMaxRows + r) * DV + c] * __expf(m - M);
    }
    o[c] = __float2bfloat16(acc * inv);
  }
}

int decode_smem_bytes(int DQ, int DV, int kv_bytes, bool latent) {
  return kMaxRows * DQ * 2 + 2 * kKT * DQ * kv_bytes + (latent ? 0 : 2 * kKT * DV * kv_bytes) +
         (kMaxRows * kKT + 3 * kMaxRows) * 4 + kMaxRows * 4 + 128;
}

template <typename KV, bool LATENT>
void launch_split(const DecArgs& a, dim3 grid, int smem, cudaStream_t s) {
  auto kern = decode_split_kernel<KV, LATENT>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  kern<<<grid, kDecThreads, smem, s>>>(a);
}

}  // namespace

int decode_splits(int B, int Hk, int max_len) {
  const int ctas = B * Hk;
  int splits = std::max(1, (2 * 148 + ctas - 1) / ctas);
  splits = std::min(splits, std::max(1, (max_len + kKT - 1) / kKT));
  return std::min(splits, 64);
}

size_t decode_workspace_floats(int B, int Hk, int splits, int DV) {
  return (size_t)B * Hk * splits * kMaxRows * (DV + 2);
}

void attn_decode(const void* q, const void* k, const void* v, const float* ks, const float* vs, bool int8_kv,
                 const int* q_pos, const int* kv_len, void* out, float* workspace, int B, int Tn, int H, int Hk,
                 int L, int DQ, int DV, long long k_b, long long k_l, long long v_b, long long v_l, long long s_b,
                 long long s_l, int window, float scale, int splits, int sink_rows, int n_sink, cudaStream_t s) {
  const bool latent = v == nullptr;
  const int G = H / Hk;
  if (Tn * G > kMaxRows) throw std::runtime_error("attn_decode: Tn * heads-per-kv-group must be <= 64");
  if (DQ % 16 != 0 || DV % 4 != 0 || DV > 4 * kDecThreads) throw std::runtime_error("attn_decode: head dims");
  if ((DV / 4 < kDecThreads) && (kDecThreads % (DV / 4) != 0))
    throw std::runtime_error("attn_decode: DV/4 must divide 256");
  {
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
  a.part_ml = workspace + (size_t)B * Hk * splits * kMaxRows * DV;
  a.B = B;
  a.Tn = Tn;
  a.H = H;
  a.Hk = Hk;
  a.L = L;
  a.DQ = DQ;
  a.DV = DV;
  a.window = window;
  a.splits = splits;
  a.sink_rows = sink_rows;
  a.n_sink = n_sink;
  a.k_b = k_b;
  a.k_l = k_l;
  a.v_b = v_b;
  a.v_l = v_l;
  a.s_b = s_b;
  a.s_l = s_l;
  a.scale = scale;
  const dim3 grid(B, Hk, splits);
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
  decode_combine_kernel<<<B * Hk * Tn * G, 128, 0, s>>>(a.part_o, a.part_ml, (bf16*)out, B, Tn, H, Hk, DV, splits);
}

}  // namespace omni
