// Flash attention for sm_100a: tcgen05 MMAs with TMEM accumulators, TMA loads,
// one elected thread issuing MMAs, four warps doing the softmax.
//
// Layout (token-major, sequences of length S packed back to back, T = B*S):
//   q  [T, H,  DQ]          (row/head strides given)
//   k  [T, Hk, DQ - DR]     (strided view allowed; GQA: head h reads kv head h/(H/Hk))
//   kr [T, DR]              rope key shared by all heads (MLA), DR = 64, optional
//   v  [T, Hk, DV]          (strided view allowed)
//   o  [T, H, DV], lse [H, T] (natural log of the softmax denominator)
//
// Kernels:
//   attn_fwd   : CTA = (q tile of 128 rows, head, sequence).  S_j = Q K_j^T goes
//                to one of two TMEM buffers while the softmax warps turn the
//                other into P (bf16, written to shared memory in the 128B
//                swizzled K-major layout the next MMA reads) and O += P V_j
//                accumulates in TMEM.  O is rescaled in TMEM only when a row
//                maximum grows by more than 2^8 (lazy rescaling).
//   attn_dkdv  : CTA = (kv tile, kv head, sequence), loops over the q tiles
//                (and over the q heads of a GQA group): S^T = K Q^T and
//                dP^T = V dO^T share TMEM columns; dV += P^T dO and
//                dK += dS^T Q accumulate in TMEM.
//   attn_dq    : CTA = (q tile, head, sequence), loops over kv tiles:
//                dQ += dS K in TMEM.
//   attn_delta : delta = rowsum(dO * O).
//
// Every mbarrier wait is bounded (see common.cuh); a timeout records a status
// code and the role leaves its loop.
//
// This replaces the reference's prefill/decode latent attention, which runs
// as ATen bmm + masked softmax over a 16-slot window
// (src/omnicoder/modeling/attention.py:1034-1262, 1265-1612).
#include <cstdio>
#include <stdexcept>

#include "common.cuh"
#include "tma_host.h"
#include "attention.h"

namespace omni {

using bf16 = __nv_bfloat16;

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr int kTile = 128;
constexpr int kAttnThreads = 192;
// backward kernels: producer warp, MMA warp and 8 softmax warps (two per TMEM lane
// quadrant, each taking half of the 64 columns of a tile)
constexpr int kBwdThreads = 320;
constexpr int kBwdSoftmaxWarps = 8;
constexpr int kSubTile = 16384;  // one [128 rows x 64 bf16] swizzled sub-tile

struct AttnArgs {
  int T, S, H, Hk;
  float scale_log2;  // softmax scale * log2(e)
  float scale;       // softmax scale
  int causal, window;
  bf16* o;
  long long o_row, o_head;
  float* lse;
  const bf16* dO;
  long long do_row, do_head;
  const bf16* O;
  long long O_row, O_head;
  const float* delta;
  bf16* dq;
  long long dq_row, dq_head;
  bf16* dk;  // nope part [T, Hk, DQ-DR]
  long long dk_row, dk_head;
  bf16* dkr;  // rope part per head [T, Hk, DR]
  long long dkr_row, dkr_head;
  bf16* dv;
  long long dv_row, dv_head;
  StatusBlock* status;
};

// Write 128 values (one row of a [128 x 128] bf16 tile) into two swizzled
// 128B K-major sub-tiles.
__device__ __forceinline__ void store_row_sw128(uint8_t* tile, int r, const float* v) {
#pragma unroll
  for (int sub = 0; sub < 2; ++sub) {
#pragma unroll
    for (int ch = 0; ch < 8; ++ch) {
      const float* x = v + sub * 64 + ch * 8;
      uint4 w = make_uint4(pack_bf16x2(x[0], x[1]), pack_bf16x2(x[2], x[3]), pack_bf16x2(x[4], x[5]),
                           pack_bf16x2(x[6], x[7]));
      *reinterpret_cast<uint4*>(tile + sub * kSubTile + r * 128 + ((ch ^ (r & 7)) << 4)) = w;
    }
  }
}


__device__ __forceinline__ void store_global_row(bf16* dst, const float* v, int n, float mul) {
  for (int q = 0; q < n / 8; ++q) {
    uint4 w = make_uint4(pack_bf16x2(v[q * 8] * mul, v[q * 8 + 1] * mul), pack_bf16x2(v[q * 8 + 2] * mul, v[q * 8 + 3] * mul),
                         pack_bf16x2(v[q * 8 + 4] * mul, v[q * 8 + 5] * mul), pack_bf16x2(v[q * 8 + 6] * mul, v[q * 8 + 7] * mul));
    *reinterpret_cast<uint4*>(dst + q * 8) = w;
  }
}

// ===========================================================================
// Forward
// ===========================================================================
template <int DQ, int DV, bool ROPE>
struct FwdSmem {
  static constexpr int NQC = DQ / 64;
  static constexpr int kQ = NQC * kSubTile;
  static constexpr int kK = NQC * kSubTile;
  static constexpr int kV = kTile * DV * 2;
  static constexpr int kOffQ = 0;
  static constexpr int kOffK = kOffQ + kQ;           // 2 stages
  static constexpr int kOffV = kOffK + 2 * kK;       // 2 stages (P lives in tensor memory)
  static constexpr int kOffBar = kOffV + 2 * kV;
  static constexpr int kBytes = kOffBar + 256 + 1024;
};

template <int DQ, int DV, bool ROPE>
__global__ void __launch_bounds__(kAttnThreads, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmKR, const __grid_constant__ CUtensorMap tmV, AttnArgs p) {
  using L = FwdSmem<DQ, DV, ROPE>;
  constexpr int NQC = L::NQC;
  constexpr int NKC = ROPE ? NQC - 1 : NQC;
  constexpr int VCH = DV / 64;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem + L::kOffQ;
  uint8_t* sK = smem + L::kOffK;
  uint8_t* sV = smem + L::kOffV;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kOffBar);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;   // [2]
  uint64_t* k_empty = bars + 3;  // [2]
  uint64_t* v_full = bars + 5;   // [2]
  uint64_t* v_empty = bars + 7;  // [2]
  uint64_t* s_full = bars + 9;   // [2]
  uint64_t* s_empty = bars + 11; // [2]  S/P stage free again (P.V of the stage's tile completed)
  uint64_t* p_full = bars + 13;   // [2] per S/P stage, so the softmax can never run two phases ahead
  uint64_t* o_done = bars + 15;
  uint64_t* drain = bars + 16;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 17);
  // Completes once, after the last P.V: o_done completes once per tile, and when
  // the softmax warps finish the last tile it may still be two completions short
  // (only P.V of tile n-3 is ordered before S of tile n-1), where a parity wait
  // on o_done could not tell phase n-1 from phase n-3.
  uint64_t* o_last = bars + 18;

  const int warp = warp_id(), lane = lane_id();
  const int nqt = p.S / kTile;
  const int qt = nqt - 1 - blockIdx.x;
  const int h = blockIdx.y, b = blockIdx.z;
  const int hk = h / (p.H / p.Hk);
  const int t0 = b * p.S + qt * kTile;
  const int qpos0 = qt * kTile;
  const int j_hi = p.causal ? qt : nqt - 1;
  const int j_lo = p.window > 0 ? max(0, qpos0 - p.window + 1) / kTile : 0;
  const int n = j_hi - j_lo + 1;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], 1);
      mbar_init(&p_full[i], 4);
    }
    mbar_init(o_done, 1);
    mbar_init(o_last, 1);
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
  // TMEM: S stages at columns [0, 128) and [128, 256) (fp32); P of a tile is written as
  // bf16 pairs over the first 64 columns of its own S stage; O at [256, 256 + DV).
  const uint32_t tS0 = tmem, tO = tmem + 256;

  if (warp == 0) {
    if (lane == 0) {
      mbar_arrive_expect_tx(q_full, L::kQ);
#pragma unroll
      for (int c = 0; c < NQC; ++c) tma_load_3d(sQ + c * kSubTile, &tmQ, q_full, c * 64, h, t0);
      bool ok = true;
      for (int jj = 0; jj < n && ok; ++jj) {
        const int kt0 = b * p.S + (j_lo + jj) * kTile;
        const int s = jj & 1;
        const uint32_t u = jj >> 1;
        if (!mbar_wait(&k_empty[s], (u & 1) ^ 1, p.status, STATUS_TIMEOUT_TMA_EMPTY)) { ok = false; break; }
        uint8_t* dK = sK + s * L::kK;
        mbar_arrive_expect_tx(&k_full[s], L::kK);
#pragma unroll
        for (int c = 0; c < NKC; ++c) tma_load_3d(dK + c * kSubTile, &tmK, &k_full[s], c * 64, hk, kt0);
        if (ROPE) tma_load_2d(dK + NKC * kSubTile, &tmKR, &k_full[s], 0, kt0);
        if (!mbar_wait(&v_empty[s], (u & 1) ^ 1, p.status, STATUS_TIMEOUT_TMA_EMPTY)) { ok = false; break; }
        uint8_t* dV = sV + s * L::kV;
        mbar_arrive_expect_tx(&v_full[s], L::kV);
#pragma unroll
        for (int half = 0; half < 2; ++half)
#pragma unroll
          for (int c = 0; c < VCH; ++c)
            tma_load_3d(dV + (half * VCH + c) * 8192, &tmV, &v_full[s], c * 64, hk, kt0 + half * 64);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc_s = umma_idesc_f16(128, 128, false, false, true);
      constexpr uint32_t idesc_o = umma_idesc_f16(128, DV, false, true, true);
      bool ok = mbar_wait(q_full, 0, p.status, STATUS_TIMEOUT_TMA_FULL);
      auto issue_s = [&](int jj) -> bool {
        const int s = jj & 1;
        const uint32_t u = jj >> 1;
        if (!mbar_wait(&k_full[s], u & 1, p.status, STATUS_TIMEOUT_TMA_FULL)) return false;
        if (!mbar_wait(&s_empty[s], (u & 1) ^ 1, p.status, STATUS_TIMEOUT_TMEM_EMPTY)) return false;
        tc_fence_after();
        const uint32_t qa = smem_u32(sQ), ka = smem_u32(sK + s * L::kK);
#pragma unroll
        for (int kk = 0; kk < DQ / 16; ++kk) {
          const uint32_t off = (kk >> 2) * kSubTile + (kk & 3) * 32;
          tc_mma_f16(tS0 + s * 128, umma_desc_sw128(qa + off, 16, 1024), umma_desc_sw128(ka + off, 16, 1024), idesc_s,
                     kk > 0 ? 1u : 0u);
        }
        tc_commit(&s_full[s]);
        tc_commit(&k_empty[s]);
        return true;
      };
      if (ok && n > 0) ok = issue_s(0);
      for (int jj = 0; jj < n && ok; ++jj) {
        const int s = jj & 1;
        const uint32_t u = jj >> 1;
        if (jj + 1 < n && !issue_s(jj + 1)) { ok = false; break; }
        if (!mbar_wait(&p_full[s], u & 1, p.status, STATUS_TIMEOUT_TMEM_FULL)) { ok = false; break; }
        if (!mbar_wait(&v_full[s], u & 1, p.status, STATUS_TIMEOUT_TMA_FULL)) { ok = false; break; }
        tc_fence_after();
        const uint32_t va = smem_u32(sV + s * L::kV);
#pragma unroll
        for (int kk = 0; kk < kTile / 16; ++kk) {
          const uint32_t boff = (kk >> 2) * (VCH * 8192) + (kk & 3) * 2048;
          tc_mma_f16_ts(tO, tS0 + s * 128 + kk * 8, umma_desc_sw128(va + boff, 8192, 1024), idesc_o,
                        (jj > 0 || kk > 0) ? 1u : 0u);
        }
        tc_commit(o_done);
        tc_commit(&v_empty[s]);
        tc_commit(&s_empty[s]);
      }
      if (ok && n > 0) tc_commit(o_last);
      tc_commit(drain);
      mbar_wait(drain, 0, p.status, STATUS_TIMEOUT_DRAIN);
    }
  } else {
    // ------------------------------ softmax warps -----------------------------
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const int qpos = qpos0 + r;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int jj = 0; jj < n; ++jj) {
      const int s = jj & 1;
      const uint32_t u = jj >> 1;
      if (!mbar_wait(&s_full[s], u & 1, p.status, STATUS_TIMEOUT_TMEM_FULL)) { ok = false; break; }
      tc_fence_after();
      float x[128];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(tS0 + s * 128 + c * 32 + lane_off, x + c * 32);
      tc_wait_ld();
      const int kpos0 = (j_lo + jj) * kTile;
      const bool need_mask = (p.causal && kpos0 + kTile - 1 > qpos0) ||
                             (p.window > 0 && kpos0 <= qpos0 + kTile - 1 - p.window);
      float mt = -INFINITY;
      if (need_mask) {
#pragma unroll
        for (int c = 0; c < 128; ++c) {
          float v = x[c] * p.scale_log2;
          const int kp = kpos0 + c;
          if ((p.causal && kp > qpos) || (p.window > 0 && kp <= qpos - p.window)) v = -INFINITY;
          x[c] = v;
          mt = fmaxf(mt, v);
        }
      } else {
#pragma unroll
        for (int c = 0; c < 128; ++c) {
          x[c] *= p.scale_log2;
          mt = fmaxf(mt, x[c]);
        }
      }
      const float m_new = fmaxf(m, mt);
      const bool need = m_new > m + 8.0f;
      const bool warp_need = __any_sync(0xffffffffu, need);
      float alpha = 1.f;
      if (need) {
        alpha = (m == -INFINITY) ? 0.f : exp2f(m - m_new);
        m = m_new;
      }
      const float m_use = (m == -INFINITY) ? 0.f : m;
      float sum = 0.f;
      uint32_t pk[64];
#pragma unroll
      for (int c = 0; c < 64; ++c) {
        const float e0 = exp2f(x[2 * c] - m_use), e1 = exp2f(x[2 * c + 1] - m_use);
        sum += e0 + e1;
        pk[c] = pack_bf16x2(e0, e1);
      }
      l = l * alpha + sum;
      // P (bf16) over the first 64 columns of this tile's S stage (S already in registers)
      tmem_st32_u32(tS0 + s * 128 + lane_off, pk);
      tmem_st32_u32(tS0 + s * 128 + 32 + lane_off, pk + 32);
      if (jj > 0 && warp_need) {
        // O must hold P.V of the previous tile before it is rescaled
        if (!mbar_wait(o_done, (jj - 1) & 1, p.status, STATUS_TIMEOUT_TMEM_FULL)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < DV / 32; ++c) {
          float o[32];
          tmem_ld32(tO + c * 32 + lane_off, o);
          tc_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] *= alpha;
          tmem_st32(tO + c * 32 + lane_off, o);
        }
      }
      tc_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[s]);
    }
    if (ok && n > 0 && mbar_wait(o_last, 0, p.status, STATUS_TIMEOUT_TMEM_FULL)) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      bf16* dst = p.o + (long long)(t0 + r) * p.o_row + (long long)h * p.o_head;
#pragma unroll
      for (int c = 0; c < DV / 32; ++c) {
        float o[32];
        tmem_ld32(tO + c * 32 + lane_off, o);
        tc_wait_ld();
        store_global_row(dst + c * 32, o, 32, inv);
      }
      const float m_use = (m == -INFINITY) ? 0.f : m;
      p.lse[(long long)h * p.T + t0 + r] = (m_use + log2f(l)) * kLn2;
    }
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ===========================================================================
// Backward: dK, dV
// ===========================================================================
template <int DQ, int DV>
struct DkdvSmem {
  static constexpr int BQ = 64;                    // query rows per iteration
  static constexpr int NQC = DQ / 64;
  static constexpr int kK = NQC * kSubTile;        // [128 kv x DQ]
  static constexpr int kV = (DV / 64) * kSubTile;  // [128 kv x DV]
  static constexpr int kQ = NQC * 8192;            // [64 q x DQ] (64-row sub-tiles)
  static constexpr int kDO = (DV / 64) * 8192;     // [64 q x DV]
  static constexpr int kVec = 2 * BQ * 4;          // lse[64], delta[64]
  static constexpr int NS = 3;                     // Q / dO / lse-delta ring stages
  static constexpr int kOffK = 0;
  static constexpr int kOffV = kOffK + kK;
  static constexpr int kOffQ = kOffV + kV;           // NS stages
  static constexpr int kOffDO = kOffQ + NS * kQ;     // NS stages
  static constexpr int kOffVec = kOffDO + NS * kDO;  // NS stages of lse/delta
  static constexpr int kOffBar = kOffVec + NS * kVec;
  static constexpr int kBytes = kOffBar + 256 + 1024;
};

// CTA = (kv tile of 128 rows, kv head, sequence); loops over query tiles of 64
// rows (and over the query heads of a GQA group).  Q/dO (with the tile's lse and
// delta, fetched by bulk copies on the same barrier) stream through a 3-stage ring,
// so a tile's loads start two iterations before its MMAs; S^T is double buffered in
// TMEM so K Q^T of the next tile runs during this tile's softmax.  The MMA thread
// issues V dO^T of this tile before K Q^T of the next one: the softmax warps wait for
// dP^T, while the next S^T is not needed until they finish this tile.  P^T and dS^T (bf16)
// are written over the two halves of their S^T stage and feed their MMAs
// (dV += P^T dO, dK += dS^T Q) straight from tensor memory: thread r holds row r
// of both, which is the A-operand layout.  dP^T is released as soon as the
// softmax has read it, so the next tile's V dO^T does not wait for dK.
//   TMEM columns: S^T -> [P^T | dS^T] [2] = [0, 64), [64, 128); dP^T = [128, 192);
//                 dV = [192, 192 + DV); dK = [192 + DV, 192 + DV + DQ)
template <int DQ, int DV, bool ROPE>
__global__ void __launch_bounds__(kBwdThreads, 1)
    attn_dkdv_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmKR, const __grid_constant__ CUtensorMap tmV,
                     const __grid_constant__ CUtensorMap tmDO, AttnArgs p) {
  using L = DkdvSmem<DQ, DV>;
  constexpr int BQ = L::BQ;
  constexpr int NQC = L::NQC;
  constexpr int NKC = ROPE ? NQC - 1 : NQC;
  constexpr int VCH = DV / 64;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = smem + L::kOffK;
  uint8_t* sV = smem + L::kOffV;
  uint8_t* sQ = smem + L::kOffQ;
  uint8_t* sDO = smem + L::kOffDO;
  float* sVec = reinterpret_cast<float*>(smem + L::kOffVec);  // [stage][lse 64 | delta 64]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kOffBar);
  constexpr int NS = L::NS;
  uint64_t* kv_full = bars + 0;
  uint64_t* q_full = bars + 1;    // [NS] Q + lse/delta
  uint64_t* q_empty = bars + 4;   // [NS]
  uint64_t* do_full = bars + 7;   // [NS]
  uint64_t* do_empty = bars + 10; // [NS]
  uint64_t* s_full = bars + 13;   // [2]
  uint64_t* s_empty = bars + 15;  // [2] S^T / P^T / dS^T stage free (commit after dK read dS^T)
  uint64_t* pt_ready = bars + 17; // one arrival per softmax warp
  uint64_t* dp_full = bars + 18;
  uint64_t* dp_empty = bars + 19; // one arrival per softmax warp: dP^T read
  uint64_t* ds_ready = bars + 20; // one arrival per softmax warp
  uint64_t* acc_done = bars + 21;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 22);

  const int warp = warp_id(), lane = lane_id();
  const int nqt = p.S / BQ;
  const int kt = blockIdx.x, hk = blockIdx.y, b = blockIdx.z;
  const int G = p.H / p.Hk;
  const int kpos0 = kt * kTile;
  const int kt0 = b * p.S + kpos0;
  const int i_lo = p.causal ? kpos0 / BQ : 0;
  const int i_hi = p.window > 0 ? min(nqt - 1, (kpos0 + kTile - 1 + p.window - 1) / BQ) : nqt - 1;
  const int nq = max(0, i_hi - i_lo + 1);
  const int n = nq * G;  // iterations (g, i), i fastest

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int i = 0; i < NS; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
      mbar_init(&do_full[i], 1);
      mbar_init(&do_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], 1);
    }
    mbar_init(pt_ready, kBwdSoftmaxWarps);
    mbar_init(dp_full, 1);
    mbar_init(dp_empty, kBwdSoftmaxWarps);
    mbar_init(ds_ready, kBwdSoftmaxWarps);
    mbar_init(acc_done, 1);
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
  const uint32_t tS0 = tmem, tdP = tmem + 128, tdV = tmem + 192, tdK = tmem + 192 + DV;

  if (warp == 0) {
    if (lane == 0) {
      mbar_arrive_expect_tx(kv_full, L::kK + L::kV);
#pragma unroll
      for (int c = 0; c < NKC; ++c) tma_load_3d(sK + c * kSubTile, &tmK, kv_full, c * 64, hk, kt0);
      if (ROPE) tma_load_2d(sK + NKC * kSubTile, &tmKR, kv_full, 0, kt0);
#pragma unroll
      for (int c = 0; c < VCH; ++c) tma_load_3d(sV + c * kSubTile, &tmV, kv_full, c * 64, hk, kt0);
      for (int it = 0; it < n; ++it) {
        const int g = it / nq, i = i_lo + it % nq;
        const int hq = hk * G + g;
        const int qrow0 = b * p.S + i * BQ;
        const int st = it % NS;
        const uint32_t u = it / NS;
        if (!mbar_wait(&q_empty[st], (u & 1) ^ 1, p.status, STATUS_TIMEOUT_TMA_EMPTY)) break;
        mbar_arrive_expect_tx(&q_full[st], L::kQ + L::kVec);
#pragma unroll
        for (int c = 0; c < NQC; ++c) tma_load_3d(sQ + st * L::kQ + c * 8192, &tmQ, &q_full[st], c * 64, hq, qrow0);
        const long long vidx = (long long)hq * p.T + qrow0;
        bulk_load(sVec + st * 2 * BQ, p.lse + vidx, BQ * 4, &q_full[st]);
        bulk_load(sVec + st * 2 * BQ + BQ, p.delta + vidx, BQ * 4, &q_full[st]);
        if (!mbar_wait(&do_empty[st], (u & 1) ^ 1, p.status, STATUS_TIMEOUT_TMA_EMPTY)) break;
        mbar_arrive_expect_tx(&do_full[st], L::kDO);
#pragma unroll
        for (int c = 0; c < VCH; ++c) tma_load_3d(sDO + st * L::kDO + c * 8192, &tmDO, &do_full[st], c * 64, hq, qrow0);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc_s = umma_idesc_f16(128, BQ, false, false, true);    // K Q^T, V dO^T
      constexpr uint32_t idesc_dv = umma_idesc_f16(128, DV, false, true, true);    // P^T dO
      constexpr uint32_t idesc_dk = umma_idesc_f16(128, DQ, false, true, true);    // dS^T Q
      bool ok = mbar_wait(kv_full, 0, p.status, STATUS_TIMEOUT_TMA_FULL);
      const uint32_t ka = smem_u32(sK), va = smem_u32(sV);
      auto issue_s = [&](int it) -> bool {
        const int qs = it % NS;                 // Q ring stage
        const int ts = it & 1;                  // S^T tensor-memory stage
        if (!mbar_wait(&q_full[qs], (it / NS) & 1, p.status, STATUS_TIMEOUT_TMA_FULL)) return false;
        if (!mbar_wait(&s_empty[ts], ((it >> 1) & 1) ^ 1, p.status, STATUS_TIMEOUT_TMEM_EMPTY)) return false;
        tc_fence_after();
        const uint32_t qa = smem_u32(sQ + qs * L::kQ);
#pragma unroll
        for (int kk = 0; kk < DQ / 16; ++kk)
          tc_mma_f16(tS0 + ts * 64, umma_desc_sw128(ka + (kk >> 2) * kSubTile + (kk & 3) * 32, 16, 1024),
                     umma_desc_sw128(qa + (kk >> 2) * 8192 + (kk & 3) * 32, 16, 1024), idesc_s, kk > 0 ? 1u : 0u);
        tc_commit(&s_full[ts]);
        return true;
      };
      // dK += dS^T Q of tile j  (dS^T from tensor memory; Q read as MN-major)
      auto issue_dk = [&](int j) -> bool {
        if (!mbar_wait(ds_ready, j & 1, p.status, STATUS_TIMEOUT_TMEM_FULL)) return false;
        tc_fence_after();
        const int qs = j % NS, ts = j & 1;
        const uint32_t qa = smem_u32(sQ + qs * L::kQ);
#pragma unroll
        for (int kk = 0; kk < BQ / 16; ++kk)
          tc_mma_f16_ts(tdK, tS0 + ts * 64 + 32 + kk * 8, umma_desc_sw128(qa + kk * 2048, 8192, 1024), idesc_dk,
                        (j > 0 || kk > 0) ? 1u : 0u);
        tc_commit(&s_empty[ts]);
        tc_commit(&q_empty[qs]);
        return true;
      };
      // Software pipeline, per iteration: dP^T(it), dK(it-1), S^T(it+1), dV(it).  dP^T of a tile
      // is issued as soon as the softmax warps have read the previous one, ahead of the previous
      // tile's dK, so it is ready when they finish P^T; S^T(it+1) reuses the tensor-memory stage
      // of tile it-1 and so follows dK(it-1).
      if (ok && n > 0) ok = issue_s(0);
      for (int it = 0; it < n && ok; ++it) {
        const int qs = it % NS;
        const uint32_t uq = it / NS;
        const int ts = it & 1;
        const uint32_t ph = it & 1;
        // dP^T = V dO^T
        if (!mbar_wait(&do_full[qs], uq & 1, p.status, STATUS_TIMEOUT_TMA_FULL)) { ok = false; break; }
        if (!mbar_wait(dp_empty, ph ^ 1, p.status, STATUS_TIMEOUT_TMEM_EMPTY)) { ok = false; break; }
        tc_fence_after();
        const uint32_t da = smem_u32(sDO + qs * L::kDO);
#pragma unroll
        for (int kk = 0; kk < DV / 16; ++kk)
          tc_mma_f16(tdP, umma_desc_sw128(va + (kk >> 2) * kSubTile + (kk & 3) * 32, 16, 1024),
                     umma_desc_sw128(da + (kk >> 2) * 8192 + (kk & 3) * 32, 16, 1024), idesc_s, kk > 0 ? 1u : 0u);
        tc_commit(dp_full);
        if (it > 0 && !issue_dk(it - 1)) { ok = false; break; }
        if (it + 1 < n && !issue_s(it + 1)) { ok = false; break; }
        // dV += P^T dO  (P^T from tensor memory; dO read as MN-major: DV contiguous, 64-row sub-tiles)
        if (!mbar_wait(pt_ready, ph, p.status, STATUS_TIMEOUT_TMEM_FULL)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < BQ / 16; ++kk)
          tc_mma_f16_ts(tdV, tS0 + ts * 64 + kk * 8, umma_desc_sw128(da + kk * 2048, 8192, 1024), idesc_dv,
                        (it > 0 || kk > 0) ? 1u : 0u);
        tc_commit(&do_empty[qs]);
      }
      if (ok && n > 0) ok = issue_dk(n - 1);
      tc_commit(acc_done);
      mbar_wait(acc_done, 0, p.status, STATUS_TIMEOUT_DRAIN);
    }
  } else {
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;   // columns [32 * half, 32 * half + 32) of each tile
    const int r = quarter * 32 + lane;  // kv row
    const int kpos = kpos0 + r;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    bool ok = true;
    for (int it = 0; it < n; ++it) {
      const int i = i_lo + it % nq;
      const int qpos0 = i * BQ + half * 32;
      const int qs = it % NS;
      const int st = it & 1;
      const uint32_t u = it >> 1;
      const uint32_t ph = it & 1;
      // lse / delta of this tile arrived with Q (make the bulk-copy writes visible here)
      if (!mbar_wait(&q_full[qs], (it / NS) & 1, p.status, STATUS_TIMEOUT_TMA_FULL)) { ok = false; break; }
      if (!mbar_wait(&s_full[st], u & 1, p.status, STATUS_TIMEOUT_TMEM_FULL)) { ok = false; break; }
      tc_fence_after();
      float P[32];
      tmem_ld32(tS0 + st * 64 + half * 32 + lane_off, P);
      tc_wait_ld();
      const float* lse = sVec + qs * 2 * BQ + half * 32;
      const float* delta = lse + BQ;
      const bool need_mask = (p.causal && kpos0 + kTile - 1 > qpos0) ||
                             (p.window > 0 && kpos0 <= qpos0 + 31 - p.window);
#pragma unroll
      for (int c = 0; c < 32; ++c) {
        float v = fast_exp2(P[c] * p.scale_log2 - lse[c] * kLog2e);
        if (need_mask) {
          const int qp = qpos0 + c;
          if ((p.causal && kpos > qp) || (p.window > 0 && kpos <= qp - p.window)) v = 0.f;
        }
        P[c] = v;
      }
      {
        // P^T (bf16) into the first half of this S^T stage: the A operand of dV += P^T dO
        uint32_t pk[16];
#pragma unroll
        for (int c = 0; c < 16; ++c) pk[c] = pack_bf16x2(P[2 * c], P[2 * c + 1]);
        tmem_st16_u32(tS0 + st * 64 + half * 16 + lane_off, pk);
        tc_wait_st();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(pt_ready);
      if (!mbar_wait(dp_full, ph, p.status, STATUS_TIMEOUT_TMEM_FULL)) { ok = false; break; }
      tc_fence_after();
      float d[32];
      tmem_ld32(tdP + half * 32 + lane_off, d);
      tc_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(dp_empty);
      {
        // dS^T (bf16) into the second half of this S^T stage: the A operand of dK += dS^T Q
        uint32_t pk[16];
#pragma unroll
        for (int c = 0; c < 16; ++c)
          pk[c] = pack_bf16x2(P[2 * c] * (d[2 * c] - delta[2 * c]) * p.scale,
                              P[2 * c + 1] * (d[2 * c + 1] - delta[2 * c + 1]) * p.scale);
        tmem_st16_u32(tS0 + st * 64 + 32 + half * 16 + lane_off, pk);
        tc_wait_st();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(ds_ready);
    }
    if (ok && n > 0 && mbar_wait(acc_done, 0, p.status, STATUS_TIMEOUT_TMEM_FULL)) {
      tc_fence_after();
      const long long t = kt0 + r;
      if (half == 0) {
        bf16* dv = p.dv + t * p.dv_row + (long long)hk * p.dv_head;
#pragma unroll
        for (int c = 0; c < DV / 32; ++c) {
          float v[32];
          tmem_ld32(tdV + c * 32 + lane_off, v);
          tc_wait_ld();
          store_global_row(dv + c * 32, v, 32, 1.f);
        }
      } else {
        bf16* dk = p.dk + t * p.dk_row + (long long)hk * p.dk_head;
#pragma unroll
        for (int c = 0; c < NKC * 2; ++c) {
          float v[32];
          tmem_ld32(tdK + c * 32 + lane_off, v);
          tc_wait_ld();
          store_global_row(dk + c * 32, v, 32, 1.f);
        }
        if (ROPE) {
          bf16* dkr = p.dkr + t * p.dkr_row + (long long)hk * p.dkr_head;
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            float v[32];
            tmem_ld32(tdK + NKC * 64 + c * 32 + lane_off, v);
            tc_wait_ld();
            store_global_row(dkr + c * 32, v, 32, 1.f);
          }
        }
      }
    } else if (n == 0) {
      // no query attends to this kv tile: zero gradients
      const long long t = kt0 + r;
      float z[32] = {0};
      if (half == 0) {
        for (int c = 0; c < DV / 32; ++c) store_global_row(p.dv + t * p.dv_row + (long long)hk * p.dv_head + c * 32, z, 32, 1.f);
      } else {
        for (int c = 0; c < NKC * 2; ++c) store_global_row(p.dk + t * p.dk_row + (long long)hk * p.dk_head + c * 32, z, 32, 1.f);
        if (ROPE)
          for (int c = 0; c < 2; ++c)
            store_global_row(p.dkr + t * p.dkr_row + (long long)hk * p.dkr_head + c * 32, z, 32, 1.f);
      }
    }
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ===========================================================================
// Backward: dQ
// ===========================================================================
template <int DQ, int DV>
struct DqSmem {
  static constexpr int BK = 64;                      // key rows per iteration
  static constexpr int NQC = DQ / 64;
  static constexpr int kQ = NQC * kSubTile;          // [128 q x DQ]
  static constexpr int kDO = (DV / 64) * kSubTile;   // [128 q x DV]
  static constexpr int kK = NQC * 8192;              // [64 kv x DQ] (64-row sub-tiles)
  static constexpr int kV = (DV / 64) * 8192;        // [64 kv x DV]
  static constexpr int NS = 3;                       // K / V ring stages
  static constexpr int kOffQ = 0;
  static constexpr int kOffDO = kOffQ + kQ;
  static constexpr int kOffK = kOffDO + kDO;         // NS stages
  static constexpr int kOffV = kOffK + NS * kK;      // NS stages
  static constexpr int kOffBar = kOffV + NS * kV;
  static constexpr int kBytes = kOffBar + 256 + 1024;
};

// CTA = (query tile of 128 rows, head, sequence); loops over key tiles of 64 rows.
// K/V tiles stream through a 3-stage ring (a tile's loads start two iterations ahead)
// and the S / dP accumulators (TMEM) are double buffered: the next tile's
// S = Q K^T, dP = dO V^T run while this tile's dS is formed, and dQ += dS K of
// this tile follows.  dS (bf16) is written over its dP stage
// and read by the MMA from tensor memory (thread = query row = A-operand row).
//   TMEM columns: S[2] = [0, 128), dP / dS [2] = [128, 256), dQ = [256, 256 + DQ)
template <int DQ, int DV, bool ROPE>
__global__ void __launch_bounds__(kBwdThreads, 1)
    attn_dq_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmKR, const __grid_constant__ CUtensorMap tmV,
                   const __grid_constant__ CUtensorMap tmDO, AttnArgs p) {
  using L = DqSmem<DQ, DV>;
  constexpr int BK = L::BK;
  constexpr int NQC = L::NQC;
  constexpr int NKC = ROPE ? NQC - 1 : NQC;
  constexpr int VCH = DV / 64;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem + L::kOffQ;
  uint8_t* sDO = smem + L::kOffDO;
  uint8_t* sK = smem + L::kOffK;
  uint8_t* sV = smem + L::kOffV;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kOffBar);
  constexpr int NS = L::NS;
  uint64_t* q_full = bars + 0;
  uint64_t* kv_full = bars + 1;    // [NS]
  uint64_t* kv_empty = bars + 4;   // [NS]
  uint64_t* sdp_full = bars + 7;   // [2]
  uint64_t* sdp_empty = bars + 9;  // [2] S / dP(dS) stage free (commit after dQ read dS)
  uint64_t* ds_ready = bars + 11;  // [2] one arrival per softmax warp, per dS stage
  uint64_t* acc_done = bars + 13;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 14);

  const int warp = warp_id(), lane = lane_id();
  const int nqt = p.S / kTile;
  const int qt = nqt - 1 - blockIdx.x;
  const int h = blockIdx.y, b = blockIdx.z;
  const int hk = h / (p.H / p.Hk);
  const int t0 = b * p.S + qt * kTile;
  const int qpos0 = qt * kTile;
  const int nkt = p.S / BK;
  const int j_hi = p.causal ? (qpos0 + kTile - 1) / BK : nkt - 1;
  const int j_lo = p.window > 0 ? max(0, qpos0 - p.window + 1) / BK : 0;
  const int n = j_hi - j_lo + 1;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < NS; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sdp_full[i], 1);
      mbar_init(&sdp_empty[i], 1);
      mbar_init(&ds_ready[i], kBwdSoftmaxWarps);
    }
    mbar_init(acc_done, 1);
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
  const uint32_t tS0 = tmem, tdP0 = tmem + 128, tdQ = tmem + 256;

  if (warp == 0) {
    if (lane == 0) {
      mbar_arrive_expect_tx(q_full, L::kQ + L::kDO);
#pragma unroll
      for (int c = 0; c < NQC; ++c) tma_load_3d(sQ + c * kSubTile, &tmQ, q_full, c * 64, h, t0);
#pragma unroll
      for (int c = 0; c < VCH; ++c) tma_load_3d(sDO + c * kSubTile, &tmDO, q_full, c * 64, h, t0);
      for (int jj = 0; jj < n; ++jj) {
        const int kt0 = b * p.S + (j_lo + jj) * BK;
        const int st = jj % NS;
        const uint32_t u = jj / NS;
        if (!mbar_wait(&kv_empty[st], (u & 1) ^ 1, p.status, STATUS_TIMEOUT_TMA_EMPTY)) break;
        mbar_arrive_expect_tx(&kv_full[st], L::kK + L::kV);
        uint8_t* dK = sK + st * L::kK;
        uint8_t* dV = sV + st * L::kV;
#pragma unroll
        for (int c = 0; c < NKC; ++c) tma_load_3d(dK + c * 8192, &tmK, &kv_full[st], c * 64, hk, kt0);
        if (ROPE) tma_load_2d(dK + NKC * 8192, &tmKR, &kv_full[st], 0, kt0);
#pragma unroll
        for (int c = 0; c < VCH; ++c) tma_load_3d(dV + c * 8192, &tmV, &kv_full[st], c * 64, hk, kt0);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc_s = umma_idesc_f16(128, BK, false, false, true);
      constexpr uint32_t idesc_dq = umma_idesc_f16(128, DQ, false, true, true);
      bool ok = mbar_wait(q_full, 0, p.status, STATUS_TIMEOUT_TMA_FULL);
      const uint32_t qa = smem_u32(sQ), da = smem_u32(sDO);
      auto issue_sdp = [&](int jj) -> bool {
        const int ks = jj % NS;                 // K / V ring stage
        const int st = jj & 1;                  // S / dP tensor-memory stage
        const uint32_t u = jj >> 1;
        if (!mbar_wait(&kv_full[ks], (jj / NS) & 1, p.status, STATUS_TIMEOUT_TMA_FULL)) return false;
        if (!mbar_wait(&sdp_empty[st], (u & 1) ^ 1, p.status, STATUS_TIMEOUT_TMEM_EMPTY)) return false;
        tc_fence_after();
        const uint32_t ka = smem_u32(sK + ks * L::kK), va = smem_u32(sV + ks * L::kV);
#pragma unroll
        for (int kk = 0; kk < DQ / 16; ++kk)
          tc_mma_f16(tS0 + st * 64, umma_desc_sw128(qa + (kk >> 2) * kSubTile + (kk & 3) * 32, 16, 1024),
                     umma_desc_sw128(ka + (kk >> 2) * 8192 + (kk & 3) * 32, 16, 1024), idesc_s, kk > 0 ? 1u : 0u);
#pragma unroll
        for (int kk = 0; kk < DV / 16; ++kk)
          tc_mma_f16(tdP0 + st * 64, umma_desc_sw128(da + (kk >> 2) * kSubTile + (kk & 3) * 32, 16, 1024),
                     umma_desc_sw128(va + (kk >> 2) * 8192 + (kk & 3) * 32, 16, 1024), idesc_s, kk > 0 ? 1u : 0u);
        tc_commit(&sdp_full[st]);
        return true;
      };
      if (ok && n > 0) ok = issue_sdp(0);
      for (int jj = 0; jj < n && ok; ++jj) {
        const int st = jj & 1;
        if (jj + 1 < n && !issue_sdp(jj + 1)) { ok = false; break; }
        if (!mbar_wait(&ds_ready[st], (jj >> 1) & 1, p.status, STATUS_TIMEOUT_TMEM_FULL)) { ok = false; break; }
        tc_fence_after();
        // dQ += dS K   (dS from tensor memory; K tile read as MN-major: d contiguous, 64-row sub-tiles)
        const int ks = jj % NS;
        const uint32_t ka = smem_u32(sK + ks * L::kK);
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk)
          tc_mma_f16_ts(tdQ, tdP0 + st * 64 + kk * 8, umma_desc_sw128(ka + kk * 2048, 8192, 1024), idesc_dq,
                        (jj > 0 || kk > 0) ? 1u : 0u);
        tc_commit(&kv_empty[ks]);
        tc_commit(&sdp_empty[st]);
      }
      tc_commit(acc_done);
      mbar_wait(acc_done, 0, p.status, STATUS_TIMEOUT_DRAIN);
    }
  } else {
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;   // key columns [32 * half, 32 * half + 32) of each tile
    const int r = quarter * 32 + lane;
    const int qpos = qpos0 + r;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const long long li = (long long)h * p.T + t0 + r;
    const float lse2 = p.lse[li] * kLog2e;
    const float dlt = p.delta[li];
    bool ok = true;
    for (int jj = 0; jj < n; ++jj) {
      const int st = jj & 1;
      const uint32_t u = jj >> 1;
      const int kpos0 = (j_lo + jj) * BK + half * 32;
      if (!mbar_wait(&sdp_full[st], u & 1, p.status, STATUS_TIMEOUT_TMEM_FULL)) { ok = false; break; }
      tc_fence_after();
      float sv[32], d[32];
      tmem_ld32(tS0 + st * 64 + half * 32 + lane_off, sv);
      tmem_ld32(tdP0 + st * 64 + half * 32 + lane_off, d);
      tc_wait_ld();
      const bool need_mask = (p.causal && kpos0 + 31 > qpos0) ||
                             (p.window > 0 && kpos0 <= qpos0 + kTile - 1 - p.window);
#pragma unroll
      for (int k = 0; k < 32; ++k) {
        float pv = fast_exp2(sv[k] * p.scale_log2 - lse2);
        if (need_mask) {
          const int kp = kpos0 + k;
          if ((p.causal && kp > qpos) || (p.window > 0 && kp <= qpos - p.window)) pv = 0.f;
        }
        d[k] = pv * (d[k] - dlt) * p.scale;
      }
      {
        // dS (bf16) into this dP stage (first 32 columns): the A operand of dQ += dS K
        uint32_t pk[16];
#pragma unroll
        for (int c = 0; c < 16; ++c) pk[c] = pack_bf16x2(d[2 * c], d[2 * c + 1]);
        tmem_st16_u32(tdP0 + st * 64 + half * 16 + lane_off, pk);
        tc_wait_st();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&ds_ready[st]);
    }
    if (ok && n > 0 && mbar_wait(acc_done, 0, p.status, STATUS_TIMEOUT_TMEM_FULL)) {
      tc_fence_after();
      bf16* dst = p.dq + (long long)(t0 + r) * p.dq_row + (long long)h * p.dq_head;
      constexpr int CH = DQ / 64;  // 32-column chunks per half
#pragma unroll
      for (int c = half * CH; c < (half + 1) * CH; ++c) {
        float v[32];
        tmem_ld32(tdQ + c * 32 + lane_off, v);
        tc_wait_ld();
        store_global_row(dst + c * 32, v, 32, 1.f);
      }
    }
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// delta[h*T + t] = sum_d dO[t,h,d] * O[t,h,d]   (one warp per (t, h))
__global__ void attn_delta_kernel(const bf16* __restrict__ dO, long long do_row, long long do_head,
                                  const bf16* __restrict__ O, long long o_row, long long o_head, float* __restrict__ delta,
                                  int T, int H, int DV) {
  const long long w = blockIdx.x * (long long)(blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (w >= (long long)T * H) return;
  const int t = (int)(w / H), h = (int)(w % H);
  const bf16* a = dO + t * do_row + h * do_head;
  const bf16* c = O + t * o_row + h * o_head;
  float s = 0.f;
  for (int d = lane * 2; d < DV; d += 64) {
    s += __bfloat162float(a[d]) * __bfloat162float(c[d]) + __bfloat162float(a[d + 1]) * __bfloat162float(c[d + 1]);
  }
  s = warp_sum(s);
  if (lane == 0) delta[(long long)h * T + t] = s;
}

// ===========================================================================
// Host launchers
// ===========================================================================
static CUtensorMap map_heads(const void* base, int d, int heads, int T, long long row, long long head, int box_rows,
                             const char* what) {
  uint64_t dims[3] = {(uint64_t)d, (uint64_t)heads, (uint64_t)T};
  uint64_t str[2] = {(uint64_t)head * 2, (uint64_t)row * 2};
  uint32_t box[3] = {64, 1, (uint32_t)box_rows};
  return make_tmap_bf16(base, 3, dims, str, box, what);
}

static CUtensorMap map_rope(const void* base, int T, long long row, const char* what, int box_rows = 128) {
  uint64_t dims[2] = {64, (uint64_t)T};
  uint64_t str[1] = {(uint64_t)row * 2};
  uint32_t box[2] = {64, (uint32_t)box_rows};
  return make_tmap_bf16(base, 2, dims, str, box, what);
}

static void check_shapes(const AttnTensors& a) {
  if (a.S % kTile != 0) throw std::runtime_error("omnicoder attention: sequence length must be a multiple of 128");
  if (a.T % a.S != 0) throw std::runtime_error("omnicoder attention: token count must be a multiple of seq");
  if (a.H % a.Hk != 0) throw std::runtime_error("omnicoder attention: heads must be a multiple of kv heads");
  if (!((a.DQ == 64 || a.DQ == 128 || a.DQ == 192) && (a.DV == 64 || a.DV == 128)))
    throw std::runtime_error("omnicoder attention: head dims must be q/k in {64,128,192}, v in {64,128}");
  if (a.DR != 0 && a.DR != 64) throw std::runtime_error("omnicoder attention: shared rope key must have 64 dims");
}

template <typename K>
static void set_smem(K kern, int bytes) {
  ensure_smem_attr(reinterpret_cast<const void*>(kern), bytes);
}

template <int DQ, int DV, bool ROPE>
static void fwd_impl(const AttnTensors& a, void* o, float* lse, void* status, cudaStream_t s) {
  const int DK = DQ - (ROPE ? 64 : 0);
  CUtensorMap tq = map_heads(a.q, DQ, a.H, a.T, a.q_row, a.q_head, 128, "attention q");
  CUtensorMap tk = map_heads(a.k, DK, a.Hk, a.T, a.k_row, a.k_head, 128, "attention k");
  CUtensorMap tkr = ROPE ? map_rope(a.kr, a.T, a.kr_row, "attention k_rope") : tk;
  CUtensorMap tv = map_heads(a.v, DV, a.Hk, a.T, a.v_row, a.v_head, 64, "attention v");
  AttnArgs p{};
  p.T = a.T; p.S = a.S; p.H = a.H; p.Hk = a.Hk;
  p.scale = a.scale; p.scale_log2 = a.scale * kLog2e;
  p.causal = a.causal; p.window = a.window;
  p.o = (bf16*)o; p.o_row = (long long)a.H * DV; p.o_head = DV;
  p.lse = lse;
  p.status = (StatusBlock*)status;
  using L = FwdSmem<DQ, DV, ROPE>;
  auto kern = attn_fwd_kernel<DQ, DV, ROPE>;
  set_smem(kern, L::kBytes);
  dim3 grid(a.S / kTile, a.H, a.T / a.S);
  kern<<<grid, kAttnThreads, L::kBytes, s>>>(tq, tk, tkr, tv, p);
}

template <int DQ, int DV, bool ROPE>
static void bwd_impl(const AttnTensors& a, const void* o, const float* lse, const void* dO, float* delta, void* dq,
                     long long dq_row, long long dq_head, void* dk, long long dk_row, long long dk_head, void* dkr, long long dkr_row, long long dkr_head,
                     void* dv, long long dv_row, long long dv_head, void* status, cudaStream_t s) {
  const int DK = DQ - (ROPE ? 64 : 0);
  // delta = rowsum(dO * O)
  {
    const long long warps = (long long)a.T * a.H;
    attn_delta_kernel<<<(unsigned)((warps + 7) / 8), 256, 0, s>>>((const bf16*)dO, (long long)a.H * DV, DV,
                                                                   (const bf16*)o, (long long)a.H * DV, DV, delta,
                                                                   a.T, a.H, DV);
  }
  CUtensorMap tq = map_heads(a.q, DQ, a.H, a.T, a.q_row, a.q_head, 128, "attention q");
  CUtensorMap tk = map_heads(a.k, DK, a.Hk, a.T, a.k_row, a.k_head, 128, "attention k");
  CUtensorMap tkr = ROPE ? map_rope(a.kr, a.T, a.kr_row, "attention k_rope") : tk;
  CUtensorMap tv = map_heads(a.v, DV, a.Hk, a.T, a.v_row, a.v_head, 128, "attention v");
  CUtensorMap tdo = map_heads(dO, DV, a.H, a.T, (long long)a.H * DV, DV, 128, "attention dO");
  AttnArgs p{};
  p.T = a.T; p.S = a.S; p.H = a.H; p.Hk = a.Hk;
  p.scale = a.scale; p.scale_log2 = a.scale * kLog2e;
  p.causal = a.causal; p.window = a.window;
  p.lse = const_cast<float*>(lse);
  p.delta = delta;
  p.dq = (bf16*)dq; p.dq_row = dq_row; p.dq_head = dq_head;
  p.dk = (bf16*)dk; p.dk_row = dk_row; p.dk_head = dk_head;
  p.dkr = (bf16*)dkr; p.dkr_row = dkr_row; p.dkr_head = dkr_head;
  p.dv = (bf16*)dv; p.dv_row = dv_row; p.dv_head = dv_head;
  p.status = (StatusBlock*)status;
  {
    using L = DkdvSmem<DQ, DV>;
    CUtensorMap tq64 = map_heads(a.q, DQ, a.H, a.T, a.q_row, a.q_head, L::BQ, "attention q (64-row tiles)");
    CUtensorMap tdo64 = map_heads(dO, DV, a.H, a.T, (long long)a.H * DV, DV, L::BQ, "attention dO (64-row tiles)");
    auto kern = attn_dkdv_kernel<DQ, DV, ROPE>;
    set_smem(kern, L::kBytes);
    dim3 grid(a.S / kTile, a.Hk, a.T / a.S);
    kern<<<grid, kBwdThreads, L::kBytes, s>>>(tq64, tk, tkr, tv, tdo64, p);
  }
  {
    using L = DqSmem<DQ, DV>;
    CUtensorMap tk64 = map_heads(a.k, DK, a.Hk, a.T, a.k_row, a.k_head, L::BK, "attention k (64-row tiles)");
    CUtensorMap tkr64 = ROPE ? map_rope(a.kr, a.T, a.kr_row, "attention k_rope (64-row tiles)", L::BK) : tk64;
    CUtensorMap tv64 = map_heads(a.v, DV, a.Hk, a.T, a.v_row, a.v_head, L::BK, "attention v (64-row tiles)");
    auto kern = attn_dq_kernel<DQ, DV, ROPE>;
    set_smem(kern, L::kBytes);
    dim3 grid(a.S / kTile, a.H, a.T / a.S);
    kern<<<grid, kBwdThreads, L::kBytes, s>>>(tq, tk64, tkr64, tv64, tdo, p);
  }
}

#define OMNI_ATTN_DISPATCH(FN, ...)                                                              \
  do {                                                                                           \
    const bool rope = a.DR == 64;                                                                \
    if (a.DQ == 192 && a.DV == 128 && rope) FN<192, 128, true>(__VA_ARGS__);                     \
    else if (a.DQ == 128 && a.DV == 128 && !rope) FN<128, 128, false>(__VA_ARGS__);              \
    else if (a.DQ == 64 && a.DV == 64 && !rope) FN<64, 64, false>(__VA_ARGS__);                  \
    else if (a.DQ == 128 && a.DV == 128 && rope) FN<128, 128, true>(__VA_ARGS__);                \
    else if (a.DQ == 192 && a.DV == 128 && !rope) FN<192, 128, false>(__VA_ARGS__);              \
    else throw std::runtime_error("omnicoder attention: unsupported head-dim combination");     \
  } while (0)

void attention_fwd(const AttnTensors& a, void* o, float* lse, void* status, cudaStream_t s) {
  check_shapes(a);
  OMNI_ATTN_DISPATCH(fwd_impl, a, o, lse, status, s);
}

void attention_bwd(const AttnTensors& a, const void* o, const float* lse, const void* dO, float* delta, void* dq,
                   long long dq_row, long long dq_head, void* dk, long long dk_row, long long dk_head, void* dkr, long long dkr_row, long long dkr_head,
                   void* dv, long long dv_row, long long dv_head, void* status, cudaStream_t s) {
  check_shapes(a);
  OMNI_ATTN_DISPATCH(bwd_impl, a, o, lse, dO, delta, dq, dq_row, dq_head, dk, dk_row, dk_head, dkr, dkr_row, dkr_head, dv, dv_row,
                     dv_head, status, s);
}

}  // namespace omni
