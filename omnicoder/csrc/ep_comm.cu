// Expert-parallel dispatch / combine over NVLink 5 peer memory (sm_100a).
//
// Every rank owns E / N experts.  Each rank's receive region lives in a
// symmetric (peer-mapped) allocation, so these kernels move tokens with plain
// loads and stores to other GPUs' memory over NVSwitch, fused with the work
// around the exchange:
//   ep_dispatch   router permutation + all-to-all: each (token, k) pair is
//                 written straight into its slot of the owner's expert-major,
//                 128-row padded receive slab (the layout the grouped tcgen05
//                 GEMM consumes), with its routing weight and origin.
//   ep_combine    all-to-all back + weighted sum + residual/shared-expert add:
//                 each token pulls its k expert outputs from the owners.
//   ep_owner_bwd  combine backward on the owner: routing-weight gradient
//                 <dout, y> (written back to the source rank) and dout * w.
// No TMA and no multicast is used here; ep_barrier orders the phases with
// release/acquire flags at system scope and a bounded wait (status word on
// timeout, never a trap).
//
// The reference has no expert parallelism: its launcher only sets an
// environment variable (src/omnicoder/tools/torchrun_ep.py:36-38) and the MoE
// layer keeps every expert on every rank (src/omnicoder/modeling/moe_layer.py).
#include <algorithm>

#include "common.cuh"
#include "ep_comm.h"
#include "kernels.h"

namespace omni {

using bf16 = __nv_bfloat16;

namespace {

constexpr int kWarps = 8;

__device__ __forceinline__ void acc_add8(float* acc, const uint4& v, float w) {
  const uint32_t* q = reinterpret_cast<const uint32_t*>(&v);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    acc[2 * j] += w * bf16_lo(q[j]);
    acc[2 * j + 1] += w * bf16_hi(q[j]);
  }
}

__device__ __forceinline__ uint4 pack8(const float* a) {
  uint4 o;
  o.x = pack_bf16x2(a[0], a[1]);
  o.y = pack_bf16x2(a[2], a[3]);
  o.z = pack_bf16x2(a[4], a[5]);
  o.w = pack_bf16x2(a[6], a[7]);
  return o;
}

__global__ void ep_dispatch_kernel(const bf16* __restrict__ x, const int* __restrict__ idx,
                                   const int* __restrict__ pos, const int* __restrict__ loc_off,
                                   const int* __restrict__ dst_base, const int* __restrict__ keep_lim,
                                   const float* __restrict__ wts, EpPeers xr, EpPeers meta, int* __restrict__ slot,
                                   int TK, int K, int E, int El, int D, int me, StatusBlock* st) {
  const int lane = threadIdx.x & 31;
  for (int i = blockIdx.x * kWarps + (threadIdx.x >> 5); i < TK; i += gridDim.x * kWarps) {
    const int e = idx[i];
    const int p = pos[i];
    int row = -1, owner = 0;
    if (e >= 0 && e < E && p >= 0) {
      const int lr = p - loc_off[e];
      if (lr >= 0 && lr < keep_lim[e]) {
        owner = e / El;
        row = dst_base[e] + lr;
        if (row >= xr.rows[owner]) {
          if (lane == 0) report_error(st, STATUS_BAD_INDEX, row);
          row = -1;
        }
      }
    } else if (lane == 0 && (e < 0 || e >= E)) {
      report_error(st, STATUS_BAD_INDEX, e);
    }
    if (lane == 0) slot[i] = row;
    if (row < 0) continue;
    const bf16* src = x + (long long)(i / K) * D;
    bf16* dst = reinterpret_cast<bf16*>(xr.ptr[owner]) + (long long)row * D;
    for (int c = lane * 8; c < D; c += 256)
      *reinterpret_cast<uint4*>(dst + c) = *reinterpret_cast<const uint4*>(src + c);
    if (lane == 0 && meta.ptr[owner] != 0ull) {
      int4 m = make_int4(__float_as_int(wts[i]), me, i, 0);
      reinterpret_cast<int4*>(meta.ptr[owner])[row] = m;
    }
  }
}

__global__ void ep_push_kernel(const bf16* __restrict__ src, const int* __restrict__ slot,
                               const int* __restrict__ idx, EpPeers dst, int TK, int K, int El, int D,
                               StatusBlock* st) {
  const int lane = threadIdx.x & 31;
  for (int i = blockIdx.x * kWarps + (threadIdx.x >> 5); i < TK; i += gridDim.x * kWarps) {
    const int row = slot[i];
    if (row < 0) continue;
    const int owner = idx[i] / El;
    if (owner < 0 || owner >= kEpMaxRanks || row >= dst.rows[owner]) {
      if (lane == 0) report_error(st, STATUS_BAD_INDEX, row);
      continue;
    }
    const bf16* s = src + (long long)(i / K) * D;
    bf16* d = reinterpret_cast<bf16*>(dst.ptr[owner]) + (long long)row * D;
    for (int c = lane * 8; c < D; c += 256)
      *reinterpret_cast<uint4*>(d + c) = *reinterpret_cast<const uint4*>(s + c);
  }
}

// One warp per token; the k remote rows of a 256-column chunk are loaded
// before they are accumulated so that up to 8 NVLink loads are in flight per lane.
template <int KMAX>
__global__ void ep_combine_kernel(const int* __restrict__ slot, const int* __restrict__ idx,
                                  const float* __restrict__ w, EpPeers y, const bf16* __restrict__ add,
                                  bf16* __restrict__ out, int T, int K, int El, int D,
                                  const bf16* __restrict__ local) {
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * kWarps + (threadIdx.x >> 5);
  if (t >= T) return;
  const bf16* rows[KMAX];
  float wk[KMAX];
#pragma unroll
  for (int k = 0; k < KMAX; ++k) {
    rows[k] = nullptr;
    wk[k] = 0.f;
    if (k < K) {
      const int s = slot[(long long)t * K + k];
      if (s >= 0 && local != nullptr) {
        // the owners pushed their output rows to this rank's (token, k) slots
        rows[k] = local + ((long long)t * K + k) * D;
        wk[k] = w != nullptr ? w[(long long)t * K + k] : 1.f;
      } else if (s >= 0) {
        const int owner = idx[(long long)t * K + k] / El;
        if (owner >= 0 && owner < kEpMaxRanks && s < y.rows[owner]) {
          rows[k] = reinterpret_cast<const bf16*>(y.ptr[owner]) + (long long)s * D;
          wk[k] = w != nullptr ? w[(long long)t * K + k] : 1.f;
        }
      }
    }
  }
  for (int c = lane * 8; c < D; c += 256) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if (add != nullptr) acc_add8(acc, *reinterpret_cast<const uint4*>(add + (long long)t * D + c), 1.f);
    uint4 v[KMAX];
#pragma unroll
    for (int k = 0; k < KMAX; ++k)
      if (rows[k] != nullptr) v[k] = *reinterpret_cast<const uint4*>(rows[k] + c);
#pragma unroll
    for (int k = 0; k < KMAX; ++k)
      if (rows[k] != nullptr) acc_add8(acc, v[k], wk[k]);
    *reinterpret_cast<uint4*>(out + (long long)t * D + c) = pack8(acc);
  }
}

// Owner rows back to their origins: row r of y (r < offsets[El]) goes to ys_peer[s] + i * D with
// (-, s, i, -) = meta[r]; padding rows (s < 0) stay.  One warp per row, whole rows per store
// sequence.  (The block-scaled GEMM writes its expert outputs locally and this kernel returns
// them; the bf16 GEMM returns them from its epilogue.)
__global__ void ep_return_rows_kernel(const bf16* __restrict__ y, const int4* __restrict__ meta,
                                      const int* __restrict__ offsets, int El, EpPeers ys, int rows, int D,
                                      StatusBlock* st) {
  const int lane = threadIdx.x & 31;
  const int total = min(rows, offsets[El]);
  for (int r = blockIdx.x * kWarps + (threadIdx.x >> 5); r < total; r += gridDim.x * kWarps) {
    const int4 m = meta[r];
    if (m.y < 0) continue;
    if (m.y >= kEpMaxRanks || m.z < 0 || m.z >= ys.rows[m.y]) {
      if (lane == 0) report_error(st, STATUS_BAD_INDEX, m.z);
      continue;
    }
    const bf16* src = y + (long long)r * D;
    bf16* dst = reinterpret_cast<bf16*>(ys.ptr[m.y]) + (long long)m.z * D;
    for (int c = lane * 8; c < D; c += 256)
      *reinterpret_cast<uint4*>(dst + c) = *reinterpret_cast<const uint4*>(src + c);
  }
}

// Combine backward on the source rank when the owners pushed their outputs to its (token, k)
// slots ys: dwts[pair] = <dout[t], ys[pair]> (read locally) and the weighted output gradient
// dout[t] * w[pair] pushed into the owner's receive row slot[pair].  One warp per pair.
__global__ void ep_source_bwd_kernel(const bf16* __restrict__ dout, const bf16* __restrict__ ys,
                                     const int* __restrict__ slot, const int* __restrict__ idx,
                                     const float* __restrict__ w, float* __restrict__ dwts, EpPeers dy, int TK, int K,
                                     int El, int D, StatusBlock* st) {
  const int lane = threadIdx.x & 31;
  for (int i = blockIdx.x * kWarps + (threadIdx.x >> 5); i < TK; i += gridDim.x * kWarps) {
    const int row = slot[i];
    if (row < 0) {
      if (lane == 0) dwts[i] = 0.f;
      continue;
    }
    const int owner = idx[i] / El;
    if (owner < 0 || owner >= kEpMaxRanks || row >= dy.rows[owner]) {
      if (lane == 0) {
        dwts[i] = 0.f;
        report_error(st, STATUS_BAD_INDEX, row);
      }
      continue;
    }
    const float wi = w[i];
    const bf16* g = dout + (long long)(i / K) * D;
    const bf16* yr = ys + (long long)i * D;
    bf16* d = reinterpret_cast<bf16*>(dy.ptr[owner]) + (long long)row * D;
    float dot = 0.f;
    for (int c = lane * 8; c < D; c += 256) {
      const uint4 gv = *reinterpret_cast<const uint4*>(g + c);
      const uint4 yv = *reinterpret_cast<const uint4*>(yr + c);
      const uint32_t* gq = reinterpret_cast<const uint32_t*>(&gv);
      const uint32_t* yq = reinterpret_cast<const uint32_t*>(&yv);
      float o[8];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float g0 = bf16_lo(gq[j]), g1 = bf16_hi(gq[j]);
        dot += g0 * bf16_lo(yq[j]) + g1 * bf16_hi(yq[j]);
        o[2 * j] = g0 * wi;
        o[2 * j + 1] = g1 * wi;
      }
      *reinterpret_cast<uint4*>(d + c) = pack8(o);
    }
    dot = warp_sum(dot);
    if (lane == 0) dwts[i] = dot;
  }
}

__device__ __forceinline__ int group_of(const int* off, int G, int r) {
  int g = 0;
  while (g + 1 < G && off[g + 1] <= r) ++g;
  return g;
}

__global__ void ep_owner_bwd_kernel(bf16* __restrict__ dy, const bf16* __restrict__ y, const int4* __restrict__ meta,
                                    const int* __restrict__ offsets, const int* __restrict__ kept, int El, EpPeers dw,
                                    int rows, int D, StatusBlock* st) {
  __shared__ int s_off[kEpMaxRanks * 32 + 1];
  __shared__ int s_kept[kEpMaxRanks * 32];
  for (int g = threadIdx.x; g <= El; g += blockDim.x) s_off[g] = offsets[g];
  for (int g = threadIdx.x; g < El; g += blockDim.x) s_kept[g] = kept[g];
  __syncthreads();
  const int total = min(rows, s_off[El]);
  const int lane = threadIdx.x & 31;
  for (int r = blockIdx.x * kWarps + (threadIdx.x >> 5); r < total; r += gridDim.x * kWarps) {
    const int g = group_of(s_off, El, r);
    bf16* d = dy + (long long)r * D;
    if (r - s_off[g] >= s_kept[g]) {
      for (int c = lane * 8; c < D; c += 256) *reinterpret_cast<uint4*>(d + c) = make_uint4(0, 0, 0, 0);
      continue;
    }
    const int4 m = meta[r];
    const float wr = __int_as_float(m.x);
    const bf16* yr = y + (long long)r * D;
    float dot = 0.f;
    for (int c = lane * 8; c < D; c += 256) {
      uint4 dv = *reinterpret_cast<const uint4*>(d + c);
      uint4 yv = *reinterpret_cast<const uint4*>(yr + c);
      const uint32_t* dq = reinterpret_cast<const uint32_t*>(&dv);
      const uint32_t* yq = reinterpret_cast<const uint32_t*>(&yv);
      float o[8];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float d0 = bf16_lo(dq[j]), d1 = bf16_hi(dq[j]);
        dot += d0 * bf16_lo(yq[j]) + d1 * bf16_hi(yq[j]);
        o[2 * j] = d0 * wr;
        o[2 * j + 1] = d1 * wr;
      }
      *reinterpret_cast<uint4*>(d + c) = pack8(o);
    }
    dot = warp_sum(dot);
    if (lane == 0) {
      const int src = m.y, pair = m.z;
      if (src >= 0 && src < kEpMaxRanks && pair >= 0 && pair < dw.rows[src])
        reinterpret_cast<float*>(dw.ptr[src])[pair] = dot;
      else
        report_error(st, STATUS_BAD_INDEX, pair);
    }
  }
}

__global__ void ep_pad_rows_kernel(bf16* __restrict__ x, int4* __restrict__ meta, const int* __restrict__ offsets,
                                   const int* __restrict__ kept, int El, int rows, int D) {
  // one block per local expert group: zero rows [off + kept, next off)
  const int g = blockIdx.x;
  if (g >= El) return;
  const int r0 = offsets[g] + kept[g];
  const int r1 = min(offsets[g + 1], rows);
  const int lane = threadIdx.x & 31;
  for (int r = r0 + (threadIdx.x >> 5); r < r1; r += kWarps) {
    bf16* d = x + (long long)r * D;
    for (int c = lane * 8; c < D; c += 256) *reinterpret_cast<uint4*>(d + c) = make_uint4(0, 0, 0, 0);
    if (meta != nullptr && lane == 0) meta[r] = make_int4(0, -1, -1, 0);
  }
}

__global__ void ep_barrier_kernel(EpPeers sig, int me, int n, unsigned epoch, StatusBlock* st) {
  const int t = threadIdx.x;
  if (t >= n) return;
  // release: everything this GPU wrote before this kernel (previous kernels on
  // the stream, including stores to peers) is visible before the flag.
  __threadfence_system();
  unsigned* peer_flag = reinterpret_cast<unsigned*>(sig.ptr[t]) + me;
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(peer_flag), "r"(epoch) : "memory");
  const unsigned* mine = reinterpret_cast<const unsigned*>(sig.ptr[me]) + t;
  const uint64_t t0 = globaltimer_ns();
  uint32_t spins = 0;
  while (true) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(mine) : "memory");
    if ((int)(v - epoch) >= 0) break;
    if ((++spins & 63u) == 0u && globaltimer_ns() - t0 > kWaitBudgetNs) {
      report_error(st, STATUS_TIMEOUT_PEER_FLAG, t);
      break;
    }
  }
  __threadfence_system();
}

// Signal every rank with the next epoch of the device counter and wait (bounded) until every
// rank has signalled it.  Every rank runs the same sequence of these barriers, so the
// counters advance in step; the epoch is read on the device, which lets a CUDA graph
// replay the barrier.  Called by one block: threads [0, n) each serve one peer.
__device__ __forceinline__ void dev_barrier(const EpPeers& sig, int me, int n, unsigned* epoch_ctr,
                                            StatusBlock* st) {
  __shared__ unsigned s_epoch;
  __syncthreads();
  if (threadIdx.x == 0) {
    s_epoch = *reinterpret_cast<volatile unsigned*>(epoch_ctr) + 1u;
    *reinterpret_cast<volatile unsigned*>(epoch_ctr) = s_epoch;
  }
  __syncthreads();
  const unsigned epoch = s_epoch;
  const int t = threadIdx.x;
  if (t < n) {
    __threadfence_system();
    unsigned* peer_flag = reinterpret_cast<unsigned*>(sig.ptr[t]) + me;
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(peer_flag), "r"(epoch) : "memory");
    const unsigned* mine = reinterpret_cast<const unsigned*>(sig.ptr[me]) + t;
    const uint64_t t0 = globaltimer_ns();
    uint32_t spins = 0;
    while (true) {
      unsigned v;
      asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(mine) : "memory");
      if ((int)(v - epoch) >= 0) break;
      if ((++spins & 63u) == 0u && globaltimer_ns() - t0 > kWaitBudgetNs) {
        report_error(st, STATUS_TIMEOUT_PEER_FLAG, t);
        break;
      }
    }
    __threadfence_system();
  }
  __syncthreads();
}

__global__ void ep_barrier_dev_kernel(EpPeers sig, int me, int n, unsigned* epoch_ctr, StatusBlock* st) {
  dev_barrier(sig, me, n, epoch_ctr, st);
}

// One-way readiness signal: advance this rank's signal counter and store it, with release order
// behind everything this GPU wrote before (the preceding kernels' peer stores included), into
// slot `me` of every rank's flag array.  Nothing is waited for here; consumers wait per source.
__global__ void ep_signal_kernel(EpPeers flags, int me, int n, unsigned* sig_ctr) {
  __shared__ unsigned s_epoch;
  if (threadIdx.x == 0) {
    s_epoch = *reinterpret_cast<volatile unsigned*>(sig_ctr) + 1u;
    *reinterpret_cast<volatile unsigned*>(sig_ctr) = s_epoch;
  }
  __syncthreads();
  const int t = threadIdx.x;
  if (t < n) {
    __threadfence_system();
    unsigned* f = reinterpret_cast<unsigned*>(flags.ptr[t]) + me;
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(f), "r"(s_epoch) : "memory");
  }
}

// Routing-count exchange and receive layout, computed on the device by every rank alike.
// Each rank stores its per-expert pair counts into row `me` of every rank's count board
// [N][E], passes a device barrier, then derives from the board (C[s][e] = pairs of source s
// for expert e) the layout that the host used to compute from all-gathered counts:
//   kept[s,e] = clamp(min(C[s,e], cap - sum_{s'<s} C[s',e]), 0)    (cap: the capacity, or none)
//   seg[e]    = sum_s kept[s,e], padded to 128 rows; segments of one owner back to back
//   dst_base[e] = base of e's segment + sum_{s<me} kept[s,e];  keep_lim[e] = kept[me,e]
//   offs_local / kept_local: this rank's El segments
// Each owner's slab holds El * seg_cap rows.  When an owner's padded segments do not fit, each
// of its experts is limited to seg_cap rows (cap = min(capacity, seg_cap)), which always fits;
// *dropped counts this rank's pairs lost to that bound (not those the capacity alone drops).
// The slabs are allocated once and no count reaches the host.  One block of >= E threads.
__global__ void ep_exchange_layout_kernel(EpPeers board, EpPeers sig, int me, int n, unsigned* epoch_ctr,
                                          const int* __restrict__ counts, int E, int El, int capacity, int seg_cap,
                                          int* __restrict__ dst_base, int* __restrict__ keep_lim,
                                          int* __restrict__ offs_local, int* __restrict__ kept_local,
                                          int* __restrict__ dropped, int* __restrict__ src_pref, StatusBlock* st) {
  extern __shared__ int sh[];
  int* C = sh;                 // [n][E]
  int* seg_pad = sh + n * E;   // [E]
  const int e = threadIdx.x;
  if (e < E) {
    const int c = counts[e];
    for (int t = 0; t < n; ++t) reinterpret_cast<volatile int*>(board.ptr[t])[me * E + e] = c;
  }
  dev_barrier(sig, me, n, epoch_ctr, st);
  const volatile int* mine = reinterpret_cast<const volatile int*>(board.ptr[me]);
  for (int i = threadIdx.x; i < n * E; i += blockDim.x) C[i] = mine[i];
  __syncthreads();
  // pass 1: segments under the capacity alone
  const int cap0 = capacity > 0 ? capacity : 0x3fffffff;
  if (e < E) {
    int before = 0, seg = 0;
    for (int s = 0; s < n; ++s) {
      const int c = C[s * E + e];
      seg += max(0, min(c, cap0 - before));
      before += c;
    }
    seg_pad[e] = (seg + 127) / 128 * 128;
  }
  __syncthreads();
  bool bounded = false;
  if (e < E) {
    const int owner = e / El;
    long long total = 0;
    for (int j = owner * El; j < owner * El + El; ++j) total += seg_pad[j];
    bounded = total > (long long)El * seg_cap;
  }
  __syncthreads();
  // pass 2: the final per-expert limit
  int kept_me = 0, before_me = 0, seg = 0, lost_me = 0;
  if (e < E) {
    const int cap = bounded ? min(cap0, seg_cap) : cap0;
    const bool local = e / El == me;
    int before = 0;
    for (int s = 0; s < n; ++s) {
      const int c = C[s * E + e];
      const int k = max(0, min(c, cap - before));
      // rows of source s in this rank's segment of expert e start at seg (sources in rank order)
      if (local && src_pref != nullptr) src_pref[(e - me * El) * (n + 1) + s] = seg;
      if (s < me) before_me += k;
      if (s == me) {
        kept_me = k;
        lost_me = max(0, min(c, cap0 - before)) - k;
      }
      seg += k;
      before += c;
    }
    if (local && src_pref != nullptr) src_pref[(e - me * El) * (n + 1) + n] = seg;
    seg_pad[e] = (seg + 127) / 128 * 128;
  }
  __syncthreads();
  if (e < E) {
    const int owner = e / El;
    int base = 0;
    for (int j = owner * El; j < e; ++j) base += seg_pad[j];
    dst_base[e] = base + before_me;
    keep_lim[e] = kept_me;
    if (owner == me) {
      offs_local[e - me * El] = base;
      kept_local[e - me * El] = seg;
      if (e == me * El + El - 1) offs_local[El] = base + seg_pad[e];
    }
    if (lost_me > 0 && dropped != nullptr) atomicAdd(dropped, lost_me);
  }
}

int grid_for(long long work_warps) {
  long long b = (work_warps + kWarps - 1) / kWarps;
  return (int)std::max(1ll, std::min(b, 148ll * 16));
}

}  // namespace

void ep_dispatch(const void* x, const int* idx, const int* pos, const int* loc_off, const int* dst_base,
                 const int* keep_lim, const float* wts, const EpPeers& xr, const EpPeers& meta, int* slot, int T,
                 int K, int E, int El, int D, int me, cudaStream_t s) {
  const int TK = T * K;
  if (TK == 0) return;
  ep_dispatch_kernel<<<grid_for(TK), kWarps * 32, 0, s>>>((const bf16*)x, idx, pos, loc_off, dst_base, keep_lim,
                                                          wts, xr, meta, slot, TK, K, E, El, D, me,
                                                          (StatusBlock*)status_ptr());
}

void ep_push(const void* src, const int* slot, const int* idx, const EpPeers& dst, int T, int K, int El, int D,
             cudaStream_t s) {
  const int TK = T * K;
  if (TK == 0) return;
  ep_push_kernel<<<grid_for(TK), kWarps * 32, 0, s>>>((const bf16*)src, slot, idx, dst, TK, K, El, D,
                                                      (StatusBlock*)status_ptr());
}

void ep_combine(const int* slot, const int* idx, const float* w, const EpPeers& y, const void* add, void* out, int T,
                int K, int El, int D, cudaStream_t s, const void* local) {
  if (T == 0) return;
  const int grid = (T + kWarps - 1) / kWarps;
  if (K <= 4)
    ep_combine_kernel<4><<<grid, kWarps * 32, 0, s>>>(slot, idx, w, y, (const bf16*)add, (bf16*)out, T, K, El, D,
                                                       (const bf16*)local);
  else if (K <= 8)
    ep_combine_kernel<8><<<grid, kWarps * 32, 0, s>>>(slot, idx, w, y, (const bf16*)add, (bf16*)out, T, K, El, D,
                                                       (const bf16*)local);
  else
    ep_combine_kernel<16><<<grid, kWarps * 32, 0, s>>>(slot, idx, w, y, (const bf16*)add, (bf16*)out, T, K, El, D,
                                                       (const bf16*)local);
}

void ep_return_rows(const void* y, const void* meta, const int* offsets, int El, const EpPeers& ys, int rows, int D,
                    cudaStream_t s) {
  if (rows == 0) return;
  ep_return_rows_kernel<<<grid_for(rows), kWarps * 32, 0, s>>>((const bf16*)y, (const int4*)meta, offsets, El, ys,
                                                                rows, D, (StatusBlock*)status_ptr());
}

void ep_source_bwd(const void* dout, const void* ys, const int* slot, const int* idx, const float* w, float* dwts,
                   const EpPeers& dy, int T, int K, int El, int D, cudaStream_t s) {
  const int TK = T * K;
  if (TK == 0) return;
  ep_source_bwd_kernel<<<grid_for(TK), kWarps * 32, 0, s>>>((const bf16*)dout, (const bf16*)ys, slot, idx, w, dwts,
                                                            dy, TK, K, El, D, (StatusBlock*)status_ptr());
}

void ep_owner_bwd(void* dy, const void* y, const void* meta, const int* offsets, const int* kept, int El,
                  const EpPeers& dw, int rows, int D, cudaStream_t s) {
  if (rows == 0) return;
  ep_owner_bwd_kernel<<<grid_for(rows), kWarps * 32, 0, s>>>((bf16*)dy, (const bf16*)y, (const int4*)meta, offsets,
                                                              kept, El, dw, rows, D, (StatusBlock*)status_ptr());
}

void ep_pad_rows(void* x, void* meta, const int* offsets, const int* kept, int El, int rows, int D, cudaStream_t s) {
  if (El == 0) return;
  ep_pad_rows_kernel<<<El, kWarps * 32, 0, s>>>((bf16*)x, (int4*)meta, offsets, kept, El, rows, D);
}

void ep_barrier_dev(const EpPeers& sig, int me, int n, unsigned* epoch_ctr, cudaStream_t s) {
  ep_barrier_dev_kernel<<<1, 32, 0, s>>>(sig, me, n, epoch_ctr, (StatusBlock*)status_ptr());
}

void ep_exchange_layout(const EpPeers& board, const EpPeers& sig, int me, int n, unsigned* epoch_ctr,
                        const int* counts, int E, int El, int capacity, int seg_cap, int* dst_base, int* keep_lim,
                        int* offs_local, int* kept_local, int* dropped, cudaStream_t s, int* src_pref) {
  const int threads = std::max(32, (E + 31) / 32 * 32);
  const size_t smem = (size_t)(n * E + E) * sizeof(int);
  ep_exchange_layout_kernel<<<1, threads, smem, s>>>(board, sig, me, n, epoch_ctr, counts, E, El, capacity, seg_cap,
                                                     dst_base, keep_lim, offs_local, kept_local, dropped, src_pref,
                                                     (StatusBlock*)status_ptr());
}

void ep_signal(const EpPeers& flags, int me, int n, unsigned* sig_ctr, cudaStream_t s) {
  ep_signal_kernel<<<1, 32, 0, s>>>(flags, me, n, sig_ctr);
}

void ep_barrier(const EpPeers& sig, int me, int n, unsigned epoch, cudaStream_t s) {
  ep_barrier_kernel<<<1, 32, 0, s>>>(sig, me, n, epoch, (StatusBlock*)status_ptr());
}

}  // namespace omni
