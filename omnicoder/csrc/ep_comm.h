// Expert-parallel token exchange over NVLink peer memory (see ep_comm.cu).
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

namespace omni {

constexpr int kEpMaxRanks = 8;

// Per-rank device addresses (valid in this process: peer-mapped symmetric
// memory) and the row capacity of each rank's region.
struct EpPeers {
  unsigned long long ptr[kEpMaxRanks];
  int rows[kEpMaxRanks];
};

// Push every kept (token, k) pair's row of x [T, D] into row
// dst_base[e] + (pos - loc_off[e]) of its owner's receive region (owner = e / El);
// meta (optional) receives {w bits, source rank, pair index, 0} per row.
// slot[pair] = destination row, -1 when dropped (capacity) or invalid.
void ep_dispatch(const void* x, const int* idx, const int* pos, const int* loc_off, const int* dst_base,
                 const int* keep_lim, const float* wts, const EpPeers& xr, const EpPeers& meta, int* slot, int T,
                 int K, int E, int El, int D, int me, cudaStream_t s);
// Push rows of src [T, D] along a slot table computed by ep_dispatch.
void ep_push(const void* src, const int* slot, const int* idx, const EpPeers& dst, int T, int K, int El, int D,
             cudaStream_t s);
// out[t] = add[t] + sum_k w[t,k] * Y_owner[slot[t,k]] (w == nullptr: weight 1); peer loads.
// local != nullptr: the owners pushed their rows into this rank's slots local[t * K + k] (read
// locally, y unused).
void ep_combine(const int* slot, const int* idx, const float* w, const EpPeers& y, const void* add, void* out, int T,
                int K, int El, int D, cudaStream_t s, const void* local = nullptr);
// Owner output rows y [rows, D] back to their origins' (token, k) slots: row r -> ys.ptr[s] + i * D,
// (-, s, i, -) = meta[r]; rows past offsets[El] and padding rows (s < 0) are skipped.
void ep_return_rows(const void* y, const void* meta, const int* offsets, int El, const EpPeers& ys, int rows, int D,
                    cudaStream_t s);
// Combine backward on the source when the owners pushed outputs to its slots ys [T*K, D]:
//   dwts[t,k] = <dout[t], ys[t*K+k]>;  owner's dy row slot[t,k] <- dout[t] * w[t,k] (peer store).
void ep_source_bwd(const void* dout, const void* ys, const int* slot, const int* idx, const float* w, float* dwts,
                   const EpPeers& dy, int T, int K, int El, int D, cudaStream_t s);
// Owner side of the combine backward, over the local receive rows:
//   dot = <dy[r], y[r]> -> written to dw_src_rank[pair] (peer store);  dy[r] *= w[r];
// padding rows (beyond kept[g] in each 128-padded group) are zeroed.
void ep_owner_bwd(void* dy, const void* y, const void* meta, const int* offsets, const int* kept, int El,
                  const EpPeers& dw, int rows, int D, cudaStream_t s);
// Zero the padding rows of a receive region (and mark their meta invalid).
void ep_pad_rows(void* x, void* meta, const int* offsets, const int* kept, int El, int rows, int D, cudaStream_t s);
// Signal every rank and wait until every rank has signalled `epoch` (bounded wait).
void ep_barrier(const EpPeers& sig, int me, int n, unsigned epoch, cudaStream_t s);
// Same, with the epoch taken from (and advanced in) the device counter *epoch_ctr, so that a
// CUDA graph can replay it.
void ep_barrier_dev(const EpPeers& sig, int me, int n, unsigned* epoch_ctr, cudaStream_t s);
// Exchange per-expert routing counts [E] through the peer-mapped count boards ([N][E] int32
// per rank) and compute the receive layout on the device (dst_base / keep_lim [E], this rank's
// offs_local [El + 1] / kept_local [El]; pairs beyond min(capacity, seg_cap) per expert are
// dropped and counted into *dropped).  E <= 1024.
void ep_exchange_layout(const EpPeers& board, const EpPeers& sig, int me, int n, unsigned* epoch_ctr,
                        const int* counts, int E, int El, int capacity, int seg_cap, int* dst_base, int* keep_lim,
                        int* offs_local, int* kept_local, int* dropped, cudaStream_t s, int* src_pref = nullptr);
// src_pref (optional, [El][n + 1]): row offset of each source's rows inside this rank's segment of
// each local expert (sources in rank order; entry n = the segment's kept rows).
// One-way readiness signal: *sig_ctr += 1, then flags.ptr[r][me] = *sig_ctr on every rank r
// (release order behind this GPU's earlier writes).  Consumers wait per source (bounded).
void ep_signal(const EpPeers& flags, int me, int n, unsigned* sig_ctr, cudaStream_t s);

// ZeRO-1 step over peer memory (zero_p2p.cu): reduce-scatter of rank-local bf16 gradient
// buckets g.ptr[r] into this rank's fp32 shard out[0, n) = scale * sum_r g_r[lo + i] (+ its
// squared norm into *norm_sq), and the AdamW update of that shard whose bf16 result is stored
// into every rank's parameter bucket dst.ptr[r] at [lo, lo + n).  lo must be a multiple of 8.
void zero_rs(const EpPeers& g, int world, long long lo, long long n, float scale, float* out, float* norm_sq,
             cudaStream_t s);
void zero_adamw_push(float* p, float* m, float* v, const float* g, const EpPeers& dst, int world, long long lo,
                     long long n, float lr, float b1, float b2, float eps, float wd, int step, const float* norm_sq,
                     float max_norm, cudaStream_t s);

}  // namespace omni
