// Raw-pointer launchers of the memory-bound and routing kernels.  The .cu
// files that define them include no torch headers; bindings live in
// ops_bindings.cpp.
#pragma once
#include <cuda_runtime.h>
#include <cstdint>

namespace pybind11 {
class module_;
}

namespace omni {

void* status_ptr();
void register_kernels(pybind11::module_& m);
void register_ep(pybind11::module_& m);

// ---- normalisation -------------------------------------------------------
// y = rmsnorm(x (+ r)) * w ; h = x + r is written when r != nullptr.
void rmsnorm_fwd(const void* x, const void* r, void* h, const void* w, void* y, float* rstd, int rows, int dim,
                 float eps, cudaStream_t s);
// dx = d(rmsnorm)/dx * dy (+ dres when dres != nullptr); dw (fp32) += sum over rows.
void rmsnorm_bwd(const void* x, const void* w, const float* rstd, const void* dy, const void* dres, void* dx,
                 float* dw, int rows, int dim, cudaStream_t s);
// LayerNorm with affine weight and bias (compat family).
void layernorm_fwd(const void* x, const void* w, const void* b, void* y, float* mean, float* rstd, int rows,
                   int dim, float eps, cudaStream_t s);
void layernorm_bwd(const void* x, const void* w, const float* mean, const float* rstd, const void* dy, void* dx,
                   float* dw, float* db, int rows, int dim, cudaStream_t s);

// ---- speculative decoding ---------------------------------------------------
// Verify k draft tokens per sequence: logits [B, K+1, V] fp32 of the target, pdraft [B, K, V]
// fp32 draft distributions (unused when temperature <= 0), draft [B, K] and next [B] token ids
// (int64 when draft_i64, else int32), u [B, K+1] uniforms, base_len / new_len [B] cache lengths
// (int64 when len_i64).  Writes n_acc [B], next, new_len = base_len + n_acc + 1.
void spec_verify(const float* logits, const float* pdraft, const void* draft, bool draft_i64, const float* u,
                 const void* base_len, bool len_i64, int B, int K, int V, float temperature, int* n_acc, void* next,
                 void* new_len, cudaStream_t s);

// ---- rotary embedding ------------------------------------------------------
// In-place rotation of dims [off, off+rot) of each head of x (bf16).
// x row t, head h starts at x + t*row_stride + h*head_stride.  Positions are
// pos[t] (int32) if pos != nullptr, else pos0 + (t % seq).  cs holds
// [max_pos, rot/2] cos values followed by the same number of sin values.
// interleaved: pairs (2i, 2i+1); else halves (i, i+rot/2).  sign = -1 undoes.
void rope_apply(void* x, const float* cs, int max_pos, const int* pos, int pos0, int seq, int tokens, int heads,
                long long row_stride, long long head_stride, int off, int rot, bool interleaved, float sign,
                cudaStream_t s);

// ---- embedding -------------------------------------------------------------
void embedding_fwd(const int64_t* ids, const void* w, void* out, int tokens, int dim, int vocab, cudaStream_t s);
void embedding_bwd(const int64_t* ids, const void* dout, float* dw, int tokens, int dim, int vocab, cudaStream_t s);

// ---- loss ------------------------------------------------------------------
// Row-wise softmax cross entropy on bf16 logits [rows, vocab] (row stride ld).
// loss[row] (fp32) = lse - logit[label]; lse[row] saved.  When dlogits !=
// nullptr the gradient (softmax - onehot) * grad_scale (+ z-loss term) is
// written there (may alias logits).  label < 0 is ignored (loss 0, grad 0).
void cross_entropy_fwd_bwd(const void* logits, long long ld, const int64_t* labels, float* loss, float* lse,
                           void* dlogits, int rows, int vocab, float grad_scale, float z_loss, cudaStream_t s);

// ---- optimiser ---------------------------------------------------------------
// Flat AdamW over n elements: fp32 master p, m, v; bf16 grad g (scaled by
// grad_scale * clip, where clip comes from *norm_sq when max_norm > 0); writes
// the bf16 copy of p into p_bf16 (may be nullptr).
void adamw_step(float* p, float* m, float* v, const void* g, void* p_bf16, long long n, float lr, float beta1,
                float beta2, float eps, float wd, float bc1, float bc2, float grad_scale, const float* norm_sq,
                float max_norm, cudaStream_t s);
// *out += sum(g^2) * scale^2 over a bf16 vector (for global-norm clipping).
void sq_norm_accum(const void* g, long long n, float scale, float* out, cudaStream_t s);
// Many small tensors per launch (one block each): AdamW update / squared-norm accumulation.
constexpr int kMultiItems = 48;
struct AdamwItem {
  float* p;
  float* m;
  float* v;
  const void* g;  // bf16 gradient
  void* pb;       // bf16 parameter copy (or nullptr)
  long long n;
  float wd;
};
struct AdamwMulti {
  AdamwItem item[kMultiItems];
  int count;
};
void adamw_multi(const AdamwMulti& t, float lr, float b1, float b2, float eps, float bc1, float bc2, float grad_scale,
                 const float* norm_sq, float max_norm, cudaStream_t s);
void sq_norm_multi(const AdamwMulti& t, float scale, float* out, cudaStream_t s);

// ---- MoE routing -------------------------------------------------------------
// Softmax over E router logits (fp32 [T, E]), top-k, optional renormalisation.
void router_topk(const float* logits, int* idx, float* wts, float* probs, int T, int E, int K, bool renorm,
                 cudaStream_t s);
// Deterministic permutation into expert-major, 128-row padded segments.
//   counts[E], offsets[E+1] (padded), pos[T*K] (-1 = dropped), src[cap_rows]
//   (token*K + k of each permuted row, -1 for padding).  capacity <= 0: no drop.
// workspace: int32 of size (E * nblocks) * 2 where nblocks = ceil(T*K/1024).
void moe_permute_plan(const int* idx, int T, int K, int E, int capacity, int* counts, int* offsets, int* pos,
                      int* src, int cap_rows, int* workspace, cudaStream_t s, int align = 128);
// X_perm[r] = X[src[r]/K] for valid rows, zero for padding rows r < cap_rows.
void moe_gather(const void* x, const int* src, void* x_perm, int cap_rows, int K, int dim, const int* offsets,
                int E, cudaStream_t s);
// out[t] = sum_k w[t,k] * Y[pos[t,k]] (+ add[t] when add != nullptr).
void moe_combine(const void* y_perm, const int* pos, const float* w, const void* add, void* out, int T, int K,
                 int dim, cudaStream_t s);
// dY_perm[r] = w[t,k] * dout[t] (zero for padding); dw[t,k] = <dout[t], Y[r]>.
void moe_combine_bwd(const void* dout, const void* y_perm, const int* src, const float* w, void* dy_perm,
                     float* dw, int cap_rows, int K, int dim, const int* offsets, int E, cudaStream_t s);
// dx[t] = sum_k dX_perm[pos[t,k]] (+ dx_add[t]).
void moe_scatter_add(const void* dx_perm, const int* pos, const void* dx_add, void* dx, int T, int K, int dim,
                     cudaStream_t s);
// Router backward: from dw (grad of the kept top-k weights) to dlogits (bf16),
// including load-balance (alpha) and z-loss (beta) terms.
void router_bwd(const float* logits, const float* probs, const int* idx, const float* dw, const int* counts,
                void* dlogits, int T, int E, int K, bool renorm, float aux_alpha, float z_beta, float* aux_out,
                cudaStream_t s);

// ---- KV-cache append ---------------------------------------------------------
// src [B, T, G, D] bf16 -> dst rows row_offset + pos[b, t] of [B, L, G, D]
// (bf16 copy, or int8 with one fp32 scale per (b, row, g)); see kv_write.cu.
void kv_cache_write(const void* src, const long long* pos, void* dst, float* scale, bool int8, int B, int T, int G,
                    int D, long long d_b, long long d_l, long long s_b, long long s_l, int row_offset, int L,
                    cudaStream_t s);

// ---- decode attention ----------------------------------------------------------
// Split-KV attention of new tokens against a (bf16 or int8) KV cache; see
// decode_sm100.cu for the layouts.  v == nullptr: MLA latent cache (the value
// is the first DV dims of each key row).  workspace: decode_plan().ws_floats.
// Token position t lives in cache row sink_rows + t; rows [0, n_sink) are
// compressed-memory rows every query attends to.
struct DecodePlan {
  bool tc;           // tensor-core kernel (MLA latent caches of supported dims)
  bool gemv;         // few-row kernel (MHA / GQA with <= 16 query rows per kv head)
  int rg, groups;    // query rows per CTA, row groups
  int splits;        // key-range splits per sequence
  int rstride;       // rows per (sequence, kv head, split) slab of the workspace
  size_t ws_floats;  // workspace size
};
DecodePlan decode_plan(int B, int Tn, int H, int Hk, int L, int DQ, int DV, bool latent, int window, int sink_rows,
                       int kv_bytes);
void attn_decode(const void* q, const void* k, const void* v, const float* ks, const float* vs, bool int8_kv,
                 const int* q_pos, const int* kv_len, void* out, float* workspace, int B, int Tn, int H, int Hk,
                 int L, int DQ, int DV, long long k_b, long long k_l, long long v_b, long long v_l, long long s_b,
                 long long s_l, int window, float scale, const DecodePlan& plan, int sink_rows, int n_sink,
                 void* status, cudaStream_t s);

// ---- int4 weight-only linear ----------------------------------------------------
// y[M, N] = x[M, K] (bf16) . dequant(w)^T, w packed [N, ldw] bytes (two nibbles per
// byte, low first), value = (q - offset) * scale[n].  M <= 8.
void int4_gemv(const void* x, const uint8_t* w, const float* scale, void* y, int M, int N, int K, int ldw,
               float offset, cudaStream_t s);
// out[N, K] (bf16) = (q - offset) * scale[n]
void int4_dequant(const uint8_t* w, const float* scale, void* out, int N, int K, int ldw, float offset,
                  cudaStream_t s);

// ---- Gaussian splatting ------------------------------------------------------
// Splat B*N projected Gaussians (u, v, sx, sy, opacity, rgb [.., 3], depth z or
// nullptr) with a k x k footprint; acc: 5 * B * H * W fp32 scratch, 16-byte aligned; writes
// out_rgb [B, 3, H, W] and out_depth [B, 1, H, W] (when z != nullptr).
void gsplat_forward(const float* u, const float* v, const float* sx, const float* sy, const float* opa,
                    const float* rgb, const float* z, float* acc, float* out_rgb, float* out_depth, int B, int N,
                    int H, int W, int k, cudaStream_t s);

}  // namespace omni
