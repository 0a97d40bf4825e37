// Host interface of the tcgen05 GEMM (see gemm_sm100.cu).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

namespace omni {

enum GemmMode : int {
  GEMM_DENSE = 0,
  GEMM_GROUPED_M = 1,
  GEMM_GROUPED_K = 2,
  GEMM_AG = 3,  // dense, rows [r*src_rows, (r+1)*src_rows) of A read from source r's buffer (peer memory)
};

enum GemmEpi : int {
  EPI_STORE_BF16 = 0,  // C(bf16) = alpha * acc
  EPI_STORE_F32 = 1,   // C(f32)  = alpha * acc
  EPI_ACCUM_F32 = 2,   // C(f32) += alpha * acc
  EPI_ADD_BF16 = 3,    // C(bf16) = alpha * acc + R(bf16)   (R may alias C)
  EPI_SWIGLU = 4,      // acc = [gate|up] interleaved by 32; C = silu(gate)*up (bf16, N/2 cols); H = acc (bf16)
  EPI_SWIGLU_BWD = 5,  // acc = dAct; R = saved H; C = dH (bf16, 2N cols, interleaved by 32)
  EPI_PEER_BF16 = 6,   // bf16 partial tile stored into its row owner's staging buffer (peer memory):
                       // row -> owner r = row / src_rows, slot me: peer_c[r] + (me*src_rows + row%src_rows)*ldc
  EPI_EP_PUSH = 7,     // grouped-M: row r goes to its origin (expert-parallel combine from the epilogue):
                       // row_meta[r] = (weight, source rank s, pair index i, -) -> peer_c[s] + i*ldc
                       // (rows with s < 0 are padding and are not stored; i < src_rows is checked)
};

constexpr int GEMM_MAX_PEERS = 8;

constexpr int GEMM_MAX_GROUPS = 256;

struct GemmDesc {
  int mode = GEMM_DENSE;
  int epilogue = EPI_STORE_BF16;
  int block_n = 256;  // 128 or 256
  int pair = -1;      // CTA-pair (cta_group::2) 256-row tiles: -1 automatic, 0 off, 1 on (block_n 256 only)
  bool a_mn_major = false;
  bool b_mn_major = false;
  int M = 0, N = 0, K = 0;
  // A: K-major -> stored [rows_a, K_extent_a]; MN-major -> stored [K_extent_a, M]
  const void* A = nullptr;
  long long lda = 0;
  long long rows_a = 0;
  long long K_extent_a = 0;
  // B: K-major -> stored [N, K_extent_b] (or [G, N, K]); MN-major -> stored [K_extent_b, N] (or [G, K, N])
  const void* B = nullptr;
  long long ldb = 0;
  long long b_group_stride = 0;
  long long K_extent_b = 0;
  int num_groups = 1;
  const int* group_offsets = nullptr;  // device [G+1], multiples of 128
  int max_rows_hint = 0;               // grouped-M: upper bound on total rows (0 = unknown)
  void* C = nullptr;
  long long ldc = 0;
  long long rows_c = 0;  // rows of C (0: M); grouped-M outputs are as tall as A
  long long c_group_stride = 0;
  const void* R = nullptr;
  long long ldr = 0;
  void* H = nullptr;
  long long ldh = 0;
  float alpha = 1.0f;
  void* status = nullptr;  // omni::StatusBlock*
  // tensor-parallel fused collectives (GEMM_AG mode / EPI_PEER_BF16 epilogue)
  int nsrc = 0;                              // ranks in the group
  int me = 0;                                // this rank
  int src_rows = 0;                          // rows per rank (multiple of 128)
  const void* peer_a[GEMM_MAX_PEERS] = {};   // GEMM_AG: each rank's A row block ([src_rows, K], stride lda)
  void* peer_c[GEMM_MAX_PEERS] = {};         // EPI_PEER_BF16: each rank's staging buffer
  const void* row_meta = nullptr;            // EPI_EP_PUSH: int4 per row of A
  // grouped-M, expert-parallel receive rows: a tile is loaded once every source rank with rows in it
  // has signalled ready[s] >= *ready_epoch (src_pref [G][nsrc+1]: row prefix of each source within
  // group g; this rank's own rows are not waited for)
  const unsigned* ready = nullptr;
  const unsigned* ready_epoch = nullptr;
  const int* src_pref = nullptr;
};

// Launch on `stream`.  Throws std::runtime_error on an invalid description.
void gemm_sm100_launch(const GemmDesc& d, cudaStream_t stream);

// Process-wide switch of the automatic CTA-pair choice (default on unless OMNI_GEMM_PAIR=0).
void set_gemm_pair(bool on);
bool gemm_pair_enabled();

// out[r, :] = sum_s staging[s, r, :] (+ residual[r, :]) — the local half of a fused GEMM -> reduce-scatter.
void tp_reduce_slots(const void* staging, int nsrc, int rows, int D, long long ld, const void* residual,
                     long long ldr, void* out, long long ldo, cudaStream_t s);

// rank-2 or rank-3 bf16 tensor map with 128-byte swizzle (dims[0] contiguous,
// byte strides for dims 1..).  Throws on misaligned bases or strides.
CUtensorMap make_tmap_bf16_sw128(const void* base, int rank, const uint64_t* dims, const uint64_t* strides_bytes,
                                 const uint32_t* box);
// Same for byte-sized elements (fp8 operands).
CUtensorMap make_tmap_u8_sw128(const void* base, int rank, const uint64_t* dims, const uint64_t* strides_bytes,
                               const uint32_t* box);
int num_sms();

// ---- block-scaled fp8 GEMM (gemm_fp8.cu) ----------------------------------------
// C[M, N] (bf16) = sum over 128-wide K blocks kb of (Xq[M, kb] . Wq[N, kb]^T) * sx[kb][m] * sw[g][n / 128][kb]
// Xq, Wq: e4m3, K-major ([rows, K] row-major, K % 128 == 0).  sx: fp32 [K/128][ldsx] (ldsx >= M rounded
// up to 128; one scale per row and 128-column block).  sw: fp32 [G][ceil(N/128)][K/128] (one scale per
// 128 x 128 weight block).  Grouped-M: group g owns rows [offsets[g], offsets[g+1]) of X (multiples of
// 128, device array) and weight Wq[g] ([G, N, K]).
struct Fp8GemmDesc {
  int M = 0, N = 0, K = 0, G = 1;
  const int* offsets = nullptr;  // grouped-M when non-null
  int max_rows_hint = 0;
  const void* X = nullptr;
  long long ldx = 0;
  const float* sx = nullptr;
  long long ldsx = 0;
  const void* W = nullptr;
  long long ldw = 0;
  long long w_group_stride = 0;
  const float* sw = nullptr;
  long long ldsw = 0;  // > 0 (dense, scaled_mma): per-row B scales sw[K/128][ldsw], like sx
  void* C = nullptr;
  long long ldc = 0;
  long long rows_c = 0;  // rows of C (0: M); grouped-M outputs are as tall as A
  void* status = nullptr;
  // every scale a power of two: the tensor core applies them (block-scaled MMA, 128 x 256 tiles);
  // otherwise the epilogue promotes each K block's partial product with its fp32 scales
  bool scaled_mma = false;
  // SwiGLU + requantisation epilogue (scaled_mma, N % 256 == 0, W rows 32-interleaved gate|up):
  // C <- gate|up pre-activation; act (optional) <- silu(g) * u bf16 [rows, N/2]; actq <- the
  // same in e4m3 with act_scale fp32 [N/256][ld_as] (power-of-two 1 x 128 block scales)
  void* act = nullptr;
  long long ld_act = 0;
  void* actq = nullptr;
  long long ld_actq = 0;
  float* act_scale = nullptr;
  long long ld_as = 0;
};
void fp8_gemm_launch(const Fp8GemmDesc& d, cudaStream_t stream);
// x [M, K] bf16 -> xq e4m3 [M, K], sx fp32 [K/128][ldsx] (rows >= M zero-filled up to ldsx);
// pow2: scales rounded up to powers of two; row_limit (device int, optional): rows at or past it
// are left unwritten (grouped operands whose tiles end at the last group's offset)
void fp8_quant_act(const void* x, long long ldx, int M, int K, void* xq, float* sx, long long ldsx, bool pow2,
                   cudaStream_t s, const int* row_limit = nullptr);
// x [T, C] bf16 -> xt [C, T] e4m3, st fp32 [T/128][ldst]: per column and 128-token block
// (power-of-two scales); T % 128 == 0
void fp8_quant_t(const void* x, long long ldx, int T, int Cn, void* xt, long long ldxt, float* st, long long ldst,
                 cudaStream_t s);
// w [G, N, K] bf16 -> wq e4m3, sw fp32 [G][ceil(N/128)][K/128]
void fp8_quant_weight(const void* w, int G, int N, int K, void* wq, float* sw, bool pow2, cudaStream_t s);

// ---- few-row GEMM (decode, speculative verification) --------------------------
// Y[rows, N] = X[rows, K] W[N, K]^T for at most kSkinnyMaxRows rows per group
// (swap-AB on the tensor core: weight rows on the MMA M side, tokens on N).
// Grouped: group g owns rows [offsets[g], offsets[g+1]) of X and weight W[g]
// (W is [G, N, K]); dense: G = 1, offsets = nullptr, rows = M.  Partial sums
// are added into acc [rows, N] fp32 (zeroed by the caller); skinny_finalize
// applies the epilogue.
constexpr int kSkinnyMaxRows = 256;
struct SkinnyDesc {
  int M = 0;            // rows of X (upper bound of offsets[G] when grouped)
  int N = 0, K = 0, G = 1;
  const int* offsets = nullptr;
  const void* X = nullptr;
  long long ldx = 0;
  const void* W = nullptr;
  long long ldw = 0;
  long long w_group_stride = 0;
  float* acc = nullptr;
  void* status = nullptr;
  // direct output (only when skinny_ksplit(d) == 1): bf16 out [rows, N] = alpha * X W^T, or the
  // SwiGLU activation [rows, N/2] of 32-interleaved gate|up rows; acc is then unused
  void* out = nullptr;
  long long ldo = 0;
  int epilogue = EPI_STORE_BF16;
  float alpha = 1.0f;
};
// Number of K splits the launch will use (1: the output can be written directly).
int skinny_ksplit(const SkinnyDesc& d);
void skinny_gemm_launch(const SkinnyDesc& d, cudaStream_t stream);
// out[r, :] = epilogue(acc[r, :]) for r < rows: EPI_STORE_BF16 / EPI_STORE_F32 /
// EPI_ADD_BF16 (+ R) / EPI_SWIGLU (acc gate/up interleaved by 32 -> N/2 columns).
void skinny_finalize(const float* acc, int rows, int N, int epilogue, float alpha, void* out, long long ldo,
                     const void* R, long long ldr, cudaStream_t stream);

}  // namespace omni
