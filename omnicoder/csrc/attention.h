// Host interface of the flash-attention kernels (attention_sm100.cu).
#pragma once
#include <cuda_runtime.h>

namespace omni {

struct AttnTensors {
  const void* q; long long q_row, q_head;
  const void* k; long long k_row, k_head;
  const void* kr; long long kr_row;
  const void* v; long long v_row, v_head;
  int T, S, H, Hk, DQ, DR, DV;
  int causal, window;
  float scale;
};

void attention_fwd(const AttnTensors& a, void* o, float* lse, void* status, cudaStream_t s);
void attention_bwd(const AttnTensors& a, const void* o, const float* lse, const void* dO, float* delta, void* dq,
                   long long dq_row, long long dq_head, void* dk, long long dk_row, long long dk_head, void* dkr,
                   long long dkr_row, long long dkr_head, void* dv, long long dv_row, long long dv_head, void* status,
                   cudaStream_t s);

}  // namespace omni
