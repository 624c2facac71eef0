// Fused kernels of the multitask layer library (expert mixing, MLP activation backward).
#pragma once

#include "common.cuh"

namespace flare {

constexpr int kMixMaxExperts = 64;

// out[b, :] = sum_e softmax(logits[b, :])_e * y_e[b, :]  (fp32 softmax and accumulation, bf16 out).
// Backward: dy_e[b, :] = p_e * dout[b, :], dlogits[b, e] = p_e * (s_e - sum_e' p_e' s_e'),
// s_e = <dout[b, :], y_e[b, :]>.  Every expert output is a bf16 [B, D] matrix with row stride ld_y.
struct GateMixParams {
  const __nv_bfloat16* ys[kMixMaxExperts];
  __nv_bfloat16* dys[kMixMaxExperts];  // backward outputs (row stride ld_dy)
  const __nv_bfloat16* logits;         // [B, E] bf16, row stride ld_logits
  __nv_bfloat16* dlogits;              // backward output [B, E], row stride ld_logits
  float* probs;                        // [B, E] fp32: written by the forward, read by the backward
  __nv_bfloat16* out;                  // forward output [B, D] (row stride ld_out)
  const __nv_bfloat16* dout;           // backward input [B, D] (row stride ld_out)
  int64_t ld_y, ld_dy, ld_logits, ld_out;
  int B, E, D;
};

void gate_mix_forward(const GateMixParams& p, cudaStream_t s);
void gate_mix_backward(const GateMixParams& p, cudaStream_t s);

// g_out = g * (h > 0) (bf16) and colsum[c] += sum_r g_out[r, c] (fp32): the ReLU backward of an MLP
// layer fused with its bias gradient.  cols a multiple of 8, every row 16-byte aligned.
void relu_bwd_colsum(const __nv_bfloat16* g, int64_t ldg, const __nv_bfloat16* h, int64_t ldh, int64_t rows,
                     int cols, __nv_bfloat16* gout, int64_t ldo, float* colsum, cudaStream_t s);

}  // namespace flare
