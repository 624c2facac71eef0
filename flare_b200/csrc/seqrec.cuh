// Memory-bound kernels of the sequential-recommendation transformer (seqrec.cu); width 256.
#pragma once

#include "common.cuh"

namespace flare {

struct SampledSoftmaxParams {
  const __nv_bfloat16* y;      // [T, ldy] final hidden states
  int64_t ldy;
  const __nv_bfloat16* emb;    // pooled item embeddings (positive targets are rows of it)
  int64_t ldemb;
  const int* target_row;       // [T] row of emb holding token t's next item, -1 = no target
  const float* logits;         // [T, ldlog] fp32 scores of the N shared negatives
  int64_t ldlog;
  int64_t T;
  int N;
  const int* num_valid;        // device scalar: tokens with a target (loss mean denominator)
  __nv_bfloat16* dneg;         // [T, lddneg] d loss / d negative logits
  int64_t lddneg;
  __nv_bfloat16* dy;           // [T, lddy] positive part of d loss / d y
  int64_t lddy;
  float* dpos;                 // [T] d loss / d positive logit
  float* loss_sum;             // += sum of per-token losses
};

void seq_embed_combine(const __nv_bfloat16* pooled, int64_t ldp, int64_t T, __nv_bfloat16* x, int64_t ldx,
                       cudaStream_t s);
void seq_layernorm_fwd(const __nv_bfloat16* x, int64_t ldx, int64_t T, const __nv_bfloat16* gamma,
                       const __nv_bfloat16* beta,
                       float eps, __nv_bfloat16* y, int64_t ldy, float* mean, float* rstd, cudaStream_t s);
void seq_layernorm_bwd(const __nv_bfloat16* dy, int64_t lddy, const __nv_bfloat16* x, int64_t ldx, int64_t T,
                       const __nv_bfloat16* gamma, const float* mean, const float* rstd, const __nv_bfloat16* resid,
                       int64_t ldr, __nv_bfloat16* dx, int64_t lddx, float* dgamma, float* dbeta, cudaStream_t s);
void seq_sampled_softmax(const SampledSoftmaxParams& p, cudaStream_t s);
void seq_embed_grad_split(const __nv_bfloat16* dx, int64_t lddx, const __nv_bfloat16* y, int64_t ldy,
                          const float* dpos, const int* target_row, int64_t T, __nv_bfloat16* grad, int64_t ldg,
                          cudaStream_t s);

}  // namespace flare
