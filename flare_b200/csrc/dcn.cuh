// Elementwise / reduction kernels of the DCN-v2 model (dcn.cu).  The GEMMs of
// the model run in gemm_dist.cu / gemm_tcgen05.cu.
#pragma once

#include "common.cuh"

namespace flare {

// x0[b, :E] = pooled[b, :E]; x0[b, E:E+nd] = bf16(dense[b]); x0[b, E+nd:ld0] = 0
void dcn_concat_x0(const __nv_bfloat16* pooled, int64_t ldp, const float* dense, int nd, int64_t B, int E,
                   __nv_bfloat16* x0, int64_t ld0, cudaStream_t s);

struct DcnHeadParams {
  const __nv_bfloat16* h;  // [B, ldh] final-layer input
  int64_t ldh;
  int H;                   // used width (multiple of 8)
  int relu_from;           // columns >= relu_from came out of a ReLU (mask dh there)
  const __nv_bfloat16* w;  // [H]
  const __nv_bfloat16* bias;  // [1]
  const float* labels;     // [B]
  int64_t B;
  int valid_count;         // samples >= valid_count get zero weight (-1: all valid)
  float grad_scale;        // d loss_mean / d loss_sum
  float* logits;           // [B]
  float* dl;               // [B] d loss / d logit (scaled)
  __nv_bfloat16* dh;       // [B, lddh]
  int64_t lddh;
  float* loss_sum;         // += sum of per-sample BCE
  float* db;               // += sum of dl
};
void dcn_head(const DcnHeadParams& p, cudaStream_t s);

// out[c] += sum_b scale[b] * x[b, c] for c < cols
void dcn_scaled_colsum(const __nv_bfloat16* x, int64_t ldx, const float* scale, int64_t rows, int cols, float* out,
                       cudaStream_t s);

// Cross-layer backward elementwise part for one layer:
//   dz = g * x0 (bf16 out), acc (=|+=) g * z (fp32), db += colsum(dz)
void dcn_cross_bwd_elem(const __nv_bfloat16* g, int64_t ldg, const __nv_bfloat16* x0, const __nv_bfloat16* z, int64_t ld,
                        int64_t rows, int cols, __nv_bfloat16* dz, float* acc, int64_t ld_acc, int accumulate,
                        float* db, cudaStream_t s);

// grad[b, c] = bf16(acc[b, c]) for c < cols (the pooled-embedding gradient)
void dcn_finalize_grad(const float* acc, int64_t ld_acc, int64_t rows, int cols, __nv_bfloat16* grad, int64_t ldg,
                       cudaStream_t s);

}  // namespace flare
