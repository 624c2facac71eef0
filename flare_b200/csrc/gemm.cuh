// Host interface of the tcgen05 GEMM (gemm_tcgen05.cu).
#pragma once

#include "common.cuh"

namespace flare {

struct GemmArgs {
  const void* A;  // logical [M,K]; K-major A[m*lda+k], MN-major A[k*lda+m]
  int64_t lda;
  bool a_mn;
  const void* B;  // logical [N,K]; K-major B[n*ldb+k], MN-major B[k*ldb+n]
  int64_t ldb;
  bool b_mn;
  int M, N, K;
  void* C;  // [M, ldc] of c_dtype
  int64_t ldc;
  int c_dtype;  // kF32 or kBF16
  bool accumulate;
  const __nv_bfloat16* bias;  // bf16 [N] or null
  int act;            // 0 none, 1 relu
  float alpha;
  const void* mask;  // bf16 [M, ldm]: result *= (mask > 0); or null
  int64_t ldm;
  float* colsum;  // fp32 [N]: += column sums of the result; or null
  int* status;
  uint64_t timeout_ns;
};

void gemm_bf16_tcgen05(const GemmArgs& a, int bn_hint, cudaStream_t stream);
int device_sm_count();

}  // namespace flare
