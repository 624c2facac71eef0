// Jagged causal attention (attention.cu): 8 heads x head dim 32 over packed sequences.
#pragma once

#include "common.cuh"

namespace flare {

struct AttnFwdParams {
  const void* qkv;       // [T_cap, ld_qkv] bf16: Q | K | V (768 columns used)
  int64_t ld_qkv;
  const void* vt;        // [256, ld_vt] bf16: V transposed
  int64_t ld_vt;
  const int* offsets;    // [nseq + 1] token offsets, each a multiple of 8
  int nseq;
  int max_len;           // longest sequence the grid covers
  int64_t T_cap;         // packed token capacity (multiple of 8)
  float scale;           // softmax scale (1/sqrt(head dim))
  __nv_bfloat16* out;    // [T_cap, ld_out]
  int64_t ld_out;
  float* lse;            // [8, ld_lse] log2-domain log-sum-exp of the scaled scores
  int64_t ld_lse;
  int* status;
  uint64_t timeout_ns;
};

struct AttnBwdParams {
  const void* qkv;       // as in the forward
  int64_t ld_qkv;
  const void* dout;      // [T_cap, ld_do] bf16 gradient of the output
  const void* out;       // [T_cap, ld_do] bf16 forward output (same pitch as dout)
  int64_t ld_do;
  const void* dout_t;    // [256, ld_t] bf16 dout transposed
  const void* q_t;       // [256, ld_t] bf16 Q transposed
  int64_t ld_t;
  const int* offsets;
  int nseq;
  int max_len;
  int64_t T_cap;
  float scale;
  const float* lse;      // [8, ld_stat] from the forward
  float* delta;          // [8, ld_stat] workspace: rowsum(dout * out) per head
  int64_t ld_stat;
  float* dq_acc;         // [T_cap, ld_dq] fp32, zero on entry (left zeroed on exit)
  int64_t ld_dq;
  __nv_bfloat16* dqkv;   // [T_cap, ld_dqkv] bf16: dQ | dK | dV
  int64_t ld_dqkv;
  int* status;
  uint64_t timeout_ns;
};

void attn_forward(const AttnFwdParams& p, cudaStream_t s);
void attn_backward(const AttnBwdParams& p, cudaStream_t s);

}  // namespace flare
