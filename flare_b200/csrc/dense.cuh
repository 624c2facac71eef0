// Parameter blocks for the dense-tower kernels in dense.cu.
#pragma once

#include "common.cuh"

namespace flare {

struct InteractionParams {
  int B, F, D;  // batch, embedded features, width (bottom output width == D)
  const __nv_bfloat16* bot;
  int64_t bot_ld;
  const __nv_bfloat16* emb;  // [B, F*D] pooled embeddings
  int64_t emb_ld;
  __nv_bfloat16* out;  // forward output [B, out_ld]
  const __nv_bfloat16* dout;  // backward input [B, out_ld]
  int64_t out_ld;
  __nv_bfloat16* dbot;
  int64_t dbot_ld;
  __nv_bfloat16* demb;
  int64_t demb_ld;
  int relu_mask_bot;  // apply ReLU-backward using bot > 0
  int* status;        // device status word for the bounded tcgen05 waits (may be null)
};

struct HeadBceParams {
  int B, H, T;
  const __nv_bfloat16* h;
  int64_t h_ld;
  const __nv_bfloat16* w;     // [T, H] compute copy
  const __nv_bfloat16* bias;  // [T]
  const float* labels;
  int64_t label_ld;
  const float* target_weights;  // [T] or null
  const float* sample_weights;  // [B] or null
  int valid_count;              // samples >= valid_count are masked; -1 = all valid
  float grad_scale;             // 1 / global normaliser
  float* logits;                // [B, T]
  float* loss_sum;              // scalar (accumulated)
  __nv_bfloat16* dh;
  int64_t dh_ld;
  float* dw;  // [T, H] accumulated
  float* db;  // [T] accumulated
};

enum DenseOptKind : int { kDenseAdam = 0, kDenseSgd = 1, kDenseAdagrad = 2, kDenseRmsprop = 3 };

struct AdamParams {
  int kind;
  float lr, beta1, beta2, eps, weight_decay;
  int decoupled;  // AdamW-style decoupled weight decay
  int nesterov;
  float bias_corr1, bias_corr2;  // used when step_ptr is null
  const int* step_ptr;           // device step counter (1-based) -> bias corrections in-kernel
};

struct AdamFlatParams {
  float* master;
  float* grad;
  float* m;
  float* v;
  __nv_bfloat16* compute_copy;  // nullable
  int64_t n;
  float grad_scale;
  int zero_grad;
  AdamParams opt;
};

struct AdamDpParams {
  int world, rank;
  int64_t lo, hi;              // owned slice of the flat buffer
  float* const* peer_grad;     // [world] fp32 flat gradient buffers
  void* const* peer_param;     // [param_world] bf16 flat compute copies the update is written to
  int param_world;             // world: replicate (all-gather by push); 1: only the local copy (FSDP)
  float* master_shard;         // fp32 [hi-lo]
  float* m_shard;
  float* v_shard;
  float grad_scale;
  AdamParams opt;
  uint32_t* flags_local;
  uint32_t* const* peer_flags;
  int flag_in, flag_out;
  uint32_t* epoch_ctr;
  unsigned* block_counter;
  int* status;
  uint64_t timeout_ns;
};

int grid_for(int64_t n, int threads);
void interaction_forward(const InteractionParams& p, cudaStream_t s);
void interaction_backward(const InteractionParams& p, cudaStream_t s);
void head_bce(const HeadBceParams& p, cudaStream_t s);
void adam_flat(const AdamFlatParams& p, cudaStream_t s);
void increment_counter(int* p, cudaStream_t s);
void adam_dp_fused(const AdamDpParams& p, cudaStream_t s);
void colsum_bf16(const __nv_bfloat16* x, int64_t rows, int cols, int64_t ldx, float* out, cudaStream_t s);
void cast_pad_bf16(const float* x, int64_t rows, int cols, int64_t ldx, __nv_bfloat16* y, int ldy, cudaStream_t s,
                   float* zero = nullptr);
void init_uniform(void* out, int dtype, int64_t n, float lo, float hi, uint64_t seed, int64_t index_offset,
                  int ncols, int dim, int col_begin, int64_t row_stride, int64_t row_first, cudaStream_t s);

}  // namespace flare
