// Declarations for the padded-inverse sparse ops and GPU dedup (sparse_ops.cu).
#pragma once

#include "common.cuh"

namespace flare {

struct UniqueScratch {
  unsigned long long* tab_keys;  // [cap]
  int* tab_first;                // [cap]
  int64_t cap;                   // power of two >= 2n
  int64_t* slot_of;              // [n]
  int* is_first;                 // [n]
  int* pos;                      // [n+1]
  int* block_sums;               // [512]
};

void exclusive_scan_int(const int* in, int64_t n, int* out, int* block_sums, cudaStream_t s);
void sparse_gather(const void* emb, int dtype, const int* inv, int64_t slots, int dim, int pad, void* out,
                   cudaStream_t s);
void sparse_gather_pooled(const void* emb, int dtype, const int* inv, int64_t bags, int E, int dim, int pad,
                          void* out, cudaStream_t s);
void sparse_scatter(const void* grad, int dtype, const int* inv, int64_t slots, int dim, int pad, float* out,
                    cudaStream_t s);
void sparse_scatter_pooled(const void* grad, int dtype, const int* inv, int64_t bags, int E, int dim, int pad,
                           float* out, cudaStream_t s);
void unique_first_occurrence(const int64_t* keys, int64_t n, const UniqueScratch& w, int64_t* unique, int* inverse,
                             int64_t* first_idx, cudaStream_t s);

}  // namespace flare
