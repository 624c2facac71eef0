// Host-DRAM tier cache maintenance (host_tier.cu).
#pragma once

#include "common.cuh"

namespace flare {

struct TierCopyParams {
  int n;                  // rows to move
  int ncols;              // columns (multiple of 4)
  const int* slots;       // [n] HBM slots
  float* cache_w;         // [C, ncols] cache rows
  float* cache_row;       // [C] row-wise state or null
  float* cache_m;         // [C, ncols] or null
  float* cache_v;         // [C, ncols] or null
  float* stage_w;         // [n, ncols]
  float* stage_row;       // [n] or null
  float* stage_m;         // [n, ncols] or null
  float* stage_v;         // [n, ncols] or null
  // install only
  int* slot_map;          // [rows] row -> slot
  const int64_t* new_rows;    // [n]
  const int64_t* evict_rows;  // [n_evict]
  int n_evict;
};

void tier_gather(const TierCopyParams& p, cudaStream_t s);
void tier_install(const TierCopyParams& p, cudaStream_t s);

}  // namespace flare
