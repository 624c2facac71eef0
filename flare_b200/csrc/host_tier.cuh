// Host-DRAM tier cache placement (host_tier.cu).
#pragma once

#include "common.cuh"

namespace flare {

constexpr int kMaxTierTables = 16;

struct TierTable {
  int feature;          // KJT feature feeding the table
  int ncols;            // columns held (multiple of 4)
  int64_t rows;         // table rows (valid ids)
  int C;                // HBM cache slots
  int* slot_map;        // [rows] row -> slot (-1 absent, -2 claimed this step)
  int64_t* slot2row;    // [C] slot -> row (-1 empty)
  int* stamp;           // [C] last step that used the slot
  unsigned* hand;       // CLOCK hand
  float* cache_w;       // [C, ncols]
  float* cache_row;     // [C] row-wise optimizer state or null
  float* cache_m;       // [C, ncols] or null
  float* cache_v;       // [C, ncols] or null
  float* host_w;        // [rows, ncols] pinned host memory (device-accessible address)
  float* host_row;      // [rows] or null
  float* host_m;        // [rows, ncols] or null
  float* host_v;        // [rows, ncols] or null
  int* miss_rows;       // [miss_cap] rows missing this step
  int* num_miss;        // counter (reset by the fill kernel)
  int miss_cap;
};

struct TierParams {
  TierTable tables[kMaxTierTables];
  int num_tables;
  int world, rank, Bl;
  const int* const* peer_offsets;  // [world] KJT offsets buffers (int32[F*Bl+1])
  const int* const* peer_values;   // [world] KJT id buffers
  const int* step_ptr;             // device step counter (the step being prepared)
  uint32_t* flags_local;           // entry barrier (world > 1)
  uint32_t* const* peer_flags;
  int flag_in;
  uint32_t* epoch_ctr;
  unsigned* block_counter;
  unsigned* block_counter2;
  int* status;
  uint64_t timeout_ns;
};

void tier_prepare(const TierParams& p, int grid, cudaStream_t s);

}  // namespace flare
