// Dynamic (hash-keyed) embedding tables: placement kernels (dynamic_emb.cu).
#pragma once

#include "common.cuh"

namespace flare {

constexpr int kMaxDynTables = 16;

struct DynTable {
  int feature;          // KJT feature feeding the table
  int ncols;            // columns held
  int col_begin;        // first table column held (init hash input)
  int C;                // HBM slots (rows)
  int H;                // hash buckets (power of two, >= 2C)
  float init_scale;     // new rows ~ uniform(-init_scale, init_scale)
  uint64_t seed;
  int* keys;            // [H] key or -1 empty / -2 tombstone
  int* slot_of;         // [H] slot of the bucket's key (-1 none)
  int* bucket_of;       // [C] bucket holding the slot's key (-1 free)
  int* stamp;           // [C] last step that used the slot
  unsigned* hand;       // CLOCK hand
  float* weights;       // [C, ncols]
  float* state_row;     // [C] or null
  float* state_m;       // [C, ncols] or null
  float* state_v;       // [C, ncols] or null
  float* score;         // [C] or null
  int* new_buckets;     // [new_cap] buckets of keys inserted this step
  int* num_new;
  int new_cap;
  int* num_tomb;        // tombstones created (rebuild trigger)
};

struct DynParams {
  DynTable tables[kMaxDynTables];
  int num_tables;
  int world, rank, Bl;
  const int* const* peer_offsets;
  const int* const* peer_values;
  int* const* peer_remap;      // [world] remap buffers (same layout as the values buffers)
  const int* step_ptr;
  uint32_t* flags_local;
  uint32_t* const* peer_flags;
  int flag_in;
  uint32_t* epoch_ctr;
  unsigned* block_counter;
  unsigned* block_counter2;
  int* status;
  uint64_t timeout_ns;
};

void dyn_prepare(const DynParams& p, int grid, cudaStream_t s);
// Re-insert the live (key, slot) pairs of one table into a cleared hash map (drops tombstones).
void dyn_rebuild(int* keys, int* slot_of, int* bucket_of, int H, const int* live_keys, const int* live_slots, int n,
                 cudaStream_t s);

}  // namespace flare
