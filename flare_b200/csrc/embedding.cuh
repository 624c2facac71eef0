// Shared declarations for the sharded embedding-bag kernels.
#pragma once

#include "common.cuh"

namespace flare {

// One locally owned shard of a table: table-wise (all columns), a column-wise
// slice, or a row-wise (modulo) piece: rows i with i % rw_n == rw_idx, held at
// local row i / rw_n.  Row ids index the table directly (static vocabulary).
struct ShardDesc {
  int feature;         // index of the input feature (KJT key) feeding this table
  int col_begin;       // first table column held by this shard
  int ncols;           // number of columns held (multiple of 4)
  int out_col;         // column of the pooled output row receiving col_begin
  int64_t rows;        // rows held in HBM (the whole table, or the cache slots of a host-tier table)
  int64_t weight_off;  // element offset of the shard in the weight buffer
  int64_t row_base;    // offset of the shard's first row in per-row arrays
  int pooling;         // 0 = sum, 1 = mean
  int flags;           // bit 0: ids are read from the remap buffers (dynamic tables: key -> slot)
  int64_t id_rows;     // valid ids are [0, id_rows)
  int64_t slot_map_off;  // >= 0: ids map to HBM rows through slot_map[slot_map_off + id]; -1: id = row
  int rw_n;              // row shards of the table (1: the shard holds every row)
  int rw_idx;            // this shard's residue
  int part_col;          // row-wise: column of the fp32 partial-sum rows receiving col_begin; -1 otherwise
  int pad_;
};

// A row-wise table as the requester sees it: partial pooled rows of its rw_n
// pieces are summed into the pooled output.
struct RwTable {
  int out_col, part_col, ncols, rw_n;
};

enum SparseOptKind : int {
  kOptSgd = 0,
  kOptRowwiseAdagrad = 1,
  kOptAdam = 2,
  kOptRowwiseAdam = 3,
  kOptAdagrad = 4,
};

enum LrPolicy : int {
  kLrConstant = 0,
  kLrSqrtDecay = 1,
  kLrLogDecay = 2,
  kLrInverseDecay = 3,
  kLrCosineFrequency = 4,
  kLrCustomLut = 5,
};

struct SparseOptParams {
  int kind;
  float lr, beta1, beta2, eps, weight_decay;
  float bias_corr1, bias_corr2;  // 1 - beta^t for the current optimizer step (if step_ptr null)
  const int* step_ptr;           // device step counter (1-based); bias corrections computed in-kernel
  int lr_policy;
  float policy_a, policy_b;  // cosine: min_lr_ratio, max_score
  const float* lut;
  int lut_len;
  float* state_row;  // per-row fp32 state (row-wise adagrad sum, row-wise adam v)
  float* state_m;    // per-element first moment (adam) / accumulator (adagrad)
  float* state_v;    // per-element second moment (adam)
  float* score;      // per-row access score for frequency-based LR policies (nullable)
  float grad_scale;  // multiplies every row's gradient sum (1 / micro-steps of an accumulation window)
};

struct EmbFwdParams {
  const ShardDesc* shards;
  int num_shards;
  int world, rank, Bl, F;
  const int* const* peer_offsets;  // [world] offsets buffers, int32[F*Bl+1]
  const int* const* peer_values;   // [world] id buffers
  void* const* peer_out;           // [world] pooled outputs (bf16 rows of out_stride)
  int64_t out_stride;
  const void* weights;
  int w_dtype;
  int out_dtype;  // kBF16 or kF32
  int vec;        // float4 vectors per lane: 1 (shard width <= 128) or 2 (<= 256); bulk: 16-byte segments
                  // per lane: 1 (rows <= 512 bytes) or 2 (<= 1024)
  int bulk;       // 1: TMA bulk-gather forward (every shard's rows 16-byte aligned, <= 1024 bytes)
  const int* slot_map;  // row -> HBM slot maps of host-tier shards (ShardDesc::slot_map_off), or null
  const int* const* peer_remap;  // [world] slot buffers of dynamic tables (same layout as values), or null
  int* fetch_offs;               // multi-GPU: local copy of every (shard, source) bag-offset run [nslot][Bl + 1];
                                 // the ids are copied into the staging rows (emb_fetch_kernel), or null
  float* const* peer_part;       // [world] fp32 partial pooled rows [rw_slots][Bl][part_stride] (row-wise tables)
  int64_t part_stride;
  const RwTable* rw_tables;      // row-wise tables of the collection (reduced locally after the exchange)
  int num_rw;
  // staging for the backward pass
  int* stage_ids;    // [(sh*world+s)*stage_cap + j]
  int* stage_bag;    // same indexing: sample index of occurrence j
  int* stage_count;  // [sh*world+s] occurrences staged
  int* stage_len;    // [(sh*world+s)*Bl + b] bag length (for mean pooling)
  int64_t stage_cap;
  // cross-GPU barrier
  uint32_t* flags_local;
  uint32_t* const* peer_flags;
  int flag_in, flag_out;  // slot-array offsets in the flag buffer
  uint32_t* epoch_ctr;    // device-resident barrier epoch (advanced by the kernel)
  unsigned* block_counter;
  int* status;
  uint64_t timeout_ns;
  int fwd_minb;  // resident blocks per SM the forward is compiled for (3 or 4)
};

struct EmbBwdParams {
  const ShardDesc* shards;
  int num_shards;
  int world, rank, Bl;
  const void* const* peer_grad;  // [world] pooled-grad buffers (rows of out_stride)
  int64_t out_stride;
  int grad_dtype;                // kBF16 or kF32
  void* grad_stage;              // [(sh*world+s)*Bl + b][grad_stage_ld] (grad_dtype)
  int64_t grad_stage_ld;
  const int* stage_ids;
  const int* stage_bag;
  int* stage_rank;   // written by the counting pass (compact index: slot_start[slot] + j)
  int* slot_start;   // [nslot + 1] exclusive prefix of the staged ids per (shard, source) slot
  const int* stage_count;
  const int* stage_len;
  int64_t stage_cap;
  void* weights;
  int w_dtype;
  // dedup / segment scratch
  int* row_count;   // per-row occurrence counter (reset to zero by the apply kernels)
  int* row2u;       // per-row unique index
  int* flags;       // [T] 1 at each row's first occurrence (compact index)
  int* pos;         // [T + 1] exclusive scan of flags
  int64_t* uniq_row;
  int* uniq_shard;
  int* cnt_u;       // occurrences of unique row u
  int* first_gidx;  // staged-grad row of u's first occurrence
  int* num_unique;  // [0] U, [1] T (valid occurrences), [2] heavy rows; hash path: [3] work chunks,
                    // [4] single-occurrence rows, [5] other light rows, [6] overflow slots in use
  int* seg_start;   // [U+1]
  int* block_sums;
  int* occ;         // staged-grad row index per occurrence, grouped by unique row
  int* heavy;       // unique rows with more than light_max occurrences
  int* hcnt;        // [H] occurrence count of each heavy row
  int* heavy_start; // [H+1] exclusive prefix of heavy-row counts
  float* heavy_acc; // [max_heavy + max_occ / 256 + 2][32*4*NV] fp32 partial sums per (heavy row, chunk)
  int max_heavy;
  int light_max;
  unsigned* dirty;  // per-row dirty bits for incremental checkpoints, 32 rows a word (nullable)
  int64_t max_occ;  // capacity of the per-unique arrays
  // deterministic-reduction mode: every row adds its occurrences in staging order (run-to-run
  // bitwise identical results); needs det_keys [2 * max_occ], det_vals [max_occ] and the sort's
  // temporary storage (emb_det_temp_bytes)
  int deterministic;
  int* det_first;    // per-row first staging position (INT_MAX when idle; reset by the emit kernel)
  int* det_keys;
  int* det_vals;
  void* det_temp;
  size_t det_temp_bytes;
  // hash-dedup path (the default when not deterministic): an open-addressing table of the step's
  // touched rows replaces the per-row count / index arrays, so the dedup stays in L2
  int hash_mode;
  int grad_direct;           // 1 (one GPU): read the pooled gradients in place, no pull into grad_stage
  unsigned long long* htab;  // [hregion + hcap] slot word: key (local row, low 32 bits) | count (high 32); empty = 0xFFFFFFFF
  int* hseg;                 // [hregion + hcap] segment start of an occupied slot's occurrences in occ, or
                             // -1 - record index of a single-occurrence row
  int* ovf_list;             // [max_occ] overflow-table slots in use this step
  int64_t hcap;              // overflow table slots (power of two >= max_occ), after the region
  int64_t hregion;           // region slots (power of two, or 0): the first probes of every key
  int hprefetch;             // 1: the counting pass prefetches the region into L2
  int* occ_h;                // [max_occ] hash slot of compact occurrence k (-1: invalid id)
  int* occ_rank;             // [max_occ] rank of k among its row's occurrences
  int* occ_bag;              // [max_occ] bag index of k: slot * Bl + sample
  int4* lrec;                // [max_occ] light-row records {row, slot, seg, count}: single-occurrence rows from
                             // the front, the other light rows from the back
  int4* crec;                // [max_chunks][2] work-chunk records {row, slot, first, len}, {part, chunk, chunks, count}
  int64_t max_chunks;
  float* hpart;              // [max_parts][ncols_max] fp32 partial sums of multi-chunk rows
  int64_t max_parts;
  float* occ_scale;          // [max_occ] 1 / bag length per grouped occurrence (mean pooling), or null
  int* scan_val;             // [max_tiles][6] per-block totals of the slot scan
  int64_t max_tiles;         // scan blocks at most
  SparseOptParams opt;
  uint32_t* flags_local;
  uint32_t* const* peer_flags;
  int flag_in;
  uint32_t* epoch_ctr;
  unsigned* block_counter;
  int* status;
  uint64_t timeout_ns;
  int light_prefetch;  // fp32 tables: the light-row pass keeps the next batch's rows in flight (cp.async; opt-in)
  int chunk_variant;   // chunk pass code variant (see hash_apply_launch; 1 by default)
};

// Gradient-accumulation window: the staging of micro-step `micro` appended to the window's staging,
// which the backward then reads as one batch of micro_steps * Bl samples (bags shifted by micro * Bl).
struct EmbWindowParams {
  const int* ids;    // the step's staging: [nslot][stage_cap] ids / bags, [nslot] counts, [nslot][Bl] lengths
  const int* bag;
  const int* count;
  const int* len;
  int* wids;         // the window's staging: [nslot][micro_steps * stage_cap] ids / bags
  int* wbag;
  int* wprefix;      // [micro_steps + 1][nslot]: occurrences of each slot before micro-step k (row k)
  int* wlen;         // [nslot][micro_steps * Bl]
  int nslot, Bl, micro, micro_steps;
  int64_t stage_cap;
};

void emb_forward(const EmbFwdParams& p, int grid, cudaStream_t s);
void emb_window_append(const EmbWindowParams& p, cudaStream_t s);
void emb_backward(const EmbBwdParams& p, int ncols_max, int grid, cudaStream_t s);
void emb_backward_hash(const EmbBwdParams& p, int ncols_max, int grid, cudaStream_t s);
size_t emb_det_temp_bytes(int64_t max_occ);
// scratch sizes of the hash-dedup backward
int64_t emb_hash_tile_count(int64_t max_occ);
int64_t emb_hash_max_chunks(int64_t max_occ, int light_max);
int64_t emb_hash_max_parts(int64_t max_occ);
int emb_hash_scan_vals();

}  // namespace flare
