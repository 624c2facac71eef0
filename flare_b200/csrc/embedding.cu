// Sharded embedding-bag kernels with the all-to-alls fused in (sm_100a).
//
// Forward (one launch per step):
//   entry barrier with every peer (their ids are staged, their previous pooled
//   output has been consumed) -> for every locally owned shard and every
//   (source rank, sample) bag: read the bag's ids straight from the source
//   rank's memory over NVLink (the ids all-to-all), gather + sum/mean pool the
//   local HBM rows in fp32, and store the pooled row straight into the source
//   rank's pooled-output buffer (the pooled all-to-all); the ids are staged
//   locally for the backward -> exit barrier (every owner has written).
//
// Backward (short launches, no host sync, no global hot counters):
//   1. entry barrier; pull the pooled gradients of every (source, sample) bag
//      of the owned columns (pooled-gradient all-to-all) and, in the same
//      launch, count occurrences per row (warp-aggregated atomics), record
//      each occurrence's rank within its row and flag rank 0;
//   2. scan of the flags -> dense unique ids in occurrence order (deterministic);
//   3. emit per-unique metadata (row, shard, count, first occurrence);
//   4. scan of per-unique counts -> segment starts;
//   5. fill: occ[seg_start[u] + rank] = staged-grad row (no atomics);
//   6. light rows (<= light_max occurrences): one row per lane group, fp32
//      segment sum + optimizer applied in place, per-row counter reset;
//   7. heavy rows (Zipf head): their occurrences are cut into equal chunks
//      across warps (balanced however skewed the counts are), each
//      (row, chunk) segment stores an fp32 partial row, then one warp per row
//      adds its partials in chunk order and applies the optimizer.
//
// Reference behaviour: gather/pool/scatter semantics of
// src/flare/kernels/backends/gpu_cupy.py:52-252 and
// src/flare/ops/sparse_gather.py:40-99 (sum, mean with max(len,1)); the
// reference routes ids and values through Fluxway transport
// (src/flare/runtime/fluxway/workers/dynamic_embedding.py:362-438, 551-681)
// and updates rows in its external native store.
#include "embedding.cuh"
#include "sm100.cuh"
#include "sparse_update.cuh"

#include <cub/device/device_radix_sort.cuh>
#include "sparse_ops.cuh"

#include <algorithm>

namespace flare {
namespace {

constexpr unsigned kFull = 0xffffffffu;
constexpr int kEmbThreads = 256;
constexpr int kMaxShardsSmem = 96;

__device__ __forceinline__ unsigned lanemask_lt() {
  unsigned m;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

__device__ __forceinline__ void barrier_signal(uint32_t* const* peer_flags, int world, int rank, int slot_off,
                                               uint32_t epoch) {
  fence_sys();
  for (int s = 0; s < world; ++s) st_release_sys(peer_flags[s] + slot_off + rank, epoch);
}

__device__ __forceinline__ bool barrier_wait(const uint32_t* flags_local, int world, int slot_off, uint32_t epoch,
                                             uint64_t timeout_ns, int* status) {
  bool ok = true;
  for (int s = 0; s < world && ok; ++s) ok = wait_flag_geq(flags_local + slot_off + s, epoch, timeout_ns, status, s);
  return ok;
}

// Entry barrier executed by every block: block 0 announces this rank, every
// block waits until all peers announced. Returns false on timeout.
__device__ __forceinline__ bool entry_barrier(uint32_t* flags_local, uint32_t* const* peer_flags, int world, int rank,
                                              int slot_off, uint32_t epoch, uint64_t timeout_ns, int* status) {
  __shared__ int ok_sh;
  if (threadIdx.x == 0) {
    if (blockIdx.x == 0) barrier_signal(peer_flags, world, rank, slot_off, epoch);
    ok_sh = barrier_wait(flags_local, world, slot_off, epoch, timeout_ns, status) ? 1 : 0;
  }
  __syncthreads();
  return ok_sh != 0;
}

// ============================================================================
// Forward
// ============================================================================
// Validated local row of an id for shard d, or -1 (out of range: reported; other residue of a
// row-wise piece: skipped; host-tier row not resident: reported).
__device__ __forceinline__ int map_id(const EmbFwdParams& p, const ShardDesc& d, int id, bool report) {
  if (id < 0 || id >= d.id_rows) {
    if (report) report_error(p.status, kIndexOutOfRange, d.feature);
    return -1;
  }
  if (d.rw_n > 1) {
    const int q = id / d.rw_n;
    return id - q * d.rw_n == d.rw_idx ? q : -1;
  }
  if (d.slot_map_off >= 0) {
    const int slot = p.slot_map[d.slot_map_off + id];
    if (slot < 0 || slot >= d.rows) {
      if (report) report_error(p.status, kIndexOutOfRange, 1000 + d.feature);
      return -1;
    }
    return slot;
  }
  return id;
}

// Multi-GPU forward prologue: after the entry barrier, copy every (owned shard, source rank) run of
// bag offsets and ids from the source's memory into local buffers (the ids land in the staging rows,
// where the forward maps them in place).  Bandwidth-bound bulk reads over NVLink replace the
// forward's two dependent remote round trips per bag (offsets, then ids).
__global__ void __launch_bounds__(kEmbThreads) emb_fetch_kernel(EmbFwdParams p) {
  const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(p.epoch_ctr) + 1u;
  if (!entry_barrier(p.flags_local, p.peer_flags, p.world, p.rank, p.flag_in, epoch, p.timeout_ns, p.status))
    return;
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t nth = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int nslot = p.num_shards * p.world;
  for (int slot = 0; slot < nslot; ++slot) {
    const int sh = slot / p.world, s = slot - sh * p.world;
    const ShardDesc& d = p.shards[sh];
    const int* offs = p.peer_offsets[s] + d.feature * p.Bl;
    int* lo = p.fetch_offs + static_cast<int64_t>(slot) * (p.Bl + 1);
    for (int64_t i = tid; i <= p.Bl; i += nth) lo[i] = offs[i];
    const int fbase = offs[0];
    int64_t cnt = offs[p.Bl] - fbase;
    if (cnt > p.stage_cap) {
      if (tid == 0) report_error(p.status, kCapacityOverflow, slot);
      cnt = p.stage_cap;
    }
    const int* src = ((d.flags & 1) ? p.peer_remap[s] : p.peer_values[s]) + fbase;
    int* dst = p.stage_ids + static_cast<int64_t>(slot) * p.stage_cap;
    for (int64_t i = tid; i < cnt; i += nth) dst[i] = src[i];
  }
}

// Forward: every (source rank, sample) bag of every owned shard; a group of G lanes per bag, each
// lane owning 4*VEC columns, 8 rows in flight per lane.  (A variant that loaded the next bag's
// offsets and ids while pooling this one and bulk-prefetched its rows into L2 measured 1-3% slower
// on the DLRM benchmark: the look-ahead state cost a resident block per SM.)
template <typename TW, int VEC, int MINB>
__global__ void __launch_bounds__(kEmbThreads, MINB) emb_fwd_kernel(EmbFwdParams p) {
  const uint32_t epoch = p.world > 1 ? *reinterpret_cast<volatile uint32_t*>(p.epoch_ctr) + 1u : 0u;
  const bool fetched = p.fetch_offs != nullptr;  // offsets and ids already copied here (emb_fetch_kernel)
  if (p.world > 1 && !fetched) {
    if (!entry_barrier(p.flags_local, p.peer_flags, p.world, p.rank, p.flag_in, epoch, p.timeout_ns, p.status))
      return;
  }
  const int lane = lane_id();
  const int64_t gwarp = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + warp_id();
  const int64_t nwarps = static_cast<int64_t>(gridDim.x) * (blockDim.x / 32);
  const TW* W = reinterpret_cast<const TW*>(p.weights);
  const int64_t nitems = static_cast<int64_t>(p.world) * p.Bl;

  for (int sh = 0; sh < p.num_shards; ++sh) {
    const ShardDesc d = p.shards[sh];
    const int G = d.ncols / (4 * VEC);  // lanes per bag (power of two <= 32)
    const int gpw = 32 / G;
    const int g = lane / G;
    const int l = lane - g * G;
    const int col0 = l * 4 * VEC;
    const TW* wshard = W + d.weight_off + col0;
    for (int64_t base = gwarp * gpw; base < nitems; base += nwarps * gpw) {
      const int64_t item = base + g;
      const bool active = item < nitems;
      // item -> (sample, source) with the source fastest, so neighbouring
      // groups read from different peers.
      const int b = active ? static_cast<int>(item / p.world) : 0;
      const int s = active ? static_cast<int>(item - static_cast<int64_t>(b) * p.world) : 0;
      int beg = 0, len = 0, fbase = 0;
      if (active && l == 0) {
        const int slot = sh * p.world + s;
        const int* offs = fetched ? p.fetch_offs + static_cast<int64_t>(slot) * (p.Bl + 1)
                                  : p.peer_offsets[s] + d.feature * p.Bl;
        fbase = offs[0];
        beg = offs[b];
        len = offs[b + 1] - beg;
        p.stage_len[static_cast<int64_t>(slot) * p.Bl + b] = len;
        if (b == 0) p.stage_count[slot] = offs[p.Bl] - fbase;
      }
      beg = __shfl_sync(kFull, beg, g * G);
      len = __shfl_sync(kFull, len, g * G);
      fbase = __shfl_sync(kFull, fbase, g * G);
      const int slot = sh * p.world + s;
      const int64_t spos = beg - fbase;
      const bool stage_ok = active && (spos + len <= p.stage_cap);
      if (active && l == 0 && !stage_ok) report_error(p.status, kCapacityOverflow, slot);
      const int64_t stage_base = static_cast<int64_t>(slot) * p.stage_cap + spos;
      int maxlen = active ? len : 0;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) maxlen = max(maxlen, __shfl_xor_sync(kFull, maxlen, o));

      float4 acc[VEC];
#pragma unroll
      for (int v = 0; v < VEC; ++v) acc[v] = make_float4(0.f, 0.f, 0.f, 0.f);
      const int* vals = (d.flags & 1) ? p.peer_remap[s] : p.peer_values[s];
      for (int j = 0; j < maxlen; j += G) {
        int myid = -1;
        const bool has = active && j + l < len;
        if (has) myid = map_id(p, d, fetched ? (stage_ok ? p.stage_ids[stage_base + j + l] : -1) : vals[beg + j + l], true);
        if (has && stage_ok) {
          p.stage_ids[stage_base + j + l] = myid;
          p.stage_bag[stage_base + j + l] = b;
        }
        const int cnt = min(G, maxlen - j);
        int t = 0;
        for (; t + 8 <= cnt; t += 8) {
          int id[8];
#pragma unroll
          for (int q = 0; q < 8; ++q) id[q] = __shfl_sync(kFull, myid, g * G + t + q);
          float4 r[8][VEC];
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const TW* row = wshard + static_cast<int64_t>(id[q] < 0 ? 0 : id[q]) * d.ncols;
#pragma unroll
            for (int v = 0; v < VEC; ++v) r[q][v] = load4<TW>(row + 4 * v);
          }
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const float m = id[q] < 0 ? 0.f : 1.f;
#pragma unroll
            for (int v = 0; v < VEC; ++v) acc[v] = f4_add(acc[v], f4_scale(r[q][v], m));
          }
        }
        for (; t < cnt; ++t) {
          const int id = __shfl_sync(kFull, myid, g * G + t);
          if (id >= 0) {
            const TW* row = wshard + static_cast<int64_t>(id) * d.ncols;
#pragma unroll
            for (int v = 0; v < VEC; ++v) acc[v] = f4_add(acc[v], load4<TW>(row + 4 * v));
          }
        }
      }
      if (active) {
        if (d.pooling == 1 && len > 0) {
          const float inv = 1.f / static_cast<float>(len);
#pragma unroll
          for (int v = 0; v < VEC; ++v) acc[v] = f4_scale(acc[v], inv);
        }
        const int64_t off = static_cast<int64_t>(b) * p.out_stride + d.out_col + col0;
        if (d.part_col >= 0) {
          // row-wise piece: fp32 partial sum into the requester's partial rows of this residue
          float* out = p.peer_part[s] + (static_cast<int64_t>(d.rw_idx) * p.Bl + b) * p.part_stride + d.part_col +
                       col0;
#pragma unroll
          for (int v = 0; v < VEC; ++v) store4<float>(out + 4 * v, acc[v]);
        } else if (p.out_dtype == kBF16) {
          __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(p.peer_out[s]) + off;
#pragma unroll
          for (int v = 0; v < VEC; ++v) store4<__nv_bfloat16>(out + 4 * v, acc[v]);
        } else {
          float* out = reinterpret_cast<float*>(p.peer_out[s]) + off;
#pragma unroll
          for (int v = 0; v < VEC; ++v) store4<float>(out + 4 * v, acc[v]);
        }
      }
    }
  }

  if (p.world > 1) {
    // Exit barrier: the last block to finish tells every peer that this
    // rank's writes into their pooled buffers are complete, then waits until
    // all owners have finished writing into ours.
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
      const unsigned prev = atomicAdd(p.block_counter, 1u);
      if (prev == gridDim.x - 1) {
        *p.block_counter = 0u;
        *p.epoch_ctr = epoch;
        barrier_signal(p.peer_flags, p.world, p.rank, p.flag_out, epoch);
        barrier_wait(p.flags_local, p.world, p.flag_out, epoch, p.timeout_ns, p.status);
      }
    }
  }
}

// ----------------------------------------------------------------------------
// Forward, TMA bulk-gather variant (used when every shard's rows are 16-byte
// aligned).  A persistent CTA per SM; each warp runs its own pipeline over
// "jobs" (up to R ids of one bag): the ids of the next job are loaded one job
// ahead, each id's row is copied HBM -> shared memory by one cp.async.bulk
// issued by the lane holding the id (completion counted on the stage's
// mbarrier, no registers held while the copy is in flight), and a job is
// pooled from shared memory kBulkStages - 1 jobs after it was issued.  The
// rows of up to kBulkStages jobs per warp are in flight at once, so the
// gather runs at the memory system's rate instead of the registers' reach.
// ----------------------------------------------------------------------------
constexpr int kBulkWarps = 8;
constexpr int kBulkStages = 4;
constexpr int kBulkStageBytes = 6144;
constexpr int kBulkThreads = kBulkWarps * 32;
constexpr int kBulkMeta = 6;  // item, shard, nvalid, flags (1 first, 2 last), len, pad
constexpr size_t kBulkSmem = static_cast<size_t>(kBulkWarps) * kBulkStages * kBulkStageBytes +
                             kBulkWarps * kBulkStages * (8 + kBulkMeta * 4) + kMaxShardsSmem * sizeof(ShardDesc) + 256;

struct BulkCursor {
  int sh, item, c;       // shard, work item (source-fastest bag index), chunk within the bag
  int beg, len, fbase;   // bag (broadcast to every lane)
  bool valid;
};

template <typename TW, int VEC>
__global__ void __launch_bounds__(kBulkThreads, 1) emb_fwd_bulk_kernel(EmbFwdParams p) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  uint8_t* stages = smem_raw;
  uint64_t* bars = reinterpret_cast<uint64_t*>(stages + static_cast<size_t>(kBulkWarps) * kBulkStages *
                                                             kBulkStageBytes);
  int* meta_all = reinterpret_cast<int*>(bars + kBulkWarps * kBulkStages);
  ShardDesc* sd = reinterpret_cast<ShardDesc*>(meta_all + kBulkWarps * kBulkStages * kBulkMeta);

  const uint32_t epoch = p.world > 1 ? *reinterpret_cast<volatile uint32_t*>(p.epoch_ctr) + 1u : 0u;
  for (int i = threadIdx.x; i < p.num_shards; i += blockDim.x) sd[i] = p.shards[i];
  const int warp = warp_id(), lane = lane_id();
  uint64_t* wbars = bars + warp * kBulkStages;
  int* wmeta = meta_all + warp * kBulkStages * kBulkMeta;
  uint8_t* wst = stages + static_cast<size_t>(warp) * kBulkStages * kBulkStageBytes;
  if (lane == 0) {
    for (int i = 0; i < kBulkStages; ++i) sm100::mbar_init(wbars + i, 1);
    sm100::fence_mbar_init();
  }
  __syncthreads();
  if (p.world > 1) {
    if (!entry_barrier(p.flags_local, p.peer_flags, p.world, p.rank, p.flag_in, epoch, p.timeout_ns, p.status))
      return;
  }
  const int nitems = p.world * p.Bl;
  const int nwt = static_cast<int>(gridDim.x) * kBulkWarps;  // warps in the grid: item stride
  const int gw = static_cast<int>(blockIdx.x) * kBulkWarps + warp;
  const char* W = reinterpret_cast<const char*>(p.weights);
  constexpr int kSegVals = 16 / static_cast<int>(sizeof(TW));  // values per 16-byte segment

  auto rows_per_job = [&](const ShardDesc& d) {
    const int rb = d.ncols * static_cast<int>(sizeof(TW));
    return min(32, kBulkStageBytes / rb);
  };
  // raw bag info of (sh, item), read by lane 0 (which also records the staging metadata)
  auto load_bag_raw = [&](int sh, int item, int& beg, int& len, int& fbase) {
    beg = len = fbase = 0;
    if (lane == 0 && sh < p.num_shards && item < nitems) {
      const ShardDesc& d = sd[sh];
      const int b = item / p.world, s = item - b * p.world;
      const int* offs = p.peer_offsets[s];
      fbase = offs[d.feature * p.Bl];
      beg = offs[d.feature * p.Bl + b];
      len = offs[d.feature * p.Bl + b + 1] - beg;
      const int slot = sh * p.world + s;
      p.stage_len[static_cast<int64_t>(slot) * p.Bl + b] = len;
      if (b == 0) p.stage_count[slot] = offs[d.feature * p.Bl + p.Bl] - fbase;
    }
  };
  auto next_bag = [&](int& sh, int& item) {
    item += nwt;
    if (item >= nitems) {
      item = gw;
      ++sh;
    }
  };
  // first bag
  BulkCursor A;
  A.sh = 0;
  A.item = gw;
  A.c = 0;
  if (gw >= nitems) A.sh = p.num_shards;  // more warps than bags: nothing to do
  A.valid = A.sh < p.num_shards;
  load_bag_raw(A.sh, A.item, A.beg, A.len, A.fbase);
  A.beg = __shfl_sync(kFull, A.beg, 0);
  A.len = __shfl_sync(kFull, A.len, 0);
  A.fbase = __shfl_sync(kFull, A.fbase, 0);
  int nb_sh = A.sh, nb_item = A.item;
  next_bag(nb_sh, nb_item);
  int nb_beg, nb_len, nb_fbase;  // raw in lane 0
  load_bag_raw(nb_sh, nb_item, nb_beg, nb_len, nb_fbase);

  auto load_ids = [&](const BulkCursor& X) -> int {
    if (!X.valid) return -1;
    const ShardDesc& d = sd[X.sh];
    const int R = rows_per_job(d);
    const int j = X.c * R + lane;
    if (lane >= R || j >= X.len) return -1;
    const int s = X.item % p.world;
    const int* vals = (d.flags & 1) ? p.peer_remap[s] : p.peer_values[s];
    return vals[X.beg + j];
  };
  int ids_A = load_ids(A);

  uint32_t parity = 0;  // bit i: parity of the next completion of stage i
  int head = 0, tail = 0;
  bool abort = false;
  float acc[VEC][kSegVals];
#pragma unroll
  for (int v = 0; v < VEC; ++v)
#pragma unroll
    for (int e = 0; e < kSegVals; ++e) acc[v][e] = 0.f;

  while (A.valid || head > tail) {
    if (A.valid && head - tail < kBulkStages) {
      // ---- advance the cursor to job B and start loading its ids
      const ShardDesc& d = sd[A.sh];
      const int R = rows_per_job(d);
      const int njobs = max(1, (A.len + R - 1) / R);
      BulkCursor B = A;
      if (A.c + 1 < njobs) {
        B.c = A.c + 1;
      } else {
        B.sh = nb_sh;
        B.item = nb_item;
        B.c = 0;
        B.valid = nb_sh < p.num_shards;
        B.beg = __shfl_sync(kFull, nb_beg, 0);
        B.len = __shfl_sync(kFull, nb_len, 0);
        B.fbase = __shfl_sync(kFull, nb_fbase, 0);
        next_bag(nb_sh, nb_item);
        load_bag_raw(nb_sh, nb_item, nb_beg, nb_len, nb_fbase);
      }
      const int ids_B = load_ids(B);

      // ---- produce job A: map ids, stage them for the backward, issue the row copies
      const int b = A.item / p.world, s = A.item - b * p.world;
      const int slot = A.sh * p.world + s;
      const int cnt = min(R, max(0, A.len - A.c * R));
      const int64_t spos = A.beg - A.fbase;
      const bool stage_ok = spos + A.len <= p.stage_cap;
      if (A.c == 0 && lane == 0 && !stage_ok) report_error(p.status, kCapacityOverflow, slot);
      int row = -1;
      if (lane < cnt) {
        row = map_id(p, d, ids_A, true);
        if (stage_ok) {
          const int64_t at = static_cast<int64_t>(slot) * p.stage_cap + spos + A.c * R + lane;
          p.stage_ids[at] = row;
          p.stage_bag[at] = b;
        }
      }
      const unsigned vmask = __ballot_sync(kFull, row >= 0);
      const int nvalid = __popc(vmask);
      const int st = head % kBulkStages;
      const int rb = d.ncols * static_cast<int>(sizeof(TW));
      if (lane == 0) {
        int* m = wmeta + st * kBulkMeta;
        m[0] = A.item;
        m[1] = A.sh;
        m[2] = nvalid;
        m[3] = (A.c == 0 ? 1 : 0) | (A.c + 1 >= njobs ? 2 : 0);
        m[4] = A.len;
        sm100::mbar_arrive_expect_tx(wbars + st, static_cast<uint32_t>(nvalid * rb));
      }
      __syncwarp();
      if (row >= 0) {
        const int pos = __popc(vmask & lanemask_lt());
        sm100::bulk_load(wst + st * kBulkStageBytes + pos * rb,
                         W + (d.weight_off + static_cast<int64_t>(row) * d.ncols) * static_cast<int64_t>(sizeof(TW)),
                         static_cast<uint32_t>(rb), wbars + st);
      }
      ++head;
      A = B;
      ids_A = ids_B;
      if (A.valid && head - tail < kBulkStages) continue;  // keep the ring full
    }
    // ---- consume the oldest job
    const int st = tail % kBulkStages;
    const uint64_t limit = abort ? 1000000ull : p.timeout_ns;
    if (!sm100::mbar_wait(wbars + st, (parity >> st) & 1u, limit, p.status, 5000 + st)) {
      abort = true;    // stop issuing; drain the jobs in flight with short waits, then return
      A.valid = false;
    }
    parity ^= 1u << st;
    const int* m = wmeta + st * kBulkMeta;
    const int item = m[0], sh = m[1], nvalid = m[2], fl = m[3], len = m[4];
    const ShardDesc& d = sd[sh];
    const int rb = d.ncols * static_cast<int>(sizeof(TW));
    const int segs = rb / 16;
    const int G = segs >= 32 ? 32 : segs;  // lanes per row
    const int P = 32 / G;                   // rows per pass
    const int g = lane / G, l = lane - g * G;
    if (fl & 1) {
#pragma unroll
      for (int v = 0; v < VEC; ++v)
#pragma unroll
        for (int e = 0; e < kSegVals; ++e) acc[v][e] = 0.f;
    }
    if (!abort) {
      const uint8_t* base = wst + st * kBulkStageBytes;
      for (int r = g; r < nvalid; r += P) {
#pragma unroll
        for (int v = 0; v < VEC; ++v) {
          const int seg = l + 32 * v;
          if (seg < segs) {
            const uint4 q = *reinterpret_cast<const uint4*>(base + r * rb + seg * 16);
            const TW* t = reinterpret_cast<const TW*>(&q);
#pragma unroll
            for (int e = 0; e < kSegVals; ++e) acc[v][e] += to_f32(t[e]);
          }
        }
      }
    }
    __syncwarp();
    sm100::fence_proxy_async_smem();  // these generic reads precede the stage's next async writes
    ++tail;
    if (fl & 2) {
      // pooled row complete: add the P row groups, scale (mean), store
      for (int o = G; o < 32; o <<= 1)
#pragma unroll
        for (int v = 0; v < VEC; ++v)
#pragma unroll
          for (int e = 0; e < kSegVals; ++e) acc[v][e] += __shfl_xor_sync(kFull, acc[v][e], o);
      const int b = item / p.world, s = item - b * p.world;
      if (d.pooling == 1 && len > 0) {
        const float inv = 1.f / static_cast<float>(len);
#pragma unroll
        for (int v = 0; v < VEC; ++v)
#pragma unroll
          for (int e = 0; e < kSegVals; ++e) acc[v][e] *= inv;
      }
      if (g == 0) {
#pragma unroll
        for (int v = 0; v < VEC; ++v) {
          const int seg = l + 32 * v;
          if (seg >= segs) continue;
          const int col = seg * kSegVals;
#pragma unroll
          for (int e = 0; e < kSegVals; e += 4) {
            const float4 q = make_float4(acc[v][e], acc[v][e + 1], acc[v][e + 2], acc[v][e + 3]);
            if (d.part_col >= 0) {
              float* out = p.peer_part[s] + (static_cast<int64_t>(d.rw_idx) * p.Bl + b) * p.part_stride +
                           d.part_col + col + e;
              store4<float>(out, q);
            } else if (p.out_dtype == kBF16) {
              store4<__nv_bfloat16>(reinterpret_cast<__nv_bfloat16*>(p.peer_out[s]) +
                                        static_cast<int64_t>(b) * p.out_stride + d.out_col + col + e,
                                    q);
            } else {
              store4<float>(reinterpret_cast<float*>(p.peer_out[s]) + static_cast<int64_t>(b) * p.out_stride +
                                d.out_col + col + e,
                            q);
            }
          }
        }
      }
    }
  }

  if (p.world > 1) {
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
      const unsigned prev = atomicAdd(p.block_counter, 1u);
      if (prev == gridDim.x - 1) {
        *p.block_counter = 0u;
        *p.epoch_ctr = epoch;
        barrier_signal(p.peer_flags, p.world, p.rank, p.flag_out, epoch);
        barrier_wait(p.flags_local, p.world, p.flag_out, epoch, p.timeout_ns, p.status);
      }
    }
  }
}

// Row-wise tables: pooled row = sum of the partial rows of the table's pieces,
// in residue order (deterministic).  Runs on the requester after the forward,
// whose exit barrier guarantees that every owner's partials have landed.
template <typename TO>
__global__ void __launch_bounds__(kEmbThreads) emb_rw_reduce_kernel(EmbFwdParams p) {
  const float* part = p.peer_part[p.rank];
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t nth = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int t = 0; t < p.num_rw; ++t) {
    const RwTable rt = p.rw_tables[t];
    const int q = rt.ncols / 4;
    const int64_t total = static_cast<int64_t>(p.Bl) * q;
    for (int64_t i = tid; i < total; i += nth) {
      const int b = static_cast<int>(i / q);
      const int c = static_cast<int>(i - static_cast<int64_t>(b) * q) * 4;
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int r = 0; r < rt.rw_n; ++r)
        acc = f4_add(acc, load4<float>(part + (static_cast<int64_t>(r) * p.Bl + b) * p.part_stride + rt.part_col + c));
      TO* out = reinterpret_cast<TO*>(p.peer_out[p.rank]) + static_cast<int64_t>(b) * p.out_stride + rt.out_col + c;
      store4<TO>(out, acc);
    }
  }
}

// ============================================================================
// Backward
// ============================================================================

// Slot table of a backward pass in shared memory: compact staging index k belongs to the slot
// (shard, source) with slot_start[slot] <= k < slot_start[slot + 1].  Loops run over k with a grid
// stride (balanced however the slots differ in size) and find the slot by binary search here.
struct SlotSmem {
  int start[1025];
  long long row_base[kMaxShardsSmem];
};

__device__ __forceinline__ void load_slot_smem(const EmbBwdParams& p, SlotSmem& t) {
  const int nslot = p.num_shards * p.world;
  for (int i = threadIdx.x; i <= nslot; i += blockDim.x) t.start[i] = p.slot_start[i];
  for (int i = threadIdx.x; i < p.num_shards; i += blockDim.x) t.row_base[i] = p.shards[i].row_base;
  __syncthreads();
}

__device__ __forceinline__ int find_slot(const SlotSmem& t, int nslot, int k) {
  int lo = 0, hi = nslot;  // the largest slot with start <= k (empty slots share a start)
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (t.start[mid] <= k) lo = mid;
    else hi = mid;
  }
  return lo;
}

// 1. pooled-gradient all-to-all (pull) + occurrence counting, ranks, first-occurrence flags
__global__ void __launch_bounds__(kEmbThreads) emb_bwd_pull_count_kernel(EmbBwdParams p) {
  if (p.world > 1) {
    const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(p.epoch_ctr) + 1u;
    const bool ok =
        entry_barrier(p.flags_local, p.peer_flags, p.world, p.rank, p.flag_in, epoch, p.timeout_ns, p.status);
    if (threadIdx.x == 0) {
      if (atomicAdd(p.block_counter, 1u) == gridDim.x - 1) {  // every block has read the epoch
        *p.block_counter = 0u;
        *p.epoch_ctr = epoch;
      }
    }
    if (!ok) return;
  }
  const int tid = static_cast<int>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int nthreads = static_cast<int>(gridDim.x) * blockDim.x;
  const int esize = p.grad_dtype == kBF16 ? 2 : 4;
  for (int sh = 0; sh < p.num_shards; ++sh) {
    const ShardDesc d = p.shards[sh];
    const int chunks = d.ncols * esize / 16;  // a power of two
    const int cshift = __ffs(chunks) - 1;
    const int total = p.world * p.Bl * chunks;
    for (int i = tid; i < total; i += nthreads) {
      const int c = i & (chunks - 1);
      const int bs = i >> cshift;  // bs = b * world + s
      const int b = bs / p.world;
      const int s = bs - b * p.world;
      const char* src = reinterpret_cast<const char*>(p.peer_grad[s]) +
                        (static_cast<int64_t>(b) * p.out_stride + d.out_col) * esize + c * 16;
      char* dst = reinterpret_cast<char*>(p.grad_stage) +
                  ((static_cast<int64_t>(sh * p.world + s) * p.Bl + b) * p.grad_stage_ld) * esize + c * 16;
      *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(src);
    }
  }
  __shared__ int block_total;
  if (threadIdx.x == 0) block_total = 0;
  __syncthreads();
  // Count occurrences per row over the used staging positions only (compact index k); this
  // occurrence's rank within its row is the counter value before the add plus its position among
  // equal-row lanes.
  __shared__ SlotSmem st;
  load_slot_smem(p, st);
  const int lane = lane_id();
  const int nslot = p.num_shards * p.world;
  const int T = st.start[nslot];
  const int gw = tid >> 5, nw = nthreads >> 5;
  int local = 0;
  for (int k0 = gw * 32; k0 < T; k0 += nw * 32) {
    const int k = k0 + lane;
    long long row = -1;
    if (k < T) {
      const int slot = find_slot(st, nslot, k);
      const int id = p.stage_ids[static_cast<int64_t>(slot) * p.stage_cap + (k - st.start[slot])];
      if (id >= 0) row = st.row_base[slot / p.world] + id;
    }
    const bool valid = row >= 0;
    const unsigned vmask = __ballot_sync(kFull, valid);
    int f = 0;
    if (valid) {
      ++local;
      const unsigned peers = __match_any_sync(vmask, row);
      const int leader = __ffs(peers) - 1;
      int old = 0;
      if (lane == leader) old = atomicAdd(p.row_count + row, __popc(peers));
      old = __shfl_sync(peers, old, leader);
      const int rank = old + __popc(peers & lanemask_lt());
      p.stage_rank[k] = rank;
      f = rank == 0 ? 1 : 0;
      if (p.deterministic) atomicMin(p.det_first + row, k);  // first occurrence by position
    }
    if (k < T) p.flags[k] = f;
  }
  local = __reduce_add_sync(kFull, local);
  if (lane == 0 && local) atomicAdd(&block_total, local);
  __syncthreads();
  if (threadIdx.x == 0 && block_total) atomicAdd(p.num_unique + 1, block_total);
}

// 0. slot_start = exclusive prefix of the staged id counts per slot (one block; slots <= 1024)
__global__ void __launch_bounds__(1024) emb_slot_prefix_kernel(EmbBwdParams p) {
  __shared__ int wsum[32];
  const int nslot = p.num_shards * p.world;
  const int i = threadIdx.x, l = lane_id(), w = warp_id();
  const int c = i < nslot ? static_cast<int>(min(static_cast<int64_t>(p.stage_count[i]), p.stage_cap)) : 0;
  int x = c;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(kFull, x, o);
    if (l >= o) x += y;
  }
  if (l == 31) wsum[w] = x;
  __syncthreads();
  if (w == 0) {
    int t = l < blockDim.x / 32 ? wsum[l] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(kFull, t, o);
      if (l >= o) t += y;
    }
    wsum[l] = t;
  }
  __syncthreads();
  const int excl = (w > 0 ? wsum[w - 1] : 0) + x - c;
  if (i < nslot) p.slot_start[i] = excl;
  if (i == blockDim.x - 1) p.slot_start[nslot] = excl + c;
}

// 3. per-unique metadata (slot-major over the used staging positions)
__global__ void __launch_bounds__(kEmbThreads) emb_emit_kernel(EmbBwdParams p) {
  __shared__ SlotSmem st;
  load_slot_smem(p, st);
  const int nslot = p.num_shards * p.world;
  const int tid = static_cast<int>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int nthreads = static_cast<int>(gridDim.x) * blockDim.x;
  const int T = st.start[nslot];
  if (tid == 0) p.num_unique[0] = p.pos[T];
  for (int k = tid; k < T; k += nthreads) {
    if (!p.flags[k]) continue;
    const int slot = find_slot(st, nslot, k);
    const int64_t at = static_cast<int64_t>(slot) * p.stage_cap + (k - st.start[slot]);
    const int sh = slot / p.world;
    const int u = p.pos[k];
    const long long row = st.row_base[sh] + p.stage_ids[at];
    p.uniq_row[u] = row;
    p.uniq_shard[u] = sh;
    p.row2u[row] = u;
    if (p.deterministic) p.det_first[row] = 0x7fffffff;
    const int c = p.row_count[row];
    p.cnt_u[u] = c;
    p.first_gidx[u] = slot * p.Bl + p.stage_bag[at];
    if (c > p.light_max) {
      const int h = atomicAdd(p.num_unique + 2, 1);
      if (h < p.max_heavy) {
        p.heavy[h] = u;
        p.hcnt[h] = c;
      } else {
        report_error(p.status, kCapacityOverflow, -1);
      }
    }
  }
}

constexpr int kScanBlocks = 512;
constexpr int kScanThreads = 512;

__device__ __forceinline__ int block_reduce_sum(int v, int* sh) {
  v = __reduce_add_sync(kFull, v);
  const int w = warp_id(), l = lane_id();
  __syncthreads();
  if (l == 0) sh[w] = v;
  __syncthreads();
  int tot = 0;
  if (w == 0) {
    tot = l < blockDim.x / 32 ? sh[l] : 0;
    tot = __reduce_add_sync(kFull, tot);
    if (l == 0) sh[0] = tot;
  }
  __syncthreads();
  tot = sh[0];
  __syncthreads();
  return tot;
}

// 4. exclusive scan of cnt_u[0..U) (U read on the device) -> seg_start
__global__ void __launch_bounds__(kScanThreads) emb_seg_partial_kernel(EmbBwdParams p) {
  __shared__ int sh[32];
  const int U = p.num_unique[0];
  const int per = (U + kScanBlocks - 1) / kScanBlocks;
  const int lo = min(U, static_cast<int>(blockIdx.x) * per), hi = min(U, lo + per);
  int acc = 0;
  for (int u = lo + threadIdx.x; u < hi; u += blockDim.x) acc += p.cnt_u[u];
  acc = block_reduce_sum(acc, sh);
  if (threadIdx.x == 0) p.block_sums[blockIdx.x] = acc;
}

__global__ void __launch_bounds__(kScanThreads) emb_seg_final_kernel(EmbBwdParams p) {
  __shared__ int sh[32];
  __shared__ int wsum[32];
  const int U = p.num_unique[0];
  const int per = (U + kScanBlocks - 1) / kScanBlocks;
  const int lo = min(U, static_cast<int>(blockIdx.x) * per), hi = min(U, lo + per);
  int base = 0;
  for (int i = threadIdx.x; i < blockIdx.x; i += blockDim.x) base += p.block_sums[i];
  base = block_reduce_sum(base, sh);
  const int w = warp_id(), l = lane_id();
  for (int t0 = lo; t0 < hi; t0 += blockDim.x) {
    const int u = t0 + threadIdx.x;
    const int c = u < hi ? p.cnt_u[u] : 0;
    int x = c;  // inclusive warp scan
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(kFull, x, o);
      if (l >= o) x += y;
    }
    if (l == 31) wsum[w] = x;
    __syncthreads();
    if (w == 0) {
      int s = l < blockDim.x / 32 ? wsum[l] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(kFull, s, o);
        if (l >= o) s += y;
      }
      wsum[l] = s;
    }
    __syncthreads();
    const int warp_base = w > 0 ? wsum[w - 1] : 0;
    if (u < hi) p.seg_start[u] = base + warp_base + x - c;
    const int tile_total = wsum[blockDim.x / 32 - 1];
    __syncthreads();
    base += tile_total;
  }
  // The last block's running base ends at the grand total (blocks past U own
  // empty ranges): the sentinel seg_start[U] = T.
  if (blockIdx.x == kScanBlocks - 1 && threadIdx.x == 0) p.seg_start[U] = base;
}

// 5. occ[seg_start[u] + rank] = staged-grad row, for rows seen more than once
__global__ void __launch_bounds__(kEmbThreads) emb_fill_kernel(EmbBwdParams p) {
  __shared__ SlotSmem st;
  load_slot_smem(p, st);
  const int nslot = p.num_shards * p.world;
  const int tid = static_cast<int>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int nthreads = static_cast<int>(gridDim.x) * blockDim.x;
  const int T = st.start[nslot];
  for (int k = tid; k < T; k += nthreads) {
    const int slot = find_slot(st, nslot, k);
    const int64_t at = static_cast<int64_t>(slot) * p.stage_cap + (k - st.start[slot]);
    const int id = p.stage_ids[at];
    if (id < 0) continue;
    const int u = p.row2u[st.row_base[slot / p.world] + id];
    if (p.cnt_u[u] <= 1) continue;
    p.occ[p.seg_start[u] + p.stage_rank[k]] = slot * p.Bl + p.stage_bag[at];
  }
}

// exclusive scan of in[0..n) -> out[0..n], n = min(*n_ptr, n_max) read on the device
__global__ void __launch_bounds__(kScanThreads) dev_scan_partial_kernel(const int* in, const int* n_ptr, int n_max,
                                                                         int* block_sums) {
  __shared__ int sh[32];
  const int n = min(*n_ptr, n_max);
  const int per = (n + kScanBlocks - 1) / kScanBlocks;
  const int lo = min(n, static_cast<int>(blockIdx.x) * per), hi = min(n, lo + per);
  int acc = 0;
  for (int i = lo + threadIdx.x; i < hi; i += blockDim.x) acc += in[i];
  acc = block_reduce_sum(acc, sh);
  if (threadIdx.x == 0) block_sums[blockIdx.x] = acc;
}

__global__ void __launch_bounds__(kScanThreads) dev_scan_final_kernel(const int* in, const int* n_ptr, int n_max,
                                                                       const int* block_sums, int* out) {
  __shared__ int sh[32];
  __shared__ int wsum[32];
  const int n = min(*n_ptr, n_max);
  const int per = (n + kScanBlocks - 1) / kScanBlocks;
  const int lo = min(n, static_cast<int>(blockIdx.x) * per), hi = min(n, lo + per);
  int base = 0;
  for (int i = threadIdx.x; i < blockIdx.x; i += blockDim.x) base += block_sums[i];
  base = block_reduce_sum(base, sh);
  const int w = warp_id(), l = lane_id();
  for (int t0 = lo; t0 < hi; t0 += blockDim.x) {
    const int i = t0 + threadIdx.x;
    const int c = i < hi ? in[i] : 0;
    int x = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(kFull, x, o);
      if (l >= o) x += y;
    }
    if (l == 31) wsum[w] = x;
    __syncthreads();
    if (w == 0) {
      int t = l < blockDim.x / 32 ? wsum[l] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(kFull, t, o);
        if (l >= o) t += y;
      }
      wsum[l] = t;
    }
    __syncthreads();
    if (i < hi) out[i] = base + (w > 0 ? wsum[w - 1] : 0) + x - c;
    const int tile_total = wsum[blockDim.x / 32 - 1];
    __syncthreads();
    base += tile_total;
  }
  if (blockIdx.x == kScanBlocks - 1 && threadIdx.x == 0) out[n] = base;
}

// ---- deterministic-reduction mode -------------------------------------------
// first-occurrence flags by staging position (the counting pass flags the first by atomic order)
__global__ void __launch_bounds__(kEmbThreads) emb_det_first_kernel(EmbBwdParams p) {
  __shared__ SlotSmem st;
  load_slot_smem(p, st);
  const int nslot = p.num_shards * p.world;
  const int tid = static_cast<int>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int nthreads = static_cast<int>(gridDim.x) * blockDim.x;
  const int T = st.start[nslot];
  for (int k = tid; k < T; k += nthreads) {
    const int slot = find_slot(st, nslot, k);
    const int id = p.stage_ids[static_cast<int64_t>(slot) * p.stage_cap + (k - st.start[slot])];
    p.flags[k] = (id >= 0 && p.det_first[st.row_base[slot / p.world] + id] == k) ? 1 : 0;
  }
}

// heavy rows listed in unique-row order (the emit kernel lists them in atomic order)
__global__ void __launch_bounds__(kEmbThreads) emb_det_heavy_flags_kernel(EmbBwdParams p) {
  const int U = p.num_unique[0];
  for (int u = blockIdx.x * blockDim.x + threadIdx.x; u < U; u += gridDim.x * blockDim.x)
    p.flags[u] = p.cnt_u[u] > p.light_max ? 1 : 0;
}

__global__ void __launch_bounds__(kEmbThreads) emb_det_heavy_place_kernel(EmbBwdParams p) {
  const int U = p.num_unique[0];
  for (int u = blockIdx.x * blockDim.x + threadIdx.x; u < U; u += gridDim.x * blockDim.x) {
    if (!p.flags[u]) continue;
    const int h = p.pos[u];
    if (h < p.max_heavy) {
      p.heavy[h] = u;
      p.hcnt[h] = p.cnt_u[u];
    }
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) p.num_unique[2] = p.pos[U];
}

// sort keys: the occurrence's unique row (invalid / unused positions sort last), value: its staged-grad row
__global__ void __launch_bounds__(kEmbThreads) emb_det_keys_kernel(EmbBwdParams p, int n) {
  __shared__ SlotSmem st;
  load_slot_smem(p, st);
  const int nslot = p.num_shards * p.world;
  const int tid = static_cast<int>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int nthreads = static_cast<int>(gridDim.x) * blockDim.x;
  const int T = st.start[nslot];
  for (int k = tid; k < n; k += nthreads) {
    if (k >= T) {
      p.det_keys[k] = 0x7fffffff;
      p.det_vals[k] = 0;
      continue;
    }
    const int slot = find_slot(st, nslot, k);
    const int64_t at = static_cast<int64_t>(slot) * p.stage_cap + (k - st.start[slot]);
    const int id = p.stage_ids[at];
    p.det_keys[k] = id < 0 ? 0x7fffffff : p.row2u[st.row_base[slot / p.world] + id];
    p.det_vals[k] = slot * p.Bl + p.stage_bag[at];
  }
}

// 6. light rows: a group of G lanes per unique row, NV float4 per lane.  (A variant that loaded the
// next row's metadata one iteration ahead and bulk-prefetched its weights / optimizer state into
// L2 measured 0-5% slower on the DLRM benchmark.)
template <typename TW, typename TG, int NV, int MINB>
__global__ void __launch_bounds__(kEmbThreads, MINB) emb_apply_light_kernel(EmbBwdParams p, int G) {
  __shared__ ShardDesc sd[kMaxShardsSmem];
  for (int i = threadIdx.x; i < p.num_shards; i += blockDim.x) sd[i] = p.shards[i];
  __syncthreads();
  SparseOptParams o = p.opt;
  resolve_sparse_step(o);
  const int U = p.num_unique[0];
  const int lane = lane_id();
  const int g = lane / G, gl = lane - (lane / G) * G;
  const int leader = g * G;
  const int gpw = 32 / G;
  const int col = gl * 4 * NV;
  const int64_t gwarp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  for (int64_t base = gwarp * gpw; base < U; base += nwarps * gpw) {
    const int u = static_cast<int>(base) + g;
    const bool inr = u < U;
    // independent per-row metadata, issued together
    const int c = inr ? p.cnt_u[u] : 0;
    const long long row = inr ? p.uniq_row[u] : 0;
    const int sh = inr ? p.uniq_shard[u] : 0;
    const int ss = inr ? p.seg_start[u] : 0;
    const int g1 = inr ? p.first_gidx[u] : 0;
    const bool mine = inr && c <= p.light_max && c > 0;
    const ShardDesc& d = sd[sh];
    const bool act = mine && col < d.ncols;
    const int64_t eoff = d.weight_off + (row - d.row_base) * d.ncols + col;
    TW* w = reinterpret_cast<TW*>(p.weights) + eoff;
    float4 wv[NV], acc[NV];
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      wv[v] = act ? load4<TW>(w + 4 * v) : make_float4(0.f, 0.f, 0.f, 0.f);
      acc[v] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    const bool mean = d.pooling == 1;
    int cmax = mine ? c : 0;
#pragma unroll
    for (int o2 = 16; o2 > 0; o2 >>= 1) cmax = max(cmax, __shfl_xor_sync(kFull, cmax, o2));
    for (int k0 = 0; k0 < cmax; k0 += G) {
      // lane gl of the group loads occurrence k0 + gl of its row
      int gidx = 0;
      float sc = 1.f;
      if (mine && k0 + gl < c) {
        gidx = c == 1 ? g1 : p.occ[ss + k0 + gl];
        if (mean) sc = 1.f / static_cast<float>(max(1, p.stage_len[gidx]));
      }
      const int n = min(G, cmax - k0);
      int t = 0;
      for (; t + 2 <= n; t += 2) {
        float4 r[2][NV];
        float s2[2];
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          const int gi = __shfl_sync(kFull, gidx, leader + t + q);
          s2[q] = __shfl_sync(kFull, sc, leader + t + q);
          const bool ok = act && k0 + t + q < c;
          const TG* src =
              reinterpret_cast<const TG*>(p.grad_stage) + static_cast<int64_t>(gi) * p.grad_stage_ld + col;
#pragma unroll
          for (int v = 0; v < NV; ++v) r[q][v] = ok ? load4<TG>(src + 4 * v) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int q = 0; q < 2; ++q)
#pragma unroll
          for (int v = 0; v < NV; ++v) acc[v] = f4_add(acc[v], f4_scale(r[q][v], s2[q]));
      }
      for (; t < n; ++t) {
        const int gi = __shfl_sync(kFull, gidx, leader + t);
        const float s = __shfl_sync(kFull, sc, leader + t);
        if (act && k0 + t < c) {
          const TG* src =
              reinterpret_cast<const TG*>(p.grad_stage) + static_cast<int64_t>(gi) * p.grad_stage_ld + col;
#pragma unroll
          for (int v = 0; v < NV; ++v) acc[v] = f4_add(acc[v], f4_scale(load4<TG>(src + 4 * v), s));
        }
      }
    }
    apply_update<TW, NV>(o, w, eoff, row, mine, act, d.ncols, acc, wv, c, G, leader);
    if (mine && gl == 0) {
      p.row_count[row] = 0;
      mark_dirty(p.dirty, row);
    }
  }
}

// 7a. exclusive scan of heavy-row counts hcnt[0..H) -> heavy_start (H on device)
__global__ void __launch_bounds__(kScanThreads) emb_heavy_partial_kernel(EmbBwdParams p) {
  __shared__ int sh[32];
  const int H = min(p.num_unique[2], p.max_heavy);
  const int per = (H + kScanBlocks - 1) / kScanBlocks;
  const int lo = min(H, static_cast<int>(blockIdx.x) * per), hi = min(H, lo + per);
  int acc = 0;
  for (int h = lo + threadIdx.x; h < hi; h += blockDim.x) acc += p.hcnt[h];
  acc = block_reduce_sum(acc, sh);
  if (threadIdx.x == 0) p.block_sums[blockIdx.x] = acc;
}

__global__ void __launch_bounds__(kScanThreads) emb_heavy_final_kernel(EmbBwdParams p) {
  __shared__ int sh[32];
  __shared__ int wsum[32];
  const int H = min(p.num_unique[2], p.max_heavy);
  const int per = (H + kScanBlocks - 1) / kScanBlocks;
  const int lo = min(H, static_cast<int>(blockIdx.x) * per), hi = min(H, lo + per);
  int base = 0;
  for (int i = threadIdx.x; i < blockIdx.x; i += blockDim.x) base += p.block_sums[i];
  base = block_reduce_sum(base, sh);
  const int w = warp_id(), l = lane_id();
  for (int t0 = lo; t0 < hi; t0 += blockDim.x) {
    const int h = t0 + threadIdx.x;
    const int c = h < hi ? p.hcnt[h] : 0;
    int x = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(kFull, x, o);
      if (l >= o) x += y;
    }
    if (l == 31) wsum[w] = x;
    __syncthreads();
    if (w == 0) {
      int s2 = l < blockDim.x / 32 ? wsum[l] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(kFull, s2, o);
        if (l >= o) s2 += y;
      }
      wsum[l] = s2;
    }
    __syncthreads();
    if (h < hi) p.heavy_start[h] = base + (w > 0 ? wsum[w - 1] : 0) + x - c;
    const int tile_total = wsum[blockDim.x / 32 - 1];
    __syncthreads();
    base += tile_total;
  }
  if (blockIdx.x == kScanBlocks - 1 && threadIdx.x == 0) p.heavy_start[H] = base;
}

// 7b. heavy occurrences in fixed chunks of kHeavyChunk across warps: one fp32
// partial row per (heavy row, chunk) segment, stored (no atomics).
constexpr int kHeavyChunk = 256;
template <typename TG, int NV>
__global__ void __launch_bounds__(kEmbThreads) emb_heavy_accumulate_kernel(EmbBwdParams p) {
  const int H = min(p.num_unique[2], p.max_heavy);
  if (H == 0) return;
  const int total = p.heavy_start[H];
  const int lane = lane_id();
  const int col = lane * 4 * NV;
  const int acc_ld = 32 * 4 * NV;
  const int64_t gwarp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  const int nchunks = (total + kHeavyChunk - 1) / kHeavyChunk;
  for (int64_t c = gwarp; c < nchunks; c += nwarps) {
    const int cb = static_cast<int>(c) * kHeavyChunk;
    const int ce = min(total, cb + kHeavyChunk);
    int lo = 0, hi = H;  // largest h with heavy_start[h] <= cb
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (p.heavy_start[mid] <= cb) lo = mid; else hi = mid;
    }
    for (int h = lo; h < H; ++h) {
      const int hs = p.heavy_start[h];
      if (hs >= ce) break;
      const int he = p.heavy_start[h + 1];
      const int a = max(hs, cb), e = min(he, ce);
      const int u = p.heavy[h];
      const ShardDesc d = p.shards[p.uniq_shard[u]];
      const bool act = col < d.ncols;
      const bool mean = d.pooling == 1;
      const int ss = p.seg_start[u] - hs;  // occ index = ss + flat position
      float4 acc[NV];
#pragma unroll
      for (int v = 0; v < NV; ++v) acc[v] = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int q0 = a; q0 < e; q0 += 32) {
        int gidx = 0;
        float sc = 1.f;
        if (q0 + lane < e) {
          gidx = p.occ[ss + q0 + lane];
          if (mean) sc = 1.f / static_cast<float>(max(1, p.stage_len[gidx]));
        }
        const int n = min(32, e - q0);
        int t = 0;
        for (; t + 4 <= n; t += 4) {
          float4 r[4][NV];
          float s4[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int gi = __shfl_sync(kFull, gidx, t + q);
            s4[q] = __shfl_sync(kFull, sc, t + q);
            const TG* src =
                reinterpret_cast<const TG*>(p.grad_stage) + static_cast<int64_t>(gi) * p.grad_stage_ld + col;
#pragma unroll
            for (int v = 0; v < NV; ++v) r[q][v] = act ? load4<TG>(src + 4 * v) : make_float4(0.f, 0.f, 0.f, 0.f);
          }
#pragma unroll
          for (int q = 0; q < 4; ++q)
#pragma unroll
            for (int v = 0; v < NV; ++v) acc[v] = f4_add(acc[v], f4_scale(r[q][v], s4[q]));
        }
        for (; t < n; ++t) {
          const int gi = __shfl_sync(kFull, gidx, t);
          const float s1 = __shfl_sync(kFull, sc, t);
          if (act) {
            const TG* src =
                reinterpret_cast<const TG*>(p.grad_stage) + static_cast<int64_t>(gi) * p.grad_stage_ld + col;
#pragma unroll
            for (int v = 0; v < NV; ++v) acc[v] = f4_add(acc[v], f4_scale(load4<TG>(src + 4 * v), s1));
          }
        }
      }
      if (act) {
        // segment (row h, chunk c) has its own partial slot h + c (injective: rows occupy disjoint,
        // increasing position ranges), so the apply sums the partials in chunk order: deterministic
        float* dst = p.heavy_acc + (static_cast<int64_t>(h) + c) * acc_ld + col;
#pragma unroll
        for (int v = 0; v < NV; ++v) reinterpret_cast<float4*>(dst)[v] = acc[v];
      }
    }
  }
}

// 7c. optimizer on the heavy rows (one warp per row), accumulators re-zeroed.
template <typename TW, int NV>
__global__ void __launch_bounds__(kEmbThreads) emb_heavy_apply_kernel(EmbBwdParams p) {
  SparseOptParams o = p.opt;
  resolve_sparse_step(o);
  const int H = min(p.num_unique[2], p.max_heavy);
  const int lane = lane_id();
  const int col = lane * 4 * NV;
  const int acc_ld = 32 * 4 * NV;
  const int64_t gwarp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  for (int64_t h = gwarp; h < H; h += nwarps) {
    const int u = p.heavy[h];
    const long long row = p.uniq_row[u];
    const ShardDesc d = p.shards[p.uniq_shard[u]];
    const bool act = col < d.ncols;
    float4 acc[NV], wv[NV];
    const int64_t eoff = d.weight_off + (row - d.row_base) * d.ncols + col;
    TW* wp = reinterpret_cast<TW*>(p.weights) + eoff;
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      acc[v] = make_float4(0.f, 0.f, 0.f, 0.f);
      wv[v] = act ? load4<TW>(wp + 4 * v) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    // partials of the row's chunks, in chunk order (slot h + c)
    const int c0 = p.heavy_start[h] / kHeavyChunk, c1 = (p.heavy_start[h + 1] - 1) / kHeavyChunk;
    for (int c = c0; act && c <= c1; ++c) {
      const float4* src = reinterpret_cast<const float4*>(p.heavy_acc + (h + c) * acc_ld + col);
#pragma unroll
      for (int v = 0; v < NV; ++v) acc[v] = f4_add(acc[v], src[v]);
    }
    apply_update<TW, NV>(o, wp, eoff, row, true, act, d.ncols, acc, wv, p.cnt_u[u], 32, 0);
    if (lane == 0) {
      p.row_count[row] = 0;
      mark_dirty(p.dirty, row);
    }
  }
}

// 4 resident blocks per SM (64 registers, a few spilled) measured ~1% faster than 3 (80 registers).
template <typename TW, int VEC>
void fwd_dispatch(const EmbFwdParams& p, int grid, cudaStream_t s) {
  // 4 resident blocks per SM (64 registers; the 2-vector variant spills ~100 bytes), or 3 (85 registers,
  // no spills): 3 measured 9 % slower per DLRM step (2.40 against 2.20 ms), the id -> row chains need warps
  if (p.fwd_minb == 3) emb_fwd_kernel<TW, VEC, 3><<<grid, kEmbThreads, 0, s>>>(p);
  else emb_fwd_kernel<TW, VEC, 4><<<grid, kEmbThreads, 0, s>>>(p);
  count_launch();
}

template <typename TW, typename TG>
void bwd_apply(const EmbBwdParams& p, int ncols_max, int grid, cudaStream_t s) {
  // light rows: 2 float4 (8 columns) per lane -> ncols_max / 8 lanes per row
  const int G = std::max(1, ncols_max / 8);
  // 4 blocks per SM: ~10% faster than 3 on the DLRM benchmark despite a few spilled registers
  // (loading the row-wise state together with the weights, at 3 or 4 blocks per SM, measured 2-3 %
  // slower on the DLRM benchmark)
  emb_apply_light_kernel<TW, TG, 2, 4><<<grid, kEmbThreads, 0, s>>>(p, G);
  emb_heavy_partial_kernel<<<kScanBlocks, kScanThreads, 0, s>>>(p);
  emb_heavy_final_kernel<<<kScanBlocks, kScanThreads, 0, s>>>(p);
  if (ncols_max > 128) {
    emb_heavy_accumulate_kernel<TG, 2><<<grid, kEmbThreads, 0, s>>>(p);
    emb_heavy_apply_kernel<TW, 2><<<grid, kEmbThreads, 0, s>>>(p);
  } else {
    emb_heavy_accumulate_kernel<TG, 1><<<grid, kEmbThreads, 0, s>>>(p);
    emb_heavy_apply_kernel<TW, 1><<<grid, kEmbThreads, 0, s>>>(p);
  }
  count_launch(5);
}

template <typename TW>
void bwd_apply_g(const EmbBwdParams& p, int ncols_max, int grid, cudaStream_t s) {
  if (p.grad_dtype == kBF16) bwd_apply<TW, __nv_bfloat16>(p, ncols_max, grid, s);
  else bwd_apply<TW, float>(p, ncols_max, grid, s);
}

template <typename TW>
void fwd_bulk_launch(const EmbFwdParams& p, cudaStream_t s) {
  int dev = 0, sms = 0;
  FLARE_CUDA_CHECK(cudaGetDevice(&dev));
  FLARE_CUDA_CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  auto k1 = emb_fwd_bulk_kernel<TW, 1>;
  auto k2 = emb_fwd_bulk_kernel<TW, 2>;
  auto k = p.vec == 2 ? k2 : k1;
  FLARE_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kBulkSmem)));
  k<<<sms, kBulkThreads, kBulkSmem, s>>>(p);
  count_launch();
}

}  // namespace

void emb_forward(const EmbFwdParams& p, int grid, cudaStream_t s) {
  FLARE_CHECK(grid > 0, "grid must be positive");
  FLARE_CHECK(p.num_shards <= kMaxShardsSmem, "too many local shards");
  FLARE_CHECK(static_cast<int64_t>(p.world) * p.Bl + 2ll * grid * (kEmbThreads / 32) * 32 < (1ll << 31),
              "too many (source, sample) bags for 32-bit work indices");
  FLARE_CHECK(p.vec == 1 || p.vec == 2, "vec must be 1 or 2");
  if (p.fetch_offs != nullptr) {
    FLARE_CHECK(p.world > 1 && !p.bulk, "the id prefetch is for the multi-GPU register-gather forward");
    emb_fetch_kernel<<<grid, kEmbThreads, 0, s>>>(p);
    FLARE_CUDA_CHECK(cudaGetLastError());
    count_launch();
  }
  if (p.bulk) {
    // every shard's rows are 16-byte aligned (checked by the caller): TMA bulk-gather forward
    if (p.w_dtype == kF32) fwd_bulk_launch<float>(p, s);
    else if (p.w_dtype == kF16) fwd_bulk_launch<__half>(p, s);
    else fwd_bulk_launch<__nv_bfloat16>(p, s);
  } else if (p.w_dtype == kF32) {
    if (p.vec == 1) fwd_dispatch<float, 1>(p, grid, s); else fwd_dispatch<float, 2>(p, grid, s);
  } else if (p.w_dtype == kF16) {
    if (p.vec == 1) fwd_dispatch<__half, 1>(p, grid, s); else fwd_dispatch<__half, 2>(p, grid, s);
  } else {
    if (p.vec == 1) fwd_dispatch<__nv_bfloat16, 1>(p, grid, s); else fwd_dispatch<__nv_bfloat16, 2>(p, grid, s);
  }
  FLARE_CUDA_CHECK(cudaGetLastError());
  if (p.num_rw > 0) {
    FLARE_CHECK(p.peer_part != nullptr && p.rw_tables != nullptr, "row-wise tables need the partial buffers");
    if (p.out_dtype == kBF16) emb_rw_reduce_kernel<__nv_bfloat16><<<grid, kEmbThreads, 0, s>>>(p);
    else emb_rw_reduce_kernel<float><<<grid, kEmbThreads, 0, s>>>(p);
    FLARE_CUDA_CHECK(cudaGetLastError());
    count_launch();
  }
}

// One block row per staging slot; blocks of a row stride over its occurrences.  Row `micro` of the
// prefix is read, row `micro + 1` written (by block 0), so no block reads what another writes.
__global__ void emb_window_append_kernel(EmbWindowParams p) {
  const int slot = blockIdx.y;
  const int c = static_cast<int>(min(static_cast<int64_t>(max(p.count[slot], 0)), p.stage_cap));
  const int base = p.micro == 0 ? 0 : p.wprefix[static_cast<int64_t>(p.micro) * p.nslot + slot];
  const int64_t wcap = p.stage_cap * p.micro_steps;
  const int* src_ids = p.ids + static_cast<int64_t>(slot) * p.stage_cap;
  const int* src_bag = p.bag + static_cast<int64_t>(slot) * p.stage_cap;
  int* dst_ids = p.wids + static_cast<int64_t>(slot) * wcap + base;
  int* dst_bag = p.wbag + static_cast<int64_t>(slot) * wcap + base;
  const int shift = p.micro * p.Bl;
  const int stride = gridDim.x * blockDim.x;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < c; i += stride) {
    dst_ids[i] = __ldcs(src_ids + i);
    dst_bag[i] = __ldcs(src_bag + i) + shift;
  }
  const int* src_len = p.len + static_cast<int64_t>(slot) * p.Bl;
  int* dst_len = p.wlen + static_cast<int64_t>(slot) * p.micro_steps * p.Bl + shift;
  for (int b = blockIdx.x * blockDim.x + threadIdx.x; b < p.Bl; b += stride) dst_len[b] = src_len[b];
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    if (p.micro == 0) p.wprefix[slot] = 0;
    p.wprefix[static_cast<int64_t>(p.micro + 1) * p.nslot + slot] = base + c;
  }
}

void emb_window_append(const EmbWindowParams& p, cudaStream_t s) {
  FLARE_CHECK(p.nslot > 0 && p.nslot < 65536, "window append: slot count out of range");
  FLARE_CHECK(p.micro >= 0 && p.micro < p.micro_steps, "window append: micro-step outside the window");
  FLARE_CHECK(p.stage_cap * p.micro_steps < (1ll << 31), "window staging exceeds 32-bit positions");
  FLARE_CHECK(static_cast<int64_t>(p.micro_steps) * p.Bl < (1ll << 31), "window samples exceed 32 bits");
  constexpr int kThreads = 256;
  const int64_t per_slot = std::max<int64_t>(p.stage_cap, p.Bl);
  const int bx = static_cast<int>(std::min<int64_t>((per_slot + kThreads * 4 - 1) / (kThreads * 4), 32));
  emb_window_append_kernel<<<dim3(std::max(bx, 1), p.nslot), kThreads, 0, s>>>(p);
  FLARE_CUDA_CHECK(cudaGetLastError());
  count_launch();
}

size_t emb_det_temp_bytes(int64_t max_occ) {
  size_t bytes = 0;
  FLARE_CUDA_CHECK(cub::DeviceRadixSort::SortPairs(nullptr, bytes, static_cast<const int*>(nullptr),
                                                   static_cast<int*>(nullptr), static_cast<const int*>(nullptr),
                                                   static_cast<int*>(nullptr), static_cast<int>(max_occ), 0, 31));
  return bytes;
}

void emb_backward(const EmbBwdParams& p, int ncols_max, int grid, cudaStream_t s) {
  FLARE_CHECK(ncols_max >= 16 && ncols_max <= 256 && (ncols_max & (ncols_max - 1)) == 0,
              "the backward needs a power-of-two widest shard in [16, 256] columns");
  FLARE_CHECK(p.num_shards <= kMaxShardsSmem, "too many local shards");
  const int64_t N = static_cast<int64_t>(p.num_shards) * p.world * p.stage_cap;
  FLARE_CHECK(N < (1ll << 31) - 1, "staging space exceeds 2^31 occurrences");
  FLARE_CHECK(p.num_shards * p.world <= 1024, "at most 1024 (shard, source) slots");
  FLARE_CHECK(static_cast<int64_t>(p.world) * p.Bl * 64 < (1ll << 31), "too many pooled-gradient chunks");
  FLARE_CUDA_CHECK(cudaMemsetAsync(p.num_unique, 0, (p.hash_mode ? 8 : 4) * sizeof(int), s));
  if (p.hash_mode && !p.deterministic) {
    emb_backward_hash(p, ncols_max, grid, s);
    return;
  }
  FLARE_CHECK(p.row_count && p.row2u && p.pos && p.uniq_row && p.cnt_u && p.heavy && p.heavy_acc,
              "the sorted backward needs its per-row scratch buffers");
  emb_slot_prefix_kernel<<<1, 1024, 0, s>>>(p);
  emb_bwd_pull_count_kernel<<<grid, kEmbThreads, 0, s>>>(p);
  if (p.deterministic) {
    FLARE_CHECK(p.det_first != nullptr, "deterministic mode needs the per-row first-position array");
    emb_det_first_kernel<<<grid, kEmbThreads, 0, s>>>(p);
    count_launch();
  }
  const int nslot = p.num_shards * p.world;
  dev_scan_partial_kernel<<<kScanBlocks, kScanThreads, 0, s>>>(p.flags, p.slot_start + nslot,
                                                               static_cast<int>(N), p.block_sums);
  dev_scan_final_kernel<<<kScanBlocks, kScanThreads, 0, s>>>(p.flags, p.slot_start + nslot, static_cast<int>(N),
                                                             p.block_sums, p.pos);
  count_launch(4);
  emb_emit_kernel<<<grid, kEmbThreads, 0, s>>>(p);
  emb_seg_partial_kernel<<<kScanBlocks, kScanThreads, 0, s>>>(p);
  emb_seg_final_kernel<<<kScanBlocks, kScanThreads, 0, s>>>(p);
  count_launch(3);
  if (!p.deterministic) {
    emb_fill_kernel<<<grid, kEmbThreads, 0, s>>>(p);
    count_launch();
  } else {
    // heavy rows in unique-row order; occurrences grouped per unique row by a stable radix sort, so
    // each row adds its gradients in staging order whatever order the counting atomics ran in
    FLARE_CHECK(p.det_keys && p.det_vals && p.det_temp, "deterministic mode needs its sort buffers");
    const int n = static_cast<int>(N);
    emb_det_heavy_flags_kernel<<<grid, kEmbThreads, 0, s>>>(p);
    dev_scan_partial_kernel<<<kScanBlocks, kScanThreads, 0, s>>>(p.flags, p.num_unique, n, p.block_sums);
    dev_scan_final_kernel<<<kScanBlocks, kScanThreads, 0, s>>>(p.flags, p.num_unique, n, p.block_sums, p.pos);
    emb_det_heavy_place_kernel<<<grid, kEmbThreads, 0, s>>>(p);
    emb_det_keys_kernel<<<grid, kEmbThreads, 0, s>>>(p, n);
    size_t bytes = p.det_temp_bytes;
    FLARE_CUDA_CHECK(cub::DeviceRadixSort::SortPairs(p.det_temp, bytes, p.det_keys, p.det_keys + n, p.det_vals,
                                                     p.occ, n, 0, 31, s));
    count_launch(5);
  }
  if (p.w_dtype == kF32) bwd_apply_g<float>(p, ncols_max, grid, s);
  else if (p.w_dtype == kF16) bwd_apply_g<__half>(p, ncols_max, grid, s);
  else bwd_apply_g<__nv_bfloat16>(p, ncols_max, grid, s);
  FLARE_CUDA_CHECK(cudaGetLastError());
}

}  // namespace flare
