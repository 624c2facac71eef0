// Dynamic (hash-keyed, insert-on-first-sight) embedding tables (sm_100a).
//
// A dynamic table accepts any non-negative int32 key.  Its C rows live in HBM
// slots; a device open-addressing hash map (H buckets, power of two, linear
// probing) maps key -> slot.  Before every forward, three kernels run on the
// table owner:
//   dyn_insert : for every key occurrence of the step (every rank's batch,
//                read from the peers' exchange buffers): find its bucket, or
//                claim an empty one (CAS EMPTY -> key, exactly one winner per
//                new key) and queue it; found keys stamp their slot with the
//                step; the occurrence's bucket goes into the requester's remap
//                buffer (P2P store);
//   dyn_fill   : each new key takes a victim slot by a CLOCK sweep (a slot not
//                used this step, won by CAS on its stamp); the victim's key
//                becomes a tombstone; the row is initialised uniform(-s, s)
//                from a counter-based hash of (seed, key, column) and its
//                optimizer state zeroed;
//   dyn_remap  : every occurrence's bucket in the remap buffers becomes the
//                bucket's slot; the fused forward then reads slots from there.
// Lookups probe past tombstones; inserts reuse the first tombstone of the
// key's chain; a rebuild (host-triggered) clears them.  Every loop is bounded.  This is the lookup_or_insert behaviour of the reference's
// external embedding store (src/flare/runtime/fluxway/workers/
// dynamic_embedding.py:134-260: auto-insert with uniform(-0.01, 0.01) init and
// an LFU score); eviction here is CLOCK (least-recently-used order).
#include "dynamic_emb.cuh"

#include <algorithm>

namespace flare {

namespace {

constexpr int kEmpty = -1;
constexpr int kTomb = -2;

__device__ __forceinline__ uint32_t hash_key(int key) {
  uint32_t x = static_cast<uint32_t>(key);
  x ^= x >> 16;
  x *= 0x7feb352du;
  x ^= x >> 15;
  x *= 0x846ca68bu;
  x ^= x >> 16;
  return x;
}

// SplitMix64 finaliser (Steele, Lea, Flood 2014) of (seed, key, column) -> uniform [0, 1)
__device__ __forceinline__ float uniform01(uint64_t seed, int key, int col) {
  uint64_t z = seed + 0x9e3779b97f4a7c15ull * (static_cast<uint64_t>(static_cast<uint32_t>(key)) * 4096ull + col + 1);
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  z ^= z >> 31;
  return static_cast<float>(z >> 40) * (1.0f / 16777216.0f);
}

__device__ __forceinline__ bool barrier_in(const DynParams& p, uint32_t epoch) {
  __shared__ int ok_sh;
  if (threadIdx.x == 0) {
    ok_sh = 1;
    if (blockIdx.x == 0) {
      fence_sys();
      for (int s = 0; s < p.world; ++s) st_release_sys(p.peer_flags[s] + p.flag_in + p.rank, epoch);
    }
    for (int s = 0; s < p.world && ok_sh; ++s)
      ok_sh = wait_flag_geq(p.flags_local + p.flag_in + s, epoch, p.timeout_ns, p.status, s) ? 1 : 0;
  }
  __syncthreads();
  return ok_sh != 0;
}

__global__ void dyn_insert_kernel(DynParams p) {
  const uint32_t epoch = p.world > 1 ? *reinterpret_cast<volatile uint32_t*>(p.epoch_ctr) + 1u : 0u;
  if (p.world > 1) {
    const bool ok = barrier_in(p, epoch);
    if (threadIdx.x == 0 && atomicAdd(p.block_counter, 1u) == gridDim.x - 1) {
      *p.block_counter = 0u;
      *p.epoch_ctr = epoch;
    }
    if (!ok) return;
  }
  const int step = *p.step_ptr;
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t nth = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int k = 0; k < p.num_tables; ++k) {
    const DynTable& t = p.tables[k];
    const uint32_t mask = static_cast<uint32_t>(t.H - 1);
    for (int s = 0; s < p.world; ++s) {
      const int* offs = p.peer_offsets[s];
      const int* vals = p.peer_values[s];
      int* remap = p.peer_remap[s];
      const int beg = offs[t.feature * p.Bl], end = offs[(t.feature + 1) * p.Bl];
      for (int64_t i = beg + tid; i < end; i += nth) {
        const int key = vals[i];
        int bucket = -1;
        if (key >= 0) {
          // Probe from the key's home bucket until the key or an empty bucket; a new key takes the
          // first tombstone on its chain (else the empty bucket) by CAS.  Losing a CAS to another key
          // restarts the probe; during this kernel buckets only change empty/tombstone -> key, so the
          // restart converges.  Bounded: at most 4 passes over the table.
          const uint32_t home = hash_key(key) & mask;
          uint32_t h = home;
          int probe = 0, tomb = -1;
          for (int it = 0; it < 4 * t.H && bucket < 0; ++it) {
            const int cur = t.keys[h];
            if (cur == key) {
              bucket = static_cast<int>(h);
              const int slot = t.slot_of[h];
              if (slot >= 0) t.stamp[slot] = step;
              break;
            }
            const bool end = cur == kEmpty || probe == t.H - 1;
            if (cur == kTomb && tomb < 0) tomb = static_cast<int>(h);
            if (!end) {
              ++probe;
              h = (h + 1) & mask;
              continue;
            }
            // the key is not on its chain: claim the first tombstone, else this empty bucket
            int target = tomb, expect = kTomb;
            if (target < 0 && cur == kEmpty) {
              target = static_cast<int>(h);
              expect = kEmpty;
            }
            if (target < 0) break;  // full chain without room
            const int got = atomicCAS(t.keys + target, expect, key);
            if (got == expect) {  // inserted: this thread owns the new key
              if (expect == kTomb) atomicSub(t.num_tomb, 1);
              const int q = atomicAdd(t.num_new, 1);
              if (q < t.new_cap) t.new_buckets[q] = target;
              else report_error(p.status, kCapacityOverflow, 4000 + k);
              bucket = target;
            } else if (got == key) {  // another occurrence inserted it first
              bucket = target;
            } else {  // another key took the bucket: probe again from home
              h = home;
              probe = 0;
              tomb = -1;
            }
          }
          if (bucket < 0) report_error(p.status, kCapacityOverflow, 4100 + k);
        } else {
          report_error(p.status, kIndexOutOfRange, 4200 + k);
        }
        remap[i] = bucket;
      }
    }
  }
}

// One warp per new key: victim slot by CLOCK, tombstone the victim's key, initialise the row.
__global__ void dyn_fill_kernel(DynParams p) {
  const int lane = lane_id();
  const int step = *p.step_ptr;
  const int64_t gw = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nw = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  for (int k = 0; k < p.num_tables; ++k) {
    const DynTable& t = p.tables[k];
    const int nnew = min(*t.num_new, t.new_cap);
    for (int64_t i = gw; i < nnew; i += nw) {
      const int h = t.new_buckets[i];
      int slot = -1;
      if (lane == 0) {
        for (int64_t tries = 0; tries < 2 * t.C + 64; ++tries) {
          const int c = static_cast<int>(atomicAdd(t.hand, 1u) % static_cast<unsigned>(t.C));
          const int st = t.stamp[c];
          if (st < step && atomicCAS(t.stamp + c, st, step) == st) {
            slot = c;
            break;
          }
        }
        if (slot < 0) report_error(p.status, kCapacityOverflow, 4300 + k);
      }
      slot = __shfl_sync(0xffffffffu, slot, 0);
      if (slot < 0) continue;
      const int key = t.keys[h];
      float* row = t.weights + static_cast<int64_t>(slot) * t.ncols;
      for (int c = lane; c < t.ncols; c += 32)
        row[c] = (2.f * uniform01(t.seed, key, t.col_begin + c) - 1.f) * t.init_scale;
      if (t.state_m)
        for (int c = lane; c < t.ncols; c += 32) t.state_m[static_cast<int64_t>(slot) * t.ncols + c] = 0.f;
      if (t.state_v)
        for (int c = lane; c < t.ncols; c += 32) t.state_v[static_cast<int64_t>(slot) * t.ncols + c] = 0.f;
      if (lane == 0) {
        if (t.state_row) t.state_row[slot] = 0.f;
        if (t.score) t.score[slot] = 0.f;
        const int old = t.bucket_of[slot];
        if (old >= 0) {  // evict the previous key: tombstone keeps probe chains intact
          t.keys[old] = kTomb;
          t.slot_of[old] = -1;
          atomicAdd(t.num_tomb, 1);
        }
        t.bucket_of[slot] = h;
        t.slot_of[h] = slot;
      }
    }
  }
}

// bucket -> slot in every requester's remap buffer (P2P stores); resets the new-key counters.
__global__ void dyn_remap_kernel(DynParams p) {
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t nth = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int k = 0; k < p.num_tables; ++k) {
    const DynTable& t = p.tables[k];
    for (int s = 0; s < p.world; ++s) {
      const int* offs = p.peer_offsets[s];
      int* remap = p.peer_remap[s];
      const int beg = offs[t.feature * p.Bl], end = offs[(t.feature + 1) * p.Bl];
      for (int64_t i = beg + tid; i < end; i += nth) {
        const int b = remap[i];
        remap[i] = b >= 0 ? t.slot_of[b] : -1;
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    if (atomicAdd(p.block_counter2, 1u) == gridDim.x - 1) {
      *p.block_counter2 = 0u;
      for (int k = 0; k < p.num_tables; ++k) *p.tables[k].num_new = 0;
    }
  }
}

__global__ void dyn_rebuild_kernel(int* keys, int* slot_of, int* bucket_of, int H, const int* live_keys,
                                   const int* live_slots, int n) {
  const uint32_t mask = static_cast<uint32_t>(H - 1);
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const int key = live_keys[i];
    uint32_t h = hash_key(key) & mask;
    for (int probe = 0; probe < H; ++probe, h = (h + 1) & mask) {
      if (atomicCAS(keys + h, kEmpty, key) == kEmpty) {
        slot_of[h] = live_slots[i];
        bucket_of[live_slots[i]] = static_cast<int>(h);
        break;
      }
    }
  }
}

}  // namespace

void dyn_rebuild(int* keys, int* slot_of, int* bucket_of, int H, const int* live_keys, const int* live_slots, int n,
                 cudaStream_t s) {
  if (n <= 0) return;
  dyn_rebuild_kernel<<<std::min((n + 255) / 256, 148 * 8), 256, 0, s>>>(keys, slot_of, bucket_of, H, live_keys,
                                                                        live_slots, n);
  FLARE_CUDA_CHECK(cudaGetLastError());
  count_launch();
}

void dyn_prepare(const DynParams& p, int grid, cudaStream_t s) {
  FLARE_CHECK(p.num_tables >= 0 && p.num_tables <= kMaxDynTables, "dynamic table count out of range");
  for (int k = 0; k < p.num_tables; ++k)
    FLARE_CHECK((p.tables[k].H & (p.tables[k].H - 1)) == 0 && p.tables[k].H >= 2 * p.tables[k].C,
                "hash buckets must be a power of two >= 2 x capacity");
  dyn_insert_kernel<<<grid, 256, 0, s>>>(p);
  FLARE_CUDA_CHECK(cudaGetLastError());
  dyn_fill_kernel<<<grid, 256, 0, s>>>(p);
  FLARE_CUDA_CHECK(cudaGetLastError());
  dyn_remap_kernel<<<grid, 256, 0, s>>>(p);
  FLARE_CUDA_CHECK(cudaGetLastError());
  count_launch(3);
}

}  // namespace flare
