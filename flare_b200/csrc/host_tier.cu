// Host-DRAM tier of an embedding table: HBM cache placement on the device (sm_100a).
//
// A host-tier table keeps every row (and its optimizer state) in pinned host
// memory, which the GPU reaches directly through its unified address (PCIe),
// and a cache of hot rows in HBM slots; the fused embedding kernels reach a row
// through slot_map[row] (-1 = not resident).  Before every step two kernels
// make the step's rows resident, with no host involvement (so the whole step,
// placement included, replays from one CUDA graph):
//   tier_mark : for every id of the step (every rank's batch, read from the
//               peers' exchange buffers like the fused forward): a resident row
//               stamps its slot with the step; a missing row is claimed by
//               exactly one thread (slot_map CAS -1 -> -2) and queued;
//   tier_fill : each queued row takes a victim slot with a CLOCK sweep (a slot
//               not stamped by this step, won by CAS on its stamp), writes the
//               victim row + state back to host memory, pulls its own row +
//               state from host memory, and publishes the row -> slot mapping.
//               One warp per row, 16-byte accesses.
// The two-kernel split makes the stamps of this step's resident rows final
// before any victim is chosen.  Every wait is bounded.  The reference's
// larger-than-RAM tier is a memory limit with disk spill inside its external
// store (src/flare/runtime/fluxway/workers/sparse_storage.py); its primary
// copy is host memory and it keeps no HBM cache.
#include "host_tier.cuh"

#include <algorithm>

namespace flare {

namespace {

constexpr int kPending = -2;

__device__ __forceinline__ bool peers_ready(const TierParams& p, uint32_t epoch) {
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

__global__ void tier_mark_kernel(TierParams p) {
  const uint32_t epoch = p.world > 1 ? *reinterpret_cast<volatile uint32_t*>(p.epoch_ctr) + 1u : 0u;
  if (p.world > 1) {
    const bool ok = peers_ready(p, epoch);
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
    const TierTable& t = p.tables[k];
    for (int s = 0; s < p.world; ++s) {
      const int* offs = p.peer_offsets[s];
      const int* vals = p.peer_values[s];
      const int beg = offs[t.feature * p.Bl], end = offs[(t.feature + 1) * p.Bl];
      for (int64_t i = beg + tid; i < end; i += nth) {
        const int row = vals[i];
        if (row < 0 || row >= t.rows) continue;  // the forward reports it
        const int slot = t.slot_map[row];
        if (slot >= 0) {
          t.stamp[slot] = step;
        } else if (slot == -1 && atomicCAS(t.slot_map + row, -1, kPending) == -1) {
          const int q = atomicAdd(t.num_miss, 1);
          if (q < t.miss_cap) t.miss_rows[q] = row;
          else report_error(p.status, kCapacityOverflow, 2000 + k);
        }
      }
    }
  }
}

// One warp per missing row: claim a victim slot, write the victim back, fetch the row.
__global__ void tier_fill_kernel(TierParams p) {
  const int lane = lane_id();
  const int step = *p.step_ptr;
  const int64_t gw = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nw = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  for (int k = 0; k < p.num_tables; ++k) {
    const TierTable& t = p.tables[k];
    const int nmiss = min(*t.num_miss, t.miss_cap);
    for (int64_t i = gw; i < nmiss; i += nw) {
      const int row = t.miss_rows[i];
      int slot = -1;
      if (lane == 0) {
        // CLOCK sweep: the first slot not used by this step, won by CAS on its stamp;
        // bounded by two sweeps of the cache per miss
        for (int64_t tries = 0; tries < 2 * t.C + 64; ++tries) {
          const int c = static_cast<int>(atomicAdd(t.hand, 1u) % static_cast<unsigned>(t.C));
          const int st = t.stamp[c];
          if (st < step && atomicCAS(t.stamp + c, st, step) == st) {
            slot = c;
            break;
          }
        }
        if (slot < 0) report_error(p.status, kCapacityOverflow, 3000 + k);
      }
      slot = __shfl_sync(0xffffffffu, slot, 0);
      if (slot < 0) {
        if (lane == 0) t.slot_map[row] = -1;
        continue;
      }
      const int64_t victim = t.slot2row[slot];
      const int q = t.ncols / 4;
      float4* cw = reinterpret_cast<float4*>(t.cache_w + static_cast<int64_t>(slot) * t.ncols);
      if (victim >= 0) {
        float4* hw = reinterpret_cast<float4*>(t.host_w + victim * t.ncols);
        for (int c = lane; c < q; c += 32) hw[c] = cw[c];
        if (t.cache_m) {
          float4* hm = reinterpret_cast<float4*>(t.host_m + victim * t.ncols);
          const float4* cm = reinterpret_cast<const float4*>(t.cache_m + static_cast<int64_t>(slot) * t.ncols);
          for (int c = lane; c < q; c += 32) hm[c] = cm[c];
        }
        if (t.cache_v) {
          float4* hv = reinterpret_cast<float4*>(t.host_v + victim * t.ncols);
          const float4* cv = reinterpret_cast<const float4*>(t.cache_v + static_cast<int64_t>(slot) * t.ncols);
          for (int c = lane; c < q; c += 32) hv[c] = cv[c];
        }
        if (t.cache_row && lane == 0) t.host_row[victim] = t.cache_row[slot];
      }
      {
        const float4* hw = reinterpret_cast<const float4*>(t.host_w + static_cast<int64_t>(row) * t.ncols);
        for (int c = lane; c < q; c += 32) cw[c] = hw[c];
        if (t.cache_m) {
          const float4* hm = reinterpret_cast<const float4*>(t.host_m + static_cast<int64_t>(row) * t.ncols);
          float4* cm = reinterpret_cast<float4*>(t.cache_m + static_cast<int64_t>(slot) * t.ncols);
          for (int c = lane; c < q; c += 32) cm[c] = hm[c];
        }
        if (t.cache_v) {
          const float4* hv = reinterpret_cast<const float4*>(t.host_v + static_cast<int64_t>(row) * t.ncols);
          float4* cv = reinterpret_cast<float4*>(t.cache_v + static_cast<int64_t>(slot) * t.ncols);
          for (int c = lane; c < q; c += 32) cv[c] = hv[c];
        }
        if (t.cache_row && lane == 0) t.cache_row[slot] = t.host_row[row];
      }
      __syncwarp();
      if (lane == 0) {
        if (victim >= 0) t.slot_map[victim] = -1;
        t.slot2row[slot] = row;
        t.slot_map[row] = slot;
      }
    }
  }
  // the miss counters restart at zero for the next step (last warp to finish)
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(p.block_counter2, 1u) == gridDim.x - 1) {
      *p.block_counter2 = 0u;
      for (int k = 0; k < p.num_tables; ++k) *p.tables[k].num_miss = 0;
    }
  }
}

}  // namespace

void tier_prepare(const TierParams& p, int grid, cudaStream_t s) {
  // a rank without host-tier tables still launches: its peers wait for it at the barrier
  FLARE_CHECK(p.num_tables >= 0 && p.num_tables <= kMaxTierTables, "host-tier table count out of range");
  for (int k = 0; k < p.num_tables; ++k) FLARE_CHECK(p.tables[k].ncols % 4 == 0, "rows must be 4-float aligned");
  tier_mark_kernel<<<grid, 256, 0, s>>>(p);
  FLARE_CUDA_CHECK(cudaGetLastError());
  tier_fill_kernel<<<grid, 256, 0, s>>>(p);
  FLARE_CUDA_CHECK(cudaGetLastError());
  count_launch(2);
}

}  // namespace flare
