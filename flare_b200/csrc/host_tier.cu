// Host-DRAM tier of an embedding table: HBM cache maintenance kernels (sm_100a).
//
// A host-tier table keeps every row (and its optimizer state) in pinned host
// memory and a cache of hot rows in HBM slots; the fused embedding kernels
// reach a row through the device map slot_map[row] (-1 = not resident).  The
// host decides placement one step ahead (it knows the next batch's ids) and
// drives these two kernels on a side stream:
//   tier_gather : copy the rows (+ state) of victim slots into a device staging
//                 buffer, which one cudaMemcpyAsync then writes back to the host;
//   tier_install: mark the victims' rows non-resident, map the missed rows to
//                 their new slots, and scatter the fetched rows (+ state) from
//                 the staging buffer (filled by one pinned cudaMemcpyAsync) into
//                 the slots.
// Both are plain 16-byte copy loops.  The reference's larger-than-RAM tier is
// the external sparse_embedding store's memory limit + disk spill
// (src/flare/runtime/fluxway/workers/sparse_storage.py); there the host copy is
// the primary and nothing is cached in HBM.
#include "host_tier.cuh"

#include <algorithm>

namespace flare {

namespace {

__global__ void tier_gather_kernel(TierCopyParams p) {
  const int q = p.ncols / 4;
  const int64_t total = static_cast<int64_t>(p.n) * q;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int r = static_cast<int>(i / q), c = static_cast<int>(i - static_cast<int64_t>(r) * q);
    const int64_t src = static_cast<int64_t>(p.slots[r]) * q + c, dst = static_cast<int64_t>(r) * q + c;
    reinterpret_cast<float4*>(p.stage_w)[dst] = reinterpret_cast<const float4*>(p.cache_w)[src];
    if (p.cache_m) reinterpret_cast<float4*>(p.stage_m)[dst] = reinterpret_cast<const float4*>(p.cache_m)[src];
    if (p.cache_v) reinterpret_cast<float4*>(p.stage_v)[dst] = reinterpret_cast<const float4*>(p.cache_v)[src];
    if (c == 0 && p.cache_row) p.stage_row[r] = p.cache_row[p.slots[r]];
  }
}

__global__ void tier_install_kernel(TierCopyParams p) {
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t nth = static_cast<int64_t>(gridDim.x) * blockDim.x;
  // evicted and newly fetched rows are disjoint (victims are resident, misses are not)
  for (int64_t i = tid; i < p.n_evict; i += nth) p.slot_map[p.evict_rows[i]] = -1;
  for (int64_t i = tid; i < p.n; i += nth) p.slot_map[p.new_rows[i]] = p.slots[i];
  const int q = p.ncols / 4;
  const int64_t total = static_cast<int64_t>(p.n) * q;
  for (int64_t i = tid; i < total; i += nth) {
    const int r = static_cast<int>(i / q), c = static_cast<int>(i - static_cast<int64_t>(r) * q);
    const int64_t dst = static_cast<int64_t>(p.slots[r]) * q + c, src = static_cast<int64_t>(r) * q + c;
    reinterpret_cast<float4*>(p.cache_w)[dst] = reinterpret_cast<const float4*>(p.stage_w)[src];
    if (p.cache_m) reinterpret_cast<float4*>(p.cache_m)[dst] = reinterpret_cast<const float4*>(p.stage_m)[src];
    if (p.cache_v) reinterpret_cast<float4*>(p.cache_v)[dst] = reinterpret_cast<const float4*>(p.stage_v)[src];
    if (c == 0 && p.cache_row) p.cache_row[p.slots[r]] = p.stage_row[r];
  }
}

int grid_of(int64_t n) { return static_cast<int>(n <= 0 ? 1 : (n + 255) / 256 > 148 * 8 ? 148 * 8 : (n + 255) / 256); }

}  // namespace

void tier_gather(const TierCopyParams& p, cudaStream_t s) {
  FLARE_CHECK(p.ncols % 4 == 0, "host-tier rows must be a multiple of 4 floats");
  if (p.n <= 0) return;
  tier_gather_kernel<<<grid_of(static_cast<int64_t>(p.n) * p.ncols / 4), 256, 0, s>>>(p);
  FLARE_CUDA_CHECK(cudaGetLastError());
  count_launch();
}

void tier_install(const TierCopyParams& p, cudaStream_t s) {
  FLARE_CHECK(p.ncols % 4 == 0, "host-tier rows must be a multiple of 4 floats");
  if (p.n <= 0 && p.n_evict <= 0) return;
  const int64_t work = std::max<int64_t>(static_cast<int64_t>(p.n) * p.ncols / 4, std::max(p.n, p.n_evict));
  tier_install_kernel<<<grid_of(work), 256, 0, s>>>(p);
  FLARE_CUDA_CHECK(cudaGetLastError());
  count_launch();
}

}  // namespace flare
