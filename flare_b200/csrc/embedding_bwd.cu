// Fused sharded embedding backward, hash-dedup path (sm_100a): six launches per step.
//
//   1. emb_hash_count_kernel: entry barrier with every peer; pooled-gradient all-to-all (the
//      owner pulls its columns of every peer's pooled gradients over NVLink; at one GPU the
//      gradients are read in place instead); then, per tile of 2048 staged occurrences, equal
//      rows are aggregated in a shared-memory hash table and each distinct row is inserted into
//      (or added to) the table of the step's touched rows: a region sized for the step, which is
//      prefetched into L2 and takes every key's first probes, backed by an overflow table with
//      room for every possible key.  The add returns the row's count before this tile, which
//      ranks the tile's occurrences of the row without further atomics.
//   2. emb_hash_reduce_kernel + emb_hash_scan_kernel: reduce-then-scan over the table's region
//      slots and the overflow slots in use, in slot order (per-block totals, then each block
//      adds the totals before it): every occupied slot gets its segment start in the grouped
//      occurrence list and a work record (single-occurrence rows, other light rows, and chunks
//      of the heavy rows).
//   3. emb_hash_fill_kernel: occ[seg[slot] + rank] = gradient row of the occurrence (a counting
//      sort by row, no atomics); a single-occurrence row's offset goes straight into its record.
//   4. emb_hash_chunk_kernel: chunks of at most kChunk occurrences of the rows above light_max
//      (the Zipf head), one warp each with eight gradient-row loads in flight per lane (a row of
//      one chunk is updated by that warp; for longer rows every chunk stores an fp32 partial and
//      the last chunk to finish, found by an atomic count-down on the row's slot, adds the
//      partials in chunk order and applies the update).
//   5. emb_hash_light_kernel: batches of light rows, several per warp, the row state read with
//      the weights.  (One kernel interleaving both kinds of work measured slower than the two.)
//   Every applied row clears its slot, so the table is empty again for the next step.
//
// Gradient sums accumulate in fp32 and the row-wise optimizer is applied once per touched row
// (reference semantics: src/flare/kernels/backends/gpu_cupy.py:171-252 scatter-add into fp32,
// then src/flare/runtime/fluxway/workers/dynamic_embedding.py:481-549 optimizer_step).  The
// order of additions within a row follows atomic order, so results are not bitwise
// reproducible run to run; the deterministic mode runs the sorted path in embedding.cu.
#include "embedding.cuh"
#include "sparse_update.cuh"

#include <type_traits>

namespace flare {
namespace {

constexpr unsigned kAll = 0xffffffffu;
constexpr int kHThreads = 256;
constexpr unsigned kHSmemEmpty = 0xFFFFFFFFu;
constexpr unsigned long long kHEmpty = 0xFFFFFFFFull;  // key 0xFFFFFFFF, count 0
constexpr int kHProbeLimit = 1 << 16;    // global probes per insert before reporting overflow
constexpr int kRegionProbes = 32;        // probes in the L2-sized region before the overflow table
constexpr int kChunk = 256;              // occurrences per work chunk of a heavy row
constexpr int kScanThreads = 256;
constexpr int kMaxShards = 96;

__device__ __forceinline__ unsigned lanemask_lt() {
  unsigned m;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

__device__ __forceinline__ bool hbarrier_wait(const uint32_t* flags_local, int world, int slot_off, uint32_t epoch,
                                              uint64_t timeout_ns, int* status) {
  bool ok = true;
  for (int s = 0; s < world && ok; ++s) ok = wait_flag_geq(flags_local + slot_off + s, epoch, timeout_ns, status, s);
  return ok;
}

// Slot of probe `i` of a key: first kRegionProbes slots of the region [0, region) (a table sized
// for the step's expected unique rows, prefetched into L2), then the overflow table
// [region, region + hcap), which alone has room for every possible key.
__device__ __forceinline__ unsigned long long probe_slot(unsigned long long mixed, int i, unsigned long long region,
                                                         unsigned long long omask) {
  if (i < kRegionProbes && region != 0) return (mixed + static_cast<unsigned long long>(i)) & (region - 1);
  const int j = region != 0 ? i - kRegionProbes : i;
  return region + (((mixed >> 32) + static_cast<unsigned long long>(j)) & omask);
}

__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Shard of a local row: the largest shard whose row_base <= row (shards hold consecutive row ranges).
__device__ __forceinline__ int shard_of_row(const long long* row_base, int nsh, long long row) {
  int lo = 0, hi = nsh;
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (row_base[mid] <= row) lo = mid;
    else hi = mid;
  }
  return lo;
}

// ============================================================================
// 1. pull + tile aggregation + global insert-or-add
// ============================================================================
// kCWin: 32-occurrence windows per warp step in the counting pass (8 measured 4 % slower per step:
// 109 registers halve the resident warps, so no more atomics are in flight)
template <int kCWin>
__global__ void __launch_bounds__(kHThreads) emb_hash_count_kernel(EmbBwdParams p) {
  __shared__ int start[1025];           // compact occurrence index of each (shard, source) slot
  __shared__ long long slot_rb[1024];   // row base of each slot's shard
  __shared__ int s_valid;
  // the region of the touched-row table into L2 first (its slots take this step's atomics)
  if (p.hprefetch) {
    const int64_t rbytes = p.hregion * 8;
    for (int64_t off = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 4096; off < rbytes;
         off += static_cast<int64_t>(gridDim.x) * blockDim.x * 4096)
      prefetch_l2(reinterpret_cast<const char*>(p.htab) + off, static_cast<uint32_t>(rbytes - off < 4096 ? rbytes - off : 4096));
  }
  if (p.world > 1) {
    const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(p.epoch_ctr) + 1u;
    __shared__ int ok_sh;
    if (threadIdx.x == 0) {
      if (blockIdx.x == 0) {
        fence_sys();
        for (int s = 0; s < p.world; ++s) st_release_sys(p.peer_flags[s] + p.flag_in + p.rank, epoch);
      }
      ok_sh = hbarrier_wait(p.flags_local, p.world, p.flag_in, epoch, p.timeout_ns, p.status) ? 1 : 0;
      if (atomicAdd(p.block_counter, 1u) == gridDim.x - 1) {  // every block has read the epoch
        *p.block_counter = 0u;
        *p.epoch_ctr = epoch;
      }
    }
    __syncthreads();
    if (!ok_sh) return;
  }
  if (!p.grad_direct) {
    // pooled-gradient all-to-all: this owner's columns of every (source, sample) row, 16 B per thread
    const int tid = static_cast<int>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int nthreads = static_cast<int>(gridDim.x) * blockDim.x;
    const int esize = p.grad_dtype == kBF16 ? 2 : 4;
    for (int sh = 0; sh < p.num_shards; ++sh) {
      const ShardDesc d = p.shards[sh];
      const int chunks = d.ncols * esize / 16;
      const int cshift = __ffs(chunks) - 1;
      const int total = p.world * p.Bl * chunks;
      for (int i = tid; i < total; i += nthreads) {
        const int c = i & (chunks - 1);
        const int bs = i >> cshift;
        const int b = bs / p.world;
        const int s = bs - b * p.world;
        const char* src = reinterpret_cast<const char*>(p.peer_grad[s]) +
                          (static_cast<int64_t>(b) * p.out_stride + d.out_col) * esize + c * 16;
        char* dst = reinterpret_cast<char*>(p.grad_stage) +
                    ((static_cast<int64_t>(sh * p.world + s) * p.Bl + b) * p.grad_stage_ld) * esize + c * 16;
        *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(src);
      }
    }
  }

  // slot prefix (compact occurrence index), computed by every block from the staged counts
  const int nslot = p.num_shards * p.world;
  {
    __shared__ int wsum[32];
    int carry = 0;
    for (int base = 0; base <= nslot; base += blockDim.x) {
      const int i = base + threadIdx.x;
      const int c = i < nslot ? static_cast<int>(min(static_cast<int64_t>(p.stage_count[i]), p.stage_cap)) : 0;
      int x = c;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(kAll, x, o);
        if (lane_id() >= o) x += y;
      }
      if (lane_id() == 31) wsum[warp_id()] = x;
      __syncthreads();
      if (warp_id() == 0) {
        int t = lane_id() < kHThreads / 32 ? wsum[lane_id()] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int y = __shfl_up_sync(kAll, t, o);
          if (lane_id() >= o) t += y;
        }
        wsum[lane_id()] = t;
      }
      __syncthreads();
      const int excl = carry + (warp_id() > 0 ? wsum[warp_id() - 1] : 0) + x - c;
      if (i <= nslot) start[i] = excl;
      carry += wsum[kHThreads / 32 - 1];
      __syncthreads();
    }
  }
  for (int i = threadIdx.x; i < nslot; i += blockDim.x) slot_rb[i] = p.shards[i / p.world].row_base;
  if (threadIdx.x == 0) s_valid = 0;
  __syncthreads();
  const int T = start[nslot];
  if (blockIdx.x == 0)
    for (int i = threadIdx.x; i <= nslot; i += blockDim.x) p.slot_start[i] = start[i];
  const unsigned long long region = static_cast<unsigned long long>(p.hregion);
  const unsigned long long omask = static_cast<unsigned long long>(p.hcap - 1);
  const int lane = lane_id();
  const int gw = static_cast<int>((static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5);
  const int nw = static_cast<int>((static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5);
  int valid_local = 0;
  // Each warp step: kCWin windows of 32 consecutive occurrences.  Equal rows of a window are
  // aggregated with match_any; the window's leaders insert-or-add into the table (all windows'
  // atomics in flight together) and every occurrence's rank is the count before the add plus its
  // position among its equal-row lanes.  Steps are visited in a permuted order (a multiplicative
  // stride coprime with the step count), so the warps in flight spread over every table instead of
  // queueing on the hottest rows of the first few.
  const int64_t nsteps = (T + 32 * kCWin - 1) / (32 * kCWin);
  int64_t stride_p = 1000003;  // prime: coprime with nsteps unless it divides it
  if (nsteps % stride_p == 0) stride_p = 999983;
  for (int64_t st = gw; st < nsteps; st += nw) {
    const int base = static_cast<int>((st * stride_p) % nsteps) * 32 * kCWin;
    int slot = 0;
    {
      int lo = 0, hi = nslot;  // slot of this warp step's first occurrence
      while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (start[mid] <= base) lo = mid;
        else hi = mid;
      }
      slot = lo;
    }
    unsigned row[kCWin];
#pragma unroll
    for (int j = 0; j < kCWin; ++j) {
      const int k = base + j * 32 + lane;
      row[j] = kHSmemEmpty;
      if (k < T) {
        int sl = slot;
        while (sl + 1 < nslot && start[sl + 1] <= k) ++sl;
        const int64_t at = static_cast<int64_t>(sl) * p.stage_cap + (k - start[sl]);
        // streamed once: evict-first, so the table's region keeps its place in L2
        const int id = __ldcs(p.stage_ids + at);
        __stcs(p.occ_bag + k, sl * p.Bl + __ldcs(p.stage_bag + at));
        if (id >= 0) row[j] = static_cast<unsigned>(slot_rb[sl] + id);
      }
    }
    unsigned peers[kCWin];
    bool pend[kCWin], hit[kCWin];
    unsigned long long h[kCWin], old[kCWin], add[kCWin];
#pragma unroll
    for (int j = 0; j < kCWin; ++j) {
      peers[j] = __match_any_sync(kAll, row[j]);
      const bool lead = row[j] != kHSmemEmpty && lane == __ffs(peers[j]) - 1;
      pend[j] = lead;
      hit[j] = false;
      add[j] = static_cast<unsigned long long>(__popc(peers[j])) << 32;
      h[j] = lead ? probe_slot(hash_mix64(row[j]), 0, region, omask) : 0ull;
      old[j] = 0ull;
      valid_local += row[j] != kHSmemEmpty ? 1 : 0;
    }
    bool any = false;
#pragma unroll
    for (int j = 0; j < kCWin; ++j) any = any || pend[j];
    for (int probe = 0; any; ++probe) {
#pragma unroll
      for (int j = 0; j < kCWin; ++j)
        if (pend[j]) old[j] = atomicCAS(p.htab + h[j], kHEmpty, add[j] | row[j]);
      any = false;
#pragma unroll
      for (int j = 0; j < kCWin; ++j) {
        if (!pend[j]) continue;
        if (old[j] == kHEmpty) {  // inserted: no earlier occurrence of the row
          pend[j] = false;
          if (h[j] >= region) p.ovf_list[atomicAdd(p.num_unique + 6, 1)] = static_cast<int>(h[j]);
        } else if (static_cast<unsigned>(old[j]) == row[j]) {
          pend[j] = false;
          hit[j] = true;
        } else if (probe >= kHProbeLimit) {
          pend[j] = false;
          h[j] = ~0ull;  // table overfull: the row's occurrences are dropped and reported
          report_error(p.status, kCapacityOverflow, -2);
        } else {
          h[j] = probe_slot(hash_mix64(row[j]), probe + 1, region, omask);
          any = true;
        }
      }
    }
#pragma unroll
    for (int j = 0; j < kCWin; ++j)
      if (hit[j]) old[j] = atomicAdd(p.htab + h[j], add[j]);
#pragma unroll
    for (int j = 0; j < kCWin; ++j) {
      const int leader = __ffs(peers[j]) - 1;
      const unsigned long long hh = __shfl_sync(kAll, h[j], leader);
      const int before = __shfl_sync(kAll, static_cast<int>(old[j] >> 32), leader);
      const int k = base + j * 32 + lane;
      if (k < T) {
        if (row[j] != kHSmemEmpty && hh != ~0ull) {
          __stcs(p.occ_h + k, static_cast<int>(hh));
          __stcs(p.occ_rank + k, before + __popc(peers[j] & lanemask_lt()));
        } else {
          __stcs(p.occ_h + k, -1);
        }
      }
    }
  }
  valid_local = __reduce_add_sync(kAll, valid_local);
  if (lane == 0 && valid_local) atomicAdd(&s_valid, valid_local);
  __syncthreads();
  if (threadIdx.x == 0 && s_valid) atomicAdd(p.num_unique + 1, s_valid);
}

// ============================================================================
// 2. scan over the table's slots -> segment starts and per-row work records
// ============================================================================
// Per occupied slot (a touched row): a = occurrences, b = work chunks (rows above light_max),
// c = fp32 partial rows (rows of more than one chunk), d = 1 for a single-occurrence row,
// e = 1 for another light row, f = 1 (unique rows).
struct Q6 {
  int a, b, c, d, e, f;
};
__device__ __forceinline__ Q6 q6_add(Q6 x, Q6 y) {
  return Q6{x.a + y.a, x.b + y.b, x.c + y.c, x.d + y.d, x.e + y.e, x.f + y.f};
}
__device__ __forceinline__ Q6 q6_sub(Q6 x, Q6 y) {
  return Q6{x.a - y.a, x.b - y.b, x.c - y.c, x.d - y.d, x.e - y.e, x.f - y.f};
}
__device__ __forceinline__ Q6 q6_shfl_up(Q6 x, int o) {
  return Q6{__shfl_up_sync(kAll, x.a, o), __shfl_up_sync(kAll, x.b, o), __shfl_up_sync(kAll, x.c, o),
            __shfl_up_sync(kAll, x.d, o), __shfl_up_sync(kAll, x.e, o), __shfl_up_sync(kAll, x.f, o)};
}
__device__ __forceinline__ Q6 q6_warp_sum(Q6 x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    x.a += __shfl_xor_sync(kAll, x.a, o);
    x.b += __shfl_xor_sync(kAll, x.b, o);
    x.c += __shfl_xor_sync(kAll, x.c, o);
    x.d += __shfl_xor_sync(kAll, x.d, o);
    x.e += __shfl_xor_sync(kAll, x.e, o);
    x.f += __shfl_xor_sync(kAll, x.f, o);
  }
  return x;
}
__device__ __forceinline__ Q6 q6_load(const volatile int* v) { return Q6{v[0], v[1], v[2], v[3], v[4], v[5]}; }
__device__ __forceinline__ void q6_store(int* v, Q6 x) {
  v[0] = x.a, v[1] = x.b, v[2] = x.c, v[3] = x.d, v[4] = x.e, v[5] = x.f;
}

__device__ __forceinline__ Q6 row_work(int c, int light_max) {
  if (c <= light_max) return Q6{c, 0, 0, c == 1 ? 1 : 0, c == 1 ? 0 : 1, 1};
  const int nch = (c + kChunk - 1) / kChunk;
  return Q6{c, nch, nch > 1 ? nch : 0, 0, 0, 1};
}

constexpr int kScanPer = 4;
constexpr int kScanStep = kScanThreads * kScanPer;  // slots per block iteration

// Slot, row and work of scan item i: the region's slots, then the overflow slots in use.
struct ScanItem {
  int hs;
  unsigned row;
  Q6 v;
};
__device__ __forceinline__ ScanItem scan_item(const EmbBwdParams& p, int i, int R, int N) {
  ScanItem it;
  it.hs = i < R ? i : (i < N ? p.ovf_list[i - R] : -1);
  const unsigned long long wd = it.hs >= 0 ? p.htab[it.hs] : kHEmpty;
  it.row = static_cast<unsigned>(wd);
  it.v = it.row != 0xFFFFFFFFu ? row_work(static_cast<int>(wd >> 32), p.light_max) : Q6{0, 0, 0, 0, 0, 0};
  return it;
}

__device__ __forceinline__ Q6 block_sum_q6(Q6 v, Q6* sh) {
  v = q6_warp_sum(v);
  if (lane_id() == 0) sh[warp_id()] = v;
  __syncthreads();
  Q6 t{0, 0, 0, 0, 0, 0};
  for (int w = 0; w < kScanThreads / 32; ++w) t = q6_add(t, sh[w]);
  __syncthreads();
  return t;
}

__device__ __forceinline__ void scan_range(int N, int& lo, int& hi) {
  const int per = ((N + gridDim.x - 1) / gridDim.x + kScanStep - 1) / kScanStep * kScanStep;
  lo = min(N, static_cast<int>(blockIdx.x) * per);
  hi = min(N, lo + per);
}

// 2a. per-block totals of a contiguous range of items
__global__ void __launch_bounds__(kScanThreads) emb_hash_reduce_kernel(EmbBwdParams p) {
  __shared__ Q6 sh[kScanThreads / 32];
  const int R = static_cast<int>(p.hregion);
  const int N = R + min(p.num_unique[6], static_cast<int>(p.max_occ));
  int lo, hi;
  scan_range(N, lo, hi);
  Q6 acc{0, 0, 0, 0, 0, 0};
  for (int i = lo + threadIdx.x; i < hi; i += blockDim.x) acc = q6_add(acc, scan_item(p, i, R, N).v);
  acc = block_sum_q6(acc, sh);
  if (threadIdx.x == 0) q6_store(p.scan_val + static_cast<int64_t>(blockIdx.x) * 6, acc);
}

// 2b. block prefix from the totals of the blocks before it, then an in-order scan of its range
// writing every occupied slot's segment start and work record
__global__ void __launch_bounds__(kScanThreads) emb_hash_scan_kernel(EmbBwdParams p) {
  __shared__ Q6 sh[kScanThreads / 32];
  __shared__ Q6 s_warp[kScanThreads / 32];
  const int R = static_cast<int>(p.hregion);
  const int N = R + min(p.num_unique[6], static_cast<int>(p.max_occ));
  int lo, hi;
  scan_range(N, lo, hi);
  Q6 pre{0, 0, 0, 0, 0, 0};
  for (int b = threadIdx.x; b < static_cast<int>(blockIdx.x); b += blockDim.x)
    pre = q6_add(pre, q6_load(p.scan_val + static_cast<int64_t>(b) * 6));
  Q6 carry = block_sum_q6(pre, sh);
  for (int i0 = lo; i0 < hi; i0 += kScanStep) {
    ScanItem it[kScanPer];
    Q6 tsum{0, 0, 0, 0, 0, 0};
#pragma unroll
    for (int k = 0; k < kScanPer; ++k) {
      const int i = i0 + threadIdx.x * kScanPer + k;
      it[k] = i < hi ? scan_item(p, i, R, N) : ScanItem{-1, 0xFFFFFFFFu, Q6{0, 0, 0, 0, 0, 0}};
      tsum = q6_add(tsum, it[k].v);
    }
    Q6 x = tsum;  // inclusive warp scan of the thread sums
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const Q6 y = q6_shfl_up(x, o);
      if (lane_id() >= o) x = q6_add(x, y);
    }
    if (lane_id() == 31) s_warp[warp_id()] = x;
    __syncthreads();
    Q6 wpre{0, 0, 0, 0, 0, 0}, step{0, 0, 0, 0, 0, 0};
    for (int w = 0; w < kScanThreads / 32; ++w) {
      if (w < warp_id()) wpre = q6_add(wpre, s_warp[w]);
      step = q6_add(step, s_warp[w]);
    }
    __syncthreads();
    Q6 run = q6_add(carry, q6_add(wpre, q6_sub(x, tsum)));
#pragma unroll
    for (int k = 0; k < kScanPer; ++k) {
      const Q6& v = it[k].v;
      if (v.f) {
        const int c = v.a;
        const int hs = it[k].hs;
        const int row = static_cast<int>(it[k].row);
        // a single-occurrence row's segment start names its record instead (-1 - index): the fill
        // kernel writes the gradient offset straight into the record
        p.hseg[hs] = v.d ? -1 - run.d : run.a;
        if (v.d) {
          p.lrec[run.d] = make_int4(row, hs, 0, 0);
        } else if (v.e) {
          p.lrec[p.max_occ - 1 - run.e] = make_int4(row, hs, run.a, c);
        } else if (run.b + v.b <= p.max_chunks && run.c + v.c <= p.max_parts) {
          const int nch = v.b;
          for (int q = 0; q < nch; ++q) {
            const int a = run.a + q * kChunk;
            int4* rec = p.crec + 2 * static_cast<int64_t>(run.b + q);
            rec[0] = make_int4(row, hs, a, min(kChunk, run.a + c - a));
            rec[1] = make_int4(nch > 1 ? run.c : -1, q, nch, c);
          }
        }
      }
      run = q6_add(run, v);
    }
    carry = q6_add(carry, step);
  }
  if (blockIdx.x == gridDim.x - 1 && threadIdx.x == 0) {
    p.num_unique[0] = carry.f;
    p.num_unique[3] = carry.b;
    p.num_unique[4] = carry.d;
    p.num_unique[5] = carry.e;
    if (carry.b > p.max_chunks || carry.c > p.max_parts) report_error(p.status, kCapacityOverflow, -4);
  }
}

// ============================================================================
// 3. counting sort of the occurrences by unique row (four occurrences in flight per thread)
// ============================================================================
__global__ void __launch_bounds__(kHThreads) emb_hash_fill_kernel(EmbBwdParams p) {
  __shared__ int out_col[kMaxShards];
  __shared__ int mean[kMaxShards];
  for (int i = threadIdx.x; i < p.num_shards; i += blockDim.x) {
    out_col[i] = p.shards[i].out_col;
    mean[i] = p.shards[i].pooling == 1;
  }
  __syncthreads();
  const bool staged = !p.grad_direct;
  const int T = p.slot_start[p.num_shards * p.world];
  const int tid = static_cast<int>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int nth = static_cast<int>(gridDim.x) * blockDim.x;
  for (int k0 = tid; k0 < T; k0 += 4 * nth) {
    int h[4], rk[4], bag[4], pos[4];
#pragma unroll
    for (int x = 0; x < 4; ++x) {
      const int k = k0 + x * nth;
      h[x] = k < T ? __ldcs(p.occ_h + k) : -1;
      rk[x] = k < T ? __ldcs(p.occ_rank + k) : 0;
      bag[x] = k < T ? __ldcs(p.occ_bag + k) : 0;
    }
#pragma unroll
    for (int x = 0; x < 4; ++x) pos[x] = h[x] >= 0 ? p.hseg[h[x]] : 0;
#pragma unroll
    for (int x = 0; x < 4; ++x) {
      if (h[x] < 0) continue;
      const int slot = bag[x] / p.Bl;
      const int b = bag[x] - slot * p.Bl;
      const int goff = staged ? static_cast<int>(static_cast<int64_t>(bag[x]) * p.grad_stage_ld)
                              : static_cast<int>(static_cast<int64_t>(b) * p.out_stride + out_col[slot]);
      const float sc = (p.occ_scale != nullptr && mean[slot / p.world])
                           ? 1.f / static_cast<float>(max(1, p.stage_len[bag[x]])) : 1.f;
      if (pos[x] < 0) {  // single-occurrence row: its record carries the offset (and the mean scale)
        int* rec = reinterpret_cast<int*>(p.lrec + (-1 - pos[x]));
        rec[2] = goff;
        if (p.occ_scale != nullptr) rec[3] = __float_as_int(sc);
      } else {
        p.occ[pos[x] + rk[x]] = goff;
        if (p.occ_scale != nullptr) p.occ_scale[pos[x] + rk[x]] = sc;
      }
    }
  }
}

// ============================================================================
// 4. fp32 reduction + row-wise optimizer
// ============================================================================
// Two fp32 adds in one instruction (sm_100 packed f32x2).
__device__ __forceinline__ void add2(float& a0, float& a1, float b0, float b1) {
  unsigned long long ra, rb, rc;
  asm("mov.b64 %0, {%1, %2};" : "=l"(ra) : "f"(a0), "f"(a1));
  asm("mov.b64 %0, {%1, %2};" : "=l"(rb) : "f"(b0), "f"(b1));
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(rc) : "l"(ra), "l"(rb));
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a0), "=f"(a1) : "l"(rc));
}

// Raw 16-byte pieces of 4*NV columns of a gradient row (loaded first, widened and added later, so a
// warp keeps many rows in flight).
template <typename TG, int NV>
struct GradRaw {
  static constexpr int kQ = NV * 4 * static_cast<int>(sizeof(TG)) / 16;
  uint4 q[kQ];
  __device__ __forceinline__ void load(const TG* src) {
#pragma unroll
    for (int i = 0; i < kQ; ++i) q[i] = __ldg(reinterpret_cast<const uint4*>(src) + i);
  }
  __device__ __forceinline__ void zero() {
#pragma unroll
    for (int i = 0; i < kQ; ++i) q[i] = make_uint4(0u, 0u, 0u, 0u);
  }
  template <bool kScale, bool kPack = false>
  __device__ __forceinline__ void add(float4 (&acc)[NV], float s) const {
    float* a = reinterpret_cast<float*>(acc);
    if constexpr (kPack && !kScale && sizeof(TG) == 2 && std::is_same<TG, __nv_bfloat16>::value) {
#pragma unroll
      for (int i = 0; i < kQ; ++i) {
        const unsigned wd[4] = {q[i].x, q[i].y, q[i].z, q[i].w};
#pragma unroll
        for (int e = 0; e < 4; ++e)
          add2(a[8 * i + 2 * e], a[8 * i + 2 * e + 1], __uint_as_float(wd[e] << 16),
               __uint_as_float(wd[e] & 0xFFFF0000u));
      }
      return;
    }
#pragma unroll
    for (int i = 0; i < kQ; ++i) {
      const unsigned wd[4] = {q[i].x, q[i].y, q[i].z, q[i].w};
      if constexpr (sizeof(TG) == 4) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float f = __uint_as_float(wd[e]);
          a[4 * i + e] = kScale ? fmaf(f, s, a[4 * i + e]) : a[4 * i + e] + f;
        }
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float lo, hi;
          if constexpr (std::is_same<TG, __nv_bfloat16>::value) {
            lo = __uint_as_float(wd[e] << 16);
            hi = __uint_as_float(wd[e] & 0xFFFF0000u);
          } else {
            const float2 h2 = __half22float2(*reinterpret_cast<const __half2*>(&wd[e]));
            lo = h2.x;
            hi = h2.y;
          }
          a[8 * i + 2 * e] = kScale ? fmaf(lo, s, a[8 * i + 2 * e]) : a[8 * i + 2 * e] + lo;
          a[8 * i + 2 * e + 1] = kScale ? fmaf(hi, s, a[8 * i + 2 * e + 1]) : a[8 * i + 2 * e + 1] + hi;
        }
      }
    }
  }
};
constexpr int kBatchLoads = 8;  // gradient-row loads in flight per lane in the chunk kernel

// acc += s * (NV float4 = 4*NV columns of a gradient row of type TG).  bf16 widens with a shift.
template <typename TG, int NV, bool kScale>
__device__ __forceinline__ void add_grad(const TG* src, float4 (&acc)[NV], float s) {
  if constexpr (sizeof(TG) == 2 && NV % 2 == 0) {
#pragma unroll
    for (int v = 0; v < NV; v += 2) {
      const uint4 q = __ldg(reinterpret_cast<const uint4*>(src + 4 * v));
      const unsigned wd[4] = {q.x, q.y, q.z, q.w};
      float f[8];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        if constexpr (std::is_same<TG, __nv_bfloat16>::value) {
          f[2 * e] = __uint_as_float(wd[e] << 16);
          f[2 * e + 1] = __uint_as_float(wd[e] & 0xFFFF0000u);
        } else {
          const float2 h2 = __half22float2(*reinterpret_cast<const __half2*>(&wd[e]));
          f[2 * e] = h2.x;
          f[2 * e + 1] = h2.y;
        }
      }
      float* a0 = reinterpret_cast<float*>(&acc[v]);
      float* a1 = reinterpret_cast<float*>(&acc[v + 1]);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        a0[e] = kScale ? fmaf(f[e], s, a0[e]) : a0[e] + f[e];
        a1[e] = kScale ? fmaf(f[4 + e], s, a1[e]) : a1[e] + f[4 + e];
      }
    }
  } else {
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      const float4 g = load4<TG>(src + 4 * v);
      acc[v] = kScale ? make_float4(fmaf(g.x, s, acc[v].x), fmaf(g.y, s, acc[v].y), fmaf(g.z, s, acc[v].z),
                                    fmaf(g.w, s, acc[v].w))
                      : f4_add(acc[v], g);
    }
  }
}

// 4. Work chunks of the rows above light_max: one warp each, lanes 0..LG-1 cover one gradient row,
// 32 / LG rows per load instruction, kBatchLoads loads in flight per lane.
// 5. Batches of 32 / GL light rows (GL lanes per row): a single-occurrence row's record holds its
// gradient offset; other light rows read their occurrence list; the row state is read with the
// weights.
__device__ __forceinline__ int4 light_rec(const EmbBwdParams& p, int i, int S) {
  return p.lrec[i < S ? static_cast<int64_t>(i) : p.max_occ - 1 - (i - S)];
}

template <typename TW, typename TG, int NVC, bool kScale, int BL = kBatchLoads, bool kPack = false>
__global__ void __launch_bounds__(kHThreads, 3) emb_hash_chunk_kernel(EmbBwdParams p, int LG) {
  __shared__ ShardDesc sd[kMaxShards];
  __shared__ long long rb[kMaxShards];
  for (int i = threadIdx.x; i < p.num_shards; i += blockDim.x) {
    sd[i] = p.shards[i];
    rb[i] = p.shards[i].row_base;
  }
  __syncthreads();
  SparseOptParams o = p.opt;
  resolve_sparse_step(o);
  const int nsh = p.num_shards;
  const TG* gbase = p.grad_direct ? reinterpret_cast<const TG*>(p.peer_grad[p.rank])
                                  : reinterpret_cast<const TG*>(p.grad_stage);
  TW* const weights = reinterpret_cast<TW*>(p.weights);
  const int lane = lane_id();
  const int gwarp = static_cast<int>((static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5);
  const int nwarps = static_cast<int>((static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5);
  const int NHC = min(p.num_unique[3], static_cast<int>(p.max_chunks));
  const int S = min(p.num_unique[4], static_cast<int>(p.max_occ));
  const int N = min(S + p.num_unique[5], static_cast<int>(p.max_occ));
  int heavy_rows = 0;

  for (int64_t jj = gwarp; jj < NHC; jj += nwarps) {
      // ---------------- work chunk c0
      const int j = static_cast<int>(jj);
      const int RPI = 32 / LG;
      const int r = lane / LG, l = lane - r * LG;
      const int col = l * 4 * NVC;
      const int ld = LG * 4 * NVC;  // fp32 partial row stride (= widest shard)
      const int4 r0 = p.crec[2 * static_cast<int64_t>(j)];
      const int4 r1 = p.crec[2 * static_cast<int64_t>(j) + 1];
      const long long row = static_cast<unsigned>(r0.x);
      const int hs = r0.y, a = r0.z, len = r0.w;
      const int part = r1.x, ci = r1.y, nch = r1.z, c = r1.w;
      const ShardDesc& d = sd[shard_of_row(rb, nsh, row)];
      const bool act = col < d.ncols;
      float4 acc[NVC];
#pragma unroll
      for (int v = 0; v < NVC; ++v) acc[v] = make_float4(0.f, 0.f, 0.f, 0.f);
      // 32 occurrences per batch; the next batch's indices load while this batch's rows are in flight
      int gi_n = lane < len ? p.occ[a + lane] : 0;
      float sc_n = (kScale && lane < len) ? p.occ_scale[a + lane] : 1.f;
      for (int q0 = 0; q0 < len; q0 += 32) {
        const int n = min(32, len - q0);
        const int gi = gi_n;
        const float sc = sc_n;
        if (q0 + 32 < len) {
          gi_n = q0 + 32 + lane < len ? p.occ[a + q0 + 32 + lane] : 0;
          if (kScale) sc_n = q0 + 32 + lane < len ? p.occ_scale[a + q0 + 32 + lane] : 1.f;
        }
        for (int tt = 0; tt < n; tt += BL * RPI) {
          GradRaw<TG, NVC> raw[BL];
          float s8[BL];
#pragma unroll
          for (int x = 0; x < BL; ++x) {
            const int qq = tt + x * RPI + r;
            const int g = __shfl_sync(kAll, gi, qq & 31);
            s8[x] = kScale ? __shfl_sync(kAll, sc, qq & 31) : 1.f;
            if (act && qq < n) raw[x].load(gbase + g + col);
            else raw[x].zero();
          }
#pragma unroll
          for (int x = 0; x < BL; ++x) raw[x].template add<kScale, kPack>(acc, s8[x]);
        }
      }
      for (int off = LG; off < 32; off <<= 1)
#pragma unroll
        for (int v = 0; v < NVC; ++v) {
          acc[v].x += __shfl_xor_sync(kAll, acc[v].x, off);
          acc[v].y += __shfl_xor_sync(kAll, acc[v].y, off);
          acc[v].z += __shfl_xor_sync(kAll, acc[v].z, off);
          acc[v].w += __shfl_xor_sync(kAll, acc[v].w, off);
        }
      const bool own = act && r == 0;  // lanes 0..LG-1 hold the row's sums
      bool apply = part < 0;
      if (!apply) {
        float* dst = p.hpart + static_cast<int64_t>(part + ci) * ld + col;
        if (own) {
#pragma unroll
          for (int v = 0; v < NVC; ++v) __stcg(reinterpret_cast<float4*>(dst) + v, acc[v]);
        }
        __threadfence();
        __syncwarp();
        int last = 0;
        if (lane == 0) {
          const unsigned long long dec = 0ull - (static_cast<unsigned long long>(len) << 32);
          last = static_cast<int>(atomicAdd(p.htab + hs, dec) >> 32) == len;
        }
        apply = __shfl_sync(kAll, last, 0) != 0;
        if (apply) {
          __threadfence();
#pragma unroll
          for (int v = 0; v < NVC; ++v) acc[v] = make_float4(0.f, 0.f, 0.f, 0.f);
          if (own) {
            // partials in chunk order, four rows in flight
            const float* p0 = p.hpart + static_cast<int64_t>(part) * ld + col;
            int q = 0;
            for (; q + 4 <= nch; q += 4) {
              float4 t4[4][NVC];
#pragma unroll
              for (int x = 0; x < 4; ++x)
#pragma unroll
                for (int v = 0; v < NVC; ++v) t4[x][v] = __ldcg(reinterpret_cast<const float4*>(p0 + (q + x) * ld) + v);
#pragma unroll
              for (int x = 0; x < 4; ++x)
#pragma unroll
                for (int v = 0; v < NVC; ++v) acc[v] = f4_add(acc[v], t4[x][v]);
            }
            for (; q < nch; ++q)
#pragma unroll
              for (int v = 0; v < NVC; ++v)
                acc[v] = f4_add(acc[v], __ldcg(reinterpret_cast<const float4*>(p0 + q * ld) + v));
          }
        }
      }
      if (apply) {
        const int64_t eoff = d.weight_off + (row - d.row_base) * d.ncols + col;
        TW* w = weights + eoff;
        float4 wv[NVC];
#pragma unroll
        for (int v = 0; v < NVC; ++v) wv[v] = own ? load4<TW>(w + 4 * v) : make_float4(0.f, 0.f, 0.f, 0.f);
        apply_update<TW, NVC>(o, w, eoff, row, true, own, d.ncols, acc, wv, c, LG, 0);
        if (lane == 0) {
          p.htab[hs] = kHEmpty;
          mark_dirty(p.dirty, row);
          ++heavy_rows;
        }
      }
  }
  if (lane == 0 && heavy_rows) atomicAdd(p.num_unique + 2, heavy_rows);
}

template <typename TW, typename TG, int NVL, bool kScale>
__global__ void __launch_bounds__(kHThreads, 3) emb_hash_light_kernel(EmbBwdParams p, int GL) {
  __shared__ ShardDesc sd[kMaxShards];
  __shared__ long long rb[kMaxShards];
  for (int i = threadIdx.x; i < p.num_shards; i += blockDim.x) {
    sd[i] = p.shards[i];
    rb[i] = p.shards[i].row_base;
  }
  __syncthreads();
  SparseOptParams o = p.opt;
  resolve_sparse_step(o);
  const int nsh = p.num_shards;
  const bool row_state = o.state_row != nullptr && (o.kind == kOptRowwiseAdagrad || o.kind == kOptRowwiseAdam);
  const TG* gbase = p.grad_direct ? reinterpret_cast<const TG*>(p.peer_grad[p.rank])
                                  : reinterpret_cast<const TG*>(p.grad_stage);
  TW* const weights = reinterpret_cast<TW*>(p.weights);
  const int lane = lane_id();
  const int gwarp = static_cast<int>((static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5);
  const int nwarps = static_cast<int>((static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5);
  const int NHC = min(p.num_unique[3], static_cast<int>(p.max_chunks));
  const int S = min(p.num_unique[4], static_cast<int>(p.max_occ));
  const int N = min(S + p.num_unique[5], static_cast<int>(p.max_occ));
  const int RPW = 32 / GL;
  const int NB = (N + RPW - 1) / RPW;

  for (int64_t t = gwarp; t < NB; t += nwarps) {
    const int64_t c0 = 0;
      // ---------------- light batch t - c0
      const int g = lane / GL, gl = lane - g * GL;
      const int leader = g * GL;
      const int col = gl * 4 * NVL;
      const int i = static_cast<int>(t - c0) * RPW + g;
      const bool mine = i < N;
      const int4 rec = mine ? light_rec(p, i, S) : make_int4(0, 0, 0, 0);
      const long long row = static_cast<unsigned>(rec.x);
      const int hs = rec.y, seg = rec.z, c = mine ? (i < S ? 1 : rec.w) : 0;
      const ShardDesc& d = sd[mine ? shard_of_row(rb, nsh, row) : 0];
      const bool act = mine && col < d.ncols;
      const int64_t eoff = d.weight_off + (row - d.row_base) * d.ncols + col;
      TW* w = weights + eoff;
      const float st_old = (row_state && mine && gl == 0) ? o.state_row[row] : -1.f;
      float4 wv[NVL], acc[NVL];
#pragma unroll
      for (int v = 0; v < NVL; ++v) {
        wv[v] = act ? load4<TW>(w + 4 * v) : make_float4(0.f, 0.f, 0.f, 0.f);
        acc[v] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
      if (act && i < S) {
        // single occurrence: the record holds the gradient offset (and the mean scale)
        add_grad<TG, NVL, kScale>(gbase + seg + col, acc, kScale ? __int_as_float(rec.w) : 1.f);
      } else if (act) {
        int k = 0;
        for (; k + 2 <= c; k += 2) {
          const int g0 = p.occ[seg + k], g1 = p.occ[seg + k + 1];
          const float s0 = kScale ? p.occ_scale[seg + k] : 1.f, s1 = kScale ? p.occ_scale[seg + k + 1] : 1.f;
          add_grad<TG, NVL, kScale>(gbase + g0 + col, acc, s0);
          add_grad<TG, NVL, kScale>(gbase + g1 + col, acc, s1);
        }
        if (k < c) add_grad<TG, NVL, kScale>(gbase + p.occ[seg + k] + col, acc, kScale ? p.occ_scale[seg + k] : 1.f);
      }
      apply_update<TW, NVL>(o, w, eoff, row, mine, act, d.ncols, acc, wv, c, GL, leader, st_old);
      if (mine && gl == 0) {
        p.htab[hs] = kHEmpty;
        mark_dirty(p.dirty, row);
      }
  }
}

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const unsigned sa = static_cast<unsigned>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(sa), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// 5b. The light-row pass for fp32 tables with the next batch's weight rows in flight: while a warp
// reduces and applies batch t, cp.async copies the rows of its batch t + nwarps into shared memory
// (two buffers per lane), so a warp keeps two batches of random row reads outstanding without the
// registers of a second batch.  Every row appears in one record only, so reading a later batch's
// rows early cannot race with an update.  Opt-in (FLARE_EMB_LIGHT_PREFETCH=1): on the 26-table
// DLRM benchmark it measured 0.7 % slower per step than the register version (2.325 vs 2.309 ms),
// which already keeps the DRAM random-read rate near its ceiling with 24 warps per SM.
struct LightCur {
  long long row;
  int64_t eoff;
  int hs, seg, c, ncols;
  int rec_w;
  float st_old;
  bool mine, act, single;
};

template <typename TG, bool kScale>
__global__ void __launch_bounds__(kHThreads, 3) emb_hash_light_pf_kernel(EmbBwdParams p, int GL) {
  constexpr int NVL = 4;
  __shared__ ShardDesc sd[kMaxShards];
  __shared__ long long rb[kMaxShards];
  __shared__ __align__(16) float4 wbuf[2][kHThreads][NVL];
  for (int i = threadIdx.x; i < p.num_shards; i += blockDim.x) {
    sd[i] = p.shards[i];
    rb[i] = p.shards[i].row_base;
  }
  __syncthreads();
  SparseOptParams o = p.opt;
  resolve_sparse_step(o);
  const int nsh = p.num_shards;
  const bool row_state = o.state_row != nullptr && (o.kind == kOptRowwiseAdagrad || o.kind == kOptRowwiseAdam);
  const TG* gbase = p.grad_direct ? reinterpret_cast<const TG*>(p.peer_grad[p.rank])
                                  : reinterpret_cast<const TG*>(p.grad_stage);
  float* const weights = reinterpret_cast<float*>(p.weights);
  const int lane = lane_id();
  const int gwarp = static_cast<int>((static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5);
  const int nwarps = static_cast<int>((static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5);
  const int S = min(p.num_unique[4], static_cast<int>(p.max_occ));
  const int N = min(S + p.num_unique[5], static_cast<int>(p.max_occ));
  const int RPW = 32 / GL;
  const int NB = (N + RPW - 1) / RPW;
  const int g = lane / GL, gl = lane - g * GL;
  const int leader = g * GL;
  const int col = gl * 4 * NVL;

  auto prepare = [&](int64_t t, LightCur& x, int buf) {
    const int i = static_cast<int>(t) * RPW + g;
    x.mine = i < N;
    const int4 rec = x.mine ? light_rec(p, i, S) : make_int4(0, 0, 0, 0);
    x.row = static_cast<unsigned>(rec.x);
    x.hs = rec.y;
    x.seg = rec.z;
    x.rec_w = rec.w;
    x.single = i < S;
    x.c = x.mine ? (x.single ? 1 : rec.w) : 0;
    const ShardDesc& d = sd[x.mine ? shard_of_row(rb, nsh, x.row) : 0];
    x.ncols = d.ncols;
    x.act = x.mine && col < d.ncols;
    x.eoff = d.weight_off + (x.row - d.row_base) * d.ncols + col;
    if (x.act) {
#pragma unroll
      for (int v = 0; v < NVL; ++v) cp_async16(&wbuf[buf][threadIdx.x][v], weights + x.eoff + 4 * v);
    }
    x.st_old = (row_state && x.mine && gl == 0) ? o.state_row[x.row] : -1.f;
  };

  int64_t t = gwarp;
  if (t >= NB) return;
  LightCur cur, nxt;
  int buf = 0;
  prepare(t, cur, 0);
  cp_async_commit();
  for (; t < NB; t += nwarps) {
    const int64_t tn = t + nwarps;
    if (tn < NB) prepare(tn, nxt, buf ^ 1);
    cp_async_commit();
    cp_async_wait<1>();  // this batch's rows (this lane's own copies) have landed
    float4 wv[NVL], acc[NVL];
#pragma unroll
    for (int v = 0; v < NVL; ++v) {
      wv[v] = cur.act ? wbuf[buf][threadIdx.x][v] : make_float4(0.f, 0.f, 0.f, 0.f);
      acc[v] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    if (cur.act && cur.single) {
      add_grad<TG, NVL, kScale>(gbase + cur.seg + col, acc, kScale ? __int_as_float(cur.rec_w) : 1.f);
    } else if (cur.act) {
      int k = 0;
      for (; k + 2 <= cur.c; k += 2) {
        const int g0 = p.occ[cur.seg + k], g1 = p.occ[cur.seg + k + 1];
        const float s0 = kScale ? p.occ_scale[cur.seg + k] : 1.f, s1 = kScale ? p.occ_scale[cur.seg + k + 1] : 1.f;
        add_grad<TG, NVL, kScale>(gbase + g0 + col, acc, s0);
        add_grad<TG, NVL, kScale>(gbase + g1 + col, acc, s1);
      }
      if (k < cur.c)
        add_grad<TG, NVL, kScale>(gbase + p.occ[cur.seg + k] + col, acc, kScale ? p.occ_scale[cur.seg + k] : 1.f);
    }
    apply_update<float, NVL>(o, weights + cur.eoff, cur.eoff, cur.row, cur.mine, cur.act, cur.ncols, acc, wv,
                             cur.c, GL, leader, cur.st_old);
    if (cur.mine && gl == 0) {
      p.htab[cur.hs] = kHEmpty;
      mark_dirty(p.dirty, cur.row);
    }
    cur = nxt;
    buf ^= 1;
  }
  cp_async_wait<0>();
}

template <typename TW, typename TG, bool kScale>
void hash_apply_launch(const EmbBwdParams& p, int ncols_max, int grid, cudaStream_t s) {
  // chunks: one 16-byte gradient load per lane (two for fp32 rows wider than 128 columns);
  // light rows: 16 columns per lane
  constexpr int kNvc = sizeof(TG) == 2 ? 2 : 1;
  const int GL = std::max(1, ncols_max / 16);
  if (sizeof(TG) == 4 && ncols_max > 128) {
    emb_hash_chunk_kernel<TW, TG, 2, kScale><<<grid, kHThreads, 0, s>>>(p, ncols_max / 8);
  } else if (sizeof(TG) == 2 && p.chunk_variant != 0 && ncols_max >= 64) {
    // variants (FLARE_EMB_CHUNK_VARIANT): 1 (default) = 32-byte loads per lane (16 columns), 4 rows in
    // flight per lane: half the index shuffles and address arithmetic per gradient byte, 0.75 % faster
    // per DLRM step than 0 (16-byte loads, 8 in flight); 2 = packed f32x2 adds (no gain); 3 = both
    switch (p.chunk_variant) {
      case 1: emb_hash_chunk_kernel<TW, TG, 4, kScale, 4, false><<<grid, kHThreads, 0, s>>>(p, ncols_max / 16); break;
      case 2: emb_hash_chunk_kernel<TW, TG, 2, kScale, kBatchLoads, true><<<grid, kHThreads, 0, s>>>(p, ncols_max / 8); break;
      default: emb_hash_chunk_kernel<TW, TG, 4, kScale, 4, true><<<grid, kHThreads, 0, s>>>(p, ncols_max / 16); break;
    }
  } else {
    emb_hash_chunk_kernel<TW, TG, kNvc, kScale><<<grid, kHThreads, 0, s>>>(p, ncols_max / (4 * kNvc));
  }
  if constexpr (std::is_same<TW, float>::value) {
    if (p.light_prefetch) {
      emb_hash_light_pf_kernel<TG, kScale><<<grid, kHThreads, 0, s>>>(p, GL);
      return;
    }
  }
  emb_hash_light_kernel<TW, TG, 4, kScale><<<grid, kHThreads, 0, s>>>(p, GL);
}

template <typename TW>
void hash_apply_g(const EmbBwdParams& p, int ncols_max, int grid, cudaStream_t s) {
  const bool mean = p.occ_scale != nullptr;
  if (p.grad_dtype == kBF16) {
    if (mean) hash_apply_launch<TW, __nv_bfloat16, true>(p, ncols_max, grid, s);
    else hash_apply_launch<TW, __nv_bfloat16, false>(p, ncols_max, grid, s);
  } else {
    if (mean) hash_apply_launch<TW, float, true>(p, ncols_max, grid, s);
    else hash_apply_launch<TW, float, false>(p, ncols_max, grid, s);
  }
}

}  // namespace

void emb_backward_hash(const EmbBwdParams& p, int ncols_max, int grid, cudaStream_t s) {
  FLARE_CHECK(p.htab && p.hseg && p.ovf_list && p.occ_h && p.occ_rank && p.occ_bag && p.lrec && p.crec &&
                  p.hpart && p.scan_val,
              "the hash-dedup backward needs its scratch buffers");
  FLARE_CHECK(p.hcap >= p.max_occ && (p.hcap & (p.hcap - 1)) == 0, "hash capacity must be a power of two >= max_occ");
  FLARE_CHECK(p.hregion >= 0 && (p.hregion & (p.hregion - 1)) == 0, "hash region must be zero or a power of two");
  FLARE_CHECK(p.max_tiles >= 1, "scan block totals missing");
  FLARE_CHECK(ncols_max >= 16 && ncols_max <= 256, "hash backward: widest shard must be in [16, 256] columns");
  FLARE_CHECK(p.num_shards <= kMaxShards, "too many local shards");
  if (!p.grad_direct)
    FLARE_CHECK(static_cast<int64_t>(p.num_shards) * p.world * p.Bl * p.grad_stage_ld < (1ll << 31),
                "staged gradient offsets exceed 32 bits");
  else
    FLARE_CHECK(p.world == 1 && static_cast<int64_t>(p.Bl) * p.out_stride < (1ll << 31),
                "in-place gradient reads are for one GPU with 32-bit offsets");
  int dev = 0, sms = 0;
  FLARE_CUDA_CHECK(cudaGetDevice(&dev));
  FLARE_CUDA_CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  emb_hash_count_kernel<4><<<sms * 4, kHThreads, 0, s>>>(p);
  const int sgrid = static_cast<int>(std::min<int64_t>(p.max_tiles, static_cast<int64_t>(sms) * 8));
  emb_hash_reduce_kernel<<<sgrid, kScanThreads, 0, s>>>(p);
  emb_hash_scan_kernel<<<sgrid, kScanThreads, 0, s>>>(p);
  emb_hash_fill_kernel<<<grid, kHThreads, 0, s>>>(p);
  const int agrid = sms * 3;
  if (p.w_dtype == kF32) hash_apply_g<float>(p, ncols_max, agrid, s);
  else if (p.w_dtype == kF16) hash_apply_g<__half>(p, ncols_max, agrid, s);
  else hash_apply_g<__nv_bfloat16>(p, ncols_max, agrid, s);
  FLARE_CUDA_CHECK(cudaGetLastError());
  count_launch(6);
}

// scan blocks (their totals are kept in scan_val, 6 ints each)
int64_t emb_hash_tile_count(int64_t) { return 4096; }
int emb_hash_scan_vals() { return 6; }
int64_t emb_hash_max_chunks(int64_t max_occ, int light_max) {
  return max_occ / (light_max + 1) + max_occ / kChunk + 2;
}
int64_t emb_hash_max_parts(int64_t max_occ) { return 2 * (max_occ / kChunk) + 2; }

}  // namespace flare
