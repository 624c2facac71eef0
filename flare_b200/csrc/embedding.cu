// Sharded embedding-bag kernels with the all-to-alls fused in (sm_100a).
//
// Forward (one launch per step):
//   entry barrier with every peer (their ids are staged, their previous pooled
//   output has been consumed) -> for every locally owned shard and every
//   (source rank, sample) bag: read the bag's ids straight from the source
//   rank's memory over NVLink (the ids all-to-all), gather + sum/mean pool the
//   local HBM rows in fp32, and store the pooled row straight into the source
//   rank's pooled-output buffer (the pooled all-to-all) -> the ids are also
//   staged locally for the backward -> exit barrier (every owner has written).
//
// Backward (one pass of six short launches, no host sync):
//   1. entry barrier; pull the pooled gradients of every (source, sample) bag
//      for the owned shards (pooled-grad all-to-all) and, in the same launch,
//      count occurrences per row with warp-aggregated atomics (dedup);
//   2-3. exclusive scan of per-unique counts -> segment starts;
//   4. fill: place every occurrence into its row's segment (counters return
//      to zero, so no per-step clearing of the per-row arrays is needed);
//   5. segment reduce in fp32 over fixed-size chunks of the occurrence list
//      (balanced under Zipf skew) and apply the row-wise optimizer in place;
//      rows spanning chunks accumulate into a small carry buffer;
//   6. apply the optimizer to the spanning rows.
//
// Reference behaviour: gather/pool/scatter semantics of
// src/flare/kernels/backends/gpu_cupy.py:52-252 and
// src/flare/ops/sparse_gather.py:40-99 (sum, mean with max(len,1)); the
// reference routes ids and values through Fluxway transport
// (src/flare/runtime/fluxway/workers/dynamic_embedding.py:362-438, 551-681).
#include "embedding.cuh"

namespace flare {
namespace {

constexpr unsigned kFull = 0xffffffffu;
constexpr int kEmbThreads = 256;

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

template <typename TW, int VEC>
__global__ void __launch_bounds__(kEmbThreads) emb_fwd_kernel(EmbFwdParams p) {
  const uint32_t epoch = p.world > 1 ? *reinterpret_cast<volatile uint32_t*>(p.epoch_ctr) + 1u : 0u;
  if (p.world > 1) {
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
        const int* offs = p.peer_offsets[s];
        const int o = d.feature * p.Bl + b;
        fbase = offs[d.feature * p.Bl];
        beg = offs[o];
        len = offs[o + 1] - beg;
        const int slot = sh * p.world + s;
        p.stage_len[static_cast<int64_t>(slot) * p.Bl + b] = len;
        if (b == 0) p.stage_count[slot] = offs[d.feature * p.Bl + p.Bl] - fbase;
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
      const int* vals = p.peer_values[s];
      for (int j = 0; j < maxlen; j += G) {
        int myid = -1;
        if (active && j + l < len) {
          myid = vals[beg + j + l];
          if (stage_ok) {
            p.stage_ids[stage_base + j + l] = myid;
            p.stage_bag[stage_base + j + l] = b;
          }
          if (myid >= d.rows) {
            report_error(p.status, kIndexOutOfRange, d.feature);
            myid = -1;
          }
        }
        const int cnt = min(G, maxlen - j);
        int t = 0;
        for (; t + 4 <= cnt; t += 4) {
          int id[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) id[q] = __shfl_sync(kFull, myid, g * G + t + q);
          float4 r[4][VEC];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const TW* row = wshard + static_cast<int64_t>(id[q] < 0 ? 0 : id[q]) * d.ncols;
#pragma unroll
            for (int v = 0; v < VEC; ++v) r[q][v] = load4<TW>(row + 4 * v);
          }
#pragma unroll
          for (int q = 0; q < 4; ++q) {
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
        if (p.out_dtype == kBF16) {
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

// --------------------------------------------------------------------------
// Backward
// --------------------------------------------------------------------------
__device__ __forceinline__ unsigned lanemask_lt() {
  unsigned m;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

// Phase 1: pooled-gradient all-to-all (pull) fused with dedup counting.
__global__ void __launch_bounds__(kEmbThreads) emb_bwd_pull_count_kernel(EmbBwdParams p) {
  if (p.world > 1) {
    const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(p.epoch_ctr) + 1u;
    const bool ok =
        entry_barrier(p.flags_local, p.peer_flags, p.world, p.rank, p.flag_in, epoch, p.timeout_ns, p.status);
    if (threadIdx.x == 0) {
      // Advance the epoch once every block has read it.
      if (atomicAdd(p.block_counter, 1u) == gridDim.x - 1) {
        *p.block_counter = 0u;
        *p.epoch_ctr = epoch;
      }
    }
    if (!ok) return;
  }
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t nthreads = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int esize = p.grad_dtype == kBF16 ? 2 : 4;
  // ---- pull gradient rows of every owned shard from every source ----
  for (int sh = 0; sh < p.num_shards; ++sh) {
    const ShardDesc d = p.shards[sh];
    const int chunks = d.ncols * esize / 16;
    const int64_t total = static_cast<int64_t>(p.world) * p.Bl * chunks;
    for (int64_t i = tid; i < total; i += nthreads) {
      const int c = static_cast<int>(i % chunks);
      const int64_t bs = i / chunks;  // bs = b * world + s
      const int b = static_cast<int>(bs / p.world);
      const int s = static_cast<int>(bs - static_cast<int64_t>(b) * p.world);
      const char* src = reinterpret_cast<const char*>(p.peer_grad[s]) +
                        (static_cast<int64_t>(b) * p.out_stride + d.out_col) * esize + c * 16;
      char* dst = reinterpret_cast<char*>(p.grad_stage) +
                  ((static_cast<int64_t>(sh * p.world + s) * p.Bl + b) * p.grad_stage_ld) * esize + c * 16;
      *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(src);
    }
  }
  // ---- count occurrences per row (warp-aggregated) ----
  const int lane = lane_id();
  const int64_t gwarp = tid >> 5;
  const int64_t nwarps = nthreads >> 5;
  int local_total = 0;
  for (int sh = 0; sh < p.num_shards; ++sh) {
    const ShardDesc d = p.shards[sh];
    for (int s = 0; s < p.world; ++s) {
      const int slot = sh * p.world + s;
      const int n = min(static_cast<int64_t>(p.stage_count[slot]), p.stage_cap);
      const int* ids = p.stage_ids + static_cast<int64_t>(slot) * p.stage_cap;
      for (int64_t j0 = gwarp * 32; j0 < n; j0 += nwarps * 32) {
        const int64_t j = j0 + lane;
        const int id = j < n ? ids[j] : -1;
        const bool valid = id >= 0 && id < d.rows;
        const unsigned vmask = __ballot_sync(kFull, valid);
        bool fresh = false;
        long long row = 0;
        if (valid) {
          row = d.row_base + id;
          const unsigned peers = __match_any_sync(vmask, row);
          const int leader = __ffs(peers) - 1;
          if (lane == leader) fresh = atomicAdd(p.row_count + row, __popc(peers)) == 0;
        }
        const unsigned fmask = __ballot_sync(kFull, fresh);
        if (fmask) {
          int base = 0;
          const int first = __ffs(fmask) - 1;
          if (lane == first) base = atomicAdd(p.num_unique, __popc(fmask));
          base = __shfl_sync(kFull, base, first);
          if (fresh) {
            const int u = base + __popc(fmask & lanemask_lt());
            p.uniq_row[u] = row;
            p.uniq_shard[u] = sh;
            p.row2u[row] = u;
          }
        }
        if (lane == 0) local_total += __popc(vmask);
      }
    }
  }
  if (lane == 0 && local_total) atomicAdd(p.num_unique + 1, local_total);
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

__global__ void __launch_bounds__(kScanThreads) emb_scan_partial_kernel(EmbBwdParams p) {
  __shared__ int sh[32];
  const int U = p.num_unique[0];
  const int per = (U + kScanBlocks - 1) / kScanBlocks;
  const int lo = min(U, blockIdx.x * per), hi = min(U, lo + per);
  int acc = 0;
  for (int u = lo + threadIdx.x; u < hi; u += blockDim.x) acc += p.row_count[p.uniq_row[u]];
  acc = block_reduce_sum(acc, sh);
  if (threadIdx.x == 0) p.block_sums[blockIdx.x] = acc;
}

__global__ void __launch_bounds__(kScanThreads) emb_scan_final_kernel(EmbBwdParams p) {
  __shared__ int sh[32];
  __shared__ int wsum[32];
  const int U = p.num_unique[0];
  const int per = (U + kScanBlocks - 1) / kScanBlocks;
  const int lo = min(U, blockIdx.x * per), hi = min(U, lo + per);
  int base = 0;
  for (int i = threadIdx.x; i < blockIdx.x; i += blockDim.x) base += p.block_sums[i];
  base = block_reduce_sum(base, sh);
  const int w = warp_id(), l = lane_id();
  for (int t0 = lo; t0 < hi; t0 += blockDim.x) {
    const int u = t0 + threadIdx.x;
    const int c = u < hi ? p.row_count[p.uniq_row[u]] : 0;
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
      wsum[l] = s;  // inclusive prefix over warps
    }
    __syncthreads();
    const int warp_base = w > 0 ? wsum[w - 1] : 0;
    if (u < hi) p.seg_start[u] = base + warp_base + x - c;
    const int tile_total = wsum[blockDim.x / 32 - 1];
    __syncthreads();
    base += tile_total;
  }
  // The last block's running base ends at the grand total (blocks past U own
  // empty ranges), which is the sentinel seg_start[U] = T.
  if (blockIdx.x == kScanBlocks - 1 && threadIdx.x == 0) p.seg_start[U] = base;
}

// Phase 4: scatter occurrences into their segments.
__global__ void __launch_bounds__(kEmbThreads) emb_fill_kernel(EmbBwdParams p) {
  const int lane = lane_id();
  const int64_t gwarp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  for (int sh = 0; sh < p.num_shards; ++sh) {
    const ShardDesc d = p.shards[sh];
    for (int s = 0; s < p.world; ++s) {
      const int slot = sh * p.world + s;
      const int n = min(static_cast<int64_t>(p.stage_count[slot]), p.stage_cap);
      const int* ids = p.stage_ids + static_cast<int64_t>(slot) * p.stage_cap;
      const int* bags = p.stage_bag + static_cast<int64_t>(slot) * p.stage_cap;
      for (int64_t j0 = gwarp * 32; j0 < n; j0 += nwarps * 32) {
        const int64_t j = j0 + lane;
        const int id = j < n ? ids[j] : -1;
        const bool valid = id >= 0 && id < d.rows;
        const unsigned vmask = __ballot_sync(kFull, valid);
        if (valid) {
          const long long row = d.row_base + id;
          const unsigned peers = __match_any_sync(vmask, row);
          const int leader = __ffs(peers) - 1;
          const int k = __popc(peers);
          int old = 0;
          if (lane == leader) old = atomicSub(p.row_count + row, k);
          old = __shfl_sync(peers, old, leader);
          const int u = p.row2u[row];
          const int rank_in_group = __popc(peers & lanemask_lt());
          const int pos = p.seg_start[u] + old - k + rank_in_group;
          p.occ[pos] = (slot * p.Bl) + bags[j];
        }
      }
    }
  }
}

__device__ __forceinline__ float lr_scale(const SparseOptParams& o, float score) {
  switch (o.lr_policy) {
    case kLrSqrtDecay:
      return rsqrtf(fmaxf(score, 1.f));
    case kLrLogDecay:
      return 1.f / (1.f + log1pf(fmaxf(score, 0.f)));
    case kLrInverseDecay:
      return 1.f / fmaxf(score, 1.f);
    case kLrCosineFrequency: {
      const float x = fminf(fmaxf(score, 0.f), o.policy_b) / fmaxf(o.policy_b, 1e-12f);
      return o.policy_a + (1.f - o.policy_a) * 0.5f * (1.f + cospif(x));
    }
    case kLrCustomLut: {
      if (o.lut == nullptr || o.lut_len <= 0) return 1.f;
      const int i = min(static_cast<int>(fmaxf(score, 0.f)), o.lut_len - 1);
      return o.lut[i];
    }
    default:
      return 1.f;
  }
}

// Apply the sparse optimizer to one row; called by a whole warp, lane covers
// columns [col, col + 4*VEC) when col < ncols.
template <typename TW, int VEC>
__device__ __forceinline__ void apply_row_update(const EmbBwdParams& p, const ShardDesc& d, long long row, int col,
                                                 float4 (&g)[VEC], int count) {
  const SparseOptParams& o = p.opt;
  const bool act = col < d.ncols;
  const int64_t local = row - d.row_base;
  const int64_t eoff = d.weight_off + local * d.ncols + col;
  TW* w = reinterpret_cast<TW*>(p.weights) + eoff;
  float lr = o.lr;
  if (o.score != nullptr) {
    float sc = 0.f;
    if (lane_id() == 0) {
      sc = o.score[row] + static_cast<float>(count);
      o.score[row] = sc;
    }
    sc = __shfl_sync(kFull, sc, 0);
    lr *= lr_scale(o, sc);
  }
  float wv[VEC][4];
  float gv[VEC][4];
#pragma unroll
  for (int v = 0; v < VEC; ++v) {
    float4 x = act ? load4<TW>(w + 4 * v) : make_float4(0.f, 0.f, 0.f, 0.f);
    wv[v][0] = x.x; wv[v][1] = x.y; wv[v][2] = x.z; wv[v][3] = x.w;
    gv[v][0] = g[v].x; gv[v][1] = g[v].y; gv[v][2] = g[v].z; gv[v][3] = g[v].w;
#pragma unroll
    for (int e = 0; e < 4; ++e) gv[v][e] += o.weight_decay * wv[v][e];
  }
  if (o.kind == kOptRowwiseAdagrad || o.kind == kOptRowwiseAdam) {
    float sq = 0.f;
    if (act) {
#pragma unroll
      for (int v = 0; v < VEC; ++v)
#pragma unroll
        for (int e = 0; e < 4; ++e) sq += gv[v][e] * gv[v][e];
    }
    sq = warp_sum(sq) / static_cast<float>(d.ncols);
    float st = 0.f;
    if (lane_id() == 0) {
      const float old = o.state_row[row];
      st = o.kind == kOptRowwiseAdagrad ? old + sq : o.beta2 * old + (1.f - o.beta2) * sq;
      o.state_row[row] = st;
    }
    st = __shfl_sync(kFull, st, 0);
    if (o.kind == kOptRowwiseAdagrad) {
      const float scale = lr / (sqrtf(st) + o.eps);
#pragma unroll
      for (int v = 0; v < VEC; ++v)
#pragma unroll
        for (int e = 0; e < 4; ++e) wv[v][e] -= scale * gv[v][e];
    } else {
      const float denom = sqrtf(st / o.bias_corr2) + o.eps;
      if (act) {
#pragma unroll
        for (int v = 0; v < VEC; ++v) {
          float4 m = *reinterpret_cast<float4*>(o.state_m + eoff + 4 * v);
          float* mm = reinterpret_cast<float*>(&m);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            mm[e] = o.beta1 * mm[e] + (1.f - o.beta1) * gv[v][e];
            wv[v][e] -= lr * (mm[e] / o.bias_corr1) / denom;
          }
          *reinterpret_cast<float4*>(o.state_m + eoff + 4 * v) = m;
        }
      }
    }
  } else if (act) {
    if (o.kind == kOptSgd) {
#pragma unroll
      for (int v = 0; v < VEC; ++v)
#pragma unroll
        for (int e = 0; e < 4; ++e) wv[v][e] -= lr * gv[v][e];
    } else if (o.kind == kOptAdagrad) {
#pragma unroll
      for (int v = 0; v < VEC; ++v) {
        float4 m = *reinterpret_cast<float4*>(o.state_m + eoff + 4 * v);
        float* mm = reinterpret_cast<float*>(&m);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          mm[e] += gv[v][e] * gv[v][e];
          wv[v][e] -= lr * gv[v][e] / (sqrtf(mm[e]) + o.eps);
        }
        *reinterpret_cast<float4*>(o.state_m + eoff + 4 * v) = m;
      }
    } else if (o.kind == kOptAdam) {
#pragma unroll
      for (int v = 0; v < VEC; ++v) {
        float4 m = *reinterpret_cast<float4*>(o.state_m + eoff + 4 * v);
        float4 s2 = *reinterpret_cast<float4*>(o.state_v + eoff + 4 * v);
        float* mm = reinterpret_cast<float*>(&m);
        float* vv = reinterpret_cast<float*>(&s2);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          mm[e] = o.beta1 * mm[e] + (1.f - o.beta1) * gv[v][e];
          vv[e] = o.beta2 * vv[e] + (1.f - o.beta2) * gv[v][e] * gv[v][e];
          wv[v][e] -= lr * (mm[e] / o.bias_corr1) / (sqrtf(vv[e] / o.bias_corr2) + o.eps);
        }
        *reinterpret_cast<float4*>(o.state_m + eoff + 4 * v) = m;
        *reinterpret_cast<float4*>(o.state_v + eoff + 4 * v) = s2;
      }
    }
  }
  if (act) {
#pragma unroll
    for (int v = 0; v < VEC; ++v)
      store4<TW>(w + 4 * v, make_float4(wv[v][0], wv[v][1], wv[v][2], wv[v][3]));
  }
}

template <typename TG, int VEC>
__device__ __forceinline__ void add_grad_row(const EmbBwdParams& p, int gidx, int col, bool act, float scale,
                                             float4 (&acc)[VEC]) {
  if (!act) return;
  const TG* src = reinterpret_cast<const TG*>(p.grad_stage) + static_cast<int64_t>(gidx) * p.grad_stage_ld + col;
#pragma unroll
  for (int v = 0; v < VEC; ++v) acc[v] = f4_add(acc[v], f4_scale(load4<TG>(src + 4 * v), scale));
}

// Phase 5: fixed-size chunks of the grouped occurrence list -> fp32 segment
// sums -> optimizer (rows wholly inside the chunk) or carry (spanning rows).
__device__ __forceinline__ void resolve_sparse_step(EmbBwdParams& p) {
  if (p.opt.step_ptr != nullptr) {
    const float t = static_cast<float>(*p.opt.step_ptr);
    p.opt.bias_corr1 = 1.f - powf(p.opt.beta1, t);
    p.opt.bias_corr2 = 1.f - powf(p.opt.beta2, t);
  }
}

template <typename TW, typename TG, int VEC>
__global__ void __launch_bounds__(kEmbThreads) emb_reduce_apply_kernel(EmbBwdParams p) {
  resolve_sparse_step(p);
  const int U = p.num_unique[0];
  const int T = p.num_unique[1];
  if (U == 0) return;
  const int lane = lane_id();
  const int col = lane * 4 * VEC;
  const int64_t gwarp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  const int nchunks = (T + p.chunk - 1) / p.chunk;
  for (int64_t c = gwarp; c < nchunks; c += nwarps) {
    const int cb = static_cast<int>(c) * p.chunk;
    const int ce = min(T, cb + p.chunk);
    // largest u with seg_start[u] <= cb
    int lo = 0, hi = U;  // invariant seg_start[lo] <= cb < seg_start[hi] (seg_start[U] = T > cb)
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (p.seg_start[mid] <= cb) lo = mid; else hi = mid;
    }
    for (int u = lo; u < U; ++u) {
      const int ss = p.seg_start[u];
      if (ss >= ce) break;
      const int se = p.seg_start[u + 1];
      const int a = max(ss, cb), e = min(se, ce);
      const ShardDesc d = p.shards[p.uniq_shard[u]];
      const bool act = col < d.ncols;
      const bool mean = d.pooling == 1;
      float4 acc[VEC];
#pragma unroll
      for (int v = 0; v < VEC; ++v) acc[v] = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int q0 = a; q0 < e; q0 += 32) {
        const int mine = q0 + lane < e ? p.occ[q0 + lane] : 0;
        float myscale = 1.f;
        if (mean && q0 + lane < e) myscale = 1.f / static_cast<float>(max(1, p.stage_len[mine]));
        const int cnt = min(32, e - q0);
        int t = 0;
        for (; t + 2 <= cnt; t += 2) {
          const int g0 = __shfl_sync(kFull, mine, t), g1 = __shfl_sync(kFull, mine, t + 1);
          const float s0 = __shfl_sync(kFull, myscale, t), s1 = __shfl_sync(kFull, myscale, t + 1);
          add_grad_row<TG, VEC>(p, g0, col, act, s0, acc);
          add_grad_row<TG, VEC>(p, g1, col, act, s1, acc);
        }
        for (; t < cnt; ++t) {
          const int g0 = __shfl_sync(kFull, mine, t);
          const float s0 = __shfl_sync(kFull, myscale, t);
          add_grad_row<TG, VEC>(p, g0, col, act, s0, acc);
        }
      }
      if (ss >= cb && se <= ce) {
        apply_row_update<TW, VEC>(p, d, p.uniq_row[u], col, acc, se - ss);
      } else {
        const int start_chunk = ss / p.chunk;
        if (act) {
          float* dst = p.carry + static_cast<int64_t>(start_chunk) * (128 * VEC) + col;
#pragma unroll
          for (int v = 0; v < VEC; ++v) {
            atomicAdd(dst + 4 * v + 0, acc[v].x);
            atomicAdd(dst + 4 * v + 1, acc[v].y);
            atomicAdd(dst + 4 * v + 2, acc[v].z);
            atomicAdd(dst + 4 * v + 3, acc[v].w);
          }
        }
        if (ss >= cb && lane == 0) p.span_u[c] = u;
      }
    }
  }
}

// Phase 6: rows whose occurrences spanned several chunks.
template <typename TW, int VEC>
__global__ void __launch_bounds__(kEmbThreads) emb_finalize_spanning_kernel(EmbBwdParams p) {
  resolve_sparse_step(p);
  const int T = p.num_unique[1];
  const int lane = lane_id();
  const int col = lane * 4 * VEC;
  const int64_t gwarp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  const int nchunks = (T + p.chunk - 1) / p.chunk;
  for (int64_t c = gwarp; c < nchunks; c += nwarps) {
    const int u = p.span_u[c];
    if (u < 0) continue;
    const ShardDesc d = p.shards[p.uniq_shard[u]];
    float* src = p.carry + c * (128 * VEC) + col;
    float4 acc[VEC];
#pragma unroll
    for (int v = 0; v < VEC; ++v) {
      acc[v] = *reinterpret_cast<float4*>(src + 4 * v);
      *reinterpret_cast<float4*>(src + 4 * v) = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    apply_row_update<TW, VEC>(p, d, p.uniq_row[u], col, acc, p.seg_start[u + 1] - p.seg_start[u]);
    if (lane == 0) p.span_u[c] = -1;
  }
}

template <typename TW, int VEC>
void fwd_dispatch(const EmbFwdParams& p, int grid, cudaStream_t s) {
  emb_fwd_kernel<TW, VEC><<<grid, kEmbThreads, 0, s>>>(p);
  count_launch();
}

template <typename TW, typename TG, int VEC>
void bwd_tail(const EmbBwdParams& p, int grid, cudaStream_t s) {
  emb_reduce_apply_kernel<TW, TG, VEC><<<grid, kEmbThreads, 0, s>>>(p);
  emb_finalize_spanning_kernel<TW, VEC><<<grid, kEmbThreads, 0, s>>>(p);
  count_launch(2);
}

template <typename TW, int VEC>
void bwd_tail_g(const EmbBwdParams& p, int grid, cudaStream_t s) {
  if (p.grad_dtype == kBF16) bwd_tail<TW, __nv_bfloat16, VEC>(p, grid, s);
  else bwd_tail<TW, float, VEC>(p, grid, s);
}

}  // namespace

void emb_forward(const EmbFwdParams& p, int grid, cudaStream_t s) {
  FLARE_CHECK(grid > 0, "grid must be positive");
  FLARE_CHECK(p.vec == 1 || p.vec == 2, "vec must be 1 or 2");
  if (p.w_dtype == kF32) {
    if (p.vec == 1) fwd_dispatch<float, 1>(p, grid, s); else fwd_dispatch<float, 2>(p, grid, s);
  } else if (p.w_dtype == kF16) {
    if (p.vec == 1) fwd_dispatch<__half, 1>(p, grid, s); else fwd_dispatch<__half, 2>(p, grid, s);
  } else {
    if (p.vec == 1) fwd_dispatch<__nv_bfloat16, 1>(p, grid, s); else fwd_dispatch<__nv_bfloat16, 2>(p, grid, s);
  }
  FLARE_CUDA_CHECK(cudaGetLastError());
}

void emb_backward(const EmbBwdParams& p, int ncols_max, int grid, cudaStream_t s) {
  FLARE_CHECK(ncols_max > 0 && ncols_max <= 256, "embedding shard width must be in (0, 256]");
  FLARE_CUDA_CHECK(cudaMemsetAsync(p.num_unique, 0, 2 * sizeof(int), s));
  emb_bwd_pull_count_kernel<<<grid, kEmbThreads, 0, s>>>(p);
  emb_scan_partial_kernel<<<kScanBlocks, kScanThreads, 0, s>>>(p);
  emb_scan_final_kernel<<<kScanBlocks, kScanThreads, 0, s>>>(p);
  emb_fill_kernel<<<grid, kEmbThreads, 0, s>>>(p);
  count_launch(4);
  const int vec = ncols_max > 128 ? 2 : 1;
  if (p.w_dtype == kF32) {
    if (vec == 1) bwd_tail_g<float, 1>(p, grid, s); else bwd_tail_g<float, 2>(p, grid, s);
  } else if (p.w_dtype == kF16) {
    if (vec == 1) bwd_tail_g<__half, 1>(p, grid, s); else bwd_tail_g<__half, 2>(p, grid, s);
  } else {
    if (vec == 1) bwd_tail_g<__nv_bfloat16, 1>(p, grid, s); else bwd_tail_g<__nv_bfloat16, 2>(p, grid, s);
  }
  FLARE_CUDA_CHECK(cudaGetLastError());
}

}  // namespace flare
