// Persistent tcgen05 GEMM with the tensor/FSDP-parallel collectives fused in.
//
//   C[M,N] = epi( A[M,K] . B[N,K]^T )
//
// One kernel covers three distributed patterns of the DCN-v2 tower:
//
//  * all-gather -> GEMM.  An operand whose stored rows are sharded over a
//    group of R ranks (activations under sequence-parallel TP, or weights
//    under FSDP) lives in a "full" buffer in symmetric memory; each rank owns
//    the rows [q*S, (q+1)*S).  Two copy warps per CTA pull the peers' rows
//    chunk by chunk into the local full buffer over NVLink (plain 16-byte
//    loads from peer memory, so every remote byte crosses NVLink once) and
//    publish a per-chunk ready flag.  The TMA producer waits for the flags of
//    the rows a tile needs, then loads from LOCAL memory only.  Tiles that
//    need only local rows are scheduled first, so the copies overlap math.
//    No TMA load ever reads a peer's memory and no load uses multicast.
//  * GEMM -> reduce-scatter over output rows (row-parallel TP).  Every rank
//    computes a full partial product; tiles of rows owned by a peer are
//    converted to bf16 and stored into that peer's receive slot (P2P
//    stores), then flagged.  The owner computes its own tiles last, waits for
//    the peers' flags of the tile, adds their partials and runs the epilogue.
//  * a plain persistent GEMM (R = 1), with the same epilogues.
//
// Structure: 384 threads.  warp 0 lane 0 = TMA producer (4-stage ring of
// 128-byte-swizzled 128x64 / 256x64 bf16 tiles); warp 1 lane 0 = tcgen05.mma
// issuer into one of two TMEM accumulators (2 x 256 columns), so the
// epilogue of tile i overlaps the MMAs of tile i+1; warps 2-9 = epilogue
// (warp w reads TMEM lanes 32*(w%4)..+31, columns [128*h, 128*h+128) with
// h = (w-2)/4); warps 10-11 = copy warps.
// The launch is cooperative (all CTAs co-resident), which the cross-CTA
// chunk flags rely on; every wait is bounded and reports a status code.
//
// Epilogues: bias, ReLU, ReLU-backward mask, column sums (bias gradients),
// fp32 accumulate, "cross" (z = acc + bias; out = x0 * z + xl, z also
// stored: the DCN-v2 cross layer) and "residual" (out = acc + aux).
//
// The reference runs these layers through XLA with NCCL collectives between
// them (src/flare/jax/training/engines/distributed.py:612-716 for the step,
// src/flare/jax/training/zero/collectives.py:26-40 for the collectives); it
// has no tensor parallelism.
#include "gemm.cuh"
#include "sm100.cuh"

#include <cudaTypedefs.h>

#include <algorithm>
#include <cstring>

namespace flare {

namespace {

constexpr int kBM = 128;
constexpr int kBN = 256;
constexpr int kBK = 64;
constexpr int kStages = 4;
constexpr int kThreads = 384;
constexpr int kEpiWarps = 8;   // warps 2..9: two per TMEM lane quarter, each owning half of the columns
constexpr int kCopyWarp0 = 2 + kEpiWarps;
constexpr int kTileA = kBM * kBK * 2;  // 16 KiB
constexpr int kTileB = kBN * kBK * 2;  // 32 KiB
constexpr int kOffB = kStages * kTileA;
constexpr int kOffBar = kOffB + kStages * kTileB;
constexpr int kBarBytes = 256;
constexpr int kSmem = kOffBar + kBarBytes + 1024;
constexpr int kMaxRanks = 8;
constexpr int kCopyUnroll = 8;

__device__ __forceinline__ void st_release_gpu(uint32_t* p, uint32_t v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}
__device__ __forceinline__ bool wait_local_geq(const uint32_t* flag, uint32_t target, uint64_t timeout_ns,
                                               int* status, int detail) {
  if (static_cast<int32_t>(ld_acquire_gpu(flag) - target) >= 0) return true;
  const uint64_t t0 = global_timer_ns();
  while (static_cast<int32_t>(ld_acquire_gpu(flag) - target) < 0) {
    if (global_timer_ns() - t0 > timeout_ns) {
      report_error(status, kTimeoutPeerSignal, detail);
      return false;
    }
    __nanosleep(32);
  }
  return true;
}

struct GatherDev {
  const __nv_bfloat16* src[kMaxRanks];  // src[q]: rank q's full buffer (peer address)
  __nv_bfloat16* dst;                   // this rank's full buffer
  int64_t ld;                           // row pitch (elements), same on every rank
  int64_t rows_per_rank;                // S
  int64_t total_rows;                   // R * S
  int row_vecs;                         // 16-byte vectors copied per row
  int chunk_rows;
  int nranks, my;
  int pieces;                           // copy work items per chunk
  int piece_vecs;                       // 16-byte vectors per work item
  uint32_t* ready;                      // per chunk: epoch when its rows are local
  uint32_t* done;                       // per chunk: pieces copied so far this launch
};

struct DistParams {
  int M, N, K, num_k_tiles, n_tiles;
  const int* tiles;
  int num_tiles;
  const int* chunks;
  int num_chunks;
  int gather_a, gather_b;
  GatherDev ga, gb;
  void* C;
  int64_t ldc;
  int c_dtype, accumulate;
  const __nv_bfloat16* bias;
  int act;
  float alpha;
  const __nv_bfloat16* mask;
  int64_t ldm;
  const __nv_bfloat16* aux0;
  int64_t ld0;
  const __nv_bfloat16* aux1;
  int64_t ld1;
  __nv_bfloat16* zout;
  int64_t ldz;
  int epi;  // 0 plain, 1 cross, 2 residual
  float* colsum;
  int rs, rs_nranks, rs_my, rs_rows;
  __nv_bfloat16* rs_recv_peer[kMaxRanks];
  const __nv_bfloat16* rs_recv_local;
  int64_t ld_recv;
  uint32_t* rs_flag_peer[kMaxRanks];
  const uint32_t* rs_flag_local;
  int world, rank;
  uint32_t* bar_local;
  uint32_t* bar_peer[kMaxRanks];
  uint32_t* ctl;  // [0] epoch, [1] block counter, [2] barrier passed
  int* status;
  uint64_t timeout_ns;
};

// Wait until the chunks covering stored rows [r0, r0+n) of a gathered operand are local.
__device__ __forceinline__ bool wait_rows(const GatherDev& g, int64_t r0, int n, uint32_t epoch, uint64_t timeout_ns,
                                          int* status) {
  const int64_t r1 = min(r0 + n, g.total_rows);
  for (int64_t c = r0 / g.chunk_rows; c * g.chunk_rows < r1; ++c) {
    const int owner = static_cast<int>((c * g.chunk_rows) / g.rows_per_rank);
    if (owner == g.my) continue;
    if (!wait_local_geq(g.ready + c, epoch, timeout_ns, status, 400 + owner)) return false;
  }
  fence_proxy_async_global();
  return true;
}

// One warp copies piece `piece` of chunk `ci` of a gathered operand from its
// owner into the local full buffer.  The warp that completes the chunk's last
// piece resets the chunk's counter and publishes its ready flag.
__device__ __forceinline__ void copy_piece(const GatherDev& g, int64_t ci, int piece, int lane, uint32_t epoch) {
  const int64_t r0 = ci * g.chunk_rows;
  const int owner = static_cast<int>(r0 / g.rows_per_rank);
  const int nrows = static_cast<int>(min(static_cast<int64_t>(g.chunk_rows), g.total_rows - r0));
  const uint4* src = reinterpret_cast<const uint4*>(g.src[owner] + r0 * g.ld);
  uint4* dst = reinterpret_cast<uint4*>(g.dst + r0 * g.ld);
  const int64_t ldv = g.ld / 8;
  const int64_t total = static_cast<int64_t>(nrows) * g.row_vecs;
  const int64_t vb = static_cast<int64_t>(piece) * g.piece_vecs;
  const int64_t ve = min(total, vb + g.piece_vecs);
  for (int64_t v0 = vb + lane; v0 < ve; v0 += 32 * kCopyUnroll) {
    uint4 buf[kCopyUnroll];
    int64_t off[kCopyUnroll];
#pragma unroll
    for (int u = 0; u < kCopyUnroll; ++u) {
      const int64_t v = v0 + 32 * u;
      off[u] = -1;
      if (v < ve) {
        const int64_t rr = v / g.row_vecs, cc = v - rr * g.row_vecs;
        off[u] = rr * ldv + cc;
        buf[u] = __ldcg(src + off[u]);
      }
    }
#pragma unroll
    for (int u = 0; u < kCopyUnroll; ++u)
      if (off[u] >= 0) dst[off[u]] = buf[u];
  }
  // generic-proxy stores -> visible to the TMA (async proxy) reads of other CTAs
  fence_proxy_async_global();
  __threadfence();
  __syncwarp();
  if (lane == 0) {
    const uint32_t prev = atomicAdd(g.done + ci, 1u);
    if (prev + 1 == static_cast<uint32_t>(g.pieces)) {
      g.done[ci] = 0u;
      __threadfence();
      st_release_gpu(g.ready + ci, epoch);
    }
  }
}

__device__ __forceinline__ uint4 pack8(const float* v) {
  uint4 u;
  uint32_t* w = reinterpret_cast<uint32_t*>(&u);
#pragma unroll
  for (int t = 0; t < 4; ++t) {
    __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * t], v[2 * t + 1]);
    w[t] = *reinterpret_cast<uint32_t*>(&h);
  }
  return u;
}
__device__ __forceinline__ void unpack8_add(uint4 u, float* v) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int t = 0; t < 4; ++t) {
    const float2 f = __bfloat1622float2(h[t]);
    v[2 * t] += f.x;
    v[2 * t + 1] += f.y;
  }
}
__device__ __forceinline__ void unpack8(uint4 u, float* v) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int t = 0; t < 4; ++t) {
    const float2 f = __bfloat1622float2(h[t]);
    v[2 * t] = f.x;
    v[2 * t + 1] = f.y;
  }
}

template <bool A_MN, bool B_MN>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_dist_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                     const __grid_constant__ DistParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* empty_bar = full_bar + kStages;
  uint64_t* tfull_bar = empty_bar + kStages;  // [2]
  uint64_t* tempty_bar = tfull_bar + 2;       // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty_bar + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id();
  const int lane = lane_id();
  const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(p.ctl) + 1u;
  const bool need_barrier = p.world > 1 && (p.gather_a || p.gather_b || p.rs);

  if (threadIdx.x == 0) {
    sm100::tma_prefetch_desc(&tmap_a);
    sm100::tma_prefetch_desc(&tmap_b);
    for (int s = 0; s < kStages; ++s) {
      sm100::mbar_init(&full_bar[s], 1);
      sm100::mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      sm100::mbar_init(&tfull_bar[b], 1);
      sm100::mbar_init(&tempty_bar[b], kEpiWarps);
    }
    *abort_flag = 0;
    sm100::fence_mbar_init();
  }
  if (warp == 0) {
    sm100::tmem_alloc(tmem_slot, 2 * kBN);
    sm100::tmem_relinquish();
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------ producer ------------------------------
      int it = 0;
      for (int ti = blockIdx.x; ti < p.num_tiles && !*abort_flag; ti += gridDim.x) {
        const int mt = p.tiles[ti] >> 16, nt = p.tiles[ti] & 0xFFFF;
        const int m0 = mt * kBM, n0 = nt * kBN;
        bool ok = true;
        if (p.gather_a && !A_MN) ok = wait_rows(p.ga, m0, kBM, epoch, p.timeout_ns, p.status);
        if (ok && p.gather_b && !B_MN) ok = wait_rows(p.gb, n0, kBN, epoch, p.timeout_ns, p.status);
        for (int kt = 0; kt < p.num_k_tiles && ok; ++kt, ++it) {
          const int s = it % kStages;
          if (it >= kStages) {
            if (!sm100::mbar_wait(&empty_bar[s], ((it / kStages) - 1) & 1, p.timeout_ns, p.status, 100 + s)) {
              ok = false;
              break;
            }
          }
          const int k0 = kt * kBK;
          if (p.gather_a && A_MN) ok = wait_rows(p.ga, k0, kBK, epoch, p.timeout_ns, p.status);
          if (ok && p.gather_b && B_MN) ok = wait_rows(p.gb, k0, kBK, epoch, p.timeout_ns, p.status);
          if (!ok) break;
          uint8_t* sa = smem + s * kTileA;
          uint8_t* sb = smem + kOffB + s * kTileB;
          sm100::mbar_arrive_expect_tx(&full_bar[s], kTileA + kTileB);
          if constexpr (!A_MN) {
            sm100::tma_load_2d(sa, &tmap_a, &full_bar[s], k0, m0);
          } else {
#pragma unroll
            for (int j = 0; j < kBM / 64; ++j) sm100::tma_load_2d(sa + j * 8192, &tmap_a, &full_bar[s], m0 + 64 * j, k0);
          }
          if constexpr (!B_MN) {
            sm100::tma_load_2d(sb, &tmap_b, &full_bar[s], k0, n0);
          } else {
#pragma unroll
            for (int j = 0; j < kBN / 64; ++j) sm100::tma_load_2d(sb + j * 8192, &tmap_b, &full_bar[s], n0 + 64 * j, k0);
          }
        }
        if (!ok) *abort_flag = 1;
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------ MMA issuer ----------------------------
      constexpr uint32_t idesc = sm100::make_idesc_bf16(kBM, kBN, A_MN, B_MN);
      int it = 0, local = 0;
      for (int ti = blockIdx.x; ti < p.num_tiles && !*abort_flag; ti += gridDim.x, ++local) {
        const int b = local & 1, use = local >> 1;
        if (local >= 2 && !sm100::mbar_wait(&tempty_bar[b], (use - 1) & 1, p.timeout_ns, p.status, 250 + b)) {
          *abort_flag = 1;
          break;
        }
        sm100::tc_fence_after();
        const uint32_t d = tmem_base + static_cast<uint32_t>(b * kBN);
        bool ok = true;
        for (int kt = 0; kt < p.num_k_tiles; ++kt, ++it) {
          const int s = it % kStages;
          if (!sm100::mbar_wait(&full_bar[s], (it / kStages) & 1, p.timeout_ns, p.status, 200 + s)) {
            ok = false;
            break;
          }
          sm100::tc_fence_after();
          const uint32_t sa = smem_u32(smem + s * kTileA);
          const uint32_t sb = smem_u32(smem + kOffB + s * kTileB);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            const uint64_t da = A_MN ? sm100::make_smem_desc(sa + k * 2048, 8192, 1024)
                                     : sm100::make_smem_desc(sa + k * 32, 16, 1024);
            const uint64_t db = B_MN ? sm100::make_smem_desc(sb + k * 2048, 8192, 1024)
                                     : sm100::make_smem_desc(sb + k * 32, 16, 1024);
            sm100::mma_f16_ss(d, da, db, idesc, (kt > 0 || k > 0) ? 1u : 0u);
          }
          sm100::mma_commit(&empty_bar[s]);
        }
        if (!ok) {
          *abort_flag = 1;
          break;
        }
        sm100::mma_commit(&tfull_bar[b]);
      }
    }
  } else if (warp < kCopyWarp0) {
    // -------------------------------- epilogue --------------------------------
    const int quarter = warp & 3;  // TMEM lane quarter this warp may access
    const int half = (warp - 2) >> 2;  // which 128 columns of the tile
    const int slot = quarter * 2 + half;
    const int tiles_per_rank = p.rs ? (p.rs_rows / kBM) * p.n_tiles : 0;
    bool barrier_seen = !need_barrier;
    int local = 0;
    for (int ti = blockIdx.x; ti < p.num_tiles && !*abort_flag; ti += gridDim.x, ++local) {
      const int b = local & 1, use = local >> 1;
      const int mt = p.tiles[ti] >> 16, nt = p.tiles[ti] & 0xFFFF;
      const int m0 = mt * kBM, n0 = nt * kBN;
      if (!sm100::mbar_wait(&tfull_bar[b], use & 1, p.timeout_ns, p.status, 300 + b)) {
        *abort_flag = 1;
        break;
      }
      sm100::tc_fence_after();
      const int row = m0 + quarter * 32 + lane;
      const bool row_ok = row < p.M;
      // reduce-scatter role of this tile
      int owner = -1, lrow = row, tile_local = 0;
      bool send = false;
      if (p.rs) {
        owner = m0 / p.rs_rows;
        lrow = row - owner * p.rs_rows;
        tile_local = (mt - owner * (p.rs_rows / kBM)) * p.n_tiles + nt;
        send = owner != p.rs_my;
        if (!barrier_seen) {
          if (!wait_local_geq(p.ctl + 2, epoch, p.timeout_ns, p.status, 500)) {
            *abort_flag = 1;
            break;
          }
          barrier_seen = true;
        }
        if (!send) {
          bool ok = true;
          for (int q = 0; q < p.rs_nranks && ok; ++q) {
            if (q == p.rs_my) continue;
            ok = wait_flag_geq(p.rs_flag_local + (static_cast<int64_t>(q) * tiles_per_rank + tile_local) * 8 + slot,
                               epoch, p.timeout_ns, p.status, 600 + q);
          }
          if (!ok) {
            *abort_flag = 1;
            break;
          }
        }
      }
      const uint32_t tbase = tmem_base + static_cast<uint32_t>(b * kBN) + (static_cast<uint32_t>(quarter * 32) << 16);
#pragma unroll 1
      for (int c = half * (kBN / 2); c < (half + 1) * (kBN / 2); c += 32) {
        const int ncol = n0 + c;
        if (ncol >= p.N) break;  // warp-uniform
        uint32_t r[32];
        sm100::tmem_ld_32x32b_x32(tbase + c, r);
        sm100::tmem_ld_wait();
        const bool full_chunk = ncol + 32 <= p.N;
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]) * p.alpha;
        if (send) {
          // Partial tile -> owner.  Receive layout: one 2 KiB block per (sender, tile,
          // quarter, 32-column chunk), element (row r, col 8q+e) at q*256 + r*8 + e, so
          // each warp-wide 16-byte store writes 512 contiguous bytes over NVLink.
          __nv_bfloat16* blk = p.rs_recv_peer[owner] +
                               ((((static_cast<int64_t>(p.rs_my) * tiles_per_rank + tile_local) * 4 + quarter) * 8 +
                                 (c >> 5)) << 10);
#pragma unroll
          for (int q = 0; q < 4; ++q) *reinterpret_cast<uint4*>(blk + q * 256 + lane * 8) = pack8(v + 8 * q);
          continue;
        }
        if (p.rs) {
          for (int q = 0; q < p.rs_nranks; ++q) {
            if (q == p.rs_my) continue;
            const __nv_bfloat16* blk = p.rs_recv_local +
                                       ((((static_cast<int64_t>(q) * tiles_per_rank + tile_local) * 4 + quarter) * 8 +
                                         (c >> 5)) << 10);
#pragma unroll
            for (int t = 0; t < 4; ++t)
              unpack8_add(__ldcg(reinterpret_cast<const uint4*>(blk + t * 256 + lane * 8)), v + 8 * t);
          }
        }
        // epilogue math
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          if (p.bias != nullptr && (full_chunk || ncol + j < p.N)) v[j] += __bfloat162float(p.bias[ncol + j]);
        }
        if (p.epi == 1 && row_ok) {
          // cross layer: z = acc + bias (stored), out = x0 * z + xl
          float x0[32], xl[32];
          const __nv_bfloat16* a0 = p.aux0 + static_cast<int64_t>(lrow) * p.ld0 + ncol;
          const __nv_bfloat16* a1 = p.aux1 + static_cast<int64_t>(lrow) * p.ld1 + ncol;
          __nv_bfloat16* zr = p.zout + static_cast<int64_t>(lrow) * p.ldz + ncol;
          if (full_chunk) {
#pragma unroll
            for (int t = 0; t < 4; ++t) {
              unpack8(*reinterpret_cast<const uint4*>(a0 + 8 * t), x0 + 8 * t);
              unpack8(*reinterpret_cast<const uint4*>(a1 + 8 * t), xl + 8 * t);
              *reinterpret_cast<uint4*>(zr + 8 * t) = pack8(v + 8 * t);
            }
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const bool in = ncol + j < p.N;
              x0[j] = in ? __bfloat162float(a0[j]) : 0.f;
              xl[j] = in ? __bfloat162float(a1[j]) : 0.f;
              if (in) zr[j] = __float2bfloat16_rn(v[j]);
            }
          }
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = x0[j] * v[j] + xl[j];
        } else if (p.epi == 2 && row_ok) {
          const __nv_bfloat16* a1 = p.aux1 + static_cast<int64_t>(lrow) * p.ld1 + ncol;
          if (full_chunk) {
#pragma unroll
            for (int t = 0; t < 4; ++t) unpack8_add(*reinterpret_cast<const uint4*>(a1 + 8 * t), v + 8 * t);
          } else {
            _Pragma("unroll") for (int j = 0; j < 32; ++j) if (ncol + j < p.N) v[j] += __bfloat162float(a1[j]);
          }
        }
        if (p.act == 1) {
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = fmaxf(v[j], 0.f);
        }
        if (p.mask != nullptr && row_ok) {
          const __nv_bfloat16* mrow = p.mask + static_cast<int64_t>(lrow) * p.ldm + ncol;
          if (full_chunk) {
#pragma unroll
            for (int t = 0; t < 4; ++t) {
              float mv[8];
              unpack8(*reinterpret_cast<const uint4*>(mrow + 8 * t), mv);
#pragma unroll
              for (int e = 0; e < 8; ++e) v[8 * t + e] = mv[e] > 0.f ? v[8 * t + e] : 0.f;
            }
          } else {
            _Pragma("unroll") for (int j = 0; j < 32; ++j) if (ncol + j < p.N) v[j] = __bfloat162float(mrow[j]) > 0.f ? v[j] : 0.f;
          }
        }
        if (!row_ok) {
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = 0.f;
        }
        if (p.colsum != nullptr) {
          float t[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) t[j] = v[j];
#pragma unroll
          for (int o = 16; o >= 1; o >>= 1) {
            const bool upper = (lane & o) != 0;
#pragma unroll
            for (int j = 0; j < o; ++j) {
              const float snd = upper ? t[j] : t[j + o];
              const float keep = upper ? t[j + o] : t[j];
              t[j] = keep + __shfl_xor_sync(0xffffffffu, snd, o);
            }
          }
          if (ncol + lane < p.N) atomicAdd(p.colsum + ncol + lane, t[0]);
        }
        if (!row_ok) continue;
        if (p.c_dtype == kBF16) {
          __nv_bfloat16* crow = reinterpret_cast<__nv_bfloat16*>(p.C) + static_cast<int64_t>(lrow) * p.ldc + ncol;
          if (full_chunk) {
#pragma unroll
            for (int q = 0; q < 4; ++q) *reinterpret_cast<uint4*>(crow + 8 * q) = pack8(v + 8 * q);
          } else {
            _Pragma("unroll") for (int j = 0; j < 32; ++j) if (ncol + j < p.N) crow[j] = __float2bfloat16_rn(v[j]);
          }
        } else {
          float* crow = reinterpret_cast<float*>(p.C) + static_cast<int64_t>(lrow) * p.ldc + ncol;
          if (full_chunk) {
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              float4 o = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
              if (p.accumulate) o = f4_add(o, *reinterpret_cast<const float4*>(crow + 4 * q));
              *reinterpret_cast<float4*>(crow + 4 * q) = o;
            }
          } else {
            _Pragma("unroll") for (int j = 0; j < 32; ++j) if (ncol + j < p.N) crow[j] = p.accumulate ? crow[j] + v[j] : v[j];
          }
        }
      }
      // release the TMEM accumulator to the MMA warp
      sm100::tc_fence_before();
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(&tempty_bar[b]);
      if (send) {
        // this warp's 32 rows of the tile are in the owner's memory: publish them
        // (one flag per tile quarter and column half, so the warps never wait on each other)
        __threadfence_system();
        __syncwarp();
        if (lane == 0) {
          fence_sys();
          st_release_sys(p.rs_flag_peer[owner] + (static_cast<int64_t>(p.rs_my) * tiles_per_rank + tile_local) * 8 + slot,
                         epoch);
        }
      }
    }
  } else {
    // ------------------------------- copy warps -------------------------------
    const bool copier = p.gather_a || p.gather_b;
    if (need_barrier && blockIdx.x == 0 && warp == kCopyWarp0 && lane == 0) {
      // whole-world entry barrier: every rank finished writing what peers read
      fence_sys();
      for (int s = 0; s < p.world; ++s) st_release_sys(p.bar_peer[s] + p.rank, epoch);
      bool ok = true;
      for (int s = 0; s < p.world && ok; ++s) ok = wait_flag_geq(p.bar_local + s, epoch, p.timeout_ns, p.status, 700 + s);
      if (ok) st_release_sys(p.ctl + 2, epoch);
      else *abort_flag = 1;
    }
    if (copier) {
      bool ok = !need_barrier || wait_flag_geq(p.ctl + 2, epoch, p.timeout_ns, p.status, 501);
      const int cw = blockIdx.x * 2 + (warp - kCopyWarp0);
      for (int c = cw; c < p.num_chunks && ok; c += gridDim.x * 2) {
        const uint32_t item = static_cast<uint32_t>(p.chunks[c]);
        const int op = static_cast<int>(item >> 31);
        const int64_t ci = (item >> 12) & 0x7FFFF;
        const int piece = static_cast<int>(item & 0xFFF);
        // two call sites keep each GatherDev in parameter space (no local copy)
        if (op) copy_piece(p.gb, ci, piece, lane, epoch);
        else copy_piece(p.ga, ci, piece, lane, epoch);
      }
      if (!ok) *abort_flag = 1;
    }
  }

  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 0) sm100::tmem_dealloc(tmem_base, 2 * kBN);
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(p.ctl + 1, 1u) == gridDim.x - 1) {
      p.ctl[1] = 0u;
      __threadfence();
      *reinterpret_cast<volatile uint32_t*>(p.ctl) = epoch;
    }
  }
}

template <bool A_MN, bool B_MN>
void launch(const DistGemmArgs& a, cudaStream_t stream) {
  auto kern = gemm_dist_kernel<A_MN, B_MN>;
  static bool attr_set = false;
  if (!attr_set) {
    FLARE_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem));
    attr_set = true;
  }
  const GemmArgs& g = a.g;
  CUtensorMap ta = A_MN ? make_tmap_bf16(g.A, g.M, g.K, g.lda, kBK) : make_tmap_bf16(g.A, g.K, g.M, g.lda, kBM);
  CUtensorMap tb = B_MN ? make_tmap_bf16(g.B, g.N, g.K, g.ldb, kBK) : make_tmap_bf16(g.B, g.K, g.N, g.ldb, kBN);
  DistParams p;
  std::memset(&p, 0, sizeof(p));
  p.M = g.M;
  p.N = g.N;
  p.K = g.K;
  p.num_k_tiles = ceil_div(g.K, kBK);
  p.n_tiles = ceil_div(g.N, kBN);
  p.tiles = a.tiles;
  p.num_tiles = a.num_tiles;
  p.chunks = a.chunks;
  p.num_chunks = a.num_chunks;
  for (int op = 0; op < 2; ++op) {
    const DistGather& s = op ? a.gb : a.ga;
    GatherDev& d = op ? p.gb : p.ga;
    if (!s.enabled) continue;
    (op ? p.gather_b : p.gather_a) = 1;
    for (int q = 0; q < s.nranks; ++q) d.src[q] = reinterpret_cast<const __nv_bfloat16*>(s.src[q]);
    d.dst = reinterpret_cast<__nv_bfloat16*>(s.dst);
    d.ld = s.ld;
    d.rows_per_rank = s.rows_per_rank;
    d.total_rows = s.rows_per_rank * s.nranks;
    d.row_vecs = static_cast<int>(s.row_elems / 8);
    d.chunk_rows = s.chunk_rows;
    d.nranks = s.nranks;
    d.my = s.my;
    d.pieces = s.pieces;
    d.piece_vecs = s.piece_vecs;
    d.ready = s.ready;
    d.done = s.done;
  }
  p.C = g.C;
  p.ldc = g.ldc;
  p.c_dtype = g.c_dtype;
  p.accumulate = g.accumulate ? 1 : 0;
  p.bias = g.bias;
  p.act = g.act;
  p.alpha = g.alpha;
  p.mask = reinterpret_cast<const __nv_bfloat16*>(g.mask);
  p.ldm = g.ldm;
  p.aux0 = reinterpret_cast<const __nv_bfloat16*>(a.aux0);
  p.ld0 = a.ld0;
  p.aux1 = reinterpret_cast<const __nv_bfloat16*>(a.aux1);
  p.ld1 = a.ld1;
  p.zout = reinterpret_cast<__nv_bfloat16*>(a.zout);
  p.ldz = a.ldz;
  p.epi = a.epi;
  p.colsum = g.colsum;
  p.rs = a.rs.enabled;
  if (p.rs) {
    p.rs_nranks = a.rs.nranks;
    p.rs_my = a.rs.my;
    p.rs_rows = a.rs.rows_per_rank;
    for (int q = 0; q < a.rs.nranks; ++q) {
      p.rs_recv_peer[q] = reinterpret_cast<__nv_bfloat16*>(a.rs.recv_peer[q]);
      p.rs_flag_peer[q] = a.rs.flag_peer[q];
    }
    p.rs_recv_local = reinterpret_cast<const __nv_bfloat16*>(a.rs.recv_local);
    p.ld_recv = a.rs.ld_recv;
    p.rs_flag_local = a.rs.flag_local;
  }
  p.world = a.world;
  p.rank = a.rank;
  p.bar_local = a.bar_local;
  for (int s = 0; s < a.world; ++s) p.bar_peer[s] = a.bar_peer[s];
  p.ctl = a.ctl;
  p.status = g.status;
  p.timeout_ns = g.timeout_ns;

  const int grid = std::max(1, std::min(a.num_tiles, device_sm_count()));
  cudaLaunchConfig_t cfg;
  std::memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  FLARE_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, ta, tb, p));
  count_launch();
}

}  // namespace

void gemm_dist_tcgen05(const DistGemmArgs& a, cudaStream_t stream) {
  const GemmArgs& g = a.g;
  FLARE_CHECK(g.M > 0 && g.N > 0 && g.K > 0, "GEMM dims must be positive");
  FLARE_CHECK(g.c_dtype == kF32 || g.c_dtype == kBF16, "GEMM output must be fp32 or bf16");
  FLARE_CHECK((reinterpret_cast<uintptr_t>(g.C) & 15) == 0, "C must be 16-byte aligned");
  FLARE_CHECK(g.ldc % (g.c_dtype == kF32 ? 4 : 8) == 0, "C pitch must be a multiple of 16 bytes");
  FLARE_CHECK(g.mask == nullptr || g.ldm % 8 == 0, "mask pitch must be a multiple of 8 elements");
  FLARE_CHECK(a.num_tiles == ceil_div(g.M, kBM) * ceil_div(g.N, kBN), "tile list does not cover the output");
  FLARE_CHECK(a.world >= 1 && a.world <= kMaxRanks, "world size out of range");
  FLARE_CHECK(!(a.rs.enabled && a.ga.enabled), "reduce-scatter of the rows of a gathered A");
  if (a.epi == 1) FLARE_CHECK(a.aux0 && a.aux1 && a.zout, "cross epilogue needs x0, xl and z");
  if (a.epi == 2) FLARE_CHECK(a.aux1 != nullptr, "residual epilogue needs aux1");
  if (a.epi != 0 || a.aux0 || a.aux1)
    FLARE_CHECK(a.ld0 % 8 == 0 && a.ld1 % 8 == 0 && a.ldz % 8 == 0, "aux pitches must be multiples of 8");
  if (a.rs.enabled) {
    FLARE_CHECK(a.rs.rows_per_rank % kBM == 0, "reduce-scatter rows per rank must be a multiple of 128");
    FLARE_CHECK(static_cast<int64_t>(a.rs.rows_per_rank) * a.rs.nranks == g.M, "reduce-scatter rows mismatch");
  }
  for (int op = 0; op < 2; ++op) {
    const DistGather& s = op ? a.gb : a.ga;
    if (!s.enabled) continue;
    FLARE_CHECK(s.nranks >= 1 && s.nranks <= kMaxRanks && s.my >= 0 && s.my < s.nranks, "bad gather group");
    FLARE_CHECK(s.row_elems % 8 == 0 && s.row_elems <= s.ld && s.ld % 8 == 0, "gather rows must be 16-byte units");
    FLARE_CHECK(s.chunk_rows > 0 && s.rows_per_rank % s.chunk_rows == 0, "chunk rows must divide rows per rank");
    FLARE_CHECK(s.rows_per_rank * s.nranks <= (int64_t(1) << 19) * s.chunk_rows, "too many chunks");
    FLARE_CHECK(s.pieces >= 1 && s.pieces <= 4096 && s.done != nullptr, "bad copy pieces");
    FLARE_CHECK(static_cast<int64_t>(s.pieces) * s.piece_vecs >= s.chunk_rows * (s.row_elems / 8),
                "copy pieces do not cover a chunk");
  }
  FLARE_CHECK(a.num_chunks == 0 || a.chunks != nullptr, "chunk list missing");
  if (!g.a_mn && !g.b_mn) launch<false, false>(a, stream);
  else if (!g.a_mn && g.b_mn) launch<false, true>(a, stream);
  else if (g.a_mn && !g.b_mn) launch<true, false>(a, stream);
  else launch<true, true>(a, stream);
}

}  // namespace flare
