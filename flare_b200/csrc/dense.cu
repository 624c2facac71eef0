// Dense-tower kernels other than the GEMM (sm_100a):
//   * DLRM pairwise dot interaction, forward and backward: tcgen05 MMAs over
//     four samples per 128-row tile (up to 32 vectors a sample), and the
//     CUDA-core kernels (one warp per sample) for 33 vectors
//   * fused prediction head + multi-target weighted sigmoid BCE, forward and
//     backward in one pass (replaces optax sigmoid_binary_cross_entropy used by
//     recipes/recsys/ranking/losses.py:69-95 of the reference)
//   * flat fused Adam / AdamW / SGD over fp32 master weights that also writes
//     the bf16 compute copy
//   * data-parallel fused reduce-scatter -> Adam -> all-gather over NVLink peer
//     memory (ZeRO-1 semantics of src/flare/training/zero/contracts.py:40-48)
//   * small helpers: fp32 -> bf16 cast with padding, counter-based uniform init
#include "dense.cuh"
#include "gemm.cuh"
#include "sm100.cuh"

#include <algorithm>

namespace flare {
namespace {

// ------------------------------- interaction -------------------------------
// Vector index pairs (i > j) enumerated row by row: p = i*(i-1)/2 + j.
__device__ __forceinline__ void pair_of(int p, int& i, int& j) {
  int r = static_cast<int>((1.f + sqrtf(1.f + 8.f * static_cast<float>(p))) * 0.5f);
  while (r * (r - 1) / 2 > p) --r;
  while ((r + 1) * r / 2 <= p) ++r;
  i = r;
  j = p - r * (r - 1) / 2;
}

constexpr int kInterWarps = 4;

// Stage Z = [bot, emb_0..emb_{F-1}] of one sample into shared memory (bf16
// pairs, row pitch `rowp` words).  All 16-byte global loads of a lane are
// issued before its shared-memory stores, so the staging costs about one
// memory round trip instead of one per word.  Rows in [T, TP) are zeroed.
__device__ __forceinline__ void stage_z(uint32_t* z, int rowp, const __nv_bfloat16* bot,
                                        const __nv_bfloat16* emb, int T, int TP, int D) {
  const int lane = lane_id();
  const int qpr = D / 8;           // uint4 per row
  constexpr int kBatch = 8;        // uint4 loads in flight per lane
  const int total = T * qpr;
  for (int q0 = 0; q0 < total; q0 += 32 * kBatch) {
    uint4 buf[kBatch];
#pragma unroll
    for (int k = 0; k < kBatch; ++k) {
      const int q = q0 + lane + 32 * k;
      if (q < total) {
        const int r = q / qpr, c = q - r * qpr;
        const __nv_bfloat16* src = r == 0 ? bot + 8 * c : emb + (r - 1) * D + 8 * c;
        buf[k] = *reinterpret_cast<const uint4*>(src);
      }
    }
#pragma unroll
    for (int k = 0; k < kBatch; ++k) {
      const int q = q0 + lane + 32 * k;
      if (q < total) {
        const int r = q / qpr, c = q - r * qpr;
        uint32_t* dst = z + r * rowp + 4 * c;
        dst[0] = buf[k].x;
        dst[1] = buf[k].y;
        dst[2] = buf[k].z;
        dst[3] = buf[k].w;
      }
    }
  }
  for (int w = T * (D / 2) + lane; w < TP * (D / 2); w += 32) {
    const int r = w / (D / 2), c = w - r * (D / 2);
    z[r * rowp + c] = 0u;
  }
}

// Z = [bot, emb_0..emb_{F-1}] (T = F+1 vectors of width D, D % 64 == 0, D <= 256)
// out[b] = [bot (D), dots (T(T-1)/2), zero padding up to out_ld]
// One warp per sample; Z staged in shared memory as bf16 pairs with an odd
// row pitch (conflict-free).  Each lane computes a 3x3 tile of Z.Z^T from the
// lower triangle (i >= j blocks): 6 shared loads feed 18 FMAs per k-pair.
__global__ void __launch_bounds__(kInterWarps * 32) interaction_fwd_kernel(InteractionParams p) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int T = p.F + 1;
  const int TB = (T + 2) / 3;          // 3-row blocks
  const int TP = TB * 3;               // padded vector count
  const int rowp = p.D / 2 + 1;        // row pitch in 32-bit words
  const int orow_words = (p.out_ld + 1) / 2 + 4;
  uint32_t* z = reinterpret_cast<uint32_t*>(smem) + warp_id() * (TP * rowp + orow_words);
  // 16-byte aligned staging row for the output
  __nv_bfloat16* orow = reinterpret_cast<__nv_bfloat16*>(
      reinterpret_cast<uintptr_t>(z + TP * rowp + 3) & ~static_cast<uintptr_t>(15));
  const int lane = lane_id();
  const int nblk = TB * (TB + 1) / 2;  // lower-triangle blocks incl. diagonal
  const int KW = p.D / 2;
  for (int b = blockIdx.x * kInterWarps + warp_id(); b < p.B; b += gridDim.x * kInterWarps) {
    const __nv_bfloat16* bot = p.bot + static_cast<int64_t>(b) * p.bot_ld;
    const __nv_bfloat16* emb = p.emb + static_cast<int64_t>(b) * p.emb_ld;
    __nv_bfloat16* out = p.out + static_cast<int64_t>(b) * p.out_ld;
    stage_z(z, rowp, bot, emb, T, TP, p.D);
    __syncwarp();
    for (int blk = lane; blk < nblk; blk += 32) {
      // blk -> (I, J) with I >= J, row-major over the lower triangle
      int I = static_cast<int>((sqrtf(8.f * blk + 1.f) - 1.f) * 0.5f);
      while (I * (I + 1) / 2 > blk) --I;
      while ((I + 1) * (I + 2) / 2 <= blk) ++I;
      const int J = blk - I * (I + 1) / 2;
      const uint32_t* zi = z + (3 * I) * rowp;
      const uint32_t* zj = z + (3 * J) * rowp;
      float acc[3][3];
#pragma unroll
      for (int x = 0; x < 3; ++x)
#pragma unroll
        for (int y = 0; y < 3; ++y) acc[x][y] = 0.f;
#pragma unroll 4
      for (int c = 0; c < KW; ++c) {
        float2 a[3], bb[3];
#pragma unroll
        for (int x = 0; x < 3; ++x) {
          a[x] = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(zi + x * rowp + c));
          bb[x] = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(zj + x * rowp + c));
        }
#pragma unroll
        for (int x = 0; x < 3; ++x)
#pragma unroll
          for (int y = 0; y < 3; ++y) acc[x][y] = fmaf(a[x].x, bb[y].x, fmaf(a[x].y, bb[y].y, acc[x][y]));
      }
#pragma unroll
      for (int x = 0; x < 3; ++x)
#pragma unroll
        for (int y = 0; y < 3; ++y) {
          const int i = 3 * I + x, j = 3 * J + y;
          if (i < T && j < i) orow[p.D + i * (i - 1) / 2 + j] = __float2bfloat16_rn(acc[x][y]);
        }
    }
    const int npairs = T * (T - 1) / 2;
    for (int c = lane; c < p.D / 2; c += 32) reinterpret_cast<uint32_t*>(orow)[c] = z[c];  // bot (row 0)
    for (int c = p.D + npairs + lane; c < p.out_ld; c += 32) orow[c] = __float2bfloat16_rn(0.f);
    __syncwarp();
    for (int q = lane; q < p.out_ld / 8; q += 32)
      reinterpret_cast<uint4*>(out)[q] = reinterpret_cast<const uint4*>(orow)[q];
    __syncwarp();
  }
}

// dZ_i = sum_{j != i} dDot(i,j) Z_j ; d(bot) += dOut[:, :D]; ReLU mask of bot.
// One warp per sample: the symmetric T x T matrix S is built in shared memory;
// a lane owns D/32 columns and accumulates 9 output rows at a time.
template <int PER>
__global__ void __launch_bounds__(kInterWarps * 32) interaction_bwd_kernel(InteractionParams p) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int T = p.F + 1;
  const int rowp = p.D / 2 + 1;
  uint32_t* z = reinterpret_cast<uint32_t*>(smem) + warp_id() * (T * rowp + T * T);
  float* S = reinterpret_cast<float*>(z + T * rowp);
  const int lane = lane_id();
  const int npairs = T * (T - 1) / 2;
  constexpr int per_lane = PER;   // columns per lane (D / 32)
  constexpr int wpl = PER / 2;     // 32-bit words per lane
  for (int b = blockIdx.x * kInterWarps + warp_id(); b < p.B; b += gridDim.x * kInterWarps) {
    const __nv_bfloat16* bot = p.bot + static_cast<int64_t>(b) * p.bot_ld;
    const __nv_bfloat16* emb = p.emb + static_cast<int64_t>(b) * p.emb_ld;
    const __nv_bfloat16* dout = p.dout + static_cast<int64_t>(b) * p.out_ld;
    stage_z(z, rowp, bot, emb, T, T, p.D);
    for (int q = lane; q < T; q += 32) S[q * T + q] = 0.f;
    for (int q = lane; q < npairs; q += 32) {
      int i, j;
      pair_of(q, i, j);
      const float g = __bfloat162float(dout[p.D + q]);
      S[i * T + j] = g;
      S[j * T + i] = g;
    }
    __syncwarp();
    const int w0 = lane * wpl;  // first word of this lane's columns
    for (int i0 = 0; i0 < T; i0 += 9) {
      float acc[9][PER];
#pragma unroll
      for (int x = 0; x < 9; ++x)
#pragma unroll
        for (int e = 0; e < PER; ++e) acc[x][e] = 0.f;
      for (int j = 0; j < T; ++j) {
        float zv[PER];
#pragma unroll
        for (int e = 0; e < wpl; ++e) {
          const float2 v = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(z + j * rowp + w0 + e));
          zv[2 * e] = v.x;
          zv[2 * e + 1] = v.y;
        }
#pragma unroll
        for (int x = 0; x < 9; ++x) {
          const float sv = (i0 + x < T) ? S[(i0 + x) * T + j] : 0.f;
#pragma unroll
          for (int e = 0; e < PER; ++e) acc[x][e] = fmaf(sv, zv[e], acc[x][e]);
        }
      }
#pragma unroll
      for (int x = 0; x < 9; ++x) {
        const int i = i0 + x;
        if (i >= T) break;
        const int c0 = lane * per_lane;
        if (i == 0) {
          __nv_bfloat16* dbot = p.dbot + static_cast<int64_t>(b) * p.dbot_ld;
#pragma unroll
          for (int e = 0; e < PER; ++e) {
            const int c = c0 + e;
            float v = acc[x][e] + __bfloat162float(dout[c]);
            if (p.relu_mask_bot && __bfloat162float(bot[c]) <= 0.f) v = 0.f;
            dbot[c] = __float2bfloat16_rn(v);
          }
        } else {
          __nv_bfloat16* demb = p.demb + static_cast<int64_t>(b) * p.demb_ld + (i - 1) * p.D;
#pragma unroll
          for (int e = 0; e < PER; e += 2)
            *reinterpret_cast<__nv_bfloat162*>(demb + c0 + e) = __floats2bfloat162_rn(acc[x][e], acc[x][e + 1]);
        }
      }
    }
    __syncwarp();
  }
}

// ----------------------- interaction on tcgen05 ---------------------------
// Four samples share one 128-row tile: row 32*s + i holds vector i of sample
// s (bot, then the F pooled embeddings; rows T..31 zero), stored K-major with
// the 128-byte swizzle in D/64 atoms of 16 KB.
//   forward:  one 128 x 128 x D MMA (A = B = the tile) gives every dot product
//             inside the group; warp s reads its sample's diagonal 32 x 32
//             block from TMEM with one tcgen05.ld and keeps the strict lower
//             triangle (the other 12 blocks are the price of a full tile).
//   backward: dZ = S Z per sample, with S the symmetric dDot matrix (zero
//             diagonal).  The four S's sit on the diagonal of a 128 x 128 bf16
//             tile (off-diagonal blocks zero), and the same Z tile read as an
//             MN-major operand (K = vector index, N = column) is B: one
//             128 x D x 128 MMA.  dDot is bf16 already, so S loses nothing.
// One CTA of 4 warps (one per sample of the group) loops over groups; a
// thread owns tile row 32*warp + lane in both epilogues.
constexpr int kItThreads = 128;
constexpr int kItAtom = 16384;  // one 64-column atom of a 128-row tile
constexpr uint64_t kItTimeoutNs = 2000000000ull;

__device__ __forceinline__ void st_sw128(uint8_t* tile, int r, int c, uint4 v) {
  const int atom = c >> 3, ch = c & 7;
  *reinterpret_cast<uint4*>(tile + atom * kItAtom + r * 128 + ((ch ^ (r & 7)) << 4)) = v;
}
// K-major operand, k-step k (16 columns): atom k / 4, 32 bytes per step inside the 128-byte row
__device__ __forceinline__ uint64_t it_desc_k(uint32_t base, int k) {
  return sm100::make_smem_desc(base + (k >> 2) * kItAtom + (k & 3) * 32, 16, 1024);
}
// MN-major operand, k-step k (16 tile rows of 128 bytes); 64-column atoms kItAtom apart
__device__ __forceinline__ uint64_t it_desc_mn(uint32_t base, int k) {
  return sm100::make_smem_desc(base + k * 2048, kItAtom, 1024);
}

// rows [32*w, 32*w + 32) of the Z tile from sample b (zeros past T, or for a sample past the batch);
// every global load of a lane is issued before its shared-memory stores
__device__ __forceinline__ void stage_group_z(uint8_t* tile, int w, const InteractionParams& p, int b, bool valid,
                                              int T) {
  const int lane = lane_id();
  const int qpr = p.D / 8;  // 16-byte chunks per row
  const int total = 32 * qpr;
  const __nv_bfloat16* bot = p.bot + static_cast<int64_t>(b) * p.bot_ld;
  const __nv_bfloat16* emb = p.emb + static_cast<int64_t>(b) * p.emb_ld;
  constexpr int kBatch = 16;  // D = 128: the whole sample in one round trip
  for (int q0 = 0; q0 < total; q0 += 32 * kBatch) {
    uint4 buf[kBatch];
#pragma unroll
    for (int k = 0; k < kBatch; ++k) {
      const int q = q0 + lane + 32 * k;
      const int r = q / qpr, c = q - r * qpr;
      buf[k] = make_uint4(0u, 0u, 0u, 0u);
      if (valid && q < total && r < T)
        buf[k] = *reinterpret_cast<const uint4*>(r == 0 ? bot + 8 * c : emb + static_cast<int64_t>(r - 1) * p.D + 8 * c);
    }
#pragma unroll
    for (int k = 0; k < kBatch; ++k) {
      const int q = q0 + lane + 32 * k;
      if (q < total) {
        const int r = q / qpr, c = q - r * qpr;
        st_sw128(tile, 32 * w + r, c, buf[k]);
      }
    }
  }
}

__global__ void __launch_bounds__(kItThreads) interaction_fwd_tc_kernel(InteractionParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* sm = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  const int natoms = p.D / 64;
  const int opitch = static_cast<int>(p.out_ld) + 8;  // bf16 per output staging row (16-byte multiple)
  uint8_t* ztile = sm;
  const int tid = threadIdx.x, w = warp_id(), lane = lane_id();
  __nv_bfloat16* orow = reinterpret_cast<__nv_bfloat16*>(sm + natoms * kItAtom) + w * opitch;
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + natoms * kItAtom + 4 * opitch * 2);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bar + 1);
  const int T = p.F + 1, npairs = T * (T - 1) / 2;
  if (tid == 0) {
    sm100::mbar_init(bar, 1);
    sm100::fence_mbar_init();
  }
  if (w == 0) {
    sm100::tmem_alloc(tslot, 128);
    sm100::tmem_relinquish();
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *tslot;
  const uint32_t zaddr = smem_u32(ztile);
  constexpr uint32_t idesc = sm100::make_idesc_bf16(128, 128, false, false);
  const int ngroups = (p.B + 3) / 4;
  uint32_t phase = 0;
  for (int g = blockIdx.x; g < ngroups; g += gridDim.x) {
    const int b = 4 * g + w;
    const bool valid = b < p.B;
    stage_group_z(ztile, w, p, b, valid, T);
    if (valid) {  // the output row: bot, (dots later), zero tail
      const uint4* bot = reinterpret_cast<const uint4*>(p.bot + static_cast<int64_t>(b) * p.bot_ld);
      for (int c = lane; c < p.D / 8; c += 32) reinterpret_cast<uint4*>(orow)[c] = bot[c];
      for (int c = p.D + npairs + lane; c < p.out_ld; c += 32) orow[c] = __float2bfloat16_rn(0.f);
    }
    sm100::fence_proxy_async_smem();  // the tile's generic-proxy stores, visible to the tensor core
    sm100::tc_fence_before();
    __syncthreads();
    sm100::tc_fence_after();
    if (tid == 0) {
      for (int k = 0; k < p.D / 16; ++k)
        sm100::mma_f16_ss(tmem, it_desc_k(zaddr, k), it_desc_k(zaddr, k), idesc, k > 0 ? 1u : 0u);
      sm100::mma_commit(bar);
    }
    const bool done = sm100::mbar_wait(bar, phase, kItTimeoutNs, p.status, g);
    phase ^= 1u;
    if (!__syncthreads_and(done ? 1 : 0)) break;  // the status word holds the timeout
    sm100::tc_fence_after();
    uint32_t r[32];
    sm100::tmem_ld_32x32b_x32(tmem + (static_cast<uint32_t>(32 * w) << 16) + static_cast<uint32_t>(32 * w), r);
    sm100::tmem_ld_wait();
    if (valid) {
      const int i = lane;
      if (i >= 1 && i < T) {
        __nv_bfloat16* dst = orow + p.D + i * (i - 1) / 2;
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (j < i) dst[j] = __float2bfloat16_rn(__uint_as_float(r[j]));
      }
      __syncwarp();
      uint4* out = reinterpret_cast<uint4*>(p.out + static_cast<int64_t>(b) * p.out_ld);
      for (int q = lane; q < p.out_ld / 8; q += 32) out[q] = reinterpret_cast<const uint4*>(orow)[q];
    }
    sm100::tc_fence_before();
    __syncthreads();  // TMEM read and tile / staging row consumed before the next group
  }
  sm100::tc_fence_after();
  if (w == 0) sm100::tmem_dealloc(tmem, 128);
}

__global__ void __launch_bounds__(kItThreads) interaction_bwd_tc_kernel(InteractionParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* sm = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  const int natoms = p.D / 64;
  const int T = p.F + 1, npairs = T * (T - 1) / 2;
  const int dlen = p.D + (npairs + 7) / 8 * 8;  // staged dOut prefix: d(bot) part + dDot (16-byte chunks)
  const int dpitch = dlen + 8;                  // bf16 per staging row
  uint8_t* ztile = sm;
  uint8_t* stile = sm + natoms * kItAtom;  // 128 x 128 bf16: two atoms
  const int tid = threadIdx.x, w = warp_id(), lane = lane_id();
  __nv_bfloat16* drow = reinterpret_cast<__nv_bfloat16*>(stile + 2 * kItAtom) + w * dpitch;
  uint64_t* bar = reinterpret_cast<uint64_t*>(stile + 2 * kItAtom + 4 * dpitch * 2);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bar + 1);
  // the off-diagonal blocks of S stay zero; the diagonal blocks are rewritten for every group
  for (int q = tid; q < 2 * kItAtom / 16; q += kItThreads)
    reinterpret_cast<uint4*>(stile)[q] = make_uint4(0u, 0u, 0u, 0u);
  if (tid == 0) {
    sm100::mbar_init(bar, 1);
    sm100::fence_mbar_init();
  }
  if (w == 0) {
    sm100::tmem_alloc(tslot, static_cast<uint32_t>(p.D));
    sm100::tmem_relinquish();
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *tslot;
  const uint32_t zaddr = smem_u32(ztile), saddr = smem_u32(stile);
  const uint32_t idesc = sm100::make_idesc_bf16(128, p.D, false, true);
  const int ngroups = (p.B + 3) / 4;
  uint32_t phase = 0;
  for (int g = blockIdx.x; g < ngroups; g += gridDim.x) {
    const int b = 4 * g + w;
    const bool valid = b < p.B;
    // this sample's dOut row up to the last dDot (out_ld covers the rounded tail): loads first, so
    // they overlap the tile staging
    uint4 dq[4];
    const uint4* dsrc = reinterpret_cast<const uint4*>(p.dout + static_cast<int64_t>(b) * p.out_ld);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int q = lane + 32 * k;
      dq[k] = (valid && q < dlen / 8) ? dsrc[q] : make_uint4(0u, 0u, 0u, 0u);
    }
    stage_group_z(ztile, w, p, b, valid, T);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int q = lane + 32 * k;
      if (q < dlen / 8) reinterpret_cast<uint4*>(drow)[q] = dq[k];
    }
    __syncwarp();
    // row i = lane of S_b: S[i][j] = dDot(max, min) for i != j < T, else 0 (columns 32*w + j)
#pragma unroll
    for (int c4 = 0; c4 < 4; ++c4) {
      uint32_t wd[4];
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        uint32_t h[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int j = c4 * 8 + t * 2 + e;
          h[e] = 0u;
          if (valid && lane < T && j < T && j != lane) {
            const int hi = max(lane, j), lo = min(lane, j);
            h[e] = __bfloat16_as_ushort(drow[p.D + hi * (hi - 1) / 2 + lo]);
          }
        }
        wd[t] = h[0] | (h[1] << 16);
      }
      st_sw128(stile, 32 * w + lane, 4 * w + c4, make_uint4(wd[0], wd[1], wd[2], wd[3]));
    }
    sm100::fence_proxy_async_smem();
    sm100::tc_fence_before();
    __syncthreads();
    sm100::tc_fence_after();
    if (tid == 0) {
      for (int k = 0; k < 8; ++k)  // K = 128 tile rows
        sm100::mma_f16_ss(tmem, it_desc_k(saddr, k), it_desc_mn(zaddr, k), idesc, k > 0 ? 1u : 0u);
      sm100::mma_commit(bar);
    }
    const bool done = sm100::mbar_wait(bar, phase, kItTimeoutNs, p.status, g);
    phase ^= 1u;
    if (!__syncthreads_and(done ? 1 : 0)) break;
    sm100::tc_fence_after();
    const int i = lane;
    const bool act = valid && i < T;
    __nv_bfloat16* dst = i == 0 ? p.dbot + static_cast<int64_t>(b) * p.dbot_ld
                                : p.demb + static_cast<int64_t>(b) * p.demb_ld + static_cast<int64_t>(i - 1) * p.D;
    for (int cc = 0; cc < p.D / 32; ++cc) {
      __syncwarp();  // tcgen05.ld is warp-collective: reconverge after the previous chunk's stores
      uint32_t r[32];
      sm100::tmem_ld_32x32b_x32(tmem + (static_cast<uint32_t>(32 * w) << 16) + static_cast<uint32_t>(32 * cc), r);
      sm100::tmem_ld_wait();
      if (!act) continue;
      float v[32];
#pragma unroll
      for (int e = 0; e < 32; ++e) v[e] = __uint_as_float(r[e]);
      if (i == 0) {  // d(bot) = dZ_0 + dOut[:, :D], masked by the bottom MLP's ReLU (bot = tile row 32*w)
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int c = 4 * cc + q;  // 16-byte chunk of the row
          const uint4 zb = *reinterpret_cast<const uint4*>(ztile + (c >> 3) * kItAtom + (32 * w) * 128 +
                                                           (((c & 7) ^ 0) << 4));
          const uint4 gd = reinterpret_cast<const uint4*>(drow)[c];
          const __nv_bfloat16* zbh = reinterpret_cast<const __nv_bfloat16*>(&zb);
          const __nv_bfloat16* gdh = reinterpret_cast<const __nv_bfloat16*>(&gd);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            float x = v[8 * q + e] + __bfloat162float(gdh[e]);
            if (p.relu_mask_bot && __bfloat162float(zbh[e]) <= 0.f) x = 0.f;
            v[8 * q + e] = x;
          }
        }
      }
      uint4* o = reinterpret_cast<uint4*>(dst + 32 * cc);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint32_t wd[4];
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          __nv_bfloat162 hv = __floats2bfloat162_rn(v[8 * q + 2 * t], v[8 * q + 2 * t + 1]);
          wd[t] = *reinterpret_cast<uint32_t*>(&hv);
        }
        o[q] = make_uint4(wd[0], wd[1], wd[2], wd[3]);
      }
    }
    sm100::tc_fence_before();
    __syncthreads();
  }
  sm100::tc_fence_after();
  if (w == 0) sm100::tmem_dealloc(tmem, static_cast<uint32_t>(p.D));
}

// --------------------------- fused head + BCE ------------------------------
// logits[b,t] = h[b,:] . w[t,:] + bias[t]
// loss = sum_b sum_t weight[b,t] * (softplus(x) - y*x)  (accumulated into loss_sum)
// dlogit = weight * (sigmoid(x) - y) * grad_scale
// dh = sum_t dlogit[b,t] * w[t,:] masked by (h > 0) ; dw[t,:] += sum_b dlogit h ; db[t] += sum_b dlogit
constexpr int kHeadWarps = 8;
template <int PER>
__global__ void __launch_bounds__(kHeadWarps * 32) head_bce_kernel(HeadBceParams p) {
  extern __shared__ __align__(16) float hs[];  // per warp: [T][H] dw partials, then [T] db partials
  const int H = p.H, T = p.T;
  const int lane = lane_id();
  float* mine = hs + warp_id() * T * (H + 1);
  for (int i = lane; i < T * (H + 1); i += 32) mine[i] = 0.f;
  __syncwarp();
  float loss_acc = 0.f;
  for (int b = blockIdx.x * kHeadWarps + warp_id(); b < p.B; b += gridDim.x * kHeadWarps) {
    const __nv_bfloat16* h = p.h + static_cast<int64_t>(b) * p.h_ld + lane * PER;
    float hv[PER], dh[PER];
#pragma unroll
    for (int e = 0; e < PER; ++e) {
      hv[e] = __bfloat162float(h[e]);
      dh[e] = 0.f;
    }
    for (int t = 0; t < T; ++t) {
      const __nv_bfloat16* wrow = p.w + static_cast<int64_t>(t) * H + lane * PER;
      float w[PER];
#pragma unroll
      for (int e = 0; e < PER; ++e) w[e] = __bfloat162float(wrow[e]);
      float acc = 0.f;
#pragma unroll
      for (int e = 0; e < PER; ++e) acc = fmaf(hv[e], w[e], acc);
      const float x = warp_sum(acc) + __bfloat162float(p.bias[t]);
      if (lane == 0) p.logits[static_cast<int64_t>(b) * T + t] = x;
      const float y = p.labels[static_cast<int64_t>(b) * p.label_ld + t];
      float wt = p.target_weights ? p.target_weights[t] : 1.f;
      if (p.sample_weights) wt *= p.sample_weights[b];
      if (p.valid_count >= 0 && b >= p.valid_count) wt = 0.f;
      // softplus(x) - y*x = max(x,0) - x*y + log1p(exp(-|x|))
      const float l = fmaxf(x, 0.f) - x * y + log1pf(__expf(-fabsf(x)));
      if (lane == 0) loss_acc += wt * l;  // x is warp-uniform: count each sample once
      const float sg = 1.f / (1.f + __expf(-x));
      const float dl = wt * (sg - y) * p.grad_scale;
      float* dwp = mine + t * H + lane * PER;
#pragma unroll
      for (int e = 0; e < PER; ++e) {
        dh[e] = fmaf(dl, w[e], dh[e]);
        dwp[e] = fmaf(dl, hv[e], dwp[e]);
      }
      if (lane == 0) mine[T * H + t] += dl;
    }
    __nv_bfloat16* dho = p.dh + static_cast<int64_t>(b) * p.dh_ld + lane * PER;
#pragma unroll
    for (int e = 0; e < PER; ++e) dho[e] = __float2bfloat16_rn(hv[e] > 0.f ? dh[e] : 0.f);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < T * (H + 1); i += blockDim.x) {
    float acc = 0.f;
    for (int w = 0; w < kHeadWarps; ++w) acc += hs[w * T * (H + 1) + i];
    if (acc != 0.f) atomicAdd(i < T * H ? p.dw + i : p.db + (i - T * H), acc);
  }
  if (lane == 0 && loss_acc != 0.f) atomicAdd(p.loss_sum, loss_acc);
}

// ------------------------------ optimizers --------------------------------
__device__ __forceinline__ AdamParams resolve_step(AdamParams o) {
  if (o.step_ptr != nullptr) {
    const float t = static_cast<float>(*o.step_ptr);
    o.bias_corr1 = 1.f - powf(o.beta1, t);
    o.bias_corr2 = 1.f - powf(o.beta2, t);
  }
  return o;
}

__device__ __forceinline__ void adam_elem(const AdamParams& o, float& w, float& m, float& v, float g) {
  if (o.weight_decay != 0.f) {
    if (o.decoupled) w -= o.lr * o.weight_decay * w;
    else g += o.weight_decay * w;
  }
  if (o.kind == kDenseSgd) {
    if (o.beta1 != 0.f) {  // momentum
      m = o.beta1 * m + g;
      g = o.nesterov ? g + o.beta1 * m : m;
    }
    w -= o.lr * g;
    return;
  }
  if (o.kind == kDenseAdagrad) {
    m += g * g;
    w -= o.lr * g / (sqrtf(m) + o.eps);
    return;
  }
  if (o.kind == kDenseRmsprop) {
    v = o.beta2 * v + (1.f - o.beta2) * g * g;
    w -= o.lr * g / (sqrtf(v) + o.eps);
    return;
  }
  m = o.beta1 * m + (1.f - o.beta1) * g;
  v = o.beta2 * v + (1.f - o.beta2) * g * g;
  w -= o.lr * (m / o.bias_corr1) / (sqrtf(v / o.bias_corr2) + o.eps);
}

__global__ void adam_flat_kernel(AdamFlatParams p) {
  const AdamParams opt = resolve_step(p.opt);
  const int64_t n4 = p.n / 4;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float4 w = reinterpret_cast<float4*>(p.master)[i];
    float4 g = reinterpret_cast<const float4*>(p.grad)[i];
    float4 m = reinterpret_cast<float4*>(p.m)[i];
    float4 v = reinterpret_cast<float4*>(p.v)[i];
    float* wp = reinterpret_cast<float*>(&w);
    float* gp = reinterpret_cast<float*>(&g);
    float* mp = reinterpret_cast<float*>(&m);
    float* vp = reinterpret_cast<float*>(&v);
#pragma unroll
    for (int e = 0; e < 4; ++e) adam_elem(opt, wp[e], mp[e], vp[e], gp[e] * p.grad_scale);
    reinterpret_cast<float4*>(p.master)[i] = w;
    reinterpret_cast<float4*>(p.m)[i] = m;
    reinterpret_cast<float4*>(p.v)[i] = v;
    if (p.compute_copy) store4<__nv_bfloat16>(p.compute_copy + 4 * i, w);
    if (p.zero_grad) reinterpret_cast<float4*>(p.grad)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
}

// Data-parallel ZeRO-1 update in one launch: rank r owns [lo, hi) of the flat
// buffer. Sum every peer's gradient slice over NVLink (reduce-scatter), run the
// optimizer on the local fp32 master/state shard, push the new bf16 values
// into every peer's compute copy (all-gather), zero the consumed gradient
// slices, and finish with a barrier so every rank sees complete parameters.
template <int R, bool PUSH_ALL>
__global__ void __launch_bounds__(256, (R == 8 && PUSH_ALL) ? 3 : 4) adam_dp_fused_kernel(AdamDpParams p) {
  __shared__ int ok_sh;
  const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(p.epoch_ctr) + 1u;
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
  if (!ok_sh) return;
  const AdamParams opt = resolve_step(p.opt);
  const int64_t lo4 = p.lo / 4, hi4 = p.hi / 4;
  // R (group size) and PUSH_ALL (write the bf16 result into every member's copy,
  // or only the local one) are compile-time, so the peer pointers stay in a few
  // registers and every load of an element group is issued before its stores.
  constexpr int PW = PUSH_ALL ? R : 1;
  float4* gsrc[R];
  __nv_bfloat16* pdst[PW];
#pragma unroll
  for (int s = 0; s < R; ++s) gsrc[s] = reinterpret_cast<float4*>(p.peer_grad[s]);
#pragma unroll
  for (int s = 0; s < PW; ++s) pdst[s] = reinterpret_cast<__nv_bfloat16*>(p.peer_param[s]);
  float4* __restrict__ ws = reinterpret_cast<float4*>(p.master_shard);
  float4* __restrict__ ms = reinterpret_cast<float4*>(p.m_shard);
  float4* __restrict__ vs = reinterpret_cast<float4*>(p.v_shard);
  const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int64_t i = lo4 + static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < hi4;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t li = i - lo4;  // index into the local shard state
    float4 w = ws[li], m = ms[li], v = vs[li];
    float4 gv[R];
#pragma unroll
    for (int s = 0; s < R; ++s) gv[s] = __ldcg(gsrc[s] + i);
    float4 g = gv[0];
#pragma unroll
    for (int s = 1; s < R; ++s) g = f4_add(g, gv[s]);
#pragma unroll
    for (int s = 0; s < R; ++s) __stcg(gsrc[s] + i, zero);
    float* wp = reinterpret_cast<float*>(&w);
    float* gp = reinterpret_cast<float*>(&g);
    float* mp = reinterpret_cast<float*>(&m);
    float* vp = reinterpret_cast<float*>(&v);
#pragma unroll
    for (int e = 0; e < 4; ++e) adam_elem(opt, wp[e], mp[e], vp[e], gp[e] * p.grad_scale);
    ws[li] = w;
    ms[li] = m;
    vs[li] = v;
#pragma unroll
    for (int s = 0; s < PW; ++s) store4<__nv_bfloat16>(pdst[s] + 4 * i, w);
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned prev = atomicAdd(p.block_counter, 1u);
    if (prev == gridDim.x - 1) {
      *p.block_counter = 0u;
      *p.epoch_ctr = epoch;
      fence_sys();
      for (int s = 0; s < p.world; ++s) st_release_sys(p.peer_flags[s] + p.flag_out + p.rank, epoch);
      for (int s = 0; s < p.world; ++s)
        if (!wait_flag_geq(p.flags_local + p.flag_out + s, epoch, p.timeout_ns, p.status, s)) break;
    }
  }
}

// ------------------------------- helpers -----------------------------------
// out[c] += sum_r x[r, c]: block = 32 columns x 8 row-groups, one atomic per
// column per block.
__global__ void colsum_kernel(const __nv_bfloat16* __restrict__ x, int64_t rows, int cols, int64_t ldx,
                              float* __restrict__ out) {
  __shared__ float part[8][33];
  const int c = blockIdx.x * 32 + threadIdx.x;
  float acc = 0.f;
  if (c < cols) {
    for (int64_t r = blockIdx.y * 8 + threadIdx.y; r < rows; r += static_cast<int64_t>(gridDim.y) * 8)
      acc += __bfloat162float(x[r * ldx + c]);
  }
  part[threadIdx.y][threadIdx.x] = acc;
  __syncthreads();
  if (threadIdx.y == 0 && c < cols) {
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) s += part[i][threadIdx.x];
    atomicAdd(out + c, s);
  }
}

__global__ void cast_pad_kernel(const float* __restrict__ x, int64_t rows, int cols, int64_t ldx,
                                __nv_bfloat16* __restrict__ y, int ldy, float* __restrict__ zero) {
  // the step's first kernel also clears the step's loss accumulator (no separate fill launch)
  if (zero != nullptr && blockIdx.x == 0 && threadIdx.x == 0) *zero = 0.f;
  const int64_t n = rows * ldy;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / ldy;
    const int c = static_cast<int>(i - r * ldy);
    y[i] = __float2bfloat16_rn(c < cols ? x[r * ldx + c] : 0.f);
  }
}

// splitmix64 finaliser as a counter-based generator: value i of stream `seed`.
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
  return z ^ (z >> 31);
}

// Element i of a [rows, ncols] slice holding columns [col_begin, col_begin +
// ncols) of a table with row length `dim` gets value index
// (i / ncols) * dim + col_begin + i % ncols (+ index_offset) in the stream, so
// a table initialised in column shards equals the table initialised whole.
template <typename T>
__global__ void init_uniform_kernel(T* __restrict__ out, int64_t n, float lo, float hi, uint64_t seed,
                                    int64_t index_offset, int ncols, int dim, int col_begin, int64_t row_stride,
                                    int64_t row_first) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / ncols;
    // local row r is table row row_first + r * row_stride (row-wise pieces hold every row_stride-th row)
    const int64_t idx = (row_first + r * row_stride) * dim + col_begin + (i - r * ncols) + index_offset;
    const uint64_t rnd = mix64(seed * 0x9e3779b97f4a7c15ULL + static_cast<uint64_t>(idx));
    const float u = static_cast<float>(rnd >> 40) * (1.0f / 16777216.0f);  // 24 random bits in [0,1)
    out[i] = from_f32<T>(lo + (hi - lo) * u);
  }
}

}  // namespace

int grid_for(int64_t n, int threads) {
  const int64_t want = (n + threads - 1) / threads;
  const int cap = 148 * 16;
  return static_cast<int>(want < 1 ? 1 : (want > cap ? cap : want));
}

// CTAs of an interaction kernel that share an SM: shared memory (with the per-block reservation),
// capped by the TMEM columns (`tmem_cap` CTAs); the grid is this many per SM, so every CTA is resident
int it_ctas_per_sm(size_t smem, int tmem_cap) {
  static int sm_bytes = -1, reserved = 0;
  if (sm_bytes < 0) {
    int dev = 0;
    FLARE_CUDA_CHECK(cudaGetDevice(&dev));
    FLARE_CUDA_CHECK(cudaDeviceGetAttribute(&sm_bytes, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev));
    FLARE_CUDA_CHECK(cudaDeviceGetAttribute(&reserved, cudaDevAttrReservedSharedMemoryPerBlock, dev));
  }
  const int by_smem = static_cast<int>(static_cast<size_t>(sm_bytes) / (smem + static_cast<size_t>(reserved)));
  return std::max(1, std::min(by_smem, tmem_cap));
}

void interaction_forward(const InteractionParams& p, cudaStream_t s) {
  FLARE_CHECK(p.D % 64 == 0 && p.D <= 256, "interaction width must be a multiple of 64 and <= 256");
  const int T = p.F + 1;
  FLARE_CHECK(p.out_ld >= p.D + T * (T - 1) / 2, "interaction output too narrow");
  const int TP = (T + 2) / 3 * 3;
  FLARE_CHECK(p.out_ld % 8 == 0 && T <= 33, "interaction: out_ld must be a multiple of 8 and F <= 32");
  if (p.B <= 0) return;
  if (T <= 32) {
    // at least 56 KB per CTA: at most 4 CTAs (4 x 128 TMEM columns) share an SM
    const size_t tc_smem = std::max<size_t>(
        1024 + static_cast<size_t>(p.D / 64) * kItAtom + 4 * static_cast<size_t>(p.out_ld + 8) * 2 + 64, 57344);
    FLARE_CUDA_CHECK(cudaFuncSetAttribute(interaction_fwd_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          static_cast<int>(tc_smem)));
    // shared memory is what limits residency: ask for the full carveout, or the occupancy query (and
    // the launch) assume the default L1 / shared split and allow one CTA per SM
    FLARE_CUDA_CHECK(cudaFuncSetAttribute(interaction_fwd_tc_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                                          cudaSharedmemCarveoutMaxShared));
    const int grid = std::min(ceil_div(p.B, 4), device_sm_count() * it_ctas_per_sm(tc_smem, 4));
    interaction_fwd_tc_kernel<<<grid, kItThreads, tc_smem, s>>>(p);
    FLARE_CUDA_CHECK(cudaGetLastError());
    count_launch();
    return;
  }
  const size_t smem = static_cast<size_t>(kInterWarps) * (TP * (p.D / 2 + 1) + (p.out_ld + 1) / 2 + 4) * 4;
  FLARE_CUDA_CHECK(cudaFuncSetAttribute(interaction_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        static_cast<int>(smem)));
  const int grid = std::min(ceil_div(p.B, kInterWarps), 148 * 8);
  interaction_fwd_kernel<<<grid, kInterWarps * 32, smem, s>>>(p);
  FLARE_CUDA_CHECK(cudaGetLastError());
  count_launch();
}

template <int PER>
void interaction_bwd_launch(const InteractionParams& p, cudaStream_t s) {
  const int T = p.F + 1;
  const size_t smem = static_cast<size_t>(kInterWarps) * (T * (p.D / 2 + 1) + T * T) * 4;
  FLARE_CUDA_CHECK(cudaFuncSetAttribute(interaction_bwd_kernel<PER>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        static_cast<int>(smem)));
  const int grid = std::min(ceil_div(p.B, kInterWarps), 148 * 8);
  interaction_bwd_kernel<PER><<<grid, kInterWarps * 32, smem, s>>>(p);
  FLARE_CUDA_CHECK(cudaGetLastError());
  count_launch();
}

void interaction_backward(const InteractionParams& p, cudaStream_t s) {
  FLARE_CHECK(p.D % 64 == 0 && p.D <= 256, "interaction width must be a multiple of 64 and <= 256");
  FLARE_CHECK(p.F + 1 <= 33, "interaction supports up to 32 embedded features");
  const int T = p.F + 1;
  FLARE_CHECK(p.out_ld % 8 == 0 && p.out_ld >= p.D + T * (T - 1) / 2, "interaction gradient too narrow");
  if (p.B <= 0) return;
  if (T <= 32) {
    // Z + S + dDot rows: 2 (D = 256) to 4 (D = 64) CTAs per SM, each with D TMEM columns (<= 512 in all)
    const size_t dpitch = static_cast<size_t>(p.D + (T * (T - 1) / 2 + 7) / 8 * 8 + 8);
    FLARE_CHECK(p.D + (T * (T - 1) / 2 + 7) / 8 * 8 <= 4 * 32 * 8, "interaction: dOut row staging too long");
    const size_t tc_smem =
        1024 + static_cast<size_t>(p.D / 64 + 2) * kItAtom + 4 * dpitch * 2 + 64;
    FLARE_CUDA_CHECK(cudaFuncSetAttribute(interaction_bwd_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          static_cast<int>(tc_smem)));
    FLARE_CUDA_CHECK(cudaFuncSetAttribute(interaction_bwd_tc_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                                          cudaSharedmemCarveoutMaxShared));
    const int grid = std::min(ceil_div(p.B, 4), device_sm_count() * it_ctas_per_sm(tc_smem, 512 / p.D));
    interaction_bwd_tc_kernel<<<grid, kItThreads, tc_smem, s>>>(p);
    FLARE_CUDA_CHECK(cudaGetLastError());
    count_launch();
    return;
  }
  if (p.D == 64) interaction_bwd_launch<2>(p, s);
  else if (p.D == 128) interaction_bwd_launch<4>(p, s);
  else interaction_bwd_launch<8>(p, s);
}

template <int PER>
void head_bce_launch(const HeadBceParams& p, cudaStream_t s) {
  const size_t smem = static_cast<size_t>(kHeadWarps) * p.T * (p.H + 1) * 4;
  FLARE_CUDA_CHECK(cudaFuncSetAttribute(head_bce_kernel<PER>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        static_cast<int>(smem)));
  const int grid = std::min(ceil_div(p.B, kHeadWarps * 8), 148 * 2);
  head_bce_kernel<PER><<<grid, kHeadWarps * 32, smem, s>>>(p);
  count_launch();
}

void head_bce(const HeadBceParams& p, cudaStream_t s) {
  FLARE_CHECK(p.H % 32 == 0 && p.H <= 1024, "head width must be a multiple of 32 and <= 1024");
  FLARE_CHECK(p.T >= 1 && p.T * p.H <= 4096, "targets x head width must be <= 4096");
  switch (p.H / 32) {
    case 1: head_bce_launch<1>(p, s); break;
    case 2: head_bce_launch<2>(p, s); break;
    case 4: head_bce_launch<4>(p, s); break;
    case 8: head_bce_launch<8>(p, s); break;
    case 16: head_bce_launch<16>(p, s); break;
    case 32: head_bce_launch<32>(p, s); break;
    default: FLARE_CHECK(false, "head width / 32 must be a power of two");
  }
  FLARE_CUDA_CHECK(cudaGetLastError());
}

void adam_flat(const AdamFlatParams& p, cudaStream_t s) {
  FLARE_CHECK(p.n % 4 == 0, "flat optimizer buffers must be padded to a multiple of 4");
  adam_flat_kernel<<<grid_for(p.n / 4, 256), 256, 0, s>>>(p);
  FLARE_CUDA_CHECK(cudaGetLastError());
  count_launch();
}

void adam_dp_fused(const AdamDpParams& p, cudaStream_t s) {
  FLARE_CHECK(p.lo % 4 == 0 && p.hi % 4 == 0, "shard bounds must be multiples of 4");
  FLARE_CHECK(p.world == 1 || p.world == 2 || p.world == 4 || p.world == 8, "group size must be 1, 2, 4 or 8");
  FLARE_CHECK(p.param_world == 1 || p.param_world == p.world, "the update goes to the local copy or to all copies");
  const int grid = std::max(1, std::min(grid_for((p.hi - p.lo) / 4, 256), 148 * 4));
  const bool all = p.param_world == p.world && p.world > 1;
  switch (p.world) {
    case 1: adam_dp_fused_kernel<1, false><<<grid, 256, 0, s>>>(p); break;
    case 2: all ? adam_dp_fused_kernel<2, true><<<grid, 256, 0, s>>>(p) : adam_dp_fused_kernel<2, false><<<grid, 256, 0, s>>>(p); break;
    case 4: all ? adam_dp_fused_kernel<4, true><<<grid, 256, 0, s>>>(p) : adam_dp_fused_kernel<4, false><<<grid, 256, 0, s>>>(p); break;
    default: all ? adam_dp_fused_kernel<8, true><<<grid, 256, 0, s>>>(p) : adam_dp_fused_kernel<8, false><<<grid, 256, 0, s>>>(p); break;
  }
  FLARE_CUDA_CHECK(cudaGetLastError());
  count_launch();
}

void colsum_bf16(const __nv_bfloat16* x, int64_t rows, int cols, int64_t ldx, float* out, cudaStream_t s) {
  dim3 block(32, 8);
  const int gx = ceil_div(cols, 32);
  const int gy = std::max(1, std::min<int>(ceil_div(rows, 256), std::max(1, 148 * 8 / gx)));
  colsum_kernel<<<dim3(gx, gy), block, 0, s>>>(x, rows, cols, ldx, out);
  FLARE_CUDA_CHECK(cudaGetLastError());
  count_launch();
}

void cast_pad_bf16(const float* x, int64_t rows, int cols, int64_t ldx, __nv_bfloat16* y, int ldy,
                   cudaStream_t s, float* zero) {
  cast_pad_kernel<<<grid_for(rows * ldy, 256), 256, 0, s>>>(x, rows, cols, ldx, y, ldy, zero);
  FLARE_CUDA_CHECK(cudaGetLastError());
  count_launch();
}

void init_uniform(void* out, int dtype, int64_t n, float lo, float hi, uint64_t seed, int64_t index_offset,
                  int ncols, int dim, int col_begin, int64_t row_stride, int64_t row_first, cudaStream_t s) {
  FLARE_CHECK(ncols > 0 && dim >= ncols && row_stride >= 1, "bad init slice");
  const int grid = grid_for(n, 256);
  if (dtype == kF32)
    init_uniform_kernel<float><<<grid, 256, 0, s>>>(static_cast<float*>(out), n, lo, hi, seed, index_offset, ncols,
                                                     dim, col_begin, row_stride, row_first);
  else if (dtype == kBF16)
    init_uniform_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(static_cast<__nv_bfloat16*>(out), n, lo, hi, seed,
                                                             index_offset, ncols, dim, col_begin, row_stride,
                                                             row_first);
  else
    init_uniform_kernel<__half><<<grid, 256, 0, s>>>(static_cast<__half*>(out), n, lo, hi, seed, index_offset,
                                                      ncols, dim, col_begin, row_stride, row_first);
  FLARE_CUDA_CHECK(cudaGetLastError());
  count_launch();
}

}  // namespace flare
