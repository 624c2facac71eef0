// bf16 GEMM on the 5th-generation tensor cores (tcgen05) for sm_100a.
//
//   C[M,N] (+)= alpha * A[M,K] . B[N,K]^T   (+ bias[N]) -> act -> * mask -> C
//
// A and B may each be K-major (row-major [rows][K]) or MN-major (the
// transpose is what is stored, row-major [K][rows]); MN-major operands are fed
// to the tensor core with the descriptor's transpose bit, so the backward
// GEMMs (dX = dY.W and dW = dY^T.X) never materialise a transpose.
//
// Structure (one 128 x BN output tile per CTA, 128 threads):
//   warp 0 / lane 0 : TMA producer, STAGES-deep ring of 128-byte-swizzled tiles
//   warp 1 / lane 0 : tcgen05.mma issuer; accumulator lives in TMEM
//   warps 0..3      : epilogue, warp w reads TMEM lanes 32w..32w+31 (= rows)
// Epilogue fusions used by the MLP towers:
//   bias + ReLU (forward), ReLU-backward mask from the saved activation,
//   per-column sums (bias gradient) via warp butterfly + one atomic per column,
//   fp32 output with accumulate (gradient accumulation windows).
//
// This replaces the XLA/cuBLAS dense GEMMs of the reference's JAX engine
// (src/flare/jax/training/engines/distributed.py:612-716 runs them via XLA).
#include "gemm.cuh"
#include "sm100.cuh"

#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdlib>
#include <mutex>

namespace flare {

// ----------------------------- host side ------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    FLARE_CUDA_CHECK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q));
    FLARE_CHECK(q == cudaDriverEntryPointSuccess && ptr != nullptr, "cuTensorMapEncodeTiled unavailable");
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

// Row-major bf16 matrix with `inner` contiguous elements per row and `outer`
// rows, row pitch `ld` elements; box = 64 x box_outer with 128-byte swizzle.
CUtensorMap make_tmap_bf16(const void* base, int64_t inner, int64_t outer, int64_t ld, int box_outer) {
  FLARE_CHECK((reinterpret_cast<uintptr_t>(base) & 15) == 0, "TMA base must be 16-byte aligned");
  FLARE_CHECK((ld * 2) % 16 == 0, "TMA row pitch must be a multiple of 16 bytes");
  CUtensorMap m;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(outer)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * 2)};
  cuuint32_t box[2] = {64u, static_cast<cuuint32_t>(box_outer)};
  cuuint32_t estr[2] = {1u, 1u};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
                           estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  FLARE_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed (code " + std::to_string(static_cast<int>(r)) + ")");
  return m;
}


namespace {

constexpr int kBM = 128;
constexpr int kBK = 64;                 // one 128-byte swizzle atom of bf16 along K
constexpr int kThreads = 128;
constexpr int kTileBytesA = kBM * kBK * 2;  // 16 KiB

struct EpiParams {
  int M, N;
  void* C;
  int64_t ldc;
  int c_dtype;
  int accumulate;
  const __nv_bfloat16* bias;
  int act;
  float alpha;
  const __nv_bfloat16* mask;
  int64_t ldm;
  float* colsum;
  int* status;
  uint64_t timeout_ns;
  int num_k_tiles;
  int splits;       // split-K factor (gridDim.z); > 1 reduces into fp32 C with atomics
  int fast_epi;     // 1 (default): staged epilogue (epilogue_rows_staged) in the one-SM kernel
  int bias_vec;     // bias is 16-byte aligned: 16-byte bias loads in the staged epilogue
};

template <int BN, int STAGES>
struct SmemLayout {
  static_assert(STAGES * kTileBytesA >= (kThreads / 32) * 2048, "the staged epilogue reuses the A ring");
  static constexpr int kTileBytesB = BN * kBK * 2;
  static constexpr int kOffA = 0;
  static constexpr int kOffB = STAGES * kTileBytesA;
  static constexpr int kOffBar = kOffB + STAGES * kTileBytesB;
  static constexpr int kBytes = kOffBar + (2 * STAGES + 1) * 8 + 16;
  static constexpr int kAlloc = kBytes + 1024;  // slack for manual 1 KiB alignment
};

// Epilogue of one 128 x BN accumulator tile in this CTA's TMEM: warp w owns
// TMEM lanes (= output rows m0 + 32w ..) and walks the columns 32 at a time.
template <int BN>
__device__ __forceinline__ void epilogue_rows(const EpiParams& p, uint32_t tmem_base, int m0, int n0, int warp,
                                              int lane, bool done) {
  const int row = m0 + warp * 32 + lane;
  const bool row_ok = row < p.M;
  if (done) {
#pragma unroll 1
    for (int c = 0; c < BN; c += 32) {
      const int ncol = n0 + c;
      if (ncol >= p.N) break;  // warp-uniform
      uint32_t r[32];
      sm100::tmem_ld_32x32b_x32(tmem_base + (static_cast<uint32_t>(warp * 32) << 16) + c, r);
      sm100::tmem_ld_wait();
      float v[32];
      const bool full_chunk = (ncol + 32 <= p.N);
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        float x = __uint_as_float(r[j]) * p.alpha;
        if (p.bias != nullptr && (full_chunk || ncol + j < p.N)) x += __bfloat162float(p.bias[ncol + j]);
        if (p.act == 1) x = fmaxf(x, 0.f);
        v[j] = x;
      }
      if (p.mask != nullptr && row_ok) {
        const __nv_bfloat16* mrow = p.mask + static_cast<int64_t>(row) * p.ldm + ncol;
        if (full_chunk) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint4 u = *reinterpret_cast<const uint4*>(mrow + q * 8);
            const __nv_bfloat16* mb = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
            for (int t = 0; t < 8; ++t) v[q * 8 + t] = (__bfloat162float(mb[t]) > 0.f) ? v[q * 8 + t] : 0.f;
          }
        } else {
          for (int j = 0; j < 32; ++j)
            if (ncol + j < p.N) v[j] = (__bfloat162float(mrow[j]) > 0.f) ? v[j] : 0.f;
        }
      }
      if (!row_ok) {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = 0.f;
      }
      if (p.colsum != nullptr) {
        // Butterfly reduce-scatter across the warp: afterwards lane l holds the
        // sum over the warp's 32 rows of column (ncol + l).
        float t[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) t[j] = v[j];
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) {
          const bool upper = (lane & o) != 0;
#pragma unroll
          for (int j = 0; j < o; ++j) {
            const float send = upper ? t[j] : t[j + o];
            const float keep = upper ? t[j + o] : t[j];
            t[j] = keep + __shfl_xor_sync(0xffffffffu, send, o);
          }
        }
        if (ncol + lane < p.N) atomicAdd(p.colsum + ncol + lane, t[0]);
      }
      if (row_ok && p.splits > 1) {
        // split-K partial: reduce into the fp32 output
        float* crow = reinterpret_cast<float*>(p.C) + static_cast<int64_t>(row) * p.ldc + ncol;
        if (full_chunk) {
#pragma unroll
          for (int q = 0; q < 8; ++q)
            atomicAdd(reinterpret_cast<float4*>(crow + 4 * q), make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]));
        } else {
          for (int j = 0; j < 32; ++j)
            if (ncol + j < p.N) atomicAdd(crow + j, v[j]);
        }
      } else if (row_ok) {
        if (p.c_dtype == kBF16) {
          __nv_bfloat16* crow = reinterpret_cast<__nv_bfloat16*>(p.C) + static_cast<int64_t>(row) * p.ldc + ncol;
          if (full_chunk) {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              uint4 u;
              uint32_t* w = reinterpret_cast<uint32_t*>(&u);
#pragma unroll
              for (int t = 0; t < 4; ++t) {
                __nv_bfloat162 h = __floats2bfloat162_rn(v[q * 8 + 2 * t], v[q * 8 + 2 * t + 1]);
                w[t] = *reinterpret_cast<uint32_t*>(&h);
              }
              *reinterpret_cast<uint4*>(crow + q * 8) = u;
            }
          } else {
            for (int j = 0; j < 32; ++j)
              if (ncol + j < p.N) crow[j] = __float2bfloat16_rn(v[j]);
          }
        } else {
          float* crow = reinterpret_cast<float*>(p.C) + static_cast<int64_t>(row) * p.ldc + ncol;
          if (full_chunk) {
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              float4 o = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
              if (p.accumulate) o = f4_add(o, *reinterpret_cast<const float4*>(crow + 4 * q));
              *reinterpret_cast<float4*>(crow + 4 * q) = o;
            }
          } else {
            for (int j = 0; j < 32; ++j)
              if (ncol + j < p.N) crow[j] = p.accumulate ? crow[j] + v[j] : v[j];
          }
        }
      }
    }
  }
}

// Staged epilogue (the default; FLARE_GEMM_EPI=0 selects epilogue_rows), for the one-SM kernel once
// its mainloop is done (24-39 % less time than epilogue_rows on the DLRM tower shapes, 8192 x 128..1024
// x 256..1024; 2.205 -> 2.089 ms per DLRM step):
//  * the TMEM load of column chunk c + 1 is in flight while chunk c is processed;
//  * bias is read with four 16-byte loads per chunk when it is 16-byte aligned;
//  * a full chunk of bf16 output goes through a 2 KiB block of the (now idle) operand ring per
//    warp: each thread writes its row's 64 bytes, then each lane stores 16 bytes of row
//    i * 8 + lane / 4, so four lanes write one row's 64 contiguous bytes (full 32-byte sectors)
//    instead of every lane writing 16 bytes of its own row.  The row's four 16-byte pieces are
//    placed at piece ^ ((row / 2) % 4), which spreads both the writes and the reads of a warp over
//    all eight 16-byte bank groups.
// fp32 outputs, split-K partials and partial chunks keep the per-row stores of epilogue_rows.
__device__ __forceinline__ void tmem_regs_ready(uint32_t (&r)[32]) {
#pragma unroll
  for (int j = 0; j < 32; ++j) asm volatile("" : "+r"(r[j]));
}

__device__ __forceinline__ void epi_chunk_staged(const EpiParams& p, uint32_t (&r)[32], int row, bool row_ok,
                                                 int ncol, int lane, uint8_t* wst, int wrow0) {
  const bool full_chunk = (ncol + 32 <= p.N);
  float v[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]) * p.alpha;
  if (p.bias != nullptr) {
    if (full_chunk && p.bias_vec) {
      const uint4* bp = reinterpret_cast<const uint4*>(p.bias + ncol);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint4 u = __ldg(bp + q);
        const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
        for (int t = 0; t < 8; ++t) v[q * 8 + t] += __bfloat162float(b[t]);
      }
    } else {
      for (int j = 0; j < 32; ++j)
        if (ncol + j < p.N) v[j] += __bfloat162float(p.bias[ncol + j]);
    }
  }
  if (p.act == 1) {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = fmaxf(v[j], 0.f);
  }
  if (p.mask != nullptr && row_ok) {
    const __nv_bfloat16* mrow = p.mask + static_cast<int64_t>(row) * p.ldm + ncol;
    if (full_chunk) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint4 u = *reinterpret_cast<const uint4*>(mrow + q * 8);
        const __nv_bfloat16* mb = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
        for (int t = 0; t < 8; ++t) v[q * 8 + t] = (__bfloat162float(mb[t]) > 0.f) ? v[q * 8 + t] : 0.f;
      }
    } else {
      for (int j = 0; j < 32; ++j)
        if (ncol + j < p.N) v[j] = (__bfloat162float(mrow[j]) > 0.f) ? v[j] : 0.f;
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
        const float send = upper ? t[j] : t[j + o];
        const float keep = upper ? t[j + o] : t[j];
        t[j] = keep + __shfl_xor_sync(0xffffffffu, send, o);
      }
    }
    if (ncol + lane < p.N) atomicAdd(p.colsum + ncol + lane, t[0]);
  }
  if (p.splits == 1 && p.c_dtype == kBF16 && full_chunk) {
    // warp-uniform branch: stage the 32 x 32 bf16 block, then coalesced 16-byte stores
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint4 u;
      uint32_t* w = reinterpret_cast<uint32_t*>(&u);
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        __nv_bfloat162 h = __floats2bfloat162_rn(v[q * 8 + 2 * t], v[q * 8 + 2 * t + 1]);
        w[t] = *reinterpret_cast<uint32_t*>(&h);
      }
      *reinterpret_cast<uint4*>(wst + lane * 64 + ((q ^ ((lane >> 1) & 3)) << 4)) = u;
    }
    __syncwarp();
    const int q = lane & 3;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int rr = i * 8 + (lane >> 2);
      const uint4 u = *reinterpret_cast<const uint4*>(wst + rr * 64 + ((q ^ ((rr >> 1) & 3)) << 4));
      const int grow = wrow0 + rr;
      if (grow < p.M)
        *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(p.C) + static_cast<int64_t>(grow) * p.ldc +
                                  ncol + q * 8) = u;
    }
    __syncwarp();  // the block is rewritten by the next chunk
    return;
  }
  if (!row_ok) return;
  if (p.splits > 1) {
    float* crow = reinterpret_cast<float*>(p.C) + static_cast<int64_t>(row) * p.ldc + ncol;
    if (full_chunk) {
#pragma unroll
      for (int q = 0; q < 8; ++q)
        atomicAdd(reinterpret_cast<float4*>(crow + 4 * q), make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]));
    } else {
      for (int j = 0; j < 32; ++j)
        if (ncol + j < p.N) atomicAdd(crow + j, v[j]);
    }
  } else if (p.c_dtype == kBF16) {
    __nv_bfloat16* crow = reinterpret_cast<__nv_bfloat16*>(p.C) + static_cast<int64_t>(row) * p.ldc + ncol;
    for (int j = 0; j < 32; ++j)
      if (ncol + j < p.N) crow[j] = __float2bfloat16_rn(v[j]);
  } else {
    float* crow = reinterpret_cast<float*>(p.C) + static_cast<int64_t>(row) * p.ldc + ncol;
    if (full_chunk) {
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        float4 o = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
        if (p.accumulate) o = f4_add(o, *reinterpret_cast<const float4*>(crow + 4 * q));
        *reinterpret_cast<float4*>(crow + 4 * q) = o;
      }
    } else {
      for (int j = 0; j < 32; ++j)
        if (ncol + j < p.N) crow[j] = p.accumulate ? crow[j] + v[j] : v[j];
    }
  }
}

// `stage`: 8 KiB of shared memory no async copy or MMA touches any more (2 KiB per warp).
template <int BN>
__device__ __forceinline__ void epilogue_rows_staged(const EpiParams& p, uint32_t tmem_base, int m0, int n0,
                                                     int warp, int lane, bool done, uint8_t* stage) {
  if (!__all_sync(0xffffffffu, done)) return;  // the TMEM loads below are warp-collective
  const int wrow0 = m0 + warp * 32;
  const int row = wrow0 + lane;
  const bool row_ok = row < p.M;
  uint8_t* wst = stage + warp * 2048;
  const uint32_t taddr = tmem_base + (static_cast<uint32_t>(warp * 32) << 16);
  const int nch = min(BN / 32, (p.N - n0 + 31) / 32);  // chunks with at least one column inside N
  if (nch <= 0) return;
  sm100::fence_proxy_async_smem();  // the ring was last written by TMA: order our generic writes after it
  uint32_t ra[32], rb[32];
  sm100::tmem_ld_32x32b_x32(taddr, ra);
#pragma unroll 1
  for (int c = 0; c < nch; c += 2) {
    sm100::tmem_ld_wait();
    tmem_regs_ready(ra);
    if (c + 1 < nch) sm100::tmem_ld_32x32b_x32(taddr + (c + 1) * 32, rb);
    epi_chunk_staged(p, ra, row, row_ok, n0 + c * 32, lane, wst, wrow0);
    if (c + 1 < nch) {
      sm100::tmem_ld_wait();
      tmem_regs_ready(rb);
      if (c + 2 < nch) sm100::tmem_ld_32x32b_x32(taddr + (c + 2) * 32, ra);
      epi_chunk_staged(p, rb, row, row_ok, n0 + (c + 1) * 32, lane, wst, wrow0);
    }
  }
}

template <int BN, int STAGES, bool A_MN, bool B_MN>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_bf16_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                     EpiParams p) {
  using L = SmemLayout<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + L::kOffBar);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* done_bar = empty_bar + STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done_bar + 1);

  const int warp = warp_id();
  const int lane = lane_id();
  const int m0 = blockIdx.x * kBM;
  const int n0 = blockIdx.y * BN;
  // split-K: this CTA owns k-tiles [kt_begin, kt_end)
  const int kt_begin = static_cast<int>((static_cast<int64_t>(p.num_k_tiles) * blockIdx.z) / p.splits);
  const int kt_end = static_cast<int>((static_cast<int64_t>(p.num_k_tiles) * (blockIdx.z + 1)) / p.splits);

  if (threadIdx.x == 0) {
    sm100::tma_prefetch_desc(&tmap_a);
    sm100::tma_prefetch_desc(&tmap_b);
    for (int s = 0; s < STAGES; ++s) {
      sm100::mbar_init(&full_bar[s], 1);
      sm100::mbar_init(&empty_bar[s], 1);
    }
    sm100::mbar_init(done_bar, 1);
    sm100::fence_mbar_init();
  }
  if (warp == 0) {
    sm100::tmem_alloc(tmem_slot, BN);
    sm100::tmem_relinquish();
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int KT = kt_end - kt_begin;

  if (warp == 0 && lane == 0) {
    // ------------------------------ producer ------------------------------
    for (int kt = 0; kt < KT; ++kt) {
      const int s = kt % STAGES;
      if (kt >= STAGES) {
        if (!sm100::mbar_wait(&empty_bar[s], ((kt / STAGES) - 1) & 1, p.timeout_ns, p.status, 100 + s)) break;
      }
      uint8_t* sa = smem + L::kOffA + s * kTileBytesA;
      uint8_t* sb = smem + L::kOffB + s * L::kTileBytesB;
      sm100::mbar_arrive_expect_tx(&full_bar[s], kTileBytesA + L::kTileBytesB);
      const int k0 = (kt_begin + kt) * kBK;
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
        for (int j = 0; j < BN / 64; ++j) sm100::tma_load_2d(sb + j * 8192, &tmap_b, &full_bar[s], n0 + 64 * j, k0);
      }
    }
  } else if (warp == 1 && lane == 0) {
    // ------------------------------ MMA issuer ----------------------------
    constexpr uint32_t idesc = sm100::make_idesc_bf16(kBM, BN, A_MN, B_MN);
    bool ok = true;
    for (int kt = 0; kt < KT; ++kt) {
      const int s = kt % STAGES;
      if (!sm100::mbar_wait(&full_bar[s], (kt / STAGES) & 1, p.timeout_ns, p.status, 200 + s)) {
        ok = false;
        break;
      }
      sm100::tc_fence_after();
      const uint32_t sa = smem_u32(smem + L::kOffA + s * kTileBytesA);
      const uint32_t sb = smem_u32(smem + L::kOffB + s * L::kTileBytesB);
#pragma unroll
      for (int k = 0; k < kBK / 16; ++k) {
        // K-major: 16 bf16 = 32 bytes further along the swizzled 128-byte row.
        // MN-major: 16 K-rows of 128 bytes further down the tile.
        const uint64_t da = A_MN ? sm100::make_smem_desc(sa + k * 2048, 8192, 1024)
                                 : sm100::make_smem_desc(sa + k * 32, 16, 1024);
        const uint64_t db = B_MN ? sm100::make_smem_desc(sb + k * 2048, 8192, 1024)
                                 : sm100::make_smem_desc(sb + k * 32, 16, 1024);
        sm100::mma_f16_ss(tmem_base, da, db, idesc, (kt > 0 || k > 0) ? 1u : 0u);
      }
      sm100::mma_commit(&empty_bar[s]);
    }
    if (ok) sm100::mma_commit(done_bar);
  }
  __syncwarp();

  // -------------------------------- epilogue --------------------------------
  const bool done = sm100::mbar_wait(done_bar, 0, p.timeout_ns, p.status, 300);
  sm100::tc_fence_after();
  if (p.fast_epi) epilogue_rows_staged<BN>(p, tmem_base, m0, n0, warp, lane, done, smem + L::kOffA);
  else epilogue_rows<BN>(p, tmem_base, m0, n0, warp, lane, done);
  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 0) sm100::tmem_dealloc(tmem_base, BN);
}

EpiParams epi_params(const GemmArgs& a, int splits) {
  EpiParams p;
  p.M = a.M;
  p.N = a.N;
  p.C = a.C;
  p.ldc = a.ldc;
  p.c_dtype = a.c_dtype;
  p.accumulate = a.accumulate ? 1 : 0;
  p.bias = a.bias;
  p.act = a.act;
  p.alpha = a.alpha;
  p.mask = reinterpret_cast<const __nv_bfloat16*>(a.mask);
  p.ldm = a.ldm;
  p.colsum = a.colsum;
  p.status = a.status;
  p.timeout_ns = a.timeout_ns;
  p.num_k_tiles = ceil_div(a.K, kBK);
  p.splits = splits;
  static int epi_env = -1;
  if (epi_env < 0) {
    const char* v = std::getenv("FLARE_GEMM_EPI");  // "0": the per-row epilogue (epilogue_rows)
    epi_env = (v != nullptr && v[0] == '0') ? 0 : 1;
  }
  p.fast_epi = epi_env;
  p.bias_vec = (reinterpret_cast<uintptr_t>(a.bias) & 15) == 0 ? 1 : 0;
  return p;
}

template <int BN, int STAGES, bool A_MN, bool B_MN>
void launch_cfg(const GemmArgs& a, int splits, cudaStream_t stream) {
  using L = SmemLayout<BN, STAGES>;
  auto kern = gemm_bf16_kernel<BN, STAGES, A_MN, B_MN>;
  static bool attr_set = false;  // one per instantiation; set before first launch
  if (!attr_set) {
    FLARE_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kAlloc));
    attr_set = true;
  }
  // A: K-major -> inner K, outer M, box rows 128; MN-major -> inner M, outer K, box 64 rows of K.
  CUtensorMap ta = A_MN ? make_tmap_bf16(a.A, a.M, a.K, a.lda, kBK) : make_tmap_bf16(a.A, a.K, a.M, a.lda, kBM);
  CUtensorMap tb = B_MN ? make_tmap_bf16(a.B, a.N, a.K, a.ldb, kBK) : make_tmap_bf16(a.B, a.K, a.N, a.ldb, BN);
  EpiParams p = epi_params(a, splits);
  dim3 grid(ceil_div(a.M, kBM), ceil_div(a.N, BN), splits);
  kern<<<grid, kThreads, L::kAlloc, stream>>>(ta, tb, p);
  FLARE_CUDA_CHECK(cudaGetLastError());
  count_launch();
}

// ---------------------------------------------------------------------------
// CTA-pair variant (cta_group::2).  A cluster of two CTAs computes a 256 x BN
// tile: CTA r stages rows [128r, 128r + 128) of the tile's A and rows
// [r BN/2, (r+1) BN/2) of its B (32 KiB per 64-deep stage at BN = 256, against
// 48 KiB for a 128 x 256 tile on one SM), so the same shared memory holds
// STAGES = 6 stages in flight and each SM reads a third less per MMA cycle.
// Both producers count their bytes on the even CTA's full barrier; the even
// CTA's MMA warp issues the 256-row MMAs and commits to the empty / done
// barriers of both CTAs (one commit per CTA, addressed through mapa); each CTA
// runs the epilogue on its own 128 accumulator rows.  Every wait is bounded.
template <int BN, int STAGES>
struct PairLayout {
  static constexpr int kTileBytesB = (BN / 2) * kBK * 2;
  static constexpr int kStageBytes = kTileBytesA + kTileBytesB;
  static constexpr int kOffB = STAGES * kTileBytesA;
  static constexpr int kOffBar = kOffB + STAGES * kTileBytesB;
  static constexpr int kBytes = kOffBar + (2 * STAGES + 1) * 8 + 16;
  static constexpr int kAlloc = kBytes + 1024;
};

template <int BN, int STAGES, bool A_MN, bool B_MN>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    gemm_bf16_pair_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                          EpiParams p) {
  using L = PairLayout<BN, STAGES>;
  constexpr int kHalfN = BN / 2;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + L::kOffBar);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* done_bar = empty_bar + STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done_bar + 1);

  const int warp = warp_id();
  const int lane = lane_id();
  const uint32_t rank = sm100::cluster_ctarank();
  const bool leader = rank == 0;
  const int m0 = blockIdx.x * kBM;                            // this CTA's 128 rows of the pair's 256
  const int n0 = blockIdx.y * BN;                             // the pair's BN columns
  const int nb0 = n0 + static_cast<int>(rank) * kHalfN;       // the B rows this CTA stages
  const int kt_begin = static_cast<int>((static_cast<int64_t>(p.num_k_tiles) * blockIdx.z) / p.splits);
  const int kt_end = static_cast<int>((static_cast<int64_t>(p.num_k_tiles) * (blockIdx.z + 1)) / p.splits);

  if (threadIdx.x == 0) {
    sm100::tma_prefetch_desc(&tmap_a);
    sm100::tma_prefetch_desc(&tmap_b);
    for (int s = 0; s < STAGES; ++s) {
      sm100::mbar_init(&full_bar[s], 1);
      sm100::mbar_init(&empty_bar[s], 1);
    }
    sm100::mbar_init(done_bar, 1);
    sm100::fence_mbar_init();
  }
  if (warp == 0) {
    sm100::tmem_alloc_pair(tmem_slot, BN);
    sm100::tmem_relinquish_pair();
  }
  sm100::tc_fence_before();
  sm100::cluster_sync();  // both CTAs: barriers initialised and TMEM allocated before any cross-CTA use
  sm100::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int KT = kt_end - kt_begin;

  if (warp == 0 && lane == 0) {
    // ------------------------------ producer (both CTAs) ------------------------------
    for (int kt = 0; kt < KT; ++kt) {
      const int s = kt % STAGES;
      if (kt >= STAGES) {
        if (!sm100::mbar_wait(&empty_bar[s], ((kt / STAGES) - 1) & 1, p.timeout_ns, p.status, 100 + s)) break;
      }
      uint8_t* sa = smem + s * kTileBytesA;
      uint8_t* sb = smem + L::kOffB + s * L::kTileBytesB;
      if (leader) sm100::mbar_arrive_expect_tx(&full_bar[s], 2 * L::kStageBytes);
      const uint32_t bar = sm100::mapa_shared(&full_bar[s], 0);
      const int k0 = (kt_begin + kt) * kBK;
      if constexpr (!A_MN) {
        sm100::tma_load_2d_pair(sa, &tmap_a, bar, k0, m0);
      } else {
#pragma unroll
        for (int j = 0; j < kBM / 64; ++j) sm100::tma_load_2d_pair(sa + j * 8192, &tmap_a, bar, m0 + 64 * j, k0);
      }
      if constexpr (!B_MN) {
        sm100::tma_load_2d_pair(sb, &tmap_b, bar, k0, nb0);
      } else {
#pragma unroll
        for (int j = 0; j < kHalfN / 64; ++j) sm100::tma_load_2d_pair(sb + j * 8192, &tmap_b, bar, nb0 + 64 * j, k0);
      }
    }
  } else if (warp == 1 && lane == 0 && leader) {
    // ------------------------------ MMA issuer (even CTA) ------------------------------
    constexpr uint32_t idesc = sm100::make_idesc_bf16(2 * kBM, BN, A_MN, B_MN);
    bool ok = true;
    for (int kt = 0; kt < KT; ++kt) {
      const int s = kt % STAGES;
      if (!sm100::mbar_wait(&full_bar[s], (kt / STAGES) & 1, p.timeout_ns, p.status, 200 + s)) {
        ok = false;
        break;
      }
      sm100::tc_fence_after();
      const uint32_t sa = smem_u32(smem + s * kTileBytesA);
      const uint32_t sb = smem_u32(smem + L::kOffB + s * L::kTileBytesB);
#pragma unroll
      for (int k = 0; k < kBK / 16; ++k) {
        const uint64_t da = A_MN ? sm100::make_smem_desc(sa + k * 2048, 8192, 1024)
                                 : sm100::make_smem_desc(sa + k * 32, 16, 1024);
        const uint64_t db = B_MN ? sm100::make_smem_desc(sb + k * 2048, 8192, 1024)
                                 : sm100::make_smem_desc(sb + k * 32, 16, 1024);
        sm100::mma_f16_ss_pair(tmem_base, da, db, idesc, (kt > 0 || k > 0) ? 1u : 0u);
      }
      sm100::mma_commit_pair(sm100::mapa_shared(&empty_bar[s], 0));
      sm100::mma_commit_pair(sm100::mapa_shared(&empty_bar[s], 1));
    }
    if (ok) {
      sm100::mma_commit_pair(sm100::mapa_shared(done_bar, 0));
      sm100::mma_commit_pair(sm100::mapa_shared(done_bar, 1));
    }
  }
  __syncwarp();

  const bool done = sm100::mbar_wait(done_bar, 0, p.timeout_ns, p.status, 300);
  sm100::tc_fence_after();
  epilogue_rows<BN>(p, tmem_base, m0, n0, warp, lane, done);
  sm100::tc_fence_before();
  __syncthreads();
  sm100::cluster_sync();  // neither CTA frees the pair's TMEM while the other may still read it
  if (warp == 0) sm100::tmem_dealloc_pair(tmem_base, BN);
}

template <int BN, int STAGES, bool A_MN, bool B_MN>
void launch_pair_cfg(const GemmArgs& a, int splits, cudaStream_t stream) {
  using L = PairLayout<BN, STAGES>;
  auto kern = gemm_bf16_pair_kernel<BN, STAGES, A_MN, B_MN>;
  static bool attr_set = false;
  if (!attr_set) {
    FLARE_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kAlloc));
    attr_set = true;
  }
  CUtensorMap ta = A_MN ? make_tmap_bf16(a.A, a.M, a.K, a.lda, kBK) : make_tmap_bf16(a.A, a.K, a.M, a.lda, kBM);
  CUtensorMap tb = B_MN ? make_tmap_bf16(a.B, a.N, a.K, a.ldb, kBK) : make_tmap_bf16(a.B, a.K, a.N, a.ldb, BN / 2);
  EpiParams p = epi_params(a, splits);
  dim3 grid(2 * ceil_div(a.M, 2 * kBM), ceil_div(a.N, BN), splits);
  kern<<<grid, kThreads, L::kAlloc, stream>>>(ta, tb, p);
  FLARE_CUDA_CHECK(cudaGetLastError());
  count_launch();
}

template <int BN, int STAGES>
void launch_pair_majors(const GemmArgs& a, int splits, cudaStream_t s) {
  if (!a.a_mn && !a.b_mn) launch_pair_cfg<BN, STAGES, false, false>(a, splits, s);
  else if (!a.a_mn && a.b_mn) launch_pair_cfg<BN, STAGES, false, true>(a, splits, s);
  else if (a.a_mn && !a.b_mn) launch_pair_cfg<BN, STAGES, true, false>(a, splits, s);
  else launch_pair_cfg<BN, STAGES, true, true>(a, splits, s);
}

template <int BN, int STAGES>
void launch_majors(const GemmArgs& a, int splits, cudaStream_t s) {
  if (!a.a_mn && !a.b_mn) launch_cfg<BN, STAGES, false, false>(a, splits, s);
  else if (!a.a_mn && a.b_mn) launch_cfg<BN, STAGES, false, true>(a, splits, s);
  else if (a.a_mn && !a.b_mn) launch_cfg<BN, STAGES, true, false>(a, splits, s);
  else launch_cfg<BN, STAGES, true, true>(a, splits, s);
}

}  // namespace

// Number of streaming multiprocessors on the current device (cached).
int device_sm_count() {
  static int count = 0;
  if (count == 0) {
    int dev = 0;
    FLARE_CUDA_CHECK(cudaGetDevice(&dev));
    FLARE_CUDA_CHECK(cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, dev));
  }
  return count;
}

// CTA pairs are used for tiles of at least 256 rows and 128 columns when the
// call asks for them (a.pair = 1) or, with a.pair = -1, when FLARE_GEMM_PAIR=1.
static bool use_pair(const GemmArgs& a) {
  static int env = -1;
  if (env < 0) {
    const char* v = std::getenv("FLARE_GEMM_PAIR");
    env = (v != nullptr && v[0] == '1') ? 1 : 0;
  }
  const bool want = a.pair > 0 || (a.pair < 0 && env == 1);
  return want && a.M >= 2 * kBM && a.N >= 128;
}

void gemm_bf16_tcgen05(const GemmArgs& a, int bn_hint, cudaStream_t stream) {
  FLARE_CHECK(a.M > 0 && a.N > 0 && a.K > 0, "GEMM dims must be positive");
  FLARE_CHECK(a.c_dtype == kF32 || a.c_dtype == kBF16, "GEMM output must be fp32 or bf16");
  FLARE_CHECK(a.ldm % 8 == 0 || a.mask == nullptr, "mask pitch must be a multiple of 8 elements");
  FLARE_CHECK((reinterpret_cast<uintptr_t>(a.C) & 15) == 0, "C must be 16-byte aligned");
  FLARE_CHECK(a.ldc % (a.c_dtype == kF32 ? 4 : 8) == 0, "C pitch must be a multiple of 16 bytes");
  const int sms = device_sm_count();
  const int kt = ceil_div(a.K, kBK);
  const bool can_split = a.c_dtype == kF32 && a.accumulate && a.bias == nullptr && a.act == 0 &&
                         a.mask == nullptr && a.colsum == nullptr;
  int bn = bn_hint;
  if (bn == 0) {
    const int mt = ceil_div(a.M, kBM);
    if (can_split && kt >= 16 && static_cast<int64_t>(mt) * ceil_div(a.N, 128) < sms) {
      bn = a.N > 64 ? 128 : 64;  // split-K fills the GPU; keep tiles wide for operand reuse
    } else {
      // Pick the widest tile that still yields at least one wave of CTAs.
      bn = 256;
      while (bn > 64 && static_cast<int64_t>(mt) * ceil_div(a.N, bn) < sms) bn >>= 1;
      if (a.N <= 64) bn = 64;
    }
  }
  // Split-K when the output tiles cannot fill the GPU and K is long (weight
  // gradients: K = batch).  Partials reduce into fp32 C, which therefore must
  // already hold the value to accumulate onto (accumulate semantics).
  if (use_pair(a)) {
    // CTA pairs: 256 x bn tiles, two SMs each.
    const int pbn = (bn_hint == 128 || bn_hint == 256) ? bn_hint : (a.N > 128 ? 256 : 128);
    const int ctas = 2 * ceil_div(a.M, 2 * kBM) * ceil_div(a.N, pbn);
    int psplits = 1;
    if (can_split && ctas < sms && kt >= 16)
      psplits = std::min(std::min(kt / 8, 16), std::max(1, (2 * sms + ctas - 1) / ctas));
    if (pbn == 256) launch_pair_majors<256, 6>(a, psplits, stream);
    else launch_pair_majors<128, 8>(a, psplits, stream);
    return;
  }
  int splits = 1;
  const int tiles = ceil_div(a.M, kBM) * ceil_div(a.N, bn);
  if (can_split && tiles < sms && kt >= 16) {
    splits = std::min(std::min(kt / 8, 16), std::max(1, (2 * sms + tiles - 1) / tiles));
  }
  if (bn == 64) launch_majors<64, 4>(a, splits, stream);
  else if (bn == 128) launch_majors<128, 3>(a, splits, stream);
  else launch_majors<256, 4>(a, splits, stream);
}

}  // namespace flare
