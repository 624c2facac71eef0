// Padded-inverse sparse ops (the SparseEmbeddingOperator contract of the
// reference, src/flare/kernels/contracts.py:53-96) and GPU first-occurrence
// deduplication (src/flare/ops/sparse_unique.py:52 semantics), for sm_100a.
//
//   gather          out[slot,:] = inv[slot]==pad ? 0 : emb[inv[slot],:]
//   gather_pooled   out[b,f,:]  = sum_e emb[inv[(b*F+f)*E+e],:] over non-pad e
//                   (fp32 accumulation, stored in the table dtype)
//   scatter         out[inv[slot],:] += grad[slot,:]           (fp32 output)
//   scatter_pooled  out[inv[(b*F+f)*E+e],:] += grad[b,f,:]     (fp32 output)
//   unique_first_occurrence: unique keys in first-occurrence order, int32
//   inverse, int64 first indices - deterministic (hash + atomicMin on the
//   occurrence index, then an order-preserving scan). INT64_MAX is reserved.
#include "sparse_ops.cuh"

namespace flare {
namespace {

template <typename T>
__global__ void gather_pad_kernel(const T* __restrict__ emb, const int* __restrict__ inv, int64_t slots, int dim,
                                  int pad, T* __restrict__ out) {
  const int64_t n = slots * dim;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t slot = i / dim;
    const int d = static_cast<int>(i - slot * dim);
    const int row = inv[slot];
    out[i] = row == pad ? from_f32<T>(0.f) : emb[static_cast<int64_t>(row) * dim + d];
  }
}

template <typename T>
__global__ void gather_pool_kernel(const T* __restrict__ emb, const int* __restrict__ inv, int64_t bags, int E,
                                   int dim, int pad, T* __restrict__ out) {
  const int64_t n = bags * dim;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t bag = i / dim;
    const int d = static_cast<int>(i - bag * dim);
    float acc = 0.f;
    for (int e = 0; e < E; ++e) {
      const int row = inv[bag * E + e];
      if (row != pad) acc += to_f32(emb[static_cast<int64_t>(row) * dim + d]);
    }
    out[i] = from_f32<T>(acc);
  }
}

template <typename T>
__global__ void scatter_pad_kernel(const T* __restrict__ grad, const int* __restrict__ inv, int64_t slots, int dim,
                                   int pad, float* __restrict__ out) {
  const int64_t n = slots * dim;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t slot = i / dim;
    const int d = static_cast<int>(i - slot * dim);
    const int row = inv[slot];
    if (row != pad) atomicAdd(out + static_cast<int64_t>(row) * dim + d, to_f32(grad[i]));
  }
}

// One lane per pooled-gradient element; the value stays in a register while
// the lane walks the bag's inverse slots.
template <typename T>
__global__ void scatter_pool_kernel(const T* __restrict__ grad, const int* __restrict__ inv, int64_t bags, int E,
                                    int dim, int pad, float* __restrict__ out) {
  const int64_t n = bags * dim;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t bag = i / dim;
    const int d = static_cast<int>(i - bag * dim);
    const float g = to_f32(grad[i]);
    for (int e = 0; e < E; ++e) {
      const int row = inv[bag * E + e];
      if (row != pad) atomicAdd(out + static_cast<int64_t>(row) * dim + d, g);
    }
  }
}

// ---------------------------- first-occurrence unique -----------------------
constexpr unsigned long long kEmptyKey = 0xFFFFFFFFFFFFFFFFull;

__global__ void unique_insert_kernel(const int64_t* __restrict__ keys, int64_t n, unsigned long long* tab_keys,
                                     int* tab_first, int64_t cap_mask, int64_t* slot_of) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    // Flip the sign bit so the empty sentinel (all ones) corresponds to the
    // key INT64_MAX, which is reserved; -1 and every other key are usable.
    const unsigned long long k = static_cast<unsigned long long>(keys[i]) ^ 0x8000000000000000ull;
    int64_t slot = static_cast<int64_t>(hash_mix64(k) & static_cast<unsigned long long>(cap_mask));
    while (true) {
      const unsigned long long cur = tab_keys[slot];
      if (cur == k) break;
      if (cur == kEmptyKey) {
        const unsigned long long prev = atomicCAS(tab_keys + slot, kEmptyKey, k);
        if (prev == kEmptyKey || prev == k) break;
      }
      slot = (slot + 1) & cap_mask;
    }
    atomicMin(tab_first + slot, static_cast<int>(i));
    slot_of[i] = slot;
  }
}

__global__ void unique_mark_kernel(int64_t n, const int* tab_first, const int64_t* slot_of, int* is_first) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    is_first[i] = tab_first[slot_of[i]] == static_cast<int>(i) ? 1 : 0;
}

__global__ void unique_emit_kernel(const int64_t* __restrict__ keys, int64_t n, const int* tab_first,
                                   const int64_t* slot_of, const int* is_first, const int* pos, int64_t* unique,
                                   int* inverse, int64_t* first_idx) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    if (is_first[i]) {
      unique[pos[i]] = keys[i];
      first_idx[pos[i]] = i;
    }
    inverse[i] = pos[tab_first[slot_of[i]]];
  }
}

// ----------------------------- generic int scan ------------------------------
constexpr int kScanBlocks = 512;
constexpr int kScanThreads = 512;

__device__ int block_sum(int v, int* sh) {
  v = __reduce_add_sync(0xffffffffu, v);
  if (lane_id() == 0) sh[warp_id()] = v;
  __syncthreads();
  int tot = 0;
  if (warp_id() == 0) {
    tot = lane_id() < blockDim.x / 32 ? sh[lane_id()] : 0;
    tot = __reduce_add_sync(0xffffffffu, tot);
    if (lane_id() == 0) sh[0] = tot;
  }
  __syncthreads();
  tot = sh[0];
  __syncthreads();
  return tot;
}

__global__ void scan_partial_kernel(const int* in, int64_t n, int* block_sums) {
  __shared__ int sh[32];
  const int64_t per = (n + kScanBlocks - 1) / kScanBlocks;
  const int64_t lo = min(n, blockIdx.x * per), hi = min(n, lo + per);
  int acc = 0;
  for (int64_t i = lo + threadIdx.x; i < hi; i += blockDim.x) acc += in[i];
  acc = block_sum(acc, sh);
  if (threadIdx.x == 0) block_sums[blockIdx.x] = acc;
}

__global__ void scan_final_kernel(const int* in, int64_t n, const int* block_sums, int* out) {
  __shared__ int sh[32];
  __shared__ int wsum[32];
  const int64_t per = (n + kScanBlocks - 1) / kScanBlocks;
  const int64_t lo = min(n, blockIdx.x * per), hi = min(n, lo + per);
  int base = 0;
  for (int i = threadIdx.x; i < blockIdx.x; i += blockDim.x) base += block_sums[i];
  base = block_sum(base, sh);
  const int w = warp_id(), l = lane_id();
  for (int64_t t0 = lo; t0 < hi; t0 += blockDim.x) {
    const int64_t i = t0 + threadIdx.x;
    const int c = i < hi ? in[i] : 0;
    int x = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, o);
      if (l >= o) x += y;
    }
    if (l == 31) wsum[w] = x;
    __syncthreads();
    if (w == 0) {
      int s = l < blockDim.x / 32 ? wsum[l] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, s, o);
        if (l >= o) s += y;
      }
      wsum[l] = s;
    }
    __syncthreads();
    const int warp_base = w > 0 ? wsum[w - 1] : 0;
    if (i < hi) out[i] = base + warp_base + x - c;
    const int tile_total = wsum[blockDim.x / 32 - 1];
    __syncthreads();
    base += tile_total;
  }
  if (blockIdx.x == kScanBlocks - 1 && threadIdx.x == 0) out[n] = base;
}

int grid_1d(int64_t n) {
  const int64_t want = (n + 255) / 256;
  return static_cast<int>(want < 1 ? 1 : (want > 148 * 16 ? 148 * 16 : want));
}

}  // namespace

void exclusive_scan_int(const int* in, int64_t n, int* out, int* block_sums, cudaStream_t s) {
  scan_partial_kernel<<<kScanBlocks, kScanThreads, 0, s>>>(in, n, block_sums);
  scan_final_kernel<<<kScanBlocks, kScanThreads, 0, s>>>(in, n, block_sums, out);
  FLARE_CUDA_CHECK(cudaGetLastError());
  count_launch(2);
}

#define FLARE_DISPATCH_FLOAT(dtype, T, ...)                    \
  do {                                                         \
    count_launch();                                            \
    if ((dtype) == kF32) {                                     \
      using T = float;                                         \
      __VA_ARGS__;                                             \
    } else if ((dtype) == kBF16) {                             \
      using T = __nv_bfloat16;                                 \
      __VA_ARGS__;                                             \
    } else {                                                   \
      using T = __half;                                        \
      __VA_ARGS__;                                             \
    }                                                          \
  } while (0)

void sparse_gather(const void* emb, int dtype, const int* inv, int64_t slots, int dim, int pad, void* out,
                   cudaStream_t s) {
  FLARE_DISPATCH_FLOAT(dtype, T,
                       gather_pad_kernel<T><<<grid_1d(slots * dim), 256, 0, s>>>(
                           static_cast<const T*>(emb), inv, slots, dim, pad, static_cast<T*>(out)));
  FLARE_CUDA_CHECK(cudaGetLastError());
}

void sparse_gather_pooled(const void* emb, int dtype, const int* inv, int64_t bags, int E, int dim, int pad,
                          void* out, cudaStream_t s) {
  FLARE_DISPATCH_FLOAT(dtype, T,
                       gather_pool_kernel<T><<<grid_1d(bags * dim), 256, 0, s>>>(
                           static_cast<const T*>(emb), inv, bags, E, dim, pad, static_cast<T*>(out)));
  FLARE_CUDA_CHECK(cudaGetLastError());
}

void sparse_scatter(const void* grad, int dtype, const int* inv, int64_t slots, int dim, int pad, float* out,
                    cudaStream_t s) {
  FLARE_DISPATCH_FLOAT(dtype, T,
                       scatter_pad_kernel<T><<<grid_1d(slots * dim), 256, 0, s>>>(
                           static_cast<const T*>(grad), inv, slots, dim, pad, out));
  FLARE_CUDA_CHECK(cudaGetLastError());
}

void sparse_scatter_pooled(const void* grad, int dtype, const int* inv, int64_t bags, int E, int dim, int pad,
                           float* out, cudaStream_t s) {
  FLARE_DISPATCH_FLOAT(dtype, T,
                       scatter_pool_kernel<T><<<grid_1d(bags * dim), 256, 0, s>>>(
                           static_cast<const T*>(grad), inv, bags, E, dim, pad, out));
  FLARE_CUDA_CHECK(cudaGetLastError());
}

void unique_first_occurrence(const int64_t* keys, int64_t n, const UniqueScratch& w, int64_t* unique, int* inverse,
                             int64_t* first_idx, cudaStream_t s) {
  FLARE_CHECK(n < (1ll << 31) - 1, "unique supports fewer than 2^31 keys");
  FLARE_CHECK((w.cap & (w.cap - 1)) == 0 && w.cap >= 2 * n, "hash capacity must be a power of two >= 2n");
  FLARE_CUDA_CHECK(cudaMemsetAsync(w.tab_keys, 0xFF, w.cap * sizeof(unsigned long long), s));
  FLARE_CUDA_CHECK(cudaMemsetAsync(w.tab_first, 0x7F, w.cap * sizeof(int), s));
  const int g = grid_1d(n);
  unique_insert_kernel<<<g, 256, 0, s>>>(keys, n, w.tab_keys, w.tab_first, w.cap - 1, w.slot_of);
  unique_mark_kernel<<<g, 256, 0, s>>>(n, w.tab_first, w.slot_of, w.is_first);
  exclusive_scan_int(w.is_first, n, w.pos, w.block_sums, s);
  unique_emit_kernel<<<g, 256, 0, s>>>(keys, n, w.tab_first, w.slot_of, w.is_first, w.pos, unique, inverse,
                                       first_idx);
  FLARE_CUDA_CHECK(cudaGetLastError());
  count_launch(3);
}

}  // namespace flare
