// On-device exact ranking metrics: AUC (ties get half credit) and grouped AUC.
//
// Semantics follow the reference's exact distributed AUC
// (recipes/recsys/ranking/metrics/ray_data.py:242-523): positives get full
// credit for every negative with a lower score and half credit for every
// negative with an equal score; GAUC averages per-group AUC over groups that
// have both classes, weighted by (positives + negative_factor * negatives).
//
// Method: a stable LSD radix sort of 64-bit keys (score bits mapped to an
// order-preserving unsigned integer, optionally prefixed by the group id)
// carrying the labels, then an exclusive scan of negatives, then per positive
// two binary searches (first and one-past-last index of its key) give the
// negatives strictly below and tied.  Per-group sums are accumulated at the
// group's first index.  All sums are exact integers or fp64.
#include "common.cuh"
#include "sparse_ops.cuh"

#include <algorithm>

namespace flare {
namespace {

constexpr int kSortThreads = 256;
constexpr int kTile = 4096;  // elements per block per pass
constexpr int kBins = 256;

__device__ __forceinline__ unsigned lanemask_lt_m() {
  unsigned m;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

// Per-tile digit histogram.
__global__ void radix_hist_kernel(const unsigned long long* keys, int64_t n, int shift, int* hist, int ntiles) {
  __shared__ int h[kBins];
  for (int i = threadIdx.x; i < kBins; i += blockDim.x) h[i] = 0;
  __syncthreads();
  const int64_t lo = static_cast<int64_t>(blockIdx.x) * kTile;
  const int64_t hi = min(n, lo + kTile);
  for (int64_t i = lo + threadIdx.x; i < hi; i += blockDim.x) atomicAdd(&h[(keys[i] >> shift) & 0xFF], 1);
  __syncthreads();
  // digit-major layout: hist[d * ntiles + tile]
  for (int d = threadIdx.x; d < kBins; d += blockDim.x) hist[d * ntiles + blockIdx.x] = h[d];
}

// Stable scatter: the tile is processed in rounds of blockDim elements; an
// element's rank among equal digits is (earlier rounds) + (earlier warps of
// this round) + (earlier lanes of its warp).
__global__ void radix_scatter_kernel(const unsigned long long* keys_in, const int* vals_in,
                                     unsigned long long* keys_out, int* vals_out, int64_t n, int shift,
                                     const int* offsets, int ntiles) {
  __shared__ int base[kBins];
  __shared__ int wcount[kSortThreads / 32][kBins];
  const int warp = warp_id(), lane = lane_id();
  for (int d = threadIdx.x; d < kBins; d += blockDim.x) base[d] = offsets[d * ntiles + blockIdx.x];
  const int64_t lo = static_cast<int64_t>(blockIdx.x) * kTile;
  const int64_t hi = min(n, lo + kTile);
  for (int64_t r0 = lo; r0 < hi; r0 += blockDim.x) {
    for (int i = threadIdx.x; i < (kSortThreads / 32) * kBins; i += blockDim.x) (&wcount[0][0])[i] = 0;
    __syncthreads();
    const int64_t i = r0 + threadIdx.x;
    const bool valid = i < hi;
    unsigned long long k = 0;
    int v = 0, dgt = -1;
    if (valid) {
      k = keys_in[i];
      v = vals_in[i];
      dgt = static_cast<int>((k >> shift) & 0xFF);
    }
    const unsigned vmask = __ballot_sync(0xffffffffu, valid);
    int rank_in_warp = 0;
    if (valid) {
      const unsigned peers = __match_any_sync(vmask, dgt);
      rank_in_warp = __popc(peers & lanemask_lt_m());
      if (rank_in_warp == 0) wcount[warp][dgt] = __popc(peers);
    }
    __syncthreads();
    if (valid) {
      int before = 0;
      for (int w = 0; w < warp; ++w) before += wcount[w][dgt];
      const int pos = base[dgt] + before + rank_in_warp;
      keys_out[pos] = k;
      vals_out[pos] = v;
    }
    __syncthreads();
    // advance per-digit bases by this round's counts
    for (int d = threadIdx.x; d < kBins; d += blockDim.x) {
      int c = 0;
      for (int w = 0; w < kSortThreads / 32; ++w) c += wcount[w][d];
      base[d] += c;
    }
    __syncthreads();
  }
}

// Order-preserving map of an fp32 score to uint32.
__device__ __forceinline__ uint32_t score_key(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__global__ void make_keys_kernel(const float* scores, const int64_t* groups, int64_t n, unsigned long long* keys,
                                 int* vals, const float* labels) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const unsigned long long g = groups ? static_cast<unsigned long long>(static_cast<uint32_t>(groups[i])) : 0ull;
    keys[i] = (g << 32) | score_key(scores[i]);
    vals[i] = labels[i] > 0.5f ? 1 : 0;
  }
}

__global__ void neg_flags_kernel(const int* vals, int64_t n, int* negs) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    negs[i] = 1 - vals[i];
}

__device__ __forceinline__ int64_t lower_bound_u64(const unsigned long long* a, int64_t n, unsigned long long x) {
  int64_t lo = 0, hi = n;
  while (lo < hi) {
    const int64_t mid = (lo + hi) >> 1;
    if (a[mid] < x) lo = mid + 1; else hi = mid;
  }
  return lo;
}

// Per positive: credit = negatives below + 0.5 * negatives tied (within its
// group when grouped).  Accumulates per group at the group's first index.
__global__ void auc_credit_kernel(const unsigned long long* keys, const int* vals, const int* neg_prefix, int64_t n,
                                  int grouped, double* credit, unsigned long long* pos_cnt, unsigned long long* neg_cnt,
                                  double* total_credit) {
  double local = 0.0;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const unsigned long long k = keys[i];
    const int64_t gs = grouped ? lower_bound_u64(keys, n, k & 0xFFFFFFFF00000000ull) : 0;
    if (vals[i] == 1) {
      const int64_t lb = lower_bound_u64(keys, n, k);
      const int64_t ub = lower_bound_u64(keys, n, k + 1);  // keys are < 2^64 - 1 in practice
      const double below = static_cast<double>(neg_prefix[lb] - neg_prefix[gs]);
      const double tied = static_cast<double>(neg_prefix[ub] - neg_prefix[lb]);
      const double c = below + 0.5 * tied;
      if (grouped) {
        atomicAdd(credit + gs, c);
        atomicAdd(pos_cnt + gs, 1ull);
      } else {
        local += c;
      }
    } else if (grouped) {
      atomicAdd(neg_cnt + gs, 1ull);
    }
  }
  if (!grouped) {
    for (int o = 16; o > 0; o >>= 1) local += __shfl_xor_sync(0xffffffffu, local, o);
    if (lane_id() == 0 && local != 0.0) atomicAdd(total_credit, local);
  }
}

// GAUC reduction over group starts.
__global__ void gauc_reduce_kernel(const double* credit, const unsigned long long* pos_cnt,
                                   const unsigned long long* neg_cnt,
                                   int64_t n, double negative_factor, double* out /* [2]: weighted sum, weight */) {
  double s = 0.0, w = 0.0;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const unsigned long long P = pos_cnt[i], N = neg_cnt[i];
    if (P > 0 && N > 0) {
      const double auc = credit[i] / (static_cast<double>(P) * static_cast<double>(N));
      const double wt = static_cast<double>(P) + negative_factor * static_cast<double>(N);
      s += auc * wt;
      w += wt;
    }
  }
  for (int o = 16; o > 0; o >>= 1) {
    s += __shfl_xor_sync(0xffffffffu, s, o);
    w += __shfl_xor_sync(0xffffffffu, w, o);
  }
  if (lane_id() == 0) {
    if (s != 0.0) atomicAdd(out, s);
    if (w != 0.0) atomicAdd(out + 1, w);
  }
}

int grid_m(int64_t n) {
  const int64_t want = (n + 255) / 256;
  return static_cast<int>(want < 1 ? 1 : (want > 148 * 16 ? 148 * 16 : want));
}

}  // namespace

// Stable LSD radix sort of (key, value) pairs on the low `bits` bits; the
// sorted result ends in keys_a / vals_a (the b buffers are ping-pong scratch).
void radix_sort_pairs(unsigned long long* keys_a, int* vals_a, unsigned long long* keys_b, int* vals_b, int64_t n,
                      int bits, int* hist, int* hist_scan, int* block_sums, cudaStream_t s) {
  const int ntiles = static_cast<int>((n + kTile - 1) / kTile);
  unsigned long long* kin = keys_a;
  int* vin = vals_a;
  unsigned long long* kout = keys_b;
  int* vout = vals_b;
  int passes = (bits + 7) / 8;
  for (int p = 0; p < passes; ++p) {
    const int shift = 8 * p;
    radix_hist_kernel<<<ntiles, kSortThreads, 0, s>>>(kin, n, shift, hist, ntiles);
    exclusive_scan_int(hist, static_cast<int64_t>(kBins) * ntiles, hist_scan, block_sums, s);
    radix_scatter_kernel<<<ntiles, kSortThreads, 0, s>>>(kin, vin, kout, vout, n, shift, hist_scan, ntiles);
    count_launch(2);
    std::swap(kin, kout);
    std::swap(vin, vout);
  }
  if (kin != keys_a) {
    FLARE_CUDA_CHECK(cudaMemcpyAsync(keys_a, kin, n * sizeof(unsigned long long), cudaMemcpyDeviceToDevice, s));
    FLARE_CUDA_CHECK(cudaMemcpyAsync(vals_a, vin, n * sizeof(int), cudaMemcpyDeviceToDevice, s));
  }
  FLARE_CUDA_CHECK(cudaGetLastError());
}

struct AucWork {
  unsigned long long* keys_a;
  unsigned long long* keys_b;
  int* vals_a;
  int* vals_b;
  int* negs;
  int* neg_prefix;  // [n+1]
  int* hist;        // [256 * ntiles]
  int* hist_scan;   // [256 * ntiles + 1]
  int* block_sums;  // [512]
  double* credit;   // [n] (grouped)
  unsigned long long* pos_cnt;
  unsigned long long* neg_cnt;
  double* out;      // [2]
};

// out[0] = AUC numerator (credit) for ungrouped, or weighted GAUC sum; out[1]
// = weight sum (grouped).  The caller divides.
void auc_device(const float* scores, const float* labels, const int64_t* groups, int64_t n, double negative_factor,
                const AucWork& w, cudaStream_t s) {
  FLARE_CHECK(n > 0 && n < (1ll << 31) - 1, "auc: 0 < n < 2^31");
  FLARE_CUDA_CHECK(cudaMemsetAsync(w.out, 0, 2 * sizeof(double), s));
  const int g = grid_m(n);
  make_keys_kernel<<<g, 256, 0, s>>>(scores, groups, n, w.keys_a, w.vals_a, labels);
  radix_sort_pairs(w.keys_a, w.vals_a, w.keys_b, w.vals_b, n, groups ? 64 : 32, w.hist, w.hist_scan, w.block_sums,
                   s);
  neg_flags_kernel<<<g, 256, 0, s>>>(w.vals_a, n, w.negs);
  exclusive_scan_int(w.negs, n, w.neg_prefix, w.block_sums, s);
  if (groups) {
    FLARE_CUDA_CHECK(cudaMemsetAsync(w.credit, 0, n * sizeof(double), s));
    FLARE_CUDA_CHECK(cudaMemsetAsync(w.pos_cnt, 0, n * sizeof(long long), s));
    FLARE_CUDA_CHECK(cudaMemsetAsync(w.neg_cnt, 0, n * sizeof(long long), s));
  }
  auc_credit_kernel<<<g, 256, 0, s>>>(w.keys_a, w.vals_a, w.neg_prefix, n, groups ? 1 : 0, w.credit, w.pos_cnt,
                                      w.neg_cnt, w.out);
  if (groups) gauc_reduce_kernel<<<g, 256, 0, s>>>(w.credit, w.pos_cnt, w.neg_cnt, n, negative_factor, w.out);
  count_launch(groups ? 4 : 3);
  FLARE_CUDA_CHECK(cudaGetLastError());
}

}  // namespace flare
