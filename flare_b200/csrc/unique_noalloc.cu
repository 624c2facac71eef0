// Allocation-free variant of the GPU first-occurrence deduplication.
//
// This entry point has no counterpart in the reference; it is an addition of
// this library.
//
//   extern "C" int flare_unique_first_occurrence_noalloc(
//       const int64_t* keys, int64_t n, int64_t* unique, int32_t* inverse,
//       int64_t* first_index, int32_t* num_unique, void* stream);
//
// Who it is for: callers that cannot call cudaMalloc.  Some host programs own
// every byte of device memory through their own pool and reserve it up front
// (for example an inference or feature-serving process that embeds this
// library and must keep its memory footprint fixed after start-up), and some
// call sites sit on latency-critical paths where an allocation, with the
// device synchronisation it can imply, is not acceptable.  Such callers pass
// their own input and output buffers and need the library to bring its own
// working memory.
//
// What it does: same contract as flare_b200.ops.sparse.unique_first_occurrence
// (the allocating entry point): `unique[0:k]` are the distinct keys in the
// order of their first occurrence, `inverse[i]` is the position of keys[i] in
// `unique`, `first_index[j]` is the index of unique[j]'s first occurrence, and
// k is written to `*num_unique` (all outputs are device memory with room for
// n entries).  INT64_MAX is reserved and must not appear as a key.
//
// Scratch memory: a file-scope `static __device__` array of about 9 MiB
// (kNaScratchBytes) that every GPU which loads this library keeps until the
// process exits.  It bounds one call to kNaMaxKeys = 262,144 keys; larger n is
// rejected with return code -1 and a message on stderr, before any work is
// enqueued.  The first call on a device looks up the array's device address
// with cudaGetSymbolAddress (with that device current) and caches it; make
// that first call before any stream capture on that device.  Every call uses
// the same array and the array keeps the previous call's contents, so each
// call first clears the part it uses; calls whose execution overlaps on the
// GPU (different streams, or different host threads without ordering) race on
// the array and must be serialised by the caller.
//
// The cached address belongs to the device's primary context: after
// cudaDeviceReset (or anything else that destroys and recreates the primary
// context) the module is loaded again at a possibly different address, so a
// caller that resets a device must call flare_unique_noalloc_forget_device()
// for it before the next call on that device.
//
// Return codes: 0 ok, -1 n out of range, -2 the scratch address could not be
// obtained, -3 a kernel launch failed.  Launch errors are read with
// cudaPeekAtLastError, which leaves the error state as it is: an error that
// was already pending before the call (left by other code) is also reported
// as -3, and stays pending for its owner to see.  The function performs no cudaMalloc,
// cudaFree or other allocating call; work is enqueued on `stream` and the
// function does not wait for it.
#include "unique_noalloc.h"

#include "common.cuh"

#include <mutex>

namespace flare {
namespace {

constexpr int64_t kNaMaxKeys = 1 << 18;    // keys per call
constexpr int64_t kNaTableSlots = 1 << 19;  // hash slots, >= 2 * kNaMaxKeys
constexpr int kNaScanBlocks = 256;
constexpr int kNaThreads = 256;
constexpr int kNaMaxDevices = 64;
constexpr unsigned long long kNaEmpty = 0xFFFFFFFFFFFFFFFFull;

struct NaScratch {
  unsigned long long tab_keys[kNaTableSlots];  // 4 MiB
  int tab_first[kNaTableSlots];                // 2 MiB
  int slot_of[kNaMaxKeys];                     // 1 MiB
  int is_first[kNaMaxKeys];                    // 1 MiB
  int pos[kNaMaxKeys + 1];                     // 1 MiB
  int block_sums[kNaScanBlocks];
};
constexpr size_t kNaScratchBytes = sizeof(NaScratch);

static __device__ __align__(256) NaScratch g_na_scratch;

__global__ void na_clear_kernel(NaScratch* s, int64_t cap) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < cap;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    s->tab_keys[i] = kNaEmpty;
    s->tab_first[i] = 0x7FFFFFFF;
  }
}

__global__ void na_insert_kernel(NaScratch* s, const int64_t* __restrict__ keys, int64_t n, int64_t cap_mask) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    // sign bit flipped so the empty pattern stands for the reserved INT64_MAX
    const unsigned long long k = static_cast<unsigned long long>(keys[i]) ^ 0x8000000000000000ull;
    int64_t slot = static_cast<int64_t>(hash_mix64(k) & static_cast<unsigned long long>(cap_mask));
    while (true) {
      const unsigned long long cur = s->tab_keys[slot];
      if (cur == k) break;
      if (cur == kNaEmpty) {
        const unsigned long long prev = atomicCAS(s->tab_keys + slot, kNaEmpty, k);
        if (prev == kNaEmpty || prev == k) break;
      }
      slot = (slot + 1) & cap_mask;
    }
    atomicMin(s->tab_first + slot, static_cast<int>(i));
    s->slot_of[i] = static_cast<int>(slot);
  }
}

__global__ void na_mark_kernel(NaScratch* s, int64_t n) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    s->is_first[i] = s->tab_first[s->slot_of[i]] == static_cast<int>(i) ? 1 : 0;
}

__device__ int na_block_sum(int v, int* sh) {
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

__global__ void na_scan_partial_kernel(NaScratch* s, int64_t n) {
  __shared__ int sh[32];
  const int64_t per = (n + kNaScanBlocks - 1) / kNaScanBlocks;
  const int64_t lo = min(n, blockIdx.x * per), hi = min(n, lo + per);
  int acc = 0;
  for (int64_t i = lo + threadIdx.x; i < hi; i += blockDim.x) acc += s->is_first[i];
  acc = na_block_sum(acc, sh);
  if (threadIdx.x == 0) s->block_sums[blockIdx.x] = acc;
}

__global__ void na_scan_final_kernel(NaScratch* s, int64_t n) {
  __shared__ int sh[32];
  __shared__ int wsum[32];
  const int64_t per = (n + kNaScanBlocks - 1) / kNaScanBlocks;
  const int64_t lo = min(n, blockIdx.x * per), hi = min(n, lo + per);
  int base = 0;
  for (int i = threadIdx.x; i < blockIdx.x; i += blockDim.x) base += s->block_sums[i];
  base = na_block_sum(base, sh);
  const int w = warp_id(), l = lane_id();
  for (int64_t t0 = lo; t0 < hi; t0 += blockDim.x) {
    const int64_t i = t0 + threadIdx.x;
    const int c = i < hi ? s->is_first[i] : 0;
    int x = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, o);
      if (l >= o) x += y;
    }
    if (l == 31) wsum[w] = x;
    __syncthreads();
    if (w == 0) {
      int v = l < blockDim.x / 32 ? wsum[l] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, v, o);
        if (l >= o) v += y;
      }
      wsum[l] = v;
    }
    __syncthreads();
    if (i < hi) s->pos[i] = base + (w > 0 ? wsum[w - 1] : 0) + x - c;
    const int tile_total = wsum[blockDim.x / 32 - 1];
    __syncthreads();
    base += tile_total;
  }
  if (blockIdx.x == kNaScanBlocks - 1 && threadIdx.x == 0) s->pos[n] = base;
}

__global__ void na_emit_kernel(NaScratch* s, const int64_t* __restrict__ keys, int64_t n, int64_t* unique,
                               int32_t* inverse, int64_t* first_index, int32_t* num_unique) {
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (tid == 0) *num_unique = s->pos[n];
  for (int64_t i = tid; i < n; i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    if (s->is_first[i]) {
      unique[s->pos[i]] = keys[i];
      first_index[s->pos[i]] = i;
    }
    inverse[i] = s->pos[s->tab_first[s->slot_of[i]]];
  }
}

__global__ void na_zero_count_kernel(int32_t* num_unique) { *num_unique = 0; }

std::mutex g_na_mu;
NaScratch* g_na_cache[kNaMaxDevices] = {};

NaScratch* na_scratch_for_current_device() {
  std::mutex& mu = g_na_mu;
  NaScratch** cache = g_na_cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kNaMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (cache[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_na_scratch);
    if (e != cudaSuccess || p == nullptr) {
      std::fprintf(stderr, "flare_unique_first_occurrence_noalloc: cudaGetSymbolAddress failed: %s\n",
                   cudaGetErrorString(e));
      return nullptr;
    }
    cache[dev] = static_cast<NaScratch*>(p);
  }
  return cache[dev];
}

int na_grid(int64_t n) {
  const int64_t want = (n + kNaThreads - 1) / kNaThreads;
  return static_cast<int>(want < 1 ? 1 : (want > 148 * 8 ? 148 * 8 : want));
}

}  // namespace
}  // namespace flare

extern "C" __attribute__((visibility("default"))) int flare_unique_first_occurrence_noalloc(
    const int64_t* keys, int64_t n, int64_t* unique, int32_t* inverse, int64_t* first_index, int32_t* num_unique,
    void* stream) {
  using namespace flare;
  if (n < 0 || n > kNaMaxKeys) {
    std::fprintf(stderr,
                 "flare_unique_first_occurrence_noalloc: n=%lld keys is outside the supported range [0, %lld] "
                 "(fixed scratch of %zu bytes)\n",
                 static_cast<long long>(n), static_cast<long long>(kNaMaxKeys), kNaScratchBytes);
    return -1;
  }
  NaScratch* s = na_scratch_for_current_device();
  if (s == nullptr) return -2;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (n == 0) {
    na_zero_count_kernel<<<1, 1, 0, st>>>(num_unique);
    return cudaPeekAtLastError() == cudaSuccess ? 0 : -3;
  }
  int64_t cap = 1;
  while (cap < 2 * n) cap <<= 1;
  const int g = na_grid(n);
  na_clear_kernel<<<na_grid(cap), kNaThreads, 0, st>>>(s, cap);
  na_insert_kernel<<<g, kNaThreads, 0, st>>>(s, keys, n, cap - 1);
  na_mark_kernel<<<g, kNaThreads, 0, st>>>(s, n);
  na_scan_partial_kernel<<<kNaScanBlocks, kNaThreads, 0, st>>>(s, n);
  na_scan_final_kernel<<<kNaScanBlocks, kNaThreads, 0, st>>>(s, n);
  na_emit_kernel<<<g, kNaThreads, 0, st>>>(s, keys, n, unique, inverse, first_index, num_unique);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -3;
}

// Drop the cached scratch address of `device` (after cudaDeviceReset on it); the next call on that
// device looks the address up again.  Returns 0, or -1 for a device number out of range.
extern "C" __attribute__((visibility("default"))) int flare_unique_noalloc_forget_device(int device) {
  using namespace flare;
  if (device < 0 || device >= kNaMaxDevices) return -1;
  std::lock_guard<std::mutex> lock(g_na_mu);
  g_na_cache[device] = nullptr;
  return 0;
}
