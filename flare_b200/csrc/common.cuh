// Shared device/host helpers for every flare_b200 CUDA kernel (sm_100a only).
//
// Every spin-wait in this code base is bounded: waits read %globaltimer and
// give up after a caller-provided budget, record an error code in a device
// status word and return, so that a missing peer or a lost signal surfaces as
// a host-side exception instead of a hung GPU.
#pragma once

#include <cstdint>
#include <cstdio>
#include <stdexcept>
#include <string>

#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#define FLARE_CUDA_CHECK(expr)                                                   \
  do {                                                                           \
    cudaError_t _e = (expr);                                                     \
    if (_e != cudaSuccess) {                                                     \
      throw std::runtime_error(std::string("CUDA error ") +                      \
                               cudaGetErrorString(_e) + " at " __FILE__ ":" +    \
                               std::to_string(__LINE__) + " in " #expr);        \
    }                                                                            \
  } while (0)

#define FLARE_CHECK(cond, msg)                                                   \
  do {                                                                           \
    if (!(cond)) {                                                               \
      throw std::runtime_error(std::string("flare_b200: ") + (msg) + " [" #cond  \
                               "] at " __FILE__ ":" + std::to_string(__LINE__)); \
    }                                                                            \
  } while (0)

namespace flare {

// Device status word layout (int32[4] per status buffer):
//   [0] first error code (0 = ok), [1] detail (e.g. peer / stage),
//   [2] count of errors, [3] reserved.
enum StatusCode : int {
  kOk = 0,
  kTimeoutMbarrier = 1,
  kTimeoutPeerSignal = 2,
  kIndexOutOfRange = 3,
  kCapacityOverflow = 4,
  kBadArgument = 5,
};

#if defined(__CUDACC__)
__device__ __forceinline__ void report_error(int* status, int code, int detail) {
  if (status == nullptr) return;
  if (atomicCAS(status, 0, code) == 0) status[1] = detail;
  atomicAdd(status + 2, 1);
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Mark `row` dirty in a bitmap of 32 rows per word (the bitmap of a 200M-row collection is 25 MB and
// stays in L2, where a byte per row would cost a DRAM sector read-modify-write per touched row).
__device__ __forceinline__ void mark_dirty(unsigned* bits, long long row) {
  if (bits != nullptr) atomicOr(bits + (row >> 5), 1u << (row & 31));
}

__device__ __forceinline__ int lane_id() { return threadIdx.x & 31; }
__device__ __forceinline__ int warp_id() { return threadIdx.x >> 5; }

// ---------------------------------------------------------------------------
// System-scope flag primitives used for cross-GPU signalling over NVLink.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void st_release_sys(volatile uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const volatile uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void fence_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

// Wait until *flag >= target (wrap-safe compare), bounded by timeout_ns.
// Returns true on success, false (and records kTimeoutPeerSignal) on timeout.
__device__ __forceinline__ bool wait_flag_geq(const volatile uint32_t* flag, uint32_t target,
                                              uint64_t timeout_ns, int* status, int detail) {
  uint64_t t0 = global_timer_ns();
  while (true) {
    uint32_t v = ld_acquire_sys(flag);
    if (static_cast<int32_t>(v - target) >= 0) return true;
    if (global_timer_ns() - t0 > timeout_ns) {
      report_error(status, kTimeoutPeerSignal, detail);
      return false;
    }
    __nanosleep(64);
  }
}

// ---------------------------------------------------------------------------
// bf16 / fp16 vector helpers
// ---------------------------------------------------------------------------
template <typename T> struct VecT;
template <> struct VecT<float> { static constexpr int kPer16B = 4; };
template <> struct VecT<__nv_bfloat16> { static constexpr int kPer16B = 8; };
template <> struct VecT<__half> { static constexpr int kPer16B = 8; };

__device__ __forceinline__ float to_f32(float v) { return v; }
__device__ __forceinline__ float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float to_f32(__half v) { return __half2float(v); }

template <typename T> __device__ __forceinline__ T from_f32(float v);
template <> __device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}
template <> __device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }

// Load 4 consecutive elements of T starting at p (p aligned to 4*sizeof(T)), as fp32.
template <typename T> __device__ __forceinline__ float4 load4(const T* p);
template <> __device__ __forceinline__ float4 load4<float>(const float* p) {
  return *reinterpret_cast<const float4*>(p);
}
template <> __device__ __forceinline__ float4 load4<__nv_bfloat16>(const __nv_bfloat16* p) {
  uint2 u = *reinterpret_cast<const uint2*>(p);
  __nv_bfloat162 a = *reinterpret_cast<__nv_bfloat162*>(&u.x);
  __nv_bfloat162 b = *reinterpret_cast<__nv_bfloat162*>(&u.y);
  float2 fa = __bfloat1622float2(a), fb = __bfloat1622float2(b);
  return make_float4(fa.x, fa.y, fb.x, fb.y);
}
template <> __device__ __forceinline__ float4 load4<__half>(const __half* p) {
  uint2 u = *reinterpret_cast<const uint2*>(p);
  __half2 a = *reinterpret_cast<__half2*>(&u.x);
  __half2 b = *reinterpret_cast<__half2*>(&u.y);
  float2 fa = __half22float2(a), fb = __half22float2(b);
  return make_float4(fa.x, fa.y, fb.x, fb.y);
}

template <typename T> __device__ __forceinline__ void store4(T* p, float4 v);
template <> __device__ __forceinline__ void store4<float>(float* p, float4 v) {
  *reinterpret_cast<float4*>(p) = v;
}
template <> __device__ __forceinline__ void store4<__nv_bfloat16>(__nv_bfloat16* p, float4 v) {
  __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y);
  __nv_bfloat162 b = __floats2bfloat162_rn(v.z, v.w);
  uint2 u;
  u.x = *reinterpret_cast<uint32_t*>(&a);
  u.y = *reinterpret_cast<uint32_t*>(&b);
  *reinterpret_cast<uint2*>(p) = u;
}
template <> __device__ __forceinline__ void store4<__half>(__half* p, float4 v) {
  __half2 a = __floats2half2_rn(v.x, v.y);
  __half2 b = __floats2half2_rn(v.z, v.w);
  uint2 u;
  u.x = *reinterpret_cast<uint32_t*>(&a);
  u.y = *reinterpret_cast<uint32_t*>(&b);
  *reinterpret_cast<uint2*>(p) = u;
}

__device__ __forceinline__ float4 f4_add(float4 a, float4 b) {
  return make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w);
}
__device__ __forceinline__ float4 f4_scale(float4 a, float s) {
  return make_float4(a.x * s, a.y * s, a.z * s, a.w * s);
}

// 64-bit finaliser of MurmurHash3 (Austin Appleby, public domain): every output bit depends on
// every input bit, so masking its low bits to a power-of-two table spreads keys that differ only
// in their high bits (ids with a table tag packed above bit 32, multiples of 2^20, ...).
__device__ __forceinline__ unsigned long long hash_mix64(unsigned long long k) {
  k ^= k >> 33;
  k *= 0xff51afd7ed558ccdull;
  k ^= k >> 33;
  k *= 0xc4ceb9fe1a85ec53ull;
  k ^= k >> 33;
  return k;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

#endif  // __CUDACC__

inline int ceil_div(int64_t a, int64_t b) { return static_cast<int>((a + b - 1) / b); }

// Host-side count of kernels launched by this library (inspected by tests and
// by the benchmark's launch accounting; under stream capture it counts the
// kernel nodes recorded into the graph).
void count_launch(int n = 1);
long long launch_count();

// Element type tag shared between Python and C++ (matches flare_b200/ops/_dtypes.py).
enum DType : int { kF32 = 0, kBF16 = 1, kF16 = 2 };

}  // namespace flare
