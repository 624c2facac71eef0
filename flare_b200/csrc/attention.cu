// Jagged causal multi-head attention on tcgen05 (sm_100a), forward and backward.
//
// Layout (T tokens of many sequences packed back to back; every sequence
// starts at a token index that is a multiple of 8, so TMA x-coordinates along
// the token axis are 16-byte aligned):
//   QKV  [T, 768] bf16   Q | K | V, head h at columns h*32 .. h*32+31 of each
//   VT   [256, T] bf16   V transposed (row = head*32 + d)
//   QT   [256, T] bf16   Q transposed (backward only)
//   O    [T, 256] bf16,  LSE [8, T] fp32 (log2 domain, scale folded in)
// Head dim 32, 8 heads.  A CTA handles TWO heads: a 64-column (128-byte)
// TMA box of Q/K covers both, and each head's QK^T is the two 16-wide
// k-steps of its own 32 columns, so every operand uses the 128-byte swizzle.
//
// Forward (CTA = sequence x head pair x 128-row query tile, 128 threads,
// thread i = query row i = TMEM lane i):
//   pass 1: for each causal key tile, S = Q K^T into TMEM (both heads), each
//           thread reduces its row to the running max / sum;
//   pass 2: recompute S, P = exp2(S' - lse) (final, no rescaling of O), write
//           P as bf16 into shared memory in the 128-byte-swizzled K-major
//           layout and issue O += P V^T-tile (A = P from smem, B = V^T tile).
//   S is computed one head at a time into a 128-column accumulator (256 TMEM
//   columns and 82 KB of shared memory per CTA), so two CTAs share an SM and
//   one CTA's softmax overlaps the other's TMA / MMA waits; fully visible key
//   tiles skip the causal / length mask.
// Backward (CTA = sequence x head pair x 128-row key tile, thread i = key row
// i): for each causal query tile and head, S^T = K Q^T and dP^T = V dO^T into
// TMEM; P^T, dS^T = P^T (dP^T - Delta) go to shared memory; then
// dV += P^T dO, dK += dS^T Q (A = smem, B = transposed tiles), and
// dQ(tile) = dS K with dS read MN-major from the same smem buffer and K read
// MN-major from the K tile; dQ is accumulated across key tiles with fp32
// vector atomics.
//
// One elected thread issues every TMA load and MMA; waits are bounded and
// report a status code (no hang on a lost completion).
// The reference has no attention operator; the sequential-recommendation
// model is one of the benchmark configurations built on this framework.
#include "attention.cuh"
#include "gemm.cuh"
#include "sm100.cuh"

#include <cmath>
#include <algorithm>
#include <cstring>

namespace flare {

namespace {

constexpr int kT = 128;          // query / key tile
constexpr int kHD = 32;          // head dim
constexpr int kHeads = 8;
constexpr int kThreadsA = 128;
constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ void fence_proxy_async_smem_() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Write 8 consecutive bf16 values (one 16-byte chunk) of row `r`, chunk `c`
// (0..15 over a 128-wide row split in two 64-wide atoms) into a K-major
// 128-byte-swizzled tile whose atoms are `atom_bytes` apart.
__device__ __forceinline__ void st_swizzled(uint8_t* tile, int atom_bytes, int r, int c, uint4 v) {
  const int atom = c >> 3, ch = c & 7;
  uint8_t* p = tile + atom * atom_bytes + r * 128 + ((ch ^ (r & 7)) << 4);
  *reinterpret_cast<uint4*>(p) = v;
}

__device__ __forceinline__ uint4 pack_bf16x8(const float* v) {
  uint4 u;
  uint32_t* w = reinterpret_cast<uint32_t*>(&u);
#pragma unroll
  for (int t = 0; t < 4; ++t) {
    __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * t], v[2 * t + 1]);
    w[t] = *reinterpret_cast<uint32_t*>(&h);
  }
  return u;
}

// K-major SW128 descriptor for k-step k (16 elements) of an operand whose K
// extent spans atoms `atom_bytes` apart (64 elements per atom).
__device__ __forceinline__ uint64_t desc_k(uint32_t base, int atom_bytes, int k) {
  return sm100::make_smem_desc(base + (k >> 2) * atom_bytes + (k & 3) * 32, 16, 1024);
}
// MN-major SW128 descriptor for k-step k: K rows are 128-byte rows, MN atoms `lbo` apart.
__device__ __forceinline__ uint64_t desc_mn(uint32_t base, int lbo, int k) {
  return sm100::make_smem_desc(base + k * 2048, lbo, 1024);
}

struct AttnSmemF {
  static constexpr int Q = 0;            // [128 x 64] 16 KB
  static constexpr int K = 16384;        // [128 x 64] 16 KB
  static constexpr int VT = 32768;       // 2 atoms of [64 rows x 64 kv] = 16 KB
  static constexpr int P = 49152;        // one head: 2 atoms x 16 KB = 32 KB
  static constexpr int BAR = 81920;
  static constexpr int BYTES = BAR + 128 + 1024;  // two CTAs fit in one SM's shared memory
};

__global__ void __launch_bounds__(kThreadsA, 2)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tm_qkv, const __grid_constant__ CUtensorMap tm_vt,
                    AttnFwdParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* sm = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + AttnSmemF::BAR);  // 0 q, 1 kv, 2 mma
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bar + 4);
  const int tid = threadIdx.x, warp = warp_id(), lane = lane_id();
  const int qt = blockIdx.x, seq = blockIdx.y, hp = blockIdx.z;
  const int s0 = p.offsets[seq];
  const int L = p.offsets[seq + 1] - s0;
  if (qt * kT >= L) return;
  if (s0 < 0 || (s0 & 7) || static_cast<int64_t>(s0) + L > p.T_cap) {  // bad offsets: report, touch nothing
    if (threadIdx.x == 0) report_error(p.status, kIndexOutOfRange, seq);
    return;
  }
  const int q0 = s0 + qt * kT;

  if (tid == 0) {
    sm100::tma_prefetch_desc(&tm_qkv);
    sm100::tma_prefetch_desc(&tm_vt);
    for (int i = 0; i < 3; ++i) sm100::mbar_init(&bar[i], 1);
    sm100::fence_mbar_init();
  }
  if (warp == 0) {
    sm100::tmem_alloc(tslot, 256);
    sm100::tmem_relinquish();
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *tslot;
  const uint32_t tS = tmem, tO = tmem + 128;  // S: one head at a time; O: heads at +128 / +160
  const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
  constexpr uint32_t idesc_s = sm100::make_idesc_bf16(128, 128, false, false);
  constexpr uint32_t idesc_o = sm100::make_idesc_bf16(128, 32, false, false);
  const float c2 = p.scale * kLog2e;
  const int qi = qt * kT + tid;  // query index within the sequence
  uint32_t ph_mma = 0;
  bool ok = true;

  // Per key step: TMA K (+ V^T in pass 2); for each head: S_h = Q_h K_h^T into the one 128-column S
  // accumulator, softmax on it (pass 1: running max / sum; pass 2: P_h to shared memory and
  // O_h += P_h V_h^T).  256 TMEM columns and 82 KB of shared memory per CTA let two CTAs share an
  // SM, so one CTA's softmax overlaps the other's TMA and MMA waits.
  if (tid == 0) {
    sm100::mbar_arrive_expect_tx(&bar[0], kT * 64 * 2);
    sm100::tma_load_2d(sm + AttnSmemF::Q, &tm_qkv, &bar[0], hp * 64, q0);
    ok = sm100::mbar_wait(&bar[0], 0, p.timeout_ns, p.status, 10);
  }
  uint32_t ph_kv = 0;
  float m2[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
  for (int pass = 0; pass < 2; ++pass) {
    for (int kt = 0; kt <= qt; ++kt) {
      const int k0 = s0 + kt * kT;
      if (tid == 0 && ok) {
        sm100::mbar_arrive_expect_tx(&bar[1], kT * 64 * 2 + (pass ? 2 * 64 * 64 * 2 : 0));
        sm100::tma_load_2d(sm + AttnSmemF::K, &tm_qkv, &bar[1], 256 + hp * 64, k0);
        if (pass) {
          sm100::tma_load_2d(sm + AttnSmemF::VT, &tm_vt, &bar[1], k0, hp * 64);
          sm100::tma_load_2d(sm + AttnSmemF::VT + 8192, &tm_vt, &bar[1], k0 + 64, hp * 64);
        }
        ok = sm100::mbar_wait(&bar[1], ph_kv, p.timeout_ns, p.status, 11);
      }
      ph_kv ^= 1;
      // a fully visible key tile (below the diagonal, inside the sequence) needs no mask
      const bool full = kt < qt && (kt + 1) * kT <= L && qi < L;
#pragma unroll 1
      for (int h = 0; h < 2; ++h) {
        if (tid == 0 && ok) {
          sm100::tc_fence_after();
          const uint32_t qa = smem_u32(sm + AttnSmemF::Q), ka = smem_u32(sm + AttnSmemF::K);
#pragma unroll
          for (int k = 0; k < 2; ++k)
            sm100::mma_f16_ss(tS, desc_k(qa, 16384, 2 * h + k), desc_k(ka, 16384, 2 * h + k), idesc_s,
                              k > 0 ? 1u : 0u);
          sm100::mma_commit(&bar[2]);  // also covers the previous step's P.V MMAs
        }
        if (!sm100::mbar_wait(&bar[2], ph_mma, p.timeout_ns, p.status, 12)) ok = false;
        ph_mma ^= 1;
        sm100::tc_fence_after();
        float pv[128];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t r[32];
          sm100::tmem_ld_32x32b_x32(tS + lane_off + c * 32, r);
          sm100::tmem_ld_wait();
          if (full) {
#pragma unroll
            for (int j = 0; j < 32; ++j) pv[c * 32 + j] = __uint_as_float(r[j]) * c2;
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const int kj = kt * kT + c * 32 + j;
              const bool valid = kj <= qi && kj < L && qi < L;
              pv[c * 32 + j] = valid ? __uint_as_float(r[j]) * c2 : -INFINITY;
            }
          }
        }
        if (pass == 0) {
          float mx = m2[h];
#pragma unroll
          for (int j = 0; j < 128; ++j) mx = fmaxf(mx, pv[j]);
          if (mx != -INFINITY) {
            float sum = 0.f;
#pragma unroll
            for (int j = 0; j < 128; ++j) sum += exp2f(pv[j] - mx);
            l[h] = l[h] * exp2f(m2[h] - mx) + sum;
            m2[h] = mx;
          }
        } else {
          const float lse = (l[h] > 0.f) ? m2[h] + log2f(l[h]) : 0.f;
          uint8_t* pt = sm + AttnSmemF::P;  // the previous head's P.V MMAs finished (S commit above)
#pragma unroll
          for (int c = 0; c < 16; ++c) {
            float e[8];
#pragma unroll
            for (int t = 0; t < 8; ++t) e[t] = exp2f(pv[c * 8 + t] - lse);
            st_swizzled(pt, 16384, tid, c, pack_bf16x8(e));
          }
        }
        if (pass == 1) fence_proxy_async_smem_();
        sm100::tc_fence_before();
        __syncthreads();  // S read by every thread before the next S MMA overwrites it; P written
        if (pass == 1 && tid == 0 && ok) {
          // O_h += P_h V_h^T; the next S MMA's commit (or the one below) covers these MMAs
          sm100::tc_fence_after();
          const uint32_t va = smem_u32(sm + AttnSmemF::VT), pa = smem_u32(sm + AttnSmemF::P);
#pragma unroll
          for (int k = 0; k < 8; ++k)
            sm100::mma_f16_ss(tO + h * 32, desc_k(pa, 16384, k), desc_k(va + h * 4096, 8192, k), idesc_o,
                              (kt > 0 || k > 0) ? 1u : 0u);
          if (h == 1) sm100::mma_commit(&bar[2]);
        }
      }
      if (pass == 1) {
        // P and the V^T tile are overwritten next step: wait for the P.V MMAs
        if (!sm100::mbar_wait(&bar[2], ph_mma, p.timeout_ns, p.status, 13)) ok = false;
        ph_mma ^= 1;
      }
    }
  }
  // ---- epilogue: O and LSE
  sm100::tc_fence_after();
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    uint32_t r[32];
    sm100::tmem_ld_32x32b_x32(tO + h * 32 + lane_off, r);
    sm100::tmem_ld_wait();
    if (qi < L && ok) {
      const int head = hp * 2 + h;
      __nv_bfloat16* o = p.out + static_cast<int64_t>(q0 + tid) * p.ld_out + head * kHD;
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        float v[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] = __uint_as_float(r[t * 8 + e]);
        *reinterpret_cast<uint4*>(o + t * 8) = pack_bf16x8(v);
      }
      p.lse[static_cast<int64_t>(head) * p.ld_lse + q0 + tid] = (l[h] > 0.f) ? m2[h] + log2f(l[h]) : 0.f;
    }
  }
  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 0) sm100::tmem_dealloc(tmem, 256);
}

// ------------------------------------------------------------------ backward
struct AttnSmemB {
  static constexpr int K = 0;            // [128 kv x 64]
  static constexpr int V = 16384;        // [128 kv x 64]
  static constexpr int Q = 32768;        // [128 q x 64]
  static constexpr int DO = 49152;       // [128 q x 64]
  static constexpr int DOT = 65536;      // 2 atoms of [64 rows x 64 q] (dO^T)
  static constexpr int QT = 81920;       // 2 atoms of [64 rows x 64 q] (Q^T)
  static constexpr int P = 98304;        // P^T: 2 atoms of [128 kv x 64 q]
  static constexpr int DS = 131072;      // dS^T: 2 atoms of [128 kv x 64 q]
  static constexpr int STAT = 163840;    // lse[2][128], delta[2][128] fp32 = 2 KB
  static constexpr int BAR = 165888;
  static constexpr int BYTES = BAR + 128 + 1024;
};

__global__ void __launch_bounds__(kThreadsA, 1)
    attn_bwd_kernel(const __grid_constant__ CUtensorMap tm_qkv, const __grid_constant__ CUtensorMap tm_do,
                    const __grid_constant__ CUtensorMap tm_dot, const __grid_constant__ CUtensorMap tm_qt,
                    AttnBwdParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* sm = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + AttnSmemB::BAR);  // 0 kv, 1 q tiles, 2 mma
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bar + 4);
  float* st_lse = reinterpret_cast<float*>(sm + AttnSmemB::STAT);
  float* st_delta = st_lse + 256;
  const int tid = threadIdx.x, warp = warp_id(), lane = lane_id();
  const int kt = blockIdx.x, seq = blockIdx.y, hp = blockIdx.z;
  const int s0 = p.offsets[seq];
  const int L = p.offsets[seq + 1] - s0;
  if (kt * kT >= L) return;
  if (s0 < 0 || (s0 & 7) || static_cast<int64_t>(s0) + L > p.T_cap) {
    if (threadIdx.x == 0) report_error(p.status, kIndexOutOfRange, seq);
    return;
  }
  const int k0 = s0 + kt * kT;
  const int nq = (L + kT - 1) / kT;

  if (tid == 0) {
    sm100::tma_prefetch_desc(&tm_qkv);
    sm100::tma_prefetch_desc(&tm_do);
    sm100::tma_prefetch_desc(&tm_dot);
    sm100::tma_prefetch_desc(&tm_qt);
    for (int i = 0; i < 3; ++i) sm100::mbar_init(&bar[i], 1);
    sm100::fence_mbar_init();
  }
  if (warp == 0) {
    sm100::tmem_alloc(tslot, 512);
    sm100::tmem_relinquish();
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *tslot;
  // TMEM columns: S^T [0,128), dP^T [128,256), dQ [256,320), dV h0/h1 [320,384), dK h0/h1 [384,448)
  const uint32_t tS = tmem, tdP = tmem + 128, tdQ = tmem + 256, tdV = tmem + 320, tdK = tmem + 384;
  const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
  constexpr uint32_t idesc_s = sm100::make_idesc_bf16(128, 128, false, false);
  constexpr uint32_t idesc_d = sm100::make_idesc_bf16(128, 32, false, false);
  constexpr uint32_t idesc_q = sm100::make_idesc_bf16(128, 64, true, true);
  const float c2 = p.scale * kLog2e;
  const int ki = kt * kT + tid;  // key index within the sequence (thread = key row)
  uint32_t ph_q = 0, ph_mma = 0;
  bool ok = true;

  if (tid == 0) {
    sm100::mbar_arrive_expect_tx(&bar[0], 2 * kT * 64 * 2);
    sm100::tma_load_2d(sm + AttnSmemB::K, &tm_qkv, &bar[0], 256 + hp * 64, k0);
    sm100::tma_load_2d(sm + AttnSmemB::V, &tm_qkv, &bar[0], 512 + hp * 64, k0);
    ok = sm100::mbar_wait(&bar[0], 0, p.timeout_ns, p.status, 20);
  }
  bool first = true;
  for (int qt = kt; qt < nq; ++qt) {
    const int q0 = s0 + qt * kT;
    if (tid == 0 && ok) {
      sm100::mbar_arrive_expect_tx(&bar[1], 2 * kT * 64 * 2 + 4 * 64 * 64 * 2);
      sm100::tma_load_2d(sm + AttnSmemB::Q, &tm_qkv, &bar[1], hp * 64, q0);
      sm100::tma_load_2d(sm + AttnSmemB::DO, &tm_do, &bar[1], hp * 64, q0);
      sm100::tma_load_2d(sm + AttnSmemB::DOT, &tm_dot, &bar[1], q0, hp * 64);
      sm100::tma_load_2d(sm + AttnSmemB::DOT + 8192, &tm_dot, &bar[1], q0 + 64, hp * 64);
      sm100::tma_load_2d(sm + AttnSmemB::QT, &tm_qt, &bar[1], q0, hp * 64);
      sm100::tma_load_2d(sm + AttnSmemB::QT + 8192, &tm_qt, &bar[1], q0 + 64, hp * 64);
    }
    // per-query statistics of this tile (both heads)
    for (int i = tid; i < 2 * kT; i += kThreadsA) {
      const int h = i >> 7, c = i & (kT - 1);
      const int qidx = qt * kT + c;
      const int64_t col = q0 + c;
      const int head = hp * 2 + h;
      st_lse[i] = qidx < L ? p.lse[static_cast<int64_t>(head) * p.ld_stat + col] : 0.f;
      st_delta[i] = qidx < L ? p.delta[static_cast<int64_t>(head) * p.ld_stat + col] : 0.f;
    }
    if (tid == 0 && ok) ok = sm100::mbar_wait(&bar[1], ph_q, p.timeout_ns, p.status, 21);
    ph_q ^= 1;
    __syncthreads();
    for (int h = 0; h < 2; ++h) {
      if (tid == 0 && ok) {
        sm100::tc_fence_after();
        const uint32_t ka = smem_u32(sm + AttnSmemB::K), va = smem_u32(sm + AttnSmemB::V);
        const uint32_t qa = smem_u32(sm + AttnSmemB::Q), da = smem_u32(sm + AttnSmemB::DO);
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          sm100::mma_f16_ss(tS, desc_k(ka, 16384, 2 * h + k), desc_k(qa, 16384, 2 * h + k), idesc_s, k > 0);
          sm100::mma_f16_ss(tdP, desc_k(va, 16384, 2 * h + k), desc_k(da, 16384, 2 * h + k), idesc_s, k > 0);
        }
        sm100::mma_commit(&bar[2]);
      }
      if (!sm100::mbar_wait(&bar[2], ph_mma, p.timeout_ns, p.status, 22)) ok = false;
      ph_mma ^= 1;
      sm100::tc_fence_after();
      const float* lse_h = st_lse + h * kT;
      const float* del_h = st_delta + h * kT;
      // a query tile entirely after this key tile and inside the sequence needs no mask
      const bool full = qt > kt && (qt + 1) * kT <= L && ki < L;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t rs[32], rd[32];
        sm100::tmem_ld_32x32b_x32(tS + lane_off + c * 32, rs);
        sm100::tmem_ld_32x32b_x32(tdP + lane_off + c * 32, rd);
        sm100::tmem_ld_wait();
        float pt[32], ds[32];
        if (full) {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int qc = c * 32 + j;
            const float pp = exp2f(__uint_as_float(rs[j]) * c2 - lse_h[qc]);
            pt[j] = pp;
            ds[j] = pp * (__uint_as_float(rd[j]) - del_h[qc]);
          }
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int qc = c * 32 + j;
            const int qidx = qt * kT + qc;
            const bool valid = qidx >= ki && qidx < L && ki < L;
            const float pp = valid ? exp2f(__uint_as_float(rs[j]) * c2 - lse_h[qc]) : 0.f;
            pt[j] = pp;
            ds[j] = pp * (__uint_as_float(rd[j]) - del_h[qc]);
          }
        }
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          st_swizzled(sm + AttnSmemB::P, 16384, tid, c * 4 + t, pack_bf16x8(pt + 8 * t));
          st_swizzled(sm + AttnSmemB::DS, 16384, tid, c * 4 + t, pack_bf16x8(ds + 8 * t));
        }
      }
      fence_proxy_async_smem_();
      sm100::tc_fence_before();
      __syncthreads();
      if (tid == 0 && ok) {
        sm100::tc_fence_after();
        const uint32_t pa = smem_u32(sm + AttnSmemB::P), sa = smem_u32(sm + AttnSmemB::DS);
        const uint32_t dota = smem_u32(sm + AttnSmemB::DOT) + h * 4096, qta = smem_u32(sm + AttnSmemB::QT) + h * 4096;
        const uint32_t ka = smem_u32(sm + AttnSmemB::K);
        const uint32_t acc_first = (first) ? 0u : 1u;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          // dV_h += P^T dO_h ; dK_h += dS^T Q_h   (A: smem [kv x q], B: transposed tiles [32 x q])
          sm100::mma_f16_ss(tdV + h * 32, desc_k(pa, 16384, k), desc_k(dota, 8192, k), idesc_d,
                            (k > 0 || !first) ? 1u : acc_first);
          sm100::mma_f16_ss(tdK + h * 32, desc_k(sa, 16384, k), desc_k(qta, 8192, k), idesc_d,
                            (k > 0 || !first) ? 1u : acc_first);
          // dQ(tile) = dS K   (A: dS^T smem read MN-major; B: K tile read MN-major, N = both heads)
          sm100::mma_f16_ss(tdQ, desc_mn(sa, 16384, k), desc_mn(ka, 16384, k), idesc_q, k > 0 ? 1u : 0u);
        }
        sm100::mma_commit(&bar[2]);
      }
      if (!sm100::mbar_wait(&bar[2], ph_mma, p.timeout_ns, p.status, 23)) ok = false;
      ph_mma ^= 1;
      sm100::tc_fence_after();
      // dQ rows of this query tile (thread = query row), head h's 32 columns
      {
        uint32_t r[32];
        sm100::tmem_ld_32x32b_x32(tdQ + lane_off + h * 32, r);
        sm100::tmem_ld_wait();
        const int qidx = qt * kT + tid;
        if (qidx < L && ok) {
          float* dq = p.dq_acc + static_cast<int64_t>(q0 + tid) * p.ld_dq + (hp * 2 + h) * kHD;
#pragma unroll
          for (int t = 0; t < 8; ++t)
            atomicAdd(reinterpret_cast<float4*>(dq + 4 * t),
                      make_float4(__uint_as_float(r[4 * t]) * p.scale, __uint_as_float(r[4 * t + 1]) * p.scale,
                                  __uint_as_float(r[4 * t + 2]) * p.scale, __uint_as_float(r[4 * t + 3]) * p.scale));
        }
      }
      sm100::tc_fence_before();
      __syncthreads();
    }
    first = false;
  }
  // ---- dK, dV of this key tile (thread = key row)
  for (int h = 0; h < 2; ++h) {
    uint32_t rv[32], rk[32];
    sm100::tmem_ld_32x32b_x32(tdV + h * 32 + lane_off, rv);
    sm100::tmem_ld_32x32b_x32(tdK + h * 32 + lane_off, rk);
    sm100::tmem_ld_wait();
    if (ki < L && ok) {
      const int head = hp * 2 + h;
      __nv_bfloat16* dk = p.dqkv + static_cast<int64_t>(k0 + tid) * p.ld_dqkv + 256 + head * kHD;
      __nv_bfloat16* dv = p.dqkv + static_cast<int64_t>(k0 + tid) * p.ld_dqkv + 512 + head * kHD;
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        float a[8], b[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          a[e] = __uint_as_float(rk[t * 8 + e]) * p.scale;
          b[e] = __uint_as_float(rv[t * 8 + e]);
        }
        *reinterpret_cast<uint4*>(dk + t * 8) = pack_bf16x8(a);
        *reinterpret_cast<uint4*>(dv + t * 8) = pack_bf16x8(b);
      }
    }
  }
  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 0) sm100::tmem_dealloc(tmem, 512);
}

// Delta[h, t] = sum_d dO[t, h*32+d] * O[t, h*32+d]   (warp per token, lane = 8 columns)
__global__ void attn_delta_kernel(const __nv_bfloat16* __restrict__ dout, const __nv_bfloat16* __restrict__ out,
                                  int64_t ld, int64_t T, float* __restrict__ delta, int64_t ld_stat) {
  const int lane = lane_id();
  for (int64_t t = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; t < T;
       t += (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5) {
    const uint4 a = *reinterpret_cast<const uint4*>(dout + t * ld + lane * 8);
    const uint4 b = *reinterpret_cast<const uint4*>(out + t * ld + lane * 8);
    const __nv_bfloat162* ha = reinterpret_cast<const __nv_bfloat162*>(&a);
    const __nv_bfloat162* hb = reinterpret_cast<const __nv_bfloat162*>(&b);
    float s = 0.f;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 fa = __bfloat1622float2(ha[e]), fb = __bfloat1622float2(hb[e]);
      s += fa.x * fb.x + fa.y * fb.y;
    }
    // 4 lanes per head (32 columns)
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    s += __shfl_xor_sync(0xffffffffu, s, 2);
    if ((lane & 3) == 0) delta[static_cast<int64_t>(lane >> 2) * ld_stat + t] = s;
  }
}

// dqkv[:, :256] = bf16(dq_acc); dq_acc = 0
__global__ void attn_dq_finalize_kernel(float* __restrict__ dq, int64_t ld_dq, int64_t T, __nv_bfloat16* __restrict__ dqkv,
                                        int64_t ld_dqkv) {
  const int64_t n = T * 32;  // 8-element groups
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t t = i >> 5;
    const int c = static_cast<int>(i & 31) * 8;
    float4* s = reinterpret_cast<float4*>(dq + t * ld_dq + c);
    const float4 a = s[0], b = s[1];
    const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    *reinterpret_cast<uint4*>(dqkv + t * ld_dqkv + c) = pack_bf16x8(v);
    s[0] = make_float4(0.f, 0.f, 0.f, 0.f);
    s[1] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
}

}  // namespace

void attn_forward(const AttnFwdParams& p, cudaStream_t s) {
  FLARE_CHECK(p.T_cap % 8 == 0 && p.ld_qkv % 8 == 0 && p.ld_out % 8 == 0, "attention pitches must be multiples of 8");
  FLARE_CHECK(p.ld_vt % 8 == 0, "V^T pitch must be a multiple of 8");
  static bool attr = false;
  if (!attr) {
    FLARE_CUDA_CHECK(cudaFuncSetAttribute(attn_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          AttnSmemF::BYTES));
    attr = true;
  }
  const CUtensorMap tq = make_tmap_bf16(p.qkv, 768, p.T_cap, p.ld_qkv, kT);
  const CUtensorMap tv = make_tmap_bf16(p.vt, p.T_cap, 256, p.ld_vt, 64);
  dim3 grid(p.max_len / kT + (p.max_len % kT ? 1 : 0), p.nseq, kHeads / 2);
  attn_fwd_kernel<<<grid, kThreadsA, AttnSmemF::BYTES, s>>>(tq, tv, p);
  FLARE_CUDA_CHECK(cudaGetLastError());
  count_launch();
}

void attn_backward(const AttnBwdParams& p, cudaStream_t s) {
  FLARE_CHECK(p.T_cap % 8 == 0 && p.ld_qkv % 8 == 0 && p.ld_do % 8 == 0 && p.ld_t % 8 == 0 && p.ld_dqkv % 8 == 0,
              "attention pitches must be multiples of 8");
  static bool attr = false;
  if (!attr) {
    FLARE_CUDA_CHECK(cudaFuncSetAttribute(attn_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          AttnSmemB::BYTES));
    attr = true;
  }
  // Delta = rowsum(dO * O) per head
  {
    const int64_t threads = p.T_cap * 32;
    const int grid = static_cast<int>(std::min<int64_t>((threads + 255) / 256, 148 * 16));
    attn_delta_kernel<<<grid, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(p.dout),
                                           static_cast<const __nv_bfloat16*>(p.out), p.ld_do, p.T_cap, p.delta,
                                           p.ld_stat);
    FLARE_CUDA_CHECK(cudaGetLastError());
    count_launch();
  }
  const CUtensorMap tq = make_tmap_bf16(p.qkv, 768, p.T_cap, p.ld_qkv, kT);
  const CUtensorMap td = make_tmap_bf16(p.dout, 256, p.T_cap, p.ld_do, kT);
  const CUtensorMap tdt = make_tmap_bf16(p.dout_t, p.T_cap, 256, p.ld_t, 64);
  const CUtensorMap tqt = make_tmap_bf16(p.q_t, p.T_cap, 256, p.ld_t, 64);
  dim3 grid(p.max_len / kT + (p.max_len % kT ? 1 : 0), p.nseq, kHeads / 2);
  attn_bwd_kernel<<<grid, kThreadsA, AttnSmemB::BYTES, s>>>(tq, td, tdt, tqt, p);
  FLARE_CUDA_CHECK(cudaGetLastError());
  count_launch();
  {
    const int64_t n = p.T_cap * 32;
    const int grid2 = static_cast<int>(std::min<int64_t>((n + 255) / 256, 148 * 16));
    attn_dq_finalize_kernel<<<grid2, 256, 0, s>>>(p.dq_acc, p.ld_dq, p.T_cap, p.dqkv, p.ld_dqkv);
    FLARE_CUDA_CHECK(cudaGetLastError());
    count_launch();
  }
}

}  // namespace flare
