// Row-wise sparse optimizer update shared by the fused embedding backward passes.
//
// One row's fp32 gradient sum is held by a group of G lanes (each lane covers
// 4*NV consecutive columns); the update reads the row's optimizer state,
// applies the LR policy (frequency score) and weight decay, and writes the
// weights back.  Reference semantics: the row-wise optimizers and LR policies
// of the reference's embedding store (src/flare/runtime/fluxway/workers/
// dynamic_embedding.py:481-549, optimizer_step after fp32 accumulation).
#pragma once

#include "embedding.cuh"

namespace flare {

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

__device__ __forceinline__ void resolve_sparse_step(SparseOptParams& o) {
  if (o.step_ptr != nullptr) {
    const float t = static_cast<float>(*o.step_ptr);
    o.bias_corr1 = 1.f - powf(o.beta1, t);
    o.bias_corr2 = 1.f - powf(o.beta2, t);
  }
}

// Sum over the G lanes of an aligned lane group (G a power of two).
__device__ __forceinline__ float group_sum(float v, int G) {
  for (int o = G >> 1; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Apply the sparse optimizer to one row.  Called by every lane of the warp in
// lockstep; a group of G lanes owns the row and lane `leader` is its first
// lane; a lane covers columns [col, col + 4*NV) of the row when `act`.
// `state_row_old` (row-wise optimizers): the row's state, if the leader lane
// loaded it already (a negative value: load it here).
template <typename TW, int NV>
__device__ __forceinline__ void apply_update(const SparseOptParams& o, TW* w, int64_t eoff, long long row,
                                             bool row_ok, bool act, int ncols, float4 (&gv4)[NV],
                                             float4 (&wv4)[NV], int count, int G, int leader,
                                             float state_row_old = -1.f) {
  float* g = reinterpret_cast<float*>(gv4);
  float* wv = reinterpret_cast<float*>(wv4);
  float lr = o.lr;
  if (o.score != nullptr) {
    float sc = 0.f;
    if (row_ok && lane_id() == leader) {
      sc = o.score[row] + static_cast<float>(count);
      o.score[row] = sc;
    }
    sc = __shfl_sync(0xffffffffu, sc, leader);
    lr *= lr_scale(o, sc);
  }
#pragma unroll
  for (int e = 0; e < 4 * NV; ++e) g[e] = g[e] * o.grad_scale + o.weight_decay * wv[e];
  if (o.kind == kOptRowwiseAdagrad || o.kind == kOptRowwiseAdam) {
    float sq = 0.f;
    if (act) {
#pragma unroll
      for (int e = 0; e < 4 * NV; ++e) sq += g[e] * g[e];
    }
    sq = group_sum(sq, G) / static_cast<float>(ncols);
    float st = 0.f;
    if (row_ok && lane_id() == leader) {
      // a caller that loaded the (non-negative) row state early passes it in
      const float old = state_row_old >= 0.f ? state_row_old : o.state_row[row];
      st = o.kind == kOptRowwiseAdagrad ? old + sq : o.beta2 * old + (1.f - o.beta2) * sq;
      o.state_row[row] = st;
    }
    st = __shfl_sync(0xffffffffu, st, leader);
    if (o.kind == kOptRowwiseAdagrad) {
      const float scale = lr / (sqrtf(st) + o.eps);
#pragma unroll
      for (int e = 0; e < 4 * NV; ++e) wv[e] -= scale * g[e];
    } else if (act) {
      const float denom = sqrtf(st / o.bias_corr2) + o.eps;
#pragma unroll
      for (int v = 0; v < NV; ++v) {
        float4 m = *reinterpret_cast<float4*>(o.state_m + eoff + 4 * v);
        float* mm = reinterpret_cast<float*>(&m);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          mm[e] = o.beta1 * mm[e] + (1.f - o.beta1) * g[4 * v + e];
          wv[4 * v + e] -= lr * (mm[e] / o.bias_corr1) / denom;
        }
        *reinterpret_cast<float4*>(o.state_m + eoff + 4 * v) = m;
      }
    }
  } else if (act) {
    if (o.kind == kOptSgd) {
#pragma unroll
      for (int e = 0; e < 4 * NV; ++e) wv[e] -= lr * g[e];
    } else if (o.kind == kOptAdagrad) {
#pragma unroll
      for (int v = 0; v < NV; ++v) {
        float4 m = *reinterpret_cast<float4*>(o.state_m + eoff + 4 * v);
        float* mm = reinterpret_cast<float*>(&m);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          mm[e] += g[4 * v + e] * g[4 * v + e];
          wv[4 * v + e] -= lr * g[4 * v + e] / (sqrtf(mm[e]) + o.eps);
        }
        *reinterpret_cast<float4*>(o.state_m + eoff + 4 * v) = m;
      }
    } else if (o.kind == kOptAdam) {
#pragma unroll
      for (int v = 0; v < NV; ++v) {
        float4 m = *reinterpret_cast<float4*>(o.state_m + eoff + 4 * v);
        float4 s2 = *reinterpret_cast<float4*>(o.state_v + eoff + 4 * v);
        float* mm = reinterpret_cast<float*>(&m);
        float* vv = reinterpret_cast<float*>(&s2);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float ge = g[4 * v + e];
          mm[e] = o.beta1 * mm[e] + (1.f - o.beta1) * ge;
          vv[e] = o.beta2 * vv[e] + (1.f - o.beta2) * ge * ge;
          wv[4 * v + e] -= lr * (mm[e] / o.bias_corr1) / (sqrtf(vv[e] / o.bias_corr2) + o.eps);
        }
        *reinterpret_cast<float4*>(o.state_m + eoff + 4 * v) = m;
        *reinterpret_cast<float4*>(o.state_v + eoff + 4 * v) = s2;
      }
    }
  }
  if (act) {
#pragma unroll
    for (int v = 0; v < NV; ++v) store4<TW>(w + 4 * v, wv4[v]);
  }
}

}  // namespace flare
