// Memory-bound kernels of the sequential-recommendation transformer (sm_100a).
//
// Width is fixed at d = 256 (8 heads x 32): a warp owns one token row and
// each lane 8 consecutive columns (one 16-byte vector), so every kernel is a
// single pass of 16-byte loads/stores with warp-shuffle reductions.
//   * token embedding combine: x = item + [side_0 | side_1 | side_2 | side_3]
//   * LayerNorm forward (saves mean / rstd) and backward (adds the residual
//     gradient, accumulates gamma / beta gradients per block then atomically)
//   * sampled softmax over [positive | 512 shared negatives]: loss, d logits,
//     and the positive-side gradients (d y and d e_pos) in one pass
//   * split of the input-embedding gradient back into item / side columns.
// The GEMMs (QKV, V^T, Q^T, output projection, FFN) run on the tcgen05 GEMMs
// and the attention in attention.cu.  The reference has no sequential model;
// this is the framework's own design for that benchmark configuration.
#include "seqrec.cuh"

#include <algorithm>

namespace flare {

namespace {

constexpr int kD = 256;
constexpr int kWarps = 8;

__device__ __forceinline__ void ld8(const __nv_bfloat16* p, float* v) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int t = 0; t < 4; ++t) {
    const float2 f = __bfloat1622float2(h[t]);
    v[2 * t] = f.x;
    v[2 * t + 1] = f.y;
  }
}
__device__ __forceinline__ void st8(__nv_bfloat16* p, const float* v) {
  uint4 u;
  uint32_t* w = reinterpret_cast<uint32_t*>(&u);
#pragma unroll
  for (int t = 0; t < 4; ++t) {
    __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * t], v[2 * t + 1]);
    w[t] = *reinterpret_cast<uint32_t*>(&h);
  }
  *reinterpret_cast<uint4*>(p) = u;
}

int rows_grid(int64_t rows) {
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((rows + kWarps - 1) / kWarps, 148 * 16)));
}

__global__ void __launch_bounds__(kWarps * 32) embed_combine_kernel(const __nv_bfloat16* __restrict__ pooled,
                                                                     int64_t ldp, int64_t T,
                                                                     __nv_bfloat16* __restrict__ x, int64_t ldx) {
  const int lane = lane_id();
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * kWarps + warp_id(); t < T;
       t += static_cast<int64_t>(gridDim.x) * kWarps) {
    float a[8], b[8];
    ld8(pooled + t * ldp + lane * 8, a);
    ld8(pooled + t * ldp + kD + lane * 8, b);
#pragma unroll
    for (int e = 0; e < 8; ++e) a[e] += b[e];
    st8(x + t * ldx + lane * 8, a);
  }
}

__global__ void __launch_bounds__(kWarps * 32) layernorm_fwd_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx,
                                                                     int64_t T, const __nv_bfloat16* __restrict__ gamma,
                                                                     const __nv_bfloat16* __restrict__ beta, float eps,
                                                                     __nv_bfloat16* __restrict__ y, int64_t ldy,
                                                                     float* __restrict__ mean,
                                                                     float* __restrict__ rstd) {
  const int lane = lane_id();
  float g[8], bb[8];
  ld8(gamma + lane * 8, g);
  ld8(beta + lane * 8, bb);
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * kWarps + warp_id(); t < T;
       t += static_cast<int64_t>(gridDim.x) * kWarps) {
    float v[8];
    ld8(x + t * ldx + lane * 8, v);
    float s = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) s += v[e];
    const float mu = warp_sum(s) * (1.f / kD);
    float q = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) q += (v[e] - mu) * (v[e] - mu);
    const float rs = rsqrtf(warp_sum(q) * (1.f / kD) + eps);
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = (v[e] - mu) * rs * g[e] + bb[e];
    st8(y + t * ldy + lane * 8, v);
    if (lane == 0) {
      mean[t] = mu;
      rstd[t] = rs;
    }
  }
}

// dx = rstd * (g*dy - mean(g*dy) - xhat * mean(g*dy*xhat)) (+ residual); dgamma += dy*xhat; dbeta += dy
__global__ void __launch_bounds__(kWarps * 32) layernorm_bwd_kernel(
    const __nv_bfloat16* __restrict__ dy, int64_t lddy, const __nv_bfloat16* __restrict__ x, int64_t ldx, int64_t T,
    const __nv_bfloat16* __restrict__ gamma, const float* __restrict__ mean, const float* __restrict__ rstd,
    const __nv_bfloat16* __restrict__ resid, int64_t ldr, __nv_bfloat16* __restrict__ dx, int64_t lddx,
    float* __restrict__ dgamma, float* __restrict__ dbeta) {
  __shared__ float red[2][kWarps][kD];
  const int lane = lane_id(), warp = warp_id();
  float g[8], dg[8], db[8];
  ld8(gamma + lane * 8, g);
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    dg[e] = 0.f;
    db[e] = 0.f;
  }
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * kWarps + warp; t < T;
       t += static_cast<int64_t>(gridDim.x) * kWarps) {
    float d[8], v[8];
    ld8(dy + t * lddy + lane * 8, d);
    ld8(x + t * ldx + lane * 8, v);
    const float mu = mean[t], rs = rstd[t];
    float a = 0.f, b = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float xh = (v[e] - mu) * rs;
      const float gd = g[e] * d[e];
      a += gd;
      b += gd * xh;
      dg[e] += d[e] * xh;
      db[e] += d[e];
      v[e] = xh;
    }
    a = warp_sum(a) * (1.f / kD);
    b = warp_sum(b) * (1.f / kD);
    float o[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] = rs * (g[e] * d[e] - a - v[e] * b);
    if (resid != nullptr) {
      float r[8];
      ld8(resid + t * ldr + lane * 8, r);
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] += r[e];
    }
    st8(dx + t * lddx + lane * 8, o);
  }
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    red[0][warp][lane * 8 + e] = dg[e];
    red[1][warp][lane * 8 + e] = db[e];
  }
  __syncthreads();
  for (int c = threadIdx.x; c < kD; c += blockDim.x) {
    float s0 = 0.f, s1 = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      s0 += red[0][w][c];
      s1 += red[1][w][c];
    }
    atomicAdd(dgamma + c, s0);
    atomicAdd(dbeta + c, s1);
  }
}

// Sampled softmax, one warp per token t (a valid token with a next token):
//   pos = y_t . e_t (e_t = target item embedding row), neg = logits[t, 0..N)
//   loss_t = logsumexp(pos, neg) - pos; p = softmax
//   dneg[t, j] = p_j * w ; dpos_t = (p_pos - 1) * w  with w = 1 / num_valid
//   dy_t = dpos_t * e_t  (the negative part is added by the following GEMM)
// The target row's gradient dpos_t * y_t is added by the gradient-split kernel.
__global__ void __launch_bounds__(kWarps * 32) sampled_softmax_kernel(SampledSoftmaxParams p) {
  __shared__ float lsum[kWarps];
  const int lane = lane_id(), warp = warp_id();
  float loss_acc = 0.f;
  const float w = 1.f / fmaxf(static_cast<float>(*p.num_valid), 1.f);
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * kWarps + warp; t < p.T;
       t += static_cast<int64_t>(gridDim.x) * kWarps) {
    const int tgt = p.target_row[t];
    if (tgt < 0) {  // padding / last token of a sequence: zero gradients
      float z[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      st8(p.dy + t * p.lddy + lane * 8, z);
      for (int j = lane; j < p.N; j += 32) p.dneg[t * p.lddneg + j] = __float2bfloat16_rn(0.f);
      if (lane == 0) p.dpos[t] = 0.f;
      continue;
    }
    float y[8], e[8];
    ld8(p.y + t * p.ldy + lane * 8, y);
    ld8(p.emb + static_cast<int64_t>(tgt) * p.ldemb + lane * 8, e);
    float dot = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) dot += y[k] * e[k];
    const float pos = warp_sum(dot);
    const float* lg = p.logits + t * p.ldlog;
    float mx = pos;
    for (int j = lane; j < p.N; j += 32) mx = fmaxf(mx, lg[j]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float se = 0.f;
    for (int j = lane; j < p.N; j += 32) se += __expf(lg[j] - mx);
    se = warp_sum(se) + __expf(pos - mx);
    const float lse = mx + __logf(se);
    const float inv = 1.f / se;
    for (int j = lane; j < p.N; j += 32) p.dneg[t * p.lddneg + j] = __float2bfloat16_rn(__expf(lg[j] - mx) * inv * w);
    const float dpos = (__expf(pos - mx) * inv - 1.f) * w;
    if (lane == 0) {
      loss_acc += lse - pos;
      p.dpos[t] = dpos;
    }
    float o[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) o[k] = dpos * e[k];
    st8(p.dy + t * p.lddy + lane * 8, o);
  }
  if (lane == 0) lsum[warp] = loss_acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    float s = 0.f;
    for (int i = 0; i < kWarps; ++i) s += lsum[i];
    if (s != 0.f) atomicAdd(p.loss_sum, s);
  }
}

// Pooled-embedding gradient of token row r (r < T):
//   item part  = dx[r] + dpos[r-1] * y[r-1]   when token r-1 predicts row r
//   side parts = dx[r]                          (x = item + [sides])
__global__ void __launch_bounds__(kWarps * 32) embed_grad_split_kernel(
    const __nv_bfloat16* __restrict__ dx, int64_t lddx, const __nv_bfloat16* __restrict__ y, int64_t ldy,
    const float* __restrict__ dpos, const int* __restrict__ target_row, int64_t T, __nv_bfloat16* __restrict__ grad,
    int64_t ldg) {
  const int lane = lane_id();
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * kWarps + warp_id(); r < T;
       r += static_cast<int64_t>(gridDim.x) * kWarps) {
    float d[8], g[8];
    ld8(dx + r * lddx + lane * 8, d);
#pragma unroll
    for (int e = 0; e < 8; ++e) g[e] = d[e];
    if (r > 0 && target_row[r - 1] == r) {
      float yv[8];
      ld8(y + (r - 1) * ldy + lane * 8, yv);
      const float dp = dpos[r - 1];
#pragma unroll
      for (int e = 0; e < 8; ++e) g[e] += dp * yv[e];
    }
    st8(grad + r * ldg + lane * 8, g);
    st8(grad + r * ldg + kD + lane * 8, d);
  }
}

}  // namespace

void seq_embed_combine(const __nv_bfloat16* pooled, int64_t ldp, int64_t T, __nv_bfloat16* x, int64_t ldx,
                       cudaStream_t s) {
  FLARE_CHECK(ldp % 8 == 0 && ldx % 8 == 0, "pitches must be multiples of 8");
  embed_combine_kernel<<<rows_grid(T), kWarps * 32, 0, s>>>(pooled, ldp, T, x, ldx);
  FLARE_CUDA_CHECK(cudaGetLastError());
  count_launch();
}

void seq_layernorm_fwd(const __nv_bfloat16* x, int64_t ldx, int64_t T, const __nv_bfloat16* gamma,
                       const __nv_bfloat16* beta,
                       float eps, __nv_bfloat16* y, int64_t ldy, float* mean, float* rstd, cudaStream_t s) {
  FLARE_CHECK(ldx % 8 == 0 && ldy % 8 == 0, "pitches must be multiples of 8");
  layernorm_fwd_kernel<<<rows_grid(T), kWarps * 32, 0, s>>>(x, ldx, T, gamma, beta, eps, y, ldy, mean, rstd);
  FLARE_CUDA_CHECK(cudaGetLastError());
  count_launch();
}

void seq_layernorm_bwd(const __nv_bfloat16* dy, int64_t lddy, const __nv_bfloat16* x, int64_t ldx, int64_t T,
                       const __nv_bfloat16* gamma, const float* mean, const float* rstd, const __nv_bfloat16* resid,
                       int64_t ldr, __nv_bfloat16* dx, int64_t lddx, float* dgamma, float* dbeta, cudaStream_t s) {
  FLARE_CHECK(lddy % 8 == 0 && ldx % 8 == 0 && lddx % 8 == 0 && (resid == nullptr || ldr % 8 == 0),
              "pitches must be multiples of 8");
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((T + 255) / 256, 148 * 4)));
  layernorm_bwd_kernel<<<grid, kWarps * 32, 0, s>>>(dy, lddy, x, ldx, T, gamma, mean, rstd, resid, ldr, dx, lddx,
                                                   dgamma, dbeta);
  FLARE_CUDA_CHECK(cudaGetLastError());
  count_launch();
}

void seq_sampled_softmax(const SampledSoftmaxParams& p, cudaStream_t s) {
  FLARE_CHECK(p.ldy % 8 == 0 && p.lddy % 8 == 0 && p.ldemb % 8 == 0, "pitches must be multiples of 8");
  sampled_softmax_kernel<<<rows_grid(p.T), kWarps * 32, 0, s>>>(p);
  FLARE_CUDA_CHECK(cudaGetLastError());
  count_launch();
}

void seq_embed_grad_split(const __nv_bfloat16* dx, int64_t lddx, const __nv_bfloat16* y, int64_t ldy,
                          const float* dpos, const int* target_row, int64_t T, __nv_bfloat16* grad, int64_t ldg,
                          cudaStream_t s) {
  FLARE_CHECK(lddx % 8 == 0 && ldy % 8 == 0 && ldg % 8 == 0, "pitches must be multiples of 8");
  embed_grad_split_kernel<<<rows_grid(T), kWarps * 32, 0, s>>>(dx, lddx, y, ldy, dpos, target_row, T, grad, ldg);
  FLARE_CUDA_CHECK(cudaGetLastError());
  count_launch();
}

}  // namespace flare
