// DCN-v2 elementwise and reduction kernels (sm_100a).
//
// The model (flare_b200/models/dcn.py) is 3 low-rank cross layers
//   x_{l+1} = x0 * (U_l (V_l x_l) + b_l) + x_l
// in parallel with a 4-layer ReLU tower, and a logistic head over
// [x_L, h_4].  The GEMMs (with the tensor/FSDP collectives fused in) are in
// gemm_dist.cu; this file holds the memory-bound pieces around them, each a
// single pass over its operands with 16-byte vector accesses:
//   * concat of the pooled embeddings and the dense features into x0;
//   * the wide BCE head (logit, loss, d logit, d input) - warp per sample;
//   * column sums weighted by a per-row scale (head weight gradient);
//   * the cross-layer backward elementwise part with the bias-gradient
//     column sums fused in;
//   * the fp32 -> bf16 pooled-embedding gradient.
// The reference expresses the same model family through Flax layers compiled
// by XLA (src/flare/jax/layers/base.py:27 MLP; the DCN-v2 cross layer is a
// config of the benchmark suite, not a reference kernel).
#include "dcn.cuh"

#include <algorithm>

namespace flare {

namespace {

constexpr int kWarps = 8;

__device__ __forceinline__ void bf8_to_f(uint4 u, float* v) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int t = 0; t < 4; ++t) {
    const float2 f = __bfloat1622float2(h[t]);
    v[2 * t] = f.x;
    v[2 * t + 1] = f.y;
  }
}
__device__ __forceinline__ uint4 f_to_bf8(const float* v) {
  uint4 u;
  uint32_t* w = reinterpret_cast<uint32_t*>(&u);
#pragma unroll
  for (int t = 0; t < 4; ++t) {
    __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * t], v[2 * t + 1]);
    w[t] = *reinterpret_cast<uint32_t*>(&h);
  }
  return u;
}

__global__ void __launch_bounds__(kWarps * 32) concat_x0_kernel(const __nv_bfloat16* __restrict__ pooled, int64_t ldp,
                                                                 const float* __restrict__ dense, int nd, int64_t B,
                                                                 int E, __nv_bfloat16* __restrict__ x0, int64_t ld0) {
  const int lane = lane_id();
  for (int64_t b = static_cast<int64_t>(blockIdx.x) * kWarps + warp_id(); b < B;
       b += static_cast<int64_t>(gridDim.x) * kWarps) {
    const uint4* src = reinterpret_cast<const uint4*>(pooled + b * ldp);
    uint4* dst = reinterpret_cast<uint4*>(x0 + b * ld0);
    for (int v = lane; v < E / 8; v += 32) dst[v] = src[v];
    for (int c = E + lane; c < ld0; c += 32) {
      const int j = c - E;
      x0[b * ld0 + c] = __float2bfloat16_rn(j < nd ? dense[b * nd + j] : 0.f);
    }
  }
}

__global__ void __launch_bounds__(kWarps * 32) dcn_head_kernel(DcnHeadParams p) {
  __shared__ float red[2][kWarps];
  const int lane = lane_id(), warp = warp_id();
  float loss_acc = 0.f, db_acc = 0.f;
  const int nv = p.H / 8;
  for (int64_t b = static_cast<int64_t>(blockIdx.x) * kWarps + warp; b < p.B;
       b += static_cast<int64_t>(gridDim.x) * kWarps) {
    const uint4* h = reinterpret_cast<const uint4*>(p.h + b * p.ldh);
    const uint4* w = reinterpret_cast<const uint4*>(p.w);
    float acc = 0.f;
    for (int v = lane; v < nv; v += 32) {
      float hv[8], wv[8];
      bf8_to_f(h[v], hv);
      bf8_to_f(w[v], wv);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc = fmaf(hv[e], wv[e], acc);
    }
    const float x = warp_sum(acc) + __bfloat162float(p.bias[0]);
    const float y = p.labels[b];
    const float wt = (p.valid_count >= 0 && b >= p.valid_count) ? 0.f : 1.f;
    // softplus(x) - y*x = max(x,0) - x*y + log1p(exp(-|x|))
    const float l = fmaxf(x, 0.f) - x * y + log1pf(__expf(-fabsf(x)));
    const float sg = 1.f / (1.f + __expf(-x));
    const float dl = wt * (sg - y) * p.grad_scale;
    if (lane == 0) {
      p.logits[b] = x;
      p.dl[b] = dl;
      loss_acc += wt * l;
      db_acc += dl;
    }
    uint4* dh = reinterpret_cast<uint4*>(p.dh + b * p.lddh);
    for (int v = lane; v < nv; v += 32) {
      float hv[8], wv[8], o[8];
      bf8_to_f(h[v], hv);
      bf8_to_f(w[v], wv);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const bool relu = v * 8 + e >= p.relu_from;
        o[e] = (relu && hv[e] <= 0.f) ? 0.f : dl * wv[e];
      }
      dh[v] = f_to_bf8(o);
    }
  }
  if (lane == 0) {
    red[0][warp] = loss_acc;
    red[1][warp] = db_acc;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float a = 0.f, d = 0.f;
    for (int i = 0; i < kWarps; ++i) {
      a += red[0][i];
      d += red[1][i];
    }
    if (a != 0.f) atomicAdd(p.loss_sum, a);
    if (d != 0.f) atomicAdd(p.db, d);
  }
}

// Block = 8 warps x 256 columns (8 per lane); grid.y splits the rows.
constexpr int kColBlock = 256;
constexpr int kRowsPerBlock = 256;

__global__ void __launch_bounds__(kWarps * 32) scaled_colsum_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx,
                                                                     const float* __restrict__ scale, int64_t rows,
                                                                     int cols, float* __restrict__ out) {
  __shared__ float part[kWarps][kColBlock];
  const int lane = lane_id(), warp = warp_id();
  const int c0 = blockIdx.x * kColBlock + lane * 8;
  const int64_t r0 = static_cast<int64_t>(blockIdx.y) * kRowsPerBlock;
  const int64_t r1 = min(r0 + kRowsPerBlock, rows);
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  if (c0 < cols) {
    for (int64_t r = r0 + warp; r < r1; r += kWarps) {
      float v[8];
      bf8_to_f(*reinterpret_cast<const uint4*>(x + r * ldx + c0), v);
      const float s = scale[r];
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] = fmaf(s, v[e], acc[e]);
    }
  }
#pragma unroll
  for (int e = 0; e < 8; ++e) part[warp][lane * 8 + e] = acc[e];
  __syncthreads();
  const int c = blockIdx.x * kColBlock + threadIdx.x;
  if (c < cols) {
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) s += part[w][threadIdx.x];
    atomicAdd(out + c, s);
  }
}

__global__ void __launch_bounds__(kWarps * 32) cross_bwd_elem_kernel(
    const __nv_bfloat16* __restrict__ g, int64_t ldg, const __nv_bfloat16* __restrict__ x0,
    const __nv_bfloat16* __restrict__ z, int64_t ld, int64_t rows, int cols, __nv_bfloat16* __restrict__ dz, float* __restrict__ acc_out, int64_t ld_acc,
    int accumulate, float* __restrict__ db) {
  __shared__ float part[kWarps][kColBlock];
  const int lane = lane_id(), warp = warp_id();
  const int c0 = blockIdx.x * kColBlock + lane * 8;
  const int64_t r0 = static_cast<int64_t>(blockIdx.y) * kRowsPerBlock;
  const int64_t r1 = min(r0 + kRowsPerBlock, rows);
  float cs[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  if (c0 < cols) {
    for (int64_t r = r0 + warp; r < r1; r += kWarps) {
      float gv[8], xv[8], zv[8], d[8];
      const int64_t o = r * ld + c0;
      bf8_to_f(*reinterpret_cast<const uint4*>(g + r * ldg + c0), gv);
      bf8_to_f(*reinterpret_cast<const uint4*>(x0 + o), xv);
      bf8_to_f(*reinterpret_cast<const uint4*>(z + o), zv);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        d[e] = gv[e] * xv[e];
        cs[e] += d[e];
      }
      *reinterpret_cast<uint4*>(dz + o) = f_to_bf8(d);
      float4* a = reinterpret_cast<float4*>(acc_out + r * ld_acc + c0);
      float4 a0 = make_float4(gv[0] * zv[0], gv[1] * zv[1], gv[2] * zv[2], gv[3] * zv[3]);
      float4 a1 = make_float4(gv[4] * zv[4], gv[5] * zv[5], gv[6] * zv[6], gv[7] * zv[7]);
      if (accumulate) {
        a0 = f4_add(a0, a[0]);
        a1 = f4_add(a1, a[1]);
      }
      a[0] = a0;
      a[1] = a1;
    }
  }
#pragma unroll
  for (int e = 0; e < 8; ++e) part[warp][lane * 8 + e] = cs[e];
  __syncthreads();
  const int c = blockIdx.x * kColBlock + threadIdx.x;
  if (c < cols) {
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) s += part[w][threadIdx.x];
    atomicAdd(db + c, s);
  }
}

__global__ void finalize_grad_kernel(const float* __restrict__ acc, int64_t ld_acc, int64_t rows, int cols,
                                     __nv_bfloat16* __restrict__ grad, int64_t ldg) {
  const int nv = cols / 8;
  const int64_t n = rows * nv;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / nv;
    const int c = static_cast<int>(i - r * nv) * 8;
    const float4* a = reinterpret_cast<const float4*>(acc + r * ld_acc + c);
    const float4 a0 = a[0], a1 = a[1];
    const float v[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
    *reinterpret_cast<uint4*>(grad + r * ldg + c) = f_to_bf8(v);
  }
}

int grid_rows(int64_t rows, int per_block) {
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((rows + per_block - 1) / per_block, 148 * 16)));
}

}  // namespace

void dcn_concat_x0(const __nv_bfloat16* pooled, int64_t ldp, const float* dense, int nd, int64_t B, int E,
                   __nv_bfloat16* x0, int64_t ld0, cudaStream_t s) {
  FLARE_CHECK(E % 8 == 0 && ldp % 8 == 0 && ld0 % 8 == 0 && ld0 >= E + nd, "bad x0 layout");
  concat_x0_kernel<<<grid_rows(B, kWarps), kWarps * 32, 0, s>>>(pooled, ldp, dense, nd, B, E, x0, ld0);
  FLARE_CUDA_CHECK(cudaGetLastError());
  count_launch();
}

void dcn_head(const DcnHeadParams& p, cudaStream_t s) {
  FLARE_CHECK(p.H % 8 == 0 && p.ldh % 8 == 0 && p.lddh % 8 == 0, "head width and pitches must be multiples of 8");
  dcn_head_kernel<<<grid_rows(p.B, kWarps), kWarps * 32, 0, s>>>(p);
  FLARE_CUDA_CHECK(cudaGetLastError());
  count_launch();
}

void dcn_scaled_colsum(const __nv_bfloat16* x, int64_t ldx, const float* scale, int64_t rows, int cols, float* out,
                       cudaStream_t s) {
  FLARE_CHECK(cols % 8 == 0 && ldx % 8 == 0, "columns and pitch must be multiples of 8");
  dim3 grid(ceil_div(cols, kColBlock), ceil_div(rows, kRowsPerBlock));
  scaled_colsum_kernel<<<grid, kWarps * 32, 0, s>>>(x, ldx, scale, rows, cols, out);
  FLARE_CUDA_CHECK(cudaGetLastError());
  count_launch();
}

void dcn_cross_bwd_elem(const __nv_bfloat16* g, int64_t ldg, const __nv_bfloat16* x0, const __nv_bfloat16* z, int64_t ld,
                        int64_t rows, int cols, __nv_bfloat16* dz, float* acc, int64_t ld_acc, int accumulate,
                        float* db, cudaStream_t s) {
  FLARE_CHECK(cols % 8 == 0 && ld % 8 == 0 && ldg % 8 == 0 && ld_acc % 4 == 0,
              "columns and pitches must be multiples of 8");
  dim3 grid(ceil_div(cols, kColBlock), ceil_div(rows, kRowsPerBlock));
  cross_bwd_elem_kernel<<<grid, kWarps * 32, 0, s>>>(g, ldg, x0, z, ld, rows, cols, dz, acc, ld_acc, accumulate, db);
  FLARE_CUDA_CHECK(cudaGetLastError());
  count_launch();
}

void dcn_finalize_grad(const float* acc, int64_t ld_acc, int64_t rows, int cols, __nv_bfloat16* grad, int64_t ldg,
                       cudaStream_t s) {
  FLARE_CHECK(cols % 8 == 0 && ld_acc % 4 == 0 && ldg % 8 == 0, "columns and pitches must be multiples of 8");
  const int64_t n = rows * (cols / 8);
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, 148 * 8)));
  finalize_grad_kernel<<<grid, 256, 0, s>>>(acc, ld_acc, rows, cols, grad, ldg);
  FLARE_CUDA_CHECK(cudaGetLastError());
  count_launch();
}

}  // namespace flare
