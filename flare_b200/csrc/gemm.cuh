// Host interface of the tcgen05 GEMM (gemm_tcgen05.cu).
#pragma once

#include "common.cuh"

namespace flare {

struct GemmArgs {
  const void* A;  // logical [M,K]; K-major A[m*lda+k], MN-major A[k*lda+m]
  int64_t lda;
  bool a_mn;
  const void* B;  // logical [N,K]; K-major B[n*ldb+k], MN-major B[k*ldb+n]
  int64_t ldb;
  bool b_mn;
  int M, N, K;
  void* C;  // [M, ldc] of c_dtype
  int64_t ldc;
  int c_dtype;  // kF32 or kBF16
  bool accumulate;
  const __nv_bfloat16* bias;  // bf16 [N] or null
  int act;            // 0 none, 1 relu
  float alpha;
  const void* mask;  // bf16 [M, ldm]: result *= (mask > 0); or null
  int64_t ldm;
  float* colsum;  // fp32 [N]: += column sums of the result; or null
  int* status;
  uint64_t timeout_ns;
  int pair = -1;  // CTA-pair (cta_group::2) tiles: 1 use, 0 never, -1 as FLARE_GEMM_PAIR says
};

void gemm_bf16_tcgen05(const GemmArgs& a, int bn_hint, cudaStream_t stream);
int device_sm_count();

// Row-major bf16 matrix as a 2-D TMA map with 128-byte swizzle, box 64 x box_outer.
CUtensorMap make_tmap_bf16(const void* base, int64_t inner, int64_t outer, int64_t ld, int box_outer);

// ---------------------------------------------------------------------------
// Persistent GEMM with fused all-gather / reduce-scatter (gemm_dist.cu).
// ---------------------------------------------------------------------------
// An operand whose stored rows are sharded over `nranks` ranks: rank q owns
// stored rows [q*rows_per_rank, (q+1)*rows_per_rank) of a full buffer that
// sits at the same offset of every rank's symmetric heap.
struct DistGather {
  int enabled = 0;
  int nranks = 1, my = 0;
  const void* src[8] = {};  // rank q's full buffer (peer address for q != my)
  void* dst = nullptr;      // this rank's full buffer (also the GEMM operand)
  int64_t ld = 0;           // row pitch in elements
  int64_t rows_per_rank = 0;
  int64_t row_elems = 0;    // elements copied per row (multiple of 8, <= ld)
  int chunk_rows = 128;     // rows per ready flag
  int pieces = 1;           // copy work items per chunk
  int piece_vecs = 0;       // 16-byte vectors per work item
  uint32_t* ready = nullptr;  // [nranks * rows_per_rank / chunk_rows]
  uint32_t* done = nullptr;   // [same], zero between launches
};

// Reduce-scatter of the output rows over `nranks` ranks (rank q owns output
// rows [q*rows_per_rank, ...)); partial tiles travel as bf16.
struct DistRS {
  int enabled = 0;
  int nranks = 1, my = 0;
  int rows_per_rank = 0;
  void* recv_peer[8] = {};        // rank q's receive buffer: [nranks][tiles][4][8] blocks of 32 x 32 bf16
  const void* recv_local = nullptr;
  int64_t ld_recv = 0;            // unused (kept for the binding's field list)
  uint32_t* flag_peer[8] = {};    // rank q's flags [nranks][tiles_per_rank][8]
  const uint32_t* flag_local = nullptr;
};

struct DistGemmArgs {
  GemmArgs g;                     // C rows are LOCAL rows when rs.enabled
  const int* tiles = nullptr;     // (m_tile << 16 | n_tile) in processing order
  int num_tiles = 0;
  const int* chunks = nullptr;    // (operand << 31 | chunk << 12 | piece) in copy order (remote chunks only)
  int num_chunks = 0;
  DistGather ga, gb;
  DistRS rs;
  int epi = 0;                    // 0 plain, 1 cross (z = acc + bias; out = aux0*z + aux1), 2 residual (+aux1)
  const void* aux0 = nullptr;
  int64_t ld0 = 0;
  const void* aux1 = nullptr;
  int64_t ld1 = 0;
  void* zout = nullptr;
  int64_t ldz = 0;
  int world = 1, rank = 0;        // entry barrier over the whole world
  uint32_t* bar_local = nullptr;
  uint32_t* bar_peer[8] = {};
  uint32_t* ctl = nullptr;        // [epoch, block counter, barrier passed]
};

void gemm_dist_tcgen05(const DistGemmArgs& a, cudaStream_t stream);

}  // namespace flare
