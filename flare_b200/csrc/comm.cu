// Symmetric-memory plumbing for the fused collectives: raw device
// allocations whose CUDA IPC handles are exchanged over torch.distributed so
// every rank maps every peer's buffer (NVLink 5 / NVSwitch peer access), plus
// the status-word helpers shared by all kernels with bounded waits.
//
// The reference has no equivalent native layer: its dense collectives are XLA
// NCCL calls (src/flare/jax/training/zero/collectives.py:14-40) and its sparse
// exchange is Fluxway transport over Ray
// (src/flare/runtime/fluxway/workers/sparse_input.py:447-455).
#include "common.cuh"

#include <atomic>
#include <cstring>
#include <vector>

namespace flare {

static std::atomic<long long> g_launches{0};
void count_launch(int n) { g_launches.fetch_add(n, std::memory_order_relaxed); }
long long launch_count() { return g_launches.load(std::memory_order_relaxed); }

__global__ void increment_counter_kernel(int* p) { *p += 1; }
void increment_counter(int* p, cudaStream_t s) {
  increment_counter_kernel<<<1, 1, 0, s>>>(p);
  FLARE_CUDA_CHECK(cudaGetLastError());
  count_launch();
}

// One thread waits (bounded) for *flag >= target; used to exercise the
// timeout path of cross-GPU waits without involving another GPU.
__global__ void wait_flag_probe_kernel(const uint32_t* flag, uint32_t target, uint64_t timeout_ns, int* status) {
  if (threadIdx.x == 0 && blockIdx.x == 0) wait_flag_geq(flag, target, timeout_ns, status, 0);
}
void wait_flag_probe(const uint32_t* flag, uint32_t target, uint64_t timeout_ns, int* status, cudaStream_t s) {
  wait_flag_probe_kernel<<<1, 32, 0, s>>>(flag, target, timeout_ns, status);
  FLARE_CUDA_CHECK(cudaGetLastError());
  count_launch();
}

void* dev_malloc(size_t bytes) {
  void* p = nullptr;
  FLARE_CUDA_CHECK(cudaMalloc(&p, bytes));
  FLARE_CUDA_CHECK(cudaMemset(p, 0, bytes));
  return p;
}

void dev_free(void* p) {
  if (p) FLARE_CUDA_CHECK(cudaFree(p));
}

std::vector<char> ipc_get_handle(void* p) {
  cudaIpcMemHandle_t h;
  FLARE_CUDA_CHECK(cudaIpcGetMemHandle(&h, p));
  std::vector<char> out(sizeof(h));
  std::memcpy(out.data(), &h, sizeof(h));
  return out;
}

void* ipc_open_handle(const std::vector<char>& bytes) {
  FLARE_CHECK(bytes.size() == sizeof(cudaIpcMemHandle_t), "bad IPC handle size");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, bytes.data(), sizeof(h));
  void* p = nullptr;
  FLARE_CUDA_CHECK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  return p;
}

void ipc_close_handle(void* p) {
  if (p) FLARE_CUDA_CHECK(cudaIpcCloseMemHandle(p));
}

bool can_access_peer(int dev, int peer) {
  int ok = 0;
  FLARE_CUDA_CHECK(cudaDeviceCanAccessPeer(&ok, dev, peer));
  return ok != 0;
}

}  // namespace flare
