// Python bindings for the flare_b200 native kernels. Kernels take raw device
// pointers (Python passes tensor.data_ptr()) and run on PyTorch's current CUDA
// stream, so they compose with torch streams, events and CUDA graph capture.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <pybind11/stl.h>

#include "common.cuh"
#include "attention.cuh"
#include "dcn.cuh"
#include "dense.cuh"
#include "dynamic_emb.cuh"
#include "embedding.cuh"
#include "gemm.cuh"
#include "host_tier.cuh"
#include "mixing.cuh"
#include "seqrec.cuh"
#include "sparse_ops.cuh"

namespace flare {
struct AucWork {
  unsigned long long* keys_a;
  unsigned long long* keys_b;
  int* vals_a;
  int* vals_b;
  int* negs;
  int* neg_prefix;
  int* hist;
  int* hist_scan;
  int* block_sums;
  double* credit;
  unsigned long long* pos_cnt;
  unsigned long long* neg_cnt;
  double* out;
};
void auc_device(const float* scores, const float* labels, const int64_t* groups, int64_t n, double negative_factor,
                const AucWork& w, cudaStream_t s);
void radix_sort_pairs(unsigned long long* keys_a, int* vals_a, unsigned long long* keys_b, int* vals_b, int64_t n,
                      int bits, int* hist, int* hist_scan, int* block_sums, cudaStream_t s);
void wait_flag_probe(const uint32_t* flag, uint32_t target, uint64_t timeout_ns, int* status, cudaStream_t s);
void* dev_malloc(size_t bytes);
void dev_free(void* p);
std::vector<char> ipc_get_handle(void* p);
void* ipc_open_handle(const std::vector<char>& bytes);
void ipc_close_handle(void* p);
bool can_access_peer(int dev, int peer);
}  // namespace flare

namespace py = pybind11;
using flare::kBF16;

namespace {

cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream().stream(); }

template <typename T>
T* P(uintptr_t v) {
  return reinterpret_cast<T*>(v);
}

template <typename T>
T get(const py::dict& d, const char* k) {
  if (!d.contains(k)) throw std::runtime_error(std::string("missing parameter: ") + k);
  return d[k].cast<T>();
}

template <typename T>
T get_or(const py::dict& d, const char* k, T dflt) {
  return d.contains(k) ? d[k].cast<T>() : dflt;
}

flare::SparseOptParams parse_sparse_opt(const py::dict& d) {
  flare::SparseOptParams o{};
  o.kind = get<int>(d, "kind");
  o.lr = get<float>(d, "lr");
  o.beta1 = get_or<float>(d, "beta1", 0.9f);
  o.beta2 = get_or<float>(d, "beta2", 0.999f);
  o.eps = get_or<float>(d, "eps", 1e-8f);
  o.weight_decay = get_or<float>(d, "weight_decay", 0.f);
  o.bias_corr1 = get_or<float>(d, "bias_corr1", 1.f);
  o.bias_corr2 = get_or<float>(d, "bias_corr2", 1.f);
  o.lr_policy = get_or<int>(d, "lr_policy", 0);
  o.policy_a = get_or<float>(d, "policy_a", 0.f);
  o.policy_b = get_or<float>(d, "policy_b", 1.f);
  o.lut = P<const float>(get_or<uintptr_t>(d, "lut", 0));
  o.lut_len = get_or<int>(d, "lut_len", 0);
  o.state_row = P<float>(get_or<uintptr_t>(d, "state_row", 0));
  o.state_m = P<float>(get_or<uintptr_t>(d, "state_m", 0));
  o.state_v = P<float>(get_or<uintptr_t>(d, "state_v", 0));
  o.score = P<float>(get_or<uintptr_t>(d, "score", 0));
  o.step_ptr = P<const int>(get_or<uintptr_t>(d, "step_ptr", 0));
  o.grad_scale = get_or<float>(d, "grad_scale", 1.f);
  return o;
}

flare::AdamParams parse_adam(const py::dict& d) {
  flare::AdamParams o{};
  o.kind = get_or<int>(d, "kind", 0);
  o.lr = get<float>(d, "lr");
  o.beta1 = get_or<float>(d, "beta1", 0.9f);
  o.beta2 = get_or<float>(d, "beta2", 0.999f);
  o.eps = get_or<float>(d, "eps", 1e-8f);
  o.weight_decay = get_or<float>(d, "weight_decay", 0.f);
  o.decoupled = get_or<int>(d, "decoupled", 0);
  o.nesterov = get_or<int>(d, "nesterov", 0);
  o.bias_corr1 = get_or<float>(d, "bias_corr1", 1.f);
  o.bias_corr2 = get_or<float>(d, "bias_corr2", 1.f);
  o.step_ptr = P<const int>(get_or<uintptr_t>(d, "step_ptr", 0));
  return o;
}

}  // namespace

void register_etl(py::module_& m);
void register_sparse_cpu(py::module_& m);
void register_paged_store(py::module_& m);
void register_dyn_map(py::module_& m);

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  register_etl(m);
  register_sparse_cpu(m);
  register_paged_store(m);
  register_dyn_map(m);
  m.doc() = "flare_b200 native kernels (sm_100a)";

  m.def("device_sm_count", &flare::device_sm_count);
  m.def("launch_count", &flare::launch_count);
  m.def("increment_counter", [](uintptr_t p) { flare::increment_counter(P<int>(p), cur_stream()); });

  m.def(
      "gemm",
      [](uintptr_t A, int64_t lda, bool a_mn, uintptr_t B, int64_t ldb, bool b_mn, int M, int N, int K, uintptr_t C,
         int64_t ldc, int c_dtype, bool accumulate, uintptr_t bias, int act, float alpha, uintptr_t mask,
         int64_t ldm, uintptr_t colsum, uintptr_t status, uint64_t timeout_ns, int bn, int pair) {
        flare::GemmArgs a{};
        a.A = P<const void>(A);
        a.lda = lda;
        a.a_mn = a_mn;
        a.B = P<const void>(B);
        a.ldb = ldb;
        a.b_mn = b_mn;
        a.M = M;
        a.N = N;
        a.K = K;
        a.C = P<void>(C);
        a.ldc = ldc;
        a.c_dtype = c_dtype;
        a.accumulate = accumulate;
        a.bias = P<const __nv_bfloat16>(bias);
        a.act = act;
        a.alpha = alpha;
        a.mask = P<const void>(mask);
        a.ldm = ldm;
        a.colsum = P<float>(colsum);
        a.status = P<int>(status);
        a.timeout_ns = timeout_ns;
        a.pair = pair;
        flare::gemm_bf16_tcgen05(a, bn, cur_stream());
      },
      py::arg("A"), py::arg("lda"), py::arg("a_mn"), py::arg("B"), py::arg("ldb"), py::arg("b_mn"), py::arg("M"),
      py::arg("N"), py::arg("K"), py::arg("C"), py::arg("ldc"), py::arg("c_dtype"), py::arg("accumulate"),
      py::arg("bias"), py::arg("act"), py::arg("alpha"), py::arg("mask"), py::arg("ldm"), py::arg("colsum"),
      py::arg("status"), py::arg("timeout_ns"), py::arg("bn") = 0, py::arg("pair") = -1);

  m.def("gemm_dist", [](const py::dict& d) {
    flare::DistGemmArgs a;
    const py::dict g = get<py::dict>(d, "g");
    a.g.A = P<const void>(get<uintptr_t>(g, "A"));
    a.g.lda = get<int64_t>(g, "lda");
    a.g.a_mn = get<bool>(g, "a_mn");
    a.g.B = P<const void>(get<uintptr_t>(g, "B"));
    a.g.ldb = get<int64_t>(g, "ldb");
    a.g.b_mn = get<bool>(g, "b_mn");
    a.g.M = get<int>(g, "M");
    a.g.N = get<int>(g, "N");
    a.g.K = get<int>(g, "K");
    a.g.C = P<void>(get<uintptr_t>(g, "C"));
    a.g.ldc = get<int64_t>(g, "ldc");
    a.g.c_dtype = get<int>(g, "c_dtype");
    a.g.accumulate = get_or<bool>(g, "accumulate", false);
    a.g.bias = P<const __nv_bfloat16>(get_or<uintptr_t>(g, "bias", 0));
    a.g.act = get_or<int>(g, "act", 0);
    a.g.alpha = get_or<float>(g, "alpha", 1.f);
    a.g.mask = P<const void>(get_or<uintptr_t>(g, "mask", 0));
    a.g.ldm = get_or<int64_t>(g, "ldm", 0);
    a.g.colsum = P<float>(get_or<uintptr_t>(g, "colsum", 0));
    a.g.status = P<int>(get<uintptr_t>(g, "status"));
    a.g.timeout_ns = get<uint64_t>(g, "timeout_ns");
    a.tiles = P<const int>(get<uintptr_t>(d, "tiles"));
    a.num_tiles = get<int>(d, "num_tiles");
    a.chunks = P<const int>(get_or<uintptr_t>(d, "chunks", 0));
    a.num_chunks = get_or<int>(d, "num_chunks", 0);
    for (int op = 0; op < 2; ++op) {
      const char* key = op ? "gb" : "ga";
      if (!d.contains(key) || d[key].is_none()) continue;
      const py::dict gd = d[key].cast<py::dict>();
      flare::DistGather& x = op ? a.gb : a.ga;
      x.enabled = 1;
      x.nranks = get<int>(gd, "nranks");
      x.my = get<int>(gd, "my");
      const auto src = get<std::vector<uintptr_t>>(gd, "src");
      if (static_cast<int>(src.size()) != x.nranks || x.nranks > 8) throw std::runtime_error("gather: bad src list");
      for (int q = 0; q < x.nranks; ++q) x.src[q] = P<const void>(src[q]);
      x.dst = P<void>(get<uintptr_t>(gd, "dst"));
      x.ld = get<int64_t>(gd, "ld");
      x.rows_per_rank = get<int64_t>(gd, "rows_per_rank");
      x.row_elems = get<int64_t>(gd, "row_elems");
      x.chunk_rows = get<int>(gd, "chunk_rows");
      x.pieces = get<int>(gd, "pieces");
      x.piece_vecs = get<int>(gd, "piece_vecs");
      x.ready = P<uint32_t>(get<uintptr_t>(gd, "ready"));
      x.done = P<uint32_t>(get<uintptr_t>(gd, "done"));
    }
    if (d.contains("rs") && !d["rs"].is_none()) {
      const py::dict rd = d["rs"].cast<py::dict>();
      a.rs.enabled = 1;
      a.rs.nranks = get<int>(rd, "nranks");
      a.rs.my = get<int>(rd, "my");
      a.rs.rows_per_rank = get<int>(rd, "rows_per_rank");
      const auto recv = get<std::vector<uintptr_t>>(rd, "recv_peer");
      const auto flags = get<std::vector<uintptr_t>>(rd, "flag_peer");
      if (static_cast<int>(recv.size()) != a.rs.nranks || static_cast<int>(flags.size()) != a.rs.nranks ||
          a.rs.nranks > 8)
        throw std::runtime_error("reduce-scatter: bad peer lists");
      for (int q = 0; q < a.rs.nranks; ++q) {
        a.rs.recv_peer[q] = P<void>(recv[q]);
        a.rs.flag_peer[q] = P<uint32_t>(flags[q]);
      }
      a.rs.recv_local = P<const void>(get<uintptr_t>(rd, "recv_local"));
      a.rs.ld_recv = get_or<int64_t>(rd, "ld_recv", 0);
      a.rs.flag_local = P<const uint32_t>(get<uintptr_t>(rd, "flag_local"));
    }
    a.epi = get_or<int>(d, "epi", 0);
    a.aux0 = P<const void>(get_or<uintptr_t>(d, "aux0", 0));
    a.ld0 = get_or<int64_t>(d, "ld0", 0);
    a.aux1 = P<const void>(get_or<uintptr_t>(d, "aux1", 0));
    a.ld1 = get_or<int64_t>(d, "ld1", 0);
    a.zout = P<void>(get_or<uintptr_t>(d, "zout", 0));
    a.ldz = get_or<int64_t>(d, "ldz", 0);
    a.world = get_or<int>(d, "world", 1);
    a.rank = get_or<int>(d, "rank", 0);
    a.bar_local = P<uint32_t>(get_or<uintptr_t>(d, "bar_local", 0));
    if (d.contains("bar_peer")) {
      const auto bp = get<std::vector<uintptr_t>>(d, "bar_peer");
      if (static_cast<int>(bp.size()) > 8) throw std::runtime_error("barrier: too many ranks");
      for (size_t s = 0; s < bp.size(); ++s) a.bar_peer[s] = P<uint32_t>(bp[s]);
    }
    a.ctl = P<uint32_t>(get<uintptr_t>(d, "ctl"));
    flare::gemm_dist_tcgen05(a, cur_stream());
  });

  m.def("emb_forward", [](const py::dict& d) {
    flare::EmbFwdParams p{};
    p.shards = P<const flare::ShardDesc>(get<uintptr_t>(d, "shards"));
    p.num_shards = get<int>(d, "num_shards");
    p.world = get<int>(d, "world");
    p.rank = get<int>(d, "rank");
    p.Bl = get<int>(d, "Bl");
    p.F = get<int>(d, "F");
    p.peer_offsets = P<const int* const>(get<uintptr_t>(d, "peer_offsets"));
    p.peer_values = P<const int* const>(get<uintptr_t>(d, "peer_values"));
    p.peer_out = P<void* const>(get<uintptr_t>(d, "peer_out"));
    p.out_stride = get<int64_t>(d, "out_stride");
    p.weights = P<const void>(get<uintptr_t>(d, "weights"));
    p.w_dtype = get<int>(d, "w_dtype");
    p.out_dtype = get_or<int>(d, "out_dtype", kBF16);
    p.vec = get_or<int>(d, "vec", 1);
    p.bulk = get_or<int>(d, "bulk", 0);
    p.slot_map = P<const int>(get_or<uintptr_t>(d, "slot_map", 0));
    p.peer_remap = P<const int* const>(get_or<uintptr_t>(d, "peer_remap", 0));
    p.fetch_offs = P<int>(get_or<uintptr_t>(d, "fetch_offs", 0));
    p.peer_part = P<float* const>(get_or<uintptr_t>(d, "peer_part", 0));
    p.part_stride = get_or<int64_t>(d, "part_stride", 0);
    p.rw_tables = P<const flare::RwTable>(get_or<uintptr_t>(d, "rw_tables", 0));
    p.num_rw = get_or<int>(d, "num_rw", 0);
    p.stage_ids = P<int>(get<uintptr_t>(d, "stage_ids"));
    p.stage_bag = P<int>(get<uintptr_t>(d, "stage_bag"));
    p.stage_count = P<int>(get<uintptr_t>(d, "stage_count"));
    p.stage_len = P<int>(get<uintptr_t>(d, "stage_len"));
    p.stage_cap = get<int64_t>(d, "stage_cap");
    p.flags_local = P<uint32_t>(get_or<uintptr_t>(d, "flags_local", 0));
    p.peer_flags = P<uint32_t* const>(get_or<uintptr_t>(d, "peer_flags", 0));
    p.flag_in = get_or<int>(d, "flag_in", 0);
    p.flag_out = get_or<int>(d, "flag_out", 0);
    p.epoch_ctr = P<uint32_t>(get_or<uintptr_t>(d, "epoch_ctr", 0));
    p.block_counter = P<unsigned>(get_or<uintptr_t>(d, "block_counter", 0));
    p.status = P<int>(get_or<uintptr_t>(d, "status", 0));
    p.timeout_ns = get_or<uint64_t>(d, "timeout_ns", 2000000000ull);
    p.fwd_minb = get_or<int>(d, "fwd_minb", 4);
    flare::emb_forward(p, get<int>(d, "grid"), cur_stream());
  });

  m.def("emb_window_append", [](const py::dict& d) {
    flare::EmbWindowParams p{};
    p.ids = P<const int>(get<uintptr_t>(d, "ids"));
    p.bag = P<const int>(get<uintptr_t>(d, "bag"));
    p.count = P<const int>(get<uintptr_t>(d, "count"));
    p.len = P<const int>(get<uintptr_t>(d, "len"));
    p.wids = P<int>(get<uintptr_t>(d, "wids"));
    p.wbag = P<int>(get<uintptr_t>(d, "wbag"));
    p.wprefix = P<int>(get<uintptr_t>(d, "wprefix"));
    p.wlen = P<int>(get<uintptr_t>(d, "wlen"));
    p.nslot = get<int>(d, "nslot");
    p.Bl = get<int>(d, "Bl");
    p.micro = get<int>(d, "micro");
    p.micro_steps = get<int>(d, "micro_steps");
    p.stage_cap = get<int64_t>(d, "stage_cap");
    flare::emb_window_append(p, cur_stream());
  });
  m.def("emb_det_temp_bytes", [](int64_t max_occ) { return flare::emb_det_temp_bytes(max_occ); });
  m.def("emb_hash_sizes", [](int64_t max_occ, int light_max) {
    return py::make_tuple(flare::emb_hash_tile_count(max_occ), flare::emb_hash_max_chunks(max_occ, light_max),
                          flare::emb_hash_max_parts(max_occ), flare::emb_hash_scan_vals());
  });
  m.def("emb_backward", [](const py::dict& d) {
    flare::EmbBwdParams p{};
    p.shards = P<const flare::ShardDesc>(get<uintptr_t>(d, "shards"));
    p.num_shards = get<int>(d, "num_shards");
    p.world = get<int>(d, "world");
    p.rank = get<int>(d, "rank");
    p.Bl = get<int>(d, "Bl");
    p.peer_grad = P<const void* const>(get<uintptr_t>(d, "peer_grad"));
    p.out_stride = get<int64_t>(d, "out_stride");
    p.grad_dtype = get_or<int>(d, "grad_dtype", kBF16);
    p.grad_stage = P<void>(get<uintptr_t>(d, "grad_stage"));
    p.grad_stage_ld = get<int64_t>(d, "grad_stage_ld");
    p.stage_ids = P<const int>(get<uintptr_t>(d, "stage_ids"));
    p.stage_bag = P<const int>(get<uintptr_t>(d, "stage_bag"));
    p.stage_rank = P<int>(get<uintptr_t>(d, "stage_rank"));
    p.slot_start = P<int>(get<uintptr_t>(d, "slot_start"));
    p.stage_count = P<const int>(get<uintptr_t>(d, "stage_count"));
    p.stage_len = P<const int>(get<uintptr_t>(d, "stage_len"));
    p.stage_cap = get<int64_t>(d, "stage_cap");
    p.weights = P<void>(get<uintptr_t>(d, "weights"));
    p.w_dtype = get<int>(d, "w_dtype");
    p.row_count = P<int>(get_or<uintptr_t>(d, "row_count", 0));
    p.row2u = P<int>(get_or<uintptr_t>(d, "row2u", 0));
    p.flags = P<int>(get<uintptr_t>(d, "flags"));
    p.pos = P<int>(get_or<uintptr_t>(d, "pos", 0));
    p.uniq_row = P<int64_t>(get_or<uintptr_t>(d, "uniq_row", 0));
    p.uniq_shard = P<int>(get_or<uintptr_t>(d, "uniq_shard", 0));
    p.cnt_u = P<int>(get_or<uintptr_t>(d, "cnt_u", 0));
    p.first_gidx = P<int>(get_or<uintptr_t>(d, "first_gidx", 0));
    p.num_unique = P<int>(get<uintptr_t>(d, "num_unique"));
    p.seg_start = P<int>(get<uintptr_t>(d, "seg_start"));
    p.block_sums = P<int>(get_or<uintptr_t>(d, "block_sums", 0));
    p.occ = P<int>(get<uintptr_t>(d, "occ"));
    p.heavy = P<int>(get_or<uintptr_t>(d, "heavy", 0));
    p.heavy_start = P<int>(get_or<uintptr_t>(d, "heavy_start", 0));
    p.hcnt = P<int>(get_or<uintptr_t>(d, "hcnt", 0));
    p.heavy_acc = P<float>(get_or<uintptr_t>(d, "heavy_acc", 0));
    p.max_heavy = get_or<int>(d, "max_heavy", 0);
    p.light_max = get_or<int>(d, "light_max", 64);
    p.dirty = P<unsigned>(get_or<uintptr_t>(d, "dirty", 0));
    p.max_occ = get<int64_t>(d, "max_occ");
    p.deterministic = get_or<int>(d, "deterministic", 0);
    p.det_first = P<int>(get_or<uintptr_t>(d, "det_first", 0));
    p.det_keys = P<int>(get_or<uintptr_t>(d, "det_keys", 0));
    p.det_vals = P<int>(get_or<uintptr_t>(d, "det_vals", 0));
    p.det_temp = P<void>(get_or<uintptr_t>(d, "det_temp", 0));
    p.det_temp_bytes = get_or<size_t>(d, "det_temp_bytes", 0);
    p.hash_mode = get_or<int>(d, "hash_mode", 0);
    if (p.hash_mode) {
      p.htab = P<unsigned long long>(get<uintptr_t>(d, "htab"));
      p.hseg = P<int>(get<uintptr_t>(d, "hseg"));
      p.ovf_list = P<int>(get<uintptr_t>(d, "ovf_list"));
      p.hcap = get<int64_t>(d, "hcap");
      p.hregion = get_or<int64_t>(d, "hregion", 0);
      p.hprefetch = get_or<int>(d, "hprefetch", 1);
      p.grad_direct = get_or<int>(d, "grad_direct", 0);
      p.occ_h = P<int>(get<uintptr_t>(d, "occ_h"));
      p.occ_rank = P<int>(get<uintptr_t>(d, "occ_rank"));
      p.occ_bag = P<int>(get<uintptr_t>(d, "occ_bag"));
      p.lrec = P<int4>(get<uintptr_t>(d, "lrec"));
      p.crec = P<int4>(get<uintptr_t>(d, "crec"));
      p.max_chunks = get<int64_t>(d, "max_chunks");
      p.hpart = P<float>(get<uintptr_t>(d, "hpart"));
      p.max_parts = get<int64_t>(d, "max_parts");
      p.occ_scale = P<float>(get_or<uintptr_t>(d, "occ_scale", 0));
      p.scan_val = P<int>(get<uintptr_t>(d, "scan_val"));
      p.max_tiles = get<int64_t>(d, "max_tiles");
    }
    p.opt = parse_sparse_opt(get<py::dict>(d, "opt"));
    p.flags_local = P<uint32_t>(get_or<uintptr_t>(d, "flags_local", 0));
    p.peer_flags = P<uint32_t* const>(get_or<uintptr_t>(d, "peer_flags", 0));
    p.flag_in = get_or<int>(d, "flag_in", 0);
    p.epoch_ctr = P<uint32_t>(get_or<uintptr_t>(d, "epoch_ctr", 0));
    p.block_counter = P<unsigned>(get_or<uintptr_t>(d, "block_counter", 0));
    p.status = P<int>(get_or<uintptr_t>(d, "status", 0));
    p.timeout_ns = get_or<uint64_t>(d, "timeout_ns", 2000000000ull);
    p.light_prefetch = get_or<int>(d, "light_prefetch", 0);
    p.chunk_variant = get_or<int>(d, "chunk_variant", 1);
    flare::emb_backward(p, get<int>(d, "ncols_max"), get<int>(d, "grid"), cur_stream());
  });

  auto parse_inter = [](const py::dict& d) {
    flare::InteractionParams p{};
    p.B = get<int>(d, "B");
    p.F = get<int>(d, "F");
    p.D = get<int>(d, "D");
    p.bot = P<const __nv_bfloat16>(get<uintptr_t>(d, "bot"));
    p.bot_ld = get<int64_t>(d, "bot_ld");
    p.emb = P<const __nv_bfloat16>(get<uintptr_t>(d, "emb"));
    p.emb_ld = get<int64_t>(d, "emb_ld");
    p.out = P<__nv_bfloat16>(get_or<uintptr_t>(d, "out", 0));
    p.dout = P<const __nv_bfloat16>(get_or<uintptr_t>(d, "dout", 0));
    p.out_ld = get<int64_t>(d, "out_ld");
    p.dbot = P<__nv_bfloat16>(get_or<uintptr_t>(d, "dbot", 0));
    p.dbot_ld = get_or<int64_t>(d, "dbot_ld", 0);
    p.demb = P<__nv_bfloat16>(get_or<uintptr_t>(d, "demb", 0));
    p.demb_ld = get_or<int64_t>(d, "demb_ld", 0);
    p.relu_mask_bot = get_or<int>(d, "relu_mask_bot", 1);
    p.status = P<int>(get_or<uintptr_t>(d, "status", 0));
    return p;
  };
  m.def("interaction_forward", [parse_inter](const py::dict& d) { flare::interaction_forward(parse_inter(d), cur_stream()); });
  m.def("interaction_backward", [parse_inter](const py::dict& d) { flare::interaction_backward(parse_inter(d), cur_stream()); });

  m.def("head_bce", [](const py::dict& d) {
    flare::HeadBceParams p{};
    p.B = get<int>(d, "B");
    p.H = get<int>(d, "H");
    p.T = get<int>(d, "T");
    p.h = P<const __nv_bfloat16>(get<uintptr_t>(d, "h"));
    p.h_ld = get<int64_t>(d, "h_ld");
    p.w = P<const __nv_bfloat16>(get<uintptr_t>(d, "w"));
    p.bias = P<const __nv_bfloat16>(get<uintptr_t>(d, "bias"));
    p.labels = P<const float>(get<uintptr_t>(d, "labels"));
    p.label_ld = get<int64_t>(d, "label_ld");
    p.target_weights = P<const float>(get_or<uintptr_t>(d, "target_weights", 0));
    p.sample_weights = P<const float>(get_or<uintptr_t>(d, "sample_weights", 0));
    p.valid_count = get_or<int>(d, "valid_count", -1);
    p.grad_scale = get<float>(d, "grad_scale");
    p.logits = P<float>(get<uintptr_t>(d, "logits"));
    p.loss_sum = P<float>(get<uintptr_t>(d, "loss_sum"));
    p.dh = P<__nv_bfloat16>(get<uintptr_t>(d, "dh"));
    p.dh_ld = get<int64_t>(d, "dh_ld");
    p.dw = P<float>(get<uintptr_t>(d, "dw"));
    p.db = P<float>(get<uintptr_t>(d, "db"));
    flare::head_bce(p, cur_stream());
  });

  m.def("adam_flat", [](const py::dict& d) {
    flare::AdamFlatParams p{};
    p.master = P<float>(get<uintptr_t>(d, "master"));
    p.grad = P<float>(get<uintptr_t>(d, "grad"));
    p.m = P<float>(get<uintptr_t>(d, "m"));
    p.v = P<float>(get<uintptr_t>(d, "v"));
    p.compute_copy = P<__nv_bfloat16>(get_or<uintptr_t>(d, "compute_copy", 0));
    p.n = get<int64_t>(d, "n");
    p.grad_scale = get_or<float>(d, "grad_scale", 1.f);
    p.zero_grad = get_or<int>(d, "zero_grad", 1);
    p.opt = parse_adam(get<py::dict>(d, "opt"));
    flare::adam_flat(p, cur_stream());
  });

  m.def("adam_dp_fused", [](const py::dict& d) {
    flare::AdamDpParams p{};
    p.world = get<int>(d, "world");
    p.rank = get<int>(d, "rank");
    p.lo = get<int64_t>(d, "lo");
    p.hi = get<int64_t>(d, "hi");
    p.peer_grad = P<float* const>(get<uintptr_t>(d, "peer_grad"));
    p.peer_param = P<void* const>(get<uintptr_t>(d, "peer_param"));
    p.param_world = get_or<int>(d, "param_world", p.world);
    p.master_shard = P<float>(get<uintptr_t>(d, "master_shard"));
    p.m_shard = P<float>(get<uintptr_t>(d, "m_shard"));
    p.v_shard = P<float>(get<uintptr_t>(d, "v_shard"));
    p.grad_scale = get_or<float>(d, "grad_scale", 1.f);
    p.opt = parse_adam(get<py::dict>(d, "opt"));
    p.flags_local = P<uint32_t>(get<uintptr_t>(d, "flags_local"));
    p.peer_flags = P<uint32_t* const>(get<uintptr_t>(d, "peer_flags"));
    p.flag_in = get<int>(d, "flag_in");
    p.flag_out = get<int>(d, "flag_out");
    p.epoch_ctr = P<uint32_t>(get<uintptr_t>(d, "epoch_ctr"));
    p.block_counter = P<unsigned>(get<uintptr_t>(d, "block_counter"));
    p.status = P<int>(get_or<uintptr_t>(d, "status", 0));
    p.timeout_ns = get_or<uint64_t>(d, "timeout_ns", 2000000000ull);
    flare::adam_dp_fused(p, cur_stream());
  });

  m.def("attn_forward", [](const py::dict& d) {
    flare::AttnFwdParams p{};
    p.qkv = P<const void>(get<uintptr_t>(d, "qkv"));
    p.ld_qkv = get<int64_t>(d, "ld_qkv");
    p.vt = P<const void>(get<uintptr_t>(d, "vt"));
    p.ld_vt = get<int64_t>(d, "ld_vt");
    p.offsets = P<const int>(get<uintptr_t>(d, "offsets"));
    p.nseq = get<int>(d, "nseq");
    p.max_len = get<int>(d, "max_len");
    p.T_cap = get<int64_t>(d, "T_cap");
    p.scale = get<float>(d, "scale");
    p.out = P<__nv_bfloat16>(get<uintptr_t>(d, "out"));
    p.ld_out = get<int64_t>(d, "ld_out");
    p.lse = P<float>(get<uintptr_t>(d, "lse"));
    p.ld_lse = get<int64_t>(d, "ld_lse");
    p.status = P<int>(get<uintptr_t>(d, "status"));
    p.timeout_ns = get<uint64_t>(d, "timeout_ns");
    flare::attn_forward(p, cur_stream());
  });
  m.def("attn_backward", [](const py::dict& d) {
    flare::AttnBwdParams p{};
    p.qkv = P<const void>(get<uintptr_t>(d, "qkv"));
    p.ld_qkv = get<int64_t>(d, "ld_qkv");
    p.dout = P<const void>(get<uintptr_t>(d, "dout"));
    p.out = P<const void>(get<uintptr_t>(d, "out"));
    p.ld_do = get<int64_t>(d, "ld_do");
    p.dout_t = P<const void>(get<uintptr_t>(d, "dout_t"));
    p.q_t = P<const void>(get<uintptr_t>(d, "q_t"));
    p.ld_t = get<int64_t>(d, "ld_t");
    p.offsets = P<const int>(get<uintptr_t>(d, "offsets"));
    p.nseq = get<int>(d, "nseq");
    p.max_len = get<int>(d, "max_len");
    p.T_cap = get<int64_t>(d, "T_cap");
    p.scale = get<float>(d, "scale");
    p.lse = P<const float>(get<uintptr_t>(d, "lse"));
    p.delta = P<float>(get<uintptr_t>(d, "delta"));
    p.ld_stat = get<int64_t>(d, "ld_stat");
    p.dq_acc = P<float>(get<uintptr_t>(d, "dq_acc"));
    p.ld_dq = get<int64_t>(d, "ld_dq");
    p.dqkv = P<__nv_bfloat16>(get<uintptr_t>(d, "dqkv"));
    p.ld_dqkv = get<int64_t>(d, "ld_dqkv");
    p.status = P<int>(get<uintptr_t>(d, "status"));
    p.timeout_ns = get<uint64_t>(d, "timeout_ns");
    flare::attn_backward(p, cur_stream());
  });

  m.def("seq_embed_combine", [](uintptr_t pooled, int64_t ldp, int64_t T, uintptr_t x, int64_t ldx) {
    flare::seq_embed_combine(P<const __nv_bfloat16>(pooled), ldp, T, P<__nv_bfloat16>(x), ldx, cur_stream());
  });
  m.def("seq_layernorm_fwd", [](uintptr_t x, int64_t ldx, int64_t T, uintptr_t gamma, uintptr_t beta, float eps,
                                uintptr_t y, int64_t ldy, uintptr_t mean, uintptr_t rstd) {
    flare::seq_layernorm_fwd(P<const __nv_bfloat16>(x), ldx, T, P<const __nv_bfloat16>(gamma),
                             P<const __nv_bfloat16>(beta), eps,
                             P<__nv_bfloat16>(y), ldy, P<float>(mean), P<float>(rstd), cur_stream());
  });
  m.def("seq_layernorm_bwd", [](uintptr_t dy, int64_t lddy, uintptr_t x, int64_t ldx, int64_t T, uintptr_t gamma,
                                uintptr_t mean, uintptr_t rstd, uintptr_t resid, int64_t ldr, uintptr_t dx,
                                int64_t lddx, uintptr_t dgamma, uintptr_t dbeta) {
    flare::seq_layernorm_bwd(P<const __nv_bfloat16>(dy), lddy, P<const __nv_bfloat16>(x), ldx, T,
                             P<const __nv_bfloat16>(gamma), P<const float>(mean), P<const float>(rstd),
                             P<const __nv_bfloat16>(resid), ldr, P<__nv_bfloat16>(dx), lddx, P<float>(dgamma),
                             P<float>(dbeta), cur_stream());
  });
  m.def("seq_sampled_softmax", [](const py::dict& d) {
    flare::SampledSoftmaxParams p{};
    p.y = P<const __nv_bfloat16>(get<uintptr_t>(d, "y"));
    p.ldy = get<int64_t>(d, "ldy");
    p.emb = P<const __nv_bfloat16>(get<uintptr_t>(d, "emb"));
    p.ldemb = get<int64_t>(d, "ldemb");
    p.target_row = P<const int>(get<uintptr_t>(d, "target_row"));
    p.logits = P<const float>(get<uintptr_t>(d, "logits"));
    p.ldlog = get<int64_t>(d, "ldlog");
    p.T = get<int64_t>(d, "T");
    p.N = get<int>(d, "N");
    p.num_valid = P<const int>(get<uintptr_t>(d, "num_valid"));
    p.dneg = P<__nv_bfloat16>(get<uintptr_t>(d, "dneg"));
    p.lddneg = get<int64_t>(d, "lddneg");
    p.dy = P<__nv_bfloat16>(get<uintptr_t>(d, "dy"));
    p.lddy = get<int64_t>(d, "lddy");
    p.dpos = P<float>(get<uintptr_t>(d, "dpos"));
    p.loss_sum = P<float>(get<uintptr_t>(d, "loss_sum"));
    flare::seq_sampled_softmax(p, cur_stream());
  });
  m.def("seq_embed_grad_split", [](uintptr_t dx, int64_t lddx, uintptr_t y, int64_t ldy, uintptr_t dpos,
                                   uintptr_t target_row, int64_t T, uintptr_t grad, int64_t ldg) {
    flare::seq_embed_grad_split(P<const __nv_bfloat16>(dx), lddx, P<const __nv_bfloat16>(y), ldy,
                                P<const float>(dpos), P<const int>(target_row), T, P<__nv_bfloat16>(grad), ldg,
                                cur_stream());
  });

  m.def("dyn_prepare", [](const py::dict& d) {
    flare::DynParams p{};
    const auto tabs = get<py::list>(d, "tables");
    p.num_tables = static_cast<int>(tabs.size());
    if (p.num_tables > flare::kMaxDynTables) throw std::runtime_error("too many dynamic tables");
    for (int k = 0; k < p.num_tables; ++k) {
      const py::dict t = tabs[k].cast<py::dict>();
      flare::DynTable& x = p.tables[k];
      x.feature = get<int>(t, "feature");
      x.ncols = get<int>(t, "ncols");
      x.col_begin = get<int>(t, "col_begin");
      x.C = get<int>(t, "C");
      x.H = get<int>(t, "H");
      x.init_scale = get<float>(t, "init_scale");
      x.seed = get<uint64_t>(t, "seed");
      x.keys = P<int>(get<uintptr_t>(t, "keys"));
      x.slot_of = P<int>(get<uintptr_t>(t, "slot_of"));
      x.bucket_of = P<int>(get<uintptr_t>(t, "bucket_of"));
      x.stamp = P<int>(get<uintptr_t>(t, "stamp"));
      x.hand = P<unsigned>(get<uintptr_t>(t, "hand"));
      x.weights = P<float>(get<uintptr_t>(t, "weights"));
      x.state_row = P<float>(get_or<uintptr_t>(t, "state_row", 0));
      x.state_m = P<float>(get_or<uintptr_t>(t, "state_m", 0));
      x.state_v = P<float>(get_or<uintptr_t>(t, "state_v", 0));
      x.score = P<float>(get_or<uintptr_t>(t, "score", 0));
      x.new_buckets = P<int>(get<uintptr_t>(t, "new_buckets"));
      x.num_new = P<int>(get<uintptr_t>(t, "num_new"));
      x.new_cap = get<int>(t, "new_cap");
      x.num_tomb = P<int>(get<uintptr_t>(t, "num_tomb"));
    }
    p.world = get<int>(d, "world");
    p.rank = get<int>(d, "rank");
    p.Bl = get<int>(d, "Bl");
    p.peer_offsets = P<const int* const>(get<uintptr_t>(d, "peer_offsets"));
    p.peer_values = P<const int* const>(get<uintptr_t>(d, "peer_values"));
    p.peer_remap = P<int* const>(get<uintptr_t>(d, "peer_remap"));
    p.step_ptr = P<const int>(get<uintptr_t>(d, "step_ptr"));
    p.flags_local = P<uint32_t>(get_or<uintptr_t>(d, "flags_local", 0));
    p.peer_flags = P<uint32_t* const>(get_or<uintptr_t>(d, "peer_flags", 0));
    p.flag_in = get_or<int>(d, "flag_in", 0);
    p.epoch_ctr = P<uint32_t>(get_or<uintptr_t>(d, "epoch_ctr", 0));
    p.block_counter = P<unsigned>(get<uintptr_t>(d, "block_counter"));
    p.block_counter2 = P<unsigned>(get<uintptr_t>(d, "block_counter2"));
    p.status = P<int>(get_or<uintptr_t>(d, "status", 0));
    p.timeout_ns = get_or<uint64_t>(d, "timeout_ns", 2000000000ull);
    flare::dyn_prepare(p, get<int>(d, "grid"), cur_stream());
  });
  m.def("dyn_rebuild", [](uintptr_t keys, uintptr_t slot_of, uintptr_t bucket_of, int H, uintptr_t live_keys,
                          uintptr_t live_slots, int n) {
    flare::dyn_rebuild(P<int>(keys), P<int>(slot_of), P<int>(bucket_of), H, P<const int>(live_keys),
                       P<const int>(live_slots), n, cur_stream());
  });

  m.def("tier_prepare", [](const py::dict& d) {
    flare::TierParams p{};
    const auto tabs = get<py::list>(d, "tables");
    p.num_tables = static_cast<int>(tabs.size());
    if (p.num_tables > flare::kMaxTierTables) throw std::runtime_error("too many host-tier tables");
    for (int k = 0; k < p.num_tables; ++k) {
      const py::dict t = tabs[k].cast<py::dict>();
      flare::TierTable& x = p.tables[k];
      x.feature = get<int>(t, "feature");
      x.ncols = get<int>(t, "ncols");
      x.rows = get<int64_t>(t, "rows");
      x.C = get<int>(t, "C");
      x.slot_map = P<int>(get<uintptr_t>(t, "slot_map"));
      x.slot2row = P<int64_t>(get<uintptr_t>(t, "slot2row"));
      x.stamp = P<int>(get<uintptr_t>(t, "stamp"));
      x.hand = P<unsigned>(get<uintptr_t>(t, "hand"));
      x.cache_w = P<float>(get<uintptr_t>(t, "cache_w"));
      x.cache_row = P<float>(get_or<uintptr_t>(t, "cache_row", 0));
      x.cache_m = P<float>(get_or<uintptr_t>(t, "cache_m", 0));
      x.cache_v = P<float>(get_or<uintptr_t>(t, "cache_v", 0));
      x.host_w = P<float>(get<uintptr_t>(t, "host_w"));
      x.host_row = P<float>(get_or<uintptr_t>(t, "host_row", 0));
      x.host_m = P<float>(get_or<uintptr_t>(t, "host_m", 0));
      x.host_v = P<float>(get_or<uintptr_t>(t, "host_v", 0));
      x.miss_rows = P<int>(get<uintptr_t>(t, "miss_rows"));
      x.num_miss = P<int>(get<uintptr_t>(t, "num_miss"));
      x.miss_cap = get<int>(t, "miss_cap");
    }
    p.world = get<int>(d, "world");
    p.rank = get<int>(d, "rank");
    p.Bl = get<int>(d, "Bl");
    p.peer_offsets = P<const int* const>(get<uintptr_t>(d, "peer_offsets"));
    p.peer_values = P<const int* const>(get<uintptr_t>(d, "peer_values"));
    p.step_ptr = P<const int>(get<uintptr_t>(d, "step_ptr"));
    p.flags_local = P<uint32_t>(get_or<uintptr_t>(d, "flags_local", 0));
    p.peer_flags = P<uint32_t* const>(get_or<uintptr_t>(d, "peer_flags", 0));
    p.flag_in = get_or<int>(d, "flag_in", 0);
    p.epoch_ctr = P<uint32_t>(get_or<uintptr_t>(d, "epoch_ctr", 0));
    p.block_counter = P<unsigned>(get<uintptr_t>(d, "block_counter"));
    p.block_counter2 = P<unsigned>(get<uintptr_t>(d, "block_counter2"));
    p.status = P<int>(get_or<uintptr_t>(d, "status", 0));
    p.timeout_ns = get_or<uint64_t>(d, "timeout_ns", 2000000000ull);
    flare::tier_prepare(p, get<int>(d, "grid"), cur_stream());
  });

  m.def("dcn_concat_x0", [](uintptr_t pooled, int64_t ldp, uintptr_t dense, int nd, int64_t B, int E, uintptr_t x0,
                            int64_t ld0) {
    flare::dcn_concat_x0(P<const __nv_bfloat16>(pooled), ldp, P<const float>(dense), nd, B, E, P<__nv_bfloat16>(x0),
                         ld0, cur_stream());
  });
  m.def("dcn_head", [](const py::dict& d) {
    flare::DcnHeadParams p{};
    p.h = P<const __nv_bfloat16>(get<uintptr_t>(d, "h"));
    p.ldh = get<int64_t>(d, "ldh");
    p.H = get<int>(d, "H");
    p.relu_from = get<int>(d, "relu_from");
    p.w = P<const __nv_bfloat16>(get<uintptr_t>(d, "w"));
    p.bias = P<const __nv_bfloat16>(get<uintptr_t>(d, "bias"));
    p.labels = P<const float>(get<uintptr_t>(d, "labels"));
    p.B = get<int64_t>(d, "B");
    p.valid_count = get_or<int>(d, "valid_count", -1);
    p.grad_scale = get<float>(d, "grad_scale");
    p.logits = P<float>(get<uintptr_t>(d, "logits"));
    p.dl = P<float>(get<uintptr_t>(d, "dl"));
    p.dh = P<__nv_bfloat16>(get<uintptr_t>(d, "dh"));
    p.lddh = get<int64_t>(d, "lddh");
    p.loss_sum = P<float>(get<uintptr_t>(d, "loss_sum"));
    p.db = P<float>(get<uintptr_t>(d, "db"));
    flare::dcn_head(p, cur_stream());
  });
  m.def("dcn_scaled_colsum", [](uintptr_t x, int64_t ldx, uintptr_t scale, int64_t rows, int cols, uintptr_t out) {
    flare::dcn_scaled_colsum(P<const __nv_bfloat16>(x), ldx, P<const float>(scale), rows, cols, P<float>(out),
                             cur_stream());
  });
  m.def("dcn_cross_bwd_elem", [](uintptr_t g, int64_t ldg, uintptr_t x0, uintptr_t z, int64_t ld, int64_t rows,
                                 int cols, uintptr_t dz, uintptr_t acc, int64_t ld_acc, int accumulate, uintptr_t db) {
    flare::dcn_cross_bwd_elem(P<const __nv_bfloat16>(g), ldg, P<const __nv_bfloat16>(x0), P<const __nv_bfloat16>(z), ld,
                              rows, cols, P<__nv_bfloat16>(dz), P<float>(acc), ld_acc, accumulate, P<float>(db),
                              cur_stream());
  });
  m.def("dcn_finalize_grad", [](uintptr_t acc, int64_t ld_acc, int64_t rows, int cols, uintptr_t grad, int64_t ldg) {
    flare::dcn_finalize_grad(P<const float>(acc), ld_acc, rows, cols, P<__nv_bfloat16>(grad), ldg, cur_stream());
  });

  m.def("gate_mix", [](const py::dict& d, bool backward) {
    flare::GateMixParams p{};
    const auto ys = get<std::vector<uintptr_t>>(d, "ys");
    FLARE_CHECK(!ys.empty() && ys.size() <= static_cast<size_t>(flare::kMixMaxExperts), "gate_mix: 1..64 experts");
    p.E = static_cast<int>(ys.size());
    for (int e = 0; e < p.E; ++e) p.ys[e] = P<const __nv_bfloat16>(ys[e]);
    p.logits = P<const __nv_bfloat16>(get<uintptr_t>(d, "logits"));
    p.ld_logits = get<int64_t>(d, "ld_logits");
    p.probs = P<float>(get<uintptr_t>(d, "probs"));
    p.ld_y = get<int64_t>(d, "ld_y");
    p.ld_out = get<int64_t>(d, "ld_out");
    p.B = get<int>(d, "B");
    p.D = get<int>(d, "D");
    if (backward) {
      const auto dys = get<std::vector<uintptr_t>>(d, "dys");
      FLARE_CHECK(dys.size() == ys.size(), "gate_mix: one gradient per expert output");
      for (int e = 0; e < p.E; ++e) p.dys[e] = P<__nv_bfloat16>(dys[e]);
      p.ld_dy = get<int64_t>(d, "ld_dy");
      p.dlogits = P<__nv_bfloat16>(get<uintptr_t>(d, "dlogits"));
      p.dout = P<const __nv_bfloat16>(get<uintptr_t>(d, "dout"));
      flare::gate_mix_backward(p, cur_stream());
    } else {
      p.out = P<__nv_bfloat16>(get<uintptr_t>(d, "out"));
      flare::gate_mix_forward(p, cur_stream());
    }
  });
  m.def("relu_bwd_colsum", [](uintptr_t g, int64_t ldg, uintptr_t h, int64_t ldh, int64_t rows, int cols,
                              uintptr_t gout, int64_t ldo, uintptr_t colsum) {
    flare::relu_bwd_colsum(P<const __nv_bfloat16>(g), ldg, P<const __nv_bfloat16>(h), ldh, rows, cols,
                           P<__nv_bfloat16>(gout), ldo, P<float>(colsum), cur_stream());
  });
  m.def("colsum_bf16", [](uintptr_t x, int64_t rows, int cols, int64_t ldx, uintptr_t out) {
    flare::colsum_bf16(P<const __nv_bfloat16>(x), rows, cols, ldx, P<float>(out), cur_stream());
  });
  m.def("cast_pad_bf16", [](uintptr_t x, int64_t rows, int cols, int64_t ldx, uintptr_t y, int ldy, uintptr_t zero) {
    flare::cast_pad_bf16(P<const float>(x), rows, cols, ldx, P<__nv_bfloat16>(y), ldy, cur_stream(), P<float>(zero));
  });
  m.def("init_uniform", [](uintptr_t out, int dtype, int64_t n, float lo, float hi, uint64_t seed, int64_t off,
                           int ncols, int dim, int col_begin, int64_t row_stride, int64_t row_first) {
    flare::init_uniform(P<void>(out), dtype, n, lo, hi, seed, off, ncols, dim, col_begin, row_stride, row_first,
                        cur_stream());
  }, py::arg("out"), py::arg("dtype"), py::arg("n"), py::arg("lo"), py::arg("hi"), py::arg("seed"), py::arg("off"),
     py::arg("ncols"), py::arg("dim"), py::arg("col_begin"), py::arg("row_stride") = 1, py::arg("row_first") = 0);

  m.def("sparse_gather", [](uintptr_t emb, int dtype, uintptr_t inv, int64_t slots, int dim, int pad, uintptr_t out) {
    flare::sparse_gather(P<const void>(emb), dtype, P<const int>(inv), slots, dim, pad, P<void>(out), cur_stream());
  });
  m.def("sparse_gather_pooled", [](uintptr_t emb, int dtype, uintptr_t inv, int64_t bags, int E, int dim, int pad,
                                   uintptr_t out) {
    flare::sparse_gather_pooled(P<const void>(emb), dtype, P<const int>(inv), bags, E, dim, pad, P<void>(out),
                                cur_stream());
  });
  m.def("sparse_scatter", [](uintptr_t g, int dtype, uintptr_t inv, int64_t slots, int dim, int pad, uintptr_t out) {
    flare::sparse_scatter(P<const void>(g), dtype, P<const int>(inv), slots, dim, pad, P<float>(out), cur_stream());
  });
  m.def("sparse_scatter_pooled", [](uintptr_t g, int dtype, uintptr_t inv, int64_t bags, int E, int dim, int pad,
                                    uintptr_t out) {
    flare::sparse_scatter_pooled(P<const void>(g), dtype, P<const int>(inv), bags, E, dim, pad, P<float>(out),
                                 cur_stream());
  });
  m.def("unique_first_occurrence", [](uintptr_t keys, int64_t n, const py::dict& w, uintptr_t unique,
                                      uintptr_t inverse, uintptr_t first_idx) {
    flare::UniqueScratch s{};
    s.tab_keys = P<unsigned long long>(get<uintptr_t>(w, "tab_keys"));
    s.tab_first = P<int>(get<uintptr_t>(w, "tab_first"));
    s.cap = get<int64_t>(w, "cap");
    s.slot_of = P<int64_t>(get<uintptr_t>(w, "slot_of"));
    s.is_first = P<int>(get<uintptr_t>(w, "is_first"));
    s.pos = P<int>(get<uintptr_t>(w, "pos"));
    s.block_sums = P<int>(get<uintptr_t>(w, "block_sums"));
    flare::unique_first_occurrence(P<const int64_t>(keys), n, s, P<int64_t>(unique), P<int>(inverse),
                                   P<int64_t>(first_idx), cur_stream());
  });
  m.def("exclusive_scan_int", [](uintptr_t in, int64_t n, uintptr_t out, uintptr_t block_sums) {
    flare::exclusive_scan_int(P<const int>(in), n, P<int>(out), P<int>(block_sums), cur_stream());
  });

  m.def("auc_device", [](uintptr_t scores, uintptr_t labels, uintptr_t groups, int64_t n, double negative_factor,
                         const py::dict& w) {
    flare::AucWork a{};
    a.keys_a = P<unsigned long long>(get<uintptr_t>(w, "keys_a"));
    a.keys_b = P<unsigned long long>(get<uintptr_t>(w, "keys_b"));
    a.vals_a = P<int>(get<uintptr_t>(w, "vals_a"));
    a.vals_b = P<int>(get<uintptr_t>(w, "vals_b"));
    a.negs = P<int>(get<uintptr_t>(w, "negs"));
    a.neg_prefix = P<int>(get<uintptr_t>(w, "neg_prefix"));
    a.hist = P<int>(get<uintptr_t>(w, "hist"));
    a.hist_scan = P<int>(get<uintptr_t>(w, "hist_scan"));
    a.block_sums = P<int>(get<uintptr_t>(w, "block_sums"));
    a.credit = P<double>(get_or<uintptr_t>(w, "credit", 0));
    a.pos_cnt = P<unsigned long long>(get_or<uintptr_t>(w, "pos_cnt", 0));
    a.neg_cnt = P<unsigned long long>(get_or<uintptr_t>(w, "neg_cnt", 0));
    a.out = P<double>(get<uintptr_t>(w, "out"));
    flare::auc_device(P<const float>(scores), P<const float>(labels), P<const int64_t>(groups), n, negative_factor, a,
                      cur_stream());
  });
  m.def("radix_sort_pairs", [](uintptr_t ka, uintptr_t va, uintptr_t kb, uintptr_t vb, int64_t n, int bits,
                               uintptr_t hist, uintptr_t hist_scan, uintptr_t block_sums) {
    flare::radix_sort_pairs(P<unsigned long long>(ka), P<int>(va), P<unsigned long long>(kb), P<int>(vb), n, bits,
                            P<int>(hist), P<int>(hist_scan), P<int>(block_sums), cur_stream());
  });

  // ---- symmetric memory plumbing ----
  m.def("wait_flag_probe", [](uintptr_t flag, uint32_t target, uint64_t timeout_ns, uintptr_t status) {
    flare::wait_flag_probe(P<const uint32_t>(flag), target, timeout_ns, P<int>(status), cur_stream());
  });
  m.def("dev_malloc", [](size_t bytes) { return reinterpret_cast<uintptr_t>(flare::dev_malloc(bytes)); });
  m.def("dev_free", [](uintptr_t p) { flare::dev_free(P<void>(p)); });
  m.def("ipc_get_handle", [](uintptr_t p) {
    auto v = flare::ipc_get_handle(P<void>(p));
    return py::bytes(v.data(), v.size());
  });
  m.def("ipc_open_handle", [](py::bytes b) {
    std::string s = b;
    std::vector<char> v(s.begin(), s.end());
    return reinterpret_cast<uintptr_t>(flare::ipc_open_handle(v));
  });
  m.def("ipc_close_handle", [](uintptr_t p) { flare::ipc_close_handle(P<void>(p)); });
  m.def("can_access_peer", &flare::can_access_peer);
  m.def("tensor_from_ptr", [](uintptr_t ptr, std::vector<int64_t> sizes, at::ScalarType dtype, int device) {
    auto opts = at::TensorOptions().dtype(dtype).device(at::Device(at::kCUDA, device));
    return torch::from_blob(reinterpret_cast<void*>(ptr), sizes, [](void*) {}, opts);
  });
}
