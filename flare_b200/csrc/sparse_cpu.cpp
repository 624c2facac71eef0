// CPU sparse embedding ops (host C++, at::parallel_for): the CPU backend of the
// padded gather / pool / scatter contract and the first-occurrence dedup.
//
//   cpu_gather         out[slot] = inv == pad ? 0 : emb[inv]              (value dtype kept)
//   cpu_gather_pooled  out[bag] = sum_e emb[inv[bag, e]] over non-pad e  (fp32 accumulation)
//   cpu_scatter        out[row] += grad[slot] for slots with inv == row  (fp32)
//   cpu_scatter_pooled out[row] += grad[bag] for every non-pad id of the bag
//   cpu_unique_first   unique keys in first-occurrence order, inverse, first index
//
// The scatters are deterministic: slots are deduplicated first, grouped per
// unique row by a counting sort (slot order kept) and each unique row sums its
// slots in order, rows in parallel; no atomics, no private copies of the table.
// fp16 / bf16 values are decoded to fp32 with the library conversions.
// Reference behaviour: src/flare/ops/sparse_gather.py:16-148,
// sparse_scatter.py:15-144 and sparse_unique.py:17-49 (Numba kernels).
#include <torch/extension.h>
#include <ATen/Parallel.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <vector>

namespace py = pybind11;

namespace flare_cpu {

enum : int { kF32 = 0, kBF16 = 1, kF16 = 2 };

inline float load_val(const void* base, int dtype, int64_t i) {
  if (dtype == kF32) return static_cast<const float*>(base)[i];
  if (dtype == kBF16) return static_cast<float>(static_cast<const c10::BFloat16*>(base)[i]);
  return static_cast<float>(static_cast<const c10::Half*>(base)[i]);
}

inline void store_val(void* base, int dtype, int64_t i, float v) {
  if (dtype == kF32) static_cast<float*>(base)[i] = v;
  else if (dtype == kBF16) static_cast<c10::BFloat16*>(base)[i] = c10::BFloat16(v);
  else static_cast<c10::Half*>(base)[i] = c10::Half(v);
}

inline int64_t esize(int dtype) { return dtype == kF32 ? 4 : 2; }

void cpu_gather(uintptr_t emb, int dtype, uintptr_t inv, int64_t slots, int dim, int pad, uintptr_t out) {
  const int32_t* iv = reinterpret_cast<const int32_t*>(inv);
  const char* e = reinterpret_cast<const char*>(emb);
  char* o = reinterpret_cast<char*>(out);
  const int64_t rb = dim * esize(dtype);
  at::parallel_for(0, slots, 1024, [&](int64_t lo, int64_t hi) {
    for (int64_t s = lo; s < hi; ++s) {
      if (iv[s] == pad) std::memset(o + s * rb, 0, rb);
      else std::memcpy(o + s * rb, e + static_cast<int64_t>(iv[s]) * rb, rb);
    }
  });
}

void cpu_gather_pooled(uintptr_t emb, int dtype, uintptr_t inv, int64_t bags, int E, int dim, int pad,
                       uintptr_t out) {
  const int32_t* iv = reinterpret_cast<const int32_t*>(inv);
  const void* e = reinterpret_cast<const void*>(emb);
  void* o = reinterpret_cast<void*>(out);
  at::parallel_for(0, bags, 256, [&](int64_t lo, int64_t hi) {
    std::vector<float> acc(dim);
    for (int64_t b = lo; b < hi; ++b) {
      std::fill(acc.begin(), acc.end(), 0.f);
      for (int k = 0; k < E; ++k) {
        const int32_t r = iv[b * E + k];
        if (r == pad) continue;
        const int64_t base = static_cast<int64_t>(r) * dim;
        for (int d = 0; d < dim; ++d) acc[d] += load_val(e, dtype, base + d);
      }
      for (int d = 0; d < dim; ++d) store_val(o, dtype, b * dim + d, acc[d]);
    }
  });
}

// first-occurrence dedup with an open-addressing table (Fibonacci hashing)
struct Dedup {
  std::vector<int64_t> unique, first;
  std::vector<int32_t> inverse;
};

Dedup dedup(const int64_t* keys, int64_t n, bool skip, int64_t skip_key) {
  Dedup r;
  r.inverse.assign(n, -1);
  int64_t cap = 16;
  while (cap < 2 * n) cap <<= 1;
  std::vector<int64_t> tk(cap);
  std::vector<int32_t> tu(cap, -1);
  const int shift = 64 - __builtin_ctzll(static_cast<uint64_t>(cap));
  for (int64_t i = 0; i < n; ++i) {
    const int64_t k = keys[i];
    if (skip && k == skip_key) continue;
    uint64_t h = (static_cast<uint64_t>(k) * 11400714819323198485ull) >> shift;
    while (true) {
      if (tu[h] < 0) {
        tu[h] = static_cast<int32_t>(r.unique.size());
        tk[h] = k;
        r.unique.push_back(k);
        r.first.push_back(i);
        break;
      }
      if (tk[h] == k) break;
      h = (h + 1) & static_cast<uint64_t>(cap - 1);
    }
    r.inverse[i] = tu[h];
  }
  return r;
}

py::tuple cpu_unique_first(torch::Tensor keys) {
  TORCH_CHECK(!keys.is_cuda() && (keys.scalar_type() == torch::kInt64 || keys.scalar_type() == torch::kInt32),
              "cpu_unique_first: int32/int64 CPU keys");
  auto k64 = keys.reshape(-1).to(torch::kInt64).contiguous();
  const int64_t n = k64.numel();
  Dedup d = dedup(k64.data_ptr<int64_t>(), n, false, 0);
  const int64_t u = static_cast<int64_t>(d.unique.size());
  auto uniq = torch::from_blob(d.unique.data(), {u}, torch::kInt64).clone().to(keys.scalar_type());
  auto inv = torch::from_blob(d.inverse.data(), {n}, torch::kInt32).clone();
  auto first = torch::from_blob(d.first.data(), {u}, torch::kInt64).clone();
  return py::make_tuple(uniq, inv, first);
}

// rows of `inv` (pad skipped) -> per unique row its source indices in order; then out[row] = sum
void scatter_grouped(const int32_t* iv, int64_t n, int pad, int dim, const void* g, int gdtype, int64_t g_div,
                     float* out) {
  std::vector<int64_t> k(n);
  for (int64_t i = 0; i < n; ++i) k[i] = iv[i];
  Dedup d = dedup(k.data(), n, true, pad);
  const int64_t U = static_cast<int64_t>(d.unique.size());
  std::vector<int64_t> start(U + 1, 0);
  for (int64_t i = 0; i < n; ++i)
    if (d.inverse[i] >= 0) ++start[d.inverse[i] + 1];
  for (int64_t u = 0; u < U; ++u) start[u + 1] += start[u];
  std::vector<int64_t> pos(start.begin(), start.end() - 1), order(start[U]);
  for (int64_t i = 0; i < n; ++i)
    if (d.inverse[i] >= 0) order[pos[d.inverse[i]]++] = i;
  at::parallel_for(0, U, 64, [&](int64_t lo, int64_t hi) {
    for (int64_t u = lo; u < hi; ++u) {
      float* o = out + d.unique[u] * dim;
      for (int64_t q = start[u]; q < start[u + 1]; ++q) {
        const int64_t src = (order[q] / g_div) * dim;  // g_div = E for pooled gradients (one per bag)
        for (int c = 0; c < dim; ++c) o[c] += load_val(g, gdtype, src + c);
      }
    }
  });
}

void cpu_scatter(uintptr_t grad, int gdtype, uintptr_t inv, int64_t slots, int dim, int pad, uintptr_t out) {
  scatter_grouped(reinterpret_cast<const int32_t*>(inv), slots, pad, dim, reinterpret_cast<const void*>(grad),
                  gdtype, 1, reinterpret_cast<float*>(out));
}

void cpu_scatter_pooled(uintptr_t grad, int gdtype, uintptr_t inv, int64_t bags, int E, int dim, int pad,
                        uintptr_t out) {
  scatter_grouped(reinterpret_cast<const int32_t*>(inv), bags * E, pad, dim, reinterpret_cast<const void*>(grad),
                  gdtype, E, reinterpret_cast<float*>(out));
}

// ---- keyed-jagged collection ops (the CPU configuration's sparse step) ----
// offsets [F*B+1] (int32) cut `values` (int32 ids) into bags, feature-major;
// table f is `weights[f]` [rows_f, dims_f] (fp32 / bf16 / fp16).

inline int dtype_code(const torch::Tensor& t) {
  if (t.scalar_type() == torch::kFloat32) return kF32;
  if (t.scalar_type() == torch::kBFloat16) return kBF16;
  TORCH_CHECK(t.scalar_type() == torch::kFloat16, "tables must be float32, bfloat16 or float16");
  return kF16;
}

void check_bags(const torch::Tensor& offsets, const torch::Tensor& values, int64_t F, int64_t B) {
  TORCH_CHECK(!offsets.is_cuda() && !values.is_cuda() && offsets.scalar_type() == torch::kInt32 &&
                  values.scalar_type() == torch::kInt32 && offsets.is_contiguous() && values.is_contiguous(),
              "offsets / values: contiguous int32 CPU tensors");
  TORCH_CHECK(offsets.numel() == F * B + 1, "offsets must have F*B+1 entries");
  const int32_t* off = offsets.data_ptr<int32_t>();
  TORCH_CHECK(off[0] >= 0 && off[F * B] <= values.numel(), "offsets outside the id array");
  for (int64_t k = 0; k < F * B; ++k) TORCH_CHECK(off[k + 1] >= off[k], "offsets must not decrease");
}

// out[b, col_f:col_f+d_f] = sum (mean) of table f's rows over bag (f, b); ids < 0 are skipped
torch::Tensor cpu_bag_pool(std::vector<torch::Tensor> weights, torch::Tensor offsets, torch::Tensor values,
                           int64_t B, std::vector<int64_t> mean) {
  const int64_t F = static_cast<int64_t>(weights.size());
  TORCH_CHECK(static_cast<int64_t>(mean.size()) == F, "one pooling flag per table");
  check_bags(offsets, values, F, B);
  std::vector<int64_t> cols(F + 1, 0);
  for (int64_t f = 0; f < F; ++f) {
    TORCH_CHECK(!weights[f].is_cuda() && weights[f].dim() == 2 && weights[f].is_contiguous(), "tables: 2-D CPU");
    cols[f + 1] = cols[f] + weights[f].size(1);
  }
  const int32_t* off = offsets.data_ptr<int32_t>();
  const int32_t* ids = values.data_ptr<int32_t>();
  for (int64_t f = 0; f < F; ++f)  // id range, before any parallel work
    for (int64_t e = off[f * B]; e < off[(f + 1) * B]; ++e)
      TORCH_CHECK(ids[e] < weights[f].size(0), "id ", ids[e], " of table ", f, " >= ", weights[f].size(0));
  auto out = torch::zeros({B, cols[F]}, torch::kFloat32);
  float* o = out.data_ptr<float>();
  at::parallel_for(0, F * B, 64, [&](int64_t lo, int64_t hi) {
    for (int64_t k = lo; k < hi; ++k) {
      const int64_t f = k / B, b = k - f * B, d = weights[f].size(1);
      const void* w = weights[f].data_ptr();
      const int dt = dtype_code(weights[f]);
      float* acc = o + b * cols[F] + cols[f];
      for (int64_t e = off[k]; e < off[k + 1]; ++e) {
        if (ids[e] < 0) continue;
        const int64_t base = static_cast<int64_t>(ids[e]) * d;
        for (int64_t c = 0; c < d; ++c) acc[c] += load_val(w, dt, base + c);
      }
      if (mean[f]) {
        const float inv = 1.f / static_cast<float>(std::max<int64_t>(1, off[k + 1] - off[k]));
        for (int64_t c = 0; c < d; ++c) acc[c] *= inv;
      }
    }
  });
  return out;
}

// Per table: (unique ids ascending [U] int64, summed fp32 gradient rows [U, d], occurrence counts [U] fp32).
// Each unique id adds its occurrences' pooled gradients in occurrence order (deterministic; no atomics).
std::vector<py::tuple> cpu_bag_row_grads(torch::Tensor grad, torch::Tensor offsets, torch::Tensor values,
                                         int64_t B, std::vector<int64_t> dims, std::vector<int64_t> mean) {
  const int64_t F = static_cast<int64_t>(dims.size());
  check_bags(offsets, values, F, B);
  TORCH_CHECK(!grad.is_cuda() && grad.scalar_type() == torch::kFloat32 && grad.is_contiguous() && grad.dim() == 2 &&
                  grad.size(0) == B, "grad: contiguous float32 [B, total_dim] CPU tensor");
  const int64_t total = grad.size(1);
  const int32_t* off = offsets.data_ptr<int32_t>();
  const int32_t* ids = values.data_ptr<int32_t>();
  const float* g = grad.data_ptr<float>();
  std::vector<int64_t> cols(F + 1, 0);
  for (int64_t f = 0; f < F; ++f) cols[f + 1] = cols[f] + dims[f];
  TORCH_CHECK(cols[F] == total, "table widths must add up to the gradient width");
  std::vector<torch::Tensor> uq(F), acc(F), cnt(F);
  at::parallel_for(0, F, 1, [&](int64_t lo, int64_t hi) {
    for (int64_t f = lo; f < hi; ++f) {
      const int64_t e0 = off[f * B], e1 = off[(f + 1) * B], d = dims[f];
      // occurrences (id, bag) in order, stably sorted by id
      std::vector<int64_t> occ;
      occ.reserve(static_cast<size_t>(e1 - e0));
      std::vector<int64_t> bag_of(static_cast<size_t>(e1 - e0));
      for (int64_t b = 0; b < B; ++b)
        for (int64_t e = off[f * B + b]; e < off[f * B + b + 1]; ++e) bag_of[e - e0] = b;
      for (int64_t e = e0; e < e1; ++e)
        if (ids[e] >= 0) occ.push_back(e);
      std::stable_sort(occ.begin(), occ.end(), [&](int64_t a, int64_t c) { return ids[a] < ids[c]; });
      int64_t U = 0;
      for (size_t i = 0; i < occ.size(); ++i)
        if (i == 0 || ids[occ[i]] != ids[occ[i - 1]]) ++U;
      auto u = torch::empty({U}, torch::kInt64);
      auto a = torch::zeros({U, d}, torch::kFloat32);
      auto n = torch::zeros({U}, torch::kFloat32);
      int64_t* up = u.data_ptr<int64_t>();
      float* ap = a.data_ptr<float>();
      float* np = n.data_ptr<float>();
      int64_t j = -1;
      for (size_t i = 0; i < occ.size(); ++i) {
        const int64_t e = occ[i];
        if (i == 0 || ids[e] != ids[occ[i - 1]]) up[++j] = ids[e];
        const int64_t b = bag_of[e - e0];
        float scale = 1.f;
        if (mean[f]) scale = 1.f / static_cast<float>(std::max<int64_t>(1, off[f * B + b + 1] - off[f * B + b]));
        const float* src = g + b * total + cols[f];
        float* dst = ap + j * d;
        for (int64_t c = 0; c < d; ++c) dst[c] += src[c] * scale;
        np[j] += 1.f;
      }
      uq[f] = u;
      acc[f] = a;
      cnt[f] = n;
    }
  });
  std::vector<py::tuple> res;
  for (int64_t f = 0; f < F; ++f) res.push_back(py::make_tuple(uq[f], acc[f], cnt[f]));
  return res;
}

// ---- row-wise sparse optimizer on the touched rows (host) ----
// w[rows[u]] updated from the summed gradient g[u] (fp32 math, the weights' dtype on store); the
// optimizer state lives in full-table fp32 tensors (row: [rows], m / v: [rows, d], score: [rows]).
enum OptKind : int { kSgd = 0, kRowAdagrad = 1, kAdam = 2, kRowAdam = 3, kAdagrad = 4 };  // sparse/config.py codes
enum LrPolicy : int { kConst = 0, kSqrt = 1, kLog = 2, kInverse = 3, kCosine = 4, kLut = 5 };

struct OptArgs {
  int kind, policy;
  float lr, b1, b2, eps, wd, cos_min, cos_max;
  int64_t step;
  std::vector<float> lut;
};

inline float lr_scale(const OptArgs& o, float score) {
  switch (o.policy) {
    case kSqrt: return 1.f / std::sqrt(std::max(score, 1.f));
    case kLog: return 1.f / (1.f + std::log1p(std::max(score, 0.f)));
    case kInverse: return 1.f / std::max(score, 1.f);
    case kCosine: {
      const float S = std::max(o.cos_max, 1e-12f);
      const float x = std::min(std::max(score, 0.f), o.cos_max) / S;
      return o.cos_min + (1.f - o.cos_min) * 0.5f * (1.f + std::cos(3.14159265358979323846f * x));
    }
    case kLut: {
      const int64_t i = std::min<int64_t>(static_cast<int64_t>(std::floor(std::max(score, 0.f))),
                                          static_cast<int64_t>(o.lut.size()) - 1);
      return o.lut[static_cast<size_t>(i)];
    }
    default: return 1.f;
  }
}

void cpu_apply_rows(int kind, int policy, std::vector<double> hp, std::vector<double> lut, int64_t step,
                    torch::Tensor w, torch::Tensor rows, torch::Tensor g, torch::Tensor cnt, torch::Tensor row_state,
                    torch::Tensor m, torch::Tensor v, torch::Tensor score) {
  TORCH_CHECK(hp.size() == 7, "hyper-parameters: lr, beta1, beta2, eps, weight_decay, cos_min, cos_max");
  OptArgs o{kind, policy, static_cast<float>(hp[0]), static_cast<float>(hp[1]), static_cast<float>(hp[2]),
            static_cast<float>(hp[3]), static_cast<float>(hp[4]), static_cast<float>(hp[5]),
            static_cast<float>(hp[6]), std::max<int64_t>(step, 1), {}};
  for (double x : lut) o.lut.push_back(static_cast<float>(x));
  TORCH_CHECK(policy != kLut || !o.lut.empty(), "custom LUT policy needs a LUT");
  TORCH_CHECK(w.dim() == 2 && w.is_contiguous() && !w.is_cuda(), "w: contiguous 2-D CPU table");
  TORCH_CHECK(rows.scalar_type() == torch::kInt64 && rows.is_contiguous(), "rows: contiguous int64");
  TORCH_CHECK(g.scalar_type() == torch::kFloat32 && g.is_contiguous() && g.dim() == 2 && g.size(0) == rows.numel() &&
                  g.size(1) == w.size(1), "g: contiguous float32 [U, d]");
  TORCH_CHECK(cnt.scalar_type() == torch::kFloat32 && cnt.numel() == rows.numel(), "cnt: float32 [U]");
  const bool need_row = kind == kRowAdagrad || kind == kRowAdam, need_m = kind == kAdagrad || kind == kAdam ||
                                                                          kind == kRowAdam,
             need_v = kind == kAdam, need_score = policy != kConst;
  auto ok = [&](const torch::Tensor& t, bool need, bool two_d) {
    if (!need) return;
    TORCH_CHECK(t.defined() && t.numel() > 0 && t.scalar_type() == torch::kFloat32 && t.is_contiguous() &&
                    t.size(0) == w.size(0) && (two_d ? t.dim() == 2 && t.size(1) == w.size(1) : t.dim() == 1),
                "optimizer state tensor has the wrong shape / dtype");
  };
  ok(row_state, need_row, false);
  ok(m, need_m, true);
  ok(v, need_v, true);
  ok(score, need_score, false);
  const int64_t U = rows.numel(), d = w.size(1), R = w.size(0);
  const int64_t* rp = rows.data_ptr<int64_t>();
  for (int64_t u = 0; u < U; ++u) TORCH_CHECK(rp[u] >= 0 && rp[u] < R, "row ", rp[u], " outside the table");
  const float* gp = g.data_ptr<float>();
  const float* cp = cnt.data_ptr<float>();
  float* rs = need_row ? row_state.data_ptr<float>() : nullptr;
  float* mp = need_m ? m.data_ptr<float>() : nullptr;
  float* vp = need_v ? v.data_ptr<float>() : nullptr;
  float* sp = need_score ? score.data_ptr<float>() : nullptr;
  void* wp = w.data_ptr();
  const int wdt = dtype_code(w);
  const float bc1 = 1.f - std::pow(o.b1, static_cast<float>(o.step));
  const float bc2 = 1.f - std::pow(o.b2, static_cast<float>(o.step));
  at::parallel_for(0, U, 64, [&](int64_t lo, int64_t hi) {
    std::vector<float> wr(static_cast<size_t>(d)), gr(static_cast<size_t>(d));
    for (int64_t u = lo; u < hi; ++u) {
      const int64_t r = rp[u];
      float g2 = 0.f;
      for (int64_t c = 0; c < d; ++c) {
        wr[c] = load_val(wp, wdt, r * d + c);
        gr[c] = gp[u * d + c] + o.wd * wr[c];
        g2 += gr[c] * gr[c];
      }
      g2 /= static_cast<float>(d);
      float lr = o.lr;
      if (sp) {
        sp[r] += cp[u];
        lr *= lr_scale(o, sp[r]);
      }
      switch (kind) {
        case kSgd:
          for (int64_t c = 0; c < d; ++c) wr[c] -= lr * gr[c];
          break;
        case kRowAdagrad: {
          rs[r] += g2;
          const float den = std::sqrt(rs[r]) + o.eps;
          for (int64_t c = 0; c < d; ++c) wr[c] -= lr * gr[c] / den;
          break;
        }
        case kAdagrad:
          for (int64_t c = 0; c < d; ++c) {
            float& acc = mp[r * d + c];
            acc += gr[c] * gr[c];
            wr[c] -= lr * gr[c] / (std::sqrt(acc) + o.eps);
          }
          break;
        case kAdam:
          for (int64_t c = 0; c < d; ++c) {
            float& mm = mp[r * d + c];
            float& vv = vp[r * d + c];
            mm = o.b1 * mm + (1.f - o.b1) * gr[c];
            vv = o.b2 * vv + (1.f - o.b2) * gr[c] * gr[c];
            wr[c] -= lr * (mm / bc1) / (std::sqrt(vv / bc2) + o.eps);
          }
          break;
        case kRowAdam: {
          rs[r] = o.b2 * rs[r] + (1.f - o.b2) * g2;
          const float den = std::sqrt(rs[r] / bc2) + o.eps;
          for (int64_t c = 0; c < d; ++c) {
            float& mm = mp[r * d + c];
            mm = o.b1 * mm + (1.f - o.b1) * gr[c];
            wr[c] -= lr * (mm / bc1) / den;
          }
          break;
        }
        default: break;
      }
      for (int64_t c = 0; c < d; ++c) store_val(wp, wdt, r * d + c, wr[c]);
    }
  });
}

}  // namespace flare_cpu

void register_sparse_cpu(py::module_& m) {
  auto c = m.def_submodule("cpu", "CPU sparse embedding ops (host)");
  c.def("gather", &flare_cpu::cpu_gather);
  c.def("gather_pooled", &flare_cpu::cpu_gather_pooled);
  c.def("scatter", &flare_cpu::cpu_scatter);
  c.def("scatter_pooled", &flare_cpu::cpu_scatter_pooled);
  c.def("unique_first", &flare_cpu::cpu_unique_first);
  c.def("bag_pool", &flare_cpu::cpu_bag_pool);
  c.def("bag_row_grads", &flare_cpu::cpu_bag_row_grads);
  c.def("apply_rows", &flare_cpu::cpu_apply_rows);
}
