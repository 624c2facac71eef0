// Native feature-ETL kernels for the offline production pipeline (host C++).
//
// Record format (the data contract of the production logs): lines separated
// by '\n'; columns separated by TAB; the feature column holds
// `code\x03value` items separated by \x02; a list value is comma separated.
// Missing / unparsable values take the null sentinel -3.
//
//   scan_records   : one pass over a byte buffer of many lines with memchr;
//                    numbers are parsed straight into caller-owned NumPy
//                    buffers according to a field plan (code -> buffer, length,
//                    float?) and a per-buffer validity mask is set;
//   fnv1a_lists    : FNV-1a 64 over the int64 items of each list (optionally
//                    modulo a bucket count);
//   fnv1a_seeded   : FNV-1a 64 over the significant little-endian bytes of seed,
//                    then of the value (zero: one zero byte; negative: none);
//   hash_bucket    : value mod bucket (as uint64), sentinel / default -> sentinel;
//   bucketize      : index of the first bound >= value (sorted bounds);
//   fixed_width    : trunc(value / width);
//   pack_fids      : slot in the top 16 bits, the value's low 48 bits below;
//   intersect_lists: per row, how many items of list A occur in list B;
//   parse_rows     : the record format read from an Arrow string column's
//                    buffers, with category vocabularies, variable-length
//                    lists, direct and metadata columns (details below).
// The reference implements these with Cython (processing/native/_scan.pyx:73,
// builder/_fast_parse.pyx:87-350)
// and Numba (builder/encoding/sparse_id.py:206,253,269, encoding/dense.py:30,40,
// cross/fea_ops.py:63-94); this is a separate implementation of the same
// record format and encodings.
#include <torch/extension.h>
#include <pybind11/numpy.h>
#include <pybind11/stl.h>

#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>

namespace py = pybind11;

namespace flare_etl {

constexpr int64_t kNull = -3;
constexpr uint64_t kFnvOffset = 14695981039346656037ull;
constexpr uint64_t kFnvPrime = 1099511628211ull;

// Integer with at most 18 digits (and optional sign), else strtod; empty -> null.
inline int64_t parse_int(const char* s, const char* e) {
  if (s >= e) return kNull;
  const char* p = s;
  bool neg = false;
  if (*p == '-' || *p == '+') {
    neg = *p == '-';
    ++p;
  }
  if (p >= e || e - p > 18) {
    char buf[64];
    const size_t n = static_cast<size_t>(e - s);
    if (n == 0 || n >= sizeof(buf)) return kNull;
    std::memcpy(buf, s, n);
    buf[n] = 0;
    char* end = nullptr;
    const double v = std::strtod(buf, &end);
    return end == buf ? kNull : static_cast<int64_t>(v);
  }
  int64_t v = 0;
  for (; p < e; ++p) {
    const int d = *p - '0';
    if (d < 0 || d > 9) {
      char buf[64];
      const size_t n = static_cast<size_t>(e - s);
      if (n >= sizeof(buf)) return kNull;
      std::memcpy(buf, s, n);
      buf[n] = 0;
      char* end = nullptr;
      const double f = std::strtod(buf, &end);
      return end == buf ? kNull : static_cast<int64_t>(f);
    }
    v = v * 10 + d;
  }
  return neg ? -v : v;
}

inline double parse_float(const char* s, const char* e) {
  char buf[64];
  const size_t n = static_cast<size_t>(e - s);
  if (n == 0 || n >= sizeof(buf)) return static_cast<double>(kNull);
  std::memcpy(buf, s, n);
  buf[n] = 0;
  char* end = nullptr;
  const double v = std::strtod(buf, &end);
  return end == buf ? static_cast<double>(kNull) : v;
}

struct Field {
  int buffer;
  int length;
  bool is_float;
};

// buffers[i]: float64 or int64 array [rows, length_i] (contiguous); validity[i]: uint8 [rows] or None.
py::tuple scan_records(py::bytes data, int num_columns, int feature_column, py::dict plan, py::list buffers,
                       py::list validity) {
  std::unordered_map<int64_t, Field> fields;
  for (auto item : plan) {
    const auto t = item.second.cast<py::tuple>();
    fields[item.first.cast<int64_t>()] = Field{t[0].cast<int>(), t[1].cast<int>(), t[2].cast<bool>()};
  }
  const int nb = static_cast<int>(buffers.size());
  std::vector<char*> bufp(nb);
  std::vector<int64_t> rows_cap(nb);
  std::vector<uint8_t*> valp(nb, nullptr);
  for (int i = 0; i < nb; ++i) {
    py::array a = buffers[i].cast<py::array>();
    if (!(a.flags() & py::array::c_style)) throw std::invalid_argument("buffers must be C-contiguous");
    bufp[i] = static_cast<char*>(a.mutable_data());
    rows_cap[i] = a.shape(0);
    if (!validity[i].is_none()) valp[i] = static_cast<uint8_t*>(validity[i].cast<py::array>().mutable_data());
  }
  std::string_view buf = data;
  const char* p = buf.data();
  const char* end = p + buf.size();
  int64_t row = 0;
  while (p < end) {
    const char* nl = static_cast<const char*>(std::memchr(p, '\n', end - p));
    const char* le = nl ? nl : end;
    if (le > p) {
      const char* col = p;
      for (int c = 0; c < num_columns && col <= le; ++c) {
        const char* tab = static_cast<const char*>(std::memchr(col, '\t', le - col));
        const char* ce = tab ? tab : le;
        if (c == feature_column) {
          const char* kv = col;
          while (kv < ce) {
            const char* sep = static_cast<const char*>(std::memchr(kv, '\x02', ce - kv));
            const char* kve = sep ? sep : ce;
            const char* eq = static_cast<const char*>(std::memchr(kv, '\x03', kve - kv));
            if (eq) {
              const auto it = fields.find(parse_int(kv, eq));
              if (it != fields.end()) {
                const Field& f = it->second;
                if (row >= rows_cap[f.buffer]) throw std::out_of_range("more records than buffer rows");
                const char* v = eq + 1;
                for (int k = 0; k < f.length && v <= kve; ++k) {
                  const char* comma = static_cast<const char*>(std::memchr(v, ',', kve - v));
                  const char* vend = (f.length > 1 && comma) ? comma : kve;
                  const int64_t off = row * f.length + k;
                  if (f.is_float) reinterpret_cast<double*>(bufp[f.buffer])[off] = parse_float(v, vend);
                  else reinterpret_cast<int64_t*>(bufp[f.buffer])[off] = parse_int(v, vend);
                  if (vend == kve) break;
                  v = vend + 1;
                }
                if (valp[f.buffer]) valp[f.buffer][row] = 1;
              }
            }
            if (!sep) break;
            kv = sep + 1;
          }
        }
        if (!tab) break;
        col = tab + 1;
      }
      ++row;
    }
    if (!nl) break;
    p = nl + 1;
  }
  return py::make_tuple(row);
}

py::array_t<uint64_t> fnv1a_lists(py::array_t<int64_t, py::array::c_style> values,
                                  py::array_t<int64_t, py::array::c_style> offsets, uint64_t buckets) {
  const int64_t n = offsets.size() - 1;
  py::array_t<uint64_t> out(n);
  const int64_t* v = values.data();
  const int64_t* o = offsets.data();
  uint64_t* r = out.mutable_data();
  for (int64_t i = 0; i < n; ++i) {
    uint64_t h = kFnvOffset;
    for (int64_t j = o[i]; j < o[i + 1]; ++j) {
      h ^= static_cast<uint64_t>(v[j]);
      h *= kFnvPrime;
    }
    r[i] = buckets ? h % buckets : h;
  }
  return out;
}

inline uint64_t fnv_bytes(uint64_t h, uint64_t x, bool zero_is_byte) {
  if (x == 0 && zero_is_byte) {
    h ^= 0;
    return h * kFnvPrime;
  }
  while (x > 0) {
    h ^= (x & 0xFF);
    h *= kFnvPrime;
    x >>= 8;
  }
  return h;
}

py::array_t<uint64_t> fnv1a_seeded(py::array_t<int64_t, py::array::c_style> values, uint64_t seed) {
  const int64_t n = values.size();
  py::array_t<uint64_t> out(n);
  const int64_t* v = values.data();
  uint64_t* r = out.mutable_data();
  const uint64_t hs = fnv_bytes(kFnvOffset, seed, false);
  // zero hashes one zero byte; negative values contribute no bytes
  for (int64_t i = 0; i < n; ++i) r[i] = v[i] < 0 ? hs : fnv_bytes(hs, static_cast<uint64_t>(v[i]), true);
  return out;
}

py::array_t<int64_t> hash_bucket(py::array_t<int64_t, py::array::c_style> values, uint64_t buckets,
                                 int64_t default_value) {
  if (buckets == 0) throw std::invalid_argument("bucket count must be positive");
  const int64_t n = values.size();
  py::array_t<int64_t> out(n);
  const int64_t* v = values.data();
  int64_t* r = out.mutable_data();
  for (int64_t i = 0; i < n; ++i)
    r[i] = (v[i] == default_value || v[i] == kNull) ? kNull
                                                      : static_cast<int64_t>(static_cast<uint64_t>(v[i]) % buckets);
  return out;
}

py::array_t<int32_t> bucketize(py::array_t<float, py::array::c_style> values,
                               py::array_t<float, py::array::c_style> bounds, float default_value) {
  const int64_t n = values.size(), nb = bounds.size();
  py::array_t<int32_t> out(n);
  const float* v = values.data();
  const float* b = bounds.data();
  int32_t* r = out.mutable_data();
  for (int64_t i = 0; i < n; ++i) {
    if (v[i] == static_cast<float>(kNull) || v[i] == default_value) {
      r[i] = static_cast<int32_t>(kNull);
      continue;
    }
    int64_t lo = 0, hi = nb;  // first bound >= value
    while (lo < hi) {
      const int64_t mid = (lo + hi) / 2;
      if (b[mid] < v[i]) lo = mid + 1;
      else hi = mid;
    }
    r[i] = static_cast<int32_t>(lo);
  }
  return out;
}

py::array_t<int32_t> fixed_width(py::array_t<float, py::array::c_style> values, float width, float default_value) {
  const int64_t n = values.size();
  py::array_t<int32_t> out(n);
  const float* v = values.data();
  int32_t* r = out.mutable_data();
  for (int64_t i = 0; i < n; ++i)
    r[i] = (v[i] == static_cast<float>(kNull) || v[i] == default_value) ? static_cast<int32_t>(kNull)
                                                                          : static_cast<int32_t>(v[i] / width);
  return out;
}

py::array_t<int64_t> pack_fids(py::array_t<int64_t, py::array::c_style> values, int slot) {
  if (slot < 0 || slot >= (1 << 16)) throw std::invalid_argument("slot must be in [0, 65536)");
  const int64_t n = values.size();
  py::array_t<int64_t> out(n);
  const int64_t* v = values.data();
  int64_t* r = out.mutable_data();
  const uint64_t hi = static_cast<uint64_t>(slot) << 48;
  for (int64_t i = 0; i < n; ++i)
    r[i] = static_cast<int64_t>(hi | (static_cast<uint64_t>(v[i]) & ((1ull << 48) - 1)));
  return out;
}

py::array_t<int32_t> intersect_lists(py::array_t<int64_t, py::array::c_style> a, py::array_t<int64_t, py::array::c_style> oa,
                                     py::array_t<int64_t, py::array::c_style> b, py::array_t<int64_t, py::array::c_style> ob) {
  const int64_t n = oa.size() - 1;
  if (ob.size() - 1 != n) throw std::invalid_argument("row counts differ");
  py::array_t<int32_t> out(n);
  const int64_t *va = a.data(), *pa = oa.data(), *vb = b.data(), *pb = ob.data();
  int32_t* r = out.mutable_data();
  for (int64_t i = 0; i < n; ++i) {
    int32_t c = 0;
    for (int64_t x = pa[i]; x < pa[i + 1]; ++x) {
      if (va[x] == kNull) continue;
      for (int64_t y = pb[i]; y < pb[i + 1]; ++y)
        if (vb[y] == va[x]) ++c;
    }
    r[i] = c;
  }
  return out;
}

// ---------------------------------------------------------------------------
// parse_rows: the same record format read straight from an Arrow string
// column (its data buffer + int64 offsets, no per-row Python objects), with
// four kinds of outputs:
//   fixed    : code -> [rows, length] int64 / float64 (as scan_records);
//   list     : code -> variable-length int64 / float64 values + [rows + 1]
//              offsets (caller-sized value capacity);
//   category : code -> int32 [rows]: the value token looked up in that code's
//              vocabulary (token bytes -> index), unknown tokens -> the code's
//              default index, missing -> -3;
//   direct   : TAB column -> int64 [rows] (the column parsed as an integer);
//   metadata : TAB column -> int32 [rows] through a string -> id table
//              (unknown -> the table's default).
// Validity bytes are set per output row where a value was seen.
// ---------------------------------------------------------------------------
struct Out {
  int kind;  // 0 fixed, 1 list, 2 category
  int length;
  bool is_float;
  char* data;
  int64_t cap;  // rows (fixed/category) or value capacity (list)
  int64_t* offs;
  uint8_t* valid;
  const std::unordered_map<std::string, int32_t>* vocab;
  int32_t dflt;
};

template <typename T>
T* arr_ptr(py::handle h, int64_t& n) {
  py::array a = py::reinterpret_borrow<py::array>(h);
  if (!(a.flags() & py::array::c_style)) throw std::invalid_argument("arrays must be C-contiguous");
  if (a.itemsize() != sizeof(T)) throw std::invalid_argument("array has the wrong element size");
  n = a.shape(0);
  return static_cast<T*>(a.mutable_data());
}

py::tuple parse_rows(py::array_t<uint8_t, py::array::c_style> data, py::array_t<int64_t, py::array::c_style> offsets,
                     int64_t n_rows, int feature_column, py::dict plan, py::dict categories, py::list direct,
                     py::list metadata) {
  if (offsets.size() < n_rows + 1) throw std::invalid_argument("offsets shorter than n_rows + 1");
  const uint8_t* base = data.data();
  const int64_t* ro = offsets.data();
  if (n_rows > 0 && (ro[0] < 0 || ro[n_rows] > data.size())) throw std::out_of_range("offsets outside the data");
  // category vocabularies
  std::unordered_map<int64_t, std::unordered_map<std::string, int32_t>> vocabs;
  std::unordered_map<int64_t, int32_t> dflts;
  for (auto item : categories) {
    const int64_t code = item.first.cast<int64_t>();
    const auto t = item.second.cast<py::tuple>();
    auto& v = vocabs[code];
    for (auto kv : t[0].cast<py::dict>()) v[kv.first.cast<std::string>()] = kv.second.cast<int32_t>();
    dflts[code] = t[1].cast<int32_t>();
  }
  // plan: code -> (kind, length, is_float, buffer, offsets or None, validity or None)
  std::unordered_map<int64_t, Out> outs;
  for (auto item : plan) {
    const int64_t code = item.first.cast<int64_t>();
    const auto t = item.second.cast<py::tuple>();
    Out o{};
    o.kind = t[0].cast<int>();
    o.length = t[1].cast<int>();
    o.is_float = t[2].cast<bool>();
    int64_t n = 0;
    o.data = o.kind == 2 ? reinterpret_cast<char*>(arr_ptr<int32_t>(t[3], n))
                         : (o.is_float ? reinterpret_cast<char*>(arr_ptr<double>(t[3], n))
                                       : reinterpret_cast<char*>(arr_ptr<int64_t>(t[3], n)));
    o.cap = n;
    if (o.kind == 1) {
      int64_t no = 0;
      o.offs = arr_ptr<int64_t>(t[4], no);
      if (no < n_rows + 1) throw std::invalid_argument("list offsets shorter than n_rows + 1");
      o.offs[0] = 0;
    }
    if (!t[5].is_none()) {
      int64_t nv = 0;
      o.valid = arr_ptr<uint8_t>(t[5], nv);
      if (nv < n_rows) throw std::invalid_argument("validity shorter than n_rows");
    }
    if (o.kind == 2) {
      const auto it = vocabs.find(code);
      if (it == vocabs.end()) throw std::invalid_argument("category output without a vocabulary");
      o.vocab = &it->second;
      o.dflt = dflts[code];
    }
    if (o.kind != 1 && o.cap < n_rows) throw std::invalid_argument("output has fewer rows than n_rows");
    outs[code] = o;
  }
  struct Direct {
    int col;
    int64_t* out;
    uint8_t* valid;
  };
  std::vector<Direct> dcols;
  for (auto h : direct) {
    const auto t = h.cast<py::tuple>();
    int64_t n = 0, nv = 0;
    Direct d{t[0].cast<int>(), arr_ptr<int64_t>(t[1], n), t[2].is_none() ? nullptr : arr_ptr<uint8_t>(t[2], nv)};
    if (n < n_rows) throw std::invalid_argument("direct output shorter than n_rows");
    dcols.push_back(d);
  }
  struct Meta {
    int col;
    std::unordered_map<std::string, int32_t> table;
    int32_t dflt;
    int32_t* out;
  };
  std::vector<Meta> mcols;
  for (auto h : metadata) {
    const auto t = h.cast<py::tuple>();
    Meta m;
    m.col = t[0].cast<int>();
    for (auto kv : t[1].cast<py::dict>()) m.table[kv.first.cast<std::string>()] = kv.second.cast<int32_t>();
    m.dflt = t[2].cast<int32_t>();
    int64_t n = 0;
    m.out = arr_ptr<int32_t>(t[3], n);
    if (n < n_rows) throw std::invalid_argument("metadata output shorter than n_rows");
    mcols.push_back(std::move(m));
  }
  // outputs start as null / empty
  for (auto& kv : outs) {
    Out& o = kv.second;
    if (o.kind == 0) {
      for (int64_t i = 0; i < n_rows * o.length; ++i) {
        if (o.is_float) reinterpret_cast<double*>(o.data)[i] = static_cast<double>(kNull);
        else reinterpret_cast<int64_t*>(o.data)[i] = kNull;
      }
    } else if (o.kind == 2) {
      for (int64_t i = 0; i < n_rows; ++i) reinterpret_cast<int32_t*>(o.data)[i] = static_cast<int32_t>(kNull);
    }
    if (o.valid) std::memset(o.valid, 0, static_cast<size_t>(n_rows));
  }
  for (auto& d : dcols) {
    for (int64_t i = 0; i < n_rows; ++i) d.out[i] = kNull;
    if (d.valid) std::memset(d.valid, 0, static_cast<size_t>(n_rows));
  }
  for (auto& m : mcols)
    for (int64_t i = 0; i < n_rows; ++i) m.out[i] = m.dflt;
  std::unordered_map<int64_t, int64_t> fill;  // list outputs: values written so far
  for (auto& kv : outs)
    if (kv.second.kind == 1) fill[kv.first] = 0;

  for (int64_t row = 0; row < n_rows; ++row) {
    const char* p = reinterpret_cast<const char*>(base + ro[row]);
    const char* le = reinterpret_cast<const char*>(base + ro[row + 1]);
    if (le > p && le[-1] == '\n') --le;
    const char* col = p;
    for (int c = 0; col <= le; ++c) {
      const char* tab = static_cast<const char*>(std::memchr(col, '\t', le - col));
      const char* ce = tab ? tab : le;
      for (auto& d : dcols)
        if (d.col == c && ce > col) {
          d.out[row] = parse_int(col, ce);
          if (d.valid) d.valid[row] = 1;
        }
      for (auto& m : mcols)
        if (m.col == c) {
          const auto it = m.table.find(std::string(col, ce));
          m.out[row] = it == m.table.end() ? m.dflt : it->second;
        }
      if (c == feature_column) {
        const char* kvp = col;
        while (kvp < ce) {
          const char* sep = static_cast<const char*>(std::memchr(kvp, '\x02', ce - kvp));
          const char* kve = sep ? sep : ce;
          const char* eq = static_cast<const char*>(std::memchr(kvp, '\x03', kve - kvp));
          if (eq) {
            const int64_t code = parse_int(kvp, eq);
            const auto it = outs.find(code);
            if (it != outs.end()) {
              Out& o = it->second;
              const char* v = eq + 1;
              if (o.kind == 2) {
                const auto f = o.vocab->find(std::string(v, kve));
                reinterpret_cast<int32_t*>(o.data)[row] = f == o.vocab->end() ? o.dflt : f->second;
              } else if (o.kind == 0) {
                for (int k = 0; k < o.length && v <= kve; ++k) {
                  const char* comma = static_cast<const char*>(std::memchr(v, ',', kve - v));
                  const char* vend = (o.length > 1 && comma) ? comma : kve;
                  const int64_t off = row * o.length + k;
                  if (o.is_float) reinterpret_cast<double*>(o.data)[off] = parse_float(v, vend);
                  else reinterpret_cast<int64_t*>(o.data)[off] = parse_int(v, vend);
                  if (vend == kve) break;
                  v = vend + 1;
                }
              } else {
                int64_t& n = fill[code];
                while (v < kve) {
                  const char* comma = static_cast<const char*>(std::memchr(v, ',', kve - v));
                  const char* vend = comma ? comma : kve;
                  if (n >= o.cap) throw std::out_of_range("list values exceed the output capacity");
                  if (o.is_float) reinterpret_cast<double*>(o.data)[n] = parse_float(v, vend);
                  else reinterpret_cast<int64_t*>(o.data)[n] = parse_int(v, vend);
                  ++n;
                  v = comma ? comma + 1 : kve;
                }
              }
              if (o.valid) o.valid[row] = 1;
            }
          }
          if (!sep) break;
          kvp = sep + 1;
        }
      }
      if (!tab) break;
      col = tab + 1;
    }
    for (auto& kv : outs)
      if (kv.second.kind == 1) kv.second.offs[row + 1] = fill[kv.first];
  }
  py::dict counts;
  for (auto& kv : fill) counts[py::int_(kv.first)] = kv.second;
  return py::make_tuple(n_rows, counts);
}

}  // namespace flare_etl

void register_etl(py::module_& m) {
  auto e = m.def_submodule("etl", "native feature-ETL kernels (host)");
  e.def("scan_records", &flare_etl::scan_records);
  e.def("parse_rows", &flare_etl::parse_rows);
  e.def("fnv1a_lists", &flare_etl::fnv1a_lists, py::arg("values"), py::arg("offsets"), py::arg("buckets") = 0);
  e.def("fnv1a_seeded", &flare_etl::fnv1a_seeded);
  e.def("hash_bucket", &flare_etl::hash_bucket);
  e.def("bucketize", &flare_etl::bucketize);
  e.def("fixed_width", &flare_etl::fixed_width);
  e.def("pack_fids", &flare_etl::pack_fids);
  e.def("intersect_lists", &flare_etl::intersect_lists);
  e.attr("NULL_SENTINEL") = flare_etl::kNull;
}
