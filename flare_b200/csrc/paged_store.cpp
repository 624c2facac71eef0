// Paged row store with a memory limit and disk spill (host C++): the storage
// tier for tables larger than host memory.
//
// A table of `rows` records of `width` fp32 values (an embedding row followed
// by its optimizer state) is cut into pages of `rows_per_page` records.  A
// page comes into memory on first touch (initialised: the first `init_cols`
// values of a record uniform in [-init_scale, init_scale] from a counter-based
// hash of (seed, row, col), the rest zero) or from the spill file.  When the
// resident pages would exceed `memory_limit_bytes`, the least recently used
// page leaves memory; a page that changed since it was loaded is written to
// its slot in the spill file first (slots are assigned on first spill and
// reused), and the spill file may not grow past `max_spill_bytes` (<= 0: no
// limit).  A page that never changed is dropped and re-initialised on return.
//
// Reads and writes go record by record, so a gather or scatter of any number
// of rows needs only one resident page at a time.  Calls are serialised by the
// caller (the Python wrapper holds the GIL); no internal threads.
//
// Reference behaviour: the AutoStorage memory limit, spill directory and
// maximum spill bytes of the reference's sparse store options
// (src/flare/runtime/sparse_storage.py:8-47; entries per page 4096 / 8192 /
// 16384), whose store is external and was not inspected.
#include <torch/extension.h>

#include <fcntl.h>
#include <unistd.h>

#include <cerrno>
#include <cstdint>
#include <cstring>
#include <list>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

namespace py = pybind11;

namespace flare_store {

// splitmix64 finaliser (Steele, Lea and Flood 2014): a bijective 64-bit mix
inline uint64_t mix64(uint64_t z) {
  z += 0x9e3779b97f4a7c15ull;
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  return z ^ (z >> 31);
}

class PagedRowStore {
 public:
  PagedRowStore(int64_t rows, int64_t width, int64_t rows_per_page, int64_t memory_limit_bytes,
                std::string spill_path, int64_t max_spill_bytes, int64_t init_cols, double init_scale,
                int64_t seed)
      : rows_(rows), width_(width), rpp_(rows_per_page), init_cols_(init_cols), init_scale_(init_scale),
        seed_(static_cast<uint64_t>(seed)), spill_path_(std::move(spill_path)), max_spill_(max_spill_bytes) {
    if (rows < 1 || width < 1 || rows_per_page < 1) throw std::invalid_argument("rows, width, rows_per_page >= 1");
    if (init_cols < 0 || init_cols > width) throw std::invalid_argument("init_cols must be in [0, width]");
    page_bytes_ = rpp_ * width_ * static_cast<int64_t>(sizeof(float));
    const int64_t npages = (rows_ + rpp_ - 1) / rpp_;
    pages_.resize(static_cast<size_t>(npages));
    max_resident_ = memory_limit_bytes <= 0 ? npages : std::max<int64_t>(1, memory_limit_bytes / page_bytes_);
    if (max_resident_ < npages && spill_path_.empty())
      throw std::invalid_argument("a memory limit below the table size needs a spill path");
  }
  ~PagedRowStore() {
    if (fd_ >= 0) {
      ::close(fd_);
      ::unlink(spill_path_.c_str());
    }
  }

  void gather(torch::Tensor ids, torch::Tensor out) {
    check_ids(ids);
    TORCH_CHECK(out.is_contiguous() && out.scalar_type() == torch::kFloat32 && out.dim() == 2 &&
                    out.size(0) == ids.numel() && out.size(1) == width_,
                "out must be a contiguous float32 [n, width] tensor");
    const int64_t* id = ids.data_ptr<int64_t>();
    float* dst = out.data_ptr<float>();
    for (int64_t i = 0; i < ids.numel(); ++i)
      std::memcpy(dst + i * width_, record(id[i], false), static_cast<size_t>(width_) * sizeof(float));
  }

  void scatter(torch::Tensor ids, torch::Tensor src) {
    check_ids(ids);
    TORCH_CHECK(src.is_contiguous() && src.scalar_type() == torch::kFloat32 && src.dim() == 2 &&
                    src.size(0) == ids.numel() && src.size(1) == width_,
                "src must be a contiguous float32 [n, width] tensor");
    const int64_t* id = ids.data_ptr<int64_t>();
    const float* s = src.data_ptr<float>();
    for (int64_t i = 0; i < ids.numel(); ++i)
      std::memcpy(record(id[i], true), s + i * width_, static_cast<size_t>(width_) * sizeof(float));
  }

  py::dict stats() const {
    py::dict d;
    d["pages"] = static_cast<int64_t>(pages_.size());
    d["resident_pages"] = resident_;
    d["max_resident_pages"] = max_resident_;
    d["page_bytes"] = page_bytes_;
    d["resident_bytes"] = resident_ * page_bytes_;
    d["spill_slots"] = slots_;
    d["spill_bytes"] = slots_ * page_bytes_;
    d["faults"] = faults_;
    d["loads_from_spill"] = loads_;
    d["evictions"] = evictions_;
    d["writebacks"] = writebacks_;
    return d;
  }

 private:
  struct Page {
    std::unique_ptr<float[]> mem;
    int64_t slot = -1;  // spill file slot (-1: never spilled)
    bool dirty = false;
    std::list<int64_t>::iterator lru;
  };

  void check_ids(const torch::Tensor& ids) const {
    TORCH_CHECK(ids.device().is_cpu() && ids.is_contiguous() && ids.scalar_type() == torch::kInt64 && ids.dim() == 1,
                "ids must be a contiguous int64 CPU vector");
    const int64_t* id = ids.data_ptr<int64_t>();
    for (int64_t i = 0; i < ids.numel(); ++i)
      TORCH_CHECK(id[i] >= 0 && id[i] < rows_, "row id ", id[i], " outside [0, ", rows_, ")");
  }

  float* record(int64_t row, bool write) {
    const int64_t p = row / rpp_;
    Page& pg = pages_[static_cast<size_t>(p)];
    if (!pg.mem) load(p);
    else lru_.splice(lru_.end(), lru_, pg.lru);  // most recently used at the back
    if (write) pg.dirty = true;
    return pg.mem.get() + (row - p * rpp_) * width_;
  }

  void load(int64_t p) {
    while (resident_ >= max_resident_) evict();
    Page& pg = pages_[static_cast<size_t>(p)];
    pg.mem.reset(new float[static_cast<size_t>(rpp_ * width_)]);
    ++faults_;
    if (pg.slot >= 0) {
      io(false, pg.mem.get(), pg.slot);
      ++loads_;
    } else {
      init_page(p, pg.mem.get());
    }
    pg.dirty = false;
    pg.lru = lru_.insert(lru_.end(), p);
    ++resident_;
  }

  // A clean page leaves memory without a write: its spill slot (or, if it never changed, its
  // deterministic initial values) already holds it.  The limit is checked before any state changes.
  void evict() {
    const int64_t p = lru_.front();
    Page& pg = pages_[static_cast<size_t>(p)];
    if (pg.dirty) {
      if (pg.slot < 0) {
        if (max_spill_ > 0 && (slots_ + 1) * page_bytes_ > max_spill_)
          throw std::runtime_error("spill file would exceed max_spill_bytes (" + std::to_string(max_spill_) + ")");
        pg.slot = slots_++;
      }
      io(true, pg.mem.get(), pg.slot);
      ++writebacks_;
    }
    lru_.pop_front();
    pg.mem.reset();
    pg.dirty = false;
    --resident_;
    ++evictions_;
  }

  void io(bool write, float* buf, int64_t slot) {
    if (fd_ < 0) {
      fd_ = ::open(spill_path_.c_str(), O_RDWR | O_CREAT | O_TRUNC, 0600);
      if (fd_ < 0) throw std::runtime_error("cannot open spill file " + spill_path_ + ": " + std::strerror(errno));
    }
    char* b = reinterpret_cast<char*>(buf);
    int64_t done = 0;
    const off_t base = static_cast<off_t>(slot * page_bytes_);
    while (done < page_bytes_) {
      const ssize_t r = write ? ::pwrite(fd_, b + done, static_cast<size_t>(page_bytes_ - done), base + done)
                              : ::pread(fd_, b + done, static_cast<size_t>(page_bytes_ - done), base + done);
      if (r < 0 && errno == EINTR) continue;
      if (r <= 0) throw std::runtime_error(std::string("spill file ") + (write ? "write" : "read") + " failed: " +
                                           (r < 0 ? std::strerror(errno) : "short read"));
      done += r;
    }
  }

  void init_page(int64_t p, float* mem) const {
    std::memset(mem, 0, static_cast<size_t>(page_bytes_));
    const int64_t r0 = p * rpp_, r1 = std::min(rows_, r0 + rpp_);
    for (int64_t r = r0; r < r1; ++r) {
      float* rec = mem + (r - r0) * width_;
      for (int64_t c = 0; c < init_cols_; ++c) {
        const uint64_t h = mix64(seed_ ^ mix64(static_cast<uint64_t>(r) * static_cast<uint64_t>(init_cols_) +
                                               static_cast<uint64_t>(c)));
        const double u = static_cast<double>(h >> 40) * (1.0 / 16777216.0);  // 24 bits -> [0, 1)
        rec[c] = static_cast<float>((2.0 * u - 1.0) * init_scale_);
      }
    }
  }

  int64_t rows_, width_, rpp_, init_cols_;
  double init_scale_;
  uint64_t seed_;
  std::string spill_path_;
  int64_t max_spill_;
  int64_t page_bytes_ = 0, max_resident_ = 0, resident_ = 0, slots_ = 0;
  int64_t faults_ = 0, loads_ = 0, evictions_ = 0, writebacks_ = 0;
  int fd_ = -1;
  std::vector<Page> pages_;
  std::list<int64_t> lru_;
};

}  // namespace flare_store

void register_paged_store(py::module_& m) {
  py::class_<flare_store::PagedRowStore>(m, "PagedRowStore")
      .def(py::init<int64_t, int64_t, int64_t, int64_t, std::string, int64_t, int64_t, double, int64_t>(),
           py::arg("rows"), py::arg("width"), py::arg("rows_per_page"), py::arg("memory_limit_bytes"),
           py::arg("spill_path"), py::arg("max_spill_bytes"), py::arg("init_cols"), py::arg("init_scale"),
           py::arg("seed"))
      .def("gather", &flare_store::PagedRowStore::gather)
      .def("scatter", &flare_store::PagedRowStore::scatter)
      .def("stats", &flare_store::PagedRowStore::stats);
}
