// Host key -> slot map for hash-keyed tables (insert on first sight, LFU eviction).
//
// A table of `capacity` slots holds rows for arbitrary int64 keys.  A
// training lookup (`insert` true) gives every key of the batch a slot: known
// keys keep theirs; new keys take a free slot or, when none is left, the slot
// of a key that the batch does not use, chosen least frequently used first
// (ties: least recently used, then lowest slot), once per batch with a
// partial selection over the slots.  Every touched key's use count and last
// batch are updated.  The caller re-initialises the rows of the slots it is
// told are new.  An evaluation lookup (`insert` false) maps unknown keys to
// -1 and changes nothing.
//
// Reference behaviour: `lookup_or_insert` with auto-insert and an LFU score
// policy of the reference's external sparse store
// (src/flare/runtime/fluxway/workers/dynamic_embedding.py:251-302, 362-397),
// whose implementation is not in the reference tree.
#include <torch/extension.h>

#include <algorithm>
#include <cstdint>
#include <stdexcept>
#include <tuple>
#include <unordered_map>
#include <unordered_set>
#include <vector>

namespace py = pybind11;

namespace flare_dyn {

class DynamicKeyMap {
 public:
  explicit DynamicKeyMap(int64_t capacity) : cap_(capacity) {
    if (capacity < 1) throw std::invalid_argument("capacity must be positive");
    slot_key_.assign(static_cast<size_t>(capacity), -1);
    uses_.assign(static_cast<size_t>(capacity), 0);
    last_.assign(static_cast<size_t>(capacity), 0);
    free_.reserve(static_cast<size_t>(capacity));
    for (int64_t s = capacity - 1; s >= 0; --s) free_.push_back(s);
    map_.reserve(static_cast<size_t>(capacity) * 2);
  }

  // (slots [n] int64, new_slots [m] int64, evicted_keys [e] int64)
  py::tuple lookup(torch::Tensor keys, bool insert) {
    TORCH_CHECK(!keys.is_cuda() && keys.scalar_type() == torch::kInt64 && keys.is_contiguous() && keys.dim() == 1,
                "keys: contiguous int64 CPU vector");
    const int64_t n = keys.numel();
    const int64_t* k = keys.data_ptr<int64_t>();
    auto slots = torch::empty({n}, torch::kInt64);
    int64_t* out = slots.data_ptr<int64_t>();
    ++batch_;
    std::vector<int64_t> fresh;  // distinct new keys, first-seen order
    std::unordered_map<int64_t, int64_t> fresh_idx;
    for (int64_t i = 0; i < n; ++i) {
      auto it = map_.find(k[i]);
      if (it != map_.end()) {
        out[i] = it->second;
        if (insert) touch(it->second);
      } else if (!insert || k[i] < 0) {
        out[i] = -1;
      } else {
        out[i] = -2;  // resolved below
        if (fresh_idx.emplace(k[i], static_cast<int64_t>(fresh.size())).second) fresh.push_back(k[i]);
      }
    }
    std::vector<int64_t> new_slots, evicted;
    if (!fresh.empty()) {
      const int64_t need = static_cast<int64_t>(fresh.size());
      std::vector<int64_t> got;
      while (!free_.empty() && static_cast<int64_t>(got.size()) < need) {
        got.push_back(free_.back());
        free_.pop_back();
      }
      if (static_cast<int64_t>(got.size()) < need) {
        // victims: occupied slots this batch does not use, least frequently (then least recently) used first
        std::vector<int64_t> cand;
        for (int64_t s = 0; s < cap_; ++s)
          if (slot_key_[s] >= 0 && last_[s] != batch_) cand.push_back(s);
        const int64_t want = need - static_cast<int64_t>(got.size());
        if (static_cast<int64_t>(cand.size()) < want) {
          for (int64_t s : got) free_.push_back(s);
          throw std::runtime_error("dynamic table full: " + std::to_string(need) + " new keys, " +
                                   std::to_string(cand.size() + got.size()) + " slots available this batch");
        }
        auto less = [&](int64_t a, int64_t b) {
          return std::make_tuple(uses_[a], last_[a], a) < std::make_tuple(uses_[b], last_[b], b);
        };
        std::nth_element(cand.begin(), cand.begin() + (want - 1), cand.end(), less);
        std::sort(cand.begin(), cand.begin() + want, less);
        for (int64_t i = 0; i < want; ++i) {
          const int64_t s = cand[i];
          evicted.push_back(slot_key_[s]);
          map_.erase(slot_key_[s]);
          slot_key_[s] = -1;
          got.push_back(s);
        }
      }
      for (int64_t j = 0; j < need; ++j) {
        const int64_t s = got[j];
        slot_key_[s] = fresh[j];
        map_[fresh[j]] = s;
        uses_[s] = 0;
        touch(s);
        new_slots.push_back(s);
      }
      std::unordered_set<int64_t> counted;  // the insert counted a new key's first occurrence
      for (int64_t i = 0; i < n; ++i)
        if (out[i] == -2) {
          const int64_t s = map_[k[i]];
          out[i] = s;
          if (!counted.insert(k[i]).second) touch(s);  // later occurrences count as uses
        }
    }
    auto vec = [](const std::vector<int64_t>& v) {
      auto t = torch::empty({static_cast<int64_t>(v.size())}, torch::kInt64);
      std::copy(v.begin(), v.end(), t.data_ptr<int64_t>());
      return t;
    };
    return py::make_tuple(slots, vec(new_slots), vec(evicted));
  }

  int64_t size() const { return static_cast<int64_t>(map_.size()); }
  int64_t capacity() const { return cap_; }

  // (keys, slots, uses, last-use batch) of every occupied slot, by slot
  py::tuple items() const {
    std::vector<int64_t> ks, ss, us, ls;
    for (int64_t s = 0; s < cap_; ++s)
      if (slot_key_[s] >= 0) {
        ks.push_back(slot_key_[s]);
        ss.push_back(s);
        us.push_back(static_cast<int64_t>(uses_[s]));
        ls.push_back(static_cast<int64_t>(last_[s]));
      }
    auto vec = [](const std::vector<int64_t>& v) {
      auto t = torch::empty({static_cast<int64_t>(v.size())}, torch::kInt64);
      std::copy(v.begin(), v.end(), t.data_ptr<int64_t>());
      return t;
    };
    return py::make_tuple(vec(ks), vec(ss), vec(us), vec(ls));
  }

  // rebuild from items() output (restore); the batch counter resumes after the latest last-use
  void load(torch::Tensor keys, torch::Tensor slots, torch::Tensor uses, torch::Tensor last) {
    TORCH_CHECK(keys.numel() == slots.numel() && keys.numel() == uses.numel() && keys.numel() == last.numel(),
                "items must align");
    auto k = keys.to(torch::kInt64).contiguous(), s = slots.to(torch::kInt64).contiguous(),
         u = uses.to(torch::kInt64).contiguous(), l = last.to(torch::kInt64).contiguous();
    std::fill(slot_key_.begin(), slot_key_.end(), -1);
    std::fill(uses_.begin(), uses_.end(), 0);
    std::fill(last_.begin(), last_.end(), 0);
    map_.clear();
    for (int64_t i = 0; i < k.numel(); ++i) {
      const int64_t sl = s.data_ptr<int64_t>()[i];
      TORCH_CHECK(sl >= 0 && sl < cap_ && slot_key_[sl] < 0, "bad or repeated slot ", sl);
      slot_key_[sl] = k.data_ptr<int64_t>()[i];
      uses_[sl] = static_cast<uint64_t>(u.data_ptr<int64_t>()[i]);
      last_[sl] = static_cast<uint64_t>(l.data_ptr<int64_t>()[i]);
      batch_ = std::max(batch_, last_[sl]);
      map_[slot_key_[sl]] = sl;
    }
    free_.clear();
    for (int64_t sl = cap_ - 1; sl >= 0; --sl)
      if (slot_key_[sl] < 0) free_.push_back(sl);
  }

 private:
  void touch(int64_t s) {
    ++uses_[s];
    last_[s] = batch_;
  }

  int64_t cap_;
  uint64_t batch_ = 0;
  std::vector<int64_t> slot_key_;
  std::vector<uint64_t> uses_, last_;
  std::vector<int64_t> free_;
  std::unordered_map<int64_t, int64_t> map_;
};

}  // namespace flare_dyn

void register_dyn_map(py::module_& m) {
  py::class_<flare_dyn::DynamicKeyMap>(m, "DynamicKeyMap")
      .def(py::init<int64_t>(), py::arg("capacity"))
      .def("lookup", &flare_dyn::DynamicKeyMap::lookup, py::arg("keys"), py::arg("insert") = true)
      .def("size", &flare_dyn::DynamicKeyMap::size)
      .def("capacity", &flare_dyn::DynamicKeyMap::capacity)
      .def("items", &flare_dyn::DynamicKeyMap::items)
      .def("load", &flare_dyn::DynamicKeyMap::load);
}
