// Byte-level BPE: trainer and encoder (the tokenizer of the data-preparation step).
//
// Training follows the usual byte-pair-encoding procedure over pre-tokenized chunks with counts (the
// reference trains rustbpe through scripts/prepare_wasm.ts:276-282): every chunk starts as its UTF-8
// bytes (token ids 0..255); each step merges the most frequent adjacent pair, weighted by chunk
// counts, into the next id. Ties go to the numerically smallest (left, right) pair so training is
// deterministic. Pair counts are maintained incrementally: only the chunks that contain the merged
// pair are rescanned, and a max-heap with lazy invalidation yields the next pair.
//
// Encoding applies merges by rank: within a chunk, the adjacent pair with the lowest merge rank is
// merged everywhere (left to right) until no learned pair remains. Encoded chunks are cached.
#include <pybind11/numpy.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <algorithm>
#include <cstdint>
#include <queue>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <utility>
#include <vector>

namespace py = pybind11;

namespace {

inline uint64_t key_of(int32_t a, int32_t b) { return (uint64_t(uint32_t(a)) << 32) | uint32_t(b); }

struct HeapItem {
  int64_t count;
  uint64_t key;
  bool operator<(const HeapItem& o) const {  // std::priority_queue pops the largest
    if (count != o.count) return count < o.count;
    return key > o.key;  // equal counts: the smaller pair first
  }
};

std::vector<std::pair<int32_t, int32_t>> bpe_train(const std::vector<std::string>& chunks,
                                                   const std::vector<int64_t>& counts, int64_t vocab_size) {
  if (chunks.size() != counts.size()) throw std::invalid_argument("bpe_train: chunks and counts differ in length");
  if (vocab_size < 256) throw std::invalid_argument("bpe_train: vocab_size must be at least 256");
  const size_t n = chunks.size();
  std::vector<std::vector<int32_t>> words(n);
  std::unordered_map<uint64_t, int64_t> pc;              // pair -> weighted count
  std::unordered_map<uint64_t, std::vector<int32_t>> where;  // pair -> chunks that may contain it
  for (size_t i = 0; i < n; ++i) {
    const std::string& s = chunks[i];
    auto& w = words[i];
    w.reserve(s.size());
    for (unsigned char ch : s) w.push_back(ch);
    for (size_t j = 0; j + 1 < w.size(); ++j) {
      const uint64_t k = key_of(w[j], w[j + 1]);
      pc[k] += counts[i];
      auto& v = where[k];
      if (v.empty() || v.back() != (int32_t)i) v.push_back((int32_t)i);
    }
  }
  std::priority_queue<HeapItem> heap;
  for (const auto& kv : pc)
    if (kv.second > 0) heap.push({kv.second, kv.first});

  std::vector<std::pair<int32_t, int32_t>> merges;
  const int64_t num_merges = vocab_size - 256;
  merges.reserve((size_t)num_merges);
  std::unordered_map<uint64_t, int64_t> delta;
  std::vector<int32_t> nw;
  while ((int64_t)merges.size() < num_merges && !heap.empty()) {
    const HeapItem top = heap.top();
    heap.pop();
    auto it = pc.find(top.key);
    if (it == pc.end() || it->second != top.count || top.count <= 0) continue;  // stale entry
    const int32_t a = int32_t(top.key >> 32), b = int32_t(top.key & 0xffffffffu);
    const int32_t id = 256 + (int32_t)merges.size();
    merges.emplace_back(a, b);
    std::vector<int32_t> cand;
    cand.swap(where[top.key]);
    delta.clear();
    for (int32_t ci : cand) {
      auto& w = words[ci];
      bool has = false;
      for (size_t j = 0; j + 1 < w.size(); ++j)
        if (w[j] == a && w[j + 1] == b) {
          has = true;
          break;
        }
      if (!has) continue;
      const int64_t c = counts[ci];
      for (size_t j = 0; j + 1 < w.size(); ++j) delta[key_of(w[j], w[j + 1])] -= c;
      nw.clear();
      for (size_t j = 0; j < w.size();) {
        if (j + 1 < w.size() && w[j] == a && w[j + 1] == b) {
          nw.push_back(id);
          j += 2;
        } else {
          nw.push_back(w[j]);
          ++j;
        }
      }
      w.swap(nw);
      for (size_t j = 0; j + 1 < w.size(); ++j) {
        const uint64_t k = key_of(w[j], w[j + 1]);
        delta[k] += c;
        if (w[j] == id || w[j + 1] == id) {
          auto& v = where[k];
          if (v.empty() || v.back() != ci) v.push_back(ci);
        }
      }
    }
    for (const auto& kv : delta) {
      if (kv.second == 0) continue;
      int64_t& cnt = pc[kv.first];
      cnt += kv.second;
      if (cnt > 0) heap.push({cnt, kv.first});
    }
    pc.erase(top.key);
  }
  return merges;
}

class BPEEncoder {
 public:
  explicit BPEEncoder(const std::vector<std::pair<int32_t, int32_t>>& merges) : merges_(merges) {
    rank_.reserve(merges.size() * 2);
    for (size_t i = 0; i < merges.size(); ++i) rank_[key_of(merges[i].first, merges[i].second)] = (int32_t)i;
  }

  const std::vector<int32_t>& encode_chunk(const std::string& s) {
    auto it = cache_.find(s);
    if (it != cache_.end()) return it->second;
    std::vector<int32_t> w;
    w.reserve(s.size());
    for (unsigned char ch : s) w.push_back(ch);
    std::vector<int32_t> nw;
    while (w.size() > 1) {
      int32_t best = INT32_MAX;
      for (size_t j = 0; j + 1 < w.size(); ++j) {
        auto r = rank_.find(key_of(w[j], w[j + 1]));
        if (r != rank_.end() && r->second < best) best = r->second;
      }
      if (best == INT32_MAX) break;
      const int32_t a = merges_[best].first, b = merges_[best].second, id = 256 + best;
      nw.clear();
      for (size_t j = 0; j < w.size();) {
        if (j + 1 < w.size() && w[j] == a && w[j + 1] == b) {
          nw.push_back(id);
          j += 2;
        } else {
          nw.push_back(w[j]);
          ++j;
        }
      }
      w.swap(nw);
    }
    if (cache_.size() > (1u << 22)) cache_.clear();
    return cache_.emplace(s, std::move(w)).first->second;
  }

  // Encodes pre-tokenized chunks of one document into one int32 array.
  py::array_t<int32_t> encode_chunks(const std::vector<std::string>& chunks) {
    std::vector<int32_t> out;
    for (const auto& c : chunks) {
      const auto& ids = encode_chunk(c);
      out.insert(out.end(), ids.begin(), ids.end());
    }
    py::array_t<int32_t> arr((py::ssize_t)out.size());
    std::copy(out.begin(), out.end(), arr.mutable_data());
    return arr;
  }

 private:
  std::vector<std::pair<int32_t, int32_t>> merges_;
  std::unordered_map<uint64_t, int32_t> rank_;
  std::unordered_map<std::string, std::vector<int32_t>> cache_;
};

}  // namespace

void register_bpe(py::module& m) {
  m.def("bpe_train", &bpe_train, py::arg("chunks"), py::arg("counts"), py::arg("vocab_size"),
        "Train byte-level BPE merges over (chunk, count) pairs; returns [(left, right)] in merge order.");
  py::class_<BPEEncoder>(m, "BPEEncoder")
      .def(py::init<const std::vector<std::pair<int32_t, int32_t>>&>(), py::arg("merges"))
      .def("encode_chunks", &BPEEncoder::encode_chunks, py::arg("chunks"));
}
