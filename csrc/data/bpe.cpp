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

// ---------------------------------------------------------------------------------------- native pre-split
// The GPT-4 split pattern
//   '(?i:[sdmt]|ll|ve|re) | [^\r\n\p{L}\p{N}]?+\p{L}+ | \p{N}{1,2} | ?[^\s\p{L}\p{N}]++[\r\n]* |
//   \s*[\r\n] | \s+(?!\S) | \s+
// restated as a scanner over code points. A class table gives each code point one of: letter (\p{L}),
// number (\p{N}), newline (\r \n), other whitespace (\s), other, or "bad" (not handled here: the caller
// uses the regex); its high bits name the contraction letter (s d m t l v e r) that the code point matches
// case-insensitively. By default the table covers printable ASCII plus the ASCII whitespace; the Python
// side installs a full table computed with the regex engine itself (set_split_table). At each position
// the alternatives are tried in the pattern's order and the first match is taken, as a regex engine does.
enum : uint8_t { C_LET, C_DIG, C_NL, C_WS, C_OTH, C_BAD };
constexpr uint32_t kMaxCp = 0x110000;

std::vector<uint8_t>& split_table() {
  static std::vector<uint8_t> t = [] {
    std::vector<uint8_t> v(128, C_BAD);
    for (int i = 0x20; i < 0x7F; ++i) v[i] = C_OTH;
    for (int i = '0'; i <= '9'; ++i) v[i] = C_DIG;
    const char* fold = "sdmtlver";
    for (int i = 0; i < 26; ++i) {
      uint8_t id = 0;
      for (int k = 0; k < 8; ++k)
        if ('a' + i == fold[k]) id = (uint8_t)(k + 1);
      v['a' + i] = v['A' + i] = (uint8_t)(C_LET | (id << 3));
    }
    v[' '] = v['\t'] = v[0x0B] = v[0x0C] = C_WS;
    v['\n'] = v['\r'] = C_NL;
    return v;
  }();
  return t;
}

void set_split_table(py::array_t<uint8_t, py::array::c_style> table) {
  if (table.ndim() != 1 || table.shape(0) != (py::ssize_t)kMaxCp)
    throw std::invalid_argument("split table must be uint8[0x110000]");
  auto& t = split_table();
  if (t.size() == kMaxCp) return;  // installed once; readers may run without the GIL, so never replaced
  t.assign(table.data(), table.data() + kMaxCp);
}

// UTF-8 -> per-code-point table entries and byte offsets (offs has one extra entry: the end).
bool decode_classes(const std::string& s, std::vector<uint8_t>& cls, std::vector<size_t>& offs) {
  const auto& t = split_table();
  const unsigned char* p = reinterpret_cast<const unsigned char*>(s.data());
  const size_t n = s.size();
  cls.clear();
  offs.clear();
  for (size_t i = 0; i < n;) {
    uint32_t cp;
    size_t len;
    const unsigned char c = p[i];
    if (c < 0x80) {
      cp = c;
      len = 1;
    } else if ((c >> 5) == 6 && i + 1 < n) {
      cp = ((c & 0x1F) << 6) | (p[i + 1] & 0x3F);
      len = 2;
    } else if ((c >> 4) == 14 && i + 2 < n) {
      cp = ((c & 0x0F) << 12) | ((p[i + 1] & 0x3F) << 6) | (p[i + 2] & 0x3F);
      len = 3;
    } else if ((c >> 3) == 30 && i + 3 < n) {
      cp = ((c & 0x07) << 18) | ((p[i + 1] & 0x3F) << 12) | ((p[i + 2] & 0x3F) << 6) | (p[i + 3] & 0x3F);
      len = 4;
    } else {
      return false;
    }
    const uint8_t k = cp < t.size() ? t[cp] : (uint8_t)C_BAD;
    if ((k & 7) == C_BAD) return false;
    cls.push_back(k);
    offs.push_back(i);
    i += len;
  }
  offs.push_back(n);
  return true;
}

// Appends [begin, end) byte ranges of the chunks of s; false if s holds a code point the table leaves out.
bool native_split(const std::string& s, std::vector<std::pair<size_t, size_t>>& out) {
  thread_local std::vector<uint8_t> kl;
  thread_local std::vector<size_t> off;
  if (!decode_classes(s, kl, off)) return false;
  const size_t n = kl.size();
  auto cls = [&](size_t i) -> uint8_t { return i < n ? (uint8_t)(kl[i] & 7) : (uint8_t)C_BAD; };
  auto letter = [&](size_t i) -> uint8_t { return i < n ? (uint8_t)(kl[i] >> 3) : (uint8_t)0; };
  auto is_ws = [&](size_t i) { const uint8_t k = cls(i); return k == C_WS || k == C_NL; };
  auto emit = [&](size_t a, size_t b) { out.emplace_back(off[a], off[b]); };
  enum : uint8_t { L_S = 1, L_D, L_M, L_T, L_L, L_V, L_E, L_R };
  size_t i = 0;
  while (i < n) {
    const uint8_t k = cls(i);
    // 1. contractions (the apostrophe is U+0027 only)
    if (s[off[i]] == '\'' && off[i + 1] - off[i] == 1) {
      const uint8_t a = letter(i + 1), b = letter(i + 2);
      if (a == L_S || a == L_D || a == L_M || a == L_T) {
        emit(i, i + 2);
        i += 2;
        continue;
      }
      if ((a == L_L && b == L_L) || (a == L_V && b == L_E) || (a == L_R && b == L_E)) {
        emit(i, i + 3);
        i += 3;
        continue;
      }
    }
    // 2. an optional non-letter, non-number, non-newline code point (possessive), then letters
    if (k == C_LET || ((k == C_WS || k == C_OTH) && cls(i + 1) == C_LET)) {
      size_t j = (k == C_LET) ? i : i + 1;
      while (cls(j) == C_LET) ++j;
      emit(i, j);
      i = j;
      continue;
    }
    // 3. one or two numbers
    if (k == C_DIG) {
      const size_t j = (cls(i + 1) == C_DIG) ? i + 2 : i + 1;
      emit(i, j);
      i = j;
      continue;
    }
    // 4. an optional space (U+0020), others (possessive), then newlines
    if (k == C_OTH || (s[off[i]] == ' ' && cls(i + 1) == C_OTH)) {
      size_t j = (k == C_OTH) ? i : i + 1;
      while (cls(j) == C_OTH) ++j;
      while (cls(j) == C_NL) ++j;
      emit(i, j);
      i = j;
      continue;
    }
    // whitespace from here on: the run [i, r)
    size_t r = i;
    while (r < n && is_ws(r)) ++r;
    // 5. whitespace up to and including its last newline
    size_t last_nl = n;
    for (size_t j = i; j < r; ++j)
      if (cls(j) == C_NL) last_nl = j;
    if (last_nl != n) {
      emit(i, last_nl + 1);
      i = last_nl + 1;
      continue;
    }
    // 6. whitespace not followed by a non-space: all of it at the end of the text, else all but its last
    if (r == n) {
      emit(i, r);
      i = r;
      continue;
    }
    if (r - i >= 2) {
      emit(i, r - 1);
      i = r - 1;
      continue;
    }
    // 7. the rest of the whitespace
    emit(i, r);
    i = r;
  }
  return true;
}

py::object split_text(const std::string& s) {
  std::vector<std::pair<size_t, size_t>> sp;
  if (!native_split(s, sp)) return py::none();
  py::list out;
  for (const auto& [a, b] : sp) out.append(py::str(s.data() + a, b - a));
  return out;
}

// Chunk counts of many texts: (chunks as UTF-8 bytes, counts, indices of texts the table cannot split,
// which the caller splits with the regex). Chunks are listed in first-seen order.
py::tuple count_chunks_native(const std::vector<std::string>& texts) {
  std::unordered_map<std::string, int64_t> idx;
  std::vector<std::string> keys;
  std::vector<int64_t> counts;
  std::vector<int64_t> rest;
  {
    py::gil_scoped_release nogil;
    std::vector<std::pair<size_t, size_t>> sp;
    for (size_t t = 0; t < texts.size(); ++t) {
      sp.clear();
      if (!native_split(texts[t], sp)) {
        rest.push_back((int64_t)t);
        continue;
      }
      for (const auto& [a, b] : sp) {
        std::string c = texts[t].substr(a, b - a);
        auto it = idx.find(c);
        if (it == idx.end()) {
          idx.emplace(c, (int64_t)keys.size());
          keys.push_back(std::move(c));
          counts.push_back(1);
        } else {
          counts[it->second] += 1;
        }
      }
    }
  }
  py::list ks;
  for (const auto& k : keys) ks.append(py::bytes(k));
  return py::make_tuple(ks, counts, rest);
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

  // Splits and encodes one document when the split table covers it; None otherwise. The work runs
  // without the GIL, so threads with an encoder each encode in parallel (one encoder is not thread-safe:
  // its chunk cache is shared by its calls).
  py::object encode_text(const std::string& text) {
    std::vector<int32_t> out;
    bool ok;
    {
      py::gil_scoped_release nogil;
      std::vector<std::pair<size_t, size_t>> sp;
      ok = native_split(text, sp);
      if (ok) {
        out.reserve(text.size() / 3 + 1);
        std::string c;
        for (const auto& [a, b] : sp) {
          c.assign(text.data() + a, b - a);
          const auto& ids = encode_chunk(c);
          out.insert(out.end(), ids.begin(), ids.end());
        }
      }
    }
    if (!ok) return py::none();
    py::array_t<int32_t> arr((py::ssize_t)out.size());
    std::copy(out.begin(), out.end(), arr.mutable_data());
    return std::move(arr);
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
      .def("encode_chunks", &BPEEncoder::encode_chunks, py::arg("chunks"))
      .def("encode_text", &BPEEncoder::encode_text, py::arg("text"));
  m.def("split_text", &split_text, py::arg("text"),
        "GPT-4 pattern chunks of a text, or None when the split table does not cover it.");
  m.def("count_chunks_native", &count_chunks_native, py::arg("texts"));
  m.def("set_split_table", &set_split_table, py::arg("table"),
        "Installs the per-code-point class table (uint8[0x110000]: class | contraction letter << 3).");
}
