// Native token-batch producer: seeded document sources + BOS best-fit row packing.
//
// Packing semantics match the reference packer (src/data/bestFitPacking.ts:131-176): each row of
// capacity T+1 is filled by repeatedly refilling a buffer of `buffer_size` BOS-prefixed documents,
// taking the largest buffered document that fits the remaining space (first one on ties), or else
// cropping the shortest one (first one on ties) to the remaining space and discarding its tail.
// inputs = row[:T], targets = row[1:].
//
// Document sources:
//   * Zipf: lengths ~ Geometric(1/mean_len) (support 1,2,...), tokens ~ Zipf(s) over ids
//     [0, V-1) through a seeded rank->id permutation; BOS = V-1 is prepended by the packer.
//   * Corpus: a fixed list of documents pushed from Python, cycled with an epoch counter.
// The RNG is splitmix64-seeded xoshiro256**; Python's numpy generator is not reproduced.
//
// The hot loop releases the GIL so a Python prefetch thread can overlap it with GPU work.
#include <pybind11/numpy.h>
#include <pybind11/pybind11.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <deque>
#include <memory>
#include <stdexcept>
#include <vector>

namespace py = pybind11;

namespace {

struct Rng {
  uint64_t s[4];
  explicit Rng(uint64_t seed) {
    for (int i = 0; i < 4; ++i) {
      seed += 0x9E3779B97F4A7C15ull;
      uint64_t z = seed;
      z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
      z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
      s[i] = z ^ (z >> 31);
    }
  }
  static uint64_t rotl(uint64_t x, int k) { return (x << k) | (x >> (64 - k)); }
  uint64_t next() {
    uint64_t r = rotl(s[1] * 5, 7) * 9;
    uint64_t t = s[1] << 17;
    s[2] ^= s[0];
    s[3] ^= s[1];
    s[1] ^= s[2];
    s[0] ^= s[3];
    s[2] ^= t;
    s[3] = rotl(s[3], 45);
    return r;
  }
  double uniform() { return (next() >> 11) * (1.0 / 9007199254740992.0); }  // [0,1)
};

using Doc = std::vector<int32_t>;

struct Packer {
  int32_t bos;
  size_t buffer_size;
  int64_t epoch = 1;
  // source
  bool zipf = false;
  std::unique_ptr<Rng> rng;
  std::vector<double> cdf;
  std::vector<int32_t> perm;
  double log1mp = 0.0;  // log(1 - 1/mean_len) for geometric sampling
  int64_t max_len = 0;
  std::vector<Doc> corpus;
  size_t corpus_idx = 0;
  // buffered BOS-prefixed documents
  std::vector<Doc> buffer;

  Doc next_doc() {
    Doc d;
    if (zipf) {
      double u = rng->uniform();
      // geometric on {1,2,...}: ceil(log(1-u)/log(1-p))
      int64_t len = (int64_t)std::ceil(std::log1p(-u) / log1mp);
      if (len < 1) len = 1;
      if (max_len > 0 && len > max_len) len = max_len;
      d.resize((size_t)len + 1);
      d[0] = bos;
      for (int64_t i = 0; i < len; ++i) {
        double v = rng->uniform();
        size_t r = (size_t)(std::upper_bound(cdf.begin(), cdf.end(), v) - cdf.begin());
        if (r >= perm.size()) r = perm.size() - 1;
        d[(size_t)i + 1] = perm[r];
      }
      return d;
    }
    if (corpus.empty()) throw std::runtime_error("packer has no documents");
    if (corpus_idx >= corpus.size()) {
      corpus_idx = 0;
      epoch += 1;
    }
    return corpus[corpus_idx++];
  }

  void refill() {
    while (buffer.size() < buffer_size) buffer.push_back(next_doc());
  }

  void pack(int32_t* rows, int64_t batch, int64_t seq) {
    const int64_t cap = seq + 1;
    for (int64_t r = 0; r < batch; ++r) {
      int32_t* row = rows + r * cap;
      int64_t pos = 0;
      while (pos < cap) {
        refill();
        const int64_t rem = cap - pos;
        int64_t best = -1, best_len = 0;
        for (size_t i = 0; i < buffer.size(); ++i) {
          int64_t L = (int64_t)buffer[i].size();
          if (L <= rem && L > best_len) {
            best = (int64_t)i;
            best_len = L;
          }
        }
        if (best >= 0) {
          std::copy(buffer[best].begin(), buffer[best].end(), row + pos);
          pos += best_len;
          buffer.erase(buffer.begin() + best);
          continue;
        }
        size_t si = 0;
        for (size_t i = 1; i < buffer.size(); ++i)
          if (buffer[i].size() < buffer[si].size()) si = i;
        std::copy(buffer[si].begin(), buffer[si].begin() + rem, row + pos);
        pos = cap;
        buffer.erase(buffer.begin() + si);
      }
    }
  }
};

std::shared_ptr<Packer> new_zipf(int32_t vocab, double s, double mean_len, uint64_t seed, int64_t buffer_size,
                                 int64_t max_len) {
  if (vocab < 2) throw std::invalid_argument("vocab must be >= 2");
  auto p = std::make_shared<Packer>();
  p->bos = vocab - 1;
  p->buffer_size = (size_t)std::max<int64_t>(1, buffer_size);
  p->zipf = true;
  p->rng = std::make_unique<Rng>(seed);
  const int32_t n = vocab - 1;
  p->cdf.resize(n);
  double tot = 0.0;
  for (int32_t r = 1; r <= n; ++r) tot += std::pow((double)r, -s);
  double acc = 0.0;
  for (int32_t r = 1; r <= n; ++r) {
    acc += std::pow((double)r, -s) / tot;
    p->cdf[r - 1] = acc;
  }
  p->cdf[n - 1] = 1.0;
  p->perm.resize(n);
  for (int32_t i = 0; i < n; ++i) p->perm[i] = i;
  Rng prng(seed ^ 0x5EEDull);
  for (int32_t i = n - 1; i > 0; --i) std::swap(p->perm[i], p->perm[prng.next() % (uint64_t)(i + 1)]);
  p->log1mp = std::log1p(-1.0 / std::max(1.0, mean_len));
  if (mean_len <= 1.0) p->log1mp = -1e30;  // every document has length 1
  p->max_len = max_len;
  return p;
}

std::shared_ptr<Packer> new_corpus(int32_t bos, int64_t buffer_size, py::array_t<int32_t, py::array::c_style> toks,
                                   py::array_t<int64_t, py::array::c_style> offs, bool prefixed) {
  auto p = std::make_shared<Packer>();
  p->bos = bos;
  p->buffer_size = (size_t)std::max<int64_t>(1, buffer_size);
  auto t = toks.unchecked<1>();
  auto o = offs.unchecked<1>();
  for (py::ssize_t i = 0; i + 1 < o.shape(0); ++i) {
    Doc d;
    if (!prefixed) d.push_back(bos);
    for (int64_t j = o(i); j < o(i + 1); ++j) d.push_back(t(j));
    p->corpus.push_back(std::move(d));
  }
  if (p->corpus.empty()) throw std::invalid_argument("corpus must contain at least one document");
  return p;
}

// rows: int32 [batch, seq+1] C-contiguous, written in place; returns the epoch after packing.
int64_t pack_rows(Packer& p, py::array_t<int32_t, py::array::c_style> rows, int64_t batch, int64_t seq) {
  auto buf = rows.request();
  if (buf.ndim != 2 || buf.shape[0] != batch || buf.shape[1] != seq + 1)
    throw std::invalid_argument("rows must be int32 [batch, seq+1]");
  int32_t* ptr = static_cast<int32_t*>(buf.ptr);
  {
    py::gil_scoped_release nogil;
    p.pack(ptr, batch, seq);
  }
  return p.epoch;
}

// Split packed rows into inputs/targets written at raw addresses (e.g. pinned host tensors).
void pack_split(Packer& p, uintptr_t inputs, uintptr_t targets, int64_t batch, int64_t seq) {
  std::vector<int32_t> rows((size_t)(batch * (seq + 1)));
  {
    py::gil_scoped_release nogil;
    p.pack(rows.data(), batch, seq);
    int32_t* in = reinterpret_cast<int32_t*>(inputs);
    int32_t* tg = reinterpret_cast<int32_t*>(targets);
    for (int64_t r = 0; r < batch; ++r) {
      const int32_t* row = rows.data() + r * (seq + 1);
      std::copy(row, row + seq, in + r * seq);
      std::copy(row + 1, row + seq + 1, tg + r * seq);
    }
  }
}

}  // namespace

void register_bpe(py::module& m);

PYBIND11_MODULE(_native_data, m) {
  register_bpe(m);
  m.doc() = "native document source + BOS best-fit packer";
  py::class_<Packer, std::shared_ptr<Packer>>(m, "Packer")
      .def_property_readonly("epoch", [](const Packer& p) { return p.epoch; })
      .def_property_readonly("buffered", [](const Packer& p) { return p.buffer.size(); });
  m.def("zipf_packer", &new_zipf, py::arg("vocab"), py::arg("s"), py::arg("mean_len"), py::arg("seed"),
        py::arg("buffer_size") = 1000, py::arg("max_len") = 0);
  m.def("corpus_packer", &new_corpus, py::arg("bos"), py::arg("buffer_size"), py::arg("tokens"),
        py::arg("offsets"), py::arg("prefixed") = false);
  m.def("pack_rows", &pack_rows);
  m.def("pack_split", &pack_split);
}
