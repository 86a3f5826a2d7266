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
//   * Markov: the same lengths and the same unigram law for a document's first token; every later
//     token is, with probability p1, a successor of the previous token, with probability p2 a
//     successor of the previous two tokens (BOS standing in before the first), and otherwise a
//     fresh unigram draw. A context has `branch` successors, each a Zipf draw through the
//     permutation taken from a hash of (table seed, context, k); successor k is picked with weight
//     2^-k. The tables are never stored: a successor is recomputed from the hash when needed.
//   * Corpus: a fixed list of documents pushed from Python, cycled with an epoch counter.
// Two seeds: the table seed fixes the "language" (the rank->id permutation and the Markov
// successors) and is shared by every rank and by the validation split; the stream seed drives the
// sampling and differs per rank and split, so ranks see disjoint samples of one distribution.
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

uint64_t mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

using Doc = std::vector<int32_t>;

struct Packer {
  int32_t bos;
  size_t buffer_size;
  int64_t epoch = 1;
  // source
  bool zipf = false;
  bool markov = false;
  std::unique_ptr<Rng> rng;
  uint64_t table_seed = 0;
  double p1 = 0.0, p2 = 0.0;
  std::vector<double> branch_cdf;
  std::vector<double> cdf;
  std::vector<int32_t> perm;
  double log1mp = 0.0;  // log(1 - 1/mean_len) for geometric sampling
  int64_t max_len = 0;
  std::vector<Doc> corpus;
  size_t corpus_idx = 0;
  // buffered BOS-prefixed documents
  std::vector<Doc> buffer;

  int32_t zipf_id(double v) const {
    size_t r = (size_t)(std::upper_bound(cdf.begin(), cdf.end(), v) - cdf.begin());
    if (r >= perm.size()) r = perm.size() - 1;
    return perm[r];
  }

  // successor k of a context (contexts of order 1 are odd, of order 2 even, so they never collide)
  int32_t successor(uint64_t ctx, uint64_t k) const {
    const uint64_t h = mix64(table_seed ^ mix64(ctx * 0x9E3779B97F4A7C15ull + k));
    return zipf_id((h >> 11) * (1.0 / 9007199254740992.0));
  }

  int32_t markov_next(int32_t prev2, int32_t prev1) {
    const double r = rng->uniform();
    if (r >= p1 + p2) return zipf_id(rng->uniform());
    const uint64_t ctx = r < p1 ? (((uint64_t)(uint32_t)prev1 << 1) | 1ull)
                                : ((((uint64_t)(uint32_t)prev2 << 32) | (uint32_t)prev1) << 1);
    const double u = rng->uniform();
    size_t k = (size_t)(std::upper_bound(branch_cdf.begin(), branch_cdf.end(), u) - branch_cdf.begin());
    if (k >= branch_cdf.size()) k = branch_cdf.size() - 1;
    return successor(ctx, (uint64_t)k);
  }

  Doc next_doc() {
    Doc d;
    if (zipf || markov) {
      double u = rng->uniform();
      // geometric on {1,2,...}: ceil(log(1-u)/log(1-p))
      int64_t len = (int64_t)std::ceil(std::log1p(-u) / log1mp);
      if (len < 1) len = 1;
      if (max_len > 0 && len > max_len) len = max_len;
      d.resize((size_t)len + 1);
      d[0] = bos;
      for (int64_t i = 0; i < len; ++i)
        d[(size_t)i + 1] = (markov && i > 0) ? markov_next(d[(size_t)i - 1], d[(size_t)i]) : zipf_id(rng->uniform());
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
                                 int64_t max_len, uint64_t table_seed) {
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
  p->table_seed = table_seed;
  Rng prng(table_seed ^ 0x5EEDull);
  for (int32_t i = n - 1; i > 0; --i) std::swap(p->perm[i], p->perm[prng.next() % (uint64_t)(i + 1)]);
  p->log1mp = std::log1p(-1.0 / std::max(1.0, mean_len));
  if (mean_len <= 1.0) p->log1mp = -1e30;  // every document has length 1
  p->max_len = max_len;
  return p;
}

std::shared_ptr<Packer> new_markov(int32_t vocab, double s, double mean_len, uint64_t seed, uint64_t table_seed,
                                   double p1, double p2, int64_t branch, int64_t buffer_size, int64_t max_len) {
  if (p1 < 0 || p2 < 0 || p1 + p2 > 1.0) throw std::invalid_argument("markov: need p1, p2 >= 0 and p1 + p2 <= 1");
  if (branch < 1) throw std::invalid_argument("markov: branch must be >= 1");
  auto p = new_zipf(vocab, s, mean_len, seed, buffer_size, max_len, table_seed);
  p->zipf = false;
  p->markov = true;
  p->p1 = p1;
  p->p2 = p2;
  double tot = 0.0;
  for (int64_t k = 0; k < branch; ++k) tot += std::ldexp(1.0, -(int)k);
  double acc = 0.0;
  for (int64_t k = 0; k < branch; ++k) {
    acc += std::ldexp(1.0, -(int)k) / tot;
    p->branch_cdf.push_back(acc);
  }
  p->branch_cdf.back() = 1.0;
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

// Exact negative log-likelihood (nats) of each target of packed Markov rows under the generating
// process: a document's first token has its unigram probability, every later one the mixture
// p1 q1(x | prev) + p2 q2(x | prev2, prev) + (1 - p1 - p2) unigram(x). Targets that are BOS (document
// boundaries) get 0; they carry no bytes in bits-per-byte. The mean over non-BOS targets is the loss
// floor that a perfect model reaches.
py::array_t<double> markov_nll(const Packer& p, py::array_t<int32_t, py::array::c_style> rows, int64_t batch,
                               int64_t seq) {
  if (!p.markov) throw std::invalid_argument("markov_nll needs a markov_packer");
  auto buf = rows.request();
  if (buf.ndim != 2 || buf.shape[0] != batch || buf.shape[1] != seq + 1)
    throw std::invalid_argument("rows must be int32 [batch, seq+1]");
  const int32_t* r = static_cast<const int32_t*>(buf.ptr);
  py::array_t<double> out({batch, seq});
  double* o = out.mutable_data();
  const size_t n = p.perm.size();
  std::vector<int32_t> rank_of(n);
  for (size_t i = 0; i < n; ++i) rank_of[(size_t)p.perm[i]] = (int32_t)i;
  auto unigram = [&](int32_t x) { const int32_t k = rank_of[(size_t)x]; return p.cdf[k] - (k ? p.cdf[k - 1] : 0.0); };
  const double pu = 1.0 - p.p1 - p.p2;
  {
    py::gil_scoped_release nogil;
    for (int64_t b = 0; b < batch; ++b) {
      const int32_t* row = r + b * (seq + 1);
      // position of the current document's BOS in this row (-1: the row starts inside a document,
      // which the packer never does: every row begins with a BOS)
      int64_t bos_at = -1;
      for (int64_t t = 0; t < seq; ++t) {
        if (row[t] == p.bos) bos_at = t;
        const int32_t x = row[t + 1];
        double nll = 0.0;
        if (x != p.bos) {
          const int64_t i = t - bos_at;  // document position of x minus one
          double pr;
          if (bos_at < 0 || i == 0) {
            pr = unigram(x);
          } else {
            const int32_t prev1 = row[t];
            const int32_t prev2 = row[t - 1];
            const uint64_t c1 = ((uint64_t)(uint32_t)prev1 << 1) | 1ull;
            const uint64_t c2 = (((uint64_t)(uint32_t)prev2 << 32) | (uint32_t)prev1) << 1;
            double q1 = 0.0, q2 = 0.0, prevc = 0.0;
            for (size_t k = 0; k < p.branch_cdf.size(); ++k) {
              const double w = p.branch_cdf[k] - prevc;
              prevc = p.branch_cdf[k];
              if (p.successor(c1, k) == x) q1 += w;
              if (p.successor(c2, k) == x) q2 += w;
            }
            pr = p.p1 * q1 + p.p2 * q2 + pu * unigram(x);
          }
          nll = -std::log(pr);
        }
        o[b * seq + t] = nll;
      }
    }
  }
  return out;
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
        py::arg("buffer_size") = 1000, py::arg("max_len") = 0, py::arg("table_seed") = 0);
  m.def("markov_packer", &new_markov, py::arg("vocab"), py::arg("s"), py::arg("mean_len"), py::arg("seed"),
        py::arg("table_seed"), py::arg("p1"), py::arg("p2"), py::arg("branch"), py::arg("buffer_size") = 1000,
        py::arg("max_len") = 0);
  m.def("corpus_packer", &new_corpus, py::arg("bos"), py::arg("buffer_size"), py::arg("tokens"),
        py::arg("offsets"), py::arg("prefixed") = false);
  m.def("markov_nll", &markov_nll);
  m.def("pack_rows", &pack_rows);
  m.def("pack_split", &pack_split);
}
