// Host-side native runtime of nexttransformer_b200 (CPU, C++17, pybind11):
//
//  * BestFitPacker - BOS best-fit packing of tokenised documents into fixed-length rows: for
//    each row, repeatedly take the longest buffered document that still fits the remaining
//    space (ties: the earliest), and when none fits, crop the shortest one.  Same algorithm and
//    tie order as nanochat's BOS best-fit loader; the O(buffer) scan per pick runs here instead
//    of in Python.  State (the buffer, in order) round-trips through Python for checkpoints.
//  * train_bpe - byte-pair-encoding merge learning over pre-split words with counts: the most
//    frequent adjacent pair is merged repeatedly (ties: the smallest pair id), pair counts are
//    maintained incrementally through an inverted index from pairs to words.
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <algorithm>
#include <cstdint>
#include <map>
#include <queue>
#include <stdexcept>
#include <unordered_map>
#include <unordered_set>
#include <vector>

namespace py = pybind11;

class BestFitPacker {
 public:
  void add(const std::vector<std::vector<int32_t>>& docs) {
    for (const auto& d : docs) buf_.push_back(d);
  }
  size_t size() const { return buf_.size(); }

  // Pops the document placed next into a row with `remaining` free slots (cropped to fit).
  std::vector<int32_t> pick(int64_t remaining) {
    if (buf_.empty()) throw std::runtime_error("best-fit buffer is empty");
    int64_t best = -1, best_len = 0;
    for (size_t i = 0; i < buf_.size(); ++i) {
      const int64_t n = static_cast<int64_t>(buf_[i].size());
      if (best_len < n && n <= remaining) {
        best = static_cast<int64_t>(i);
        best_len = n;
      }
    }
    if (best < 0) {  // nothing fits: the shortest document, cropped
      size_t s = 0;
      for (size_t i = 1; i < buf_.size(); ++i)
        if (buf_[i].size() < buf_[s].size()) s = i;
      best = static_cast<int64_t>(s);
    }
    std::vector<int32_t> doc = std::move(buf_[best]);
    buf_.erase(buf_.begin() + best);
    if (static_cast<int64_t>(doc.size()) > remaining) doc.resize(remaining);
    return doc;
  }

  std::vector<std::vector<int32_t>> state() const { return buf_; }
  void set_state(const std::vector<std::vector<int32_t>>& s) { buf_ = s; }

 private:
  std::vector<std::vector<int32_t>> buf_;
};

namespace {
using Pair = std::pair<int32_t, int32_t>;
struct PairHash {
  size_t operator()(const Pair& p) const { return (static_cast<uint64_t>(p.first) << 32) ^ static_cast<uint32_t>(p.second); }
};
}  // namespace

// words: token-id sequences (initially bytes 0..255) with their counts.  Returns the merges in
// order as (left, right) pairs; merge i creates token id `first_id + i`.
std::vector<Pair> train_bpe(std::vector<std::vector<int32_t>> words, const std::vector<int64_t>& counts,
                            int num_merges, int32_t first_id) {
  if (words.size() != counts.size()) throw std::runtime_error("words/counts length mismatch");
  std::unordered_map<Pair, int64_t, PairHash> pc;
  std::unordered_map<Pair, std::unordered_set<int32_t>, PairHash> where;
  for (size_t w = 0; w < words.size(); ++w) {
    const auto& t = words[w];
    for (size_t i = 0; i + 1 < t.size(); ++i) {
      Pair p{t[i], t[i + 1]};
      pc[p] += counts[w];
      where[p].insert(static_cast<int32_t>(w));
    }
  }
  // max-heap on (count, -pair) with lazy invalidation: an entry is live only while its count is
  // still the pair's current count.
  struct Entry {
    int64_t n;
    Pair p;
    bool operator<(const Entry& o) const { return n != o.n ? n < o.n : o.p < p; }
  };
  std::priority_queue<Entry> heap;
  for (const auto& kv : pc) heap.push({kv.second, kv.first});
  std::vector<Pair> merges;
  merges.reserve(num_merges);
  for (int m = 0; m < num_merges; ++m) {
    Pair best{0, 0};
    bool found = false;
    while (!heap.empty()) {
      Entry e = heap.top();
      heap.pop();
      auto it = pc.find(e.p);
      if (it != pc.end() && it->second == e.n && e.n > 0) {
        best = e.p;
        found = true;
        break;
      }
    }
    if (!found) break;
    const int32_t nid = first_id + m;
    merges.push_back(best);
    std::vector<int32_t> affected(where[best].begin(), where[best].end());
    std::sort(affected.begin(), affected.end());
    std::unordered_set<Pair, PairHash> touched;
    for (int32_t w : affected) {
      auto& t = words[w];
      const int64_t c = counts[w];
      for (size_t i = 0; i + 1 < t.size(); ++i) {
        Pair p{t[i], t[i + 1]};
        auto it = pc.find(p);
        if (it != pc.end() && (it->second -= c) <= 0) pc.erase(it);
        auto wi = where.find(p);
        if (wi != where.end()) wi->second.erase(w);
        touched.insert(p);
      }
      std::vector<int32_t> out;
      out.reserve(t.size());
      for (size_t i = 0; i < t.size();) {
        if (i + 1 < t.size() && t[i] == best.first && t[i + 1] == best.second) {
          out.push_back(nid);
          i += 2;
        } else {
          out.push_back(t[i]);
          i += 1;
        }
      }
      t.swap(out);
      for (size_t i = 0; i + 1 < t.size(); ++i) {
        Pair p{t[i], t[i + 1]};
        pc[p] += c;
        where[p].insert(w);
        touched.insert(p);
      }
    }
    where.erase(best);
    pc.erase(best);
    for (const auto& p : touched) {
      auto it = pc.find(p);
      if (it != pc.end()) heap.push({it->second, p});
    }
  }
  return merges;
}

PYBIND11_MODULE(_native, m) {
  m.doc() = "nexttransformer_b200 host-side native runtime";
  py::class_<BestFitPacker>(m, "BestFitPacker")
      .def(py::init<>())
      .def("add", &BestFitPacker::add)
      .def("size", &BestFitPacker::size)
      .def("pick", &BestFitPacker::pick)
      .def("state", &BestFitPacker::state)
      .def("set_state", &BestFitPacker::set_state);
  m.def("train_bpe", &train_bpe, py::arg("words"), py::arg("counts"), py::arg("num_merges"), py::arg("first_id"));
}
