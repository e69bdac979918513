// Native LPT multipack allocator for the packed corpus sampler (CPU).
//
// Behaviour (reference: src/mimir/corpus/multipack.py:10-110): a global batch is the longest
// prefix of the remaining rows whose lengths can be spread over `n` ranks with at most `c`
// tokens each by Longest-Processing-Time-first scheduling (binary search on the prefix
// length); each rank then receives its LPT share.  Row order, tie breaking (descending
// lengths, later index first among equals) and the min-heap discipline are kept exactly so
// the same corpus yields the same batches as the reference sampler.
#include <pybind11/numpy.h>
#include <pybind11/pybind11.h>

#include <algorithm>
#include <cstdint>
#include <numeric>
#include <vector>

namespace py = pybind11;

namespace {

// Min-heap of bin loads stored at [1, n]; ids (optional) follow the swaps.
inline void sift_down(std::vector<int64_t>& heap, std::vector<int64_t>* ids, int64_t n) {
  int64_t u = 1;
  while ((u << 1) <= n) {
    int64_t v = u << 1;
    const int64_t rch = v | 1;
    if (rch <= n && heap[rch] < heap[v]) v = rch;
    if (heap[u] <= heap[v]) break;
    std::swap(heap[u], heap[v]);
    if (ids) std::swap((*ids)[u], (*ids)[v]);
    u = v;
  }
}

bool lpt_fits(const int64_t* a, int64_t m, int64_t c, int64_t n, std::vector<int64_t>& heap,
              std::vector<int64_t>& sorted) {
  sorted.assign(a, a + m);
  std::sort(sorted.begin(), sorted.end(), std::greater<int64_t>());
  std::fill(heap.begin(), heap.end(), 0);
  for (int64_t size : sorted) {
    heap[1] += size;
    if (heap[1] > c) return false;
    sift_down(heap, nullptr, n);
  }
  return true;
}

std::vector<int64_t> lpt_assign(const int64_t* a, int64_t m, int64_t n, int64_t rank, std::vector<int64_t>& heap) {
  // Stable ascending argsort, then reversed: descending lengths, later index first on ties.
  std::vector<int64_t> order(m);
  std::iota(order.begin(), order.end(), 0);
  std::stable_sort(order.begin(), order.end(), [&](int64_t x, int64_t y) { return a[x] < a[y]; });
  std::reverse(order.begin(), order.end());
  std::fill(heap.begin(), heap.end(), 0);
  std::vector<int64_t> ids(n + 1);
  for (int64_t i = 0; i <= n; ++i) ids[i] = i - 1;
  std::vector<int64_t> mine;
  for (int64_t idx : order) {
    heap[1] += a[idx];
    if (ids[1] == rank) mine.push_back(idx);
    sift_down(heap, &ids, n);
  }
  return mine;
}

// Returns (is_full, rows_used, this_rank_rows (absolute indices), tokens_used).
py::tuple allocate(py::array_t<int64_t, py::array::c_style | py::array::forcecast> lengths, int64_t start,
                   int64_t rank, int64_t c, int64_t n) {
  auto buf = lengths.unchecked<1>();
  const int64_t size = buf.shape(0);
  const int64_t* data = lengths.data();
  int64_t total = 0, end = start;
  while (end < size) {
    total += buf(end);
    ++end;
    if (total >= c * n) break;
  }
  const int64_t* a = data + start;
  const int64_t avail = end - start;
  std::vector<int64_t> heap(n + 1), sorted;
  int64_t lo = 1, hi = 1 + avail;
  {
    py::gil_scoped_release release;
    while (hi - lo > 1) {
      const int64_t mid = (lo + hi) / 2;
      if (lpt_fits(a, mid, c, n, heap, sorted)) lo = mid;
      else hi = mid;
    }
  }
  std::vector<int64_t> mine = lpt_assign(a, lo, n, rank, heap);
  py::array_t<int64_t> batch(mine.size());
  auto out = batch.mutable_unchecked<1>();
  for (size_t i = 0; i < mine.size(); ++i) out(i) = start + mine[i];
  int64_t used_tokens = 0;
  for (int64_t i = 0; i < lo && i < avail; ++i) used_tokens += a[i];
  return py::make_tuple(lo >= n, lo, batch, used_tokens);
}

}  // namespace

PYBIND11_MODULE(_host, m) {
  m.doc() = "mimir_b200 native host-side runtime helpers";
  m.def("multipack_allocate", &allocate, py::arg("lengths"), py::arg("start"), py::arg("rank"), py::arg("c"),
        py::arg("n"));
}
