// Prompt-lookup drafting index (see ngram.h). Each appended token adds one entry per n-gram
// length that ends at it, so a proposal is a hash lookup plus a backwards walk over the
// matching end positions instead of a scan of the window; entries older than the window
// are skipped by the walk (the window only moves forward).
#include "ngram.h"

#ifndef AXR_NO_PYBIND
#include <pybind11/numpy.h>
#include <pybind11/stl.h>
namespace py = pybind11;
#endif

#include <algorithm>
#include <stdexcept>

namespace axr {

namespace {
inline std::uint64_t mix(std::uint64_t h, std::uint32_t v) {
  h ^= v + 0x9e3779b97f4a7c15ull + (h << 6) + (h >> 2);
  h *= 0xff51afd7ed558ccdull;
  return h ^ (h >> 33);
}
}  // namespace

NgramTable::NgramTable(int max_n, int min_n, int window)
    : max_n_(max_n), min_n_(min_n), window_(window), ends_(std::max(0, max_n - min_n + 1)) {
  if (min_n < 1 || max_n < min_n || window < 1) throw std::invalid_argument("NgramTable: need 1 <= min_n <= max_n, window >= 1");
}

std::uint64_t NgramTable::hash(std::size_t end, int n) const {
  std::uint64_t h = 0x243f6a8885a308d3ull ^ static_cast<std::uint64_t>(n);
  for (std::size_t i = end - n; i < end; ++i) h = mix(h, static_cast<std::uint32_t>(toks_[i]));
  return h;
}

void NgramTable::extend(const std::int32_t* t, std::size_t n) {
  toks_.reserve(toks_.size() + n);
  for (std::size_t j = 0; j < n; ++j) {
    toks_.push_back(t[j]);
    const std::size_t end = toks_.size();
    for (int g = min_n_; g <= max_n_; ++g)
      if (end >= static_cast<std::size_t>(g)) ends_[g - min_n_][hash(end, g)].push_back(static_cast<std::int32_t>(end));
  }
}

std::vector<std::int32_t> NgramTable::propose(int k, int skip) const {
  const long long L = static_cast<long long>(toks_.size());
  std::vector<std::int32_t> out;
  if (k <= 0) return out;
  const long long lo = std::max(0LL, L - window_);  // first start position inside the window
  for (int n = max_n_; n >= min_n_; --n) {
    if (L - lo <= n) continue;  // the window holds no earlier n-gram with a successor
    const auto& m = ends_[n - min_n_];
    const auto it = m.find(hash(static_cast<std::size_t>(L), n));
    if (it == m.end()) continue;
    int left = skip;
    const auto& ends = it->second;
    for (auto e = ends.rbegin(); e != ends.rend(); ++e) {
      const long long end = *e;
      if (end >= L) continue;        // the tail itself: no successor
      if (end - n < lo) break;       // older occurrences start before the window
      if (!std::equal(toks_.begin() + (end - n), toks_.begin() + end, toks_.end() - n)) continue;  // collision
      if (left > 0) {
        --left;
        continue;
      }
      const long long stop = std::min(L, end + k);
      out.assign(toks_.begin() + end, toks_.begin() + stop);
      while (static_cast<int>(out.size()) < k) out.push_back(out.back());
      return out;
    }
  }
  out.assign(k, L ? toks_.back() : 0);
  return out;
}

#ifndef AXR_NO_PYBIND
void bind_ngram(py::module_& m) {
  py::class_<NgramTable>(m, "NgramTable")
      .def(py::init<int, int, int>(), py::arg("max_n"), py::arg("min_n"), py::arg("window"))
      .def("extend",
           [](NgramTable& t, py::array_t<std::int32_t, py::array::c_style | py::array::forcecast> a) {
             const std::int32_t* p = a.data();
             const std::size_t n = static_cast<std::size_t>(a.size());
             py::gil_scoped_release rel;
             t.extend(p, n);
           })
      .def("propose",
           [](const NgramTable& t, int k, int skip) {
             std::vector<std::int32_t> v;
             {
               py::gil_scoped_release rel;
               v = t.propose(k, skip);
             }
             return v;
           },
           py::arg("k"), py::arg("skip") = 0)
      .def("__len__", &NgramTable::size);
}

#endif

}  // namespace axr
