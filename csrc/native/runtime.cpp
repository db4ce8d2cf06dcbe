// Runtime helpers and controller bindings.
#include "runtime.h"

#include <pybind11/numpy.h>

#include <cstdint>

namespace py = pybind11;

namespace axr {
namespace {

inline std::uint64_t mix64(std::uint64_t x) {
  x ^= x >> 30;
  x *= 0xbf58476d1ce4e5b9ull;
  x ^= x >> 27;
  x *= 0x94d049bb133111ebull;
  x ^= x >> 31;
  return x;
}

// Chained 128-bit content hashes of full 16-token blocks: block i's hash covers the
// hash of block i-1 and its own tokens, so equal hashes mean equal whole prefixes.
py::array_t<std::uint64_t> block_chain_hashes(py::array_t<std::int32_t, py::array::c_style | py::array::forcecast> toks,
                                              int page, long long n_blocks) {
  const long long n = toks.size();
  const long long nb = std::min<long long>(n_blocks < 0 ? n / page : n_blocks, n / page);
  py::array_t<std::uint64_t> out({nb, 2LL});
  auto* o = out.mutable_data();
  const std::int32_t* t = toks.data();
  std::uint64_t a = 0x6a09e667f3bcc908ull, b = 0xbb67ae8584caa73bull;
  {
    py::gil_scoped_release rel;
    for (long long i = 0; i < nb; ++i) {
      std::uint64_t ha = mix64(a ^ 0x3c6ef372fe94f82bull), hb = mix64(b + 0xa54ff53a5f1d36f1ull);
      for (int j = 0; j < page; ++j) {
        const std::uint64_t v = static_cast<std::uint32_t>(t[i * page + j]);
        ha = mix64(ha ^ (v * 0x9e3779b97f4a7c15ull + static_cast<std::uint64_t>(j)));
        hb = mix64(hb + v * 0xc2b2ae3d27d4eb4full + (ha << 1));
      }
      a = ha;
      b = hb;
      o[2 * i] = a;
      o[2 * i + 1] = b;
    }
  }
  return out;
}

}  // namespace

void bind_runtime(py::module_& m) {
  m.def("block_chain_hashes", &block_chain_hashes, py::arg("tokens"), py::arg("page") = 16,
        py::arg("n_blocks") = -1);
}

}  // namespace axr
