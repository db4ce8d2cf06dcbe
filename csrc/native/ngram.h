// Incremental n-gram index of one token sequence for prompt-lookup drafting: proposes the
// tokens that followed the most recent earlier occurrence of the sequence's tail.
#pragma once

#ifndef AXR_NO_PYBIND
#include <pybind11/pybind11.h>
#endif

#include <cstdint>
#include <unordered_map>
#include <vector>

namespace axr {

class NgramTable {
 public:
  NgramTable(int max_n, int min_n, int window);
  // Appends tokens to the sequence and indexes the n-grams that end at each of them.
  void extend(const std::int32_t* t, std::size_t n);
  // k tokens after the (skip + 1)-th most recent earlier occurrence of the longest tail
  // n-gram (max_n down to min_n) that starts inside the last `window` tokens and has a
  // successor; padded with its last token; the last token repeated when nothing matches.
  std::vector<std::int32_t> propose(int k, int skip) const;
  std::size_t size() const { return toks_.size(); }

 private:
  std::uint64_t hash(std::size_t end, int n) const;
  int max_n_, min_n_, window_;
  std::vector<std::int32_t> toks_;
  // per n (index n - min_n): n-gram hash -> end positions (exclusive), ascending
  std::vector<std::unordered_map<std::uint64_t, std::vector<std::int32_t>>> ends_;
};

#ifndef AXR_NO_PYBIND
void bind_ngram(pybind11::module_& m);
#endif

}  // namespace axr
