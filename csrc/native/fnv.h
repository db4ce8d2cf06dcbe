// FNV-1a 64-bit hashing used by every AMF key namespace that lives on disk.
//
// The constants and the two step functions define the on-disk key format of the
// AMF store (prefix hash of int32 token ids, tenant hash of UTF-8 bytes, index and
// blob checksums), so they must match the reference store bit for bit
// (reference: core/amf_store.cpp:27-28, :118-129).  Everything else here is new.
#pragma once

#include <cstddef>
#include <cstdint>

namespace axr {

constexpr std::uint64_t kFnvOffset = 1469598103934665603ull;
constexpr std::uint64_t kFnvPrime = 1099511628211ull;

// Byte-serial FNV-1a: h ^= byte; h *= prime.
inline std::uint64_t fnv1a_bytes(std::uint64_t h, const void* data, std::size_t n) {
  const auto* p = static_cast<const std::uint8_t*>(data);
  // Unrolled by 8: the dependency chain is serial, unrolling only trims loop overhead.
  std::size_t i = 0;
  for (; i + 8 <= n; i += 8) {
    h = (h ^ p[i + 0]) * kFnvPrime;
    h = (h ^ p[i + 1]) * kFnvPrime;
    h = (h ^ p[i + 2]) * kFnvPrime;
    h = (h ^ p[i + 3]) * kFnvPrime;
    h = (h ^ p[i + 4]) * kFnvPrime;
    h = (h ^ p[i + 5]) * kFnvPrime;
    h = (h ^ p[i + 6]) * kFnvPrime;
    h = (h ^ p[i + 7]) * kFnvPrime;
  }
  for (; i < n; ++i) h = (h ^ p[i]) * kFnvPrime;
  return h;
}

// Token step: the whole 32-bit token id is xor-ed in at once (not byte by byte).
inline std::uint64_t fnv1a_token(std::uint64_t h, std::int32_t tok) {
  return (h ^ static_cast<std::uint64_t>(static_cast<std::uint32_t>(tok))) * kFnvPrime;
}

inline std::uint64_t fnv1a_tokens(const std::int32_t* toks, std::size_t n) {
  std::uint64_t h = kFnvOffset;
  for (std::size_t i = 0; i < n; ++i) h = fnv1a_token(h, toks[i]);
  return h;
}

}  // namespace axr
