// Polynomial rolling hash over operator sequences (BASE 131, arithmetic mod 2^64), with
// O(1) sub-sequence hashes from a prefix table. The per-op prime codes are the
// reference's (src/C3/RollingHash.cpp:42-72): region kernels installed by this build are
// found under the same keys a C3 host dispatcher computes.
#pragma once

#include <cstddef>
#include <cstdint>
#include <vector>

#include "Ctools.h"

namespace ct {
namespace c3 {

class RollingHash {
 public:
  static constexpr uint64_t kBase = 131;

  static void precompute(size_t max_len);
  // prefix[i] = hash of ops[0..i-1]; prefix[0] = 0
  static std::vector<uint64_t> computePrefixHashes(const std::vector<op>& ops);
  // hash of ops[l..r] (inclusive), given prefix hashes of length > r + 1
  static uint64_t getSubHash(const std::vector<uint64_t>& prefix, size_t l, size_t r);
  static uint64_t getOpCode(op op_type);
  static size_t maxLen();
  // Convenience: hash of a whole sequence.
  static uint64_t hashSequence(const std::vector<op>& ops);
};

}  // namespace c3
}  // namespace ct
