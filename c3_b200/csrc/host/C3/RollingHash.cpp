#include "C3/RollingHash.h"

#include <mutex>

namespace ct {
namespace c3 {

namespace {
std::mutex g_mu;
std::vector<uint64_t> g_pow{1};
}  // namespace

void RollingHash::precompute(size_t max_len) {
  std::lock_guard<std::mutex> lock(g_mu);
  while (g_pow.size() <= max_len) g_pow.push_back(g_pow.back() * kBase);
}

size_t RollingHash::maxLen() {
  std::lock_guard<std::mutex> lock(g_mu);
  return g_pow.size() - 1;
}

std::vector<uint64_t> RollingHash::computePrefixHashes(const std::vector<op>& ops) {
  precompute(ops.size());
  std::vector<uint64_t> prefix(ops.size() + 1, 0);
  for (size_t i = 0; i < ops.size(); ++i) prefix[i + 1] = prefix[i] * kBase + getOpCode(ops[i]);
  return prefix;
}

uint64_t RollingHash::getSubHash(const std::vector<uint64_t>& prefix, size_t l, size_t r) {
  const size_t len = r - l + 1;
  precompute(len);
  uint64_t p;
  {
    std::lock_guard<std::mutex> lock(g_mu);
    p = g_pow[len];
  }
  return prefix[r + 1] - prefix[l] * p;
}

uint64_t RollingHash::hashSequence(const std::vector<op>& ops) {
  if (ops.empty()) return 0;
  return getSubHash(computePrefixHashes(ops), 0, ops.size() - 1);
}

uint64_t RollingHash::getOpCode(op o) {
  switch (o) {
    case op::Add: return 2;
    case op::Sub: return 3;
    case op::Neg: return 5;
    case op::Mul: return 7;
    case op::Div: return 11;
    case op::MatMul: return 13;
    case op::Dot: return 17;
    case op::Cos: return 19;
    case op::Sin: return 23;
    case op::ReLU: return 29;
    case op::Tanh: return 31;
    case op::Sigmoid: return 37;
    case op::GELU: return 41;
    case op::LReLU: return 43;
    case op::Log: return 47;
    case op::Exp: return 53;
    case op::Abs: return 59;
    case op::Softmax: return 61;
    case op::Min: return 67;
    case op::Max: return 71;
    case op::MSE: return 73;
    case op::CE: return 79;
    case op::MAE: return 83;
    case op::Conv: return 89;
    case op::Pool: return 97;
    default: return 101;
  }
}

}  // namespace c3
}  // namespace ct
