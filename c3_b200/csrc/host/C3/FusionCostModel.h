// Read/write-count cost model gating region fusion, as in the reference
// (include/C3/FusionCostModel.h:71-106): eager = sum of outputs written + intermediates read;
// fusing saves one write and one read of every non-MatMul intermediate; a region is worth
// fusing when it saves something and the saved fraction reaches the threshold (0.20).
#pragma once

#include <atomic>
#include <cstddef>
#include <vector>

#include "Ctools.h"

namespace ct {
namespace c3 {

struct FusionCost {
  size_t eager_accesses = 0;
  size_t fused_accesses = 0;
  size_t saved_accesses = 0;
  double gain_ratio = 0.0;
  bool worthwhile = false;
};

class FusionCostModel {
 public:
  static constexpr double kDefaultMinGainRatio = 0.20;
  static double minGainRatio() { return ratio().load(); }
  static void setMinGainRatio(double r) { ratio().store(r); }
  static bool isComputeIntensive(op t) { return t == op::MatMul; }

  static FusionCost estimate(const std::vector<op>& op_seq, const std::vector<size_t>& out_numels) {
    FusionCost c;
    const size_t n = op_seq.size() < out_numels.size() ? op_seq.size() : out_numels.size();
    if (n == 0) return c;
    size_t write_all = 0, read_mid = 0;
    for (size_t i = 0; i < n; ++i) {
      write_all += out_numels[i];
      if (i + 1 < n) read_mid += out_numels[i];
    }
    c.eager_accesses = write_all + read_mid;
    for (size_t i = 0; i + 1 < n; ++i)
      if (!isComputeIntensive(op_seq[i])) c.saved_accesses += out_numels[i] * 2;
    c.fused_accesses = c.eager_accesses > c.saved_accesses ? c.eager_accesses - c.saved_accesses : 0;
    if (c.eager_accesses > 0)
      c.gain_ratio = static_cast<double>(c.saved_accesses) / static_cast<double>(c.eager_accesses);
    c.worthwhile = c.saved_accesses > 0 && c.gain_ratio >= minGainRatio();
    return c;
  }

 private:
  static std::atomic<double>& ratio() {
    static std::atomic<double> r{kDefaultMinGainRatio};
    return r;
  }
};

}  // namespace c3
}  // namespace ct
