#include "C3/C3BackwardCapture.h"

#include <algorithm>
#include <sstream>
#include <typeinfo>

#include "C3/CudaKernels.h"
#include "c3cu.h"

#include "C3/C3Config.h"
#include "CtorchError.h"

namespace ct {
namespace c3 {

C3BackwardCapture& C3BackwardCapture::getInstance() {
  static C3BackwardCapture instance;
  return instance;
}

C3BackwardCapture::~C3BackwardCapture() {
  std::lock_guard<std::mutex> lock(pending_mutex_);
  for (auto& f : futures_)
    if (f.valid()) f.wait_for(std::chrono::milliseconds(100));
}

std::string C3BackwardCapture::makeBaseKey(const std::string& type_name, const std::vector<size_t>& grad_shape,
                                           const std::vector<std::vector<size_t>>& input_shapes) {
  std::stringstream ss;
  ss << type_name << "|grad:";
  for (size_t s : grad_shape) ss << s << ",";
  ss << "|inputs:";
  for (const auto& sh : input_shapes)
    for (size_t s : sh) ss << s << ",";
  return ss.str();
}

std::optional<std::vector<Tensor>> C3BackwardCapture::tryExecuteBackward(const ::Node* node, const Tensor& grad,
                                                                         const std::vector<Tensor>& forward_inputs) {
  static const bool disabled = [] {
    const char* k = std::getenv("CTORCH_DISABLE_C3_BACKWARD");
    if (k && std::string(k) == "1") return true;
    return !backwardFusionEnabled();
  }();
  if (disabled || !node) return std::nullopt;
  {
    std::lock_guard<std::mutex> lock(stats_mutex_);
    capture_count_++;
  }
  size_t n_inputs = forward_inputs.empty() ? node->getInputs().size() : forward_inputs.size();
  if (n_inputs == 0) n_inputs = 1;
  std::vector<std::vector<size_t>> shapes;
  for (const auto& t : forward_inputs) shapes.push_back(t.sizes());
  const std::string base = makeBaseKey(typeid(*node).name(), grad.sizes(), shapes);
  std::vector<Tensor> out;
  out.reserve(n_inputs);
  for (size_t i = 0; i < n_inputs; ++i) {
    auto r = C3KernelRegistry::getInstance().tryExecuteBackward(base + "|in:" + std::to_string(i), grad,
                                                                forward_inputs);
    if (!r || r->empty()) {
      {
        std::lock_guard<std::mutex> lock(stats_mutex_);
        cache_miss_count_++;
      }
      compileBackwardAsyncForInput(node, grad, i);
      return std::nullopt;
    }
    out.push_back(std::move(r->at(0)));
  }
  std::lock_guard<std::mutex> lock(stats_mutex_);
  cache_hit_count_++;
  return out;
}

void C3BackwardCapture::compileBackwardAsync(const ::Node* node, const Tensor& grad) {
  if (!node) return;
  const size_t n = node->getInputs().empty() ? 1 : node->getInputs().size();
  for (size_t i = 0; i < n; ++i) compileBackwardAsyncForInput(node, grad, i);
}

void C3BackwardCapture::compileBackwardAsyncForInput(const ::Node* node, const Tensor& grad, size_t input_index) {
  if (!node) return;
  const DeviceType dev = grad.device();
  if (dev != DeviceType::kCPU && dev != DeviceType::kCUDA) {
    CtorchError::log(ErrorLevel::WARN, ErrorPlatform::kGENERAL, ErrorType::DEVICE_COMPAT,
                     "C3 backward: unsupported device " + std::to_string(static_cast<int>(dev)));
    return;
  }
  const std::string type = typeid(*node).name();
  std::vector<std::vector<size_t>> shapes;
  std::vector<TensorDesc> input_descs;
  for (const auto& t : node->getInputs()) {
    shapes.push_back(t.sizes());
    input_descs.push_back(TensorDesc{t.sizes(), t.dtype(), t.device(), TensorDesc::computeNumel(t.sizes())});
  }
  const std::string per_key = makeBaseKey(type, grad.sizes(), shapes) + "|in:" + std::to_string(input_index);
  if (C3KernelRegistry::getInstance().hasBackwardKey(per_key)) return;
  {
    std::lock_guard<std::mutex> lock(pending_mutex_);
    if (pending_compiles_.count(per_key)) return;
    pending_compiles_[per_key] = true;
  }
  const TensorDesc grad_desc{grad.sizes(), grad.dtype(), grad.device(), TensorDesc::computeNumel(grad.sizes())};
  auto task = [this, type, input_index, grad_desc, input_descs, per_key]() {
    try {
      auto bg = buildBackwardGraphForTypeAndIndex(type, input_index, grad_desc, input_descs);
      // identity gradients (no compute node) are not compiled: the host passes grad through
      if (bg && bg->first.nodeCount() > bg->first.inputCount() && !bg->first.computeNodes().empty()) {
        CompileOptions opts;
        auto kernel = C3Engine::getInstance().compile(bg->first, opts);
        const std::vector<size_t> out_shape =
            input_descs.empty() ? grad_desc.shape : input_descs[input_index].shape;
        C3KernelRegistry::getInstance().installBackward(per_key, kernel, grad_desc.shape, out_shape, bg->second,
                                                        bg->first.inputCount());
        std::lock_guard<std::mutex> lock(stats_mutex_);
        compile_count_++;
      }
    } catch (const std::exception& e) {
      C3Engine::getInstance().recordCompileError("backward", std::string(e.what()) + " key=" + per_key);
      std::lock_guard<std::mutex> lock(stats_mutex_);
      execution_failures_++;
    }
    std::lock_guard<std::mutex> lock(pending_mutex_);
    pending_compiles_.erase(per_key);
  };
  std::lock_guard<std::mutex> lock(pending_mutex_);
  futures_.push_back(std::async(std::launch::async, task));
}

void C3BackwardCapture::waitForPendingCompiles() {
  std::vector<std::future<void>> fs;
  {
    std::lock_guard<std::mutex> lock(pending_mutex_);
    fs.swap(futures_);
  }
  for (auto& f : fs)
    if (f.valid()) f.wait_for(std::chrono::seconds(30));
}

std::optional<Graph> C3BackwardCapture::buildBackwardGraph(const ::Node* node, const TensorDesc& grad_desc,
                                                           const std::vector<TensorDesc>& input_descs) {
  return buildBackwardGraphForInput(node, 0, grad_desc, input_descs);
}

std::optional<Graph> C3BackwardCapture::buildBackwardGraphForInput(const ::Node* node, size_t input_index,
                                                                   const TensorDesc& grad_desc,
                                                                   const std::vector<TensorDesc>& input_descs) {
  if (!node) return std::nullopt;
  auto bg = buildBackwardGraphForTypeAndIndex(typeid(*node).name(), input_index, grad_desc, input_descs);
  if (!bg) return std::nullopt;
  return bg->first;
}

bool C3BackwardCapture::supportsNodeType(const std::string& t) {
  for (const char* n : {"ReLUNode", "SigmoidNode", "TanhNode", "AddNode", "MulNode", "MatMulNode", "NegNode",
                        "SubNode", "DivNode", "ExpNode", "LogNode"})
    if (t.find(n) != std::string::npos) return true;
  return false;
}

std::optional<C3BackwardCapture::BackwardGraph> C3BackwardCapture::buildBackwardGraphForTypeAndIndex(
    const std::string& t, size_t i, const TensorDesc& grad, const std::vector<TensorDesc>& in) {
  auto has = [&t](const char* s) { return t.find(s) != std::string::npos; };
  if (has("ReLUNode")) return (i == 0 && !in.empty()) ? std::optional(buildReLUBackwardGraph(grad, in[0])) : std::nullopt;
  if (has("SigmoidNode")) return (i == 0 && !in.empty()) ? std::optional(buildSigmoidBackwardGraph(grad, in[0])) : std::nullopt;
  if (has("TanhNode")) return (i == 0 && !in.empty()) ? std::optional(buildTanhBackwardGraph(grad, in[0])) : std::nullopt;
  if (has("AddNode")) return (i < in.size() && in.size() >= 2) ? std::optional(buildAddBackwardGraph(grad, in[0], in[1], i)) : std::nullopt;
  // MatMulNode before MulNode: "MulNode" is a substring of "MatMulNode"
  if (has("MatMulNode")) return (i < in.size() && in.size() >= 2) ? std::optional(buildMatMulBackwardGraph(grad, in[0], in[1], i)) : std::nullopt;
  if (has("MulNode")) return (i < in.size() && in.size() >= 2) ? std::optional(buildMulBackwardGraph(grad, in[0], in[1], i)) : std::nullopt;
  if (has("NegNode")) return i == 0 ? std::optional(buildNegBackwardGraph(grad)) : std::nullopt;
  if (has("SubNode")) return i < std::max<size_t>(in.size(), 2) ? std::optional(buildSubBackwardGraph(grad, i)) : std::nullopt;
  if (has("DivNode")) return (i < in.size() && in.size() >= 2) ? std::optional(buildDivBackwardGraph(grad, in[0], in[1], i)) : std::nullopt;
  if (has("ExpNode")) return (i == 0 && !in.empty()) ? std::optional(buildExpBackwardGraph(grad, in[0])) : std::nullopt;
  if (has("LogNode")) return (i == 0 && !in.empty()) ? std::optional(buildLogBackwardGraph(grad, in[0])) : std::nullopt;
  return std::nullopt;
}

C3BackwardCapture::Stats C3BackwardCapture::getStats() const {
  std::lock_guard<std::mutex> lock(stats_mutex_);
  Stats s;
  s.capture_count = capture_count_;
  s.compile_count = compile_count_;
  s.cache_hit_count = cache_hit_count_;
  s.cache_miss_count = cache_miss_count_;
  s.execution_failures = execution_failures_;
  s.fusion_compile_count = fusion_compile_count_;
  s.fusion_hit_count = fusion_hit_count_;
  s.fusion_miss_count = fusion_miss_count_;
  return s;
}

void C3BackwardCapture::clear() {
  {
    std::lock_guard<std::mutex> lock(stats_mutex_);
    capture_count_ = compile_count_ = cache_hit_count_ = cache_miss_count_ = execution_failures_ = 0;
    fusion_compile_count_ = fusion_hit_count_ = fusion_miss_count_ = 0;
  }
  waitForPendingCompiles();
  {
    std::lock_guard<std::mutex> lock(fusion_mutex_);
    recent_sequence_.clear();
    recent_grad_shapes_.clear();
    recent_input_shapes_.clear();
    sequence_counts_.clear();
  }
  clearInterceptedState();
  std::lock_guard<std::mutex> lock(pending_mutex_);
  pending_compiles_.clear();
}

void C3BackwardCapture::clearCallScopedState() { clearInterceptedState(); }

// ============================================================================ fused sequences
bool C3BackwardCapture::isElementWiseBackward(const std::string& t) {
  // single-input, single-output nodes only (src/C3/C3BackwardCapture.cpp:463-483)
  for (const char* n : {"ReLUNode", "SigmoidNode", "TanhNode", "NegNode", "GELUNode", "LReLUNode", "SinNode",
                        "CosNode", "AbsNode", "ExpNode", "LogNode", "MinNode", "MaxNode"})
    if (t.find(n) != std::string::npos) return true;
  return false;
}

bool C3BackwardCapture::isFusableSequence(const std::vector<std::string>& types) {
  if (types.size() < 2) return false;
  for (const auto& t : types)
    if (!isElementWiseBackward(t)) return false;
  return true;
}

std::string C3BackwardCapture::makeSequenceKey(const std::vector<std::string>& types) {
  std::string key;
  for (const auto& t : types) {
    if (!key.empty()) key += "+";
    const char* names[][2] = {{"ReLUNode", "ReLU"}, {"SigmoidNode", "Sigmoid"}, {"TanhNode", "Tanh"},
                              {"NegNode", "Neg"},   {"AddNode", "Add"},         {"SubNode", "Sub"},
                              {"MulNode", "Mul"},   {"DivNode", "Div"},         {"ExpNode", "Exp"},
                              {"LogNode", "Log"}};
    const char* shortname = "Other";
    for (const auto& nm : names)
      if (t.find(nm[0]) != std::string::npos) {
        shortname = nm[1];
        break;
      }
    key += shortname;
  }
  return key;
}

std::string C3BackwardCapture::makeFusedBackwardKey(const std::string& seq_key, const std::vector<size_t>& g,
                                                    const std::vector<size_t>& in) {
  std::stringstream ss;
  ss << "backward_fused_" << seq_key << "|g:";
  for (size_t v : g) ss << v << ",";
  ss << "|i:";
  for (size_t v : in) ss << v << ",";
  return ss.str();
}

void C3BackwardCapture::countSequence(std::vector<std::string> types, std::vector<std::vector<size_t>> gs,
                                      std::vector<std::vector<size_t>> is) {
  // registration key: the most downstream gradient shape and the most upstream input shape
  const std::string full_key = makeFusedBackwardKey(makeSequenceKey(types), gs.front(), is.back());
  auto& entry = sequence_counts_[full_key];
  if (entry.node_types.empty()) {
    entry.node_types = std::move(types);
    entry.grad_shapes = std::move(gs);
    entry.input_shapes = std::move(is);
  }
  entry.frequency++;
  if (entry.frequency >= kFusionThreshold && !entry.compiling) {
    entry.compiling = true;
    compileFusedBackwardAsync(entry);
  }
}

void C3BackwardCapture::recordBackwardNode(const std::string& node_type, const std::vector<size_t>& grad_shape,
                                           const std::vector<size_t>& input_shape,
                                           const std::vector<Tensor>& forward_inputs) {
  (void)forward_inputs;
  if (!isElementWiseBackward(node_type)) return;  // other nodes never enter the window
  std::lock_guard<std::mutex> lock(fusion_mutex_);
  // A complete two-node chain from the previous pass is counted and the window restarted,
  // so that the tail of one iteration never pairs with the head of the next
  // (src/C3/C3BackwardCapture.cpp:886-931).
  if (recent_sequence_.size() == 2) {
    std::vector<std::string> chain(recent_sequence_.begin(), recent_sequence_.end());
    std::vector<std::vector<size_t>> gs(recent_grad_shapes_.begin(), recent_grad_shapes_.end());
    std::vector<std::vector<size_t>> is(recent_input_shapes_.begin(), recent_input_shapes_.end());
    bool same_shape = true;
    for (size_t i = 1; i < gs.size(); ++i) same_shape = same_shape && gs[i] == gs[0];
    if (same_shape && isFusableSequence(chain)) countSequence(std::move(chain), std::move(gs), std::move(is));
    recent_sequence_.clear();
    recent_grad_shapes_.clear();
    recent_input_shapes_.clear();
  }
  recent_sequence_.push_back(node_type);
  recent_grad_shapes_.push_back(grad_shape);
  recent_input_shapes_.push_back(input_shape);
  if (recent_sequence_.size() > kFusionWindowSize) {
    recent_sequence_.pop_front();
    recent_grad_shapes_.pop_front();
    recent_input_shapes_.pop_front();
  }
  // every fusable tail window of length 2..kFusionWindowSize is counted
  const size_t L = recent_sequence_.size();
  for (size_t w = 2; w <= kFusionWindowSize && w <= L; ++w) {
    const size_t start = L - w;
    std::vector<std::string> types(recent_sequence_.begin() + start, recent_sequence_.end());
    if (!isFusableSequence(types)) continue;
    std::vector<std::vector<size_t>> gs(recent_grad_shapes_.begin() + start, recent_grad_shapes_.end());
    std::vector<std::vector<size_t>> is(recent_input_shapes_.begin() + start, recent_input_shapes_.end());
    countSequence(std::move(types), std::move(gs), std::move(is));
  }
}

namespace {
int chainOp(const std::string& t) {
  if (t.find("ReLUNode") != std::string::npos) return C3CU_BW_RELU;
  if (t.find("SigmoidNode") != std::string::npos) return C3CU_BW_SIGMOID;
  if (t.find("TanhNode") != std::string::npos) return C3CU_BW_TANH;
  if (t.find("NegNode") != std::string::npos) return C3CU_BW_NEG;
  if (t.find("ExpNode") != std::string::npos) return C3CU_BW_EXP;
  if (t.find("LogNode") != std::string::npos) return C3CU_BW_LOG;
  return 0;  // no backward graph for this type: the sequence is not compiled
}
}  // namespace

void C3BackwardCapture::compileFusedBackwardAsync(const BackwardSequence& seq) {
  if (!isFusableSequence(seq.node_types) || seq.grad_shapes.empty() || seq.input_shapes.empty()) return;
  const std::string key =
      makeFusedBackwardKey(makeSequenceKey(seq.node_types), seq.grad_shapes.front(), seq.input_shapes.back());
  {
    std::lock_guard<std::mutex> lock(pending_mutex_);
    if (pending_compiles_.count(key)) return;
    pending_compiles_[key] = true;
  }
  auto task = [this, seq, key]() {
    std::vector<int> ops;
    for (const auto& t : seq.node_types) ops.push_back(chainOp(t));
    const bool supported = std::find(ops.begin(), ops.end(), 0) == ops.end();
    if (supported) {
      // inputs [grad, fwd_0[0], ..., fwd_{N-1}[0]]: identity map onto the forward inputs
      auto kernel = std::make_shared<CudaFusedBackwardKernel>(key, ops, seq.grad_shapes.front());
      std::vector<size_t> fwd_map(seq.node_types.size());
      for (size_t i = 0; i < fwd_map.size(); ++i) fwd_map[i] = i;
      C3KernelRegistry::getInstance().installBackward(key, kernel, seq.grad_shapes.front(), seq.input_shapes.back(),
                                                      fwd_map, 1 + seq.node_types.size());
      std::lock_guard<std::mutex> lock(stats_mutex_);
      fusion_compile_count_++;
    }
    std::lock_guard<std::mutex> lock(pending_mutex_);
    pending_compiles_.erase(key);
  };
  std::lock_guard<std::mutex> lock(pending_mutex_);
  futures_.push_back(std::async(std::launch::async, task));
}

std::optional<Tensor> C3BackwardCapture::tryExecuteFusedBackward(const ::Node* node, const Tensor& grad,
                                                                 const std::vector<Tensor>& forward_inputs) {
  if (!node) return std::nullopt;
  const std::string current_type = typeid(*node).name();
  // Path A: the gradient was computed when the fused kernel ran at a downstream node.
  {
    std::unique_lock<std::shared_mutex> lock(intercepted_mutex_);
    auto it = pending_intercepted_.find(node);
    if (it != pending_intercepted_.end()) {
      if (it->second.first == current_type) {
        Tensor t = std::move(it->second.second);
        pending_intercepted_.erase(it);
        lock.unlock();
        std::lock_guard<std::mutex> slock(stats_mutex_);
        fusion_hit_count_++;
        return t;
      }
      pending_intercepted_.erase(it);  // a reused address with another type: stale entry
    }
  }
  {
    std::lock_guard<std::mutex> mlock(miss_marker_mutex_);
    if (miss_marker_nodes_.count(node)) {
      std::lock_guard<std::mutex> slock(stats_mutex_);
      fusion_miss_count_++;
      return std::nullopt;
    }
  }
  if (!isElementWiseBackward(current_type)) return std::nullopt;
  // Path B: this node is the most downstream one of a chain. Walk upstream (skipping up to
  // kSkipMax single-upstream wrapper nodes between elementwise nodes); every node of the
  // chain must take an input of the gradient's shape.
  constexpr size_t kSkipMax = 4;
  std::vector<std::shared_ptr<::Node>> chain_nodes{nullptr};
  std::vector<std::string> chain_types{current_type};
  std::vector<std::vector<Tensor>> chain_inputs{forward_inputs.empty() ? node->getInputs() : forward_inputs};
  const ::Node* cur = node;
  for (size_t step = 1; step < kFusionWindowSize; ++step) {
    std::shared_ptr<::Node> next;
    const ::Node* c = cur;
    for (size_t skips = 0; skips <= kSkipMax; ++skips) {
      const auto& ups = c->getUpStreamNodes();
      if (ups.size() != 1 || !ups[0]) break;
      if (isElementWiseBackward(typeid(*ups[0]).name())) {
        next = ups[0];
        break;
      }
      c = ups[0].get();
    }
    if (!next) break;
    const auto& ins = next->getInputs();
    if (ins.empty() || ins[0].sizes() != grad.sizes()) break;
    chain_nodes.push_back(next);
    chain_types.push_back(typeid(*next).name());
    chain_inputs.push_back(ins);
    cur = next.get();
  }
  for (size_t w = std::min(kFusionWindowSize, chain_types.size()); w >= 2; --w) {
    std::vector<std::string> types(chain_types.begin(), chain_types.begin() + w);
    if (!isFusableSequence(types)) continue;
    const auto& up_shape = chain_inputs[w - 1].empty() ? grad.sizes() : chain_inputs[w - 1][0].sizes();
    const std::string key = makeFusedBackwardKey(makeSequenceKey(types), grad.sizes(), up_shape);
    if (!C3KernelRegistry::getInstance().hasBackwardKey(key)) continue;
    std::vector<Tensor> fwd;
    for (size_t k = 0; k < w; ++k) {
      if (chain_inputs[k].empty()) break;
      fwd.push_back(chain_inputs[k][0]);
    }
    if (fwd.size() != w) continue;
    auto outs = C3KernelRegistry::getInstance().tryExecuteBackward(key, grad, fwd);
    if (!outs || outs->size() != w) continue;
    {
      std::unique_lock<std::shared_mutex> lock(intercepted_mutex_);
      for (size_t k = 1; k < w; ++k)
        pending_intercepted_[chain_nodes[k].get()] = {chain_types[k], std::move((*outs)[k])};
    }
    std::lock_guard<std::mutex> slock(stats_mutex_);
    fusion_hit_count_++;
    return std::move((*outs)[0]);
  }
  {
    std::lock_guard<std::mutex> mlock(miss_marker_mutex_);
    miss_marker_nodes_[node] = true;
  }
  std::lock_guard<std::mutex> slock(stats_mutex_);
  fusion_miss_count_++;
  return std::nullopt;
}

void C3BackwardCapture::clearInterceptedState() {
  {
    std::unique_lock<std::shared_mutex> lock(intercepted_mutex_);
    pending_intercepted_.clear();
  }
  std::lock_guard<std::mutex> lock(miss_marker_mutex_);
  miss_marker_nodes_.clear();
}

bool C3BackwardCapture::needsSumReduce(const std::vector<size_t>& g, const std::vector<size_t>& t) {
  if (g == t) return false;
  if (g.empty() || t.empty()) return true;
  if (g.size() > t.size()) return true;
  for (size_t i = 0; i < g.size(); ++i) {
    const size_t gd = g[g.size() - 1 - i];
    const size_t td = i < t.size() ? t[t.size() - 1 - i] : 1;
    if (gd != td) return true;
  }
  return false;
}

int C3BackwardCapture::computeReduceAxis(const std::vector<size_t>& g, const std::vector<size_t>& t) {
  if (g == t || g.empty() || t.empty()) return -1;
  if (g.size() > t.size()) return 0;
  const size_t offset = g.size() - t.size();
  for (size_t i = 0; i < g.size(); ++i) {
    if (i < offset) return static_cast<int>(i);
    if (g[i] != t[i - offset] && t[i - offset] == 1) return static_cast<int>(i);
  }
  return -1;
}

// ------------------------------------------------------------------ builders
// Each follows the reference's graph for that node type (src/C3/C3BackwardCapture.cpp:501-873).

C3BackwardCapture::BackwardGraph C3BackwardCapture::buildReLUBackwardGraph(const TensorDesc& grad, const TensorDesc& x) {
  Graph g;
  const size_t gi = g.addInput(grad), xi = g.addInput(x);
  const auto zero = TensorDesc::fromShape({1});
  const size_t z = g.addConstant(0.0, zero);
  const size_t gt = g.addNode(GtNode{x, zero}, {xi, z}, TensorDesc::fromShape(x.shape));
  g.markOutput(g.addNode(MulNode{TensorDesc::fromShape(x.shape), grad}, {gt, gi}, TensorDesc::fromShape(x.shape)));
  return {std::move(g), {0}};
}

C3BackwardCapture::BackwardGraph C3BackwardCapture::buildSigmoidBackwardGraph(const TensorDesc& grad, const TensorDesc& x) {
  Graph g;
  const size_t gi = g.addInput(grad), xi = g.addInput(x);
  const auto d = TensorDesc::fromShape(x.shape);
  const size_t neg = g.addNode(NegNode{d}, {xi}, d);
  const size_t ex = g.addNode(ExpNode{d}, {neg}, d);
  const size_t one = g.addConstant(1.0, TensorDesc::fromShape({1}));
  const size_t den = g.addNode(AddNode{d, d}, {one, ex}, d);
  const size_t sig = g.addNode(DivNode{d, d}, {one, den}, d);
  const size_t oms = g.addNode(SubNode{d, d}, {one, sig}, d);
  const size_t prod = g.addNode(MulNode{d, d}, {sig, oms}, d);
  g.markOutput(g.addNode(MulNode{grad, d}, {gi, prod}, d));
  return {std::move(g), {0}};
}

C3BackwardCapture::BackwardGraph C3BackwardCapture::buildTanhBackwardGraph(const TensorDesc& grad, const TensorDesc& x) {
  Graph g;
  const size_t gi = g.addInput(grad), xi = g.addInput(x);
  const auto d = TensorDesc::fromShape(x.shape);
  const size_t ex = g.addNode(ExpNode{d}, {xi}, d);
  const size_t nx = g.addNode(NegNode{d}, {xi}, d);
  const size_t enx = g.addNode(ExpNode{d}, {nx}, d);
  const size_t num = g.addNode(SubNode{d, d}, {ex, enx}, d);
  const size_t den = g.addNode(AddNode{d, d}, {ex, enx}, d);
  const size_t th = g.addNode(DivNode{d, d}, {num, den}, d);
  const size_t sq = g.addNode(MulNode{d, d}, {th, th}, d);
  const size_t one = g.addConstant(1.0, TensorDesc::fromShape({1}));
  const size_t om = g.addNode(SubNode{d, TensorDesc::fromShape({1})}, {one, sq}, d);
  g.markOutput(g.addNode(MulNode{grad, d}, {gi, om}, d));
  return {std::move(g), {0}};
}

C3BackwardCapture::BackwardGraph C3BackwardCapture::buildAddBackwardGraph(const TensorDesc& grad, const TensorDesc& lhs,
                                                                          const TensorDesc& rhs, size_t index) {
  Graph g;
  const size_t gi = g.addInput(grad);
  const TensorDesc& target = index == 0 ? lhs : rhs;
  if (needsSumReduce(grad.shape, target.shape)) {
    const int axis = computeReduceAxis(grad.shape, target.shape);
    g.markOutput(g.addNode(SumReduceNode{grad, axis}, {gi}, TensorDesc::fromShape(target.shape)));
  } else {
    g.markOutput(gi);
  }
  return {std::move(g), {}};
}

C3BackwardCapture::BackwardGraph C3BackwardCapture::buildMulBackwardGraph(const TensorDesc& grad, const TensorDesc& a,
                                                                          const TensorDesc& b, size_t index) {
  Graph g;
  const size_t gi = g.addInput(grad);
  if (index == 0) {
    const size_t bi = g.addInput(b);
    g.markOutput(g.addNode(MulNode{grad, b}, {gi, bi}, TensorDesc::fromShape(a.shape)));
    return {std::move(g), {1}};
  }
  const size_t ai = g.addInput(a);
  g.markOutput(g.addNode(MulNode{a, grad}, {ai, gi}, TensorDesc::fromShape(b.shape)));
  return {std::move(g), {0}};
}

C3BackwardCapture::BackwardGraph C3BackwardCapture::buildMatMulBackwardGraph(const TensorDesc& grad, const TensorDesc& a,
                                                                             const TensorDesc& b, size_t index) {
  Graph g;
  const size_t gi = g.addInput(grad);
  if (index == 0) {
    // grad_A = grad @ B^T: the transpose is folded into the GEMM's operand read
    const size_t bi = g.addInput(b);
    const auto bt = TensorDesc::fromShape({b.shape[1], b.shape[0]});
    const size_t t = g.addNode(TransposeNode{b, 0, 1}, {bi}, bt);
    g.markOutput(g.addNode(MatMulNode{grad, bt}, {gi, t}, TensorDesc::fromShape({grad.shape[0], bt.shape[1]})));
    return {std::move(g), {1}};
  }
  const size_t ai = g.addInput(a);
  const auto at = TensorDesc::fromShape({a.shape[1], a.shape[0]});
  const size_t t = g.addNode(TransposeNode{a, 0, 1}, {ai}, at);
  g.markOutput(g.addNode(MatMulNode{at, grad}, {t, gi}, TensorDesc::fromShape({at.shape[0], grad.shape[1]})));
  return {std::move(g), {0}};
}

C3BackwardCapture::BackwardGraph C3BackwardCapture::buildNegBackwardGraph(const TensorDesc& grad) {
  Graph g;
  const size_t gi = g.addInput(grad);
  g.markOutput(g.addNode(NegNode{grad}, {gi}, grad));
  return {std::move(g), {}};
}

C3BackwardCapture::BackwardGraph C3BackwardCapture::buildSubBackwardGraph(const TensorDesc& grad, size_t index) {
  Graph g;
  const size_t gi = g.addInput(grad);
  if (index == 0)
    g.markOutput(gi);
  else
    g.markOutput(g.addNode(NegNode{grad}, {gi}, grad));
  return {std::move(g), {}};
}

C3BackwardCapture::BackwardGraph C3BackwardCapture::buildDivBackwardGraph(const TensorDesc& grad, const TensorDesc& a,
                                                                          const TensorDesc& b, size_t index) {
  Graph g;
  const size_t gi = g.addInput(grad);
  if (index == 0) {
    const size_t bi = g.addInput(b);
    g.markOutput(g.addNode(DivNode{grad, b}, {gi, bi}, TensorDesc::fromShape(a.shape)));
    return {std::move(g), {1}};
  }
  const size_t ai = g.addInput(a), bi = g.addInput(b);
  const size_t b2 = g.addNode(MulNode{b, b}, {bi, bi}, b);
  const size_t q = g.addNode(DivNode{a, b}, {ai, b2}, a);
  const size_t m = g.addNode(MulNode{a, grad}, {q, gi}, TensorDesc::fromShape(b.shape));
  g.markOutput(g.addNode(NegNode{TensorDesc::fromShape(b.shape)}, {m}, TensorDesc::fromShape(b.shape)));
  return {std::move(g), {0, 1}};
}

C3BackwardCapture::BackwardGraph C3BackwardCapture::buildExpBackwardGraph(const TensorDesc& grad, const TensorDesc& x) {
  Graph g;
  const size_t gi = g.addInput(grad), xi = g.addInput(x);
  const size_t e = g.addNode(ExpNode{x}, {xi}, x);
  g.markOutput(g.addNode(MulNode{x, grad}, {e, gi}, TensorDesc::fromShape(x.shape)));
  return {std::move(g), {0}};
}

C3BackwardCapture::BackwardGraph C3BackwardCapture::buildLogBackwardGraph(const TensorDesc& grad, const TensorDesc& x) {
  Graph g;
  const size_t gi = g.addInput(grad), xi = g.addInput(x);
  g.markOutput(g.addNode(DivNode{grad, x}, {gi, xi}, TensorDesc::fromShape(x.shape)));
  return {std::move(g), {0}};
}

}  // namespace c3
}  // namespace ct
