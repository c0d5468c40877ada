#include "CtorchError.h"

#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

namespace {
std::mutex g_mu;
std::string g_last;
std::atomic<size_t> g_counts[4];

ErrorLevel threshold() {
  static const ErrorLevel t = [] {
    const char* v = std::getenv("C3_LOG_LEVEL");
    if (!v) return ErrorLevel::WARN;
    if (!std::strcmp(v, "debug")) return ErrorLevel::DEBUG;
    if (!std::strcmp(v, "info")) return ErrorLevel::INFO;
    if (!std::strcmp(v, "error")) return ErrorLevel::ERROR;
    return ErrorLevel::WARN;
  }();
  return t;
}

const char* levelName(ErrorLevel l) {
  switch (l) {
    case ErrorLevel::DEBUG: return "DEBUG";
    case ErrorLevel::INFO: return "INFO";
    case ErrorLevel::WARN: return "WARN";
    default: return "ERROR";
  }
}
}  // namespace

void CtorchError::log(ErrorLevel level, ErrorPlatform, ErrorType, const std::string& msg) {
  g_counts[static_cast<int>(level)].fetch_add(1, std::memory_order_relaxed);
  if (level >= ErrorLevel::WARN) {
    std::lock_guard<std::mutex> lock(g_mu);
    g_last = msg;
  }
  if (level >= threshold()) std::fprintf(stderr, "[c3 %s] %s\n", levelName(level), msg.c_str());
}

std::string CtorchError::lastMessage() {
  std::lock_guard<std::mutex> lock(g_mu);
  return g_last;
}

size_t CtorchError::count(ErrorLevel level) {
  return g_counts[static_cast<int>(level)].load(std::memory_order_relaxed);
}
