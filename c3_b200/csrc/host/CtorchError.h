// Logging facade with the signature C3 calls (CtorchError::log(level, platform, type, msg)).
// Messages at or above the threshold (env C3_LOG_LEVEL = debug|info|warn|error, default warn)
// go to stderr; the last WARN/ERROR message is kept for diagnostics.
#pragma once

#include <string>

enum class ErrorLevel { DEBUG = 0, INFO = 1, WARN = 2, ERROR = 3 };
enum class ErrorPlatform { kGENERAL, kCPU, kCUDA };
enum class ErrorType { UNKNOWN, DIMENSION, DEVICE_COMPAT, TYPE, MEMORY, RUNTIME };

class CtorchError {
 public:
  static void log(ErrorLevel level, ErrorPlatform platform, ErrorType type, const std::string& msg);
  static std::string lastMessage();
  static size_t count(ErrorLevel level);
};
