// felix::FelixStatus — error object returned by every felix:: operator.
// Same type, fields and semantics as the reference (include/felix/status.hpp:6-41,
// src/felix/base/status.cpp:16-49); KERNEL_RUNTIME_ERROR is produced here by the
// device watchdog (felix::check_watchdog).
#pragma once
#include <cuda_runtime.h>
#include <source_location>
#include <string>

namespace felix {
struct FelixStatus {
  enum class Type { SUCCESS, KERNEL_LAUNCH_FAILED, KERNEL_RUNTIME_ERROR, API_ERROR };

  Type type;
  cudaError_t cuda_code;
  std::string message;
  std::string file;
  int line;
  std::string func;

  FelixStatus();
  FelixStatus(Type t, cudaError_t code, std::string msg, std::string file, int line,
              std::string func);

  [[nodiscard]] bool ok() const;
  [[nodiscard]] std::string str() const;

  static FelixStatus make(Type t, cudaError_t code, std::string msg = "",
                          const std::source_location& loc = std::source_location::current());

  static FelixStatus success() noexcept { return FelixStatus(); }

 private:
  const char* type_string() const;
};
}  // namespace felix
