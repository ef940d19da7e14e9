// common.h -- errors, logging and CUDA checks shared by the host side.
//
// Error model (same contract as the reference's src/common.h:55-58 and
// src/engine.cc:231-239): internal code throws rpgb::Error; every extern "C"
// entry point catches, stores the message in a thread-local slot and returns a
// negative value or NULL.  CUDA failures become rpgb::Error too.
#pragma once

#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <stdexcept>
#include <string>

namespace rpgb {

class Error : public std::runtime_error {
 public:
  explicit Error(const std::string& m) : std::runtime_error(m) {}
};

[[noreturn]] void Throw(const char* fmt, ...) __attribute__((format(printf, 1, 2)));

void SetLastError(const char* msg);
const char* LastError();

enum class LogLevel { kInfo = 0, kWarn = 1, kOff = 2 };
void Log(LogLevel lv, const char* fmt, ...) __attribute__((format(printf, 2, 3)));

}  // namespace rpgb

#define RPGB_CHECK(cond, ...)      \
  do {                             \
    if (!(cond)) {                 \
      ::rpgb::Throw(__VA_ARGS__);  \
    }                              \
  } while (0)

#define RPGB_CUDA(call)                                                                  \
  do {                                                                                   \
    const cudaError_t rpgb_e_ = (call);                                                  \
    if (rpgb_e_ != cudaSuccess) {                                                        \
      ::rpgb::Throw("CUDA error %s at %s:%d: %s", cudaGetErrorName(rpgb_e_), __FILE__,   \
                    __LINE__, cudaGetErrorString(rpgb_e_));                              \
    }                                                                                    \
  } while (0)

#define RPGB_INFO(...) ::rpgb::Log(::rpgb::LogLevel::kInfo, __VA_ARGS__)
#define RPGB_WARN(...) ::rpgb::Log(::rpgb::LogLevel::kWarn, __VA_ARGS__)
