#include "common.h"

#include <atomic>
#include <cstdlib>
#include <cstring>

namespace rpgb {

namespace {
thread_local std::string g_last_error;

LogLevel Threshold() {
  static const LogLevel lv = [] {
    const char* e = std::getenv("RPGBAR_ENGINE_LOG");
    if (e == nullptr) return LogLevel::kWarn;
    if (std::strcmp(e, "off") == 0) return LogLevel::kOff;
    if (std::strcmp(e, "info") == 0) return LogLevel::kInfo;
    return LogLevel::kWarn;
  }();
  return lv;
}
}  // namespace

void Throw(const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  std::vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  throw Error(buf);
}

namespace {
std::atomic<int64_t> g_launches{0};
}  // namespace

void CountLaunches(int64_t n) { g_launches.fetch_add(n, std::memory_order_relaxed); }
int64_t LaunchCount() { return g_launches.load(std::memory_order_relaxed); }

void SetLastError(const char* msg) { g_last_error = msg != nullptr ? msg : ""; }

const char* LastError() { return g_last_error.c_str(); }

void Log(LogLevel lv, const char* fmt, ...) {
  if (static_cast<int>(lv) < static_cast<int>(Threshold())) return;
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  std::vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  std::fprintf(stderr, "[rpgb %s] %s\n", lv == LogLevel::kWarn ? "warn" : "info", buf);
}

}  // namespace rpgb
