#include "core/logger.h"

#include <atomic>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <ctime>
#include <mutex>
#include <unistd.h>

namespace bccl {
namespace {

LogLevel ParseLevel(const char* s) {
    if (s == nullptr) return LogLevel::kWarn;
    if (!strcasecmp(s, "DEBUG") || !strcmp(s, "0")) return LogLevel::kDebug;
    if (!strcasecmp(s, "INFO") || !strcmp(s, "1")) return LogLevel::kInfo;
    if (!strcasecmp(s, "WARN") || !strcasecmp(s, "WARNING") || !strcmp(s, "2")) return LogLevel::kWarn;
    if (!strcasecmp(s, "ERROR") || !strcmp(s, "3")) return LogLevel::kError;
    if (!strcasecmp(s, "NONE") || !strcmp(s, "4")) return LogLevel::kNone;
    return LogLevel::kWarn;
}

std::atomic<int>& LevelStore() {
    static std::atomic<int> level{static_cast<int>(ParseLevel(std::getenv("BCCL_LOG_LEVEL")))};
    return level;
}

const char* LevelTag(LogLevel l) {
    switch (l) {
    case LogLevel::kDebug: return "DEBUG";
    case LogLevel::kInfo: return "INFO";
    case LogLevel::kWarn: return "WARN";
    case LogLevel::kError: return "ERROR";
    default: return "?";
    }
}

thread_local char t_last_error[512] = {0};
std::mutex g_write_mu;

}  // namespace

LogLevel CurrentLogLevel() { return static_cast<LogLevel>(LevelStore().load(std::memory_order_relaxed)); }
void SetLogLevel(LogLevel level) { LevelStore().store(static_cast<int>(level)); }

void LogWrite(LogLevel level, const char* file, int line, const char* fmt, ...) {
    char msg[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(msg, sizeof(msg), fmt, ap);
    va_end(ap);
    auto now = std::chrono::system_clock::now();
    auto us = std::chrono::duration_cast<std::chrono::microseconds>(now.time_since_epoch()).count();
    time_t secs = static_cast<time_t>(us / 1000000);
    struct tm tmv;
    localtime_r(&secs, &tmv);
    char ts[32];
    strftime(ts, sizeof(ts), "%H:%M:%S", &tmv);
    const char* base = strrchr(file, '/');
    base = base ? base + 1 : file;
    std::lock_guard<std::mutex> lk(g_write_mu);
    fprintf(stderr, "[%s.%06lld bccl %s pid=%d %s:%d] %s\n", ts, static_cast<long long>(us % 1000000),
            LevelTag(level), static_cast<int>(getpid()), base, line, msg);
}

const char* LastErrorMessage() { return t_last_error; }

void SetLastError(const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(t_last_error, sizeof(t_last_error), fmt, ap);
    va_end(ap);
}

}  // namespace bccl
