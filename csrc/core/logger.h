// Level-filtered, timestamped logging to stderr.
//
// Parity: the reference's Logger singleton and LOG_* macros (OriginCCL include/logger.h:16-94).
// The level comes from BCCL_LOG_LEVEL (DEBUG | INFO | WARN | ERROR | NONE; default WARN).
// printf-style formatting keeps the library free of a formatting dependency.
#pragma once

#include <cstdarg>

namespace bccl {

enum class LogLevel : int { kDebug = 0, kInfo = 1, kWarn = 2, kError = 3, kNone = 4 };

LogLevel CurrentLogLevel();
void SetLogLevel(LogLevel level);
void LogWrite(LogLevel level, const char* file, int line, const char* fmt, ...)
    __attribute__((format(printf, 4, 5)));
// Last error message produced on this thread (kept for the C API's bcclGetLastError()).
const char* LastErrorMessage();
void SetLastError(const char* fmt, ...) __attribute__((format(printf, 1, 2)));

}  // namespace bccl

#define BCCL_LOG(level, ...)                                                  \
    do {                                                                      \
        if (static_cast<int>(level) >= static_cast<int>(::bccl::CurrentLogLevel())) \
            ::bccl::LogWrite(level, __FILE__, __LINE__, __VA_ARGS__);         \
    } while (0)

#define LOG_DEBUG(...) BCCL_LOG(::bccl::LogLevel::kDebug, __VA_ARGS__)
#define LOG_INFO(...) BCCL_LOG(::bccl::LogLevel::kInfo, __VA_ARGS__)
#define LOG_WARN(...) BCCL_LOG(::bccl::LogLevel::kWarn, __VA_ARGS__)
// Errors are always recorded as the thread's last error, even when not printed.
#define LOG_ERROR(...)                                                        \
    do {                                                                      \
        ::bccl::SetLastError(__VA_ARGS__);                                    \
        BCCL_LOG(::bccl::LogLevel::kError, __VA_ARGS__);                      \
    } while (0)
