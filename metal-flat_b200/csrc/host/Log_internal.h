// SPDX-License-Identifier: Apache-2.0
// Log_internal.h -- library-internal logging entry points and MFLAT_LOG_*
// macros.  The macros test the threshold before evaluating their arguments,
// as the reference's src/Log_internal.h:21-26 does.
#pragma once

#include "metalflat/Log.h"

namespace mflat {
namespace detail {

bool logEnabled(LogLevel level);
void logMessage(LogLevel level, const char* msg);
void logf(LogLevel level, const char* fmt, ...) __attribute__((format(printf, 2, 3)));

}  // namespace detail
}  // namespace mflat

#define MFLAT_LOG_AT(lvl, ...)                                                \
    do {                                                                      \
        if (::mflat::detail::logEnabled(lvl)) ::mflat::detail::logf(lvl, __VA_ARGS__); \
    } while (0)
#define MFLAT_LOG_ERROR(...) MFLAT_LOG_AT(::mflat::LogLevel::Error, __VA_ARGS__)
#define MFLAT_LOG_WARN(...)  MFLAT_LOG_AT(::mflat::LogLevel::Warn, __VA_ARGS__)
#define MFLAT_LOG_INFO(...)  MFLAT_LOG_AT(::mflat::LogLevel::Info, __VA_ARGS__)
