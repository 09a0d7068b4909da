// SPDX-License-Identifier: Apache-2.0
// Log.cpp -- process-global log sink and threshold.
//
// Behaviour follows the reference's src/Log.cpp:11-62: lock-free atomics
// (constant-initialised, safe during static init / teardown), a handler of
// nullptr means the built-in stderr sink, the threshold Off drops all
// messages, and a message is formatted only when it will be delivered.
#include <atomic>
#include <cstdarg>
#include <cstdio>

#include "Log_internal.h"
#include "metalflat/Log.h"

namespace mflat {
namespace {

std::atomic<LogHandler> g_handler{nullptr};
std::atomic<void*> g_user{nullptr};
std::atomic<int> g_threshold{static_cast<int>(LogLevel::Info)};

const char* level_tag(LogLevel l) {
    switch (l) {
        case LogLevel::Error: return "error";
        case LogLevel::Warn: return "warn";
        default: return "info";
    }
}

void stderr_sink(LogLevel l, const char* msg) {
    std::fprintf(stderr, "[metalflat] %s: %s\n", level_tag(l), msg);
}

}  // namespace

void setLogHandler(LogHandler handler, void* user) {
    g_user.store(user, std::memory_order_release);
    g_handler.store(handler, std::memory_order_release);
}

void setLogLevel(LogLevel threshold) {
    g_threshold.store(static_cast<int>(threshold), std::memory_order_relaxed);
}

LogLevel logLevel() { return static_cast<LogLevel>(g_threshold.load(std::memory_order_relaxed)); }

namespace detail {

bool logEnabled(LogLevel level) {
    const int t = g_threshold.load(std::memory_order_relaxed);
    return t != static_cast<int>(LogLevel::Off) && static_cast<int>(level) >= t;
}

void logMessage(LogLevel level, const char* msg) {
    if (!logEnabled(level)) return;
    LogHandler h = g_handler.load(std::memory_order_acquire);
    if (h) {
        h(level, msg, g_user.load(std::memory_order_acquire));
        return;
    }
    stderr_sink(level, msg);
}

void logf(LogLevel level, const char* fmt, ...) {
    if (!logEnabled(level)) return;
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    const int n = std::vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    if (n < 0) return;
    logMessage(level, buf);
}

}  // namespace detail
}  // namespace mflat
