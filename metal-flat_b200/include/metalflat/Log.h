// SPDX-License-Identifier: Apache-2.0
// metalflat/Log.h -- process-global log sink control (same API and semantics as
// the reference's include/metalflat/Log.h:11-33).
//
// Default sink: stderr, "[metalflat] <level>: <message>".  A handler replaces
// it; handler == nullptr restores it; LogLevel::Off silences everything.
// Handlers run synchronously on the logging thread and must not throw.
#pragma once

#include "metalflat/Export.h"

namespace mflat {

enum class LogLevel : int { Info = 0, Warn = 1, Error = 2, Off = 3 };

using LogHandler = void (*)(LogLevel level, const char* msg, void* user);

MFLAT_CXX_API void     setLogHandler(LogHandler handler, void* user = nullptr);
MFLAT_CXX_API void     setLogLevel(LogLevel threshold);
MFLAT_CXX_API LogLevel logLevel();

}  // namespace mflat
