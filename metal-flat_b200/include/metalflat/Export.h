// SPDX-License-Identifier: Apache-2.0
// metalflat/Export.h -- visibility of the C++ API.
//
// libmetalflat_c.so is built with hidden default visibility (its C ABI entry
// points carry MFLAT_API); the C++ classes and functions a C++ caller links
// against carry MFLAT_CXX_API, so the same library serves both.
#pragma once

#if defined(_WIN32)
#  define MFLAT_CXX_API
#else
#  define MFLAT_CXX_API __attribute__((visibility("default")))
#endif
