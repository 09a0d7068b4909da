// SPDX-License-Identifier: Apache-2.0
// metalflat/Metric.h -- distance / similarity metrics for flat (exact) search.
// Same enumerators and values as the reference (include/metalflat/Metric.h:10-20).
#pragma once

namespace mflat {

enum class Metric {
    L2,            // squared Euclidean distance, smaller = nearer
    InnerProduct,  // dot product, larger = nearer, vectors used as-is
    Cosine,        // dot product of L2-normalised copies, larger = nearer
};

}  // namespace mflat
