// cxx_load_probe.cpp -- FlatIndex::load into an index that already holds rows
// (C++ API, run on a GPU by tests/test_gpu_persist.py).  argv[1]: a complete
// index file, argv[2]: the same file truncated.  Prints "ok" when a failed
// (truncated) load leaves the index's rows and results unchanged and the
// complete file then replaces them.
#include <cstdio>
#include <vector>

#include "metalflat/FlatIndex.h"
#include "metalflat/Log.h"

int main(int argc, char** argv) {
    if (argc < 3) return 2;
    mflat::setLogLevel(mflat::LogLevel::Off);
    const int dim = 37, n = 500, k = 7;
    std::vector<float> rows(static_cast<size_t>(n) * dim), q(3 * dim);
    for (size_t i = 0; i < rows.size(); ++i) rows[i] = static_cast<float>((i * 2654435761u) % 1000) / 997.0f;
    for (size_t i = 0; i < q.size(); ++i) q[i] = static_cast<float>((i * 40503u) % 1000) / 991.0f;
    mflat::FlatIndex idx(dim, mflat::Metric::L2, mflat::Storage::FP32);
    idx.add(rows.data(), n);
    std::vector<int32_t> id0(3 * k), id1(3 * k);
    std::vector<float> d0(3 * k), d1(3 * k);
    idx.searchInto(q.data(), 3, k, id0.data(), d0.data());
    if (idx.load(argv[2])) { std::printf("truncated file accepted\n"); return 1; }
    if (idx.size() != n) { std::printf("size changed to %d\n", idx.size()); return 1; }
    idx.searchInto(q.data(), 3, k, id1.data(), d1.data());
    if (id0 != id1 || d0 != d1) { std::printf("results changed\n"); return 1; }
    if (!idx.load(argv[1])) { std::printf("complete file rejected\n"); return 1; }
    std::printf("ok %d\n", idx.size());
    return 0;
}
