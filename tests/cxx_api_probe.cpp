// cxx_api_probe.cpp -- a C++ caller of the metalflat C++ API, linked against
// libmetalflat_c.so, for the CPU test suite (no CUDA device needed): the
// exported classes and functions resolve, exceptions cross the library
// boundary, and the host-side pieces (log level, index-file header,
// k-means seed permutation) behave as specified.  argv[1]: an index file.
#include <cstdio>
#include <stdexcept>
#include <vector>

#include "metalflat/CoarseQuantizer.h"
#include "metalflat/FlatIndex.h"
#include "metalflat/Log.h"

int main(int argc, char** argv) {
    mflat::setLogLevel(mflat::LogLevel::Off);
    std::printf("loglevel %d\n", static_cast<int>(mflat::logLevel()));

    mflat::FlatIndex idx(8, mflat::Metric::InnerProduct);
    std::printf("index %d %d %d %d\n", idx.ready() ? 1 : 0, idx.dim(), idx.size(),
                static_cast<int>(idx.metric()));
    std::vector<float> q(8, 0.0f);
    std::vector<int32_t> ids(5);
    std::vector<float> dist(5);
    try {
        idx.search(q.data(), 1, 5);
        std::printf("search returned\n");
    } catch (const mflat::DeviceError&) {
        std::printf("search DeviceError\n");
    }
    try {
        idx.searchInto(q.data(), 1, 5, ids.data(), dist.data());
        std::printf("searchInto returned\n");
    } catch (const mflat::DeviceError&) {
        std::printf("searchInto DeviceError\n");
    }
    std::printf("empty %d\n", idx.searchInto(q.data(), 0, 5, ids.data(), dist.data()));

    int dim = 0, n = 0;
    mflat::Metric metric = mflat::Metric::L2;
    mflat::Storage storage = mflat::Storage::FP32;
    const bool ok = argc > 1 && mflat::readFlatFileInfo(argv[1], dim, metric, storage, n);
    std::printf("info %d %d %d %d %d\n", ok ? 1 : 0, dim, static_cast<int>(metric),
                static_cast<int>(storage), n);

    try {
        mflat::CoarseQuantizer bad(0);
        std::printf("coarse_dim0 constructed\n");
    } catch (const std::invalid_argument&) {
        std::printf("coarse_dim0 invalid_argument\n");
    }
    mflat::CoarseQuantizer cq(8);
    std::printf("coarse %d %d %d\n", cq.dim(), cq.nlist(), cq.size());
    try {
        cq.setShard(2, 2, nullptr, nullptr);
        std::printf("coarse_shard accepted\n");
    } catch (const std::invalid_argument&) {
        std::printf("coarse_shard invalid_argument\n");
    }
    std::vector<float> pts(8 * 64, 0.5f);
    try {
        cq.train(pts.data(), 64, 4, 2);
        std::printf("coarse_train returned\n");
    } catch (const mflat::DeviceError&) {
        std::printf("coarse_train DeviceError\n");
    }

    std::vector<int> perm;
    mflat::kmeansSeedPermutation(37, 12345u, perm);
    std::printf("perm");
    for (int v : perm) std::printf(" %d", v);
    std::printf("\n");
    return 0;
}
