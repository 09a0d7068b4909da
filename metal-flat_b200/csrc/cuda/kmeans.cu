// kmeans.cu -- the k-means assignment step on the flat-search kernel pair.
//
// Reference: the final all-points assignment of kmeansGpu
// (src/Internal.h:321-359, kernel kmeans_assign_reg :138-183) and its
// GEMM fallback through FlatIndex::search(k=1) (:366-381); the CPU rule the
// result must reproduce bit-for-bit is src/CoarseQuantizer.mm:122-130
// (argmin of the fp32 sequential sqL2 of Distance.h:33-37, strict '<').
// Here every dimension uses the same path: the centroids become a temporary
// L2 index, the points are screened with the tcgen05 kernel (top-4), and the
// select stage re-checks the near-ties with the reference's exact fp32
// operation order.
#include <cuda_runtime.h>

#include <climits>
#include <cmath>
#include <map>
#include <mutex>
#include <utility>

#include "index_impl.cuh"
#include "kernels.cuh"
#include "mflat_cuda.h"

using namespace mflat_cu;

extern "C" int mflat_cu_kmeans_assign(const float* points, int64_t n, const float* centroids,
                                      int ncentroids, int dim, int32_t* out_assign, int device,
                                      int on_device, void* stream) {
    if (n < 0 || ncentroids < 1 || dim < 1) return fail(ST_BAD_ARG, "bad argument");
    if (n == 0) return ST_OK;
    if (!points || !centroids || !out_assign) return fail(ST_BAD_ARG, "null argument");
    if (n > INT_MAX - kBM) return fail(ST_BAD_ARG, "too many points for one call");
    // One assignment index per (device, dim), reused across calls so that
    // repeated k-means iterations do not re-allocate their scratch; calls on
    // the same device are serialised by the cache mutex.
    device = mflat_cu_default_device(device);
    static std::mutex cache_mu;
    static std::map<std::pair<int, int>, mflat_cu_index*> cache;
    std::lock_guard<std::mutex> lk(cache_mu);
    mflat_cu_index*& ix = cache[{device, dim}];
    int rc;
    if (!ix) {
        rc = mflat_cu_index_create(device, dim, kL2, 0, &ix);
        if (rc != ST_OK) {
            ix = nullptr;
            return rc;
        }
    } else {
        rc = mflat_cu_index_reset(ix);
        if (rc != ST_OK) return rc;
    }
    DeviceGuard g(ix->device);
    cudaStream_t st = on_device ? static_cast<cudaStream_t>(stream) : ix->stream;
    rc = mflat_cu_index_add(ix, centroids, ncentroids, on_device, stream);
    if (rc != ST_OK) return rc;

    const int m = static_cast<int>(n);
    ScreenRun run;
    rc = run_screen(ix, points, m, 4, on_device, st, run, 32);
    if (rc != ST_OK) return rc;
    CU_TRY(ix->flag_list.ensure(static_cast<size_t>(m) * sizeof(int)), "fallback list");
    cudaMemsetAsync(ix->flag_count, 0, sizeof(int), st);

    int32_t* d_out = out_assign;
    if (!on_device) {
        CU_TRY(ix->out_ids.ensure(static_cast<size_t>(m) * sizeof(int32_t)), "result buffer");
        d_out = ix->out_ids.as<int32_t>();
    }
    SelectParams sel{};
    sel.m = m;
    sel.m_pad = run.m_pad;
    sel.dim = dim;
    sel.d_pad = ix->d_pad;
    sel.k_out = 1;
    sel.n_chunks = run.n_lists;
    sel.metric = kL2;
    sel.n = ix->n;
    sel.part_score = run.part_s;
    sel.part_id = run.part_i;
    sel.q_x = run.q_x;
    sel.qnorm = run.qnorm;
    sel.db_x = ix->db_x;
    sel.xmax_bits = ix->xmax_bits;
    sel.gamma = screen_gamma(ix->d_pad);
    sel.flag_count = ix->flag_count;
    sel.flag_list = ix->flag_list.as<int>();
    sel.err = ix->err;
    CU_TRY(launch_kmeans_select(sel, d_out, ix->num_sms, st), "assignment launch");
    cudaMemcpyAsync(&ix->host_words[0], ix->err, sizeof(int), cudaMemcpyDeviceToHost, st);
    if (!on_device)
        CU_TRY(cudaMemcpyAsync(out_assign, d_out, static_cast<size_t>(m) * sizeof(int32_t),
                               cudaMemcpyDeviceToHost, st),
               "download");
    // The cached index's scratch is reused by the next call: finish first.
    CU_TRY(cudaStreamSynchronize(st), "assignment");
    return check_device_error(ix, st);
}
