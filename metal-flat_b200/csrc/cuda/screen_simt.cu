// screen_simt.cu -- CUDA-core screen with exactly the inputs and outputs of
// the tcgen05 kernel (per (query, chunk) top-KP lists).  It is the
// independent GPU cross-check of screen.cu (fp32 storage), selected with
// MFLAT_SCREEN=simt; the fp32 dot product here is computed directly from the
// stored fp32 rows, in index order.
#include "kernels.cuh"
#include "ptx.cuh"

namespace mflat_cu {
namespace {

template <int KP>
__global__ void __launch_bounds__(128) screen_simt_kernel(const ScreenParams p) {
    const int qt = blockIdx.x;
    const int ch = blockIdx.y;
    const int row = qt * kBM + threadIdx.x;
    const int64_t t0 = static_cast<int64_t>(ch) * p.tiles_per_chunk;
    const int64_t t1 = min(t0 + p.tiles_per_chunk, static_cast<int64_t>(p.n_tiles));
    TopList<KP> L;
    L.init();
    if (row < p.m) {
        const float* qx = p.q_x + static_cast<int64_t>(row) * p.d_pad;
        for (int64_t t = t0; t < t1; ++t) {
            const int64_t j0 = t * p.tile_stride * kBN;
            const int64_t j1 = min(j0 + kBN, p.n);
            for (int64_t j = j0; j < j1; ++j) {
                const float* x = p.db_x + j * p.d_pad;
                float acc = 0.0f;
                for (int c = 0; c < p.d_pad; ++c) acc = fmaf(qx[c], x[c], acc);
                const float s = fmaf(p.alpha, acc, p.colbias[j]);
                if (s > L.worst()) L.insert(s, static_cast<int>(j));
            }
        }
        const int64_t o = (static_cast<int64_t>(ch) * p.m_pad + row) * KP;
        for (int i = 0; i < KP; ++i) {
            p.part_score[o + i] = L.s[i];
            p.part_id[o + i] = L.id[i];
        }
    }
}

// Buffer mode: append every score at or above the query's floor.
__global__ void __launch_bounds__(128) screen_simt_buffer_kernel(const ScreenParams p) {
    const int qt = blockIdx.x;
    const int ch = blockIdx.y;
    const int row = qt * kBM + threadIdx.x;
    if (row >= p.m) return;
    const int64_t t0 = static_cast<int64_t>(ch) * p.tiles_per_chunk;
    const int64_t t1 = min(t0 + p.tiles_per_chunk, static_cast<int64_t>(p.n_tiles));
    const float floor_adj = floor_below(p.thr[row]);
    const float* qx = p.q_x + static_cast<int64_t>(row) * p.d_pad;
    for (int64_t t = t0; t < t1; ++t) {
        const int64_t j0 = t * p.tile_stride * kBN;
        const int64_t j1 = min(j0 + kBN, p.n);
        for (int64_t j = j0; j < j1; ++j) {
            const float* x = p.db_x + j * p.d_pad;
            float acc = 0.0f;
            for (int c = 0; c < p.d_pad; ++c) acc = fmaf(qx[c], x[c], acc);
            const float s = fmaf(p.alpha, acc, p.colbias[j]);
            if (s > floor_adj) {
                const uint32_t slot = atomicAdd(p.buf_cnt + row, 1u);
                if (slot < p.cap) {
                    p.buf_s[static_cast<int64_t>(row) * p.cap + slot] = s;
                    p.buf_i[static_cast<int64_t>(row) * p.cap + slot] = static_cast<int>(j);
                }
            }
        }
    }
}

template <int KP>
cudaError_t launch_kp(const ScreenParams& p, cudaStream_t stream) {
    dim3 grid(p.n_qtiles, p.n_chunks);
    screen_simt_kernel<KP><<<grid, kBM, 0, stream>>>(p);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_screen_simt(int kp, const ScreenParams& p, cudaStream_t stream) {
    switch (kp) {
        case 0: {
            dim3 grid(p.n_qtiles, p.n_chunks);
            screen_simt_buffer_kernel<<<grid, kBM, 0, stream>>>(p);
            return cudaGetLastError();
        }
        case 4: return launch_kp<4>(p, stream);
        case 8: return launch_kp<8>(p, stream);
        case 16: return launch_kp<16>(p, stream);
        case 32: return launch_kp<32>(p, stream);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace mflat_cu
