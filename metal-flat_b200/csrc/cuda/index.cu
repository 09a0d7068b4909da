// index.cu -- device-side flat index behind the extern "C" layer
// (mflat_cuda.h).  The host engine (FlatIndex.cpp) owns argument checking,
// k clamping and logging; this file owns device memory, streams, kernel
// orchestration and the device error word.
//
// Replaces the device half of the reference's FlatIndex::Impl
// (src/FlatIndex.mm:137-189 buffers, :160-178 ensureBuffer, :294-421 search
// tile loop) with a device-authoritative layout: rows are appended on the
// device (no host copy, no whole-database re-upload per add) and norms are
// computed on the device with the reference's double accumulation
// (src/Distance.h:40-60).
#include <cudaTypedefs.h>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>

#include "index_impl.cuh"
#include "kernels.cuh"
#include "mflat_cuda.h"
#include "ptx.cuh"

namespace mflat_cu {

namespace {
thread_local std::string g_last_error;
}

int fail(int status, const char* what, cudaError_t e) {
    char buf[512];
    if (e != cudaSuccess)
        std::snprintf(buf, sizeof buf, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
    else
        std::snprintf(buf, sizeof buf, "%s", what);
    g_last_error = buf;
    return status;
}

const char* last_error_message() { return g_last_error.c_str(); }

cudaError_t DevBuf::ensure(size_t need) {
    if (need <= bytes) return cudaSuccess;
    if (p) cudaFree(p);
    p = nullptr;
    bytes = 0;
    const size_t want = need + need / 4;
    cudaError_t e = cudaMalloc(&p, want);
    if (e != cudaSuccess) { p = nullptr; return e; }
    bytes = want;
    return cudaSuccess;
}

void DevBuf::release() {
    if (p) cudaFree(p);
    p = nullptr;
    bytes = 0;
}

DeviceGuard::DeviceGuard(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
}

DeviceGuard::~DeviceGuard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
}

namespace {

const float kInf = INFINITY;

// ------------------------------------------------------------- TMA encode
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

bool get_encoder() {
    std::call_once(g_encode_once, [] {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    });
    return g_encode != nullptr;
}

// 16-bit rows [rows][inner] (fp16 / bf16 bits): box [box_rows][64 halves].
bool make_map_u16(CUtensorMap* map, const void* base, uint64_t inner, uint64_t rows,
                  uint32_t box_rows) {
    if (!get_encoder()) return false;
    cuuint64_t dims[2] = {inner, rows};
    cuuint64_t strides[1] = {inner * 2};
    cuuint32_t box[2] = {64u, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void*>(base), dims,
                          strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                          CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

// Bias parts of the screens' bias MMA: [rows][8] bf16 (h, m, l, zeros),
// 8-wide boxes of box_rows rows (a CTA's share of a tile), no swizzle (the
// MMA's K-major core-matrix layout).
bool make_map_bias16(CUtensorMap* map, const void* base, uint64_t rows, uint32_t box_rows) {
    if (!get_encoder()) return false;
    cuuint64_t dims[2] = {8, rows};
    cuuint64_t strides[1] = {16};
    cuuint32_t box[2] = {8u, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void*>(base), dims,
                          strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                          CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

// ------------------------------------------------------------- kernels
// b = colbias * scale (scale = 1 / alpha, an exact power of two) as
// h + m + l: h and m truncated to bf16 (round toward zero), l the remainder
// (8 bits, exact).  The three parts share b's sign and cover disjoint bit
// ranges of its 24-bit significand, so every partial sum is exact in fp32 and
// the tensor core's addition order cannot change the result.  -inf (rows past
// n) becomes (-inf, 0, 0).  Rows [row0, row1).
__global__ void split_bias_kernel(const float* __restrict__ colbias, int64_t row0, int64_t row1,
                                  float scale, uint4* __restrict__ out) {
    const int64_t i = row0 + static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= row1) return;
    const float b = scale * colbias[i];
    uint16_t h, m = 0, l = 0;
    if (isinf(b)) {
        h = __bfloat16_as_ushort(__float2bfloat16_rn(b));
    } else {
        const __nv_bfloat16 hb = __float2bfloat16_rz(b);
        const float r1 = b - __bfloat162float(hb);
        const __nv_bfloat16 mb = __float2bfloat16_rz(r1);
        const float r2 = r1 - __bfloat162float(mb);
        h = __bfloat16_as_ushort(hb);
        m = __bfloat16_as_ushort(mb);
        l = __bfloat16_as_ushort(__float2bfloat16_rn(r2));
    }
    out[i] = make_uint4(static_cast<uint32_t>(h) | (static_cast<uint32_t>(m) << 16), l, 0u, 0u);
}

// fp32 -> 16-bit storage bits, round to nearest even.
__device__ __forceinline__ uint16_t to_half_bits(float x, bool bf16) {
    if (bf16) return __bfloat16_as_ushort(__float2bfloat16_rn(x));
    return __half_as_ushort(__float2half_rn(x));
}
__device__ __forceinline__ float from_half_bits(uint16_t u, bool bf16) {
    return bf16 ? __bfloat162float(__ushort_as_bfloat16(u)) : __half2float(__ushort_as_half(u));
}

// 16-bit storage ingest: Cosine normalisation as for fp32 (Distance.h:50-60),
// then conversion; the norm term is that of the stored 16-bit row.
__global__ void ingest_rows_half_kernel(const float* __restrict__ src, int64_t n, int dim, int d_pad,
                                        int metric, bool bf16, int64_t row0, uint16_t* __restrict__ db,
                                        float* __restrict__ colbias, float* __restrict__ dnorm) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float* row = src + i * dim;
    uint16_t* o = db + (row0 + i) * d_pad;
    float inv = 1.0f;
    bool scale = false;
    if (metric == kCosine) {
        double s = 0.0;
        for (int c = 0; c < dim; ++c) s += static_cast<double>(row[c]) * row[c];
        if (s > 0.0) { inv = static_cast<float>(1.0 / sqrt(s)); scale = true; }
    }
    double s2 = 0.0;
    for (int c = 0; c < dim; ++c) {
        const uint16_t h = to_half_bits(scale ? row[c] * inv : row[c], bf16);
        const float x = from_half_bits(h, bf16);
        s2 += static_cast<double>(x) * x;
        o[c] = h;
    }
    for (int c = dim; c < d_pad; ++c) o[c] = 0;
    dnorm[row0 + i] = static_cast<float>(s2);
    colbias[row0 + i] = metric == kL2 ? -static_cast<float>(s2) : 0.0f;
}

// 16-bit rows that are already stored values (a reloaded index): copied bit
// for bit; the norm term is recomputed from them exactly as at first ingest.
__global__ void ingest_rows_bits_kernel(const uint16_t* __restrict__ src, int64_t n, int dim,
                                        int d_pad, int metric, bool bf16, int64_t row0,
                                        uint16_t* __restrict__ db, float* __restrict__ colbias,
                                        float* __restrict__ dnorm) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const uint16_t* row = src + i * dim;
    uint16_t* o = db + (row0 + i) * d_pad;
    double s2 = 0.0;
    for (int c = 0; c < dim; ++c) {
        const float x = from_half_bits(row[c], bf16);
        s2 += static_cast<double>(x) * x;
        o[c] = row[c];
    }
    for (int c = dim; c < d_pad; ++c) o[c] = 0;
    dnorm[row0 + i] = static_cast<float>(s2);
    colbias[row0 + i] = metric == kL2 ? -static_cast<float>(s2) : 0.0f;
}

// Stored rows [row0, row0 + n) in storage precision without padding: fp32
// rows as ingested, 16-bit rows bit for bit.
__global__ void export_rows_f32_kernel(const float* __restrict__ db_x, int64_t row0, int64_t n,
                                       int dim, int d_pad, float* __restrict__ out) {
    const int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (e >= n * dim) return;
    const int64_t r = e / dim;
    const int c = static_cast<int>(e - r * dim);
    out[e] = db_x[(row0 + r) * d_pad + c];
}

__global__ void export_rows_bits_kernel(const uint16_t* __restrict__ db, int64_t row0, int64_t n,
                                        int dim, int d_pad, uint16_t* __restrict__ out) {
    const int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (e >= n * dim) return;
    const int64_t r = e / dim;
    const int c = static_cast<int>(e - r * dim);
    out[e] = db[(row0 + r) * d_pad + c];
}

// 16-bit query preparation (Cosine normalisation, rounding to the storage
// type, sum of squares of the rounded values): 32 rows per 128-thread block
// through shared memory in 64-column slabs, so global reads and writes are
// coalesced; each row's arithmetic stays with one thread in ascending
// coordinate order, the same operations as the per-row form.
constexpr int kHalfPrepRows = 32;
constexpr int kHalfPrepCols = 64;

__global__ void __launch_bounds__(128) prep_queries_half_kernel(const float* __restrict__ src, int m, int m_pad,
                                                                int dim, int d_pad, int metric, bool bf16,
                                                                uint16_t* __restrict__ q, float* __restrict__ qsq) {
    __shared__ float tin[kHalfPrepRows][kHalfPrepCols + 1];
    __shared__ uint16_t tq[kHalfPrepRows][kHalfPrepCols + 2];
    const int r0 = blockIdx.x * kHalfPrepRows;
    const int t = threadIdx.x;
    const int row = r0 + t;
    const bool own = t < kHalfPrepRows && row < m_pad;   // this thread's row
    const bool live = own && row < m;
    auto load = [&](int c0) {
        for (int i = t; i < kHalfPrepRows * kHalfPrepCols; i += blockDim.x) {
            const int rr = i / kHalfPrepCols, cc = i % kHalfPrepCols;
            const int r = r0 + rr, c = c0 + cc;
            tin[rr][cc] = (r < m && c < dim) ? src[static_cast<int64_t>(r) * dim + c] : 0.0f;
        }
    };
    float inv = 1.0f;
    bool scale = false;
    if (metric == kCosine) {
        double s = 0.0;
        for (int c0 = 0; c0 < dim; c0 += kHalfPrepCols) {
            load(c0);
            __syncthreads();
            if (live)
                for (int cc = 0; cc < kHalfPrepCols && c0 + cc < dim; ++cc)
                    s += static_cast<double>(tin[t][cc]) * tin[t][cc];
            __syncthreads();
        }
        if (live && s > 0.0) { inv = static_cast<float>(1.0 / sqrt(s)); scale = true; }
    }
    double s2 = 0.0;
    for (int c0 = 0; c0 < d_pad; c0 += kHalfPrepCols) {
        load(c0);
        __syncthreads();
        if (own) {
            for (int cc = 0; cc < kHalfPrepCols; ++cc) {
                uint16_t h = 0;
                if (live && c0 + cc < dim) {
                    h = to_half_bits(scale ? tin[t][cc] * inv : tin[t][cc], bf16);
                    const float x = from_half_bits(h, bf16);
                    s2 += static_cast<double>(x) * x;
                }
                tq[t][cc] = h;
            }
        }
        __syncthreads();
        for (int i = t; i < kHalfPrepRows * kHalfPrepCols; i += blockDim.x) {
            const int rr = i / kHalfPrepCols, cc = i % kHalfPrepCols;
            const int r = r0 + rr, c = c0 + cc;
            if (r < m_pad && c < d_pad) q[static_cast<int64_t>(r) * d_pad + c] = tq[rr][cc];
        }
        __syncthreads();
    }
    if (own) qsq[row] = live ? static_cast<float>(s2) : 0.0f;
}

// x ~ h + l: h = bf16(x), l = bf16(x - h), both round to nearest (x - h is
// exact in fp32); |x - h - l| <= 2^-8 |x - h| <= 2^-16 |x|.
__device__ __forceinline__ void split_bf16(float x, uint16_t& h, uint16_t& l) {
    const __nv_bfloat16 hb = __float2bfloat16_rn(x);
    h = __bfloat16_as_ushort(hb);
    l = __bfloat16_as_ushort(__float2bfloat16_rn(x - __bfloat162float(hb)));
}

// One thread per row: optional Cosine normalisation (src/Distance.h:50-60),
// squared norm with double accumulation (Distance.h:40-47), the stored fp32
// row and its bf16 split planes, zero padding to d_pad, score bias and running
// max row norm.  `normalize` = 0 for rows that are already stored values (a
// reloaded index).
__global__ void ingest_rows_kernel(const float* __restrict__ src, int64_t n, int dim, int d_pad,
                                   int metric, int normalize, int64_t row0, float* __restrict__ db_x,
                                   uint16_t* __restrict__ db_h, uint16_t* __restrict__ db_l,
                                   float* __restrict__ colbias, float* __restrict__ dnorm,
                                   unsigned* xmax_bits) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float* row = src + i * dim;
    float* ox = db_x + (row0 + i) * d_pad;
    uint16_t* oh = db_h + (row0 + i) * d_pad;
    uint16_t* ol = db_l + (row0 + i) * d_pad;
    float inv = 1.0f;
    bool scale = false;
    if (metric == kCosine && normalize) {
        double s = 0.0;
        for (int c = 0; c < dim; ++c) s += static_cast<double>(row[c]) * row[c];
        if (s > 0.0) { inv = static_cast<float>(1.0 / sqrt(s)); scale = true; }
    }
    double s2 = 0.0;
    for (int c = 0; c < dim; ++c) {
        const float x = scale ? row[c] * inv : row[c];
        s2 += static_cast<double>(x) * x;
        uint16_t h, l;
        split_bf16(x, h, l);
        ox[c] = x;
        oh[c] = h;
        ol[c] = l;
    }
    for (int c = dim; c < d_pad; ++c) { ox[c] = 0.0f; oh[c] = 0; ol[c] = 0; }
    const float dn = static_cast<float>(s2);
    dnorm[row0 + i] = dn;
    colbias[row0 + i] = metric == kL2 ? -dn : 0.0f;
    const float nrm = static_cast<float>(sqrt(s2) * (1.0 + 1e-7));   // rounded up
    atomicMax(xmax_bits, __float_as_uint(nrm));
}

// Query preparation: Cosine normalisation, the fp32 query and its bf16 split,
// ||q|| (rounded up) for the error bound; rows >= m are zero.  32 rows per
// 128-thread block pass through shared memory in 64-column slabs, so every
// global read and write is coalesced (one thread per row walked its own row
// before, which made the k-means step's 10M points cost 36 ms).  Each row's
// arithmetic stays with one thread in ascending coordinate order: the same
// operations, bit for bit, as the per-row form (src/Distance.h:40-60).
constexpr int kPrepRows = 32;
constexpr int kPrepCols = 64;

__global__ void __launch_bounds__(128) prep_queries_kernel(const float* __restrict__ src, int m, int m_pad,
                                                           int dim, int d_pad, int metric,
                                                           float* __restrict__ q_x, uint16_t* __restrict__ q_h,
                                                           uint16_t* __restrict__ q_l, float* __restrict__ qnorm) {
    __shared__ float tin[kPrepRows][kPrepCols + 1];
    __shared__ float tx[kPrepRows][kPrepCols + 1];
    __shared__ uint16_t th[kPrepRows][kPrepCols + 2];
    __shared__ uint16_t tl[kPrepRows][kPrepCols + 2];
    const int r0 = blockIdx.x * kPrepRows;
    const int t = threadIdx.x;
    const int row = r0 + t;
    const bool own = t < kPrepRows && row < m_pad;   // this thread's row
    const bool live = own && row < m;
    auto load = [&](int c0) {
        for (int i = t; i < kPrepRows * kPrepCols; i += blockDim.x) {
            const int rr = i / kPrepCols, cc = i % kPrepCols;
            const int r = r0 + rr, c = c0 + cc;
            tin[rr][cc] = (r < m && c < dim) ? src[static_cast<int64_t>(r) * dim + c] : 0.0f;
        }
    };
    float inv = 1.0f;
    bool scale = false;
    if (metric == kCosine) {
        double s = 0.0;
        for (int c0 = 0; c0 < dim; c0 += kPrepCols) {
            load(c0);
            __syncthreads();
            if (live)
                for (int cc = 0; cc < kPrepCols && c0 + cc < dim; ++cc)
                    s += static_cast<double>(tin[t][cc]) * tin[t][cc];
            __syncthreads();
        }
        if (live && s > 0.0) { inv = static_cast<float>(1.0 / sqrt(s)); scale = true; }
    }
    double s2 = 0.0;
    for (int c0 = 0; c0 < d_pad; c0 += kPrepCols) {
        load(c0);
        __syncthreads();
        if (own) {
            for (int cc = 0; cc < kPrepCols; ++cc) {
                float x = 0.0f;
                uint16_t h = 0, l = 0;
                if (live && c0 + cc < dim) {
                    x = scale ? tin[t][cc] * inv : tin[t][cc];
                    s2 += static_cast<double>(x) * x;
                    split_bf16(x, h, l);
                }
                tx[t][cc] = x;
                th[t][cc] = h;
                tl[t][cc] = l;
            }
        }
        __syncthreads();
        for (int i = t; i < kPrepRows * kPrepCols; i += blockDim.x) {
            const int rr = i / kPrepCols, cc = i % kPrepCols;
            const int r = r0 + rr, c = c0 + cc;
            if (r < m_pad && c < d_pad) {
                const int64_t o = static_cast<int64_t>(r) * d_pad + c;
                q_x[o] = tx[rr][cc];
                q_h[o] = th[rr][cc];
                q_l[o] = tl[rr][cc];
            }
        }
        __syncthreads();
    }
    if (own) qnorm[row] = live ? static_cast<float>(sqrt(s2) * (1.0 + 1e-7)) : 0.0f;
}

__global__ void fill_f32_kernel(float* p, int64_t n, float v) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < n) p[i] = v;
}

__global__ void fill_empty_kernel(int32_t* ids, float* dist, int64_t n, float v) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < n) { ids[i] = -1; dist[i] = v; }
}

cudaError_t grow(mflat_cu_index* ix, int64_t need) {
    if (need <= ix->cap) return cudaSuccess;
    cudaStream_t st = ix->stream;
    int64_t cap = std::max<int64_t>(need, ix->cap + ix->cap / 2);
    cap = (cap + kBN - 1) / kBN * kBN;
    // fp32 storage: x (4 B) + h, l (2 B each) per element; 16-bit: one plane
    void *x = nullptr, *h = nullptr, *l = nullptr, *bp = nullptr;
    float *cb = nullptr, *dn = nullptr;
    const bool half = ix->storage != 0;
    const size_t row16 = static_cast<size_t>(ix->d_pad) * 2;
    const size_t row32 = static_cast<size_t>(ix->d_pad) * sizeof(float);
    cudaError_t e;
    if ((e = cudaMalloc(&h, cap * row16)) != cudaSuccess) goto bad;
    if (!half && (e = cudaMalloc(&l, cap * row16)) != cudaSuccess) goto bad;
    if (!half && (e = cudaMalloc(&x, cap * row32)) != cudaSuccess) goto bad;
    if ((e = cudaMalloc(&cb, cap * sizeof(float))) != cudaSuccess) goto bad;
    if ((e = cudaMalloc(&dn, cap * sizeof(float))) != cudaSuccess) goto bad;
    if ((e = cudaMalloc(&bp, cap * sizeof(uint4))) != cudaSuccess) goto bad;
    if (ix->bias16_rows > 0)
        cudaMemcpyAsync(bp, ix->bias16, ix->bias16_rows * sizeof(uint4), cudaMemcpyDeviceToDevice, st);
    if (ix->n > 0) {
        cudaMemcpyAsync(h, half ? ix->db16 : static_cast<void*>(ix->db_h), ix->n * row16,
                        cudaMemcpyDeviceToDevice, st);
        if (!half) {
            cudaMemcpyAsync(l, ix->db_l, ix->n * row16, cudaMemcpyDeviceToDevice, st);
            cudaMemcpyAsync(x, ix->db_x, ix->n * row32, cudaMemcpyDeviceToDevice, st);
        }
        cudaMemcpyAsync(cb, ix->colbias, ix->n * sizeof(float), cudaMemcpyDeviceToDevice, st);
        cudaMemcpyAsync(dn, ix->dnorm, ix->n * sizeof(float), cudaMemcpyDeviceToDevice, st);
    }
    fill_f32_kernel<<<blocks_for(cap - ix->n, 256), 256, 0, st>>>(cb + ix->n, cap - ix->n, -kInf);
    if ((e = cudaStreamSynchronize(st)) != cudaSuccess) goto bad;
    cudaFree(ix->db16);
    cudaFree(ix->db_h);
    cudaFree(ix->db_l);
    cudaFree(ix->db_x);
    cudaFree(ix->colbias);
    cudaFree(ix->dnorm);
    cudaFree(ix->bias16);
    ix->bias16 = static_cast<uint4*>(bp);
    if (half) {
        ix->db16 = h;
    } else {
        ix->db_h = static_cast<uint16_t*>(h);
        ix->db_l = static_cast<uint16_t*>(l);
        ix->db_x = static_cast<float*>(x);
    }
    ix->colbias = cb;
    ix->dnorm = dn;
    ix->cap = cap;
    return cudaSuccess;
bad:
    cudaFree(bp);
    cudaFree(x);
    cudaFree(h);
    cudaFree(l);
    cudaFree(cb);
    cudaFree(dn);
    return e;
}

// Make `waiter` wait for everything enqueued so far on `producer`.
void order_after(cudaStream_t waiter, cudaStream_t producer) {
    if (waiter == producer) return;
    cudaEvent_t e;
    cudaEventCreateWithFlags(&e, cudaEventDisableTiming);
    cudaEventRecord(e, producer);
    cudaStreamWaitEvent(waiter, e, 0);
    cudaEventDestroy(e);
}

// Candidate-list length for the exact path: k plus a margin (>= 11 rows)
// that absorbs the rows whose screen scores fall inside the proven error
// band, so that the exact fallback stays rare.
int kp_for(int k) { return k <= 21 ? 32 : 0; }

// Bytes of one 256-row database tile as the screens read it.
size_t tile_bytes(const mflat_cu_index* ix) {
    return static_cast<size_t>(kBN) * ix->d_pad * (ix->storage != 0 ? 2 : 4);
}

}  // namespace

// Entry points for other translation units of this library (noalloc.cu).
bool encode_map_bf16(CUtensorMap* map, const void* base, uint64_t inner, uint64_t rows,
                     uint32_t box_rows) {
    return make_map_u16(map, base, inner, rows, box_rows);
}

cudaError_t launch_prep_queries(const float* src, int m, int m_pad, int dim, int d_pad, int metric,
                                float* q_x, uint16_t* q_h, uint16_t* q_l, float* qnorm,
                                cudaStream_t st) {
    prep_queries_kernel<<<blocks_for(m_pad, kPrepRows), 128, 0, st>>>(src, m, m_pad, dim, d_pad, metric,
                                                                      q_x, q_h, q_l, qnorm);
    return cudaGetLastError();
}

cudaError_t launch_fill_empty(int32_t* ids, float* dist, int64_t n, float v, cudaStream_t st) {
    fill_empty_kernel<<<blocks_for(n, 256), 256, 0, st>>>(ids, dist, n, v);
    return cudaGetLastError();
}

void plan_screen_chunks(int n_qtiles, int n_tiles, int num_sms, int max_chunks, int& n_chunks,
                        int& tiles_per_chunk) {
    plan_chunks(n_qtiles, n_tiles, num_sms, max_chunks, n_chunks, tiles_per_chunk);
}

int check_device_error(mflat_cu_index* ix, cudaStream_t st) {
    if (ix->host_words[0] != 0) {
        const int code = ix->host_words[0];
        ix->host_words[0] = 0;
        // cleared on the stream of the next kernels, ordered before them
        cudaMemsetAsync(ix->err, 0, sizeof(int), st);
        char buf[128];
        std::snprintf(buf, sizeof buf, "device kernel reported error code %d (%s)", code,
                      code == kErrTimeout ? "bounded wait timed out" : "bad launch configuration");
        return fail(ST_DEVICE, buf);
    }
    return ST_OK;
}

bool screen_pair_for(const mflat_cu_index* ix, int n_qtiles) {
    return screen_pair_for(ix->screen_pair && !ix->force_simt, n_qtiles);
}

int screen_grid(const mflat_cu_index* ix, int n_qtiles, int n_chunks, bool pair) {
    const int64_t units = static_cast<int64_t>(screen_qunits(n_qtiles, pair)) * n_chunks;
    const int slots = static_cast<int>(std::min<int64_t>(units, screen_slots(ix->num_sms, pair)));
    return pair ? 2 * slots : slots;
}

int prepare_bias_parts(mflat_cu_index* ix, cudaStream_t st, CUtensorMap* map, bool pair) {
    const int64_t rows_pad = (ix->n + kBN - 1) / kBN * kBN;
    if (rows_pad == 0 || !ix->bias16 || rows_pad > ix->cap)
        return fail(ST_INTERNAL, "screen bias parts: no rows");
    if (ix->bias16_rows < rows_pad) {
        const int64_t r0 = ix->bias16_rows;
        const float scale = ix->metric == kL2 ? 0.5f : 1.0f;   // 1 / alpha
        split_bias_kernel<<<blocks_for(rows_pad - r0, 256), 256, 0, st>>>(ix->colbias, r0, rows_pad,
                                                                          scale, ix->bias16);
        CU_TRY(cudaGetLastError(), "bias parts");
        ix->bias16_rows = rows_pad;
    }
    if (!make_map_bias16(map, ix->bias16, static_cast<uint64_t>(rows_pad),
                         static_cast<uint32_t>(screen_rows_per_cta(pair))))
        return fail(ST_DEVICE, "tensor map encoding failed");
    return ST_OK;
}

int fp32_lists_per_chunk(const mflat_cu_index* ix) {
    return ix->force_simt ? 1 : kScreenListsPerChunk;
}

// The fp32-storage screen over sp's query batch (bf16 planes in ix->q_h /
// ix->q_l, rows in ix->db_h / ix->db_l), or the CUDA-core cross-check.
cudaError_t launch_fp32_screen(mflat_cu_index* ix, const ScreenParams& sp_in, int kp, cudaStream_t st) {
    if (ix->force_simt) return launch_screen_simt(kp, sp_in, st);
    ScreenParams sp = sp_in;
    sp.wait_ns = ix->wait_ns;
    sp.test_stall = ix->test_stall;
    ix->test_stall = 0;
    const bool pair = screen_pair_for(ix, sp.n_qtiles);
    const uint32_t rows_b = static_cast<uint32_t>(screen_rows_per_cta(pair));
    ScreenMaps maps;
    if (!make_map_u16(&maps.a, ix->q_h.p, sp.d_pad, sp.m_pad, kBM) ||
        !make_map_u16(&maps.a2, ix->q_l.p, sp.d_pad, sp.m_pad, kBM) ||
        !make_map_u16(&maps.b, ix->db_h, sp.d_pad, ix->n, rows_b) ||
        !make_map_u16(&maps.b2, ix->db_l, sp.d_pad, ix->n, rows_b))
        return cudaErrorInvalidValue;
    if (prepare_bias_parts(ix, st, &maps.bias, pair) != ST_OK) return cudaErrorInvalidValue;
    return launch_screen(kp, ScreenKind::kBF16x3, maps, sp, screen_grid(ix, sp.n_qtiles, sp.n_chunks, pair),
                         pair, st);
}

int run_screen(mflat_cu_index* ix, const float* queries, int m, int kp, int on_device,
               cudaStream_t st, ScreenRun& out, int max_chunks) {
    const int m_pad = (m + kBM - 1) / kBM * kBM;
    const int d_pad = ix->d_pad;
    const int n_tiles = static_cast<int>((ix->n + kBN - 1) / kBN);
    const int n_qtiles = m_pad / kBM;
    int n_chunks = 1, tpc = n_tiles;
    const int lpc = fp32_lists_per_chunk(ix);
    const bool pair = screen_pair_for(ix, n_qtiles);
    plan_chunks(screen_qunits(n_qtiles, pair), n_tiles, screen_slots(ix->num_sms, pair), max_chunks / lpc,
                n_chunks, tpc);

    const float* qsrc = queries;
    if (!on_device) {
        CU_TRY(ix->q_in.ensure(static_cast<size_t>(m) * ix->dim * sizeof(float)), "query buffer");
        CU_TRY(cudaMemcpyAsync(ix->q_in.p, queries, static_cast<size_t>(m) * ix->dim * sizeof(float),
                               cudaMemcpyHostToDevice, st),
               "query upload");
        qsrc = ix->q_in.as<float>();
    }
    CU_TRY(ix->q_x.ensure(static_cast<size_t>(m_pad) * d_pad * sizeof(float)), "query buffer");
    CU_TRY(ix->q_h.ensure(static_cast<size_t>(m_pad) * d_pad * 2), "query split");
    CU_TRY(ix->q_l.ensure(static_cast<size_t>(m_pad) * d_pad * 2), "query split");
    CU_TRY(ix->qnorm.ensure(static_cast<size_t>(m_pad) * sizeof(float)), "query norms");
    const size_t parts = static_cast<size_t>(n_chunks) * lpc * m_pad * kp;
    CU_TRY(ix->part_s.ensure(parts * sizeof(float)), "candidate lists");
    CU_TRY(ix->part_i.ensure(parts * sizeof(int32_t)), "candidate lists");
    CU_TRY(ix->thr.ensure(static_cast<size_t>(m_pad) * sizeof(uint32_t)), "score floors");
    CU_TRY(cudaMemsetAsync(ix->thr.p, 0, static_cast<size_t>(m_pad) * sizeof(uint32_t), st), "floors");

    if (ix->timing) cudaEventRecord(ix->ev[0], st);
    CU_TRY(launch_prep_queries(qsrc, m, m_pad, ix->dim, d_pad, ix->metric, ix->q_x.as<float>(),
                               ix->q_h.as<uint16_t>(), ix->q_l.as<uint16_t>(), ix->qnorm.as<float>(), st),
           "query prep launch");

    ScreenParams sp{};
    sp.m = m;
    sp.m_pad = m_pad;
    sp.d_pad = d_pad;
    sp.n = ix->n;
    sp.n_tiles = n_tiles;
    sp.n_qtiles = n_qtiles;
    sp.n_chunks = n_chunks;
    sp.tiles_per_chunk = tpc;
    sp.alpha = ix->metric == kL2 ? 2.0f : 1.0f;
    sp.colbias = ix->colbias;
    sp.part_score = ix->part_s.as<float>();
    sp.part_id = ix->part_i.as<int32_t>();
    sp.err = ix->err;
    sp.thr = ix->thr.as<uint32_t>();
    sp.tile_stride = 1;
    sp.use_floor = 1;
    sp.q_x = ix->q_x.as<float>();
    sp.db_x = ix->db_x;

    if (ix->timing) cudaEventRecord(ix->ev[1], st);
    CU_TRY(launch_fp32_screen(ix, sp, kp, st), "screen launch");
    if (ix->timing) cudaEventRecord(ix->ev[2], st);

    out.kp = kp;
    out.m = m;
    out.m_pad = m_pad;
    out.n_chunks = n_chunks;
    out.n_lists = n_chunks * lpc;
    out.q_x = sp.q_x;
    out.qnorm = ix->qnorm.as<float>();
    out.part_s = sp.part_score;
    out.part_i = sp.part_id;
    out.launches = 2;
    return ST_OK;
}

// ---------------------------------------------------------------------------
// Large k (22..1024) on fp32 storage: strided-sample floor pre-pass (list
// mode), buffer-mode screen over every row, radix select + exact window
// re-rank (select_large.cu).  Queries are processed in batches sized so the
// candidate buffers stay within a fixed budget.
namespace {

// Bytes the candidate buffers of one query batch may take: a quarter of the
// device memory that is free or already held by this index's buffers, within
// [1 GB, 16 GB].  Fixed at the index's first large-k search, so the plan (and
// the buffers) of later searches do not follow the device's changing free
// memory, and no later search queries it.
size_t buffer_budget(mflat_cu_index* ix) {
    if (ix->lk_budget) return ix->lk_budget;
    size_t free_b = 0, total_b = 0;
    if (cudaMemGetInfo(&free_b, &total_b) != cudaSuccess) return size_t(4) << 30;
    const size_t held = ix->buf_s.bytes + ix->buf_i.bytes;
    ix->lk_budget = std::max<size_t>(size_t(1) << 30,
                                     std::min<size_t>(size_t(16) << 30, (free_b + held) / 4));
    return ix->lk_budget;
}

// Floor estimate for one query batch (see plan_large): stage A list-mode
// pass + union select, then (two-stage plans) stage B buffer-mode pass + the
// want-th best of each buffer (valid floor, in base.thr) and its r_stat-th
// best (statistical floor, in thr_stat).  list_pass / buffer_pass launch the storage's
// screen kernel; `base` carries the batch's queries and buffers.
template <class ListPass, class BufferPass>
int estimate_floor(mflat_cu_index* ix, const LargePlan& P, const ScreenParams& base, int want,
                   int kp1, int lists_per_chunk, ListPass list_pass, BufferPass buffer_pass,
                   uint32_t* thr_stat, int* words, cudaStream_t st) {
    ScreenParams pa = base;
    pa.use_floor = 0;
    pa.tile_stride = P.stride_a;
    pa.n_tiles = P.sample_a;
    pa.tiles_per_chunk = P.tpc_a;
    pa.n_chunks = P.chunks_a;
    CU_TRY(list_pass(pa, kp1), "floor pre-pass launch");
    const bool guess = P.two_stage && P.r_guess > 0;
    CU_TRY(launch_prepass_floor(pa.part_score, pa.part_id, pa.n_chunks * lists_per_chunk, base.m,
                                base.m_pad, kp1, want, guess ? P.r_guess : 0, base.thr,
                                guess ? thr_stat : nullptr, st),
           "floor launch");
    if (!P.two_stage) return ST_OK;
    ScreenParams pb = base;
    pb.use_floor = 1;
    pb.tile_stride = P.stride_b;
    pb.n_tiles = P.sample_b;
    int n_chunks = 1, tpc = P.sample_b;
    const bool pair = screen_pair_for(ix, pb.n_qtiles);
    plan_buffer_chunks(screen_qunits(pb.n_qtiles, pair), P.sample_b, screen_slots(ix->num_sms, pair),
                       tile_bytes(ix), n_chunks, tpc);
    pb.n_chunks = n_chunks;
    pb.tiles_per_chunk = tpc;
    // Stage B runs above the stage-A guess (about want * stride_b / stride_a
    // union rows, plus six standard deviations); when it kept fewer than `want`
    // rows for some query the guess was too high and stage B is redone above
    // the valid stage-A floor.
    for (int attempt = 0; attempt < 2; ++attempt) {
        const bool g = guess && attempt == 0;
        pb.thr = g ? thr_stat : base.thr;
        CU_TRY(cudaMemsetAsync(base.buf_cnt, 0, static_cast<size_t>(base.m_pad) * sizeof(uint32_t), st),
               "counts");
        CU_TRY(buffer_pass(pb), "floor buffer pass launch");
        if (g) CU_TRY(cudaMemsetAsync(words + 3, 0, sizeof(int), st), "status word");
        CU_TRY(launch_buffer_floor(base.buf_cnt, base.buf_s, base.cap, want, P.r_stat, base.m, base.thr,
                                   thr_stat, g ? words + 3 : nullptr, st),
               "floor select launch");
        if (!g) break;
        CU_TRY(cudaMemcpyAsync(&ix->host_words[7], words + 3, sizeof(int), cudaMemcpyDeviceToHost, st),
               "status");
        CU_TRY(cudaStreamSynchronize(st), "floor estimate");
        if (ix->host_words[7] == 0) break;
    }
    return ST_OK;
}

cudaError_t launch_pass(mflat_cu_index* ix, const ScreenParams& sp, int kp, cudaStream_t st) {
    return launch_fp32_screen(ix, sp, kp, st);
}

}  // namespace

int search_large(mflat_cu_index* ix, const float* queries, int m, int k_out, int32_t* d_ids,
                 float* d_dist, int on_device, cudaStream_t st) {
    constexpr int kKP1 = 32;
    const int lpc = fp32_lists_per_chunk(ix);   // stage-A lists per chunk
    const LargePlan P = plan_large(ix->n, k_out, m, kKP1, 2 * k_out, lpc, ix->num_sms, buffer_budget(ix),
                                   ix->screen_pair && !ix->force_simt);
    const int d_pad = ix->d_pad;
    const int n_tiles = static_cast<int>((ix->n + kBN - 1) / kBN);
    const float* qsrc = queries;
    if (!on_device) {
        CU_TRY(ix->q_in.ensure(static_cast<size_t>(m) * ix->dim * sizeof(float)), "query buffer");
        CU_TRY(cudaMemcpyAsync(ix->q_in.p, queries, static_cast<size_t>(m) * ix->dim * sizeof(float),
                               cudaMemcpyHostToDevice, st),
               "query upload");
        qsrc = ix->q_in.as<float>();
    }
    const int bm_pad = (P.batch + kBM - 1) / kBM * kBM;
    CU_TRY(ix->q_x.ensure(static_cast<size_t>(bm_pad) * d_pad * sizeof(float)), "query buffer");
    CU_TRY(ix->q_h.ensure(static_cast<size_t>(bm_pad) * d_pad * 2), "query split");
    CU_TRY(ix->q_l.ensure(static_cast<size_t>(bm_pad) * d_pad * 2), "query split");
    CU_TRY(ix->qnorm.ensure(static_cast<size_t>(bm_pad) * sizeof(float)), "query norms");
    CU_TRY(ix->thr.ensure(static_cast<size_t>(bm_pad) * sizeof(uint32_t)), "floors");
    CU_TRY(ix->buf_cnt.ensure(static_cast<size_t>(bm_pad) * sizeof(uint32_t)), "buffer counts");
    CU_TRY(ix->buf_s.ensure(static_cast<size_t>(bm_pad) * P.cap * sizeof(float)), "candidate buffer");
    CU_TRY(ix->buf_i.ensure(static_cast<size_t>(bm_pad) * P.cap * sizeof(int32_t)), "candidate buffer");
    CU_TRY(ix->flag_list.ensure(static_cast<size_t>(bm_pad) * sizeof(int)), "flag list");
    CU_TRY(ix->lk_words.ensure(4 * sizeof(int)), "status words");
    CU_TRY(ix->thr_stat.ensure(static_cast<size_t>(bm_pad) * sizeof(uint32_t)), "floors");
    if (P.prepass) {
        const size_t parts = static_cast<size_t>(P.chunks_a) * lpc * bm_pad * kKP1;
        CU_TRY(ix->part_s.ensure(parts * sizeof(float)), "pre-pass lists");
        CU_TRY(ix->part_i.ensure(parts * sizeof(int32_t)), "pre-pass lists");
    } else {
        CU_TRY(ix->part_s.ensure(sizeof(float)), "pre-pass lists");
        CU_TRY(ix->part_i.ensure(sizeof(int32_t)), "pre-pass lists");
    }
    // per batch: [0] overflows, [1] unproven queries, [2] statistical-floor misses
    int* words = ix->lk_words.as<int>();
    const bool use_stat = P.prepass && P.two_stage && P.r_stat > 0;
    int overflows = 0, unproven = 0, redone = 0;
    if (ix->timing) cudaEventRecord(ix->ev[0], st);

    for (int b0 = 0; b0 < m; b0 += P.batch) {
        const int mb = std::min(P.batch, m - b0);
        const int mb_pad = (mb + kBM - 1) / kBM * kBM;
        CU_TRY(launch_prep_queries(qsrc + static_cast<int64_t>(b0) * ix->dim, mb, mb_pad, ix->dim,
                                   d_pad, ix->metric, ix->q_x.as<float>(), ix->q_h.as<uint16_t>(),
                                   ix->q_l.as<uint16_t>(), ix->qnorm.as<float>(), st),
               "query prep launch");
        CU_TRY(cudaMemsetAsync(ix->thr.p, 0, static_cast<size_t>(mb_pad) * sizeof(uint32_t), st), "floors");
        CU_TRY(cudaMemsetAsync(ix->buf_cnt.p, 0, static_cast<size_t>(mb_pad) * sizeof(uint32_t), st), "counts");
        CU_TRY(cudaMemsetAsync(ix->flag_count, 0, sizeof(int), st), "flag count");
        CU_TRY(cudaMemsetAsync(words, 0, 4 * sizeof(int), st), "status words");

        ScreenParams sp{};
        sp.m = mb;
        sp.m_pad = mb_pad;
        sp.d_pad = d_pad;
        sp.n = ix->n;
        sp.n_qtiles = mb_pad / kBM;
        sp.alpha = ix->metric == kL2 ? 2.0f : 1.0f;
        sp.colbias = ix->colbias;
        sp.err = ix->err;
        sp.thr = ix->thr.as<uint32_t>();
        sp.q_x = ix->q_x.as<float>();
        sp.db_x = ix->db_x;
        sp.buf_cnt = ix->buf_cnt.as<uint32_t>();
        sp.buf_s = ix->buf_s.as<float>();
        sp.buf_i = ix->buf_i.as<int32_t>();
        sp.cap = P.cap;
        sp.part_score = ix->part_s.as<float>();
        sp.part_id = ix->part_i.as<int32_t>();
        if (P.prepass) {
            const int rc = estimate_floor(
                ix, P, sp, 2 * k_out, kKP1, lpc,
                [&](const ScreenParams& q, int kp) { return launch_pass(ix, q, kp, st); },
                [&](const ScreenParams& q) { return launch_pass(ix, q, 0, st); },
                ix->thr_stat.as<uint32_t>(), words, st);
            if (rc != ST_OK) return rc;
        }
        sp.use_floor = 1;
        sp.tile_stride = 1;
        sp.n_tiles = n_tiles;
        int n_chunks = 1, tpc = n_tiles;
        const bool pair = screen_pair_for(ix, sp.n_qtiles);
        plan_buffer_chunks(screen_qunits(sp.n_qtiles, pair), n_tiles, screen_slots(ix->num_sms, pair),
                           tile_bytes(ix), n_chunks, tpc);
        sp.n_chunks = n_chunks;
        sp.tiles_per_chunk = tpc;

        LargeSelectParams ls{};
        ls.n = ix->n;
        ls.err = ix->err;
        ls.m = mb;
        ls.m_pad = mb_pad;
        ls.dim = ix->dim;
        ls.d_pad = d_pad;
        ls.k_out = k_out;
        ls.metric = ix->metric == kL2 ? kL2 : kIP;
        ls.cnt = sp.buf_cnt;
        ls.buf_s = sp.buf_s;
        ls.buf_i = sp.buf_i;
        ls.cap = P.cap;
        ls.exact = 1;
        ls.q_x = sp.q_x;
        ls.qnorm = ix->qnorm.as<float>();
        ls.db_x = ix->db_x;
        ls.xmax_bits = ix->xmax_bits;
        ls.gamma = screen_gamma(d_pad);
        ls.id_base = ix->world > 1 ? ix->id_base : 0;
        ls.out_ids = d_ids + static_cast<int64_t>(b0) * k_out;
        ls.out_dist = d_dist + static_cast<int64_t>(b0) * k_out;
        ls.flag_count = words + 1;
        ls.flag_list = ix->flag_list.as<int>();
        ls.overflow = words;

        // The statistical floor first; when it failed for any query of the
        // batch (too few rows reached it, an overflow or an unproven window),
        // the batch is redone with the valid floor.
        for (int attempt = 0; attempt < 2; ++attempt) {
            const bool stat = use_stat && attempt == 0;
            sp.thr = stat ? ix->thr_stat.as<uint32_t>() : ix->thr.as<uint32_t>();
            ls.thr = sp.thr;
            CU_TRY(cudaMemsetAsync(ix->buf_cnt.p, 0, static_cast<size_t>(mb_pad) * sizeof(uint32_t), st),
                   "counts");
            if (ix->timing && b0 == 0 && attempt == 0) cudaEventRecord(ix->ev[1], st);
            CU_TRY(launch_pass(ix, sp, 0, st), "buffer screen launch");
            if (ix->timing && b0 == 0 && attempt == 0) cudaEventRecord(ix->ev[2], st);
            if (stat)
                CU_TRY(launch_floor_check(sp.buf_cnt, ix->thr_stat.as<uint32_t>(), ix->thr.as<uint32_t>(),
                                          2 * k_out, mb, words + 2, st),
                       "floor check launch");
            CU_TRY(launch_select_large(ls, st), "large select launch");
            CU_TRY(cudaMemcpyAsync(&ix->host_words[4], words, 3 * sizeof(int), cudaMemcpyDeviceToHost, st),
                   "status");
            CU_TRY(cudaStreamSynchronize(st), "large-k search");
            if (!stat || (ix->host_words[4] == 0 && ix->host_words[5] == 0 && ix->host_words[6] == 0))
                break;
            ++redone;
            CU_TRY(cudaMemsetAsync(words, 0, 4 * sizeof(int), st), "status words");
        }
        overflows += ix->host_words[4];
        unproven += ix->host_words[5];
    }
    if (ix->timing) cudaEventRecord(ix->ev[3], st);
    // Overflows and unproven queries are rare; surface them as errors.
    if (overflows > 0) return fail(ST_INTERNAL, "candidate buffer overflow (too many rows tie with the k-th best)");
    if (unproven > 0) return fail(ST_INTERNAL, "exactness could not be proven for some queries (near-ties)");
    ix->last.screen_launches = 1 + redone;
    ix->last.launches = (P.prepass ? (P.two_stage ? 7 : 5) : 3) * ((m + P.batch - 1) / P.batch);
    return ST_OK;
}

// ---------------------------------------------------------------------------
// fp16 / bf16 storage (recall path).  k <= 16: list-mode screen (two lists per
// chunk) + recall select.  k > 16: strided floor pre-pass (list mode, 16 per
// list), buffer-mode screen, radix select.
int search_half(mflat_cu_index* ix, const float* queries, int m, int k_out, int32_t* d_ids,
                float* d_dist, int on_device, cudaStream_t st) {
    const bool bf16 = ix->storage == 2;
    const int d_pad = ix->d_pad;
    const int n_tiles = static_cast<int>((ix->n + kBN - 1) / kBN);
    const float* qsrc = queries;
    if (!on_device) {
        CU_TRY(ix->q_in.ensure(static_cast<size_t>(m) * ix->dim * sizeof(float)), "query buffer");
        CU_TRY(cudaMemcpyAsync(ix->q_in.p, queries, static_cast<size_t>(m) * ix->dim * sizeof(float),
                               cudaMemcpyHostToDevice, st),
               "query upload");
        qsrc = ix->q_in.as<float>();
    }
    // Small k on a small problem: per-(query, chunk) top lists (one launch
    // pair, no floor estimate).  Otherwise the
    // buffer path (floor estimate, then append above the floor), whose 4
    // epilogue warpgroups keep up with the d = 128 MMA better than the 2 that
    // per-thread lists leave room for.
    const bool list_mode =
        k_out <= 16 && (ix->n <= kAllRowsBuffered || static_cast<double>(m) * ix->n <= 8e8);
    const int kp = k_out <= 4 ? 4 : (k_out <= 8 ? 8 : 16);
    constexpr int kKP1 = 16;
    LargePlan P;
    if (list_mode) {
        P.batch = m;
    } else {
        // two lists (column halves) per chunk
        P = plan_large(ix->n, k_out, m, kKP1, k_out, 2, ix->num_sms, buffer_budget(ix), ix->screen_pair);
    }
    const int bm_pad = (P.batch + kBM - 1) / kBM * kBM;
    CU_TRY(ix->q16.ensure(static_cast<size_t>(bm_pad) * d_pad * 2), "query conversion");
    CU_TRY(ix->qsq.ensure(static_cast<size_t>(bm_pad) * sizeof(float)), "query norms");
    CU_TRY(ix->thr.ensure(static_cast<size_t>(bm_pad) * sizeof(uint32_t)), "floors");
    if (!list_mode) {
        CU_TRY(ix->buf_cnt.ensure(static_cast<size_t>(bm_pad) * sizeof(uint32_t)), "buffer counts");
        CU_TRY(ix->buf_s.ensure(static_cast<size_t>(bm_pad) * P.cap * sizeof(float)), "candidate buffer");
        CU_TRY(ix->buf_i.ensure(static_cast<size_t>(bm_pad) * P.cap * sizeof(int32_t)), "candidate buffer");
        CU_TRY(ix->lk_words.ensure(4 * sizeof(int)), "status words");
        CU_TRY(ix->thr_stat.ensure(static_cast<size_t>(bm_pad) * sizeof(uint32_t)), "floors");
    }
    // per batch: [0] overflows, [2] statistical-floor misses
    int* words = list_mode ? nullptr : ix->lk_words.as<int>();
    const bool use_stat = !list_mode && P.prepass && P.two_stage && P.r_stat > 0;
    int overflows = 0, redone = 0;
    const int max_lists = list_mode ? kMaxChunks / 2 : P.chunks_a;
    const int lk = list_mode ? kp : kKP1;
    const size_t parts = static_cast<size_t>(2 * std::max(max_lists, 1)) * bm_pad * lk;
    CU_TRY(ix->part_s.ensure(parts * sizeof(float)), "candidate lists");
    CU_TRY(ix->part_i.ensure(parts * sizeof(int32_t)), "candidate lists");
    // tensor maps of the rows for single-CTA [0] and CTA-pair [1] screens
    ScreenMaps maps[2];
    for (int pr = 0; pr < 2; ++pr) {
        if (!make_map_u16(&maps[pr].b, ix->db16, d_pad, ix->n,
                          static_cast<uint32_t>(screen_rows_per_cta(pr != 0))))
            return fail(ST_DEVICE, "tensor map encoding failed");
        maps[pr].b2 = maps[pr].b;
        const int rc = prepare_bias_parts(ix, st, &maps[pr].bias, pr != 0);
        if (rc != ST_OK) return rc;
    }
    const ScreenKind kind = bf16 ? ScreenKind::kBF16 : ScreenKind::kF16;
    if (ix->timing) cudaEventRecord(ix->ev[0], st);

    for (int b0 = 0; b0 < m; b0 += P.batch) {
        const int mb = std::min(P.batch, m - b0);
        const int mb_pad = (mb + kBM - 1) / kBM * kBM;
        prep_queries_half_kernel<<<blocks_for(mb_pad, kHalfPrepRows), 128, 0, st>>>(
            qsrc + static_cast<int64_t>(b0) * ix->dim, mb, mb_pad, ix->dim, d_pad, ix->metric, bf16,
            ix->q16.as<uint16_t>(), ix->qsq.as<float>());
        CU_TRY(cudaGetLastError(), "query prep launch");
        CU_TRY(cudaMemsetAsync(ix->thr.p, 0, static_cast<size_t>(mb_pad) * sizeof(uint32_t), st), "floors");
        for (int pr = 0; pr < 2; ++pr) {
            if (!make_map_u16(&maps[pr].a, ix->q16.p, d_pad, mb_pad, kBM))
                return fail(ST_DEVICE, "tensor map encoding failed");
            maps[pr].a2 = maps[pr].a;
        }
        const bool pair = screen_pair_for(ix->screen_pair, mb_pad / kBM);   // no CUDA-core variant here
        ScreenParams sp{};
        sp.m = mb;
        sp.m_pad = mb_pad;
        sp.d_pad = d_pad;
        sp.n = ix->n;
        sp.n_qtiles = mb_pad / kBM;
        sp.alpha = ix->metric == kL2 ? 2.0f : 1.0f;
        sp.colbias = ix->colbias;
        sp.err = ix->err;
        sp.thr = ix->thr.as<uint32_t>();
        sp.part_score = ix->part_s.as<float>();
        sp.part_id = ix->part_i.as<int32_t>();
        sp.wait_ns = ix->wait_ns;
        auto launch = [&](const ScreenParams& q, int kpp) {
            return launch_screen(kpp, kind, maps[pair ? 1 : 0], q, screen_grid(ix, q.n_qtiles, q.n_chunks, pair),
                                 pair, st);
        };
        if (list_mode) {
            sp.use_floor = 1;
            sp.tile_stride = 1;
            sp.n_tiles = n_tiles;
            int n_chunks = 1, tpc = n_tiles;
            plan_chunks(screen_qunits(sp.n_qtiles, pair), n_tiles, screen_slots(ix->num_sms, pair), kMaxChunks / 2,
                        n_chunks, tpc);
            sp.n_chunks = n_chunks;
            sp.tiles_per_chunk = tpc;
            if (ix->timing) cudaEventRecord(ix->ev[1], st);
            CU_TRY(launch(sp, kp), "screen launch");
            if (ix->timing) cudaEventRecord(ix->ev[2], st);
            SelectParams sel{};
            sel.m = mb;
            sel.m_pad = mb_pad;
            sel.k_out = k_out;
            sel.n_chunks = 2 * n_chunks;
            sel.metric = ix->metric == kL2 ? kL2 : kIP;
            sel.part_score = sp.part_score;
            sel.part_id = sp.part_id;
            sel.id_base = ix->world > 1 ? ix->id_base : 0;
            sel.out_ids = d_ids + static_cast<int64_t>(b0) * k_out;
            sel.out_dist = d_dist + static_cast<int64_t>(b0) * k_out;
            CU_TRY(launch_select_recall(kp, sel, ix->qsq.as<float>(), st), "select launch");
            continue;
        }
        sp.buf_cnt = ix->buf_cnt.as<uint32_t>();
        sp.buf_s = ix->buf_s.as<float>();
        sp.buf_i = ix->buf_i.as<int32_t>();
        sp.cap = P.cap;
        CU_TRY(cudaMemsetAsync(words, 0, 4 * sizeof(int), st), "status words");
        if (P.prepass) {
            CU_TRY(cudaMemsetAsync(ix->buf_cnt.p, 0, static_cast<size_t>(mb_pad) * sizeof(uint32_t), st),
                   "counts");
            const int rc = estimate_floor(
                ix, P, sp, k_out, kKP1, 2, [&](const ScreenParams& q, int kpp) { return launch(q, kpp); },
                [&](const ScreenParams& q) { return launch(q, 0); }, ix->thr_stat.as<uint32_t>(), words,
                st);
            if (rc != ST_OK) return rc;
        }
        sp.use_floor = 1;
        sp.tile_stride = 1;
        sp.n_tiles = n_tiles;
        int n_chunks = 1, tpc = n_tiles;
        plan_buffer_chunks(screen_qunits(sp.n_qtiles, pair), n_tiles, screen_slots(ix->num_sms, pair),
                           tile_bytes(ix), n_chunks, tpc);
        sp.n_chunks = n_chunks;
        sp.tiles_per_chunk = tpc;
        LargeSelectParams ls{};
        ls.n = ix->n;
        ls.err = ix->err;
        ls.m = mb;
        ls.m_pad = mb_pad;
        ls.k_out = k_out;
        ls.metric = ix->metric == kL2 ? kL2 : kIP;
        ls.cnt = sp.buf_cnt;
        ls.buf_s = sp.buf_s;
        ls.buf_i = sp.buf_i;
        ls.cap = P.cap;
        ls.exact = 0;
        ls.qsq = ix->qsq.as<float>();
        ls.id_base = ix->world > 1 ? ix->id_base : 0;
        ls.out_ids = d_ids + static_cast<int64_t>(b0) * k_out;
        ls.out_dist = d_dist + static_cast<int64_t>(b0) * k_out;
        ls.flag_count = words + 1;
        ls.flag_list = nullptr;
        ls.overflow = words;
        // statistical floor first, the valid floor when it failed (see search_large)
        for (int attempt = 0; attempt < 2; ++attempt) {
            const bool stat = use_stat && attempt == 0;
            sp.thr = stat ? ix->thr_stat.as<uint32_t>() : ix->thr.as<uint32_t>();
            ls.thr = sp.thr;
            CU_TRY(cudaMemsetAsync(ix->buf_cnt.p, 0, static_cast<size_t>(mb_pad) * sizeof(uint32_t), st),
                   "counts");
            if (ix->timing && b0 == 0 && attempt == 0) cudaEventRecord(ix->ev[1], st);
            CU_TRY(launch(sp, 0), "buffer screen launch");
            if (ix->timing && b0 == 0 && attempt == 0) cudaEventRecord(ix->ev[2], st);
            if (stat)
                CU_TRY(launch_floor_check(sp.buf_cnt, ix->thr_stat.as<uint32_t>(), ix->thr.as<uint32_t>(),
                                          k_out, mb, words + 2, st),
                       "floor check launch");
            CU_TRY(launch_select_large(ls, st), "large select launch");
            CU_TRY(cudaMemcpyAsync(&ix->host_words[4], words, 3 * sizeof(int), cudaMemcpyDeviceToHost, st),
                   "status");
            CU_TRY(cudaStreamSynchronize(st), "large-k search");
            if (!stat || (ix->host_words[4] == 0 && ix->host_words[6] == 0)) break;
            ++redone;
            CU_TRY(cudaMemsetAsync(words, 0, 4 * sizeof(int), st), "status words");
        }
        overflows += ix->host_words[4];
    }
    if (ix->timing) cudaEventRecord(ix->ev[3], st);
    ix->last.screen_launches = 1 + redone;
    ix->last.launches = list_mode ? 3 : (P.prepass ? (P.two_stage ? 7 : 5) : 3);
    if (overflows > 0)
        return fail(ST_INTERNAL, "candidate buffer overflow (too many rows tie with the k-th best)");
    return ST_OK;
}

}  // namespace mflat_cu

using namespace mflat_cu;

namespace mflat_cu {
namespace {

// Append n rows.  raw = 0: caller vectors (Cosine rows are normalised);
// raw = 1: host rows that are already stored values, in storage precision
// (fp32, or 16-bit bit patterns), taken as they are.
int index_add(mflat_cu_index_t* ix, const void* vectors, int64_t n, int on_device, void* stream,
              int raw) {
    if (!ix || (!vectors && n > 0) || n < 0) return fail(ST_BAD_ARG, "bad argument");
    if (n == 0) return ST_OK;
    if (ix->n + n > static_cast<int64_t>(INT32_MAX) - kBN)
        return fail(ST_BAD_ARG, "database would exceed 2^31 rows");
    DeviceGuard g(ix->device);
    cudaStream_t caller = static_cast<cudaStream_t>(stream);
    if (on_device) order_after(ix->stream, caller);
    CU_TRY(grow(ix, ix->n + n), "database allocation");
    const size_t elem = raw && ix->storage != 0 ? sizeof(uint16_t) : sizeof(float);
    const int64_t chunk =
        on_device ? n : std::max<int64_t>(1, (int64_t(64) << 20) / (int64_t(ix->dim) * 4));
    for (int64_t off = 0; off < n; off += chunk) {
        const int64_t cnt = std::min(chunk, n - off);
        const void* src = static_cast<const uint8_t*>(vectors) + off * ix->dim * elem;
        if (!on_device) {
            const size_t bytes = static_cast<size_t>(cnt) * ix->dim * elem;
            CU_TRY(ix->stage_in.ensure(bytes), "staging");
            CU_TRY(cudaMemcpyAsync(ix->stage_in.p, src, bytes, cudaMemcpyHostToDevice, ix->stream), "upload");
            src = ix->stage_in.p;
        }
        if (ix->storage != 0 && raw)
            ingest_rows_bits_kernel<<<blocks_for(cnt, 128), 128, 0, ix->stream>>>(
                static_cast<const uint16_t*>(src), cnt, ix->dim, ix->d_pad, ix->metric, ix->storage == 2,
                ix->n + off, static_cast<uint16_t*>(ix->db16), ix->colbias, ix->dnorm);
        else if (ix->storage != 0)
            ingest_rows_half_kernel<<<blocks_for(cnt, 128), 128, 0, ix->stream>>>(
                static_cast<const float*>(src), cnt, ix->dim, ix->d_pad, ix->metric, ix->storage == 2,
                ix->n + off, static_cast<uint16_t*>(ix->db16), ix->colbias, ix->dnorm);
        else
            ingest_rows_kernel<<<blocks_for(cnt, 128), 128, 0, ix->stream>>>(
                static_cast<const float*>(src), cnt, ix->dim, ix->d_pad, ix->metric, raw ? 0 : 1,
                ix->n + off, ix->db_x, ix->db_h, ix->db_l, ix->colbias, ix->dnorm, ix->xmax_bits);
        CU_TRY(cudaGetLastError(), "ingest launch");
        if (!on_device) CU_TRY(cudaStreamSynchronize(ix->stream), "ingest");
    }
    // rows [n_old, rows_pad(n_old)) were padding: their bias parts change
    ix->bias16_rows = std::min(ix->bias16_rows, ix->n);
    ix->n += n;
    if (on_device) order_after(caller, ix->stream);
    return ST_OK;
}

}  // namespace
}  // namespace mflat_cu

// =====================================================================
namespace mflat_cu {

// fp32 storage, k <= 21: list-mode screen (top-32 per query and chunk), then
// the merge + exactness proof + fp64 re-rank, and the exact full scan for the
// (rare) queries whose proof fails.
int search_list_exact(mflat_cu_index* ix, const float* queries, int m, int k_out, int32_t* d_ids,
                      float* d_dist, int on_device, cudaStream_t st) {
    const int kp = kp_for(k_out);
    ScreenRun run;
    int rc = run_screen(ix, queries, m, kp, on_device, st, run);
    if (rc != ST_OK) return rc;
    ix->last.screen_launches = 1;
    CU_TRY(ix->flag_list.ensure(static_cast<size_t>(m) * sizeof(int)), "fallback list");
    CU_TRY(cudaMemsetAsync(ix->flag_count, 0, sizeof(int), st), "fallback count");

    SelectParams sel{};
    sel.m = m;
    sel.m_pad = run.m_pad;
    sel.dim = ix->dim;
    sel.d_pad = ix->d_pad;
    sel.k_out = k_out;
    sel.n_chunks = run.n_lists;
    sel.metric = ix->metric == kL2 ? kL2 : kIP;
    sel.n = ix->n;
    sel.part_score = run.part_s;
    sel.part_id = run.part_i;
    sel.q_x = run.q_x;
    sel.qnorm = run.qnorm;
    sel.db_x = ix->db_x;
    sel.xmax_bits = ix->xmax_bits;
    sel.gamma = screen_gamma(ix->d_pad);
    sel.id_base = ix->world > 1 ? ix->id_base : 0;
    sel.out_ids = d_ids;
    sel.out_dist = d_dist;
    sel.flag_count = ix->flag_count;
    sel.flag_list = ix->flag_list.as<int>();
    sel.err = ix->err;
    const size_t fb = static_cast<size_t>(m) * kFbChunks * k_out;
    CU_TRY(ix->fb_s.ensure(fb * sizeof(double)), "fallback scratch");
    CU_TRY(ix->fb_i.ensure(fb * sizeof(int32_t)), "fallback scratch");
    sel.fb_s = ix->fb_s.as<double>();
    sel.fb_i = ix->fb_i.as<int32_t>();
    CU_TRY(launch_select_exact(kp, sel, st), "select launch");
    CU_TRY(launch_fallback_exact(sel, ix->num_sms, st), "fallback launch");
    ix->last.launches = run.launches + 3;
    if (ix->timing) {
        CU_TRY(cudaMemcpyAsync(&ix->host_words[8 + ix->ring_next], ix->flag_count, sizeof(int),
                               cudaMemcpyDeviceToHost, st),
               "fallback count");
        cudaEventRecord(ix->ev[3], st);
    }
    return ST_OK;
}

}  // namespace mflat_cu

namespace mflat_cu {

// Read a pending timing slot (waits for its last event) and add it to the sums.
void fold_slot(const mflat_cu_index* ix, int slot) {
    auto& sl = ix->ring[slot];
    if (!sl.pending) return;
    sl.pending = false;
    if (cudaEventSynchronize(sl.ev[3]) != cudaSuccess) return;
    cudaEventElapsedTime(&sl.t.total_ms, sl.ev[0], sl.ev[3]);
    cudaEventElapsedTime(&sl.t.screen_ms, sl.ev[1], sl.ev[2]);
    cudaEventElapsedTime(&sl.t.select_ms, sl.ev[2], sl.ev[3]);
    sl.t.fallback_queries = ix->host_words[8 + slot];
    ix->sum.total_ms += sl.t.total_ms;
    ix->sum.screen_ms += sl.t.screen_ms;
    ix->sum.select_ms += sl.t.select_ms;
    ix->sum.screen_launches += sl.t.screen_launches;
    ix->sum.launches += sl.t.launches;
    ix->sum.fallback_queries += sl.t.fallback_queries;
    ix->sum_n += 1;
}

// Oldest first, so the sums add up in search order.
void fold_all_slots(const mflat_cu_index* ix) {
    for (int i = 0; i < kTimingRing; ++i) fold_slot(ix, (ix->ring_next + i) % kTimingRing);
}

void timing_begin(mflat_cu_index* ix) {
    if (!ix->timing) return;
    const int slot = ix->ring_next;
    fold_slot(ix, slot);                 // reused after kTimingRing searches: long finished
    ix->ev = ix->ring[slot].ev;
    ix->host_words[8 + slot] = 0;
    ix->last = mflat_cu_timing_t{};
}

void timing_end(mflat_cu_index* ix) {
    if (!ix->timing) return;
    const int slot = ix->ring_next;
    ix->ring[slot].t = ix->last;
    ix->ring[slot].pending = true;
    ix->ring_last = slot;
    ix->ring_next = (slot + 1) % kTimingRing;
}

}  // namespace mflat_cu

extern "C" {

const char* mflat_cu_last_error(void) { return last_error_message(); }

int mflat_cu_device_count(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) return 0;
    return n;
}

int mflat_cu_default_device(int device) {
    if (device >= 0) return device;
    const char* env = std::getenv("MFLAT_DEVICE");
    if (env && *env) return std::atoi(env);
    return 0;
}

int mflat_cu_index_create(int device, int dim, int metric, int storage, mflat_cu_index_t** out) {
    if (!out || dim <= 0) return fail(ST_BAD_ARG, "bad argument");
    *out = nullptr;
    device = mflat_cu_default_device(device);
    const int ndev = mflat_cu_device_count();
    if (ndev <= 0) return fail(ST_DEVICE, "no CUDA device");
    if (device >= ndev) return fail(ST_BAD_ARG, "device index out of range");
    if (storage < 0 || storage > 2) return fail(ST_BAD_ARG, "unknown storage precision");
    DeviceGuard g(device);
    int major = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device);
    if (major != 10) return fail(ST_DEVICE, "device is not sm_100 (B200)");
    auto* ix = new (std::nothrow) mflat_cu_index();
    if (!ix) return fail(ST_ALLOC, "host allocation failed");
    ix->device = device;
    ix->dim = dim;
    // one 128-byte k-block = 64 16-bit elements (the fp32 storage's screen
    // planes are bf16 too)
    ix->d_pad = (dim + kBK - 1) / kBK * kBK;
    ix->metric = (metric == kIP || metric == kCosine) ? metric : kL2;
    ix->storage = storage;
    cudaDeviceGetAttribute(&ix->num_sms, cudaDevAttrMultiProcessorCount, device);
    const char* fs = std::getenv("MFLAT_SCREEN");
    ix->force_simt = fs && std::strcmp(fs, "simt") == 0;
    if (const char* pr = std::getenv("MFLAT_SCREEN_PAIR")) ix->screen_pair = std::strcmp(pr, "0") != 0;
    if (const char* wl = std::getenv("MFLAT_WAIT_LIMIT_MS")) {
        const double ms = std::atof(wl);
        if (ms > 0.0) ix->wait_ns = static_cast<uint64_t>(ms * 1e6);
    }
    const char* stall = std::getenv("MFLAT_TEST_STALL_SCREEN");
    ix->test_stall = (stall && std::strcmp(stall, "1") == 0) ? 1 : 0;
    cudaError_t e;
    if ((e = cudaStreamCreateWithFlags(&ix->stream, cudaStreamNonBlocking)) != cudaSuccess ||
        (e = cudaMalloc(&ix->xmax_bits, sizeof(unsigned))) != cudaSuccess ||
        (e = cudaMalloc(&ix->err, sizeof(int))) != cudaSuccess ||
        (e = cudaMalloc(&ix->flag_count, sizeof(int))) != cudaSuccess ||
        (e = cudaHostAlloc(&ix->host_words, kHostWords * sizeof(int), cudaHostAllocDefault)) != cudaSuccess) {
        mflat_cu_index_destroy(ix);
        return fail(e == cudaErrorMemoryAllocation ? ST_ALLOC : ST_DEVICE, "index setup", e);
    }
    cudaMemsetAsync(ix->xmax_bits, 0, sizeof(unsigned), ix->stream);
    cudaMemsetAsync(ix->err, 0, sizeof(int), ix->stream);
    std::memset(ix->host_words, 0, kHostWords * sizeof(int));
    if ((e = cudaStreamSynchronize(ix->stream)) != cudaSuccess) {
        mflat_cu_index_destroy(ix);
        return fail(ST_DEVICE, "index setup", e);
    }
    *out = ix;
    return ST_OK;
}

void mflat_cu_index_destroy(mflat_cu_index_t* ix) {
    if (!ix) return;
    DeviceGuard g(ix->device);
    if (ix->stream) cudaStreamSynchronize(ix->stream);
    comm_release(ix);
    cudaFree(ix->db16);
    cudaFree(ix->db_x);
    cudaFree(ix->db_h);
    cudaFree(ix->db_l);
    cudaFree(ix->colbias);
    cudaFree(ix->dnorm);
    cudaFree(ix->xmax_bits);
    cudaFree(ix->err);
    cudaFree(ix->flag_count);
    if (ix->host_words) cudaFreeHost(ix->host_words);
    for (DevBuf* b : {&ix->stage_in, &ix->q_in, &ix->q_x, &ix->q_h, &ix->q_l, &ix->qnorm, &ix->part_s,
                      &ix->part_i, &ix->flag_list, &ix->out_ids, &ix->out_dist, &ix->gather_ids,
                      &ix->gather_dist, &ix->merge_tmp_ids, &ix->merge_tmp_dist, &ix->thr, &ix->thr_stat, &ix->fb_s,
                      &ix->fb_i, &ix->buf_cnt, &ix->buf_s, &ix->buf_i, &ix->lk_words,
                      &ix->q16, &ix->qsq})
        b->release();
    cudaFree(ix->bias16);
    for (auto& slot : ix->ring)
        for (auto& ev : slot.ev)
            if (ev) cudaEventDestroy(ev);
    if (ix->stream) cudaStreamDestroy(ix->stream);
    delete ix;
}

int64_t mflat_cu_index_size(const mflat_cu_index_t* ix) { return ix ? ix->n : 0; }
int mflat_cu_index_device(const mflat_cu_index_t* ix) { return ix ? ix->device : -1; }

int mflat_cu_index_add(mflat_cu_index_t* ix, const float* vectors, int64_t n, int on_device,
                       void* stream) {
    return index_add(ix, vectors, n, on_device, stream, 0);
}

int mflat_cu_index_add_raw(mflat_cu_index_t* ix, const void* host_rows, int64_t n) {
    return index_add(ix, host_rows, n, 0, nullptr, 1);
}

int mflat_cu_index_export_rows(mflat_cu_index_t* ix, int64_t start, int64_t count, void* host_out) {
    if (!ix || start < 0 || count < 0 || start + count > ix->n || (count > 0 && !host_out))
        return fail(ST_BAD_ARG, "export range outside the index");
    if (count == 0) return ST_OK;
    DeviceGuard g(ix->device);
    const size_t elem = ix->storage != 0 ? sizeof(uint16_t) : sizeof(float);
    const int64_t chunk = std::max<int64_t>(1, (int64_t(64) << 20) / (int64_t(ix->dim) * 4));
    for (int64_t off = 0; off < count; off += chunk) {
        const int64_t cnt = std::min(chunk, count - off);
        const int64_t elems = cnt * ix->dim;
        CU_TRY(ix->stage_in.ensure(static_cast<size_t>(elems) * elem), "staging");
        if (ix->storage != 0)
            export_rows_bits_kernel<<<blocks_for(elems, 256), 256, 0, ix->stream>>>(
                static_cast<const uint16_t*>(ix->db16), start + off, cnt, ix->dim, ix->d_pad,
                ix->stage_in.as<uint16_t>());
        else
            export_rows_f32_kernel<<<blocks_for(elems, 256), 256, 0, ix->stream>>>(
                ix->db_x, start + off, cnt, ix->dim, ix->d_pad, ix->stage_in.as<float>());
        CU_TRY(cudaGetLastError(), "export launch");
        CU_TRY(cudaMemcpyAsync(static_cast<uint8_t*>(host_out) + off * ix->dim * elem, ix->stage_in.p,
                               static_cast<size_t>(elems) * elem, cudaMemcpyDeviceToHost, ix->stream),
               "download");
        CU_TRY(cudaStreamSynchronize(ix->stream), "export");
    }
    return ST_OK;
}

int mflat_cu_index_storage(const mflat_cu_index_t* ix) { return ix ? ix->storage : -1; }

int mflat_cu_index_reset(mflat_cu_index_t* ix) {
    if (!ix) return fail(ST_BAD_ARG, "bad argument");
    DeviceGuard g(ix->device);
    CU_TRY(cudaStreamSynchronize(ix->stream), "reset");
    if (ix->cap > 0) {
        fill_f32_kernel<<<blocks_for(ix->cap, 256), 256, 0, ix->stream>>>(ix->colbias, ix->cap, -kInf);
        CU_TRY(cudaGetLastError(), "reset");
    }
    cudaMemsetAsync(ix->xmax_bits, 0, sizeof(unsigned), ix->stream);
    CU_TRY(cudaStreamSynchronize(ix->stream), "reset");
    ix->n = 0;
    ix->bias16_rows = 0;
    return ST_OK;
}

int mflat_cu_index_set_timing(mflat_cu_index_t* ix, int enable) {
    if (!ix) return fail(ST_BAD_ARG, "bad argument");
    DeviceGuard g(ix->device);
    fold_all_slots(ix);
    if (enable && !ix->ring[0].ev[0]) {
        for (auto& slot : ix->ring)
            for (auto& ev : slot.ev) CU_TRY(cudaEventCreate(&ev), "timing events");
    }
    if (enable) {
        ix->sum = mflat_cu_timing_t{};
        ix->sum_n = 0;
        ix->ring_last = -1;
        ix->ring_next = 0;
    }
    ix->timing = enable != 0;
    return ST_OK;
}

int mflat_cu_index_last_timing(const mflat_cu_index_t* ix, mflat_cu_timing_t* out) {
    if (!ix || !out) return fail(ST_BAD_ARG, "bad argument");
    *out = mflat_cu_timing_t{};
    if (ix->ring_last < 0) return ST_OK;
    DeviceGuard g(ix->device);
    fold_slot(ix, ix->ring_last);
    *out = ix->ring[ix->ring_last].t;
    return ST_OK;
}

int mflat_cu_index_timing_sum(const mflat_cu_index_t* ix, mflat_cu_timing_t* out, int* n_searches) {
    if (!ix || !out) return fail(ST_BAD_ARG, "bad argument");
    DeviceGuard g(ix->device);
    fold_all_slots(ix);
    *out = ix->sum;
    if (n_searches) *n_searches = ix->sum_n;
    return ST_OK;
}

int mflat_cu_index_search(mflat_cu_index_t* ix, const float* queries, int m, int k_out,
                          int32_t* out_ids, float* out_dist, int on_device, void* stream) {
    if (!ix || (!queries && m > 0) || m < 0 || k_out < 1) return fail(ST_BAD_ARG, "bad argument");
    if (m == 0) return ST_OK;
    DeviceGuard g(ix->device);
    NvtxRange range("mflat.search");
    cudaStream_t st = on_device ? static_cast<cudaStream_t>(stream) : ix->stream;
    if (on_device) {
        const int rc = check_device_error(ix, st);   // the previous asynchronous call
        if (rc != ST_OK) return rc;
    }
    const int64_t mk = static_cast<int64_t>(m) * k_out;
    int32_t* d_ids = out_ids;
    float* d_dist = out_dist;
    if (!on_device) {
        CU_TRY(ix->out_ids.ensure(mk * sizeof(int32_t)), "result buffer");
        CU_TRY(ix->out_dist.ensure(mk * sizeof(float)), "result buffer");
        d_ids = ix->out_ids.as<int32_t>();
        d_dist = ix->out_dist.as<float>();
    }
    timing_begin(ix);
    int rc = ST_OK;
    if (ix->n == 0) {
        if (ix->timing)
            for (int i = 0; i < 3; ++i) cudaEventRecord(ix->ev[i], st);
        const float empty = ix->metric == kL2 ? kInf : -kInf;
        fill_empty_kernel<<<blocks_for(mk, 256), 256, 0, st>>>(d_ids, d_dist, mk, empty);
        CU_TRY(cudaGetLastError(), "fill");
        if (ix->timing) cudaEventRecord(ix->ev[3], st);
        ix->last.launches = 1;
    } else if (ix->storage != 0) {
        rc = search_half(ix, queries, m, k_out, d_ids, d_dist, on_device, st);
    } else if (kp_for(k_out) == 0) {
        rc = search_large(ix, queries, m, k_out, d_ids, d_dist, on_device, st);
    } else {
        rc = search_list_exact(ix, queries, m, k_out, d_ids, d_dist, on_device, st);
    }
    if (rc != ST_OK) return rc;
    if (ix->world > 1) {
        NvtxRange mr("mflat.shard_merge");
        rc = shard_merge(ix, m, k_out, d_ids, d_dist, st);
        if (rc != ST_OK) return rc;
        ix->last.launches += 1;
    }
    CU_TRY(cudaMemcpyAsync(&ix->host_words[0], ix->err, sizeof(int), cudaMemcpyDeviceToHost, st),
           "status");
    if (!on_device) {
        // A copy into pageable caller memory blocks the host until the stream
        // reaches it; behind an all-gather that a dead peer never completes it
        // would block for good.  Sharded searches therefore wait under the
        // collective watchdog first.
        if (ix->world > 1) {
            rc = wait_stream_checked(ix, st);
            if (rc != ST_OK) return rc;
        }
        CU_TRY(cudaMemcpyAsync(out_ids, d_ids, mk * sizeof(int32_t), cudaMemcpyDeviceToHost, st), "download");
        CU_TRY(cudaMemcpyAsync(out_dist, d_dist, mk * sizeof(float), cudaMemcpyDeviceToHost, st), "download");
        rc = wait_stream_checked(ix, st);
        if (rc != ST_OK) return rc;
        rc = check_device_error(ix, st);
        if (rc != ST_OK) return rc;
    }
    timing_end(ix);
    return ST_OK;
}

}  // extern "C"
