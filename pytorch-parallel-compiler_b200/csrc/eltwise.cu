// Elementwise glue between wide stages and the layout-boundary copies.
// All kernels are single-pass, 16-byte vectorised where alignment allows, with
// grids sized to a few CTAs per SM and grid-stride loops.
#include "common.cuh"

namespace widek {
namespace {

__device__ __forceinline__ float unary_op(float v, int op) {
    switch (op) {
        case WIDEK_UNARY_RELU: return v > 0.f ? v : 0.f;
        case WIDEK_UNARY_GELU: return gelu_erf(v);
        case WIDEK_UNARY_SIGMOID: return 1.f / (1.f + __expf(-v));
        case WIDEK_UNARY_TANH: return tanhf(v);
        case WIDEK_UNARY_SILU: return v / (1.f + __expf(-v));
        default: return v;
    }
}
__device__ __forceinline__ float binary_op(float a, float b, int op) {
    switch (op) {
        case WIDEK_BINARY_ADD: return a + b;
        case WIDEK_BINARY_MUL: return a * b;
        case WIDEK_BINARY_SUB: return a - b;
        case WIDEK_BINARY_DIV: return a / b;
        default: return a;
    }
}

template <typename T>
__global__ void unary_kernel(const T* __restrict__ x, T* __restrict__ y, int64_t numel, int op, int vec) {
    constexpr int V = 16 / sizeof(T);
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (vec) {
        const int64_t nv = numel / V;
        for (int64_t j = i; j < nv; j += stride) {
            float v[V];
            load16<T>(x + j * V, v);
#pragma unroll
            for (int t = 0; t < V; ++t) v[t] = unary_op(v[t], op);
            store16<T>(y + j * V, v);
        }
        for (int64_t j = nv * V + i; j < numel; j += stride) y[j] = from_f<T>(unary_op(to_f<T>(x[j]), op));
    } else {
        for (int64_t j = i; j < numel; j += stride) y[j] = from_f<T>(unary_op(to_f<T>(x[j]), op));
    }
}

template <typename T>
__global__ void binary_kernel(const T* __restrict__ a, const T* __restrict__ b, T* __restrict__ y, int64_t numel,
                              int op, int vec) {
    constexpr int V = 16 / sizeof(T);
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (vec) {
        const int64_t nv = numel / V;
        for (int64_t j = i; j < nv; j += stride) {
            float va[V], vb[V];
            load16<T>(a + j * V, va);
            load16<T>(b + j * V, vb);
#pragma unroll
            for (int t = 0; t < V; ++t) va[t] = binary_op(va[t], vb[t], op);
            store16<T>(y + j * V, va);
        }
        for (int64_t j = nv * V + i; j < numel; j += stride)
            y[j] = from_f<T>(binary_op(to_f<T>(a[j]), to_f<T>(b[j]), op));
    } else {
        for (int64_t j = i; j < numel; j += stride) y[j] = from_f<T>(binary_op(to_f<T>(a[j]), to_f<T>(b[j]), op));
    }
}

unsigned grid_for(int64_t work_items, int threads) {
    const int64_t want = (work_items + threads - 1) / threads;
    const int64_t cap = (int64_t)sm_count(current_device()) * 8;
    return (unsigned)std::max<int64_t>(1, std::min<int64_t>(want, cap));
}

struct UnaryLaunch {
    const void* x;
    void* y;
    int64_t numel;
    int op;
    cudaStream_t st;
    template <typename T>
    int run() {
        const int vec = aligned16(x) && aligned16(y);
        const int64_t items = vec ? numel / (16 / sizeof(T)) + 1 : numel;
        unary_kernel<T><<<grid_for(items, 256), 256, 0, st>>>(static_cast<const T*>(x), static_cast<T*>(y), numel,
                                                              op, vec);
        return check_launch("widek_unary");
    }
};

struct BinaryLaunch {
    const void *a, *b;
    void* y;
    int64_t numel;
    int op;
    cudaStream_t st;
    template <typename T>
    int run() {
        const int vec = aligned16(a) && aligned16(b) && aligned16(y);
        const int64_t items = vec ? numel / (16 / sizeof(T)) + 1 : numel;
        binary_kernel<T><<<grid_for(items, 256), 256, 0, st>>>(static_cast<const T*>(a), static_cast<const T*>(b),
                                                               static_cast<T*>(y), numel, op, vec);
        return check_launch("widek_binary");
    }
};

// dst[j, i, :] = src[i, j, :]; rows of `row_units` units of type U.
template <typename U>
__global__ void swap01_kernel(const U* __restrict__ src, U* __restrict__ dst, int64_t a, int64_t b,
                              int64_t row_units) {
    const int64_t total = a * b * row_units;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += stride) {
        const int64_t drow = idx / row_units;
        const int64_t v = idx - drow * row_units;
        const int64_t j = drow / a;
        const int64_t i = drow - j * a;
        dst[idx] = src[(i * b + j) * row_units + v];
    }
}

// Same permutation for long rows: a job is one chunk of kRowChunk units of
// one destination row; the index arithmetic is per job, and each thread keeps
// kRowUnroll independent loads in flight.
constexpr int kRowUnroll = 4;
constexpr int kRowThreads = 256;
constexpr int64_t kRowChunk = (int64_t)kRowThreads * kRowUnroll;

template <typename U>
__global__ void __launch_bounds__(kRowThreads) swap01_rows_kernel(const U* __restrict__ src, U* __restrict__ dst,
                                                                  int64_t a, int64_t b, int64_t row_units) {
    const int64_t chunks = (row_units + kRowChunk - 1) / kRowChunk;
    const int64_t jobs = a * b * chunks;
    for (int64_t job = blockIdx.x; job < jobs; job += gridDim.x) {
        const int64_t drow = job / chunks;
        const int64_t c0 = (job - drow * chunks) * kRowChunk;
        const int64_t j = drow / a;
        const int64_t i = drow - j * a;
        const U* s = src + (i * b + j) * row_units;
        U* d = dst + drow * row_units;
        U v[kRowUnroll];
#pragma unroll
        for (int u = 0; u < kRowUnroll; ++u) {
            const int64_t k = c0 + u * kRowThreads + threadIdx.x;
            if (k < row_units) v[u] = s[k];
        }
#pragma unroll
        for (int u = 0; u < kRowUnroll; ++u) {
            const int64_t k = c0 + u * kRowThreads + threadIdx.x;
            if (k < row_units) d[k] = v[u];
        }
    }
}

// Strided 2-D copy: dst[r * dst_pitch + k] = src[r * src_pitch + k] for
// k < row_units (pitches in units of U); jobs are (row, chunk) pairs as in
// swap01_rows_kernel.
template <typename U>
__global__ void __launch_bounds__(kRowThreads) copy2d_kernel(const U* __restrict__ src, int64_t src_pitch,
                                                             U* __restrict__ dst, int64_t dst_pitch, int64_t rows,
                                                             int64_t row_units) {
    const int64_t chunks = (row_units + kRowChunk - 1) / kRowChunk;
    const int64_t jobs = rows * chunks;
    for (int64_t job = blockIdx.x; job < jobs; job += gridDim.x) {
        const int64_t r = job / chunks;
        const int64_t c0 = (job - r * chunks) * kRowChunk;
        const U* s = src + r * src_pitch;
        U* d = dst + r * dst_pitch;
        U v[kRowUnroll];
#pragma unroll
        for (int u = 0; u < kRowUnroll; ++u) {
            const int64_t k = c0 + u * kRowThreads + threadIdx.x;
            if (k < row_units) v[u] = s[k];
        }
#pragma unroll
        for (int u = 0; u < kRowUnroll; ++u) {
            const int64_t k = c0 + u * kRowThreads + threadIdx.x;
            if (k < row_units) d[k] = v[u];
        }
    }
}

template <typename U>
void launch_copy2d(const void* src, int64_t src_pitch, void* dst, int64_t dst_pitch, int64_t rows,
                   int64_t row_bytes, cudaStream_t st) {
    constexpr int64_t u = sizeof(U);
    const int64_t ru = row_bytes / u;
    const int64_t jobs = rows * ((ru + kRowChunk - 1) / kRowChunk);
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(jobs, (int64_t)sm_count(current_device()) * 8));
    copy2d_kernel<U><<<grid, kRowThreads, 0, st>>>(static_cast<const U*>(src), src_pitch / u, static_cast<U*>(dst),
                                                   dst_pitch / u, rows, ru);
}

constexpr int kPackMax = 64;
struct PackPtrs {
    const void* p[kPackMax];
};

// dst[bi, i0 + i, :] = srcs[i][bi, :] for i < cnt; rows of `row_units` U.
template <typename U>
__global__ void pack_kernel(PackPtrs srcs, int cnt, int64_t n, int64_t i0, U* __restrict__ dst, int64_t b,
                            int64_t row_units) {
    const int64_t total = b * cnt * row_units;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += stride) {
        const int64_t r = idx / row_units;
        const int64_t v = idx - r * row_units;
        const int64_t bi = r / cnt;
        const int64_t i = r - bi * cnt;
        const U* s = static_cast<const U*>(srcs.p[i]);
        dst[(bi * n + i0 + i) * row_units + v] = s[bi * row_units + v];
    }
}

}  // namespace
}  // namespace widek

extern "C" {

int widek_unary(const void* x, void* y, int64_t numel, int op, int dtype, void* stream) {
    using namespace widek;
    if (numel < 0) return set_error(WIDEK_ERR_INVALID, "unary: negative numel");
    if (op < WIDEK_UNARY_RELU || op > WIDEK_UNARY_SILU) return set_error(WIDEK_ERR_INVALID, "unary: bad op %d", op);
    if (numel == 0) return WIDEK_OK;
    if (!x || !y) return set_error(WIDEK_ERR_INVALID, "unary: null pointer");
    UnaryLaunch L{x, y, numel, op, (cudaStream_t)stream};
    return dispatch_dtype(dtype, L);
}

int widek_binary(const void* a, const void* b, void* y, int64_t numel, int op, int dtype, void* stream) {
    using namespace widek;
    if (numel < 0) return set_error(WIDEK_ERR_INVALID, "binary: negative numel");
    if (op < WIDEK_BINARY_ADD || op > WIDEK_BINARY_DIV) return set_error(WIDEK_ERR_INVALID, "binary: bad op %d", op);
    if (numel == 0) return WIDEK_OK;
    if (!a || !b || !y) return set_error(WIDEK_ERR_INVALID, "binary: null pointer");
    BinaryLaunch L{a, b, y, numel, op, (cudaStream_t)stream};
    return dispatch_dtype(dtype, L);
}

int widek_swap01(const void* src, void* dst, int64_t a, int64_t b, int64_t inner_bytes, void* stream) {
    using namespace widek;
    if (a < 0 || b < 0 || inner_bytes < 0) return set_error(WIDEK_ERR_INVALID, "swap01: negative size");
    if (a == 0 || b == 0 || inner_bytes == 0) return WIDEK_OK;
    if (!src || !dst) return set_error(WIDEK_ERR_INVALID, "swap01: null pointer");
    cudaStream_t st = (cudaStream_t)stream;
    const uintptr_t align = reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst) | (uintptr_t)inner_bytes;
    if ((align & 15) == 0 && inner_bytes / 16 >= kRowThreads) {
        // Long rows of 16-byte units: row-chunked copy.
        const int64_t ru = inner_bytes / 16;
        const int64_t jobs = a * b * ((ru + kRowChunk - 1) / kRowChunk);
        const int grid = (int)std::min<int64_t>(jobs, (int64_t)sm_count(current_device()) * 8);
        swap01_rows_kernel<uint4><<<grid, kRowThreads, 0, st>>>(static_cast<const uint4*>(src),
                                                                 static_cast<uint4*>(dst), a, b, ru);
    } else if ((align & 15) == 0) {
        const int64_t ru = inner_bytes / 16;
        swap01_kernel<uint4><<<grid_for(a * b * ru, 256), 256, 0, st>>>(static_cast<const uint4*>(src),
                                                                       static_cast<uint4*>(dst), a, b, ru);
    } else if ((align & 3) == 0) {
        const int64_t ru = inner_bytes / 4;
        swap01_kernel<uint32_t><<<grid_for(a * b * ru, 256), 256, 0, st>>>(static_cast<const uint32_t*>(src),
                                                                          static_cast<uint32_t*>(dst), a, b, ru);
    } else if ((align & 1) == 0) {
        const int64_t ru = inner_bytes / 2;
        swap01_kernel<uint16_t><<<grid_for(a * b * ru, 256), 256, 0, st>>>(static_cast<const uint16_t*>(src),
                                                                          static_cast<uint16_t*>(dst), a, b, ru);
    } else {
        swap01_kernel<uint8_t><<<grid_for(a * b * inner_bytes, 256), 256, 0, st>>>(
            static_cast<const uint8_t*>(src), static_cast<uint8_t*>(dst), a, b, inner_bytes);
    }
    return check_launch("widek_swap01");
}

int widek_copy2d(const void* src, int64_t src_pitch, void* dst, int64_t dst_pitch, int64_t rows, int64_t row_bytes,
                 void* stream) {
    using namespace widek;
    if (rows < 0 || row_bytes < 0) return set_error(WIDEK_ERR_INVALID, "copy2d: negative size");
    if (rows == 0 || row_bytes == 0) return WIDEK_OK;
    if (!src || !dst) return set_error(WIDEK_ERR_INVALID, "copy2d: null pointer");
    if (src_pitch < row_bytes || dst_pitch < row_bytes)
        return set_error(WIDEK_ERR_INVALID, "copy2d: pitch (%lld, %lld) below the row size %lld", (long long)src_pitch,
                         (long long)dst_pitch, (long long)row_bytes);
    cudaStream_t st = (cudaStream_t)stream;
    const uintptr_t align = reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst) |
                            (uintptr_t)src_pitch | (uintptr_t)dst_pitch | (uintptr_t)row_bytes;
    if ((align & 15) == 0)
        launch_copy2d<uint4>(src, src_pitch, dst, dst_pitch, rows, row_bytes, st);
    else if ((align & 7) == 0)
        launch_copy2d<uint2>(src, src_pitch, dst, dst_pitch, rows, row_bytes, st);
    else if ((align & 3) == 0)
        launch_copy2d<uint32_t>(src, src_pitch, dst, dst_pitch, rows, row_bytes, st);
    else if ((align & 1) == 0)
        launch_copy2d<uint16_t>(src, src_pitch, dst, dst_pitch, rows, row_bytes, st);
    else
        launch_copy2d<uint8_t>(src, src_pitch, dst, dst_pitch, rows, row_bytes, st);
    return check_launch("widek_copy2d");
}

int widek_pack(const void* const* srcs, int64_t n, void* dst, int64_t b, int64_t inner_bytes, void* stream) {
    using namespace widek;
    if (n < 0 || b < 0 || inner_bytes < 0) return set_error(WIDEK_ERR_INVALID, "pack: negative size");
    if (n == 0 || b == 0 || inner_bytes == 0) return WIDEK_OK;
    if (!srcs || !dst) return set_error(WIDEK_ERR_INVALID, "pack: null pointer");
    uintptr_t align = reinterpret_cast<uintptr_t>(dst) | (uintptr_t)inner_bytes;
    for (int64_t i = 0; i < n; ++i) {
        if (!srcs[i]) return set_error(WIDEK_ERR_INVALID, "pack: null source %lld", (long long)i);
        align |= reinterpret_cast<uintptr_t>(srcs[i]);
    }
    cudaStream_t st = (cudaStream_t)stream;
    for (int64_t i0 = 0; i0 < n; i0 += kPackMax) {
        const int cnt = (int)std::min<int64_t>(kPackMax, n - i0);
        PackPtrs P;
        for (int i = 0; i < cnt; ++i) P.p[i] = srcs[i0 + i];
        if ((align & 15) == 0) {
            const int64_t ru = inner_bytes / 16;
            pack_kernel<uint4><<<grid_for(b * cnt * ru, 256), 256, 0, st>>>(P, cnt, n, i0, static_cast<uint4*>(dst),
                                                                             b, ru);
        } else if ((align & 3) == 0) {
            const int64_t ru = inner_bytes / 4;
            pack_kernel<uint32_t><<<grid_for(b * cnt * ru, 256), 256, 0, st>>>(P, cnt, n, i0,
                                                                                static_cast<uint32_t*>(dst), b, ru);
        } else {
            pack_kernel<uint8_t><<<grid_for(b * cnt * inner_bytes, 256), 256, 0, st>>>(
                P, cnt, n, i0, static_cast<uint8_t*>(dst), b, inner_bytes);
        }
        const int rc = check_launch("widek_pack");
        if (rc) return rc;
    }
    return WIDEK_OK;
}

}  // extern "C"
