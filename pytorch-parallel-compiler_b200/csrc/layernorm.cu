// WideLayerNorm forward: one HBM pass, statistics in fp32.
//
// Layout: x, y are [outer][n][inner][d] rows (contiguous); the per-model
// affine w, b are [n, d]. Row r belongs to model (r / inner) % n. The
// N-first layout [n, rows_per_model, d] is outer = 1, inner = rows_per_model;
// the packed TracedWideModel boundary layout [B, n*T, d] is outer = B,
// inner = T, so LayerNorm runs on either without a layout change.
//
// Fast path: one warp per row, the row held in registers as 16-byte vectors
// (mean and the biased variance are two exact passes over registers, so the
// row is read from HBM once and written once). Rows that do not fit the
// register budget, or unaligned/odd-width rows, take the block-per-row path.
#include "common.cuh"

namespace widek {
namespace {

// Model of a row: (row / inner) % n, with 32-bit division when the values
// fit (a 64-bit division is a long instruction sequence on the critical path
// to the affine loads) and no modulo in the N-first layout (quotient < n).
__device__ __forceinline__ int64_t model_of_row(int64_t row, int64_t inner, int64_t n) {
    int64_t q;
    if (((uint64_t)row | (uint64_t)inner) <= 0xffffffffull)
        q = (int64_t)((uint32_t)row / (uint32_t)inner);
    else
        q = row / inner;
    if (q >= n) q = (n <= 0xffffffffll && q <= 0xffffffffll) ? (int64_t)((uint32_t)q % (uint32_t)n) : q % n;
    return q;
}

template <typename T, int MAXV>
__global__ void __launch_bounds__(256) layernorm_warp_kernel(
    const T* __restrict__ x, const T* __restrict__ w, const T* __restrict__ b,
    T* __restrict__ y, int64_t rows, int64_t inner, int64_t n, int d, float eps) {
    constexpr int VEC = 16 / sizeof(T);
    const int lane = threadIdx.x & 31;
    const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (row >= rows) return;
    const int nvec = d / VEC;
    const T* xr = x + row * d;
    float v[MAXV][VEC];
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
        const int vi = lane + 32 * i;
        if (vi < nvec) {
            load16<T>(xr + vi * VEC, v[i]);
#pragma unroll
            for (int j = 0; j < VEC; ++j) s += v[i][j];
        }
    }
    const float mean = warp_sum(s) / (float)d;
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
        const int vi = lane + 32 * i;
        if (vi < nvec) {
#pragma unroll
            for (int j = 0; j < VEC; ++j) {
                const float t = v[i][j] - mean;
                q += t * t;
            }
        }
    }
    const float var = warp_sum(q) / (float)d;
    const float rstd = rsqrtf(var + eps);
    const int64_t model = model_of_row(row, inner, n);
    const T* wr = w + model * d;
    const T* br = b + model * d;
    T* yr = y + row * d;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
        const int vi = lane + 32 * i;
        if (vi < nvec) {
            float wv[VEC], bv[VEC], o[VEC];
            load16<T>(wr + vi * VEC, wv);
            load16<T>(br + vi * VEC, bv);
#pragma unroll
            for (int j = 0; j < VEC; ++j) o[j] = (v[i][j] - mean) * rstd * wv[j] + bv[j];
            store16<T>(yr + vi * VEC, o);
        }
    }
}

// General path: one 256-thread block per row, scalar accesses.
template <typename T>
__global__ void __launch_bounds__(256) layernorm_block_kernel(
    const T* __restrict__ x, const T* __restrict__ w, const T* __restrict__ b,
    T* __restrict__ y, int64_t inner, int64_t n, int d, float eps) {
    __shared__ float red[32];
    const int64_t row = blockIdx.x;
    const T* xr = x + row * d;
    float s = 0.f;
    for (int i = threadIdx.x; i < d; i += blockDim.x) s += to_f<T>(xr[i]);
    s = warp_sum(s);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x < 32) {
        float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
        t = warp_sum(t);
        if (threadIdx.x == 0) red[0] = t;
    }
    __syncthreads();
    const float mean = red[0] / (float)d;
    __syncthreads();
    float q = 0.f;
    for (int i = threadIdx.x; i < d; i += blockDim.x) {
        const float t = to_f<T>(xr[i]) - mean;
        q += t * t;
    }
    q = warp_sum(q);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = q;
    __syncthreads();
    if (threadIdx.x < 32) {
        float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
        t = warp_sum(t);
        if (threadIdx.x == 0) red[0] = t;
    }
    __syncthreads();
    const float rstd = rsqrtf(red[0] / (float)d + eps);
    const int64_t model = model_of_row(row, inner, n);
    const T* wr = w + model * d;
    const T* br = b + model * d;
    T* yr = y + row * d;
    for (int i = threadIdx.x; i < d; i += blockDim.x)
        yr[i] = from_f<T>((to_f<T>(xr[i]) - mean) * rstd * to_f<T>(wr[i]) + to_f<T>(br[i]));
}

struct LayerNormLaunch {
    const void *x, *w, *b;
    void* y;
    int64_t n, outer, inner, d;
    float eps;
    cudaStream_t st;

    template <typename T>
    int run() {
        constexpr int VEC = 16 / sizeof(T);
        const int64_t rows = outer * n * inner;
        if (rows == 0 || d == 0) return WIDEK_OK;
        const bool vec_ok = (d % VEC == 0) && aligned16(x) && aligned16(w) && aligned16(b) && aligned16(y);
        const int64_t per_lane = (d / VEC + 31) / 32;
        const T* xp = static_cast<const T*>(x);
        const T* wp = static_cast<const T*>(w);
        const T* bp = static_cast<const T*>(b);
        T* yp = static_cast<T*>(y);
        if (vec_ok && per_lane <= 8) {
            const int warps = 8;
            const int64_t blocks = (rows + warps - 1) / warps;
            if (blocks > 0x7fffffff) return set_error(WIDEK_ERR_INVALID, "layernorm: too many rows");
            dim3 grid((unsigned)blocks), block(32 * warps);
            if (per_lane <= 1)
                layernorm_warp_kernel<T, 1><<<grid, block, 0, st>>>(xp, wp, bp, yp, rows, inner, n, (int)d, eps);
            else if (per_lane <= 2)
                layernorm_warp_kernel<T, 2><<<grid, block, 0, st>>>(xp, wp, bp, yp, rows, inner, n, (int)d, eps);
            else if (per_lane <= 4)
                layernorm_warp_kernel<T, 4><<<grid, block, 0, st>>>(xp, wp, bp, yp, rows, inner, n, (int)d, eps);
            else
                layernorm_warp_kernel<T, 8><<<grid, block, 0, st>>>(xp, wp, bp, yp, rows, inner, n, (int)d, eps);
        } else {
            if (rows > 0x7fffffff) return set_error(WIDEK_ERR_INVALID, "layernorm: too many rows");
            layernorm_block_kernel<T><<<(unsigned)rows, 256, 0, st>>>(xp, wp, bp, yp, inner, n, (int)d, eps);
        }
        return check_launch("widek_layernorm_fwd");
    }
};

}  // namespace
}  // namespace widek

extern "C" int widek_layernorm_fwd_ex(const void* x, const void* w, const void* b, void* y, int64_t n,
                                      int64_t outer, int64_t inner, int64_t d, double eps, int dtype,
                                      void* stream) {
    using namespace widek;
    if (n < 0 || outer < 0 || inner < 0 || d < 0 || d > (1 << 30))
        return set_error(WIDEK_ERR_INVALID, "layernorm: bad sizes n=%lld outer=%lld inner=%lld d=%lld",
                         (long long)n, (long long)outer, (long long)inner, (long long)d);
    if (n * outer * inner * d > 0 && (!x || !w || !b || !y))
        return set_error(WIDEK_ERR_INVALID, "layernorm: null pointer");
    LayerNormLaunch L{x, w, b, y, n, outer, inner, d, (float)eps, (cudaStream_t)stream};
    return dispatch_dtype(dtype, L);
}

extern "C" int widek_layernorm_fwd(const void* x, const void* w, const void* b, void* y,
                                   int64_t n, int64_t rows_per_model, int64_t d,
                                   double eps, int dtype, void* stream) {
    return widek_layernorm_fwd_ex(x, w, b, y, n, 1, rows_per_model, d, eps, dtype, stream);
}
