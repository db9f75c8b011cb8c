// CUDA-core grouped GEMM: y[i] = act(x[i] @ w[i]^T + bias[i]) for every model.
//
// Serves fp32 WideLinear (fp32 FFMA, so results keep fp32 products: the
// reference's tolerance is defined with TF32 off) and any bf16/f16 problem the
// tensor-core kernel cannot take (k not a multiple of 8, unaligned pointers).
// Classic shared-memory tiling: a CTA computes a BM x BN output tile of one
// model; each thread owns TM consecutive rows and TN columns strided by
// BN / TN (so that a warp's B-tile reads are consecutive words: no bank
// conflict, and its output stores are coalesced).
#include "common.cuh"
#include "sm100_ptx.cuh"

namespace widek {
namespace {

template <typename T, int BM, int BN, int BK, int TM, int TN>
__global__ void __launch_bounds__((BM / TM) * (BN / TN))
    gemm_simt_kernel(const T* __restrict__ x, const T* __restrict__ w, const T* __restrict__ bias,
                     T* __restrict__ y, int M, int K, int O, int act, int64_t w_ms, int64_t w_rs, int64_t x_ms,
                     int64_t x_bs, int x_rpb, int64_t y_ms, int64_t y_bs) {
    constexpr int NT = (BM / TM) * (BN / TN);
    __shared__ float As[BK][BM + 4];
    __shared__ float Bs[BK][BN + 4];
    // A programmatic dependent of this kernel (the recurrence after the RNN
    // input projection) may start its set-up now; it waits for this grid's
    // results before reading them.
    sm100::grid_dep_launch_dependents();
    const int model = blockIdx.z;
    const int m0 = blockIdx.y * BM;
    const int o0 = blockIdx.x * BN;
    x += (int64_t)model * x_ms;
    w += (int64_t)model * w_ms;
    y += (int64_t)model * y_ms;
    const int tid = threadIdx.x;
    const int tx = tid % (BN / TN);
    const int ty = tid / (BN / TN);
    // Row offsets (elements) of the x rows this thread loads (the same rows
    // in every k tile) and of the y rows it stores: block-strided rows
    // (row r at (r / x_rpb)*x_bs + (r % x_rpb)*K), one division per row
    // instead of per element.
    constexpr int LOADS = (BM * BK + NT - 1) / NT;
    int64_t xoff[LOADS];
#pragma unroll
    for (int j = 0; j < LOADS; ++j) {
        const int gm = m0 + (tid + j * NT) / BK;
        xoff[j] = gm < M ? (int64_t)(gm / x_rpb) * x_bs + (int64_t)(gm % x_rpb) * K : 0;
    }

    float acc[TM][TN];
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) acc[i][j] = 0.f;

    for (int k0 = 0; k0 < K; k0 += BK) {
#pragma unroll
        for (int j = 0; j < LOADS; ++j) {
            const int i = tid + j * NT;
            if (i < BM * BK) {
                const int r = i / BK, c = i % BK;
                const int gm = m0 + r, gk = k0 + c;
                As[c][r] = (gm < M && gk < K) ? to_f<T>(x[xoff[j] + gk]) : 0.f;
            }
        }
        for (int i = tid; i < BN * BK; i += NT) {
            const int r = i / BK, c = i % BK;
            const int go = o0 + r, gk = k0 + c;
            Bs[c][r] = (go < O && gk < K) ? to_f<T>(w[(int64_t)go * w_rs + gk]) : 0.f;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < BK; ++kk) {
            float a[TM], b[TN];
#pragma unroll
            for (int i = 0; i < TM; ++i) a[i] = As[kk][ty * TM + i];
#pragma unroll
            for (int j = 0; j < TN; ++j) b[j] = Bs[kk][tx + (BN / TN) * j];
#pragma unroll
            for (int i = 0; i < TM; ++i)
#pragma unroll
                for (int j = 0; j < TN; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < TM; ++i) {
        const int gm = m0 + ty * TM + i;
        if (gm >= M) continue;
        T* yrow = y + (int64_t)(gm / x_rpb) * y_bs + (int64_t)(gm % x_rpb) * O;
#pragma unroll
        for (int j = 0; j < TN; ++j) {
            const int go = o0 + tx + (BN / TN) * j;
            if (go >= O) continue;
            float v = acc[i][j];
            if (bias) v += to_f<T>(bias[(int64_t)model * O + go]);
            yrow[go] = from_f<T>(apply_act(v, act));
        }
    }
}

struct SimtLaunch {
    const void *x, *w, *b;
    void* y;
    int64_t n, m, k, o;
    int act;
    cudaStream_t st;
    int64_t w_ms, w_rs;     // weight model / row strides (elements)
    int64_t x_ms = -1, x_bs = 0, x_rpb = 0;   // strided x (x_ms < 0: dense)
    int64_t y_ms = -1, y_bs = 0;              // strided y (y_ms < 0: dense)

    template <typename T>
    int run() {
        if (n > 65535) return set_error(WIDEK_ERR_UNSUPPORTED, "linear (simt): n=%lld > 65535", (long long)n);
        if (m > 0x7fffffff || k > 0x7fffffff || o > 0x7fffffff)
            return set_error(WIDEK_ERR_UNSUPPORTED, "linear (simt): dimension exceeds int32");
        const T* xp = static_cast<const T*>(x);
        const T* wp = static_cast<const T*>(w);
        const T* bp = static_cast<const T*>(b);
        T* yp = static_cast<T*>(y);
        const int64_t xms = x_ms < 0 ? m * k : x_ms;
        const int64_t xbs = x_ms < 0 ? 0 : x_bs;
        const int64_t xrpb = x_ms < 0 ? m : x_rpb;
        // y rows use the same row blocks as x (dense x: one block of m rows)
        const int64_t yms = y_ms < 0 ? m * o : y_ms;
        const int64_t ybs = y_ms < 0 ? (xrpb == m ? 0 : xrpb * o) : y_bs;
        if (xrpb <= 0 || xrpb > 0x7fffffff) return set_error(WIDEK_ERR_INVALID, "linear (simt): bad row block %lld",
                                                             (long long)xrpb);
        if (m <= 32) {
            dim3 grid((unsigned)((o + 63) / 64), (unsigned)((m + 31) / 32), (unsigned)n);
            gemm_simt_kernel<T, 32, 64, 16, 2, 4><<<grid, 256, 0, st>>>(xp, wp, bp, yp, (int)m, (int)k, (int)o, act, w_ms, w_rs, xms, xbs,
                                                                    (int)xrpb, yms, ybs);
        } else {
            dim3 grid((unsigned)((o + 63) / 64), (unsigned)((m + 63) / 64), (unsigned)n);
            if (grid.y > 65535) return set_error(WIDEK_ERR_UNSUPPORTED, "linear (simt): m too large");
            gemm_simt_kernel<T, 64, 64, 16, 4, 4><<<grid, 256, 0, st>>>(xp, wp, bp, yp, (int)m, (int)k, (int)o, act, w_ms, w_rs, xms, xbs,
                                                                    (int)xrpb, yms, ybs);
        }
        return check_launch("widek_linear_fwd_simt");
    }
};

}  // namespace

int linear_simt_strided(const void* x, const void* w, const void* bias, void* y, int64_t n, int64_t m, int64_t k,
                        int64_t o, int64_t w_ms, int64_t w_rs, int dtype, int act, cudaStream_t st, int64_t x_ms,
                        int64_t x_bs, int64_t x_rpb, int64_t y_ms, int64_t y_bs) {
    if (n == 0 || m == 0 || o == 0) return WIDEK_OK;
    SimtLaunch L{x, w, bias, y, n, m, k, o, act, st, w_ms, w_rs, x_ms, x_bs, x_rpb, y_ms, y_bs};
    return dispatch_dtype(dtype, L);
}

}  // namespace widek

extern "C" int widek_linear_fwd_simt(const void* x, const void* w, const void* bias, void* y, int64_t n, int64_t m,
                                     int64_t k, int64_t o, int dtype, int act, void* stream) {
    using namespace widek;
    if (n < 0 || m < 0 || k < 0 || o < 0) return set_error(WIDEK_ERR_INVALID, "linear: negative size");
    if (act < WIDEK_ACT_NONE || act > WIDEK_ACT_GELU) return set_error(WIDEK_ERR_INVALID, "linear: bad activation %d", act);
    if (n == 0 || m == 0 || o == 0) return WIDEK_OK;
    if (!x && k > 0) return set_error(WIDEK_ERR_INVALID, "linear: null x");
    if (!y) return set_error(WIDEK_ERR_INVALID, "linear: null y");
    SimtLaunch L{x, w, bias, y, n, m, k, o, act, (cudaStream_t)stream, o * k, k};
    return dispatch_dtype(dtype, L);
}
