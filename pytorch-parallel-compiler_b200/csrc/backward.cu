// Backward kernels for WideLinear (and its fused activation) and
// WideLayerNorm.
//
// The reference trains through torch autograd over its primitives' plain
// torch forward (wide_linear.py:162-171 einsum 'noi,nbi->nbo' + bias;
// wide_layernorm.py:62-65 F.layer_norm on the [N, ..., D] view times the
// flat [N*D] affine); its gradient-flow test is wide_lstm.py:744-762. The
// gradients here are the same formulas, computed on the GPU:
//
//   WideLinear  y[i] = x[i] W[i]^T + b[i]     (x [N, M, K], W [N, O, K])
//     dX[i] = dY[i] W[i]          dW[i] = dY[i]^T x[i]      db[i] = sum_rows dY[i]
//   For bf16/f16 with 16-byte rows both products run on the tcgen05 GEMM
//   with MN-major operands read straight from W, dY and x (dX: W MN-major;
//   dW: dY and x MN-major). Otherwise (fp32: split-operand tcgen05 or CUDA
//   cores; ragged widths) they run on the forward's K-major GEMM:
//   dX = dY . (W^T)^T needs W^T [N, K, O]; dW = (dY^T) . (x^T)^T needs
//   dY^T [N, O, M] and x^T [N, K, M], from one batched transpose kernel into
//   a caller-provided workspace. The bias gradient is a column sum
//   (per-block partials in fp32, then one pass over the blocks, so the
//   result does not depend on scheduling).
//
//   activation  dpre = dY * act'(.)   ReLU from the saved output (y > 0),
//                                     exact-erf GELU from the saved
//                                     pre-activation: Phi(x) + x phi(x)
//
//   WideLayerNorm  x_hat = (x - mean) * rstd,  g = dY * gamma
//     dX = rstd * (g - mean(g) - x_hat * mean(g * x_hat))
//     dgamma = sum_rows dY * x_hat,  dbeta = sum_rows dY
//   One warp per row (statistics recomputed from the row held in
//   registers), each CTA working on rows of one model and keeping its
//   dgamma/dbeta partial sums in registers; a second kernel adds the CTAs'
//   partials per model.
#include "common.cuh"

#include <cuda_runtime.h>

#include <type_traits>

namespace widek {
namespace {

// ---------------------------------------------------------------------------
// Batched transpose: x [batch, R, C] -> y [batch, C, R]
//
// 64 x 64 tiles through shared memory. Rows are read and written as 16-byte
// vectors when the row lengths and base pointers allow it (C, resp. R, a
// multiple of the vector), else element by element; consecutive threads
// touch consecutive addresses in both phases. The shared tile's pitch
// (65 words / 66 halfwords) keeps the column reads at most 2-way
// bank-conflicted.
// ---------------------------------------------------------------------------
constexpr int kTT = 64;
constexpr int kTThreads = 256;

template <typename T>
__global__ void __launch_bounds__(kTThreads) transpose_kernel(const T* __restrict__ x, T* __restrict__ y, int64_t R,
                                                               int64_t C, bool vec_in, bool vec_out) {
    constexpr int VEC = 16 / sizeof(T);
    constexpr int PITCH = sizeof(T) == 4 ? kTT + 1 : kTT + 2;
    __shared__ T tile[kTT * PITCH];
    const int64_t b = blockIdx.z;
    const int64_t r0 = (int64_t)blockIdx.y * kTT, c0 = (int64_t)blockIdx.x * kTT;
    const T* xb = x + b * R * C;
    T* yb = y + b * R * C;
    const int tid = threadIdx.x;
    if (vec_in) {
        constexpr int PER_ROW = kTT / VEC;
        for (int i = tid; i < kTT * PER_ROW; i += kTThreads) {
            const int r = i / PER_ROW, cv = i % PER_ROW;
            const int64_t gr = r0 + r, gc = c0 + (int64_t)cv * VEC;
            if (gr < R && gc < C) {
                uint4 raw = *reinterpret_cast<const uint4*>(xb + gr * C + gc);
                const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
                for (int j = 0; j < VEC; ++j) tile[r * PITCH + cv * VEC + j] = e[j];
            }
        }
    } else {
        for (int i = tid; i < kTT * kTT; i += kTThreads) {
            const int r = i / kTT, c = i % kTT;
            const int64_t gr = r0 + r, gc = c0 + c;
            if (gr < R && gc < C) tile[r * PITCH + c] = xb[gr * C + gc];
        }
    }
    __syncthreads();
    if (vec_out) {
        constexpr int PER_COL = kTT / VEC;
        for (int i = tid; i < kTT * PER_COL; i += kTThreads) {
            const int c = i / PER_COL, rv = i % PER_COL;
            const int64_t gc = c0 + c, gr = r0 + (int64_t)rv * VEC;
            if (gc < C && gr < R) {
                uint4 raw;
                T* e = reinterpret_cast<T*>(&raw);
#pragma unroll
                for (int j = 0; j < VEC; ++j) e[j] = tile[(rv * VEC + j) * PITCH + c];
                *reinterpret_cast<uint4*>(yb + gc * R + gr) = raw;
            }
        }
    } else {
        for (int i = tid; i < kTT * kTT; i += kTThreads) {
            const int c = i / kTT, r = i % kTT;
            const int64_t gc = c0 + c, gr = r0 + r;
            if (gc < C && gr < R) yb[gc * R + gr] = tile[r * PITCH + c];
        }
    }
}

int launch_transpose(const void* x, void* y, int64_t batch, int64_t R, int64_t C, size_t esize, cudaStream_t st) {
    if (batch == 0 || R == 0 || C == 0) return WIDEK_OK;
    if (batch > 65535) return set_error(WIDEK_ERR_UNSUPPORTED, "transpose: more than 65535 matrices");
    const int64_t vec = 16 / (int64_t)esize;
    const bool vin = C % vec == 0 && aligned16(x), vout = R % vec == 0 && aligned16(y);
    const dim3 grid((unsigned)((C + kTT - 1) / kTT), (unsigned)((R + kTT - 1) / kTT), (unsigned)batch);
    if ((R + kTT - 1) / kTT > 65535) return set_error(WIDEK_ERR_UNSUPPORTED, "transpose: too many row tiles");
    if (esize == 4)
        transpose_kernel<float><<<grid, kTThreads, 0, st>>>(static_cast<const float*>(x), static_cast<float*>(y), R, C,
                                                            vin, vout);
    else
        transpose_kernel<__half><<<grid, kTThreads, 0, st>>>(static_cast<const __half*>(x), static_cast<__half*>(y),
                                                             R, C, vin, vout);
    return check_launch("transpose");
}

// ---------------------------------------------------------------------------
// Column sums: part[i][blk][c] = sum over the block's rows of x[i][r][c]
// (fp32), then out[i][c] = sum over blocks, in the storage dtype.
// ---------------------------------------------------------------------------
constexpr int kSumThreads = 256;
constexpr int kSumRows = 32;          // rows per partial

// PAIR: two adjacent 16-bit columns per thread (one 4-byte load per row, so
// a warp reads 128 contiguous bytes of a row, as in the fp32 case).
template <typename T, bool PAIR>
__global__ void __launch_bounds__(kSumThreads) colsum_part_kernel(const T* __restrict__ x, float* __restrict__ part,
                                                                   int64_t M, int64_t C, int nblk) {
    constexpr int P = PAIR ? 2 : 1;
    const int64_t i = blockIdx.z;
    const int blk = blockIdx.y;
    const int64_t c = ((int64_t)blockIdx.x * kSumThreads + threadIdx.x) * P;
    if (c >= C) return;
    const int64_t r_end = min(M, (int64_t)(blk + 1) * kSumRows);
    const T* p = x + i * M * C + c;
    float s0[P], s1[P];
#pragma unroll
    for (int q = 0; q < P; ++q) s0[q] = s1[q] = 0.f;
    int64_t r = (int64_t)blk * kSumRows;
    auto add = [&](float (&acc)[P], int64_t row) {
        if constexpr (PAIR) {
            const uint32_t w = *reinterpret_cast<const uint32_t*>(p + row * C);
            const T* e = reinterpret_cast<const T*>(&w);
            acc[0] += to_f<T>(e[0]);
            acc[P - 1] += to_f<T>(e[1]);
        } else {
            acc[0] += to_f<T>(p[row * C]);
        }
    };
    for (; r + 4 <= r_end; r += 4) {       // four independent loads in flight
        add(s0, r);
        add(s1, r + 1);
        add(s0, r + 2);
        add(s1, r + 3);
    }
    for (; r < r_end; ++r) add(s0, r);
#pragma unroll
    for (int q = 0; q < P; ++q) part[(i * nblk + blk) * C + c + q] = s0[q] + s1[q];
}

template <typename T>
__global__ void __launch_bounds__(kSumThreads) colsum_final_kernel(const float* __restrict__ part, T* __restrict__ out,
                                                                    int64_t C, int nblk) {
    const int64_t i = blockIdx.y;
    const int64_t c = (int64_t)blockIdx.x * kSumThreads + threadIdx.x;
    if (c >= C) return;
    float s = 0.f;
    for (int b = 0; b < nblk; ++b) s += part[(i * nblk + b) * C + c];
    out[i * C + c] = from_f<T>(s);
}

// ---------------------------------------------------------------------------
// Activation gradient: dpre = dy * act'(s); s = the saved output (ReLU) or
// pre-activation (GELU).
// ---------------------------------------------------------------------------
__device__ __forceinline__ float act_grad(float s, int act) {
    if (act == WIDEK_ACT_RELU) return s > 0.f ? 1.f : 0.f;
    // d/dx [x * Phi(x)] = Phi(x) + x * phi(x), Phi the standard normal CDF
    const float cdf = 0.5f * (1.0f + erff(s * 0.70710678118654752f));
    const float pdf = 0.39894228040143268f * expf(-0.5f * s * s);
    return cdf + s * pdf;
}

template <typename T>
__global__ void act_bwd_kernel(const T* __restrict__ dy, const T* __restrict__ s, T* __restrict__ out, int64_t count,
                               int act, bool vec) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (vec) {
        constexpr int V = 16 / sizeof(T);
        const int64_t nv = count / V;
        for (int64_t i = t; i < nv; i += stride) {
            float a[V], b[V];
            load16<T>(dy + i * V, a);
            load16<T>(s + i * V, b);
#pragma unroll
            for (int j = 0; j < V; ++j) a[j] *= act_grad(b[j], act);
            store16<T>(out + i * V, a);
        }
    } else {
        for (int64_t i = t; i < count; i += stride)
            out[i] = from_f<T>(to_f<T>(dy[i]) * act_grad(to_f<T>(s[i]), act));
    }
}

// ---------------------------------------------------------------------------
// LayerNorm backward. x, dy, dx: [n, outer, d] (N-first, dense); gamma flat
// [n*d]. Grid (nblk, n): CTA (blk, i) takes rows [blk*rpc, (blk+1)*rpc) of
// model i, one warp per row; lane l holds the row's chunks l, l+32, ... of V
// elements (16-byte vectors when d and the pointers allow, else V = 1).
// part: [n, nblk, 2, d] fp32 (dgamma, dbeta partial sums).
// ---------------------------------------------------------------------------
constexpr int kLnThreads = 256;
constexpr int kLnWarps = kLnThreads / 32;
constexpr int kLnMaxD = 1024;
constexpr int kLnTargetCtas = 296;    // 2 per SM on a 148-SM part

template <typename T, int V>
__device__ __forceinline__ void ln_load(const T* p, float* out) {
    if constexpr (V == 1) out[0] = to_f<T>(*p);
    else load16<T>(p, out);
}
template <typename T, int V>
__device__ __forceinline__ void ln_store(T* p, const float* in) {
    if constexpr (V == 1) *p = from_f<T>(in[0]);
    else store16<T>(p, in);
}

template <typename T, int V, int CPL>
__global__ void __launch_bounds__(kLnThreads) layernorm_bwd_kernel(const T* __restrict__ x, const T* __restrict__ w,
                                                                    const T* __restrict__ dy, T* __restrict__ dx,
                                                                    float* __restrict__ part, int64_t outer, int d,
                                                                    float eps, int64_t rpc, int nblk) {
    constexpr int E = CPL * V;
    __shared__ float red[kLnWarps * kLnMaxD];
    __shared__ float gam[kLnMaxD];
    const int64_t model = blockIdx.y;
    const int blk = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nch = d / V;
    const float inv_d = 1.0f / (float)d;
    for (int j = threadIdx.x; j < d; j += kLnThreads) gam[j] = to_f<T>(w[model * d + j]);
    __syncthreads();
    float ag[E], ab[E];
#pragma unroll
    for (int e = 0; e < E; ++e) ag[e] = ab[e] = 0.f;
    const int64_t r_begin = (int64_t)blk * rpc;
    const int64_t r_end = min(outer, r_begin + rpc);
    // The next row's raw bytes are loaded before the current row is
    // reduced, so each warp keeps two rows in flight.
    using Raw = typename std::conditional<V == 1, T, uint4>::type;
    Raw px[CPL], pg[CPL];
    auto load_raw = [&](int64_t row) {
        const int64_t o = (model * outer + row) * d;
#pragma unroll
        for (int c = 0; c < CPL; ++c) {
            const int ch = lane + 32 * c;
            if (ch < nch) {
                px[c] = *reinterpret_cast<const Raw*>(x + o + (int64_t)ch * V);
                pg[c] = *reinterpret_cast<const Raw*>(dy + o + (int64_t)ch * V);
            }
        }
    };
    if (r_begin + warp < r_end) load_raw(r_begin + warp);
    for (int64_t r = r_begin + warp; r < r_end; r += kLnWarps) {
        const int64_t off = (model * outer + r) * d;
        float xv[E], gv[E];
#pragma unroll
        for (int c = 0; c < CPL; ++c) {
            const int ch = lane + 32 * c;
            const T* ex = reinterpret_cast<const T*>(&px[c]);
            const T* eg = reinterpret_cast<const T*>(&pg[c]);
#pragma unroll
            for (int j = 0; j < V; ++j) {
                xv[c * V + j] = ch < nch ? to_f<T>(ex[j]) : 0.f;
                gv[c * V + j] = ch < nch ? to_f<T>(eg[j]) : 0.f;
            }
        }
        if (r + kLnWarps < r_end) load_raw(r + kLnWarps);
        float s = 0.f;
#pragma unroll
        for (int e = 0; e < E; ++e) s += xv[e];
        const float mean = warp_sum(s) * inv_d;
        float q = 0.f;
#pragma unroll
        for (int c = 0; c < CPL; ++c) {
            if (lane + 32 * c < nch) {
#pragma unroll
                for (int j = 0; j < V; ++j) {
                    const float t = xv[c * V + j] - mean;
                    q += t * t;
                }
            }
        }
        const float rstd = rsqrtf(warp_sum(q) * inv_d + eps);
        float s1 = 0.f, s2 = 0.f;
#pragma unroll
        for (int c = 0; c < CPL; ++c) {
            if (lane + 32 * c < nch) {
#pragma unroll
                for (int j = 0; j < V; ++j) {
                    const int e = c * V + j;
                    const float xh = (xv[e] - mean) * rstd;
                    ag[e] += gv[e] * xh;
                    ab[e] += gv[e];
                    const float g = gv[e] * gam[(lane + 32 * c) * V + j];
                    s1 += g;
                    s2 += g * xh;
                    xv[e] = xh;
                    gv[e] = g;
                }
            }
        }
        s1 = warp_sum(s1) * inv_d;
        s2 = warp_sum(s2) * inv_d;
#pragma unroll
        for (int c = 0; c < CPL; ++c) {
            const int ch = lane + 32 * c;
            if (ch < nch) {
                float o[V];
#pragma unroll
                for (int j = 0; j < V; ++j) o[j] = rstd * (gv[c * V + j] - s1 - xv[c * V + j] * s2);
                ln_store<T, V>(dx + off + (int64_t)ch * V, o);
            }
        }
    }
    // dgamma / dbeta partials of this CTA: the 8 warps' sums added in a fixed
    // order through shared memory.
    float* out = part + ((model * nblk + blk) * 2) * d;
#pragma unroll 1
    for (int a = 0; a < 2; ++a) {
        const float* acc = a == 0 ? ag : ab;
#pragma unroll
        for (int c = 0; c < CPL; ++c) {
            const int ch = lane + 32 * c;
            if (ch < nch) {
#pragma unroll
                for (int j = 0; j < V; ++j) red[warp * kLnMaxD + ch * V + j] = acc[c * V + j];
            }
        }
        __syncthreads();
        for (int j = threadIdx.x; j < d; j += kLnThreads) {
            float t = 0.f;
#pragma unroll
            for (int q = 0; q < kLnWarps; ++q) t += red[q * kLnMaxD + j];
            out[(int64_t)a * d + j] = t;
        }
        __syncthreads();
    }
}

// dgamma[i*d + j] = sum over blocks of part[i][blk][0][j] (dbeta: [1]).
// A CTA takes 32 columns; its 8 warps sum every 8th block each (lanes on
// consecutive columns), then warp 0 adds the 8 partial sums in order.
template <typename T>
__global__ void __launch_bounds__(kSumThreads) ln_param_reduce_kernel(const float* __restrict__ part, T* __restrict__ dw,
                                                                       T* __restrict__ db, int d, int nblk) {
    __shared__ float red[2][kSumThreads / 32][32];
    const int64_t i = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int j = blockIdx.x * 32 + lane;
    float sg = 0.f, sb = 0.f;
    if (j < d) {
        for (int b = warp; b < nblk; b += kSumThreads / 32) {
            const float* p = part + ((i * nblk + b) * 2) * d;
            sg += p[j];
            sb += p[d + j];
        }
    }
    red[0][warp][lane] = sg;
    red[1][warp][lane] = sb;
    __syncthreads();
    if (warp == 0 && j < d) {
        float g = 0.f, bsum = 0.f;
#pragma unroll
        for (int q = 0; q < kSumThreads / 32; ++q) {
            g += red[0][q][lane];
            bsum += red[1][q][lane];
        }
        if (dw) dw[i * d + j] = from_f<T>(g);
        if (db) db[i * d + j] = from_f<T>(bsum);
    }
}

int ln_blocks(int64_t n, int64_t outer) {
    int64_t nb = (kLnTargetCtas + n - 1) / (n > 0 ? n : 1);
    const int64_t max_nb = (outer + kLnWarps - 1) / kLnWarps;
    if (nb > max_nb) nb = max_nb;
    if (nb < 1) nb = 1;
    if (nb > 65535) nb = 65535;
    return (int)nb;
}

size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

struct LnBwdLaunch {
    const void *x, *w, *dy;
    void *dx, *dw, *db;
    float* part;
    int64_t n, outer;
    int d;
    float eps;
    int nblk;
    cudaStream_t st;

    template <typename T, int V, int CPL>
    void go(int64_t rpc) {
        layernorm_bwd_kernel<T, V, CPL><<<dim3((unsigned)nblk, (unsigned)n), kLnThreads, 0, st>>>(
            static_cast<const T*>(x), static_cast<const T*>(w), static_cast<const T*>(dy), static_cast<T*>(dx), part,
            outer, d, eps, rpc, nblk);
    }
    template <typename T>
    int run() {
        constexpr int VV = 16 / sizeof(T);
        const bool vec = d % VV == 0 && aligned16(x) && aligned16(w) && aligned16(dy) && aligned16(dx);
        const int v = vec ? VV : 1;
        const int nch = d / v;
        int cpl = 1;
        while (cpl * 32 < nch) cpl <<= 1;
        if (cpl * v > 32) return set_error(WIDEK_ERR_UNSUPPORTED, "layernorm_bwd: d = %d too large for the register row", d);
        const int64_t rpc = (outer + nblk - 1) / nblk;
        if (vec) {
            switch (cpl) {
                case 1: go<T, VV, 1>(rpc); break;
                case 2: go<T, VV, 2>(rpc); break;
                case 4: go<T, VV, 4>(rpc); break;
                default:
                    if constexpr (VV == 4) go<T, VV, 8>(rpc);   // fp32: 8 chunks of 4
                    break;
            }
        } else {
            switch (cpl) {
                case 1: go<T, 1, 1>(rpc); break;
                case 2: go<T, 1, 2>(rpc); break;
                case 4: go<T, 1, 4>(rpc); break;
                case 8: go<T, 1, 8>(rpc); break;
                case 16: go<T, 1, 16>(rpc); break;
                default: go<T, 1, 32>(rpc); break;
            }
        }
        int rc = check_launch("layernorm_bwd");
        if (rc != WIDEK_OK || (!dw && !db)) return rc;
        ln_param_reduce_kernel<T><<<dim3((unsigned)((d + 31) / 32), (unsigned)n), kSumThreads, 0, st>>>(
            part, static_cast<T*>(dw), static_cast<T*>(db), d, nblk);
        return check_launch("layernorm_bwd (parameter sums)");
    }
};

}  // namespace
}  // namespace widek

namespace widek {
namespace {

// ---------------------------------------------------------------------------
// BatchNorm / GroupNorm backward (InstanceNorm is GroupNorm with one channel
// per group). x, dy, dx: [n, B, C, L] dense (L = spatial size). A segment is
// the set of elements one statistic covers: BatchNorm (i, c): B chunks of L
// elements, C*L apart; GroupNorm (i, b, g): cg = C/G consecutive chunks of L
// elements. Chunk k of a segment has channel ch0 + k * chan_step.
//   x_hat = (x - mean) * rstd, g = dy * gamma_ch, M = elements of the segment
//   batch statistics: dx = rstd * (g - mean(g) - x_hat * mean(g * x_hat))
//   running statistics (BatchNorm in eval mode): dx = rstd * g
//   dgamma_ch = sum dy * x_hat, dbeta_ch = sum dy over the channel's elements
// One CTA per segment: pass 1 accumulates sum x, sum x^2 (shifted by the
// segment's first element), sum g and sum g * x; pass 2 (the segment again,
// mostly from L2) writes dx and the parameter sums: per segment for
// BatchNorm (the channel is the segment), per (segment, channel) partials
// for GroupNorm, added over the batch by a second kernel in a fixed order.
// ---------------------------------------------------------------------------
constexpr int kNbThreads = 256;

struct NormBwdArgs {
    const void *x, *dy, *w, *rmean, *rvar;
    void *dx, *dw, *db;
    float* part;                    // GroupNorm: [n * B][C][2] (dgamma, dbeta) partials
    int64_t n, batch, c, l;
    int groups;                     // 0: BatchNorm
    int batch_stats;                // BatchNorm: 1 = batch statistics, 0 = running statistics
    float eps;
};

__device__ __forceinline__ float nb_block_sum(float v, float* red) {
    v = warp_sum(v);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();                 // red is free (a previous sum has been read)
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = 0.f;
#pragma unroll
    for (int q = 0; q < kNbThreads / 32; ++q) t += red[q];
    return t;
}

template <typename T, bool VEC>
__global__ void __launch_bounds__(kNbThreads) norm_bwd_kernel(NormBwdArgs a) {
    __shared__ float red[kNbThreads / 32];
    constexpr int V = VEC ? 16 / (int)sizeof(T) : 1;
    const T* x = static_cast<const T*>(a.x);
    const T* dy = static_cast<const T*>(a.dy);
    const T* w = static_cast<const T*>(a.w);
    T* dx = static_cast<T*>(a.dx);
    const int64_t seg = blockIdx.x;
    const bool bn = a.groups == 0;
    int64_t base, kstride, ch0, chan_step, chunks;
    if (bn) {
        const int64_t i = seg / a.c, c = seg % a.c;
        base = (i * a.batch * a.c + c) * a.l;
        kstride = a.c * a.l;
        ch0 = i * a.c + c;
        chan_step = 0;
        chunks = a.batch;
    } else {
        const int64_t cg = a.c / a.groups;
        const int64_t g = seg % a.groups, ib = seg / a.groups, i = ib / a.batch;
        base = (ib * a.c + g * cg) * a.l;
        kstride = a.l;
        ch0 = i * a.c + g * cg;
        chan_step = 1;
        chunks = cg;
    }
    const int64_t L = a.l, M = chunks * L;
    const int64_t nv = L / V;               // vectors per chunk
    const float shift = to_f<T>(x[base]);
    auto gamma = [&](int64_t ch) { return w ? to_f<T>(w[ch]) : 1.f; };
    // pass 1
    float sx = 0.f, sxx = 0.f, sg = 0.f, sgx = 0.f;
    for (int64_t k = 0; k < chunks; ++k) {
        const int64_t off = base + k * kstride;
        const float gm = gamma(ch0 + k * chan_step);
        for (int64_t q = threadIdx.x; q < nv; q += kNbThreads) {
            float xv[V], gv[V];
            if constexpr (VEC) {
                load16<T>(x + off + q * V, xv);
                load16<T>(dy + off + q * V, gv);
            } else {
                xv[0] = to_f<T>(x[off + q]);
                gv[0] = to_f<T>(dy[off + q]);
            }
#pragma unroll
            for (int e = 0; e < V; ++e) {
                const float d = xv[e] - shift, g = gv[e] * gm;
                sx += d;
                sxx += d * d;
                sg += g;
                sgx += g * d;
            }
        }
    }
    const float inv_m = 1.0f / (float)M;
    const float m_d = nb_block_sum(sx, red) * inv_m;              // mean of x - shift
    const float var_b = fmaxf(nb_block_sum(sxx, red) * inv_m - m_d * m_d, 0.f);
    const float mg = nb_block_sum(sg, red) * inv_m;                // mean of g
    const float mgd = nb_block_sum(sgx, red) * inv_m;              // mean of g * (x - shift)
    float mean, rstd;
    if (bn && !a.batch_stats) {
        mean = to_f<T>(static_cast<const T*>(a.rmean)[ch0]);
        rstd = rsqrtf(to_f<T>(static_cast<const T*>(a.rvar)[ch0]) + a.eps);
    } else {
        mean = shift + m_d;
        rstd = rsqrtf(var_b + a.eps);
    }
    // mean(g * x_hat) = rstd * (mean(g * (x - shift)) - (mean - shift) * mean(g))
    const float mgxh = rstd * (mgd - (mean - shift) * mg);
    const bool full = !(bn && !a.batch_stats);
    // pass 2
    float pdw = 0.f, pdb = 0.f;
    for (int64_t k = 0; k < chunks; ++k) {
        const int64_t off = base + k * kstride;
        const int64_t ch = ch0 + k * chan_step;
        const float gm = gamma(ch);
        for (int64_t q = threadIdx.x; q < nv; q += kNbThreads) {
            float xv[V], gv[V], o[V];
            if constexpr (VEC) {
                load16<T>(x + off + q * V, xv);
                load16<T>(dy + off + q * V, gv);
            } else {
                xv[0] = to_f<T>(x[off + q]);
                gv[0] = to_f<T>(dy[off + q]);
            }
#pragma unroll
            for (int e = 0; e < V; ++e) {
                const float xh = (xv[e] - mean) * rstd;
                pdw += gv[e] * xh;
                pdb += gv[e];
                const float g = gv[e] * gm;
                o[e] = full ? rstd * (g - mg - xh * mgxh) : rstd * g;
            }
            if constexpr (VEC) store16<T>(dx + off + q * V, o);
            else dx[off + q] = from_f<T>(o[0]);
        }
        if (!bn) {
            // GroupNorm: this chunk is one channel; its partial sums
            const float tw = nb_block_sum(pdw, red), tb = nb_block_sum(pdb, red);
            if (threadIdx.x == 0) {
                const int64_t ib = seg / a.groups;
                const int64_t cl = ch - (ib / a.batch) * a.c;
                a.part[((ib * a.c) + cl) * 2] = tw;
                a.part[((ib * a.c) + cl) * 2 + 1] = tb;
            }
            pdw = pdb = 0.f;
        }
    }
    if (bn) {
        const float tw = nb_block_sum(pdw, red), tb = nb_block_sum(pdb, red);
        if (threadIdx.x == 0) {
            if (a.dw) static_cast<T*>(a.dw)[ch0] = from_f<T>(tw);
            if (a.db) static_cast<T*>(a.db)[ch0] = from_f<T>(tb);
        }
    }
}

// GroupNorm parameter gradients: dgamma[i*C + c] = sum over b of part[i][b][c].
template <typename T>
__global__ void __launch_bounds__(kSumThreads) gn_param_reduce_kernel(const float* __restrict__ part, T* dw, T* db,
                                                                       int64_t n, int64_t batch, int64_t c) {
    const int64_t idx = (int64_t)blockIdx.x * kSumThreads + threadIdx.x;
    if (idx >= n * c) return;
    const int64_t i = idx / c, cl = idx % c;
    float tw = 0.f, tb = 0.f;
    for (int64_t b = 0; b < batch; ++b) {
        const float* p = part + (((i * batch + b) * c) + cl) * 2;
        tw += p[0];
        tb += p[1];
    }
    if (dw) dw[idx] = from_f<T>(tw);
    if (db) db[idx] = from_f<T>(tb);
}

struct NormBwdLaunch {
    NormBwdArgs a;
    cudaStream_t st;
    template <typename T>
    int run() {
        constexpr int VV = 16 / sizeof(T);
        const bool vec = a.l % VV == 0 && aligned16(a.x) && aligned16(a.dy) && aligned16(a.dx);
        const int64_t segs = a.groups == 0 ? a.n * a.c : a.n * a.batch * a.groups;
        if (segs > 0x7fffffff) return set_error(WIDEK_ERR_UNSUPPORTED, "norm backward: too many segments");
        if (vec)
            norm_bwd_kernel<T, true><<<(unsigned)segs, kNbThreads, 0, st>>>(a);
        else
            norm_bwd_kernel<T, false><<<(unsigned)segs, kNbThreads, 0, st>>>(a);
        int rc = check_launch(a.groups == 0 ? "batchnorm_bwd" : "groupnorm_bwd");
        if (rc != WIDEK_OK || a.groups == 0 || (!a.dw && !a.db)) return rc;
        gn_param_reduce_kernel<T><<<(unsigned)((a.n * a.c + kSumThreads - 1) / kSumThreads), kSumThreads, 0, st>>>(
            a.part, static_cast<T*>(a.dw), static_cast<T*>(a.db), a.n, a.batch, a.c);
        return check_launch("groupnorm_bwd (parameter sums)");
    }
};

}  // namespace
}  // namespace widek

// ---------------------------------------------------------------------------
// C-ABI
// ---------------------------------------------------------------------------
namespace widek {
namespace {

struct LinBwdLayout {
    size_t wt, dyt, xt, part, total;    // byte offsets into the workspace
    int nblk;                           // column-sum partials per model
};

LinBwdLayout lin_bwd_layout(int64_t n, int64_t m, int64_t k, int64_t o, size_t es) {
    LinBwdLayout L{};
    L.nblk = (int)((m + widek::kSumRows - 1) / widek::kSumRows);
    if (L.nblk < 1) L.nblk = 1;
    size_t off = 0;
    L.wt = off;   off += widek::align256((size_t)n * k * o * es);
    L.dyt = off;  off += widek::align256((size_t)n * o * m * es);
    L.xt = off;   off += widek::align256((size_t)n * k * m * es);
    L.part = off; off += widek::align256((size_t)n * L.nblk * o * sizeof(float));
    L.total = off;
    return L;
}

struct ColsumLaunch {
    const void* x;
    void* out;
    float* part;
    int64_t n, m, c;
    int nblk;
    cudaStream_t st;
    template <typename T>
    int run() {
        using namespace widek;
        const unsigned cx = (unsigned)((c + kSumThreads - 1) / kSumThreads);
        const bool pair = sizeof(T) == 2 && c % 2 == 0 && (reinterpret_cast<uintptr_t>(x) & 3u) == 0;
        if (pair)
            colsum_part_kernel<T, true><<<dim3((cx + 1) / 2, (unsigned)nblk, (unsigned)n), kSumThreads, 0, st>>>(
                static_cast<const T*>(x), part, m, c, nblk);
        else
            colsum_part_kernel<T, false><<<dim3(cx, (unsigned)nblk, (unsigned)n), kSumThreads, 0, st>>>(
                static_cast<const T*>(x), part, m, c, nblk);
        int rc = check_launch("linear_bwd (bias partial sums)");
        if (rc != WIDEK_OK) return rc;
        colsum_final_kernel<T><<<dim3(cx, (unsigned)n), kSumThreads, 0, st>>>(part, static_cast<T*>(out), c, nblk);
        return check_launch("linear_bwd (bias sums)");
    }
};

struct ActBwdLaunch {
    const void *dy, *s;
    void* out;
    int64_t count;
    int act;
    cudaStream_t st;
    template <typename T>
    int run() {
        using namespace widek;
        constexpr int V = 16 / sizeof(T);
        const bool vec = count % V == 0 && aligned16(dy) && aligned16(s) && aligned16(out);
        const int64_t work = vec ? count / V : count;
        int64_t blocks = (work + 255) / 256;
        const int64_t cap = (int64_t)sm_count(current_device()) * 8;
        if (blocks > cap) blocks = cap;
        if (blocks < 1) blocks = 1;
        act_bwd_kernel<T><<<(unsigned)blocks, 256, 0, st>>>(static_cast<const T*>(dy), static_cast<const T*>(s),
                                                             static_cast<T*>(out), count, act, vec);
        return check_launch("act_bwd");
    }
};

}  // namespace
}  // namespace widek

extern "C" {

int widek_transpose(const void* x, void* y, int64_t batch, int64_t rows, int64_t cols, int dtype, void* stream) {
    using namespace widek;
    if (batch < 0 || rows < 0 || cols < 0) return set_error(WIDEK_ERR_INVALID, "transpose: negative size");
    const size_t es = dtype_size(dtype);
    if (es == 0) return set_error(WIDEK_ERR_INVALID, "transpose: unknown dtype code %d", dtype);
    if ((!x || !y) && batch * rows * cols > 0) return set_error(WIDEK_ERR_INVALID, "transpose: null pointer");
    return launch_transpose(x, y, batch, rows, cols, es, (cudaStream_t)stream);
}

int64_t widek_linear_bwd_workspace(int64_t n, int64_t m, int64_t k, int64_t o, int dtype) {
    using namespace widek;
    const size_t es = dtype_size(dtype);
    if (es == 0 || n < 0 || m < 0 || k < 0 || o < 0) return -1;
    return (int64_t)lin_bwd_layout(n, m, k, o, es).total;
}

int widek_linear_bwd(const void* x, const void* w, const void* dy, void* dx, void* dw, void* db, int64_t n, int64_t m,
                     int64_t k, int64_t o, int dtype, void* workspace, int64_t workspace_bytes, void* stream) {
    using namespace widek;
    cudaStream_t st = (cudaStream_t)stream;
    const size_t es = dtype_size(dtype);
    if (es == 0) return set_error(WIDEK_ERR_INVALID, "linear_bwd: unknown dtype code %d", dtype);
    if (n < 0 || m < 0 || k < 0 || o < 0) return set_error(WIDEK_ERR_INVALID, "linear_bwd: negative size");
    if (n > 65535) return set_error(WIDEK_ERR_UNSUPPORTED, "linear_bwd: more than 65535 models");
    const LinBwdLayout L = lin_bwd_layout(n, m, k, o, es);
    if (workspace_bytes < (int64_t)L.total || (!workspace && L.total > 0))
        return set_error(WIDEK_ERR_INVALID, "linear_bwd: workspace of %lld bytes, %lld needed",
                         (long long)workspace_bytes, (long long)L.total);
    if (n == 0) return WIDEK_OK;
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    int rc = WIDEK_OK;
    if (m == 0) {
        // no rows: the weight and bias gradients are zero, dX is empty
        if (dw && cudaMemsetAsync(dw, 0, (size_t)n * o * k * es, st) != cudaSuccess)
            return set_error(WIDEK_ERR_CUDA, "linear_bwd: memset failed");
        if (db && cudaMemsetAsync(db, 0, (size_t)n * o * es, st) != cudaSuccess)
            return set_error(WIDEK_ERR_CUDA, "linear_bwd: memset failed");
        return WIDEK_OK;
    }
    if (!dy || (dx && !w) || (dw && !x)) return set_error(WIDEK_ERR_INVALID, "linear_bwd: null pointer");
    if (dx) {
        // dX [n, m, k] = dY [n, m, o] . W [n, o, k]: W read MN-major by the
        // tcgen05 GEMM where it can, else dY . (W^T [n, k, o])^T on the
        // forward's GEMM
        rc = gemm_tc_mn(dy, w, dx, n, m, o, k, false, true, dtype, st);
        if (rc == WIDEK_ERR_UNSUPPORTED) {
            if ((rc = launch_transpose(w, ws + L.wt, n, o, k, es, st)) != WIDEK_OK) return rc;
            rc = widek_linear_fwd(dy, ws + L.wt, nullptr, dx, n, m, o, k, dtype, WIDEK_ACT_NONE, stream);
        }
        if (rc != WIDEK_OK) return rc;
    }
    if (dw) {
        // dW [n, o, k] = dY^T . x with both read MN-major where the tcgen05
        // GEMM can, else dY^T [n, o, m] . (x^T [n, k, m])^T
        rc = gemm_tc_mn(dy, x, dw, n, o, m, k, true, true, dtype, st);
        if (rc == WIDEK_ERR_UNSUPPORTED) {
            if ((rc = launch_transpose(dy, ws + L.dyt, n, m, o, es, st)) != WIDEK_OK) return rc;
            if ((rc = launch_transpose(x, ws + L.xt, n, m, k, es, st)) != WIDEK_OK) return rc;
            rc = widek_linear_fwd(ws + L.dyt, ws + L.xt, nullptr, dw, n, o, m, k, dtype, WIDEK_ACT_NONE, stream);
        }
        if (rc != WIDEK_OK) return rc;
    }
    if (db) {
        ColsumLaunch C{dy, db, reinterpret_cast<float*>(ws + L.part), n, m, o, L.nblk, st};
        if ((rc = dispatch_dtype(dtype, C)) != WIDEK_OK) return rc;
    }
    return WIDEK_OK;
}

int widek_act_bwd(const void* dy, const void* saved, void* dpre, int64_t count, int act, int dtype, void* stream) {
    using namespace widek;
    if (count < 0) return set_error(WIDEK_ERR_INVALID, "act_bwd: negative count");
    if (act != WIDEK_ACT_RELU && act != WIDEK_ACT_GELU)
        return set_error(WIDEK_ERR_INVALID, "act_bwd: activation %d has no gradient kernel", act);
    if (count == 0) return WIDEK_OK;
    if (!dy || !saved || !dpre) return set_error(WIDEK_ERR_INVALID, "act_bwd: null pointer");
    ActBwdLaunch L{dy, saved, dpre, count, act, (cudaStream_t)stream};
    return dispatch_dtype(dtype, L);
}

int64_t widek_layernorm_bwd_workspace(int64_t n, int64_t outer, int64_t d) {
    using namespace widek;
    if (n < 0 || outer < 0 || d < 0) return -1;
    return (int64_t)align256((size_t)n * ln_blocks(n, outer) * 2 * d * sizeof(float));
}

int widek_layernorm_bwd(const void* x, const void* w, const void* dy, void* dx, void* dw, void* db, int64_t n,
                        int64_t outer, int64_t d, double eps, int dtype, void* workspace, int64_t workspace_bytes,
                        void* stream) {
    using namespace widek;
    if (n < 0 || outer < 0 || d < 0) return set_error(WIDEK_ERR_INVALID, "layernorm_bwd: negative size");
    if (d > kLnMaxD) return set_error(WIDEK_ERR_UNSUPPORTED, "layernorm_bwd: d = %lld above %d", (long long)d, kLnMaxD);
    if (n > 65535) return set_error(WIDEK_ERR_UNSUPPORTED, "layernorm_bwd: more than 65535 models");
    const int64_t need = widek_layernorm_bwd_workspace(n, outer, d);
    if (workspace_bytes < need || (!workspace && need > 0))
        return set_error(WIDEK_ERR_INVALID, "layernorm_bwd: workspace of %lld bytes, %lld needed",
                         (long long)workspace_bytes, (long long)need);
    if (n == 0 || d == 0) return WIDEK_OK;
    if (!x || !w || !dy || !dx) return set_error(WIDEK_ERR_INVALID, "layernorm_bwd: null pointer");
    if (outer == 0) {
        cudaStream_t st = (cudaStream_t)stream;
        const size_t bytes = (size_t)n * d * dtype_size(dtype);
        if ((dw && cudaMemsetAsync(dw, 0, bytes, st) != cudaSuccess) ||
            (db && cudaMemsetAsync(db, 0, bytes, st) != cudaSuccess))
            return set_error(WIDEK_ERR_CUDA, "layernorm_bwd: memset failed");
        return WIDEK_OK;
    }
    LnBwdLaunch L{x, w, dy, dx, dw, db, static_cast<float*>(workspace), n, outer, (int)d, (float)eps, ln_blocks(n, outer),
                  (cudaStream_t)stream};
    return dispatch_dtype(dtype, L);
}

int widek_batchnorm_bwd(const void* x, const void* dy, const void* weight, const void* running_mean,
                        const void* running_var, void* dx, void* dw, void* db, int64_t n, int64_t batch, int64_t c,
                        int64_t l, int batch_stats, double eps, int dtype, void* stream) {
    using namespace widek;
    if (n < 0 || batch < 0 || c < 0 || l < 0) return set_error(WIDEK_ERR_INVALID, "batchnorm_bwd: negative size");
    if (n * c == 0) return WIDEK_OK;
    if (batch * l == 0) return set_error(WIDEK_ERR_INVALID, "batchnorm_bwd: a channel has no elements");
    if (!x || !dy || !dx) return set_error(WIDEK_ERR_INVALID, "batchnorm_bwd: null pointer");
    if (!batch_stats && (!running_mean || !running_var))
        return set_error(WIDEK_ERR_INVALID, "batchnorm_bwd: running statistics needed without batch statistics");
    NormBwdLaunch L{NormBwdArgs{x, dy, weight, running_mean, running_var, dx, dw, db, nullptr, n, batch, c, l, 0,
                                batch_stats ? 1 : 0, (float)eps},
                    (cudaStream_t)stream};
    return dispatch_dtype(dtype, L);
}

int64_t widek_groupnorm_bwd_workspace(int64_t n, int64_t batch, int64_t c) {
    if (n < 0 || batch < 0 || c < 0) return -1;
    return (int64_t)widek::align256((size_t)n * batch * c * 2 * sizeof(float));
}

int widek_groupnorm_bwd(const void* x, const void* dy, const void* weight, void* dx, void* dw, void* db, int64_t n,
                        int64_t batch, int64_t c, int64_t l, int64_t groups, double eps, int dtype, void* workspace,
                        int64_t workspace_bytes, void* stream) {
    using namespace widek;
    if (n < 0 || batch < 0 || c < 0 || l < 0 || groups <= 0)
        return set_error(WIDEK_ERR_INVALID, "groupnorm_bwd: bad sizes");
    if (c % groups != 0) return set_error(WIDEK_ERR_INVALID, "groupnorm_bwd: %lld channels in %lld groups",
                                          (long long)c, (long long)groups);
    const int64_t need = widek_groupnorm_bwd_workspace(n, batch, c);
    if (workspace_bytes < need || (!workspace && need > 0))
        return set_error(WIDEK_ERR_INVALID, "groupnorm_bwd: workspace of %lld bytes, %lld needed",
                         (long long)workspace_bytes, (long long)need);
    if (n * batch * c == 0) {
        const size_t bytes = (size_t)n * c * dtype_size(dtype);
        cudaStream_t st = (cudaStream_t)stream;
        if (bytes && ((dw && cudaMemsetAsync(dw, 0, bytes, st) != cudaSuccess) ||
                      (db && cudaMemsetAsync(db, 0, bytes, st) != cudaSuccess)))
            return set_error(WIDEK_ERR_CUDA, "groupnorm_bwd: memset failed");
        return WIDEK_OK;
    }
    if (l == 0) return set_error(WIDEK_ERR_INVALID, "groupnorm_bwd: empty spatial extent");
    if (!x || !dy || !dx) return set_error(WIDEK_ERR_INVALID, "groupnorm_bwd: null pointer");
    if (groups > 0x7fffffff) return set_error(WIDEK_ERR_UNSUPPORTED, "groupnorm_bwd: too many groups");
    NormBwdLaunch L{NormBwdArgs{x, dy, weight, nullptr, nullptr, dx, dw, db, static_cast<float*>(workspace), n, batch,
                                c, l, (int)groups, 1, (float)eps},
                    (cudaStream_t)stream};
    return dispatch_dtype(dtype, L);
}

}  // extern "C"
