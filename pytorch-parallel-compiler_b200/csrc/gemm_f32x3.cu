// fp32 grouped GEMM on the tensor cores by operand splitting:
//
//   y[i] = x[i] @ W_i^T + bias[i]   (fp32 in, fp32 out)
//
// Each fp32 operand a is split into three bf16 pieces, a0 = bf16(a),
// a1 = bf16(a - a0), a2 = bf16(a - a0 - a1), so that a = a0 + a1 + a2 to
// about 2^-27 relative. The product is accumulated in fp32 TMEM from the six
// piece products whose order is at most 2^-18 relative,
//   x0*w0 + x0*w1 + x1*w0 + x0*w2 + x1*w1 + x2*w0
// (six tcgen05 kind::f16 MMAs per K step; the dropped terms are below
// 2^-26), so each product is as accurate as an fp32 multiply and the sums
// differ from an fp32 FFMA GEMM by accumulation order only: the fp32
// contract (rtol 1e-3 / atol 1e-4 with TF32 off) holds however long K is.
// (Two pieces and three products leave ~2^-17 per product, which over a
// few hundred unscaled terms, e.g. a weight gradient summed over the batch,
// already reaches the 1e-4 absolute bound.) Serves fp32 WideLinear and the
// recurrent layers' input projection (all T steps of x at once), whose rows
// and weights come strided exactly as for linear_simt_strided.
//
// The tensor core's fp32 accumulation does not round to nearest: adding
// into one TMEM accumulator over all of K left errors that grow with K
// (1.1e-3 at K = 2048 with unscaled operands, against ~1e-4 for FFMA). So
// each 64-wide K chunk accumulates afresh, x0*w0 and the five small
// products into two separate TMEM accumulators, and the threads add both
// into fp32 registers (round to nearest) after the chunk: the truncation
// then acts on chunk-sized partial sums only.
//
// One CTA of 128 threads per (model, 128-row tile, 128-column tile), two
// stages: the threads load the x and W tiles of chunk c with coalesced
// 16-byte loads, split them and write the six bf16 tiles into the stage's
// shared memory in the 128-byte swizzled K-major layout (rows of 64
// values); one thread issues chunk c's MMAs into the stage's two 128-column
// TMEM accumulators; while they run, every thread drains chunk c-1's
// accumulators (its row: TMEM lane) into its registers. Epilogue: each
// thread writes its row with the bias added.
#include "common.cuh"
#include "sm100_ptx.cuh"

namespace widek {
namespace {

using namespace sm100;

constexpr int kF3Rows = 128;     // M and N of one tile
constexpr int kF3K = 64;         // K per chunk (one 128-byte swizzled bf16 row)
constexpr int kF3Threads = 128;
constexpr int kF3Batch = 8;      // 16-byte loads of x and of W in flight per thread
constexpr uint32_t kF3Tile = kF3Rows * kF3K * 2;     // one bf16 tile: 16 KB
constexpr uint32_t kF3Stage = 6 * kF3Tile;             // three pieces of x and of W
constexpr uint32_t kF3TmemCols = 4 * kF3Rows;          // per stage: x0*w0, and the small products

struct F3Args {
    const float* x;
    const float* w;
    const float* bias;       // [n, o] or null
    float* y;
    int m, k, o;
    int64_t w_ms, w_rs;      // weight model / row strides
    int64_t x_ms, x_bs;      // x: row r of model i at i*x_ms + (r / rpb)*x_bs + (r % rpb)*k
    int64_t y_ms, y_bs;      // y likewise with o
    int rpb;
};

// Byte offset of element (r, kk) (kk < 64) in a 128-byte swizzled K-major
// bf16 tile: row r at r*128, 16-byte chunk (kk / 8) at position chunk ^ (r % 8).
__device__ __forceinline__ uint32_t f3_off(int r, int kk) {
    return (uint32_t)(r * 128 + ((((kk >> 3) ^ (r & 7)) << 4) | ((kk & 7) << 1)));
}

// Splits four consecutive fp32 values into three bf16 pieces each and
// stores them at (r, kk..kk+3) of the piece tiles t0, t1, t2.
__device__ __forceinline__ void f3_split_store(uint8_t* t0, uint8_t* t1, uint8_t* t2, int r, int kk, float4 v) {
    const float a[4] = {v.x, v.y, v.z, v.w};
    uint32_t p0[2], p1[2], p2[2];
#pragma unroll
    for (int p = 0; p < 2; ++p) {
        const __nv_bfloat162 h = __floats2bfloat162_rn(a[2 * p], a[2 * p + 1]);
        const float2 hf = __bfloat1622float2(h);
        const float r0 = a[2 * p] - hf.x, r1 = a[2 * p + 1] - hf.y;          // exact in fp32
        const __nv_bfloat162 m = __floats2bfloat162_rn(r0, r1);
        const float2 mf = __bfloat1622float2(m);
        const __nv_bfloat162 l = __floats2bfloat162_rn(r0 - mf.x, r1 - mf.y);
        p0[p] = *reinterpret_cast<const uint32_t*>(&h);
        p1[p] = *reinterpret_cast<const uint32_t*>(&m);
        p2[p] = *reinterpret_cast<const uint32_t*>(&l);
    }
    const uint32_t off = f3_off(r, kk);      // 4 values = 8 bytes, inside one 16-byte chunk
    *reinterpret_cast<uint2*>(t0 + off) = make_uint2(p0[0], p0[1]);
    *reinterpret_cast<uint2*>(t1 + off) = make_uint2(p1[0], p1[1]);
    *reinterpret_cast<uint2*>(t2 + off) = make_uint2(p2[0], p2[1]);
}

// MULTI: K spans more than one chunk (register accumulation over chunks);
// otherwise the single chunk's accumulators are written out directly, and
// the kernel keeps few registers (room on the SM for a programmatic
// dependent's CTAs).
template <bool MULTI>
__global__ void __launch_bounds__(kF3Threads, 1) gemm_f32x3_kernel(F3Args a, int* err) {
    extern __shared__ uint8_t f3_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(f3_raw) + 1023) & ~uintptr_t(1023));
    // barriers in the first 1 KB, then one or two stages of six tiles (x
    // pieces 0..2, then W pieces 0..2); a single-chunk call gets one stage,
    // which leaves room on the SM for a programmatic dependent's CTAs
    uint64_t* done = reinterpret_cast<uint64_t*>(sm);      // [2], one per stage
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 2);
    uint8_t* tiles = sm + 1024;

    // A programmatic dependent (the recurrence after the RNN input
    // projection) may start its set-up now; it waits for this grid's results.
    grid_dep_launch_dependents();
    const int model = blockIdx.z;
    const int m0 = blockIdx.y * kF3Rows;
    const int o0 = blockIdx.x * kF3Rows;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const float* xm = a.x + (int64_t)model * a.x_ms;
    const float* wm = a.w + (int64_t)model * a.w_ms;

    if (tid == 0) {
        mbar_init(&done[0], 1);
        mbar_init(&done[1], 1);
        mbar_init_fence();
    }
    if (warp == 0) { tmem_alloc(tmem_slot, kF3TmemCols); tmem_relinquish(); }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    constexpr uint32_t IDESC = idesc_f16(kF3Rows, kF3Rows, true);
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;

    // Row r = warp*32 + lane of the tile, all 128 columns, summed in fp32
    // registers (round to nearest) over the K chunks.
    float acc[MULTI ? kF3Rows : 1];
#pragma unroll
    for (int j = 0; j < (MULTI ? kF3Rows : 1); ++j) acc[j] = 0.f;
    // Adds the accumulators of one stage (x0*w0 and the sum of the small
    // piece products, 128 columns each) to acc.
    auto drain = [&](int stage) {
        if constexpr (MULTI) {
            const uint32_t big = tmem + (uint32_t)(stage * 2 * kF3Rows) + lane_base;
            const uint32_t small = big + kF3Rows;
#pragma unroll
            for (int c = 0; c < kF3Rows; c += 32) {
                uint32_t vb[32], vs[32];
                tmem_ld_32x32b_x32(big + (uint32_t)c, vb);
                tmem_ld_32x32b_x32(small + (uint32_t)c, vs);
                tmem_ld_wait();
#pragma unroll
                for (int j = 0; j < 32; ++j) acc[c + j] += __uint_as_float(vb[j]) + __uint_as_float(vs[j]);
            }
        }
    };

    bool ok = true;
    int last_issued = 0;
    const volatile int no_abort = 0;
    const int chunks = (a.k + kF3K - 1) / kF3K;
    for (int ch = 0; ch < chunks && ok; ++ch) {
        const int st = ch & 1;
        uint8_t* x0 = tiles + st * kF3Stage;
        uint8_t* x1 = x0 + kF3Tile;
        uint8_t* x2 = x0 + 2 * kF3Tile;
        uint8_t* w0 = x0 + 3 * kF3Tile;
        uint8_t* w1 = x0 + 4 * kF3Tile;
        uint8_t* w2 = x0 + 5 * kF3Tile;
        const int k0 = ch * kF3K;
        // x and W tiles: 128 rows x 16 float4 each, consecutive threads on
        // consecutive 16-byte pieces of a row; rows / columns past the
        // matrix and k past K are zeros. Loads are issued in batches of
        // kF3Batch per tile before any is split and stored, so their
        // latencies overlap. The stage's previous MMAs (chunk ch - 2) were
        // waited for before chunk ch - 1's were issued.
        constexpr int kPer = kF3Rows * (kF3K / 4) / kF3Threads;     // float4 per thread per tile
#pragma unroll 1
        for (int j0 = 0; j0 < kPer; j0 += kF3Batch) {
            float4 xv[kF3Batch], wv[kF3Batch];
#pragma unroll
            for (int jj = 0; jj < kF3Batch; ++jj) {
                const int i = tid + (j0 + jj) * kF3Threads;
                const int r = i >> 4, kk = (i & 15) * 4;
                const int gk = k0 + kk;
                const int gm = m0 + r, go = o0 + r;
                xv[jj] = make_float4(0.f, 0.f, 0.f, 0.f);
                wv[jj] = xv[jj];
                if (gm < a.m && gk < a.k) {
                    const float* xr = xm + (int64_t)(gm / a.rpb) * a.x_bs + (int64_t)(gm % a.rpb) * a.k;
                    xv[jj] = __ldg(reinterpret_cast<const float4*>(xr + gk));
                }
                if (go < a.o && gk < a.k) wv[jj] = __ldg(reinterpret_cast<const float4*>(wm + (int64_t)go * a.w_rs + gk));
            }
#pragma unroll
            for (int jj = 0; jj < kF3Batch; ++jj) {
                const int i = tid + (j0 + jj) * kF3Threads;
                const int r = i >> 4, kk = (i & 15) * 4;
                f3_split_store(x0, x1, x2, r, kk, xv[jj]);
                f3_split_store(w0, w1, w2, r, kk, wv[jj]);
            }
        }
        // The tiles written by the threads become visible to the tensor
        // core; the stage's accumulators were drained (chunk ch - 2).
        fence_async_shared();
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
        if (tid == 0) {
            const uint32_t t_big = tmem + (uint32_t)(st * 2 * kF3Rows), t_small = t_big + kF3Rows;
            const uint64_t dx0 = sdesc_kmajor_sw128(smem_addr(x0)), dx1 = sdesc_kmajor_sw128(smem_addr(x1)),
                           dx2 = sdesc_kmajor_sw128(smem_addr(x2));
            const uint64_t dw0 = sdesc_kmajor_sw128(smem_addr(w0)), dw1 = sdesc_kmajor_sw128(smem_addr(w1)),
                           dw2 = sdesc_kmajor_sw128(smem_addr(w2));
#pragma unroll
            for (int k = 0; k < kF3K / 16; ++k) {
                umma_f16_ss(t_big, dx0 + 2 * k, dw0 + 2 * k, IDESC, k != 0);
                umma_f16_ss(t_small, dx0 + 2 * k, dw1 + 2 * k, IDESC, k != 0);
                umma_f16_ss(t_small, dx1 + 2 * k, dw0 + 2 * k, IDESC, 1);
                umma_f16_ss(t_small, dx0 + 2 * k, dw2 + 2 * k, IDESC, 1);
                umma_f16_ss(t_small, dx1 + 2 * k, dw1 + 2 * k, IDESC, 1);
                umma_f16_ss(t_small, dx2 + 2 * k, dw0 + 2 * k, IDESC, 1);
            }
            umma_commit(&done[st]);
        }
        last_issued = ch;
        // While chunk ch's MMAs run, drain chunk ch - 1's accumulators (its
        // MMAs are done once its barrier completes; every thread waits,
        // bounded, and the verdict is made uniform).
        if (ch > 0) {
            const int ps = st ^ 1;
            const bool got = mbar_wait(&done[ps], (uint32_t)(((ch - 1) >> 1) & 1), &no_abort);
            tc_fence_after();
            if (!__syncthreads_and(got)) { ok = false; break; }
            drain(ps);
            tc_fence_before();
        }
    }
    if (ok) {
        const int last = chunks - 1;
        const bool got = mbar_wait(&done[last & 1], (uint32_t)((last >> 1) & 1), &no_abort);
        tc_fence_after();
        ok = __syncthreads_and(got);
        if (ok && MULTI) drain(last & 1);
    }
    if (!ok) {
        // a wait ran out: report, and give the MMAs still in flight (the
        // last chunk issued) a bounded wait before the accumulators are freed
        raise_device_error(err, DEV_ERR_GEMM_TIMEOUT);
        mbar_wait(&done[last_issued & 1], (uint32_t)((last_issued >> 1) & 1), &no_abort);
    } else {
        // Epilogue: thread (warp, lane) holds row warp*32 + lane.
        const int r = warp * 32 + lane;
        const int gm = m0 + r;
        const float* bm = a.bias ? a.bias + (int64_t)model * a.o : nullptr;
        if (!MULTI) {
            // one chunk: big + small straight from TMEM (stage 0), 16 columns at a time
            float* yr = a.y + (int64_t)model * a.y_ms + (int64_t)((gm < a.m ? gm : 0) / a.rpb) * a.y_bs +
                        (int64_t)((gm < a.m ? gm : 0) % a.rpb) * a.o;
#pragma unroll 1
            for (int c = 0; c < kF3Rows; c += 16) {
                uint32_t vb[16], vs[16];
                tmem_ld_32x32b_x16(tmem + lane_base + (uint32_t)c, vb);
                tmem_ld_32x32b_x16(tmem + lane_base + kF3Rows + (uint32_t)c, vs);
                tmem_ld_wait();
                if (gm >= a.m) continue;
                const int go0 = o0 + c;
                if (go0 + 16 <= a.o && (a.o & 3) == 0) {
#pragma unroll
                    for (int j = 0; j < 16; j += 4) {
                        float4 f = make_float4(__uint_as_float(vb[j]) + __uint_as_float(vs[j]),
                                               __uint_as_float(vb[j + 1]) + __uint_as_float(vs[j + 1]),
                                               __uint_as_float(vb[j + 2]) + __uint_as_float(vs[j + 2]),
                                               __uint_as_float(vb[j + 3]) + __uint_as_float(vs[j + 3]));
                        if (bm) {
                            const float4 b = *reinterpret_cast<const float4*>(bm + go0 + j);
                            f.x += b.x; f.y += b.y; f.z += b.z; f.w += b.w;
                        }
                        *reinterpret_cast<float4*>(yr + go0 + j) = f;
                    }
                } else {
                    for (int j = 0; j < 16; ++j)
                        if (go0 + j < a.o)
                            yr[go0 + j] = __uint_as_float(vb[j]) + __uint_as_float(vs[j]) + (bm ? bm[go0 + j] : 0.f);
                }
            }
        } else if (gm < a.m) {
            float* yr = a.y + (int64_t)model * a.y_ms + (int64_t)(gm / a.rpb) * a.y_bs + (int64_t)(gm % a.rpb) * a.o;
            if (o0 + kF3Rows <= a.o && (a.o & 3) == 0) {
#pragma unroll
                for (int j = 0; j < (MULTI ? kF3Rows : 0); j += 4) {
                    float4 f = make_float4(acc[j], acc[j + 1], acc[j + 2], acc[j + 3]);
                    if (bm) {
                        const float4 b = *reinterpret_cast<const float4*>(bm + o0 + j);
                        f.x += b.x; f.y += b.y; f.z += b.z; f.w += b.w;
                    }
                    *reinterpret_cast<float4*>(yr + o0 + j) = f;
                }
            } else {
#pragma unroll
                for (int j = 0; j < (MULTI ? kF3Rows : 0); ++j)
                    if (o0 + j < a.o) yr[o0 + j] = acc[j] + (bm ? bm[o0 + j] : 0.f);
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, kF3TmemCols);
    }
}

}  // namespace

// True when the split tensor-core kernel serves the call (and it was
// launched); false when the caller should use the CUDA-core kernel.
int linear_f32x3_strided(const float* x, const float* w, const float* bias, float* y, int64_t n, int64_t m, int64_t k,
                         int64_t o, int64_t w_ms, int64_t w_rs, int64_t x_ms, int64_t x_bs, int64_t x_rpb,
                         int64_t y_ms, int64_t y_bs, cudaStream_t st) {
    if (n <= 0 || m <= 0 || o <= 0 || k <= 0) return WIDEK_ERR_UNSUPPORTED;
    if (n > 65535 || m > 0x7fffffff || o > 0x7fffffff || k > 0x7fffffff) return WIDEK_ERR_UNSUPPORTED;
    // 16-byte loads: rows of x and W start on 16-byte boundaries
    const bool vec = k % 4 == 0 && w_rs % 4 == 0 && w_ms % 4 == 0 && x_ms % 4 == 0 && x_bs % 4 == 0 &&
                     aligned16(x) && aligned16(w) && (!bias || aligned16(bias)) && aligned16(y) &&
                     y_ms % 4 == 0 && y_bs % 4 == 0;
    if (!vec) return WIDEK_ERR_UNSUPPORTED;
    const int64_t mt = (m + kF3Rows - 1) / kF3Rows, ot = (o + kF3Rows - 1) / kF3Rows;
    if (mt > 65535 || ot > 0x7fffffff) return WIDEK_ERR_UNSUPPORTED;
    F3Args a{x, w, bias, y, (int)m, (int)k, (int)o, w_ms, w_rs, x_ms, x_bs, y_ms, y_bs, (int)x_rpb};
    const size_t smem_max = 2048 + 2 * kF3Stage;
    const size_t smem = 2048 + (k > kF3K ? 2 : 1) * (size_t)kF3Stage;
    static bool attr_done[64] = {false};
    const int dev = current_device();
    if (dev >= 0 && dev < 64 && !attr_done[dev]) {
        if (cudaFuncSetAttribute(gemm_f32x3_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)smem_max) != cudaSuccess ||
            cudaFuncSetAttribute(gemm_f32x3_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)smem_max) != cudaSuccess)
            return set_error(WIDEK_ERR_CUDA, "linear (f32x3): cannot reserve %zu bytes of shared memory", smem_max);
        attr_done[dev] = true;
    }
    dim3 grid((unsigned)ot, (unsigned)mt, (unsigned)n);
    if (k > kF3K)
        gemm_f32x3_kernel<true><<<grid, kF3Threads, smem, st>>>(a, device_error_ptr());
    else
        gemm_f32x3_kernel<false><<<grid, kF3Threads, smem, st>>>(a, device_error_ptr());
    return check_launch("widek_linear_fwd (fp32 split tensor-core)");
}

}  // namespace widek
