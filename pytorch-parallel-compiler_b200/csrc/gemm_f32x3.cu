// fp32 grouped GEMM on the tensor cores by operand splitting:
//
//   y[i] = x[i] @ W_i^T + bias[i]   (fp32 in, fp32 out)
//
// Each fp32 operand a is split into two bf16 values, hi = bf16(a) and
// lo = bf16(a - hi), so that a = hi + lo to about 2^-17 relative. The
// product is accumulated in fp32 TMEM as hi_x*hi_w + hi_x*lo_w + lo_x*hi_w
// (three tcgen05 kind::f16 MMAs per K step; the dropped lo*lo term is about
// 2^-16 relative), which keeps each product within ~2^-16 of the fp32 one:
// well inside the fp32 contract (rtol 1e-3 / atol 1e-4 with TF32 off),
// while the CUDA-core kernel of gemm_simt.cu is bound by its shared-memory
// wavefronts. Serves the recurrent layers' input projection (all T steps of
// x at once), whose rows and weights come strided exactly as for
// linear_simt_strided.
//
// One CTA of 128 threads per (model, 128-row tile, 128-column tile): the
// threads load their x and W tiles with coalesced 16-byte loads, split them
// and write the four bf16 tiles into shared memory in the 128-byte swizzled
// K-major layout (rows of 64 values); one thread issues the MMAs into a
// 128-column TMEM accumulator; each warp then reads its 32 TMEM lanes (rows)
// and writes them with the bias added. K runs in chunks of 64.
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

// Splits four consecutive fp32 values into bf16 hi / lo parts and stores
// them at (r, kk..kk+3) of the hi and lo tiles.
__device__ __forceinline__ void f3_split_store(uint8_t* hi, uint8_t* lo, int r, int kk, float4 v) {
    const float a[4] = {v.x, v.y, v.z, v.w};
    uint32_t h2[2], l2[2];
#pragma unroll
    for (int p = 0; p < 2; ++p) {
        const __nv_bfloat162 h = __floats2bfloat162_rn(a[2 * p], a[2 * p + 1]);
        const float2 hf = __bfloat1622float2(h);
        const __nv_bfloat162 l = __floats2bfloat162_rn(a[2 * p] - hf.x, a[2 * p + 1] - hf.y);
        h2[p] = *reinterpret_cast<const uint32_t*>(&h);
        l2[p] = *reinterpret_cast<const uint32_t*>(&l);
    }
    const uint32_t off = f3_off(r, kk);      // 4 values = 8 bytes, inside one 16-byte chunk
    *reinterpret_cast<uint2*>(hi + off) = make_uint2(h2[0], h2[1]);
    *reinterpret_cast<uint2*>(lo + off) = make_uint2(l2[0], l2[1]);
}

__global__ void __launch_bounds__(kF3Threads, 1) gemm_f32x3_kernel(F3Args a, int* err) {
    extern __shared__ uint8_t f3_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(f3_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* xh = sm;
    uint8_t* xl = sm + kF3Tile;
    uint8_t* wh = sm + 2 * kF3Tile;
    uint8_t* wl = sm + 3 * kF3Tile;
    uint64_t* done = reinterpret_cast<uint64_t*>(sm + 4 * kF3Tile);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);

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
        mbar_init(done, 1);
        mbar_init_fence();
    }
    if (warp == 0) { tmem_alloc(tmem_slot, kF3Rows); tmem_relinquish(); }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    constexpr uint32_t IDESC = idesc_f16(kF3Rows, kF3Rows, true);

    bool ok = true;
    const int chunks = (a.k + kF3K - 1) / kF3K;
    for (int ch = 0; ch < chunks; ++ch) {
        const int k0 = ch * kF3K;
        // x and W tiles: 128 rows x 16 float4 each, consecutive threads on
        // consecutive 16-byte pieces of a row; rows / columns past the
        // matrix and k past K are zeros. Loads are issued in batches of
        // kF3Batch per tile before any is split and stored, so their
        // latencies overlap.
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
                f3_split_store(xh, xl, r, kk, xv[jj]);
                f3_split_store(wh, wl, r, kk, wv[jj]);
            }
        }
        // The tiles written by the threads become visible to the tensor core.
        fence_async_shared();
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
        if (tid == 0) {
            const uint64_t dxh = sdesc_kmajor_sw128(smem_addr(xh)), dxl = sdesc_kmajor_sw128(smem_addr(xl));
            const uint64_t dwh = sdesc_kmajor_sw128(smem_addr(wh)), dwl = sdesc_kmajor_sw128(smem_addr(wl));
#pragma unroll
            for (int k = 0; k < kF3K / 16; ++k) {
                umma_f16_ss(tmem, dxh + 2 * k, dwh + 2 * k, IDESC, (ch | k) != 0);
                umma_f16_ss(tmem, dxh + 2 * k, dwl + 2 * k, IDESC, 1);
                umma_f16_ss(tmem, dxl + 2 * k, dwh + 2 * k, IDESC, 1);
            }
            umma_commit(done);
        }
        // The MMAs have read the tiles (and, after the last chunk, written
        // the accumulator) before the tiles are overwritten / TMEM is read.
        // Every thread waits (bounded); the verdict is made uniform so that
        // no thread leaves the loop while others reach the next barrier.
        const volatile int no_abort = 0;
        const bool got = mbar_wait(done, (uint32_t)(ch & 1), &no_abort);
        tc_fence_after();
        if (!__syncthreads_and(got)) { ok = false; break; }
    }
    if (!ok) {
        raise_device_error(err, DEV_ERR_GEMM_TIMEOUT);
    } else {
        // Epilogue: warp q reads TMEM lanes 32q..32q+31 (rows), 32 columns at a time.
        const int r = warp * 32 + lane;
        const int gm = m0 + r;
        float* yr = a.y + (int64_t)model * a.y_ms + (int64_t)((gm < a.m ? gm : 0) / a.rpb) * a.y_bs +
                    (int64_t)((gm < a.m ? gm : 0) % a.rpb) * a.o;
        const float* bm = a.bias ? a.bias + (int64_t)model * a.o : nullptr;
#pragma unroll 1
        for (int c = 0; c < kF3Rows; c += 32) {
            uint32_t v[32];
            tmem_ld_32x32b_x32(tmem + (uint32_t)c + ((uint32_t)(warp * 32) << 16), v);
            tmem_ld_wait();
            if (gm < a.m) {
                const int go0 = o0 + c;
                if (go0 + 32 <= a.o && (a.o & 3) == 0) {
#pragma unroll
                    for (int j = 0; j < 32; j += 4) {
                        float4 f = make_float4(__uint_as_float(v[j]), __uint_as_float(v[j + 1]),
                                               __uint_as_float(v[j + 2]), __uint_as_float(v[j + 3]));
                        if (bm) {
                            const float4 b = *reinterpret_cast<const float4*>(bm + go0 + j);
                            f.x += b.x; f.y += b.y; f.z += b.z; f.w += b.w;
                        }
                        *reinterpret_cast<float4*>(yr + go0 + j) = f;
                    }
                } else {
                    for (int j = 0; j < 32; ++j)
                        if (go0 + j < a.o) yr[go0 + j] = __uint_as_float(v[j]) + (bm ? bm[go0 + j] : 0.f);
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, kF3Rows);
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
    const size_t smem = 1024 + 4 * kF3Tile + 16;
    static bool attr_done[64] = {false};
    const int dev = current_device();
    if (dev >= 0 && dev < 64 && !attr_done[dev]) {
        if (cudaFuncSetAttribute(gemm_f32x3_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
            cudaSuccess)
            return set_error(WIDEK_ERR_CUDA, "linear (f32x3): cannot reserve %zu bytes of shared memory", smem);
        attr_done[dev] = true;
    }
    dim3 grid((unsigned)ot, (unsigned)mt, (unsigned)n);
    gemm_f32x3_kernel<<<grid, kF3Threads, smem, st>>>(a, device_error_ptr());
    return check_launch("widek_linear_fwd (fp32 split tensor-core)");
}

}  // namespace widek
