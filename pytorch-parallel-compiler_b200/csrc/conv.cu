// Wide convolutions (1-D / 2-D / 3-D, one independent conv per model) on the
// N-first layout x [n, batch, cin, *spatial] -> y [n, batch, cout, *spatial'].
//
// Tensor-core path (bf16/f16, 2-D or 1-D, stride 1, cin % 64 == 0,
// cout % 16 == 0): implicit GEMM on tcgen05.
//   * the input is staged channels-last ([n*batch][h][w][cin], a caller
//     workspace) by one tiled transpose kernel, so that for a fixed filter tap
//     (kh, kw) the 64 input channels of an output pixel are one contiguous
//     128-byte row;
//   * the weights are pre-packed [n][cout][kh][kw][cin] (K-major with
//     k = (kh, kw, cin)) by widek_conv_pack_weight;
//   * a 128-pixel M tile is TH x TW output pixels (TW = row width rounded up
//     to a power of two, TH = 128 / TW). K-block (kh, kw, 64 channels) of A is
//     ONE TMA box {64, TW, TH, 1} of the channels-last input at coordinates
//     (c0, wo0 - pad + kw*dil, ho0 - pad + kh*dil, image): the innermost
//     coordinate stays 64-aligned, and out-of-range (padding) pixels are
//     zero-filled by the TMA unit;
//   * warp-specialised persistent kernel as the linear one (TMA warp, MMA
//     warp, 4 epilogue warps, double-buffered TMEM accumulator); the epilogue
//     writes NCHW directly (for a fixed output channel a warp stores 32
//     consecutive pixels) and can fuse bias, a per-channel scale/shift
//     (folded BatchNorm), an activation and a residual add.
// CUDA-core path (everything else, including fp32): direct convolution, one
// output element per thread, fp32 accumulation.
#include <cstring>

#include "sm100_ptx.cuh"

namespace widek {
namespace {

using namespace sm100;

// ---------------------------------------------------------------------------
// Layout helpers
// ---------------------------------------------------------------------------
// [nb][c][p] -> [nb][p][c], 32x32 tiles through shared memory (any c, p).
template <typename T>
__global__ void nchw_to_nhwc_kernel(const T* __restrict__ src, T* __restrict__ dst, int64_t nb, int c, int64_t p) {
    __shared__ T tile[32][33];
    const int tx = threadIdx.x, ty = threadIdx.y;   // 32 x 8
    const int64_t p0 = (int64_t)blockIdx.x * 32;
    const int c0 = blockIdx.y * 32;
    for (int64_t img = blockIdx.z; img < nb; img += gridDim.z) {
        const T* s = src + img * c * p;
        T* d = dst + img * c * p;
        for (int r = ty; r < 32; r += 8) {
            const int cc = c0 + r;
            const int64_t pp = p0 + tx;
            if (cc < c && pp < p) tile[r][tx] = s[(int64_t)cc * p + pp];
        }
        __syncthreads();
        for (int r = ty; r < 32; r += 8) {
            const int64_t pp = p0 + r;
            const int cc = c0 + tx;
            if (cc < c && pp < p) d[pp * c + cc] = tile[tx][r];
        }
        __syncthreads();
    }
}

// 16-bit [nb][c][p] -> [nb][p][c] for c % 64 == 0 and p % 64 == 0: 64x64
// tiles, 16-byte loads along p and 16-byte stores along c. `packed_b` > 0
// means the source is the channel-packed [b][n][c][p] layout (image
// img = n * packed_b + b), so the unpack of a TracedWideModel input is fused.
__global__ void __launch_bounds__(256) nchw_to_nhwc_vec_kernel(const uint16_t* __restrict__ src,
                                                               uint16_t* __restrict__ dst, int64_t nb, int c,
                                                               int64_t p, int64_t packed_b, int64_t packed_n) {
    __shared__ uint16_t tile[64][64 + 2];
    const int t = threadIdx.x;
    const int64_t tiles_p = p / 64, tiles_c = c / 64;
    const int64_t total = nb * tiles_c * tiles_p;
    for (int64_t job = blockIdx.x; job < total; job += gridDim.x) {
        const int64_t tp = job % tiles_p;
        const int64_t rest = job / tiles_p;
        const int64_t tc = rest % tiles_c;
        const int64_t img = rest / tiles_c;
        int64_t src_img = img;
        if (packed_b > 0) {
            const int64_t n_i = img / packed_b, b_i = img % packed_b;
            src_img = b_i * packed_n + n_i;
        }
        const uint16_t* s = src + (src_img * c + tc * 64) * p + tp * 64;
        uint16_t* d = dst + (img * p + tp * 64) * c + tc * 64;
        // load: 64 channel rows x 8 chunks of 8 pixels
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int chunk = t + 256 * i;
            const int row = chunk >> 3, col = (chunk & 7) * 8;
            const uint4 v = *reinterpret_cast<const uint4*>(s + (int64_t)row * p + col);
            const uint16_t* e = reinterpret_cast<const uint16_t*>(&v);
#pragma unroll
            for (int j = 0; j < 8; ++j) tile[row][col + j] = e[j];
        }
        __syncthreads();
        // store: 64 pixel rows x 8 chunks of 8 channels
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int chunk = t + 256 * i;
            const int pix = chunk >> 3, ch = (chunk & 7) * 8;
            uint4 v;
            uint16_t* e = reinterpret_cast<uint16_t*>(&v);
#pragma unroll
            for (int j = 0; j < 8; ++j) e[j] = tile[ch + j][pix];
            *reinterpret_cast<uint4*>(d + (int64_t)pix * c + ch) = v;
        }
        __syncthreads();
    }
}

// w [rows][cin][taps] -> wp [rows][taps][cin]
template <typename U>
__global__ void pack_weight_kernel(const U* __restrict__ w, U* __restrict__ wp, int64_t rows, int64_t cin,
                                   int64_t taps) {
    const int64_t total = rows * cin * taps;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
        const int64_t r = i / (cin * taps);
        const int64_t rem = i - r * cin * taps;
        const int64_t t = rem / cin;
        const int64_t ci = rem - t * cin;
        wp[i] = w[(r * cin + ci) * taps + t];
    }
}

unsigned grid_cap(int64_t items, int threads) {
    const int64_t want = (items + threads - 1) / threads;
    const int64_t cap = (int64_t)sm_count(current_device()) * 8;
    return (unsigned)std::max<int64_t>(1, std::min<int64_t>(want, cap));
}

struct ConvGeom {
    int n, batch, cin, cout;
    int d, h, w;          // input spatial (d = 1 for 2-D, h = d = 1 for 1-D)
    int kd, kh, kw;
    int sd, sh, sw;
    int pd, ph, pw;
    int dd, dh, dw;
    int od, oh, ow;       // output spatial
};

struct ConvEpi {
    const void* bias;     // [n*cout] or null
    const void* scale;    // [n*cout] or null (per-channel multiplier after bias)
    const void* shift;    // [n*cout] or null
    const void* residual; // same layout as y, or null
    int act;              // WIDEK_ACT_*
    int residual_first;   // 1: add the residual before the activation
};

template <typename T>
__device__ __forceinline__ float conv_epilogue(float v, int64_t ch, int64_t yoff, const ConvEpi& e) {
    if (e.bias) v += to_f<T>(static_cast<const T*>(e.bias)[ch]);
    if (e.scale) v *= to_f<T>(static_cast<const T*>(e.scale)[ch]);
    if (e.shift) v += to_f<T>(static_cast<const T*>(e.shift)[ch]);
    if (e.residual && e.residual_first) v += to_f<T>(static_cast<const T*>(e.residual)[yoff]);
    v = apply_act(v, e.act);
    if (e.residual && !e.residual_first) v += to_f<T>(static_cast<const T*>(e.residual)[yoff]);
    return v;
}

// ---------------------------------------------------------------------------
// CUDA-core direct convolution
// ---------------------------------------------------------------------------
template <typename T>
__global__ void conv_direct_kernel(const T* __restrict__ x, const T* __restrict__ w, T* __restrict__ y, ConvGeom g,
                                   ConvEpi e) {
    const int64_t osp = (int64_t)g.od * g.oh * g.ow;
    const int64_t total = (int64_t)g.n * g.batch * g.cout * osp;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t isp = (int64_t)g.d * g.h * g.w;
    const int taps = g.kd * g.kh * g.kw;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
        int64_t r = i;
        const int ox = (int)(r % g.ow); r /= g.ow;
        const int oy = (int)(r % g.oh); r /= g.oh;
        const int oz = (int)(r % g.od); r /= g.od;
        const int co = (int)(r % g.cout); r /= g.cout;
        const int64_t img = r;                       // n_i * batch + b
        const int64_t ni = img / g.batch;
        const T* xi = x + img * g.cin * isp;
        const T* wr = w + (ni * g.cout + co) * (int64_t)g.cin * taps;
        float acc = 0.f;
        for (int ci = 0; ci < g.cin; ++ci) {
            const T* xc = xi + (int64_t)ci * isp;
            const T* wc = wr + (int64_t)ci * taps;
            for (int a = 0; a < g.kd; ++a) {
                const int iz = oz * g.sd - g.pd + a * g.dd;
                if (iz < 0 || iz >= g.d) continue;
                for (int bb = 0; bb < g.kh; ++bb) {
                    const int iy = oy * g.sh - g.ph + bb * g.dh;
                    if (iy < 0 || iy >= g.h) continue;
                    for (int cc = 0; cc < g.kw; ++cc) {
                        const int ix = ox * g.sw - g.pw + cc * g.dw;
                        if (ix < 0 || ix >= g.w) continue;
                        acc = fmaf(to_f<T>(xc[((int64_t)iz * g.h + iy) * g.w + ix]),
                                   to_f<T>(wc[(a * g.kh + bb) * g.kw + cc]), acc);
                    }
                }
            }
        }
        y[i] = from_f<T>(conv_epilogue<T>(acc, ni * g.cout + co, i, e));
    }
}

// ---------------------------------------------------------------------------
// tcgen05 implicit GEMM (2-D / 1-D, stride 1)
// ---------------------------------------------------------------------------
constexpr int BM = 128;
constexpr int BK = 64;
constexpr int kThreads = 192;

template <int BN, int STAGES, bool RES_TMA = false>
struct ConvSmem {
    static constexpr uint32_t A_BYTES = BM * BK * 2;
    static constexpr uint32_t B_BYTES = BN * BK * 2;
    static constexpr uint32_t RING = STAGES * (A_BYTES + B_BYTES);
    static constexpr uint32_t STAGE_OUT = BM * BN * 2;   // output tile staged for the TMA store
    static constexpr uint32_t STAGE_RES = RES_TMA ? BM * BN * 2 : 0;   // residual tile (TMA load)
    static constexpr uint32_t BARS = 8 * (2 * STAGES + 6) + 16;
    static constexpr uint32_t TOTAL = 1024 + RING + STAGE_OUT + STAGE_RES + BARS;
};

__device__ __forceinline__ void tma_store_4d(const CUtensorMap* map, const void* src, int c0, int c1, int c2, int c3) {
    asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(smem_addr(src)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void epi_bar_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

struct ConvTcGeom {
    int n, batch, cout, ho, wo, th, tw, tiles_h, tiles_w, nt_count;
    int kh, kw, cblocks, ph, pw, dh, dw;
};

template <typename T, int BN, int STAGES, bool TMA_STORE, bool RES_TMA>
__global__ void __launch_bounds__(kThreads, 1)
    conv_tc_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
                   const __grid_constant__ CUtensorMap tm_y, const __grid_constant__ CUtensorMap tm_r,
                   T* __restrict__ y, ConvTcGeom g, ConvEpi e, int* err) {
    using S = ConvSmem<BN, STAGES, RES_TMA>;
    constexpr uint32_t IDESC = idesc_f16(BM, BN, std::is_same<T, __nv_bfloat16>::value);
    constexpr uint32_t TMEM_COLS = 2 * BN;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;
    uint8_t* sB = smem + STAGES * S::A_BYTES;
    T* sOut = reinterpret_cast<T*>(smem + S::RING);      // [BN][BM] output tile (TMA store source)
    T* sRes = reinterpret_cast<T*>(smem + S::RING + S::STAGE_OUT);   // [BN][BM] residual tile
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::RING + S::STAGE_OUT + S::STAGE_RES);
    uint64_t* empty = full + STAGES;
    uint64_t* tfull = empty + STAGES;
    uint64_t* tempty = tfull + 2;
    uint64_t* done = tempty + 2;
    uint64_t* res_bar = done + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(res_bar + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int mt_count = g.tiles_h * g.tiles_w;
    const int kb_count = g.kh * g.kw * g.cblocks;
    const int64_t tiles = (int64_t)g.n * g.nt_count * g.batch * mt_count;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
        for (int a = 0; a < 2; ++a) { mbar_init(&tfull[a], 1); mbar_init(&tempty[a], 4 * 32); }
        mbar_init(done, 1);
        mbar_init(res_bar, 1);
        *abort_flag = 0;
        mbar_init_fence();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tm_x);
        tma_prefetch_desc(&tm_w);
        if (TMA_STORE) tma_prefetch_desc(&tm_y);
        if (RES_TMA) tma_prefetch_desc(&tm_r);
    }
    if (warp == 1) { tmem_alloc(tmem_slot, TMEM_COLS); tmem_relinquish(); }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    // tile -> (model, n-tile, image-in-batch, m-tile); m-tile fastest.
    auto decode = [&](int64_t tile, int& model, int& nt, int& b, int& mt) {
        mt = (int)(tile % mt_count); tile /= mt_count;
        b = (int)(tile % g.batch); tile /= g.batch;
        nt = (int)(tile % g.nt_count);
        model = (int)(tile / g.nt_count);
    };

    if (warp == 0) {
        const uint64_t pol_x = l2_policy_evict_first();
        const uint64_t pol_w = l2_policy_evict_last();
        int s = 0, issued = 0;
        uint32_t ph = 0;
        bool ok = true;
        for (int64_t tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x) {
            int model, nt, b, mt;
            decode(tile, model, nt, b, mt);
            const int ho0 = (mt / g.tiles_w) * g.th;
            const int wo0 = (mt % g.tiles_w) * g.tw;
            const int img = model * g.batch + b;
            for (int kb = 0; kb < kb_count; ++kb) {
                const int cb = kb % g.cblocks;
                const int tap = kb / g.cblocks;
                const int ky = tap / g.kw, kx = tap % g.kw;
                if (!mbar_wait(&empty[s], ph ^ 1, abort_flag)) { ok = false; break; }
                if (lane == 0) {
                    mbar_arrive_expect_tx(&full[s], S::A_BYTES + S::B_BYTES);
                    tma_load_4d(sA + s * S::A_BYTES, &tm_x, &full[s], cb * BK, wo0 - g.pw + kx * g.dw,
                                ho0 - g.ph + ky * g.dh, img, pol_x);
                    tma_load_3d(sB + s * S::B_BYTES, &tm_w, &full[s], kb * BK, nt * BN, model, pol_w);
                }
                __syncwarp();
                ++issued;
                if (++s == STAGES) { s = 0; ph ^= 1; }
            }
        }
        if (!ok) {
            *abort_flag = 1;
            raise_device_error(err, DEV_ERR_CONV_TIMEOUT);
            const int inflight = issued < STAGES ? issued : STAGES;
            for (int j = 1; j <= inflight; ++j) {
                const int idx = issued - j;
                const volatile int never = 0;
                mbar_wait(&full[idx % STAGES], (uint32_t)((idx / STAGES) & 1), &never);
            }
        }
    } else if (warp == 1) {
        int s = 0, local = 0;
        uint32_t ph = 0;
        bool ok = true;
        for (int64_t tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x, ++local) {
            const int acc = local & 1;
            const uint32_t aph = (local >> 1) & 1;
            if (!mbar_wait(&tempty[acc], aph ^ 1, abort_flag)) { ok = false; break; }
            tc_fence_after();
            const uint32_t d_tmem = tmem_base + acc * BN;
            for (int kb = 0; kb < kb_count; ++kb) {
                if (!mbar_wait(&full[s], ph, abort_flag)) { ok = false; break; }
                tc_fence_after();
                if (lane == 0) {
                    const uint32_t a0 = smem_addr(sA + s * S::A_BYTES);
                    const uint32_t b0 = smem_addr(sB + s * S::B_BYTES);
#pragma unroll
                    for (int k = 0; k < BK / 16; ++k)
                        umma_f16_ss(d_tmem, sdesc_kmajor_sw128(a0 + k * 32), sdesc_kmajor_sw128(b0 + k * 32), IDESC,
                                    (kb | k) != 0);
                    umma_commit(&empty[s]);
                }
                __syncwarp();
                if (++s == STAGES) { s = 0; ph ^= 1; }
            }
            if (!ok) break;
            if (lane == 0) umma_commit(&tfull[acc]);
            __syncwarp();
        }
        if (!ok) {
            *abort_flag = 1;
            raise_device_error(err, DEV_ERR_CONV_TIMEOUT);
        }
        if (lane == 0) umma_commit(done);
        __syncwarp();
        const volatile int never = 0;
        mbar_wait(done, 0, &never);
    } else {
        // Epilogue: warps 2..5, TMEM lane quarter q = warp % 4 (pixels
        // q*32 .. q*32+31 of the tile). Per 32-channel chunk, lane j fetches
        // the per-channel parameters of channel co0 + j once; the values are
        // broadcast with shuffles.
        const int q = warp & 3;
        const int ep_tid = threadIdx.x - 64;            // 0..127
        const int64_t osp = (int64_t)g.ho * g.wo;
        const T* bias = static_cast<const T*>(e.bias);
        const T* scale = static_cast<const T*>(e.scale);
        const T* shift = static_cast<const T*>(e.shift);
        const T* res = static_cast<const T*>(e.residual);
        int local = 0;
        for (int64_t tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++local) {
            int model, nt, b, mt;
            decode(tile, model, nt, b, mt);
            const int acc = local & 1;
            const uint32_t aph = (local >> 1) & 1;
            const int r = q * 32 + lane;                 // pixel within the tile
            const int ho0 = (mt / g.tiles_w) * g.th, wo0 = (mt % g.tiles_w) * g.tw;
            const int ho = ho0 + r / g.tw;
            const int wo = wo0 + r % g.tw;
            const bool pix_ok = ho < g.ho && wo < g.wo;
            const int64_t img = (int64_t)model * g.batch + b;
            const int64_t pix = (int64_t)ho * g.wo + wo;
            if (TMA_STORE) {
                // The previous tile's store must have finished reading sOut and
                // every thread must be done with the previous sRes; then the
                // residual tile is requested so that it lands while this tile's
                // MMAs finish.
                if (ep_tid == 0) bulk_wait_read0();
                epi_bar_sync();
                if (RES_TMA && ep_tid == 0) {
                    mbar_arrive_expect_tx(res_bar, S::STAGE_RES);
                    tma_load_4d(sRes, &tm_r, res_bar, wo0, ho0, nt * BN, (int)img, l2_policy_evict_first());
                }
            }
            if (!mbar_wait(&tfull[acc], aph, abort_flag)) {
                *abort_flag = 1;
                raise_device_error(err, DEV_ERR_CONV_TIMEOUT);
                break;
            }
            tc_fence_after();
            if (RES_TMA && !mbar_wait(res_bar, (uint32_t)(local & 1), abort_flag)) {
                *abort_flag = 1;
                raise_device_error(err, DEV_ERR_CONV_TIMEOUT);
                break;
            }
#pragma unroll 1
            for (int c = 0; c < BN; c += 32) {
                const int co0 = nt * BN + c;
                if (co0 >= g.cout) break;    // warp-uniform
                uint32_t v[32];
                tmem_ld_32x32b_x32(tmem_base + (uint32_t)(acc * BN + c) + ((uint32_t)(q * 32) << 16), v);
                const int my_co = co0 + lane;
                const int64_t my_ch = (int64_t)model * g.cout + (my_co < g.cout ? my_co : 0);
                const float pb = bias ? to_f<T>(bias[my_ch]) : 0.f;
                const float ps = scale ? to_f<T>(scale[my_ch]) : 1.f;
                const float pt = shift ? to_f<T>(shift[my_ch]) : 0.f;
                tmem_ld_wait();
                const int64_t ybase = (img * g.cout + co0) * osp + pix;
                // residual values of this chunk: from the TMA-staged tile, or
                // 32 independent loads issued before any use
                float rv[32];
                if (res) {
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        if (RES_TMA) {
                            rv[j] = to_f<T>(sRes[(c + j) * BM + r]);
                        } else {
                            const bool ok = pix_ok && co0 + j < g.cout;
                            rv[j] = ok ? to_f<T>(res[ybase + (int64_t)j * osp]) : 0.f;
                        }
                    }
                }
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    float val = (__uint_as_float(v[j]) + __shfl_sync(0xffffffffu, pb, j)) *
                                    __shfl_sync(0xffffffffu, ps, j) +
                                __shfl_sync(0xffffffffu, pt, j);
                    const bool ok = pix_ok && co0 + j < g.cout;
                    if (res && e.residual_first) val += rv[j];
                    val = apply_act(val, e.act);
                    if (res && !e.residual_first) val += rv[j];
                    if (TMA_STORE) {
                        sOut[(c + j) * BM + r] = from_f<T>(val);
                    } else if (ok) {
                        y[ybase + (int64_t)j * osp] = from_f<T>(val);
                    }
                }
            }
            tc_fence_before();
            mbar_arrive(&tempty[acc]);
            if (TMA_STORE) {
                fence_proxy_async_smem();
                epi_bar_sync();
                if (ep_tid == 0) {
                    const int cvalid = g.cout - nt * BN;
                    if (cvalid >= BN) {
                        tma_store_4d(&tm_y, sOut, wo0, ho0, nt * BN, (int)img);
                    }
                    bulk_commit();
                }
            }
        }
        if (TMA_STORE && ep_tid == 0) bulk_wait0();
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, TMEM_COLS);
    }
}

template <typename T>
CUtensorMapDataType tmap_dt() {
    return std::is_same<T, __nv_bfloat16>::value ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
}

template <typename T, int BN, int STAGES, bool TMA_STORE, bool RES_TMA = false>
int launch_conv_tc(const T* x_nhwc, const T* wp, T* y, const ConvGeom& cg, const ConvEpi& e, cudaStream_t st) {
    using S = ConvSmem<BN, STAGES, RES_TMA>;
    ConvTcGeom g{};
    g.n = cg.n; g.batch = cg.batch; g.cout = cg.cout; g.ho = cg.oh; g.wo = cg.ow;
    int tw = 1;
    while (tw < cg.ow && tw < BM) tw <<= 1;
    g.tw = tw;
    g.th = BM / tw;
    g.tiles_h = (cg.oh + g.th - 1) / g.th;
    g.tiles_w = (cg.ow + g.tw - 1) / g.tw;
    g.nt_count = (cg.cout + BN - 1) / BN;
    g.kh = cg.kh; g.kw = cg.kw; g.cblocks = cg.cin / BK;
    g.ph = cg.ph; g.pw = cg.pw; g.dh = cg.dh; g.dw = cg.dw;
    const int64_t nb = (int64_t)cg.n * cg.batch;
    CUtensorMap tx, tw_map;
    {
        const uint64_t dims[4] = {(uint64_t)cg.cin, (uint64_t)cg.w, (uint64_t)cg.h, (uint64_t)nb};
        const uint64_t strides[3] = {(uint64_t)cg.cin * 2, (uint64_t)cg.w * cg.cin * 2,
                                     (uint64_t)cg.h * cg.w * cg.cin * 2};
        const uint32_t box[4] = {BK, (uint32_t)g.tw, (uint32_t)g.th, 1};
        int rc = encode_tmap_tiled(&tx, tmap_dt<T>(), 4, x_nhwc, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
        if (rc) return rc;
    }
    {
        const uint64_t k = (uint64_t)cg.kh * cg.kw * cg.cin;
        const uint64_t dims[3] = {k, (uint64_t)cg.cout, (uint64_t)cg.n};
        const uint64_t strides[2] = {k * 2, (uint64_t)cg.cout * k * 2};
        const uint32_t box[3] = {BK, BN, 1};
        int rc = encode_tmap_tiled(&tw_map, tmap_dt<T>(), 3, wp, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
        if (rc) return rc;
    }
    CUtensorMap ty_map;
    memset(&ty_map, 0, sizeof(ty_map));
    if (TMA_STORE) {
        // NCHW output per image: dims {W, H, C, image}; box = one tile of BN channels
        const uint64_t dims[4] = {(uint64_t)cg.ow, (uint64_t)cg.oh, (uint64_t)cg.cout, (uint64_t)nb};
        const uint64_t strides[3] = {(uint64_t)cg.ow * 2, (uint64_t)cg.oh * cg.ow * 2,
                                     (uint64_t)cg.cout * cg.oh * cg.ow * 2};
        const uint32_t box[4] = {(uint32_t)g.tw, (uint32_t)g.th, (uint32_t)BN, 1};
        int rc = encode_tmap_tiled(&ty_map, tmap_dt<T>(), 4, y, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_NONE);
        if (rc) return rc;
    }
    CUtensorMap tr_map;
    memset(&tr_map, 0, sizeof(tr_map));
    if (RES_TMA) {
        const uint64_t dims[4] = {(uint64_t)cg.ow, (uint64_t)cg.oh, (uint64_t)cg.cout, (uint64_t)nb};
        const uint64_t strides[3] = {(uint64_t)cg.ow * 2, (uint64_t)cg.oh * cg.ow * 2,
                                     (uint64_t)cg.cout * cg.oh * cg.ow * 2};
        const uint32_t box[4] = {(uint32_t)g.tw, (uint32_t)g.th, (uint32_t)BN, 1};
        int rc = encode_tmap_tiled(&tr_map, tmap_dt<T>(), 4, e.residual, dims, strides, box,
                                   CU_TENSOR_MAP_SWIZZLE_NONE);
        if (rc) return rc;
    }
    auto kern = conv_tc_kernel<T, BN, STAGES, TMA_STORE, RES_TMA>;
    static bool attr_done[64] = {false};
    const int dev = current_device();
    if (dev >= 0 && dev < 64 && !attr_done[dev]) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)S::TOTAL) != cudaSuccess)
            return set_error(WIDEK_ERR_CUDA, "conv: cannot reserve %u bytes of shared memory", S::TOTAL);
        attr_done[dev] = true;
    }
    const int64_t tiles = (int64_t)g.n * g.nt_count * g.batch * g.tiles_h * g.tiles_w;
    const int grid = (int)std::min<int64_t>(tiles, sm_count(dev));
    kern<<<grid, kThreads, S::TOTAL, st>>>(tx, tw_map, ty_map, tr_map, y, g, e, device_error_ptr());
    return check_launch("widek_conv_fwd (tcgen05)");
}

bool tc_eligible(const ConvGeom& g, int dtype) {
    return (dtype == WIDEK_BF16 || dtype == WIDEK_F16) && g.d == 1 && g.kd == 1 && g.sh == 1 && g.sw == 1 &&
           g.cin % 64 == 0 && g.cout % 16 == 0 && g.cout <= 4096 && g.h <= 65536 && g.w <= 65536;
}

struct ConvLaunch {
    const void *x, *w, *wp;
    void *y, *ws;
    size_t ws_bytes;
    ConvGeom g;
    ConvEpi e;
    int dtype;
    int64_t packed_b;     // > 0: x is channel-packed [batch][n][cin][...] (tensor-core path only)
    cudaStream_t st;
    template <typename T>
    int run() {
        if (wp && tc_eligible(g, dtype)) {
            if constexpr (!std::is_same<T, float>::value) {
                const int64_t nb = (int64_t)g.n * g.batch;
                const size_t need = (size_t)nb * g.cin * g.h * g.w * sizeof(T);
                if (ws && ws_bytes >= need && aligned16(ws) && aligned16(wp)) {
                    const int64_t p = (int64_t)g.h * g.w;
                    if (p % 64 == 0 && aligned16(x)) {
                        const int64_t jobs = nb * (g.cin / 64) * (p / 64);
                        const int blocks = (int)std::min<int64_t>(jobs, (int64_t)sm_count(current_device()) * 8);
                        nchw_to_nhwc_vec_kernel<<<blocks, 256, 0, st>>>(static_cast<const uint16_t*>(x),
                                                                        static_cast<uint16_t*>(ws), nb, g.cin, p,
                                                                        packed_b, g.n);
                    } else {
                        dim3 grid((unsigned)((p + 31) / 32), (unsigned)((g.cin + 31) / 32),
                                  (unsigned)std::min<int64_t>(nb, 65535));
                        nchw_to_nhwc_kernel<T><<<grid, dim3(32, 8), 0, st>>>(static_cast<const T*>(x),
                                                                             static_cast<T*>(ws), nb, g.cin, p);
                    }
                    int rc = check_launch("widek_conv_fwd (nhwc staging)");
                    if (rc) return rc;
                    const T* xs = static_cast<const T*>(ws);
                    const T* wpp = static_cast<const T*>(wp);
                    T* yp = static_cast<T*>(y);
                    // TMA store of the output tile: box width = tile width (>= 8 elements,
                    // 16-byte multiple), rows 16-byte aligned, whole BN-channel tiles.
                    int tw = 1;
                    while (tw < g.ow && tw < BM) tw <<= 1;
                    const bool store_ok = tw >= 8 && g.ow % 8 == 0 && aligned16(yp);
                    const bool res_tma = store_ok && e.residual && aligned16(e.residual);
                    if (g.cout <= 64) {
                        if (res_tma && g.cout == 64) return launch_conv_tc<T, 64, 8, true, true>(xs, wpp, yp, g, e, st);
                        if (store_ok && g.cout == 64) return launch_conv_tc<T, 64, 8, true>(xs, wpp, yp, g, e, st);
                        return launch_conv_tc<T, 64, 8, false>(xs, wpp, yp, g, e, st);
                    }
                    if (g.cout <= 128) {
                        if (res_tma && g.cout % 128 == 0)
                            return launch_conv_tc<T, 128, 5, true, true>(xs, wpp, yp, g, e, st);
                        if (store_ok && g.cout % 128 == 0) return launch_conv_tc<T, 128, 6, true>(xs, wpp, yp, g, e, st);
                        return launch_conv_tc<T, 128, 6, false>(xs, wpp, yp, g, e, st);
                    }
                    if (store_ok && g.cout % 256 == 0) return launch_conv_tc<T, 256, 3, true>(xs, wpp, yp, g, e, st);
                    return launch_conv_tc<T, 256, 3, false>(xs, wpp, yp, g, e, st);
                }
            }
        }
        const int64_t total = (int64_t)g.n * g.batch * g.cout * g.od * g.oh * g.ow;
        conv_direct_kernel<T><<<grid_cap(total, 256), 256, 0, st>>>(static_cast<const T*>(x),
                                                                    static_cast<const T*>(w), static_cast<T*>(y),
                                                                    g, e);
        return check_launch("widek_conv_fwd (direct)");
    }
};

}  // namespace
}  // namespace widek

extern "C" {

int widek_conv_pack_weight(const void* w, void* wp, int64_t rows, int64_t cin, int64_t taps, int64_t elem_bytes,
                           void* stream) {
    using namespace widek;
    if (rows < 0 || cin < 0 || taps < 0) return set_error(WIDEK_ERR_INVALID, "conv_pack_weight: negative size");
    if (rows * cin * taps == 0) return WIDEK_OK;
    if (!w || !wp) return set_error(WIDEK_ERR_INVALID, "conv_pack_weight: null pointer");
    cudaStream_t st = (cudaStream_t)stream;
    const int64_t total = rows * cin * taps;
    if (elem_bytes == 2)
        pack_weight_kernel<uint16_t><<<grid_cap(total, 256), 256, 0, st>>>(
            static_cast<const uint16_t*>(w), static_cast<uint16_t*>(wp), rows, cin, taps);
    else if (elem_bytes == 4)
        pack_weight_kernel<uint32_t><<<grid_cap(total, 256), 256, 0, st>>>(
            static_cast<const uint32_t*>(w), static_cast<uint32_t*>(wp), rows, cin, taps);
    else
        return set_error(WIDEK_ERR_INVALID, "conv_pack_weight: element size %lld", (long long)elem_bytes);
    return check_launch("widek_conv_pack_weight");
}

size_t widek_conv_workspace(int64_t n, int64_t batch, int64_t cin, int64_t d, int64_t h, int64_t w, int dtype) {
    return (size_t)(n * batch * cin * d * h * w) * widek::dtype_size(dtype);
}

int widek_conv_fwd(const void* x, const void* w, const void* w_packed, const void* bias, const void* scale,
                   const void* shift, const void* residual, void* y, void* workspace, size_t workspace_bytes,
                   const int64_t* geom, int act, int residual_first, int dtype, void* stream) {
    using namespace widek;
    if (!geom) return set_error(WIDEK_ERR_INVALID, "conv: null geometry");
    ConvGeom g{};
    int* f = &g.n;
    for (int i = 0; i < 22; ++i) {
        if (geom[i] < 0 || geom[i] > 0x7fffffff) return set_error(WIDEK_ERR_INVALID, "conv: geometry[%d] out of range", i);
        f[i] = (int)geom[i];
    }
    if (g.kd < 1 || g.kh < 1 || g.kw < 1 || g.sd < 1 || g.sh < 1 || g.sw < 1 || g.dd < 1 || g.dh < 1 || g.dw < 1)
        return set_error(WIDEK_ERR_INVALID, "conv: kernel/stride/dilation must be >= 1");
    auto outsz = [](int in, int p, int d, int k, int s) { return (in + 2 * p - d * (k - 1) - 1) / s + 1; };
    if (g.od != outsz(g.d, g.pd, g.dd, g.kd, g.sd) || g.oh != outsz(g.h, g.ph, g.dh, g.kh, g.sh) ||
        g.ow != outsz(g.w, g.pw, g.dw, g.kw, g.sw))
        return set_error(WIDEK_ERR_INVALID, "conv: output size does not match input/kernel/stride/padding");
    if (act < WIDEK_ACT_NONE || act > WIDEK_ACT_GELU) return set_error(WIDEK_ERR_INVALID, "conv: bad activation");
    if ((int64_t)g.n * g.batch * g.cout * g.od * g.oh * g.ow == 0) return WIDEK_OK;
    if (!x || !w || !y) return set_error(WIDEK_ERR_INVALID, "conv: null pointer");
    ConvEpi e{bias, scale, shift, residual, act, residual_first};
    ConvLaunch L{x, w, w_packed, y, workspace, workspace_bytes, g, e, dtype, 0, (cudaStream_t)stream};
    return dispatch_dtype(dtype, L);
}

}  // extern "C"
