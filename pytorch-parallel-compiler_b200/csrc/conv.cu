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
//   * with 64-channel output tiles and a tile width that is a multiple of 8,
//     conv_halo_kernel loads each input region once per tile (kw subtiles
//     covering the kh taps of each column offset) instead of once per tap,
//     and keeps the output tile's weights resident in shared memory.
// CUDA-core path (everything else, including fp32): direct convolution, one
// output element per thread, fp32 accumulation.
#include <cstring>
#include <type_traits>

#include "sm100_ptx.cuh"

namespace widek {
namespace {

using namespace sm100;

// ---------------------------------------------------------------------------
// Layout helpers
// ---------------------------------------------------------------------------
// [nb][c][p] -> [nb][p][c_dst], 32x32 tiles through shared memory (any c,
// p; c_dst >= c, channels c .. c_dst-1 written as zeros, so that a channel
// count that is not a multiple of 8 gets 16-byte pixel rows for the TMA).
template <typename T>
__global__ void nchw_to_nhwc_kernel(const T* __restrict__ src, T* __restrict__ dst, int64_t nb, int c, int64_t p,
                                    int c_dst) {
    __shared__ T tile[32][33];
    const int tx = threadIdx.x, ty = threadIdx.y;   // 32 x 8
    const int64_t p0 = (int64_t)blockIdx.x * 32;
    const int c0 = blockIdx.y * 32;
    for (int64_t img = blockIdx.z; img < nb; img += gridDim.z) {
        const T* s = src + img * c * p;
        T* d = dst + img * c_dst * p;
        for (int r = ty; r < 32; r += 8) {
            const int cc = c0 + r;
            const int64_t pp = p0 + tx;
            tile[r][tx] = cc < c && pp < p ? s[(int64_t)cc * p + pp] : from_f<T>(0.f);
        }
        __syncthreads();
        for (int r = ty; r < 32; r += 8) {
            const int64_t pp = p0 + r;
            const int cc = c0 + tx;
            if (cc < c_dst && pp < p) d[pp * c_dst + cc] = tile[tx][r];
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

// w [rows][cin][taps] -> wp [rows][taps][cin_p] (cin_p >= cin; channels
// cin .. cin_p-1 of every tap are zeros)
template <typename U>
__global__ void pack_weight_kernel(const U* __restrict__ w, U* __restrict__ wp, int64_t rows, int64_t cin,
                                   int64_t taps, int64_t cin_p) {
    const int64_t total = rows * cin_p * taps;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
        const int64_t r = i / (cin_p * taps);
        const int64_t rem = i - r * cin_p * taps;
        const int64_t t = rem / cin_p;
        const int64_t ci = rem - t * cin_p;
        wp[i] = ci < cin ? w[(r * cin + ci) * taps + t] : U(0);
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
__device__ __forceinline__ void tma_store_5d(const CUtensorMap* map, const void* src, int c0, int c1, int c2, int c3,
                                             int c4) {
    asm volatile("cp.async.bulk.tensor.5d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5, %6}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(smem_addr(src)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void epi_bar_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

struct ConvTcGeom {
    int n, batch, cout, od, ho, wo, th, tw, tiles_h, tiles_w, nt_count;
    int kd, kh, kw, cblocks;
    int pd, ph, pw, sd, sh, sw, dd, dh, dw;
};

// Per-tap implicit GEMM, any spatial rank (1-D and 2-D are 3-D with unit
// depth), stride, dilation and channel count. The channels-last input is
// read through a 5-D map {C, W, H, D, image} whose W and H traversal steps
// are the conv strides, so that one box {64, tw*sw, th*sh, 1, 1} delivers
// the tw x th output pixels' input pixels of one tap densely, at
// coordinates (c0, wo0*sw - pw + kx*dw, ho0*sh - ph + ky*dh,
// oz*sd - pd + kz*dd, image). Channels beyond the input's (the last 64-block
// of a channel count that is not a multiple of 64) arrive as zeros (TMA
// out-of-range fill); the packed weights carry zeros there too.
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
    const int taps_hw = g.kh * g.kw;
    const int kb_count = g.kd * taps_hw * g.cblocks;
    const int64_t tiles = (int64_t)g.n * g.nt_count * g.batch * g.od * mt_count;

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

    // tile -> (model, n-tile, image-in-batch, output depth, m-tile); m-tile fastest.
    auto decode = [&](int64_t tile, int& model, int& nt, int& b, int& oz, int& mt) {
        mt = (int)(tile % mt_count); tile /= mt_count;
        oz = (int)(tile % g.od); tile /= g.od;
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
            int model, nt, b, oz, mt;
            decode(tile, model, nt, b, oz, mt);
            const int hy = (mt / g.tiles_w) * g.th * g.sh - g.ph;
            const int wx = (mt % g.tiles_w) * g.tw * g.sw - g.pw;
            const int dz = oz * g.sd - g.pd;
            const int img = model * g.batch + b;
            for (int kb = 0; kb < kb_count; ++kb) {
                const int cb = kb % g.cblocks;
                const int tap = kb / g.cblocks;
                const int kz = tap / taps_hw, kyx = tap - kz * taps_hw;
                const int ky = kyx / g.kw, kx = kyx - ky * g.kw;
                if (!mbar_wait(&empty[s], ph ^ 1, abort_flag)) { ok = false; break; }
                if (lane == 0) {
                    mbar_arrive_expect_tx(&full[s], S::A_BYTES + S::B_BYTES);
                    tma_load_5d(sA + s * S::A_BYTES, &tm_x, &full[s], cb * BK, wx + kx * g.dw, hy + ky * g.dh,
                                dz + kz * g.dd, img, pol_x);
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
        const int64_t osp = (int64_t)g.od * g.ho * g.wo;
        const T* bias = static_cast<const T*>(e.bias);
        const T* scale = static_cast<const T*>(e.scale);
        const T* shift = static_cast<const T*>(e.shift);
        const T* res = static_cast<const T*>(e.residual);
        int local = 0;
        for (int64_t tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++local) {
            int model, nt, b, oz, mt;
            decode(tile, model, nt, b, oz, mt);
            const int acc = local & 1;
            const uint32_t aph = (local >> 1) & 1;
            const int r = q * 32 + lane;                 // pixel within the tile
            const int ho0 = (mt / g.tiles_w) * g.th, wo0 = (mt % g.tiles_w) * g.tw;
            const int ho = ho0 + r / g.tw;
            const int wo = wo0 + r % g.tw;
            const bool pix_ok = ho < g.ho && wo < g.wo;
            const int64_t img = (int64_t)model * g.batch + b;
            const int64_t pix = ((int64_t)oz * g.ho + ho) * g.wo + wo;
            if (TMA_STORE) {
                // The previous tile's store must have finished reading sOut and
                // every thread must be done with the previous sRes; then the
                // residual tile is requested so that it lands while this tile's
                // MMAs finish.
                if (ep_tid == 0) bulk_wait_read0();
                epi_bar_sync();
                if (RES_TMA && ep_tid == 0) {
                    mbar_arrive_expect_tx(res_bar, S::STAGE_RES);
                    tma_load_5d(sRes, &tm_r, res_bar, wo0, ho0, oz, nt * BN, (int)img, l2_policy_evict_first());
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
                        tma_store_5d(&tm_y, sOut, wo0, ho0, oz, nt * BN, (int)img);
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

// ---------------------------------------------------------------------------
// tcgen05 implicit GEMM with halo reuse (stride 1, 64-channel output tiles)
//
// The per-tap kernel above reloads its whole A tile from L2 for each of the
// kh*kw taps. Here a tile of TW x TH output pixels (TW a multiple of 8,
// TH = 128 / TW) loads, per 64-channel input block, kw subtiles of
// TH + (kh-1)*dh input rows x TW pixels (one per horizontal tap offset,
// 128-byte swizzled like the per-tap boxes). For tap (ky, kx) the A operand is
// subtile kx starting ky*dh input rows further down: the 128 rows of A are
// consecutive 128-byte rows of the subtile, at an offset that is a multiple
// of 8 rows (1 KB), so the standard K-major SW128 descriptor applies. The
// weights of the current (model, 64-channel output tile) stay resident in
// shared memory; each CTA works through a contiguous range of tiles (all
// tiles of a model are adjacent), so they are reloaded only when the range
// crosses into the next model or output tile.
// ---------------------------------------------------------------------------
constexpr int kHaloMaxStages = 8;
// Two epilogue warpgroups: for N-first / packed outputs warps 2..5 take TMEM
// lanes (pixels) 32q..32q+15 of their quarter q and warps 6..9 lanes
// 32q+16..32q+31, so such a tile drains in half the time (its epilogue, not
// the MMAs, bounded the tile with four warps: cfg3's conv2 352 -> 333 us).
constexpr int kHaloEpiWarps = 8;
constexpr int kHaloThreads = 352;   // TMA warp, MMA warp, 8 epilogue warps, second MMA warp
__device__ __forceinline__ void halo_epi_sync() {
    asm volatile("bar.sync 1, %0;" ::"n"(kHaloEpiWarps * 32) : "memory");
}
constexpr int HBN = 64;

struct ConvHaloGeom {
    int n, batch, cout, ho, wo, th, tw, tiles_h, tiles_w, nt_count;
    int kh, kw, cblocks, ph, pw, dh, dw;
    int stages;             // ring depth, one subtile per stage
    int out5, res5;         // output / residual in the packed [b][n*c][h][w] layout (5-D maps)
    int shared;             // one halo buffer per (tile, channel block) for all kw column offsets
    int pitch;              // pixels per buffer row in shared mode (a multiple of 8)
    uint32_t sub_bytes;     // (th + (kh-1)*dh) * (shared ? pitch : tw) * 128: one subtile / buffer
    uint32_t w_bytes;       // kh * kw * cblocks * HBN * 128: weights of one output tile
    int64_t tiles;
};

// Activations of the halo epilogues. GELU (erf) is out of line so that the
// unrolled loops do not carry one copy of erff per value. The channels-last
// epilogue fixes the activation at compile time (one copy of its loop per
// activation, picked once per tile); the N-first / packed epilogue keeps the
// runtime test, which measured faster there (its shared-memory accesses
// then spread out instead of competing in bursts with the MMA operand reads).
__device__ __noinline__ float conv_gelu(float v) { return gelu_erf(v); }
template <int ACT>
__device__ __forceinline__ float conv_act(float v) {
    if constexpr (ACT == WIDEK_ACT_RELU) return v > 0.f ? v : 0.f;
    else if constexpr (ACT == WIDEK_ACT_GELU) return conv_gelu(v);
    else return v;
}
__device__ __forceinline__ float conv_act_rt(float v, int act) {
    if (act == WIDEK_ACT_RELU) return v > 0.f ? v : 0.f;
    if (act == WIDEK_ACT_GELU) return conv_gelu(v);
    return v;
}

// Two output tile buffers, used by alternate tiles, so that a tile's
// epilogue only waits for the store issued two tiles earlier. With a
// TMA-loaded residual each buffer first receives the tile's residual
// (requested by the epilogue's elected thread one tile ahead, once the
// buffer's previous store has read it out), which the epilogue updates in
// place (same [channel][pixel] index) before the store.
template <bool RES_TMA>
struct HaloSmem {
    static constexpr uint32_t TILE = HBN * BM * 2;
    static constexpr uint32_t BUFS = 2;
    static constexpr uint32_t BARS = 8 * (2 * kHaloMaxStages + 12) + 16;
    static constexpr uint32_t PARAMS = HBN * 8;      // per-channel (scale, offset) of the current output tile
    static uint32_t fixed(uint32_t w_bytes) { return 1024 + w_bytes + BUFS * TILE + BARS + PARAMS; }
};

// Issues the MMAs of one input subtile (column offset kx, channel block cb):
// for each kernel row ky, 4 MMAs (K = 16 each) over the 64 channels. At
// N = 64 the tensor core consumes an MMA faster than the issuing thread can
// build one, so the descriptors are formed once per stage and advanced by
// constants (the start-address field counts 16-byte units; smem addresses
// stay below 2^18, so adding never carries out of the field), and with
// compile-time KH the loop unrolls completely.
template <int KH>
__device__ __forceinline__ void halo_issue_subtile(uint32_t d_tmem, uint64_t a_desc, uint64_t w_desc,
                                                   uint32_t row_step16, uint32_t tap_stride16, uint32_t idesc,
                                                   bool first_group, int kh_runtime) {
    const int kh = KH > 0 ? KH : kh_runtime;
#pragma unroll
    for (int ky = 0; ky < (KH > 0 ? KH : 8); ++ky) {
        if (KH == 0 && ky >= kh) break;
        const uint64_t ad = a_desc + (uint64_t)(ky * row_step16);
        const uint64_t bd = w_desc + (uint64_t)(ky * tap_stride16);
#pragma unroll
        for (int k = 0; k < BK / 16; ++k)
            umma_f16_ss(d_tmem, ad + 2 * k, bd + 2 * k, idesc, !(first_group && ky == 0 && k == 0));
    }
}

// 16 TMEM lanes x 8 consecutive 32-bit columns, 8 times along the columns
// (64 columns): thread t receives, for column group k, r[4k], r[4k+1] from
// lane (base + t/4), columns 8k + 2(t%4) and + 1, and r[4k+2], r[4k+3] from
// lane (base + 8 + t/4), the same columns.
__device__ __forceinline__ void tmem_ld_16x256b_x8(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.16x256b.x8.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]),
          "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
          "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
}
// Four 8x8 16-bit matrices whose rows (16 bytes each) start at the addresses
// given by lanes 8i..8i+7 for matrix i, transposed: register i of thread t
// holds the matrix's elements (row 2(t%4), column t/4) and (row 2(t%4)+1,
// column t/4), low half first. stmatrix...trans is the inverse.
__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t (&v)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3])
                 : "r"(addr)
                 : "memory");
}
__device__ __forceinline__ void stsm_x4_trans(uint32_t addr, const uint32_t (&v)[4]) {
    asm volatile("stmatrix.sync.aligned.m8n8.x4.trans.shared.b16 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v[0]),
                 "r"(v[1]), "r"(v[2]), "r"(v[3])
                 : "memory");
}
template <typename T>
__device__ __forceinline__ uint32_t pack2(float lo, float hi);
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float lo, float hi) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&v);
}
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float lo, float hi) {
    const __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&v);
}
template <typename T>
__device__ __forceinline__ float2 unpack2(uint32_t v);
template <>
__device__ __forceinline__ float2 unpack2<__nv_bfloat16>(uint32_t v) {
    return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&v));
}
template <>
__device__ __forceinline__ float2 unpack2<__half>(uint32_t v) {
    return __half22float2(*reinterpret_cast<const __half2*>(&v));
}

template <typename T, bool RES_TMA, int KH, int KW, bool OUT_CL>
__global__ void __launch_bounds__(kHaloThreads, 1)
    conv_halo_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
                     const __grid_constant__ CUtensorMap tm_y, const __grid_constant__ CUtensorMap tm_r,
                     ConvHaloGeom g, ConvEpi e, int* err) {
    using S = HaloSmem<RES_TMA>;
    constexpr uint32_t IDESC = idesc_f16(BM, HBN, std::is_same<T, __nv_bfloat16>::value);
    constexpr uint32_t TMEM_COLS = 2 * HBN;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sW = smem;                                    // [kb][HBN rows][128 B]
    T* sBuf = reinterpret_cast<T*>(sW + g.w_bytes);        // [BUFS][HBN][BM]
    uint8_t* sA = reinterpret_cast<uint8_t*>(sBuf) + S::BUFS * S::TILE;   // [stage][rows][tw][128 B]
    uint64_t* full = reinterpret_cast<uint64_t*>(sA + g.stages * g.sub_bytes);
    uint64_t* empty = full + kHaloMaxStages;
    uint64_t* w_full = empty + kHaloMaxStages;
    uint64_t* w_empty = w_full + 1;
    uint64_t* tfull = w_empty + 1;        // [2]
    uint64_t* tempty = tfull + 2;         // [2]
    uint64_t* done = tempty + 2;          // [2], one per MMA issuer
    uint64_t* res_full = done + 2;        // [2]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(res_full + 2);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    float2* sPar = reinterpret_cast<float2*>(reinterpret_cast<uint8_t*>(full) + S::BARS);   // [HBN]

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int mt_count = g.tiles_h * g.tiles_w;
    const int stages = g.stages;
    const int64_t per_cta = (g.tiles + gridDim.x - 1) / gridDim.x;
    const int64_t t_begin = (int64_t)blockIdx.x * per_cta;
    const int64_t t_end = t_begin + per_cta < g.tiles ? t_begin + per_cta : g.tiles;

    if (threadIdx.x == 0) {
        for (int s = 0; s < stages; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
        mbar_init(w_full, 1);
        mbar_init(w_empty, 2);            // both MMA issuers release the weights
        for (int a = 0; a < 2; ++a) {
            mbar_init(&tfull[a], 1);
            mbar_init(&tempty[a], kHaloEpiWarps * 32);
            mbar_init(&res_full[a], 1);
        }
        mbar_init(&done[0], 1);
        mbar_init(&done[1], 1);
        *abort_flag = 0;
        mbar_init_fence();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tm_x);
        tma_prefetch_desc(&tm_w);
        tma_prefetch_desc(&tm_y);
        if (RES_TMA) tma_prefetch_desc(&tm_r);
    }
    if (warp == 1) { tmem_alloc(tmem_slot, TMEM_COLS); tmem_relinquish(); }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    // tile -> (model, n-tile, image-in-batch, m-tile); m-tile fastest. The
    // launcher keeps the tile count below 2^31, so 32-bit division suffices.
    auto decode = [&](int64_t tile64, int& model, int& nt, int& b, int& mt) {
        uint32_t tile = (uint32_t)tile64;
        mt = (int)(tile % (uint32_t)mt_count); tile /= (uint32_t)mt_count;
        b = (int)(tile % (uint32_t)g.batch); tile /= (uint32_t)g.batch;
        nt = (int)(tile % (uint32_t)g.nt_count);
        model = (int)(tile / (uint32_t)g.nt_count);
    };

    if (warp == 0) {
        // TMA producer: weights when the (model, output tile) changes, then
        // per input-channel block and column offset kx one subtile per stage
        // (the residual tiles are requested by the epilogue).
        const uint64_t pol_x = l2_policy_evict_normal();
        const uint64_t pol_w = l2_policy_evict_last();
        int s = 0, issued = 0, wl = 0, local = 0;
        uint32_t ph = 0;
        int64_t cur = -1;
        bool ok = true;
        for (int64_t tile = t_begin; tile < t_end && ok; ++tile, ++local) {
            int model, nt, b, mt;
            decode(tile, model, nt, b, mt);
            const int64_t key = (int64_t)model * g.nt_count + nt;
            if (key != cur) {
                // Previous weights: every MMA that reads them has completed.
                if (wl > 0 && !mbar_wait(w_empty, (uint32_t)((wl - 1) & 1), abort_flag)) { ok = false; break; }
                if (lane == 0) {
                    mbar_arrive_expect_tx(w_full, g.w_bytes);
                    for (int kb = 0; kb < g.kh * g.kw * g.cblocks; ++kb)
                        tma_load_3d(sW + kb * (HBN * 128), &tm_w, w_full, kb * BK, nt * HBN, model, pol_w);
                }
                __syncwarp();
                ++wl;
                cur = key;
            }
            const int ho0 = (mt / g.tiles_w) * g.th;
            const int wo0 = (mt % g.tiles_w) * g.tw;
            const int img = model * g.batch + b;
            const int loads = g.shared ? 1 : g.kw;
            for (int cb = 0; cb < g.cblocks && ok; ++cb) {
                for (int kx = 0; kx < loads; ++kx) {
                    if (!mbar_wait(&empty[s], ph ^ 1, abort_flag)) { ok = false; break; }
                    if (lane == 0) {
                        mbar_arrive_expect_tx(&full[s], g.sub_bytes);
                        tma_load_4d(sA + s * g.sub_bytes, &tm_x, &full[s], cb * BK, wo0 - g.pw + kx * g.dw,
                                    ho0 - g.ph, img, pol_x);
                    }
                    __syncwarp();
                    ++issued;
                    if (++s == stages) { s = 0; ph ^= 1; }
                }
            }
        }
        if (!ok) {
            *abort_flag = 1;
            raise_device_error(err, DEV_ERR_CONV_TIMEOUT);
        }
        if (!ok || *abort_flag) {
            // Copies in flight land before the CTA's shared memory is released.
            const volatile int never = 0;
            if (wl > 0) mbar_wait(w_full, (uint32_t)((wl - 1) & 1), &never);
            const int inflight = issued < stages ? issued : stages;
            for (int j = 1; j <= inflight; ++j) {
                const int idx = issued - j;
                mbar_wait(&full[idx % stages], (uint32_t)((idx / stages) & 1), &never);
            }
        }
    } else if (warp == 1 || warp == kHaloThreads / 32 - 1) {
        // Two MMA issuers (one thread each, in warps 1 and 10): issuer i takes
        // the CTA's tiles with local index = i (mod 2) into accumulator i, so
        // one tile's MMAs go out while the other's are still being issued:
        // a single thread sustains ~60 cycles per M128-N64-K16 MMA, two reach
        // the ~48-cycle shared-memory operand bound. Both walk every tile to
        // keep the subtile ring position and to release the weights (w_empty
        // counts both) whenever the (model, output tile) changes.
        const int me = warp == 1 ? 0 : 1;
        if (lane == 0) {
            int wl = 0;
            int64_t cur = -1;
            uint32_t ring = 0;            // subtiles of all earlier tiles
            bool ok = true;
            const uint64_t a_desc0 = sdesc_kmajor_sw128(smem_addr(sA));
            const uint64_t w_desc0 = sdesc_kmajor_sw128(smem_addr(sW));
            // ky*dh input rows further down in a subtile; one kernel row further in the weights
            const uint32_t row_step16 = (uint32_t)(g.dh * g.tw * 128) >> 4;
            const uint32_t tap_stride16 = (uint32_t)((KW > 0 ? KW : g.kw) * g.cblocks * HBN * 128) >> 4;
            const int kw = KW > 0 ? KW : g.kw;
            const int kh = KH > 0 ? KH : g.kh;
            const uint32_t per_tile = (uint32_t)(g.cblocks * (g.shared ? 1 : kw));
            // Shared mode: A rows are (tile row, pixel) at a pitch of g.pitch
            // pixels, so the 8-row core groups are g.pitch*128 bytes apart
            // (a multiple of 1024); tap (ky, kx) starts ky*dh*pitch + kx*dw
            // rows into the buffer. The start need not be 1024-aligned: the
            // tensor core takes each row's 128-byte swizzle phase from its
            // shared-memory address, as the TMA wrote it (checked against
            // the oracle on B200; the descriptor's base-offset field stays 0).
            const uint64_t a_desc_sh = (a_desc0 & ~((uint64_t)0x3FFF << 32)) |
                                       ((uint64_t)(((uint32_t)g.pitch * 128u) >> 4) << 32);
            int local = 0;
            for (int64_t tile = t_begin; tile < t_end && ok; ++tile, ++local, ring += per_tile) {
                int model, nt, b, mt;
                decode(tile, model, nt, b, mt);
                const int64_t key = (int64_t)model * g.nt_count + nt;
                if (key != cur) {
                    if (wl > 0) umma_commit(w_empty);
                    if (!mbar_wait(w_full, (uint32_t)(wl & 1), abort_flag)) { ok = false; break; }
                    ++wl;
                    cur = key;
                }
                if ((local & 1) != me) continue;
                const uint32_t aph = (local >> 1) & 1;
                if (!mbar_wait(&tempty[me], aph ^ 1, abort_flag)) { ok = false; break; }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + me * HBN;
                uint32_t c = ring;
                if (g.shared) {
                    for (int cb = 0; cb < g.cblocks && ok; ++cb, ++c) {
                        const uint32_t s = c % (uint32_t)g.stages;
                        if (!mbar_wait(&full[s], (c / (uint32_t)g.stages) & 1, abort_flag)) { ok = false; break; }
                        tc_fence_after();
                        const uint64_t a_stage = a_desc_sh + (uint64_t)((s * g.sub_bytes) >> 4);
#pragma unroll 1
                        for (int ky = 0; ky < kh; ++ky) {
#pragma unroll
                            for (int kx = 0; kx < (KW > 0 ? KW : 8); ++kx) {
                                if (KW == 0 && kx >= kw) break;
                                const uint32_t off = (uint32_t)(ky * g.dh * g.pitch + kx * g.dw);
                                const uint64_t ad = a_stage + (uint64_t)(off * 8u);
                                const uint64_t bd = w_desc0 + (uint64_t)((((ky * kw + kx) * g.cblocks + cb) *
                                                                          (HBN * 128)) >> 4);
#pragma unroll
                                for (int k = 0; k < BK / 16; ++k)
                                    umma_f16_ss(d_tmem, ad + 2 * k, bd + 2 * k, IDESC,
                                                !(cb == 0 && ky == 0 && kx == 0 && k == 0));
                            }
                        }
                        umma_commit(&empty[s]);
                    }
                    if (!ok) break;
                    umma_commit(&tfull[me]);
                    continue;
                }
                for (int cb = 0; cb < g.cblocks && ok; ++cb) {
                    for (int kx = 0; kx < kw; ++kx, ++c) {
                        const uint32_t s = c % (uint32_t)g.stages;
                        if (!mbar_wait(&full[s], (c / (uint32_t)g.stages) & 1, abort_flag)) { ok = false; break; }
                        tc_fence_after();
                        const uint64_t a_desc = a_desc0 + (uint64_t)((s * g.sub_bytes) >> 4);
                        const uint64_t w_desc = w_desc0 + (uint64_t)(((kx * g.cblocks + cb) * (HBN * 128)) >> 4);
                        halo_issue_subtile<KH>(d_tmem, a_desc, w_desc, row_step16, tap_stride16, IDESC,
                                               (cb | kx) == 0, g.kh);
                        umma_commit(&empty[s]);
                    }
                }
                if (!ok) break;
                umma_commit(&tfull[me]);
            }
            if (!ok) {
                *abort_flag = 1;
                raise_device_error(err, DEV_ERR_CONV_TIMEOUT);
            }
            // Every MMA issued by this thread completes before TMEM is freed.
            umma_commit(&done[me]);
            const volatile int never = 0;
            mbar_wait(&done[me], 0, &never);
        }
        __syncwarp();
    } else {
        // Epilogue (as conv_tc_kernel with a TMA store): warps 2..9, TMEM lane
        // quarter q = warp % 4, 16-lane half eh = (warp - 2) / 4. Bias and the folded BatchNorm become one
        // (scale, offset) pair per channel, staged in shared memory when the
        // (model, output tile) changes and read as a broadcast per value.
        // Tile i uses buffer i % 2; with a residual that buffer holds the
        // tile's residual, which the output overwrites in place.
        const int q = warp & 3;
        const int eh = (warp - 2) >> 2;            // which 16-lane half of the quarter
        const int ep_tid = threadIdx.x - 64;
        const T* bias = static_cast<const T*>(e.bias);
        const T* scale = static_cast<const T*>(e.scale);
        const T* shift = static_cast<const T*>(e.shift);
        const bool res = RES_TMA && e.residual != nullptr;
        int64_t par_key = -1;
        int res_issued = 0;
        // Channels-last output: threads t and t + 16 of a warp share a pixel
        // (the 16x32bx2 TMEM read), t < 16 taking channels [0, 32) and
        // t >= 16 channels [32, 64); the lane's 32 channels' (scale, offset)
        // pairs stay in registers. The N-first / packed output reads them
        // from shared memory.
        const int ch_half = lane >> 4;
        // N-first / packed output: the lane's 16 channels are 8k + 2(lane%4) + {0, 1}
        // (the 16x256b TMEM read), their pairs likewise held in registers.
        float ps[HBN / 2], po[HBN / 2];
        // Residual tile of `tile` into buffer `rb` (elected thread only).
        auto load_residual = [&](int64_t tile, int rb) {
            int model, nt, b, mt;
            decode(tile, model, nt, b, mt);
            const int ho0 = (mt / g.tiles_w) * g.th, wo0 = (mt % g.tiles_w) * g.tw;
            mbar_arrive_expect_tx(&res_full[rb], S::TILE);
            if (g.res5)
                tma_load_5d(sBuf + rb * (HBN * BM), &tm_r, &res_full[rb], wo0, nt * HBN, ho0, b, model,
                            l2_policy_evict_first());
            else
                tma_load_4d(sBuf + rb * (HBN * BM), &tm_r, &res_full[rb], wo0, nt * HBN, ho0,
                            model * g.batch + b, l2_policy_evict_first());
            ++res_issued;
        };
        if (RES_TMA && ep_tid == 0 && t_begin < t_end) load_residual(t_begin, 0);
        int local = 0;
        for (int64_t tile = t_begin; tile < t_end; ++tile, ++local) {
            int model, nt, b, mt;
            decode(tile, model, nt, b, mt);
            const int acc = local & 1;
            const uint32_t aph = (local >> 1) & 1;
            const int buf = local & 1;
            T* sOut = sBuf + buf * (HBN * BM);
            const int ho0 = (mt / g.tiles_w) * g.th, wo0 = (mt % g.tiles_w) * g.tw;
            const int64_t img = (int64_t)model * g.batch + b;
            // Without a residual: the store issued two tiles ago (from this
            // tile's buffer) has read it out.
            if (ep_tid == 0) {
                if (RES_TMA) {
                    // The previous tile's store has read buffer buf ^ 1 out:
                    // the next tile's residual goes there, a whole tile
                    // ahead of its use.
                    bulk_wait_read0();
                    if (tile + 1 < t_end) load_residual(tile + 1, buf ^ 1);
                } else {
                    bulk_wait_read1();
                }
            }
            const int64_t key = (int64_t)model * g.nt_count + nt;
            const bool fresh = key != par_key;
            if (fresh) {
                // every read of the previous pairs finished before the last tile's second barrier
                if (ep_tid < HBN) {
                    const int64_t ch = (int64_t)model * g.cout + nt * HBN + ep_tid;
                    const float pb = bias ? to_f<T>(bias[ch]) : 0.f;
                    const float sc = scale ? to_f<T>(scale[ch]) : 1.f;
                    const float pt = shift ? to_f<T>(shift[ch]) : 0.f;
                    sPar[ep_tid] = make_float2(sc, pb * sc + pt);
                }
                par_key = key;
            }
            halo_epi_sync();
            if (fresh) {
#pragma unroll
                for (int m = 0; m < HBN / 2; ++m) {
                    const float2 pp = OUT_CL ? sPar[32 * ch_half + m] : sPar[8 * (m >> 1) + 2 * (lane & 3) + (m & 1)];
                    ps[m] = pp.x;
                    po[m] = pp.y;
                }
            }
            // With a channels-last output the second warpgroup has no pixels
            // to drain: it neither polls the accumulator nor the residual
            // (polling warps take issue slots from the MMA and TMA warps),
            // and only keeps step through the barriers and the arrival.
            const bool idle = OUT_CL && eh == 1;
            if (!idle && !mbar_wait(&tfull[acc], aph, abort_flag)) {
                *abort_flag = 1;
                raise_device_error(err, DEV_ERR_CONV_TIMEOUT);
                break;
            }
            tc_fence_after();
            if (RES_TMA && !idle && !mbar_wait(&res_full[buf], (uint32_t)((local >> 1) & 1), abort_flag)) {
                *abort_flag = 1;
                raise_device_error(err, DEV_ERR_CONV_TIMEOUT);
                break;
            }
            if constexpr (OUT_CL) {
                auto epilogue = [&](auto act_c) {
                    constexpr int ACT = decltype(act_c)::value;
                    // channels-last output: the first warpgroup drains both
                    // 16-lane halves (splitting them made conv1 slower, 279 ->
                    // 293 us at cfg3, its MMAs being fed by the input loads);
                    // the second only joins the barriers
#pragma unroll
                    for (int hs = 0; hs < (eh == 0 ? 2 : 0); ++hs) {
                        // pixels q*32 + 16*hs + (lane % 16)
                        uint32_t v[32];
                        tmem_ld_16x32bx2_x32_split32(
                            tmem_base + (uint32_t)(acc * HBN) + ((uint32_t)(q * 32 + 16 * hs) << 16), v);
                        tmem_ld_wait();
                        float ov[32];
#pragma unroll
                        for (int j = 0; j < 32; ++j) ov[j] = conv_act<ACT>(fmaf(__uint_as_float(v[j]), ps[j], po[j]));
                        // channels-last staging: pixel p's 64 channels form
                        // one 128-byte row, 16-byte unit u stored at
                        // u ^ (p % 8) (the 128-byte swizzle the TMA store reads).
                        const int px = q * 32 + 16 * hs + (lane & 15);
                        uint8_t* row = reinterpret_cast<uint8_t*>(sOut) + px * 128;
#pragma unroll
                        for (int u = 0; u < 4; ++u)
                            store16<T>(reinterpret_cast<T*>(row + (((4 * ch_half + u) ^ (px & 7)) << 4)),
                                       ov + 8 * u);
                    }
                };
                if (e.act == WIDEK_ACT_RELU)
                    epilogue(std::integral_constant<int, WIDEK_ACT_RELU>{});
                else if (e.act == WIDEK_ACT_GELU)
                    epilogue(std::integral_constant<int, WIDEK_ACT_GELU>{});
                else
                    epilogue(std::integral_constant<int, WIDEK_ACT_NONE>{});
            } else {
                // N-first / packed output through [row][channel][column]
                // staging (TMA box {tw, 64, th}; 32-byte swizzle for tw = 16):
                // per half warp of TMEM lanes (16 pixels = pixel groups g0,
                // g1 of 8) the 16x256b read gives each thread 2 channels of
                // one pixel per group and column block, which is the
                // fragment of an 8x8 transposed ldmatrix / stmatrix, so the
                // residual is read and the output written 16 bytes per row.
                const uint32_t buf_addr = smem_addr(sOut);
                const int mi = lane >> 3, ri = lane & 7;     // this lane's matrix and row in an x4 access
                // The activation and the residual order are fixed per loop copy
                // (picked once per tile): the unrolled body then has no
                // per-value branches, which keeps it small in the
                // instruction cache next to the MMA and TMA roles.
                auto epilogue = [&](auto act_c, auto rf_c) {
                    constexpr int ACT = decltype(act_c)::value;
                    constexpr bool RF = decltype(rf_c)::value;
                    {
                        const int h = eh;
                        uint32_t v[32];
                        tmem_ld_16x256b_x8(tmem_base + (uint32_t)(acc * HBN) + ((uint32_t)(q * 32 + 16 * h) << 16), v);
                        // row address of matrix mi = (group mi & 1, column block 2*jj + (mi >> 1))
                        const int pix = q * 32 + 16 * h + 8 * (mi & 1);   // first pixel of the group
                        const int py = pix / g.tw, px = pix - py * g.tw;
                        const uint32_t row0 = (uint32_t)(((py * HBN + 8 * (mi >> 1) + ri) * g.tw + px) * 2);
                        const uint32_t swz = g.tw == 16 ? 1u : 0u;
                        uint32_t rv[16];
                        if constexpr (RES_TMA) {
#pragma unroll
                            for (int jj = 0; jj < 4; ++jj) {
                                uint32_t o = row0 + (uint32_t)(16 * jj * g.tw * 2);
                                o ^= (((o >> 7) & 1u) << 4) * swz;
                                uint32_t t4[4];
                                ldsm_x4_trans(buf_addr + o, t4);
#pragma unroll
                                for (int u = 0; u < 4; ++u) rv[4 * jj + u] = t4[u];
                            }
                        }
                        tmem_ld_wait();
                        uint32_t ov[16];
#pragma unroll
                        for (int k = 0; k < 8; ++k) {
                            // column block k: registers 4k..4k+3 = (g0: ch lo, hi), (g1: ch lo, hi);
                            // x4 matrices per jj: (g0, 2jj), (g1, 2jj), (g0, 2jj+1), (g1, 2jj+1)
#pragma unroll
                            for (int gi = 0; gi < 2; ++gi) {
                                float a0 = fmaf(__uint_as_float(v[4 * k + 2 * gi]), ps[2 * k], po[2 * k]);
                                float a1 = fmaf(__uint_as_float(v[4 * k + 2 * gi + 1]), ps[2 * k + 1], po[2 * k + 1]);
                                const int slot = 4 * (k >> 1) + 2 * (k & 1) + gi;
                                if constexpr (RES_TMA && RF) {
                                    const float2 r2 = unpack2<T>(rv[slot]);
                                    a0 += r2.x;
                                    a1 += r2.y;
                                }
                                a0 = conv_act<ACT>(a0);
                                a1 = conv_act<ACT>(a1);
                                if constexpr (RES_TMA && !RF) {
                                    const float2 r2 = unpack2<T>(rv[slot]);
                                    a0 += r2.x;
                                    a1 += r2.y;
                                }
                                ov[slot] = pack2<T>(a0, a1);
                            }
                        }
#pragma unroll
                        for (int jj = 0; jj < 4; ++jj) {
                            uint32_t o = row0 + (uint32_t)(16 * jj * g.tw * 2);
                            o ^= (((o >> 7) & 1u) << 4) * swz;
                            const uint32_t t4[4] = {ov[4 * jj], ov[4 * jj + 1], ov[4 * jj + 2], ov[4 * jj + 3]};
                            stsm_x4_trans(buf_addr + o, t4);
                        }
                    }
                };
                auto with_act = [&](auto rf_c) {
                    if (e.act == WIDEK_ACT_RELU)
                        epilogue(std::integral_constant<int, WIDEK_ACT_RELU>{}, rf_c);
                    else if (e.act == WIDEK_ACT_GELU)
                        epilogue(std::integral_constant<int, WIDEK_ACT_GELU>{}, rf_c);
                    else
                        epilogue(std::integral_constant<int, WIDEK_ACT_NONE>{}, rf_c);
                };
                if (RES_TMA && e.residual_first)
                    with_act(std::true_type{});
                else
                    with_act(std::false_type{});
            }
            tc_fence_before();
            mbar_arrive(&tempty[acc]);
            fence_proxy_async_smem();
            halo_epi_sync();
            if (ep_tid == 0) {
                if (OUT_CL)
                    tma_store_4d(&tm_y, sOut, nt * HBN, wo0, ho0, (int)img);
                else if (g.out5)
                    tma_store_5d(&tm_y, sOut, wo0, nt * HBN, ho0, b, model);
                else
                    tma_store_4d(&tm_y, sOut, wo0, nt * HBN, ho0, (int)img);
                bulk_commit();
            }
        }
        if (ep_tid == 0) {
            bulk_wait0();
            if (RES_TMA && *abort_flag) {
                // residual copies in flight land before the CTA's shared memory is released
                const volatile int never = 0;
                for (int j = 1; j <= 2; ++j) {
                    const int idx = res_issued - j;
                    if (idx >= 0) mbar_wait(&res_full[idx & 1], (uint32_t)((idx >> 1) & 1), &never);
                }
            }
        }
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

// Channel stride of the staged channels-last input: the channel count
// rounded up to 8 (16-byte pixel rows, which the TMA needs); the staging
// writes zeros into the extra channels.
inline int staged_channels(int cin) { return (cin + 7) & ~7; }
// Channels per tap of the packed weights: rounded up to the 64-channel block.
inline int packed_channels(int cin) { return (cin + BK - 1) / BK * BK; }

// Output tile of the per-tap kernel: tw x th pixels of one output depth
// slice, tw a power of two covering the row (at most 128) and th = 128 / tw.
// The input box spans tile * stride elements per dimension, at most 256.
bool tc_tile(const ConvGeom& cg, int& tw, int& th) {
    tw = 1;
    while (tw < cg.ow && tw < BM) tw <<= 1;
    while (tw > 1 && tw * cg.sw > 256) tw >>= 1;
    th = BM / tw;
    return tw * cg.sw <= 256 && th * cg.sh <= 256;
}

template <typename T, int BN, int STAGES, bool TMA_STORE, bool RES_TMA = false>
int launch_conv_tc(const T* x_nhwc, const T* wp, T* y, const ConvGeom& cg, const ConvEpi& e, cudaStream_t st) {
    using S = ConvSmem<BN, STAGES, RES_TMA>;
    ConvTcGeom g{};
    g.n = cg.n; g.batch = cg.batch; g.cout = cg.cout; g.od = cg.od; g.ho = cg.oh; g.wo = cg.ow;
    if (!tc_tile(cg, g.tw, g.th)) return set_error(WIDEK_ERR_UNSUPPORTED, "conv: no tensor-core tile for this stride");
    g.tiles_h = (cg.oh + g.th - 1) / g.th;
    g.tiles_w = (cg.ow + g.tw - 1) / g.tw;
    g.nt_count = (cg.cout + BN - 1) / BN;
    g.kd = cg.kd; g.kh = cg.kh; g.kw = cg.kw;
    const int cin_s = staged_channels(cg.cin), cin_p = packed_channels(cg.cin);
    g.cblocks = cin_p / BK;
    g.pd = cg.pd; g.ph = cg.ph; g.pw = cg.pw;
    g.sd = cg.sd; g.sh = cg.sh; g.sw = cg.sw;
    g.dd = cg.dd; g.dh = cg.dh; g.dw = cg.dw;
    const int64_t nb = (int64_t)cg.n * cg.batch;
    CUtensorMap tx, tw_map;
    {
        const uint64_t row = (uint64_t)cin_s * 2;
        const uint64_t dims[5] = {(uint64_t)cin_s, (uint64_t)cg.w, (uint64_t)cg.h, (uint64_t)cg.d, (uint64_t)nb};
        const uint64_t strides[4] = {row, row * cg.w, row * cg.w * cg.h, row * cg.w * cg.h * cg.d};
        const uint32_t box[5] = {BK, (uint32_t)(g.tw * cg.sw), (uint32_t)(g.th * cg.sh), 1, 1};
        const uint32_t estr[5] = {1, (uint32_t)cg.sw, (uint32_t)cg.sh, 1, 1};
        int rc = encode_tmap_tiled(&tx, tmap_dt<T>(), 5, x_nhwc, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B, estr);
        if (rc) return rc;
    }
    {
        const uint64_t k = (uint64_t)cg.kd * cg.kh * cg.kw * cin_p;
        const uint64_t dims[3] = {k, (uint64_t)cg.cout, (uint64_t)cg.n};
        const uint64_t strides[2] = {k * 2, (uint64_t)cg.cout * k * 2};
        const uint32_t box[3] = {BK, BN, 1};
        int rc = encode_tmap_tiled(&tw_map, tmap_dt<T>(), 3, wp, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
        if (rc) return rc;
    }
    // NCDHW output / residual per image: dims {W, H, D, C, image}; box = one
    // tile of BN channels of one depth slice ([channel][row][column] in
    // shared memory).
    const uint64_t osp = (uint64_t)cg.od * cg.oh * cg.ow;
    const uint64_t odims[5] = {(uint64_t)cg.ow, (uint64_t)cg.oh, (uint64_t)cg.od, (uint64_t)cg.cout, (uint64_t)nb};
    const uint64_t ostrides[4] = {(uint64_t)cg.ow * 2, (uint64_t)cg.oh * cg.ow * 2, osp * 2, (uint64_t)cg.cout * osp * 2};
    const uint32_t obox[5] = {(uint32_t)g.tw, (uint32_t)g.th, 1, (uint32_t)BN, 1};
    CUtensorMap ty_map;
    memset(&ty_map, 0, sizeof(ty_map));
    if (TMA_STORE) {
        int rc = encode_tmap_tiled(&ty_map, tmap_dt<T>(), 5, y, odims, ostrides, obox, CU_TENSOR_MAP_SWIZZLE_NONE);
        if (rc) return rc;
    }
    CUtensorMap tr_map;
    memset(&tr_map, 0, sizeof(tr_map));
    if (RES_TMA) {
        int rc = encode_tmap_tiled(&tr_map, tmap_dt<T>(), 5, e.residual, odims, ostrides, obox,
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
    const int64_t tiles = (int64_t)g.n * g.nt_count * g.batch * g.od * g.tiles_h * g.tiles_w;
    const int grid = (int)std::min<int64_t>(tiles, sm_count(dev));
    kern<<<grid, kThreads, S::TOTAL, st>>>(tx, tw_map, ty_map, tr_map, y, g, e, device_error_ptr());
    return check_launch("widek_conv_fwd (tcgen05)");
}

// 0: halo-reuse kernel where it applies, else the per-tap kernel (default);
// 1: per-tap kernel only; 2: halo kernel with one shared halo buffer per
// tile (8 x 16 pixel tiles) for every output layout (variant 0 uses it for
// channels-last outputs only). Set with widek_conv_set_variant (measurements).
int g_conv_variant = 0;

// Halo-reuse geometry for a stride-1 conv with 64-channel output tiles, or
// false when it does not fit (tile width, box limits, shared memory).
bool halo_geometry(const ConvGeom& cg, bool res_tma, bool cl_out, ConvHaloGeom& g, uint32_t& smem) {
    if (cg.d != 1 || cg.kd != 1 || cg.sh != 1 || cg.sw != 1 || cg.cin % BK != 0) return false;
    if (cg.cout % HBN != 0 || cg.ow % 8 != 0 || cg.ow < 8) return false;
    // Shared halo buffer: 8 x 16 pixel tiles, one buffer of (16 + (kh-1)*dh)
    // rows x pitch pixels per channel block serving every tap (36 KB per
    // tile at 3x3 instead of three 20 KB column-shifted subtiles). Used for
    // channels-last outputs (128-byte output rows; on cfg3's conv1 283 vs
    // 292 us), and for every output with variant 2; the N-first / packed
    // outputs keep 16 x 8 tiles, whose 32-byte output rows make full sectors
    // (with 8-pixel tiles cfg3's conv2 went 331 -> 426 us).
    const int pitch = (8 + (cg.kw - 1) * cg.dw + 7) / 8 * 8;
    const bool shared = (g_conv_variant == 2 || (g_conv_variant == 0 && cl_out)) && pitch <= 256;
    const int tw = shared ? 8 : (cg.ow >= 16 ? 16 : 8);
    const int th = BM / tw;
    const int rows = th + (cg.kh - 1) * cg.dh;
    if (rows > 256) return false;
    g = ConvHaloGeom{};
    g.shared = shared ? 1 : 0;
    g.pitch = pitch;
    g.n = cg.n; g.batch = cg.batch; g.cout = cg.cout; g.ho = cg.oh; g.wo = cg.ow;
    g.tw = tw; g.th = th;
    g.tiles_h = (cg.oh + th - 1) / th;
    g.tiles_w = (cg.ow + tw - 1) / tw;
    g.nt_count = cg.cout / HBN;
    g.kh = cg.kh; g.kw = cg.kw; g.cblocks = cg.cin / BK;
    g.ph = cg.ph; g.pw = cg.pw; g.dh = cg.dh; g.dw = cg.dw;
    g.sub_bytes = (uint32_t)rows * (shared ? pitch : tw) * 128;
    if ((uint64_t)cg.kh * cg.kw * g.cblocks > 64) return false;
    g.w_bytes = (uint32_t)(cg.kh * cg.kw * g.cblocks) * HBN * 128;
    g.tiles = (int64_t)g.n * g.nt_count * g.batch * g.tiles_h * g.tiles_w;
    if (g.tiles > 0x7fffffff) return false;
    const uint32_t fixed = res_tma ? HaloSmem<true>::fixed(g.w_bytes) : HaloSmem<false>::fixed(g.w_bytes);
    if (fixed >= 232448) return false;
    g.stages = (int)std::min<uint32_t>(kHaloMaxStages, (232448 - fixed) / g.sub_bytes);
    if (g.stages < 2) return false;
    smem = fixed + (uint32_t)g.stages * g.sub_bytes;
    return true;
}

// Output / residual tensor maps by layout (WIDEK_LAYOUT_*): N-first NCHW
// [n*b][c][h][w] as 4-D {W, H, C, image}; packed [b][n*c][h][w] as 5-D
// {W, H, C, b, n}; channels-last [n*b][h][w][c] as 4-D {C, W, H, image} with
// a 64-channel, 128-byte-swizzled box.
template <typename T>
int halo_out_map(CUtensorMap* m, const void* base, const ConvGeom& cg, const ConvHaloGeom& g, int layout) {
    const uint64_t nb = (uint64_t)cg.n * cg.batch, sp = (uint64_t)cg.oh * cg.ow;
    if (layout == WIDEK_LAYOUT_CLAST) {
        const uint64_t dims[4] = {(uint64_t)cg.cout, (uint64_t)cg.ow, (uint64_t)cg.oh, nb};
        const uint64_t strides[3] = {(uint64_t)cg.cout * 2, (uint64_t)cg.ow * cg.cout * 2, sp * cg.cout * 2};
        const uint32_t box[4] = {HBN, (uint32_t)g.tw, (uint32_t)g.th, 1};
        return encode_tmap_tiled(m, tmap_dt<T>(), 4, base, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    }
    // NCHW-family layouts: dims ordered {W, C, H, ...} so that a box lands in
    // shared memory as [row][channel][column]; rows of 32 bytes (tw = 16)
    // are 32-byte swizzled, which spreads the epilogue's 8-channel matrix
    // rows over all banks.
    const CUtensorMapSwizzle swz = g.tw == 16 ? CU_TENSOR_MAP_SWIZZLE_32B : CU_TENSOR_MAP_SWIZZLE_NONE;
    if (layout == WIDEK_LAYOUT_PACKED) {
        const uint64_t dims[5] = {(uint64_t)cg.ow, (uint64_t)cg.cout, (uint64_t)cg.oh, (uint64_t)cg.batch,
                                  (uint64_t)cg.n};
        const uint64_t strides[4] = {sp * 2, (uint64_t)cg.ow * 2, (uint64_t)cg.n * cg.cout * sp * 2,
                                     (uint64_t)cg.cout * sp * 2};
        const uint32_t box[5] = {(uint32_t)g.tw, HBN, (uint32_t)g.th, 1, 1};
        return encode_tmap_tiled(m, tmap_dt<T>(), 5, base, dims, strides, box, swz);
    }
    const uint64_t dims[4] = {(uint64_t)cg.ow, (uint64_t)cg.cout, (uint64_t)cg.oh, nb};
    const uint64_t strides[3] = {sp * 2, (uint64_t)cg.ow * 2, (uint64_t)cg.cout * sp * 2};
    const uint32_t box[4] = {(uint32_t)g.tw, HBN, (uint32_t)g.th, 1};
    return encode_tmap_tiled(m, tmap_dt<T>(), 4, base, dims, strides, box, swz);
}

template <typename T, bool RES_TMA, bool OUT_CL>
int launch_conv_halo(const T* x_nhwc, const T* wp, T* y, const ConvGeom& cg, ConvHaloGeom g, uint32_t smem,
                     const ConvEpi& e, int out_layout, int res_layout, cudaStream_t st) {
    const int64_t nb = (int64_t)cg.n * cg.batch;
    CUtensorMap tx, tw_map, ty_map, tr_map;
    {
        const uint64_t dims[4] = {(uint64_t)cg.cin, (uint64_t)cg.w, (uint64_t)cg.h, (uint64_t)nb};
        const uint64_t strides[3] = {(uint64_t)cg.cin * 2, (uint64_t)cg.w * cg.cin * 2,
                                     (uint64_t)cg.h * cg.w * cg.cin * 2};
        const uint32_t bw = (uint32_t)(g.shared ? g.pitch : g.tw);
        const uint32_t box[4] = {BK, bw, g.sub_bytes / (bw * 128), 1};
        int rc = encode_tmap_tiled(&tx, tmap_dt<T>(), 4, x_nhwc, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
        if (rc) return rc;
    }
    {
        const uint64_t k = (uint64_t)cg.kh * cg.kw * cg.cin;
        const uint64_t dims[3] = {k, (uint64_t)cg.cout, (uint64_t)cg.n};
        const uint64_t strides[2] = {k * 2, (uint64_t)cg.cout * k * 2};
        const uint32_t box[3] = {BK, HBN, 1};
        int rc = encode_tmap_tiled(&tw_map, tmap_dt<T>(), 3, wp, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
        if (rc) return rc;
    }
    int rc = halo_out_map<T>(&ty_map, y, cg, g, out_layout);
    if (rc) return rc;
    memset(&tr_map, 0, sizeof(tr_map));
    if (RES_TMA) {
        rc = halo_out_map<T>(&tr_map, e.residual, cg, g, res_layout);
        if (rc) return rc;
    }
    g.out5 = out_layout == WIDEK_LAYOUT_PACKED;
    g.res5 = RES_TMA && res_layout == WIDEK_LAYOUT_PACKED;
    const bool k33 = cg.kh == 3 && cg.kw == 3, k11 = cg.kh == 1 && cg.kw == 1;
    auto kern = k33 ? conv_halo_kernel<T, RES_TMA, 3, 3, OUT_CL>
                    : (k11 ? conv_halo_kernel<T, RES_TMA, 1, 1, OUT_CL> : conv_halo_kernel<T, RES_TMA, 0, 0, OUT_CL>);
    // The dynamic shared memory size varies with the geometry: raise the
    // kernel's limit whenever a larger size is needed.
    static uint32_t attr_bytes[64][3] = {};
    const int dev = current_device();
    const int d = (dev >= 0 && dev < 64) ? dev : 0;
    const int spec = k33 ? 0 : (k11 ? 1 : 2);
    if (attr_bytes[d][spec] < smem) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
            return set_error(WIDEK_ERR_CUDA, "conv: cannot reserve %u bytes of shared memory", smem);
        attr_bytes[d][spec] = smem;
    }
    const int grid = (int)std::min<int64_t>(g.tiles, sm_count(dev));
    kern<<<grid, kHaloThreads, smem, st>>>(tx, tw_map, ty_map, tr_map, g, e, device_error_ptr());
    return check_launch("widek_conv_fwd (tcgen05 halo)");
}

// The tensor-core path takes bf16/f16 convs of any rank, channel count and
// dilation with strides up to 8 along H and W (the TMA traversal-step limit)
// whose output tile fits the 256-element input box.
bool tc_eligible(const ConvGeom& g, int dtype) {
    int tw, th;
    return (dtype == WIDEK_BF16 || dtype == WIDEK_F16) && g.sh <= 8 && g.sw <= 8 && g.cout <= 4096 &&
           g.d <= 65536 && g.h <= 65536 && g.w <= 65536 && tc_tile(g, tw, th);
}

struct ConvLaunch {
    const void *x, *w, *wp;
    void *y, *ws;
    size_t ws_bytes;
    ConvGeom g;
    ConvEpi e;
    int dtype;
    int in_layout, out_layout, res_layout;   // WIDEK_LAYOUT_*
    bool query;           // decide only: WIDEK_OK if the call would run, else WIDEK_ERR_UNSUPPORTED
    cudaStream_t st;
    int path = -1;        // set in query mode: WIDEK_CONV_PATH_*

    // In query mode pointers are absent: treat them as 16-byte aligned (as
    // every caching-allocator block is) and the workspace as large enough.
    bool al(const void* p) const { return query || aligned16(p); }
    int unsupported(const char* why) const {
        return query ? WIDEK_ERR_UNSUPPORTED : set_error(WIDEK_ERR_UNSUPPORTED, "conv: %s", why);
    }

    template <typename T>
    int run() {
        const bool std_layouts = in_layout == WIDEK_LAYOUT_NFIRST && out_layout == WIDEK_LAYOUT_NFIRST &&
                                 res_layout == WIDEK_LAYOUT_NFIRST;
        if ((wp || query) && tc_eligible(g, dtype)) {
            if constexpr (!std::is_same<T, float>::value) {
                const int64_t nb = (int64_t)g.n * g.batch;
                const int64_t p = (int64_t)g.d * g.h * g.w;
                const int cin_s = staged_channels(g.cin);
                const size_t need = (size_t)nb * cin_s * p * sizeof(T);
                const bool cl_in = in_layout == WIDEK_LAYOUT_CLAST;
                const bool ws_ok = query || (ws && ws_bytes >= need && aligned16(ws));
                if (cl_in || ws_ok) {
                    if (!al(wp)) return unsupported("packed weights not 16-byte aligned");
                    const bool vec_staging = g.cin % 64 == 0 && p % 64 == 0 && al(x);
                    if (!cl_in && in_layout == WIDEK_LAYOUT_PACKED && !vec_staging)
                        return unsupported("packed input needs 64-channel and 64-pixel multiples and 16-byte alignment");
                    if (cl_in && (!al(x) || g.cin != cin_s))
                        return unsupported("channels-last input needs 16-byte alignment and a multiple of 8 channels");
                    // TMA store of the output tile: box width = tile width (>= 8 elements,
                    // 16-byte multiple), rows 16-byte aligned, whole channel tiles.
                    int tw, th;
                    tc_tile(g, tw, th);
                    const bool store_ok = tw >= 8 && g.ow % 8 == 0 && al(y);
                    const bool res_tma = store_ok && e.residual && al(e.residual);
                    ConvHaloGeom hg;
                    uint32_t hsmem = 0;
                    // The halo kernel takes a residual only through its TMA
                    // path, and not with a channels-last output.
                    const bool halo = g_conv_variant != 1 && store_ok && (!e.residual || res_tma) &&
                                      !(e.residual && out_layout == WIDEK_LAYOUT_CLAST) &&
                                      halo_geometry(g, res_tma, out_layout == WIDEK_LAYOUT_CLAST, hg, hsmem);
                    // The per-tap kernels read any input layout (staged or
                    // channels-last) but write and add in the N-first layout.
                    if (!halo && (out_layout != WIDEK_LAYOUT_NFIRST || res_layout != WIDEK_LAYOUT_NFIRST))
                        return unsupported("output/residual layout needs the halo kernel, which does not apply");
                    if (query) { path = halo ? WIDEK_CONV_PATH_HALO : WIDEK_CONV_PATH_TAPS; return WIDEK_OK; }
                    const T* xs = static_cast<const T*>(cl_in ? x : ws);
                    if (!cl_in) {
                        const int64_t packed_b = in_layout == WIDEK_LAYOUT_PACKED ? g.batch : 0;
                        if (vec_staging) {
                            const int64_t jobs = nb * (g.cin / 64) * (p / 64);
                            const int blocks = (int)std::min<int64_t>(jobs, (int64_t)sm_count(current_device()) * 8);
                            nchw_to_nhwc_vec_kernel<<<blocks, 256, 0, st>>>(static_cast<const uint16_t*>(x),
                                                                            static_cast<uint16_t*>(ws), nb, g.cin, p,
                                                                            packed_b, g.n);
                        } else {
                            dim3 grid((unsigned)((p + 31) / 32), (unsigned)((cin_s + 31) / 32),
                                      (unsigned)std::min<int64_t>(nb, 65535));
                            nchw_to_nhwc_kernel<T><<<grid, dim3(32, 8), 0, st>>>(
                                static_cast<const T*>(x), static_cast<T*>(ws), nb, g.cin, p, cin_s);
                        }
                        int rc = check_launch("widek_conv_fwd (nhwc staging)");
                        if (rc) return rc;
                    }
                    const T* wpp = static_cast<const T*>(wp);
                    T* yp = static_cast<T*>(y);
                    if (halo) {
                        const bool ocl = out_layout == WIDEK_LAYOUT_CLAST;
                        if (res_tma) return launch_conv_halo<T, true, false>(xs, wpp, yp, g, hg, hsmem, e, out_layout,
                                                                            res_layout, st);
                        if (ocl) return launch_conv_halo<T, false, true>(xs, wpp, yp, g, hg, hsmem, e, out_layout,
                                                                        res_layout, st);
                        return launch_conv_halo<T, false, false>(xs, wpp, yp, g, hg, hsmem, e, out_layout,
                                                                res_layout, st);
                    }
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
        if (!std_layouts) return unsupported("non-default layouts need the tensor-core path");
        if (query) { path = WIDEK_CONV_PATH_DIRECT; return WIDEK_OK; }
        const int64_t total = (int64_t)g.n * g.batch * g.cout * g.od * g.oh * g.ow;
        conv_direct_kernel<T><<<grid_cap(total, 256), 256, 0, st>>>(static_cast<const T*>(x),
                                                                    static_cast<const T*>(w), static_cast<T*>(y),
                                                                    g, e);
        return check_launch("widek_conv_fwd (direct)");
    }
};

// Geometry array -> ConvGeom with validation (shared by the entry points).
int parse_geom(const int64_t* geom, ConvGeom& g) {
    if (!geom) return set_error(WIDEK_ERR_INVALID, "conv: null geometry");
    g = ConvGeom{};
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
    return WIDEK_OK;
}

bool layout_ok(int l) { return l == WIDEK_LAYOUT_NFIRST || l == WIDEK_LAYOUT_PACKED || l == WIDEK_LAYOUT_CLAST; }

}  // namespace
}  // namespace widek

extern "C" {

int widek_conv_set_variant(int variant) {
    if (variant < 0 || variant > 2) return widek::set_error(WIDEK_ERR_INVALID, "conv: unknown variant %d", variant);
    widek::g_conv_variant = variant;
    return WIDEK_OK;
}

int widek_conv_pack_weight(const void* w, void* wp, int64_t rows, int64_t cin, int64_t taps, int64_t elem_bytes,
                           void* stream) {
    using namespace widek;
    if (rows < 0 || cin < 0 || taps < 0) return set_error(WIDEK_ERR_INVALID, "conv_pack_weight: negative size");
    if (rows * cin * taps == 0) return WIDEK_OK;
    if (!w || !wp) return set_error(WIDEK_ERR_INVALID, "conv_pack_weight: null pointer");
    cudaStream_t st = (cudaStream_t)stream;
    const int64_t cin_p = (cin + BK - 1) / BK * BK;
    const int64_t total = rows * cin_p * taps;
    if (elem_bytes == 2)
        pack_weight_kernel<uint16_t><<<grid_cap(total, 256), 256, 0, st>>>(
            static_cast<const uint16_t*>(w), static_cast<uint16_t*>(wp), rows, cin, taps, cin_p);
    else if (elem_bytes == 4)
        pack_weight_kernel<uint32_t><<<grid_cap(total, 256), 256, 0, st>>>(
            static_cast<const uint32_t*>(w), static_cast<uint32_t*>(wp), rows, cin, taps, cin_p);
    else
        return set_error(WIDEK_ERR_INVALID, "conv_pack_weight: element size %lld", (long long)elem_bytes);
    return check_launch("widek_conv_pack_weight");
}

size_t widek_conv_workspace(int64_t n, int64_t batch, int64_t cin, int64_t d, int64_t h, int64_t w, int dtype) {
    const int64_t cin_s = (cin + 7) / 8 * 8;
    return (size_t)(n * batch * cin_s * d * h * w) * widek::dtype_size(dtype);
}

int64_t widek_conv_packed_weight_elems(int64_t rows, int64_t cin, int64_t taps) {
    if (rows < 0 || cin < 0 || taps < 0) return -1;
    return rows * taps * ((cin + widek::BK - 1) / widek::BK * widek::BK);
}

int widek_conv_fwd_ex(const void* x, const void* w, const void* w_packed, const void* bias, const void* scale,
                      const void* shift, const void* residual, void* y, void* workspace, size_t workspace_bytes,
                      const int64_t* geom, int act, int residual_first, int in_layout, int out_layout,
                      int res_layout, int dtype, void* stream) {
    using namespace widek;
    ConvGeom g;
    int rc = parse_geom(geom, g);
    if (rc) return rc;
    if (act < WIDEK_ACT_NONE || act > WIDEK_ACT_GELU) return set_error(WIDEK_ERR_INVALID, "conv: bad activation");
    if (!layout_ok(in_layout) || !layout_ok(out_layout) || !layout_ok(res_layout) ||
        res_layout == WIDEK_LAYOUT_CLAST)
        return set_error(WIDEK_ERR_INVALID, "conv: bad layout code");
    if ((int64_t)g.n * g.batch * g.cout * g.od * g.oh * g.ow == 0) return WIDEK_OK;
    if (!x || !w || !y) return set_error(WIDEK_ERR_INVALID, "conv: null pointer");
    ConvEpi e{bias, scale, shift, residual, act, residual_first};
    ConvLaunch L{x, w, w_packed, y, workspace, workspace_bytes, g, e, dtype, in_layout, out_layout, res_layout,
                 false, (cudaStream_t)stream};
    return dispatch_dtype(dtype, L);
}

int widek_conv_fwd(const void* x, const void* w, const void* w_packed, const void* bias, const void* scale,
                   const void* shift, const void* residual, void* y, void* workspace, size_t workspace_bytes,
                   const int64_t* geom, int act, int residual_first, int dtype, void* stream) {
    return widek_conv_fwd_ex(x, w, w_packed, bias, scale, shift, residual, y, workspace, workspace_bytes, geom, act,
                             residual_first, WIDEK_LAYOUT_NFIRST, WIDEK_LAYOUT_NFIRST, WIDEK_LAYOUT_NFIRST, dtype,
                             stream);
}

int widek_conv_path(const int64_t* geom, int dtype, int in_layout, int out_layout, int res_layout,
                    int has_residual) {
    using namespace widek;
    ConvGeom g;
    if (parse_geom(geom, g)) return -1;
    if (!layout_ok(in_layout) || !layout_ok(out_layout) || !layout_ok(res_layout) || res_layout == WIDEK_LAYOUT_CLAST)
        return -1;
    static const int dummy = 0;
    ConvEpi e{nullptr, nullptr, nullptr, has_residual ? &dummy : nullptr, 0, 0};
    ConvLaunch L{nullptr, nullptr, nullptr, nullptr, nullptr, 0, g, e, dtype, in_layout, out_layout, res_layout,
                 true, nullptr};
    return dispatch_dtype(dtype, L) == WIDEK_OK ? L.path : -1;
}

int widek_conv_layouts_supported(const int64_t* geom, int dtype, int in_layout, int out_layout, int res_layout,
                                 int has_residual) {
    using namespace widek;
    ConvGeom g;
    if (parse_geom(geom, g)) return 0;
    if (!layout_ok(in_layout) || !layout_ok(out_layout) || !layout_ok(res_layout) || res_layout == WIDEK_LAYOUT_CLAST)
        return 0;
    static const int dummy = 0;
    ConvEpi e{nullptr, nullptr, nullptr, has_residual ? &dummy : nullptr, 0, 0};
    ConvLaunch L{nullptr, nullptr, nullptr, nullptr, nullptr, 0, g, e, dtype, in_layout, out_layout, res_layout,
                 true, nullptr};
    return dispatch_dtype(dtype, L) == WIDEK_OK ? 1 : 0;
}

}  // extern "C"
