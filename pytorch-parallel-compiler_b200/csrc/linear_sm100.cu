// WideLinear forward on the 5th-generation tensor cores (tcgen05, sm_100a).
//
//   y[i] = act(x[i] @ w[i]^T + bias[i]),  x: [n, m, k], w: [n, o, k], y: [n, m, o]
//
// Design (one persistent CTA per SM, warp-specialised, 192 threads):
//   warp 0      TMA producer: streams 128x64 tiles of x and BNx64 tiles of w
//               (K-major, 128-byte swizzle) into a STAGES-deep smem ring.
//               4-D tensor maps [n][row blocks][rows per block][k] keep every
//               tile inside one model (rows past m or o read as zero); one
//               block per model is the N-first layout, T-row blocks B apart
//               the packed boundary layout [B, n*T, k] (read in place). w is streamed once
//               (L2 evict-first), x is re-read by every column tile of its
//               model (L2 evict-last).
//   warp 1      allocates TMEM (2 x BN fp32 columns: a double-buffered
//               accumulator); one elected thread issues tcgen05.mma
//               (M=128, N=BN, K=16 per instruction) and tcgen05.commit to
//               release smem stages and to publish finished accumulators.
//   warps 2..5  epilogue: tcgen05.ld the 128 x BN accumulator (one row per
//               thread), add the bias, apply the activation, convert, store.
//               Runs while the MMA warp fills the other accumulator.
// Tiles are ordered (model, column tile, row tile) with the row tile fastest,
// so the CTAs that share a w tile run at the same time and w crosses HBM once.
//
// fp32 (and anything the tensor-core path cannot take) goes to the CUDA-core
// kernel in gemm_simt.cu, so fp32 results keep fp32 products (TF32 off).
#include <cstring>

#include "sm100_ptx.cuh"

namespace widek {
namespace {

// Activation over one 32-value epilogue chunk: one uniform test per chunk,
// so the per-value loops carry no branch (a branch or call per value keeps
// the compiler from scheduling the shuffles, adds and stores across it);
// GELU (erf) is an out-of-line call.
__device__ __noinline__ float gemm_gelu(float v) { return gelu_erf(v); }
__device__ __forceinline__ void act_chunk(float (&v)[32], int act) {
    if (act == WIDEK_ACT_RELU) {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = v[j] > 0.f ? v[j] : 0.f;
    } else if (act == WIDEK_ACT_GELU) {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = gemm_gelu(v[j]);
    }
}

using namespace sm100;

constexpr int BM = 128;
constexpr int BK = 64;  // 64 bf16 = 128 bytes = one swizzle row
constexpr int kGemmThreads = 320;   // TMA warp, MMA warp, 2 x 4 epilogue warps

template <int BN, int STAGES, bool TMA_STORE = false>
struct GemmSmem {
    static constexpr uint32_t A_BYTES = BM * BK * 2;
    static constexpr uint32_t B_BYTES = BN * BK * 2;
    static constexpr uint32_t RING = STAGES * (A_BYTES + B_BYTES);
    // Output staging for the TMA store: per epilogue warpgroup two buffers of
    // 128 rows x 32 columns.
    static constexpr uint32_t OUT_CHUNK = BM * 32 * 2;
    static constexpr uint32_t OUT_BYTES = TMA_STORE ? 4 * OUT_CHUNK : 0;
    static constexpr uint32_t BAR_BYTES = 8 * (2 * STAGES + 4 + 1) + 16;
    static constexpr uint32_t TOTAL = 1024 + RING + OUT_BYTES + BAR_BYTES;  // 1024: alignment slack
};

__device__ __forceinline__ void tma_store_4d(const CUtensorMap* map, const void* src, int c0, int c1, int c2,
                                             int c3) {
    asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(smem_addr(src)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
                 : "memory");
}

// Rows of one model: row r of model i is row (r % rpb) of block (r / rpb);
// the tensor maps carry the block and model strides. y_ms / y_bs (elements)
// address the output rows for the direct (non-TMA) stores.
struct GemmRows {
    int rpb;
    int64_t y_ms, y_bs;
};
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void epi_bar_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }
// Named barrier of one 128-thread epilogue warpgroup (ids 1 and 2).
__device__ __forceinline__ void wg_bar_sync(int wg) { asm volatile("bar.sync %0, 128;" ::"r"(1 + wg) : "memory"); }

// A_MN / B_MN: the operand is read MN-major (its M / N index contiguous in
// memory, one row per K index), as the backward products need: x^T-like
// operands come straight from the untransposed tensors. An MN-major tile is
// loaded as 64-column boxes (128 B rows, 128-byte swizzle) of BK rows each,
// 8 KB apart; its descriptor's leading byte offset is that 8 KB (next 64
// columns), the stride byte offset 1 KB (next 8 K rows), and a K step of 16
// advances 16 rows (2 KB).
template <typename T, int BN, int STAGES, bool TMA_STORE, bool A_MN = false, bool B_MN = false>
__global__ void __launch_bounds__(kGemmThreads, 1)
    linear_tc_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
                     const __grid_constant__ CUtensorMap tm_y, const T* __restrict__ bias, T* __restrict__ y,
                     int n_models, int M, int K, int O, int act, int vec_store, int l2_hints, GemmRows rw,
                     int* err) {
    using S = GemmSmem<BN, STAGES, TMA_STORE>;
    constexpr uint32_t IDESC = idesc_f16(BM, BN, std::is_same<T, __nv_bfloat16>::value) | (A_MN ? 1u << 15 : 0u) |
                               (B_MN ? 1u << 16 : 0u);
    constexpr uint32_t kMnBlock = 64 * BK * 2;        // one 64-column box of an MN-major tile
    constexpr uint32_t A_KSTEP = A_MN ? (16 * 128) >> 4 : 2;   // descriptor units per K step of 16
    constexpr uint32_t B_KSTEP = B_MN ? (16 * 128) >> 4 : 2;
    constexpr uint32_t TMEM_COLS = 2 * BN;

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;
    uint8_t* sB = smem + STAGES * S::A_BYTES;
    uint8_t* sOut = smem + S::RING;     // [2][128 rows][64 B], 64-byte swizzled (TMA store source)
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::RING + S::OUT_BYTES);
    uint64_t* empty = full + STAGES;
    uint64_t* tfull = empty + STAGES;   // [2]
    uint64_t* tempty = tfull + 2;       // [2]
    uint64_t* done = tempty + 2;        // [1]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int mt_count = (M + BM - 1) / BM;
    const int nt_count = (O + BN - 1) / BN;
    const int kb_count = (K + BK - 1) / BK;
    const int tiles = n_models * mt_count * nt_count;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&tfull[a], 1);
            mbar_init(&tempty[a], 8 * 32);
        }
        mbar_init(done, 1);
        *abort_flag = 0;
        mbar_init_fence();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tm_x);
        tma_prefetch_desc(&tm_w);
        if (TMA_STORE) tma_prefetch_desc(&tm_y);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        // ------------------------------------------------------------------
        // TMA producer
        // ------------------------------------------------------------------
        const uint64_t pol_x = l2_hints ? l2_policy_evict_last() : l2_policy_evict_normal();
        const uint64_t pol_w = l2_hints ? l2_policy_evict_first() : l2_policy_evict_normal();
        int s = 0;
        uint32_t ph = 0;
        int issued = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x) {
            const int mt = tile % mt_count;
            const int rest = tile / mt_count;
            const int nt = rest % nt_count;
            const int model = rest / nt_count;
            for (int kb = 0; kb < kb_count; ++kb) {
                if (!mbar_wait(&empty[s], ph ^ 1, abort_flag)) { ok = false; break; }
                if (lane == 0) {
                    mbar_arrive_expect_tx(&full[s], S::A_BYTES + S::B_BYTES);
                    if constexpr (A_MN) {
#pragma unroll
                        for (int j = 0; j < BM / 64; ++j)
                            tma_load_3d(sA + s * S::A_BYTES + j * kMnBlock, &tm_x, &full[s], mt * BM + j * 64,
                                        kb * BK, model, pol_x);
                    } else {
                        tma_load_4d(sA + s * S::A_BYTES, &tm_x, &full[s], kb * BK, (mt * BM) % rw.rpb,
                                    (mt * BM) / rw.rpb, model, pol_x);
                    }
                    if constexpr (B_MN) {
#pragma unroll
                        for (int j = 0; j < BN / 64; ++j)
                            tma_load_3d(sB + s * S::B_BYTES + j * kMnBlock, &tm_w, &full[s], nt * BN + j * 64,
                                        kb * BK, model, pol_w);
                    } else {
                        tma_load_3d(sB + s * S::B_BYTES, &tm_w, &full[s], kb * BK, nt * BN, model, pol_w);
                    }
                }
                __syncwarp();
                ++issued;
                if (++s == STAGES) { s = 0; ph ^= 1; }
            }
        }
        if (!ok) {
            *abort_flag = 1;
            raise_device_error(err, DEV_ERR_GEMM_TIMEOUT);
            // Let copies already in flight land before the CTA's smem is released.
            const int inflight = issued < STAGES ? issued : STAGES;
            for (int j = 1; j <= inflight; ++j) {
                const int idx = issued - j;
                const volatile int never = 0;
                mbar_wait(&full[idx % STAGES], (uint32_t)((idx / STAGES) & 1), &never);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------------
        // MMA issuer: one thread waits, fences and issues, with descriptors
        // formed once and advanced by constants (the start-address field
        // counts 16-byte units and smem addresses stay below 2^18, so the
        // add never carries out of it); the other lanes wait at the end.
        // Warp-wide polling and per-MMA descriptor arithmetic measurably
        // slow the issue of back-to-back MMAs.
        // ------------------------------------------------------------------
        if (lane == 0) {
            int s = 0;
            uint32_t ph = 0;
            bool ok = true;
            int local = 0;
            const uint64_t a_desc0 =
                A_MN ? sdesc_mnmajor_sw128(smem_addr(sA), kMnBlock) : sdesc_kmajor_sw128(smem_addr(sA));
            const uint64_t b_desc0 =
                B_MN ? sdesc_mnmajor_sw128(smem_addr(sB), kMnBlock) : sdesc_kmajor_sw128(smem_addr(sB));
            for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x, ++local) {
                const int acc = local & 1;
                const uint32_t aph = (local >> 1) & 1;
                if (!mbar_wait(&tempty[acc], aph ^ 1, abort_flag)) { ok = false; break; }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * BN;
                for (int kb = 0; kb < kb_count; ++kb) {
                    if (!mbar_wait(&full[s], ph, abort_flag)) { ok = false; break; }
                    tc_fence_after();
                    const uint64_t ad = a_desc0 + (uint64_t)((s * S::A_BYTES) >> 4);
                    const uint64_t bd = b_desc0 + (uint64_t)((s * S::B_BYTES) >> 4);
#pragma unroll
                    for (int k = 0; k < BK / 16; ++k)   // K-major: 32 bytes along the row; MN-major: 16 rows
                        umma_f16_ss(d_tmem, ad + A_KSTEP * k, bd + B_KSTEP * k, IDESC, (kb | k) != 0);
                    umma_commit(&empty[s]);
                    if (++s == STAGES) { s = 0; ph ^= 1; }
                }
                if (!ok) break;
                umma_commit(&tfull[acc]);
            }
            if (!ok) {
                *abort_flag = 1;
                raise_device_error(err, DEV_ERR_GEMM_TIMEOUT);
            }
            // Drain: every MMA this thread issued completes before TMEM is freed.
            umma_commit(done);
            const volatile int never = 0;
            mbar_wait(done, 0, &never);
        }
        __syncwarp();
    } else {
        // ------------------------------------------------------------------
        // Epilogue: two warpgroups (warps 2..5 and 6..9), each warp owning
        // the TMEM lane quarter warp % 4; warpgroup g finishes the column
        // half [g*BN/2, (g+1)*BN/2) of the tile, so the two halves drain in
        // parallel. Per 32-column chunk: lane j fetches bias[col0 + j] once
        // (broadcast by shuffles); with TMA_STORE the chunk (128 rows x 64 B)
        // is staged in the warpgroup's shared memory (64-byte swizzle,
        // double-buffered) and written by one TMA store, so the SM issues
        // full-line writes instead of 16-byte pieces scattered over 32 rows
        // per instruction.
        // ------------------------------------------------------------------
        const int q = warp & 3;
        const int wg = (warp - 2) >> 2;
        const int ep_tid = threadIdx.x - 64 - 128 * wg;
        uint8_t* sOutW = sOut + wg * 2 * S::OUT_CHUNK;
        int local = 0;
        int oc = 0;                               // chunks stored so far (buffer parity)
        for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++local) {
            const int mt = tile % mt_count;
            const int rest = tile / mt_count;
            const int nt = rest % nt_count;
            const int model = rest / nt_count;
            const int acc = local & 1;
            const uint32_t aph = (local >> 1) & 1;
            if (!mbar_wait(&tfull[acc], aph, abort_flag)) {
                *abort_flag = 1;
                raise_device_error(err, DEV_ERR_GEMM_TIMEOUT);
                break;
            }
            tc_fence_after();
            const int rloc = q * 32 + lane;
            const int row = mt * BM + rloc;
            const bool row_ok = row < M;
            const int rr = row_ok ? row : 0;
            T* yrow = y + (int64_t)model * rw.y_ms + (int64_t)(rr / rw.rpb) * rw.y_bs + (int64_t)(rr % rw.rpb) * O;
            const T* brow = bias ? bias + (int64_t)model * O : nullptr;
#pragma unroll 1
            for (int c = wg * (BN / 2); c < (wg + 1) * (BN / 2); c += 32) {
                const int col0 = nt * BN + c;
                if (col0 >= O) break;  // warp-uniform
                uint32_t r[32];
                tmem_ld_32x32b_x32(tmem_base + (uint32_t)(acc * BN + c) + ((uint32_t)(q * 32) << 16), r);
                const float my_bias = (brow && col0 + lane < O) ? to_f<T>(brow[col0 + lane]) : 0.f;
                tmem_ld_wait();
                float v[32];
#pragma unroll
                for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]) + __shfl_sync(0xffffffffu, my_bias, j);
                act_chunk(v, act);
                if (TMA_STORE) {
                    uint8_t* buf = sOutW + (oc & 1) * S::OUT_CHUNK;
                    if (ep_tid == 0) bulk_wait_read1();       // the store that used this buffer has read it
                    wg_bar_sync(wg);
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const int phys = j ^ ((rloc >> 1) & 3);
                        store16<T>(reinterpret_cast<T*>(buf + rloc * 64 + phys * 16), v + 8 * j);
                    }
                    fence_proxy_async_smem();
                    wg_bar_sync(wg);
                    if (ep_tid == 0) {
                        tma_store_4d(&tm_y, buf, col0, (mt * BM) % rw.rpb, (mt * BM) / rw.rpb, model);
                        bulk_commit();
                    }
                    ++oc;
                } else if (row_ok) {
                    if (vec_store && col0 + 32 <= O) {
#pragma unroll
                        for (int j = 0; j < 32; j += 8) store16<T>(yrow + col0 + j, v + j);
                    } else {
#pragma unroll
                        for (int j = 0; j < 32; ++j)
                            if (col0 + j < O) yrow[col0 + j] = from_f<T>(v[j]);
                    }
                }
            }
            tc_fence_before();
            mbar_arrive(&tempty[acc]);
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
// CTA-pair form (cta_group::2): a cluster of 2 CTAs on 2 SMs computes a
// 256 x 256 tile. CTA r loads rows [r*128, r*128+128) of the x tile and rows
// [r*128, r*128+128) of the w tile, so per MMA each SM reads 8 KB of operands
// from its shared memory instead of 12 KB (and its TMA writes 32 KB per k
// block instead of 48 KB); the leader (r = 0) issues M=256, N=256 MMAs that
// read both CTAs' shared memory and write each CTA's 128 accumulator rows
// into its own TMEM. Both CTAs' TMA loads count their bytes on the leader's
// "full" barrier; the leader's commits arrive on the "empty" / "tmem full"
// barriers of both CTAs; each CTA's two epilogue warpgroups (as in
// linear_tc_kernel, one 128-column half each) release the accumulator on
// the leader's "tmem empty" barrier (remote arrive).
// ---------------------------------------------------------------------------
constexpr int kPairStages = 6;

template <bool TMA_STORE>
struct PairSmem {
    static constexpr uint32_t A_BYTES = 128 * BK * 2;
    static constexpr uint32_t B_BYTES = 128 * BK * 2;
    static constexpr uint32_t RING = kPairStages * (A_BYTES + B_BYTES);
    static constexpr uint32_t OUT_CHUNK = 128 * 32 * 2;
    static constexpr uint32_t OUT_BYTES = TMA_STORE ? 4 * OUT_CHUNK : 0;
    static constexpr uint32_t TOTAL = 1024 + RING + OUT_BYTES + 8 * (2 * kPairStages + 5) + 16;
};

template <typename T, bool TMA_STORE>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kGemmThreads, 1)
    linear_tc_pair_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
                          const __grid_constant__ CUtensorMap tm_y, const T* __restrict__ bias, T* __restrict__ y,
                          int n_models, int M, int K, int O, int act, int vec_store, GemmRows rw, int* err) {
    using S = PairSmem<TMA_STORE>;
    constexpr int BN2 = 256;                 // N per pair tile (and per CTA accumulator)
    constexpr uint32_t IDESC = idesc_f16(256, BN2, std::is_same<T, __nv_bfloat16>::value);
    constexpr uint32_t TMEM_COLS = 2 * BN2;
    constexpr int STAGES = kPairStages;

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;
    uint8_t* sB = smem + STAGES * S::A_BYTES;
    uint8_t* sOut = smem + S::RING;     // [2 warpgroups][2][128 rows][64 B], 64-byte swizzled
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::RING + S::OUT_BYTES);
    uint64_t* empty = full + STAGES;
    uint64_t* tfull = empty + STAGES;
    uint64_t* tempty = tfull + 2;
    uint64_t* done = tempty + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const int pair = blockIdx.x >> 1;
    const int npairs = gridDim.x >> 1;
    const int mt_count = (M + 255) / 256;
    const int nt_count = (O + BN2 - 1) / BN2;
    const int kb_count = (K + BK - 1) / BK;
    const int tiles = n_models * mt_count * nt_count;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&tfull[a], 1);
            mbar_init(&tempty[a], 2 * 8 * 32);   // both CTAs' epilogue threads
        }
        mbar_init(done, 1);
        *abort_flag = 0;
        mbar_init_fence();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tm_x);
        tma_prefetch_desc(&tm_w);
        if (TMA_STORE) tma_prefetch_desc(&tm_y);
    }
    if (warp == 1) {
        tmem_alloc_pair(tmem_slot, TMEM_COLS);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    cluster_sync_all();                      // barriers of both CTAs initialised, TMEM allocated
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        // TMA producer (both CTAs); bytes land on the leader's full barrier.
        const uint64_t pol_x = l2_policy_evict_last();
        const uint64_t pol_w = l2_policy_evict_first();
        int s = 0;
        uint32_t ph = 0;
        bool ok = true;
        for (int tile = pair; tile < tiles && ok; tile += npairs) {
            const int mt = tile % mt_count;
            const int rest = tile / mt_count;
            const int nt = rest % nt_count;
            const int model = rest / nt_count;
            const int row0 = mt * 256 + (int)rank * 128;
            for (int kb = 0; kb < kb_count; ++kb) {
                if (!mbar_wait(&empty[s], ph ^ 1, abort_flag)) { ok = false; break; }
                if (lane == 0) {
                    if (rank == 0) mbar_arrive_expect_tx(&full[s], 2 * (S::A_BYTES + S::B_BYTES));
                    const uint32_t leader_full = map_to_rank(smem_addr(&full[s]), 0);
                    tma_load_4d_pair(sA + s * S::A_BYTES, &tm_x, leader_full, kb * BK, row0 % rw.rpb, row0 / rw.rpb,
                                     model, pol_x);
                    tma_load_3d_pair(sB + s * S::B_BYTES, &tm_w, leader_full, kb * BK, nt * BN2 + (int)rank * 128,
                                     model, pol_w);
                }
                __syncwarp();
                if (++s == STAGES) { s = 0; ph ^= 1; }
            }
        }
        if (!ok) {
            *abort_flag = 1;
            raise_device_error(err, DEV_ERR_GEMM_TIMEOUT);
            // This CTA's copies count on the leader's barrier; give them time
            // to land (bounded) before the CTA's shared memory is released.
            const uint64_t t0 = globaltimer_ns();
            while (globaltimer_ns() - t0 < 1000000ull) { }
        }
    } else if (warp == 1) {
        if (rank == 0 && lane == 0) {
            // MMA issuer (leader CTA, one thread; descriptors formed once)
            int s = 0, local = 0;
            uint32_t ph = 0;
            bool ok = true;
            const uint64_t a_desc0 = sdesc_kmajor_sw128(smem_addr(sA));
            const uint64_t b_desc0 = sdesc_kmajor_sw128(smem_addr(sB));
            for (int tile = pair; tile < tiles && ok; tile += npairs, ++local) {
                const int acc = local & 1;
                const uint32_t aph = (local >> 1) & 1;
                if (!mbar_wait(&tempty[acc], aph ^ 1, abort_flag)) { ok = false; break; }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * BN2;
                for (int kb = 0; kb < kb_count; ++kb) {
                    if (!mbar_wait(&full[s], ph, abort_flag)) { ok = false; break; }
                    tc_fence_after();
                    const uint64_t ad = a_desc0 + (uint64_t)((s * S::A_BYTES) >> 4);
                    const uint64_t bd = b_desc0 + (uint64_t)((s * S::B_BYTES) >> 4);
#pragma unroll
                    for (int k = 0; k < BK / 16; ++k)
                        umma_f16_ss_pair(d_tmem, ad + 2 * k, bd + 2 * k, IDESC, (kb | k) != 0);
                    umma_commit_pair_mc(&empty[s], 0x3);
                    if (++s == STAGES) { s = 0; ph ^= 1; }
                }
                if (!ok) break;
                umma_commit_pair_mc(&tfull[acc], 0x3);
            }
            if (!ok) {
                *abort_flag = 1;
                raise_device_error(err, DEV_ERR_GEMM_TIMEOUT);
            }
            umma_commit_pair_mc(done, 0x1);
            const volatile int never = 0;
            mbar_wait(done, 0, &never);
        }
        __syncwarp();
    } else {
        // Epilogue: warpgroup wg (warps 2..5, 6..9) drains the column half
        // [wg*128, wg*128+128) of this CTA's 128 accumulator rows, TMEM lane
        // quarter q = warp % 4, as in linear_tc_kernel.
        const int q = warp & 3;
        const int wg = (warp - 2) >> 2;
        const int ep_tid = threadIdx.x - 64 - 128 * wg;
        uint8_t* sOutW = sOut + wg * 2 * S::OUT_CHUNK;
        const uint32_t leader_tempty0 = map_to_rank(smem_addr(&tempty[0]), 0);
        int oc = 0;
        int local = 0;
        for (int tile = pair; tile < tiles; tile += npairs, ++local) {
            const int mt = tile % mt_count;
            const int rest = tile / mt_count;
            const int nt = rest % nt_count;
            const int model = rest / nt_count;
            const int acc = local & 1;
            const uint32_t aph = (local >> 1) & 1;
            if (!mbar_wait(&tfull[acc], aph, abort_flag)) {
                *abort_flag = 1;
                raise_device_error(err, DEV_ERR_GEMM_TIMEOUT);
                break;
            }
            tc_fence_after();
            const int rloc = q * 32 + lane;
            const int row0 = mt * 256 + (int)rank * 128;
            const int row = row0 + rloc;
            const bool row_ok = row < M;
            const int rr = row_ok ? row : 0;
            T* yrow = y + (int64_t)model * rw.y_ms + (int64_t)(rr / rw.rpb) * rw.y_bs + (int64_t)(rr % rw.rpb) * O;
            const T* brow = bias ? bias + (int64_t)model * O : nullptr;
#pragma unroll 1
            for (int c = wg * (BN2 / 2); c < (wg + 1) * (BN2 / 2); c += 32) {
                const int col0 = nt * BN2 + c;
                if (col0 >= O) break;  // warp-uniform
                uint32_t r[32];
                tmem_ld_32x32b_x32(tmem_base + (uint32_t)(acc * BN2 + c) + ((uint32_t)(q * 32) << 16), r);
                const float my_bias = (brow && col0 + lane < O) ? to_f<T>(brow[col0 + lane]) : 0.f;
                tmem_ld_wait();
                float v[32];
#pragma unroll
                for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]) + __shfl_sync(0xffffffffu, my_bias, j);
                act_chunk(v, act);
                if (TMA_STORE) {
                    // Rows past M of the last tile are clipped by the store;
                    // a CTA whose 128 rows all lie past M stores nothing.
                    uint8_t* buf = sOutW + (oc & 1) * S::OUT_CHUNK;
                    if (ep_tid == 0) bulk_wait_read1();
                    wg_bar_sync(wg);
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const int phys = j ^ ((rloc >> 1) & 3);
                        store16<T>(reinterpret_cast<T*>(buf + rloc * 64 + phys * 16), v + 8 * j);
                    }
                    fence_proxy_async_smem();
                    wg_bar_sync(wg);
                    if (ep_tid == 0 && row0 < M) {
                        tma_store_4d(&tm_y, buf, col0, row0 % rw.rpb, row0 / rw.rpb, model);
                        bulk_commit();
                    }
                    ++oc;
                } else if (row_ok) {
                    if (vec_store && col0 + 32 <= O) {
#pragma unroll
                        for (int j = 0; j < 32; j += 8) store16<T>(yrow + col0 + j, v + j);
                    } else {
#pragma unroll
                        for (int j = 0; j < 32; ++j)
                            if (col0 + j < O) yrow[col0 + j] = from_f<T>(v[j]);
                    }
                }
            }
            tc_fence_before();
            mbar_arrive_remote(leader_tempty0 + acc * 8);
        }
        if (TMA_STORE && ep_tid == 0) bulk_wait0();
    }

    tc_fence_before();
    cluster_sync_all();                      // no CTA leaves while its pair may still touch its smem / TMEM
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, TMEM_COLS);
    }
}

// Kernel selection (set with widek_linear_set_variant, for measurements):
// 0 = automatic, 1 = single-CTA tiles, 2 = CTA-pair 256x256 tiles when
// m > 128 and o > 128, 3 = 128x128 tiles with a 6-stage ring, 4 = as 1
// without L2 hints, 5 = direct stores instead of the TMA store, 6 = fp32 on
// the CUDA-core kernel instead of the split-operand tensor-core kernel.
int g_linear_variant = 0;

template <typename T>
CUtensorMapDataType tmap_dtype();
template <>
CUtensorMapDataType tmap_dtype<__nv_bfloat16>() { return CU_TENSOR_MAP_DATA_TYPE_BFLOAT16; }
template <>
CUtensorMapDataType tmap_dtype<__half>() { return CU_TENSOR_MAP_DATA_TYPE_FLOAT16; }

// Row addressing of x and y: each model's m rows are nblk blocks of rpb rows
// (strides in elements). N-first: one block; packed [B, n*T, *]: B blocks
// of T rows, n*T rows apart, models T rows apart.
struct LinRows {
    int64_t rpb, nblk;
    int64_t x_bs, x_ms, y_bs, y_ms;
};

LinRows nfirst_rows(int64_t m, int64_t k, int64_t o) { return LinRows{m, 1, m * k, m * k, m * o, m * o}; }

// Box rows of one 128-row tile: (rows within a block, blocks).
bool tile_box(const LinRows& r, uint32_t& tb, uint32_t& bb) {
    if (r.nblk == 1 || r.rpb % BM == 0) { tb = BM; bb = 1; return true; }
    if (BM % r.rpb == 0) { tb = (uint32_t)r.rpb; bb = (uint32_t)(BM / r.rpb); return true; }
    return false;
}

template <typename T, int BN, int STAGES, bool TMA_STORE = false>
int launch_tc(const T* x, const T* w, const T* bias, T* y, int64_t n, int64_t m, int64_t k, int64_t o, int act,
              const LinRows& rows, cudaStream_t st) {
    using S = GemmSmem<BN, STAGES, TMA_STORE>;
    uint32_t tb, bb;
    if (!tile_box(rows, tb, bb)) return set_error(WIDEK_ERR_UNSUPPORTED, "linear: row blocks of %lld rows",
                                                  (long long)rows.rpb);
    CUtensorMap tx, tw;
    {
        const uint64_t dims[4] = {(uint64_t)k, (uint64_t)rows.rpb, (uint64_t)rows.nblk, (uint64_t)n};
        const uint64_t strides[3] = {(uint64_t)k * 2, (uint64_t)rows.x_bs * 2, (uint64_t)rows.x_ms * 2};
        const uint32_t box[4] = {BK, tb, bb, 1};
        int rc = encode_tmap_tiled(&tx, tmap_dtype<T>(), 4, x, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
        if (rc) return rc;
    }
    {
        const uint64_t dims[3] = {(uint64_t)k, (uint64_t)o, (uint64_t)n};
        const uint64_t strides[2] = {(uint64_t)k * 2, (uint64_t)o * k * 2};
        const uint32_t box[3] = {BK, BN, 1};
        int rc = encode_tmap_tiled(&tw, tmap_dtype<T>(), 3, w, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
        if (rc) return rc;
    }
    CUtensorMap ty;
    memset(&ty, 0, sizeof(ty));
    if (TMA_STORE) {
        const uint64_t dims[4] = {(uint64_t)o, (uint64_t)rows.rpb, (uint64_t)rows.nblk, (uint64_t)n};
        const uint64_t strides[3] = {(uint64_t)o * 2, (uint64_t)rows.y_bs * 2, (uint64_t)rows.y_ms * 2};
        const uint32_t box[4] = {32, tb, bb, 1};
        int rc = encode_tmap_tiled(&ty, tmap_dtype<T>(), 4, y, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_64B);
        if (rc) return rc;
    }
    auto kern = linear_tc_kernel<T, BN, STAGES, TMA_STORE>;
    static bool attr_done[64] = {false};
    const int dev = current_device();
    if (dev >= 0 && dev < 64 && !attr_done[dev]) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)S::TOTAL) != cudaSuccess)
            return set_error(WIDEK_ERR_CUDA, "linear: cannot reserve %u bytes of shared memory", S::TOTAL);
        attr_done[dev] = true;
    }
    const int64_t tiles = n * ((m + BM - 1) / BM) * ((o + BN - 1) / BN);
    const int grid = (int)std::min<int64_t>(tiles, sm_count(dev));
    const int vec_store = (o % 8 == 0) && aligned16(y);
    const GemmRows rw{(int)rows.rpb, rows.y_ms, rows.y_bs};
    kern<<<grid, kGemmThreads, S::TOTAL, st>>>(tx, tw, ty, bias, y, (int)n, (int)m, (int)k, (int)o, act, vec_store,
                                           g_linear_variant == 4 ? 0 : 1, rw, device_error_ptr());
    return check_launch("widek_linear_fwd (tcgen05)");
}

// y[i] = A_i . B_i on linear_tc_kernel with either operand MN-major (see
// gemm_tc_mn). The MN-major maps are 3-D {cols, K rows, model} with 64-column
// boxes; the K-major ones are the forward's.
template <typename T, int BN, int STAGES, bool TMA_STORE, bool A_MN, bool B_MN>
int launch_tc_mn(const T* a, const T* b, T* y, int64_t n, int64_t M, int64_t K, int64_t N, cudaStream_t st) {
    using S = GemmSmem<BN, STAGES, TMA_STORE>;
    CUtensorMap ta, tb, ty;
    memset(&ty, 0, sizeof(ty));
    if (A_MN) {
        const uint64_t dims[3] = {(uint64_t)M, (uint64_t)K, (uint64_t)n};
        const uint64_t strides[2] = {(uint64_t)M * 2, (uint64_t)K * M * 2};
        const uint32_t box[3] = {64, BK, 1};
        int rc = encode_tmap_tiled(&ta, tmap_dtype<T>(), 3, a, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
        if (rc) return rc;
    } else {
        const uint64_t dims[4] = {(uint64_t)K, (uint64_t)M, 1, (uint64_t)n};
        const uint64_t strides[3] = {(uint64_t)K * 2, (uint64_t)M * K * 2, (uint64_t)M * K * 2};
        const uint32_t box[4] = {BK, BM, 1, 1};
        int rc = encode_tmap_tiled(&ta, tmap_dtype<T>(), 4, a, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
        if (rc) return rc;
    }
    if (B_MN) {
        const uint64_t dims[3] = {(uint64_t)N, (uint64_t)K, (uint64_t)n};
        const uint64_t strides[2] = {(uint64_t)N * 2, (uint64_t)K * N * 2};
        const uint32_t box[3] = {64, BK, 1};
        int rc = encode_tmap_tiled(&tb, tmap_dtype<T>(), 3, b, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
        if (rc) return rc;
    } else {
        const uint64_t dims[3] = {(uint64_t)K, (uint64_t)N, (uint64_t)n};
        const uint64_t strides[2] = {(uint64_t)K * 2, (uint64_t)N * K * 2};
        const uint32_t box[3] = {BK, BN, 1};
        int rc = encode_tmap_tiled(&tb, tmap_dtype<T>(), 3, b, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
        if (rc) return rc;
    }
    if (TMA_STORE) {
        const uint64_t dims[4] = {(uint64_t)N, (uint64_t)M, 1, (uint64_t)n};
        const uint64_t strides[3] = {(uint64_t)N * 2, (uint64_t)M * N * 2, (uint64_t)M * N * 2};
        const uint32_t box[4] = {32, BM, 1, 1};
        int rc = encode_tmap_tiled(&ty, tmap_dtype<T>(), 4, y, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_64B);
        if (rc) return rc;
    }
    auto kern = linear_tc_kernel<T, BN, STAGES, TMA_STORE, A_MN, B_MN>;
    static bool attr_done[64] = {false};
    const int dev = current_device();
    if (dev >= 0 && dev < 64 && !attr_done[dev]) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)S::TOTAL) != cudaSuccess)
            return set_error(WIDEK_ERR_CUDA, "gemm (MN-major): cannot reserve %u bytes of shared memory", S::TOTAL);
        attr_done[dev] = true;
    }
    const int64_t tiles = n * ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
    const int grid = (int)std::min<int64_t>(tiles, sm_count(dev));
    const int vec_store = (N % 8 == 0) && aligned16(y);
    const GemmRows rw{(int)M, M * N, M * N};
    kern<<<grid, kGemmThreads, S::TOTAL, st>>>(ta, tb, ty, nullptr, y, (int)n, (int)M, (int)K, (int)N,
                                               WIDEK_ACT_NONE, vec_store, 1, rw, device_error_ptr());
    return check_launch("gemm (tcgen05, MN-major operands)");
}

template <typename T, bool A_MN, bool B_MN>
int gemm_tc_mn_t(const T* a, const T* b, T* y, int64_t n, int64_t M, int64_t K, int64_t N, cudaStream_t st) {
    if (N > 128) return launch_tc_mn<T, 256, 4, true, A_MN, B_MN>(a, b, y, n, M, K, N, st);
    if (N > 64) return launch_tc_mn<T, 128, 6, true, A_MN, B_MN>(a, b, y, n, M, K, N, st);
    return launch_tc_mn<T, 64, 8, true, A_MN, B_MN>(a, b, y, n, M, K, N, st);
}

// ---------------------------------------------------------------------------
// WideLinear with a fused LayerNorm epilogue:
//   y[i][r] = LayerNorm(x[i][r] @ w[i]^T + bias[i]) * ln_w[i] + ln_b[i]
// for o <= 512 output features (a multiple of 16): the attention output
// projection followed by WideLayerNorm. A tile is 128 rows x all o columns,
// so each row's statistics are complete in TMEM: one 512-column fp32
// accumulator (M = 128; two MMAs of N = 256 / o - 256 per K step when
// o > 256). Same warp roles as linear_tc_kernel; the accumulator is not
// double-buffered (the whole TMEM), so the next tile's MMAs wait for the
// epilogue. Epilogue: warpgroup g owns columns [256g, 256g + 256) of the
// 128 rows (one row per thread); one pass sums d = v - c and d^2 (v = acc
// + bias, c the row's first value: a shifted one-pass variance in fp32),
// the two warpgroups adding their halves through shared memory; a second
// pass writes (v - mean) * rstd * ln_w + ln_b through the staged TMA store. The output is rounded once, from the
// fp32 accumulator (the unfused path rounds the projection to the storage
// dtype before normalising).
// ---------------------------------------------------------------------------
constexpr int kLnBN = 512;
// K per stage 32 (64-byte rows, 64-byte swizzle): a stage is 8 KB of x and
// 32 KB of w, so four stages fit beside the output staging; with 128-byte
// rows (K = 64) a stage is 80 KB and only two fit, which left the TMA
// latency exposed (231 against 142 us at cfg5's size).
constexpr int kLnBK = 32;
constexpr int kLnStages = 4;

struct GemmLnSmem {
    static constexpr uint32_t A_BYTES = BM * kLnBK * 2;
    static constexpr uint32_t B_BYTES = kLnBN * kLnBK * 2;
    static constexpr uint32_t RING = kLnStages * (A_BYTES + B_BYTES);
    static constexpr uint32_t OUT_CHUNK = BM * 32 * 2;
    static constexpr uint32_t OUT_BYTES = 4 * OUT_CHUNK;
    static constexpr uint32_t RED_BYTES = 2 * 2 * BM * 4;     // [sum | sq][warpgroup][row]
    static constexpr uint32_t VEC_BYTES = 3 * kLnBN * 4;      // bias, ln_w, ln_b of the tile's model (fp32)
    static constexpr uint32_t BAR_BYTES = 8 * (2 * kLnStages + 2 + 1) + 16;
    static constexpr uint32_t TOTAL = 1024 + RING + OUT_BYTES + RED_BYTES + VEC_BYTES + BAR_BYTES;
};

// K-major operand tile with 64-byte rows and 64-byte swizzling: 8-row
// groups 512 bytes apart.
__device__ __forceinline__ uint64_t sdesc_kmajor_sw64(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFF);   // start address, 16-byte units
    d |= (uint64_t)1 << 16;                   // leading byte offset (unused when swizzled)
    d |= (uint64_t)(512 >> 4) << 32;          // stride byte offset: 8 rows * 64 B
    d |= (uint64_t)1 << 46;                   // descriptor version for sm_100
    d |= (uint64_t)4 << 61;                   // layout type 4 = 64-byte swizzle
    return d;
}

// Named barrier over the two epilogue warpgroups (256 threads).
__device__ __forceinline__ void epi_all_sync() { asm volatile("bar.sync 3, 256;" ::: "memory"); }

template <typename T>
__global__ void __launch_bounds__(kGemmThreads, 1)
    linear_ln_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
                     const __grid_constant__ CUtensorMap tm_y, const T* __restrict__ bias,
                     const T* __restrict__ ln_w, const T* __restrict__ ln_b, int n_models, int M, int K, int O,
                     float eps, GemmRows rw, int* err) {
    using S = GemmLnSmem;
    constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;
    uint8_t* sB = smem + kLnStages * S::A_BYTES;
    uint8_t* sOut = smem + S::RING;
    float* red = reinterpret_cast<float*>(smem + S::RING + S::OUT_BYTES);   // [2][2][BM]
    float* vec = red + 4 * BM;                                              // [3][kLnBN]
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::RING + S::OUT_BYTES + S::RED_BYTES + S::VEC_BYTES);
    uint64_t* empty = full + kLnStages;
    uint64_t* tfull = empty + kLnStages;
    uint64_t* tempty = tfull + 1;
    uint64_t* done = tempty + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int mt_count = (M + BM - 1) / BM;
    const int kb_count = (K + kLnBK - 1) / kLnBK;
    const int tiles = n_models * mt_count;
    const int o_pad = (O + 15) & ~15;
    const int n0 = o_pad < 256 ? o_pad : 256;          // first MMA's N
    const int n1 = o_pad - n0;                         // second MMA's N (0: none)
    // w boxes: rows [0, n0) and, when o > 256, rows [256, 512) (past o: zeros)
    const uint32_t b_bytes = (uint32_t)n0 * kLnBK * 2 + (n1 > 0 ? 256u * kLnBK * 2 : 0u);

    if (threadIdx.x == 0) {
        for (int s = 0; s < kLnStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(tfull, 1);
        mbar_init(tempty, 8 * 32);
        mbar_init(done, 1);
        *abort_flag = 0;
        mbar_init_fence();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tm_x);
        tma_prefetch_desc(&tm_w);
        tma_prefetch_desc(&tm_y);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, kLnBN);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        // TMA producer: x tile 128 x 64, w rows [0, 256) and [256, 512) as
        // two boxes (the second only when o > 256)
        const uint64_t pol_x = l2_policy_evict_first();
        const uint64_t pol_w = l2_policy_evict_last();
        int s = 0;
        uint32_t ph = 0;
        int issued = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x) {
            const int mt = tile % mt_count;
            const int model = tile / mt_count;
            for (int kb = 0; kb < kb_count; ++kb) {
                if (!mbar_wait(&empty[s], ph ^ 1, abort_flag)) { ok = false; break; }
                if (lane == 0) {
                    mbar_arrive_expect_tx(&full[s], S::A_BYTES + b_bytes);
                    tma_load_4d(sA + s * S::A_BYTES, &tm_x, &full[s], kb * kLnBK, (mt * BM) % rw.rpb,
                                (mt * BM) / rw.rpb, model, pol_x);
                    tma_load_3d(sB + s * S::B_BYTES, &tm_w, &full[s], kb * kLnBK, 0, model, pol_w);
                    if (n1 > 0)
                        tma_load_3d(sB + s * S::B_BYTES + 256 * kLnBK * 2, &tm_w, &full[s], kb * kLnBK, 256, model,
                                    pol_w);
                }
                __syncwarp();
                ++issued;
                if (++s == kLnStages) { s = 0; ph ^= 1; }
            }
        }
        if (!ok) {
            *abort_flag = 1;
            raise_device_error(err, DEV_ERR_GEMM_TIMEOUT);
            const int inflight = issued < kLnStages ? issued : kLnStages;
            for (int j = 1; j <= inflight; ++j) {
                const int idx = issued - j;
                const volatile int never = 0;
                mbar_wait(&full[idx % kLnStages], (uint32_t)((idx / kLnStages) & 1), &never);
            }
        }
    } else if (warp == 1) {
        // MMA issuer (one thread)
        if (lane == 0) {
            int s = 0;
            uint32_t ph = 0;
            bool ok = true;
            int local = 0;
            const uint32_t idesc0 = idesc_f16(BM, n0, kBf16);
            const uint32_t idesc1 = idesc_f16(BM, n1 > 0 ? n1 : 16, kBf16);
            const uint64_t a_desc0 = sdesc_kmajor_sw64(smem_addr(sA));
            const uint64_t b_desc0 = sdesc_kmajor_sw64(smem_addr(sB));
            constexpr uint64_t kB1 = (256 * kLnBK * 2) >> 4;    // rows 256.. of the w tile
            for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x, ++local) {
                if (!mbar_wait(tempty, (uint32_t)(local & 1) ^ 1, abort_flag)) { ok = false; break; }
                tc_fence_after();
                for (int kb = 0; kb < kb_count; ++kb) {
                    if (!mbar_wait(&full[s], ph, abort_flag)) { ok = false; break; }
                    tc_fence_after();
                    const uint64_t ad = a_desc0 + (uint64_t)((s * S::A_BYTES) >> 4);
                    const uint64_t bd = b_desc0 + (uint64_t)((s * S::B_BYTES) >> 4);
#pragma unroll
                    for (int k = 0; k < kLnBK / 16; ++k) {   // 16 elements = 32 bytes along the 64-byte row
                        umma_f16_ss(tmem_base, ad + 2 * k, bd + 2 * k, idesc0, (kb | k) != 0);
                        if (n1 > 0) umma_f16_ss(tmem_base + 256, ad + 2 * k, bd + kB1 + 2 * k, idesc1, (kb | k) != 0);
                    }
                    umma_commit(&empty[s]);
                    if (++s == kLnStages) { s = 0; ph ^= 1; }
                }
                if (!ok) break;
                umma_commit(tfull);
            }
            if (!ok) {
                *abort_flag = 1;
                raise_device_error(err, DEV_ERR_GEMM_TIMEOUT);
            }
            umma_commit(done);
            const volatile int never = 0;
            mbar_wait(done, 0, &never);
        }
        __syncwarp();
    } else {
        // Epilogue: warpgroup wg = columns [256 wg, 256 wg + 256), warp
        // quarter q = TMEM lanes (rows) 32q..32q+31.
        const int q = warp & 3;
        const int wg = (warp - 2) >> 2;
        const int ep_tid = threadIdx.x - 64 - 128 * wg;
        const int rloc = q * 32 + lane;
        uint8_t* sOutW = sOut + wg * 2 * S::OUT_CHUNK;
        float* red_sum = red;               // [2][BM]
        float* red_sq = red + 2 * BM;       // [2][BM]
        const float inv_o = 1.0f / (float)O;
        const int c_begin = wg * 256;
        const int c_end = (wg + 1) * 256 < O ? (wg + 1) * 256 : O;
        int local = 0;
        int oc = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++local) {
            const int mt = tile % mt_count;
            const int model = tile / mt_count;
            if (!mbar_wait(tfull, (uint32_t)(local & 1), abort_flag)) { ok = false; break; }
            tc_fence_after();
            // the tile's model's bias, ln_w and ln_b as fp32 in shared memory
            // (every epilogue thread is done with the previous tile's)
            epi_all_sync();
            for (int j = ep_tid + 128 * wg; j < O; j += 256) {
                vec[j] = bias ? to_f<T>(bias[(int64_t)model * O + j]) : 0.f;
                vec[kLnBN + j] = to_f<T>(ln_w[(int64_t)model * O + j]);
                vec[2 * kLnBN + j] = to_f<T>(ln_b[(int64_t)model * O + j]);
            }
            epi_all_sync();
            const uint32_t trow = tmem_base + ((uint32_t)(q * 32) << 16);
            // pass 1: sums of d = v - c and d^2 over this warpgroup's
            // columns, v = acc + bias, shifted by the row's first value c
            // (the same in both warpgroups) so that the one-pass variance
            // does not cancel when the mean is large against the spread
            const float c0 = __uint_as_float(tmem_ld_32x32b_x1(trow));
            tmem_ld_wait();
            const float shift = c0 + vec[0];
            float s1 = 0.f, s2 = 0.f;
#pragma unroll 1
            for (int c = c_begin; c < c_end; c += 32) {
                uint32_t r[32];
                tmem_ld_32x32b_x32(trow + (uint32_t)c, r);
                tmem_ld_wait();
                if (c + 32 <= O) {
                    const float4* vb = reinterpret_cast<const float4*>(vec + c);
#pragma unroll
                    for (int j4 = 0; j4 < 8; ++j4) {
                        const float4 bv = vb[j4];               // one 16-byte broadcast read
                        const float bj[4] = {bv.x, bv.y, bv.z, bv.w};
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const float dv = __uint_as_float(r[4 * j4 + e]) + bj[e] - shift;
                            s1 += dv;
                            s2 += dv * dv;
                        }
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        const float dv = c + j < O ? __uint_as_float(r[j]) + vec[c + j] - shift : 0.f;
                        s1 += dv;
                        s2 += dv * dv;
                    }
                }
            }
            red_sum[wg * BM + rloc] = s1;
            red_sq[wg * BM + rloc] = s2;
            epi_all_sync();
            const float m1 = (red_sum[rloc] + red_sum[BM + rloc]) * inv_o;      // mean of d
            const float var = fmaxf((red_sq[rloc] + red_sq[BM + rloc]) * inv_o - m1 * m1, 0.f);
            const float mean = shift + m1;
            const float rstd = rsqrtf(var + eps);
            // pass 2: normalise, affine, store through the staged TMA store
#pragma unroll 1
            for (int c = c_begin; c < c_end; c += 32) {
                uint32_t r[32];
                tmem_ld_32x32b_x32(trow + (uint32_t)c, r);
                tmem_ld_wait();
                float v[32];
                const float4* vb = reinterpret_cast<const float4*>(vec + c);
                const float4* vg = reinterpret_cast<const float4*>(vec + kLnBN + c);
                const float4* vh = reinterpret_cast<const float4*>(vec + 2 * kLnBN + c);
#pragma unroll
                for (int j4 = 0; j4 < 8; ++j4) {
                    const float4 bv = vb[j4], gv = vg[j4], hv = vh[j4];
                    const float bj[4] = {bv.x, bv.y, bv.z, bv.w}, gj[4] = {gv.x, gv.y, gv.z, gv.w},
                                hj[4] = {hv.x, hv.y, hv.z, hv.w};
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float u = (__uint_as_float(r[4 * j4 + e]) + bj[e] - mean) * rstd;
                        v[4 * j4 + e] = u * gj[e] + hj[e];
                    }
                }
                uint8_t* buf = sOutW + (oc & 1) * S::OUT_CHUNK;
                if (ep_tid == 0) bulk_wait_read1();
                wg_bar_sync(wg);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int phys = j ^ ((rloc >> 1) & 3);
                    store16<T>(reinterpret_cast<T*>(buf + rloc * 64 + phys * 16), v + 8 * j);
                }
                fence_proxy_async_smem();
                wg_bar_sync(wg);
                if (ep_tid == 0) {
                    tma_store_4d(&tm_y, buf, c, (mt * BM) % rw.rpb, (mt * BM) / rw.rpb, model);
                    bulk_commit();
                }
                ++oc;
            }
            tc_fence_before();
            mbar_arrive(tempty);
        }
        if (!ok) {
            *abort_flag = 1;
            raise_device_error(err, DEV_ERR_GEMM_TIMEOUT);
        }
        if (ep_tid == 0) bulk_wait0();
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, kLnBN);
    }
}

// Launches linear_ln_kernel; WIDEK_ERR_UNSUPPORTED (nothing launched) when
// the shapes, layouts or alignment do not fit it.
template <typename T>
int launch_ln(const T* x, const T* w, const T* bias, const T* lnw, const T* lnb, T* y, int64_t n, int64_t m,
              int64_t k, int64_t o, float eps, const LinRows& rows, cudaStream_t st) {
    using S = GemmLnSmem;
    uint32_t tb, bb;
    if (o < 16 || o > kLnBN || o % 16 != 0 || k % 8 != 0 || k <= 0 || !aligned16(x) || !aligned16(w) ||
        !aligned16(y) || !tile_box(rows, tb, bb) || n > 0x7fffffff || m > 0x7fffffff || k > 0x7fffffff ||
        n * ((m + BM - 1) / BM) > 0x7fffffff)
        return WIDEK_ERR_UNSUPPORTED;
    CUtensorMap tx, tw, ty;
    {
        const uint64_t dims[4] = {(uint64_t)k, (uint64_t)rows.rpb, (uint64_t)rows.nblk, (uint64_t)n};
        const uint64_t strides[3] = {(uint64_t)k * 2, (uint64_t)rows.x_bs * 2, (uint64_t)rows.x_ms * 2};
        const uint32_t box[4] = {kLnBK, tb, bb, 1};
        int rc = encode_tmap_tiled(&tx, tmap_dtype<T>(), 4, x, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_64B);
        if (rc) return rc;
    }
    {
        const uint64_t dims[3] = {(uint64_t)k, (uint64_t)o, (uint64_t)n};
        const uint64_t strides[2] = {(uint64_t)k * 2, (uint64_t)o * k * 2};
        const uint32_t box[3] = {kLnBK, (uint32_t)(o < 256 ? o : 256), 1};
        int rc = encode_tmap_tiled(&tw, tmap_dtype<T>(), 3, w, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_64B);
        if (rc) return rc;
    }
    {
        const uint64_t dims[4] = {(uint64_t)o, (uint64_t)rows.rpb, (uint64_t)rows.nblk, (uint64_t)n};
        const uint64_t strides[3] = {(uint64_t)o * 2, (uint64_t)rows.y_bs * 2, (uint64_t)rows.y_ms * 2};
        const uint32_t box[4] = {32, tb, bb, 1};
        int rc = encode_tmap_tiled(&ty, tmap_dtype<T>(), 4, y, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_64B);
        if (rc) return rc;
    }
    auto kern = linear_ln_kernel<T>;
    static bool attr_done[64] = {false};
    const int dev = current_device();
    if (dev >= 0 && dev < 64 && !attr_done[dev]) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)S::TOTAL) != cudaSuccess)
            return set_error(WIDEK_ERR_CUDA, "linear + layernorm: cannot reserve %u bytes of shared memory", S::TOTAL);
        attr_done[dev] = true;
    }
    const int64_t tiles = n * ((m + BM - 1) / BM);
    const int grid = (int)std::min<int64_t>(tiles, sm_count(dev));
    const GemmRows rw{(int)rows.rpb, rows.y_ms, rows.y_bs};
    kern<<<grid, kGemmThreads, S::TOTAL, st>>>(tx, tw, ty, bias, lnw, lnb, (int)n, (int)m, (int)k, (int)o, eps, rw,
                                               device_error_ptr());
    return check_launch("widek_linear_ln_fwd (tcgen05, LayerNorm epilogue)");
}

template <typename T>
int launch_tc_pair(const T* x, const T* w, const T* bias, T* y, int64_t n, int64_t m, int64_t k, int64_t o, int act,
                   const LinRows& rows, cudaStream_t st) {
    uint32_t tb, bb;
    if (!tile_box(rows, tb, bb)) return set_error(WIDEK_ERR_UNSUPPORTED, "linear: row blocks of %lld rows",
                                                  (long long)rows.rpb);
    CUtensorMap tx, tw;
    {
        const uint64_t dims[4] = {(uint64_t)k, (uint64_t)rows.rpb, (uint64_t)rows.nblk, (uint64_t)n};
        const uint64_t strides[3] = {(uint64_t)k * 2, (uint64_t)rows.x_bs * 2, (uint64_t)rows.x_ms * 2};
        const uint32_t box[4] = {BK, tb, bb, 1};
        int rc = encode_tmap_tiled(&tx, tmap_dtype<T>(), 4, x, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
        if (rc) return rc;
    }
    {
        const uint64_t dims[3] = {(uint64_t)k, (uint64_t)o, (uint64_t)n};
        const uint64_t strides[2] = {(uint64_t)k * 2, (uint64_t)o * k * 2};
        const uint32_t box[3] = {BK, 128, 1};
        int rc = encode_tmap_tiled(&tw, tmap_dtype<T>(), 3, w, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
        if (rc) return rc;
    }
    const int vec_store = (o % 8 == 0) && aligned16(y);
    CUtensorMap ty;
    memset(&ty, 0, sizeof(ty));
    if (vec_store) {
        const uint64_t dims[4] = {(uint64_t)o, (uint64_t)rows.rpb, (uint64_t)rows.nblk, (uint64_t)n};
        const uint64_t strides[3] = {(uint64_t)o * 2, (uint64_t)rows.y_bs * 2, (uint64_t)rows.y_ms * 2};
        const uint32_t box[4] = {32, tb, bb, 1};
        int rc = encode_tmap_tiled(&ty, tmap_dtype<T>(), 4, y, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_64B);
        if (rc) return rc;
    }
    const int dev = current_device();
    const int64_t tiles = n * ((m + 255) / 256) * ((o + 255) / 256);
    const int pairs = (int)std::min<int64_t>(tiles, sm_count(dev) / 2);
    const GemmRows rw{(int)rows.rpb, rows.y_ms, rows.y_bs};
    auto launch = [&](auto kern, uint32_t smem_bytes, bool& attr_done) -> int {
        if (!attr_done) {
            if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_bytes) !=
                cudaSuccess)
                return set_error(WIDEK_ERR_CUDA, "linear: cannot reserve %u bytes of shared memory", smem_bytes);
            attr_done = true;
        }
        kern<<<2 * pairs, kGemmThreads, smem_bytes, st>>>(tx, tw, ty, bias, y, (int)n, (int)m, (int)k, (int)o, act,
                                                           vec_store, rw, device_error_ptr());
        return check_launch("widek_linear_fwd (tcgen05 pair)");
    };
    static bool attr_store[64] = {false}, attr_plain[64] = {false};
    const int d = (dev >= 0 && dev < 64) ? dev : 0;
    if (vec_store) return launch(linear_tc_pair_kernel<T, true>, PairSmem<true>::TOTAL, attr_store[d]);
    return launch(linear_tc_pair_kernel<T, false>, PairSmem<false>::TOTAL, attr_plain[d]);
}

template <typename T>
int linear_tc(const T* x, const T* w, const T* bias, T* y, int64_t n, int64_t m, int64_t k, int64_t o, int act,
              const LinRows& r, cudaStream_t st) {
    if (g_linear_variant == 2 && o > 128 && m > 128) return launch_tc_pair<T>(x, w, bias, y, n, m, k, o, act, r, st);
    if (g_linear_variant == 3 && o > 64) return launch_tc<T, 128, 6>(x, w, bias, y, n, m, k, o, act, r, st);
    // Output through shared memory + TMA store when the output rows are
    // 16-byte aligned (o % 8 == 0); variant 5 keeps direct stores.
    const bool store_ok = (o % 8 == 0) && aligned16(y) && g_linear_variant != 5;
    if (store_ok) {
        if (o > 128) return launch_tc<T, 256, 4, true>(x, w, bias, y, n, m, k, o, act, r, st);
        if (o > 64) return launch_tc<T, 128, 6, true>(x, w, bias, y, n, m, k, o, act, r, st);
        return launch_tc<T, 64, 8, true>(x, w, bias, y, n, m, k, o, act, r, st);
    }
    if (o > 128) return launch_tc<T, 256, 4>(x, w, bias, y, n, m, k, o, act, r, st);
    if (o > 64) return launch_tc<T, 128, 6>(x, w, bias, y, n, m, k, o, act, r, st);
    return launch_tc<T, 64, 8>(x, w, bias, y, n, m, k, o, act, r, st);
}

int linear_entry(const void* x, const void* w, const void* bias, void* y, int64_t n, int64_t m, int64_t k, int64_t o,
                 const LinRows& r, int dtype, int act, cudaStream_t st) {
    if (n < 0 || m < 0 || k < 0 || o < 0)
        return set_error(WIDEK_ERR_INVALID, "linear: negative size");
    if (act < WIDEK_ACT_NONE || act > WIDEK_ACT_GELU) return set_error(WIDEK_ERR_INVALID, "linear: bad activation %d", act);
    if (n == 0 || m == 0 || o == 0) return WIDEK_OK;
    uint32_t tb, bb;
    const bool tc_ok = (dtype == WIDEK_BF16 || dtype == WIDEK_F16) && k > 0 && (k % 8 == 0) && aligned16(x) &&
                       aligned16(w) && n <= 0x7fffffff && m <= 0x7fffffff && k <= 0x7fffffff &&
                       o <= 0x7fffffff && n * ((m + 127) / 128) * ((o + 63) / 64) <= 0x7fffffff &&
                       tile_box(r, tb, bb);
    if (!tc_ok) {
        if (!x && k > 0) return set_error(WIDEK_ERR_INVALID, "linear: null x");
        if (!y) return set_error(WIDEK_ERR_INVALID, "linear: null y");
        // fp32 without an activation: the split-operand tensor-core GEMM
        // where it fits (products within ~2^-16 of fp32), else CUDA cores
        if (dtype == WIDEK_F32 && act == WIDEK_ACT_NONE && g_linear_variant != 6) {
            const int rc = linear_f32x3_strided(static_cast<const float*>(x), static_cast<const float*>(w),
                                                static_cast<const float*>(bias), static_cast<float*>(y), n, m, k, o,
                                                o * k, k, r.x_ms, r.x_bs, r.rpb, r.y_ms, r.y_bs, st);
            if (rc != WIDEK_ERR_UNSUPPORTED) return rc;
        }
        return linear_simt_strided(x, w, bias, y, n, m, k, o, o * k, k, dtype, act, st, r.x_ms, r.x_bs, r.rpb,
                                   r.y_ms, r.y_bs);
    }
    if (dtype == WIDEK_BF16)
        return linear_tc<__nv_bfloat16>((const __nv_bfloat16*)x, (const __nv_bfloat16*)w,
                                        (const __nv_bfloat16*)bias, (__nv_bfloat16*)y, n, m, k, o, act, r, st);
    return linear_tc<__half>((const __half*)x, (const __half*)w, (const __half*)bias, (__half*)y, n, m, k, o, act,
                             r, st);
}

}  // namespace

int gemm_tc_mn(const void* a, const void* b, void* y, int64_t n, int64_t M, int64_t K, int64_t N, bool a_mn,
               bool b_mn, int dtype, cudaStream_t st) {
    if (dtype != WIDEK_BF16 && dtype != WIDEK_F16) return WIDEK_ERR_UNSUPPORTED;
    if (n <= 0 || M <= 0 || K <= 0 || N <= 0 || n > 0x7fffffff || M > 0x7fffffff || K > 0x7fffffff ||
        N > 0x7fffffff || n * ((M + 127) / 128) * ((N + 63) / 64) > 0x7fffffff)
        return WIDEK_ERR_UNSUPPORTED;
    // TMA rows start on 16-byte boundaries: the contiguous extent of each
    // operand (K when K-major, M / N when MN-major) and of y a multiple of 8
    if ((a_mn ? M : K) % 8 != 0 || (b_mn ? N : K) % 8 != 0 || N % 8 != 0 || !aligned16(a) || !aligned16(b) ||
        !aligned16(y))
        return WIDEK_ERR_UNSUPPORTED;
    auto go = [&](auto tag) -> int {
        using T = decltype(tag);
        const T* A = static_cast<const T*>(a);
        const T* B = static_cast<const T*>(b);
        T* Y = static_cast<T*>(y);
        if (a_mn && b_mn) return gemm_tc_mn_t<T, true, true>(A, B, Y, n, M, K, N, st);
        if (a_mn) return gemm_tc_mn_t<T, true, false>(A, B, Y, n, M, K, N, st);
        if (b_mn) return gemm_tc_mn_t<T, false, true>(A, B, Y, n, M, K, N, st);
        return gemm_tc_mn_t<T, false, false>(A, B, Y, n, M, K, N, st);
    };
    return dtype == WIDEK_BF16 ? go(__nv_bfloat16{}) : go(__half{});
}

}  // namespace widek

extern "C" int widek_linear_set_variant(int variant) {
    if (variant < 0 || variant > 6) return widek::set_error(WIDEK_ERR_INVALID, "linear variant %d", variant);
    widek::g_linear_variant = variant;
    return WIDEK_OK;
}

extern "C" int widek_linear_fwd(const void* x, const void* w, const void* bias, void* y, int64_t n, int64_t m,
                                int64_t k, int64_t o, int dtype, int act, void* stream) {
    using namespace widek;
    return linear_entry(x, w, bias, y, n, m, k, o, nfirst_rows(m, k, o), dtype, act, (cudaStream_t)stream);
}

extern "C" int widek_linear_ln_fwd_ex(const void* x, const void* w, const void* bias, const void* ln_w,
                                      const void* ln_b, void* y, int64_t n, int64_t m, int64_t k, int64_t o,
                                      int64_t rows_per_block, int in_layout, int out_layout, double eps, int dtype,
                                      void* stream) {
    using namespace widek;
    const bool pin = in_layout == WIDEK_LAYOUT_PACKED, pout = out_layout == WIDEK_LAYOUT_PACKED;
    if ((!pin && in_layout != WIDEK_LAYOUT_NFIRST) || (!pout && out_layout != WIDEK_LAYOUT_NFIRST))
        return set_error(WIDEK_ERR_INVALID, "linear + layernorm: layouts must be N-first or packed");
    if (n < 0 || m < 0 || k < 0 || o < 0) return set_error(WIDEK_ERR_INVALID, "linear + layernorm: negative size");
    if (n == 0 || m == 0) return WIDEK_OK;
    if (!x || !w || !ln_w || !ln_b || !y) return set_error(WIDEK_ERR_INVALID, "linear + layernorm: null pointer");
    if (dtype != WIDEK_BF16 && dtype != WIDEK_F16) return WIDEK_ERR_UNSUPPORTED;
    if ((pin || pout) && (rows_per_block <= 0 || m % rows_per_block != 0))
        return set_error(WIDEK_ERR_INVALID, "linear + layernorm: %lld rows are not whole blocks of %lld", (long long)m,
                         (long long)rows_per_block);
    const int64_t t = (pin || pout) ? rows_per_block : m, nb = m / t;
    LinRows r{t, nb, pin ? n * t * k : t * k, pin ? t * k : m * k, pout ? n * t * o : t * o, pout ? t * o : m * o};
    if (dtype == WIDEK_BF16)
        return launch_ln<__nv_bfloat16>((const __nv_bfloat16*)x, (const __nv_bfloat16*)w, (const __nv_bfloat16*)bias,
                                        (const __nv_bfloat16*)ln_w, (const __nv_bfloat16*)ln_b, (__nv_bfloat16*)y,
                                        n, m, k, o, (float)eps, r, (cudaStream_t)stream);
    return launch_ln<__half>((const __half*)x, (const __half*)w, (const __half*)bias, (const __half*)ln_w,
                             (const __half*)ln_b, (__half*)y, n, m, k, o, (float)eps, r, (cudaStream_t)stream);
}

extern "C" int widek_linear_fwd_ex(const void* x, const void* w, const void* bias, void* y, int64_t n, int64_t m,
                                   int64_t k, int64_t o, int64_t rows_per_block, int in_layout, int out_layout,
                                   int dtype, int act, void* stream) {
    using namespace widek;
    const bool pin = in_layout == WIDEK_LAYOUT_PACKED, pout = out_layout == WIDEK_LAYOUT_PACKED;
    if ((!pin && in_layout != WIDEK_LAYOUT_NFIRST) || (!pout && out_layout != WIDEK_LAYOUT_NFIRST))
        return set_error(WIDEK_ERR_INVALID, "linear: layouts must be N-first or packed");
    if (!pin && !pout) return widek_linear_fwd(x, w, bias, y, n, m, k, o, dtype, act, stream);
    if (rows_per_block <= 0 || m < 0 || m % rows_per_block != 0)
        return set_error(WIDEK_ERR_INVALID, "linear: %lld rows are not blocks of %lld", (long long)m,
                         (long long)rows_per_block);
    const int64_t t = rows_per_block;
    LinRows r{t, m / t, pin ? n * t * k : t * k, pin ? t * k : m * k, pout ? n * t * o : t * o, pout ? t * o : m * o};
    return linear_entry(x, w, bias, y, n, m, k, o, r, dtype, act, (cudaStream_t)stream);
}
