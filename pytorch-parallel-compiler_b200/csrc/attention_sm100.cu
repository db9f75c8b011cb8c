// Flash-attention core on the 5th-generation tensor cores (tcgen05 + TMEM).
//
// One CTA computes 256 query rows of one head as two 128-row tiles (Q0, Q1)
// that take turns on the tensor core while the other tile's softmax runs on
// the CUDA cores. 320 threads, warp-specialised:
//   warps 0..3  softmax for Q0, warps 4..7 softmax for Q1: thread = one query
//               row = one TMEM lane (warp % 4 selects the lane quarter).
//   warp 8      TMA producer: Q0/Q1 once, then 128-key tiles of K and V
//               through a 3-stage ring (128-byte swizzle, read in place from
//               the projection output through 3-D maps [nb][t][columns]).
//   warp 9      allocates TMEM and issues the MMAs from one elected thread:
//                 S_i = Q_i K_j^T   (M=128, N=128, K=64)  -> TMEM, fp32
//                 O_i += P_i V_j    (M=128, N=64,  K=128) -> TMEM, fp32
//               P_i (bf16/f16) is written by the softmax warps into shared
//               memory in the K-major 128-byte-swizzled layout; V is used as
//               an MN-major operand straight from its TMA tile.
// TMEM columns: S0 [0,128), S1 [128,256), O0 [256,320), O1 [320,384).
//
// Online softmax (log2 domain, scale folded into one FMA before ex2): each
// thread owns a whole row, so row max and row sum need no shuffles. The
// running max is only moved (and O rescaled in TMEM) when the new tile's max
// exceeds it by more than 2^8; otherwise P entries up to 256 are kept, which
// the fp32 accumulators absorb, and the final division by the row sum
// cancels the stale scale.
//
// Causal (top-left aligned): Q0 stops one key tile before Q1; per-element
// masking only on tiles that cross the diagonal or the end of the keys. The
// output is normalised, staged in shared memory (the tile's P buffer, free by
// then) and written by one TMA store per warp (rows past tq are clipped).
//
// Every wait is bounded; on a timeout the CTA records DEV_ERR_ATTN_TIMEOUT,
// stops issuing, lets its copies and MMAs in flight finish and frees TMEM.
//
// Replaces the scaled_dot_product_attention call of
// wide_compiler/core/primitives/wide_attention.py:217-231 for head_dim 64.
#include <cstring>

#include "attention.cuh"
#include "sm100_ptx.cuh"

namespace widek {
namespace {

using namespace sm100;

constexpr int kQT = 128;        // query rows per tile
constexpr int kKT = 128;        // keys per tile
constexpr int kHD = 64;         // head dim
constexpr int kStages = 3;
constexpr int kThreads = 320;
constexpr int kTmaWarp = 8;
constexpr int kMmaWarp = 9;
constexpr uint32_t kTmemCols = 512;
constexpr float kRescaleLog2 = 8.f;

struct Smem {
    static constexpr uint32_t Q_BYTES = kQT * kHD * 2;      // 16 KB
    static constexpr uint32_t KV_BYTES = kKT * kHD * 2;     // 16 KB
    static constexpr uint32_t P_BYTES = kQT * kKT * 2;      // 32 KB: two 64-key halves of 16 KB
    static constexpr uint32_t OFF_Q = 0;
    static constexpr uint32_t OFF_K = OFF_Q + 2 * Q_BYTES;
    static constexpr uint32_t OFF_V = OFF_K + kStages * KV_BYTES;
    static constexpr uint32_t OFF_P = OFF_V + kStages * KV_BYTES;
    static constexpr uint32_t OFF_BAR = OFF_P + 2 * P_BYTES;
    // q_full, k_full[S], v_full[S], kv_empty[S], s_full[2], s_free[2], p_full[2], o_full[2], done
    static constexpr uint32_t NBAR = 1 + 3 * kStages + 8 + 1;
    static constexpr uint32_t TOTAL = 1024 + OFF_BAR + NBAR * 8 + 16;
};

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

template <typename T>
__device__ __forceinline__ uint32_t pack2(float lo, float hi);
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
}
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float lo, float hi) {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
        "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
        "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
        "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
        "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// MN-major operand tile written by TMA with 128-byte swizzling: 64 elements
// of N per 128-byte row, one row per K index, 8-row atoms 1024 bytes apart.
__device__ __forceinline__ uint64_t sdesc_mnmajor_sw128(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFF);   // start address, 16-byte units
    d |= (uint64_t)1 << 16;                   // leading byte offset: next 64-wide N block (none here)
    d |= (uint64_t)(1024 >> 4) << 32;         // stride byte offset: next 8 K rows
    d |= (uint64_t)1 << 46;                   // descriptor version for sm_100
    d |= (uint64_t)2 << 61;                   // 128-byte swizzle
    return d;
}

__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, const void* src, int c0, int c1, int c2) {
    asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(smem_addr(src)), "r"(c0), "r"(c1), "r"(c2)
                 : "memory");
}
// mbar_wait with one answer for the whole warp: a lane that gives up makes
// every lane give up, so warp-collective tcgen05 operations stay converged.
__device__ __forceinline__ bool mbar_wait_warp(uint64_t* bar, uint32_t parity, const volatile int* abort) {
    return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort));
}
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Writes 64 packed pairs (128 values of one row) into a K-major, 128-byte
// swizzled [128 rows][128 columns] tile: two 64-column halves of 16 KB, row r
// at r*128 bytes within a half, 16-byte unit u stored at unit u ^ (r % 8).
__device__ __forceinline__ void store_row_sw128(uint8_t* tile, int r, const uint32_t (&pk)[64]) {
#pragma unroll
    for (int half = 0; half < 2; ++half) {
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int base = half * 32 + u * 4;
            uint4 v = make_uint4(pk[base], pk[base + 1], pk[base + 2], pk[base + 3]);
            *reinterpret_cast<uint4*>(tile + half * 16384 + r * 128 + ((u ^ (r & 7)) << 4)) = v;
        }
    }
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                   const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_o, int heads,
                   int tq, int tk, int causal, float sl2, int* err) {
    constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
    constexpr uint32_t IDESC_S = idesc_f16(kQT, kKT, kBf16);
    constexpr uint32_t IDESC_PV = idesc_f16(kQT, kHD, kBf16) | (1u << 16);   // B (V) MN-major

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sQ = smem + Smem::OFF_Q;
    uint8_t* sK = smem + Smem::OFF_K;
    uint8_t* sV = smem + Smem::OFF_V;
    uint8_t* sP = smem + Smem::OFF_P;
    uint64_t* q_full = reinterpret_cast<uint64_t*>(smem + Smem::OFF_BAR);
    uint64_t* k_full = q_full + 1;
    uint64_t* v_full = k_full + kStages;
    uint64_t* kv_empty = v_full + kStages;
    uint64_t* s_full = kv_empty + kStages;   // [2]
    uint64_t* s_free = s_full + 2;           // [2]
    uint64_t* p_full = s_free + 2;           // [2]
    uint64_t* o_full = p_full + 2;           // [2]
    uint64_t* done = o_full + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    // Work item: CTAs of one head are adjacent (they share K/V through L2);
    // within a head the query blocks with the most keys start first.
    const int nqb = (tq + 2 * kQT - 1) / (2 * kQT);
    const int bh = blockIdx.x / nqb;
    const int qb = nqb - 1 - (int)(blockIdx.x % nqb);
    const int b = bh / heads, h = bh % heads;
    const int q0 = qb * 2 * kQT;
    int rows[2], ntile[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        rows[i] = max(0, min(kQT, tq - (q0 + i * kQT)));
        const int klim = causal ? min(tk, q0 + i * kQT + rows[i]) : tk;
        ntile[i] = rows[i] > 0 ? (klim + kKT - 1) / kKT : 0;
    }
    const int nmax = max(ntile[0], ntile[1]);

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&k_full[s], 1);
            mbar_init(&v_full[s], 1);
            mbar_init(&kv_empty[s], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&s_full[i], 1);
            mbar_init(&s_free[i], 128);
            mbar_init(&p_full[i], 128);
            mbar_init(&o_full[i], 1);
        }
        mbar_init(done, 1);
        *abort_flag = 0;
        mbar_init_fence();
    }
    if (warp == kTmaWarp && lane == 0) {
        tma_prefetch_desc(&tm_q);
        tma_prefetch_desc(&tm_k);
        tma_prefetch_desc(&tm_v);
        tma_prefetch_desc(&tm_o);
    }
    if (warp == kMmaWarp) {
        tmem_alloc(tmem_slot, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == kTmaWarp) {
        // ------------------------------------------------------------------
        // TMA producer
        // ------------------------------------------------------------------
        const uint64_t pol = l2_policy_evict_normal();
        const int col = h * kHD;
        if (lane == 0) {
            uint32_t qbytes = 0;
            for (int i = 0; i < 2; ++i) qbytes += rows[i] > 0 ? Smem::Q_BYTES : 0;
            mbar_arrive_expect_tx(q_full, qbytes);
            for (int i = 0; i < 2; ++i)
                if (rows[i] > 0) tma_load_3d(sQ + i * Smem::Q_BYTES, &tm_q, q_full, col, q0 + i * kQT, b, pol);
        }
        __syncwarp();
        int issued = 0;
        bool ok = true;
        for (int j = 0; j < nmax; ++j) {
            const int s = j % kStages;
            const uint32_t ph = (uint32_t)((j / kStages) & 1);
            if (!mbar_wait_warp(&kv_empty[s], ph ^ 1, abort_flag)) { ok = false; break; }
            if (lane == 0) {
                mbar_arrive_expect_tx(&k_full[s], Smem::KV_BYTES);
                tma_load_3d(sK + s * Smem::KV_BYTES, &tm_k, &k_full[s], col, j * kKT, b, pol);
                mbar_arrive_expect_tx(&v_full[s], Smem::KV_BYTES);
                tma_load_3d(sV + s * Smem::KV_BYTES, &tm_v, &v_full[s], col, j * kKT, b, pol);
            }
            __syncwarp();
            ++issued;
        }
        if (!ok) {
            *abort_flag = 1;
            raise_device_error(err, DEV_ERR_ATTN_TIMEOUT);
        }
        if (!ok || *abort_flag) {
            // Copies still in flight land before the CTA's smem is released.
            const volatile int never = 0;
            mbar_wait(q_full, 0, &never);
            const int inflight = issued < kStages ? issued : kStages;
            for (int t = 1; t <= inflight; ++t) {
                const int idx = issued - t;
                const uint32_t ph = (uint32_t)((idx / kStages) & 1);
                mbar_wait(&k_full[idx % kStages], ph, &never);
                mbar_wait(&v_full[idx % kStages], ph, &never);
            }
        }
    } else if (warp == kMmaWarp) {
        // ------------------------------------------------------------------
        // MMA issuer
        // ------------------------------------------------------------------
        bool ok = mbar_wait_warp(q_full, 0, abort_flag);
        const uint32_t aQ = smem_addr(sQ), aK = smem_addr(sK), aV = smem_addr(sV), aP = smem_addr(sP);
        auto issue_s = [&](int i, int s) {
            const uint32_t a0 = aQ + i * Smem::Q_BYTES, b0 = aK + s * Smem::KV_BYTES;
#pragma unroll
            for (int kk = 0; kk < kHD / 16; ++kk)
                umma_f16_ss(tmem_base + i * kKT, sdesc_kmajor_sw128(a0 + kk * 32), sdesc_kmajor_sw128(b0 + kk * 32),
                            IDESC_S, kk != 0);
            umma_commit(&s_full[i]);
        };
        auto issue_pv = [&](int i, int s, int j) {
            const uint32_t a0 = aP + i * Smem::P_BYTES, b0 = aV + s * Smem::KV_BYTES;
#pragma unroll
            for (int kk = 0; kk < kKT / 16; ++kk)
                umma_f16_ss(tmem_base + 2 * kKT + i * kHD,
                            sdesc_kmajor_sw128(a0 + (kk >> 2) * 16384 + (kk & 3) * 32),
                            sdesc_mnmajor_sw128(b0 + kk * 16 * 128), IDESC_PV, (j | kk) != 0);
            umma_commit(&o_full[i]);
        };
        if (ok && nmax > 0) {
            ok = mbar_wait_warp(&k_full[0], 0, abort_flag);
            if (ok) {
                tc_fence_after();
                if (lane == 0)
                    for (int i = 0; i < 2; ++i)
                        if (ntile[i] > 0) issue_s(i, 0);
                __syncwarp();
            }
        }
        for (int j = 0; j < nmax && ok; ++j) {
            const int s = j % kStages;
            const uint32_t ph = (uint32_t)((j / kStages) & 1);
            const int s1 = (j + 1) % kStages;
            const uint32_t ph1 = (uint32_t)(((j + 1) / kStages) & 1);
            bool k1_ready = false, v_ready = false;
            for (int i = 0; i < 2 && ok; ++i) {
                if (j + 1 < ntile[i]) {
                    // Next S of this tile as soon as its softmax has read the current one.
                    if (!k1_ready) { ok = mbar_wait_warp(&k_full[s1], ph1, abort_flag); k1_ready = true; }
                    if (ok) ok = mbar_wait_warp(&s_free[i], (uint32_t)(j & 1), abort_flag);
                    if (!ok) break;
                    tc_fence_after();
                    if (lane == 0) issue_s(i, s1);
                    __syncwarp();
                }
                if (j < ntile[i]) {
                    if (!v_ready) { ok = mbar_wait_warp(&v_full[s], ph, abort_flag); v_ready = true; }
                    if (ok) ok = mbar_wait_warp(&p_full[i], (uint32_t)(j & 1), abort_flag);
                    if (!ok) break;
                    tc_fence_after();
                    if (lane == 0) issue_pv(i, s, j);
                    __syncwarp();
                }
            }
            if (!ok) break;
            if (lane == 0) umma_commit(&kv_empty[s]);
            __syncwarp();
        }
        if (!ok) {
            *abort_flag = 1;
            raise_device_error(err, DEV_ERR_ATTN_TIMEOUT);
        }
        // Every MMA issued by this thread completes before TMEM is freed.
        if (lane == 0) umma_commit(done);
        __syncwarp();
        const volatile int never = 0;
        mbar_wait(done, 0, &never);
    } else {
        // ------------------------------------------------------------------
        // Softmax: warps 4i..4i+3 own query tile i, one row per thread.
        // ------------------------------------------------------------------
        const int i = warp >> 2;
        const int qd = warp & 3;
        const int r = qd * 32 + lane;                 // row within the tile = TMEM lane
        const int qrow = q0 + i * kQT + r;
        const int wrow0 = q0 + i * kQT + qd * 32;     // first row of this warp
        const uint32_t lane_off = (uint32_t)(qd * 32) << 16;
        const uint32_t tS = tmem_base + lane_off + i * kKT;
        const uint32_t tO = tmem_base + lane_off + 2 * kKT + i * kHD;
        uint8_t* myP = sP + i * Smem::P_BYTES;
        const int n = ntile[i];
        float m_used = -INFINITY;   // running max, log2 domain (scaled)
        float l = 0.f;
        bool ok = true;
        for (int j = 0; j < n; ++j) {
            if (!mbar_wait_warp(&s_full[i], (uint32_t)(j & 1), abort_flag)) { ok = false; break; }
            tc_fence_after();
            uint32_t su[kKT];
#pragma unroll
            for (int c = 0; c < kKT; c += 32)
                tmem_ld_32x32b_x32(tS + c, *reinterpret_cast<uint32_t(*)[32]>(su + c));
            tmem_ld_wait();
            tc_fence_before();
            mbar_arrive(&s_free[i]);

            const int kbase = j * kKT;
            const bool need_mask = (kbase + kKT > tk) || (causal && kbase + kKT - 1 > wrow0);
            float s[kKT];
#pragma unroll
            for (int c = 0; c < kKT; ++c) s[c] = __uint_as_float(su[c]);
            if (need_mask) {
                const int lim = causal ? min(tk - kbase, qrow - kbase + 1) : tk - kbase;
#pragma unroll
                for (int c = 0; c < kKT; ++c)
                    if (c >= lim) s[c] = -INFINITY;
            }
            float mx = s[0];
#pragma unroll
            for (int c = 1; c < kKT; ++c) mx = fmaxf(mx, s[c]);
            const float m_tile = mx * sl2;
            const float m_new = fmaxf(m_used, m_tile);
            const bool rescale = m_new > m_used + kRescaleLog2;
            float alpha = 1.f;
            if (rescale) {
                alpha = ex2(m_used - m_new);
                m_used = m_new;
            }
            l *= alpha;
            const float neg_m = (m_used == -INFINITY) ? 0.f : -m_used;
            uint32_t pk[kKT / 2];
#pragma unroll
            for (int c = 0; c < kKT; c += 2) {
                const float p0 = ex2(fmaf(s[c], sl2, neg_m));
                const float p1 = ex2(fmaf(s[c + 1], sl2, neg_m));
                l += p0 + p1;
                pk[c / 2] = pack2<T>(p0, p1);
            }
            if (j > 0) {
                // P_i(j-1) V has finished: the P buffer is free and O holds
                // the sum through tile j-1.
                if (!mbar_wait_warp(&o_full[i], (uint32_t)((j - 1) & 1), abort_flag)) { ok = false; break; }
                tc_fence_after();
                if (__any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll
                    for (int c = 0; c < kHD; c += 32) {
                        uint32_t o[32];
                        tmem_ld_32x32b_x32(tO + c, o);
                        tmem_ld_wait();
#pragma unroll
                        for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
                        tmem_st_32x32b_x32(tO + c, o);
                    }
                    tmem_st_wait();
                }
            }
            store_row_sw128(myP, r, pk);
            fence_proxy_async_smem();
            tc_fence_before();
            mbar_arrive(&p_full[i]);
        }
        if (!ok) {
            *abort_flag = 1;
            raise_device_error(err, DEV_ERR_ATTN_TIMEOUT);
        }
        // ok is warp-uniform here (every wait above is), and so is rows[i].
        if (ok && rows[i] > 0 && n > 0) {
            if (!mbar_wait_warp(&o_full[i], (uint32_t)((n - 1) & 1), abort_flag)) {
                *abort_flag = 1;
                raise_device_error(err, DEV_ERR_ATTN_TIMEOUT);
            } else if (wrow0 < tq) {
                tc_fence_after();
                uint32_t ou[kHD];
#pragma unroll
                for (int c = 0; c < kHD; c += 32)
                    tmem_ld_32x32b_x32(tO + c, *reinterpret_cast<uint32_t(*)[32]>(ou + c));
                tmem_ld_wait();
                const float inv = l > 0.f ? 1.f / l : 0.f;
                // Stage this warp's 32 rows x 64 columns in its own 4 KB slice
                // of the P buffer (128-byte swizzle, as the TMA store reads it)
                // and write them with one TMA store; rows past tq are clipped.
                uint8_t* stage = myP + qd * 32 * 128;
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    uint32_t w[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const int c = u * 8 + e * 2;
                        w[e] = pack2<T>(__uint_as_float(ou[c]) * inv, __uint_as_float(ou[c + 1]) * inv);
                    }
                    *reinterpret_cast<uint4*>(stage + lane * 128 + ((u ^ (lane & 7)) << 4)) =
                        make_uint4(w[0], w[1], w[2], w[3]);
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    tma_store_3d(&tm_o, stage, h * kHD, wrow0, b);
                    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
                    asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
                }
                __syncwarp();
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == kMmaWarp) {
        tc_fence_after();
        tmem_dealloc(tmem_base, kTmemCols);
    }
}

template <typename T>
CUtensorMapDataType tmap_dtype();
template <>
CUtensorMapDataType tmap_dtype<__nv_bfloat16>() { return CU_TENSOR_MAP_DATA_TYPE_BFLOAT16; }
template <>
CUtensorMapDataType tmap_dtype<__half>() { return CU_TENSOR_MAP_DATA_TYPE_FLOAT16; }

// [nb][t][heads*64] view of a row-strided operand, boxes of 64 columns x
// box_rows rows.
template <typename T>
int rows_map(CUtensorMap* m, const void* base, int64_t stride, int t, int nb, int heads, int box_rows) {
    const uint64_t dims[3] = {(uint64_t)heads * kHD, (uint64_t)t, (uint64_t)nb};
    const uint64_t strides[2] = {(uint64_t)stride * 2, (uint64_t)stride * t * 2};
    const uint32_t box[3] = {(uint32_t)kHD, (uint32_t)box_rows, 1};
    return encode_tmap_tiled(m, tmap_dtype<T>(), 3, base, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

}  // namespace

template <typename T>
int launch_attn_tc(const AttnArgs& a, cudaStream_t st) {
    if constexpr (std::is_same<T, float>::value) {
        return WIDEK_ERR_UNSUPPORTED;
    } else {
        const int64_t width = (int64_t)a.heads * kHD;
        const bool fits = a.dh == kHD && a.mask_kind == 0 && a.scale > 0.f && a.tk >= 0 &&
                          a.sq % 8 == 0 && a.sk % 8 == 0 && a.sv % 8 == 0 && a.so % 8 == 0 &&
                          a.sq >= width && a.sk >= width && a.sv >= width && a.so >= width &&
                          aligned16(a.q) && aligned16(a.k) && aligned16(a.v) && aligned16(a.o);
        if (!fits || a.tk == 0) return WIDEK_ERR_UNSUPPORTED;
        const int64_t nqb = (a.tq + 2 * kQT - 1) / (2 * kQT);
        const int64_t blocks = nqb * a.nb * (int64_t)a.heads;
        if (blocks > 0x7fffffff) return WIDEK_ERR_UNSUPPORTED;
        CUtensorMap tq_, tk_, tv_, to_;
        int rc = rows_map<T>(&tq_, a.q, a.sq, a.tq, a.nb, a.heads, kQT);
        if (!rc) rc = rows_map<T>(&tk_, a.k, a.sk, a.tk, a.nb, a.heads, kKT);
        if (!rc) rc = rows_map<T>(&tv_, a.v, a.sv, a.tk, a.nb, a.heads, kKT);
        if (!rc) rc = rows_map<T>(&to_, a.o, a.so, a.tq, a.nb, a.heads, 32);
        if (rc) return rc;
        auto kern = attn_tc_kernel<T>;
        static bool attr_done[64] = {false};
        const int dev = current_device();
        if (dev >= 0 && dev < 64 && !attr_done[dev]) {
            if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Smem::TOTAL) !=
                cudaSuccess)
                return set_error(WIDEK_ERR_CUDA, "attention: cannot reserve %u bytes of shared memory", Smem::TOTAL);
            attr_done[dev] = true;
        }
        const float sl2 = a.scale * 1.4426950408889634f;
        kern<<<(unsigned)blocks, kThreads, Smem::TOTAL, st>>>(tq_, tk_, tv_, to_, a.heads, a.tq, a.tk, a.causal,
                                                              sl2, device_error_ptr());
        return check_launch("widek_attention_fwd (tcgen05)");
    }
}

template int launch_attn_tc<float>(const AttnArgs&, cudaStream_t);
template int launch_attn_tc<__nv_bfloat16>(const AttnArgs&, cudaStream_t);
template int launch_attn_tc<__half>(const AttnArgs&, cudaStream_t);

}  // namespace widek
