// Flash-attention core on the 5th-generation tensor cores (tcgen05 + TMEM).
//
// A work item is 256 query rows of one head, as two 128-row tiles (Q0, Q1)
// that take turns on the tensor core while the other tile's softmax runs on
// the CUDA cores. The kernel is persistent: at most one CTA per SM loops over
// items, and the next item's Q load and first S = Q K^T overlap the current
// item's last softmax and output (Q is double-buffered; O's TMEM columns are
// handed back by the epilogue).
// 352 threads, warp-specialised:
//   warps 0..3  softmax for Q0, warps 4..7 softmax for Q1: thread = one query
//               row = one TMEM lane (warp % 4 selects the lane quarter).
//   warp 8      TMA producer: Q0/Q1 per item, then 128-key tiles of K and
//               V through two 3-stage rings (128-byte swizzle, read in place
//               from the projection output through 3-D maps [nb][t][columns]);
//               K of tile j+1 is fetched before V of tile j.
//   warps 9, 10 issue the MMAs of tile 0 / tile 1 from one elected thread
//               each (warp 9 also allocates TMEM):
//                 S_i = Q_i K_j^T   (M=128, N=128, K=64), A and B in smem
//                 O_i += P_i V_j    (M=128, N=64,  K=128), A (P) in TMEM,
//                                   B (V) in smem as an MN-major operand
//               S_i(j+1) is issued as soon as the softmax has read S_i(j),
//               so the next scores are ready when the softmax needs them;
//               with one issuing warp per tile neither tile's pipeline waits
//               for the other's softmax.
// TMEM columns (512): S0 [0,128), S1 [128,256), O0 [256,320), O1 [320,384),
// P0 [384,448), P1 [448,512) (P: bf16/f16 pairs, one row per lane).
// Keeping P in TMEM spares shared memory the P stores and the MMA's P reads,
// which on B200 share the 128 B/clk per SM that the S MMAs need.
//
// Online softmax (log2 domain, scale folded into one FMA before the
// exponential): each thread owns a whole row, so row max and row sum need no
// shuffles; both are computed as trees of independent partial results with
// the 2-wide fp32 instructions of sm_100. The running max is only moved (and
// O rescaled in TMEM) when the new tile's max exceeds it by more than 2^8;
// otherwise P entries up to 256 are kept, which the fp32 accumulators absorb,
// and the final division by the row sum cancels the stale scale.
//
// Exponentials: ex2.approx on the special-function unit, and for NPOLY of
// every 4 column pairs a polynomial on the FMA pipe (rint range reduction,
// 2^f on [-1/2, 1/2] by a degree-3 fit with 7.5e-5 relative error, made by
// fit_exp2_poly.py), which spreads the work over both pipes.
//
// Causal (top-left aligned): Q0 stops one key tile before Q1; on tiles that
// cross the diagonal, 32-key chunks that no row of a warp attends are not
// exponentiated. The output is normalised, staged in shared memory and
// written by one TMA store per warp (rows past tq are clipped).
//
// Every wait is bounded; on a timeout the CTA records DEV_ERR_ATTN_TIMEOUT,
// stops issuing, lets its copies and MMAs in flight finish and frees TMEM.
//
// Replaces the scaled_dot_product_attention call of
// wide_compiler/core/primitives/wide_attention.py:217-231 for head_dim 64.
#include <algorithm>
#include <cstring>
#include <numeric>

#include "attention.cuh"
#include "sm100_ptx.cuh"

namespace widek {
namespace {

using namespace sm100;

constexpr int kQT = 128;        // query rows per tile
constexpr int kKT = 128;        // keys per tile
constexpr int kHD = 64;         // head dim
constexpr int kThreads = 352;
constexpr int kTmaWarp = 8;
constexpr int kMmaWarp = 9;    // and 10: one MMA warp per query tile
constexpr uint32_t kTmemCols = 512;
constexpr float kRescaleLog2 = 8.f;

constexpr int kStages = 3;      // K ring and V ring depth

struct Smem {
    static constexpr uint32_t Q_BYTES = kQT * kHD * 2;      // 16 KB
    static constexpr uint32_t KV_BYTES = kKT * kHD * 2;     // 16 KB
    static constexpr uint32_t OFF_Q = 0;                    // [2 item buffers][2 tiles]
    static constexpr uint32_t OFF_K = OFF_Q + 4 * Q_BYTES;  // [kStages]
    static constexpr uint32_t OFF_V = OFF_K + kStages * KV_BYTES;
    static constexpr uint32_t OFF_OUT = OFF_V + kStages * KV_BYTES;   // [2 tiles] output staging
    static constexpr uint32_t OFF_BAR = OFF_OUT + 2 * Q_BYTES;
    // q_full[2], q_empty[2], k_full[S], k_empty[S], v_full[S], v_empty[S],
    // s_full[2], s_free[2], p_full[2], o_full[2], o_free[2], done[2]
    static constexpr uint32_t NBAR = 4 + 4 * kStages + 12;
    static constexpr uint32_t TOTAL = 1024 + OFF_BAR + NBAR * 8 + 16;
};
static_assert(Smem::TOTAL <= 232448, "attention smem over the per-CTA limit");

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// 2^x for two values on the FMA/ALU pipes. x = n + f with n = rint(x) (by
// adding and subtracting 1.5 * 2^23), 2^f from a degree-3 polynomial on
// [-1/2, 1/2], times 2^n built in the exponent field. x is clamped at -127,
// where 2^n is built as exactly +0, so masked scores (-inf) give exactly 0;
// results are never negative. Valid for x <= 127.
__device__ __forceinline__ float2 exp2_poly2(float2 x) {
    constexpr float kMagic = 12582912.f;   // 1.5 * 2^23
    x.x = fmaxf(x.x, -127.f);
    x.y = fmaxf(x.y, -127.f);
    const float2 t = __fadd2_rn(x, make_float2(kMagic, kMagic));
    const float2 n = __fadd2_rn(t, make_float2(-kMagic, -kMagic));
    const float2 f = __ffma2_rn(n, make_float2(-1.f, -1.f), x);
    float2 p = __ffma2_rn(make_float2(0.0551716648f, 0.0551716648f), f, make_float2(0.242611125f, 0.242611125f));
    p = __ffma2_rn(p, f, make_float2(0.693260968f, 0.693260968f));
    p = __ffma2_rn(p, f, make_float2(0.999928057f, 0.999928057f));
    // The low bits of t hold n (two's complement): (n << 23) + bits(1.0f) is
    // the float 2^n for n >= -126 and +0 for n = -127 (the 1.5 * 2^23 part of
    // t shifts out).
    const float2 two_n = make_float2(__int_as_float((__float_as_int(t.x) << 23) + 0x3F800000),
                                     __int_as_float((__float_as_int(t.y) << 23) + 0x3F800000));
    return __fmul2_rn(p, two_n);
}

__device__ __forceinline__ float max3(float a, float b, float c) {
    float r;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    return r;
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

// 32 lanes x 32 columns of fp32 into v[0..31] of each thread.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
    uint32_t r[32];
    tmem_ld_32x32b_x32(taddr, r);
#pragma unroll
    for (int e = 0; e < 32; ++e) v[e] = __uint_as_float(r[e]);
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

// S = Q K^T for one 128-row tile: 4 MMAs over the 64-wide head dim. The
// descriptors are formed once and advanced by constants (the start-address
// field counts 16-byte units and smem addresses stay below 2^18, so the add
// never carries out of the field): the issuing thread's work between MMAs
// is what limits small MMAs.
__device__ __forceinline__ void issue_qk(uint32_t d_tmem, uint64_t q_desc, uint64_t k_desc, uint32_t idesc) {
#pragma unroll
    for (int kk = 0; kk < kHD / 16; ++kk) umma_f16_ss(d_tmem, q_desc + 2 * kk, k_desc + 2 * kk, idesc, kk != 0);
}
// O (+)= P V: 8 MMAs over the 128 keys; P from TMEM (8 columns of packed
// pairs per 16 keys), V MN-major with 16 key rows (2 KB) per MMA.
__device__ __forceinline__ void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void issue_pv(uint32_t d_tmem, uint32_t t_p, uint64_t v_desc, uint32_t idesc, bool accum) {
#pragma unroll
    for (int kk = 0; kk < kKT / 16; ++kk)
        umma_f16_ts(d_tmem, t_p + kk * 8, v_desc + (uint64_t)kk * (16 * 128 / 16), idesc, accum || kk != 0);
}

// Work item w -> (batch*head index, query block of 256 rows): the query
// blocks of a head are adjacent (they share K/V through L2), the one with the
// most keys first. CTAs take items blockIdx.x, + gridDim.x, ...; the host
// picks a grid size coprime to the number of query blocks, so that each CTA
// cycles through all query-block classes (balanced work) while the items in
// flight at any time cover few heads (L2 reuse of their K/V).
__device__ __forceinline__ void item_of(int w, int nqb, int& bh, int& qb) {
    bh = w / nqb;
    qb = nqb - 1 - w % nqb;
}

// Explicit attention mask (wide_attention.py:223-228 passes attn_mask to
// scaled_dot_product_attention): element (b, h, q, k) at
// b*sb + h*sh + q*sq + k*sk of a bool (uint8: nonzero = attend) or additive
// (T or fp32) tensor. The softmax works on raw scores s (scaled into the
// log2 domain by sl2 = scale*log2(e) later), so an additive value m enters
// as s + m / scale and a masked-out key as s = -inf.
struct AttnMaskArgs {
    const void* p;
    int kind;                   // 1 bool, 2 additive T, 3 additive fp32
    int vec;                    // 16-byte loads along the keys: unit key stride, 16-byte aligned rows, tk % vector == 0
    int64_t sb, sh, sq, sk;
    float inv_scale;
};

template <typename T>
__device__ __forceinline__ void attn_apply_mask(const AttnMaskArgs& mk, int b, int h, int qrow, int kbase, int tk,
                                                float (&s)[kKT]) {
    const int64_t base = (int64_t)b * mk.sb + (int64_t)h * mk.sh + (int64_t)qrow * mk.sq;
    if (mk.kind == 1) {
        const uint8_t* m = static_cast<const uint8_t*>(mk.p) + base;
        if (mk.vec) {
#pragma unroll
            for (int g = 0; g < kKT / 16; ++g) {
                if (kbase + 16 * g < tk) {
                    const uint4 v = __ldg(reinterpret_cast<const uint4*>(m + kbase + 16 * g));
                    const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                    for (int e = 0; e < 16; ++e)
                        if (((w4[e >> 2] >> (8 * (e & 3))) & 0xffu) == 0u) s[16 * g + e] = -INFINITY;
                }
            }
        } else {
#pragma unroll
            for (int c = 0; c < kKT; ++c)
                if (kbase + c < tk && m[(int64_t)(kbase + c) * mk.sk] == 0) s[c] = -INFINITY;
        }
        return;
    }
    if (mk.kind == 2) {
        const T* m = static_cast<const T*>(mk.p) + base;
        if (mk.vec) {
#pragma unroll
            for (int g = 0; g < kKT / 8; ++g) {
                if (kbase + 8 * g < tk) {
                    float f[8];
                    load16<T>(m + kbase + 8 * g, f);
#pragma unroll
                    for (int e = 0; e < 8; ++e) s[8 * g + e] = fmaf(f[e], mk.inv_scale, s[8 * g + e]);
                }
            }
        } else {
#pragma unroll
            for (int c = 0; c < kKT; ++c)
                if (kbase + c < tk) s[c] = fmaf(to_f<T>(m[(int64_t)(kbase + c) * mk.sk]), mk.inv_scale, s[c]);
        }
        return;
    }
    const float* m = static_cast<const float*>(mk.p) + base;
    if (mk.vec) {
#pragma unroll
        for (int g = 0; g < kKT / 4; ++g) {
            if (kbase + 4 * g < tk) {
                const float4 f = __ldg(reinterpret_cast<const float4*>(m + kbase + 4 * g));
                s[4 * g] = fmaf(f.x, mk.inv_scale, s[4 * g]);
                s[4 * g + 1] = fmaf(f.y, mk.inv_scale, s[4 * g + 1]);
                s[4 * g + 2] = fmaf(f.z, mk.inv_scale, s[4 * g + 2]);
                s[4 * g + 3] = fmaf(f.w, mk.inv_scale, s[4 * g + 3]);
            }
        }
    } else {
#pragma unroll
        for (int c = 0; c < kKT; ++c)
            if (kbase + c < tk) s[c] = fmaf(m[(int64_t)(kbase + c) * mk.sk], mk.inv_scale, s[c]);
    }
}

template <typename T, int NPOLY, bool MASKED>
__global__ void __launch_bounds__(kThreads, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                   const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_o, int heads,
                   int items, int tq, int tk, int causal, float sl2, AttnMaskArgs mk, int* err) {
    constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
    constexpr uint32_t IDESC_S = idesc_f16(kQT, kKT, kBf16);
    constexpr uint32_t IDESC_PV = idesc_f16(kQT, kHD, kBf16) | (1u << 16);   // B (V) MN-major

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sQ = smem + Smem::OFF_Q;       // [item buffer][tile]
    uint8_t* sK = smem + Smem::OFF_K;
    uint8_t* sV = smem + Smem::OFF_V;
    uint8_t* sOut = smem + Smem::OFF_OUT;   // [tile]
    uint64_t* q_full = reinterpret_cast<uint64_t*>(smem + Smem::OFF_BAR);   // [2 item buffers]
    uint64_t* q_empty = q_full + 2;           // [2 item buffers]
    uint64_t* k_full = q_empty + 2;           // [kStages]
    uint64_t* k_empty = k_full + kStages;     // [kStages]
    uint64_t* v_full = k_empty + kStages;     // [kStages]
    uint64_t* v_empty = v_full + kStages;     // [kStages]
    uint64_t* s_full = v_empty + kStages;     // [2 tiles]
    uint64_t* s_free = s_full + 2;            // [2 tiles]
    uint64_t* p_full = s_free + 2;            // [2 tiles]
    uint64_t* o_full = p_full + 2;            // [2 tiles]
    uint64_t* o_free = o_full + 2;            // [2 tiles]
    uint64_t* done = o_free + 2;              // [2 MMA warps]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 2);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int nqb = (tq + 2 * kQT - 1) / (2 * kQT);

    // Per-item geometry, identical in every role: query rows and key tiles
    // of the two query tiles.
    auto geometry = [&](int qb, int (&rows)[2], int (&ntile)[2]) {
        const int q0 = qb * 2 * kQT;
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            rows[i] = max(0, min(kQT, tq - (q0 + i * kQT)));
            const int klim = causal ? min(tk, q0 + i * kQT + rows[i]) : tk;
            ntile[i] = rows[i] > 0 ? (klim + kKT - 1) / kKT : 0;
        }
    };

    if (threadIdx.x == 0) {
        for (int u = 0; u < 2; ++u) {
            mbar_init(&q_full[u], 1);
            mbar_init(&q_empty[u], 2);
        }
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&k_full[s], 1);
            mbar_init(&k_empty[s], 2);
            mbar_init(&v_full[s], 1);
            mbar_init(&v_empty[s], 2);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&s_full[i], 1);
            mbar_init(&s_free[i], 128);
            mbar_init(&p_full[i], 128);
            mbar_init(&o_full[i], 1);
            mbar_init(&o_free[i], 128);
            mbar_init(&done[i], 1);
        }
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
        // TMA producer. Per item: Q0/Q1 into item buffer u % 2 (once the
        // item two back has released it), then K(0), and per key tile j:
        // K(j+1), V(j). The K and V rings run on across items.
        // ------------------------------------------------------------------
        const uint64_t pol = l2_policy_evict_normal();
        int kc = 0, vc = 0, u = 0;      // K loads, V loads, items (running)
        bool ok = true;
        for (int w = blockIdx.x; w < items && ok; w += gridDim.x) {
            int bh, qb;
            item_of(w, nqb, bh, qb);
            const int b = bh / heads, col = (bh % heads) * kHD, q0 = qb * 2 * kQT;
            int rows[2], ntile[2];
            geometry(qb, rows, ntile);
            const int nmax = max(ntile[0], ntile[1]);
            const int qs = u & 1;
            if (!mbar_wait_warp(&q_empty[qs], (uint32_t)(((u >> 1) & 1) ^ 1), abort_flag)) { ok = false; break; }
            if (lane == 0) {
                uint32_t qbytes = 0;
                for (int i = 0; i < 2; ++i) qbytes += rows[i] > 0 ? Smem::Q_BYTES : 0;
                mbar_arrive_expect_tx(&q_full[qs], qbytes);
                for (int i = 0; i < 2; ++i)
                    if (rows[i] > 0)
                        tma_load_3d(sQ + (2 * qs + i) * Smem::Q_BYTES, &tm_q, &q_full[qs], col, q0 + i * kQT, b, pol);
            }
            __syncwarp();
            ++u;
            for (int step = 0; step <= nmax && ok; ++step) {
                // step 0 loads K(0); step j+1 loads K(j+1) (if any) and V(j).
                if (step < nmax) {
                    const int s = kc % kStages;
                    if (!mbar_wait_warp(&k_empty[s], (uint32_t)(((kc / kStages) & 1) ^ 1), abort_flag)) {
                        ok = false;
                        break;
                    }
                    if (lane == 0) {
                        mbar_arrive_expect_tx(&k_full[s], Smem::KV_BYTES);
                        tma_load_3d(sK + s * Smem::KV_BYTES, &tm_k, &k_full[s], col, step * kKT, b, pol);
                    }
                    __syncwarp();
                    ++kc;
                }
                if (step >= 1) {
                    const int s = vc % kStages;
                    if (!mbar_wait_warp(&v_empty[s], (uint32_t)(((vc / kStages) & 1) ^ 1), abort_flag)) {
                        ok = false;
                        break;
                    }
                    if (lane == 0) {
                        mbar_arrive_expect_tx(&v_full[s], Smem::KV_BYTES);
                        tma_load_3d(sV + s * Smem::KV_BYTES, &tm_v, &v_full[s], col, (step - 1) * kKT, b, pol);
                    }
                    __syncwarp();
                    ++vc;
                }
            }
        }
        if (!ok) {
            *abort_flag = 1;
            raise_device_error(err, DEV_ERR_ATTN_TIMEOUT);
        }
        if (!ok || *abort_flag) {
            // Copies still in flight land before the CTA's smem is released.
            const volatile int never = 0;
            for (int t = 1; t <= 2; ++t)
                if (u - t >= 0) mbar_wait(&q_full[(u - t) & 1], (uint32_t)(((u - t) >> 1) & 1), &never);
            for (int t = 1; t <= kStages; ++t) {
                const int jk = kc - t, jv = vc - t;
                if (jk >= 0) mbar_wait(&k_full[jk % kStages], (uint32_t)((jk / kStages) & 1), &never);
                if (jv >= 0) mbar_wait(&v_full[jv % kStages], (uint32_t)((jv / kStages) & 1), &never);
            }
        }
    } else if (warp >= kMmaWarp) {
        // ------------------------------------------------------------------
        // MMA issuers: warp 9 + i serves query tile i, so that each tile's
        // S(j+1) follows its own softmax without waiting for the other
        // tile. Both warps commit every K/V stage and Q buffer (count-2
        // "empty" barriers), also those their tile does not use; each waits
        // for a buffer's "full" barrier before committing its "empty" one,
        // so that its arrival always lands on the phase of that load.
        // The first S of an item only needs the previous S read (s_free), so
        // it overlaps the previous item's last softmax and epilogue; its
        // first P V (which overwrites O) waits for that epilogue (o_free).
        // ------------------------------------------------------------------
        const int i = warp - kMmaWarp;
        const uint64_t k_desc0 = sdesc_kmajor_sw128(smem_addr(sK));
        const uint64_t v_desc0 = sdesc_mnmajor_sw128(smem_addr(sV));
        const uint32_t dS = tmem_base + i * kKT, dO = tmem_base + 2 * kKT + i * kHD;
        const uint32_t tP = tmem_base + 2 * kKT + 2 * kHD + i * (kKT / 2);
        int kc = 0, vc = 0, u = 0;      // running K tiles, V tiles, items
        int g = 0;                      // running S/P/O tile index of this query tile
        int ue = 0;                     // items of this query tile with output (epilogues)
        bool ok = true;
        for (int w = blockIdx.x; w < items && ok; w += gridDim.x) {
            int bh, qb;
            item_of(w, nqb, bh, qb);
            int rows[2], ntile[2];
            geometry(qb, rows, ntile);
            const int n = ntile[i];
            const int nmax = max(ntile[0], ntile[1]);
            const int qs = u & 1;
            const uint64_t q_desc = sdesc_kmajor_sw128(smem_addr(sQ) + (2 * qs + i) * Smem::Q_BYTES);
            ok = mbar_wait_warp(&q_full[qs], (uint32_t)((u >> 1) & 1), abort_flag);
            for (int j = -1; j < nmax && ok; ++j) {
                // S(j+1) of this tile, then P V for tile j.
                if (j + 1 < nmax) {
                    const int s1 = kc % kStages;
                    ok = mbar_wait_warp(&k_full[s1], (uint32_t)((kc / kStages) & 1), abort_flag);
                    if (!ok) break;
                    if (j + 1 < n) {
                        const int t = g + j + 1;   // running index of this S
                        if (t > 0) ok = mbar_wait_warp(&s_free[i], (uint32_t)((t - 1) & 1), abort_flag);
                        if (!ok) break;
                        tc_fence_after();
                        if (lane == 0) {
                            issue_qk(dS, q_desc, k_desc0 + (uint64_t)((s1 * Smem::KV_BYTES) >> 4), IDESC_S);
                            umma_commit(&s_full[i]);
                        }
                    }
                    if (lane == 0) umma_commit(&k_empty[s1]);
                    __syncwarp();
                    ++kc;
                }
                if (j >= 0) {
                    const int sv = vc % kStages;
                    ok = mbar_wait_warp(&v_full[sv], (uint32_t)((vc / kStages) & 1), abort_flag);
                    if (!ok) break;
                    if (j < n) {
                        if (j == 0 && ue > 0)
                            ok = mbar_wait_warp(&o_free[i], (uint32_t)((ue - 1) & 1), abort_flag);
                        if (ok) ok = mbar_wait_warp(&p_full[i], (uint32_t)((g + j) & 1), abort_flag);
                        if (!ok) break;
                        tc_fence_after();
                        if (lane == 0) {
                            issue_pv(dO, tP, v_desc0 + (uint64_t)((sv * Smem::KV_BYTES) >> 4), IDESC_PV, j > 0);
                            umma_commit(&o_full[i]);
                        }
                    }
                    if (lane == 0) umma_commit(&v_empty[sv]);
                    __syncwarp();
                    ++vc;
                }
            }
            if (!ok) break;
            // Q buffer qs is free once this warp's MMAs of the item are done.
            if (lane == 0) umma_commit(&q_empty[qs]);
            __syncwarp();
            ++u;
            if (n > 0) {
                g += n;
                ++ue;
            }
        }
        if (!ok) {
            *abort_flag = 1;
            raise_device_error(err, DEV_ERR_ATTN_TIMEOUT);
        }
        // Every MMA issued by this thread completes before TMEM is freed.
        if (lane == 0) umma_commit(&done[i]);
        __syncwarp();
        const volatile int never = 0;
        mbar_wait(&done[i], 0, &never);
    } else {
        // ------------------------------------------------------------------
        // Softmax: warps 4i..4i+3 own query tile i, one row per thread.
        // ------------------------------------------------------------------
        const int i = warp >> 2;
        const int qd = warp & 3;
        const int r = qd * 32 + lane;                 // row within the tile = TMEM lane
        const uint32_t lane_off = (uint32_t)(qd * 32) << 16;
        const uint32_t tS = tmem_base + lane_off + i * kKT;
        const uint32_t tO = tmem_base + lane_off + 2 * kKT + i * kHD;
        const uint32_t tP = tmem_base + lane_off + 2 * kKT + 2 * kHD + i * (kKT / 2);
        uint8_t* stage = sOut + i * Smem::Q_BYTES + qd * 32 * 128;   // this warp's 32 output rows
        const float2 sl2x2 = make_float2(sl2, sl2);
        int g = 0;                      // running S/P/O tile index of this query tile
        bool ok = true;
        for (int w = blockIdx.x; w < items && ok; w += gridDim.x) {
            int bh, qb;
            item_of(w, nqb, bh, qb);
            int rows[2], ntile[2];
            geometry(qb, rows, ntile);
            const int n = ntile[i];
            if (n == 0) continue;
            const int q0 = qb * 2 * kQT;
            const int qrow = q0 + i * kQT + r;
            const int wrow0 = q0 + i * kQT + qd * 32;     // first row of this warp
            float m_used = -INFINITY;   // running max, log2 domain (scaled)
            float2 lsum[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) lsum[e] = make_float2(0.f, 0.f);
            for (int j = 0; j < n; ++j) {
                const int t = g + j;
                if (!mbar_wait_warp(&s_full[i], (uint32_t)(t & 1), abort_flag)) { ok = false; break; }
                tc_fence_after();
                const int kbase = j * kKT;
                // Keys of this tile attended by at least one row of the warp.
                int kvalid = min(kKT, tk - kbase);
                if (causal) kvalid = min(kvalid, wrow0 + 32 - kbase);
                const int nch = (max(kvalid, 0) + 31) >> 5;   // 32-key chunks to process (warp-uniform)
                // All four chunks are read (a conditional read costs
                // registers); the chunks no row attends are skipped below.
                float s[kKT];
#pragma unroll
                for (int cc = 0; cc < 4; ++cc) tmem_ld32(tS + cc * 32, s + cc * 32);
                tmem_ld_wait();
                tc_fence_before();
                mbar_arrive(&s_free[i]);

                if constexpr (MASKED) {
                    if (qrow < tq) attn_apply_mask<T>(mk, bh / heads, bh % heads, qrow, kbase, tk, s);
                }
                const bool need_mask = (kbase + kKT > tk) || (causal && kbase + kKT - 1 > wrow0);
                if (need_mask) {
                    const int lim = causal ? min(tk - kbase, qrow - kbase + 1) : tk - kbase;
#pragma unroll
                    for (int c = 0; c < kKT; ++c)
                        if (c >= lim) s[c] = -INFINITY;
                }
                // Row max: four independent 3-input max chains per chunk.
                float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
                for (int cc = 0; cc < 4; ++cc) {
                    if (cc < nch) {
#pragma unroll
                        for (int c = cc * 32; c < cc * 32 + 32; c += 8) {
                            mx4[0] = max3(mx4[0], s[c], s[c + 1]);
                            mx4[1] = max3(mx4[1], s[c + 2], s[c + 3]);
                            mx4[2] = max3(mx4[2], s[c + 4], s[c + 5]);
                            mx4[3] = max3(mx4[3], s[c + 6], s[c + 7]);
                        }
                    }
                }
                const float m_tile = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3])) * sl2;
                const float m_new = fmaxf(m_used, m_tile);
                const bool rescale = m_new > m_used + kRescaleLog2;
                float alpha = 1.f;
                if (rescale) {
                    alpha = ex2(m_used - m_new);
                    m_used = m_new;
                }
                const float neg_m = (m_used == -INFINITY) ? 0.f : -m_used;
                const float2 negm2 = make_float2(neg_m, neg_m);
                const float2 alpha2 = make_float2(alpha, alpha);
#pragma unroll
                for (int e = 0; e < 4; ++e) lsum[e] = __fmul2_rn(lsum[e], alpha2);
                uint32_t pk[kKT / 2];
#pragma unroll
                for (int cc = 0; cc < 4; ++cc) {
                    if (cc < nch) {
#pragma unroll
                        for (int c = cc * 32; c < cc * 32 + 32; c += 2) {
                            const float2 x = __ffma2_rn(make_float2(s[c], s[c + 1]), sl2x2, negm2);
                            float2 p;
                            if (((c >> 1) & 3) < NPOLY) {
                                p = exp2_poly2(x);
                            } else {
                                p.x = ex2(x.x);
                                p.y = ex2(x.y);
                            }
                            lsum[(c >> 1) & 3] = __fadd2_rn(lsum[(c >> 1) & 3], p);
                            pk[c >> 1] = pack2<T>(p.x, p.y);
                        }
                    } else {
#pragma unroll
                        for (int c = cc * 32; c < cc * 32 + 32; c += 2) pk[c >> 1] = 0u;
                    }
                }
                if (j > 0) {
                    // P_i(j-1) V has finished: P's TMEM columns are free and
                    // O holds the sum through tile j-1 (rescaled here if
                    // needed before P_i(j) V joins it). For j = 0 the previous
                    // item's epilogue already waited for its last P V.
                    if (!mbar_wait_warp(&o_full[i], (uint32_t)((t - 1) & 1), abort_flag)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    if (__any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll
                        for (int c = 0; c < kHD; c += 32) {
                            uint32_t o[32];
                            tmem_ld_32x32b_x32(tO + c, o);
                            tmem_ld_wait();
#pragma unroll
                            for (int e = 0; e < 32; e += 2) {
                                const float2 v = __fmul2_rn(
                                    make_float2(__uint_as_float(o[e]), __uint_as_float(o[e + 1])), alpha2);
                                o[e] = __float_as_uint(v.x);
                                o[e + 1] = __float_as_uint(v.y);
                            }
                            tmem_st_32x32b_x32(tO + c, o);
                        }
                    }
                }
                tmem_st_32x32b_x32(tP, *reinterpret_cast<const uint32_t(*)[32]>(pk));
                tmem_st_32x32b_x32(tP + 32, *reinterpret_cast<const uint32_t(*)[32]>(pk + 32));
                tmem_st_wait();
                tc_fence_before();
                mbar_arrive(&p_full[i]);
            }
            if (!ok) break;
            // Epilogue: O after the item's last P V; O's columns are handed
            // back (o_free) as soon as they are in registers.
            if (!mbar_wait_warp(&o_full[i], (uint32_t)((g + n - 1) & 1), abort_flag)) {
                ok = false;
                break;
            }
            tc_fence_after();
            float o[kHD];
            tmem_ld32(tO, o);
            tmem_ld32(tO + 32, o + 32);
            tmem_ld_wait();
            tc_fence_before();
            mbar_arrive(&o_free[i]);
            g += n;
            if (wrow0 < tq) {
                const float2 l2 = __fadd2_rn(__fadd2_rn(lsum[0], lsum[1]), __fadd2_rn(lsum[2], lsum[3]));
                const float l = l2.x + l2.y;
                const float inv = l > 0.f ? 1.f / l : 0.f;
                // This warp's 32 rows x 64 columns, 128-byte swizzled as the
                // TMA store reads them, once the previous store has read the
                // staging slice; rows past tq are clipped by the store.
                if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
                __syncwarp();
#pragma unroll
                for (int u8 = 0; u8 < 8; ++u8) {
                    uint32_t wv[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const int c = u8 * 8 + e * 2;
                        wv[e] = pack2<T>(o[c] * inv, o[c + 1] * inv);
                    }
                    *reinterpret_cast<uint4*>(stage + lane * 128 + ((u8 ^ (lane & 7)) << 4)) =
                        make_uint4(wv[0], wv[1], wv[2], wv[3]);
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    tma_store_3d(&tm_o, stage, (bh % heads) * kHD, wrow0, bh / heads);
                    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
                }
                __syncwarp();
            }
        }
        if (!ok) {
            *abort_flag = 1;
            raise_device_error(err, DEV_ERR_ATTN_TIMEOUT);
        }
        if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
        __syncwarp();
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

template <typename T, int NPOLY, bool MASKED = false>
int launch_tc(const CUtensorMap& q, const CUtensorMap& k, const CUtensorMap& v, const CUtensorMap& o,
              const AttnArgs& a, cudaStream_t st) {
    auto kern = attn_tc_kernel<T, NPOLY, MASKED>;
    static bool attr_done[64] = {false};
    const int dev = current_device();
    if (dev >= 0 && dev < 64 && !attr_done[dev]) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Smem::TOTAL) !=
            cudaSuccess)
            return set_error(WIDEK_ERR_CUDA, "attention: cannot reserve %u bytes of shared memory", Smem::TOTAL);
        attr_done[dev] = true;
    }
    // Persistent: at most one CTA per SM, looping over items; the grid size
    // is the largest one not above the SM count that is coprime to the
    // number of query blocks per head (see item_of).
    const int64_t nbh = (int64_t)a.nb * a.heads;
    const int64_t nqb = (a.tq + 2 * kQT - 1) / (2 * kQT);
    const int64_t items = nbh * nqb;
    if (items > 0x7fffffff) return WIDEK_ERR_UNSUPPORTED;
    int64_t grid = std::min<int64_t>(items, std::max(1, sm_count(dev)));
    while (grid > 1 && std::gcd(grid, nqb) != 1) --grid;
    const float sl2 = a.scale * 1.4426950408889634f;
    AttnMaskArgs mk{};
    if (MASKED) {
        const int64_t es = a.mask_kind == 1 ? 1 : (a.mask_kind == 2 ? (int64_t)sizeof(T) : 4);
        const int64_t vlen = 16 / es;
        mk = AttnMaskArgs{a.mask, a.mask_kind, 0, a.ms_b, a.ms_h, a.ms_q, a.ms_k, 1.f / a.scale};
        mk.vec = a.ms_k == 1 && aligned16(a.mask) && (a.ms_q * es) % 16 == 0 && (a.ms_h * es) % 16 == 0 &&
                 (a.ms_b * es) % 16 == 0 && a.tk % vlen == 0;
    }
    kern<<<(unsigned)grid, kThreads, Smem::TOTAL, st>>>(q, k, v, o, a.heads, (int)items, a.tq, a.tk, a.causal,
                                                        sl2, mk, device_error_ptr());
    return check_launch("widek_attention_fwd (tcgen05)");
}

}  // namespace

template <typename T>
int launch_attn_tc(const AttnArgs& a, cudaStream_t st) {
    if constexpr (std::is_same<T, float>::value) {
        return WIDEK_ERR_UNSUPPORTED;
    } else {
        const int64_t width = (int64_t)a.heads * kHD;
        const bool fits = a.dh == kHD && a.mask_kind >= 0 && a.mask_kind <= 3 && (a.mask_kind == 0 || a.mask) &&
                          a.scale > 0.f && a.tk > 0 &&
                          a.sq % 8 == 0 && a.sk % 8 == 0 && a.sv % 8 == 0 && a.so % 8 == 0 &&
                          a.sq >= width && a.sk >= width && a.sv >= width && a.so >= width &&
                          aligned16(a.q) && aligned16(a.k) && aligned16(a.v) && aligned16(a.o);
        if (!fits) return WIDEK_ERR_UNSUPPORTED;
        CUtensorMap tq_, tk_, tv_, to_;
        int rc = rows_map<T>(&tq_, a.q, a.sq, a.tq, a.nb, a.heads, kQT);
        if (!rc) rc = rows_map<T>(&tk_, a.k, a.sk, a.tk, a.nb, a.heads, kKT);
        if (!rc) rc = rows_map<T>(&tv_, a.v, a.sv, a.tk, a.nb, a.heads, kKT);
        if (!rc) rc = rows_map<T>(&to_, a.o, a.so, a.tq, a.nb, a.heads, 32);
        if (rc) return rc;
        if (a.mask_kind != 0) return launch_tc<T, 1, true>(tq_, tk_, tv_, to_, a, st);
        switch (attn_poly_pairs()) {
            case 0: return launch_tc<T, 0>(tq_, tk_, tv_, to_, a, st);
            case 2: return launch_tc<T, 2>(tq_, tk_, tv_, to_, a, st);
            default: return launch_tc<T, 1>(tq_, tk_, tv_, to_, a, st);
        }
    }
}

template int launch_attn_tc<float>(const AttnArgs&, cudaStream_t);
template int launch_attn_tc<__nv_bfloat16>(const AttnArgs&, cudaStream_t);
template int launch_attn_tc<__half>(const AttnArgs&, cudaStream_t);

}  // namespace widek
