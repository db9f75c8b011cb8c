// Scaled-dot-product attention core for WideAttention (N*B*H independent
// heads), flash-style: scores are never written to memory; an online softmax
// keeps a running max / sum per query row.
//
// Q, K, V are read in place from the projection outputs through row strides
// (e.g. the fused [q | k | v] projection [n, b, t, 3D] with head h at columns
// h*dh), so no head-split copies exist; the output is written directly as
// [n, b, tq, D] (head h at columns h*dh) for the output projection.
//
// bf16/f16, dh = 64, 16-byte-aligned operands with row strides a multiple of
// 8 elements (causal and/or an explicit mask of any kind): the tcgen05/TMEM
// kernel of attention_sm100.cu. Other bf16/f16 calls with dh in {64, 128}: a warp-level
// tensor-core kernel here (m16n8k16 MMA, 64 or 128 query rows per CTA,
// 64-key tiles double-buffered with cp.async, XOR-swizzled shared memory for
// conflict-free ldmatrix). fp32 and other head sizes: a CUDA-core kernel (one
// warp per query row, fp32 FFMA).
//
// Masking: causal (key index <= query index, top-left aligned as
// torch.nn.functional.scaled_dot_product_attention), and/or an explicit mask
// broadcast to [n*b, heads, tq, tk] through element strides: boolean (true =
// attend) or additive (added to the scaled scores). Rows with no attended key
// produce zeros.
#include "attention.cuh"

namespace widek {
namespace {

template <typename T>
__device__ __forceinline__ float mask_value(const AttnArgs& a, int64_t bh_b, int h, int qi, int kj, bool& keep) {
    keep = true;
    if (a.causal && kj > qi) { keep = false; return 0.f; }
    if (a.mask_kind == 0) return 0.f;
    const int64_t off = bh_b * a.ms_b + (int64_t)h * a.ms_h + (int64_t)qi * a.ms_q + (int64_t)kj * a.ms_k;
    if (a.mask_kind == 1) {
        keep = static_cast<const uint8_t*>(a.mask)[off] != 0;
        return 0.f;
    }
    if (a.mask_kind == 2) return to_f<T>(static_cast<const T*>(a.mask)[off]);
    return static_cast<const float*>(a.mask)[off];
}

// ---------------------------------------------------------------------------
// CUDA-core kernel: one warp per query row, 64-key tiles of K and V staged in
// shared memory and shared by the CTA's 4 warps (4 consecutive query rows).
// ---------------------------------------------------------------------------
constexpr int kSimtRows = 4;
constexpr int kSimtKeys = 64;

template <typename T, int DMAX>
__global__ void __launch_bounds__(32 * kSimtRows) attn_simt_kernel(AttnArgs a) {
    constexpr int DPL = DMAX / 32;      // output dims per lane
    extern __shared__ float smf[];
    float* Ks = smf;                    // [kSimtKeys][dh]
    float* Vs = Ks + kSimtKeys * a.dh;  // [kSimtKeys][dh]
    float* Qs = Vs + kSimtKeys * a.dh;  // [kSimtRows][dh]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t bh = blockIdx.y;      // nb * heads + h
    const int b = (int)(bh / a.heads), h = (int)(bh % a.heads);
    const int q0 = blockIdx.x * kSimtRows;
    const int qi = q0 + warp;
    const T* qp = static_cast<const T*>(a.q) + (int64_t)b * a.tq * a.sq + (int64_t)h * a.dh;
    const T* kp = static_cast<const T*>(a.k) + (int64_t)b * a.tk * a.sk + (int64_t)h * a.dh;
    const T* vp = static_cast<const T*>(a.v) + (int64_t)b * a.tk * a.sv + (int64_t)h * a.dh;
    for (int i = threadIdx.x; i < kSimtRows * a.dh; i += blockDim.x) {
        const int r = i / a.dh, d = i % a.dh;
        Qs[i] = (q0 + r < a.tq) ? to_f<T>(qp[(int64_t)(q0 + r) * a.sq + d]) * a.scale : 0.f;
    }
    float m = -INFINITY, l = 0.f, acc[DPL];
#pragma unroll
    for (int i = 0; i < DPL; ++i) acc[i] = 0.f;
    int kend = a.tk;
    if (a.causal) {
        const int last_q = min(q0 + kSimtRows - 1, a.tq - 1);
        kend = min(kend, last_q + 1);
    }
    for (int k0 = 0; k0 < kend; k0 += kSimtKeys) {
        __syncthreads();
        for (int i = threadIdx.x; i < kSimtKeys * a.dh; i += blockDim.x) {
            const int r = i / a.dh, d = i % a.dh;
            const bool in = k0 + r < a.tk;
            Ks[i] = in ? to_f<T>(kp[(int64_t)(k0 + r) * a.sk + d]) : 0.f;
            Vs[i] = in ? to_f<T>(vp[(int64_t)(k0 + r) * a.sv + d]) : 0.f;
        }
        __syncthreads();
        if (qi >= a.tq) continue;
        float s[2];
        bool keep[2];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int j = lane + 32 * u;
            const int kj = k0 + j;
            float dot = 0.f;
            for (int d = 0; d < a.dh; ++d) dot = fmaf(Qs[warp * a.dh + d], Ks[j * a.dh + d], dot);
            keep[u] = kj < a.tk;
            float add = 0.f;
            if (keep[u]) add = mask_value<T>(a, b, h, qi, kj, keep[u]);
            s[u] = keep[u] ? dot + add : -INFINITY;
        }
        float tmax = fmaxf(s[0], s[1]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, o));
        const float mnew = fmaxf(m, tmax);
        if (mnew == -INFINITY) continue;           // nothing attended yet
        const float alpha = expf(m - mnew);
        float p[2];
#pragma unroll
        for (int u = 0; u < 2; ++u) p[u] = keep[u] ? expf(s[u] - mnew) : 0.f;
        float psum = p[0] + p[1];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) psum += __shfl_xor_sync(0xffffffffu, psum, o);
        l = l * alpha + psum;
        m = mnew;
#pragma unroll
        for (int i = 0; i < DPL; ++i) acc[i] *= alpha;
        for (int j = 0; j < kSimtKeys; ++j) {
            const float pj = __shfl_sync(0xffffffffu, p[j >> 5], j & 31);
            if (pj == 0.f) continue;
#pragma unroll
            for (int i = 0; i < DPL; ++i) {
                const int d = lane + 32 * i;
                if (d < a.dh) acc[i] = fmaf(pj, Vs[j * a.dh + d], acc[i]);
            }
        }
    }
    if (qi >= a.tq) return;
    T* op = static_cast<T*>(a.o) + ((int64_t)b * a.tq + qi) * a.so + (int64_t)h * a.dh;
    const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll
    for (int i = 0; i < DPL; ++i) {
        const int d = lane + 32 * i;
        if (d < a.dh) op[d] = from_f<T>(acc[i] * inv);
    }
}

// ---------------------------------------------------------------------------
// Tensor-core kernel (bf16 / f16, dh = 64 or 128)
// ---------------------------------------------------------------------------
constexpr int kBN = 64;      // keys per tile (query rows per CTA: 16 per warp)

// 2^x on the special-function unit (the scores are already in the log2 domain).
__device__ __forceinline__ float fast_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

// 16-byte async copy global -> shared, zero-filled when !valid.
__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool valid) {
    const int sz = valid ? 16 : 0;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(sz) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ void ldmatrix_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                                  uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}

template <typename T>
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1);
template <>
__device__ __forceinline__ void mma16816<__nv_bfloat16>(float (&c)[4], const uint32_t (&a)[4], uint32_t b0,
                                                        uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
template <>
__device__ __forceinline__ void mma16816<__half>(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
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

// Swizzled offset (in elements) of 16-byte chunk `c` of row `r` in a tile with
// D elements per row: chunk index XOR (r % 8) spreads an 8-row ldmatrix
// access over all banks.
template <int D>
__device__ __forceinline__ int swz(int r, int c) {
    return r * D + ((c ^ (r & 7)) << 3);
}

template <typename T, int D, int NT>
__device__ __forceinline__ void load_tile(T* dst, const T* src, int64_t stride, int row0, int rows_valid,
                                          int nrows) {
    constexpr int CPR = D / 8;   // 16-byte chunks per row
    for (int i = threadIdx.x; i < nrows * CPR; i += NT) {
        const int r = i / CPR, c = i % CPR;
        const bool ok = r < rows_valid;
        const T* s = ok ? src + (int64_t)(row0 + r) * stride + c * 8 : src;
        cp_async16(dst + swz<D>(r, c), s, ok);
    }
}

template <typename T, int D, int NW>
__global__ void __launch_bounds__(NW * 32) attn_mma_kernel(AttnArgs a) {
    constexpr int kBM = 16 * NW;
    constexpr int NT = 32 * NW;
    extern __shared__ __align__(128) uint8_t smraw[];
    T* Qs = reinterpret_cast<T*>(smraw);                 // [kBM][D]
    T* Ks = Qs + kBM * D;                                // [2][kBN][D]
    T* Vs = Ks + 2 * kBN * D;                            // [2][kBN][D]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, tq4 = lane & 3;
    const int64_t bh = blockIdx.y;
    const int b = (int)(bh / a.heads), h = (int)(bh % a.heads);
    const int q0 = blockIdx.x * kBM;
    const T* qp = static_cast<const T*>(a.q) + (int64_t)b * a.tq * a.sq + (int64_t)h * D;
    const T* kp = static_cast<const T*>(a.k) + (int64_t)b * a.tk * a.sk + (int64_t)h * D;
    const T* vp = static_cast<const T*>(a.v) + (int64_t)b * a.tk * a.sv + (int64_t)h * D;

    int kend = a.tk;
    if (a.causal) kend = min(kend, min(q0 + kBM, a.tq));
    const int ntiles = (kend + kBN - 1) / kBN;

    load_tile<T, D, NT>(Qs, qp, a.sq, q0, min(kBM, a.tq - q0), kBM);
    if (ntiles > 0) {
        load_tile<T, D, NT>(Ks, kp, a.sk, 0, min(kBN, a.tk), kBN);
        load_tile<T, D, NT>(Vs, vp, a.sv, 0, min(kBN, a.tk), kBN);
    }
    cp_async_commit();

    // Q fragments for this warp's 16 rows: D/16 k-steps x 4 registers.
    uint32_t qf[D / 16][4];
    float o[D / 8][4];
#pragma unroll
    for (int i = 0; i < D / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};
    const float sl2 = a.scale * 1.4426950408889634f;   // scale * log2(e)
    const int qr0 = q0 + warp * 16 + g;                 // this thread's rows: qr0, qr0 + 8

    for (int it = 0; it < ntiles; ++it) {
        const int buf = it & 1;
        if (it + 1 < ntiles) {
            const int k1 = (it + 1) * kBN;
            load_tile<T, D, NT>(Ks + (buf ^ 1) * kBN * D, kp, a.sk, k1, min(kBN, a.tk - k1), kBN);
            load_tile<T, D, NT>(Vs + (buf ^ 1) * kBN * D, vp, a.sv, k1, min(kBN, a.tk - k1), kBN);
        }
        cp_async_commit();
        cp_async_wait<1>();
        __syncthreads();
        if (it == 0) {
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
                // A fragment: rows warp*16 + (lane%16), chunk 2*kk + lane/16
                const int r = warp * 16 + (lane & 15);
                const int c = 2 * kk + (lane >> 4);
                ldmatrix_x4(smem_u32(Qs + swz<D>(r, c)), qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3]);
            }
        }
        const T* Kt = Ks + buf * kBN * D;
        const T* Vt = Vs + buf * kBN * D;
        const int kbase = it * kBN;
        const int wrow0 = q0 + warp * 16;                  // this warp's first query row
        // Causal: a tile entirely after this warp's last row contributes nothing.
        if (a.causal && kbase > wrow0 + 15) {
            __syncthreads();
            continue;
        }
        // Per-element masking only where it can change something.
        const bool need_mask = a.mask_kind != 0 || kbase + kBN > a.tk || wrow0 + 15 >= a.tq ||
                               (a.causal && kbase + kBN - 1 > wrow0);
        // S = Q K^T : 16 x 64 per warp (8 n-tiles of 8 keys)
        float s[kBN / 8][4];
#pragma unroll
        for (int j = 0; j < kBN / 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
#pragma unroll
            for (int jp = 0; jp < kBN / 16; ++jp) {
                // two n-tiles (16 keys) x 16 dims: matrices (keys 0-7, d lo), (keys 0-7, d hi),
                // (keys 8-15, d lo), (keys 8-15, d hi)
                const int mi = lane >> 3;
                const int r = jp * 16 + (mi >> 1) * 8 + (lane & 7);
                const int c = 2 * kk + (mi & 1);
                uint32_t b0, b1, b2, b3;
                ldmatrix_x4(smem_u32(Kt + swz<D>(r, c)), b0, b1, b2, b3);
                mma16816<T>(s[2 * jp], qf[kk], b0, b1);
                mma16816<T>(s[2 * jp + 1], qf[kk], b2, b3);
            }
        }
        // scale (log2 domain), masks, online softmax
        float tmax[2] = {-INFINITY, -INFINITY};
        if (need_mask) {
#pragma unroll
            for (int j = 0; j < kBN / 8; ++j) {
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int row = qr0 + (e >> 1) * 8;
                    const int kj = kbase + j * 8 + 2 * tq4 + (e & 1);
                    float val = s[j][e] * sl2;
                    bool keep = kj < a.tk && row < a.tq;
                    if (keep && (a.causal || a.mask_kind)) {
                        const float add = mask_value<T>(a, b, h, row, kj, keep);
                        val += add * 1.4426950408889634f;
                    }
                    s[j][e] = keep ? val : -INFINITY;
                    tmax[e >> 1] = fmaxf(tmax[e >> 1], s[j][e]);
                }
            }
        } else {
#pragma unroll
            for (int j = 0; j < kBN / 8; ++j) {
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    s[j][e] *= sl2;
                    tmax[e >> 1] = fmaxf(tmax[e >> 1], s[j][e]);
                }
            }
        }
        float alpha[2];
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            tmax[r] = fmaxf(tmax[r], __shfl_xor_sync(0xffffffffu, tmax[r], 1));
            tmax[r] = fmaxf(tmax[r], __shfl_xor_sync(0xffffffffu, tmax[r], 2));
            const float mnew = fmaxf(mrow[r], tmax[r]);
            alpha[r] = (mnew == -INFINITY) ? 1.f : fast_exp2(mrow[r] - mnew);
            mrow[r] = mnew;
        }
        float psum[2] = {0.f, 0.f};
        uint32_t pf[kBN / 16][4];
#pragma unroll
        for (int j = 0; j < kBN / 8; ++j) {
            float p[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float mr = mrow[e >> 1];
                p[e] = (s[j][e] == -INFINITY) ? 0.f : fast_exp2(s[j][e] - mr);
                psum[e >> 1] += p[e];
            }
            // C fragment of n-tile j -> half of the A fragment for k-step j/2
            pf[j >> 1][(j & 1) * 2 + 0] = pack2<T>(p[0], p[1]);
            pf[j >> 1][(j & 1) * 2 + 1] = pack2<T>(p[2], p[3]);
        }
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            psum[r] += __shfl_xor_sync(0xffffffffu, psum[r], 1);
            psum[r] += __shfl_xor_sync(0xffffffffu, psum[r], 2);
            lrow[r] = lrow[r] * alpha[r] + psum[r];
        }
#pragma unroll
        for (int i = 0; i < D / 8; ++i) {
            o[i][0] *= alpha[0];
            o[i][1] *= alpha[0];
            o[i][2] *= alpha[1];
            o[i][3] *= alpha[1];
        }
        // O += P V: k = keys (4 k-steps of 16), n = dims (D/8 n-tiles)
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk) {
            // A fragment register order: (row g, k lo), (row g+8, k lo), (row g, k hi), (row g+8, k hi)
            const uint32_t af[4] = {pf[kk][0], pf[kk][1], pf[kk][2], pf[kk][3]};
#pragma unroll
            for (int dp = 0; dp < D / 16; ++dp) {
                // V^T fragments via transposed ldmatrix: matrices (keys lo, d 0-7), (keys hi, d 0-7),
                // (keys lo, d 8-15), (keys hi, d 8-15)
                const int mi = lane >> 3;
                const int r = kk * 16 + (mi & 1) * 8 + (lane & 7);
                const int c = 2 * dp + (mi >> 1);
                uint32_t b0, b1, b2, b3;
                ldmatrix_x4_trans(smem_u32(Vt + swz<D>(r, c)), b0, b1, b2, b3);
                mma16816<T>(o[2 * dp], af, b0, b1);
                mma16816<T>(o[2 * dp + 1], af, b2, b3);
            }
        }
        __syncthreads();
    }
    cp_async_wait<0>();
    // normalize and store: thread holds rows qr0, qr0+8; dims 8*i + 2*tq4 + {0,1}
    T* op = static_cast<T*>(a.o) + (int64_t)b * a.tq * a.so + (int64_t)h * D;
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const int row = qr0 + r * 8;
        if (row >= a.tq) continue;
        const float inv = lrow[r] > 0.f ? 1.f / lrow[r] : 0.f;
#pragma unroll
        for (int i = 0; i < D / 8; ++i) {
            const uint32_t pk = pack2<T>(o[i][2 * r] * inv, o[i][2 * r + 1] * inv);
            *reinterpret_cast<uint32_t*>(op + (int64_t)row * a.so + i * 8 + 2 * tq4) = pk;
        }
    }
}

int g_attn_variant = 0;
int g_attn_poly_pairs = 1;

template <typename T>
int launch_attn(AttnArgs a, cudaStream_t st) {
    if (a.nb * (int64_t)a.heads > 0 && g_attn_variant == 0) {
        const int rc = launch_attn_tc<T>(a, st);
        if (rc != WIDEK_ERR_UNSUPPORTED) return rc;
    }
    const bool mma_ok = !std::is_same<T, float>::value && (a.dh == 64 || a.dh == 128) &&
                        (a.sq % 8 == 0) && (a.sk % 8 == 0) && (a.sv % 8 == 0) && (a.so % 2 == 0) &&
                        aligned16(a.q) && aligned16(a.k) && aligned16(a.v) &&
                        ((reinterpret_cast<uintptr_t>(a.o) & 3) == 0);
    if (a.nb * (int64_t)a.heads > 65535) return set_error(WIDEK_ERR_UNSUPPORTED, "attention: too many heads");
    if (mma_ok) {
        if constexpr (!std::is_same<T, float>::value) {
            const int D = a.dh;
            // 8 warps (128 query rows) per CTA share each K/V tile; short
            // sequences use 4 warps so that more CTAs run.
            const int nw = a.tq >= 256 ? 8 : 4;
            const int bm = 16 * nw;
            const size_t smem = (size_t)(bm * D + 4 * kBN * D) * sizeof(T);
            dim3 grid((unsigned)((a.tq + bm - 1) / bm), (unsigned)(a.nb * a.heads));
            if (D == 64 && nw == 8) {
                auto k = attn_mma_kernel<T, 64, 8>;
                cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
                k<<<grid, 256, smem, st>>>(a);
            } else if (D == 64) {
                auto k = attn_mma_kernel<T, 64, 4>;
                cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
                k<<<grid, 128, smem, st>>>(a);
            } else if (nw == 8) {
                auto k = attn_mma_kernel<T, 128, 8>;
                cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
                k<<<grid, 256, smem, st>>>(a);
            } else {
                auto k = attn_mma_kernel<T, 128, 4>;
                cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
                k<<<grid, 128, smem, st>>>(a);
            }
            return check_launch("widek_attention_fwd (mma)");
        }
    }
    if (a.dh > 256) return set_error(WIDEK_ERR_UNSUPPORTED, "attention: head_dim %d > 256", a.dh);
    const size_t smem = (size_t)(2 * kSimtKeys * a.dh + kSimtRows * a.dh) * sizeof(float);
    dim3 grid((unsigned)((a.tq + kSimtRows - 1) / kSimtRows), (unsigned)(a.nb * a.heads));
    if (a.dh <= 32) {
        auto k = attn_simt_kernel<T, 32>;
        cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        k<<<grid, 32 * kSimtRows, smem, st>>>(a);
    } else if (a.dh <= 64) {
        auto k = attn_simt_kernel<T, 64>;
        cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        k<<<grid, 32 * kSimtRows, smem, st>>>(a);
    } else if (a.dh <= 128) {
        auto k = attn_simt_kernel<T, 128>;
        cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        k<<<grid, 32 * kSimtRows, smem, st>>>(a);
    } else {
        auto k = attn_simt_kernel<T, 256>;
        cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        k<<<grid, 32 * kSimtRows, smem, st>>>(a);
    }
    return check_launch("widek_attention_fwd (simt)");
}

struct AttnLaunch {
    AttnArgs a;
    cudaStream_t st;
    template <typename T>
    int run() { return launch_attn<T>(a, st); }
};

}  // namespace

int attn_variant() { return g_attn_variant; }
int attn_poly_pairs() { return g_attn_poly_pairs; }

}  // namespace widek

extern "C" int widek_attention_set_variant(int variant) {
    if (variant == 0 || variant == 1) {
        widek::g_attn_variant = variant;
        widek::g_attn_poly_pairs = 1;
        return WIDEK_OK;
    }
    if (variant >= 10 && variant <= 12) {
        widek::g_attn_variant = 0;
        widek::g_attn_poly_pairs = variant - 10;
        return WIDEK_OK;
    }
    return widek::set_error(WIDEK_ERR_INVALID, "attention: unknown variant %d", variant);
}

extern "C" int widek_attention_fwd(const void* q, const void* k, const void* v, void* o, int64_t q_row_stride,
                                   int64_t k_row_stride, int64_t v_row_stride, int64_t o_row_stride, int64_t nb,
                                   int64_t heads, int64_t tq, int64_t tk, int64_t head_dim, int causal,
                                   const void* mask, int mask_kind, const int64_t* mask_strides, double scale,
                                   int dtype, void* stream) {
    using namespace widek;
    if (nb < 0 || heads < 0 || tq < 0 || tk < 0 || head_dim <= 0)
        return set_error(WIDEK_ERR_INVALID, "attention: bad sizes");
    if (nb * heads * tq == 0) return WIDEK_OK;
    if (!q || !k || !v || !o) return set_error(WIDEK_ERR_INVALID, "attention: null pointer");
    if (mask_kind < 0 || mask_kind > 3 || (mask_kind && (!mask || !mask_strides)))
        return set_error(WIDEK_ERR_INVALID, "attention: bad mask arguments");
    if (tq > 0x7fffffff || tk > 0x7fffffff || head_dim > 256)
        return set_error(WIDEK_ERR_UNSUPPORTED, "attention: sizes outside the supported range");
    AttnArgs a{};
    a.q = q; a.k = k; a.v = v; a.o = o; a.mask = mask;
    a.sq = q_row_stride; a.sk = k_row_stride; a.sv = v_row_stride; a.so = o_row_stride;
    if (mask_kind) {
        a.ms_b = mask_strides[0]; a.ms_h = mask_strides[1]; a.ms_q = mask_strides[2]; a.ms_k = mask_strides[3];
    }
    a.nb = (int)nb; a.heads = (int)heads; a.tq = (int)tq; a.tk = (int)tk; a.dh = (int)head_dim;
    a.causal = causal ? 1 : 0; a.mask_kind = mask_kind; a.scale = (float)scale;
    AttnLaunch L{a, (cudaStream_t)stream};
    return dispatch_dtype(dtype, L);
}
