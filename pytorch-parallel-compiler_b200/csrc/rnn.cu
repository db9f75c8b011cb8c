// WideGRU / WideLSTM recurrence: one persistent launch for all T steps.
//
// The input projection for every step (x @ W_ih^T + b_ih) is computed before
// this kernel by the grouped GEMM (widek_linear_fwd) into gates_x
// [n, batch, T, G*H] (G = 3 for GRU gates r,z,n; 4 for LSTM gates i,f,g,o).
//
// Recurrence: one thread-block cluster of CL CTAs per model. CTA q of the
// cluster owns hidden units [q*U, (q+1)*U), U = H / CL, and keeps the G*U rows
// of W_hh that produce those units resident in shared memory, transposed to
// k-major fp32 ([H][G*U]) so a warp reads consecutive rows at one k
// (conflict-free) while h[b][k] is a broadcast. Each step:
//   1. thread r computes gh[b][r] = W_hh[r] . h[b] + b_hh[r] for all b;
//   2. threads (b, j) combine the gates (PyTorch formulas), update h (and c for
//      LSTM, kept in shared memory), write out[n, b, t, unit];
//   3. the new h slice is stored into every cluster CTA's next h buffer
//      through distributed shared memory; one hardware cluster barrier
//      (barrier.cluster arrive.release / wait.acquire) publishes it.
// h is double-buffered so a single barrier per step orders reads and writes.
// The cluster is as large as all models' clusters allow on the GPU at once
// (up to 8 CTAs); with resident weights the mat-vec splits each row's k
// range over S consecutive lanes (16-byte words of W and h, partial sums
// combined by shuffles), so S*R threads share the work with short
// dependency chains; the next step's input-gate values are loaded into
// registers one step ahead.
// When the weight slice does not fit in shared memory for any cluster size,
// the kernel reads W_hh rows from global memory (L2) instead.
#include <cooperative_groups.h>

#include "common.cuh"
#include "sm100_ptx.cuh"

namespace cg = cooperative_groups;

namespace widek {
namespace {

__device__ __forceinline__ float sigmoidf_(float x) { return 1.f / (1.f + expf(-x)); }
// Short-latency forms for the register-resident kernel's critical path: the
// exponential intrinsic and an approximate divide for the logistic, and tanh
// from the identity tanh(x) = 2 * sigmoid(2x) - 1 (absolute error ~1e-7 near
// 0, far inside the fp32 contract's 1e-4).
__device__ __forceinline__ float sigmoid_fast(float x) { return __fdividef(1.f, 1.f + __expf(-x)); }
__device__ __forceinline__ float tanh_fast(float x) { return 2.f * sigmoid_fast(2.f * x) - 1.f; }

struct RnnArgs {
    const void* gx;      // [n, batch, T, G*H]
    const void* w_hh;    // model i's [G*H, H] block at w_hh + i*whh_ms, rows whh_rs apart
    const void* b_hh;    // [n, G*H] or null
    const void* h0;      // [n, batch, H] or null
    const void* c0;      // [n, batch, H] or null (LSTM)
    void* out;           // [n, batch, T, H] (or packed, see out_ms / out_bs)
    void* hn;            // [n, batch, H]
    void* cn;            // [n, batch, H] or null (LSTM)
    int batch, T, H, G, cl, w_in_smem;
    int kparts;          // threads sharing one row's dot products (split k, vec4 path)
    int64_t whh_ms, whh_rs;   // W_hh model / row strides (elements)
    int64_t out_ms, out_bs;   // out model / batch strides (elements): N-first [n, batch, T, H] is
                              // (batch*T*H, T*H), the packed [batch, n*T, H] layout (T*H, n*T*H)
};

template <typename T, bool LSTM>
__global__ void __launch_bounds__(1024) rnn_cluster_kernel(RnnArgs a) {
    cg::cluster_group cluster = cg::this_cluster();
    const int q = (int)cluster.block_rank();
    const int model = blockIdx.x / a.cl;
    const int H = a.H, G = a.G, B = a.batch, U = H / a.cl, R = G * U;

    extern __shared__ float sm[];
    float* Ws = sm;                                          // [H][R] (if resident)
    float* hbuf = Ws + (a.w_in_smem ? (size_t)H * R : 0);    // [2][B][H]
    float* gates = hbuf + 2 * (size_t)B * H;                  // [B][R]
    float* cst = gates + (size_t)B * R;                       // [B][U] (LSTM)

    const T* gx = static_cast<const T*>(a.gx) + (size_t)model * B * a.T * G * H;
    const T* w = static_cast<const T*>(a.w_hh) + (size_t)model * a.whh_ms;
    const int64_t wrs = a.whh_rs;
    const T* bh = a.b_hh ? static_cast<const T*>(a.b_hh) + (size_t)model * G * H : nullptr;
    T* out = static_cast<T*>(a.out) + (size_t)model * a.out_ms;

    // global row of local row lr = g * U + j
    auto grow = [&](int lr) { return (lr / U) * H + q * U + (lr % U); };

    // Resident weights: row-major [R][H] (16-byte words of four k) for the
    // split-k mat-vec when H % 4 == 0, else k-major [H][R].
    const bool vec4 = a.w_in_smem && (H % 4 == 0);
    if (a.w_in_smem) {
        for (int i = threadIdx.x; i < R * H; i += blockDim.x) {
            const int lr = i / H, k = i % H;
            const float v = to_f<T>(w[(size_t)grow(lr) * wrs + k]);
            if (vec4) Ws[(size_t)lr * H + k] = v;
            else Ws[(size_t)k * R + lr] = v;
        }
    }
    for (int i = threadIdx.x; i < B * H; i += blockDim.x) {
        hbuf[i] = a.h0 ? to_f<T>(static_cast<const T*>(a.h0)[(size_t)model * B * H + i]) : 0.f;
    }
    if (LSTM) {
        for (int i = threadIdx.x; i < B * U; i += blockDim.x) {
            const int b = i / U, j = i % U;
            cst[i] = a.c0 ? to_f<T>(static_cast<const T*>(a.c0)[((size_t)model * B + b) * H + q * U + j]) : 0.f;
        }
    }
    cluster.sync();

    // Input-projection gates of the next step, prefetched into registers one
    // step ahead when every (b, j) pair has its own thread (i = b*U + j);
    // otherwise the gate loop reads them directly.
    const int bu = B * U;
    const bool pre = bu <= (int)blockDim.x;
    float gx_next[4] = {0.f, 0.f, 0.f, 0.f};
    auto load_gx = [&](int i, int t, float (&v)[4]) {
        const int b = i / U, j = i % U;
        const T* gxr = gx + ((size_t)b * a.T + t) * G * H + q * U + j;
#pragma unroll
        for (int gi = 0; gi < 4; ++gi)
            if (gi < G) v[gi] = to_f<T>(gxr[(size_t)gi * H]);
    };
    // The projected gates come from the kernel before this one on the
    // stream (launched as its programmatic dependent: everything above ran
    // while it finished).
    sm100::grid_dep_wait();
    if (pre && (int)threadIdx.x < bu && a.T > 0) load_gx(threadIdx.x, 0, gx_next);

    for (int t = 0; t < a.T; ++t) {
        const float* hc = hbuf + (size_t)(t & 1) * B * H;
        float* hn_local = hbuf + (size_t)((t + 1) & 1) * B * H;
        float gx_cur[4] = {gx_next[0], gx_next[1], gx_next[2], gx_next[3]};
        if (pre && (int)threadIdx.x < bu && t + 1 < a.T) load_gx(threadIdx.x, t + 1, gx_next);
        // 1. recurrent mat-vec: rows x batch
        if (vec4) {
            // Split k: S = kparts consecutive lanes share a row; lane part p
            // takes the 16-byte words k4 = i*S + p, so a quarter-warp reads
            // contiguous 128-byte runs of W and of each h row; partial sums
            // meet by shuffles. S*R threads, many warps per SM, short chains.
            const int S = a.kparts;
            const int lr = threadIdx.x / S, p = threadIdx.x % S;
            const int KS = (H >> 2) / S;
            const bool live = lr < R;
            const float4* W4 = reinterpret_cast<const float4*>(Ws) + (size_t)(live ? lr : 0) * (H >> 2);
            const float bias = (live && bh) ? to_f<T>(bh[grow(lr)]) : 0.f;
            for (int b0 = 0; b0 < B; b0 += 4) {
                const int nb = B - b0 < 4 ? B - b0 : 4;
                float acc[4] = {0.f, 0.f, 0.f, 0.f};
                const float4* H4 = reinterpret_cast<const float4*>(hc + (size_t)b0 * H);
                const int h4 = H >> 2;
#pragma unroll 2
                for (int i = 0; i < KS; ++i) {
                    const int k4 = i * S + p;
                    const float4 wv = W4[k4];
#pragma unroll
                    for (int bb = 0; bb < 4; ++bb) {
                        const float4 hv = H4[(bb < nb ? bb : 0) * h4 + k4];
                        float s2 = acc[bb];
                        s2 = fmaf(wv.x, hv.x, s2);
                        s2 = fmaf(wv.y, hv.y, s2);
                        s2 = fmaf(wv.z, hv.z, s2);
                        s2 = fmaf(wv.w, hv.w, s2);
                        acc[bb] = s2;
                    }
                }
#pragma unroll
                for (int bb = 0; bb < 4; ++bb)
                    for (int off = S >> 1; off > 0; off >>= 1) acc[bb] += __shfl_xor_sync(0xffffffffu, acc[bb], off);
                if (live && p == 0) {
#pragma unroll
                    for (int bb = 0; bb < 4; ++bb)
                        if (bb < nb) gates[(size_t)(b0 + bb) * R + lr] = acc[bb] + bias;
                }
            }
        } else {
            for (int lr = threadIdx.x; lr < R; lr += blockDim.x) {
                const float bias = bh ? to_f<T>(bh[grow(lr)]) : 0.f;
                for (int b0 = 0; b0 < B; b0 += 4) {
                    float acc[4];
#pragma unroll
                    for (int bb = 0; bb < 4; ++bb) acc[bb] = bias;
                    const int nb = B - b0 < 4 ? B - b0 : 4;
                    if (a.w_in_smem) {
#pragma unroll 4
                        for (int k = 0; k < H; ++k) {
                            const float wv = Ws[(size_t)k * R + lr];
#pragma unroll
                            for (int bb = 0; bb < 4; ++bb)
                                if (bb < nb) acc[bb] = fmaf(wv, hc[(size_t)(b0 + bb) * H + k], acc[bb]);
                        }
                    } else {
                        const T* wr = w + (size_t)grow(lr) * wrs;
#pragma unroll 4
                        for (int k = 0; k < H; ++k) {
                            const float wv = to_f<T>(wr[k]);
#pragma unroll
                            for (int bb = 0; bb < 4; ++bb)
                                if (bb < nb) acc[bb] = fmaf(wv, hc[(size_t)(b0 + bb) * H + k], acc[bb]);
                        }
                    }
#pragma unroll
                    for (int bb = 0; bb < 4; ++bb)
                        if (bb < nb) gates[(size_t)(b0 + bb) * R + lr] = acc[bb];
                }
            }
        }
        __syncthreads();
        // 2. gate math for (b, j); blockDim.x >= B*U (launcher)
        for (int i = threadIdx.x; i < B * U; i += blockDim.x) {
            const int b = i / U, j = i % U;
            const int ju = q * U + j;                            // global hidden unit
            const float* gr = gates + (size_t)b * R;
            if (!pre) load_gx(i, t, gx_cur);
            float hnew;
            if (!LSTM) {
                const float r = sigmoidf_(gx_cur[0] + gr[j]);
                const float z = sigmoidf_(gx_cur[1] + gr[U + j]);
                const float nn = tanhf(gx_cur[2] + r * gr[2 * U + j]);
                hnew = (1.f - z) * nn + z * hc[(size_t)b * H + ju];
            } else {
                const float ig = sigmoidf_(gx_cur[0] + gr[j]);
                const float fg = sigmoidf_(gx_cur[1] + gr[U + j]);
                const float gg = tanhf(gx_cur[2] + gr[2 * U + j]);
                const float og = sigmoidf_(gx_cur[3] + gr[3 * U + j]);
                const float c = fg * cst[i] + ig * gg;
                cst[i] = c;
                hnew = og * tanhf(c);
            }
            // Round through the storage type so every consumer sees the
            // value the reference would hold in a tensor of that dtype.
            const T hs = from_f<T>(hnew);
            const float hv = to_f<T>(hs);
            out[(size_t)b * a.out_bs + (size_t)t * H + ju] = hs;
            // 3. publish into every cluster CTA's next buffer (DSMEM)
            for (int r = 0; r < a.cl; ++r) {
                float* dst = cluster.map_shared_rank(hn_local, r);
                dst[(size_t)b * H + ju] = hv;
            }
        }
        cluster.sync();
    }

    // final states
    const float* hl = hbuf + (size_t)(a.T & 1) * B * H;
    for (int i = threadIdx.x; i < B * U; i += blockDim.x) {
        const int b = i / U, j = i % U;
        const int ju = q * U + j;
        static_cast<T*>(a.hn)[((size_t)model * B + b) * H + ju] = from_f<T>(hl[(size_t)b * H + ju]);
        if (LSTM && a.cn) static_cast<T*>(a.cn)[((size_t)model * B + b) * H + ju] = from_f<T>(cst[i]);
    }
    // No CTA may exit while a peer can still read its shared memory.
    cluster.sync();
}

// ---------------------------------------------------------------------------
// Register-resident variant (small hidden sizes, e.g. H = 128): W_hh lives in
// registers for all T steps and the hidden state moves by signals instead of
// a cluster-wide barrier.
//
// 256 threads per CTA; lane part p = tid % 8 of row group g = tid / 8 holds
// the 16-byte words k4 = i*8 + p (i < KS = H/32) of rows g + 32r (r < RPT),
// so each step's mat-vec reads only h from shared memory (one 16-byte word
// per k-slice and batch row) and reduces the 8 partial sums by shuffles.
// The new h slice goes into every cluster CTA's next buffer by asynchronous
// DSMEM stores (st.async, sent by the lanes of the gate math as soon as a
// 16-byte chunk is complete) that complete their bytes on that CTA's "full"
// mbarrier of the buffer; a CTA posts the B*H*4 bytes it expects for h_{t+1}
// at the start of step t and starts step t+1 once they have all landed. A
// two-deep buffer ring is enough: a CTA writes h_{t+2} into a peer only
// after receiving all of that peer's h_{t+1}, whose chunks the peer sent
// after its step-t reads of the buffer (mat-vec and gate math) had returned.
// Every wait is bounded (device error + abort flag).
// ---------------------------------------------------------------------------
constexpr int kRegThreads = 256;
constexpr int kRegParts = 8;

__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, const volatile int* abort) {
    const uint32_t addr = sm100::smem_addr(bar);
    auto try_once = [&]() {
        uint32_t ok;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}\n"
            : "=r"(ok)
            : "r"(addr), "r"(parity)
            : "memory");
        return ok != 0;
    };
    if (try_once()) return true;
    const uint64_t t0 = globaltimer_ns();
    while (true) {
#pragma unroll 1
        for (int i = 0; i < 32; ++i)
            if (try_once()) return true;
        if (*abort) return false;
        if (globaltimer_ns() - t0 > kWaitLimitNs) return false;
    }
}

template <typename T, bool LSTM, int RPT, int KS>
__global__ void __launch_bounds__(kRegThreads, 1) rnn_reg_kernel(RnnArgs a, int* err) {
    cg::cluster_group cluster = cg::this_cluster();
    const int q = (int)cluster.block_rank();
    const int cl = a.cl;
    const int model = blockIdx.x / cl;
    const int H = a.H, G = a.G, B = a.batch, U = H / cl, R = G * U;

    extern __shared__ __align__(16) float rsm[];
    float* hbuf = rsm;                                         // [2][B][H]
    float* gates = hbuf + 2 * (size_t)B * H;                   // [B][R]
    float* cst = gates + (size_t)B * R;                        // [B][U] (LSTM)
    uint64_t* full = reinterpret_cast<uint64_t*>(cst + (((size_t)B * U + 3) & ~(size_t)3));   // [2]
    volatile int* abort_flag = reinterpret_cast<volatile int*>(full + 2);

    const T* gx = static_cast<const T*>(a.gx) + (size_t)model * B * a.T * G * H;
    const T* w = static_cast<const T*>(a.w_hh) + (size_t)model * a.whh_ms;
    const T* bh = a.b_hh ? static_cast<const T*>(a.b_hh) + (size_t)model * G * H : nullptr;
    T* out = static_cast<T*>(a.out) + (size_t)model * a.out_ms;
    auto grow = [&](int lr) { return (lr / U) * H + q * U + (lr % U); };

    const int tid = threadIdx.x, grp = tid / kRegParts, p = tid % kRegParts;
    // This thread's W words and row biases, for all steps.
    float4 wr[RPT][KS];
    float brow[RPT];
#pragma unroll
    for (int r = 0; r < RPT; ++r) {
        const int lr = grp + 32 * r;
        const bool ok = lr < R;
        const T* wrow = w + (size_t)(ok ? grow(lr) : 0) * a.whh_rs;
#pragma unroll
        for (int i = 0; i < KS; ++i) {
            const int k = 4 * (i * kRegParts + p);
            wr[r][i] = ok ? make_float4(to_f<T>(wrow[k]), to_f<T>(wrow[k + 1]), to_f<T>(wrow[k + 2]),
                                        to_f<T>(wrow[k + 3]))
                          : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        brow[r] = (ok && bh) ? to_f<T>(bh[grow(lr)]) : 0.f;
    }
    for (int i = tid; i < B * H; i += blockDim.x)
        hbuf[i] = a.h0 ? to_f<T>(static_cast<const T*>(a.h0)[(size_t)model * B * H + i]) : 0.f;
    if (LSTM) {
        for (int i = tid; i < B * U; i += blockDim.x) {
            const int b = i / U, j = i % U;
            cst[i] = a.c0 ? to_f<T>(static_cast<const T*>(a.c0)[((size_t)model * B + b) * H + q * U + j]) : 0.f;
        }
    }
    // Each "full" phase has one arrival (this CTA's expect_tx of the B*H*4
    // bytes that the cl CTAs' asynchronous stores of 16-byte h chunks
    // complete).
    if (tid == 0) {
        sm100::mbar_init(&full[0], 1u);
        sm100::mbar_init(&full[1], 1u);
        *abort_flag = 0;
        sm100::mbar_init_fence();
    }
    cluster.sync();
    const uint32_t full0 = sm100::smem_addr(&full[0]);

    const int bu = B * U;
    const bool pre = bu <= (int)blockDim.x;
    float gx_next[4] = {0.f, 0.f, 0.f, 0.f};
    auto load_gx = [&](int i, int t, float (&v)[4]) {
        const int b = i / U, j = i % U;
        const T* gxr = gx + ((size_t)b * a.T + t) * G * H + q * U + j;
#pragma unroll
        for (int gi = 0; gi < 4; ++gi)
            if (gi < G) v[gi] = to_f<T>(gxr[(size_t)gi * H]);
    };
    // The projected gates come from the kernel before this one on the
    // stream (launched as its programmatic dependent: the W_hh register
    // load, the state set-up and the cluster start ran while it finished).
    sm100::grid_dep_wait();
    if (pre && tid < bu && a.T > 0) load_gx(tid, 0, gx_next);

    bool ok = true;
    int posted = 0;          // last h index whose bytes this CTA expects
    for (int t = 0; t < a.T; ++t) {
        // One thread waits for h_t (all B*H*4 bytes landed); the barrier
        // then releases the CTA, and every thread sees the same verdict.
        if (t > 0 && tid == 0 && !mbar_wait_cluster(&full[t & 1], (uint32_t)(((t - 1) >> 1) & 1), abort_flag))
            *abort_flag = 1;
        __syncthreads();     // h_t complete; the previous step's gate reads are done
        if (*abort_flag) {
            ok = false;
            break;
        }
        // The buffer that receives h_{t+1}: its previous phase (h_{t-1})
        // completed before step t-1, and no CTA can send h_{t+1} before it
        // has this CTA's h_t.
        if (tid == 0) sm100::mbar_arrive_expect_tx(&full[(t + 1) & 1], (uint32_t)(B * H * 4));
        posted = t + 1;
        const float* hc = hbuf + (size_t)(t & 1) * B * H;
        const int nxt = (t + 1) & 1;
        float gx_cur[4] = {gx_next[0], gx_next[1], gx_next[2], gx_next[3]};
        if (pre && tid < bu && t + 1 < a.T) load_gx(tid, t + 1, gx_next);
        // 1. mat-vec from registers: four batch rows at a time (their loads,
        // FMA chains and shuffle trees interleave), RPT rows x this lane's
        // k-slice
        const float4* H4 = reinterpret_cast<const float4*>(hc);
        for (int b0 = 0; b0 < B; b0 += 4) {
            const int nb = B - b0 < 4 ? B - b0 : 4;
            // v[bb*4 + r]: batch row b0+bb, gate row grp + 32r (rows past RPT stay 0)
            float v[16];
#pragma unroll
            for (int k = 0; k < 16; ++k) v[k] = 0.f;
#pragma unroll
            for (int i = 0; i < KS; ++i) {
                float4 hv[4];
#pragma unroll
                for (int bb = 0; bb < 4; ++bb)
                    hv[bb] = H4[(size_t)(b0 + (bb < nb ? bb : 0)) * (H >> 2) + i * kRegParts + p];
#pragma unroll
                for (int bb = 0; bb < 4; ++bb)
#pragma unroll
                    for (int r = 0; r < RPT; ++r) {
                        float s2 = v[bb * 4 + r];
                        s2 = fmaf(wr[r][i].x, hv[bb].x, s2);
                        s2 = fmaf(wr[r][i].y, hv[bb].y, s2);
                        s2 = fmaf(wr[r][i].z, hv[bb].z, s2);
                        s2 = fmaf(wr[r][i].w, hv[bb].w, s2);
                        v[bb * 4 + r] = s2;
                    }
            }
            // Recursive halving over the 8 lanes of the row group: each level
            // keeps the half of the values selected by one bit of the lane
            // part and adds the partner's copy of it (8 + 4 + 2 shuffles for
            // 16 sums); lane part p ends with values 2p and 2p + 1.
            float v8[8], v4[4], v2[2];
            {
                const bool hb = (p >> 2) & 1;
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    const float send = hb ? v[k] : v[k + 8], keep = hb ? v[k + 8] : v[k];
                    v8[k] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
                }
            }
            {
                const bool hb = (p >> 1) & 1;
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const float send = hb ? v8[k] : v8[k + 4], keep = hb ? v8[k + 4] : v8[k];
                    v4[k] = keep + __shfl_xor_sync(0xffffffffu, send, 2);
                }
            }
            {
                const bool hb = p & 1;
#pragma unroll
                for (int k = 0; k < 2; ++k) {
                    const float send = hb ? v4[k] : v4[k + 2], keep = hb ? v4[k + 2] : v4[k];
                    v2[k] = keep + __shfl_xor_sync(0xffffffffu, send, 1);
                }
            }
#pragma unroll
            for (int k = 0; k < 2; ++k) {
                const int idx = 2 * p + k, bb = idx >> 2, r = idx & 3;
                const int lr = grp + 32 * r;
                if (r < RPT && bb < nb && lr < R) {
                    float bias = brow[0];
#pragma unroll
                    for (int rr = 1; rr < RPT; ++rr) bias = r == rr ? brow[rr] : bias;
                    gates[(size_t)(b0 + bb) * R + lr] = v2[k] + bias;
                }
            }
        }
        __syncthreads();
        // 2. gate math for (b, j), then 3. publish: lanes 4m..4m+3 hold one
        // 16-byte chunk of the new h slice (4 consecutive j of one batch row;
        // U % 4 == 0, so a chunk never straddles rows or the end), gather it
        // by shuffles, and lane 4m+k sends it to cluster ranks k, k+4, ... as
        // asynchronous DSMEM stores that complete bytes on that CTA's "full"
        // mbarrier. No barrier separates the gate math from the publish:
        // the h_{t+1} chunks overwrite a peer's h_{t-1} buffer, and this CTA
        // reaches this point only with the peer's whole h_t, whose last chunk
        // the peer sent after its last read of h_{t-1} (a lane's loads are
        // consumed before its stores issue).
        float* hnext = hbuf + (size_t)nxt * B * H;
        const int lane = tid & 31;
        for (int base = 0; base < bu; base += (int)blockDim.x) {
            const int i = base + tid;
            const bool on = i < bu;     // the same for the 4 lanes of a chunk
            float hval = 0.f;
            if (on) {
                const int b = i / U, j = i % U;
                const int ju = q * U + j;
                const float* gr = gates + (size_t)b * R;
                if (!pre) load_gx(i, t, gx_cur);
                float hnew;
                if (!LSTM) {
                    const float r = sigmoid_fast(gx_cur[0] + gr[j]);
                    const float z = sigmoid_fast(gx_cur[1] + gr[U + j]);
                    const float nn = tanh_fast(gx_cur[2] + r * gr[2 * U + j]);
                    hnew = (1.f - z) * nn + z * hc[(size_t)b * H + ju];
                } else {
                    const float ig = sigmoid_fast(gx_cur[0] + gr[j]);
                    const float fg = sigmoid_fast(gx_cur[1] + gr[U + j]);
                    const float gg = tanh_fast(gx_cur[2] + gr[2 * U + j]);
                    const float og = sigmoid_fast(gx_cur[3] + gr[3 * U + j]);
                    const float c = fg * cst[i] + ig * gg;
                    cst[i] = c;
                    hnew = og * tanh_fast(c);
                }
                const T hs = from_f<T>(hnew);
                hval = to_f<T>(hs);
                out[(size_t)b * a.out_bs + (size_t)t * H + ju] = hs;
            }
            const int g0 = lane & ~3;
            const float v0 = __shfl_sync(0xffffffffu, hval, g0), v1 = __shfl_sync(0xffffffffu, hval, g0 + 1),
                        v2 = __shfl_sync(0xffffffffu, hval, g0 + 2), v3 = __shfl_sync(0xffffffffu, hval, g0 + 3);
            if (on) {
                const int c0 = i & ~3, b = c0 / U, j = c0 % U;
                const uint32_t src = sm100::smem_addr(hnext + (size_t)b * H + q * U + j);
                for (int r = lane & 3; r < cl; r += 4) {
                    const uint32_t dst = sm100::map_to_rank(src, (uint32_t)r);
                    const uint32_t rbar = sm100::map_to_rank(full0, (uint32_t)r) + nxt * 8;
                    asm volatile(
                        "st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.f32 [%0], {%1, %2, %3, %4}, [%5];"
                        ::"r"(dst), "f"(v0), "f"(v1), "f"(v2), "f"(v3), "r"(rbar)
                        : "memory");
                }
            }
        }
    }
    // h_T (written by every CTA of the cluster into this CTA's buffer T % 2)
    if (ok && a.T > 0 && tid == 0 &&
        !mbar_wait_cluster(&full[a.T & 1], (uint32_t)(((a.T - 1) >> 1) & 1), abort_flag))
        *abort_flag = 1;
    __syncthreads();
    if (tid == 0 && *abort_flag) {
        raise_device_error(err, DEV_ERR_RNN_TIMEOUT);
        // Stores other CTAs may still have in flight into the phase this CTA
        // posted last land (bounded wait) before its shared memory goes away.
        const volatile int never = 0;
        if (posted > 0) mbar_wait_cluster(&full[posted & 1], (uint32_t)(((posted - 1) >> 1) & 1), &never);
    }
    const float* hl = hbuf + (size_t)(a.T & 1) * B * H;
    for (int i = tid; i < bu; i += blockDim.x) {
        const int b = i / U, j = i % U;
        const int ju = q * U + j;
        static_cast<T*>(a.hn)[((size_t)model * B + b) * H + ju] = from_f<T>(hl[(size_t)b * H + ju]);
        if (LSTM && a.cn) static_cast<T*>(a.cn)[((size_t)model * B + b) * H + ju] = from_f<T>(cst[i]);
    }
    // No CTA may exit while a peer can still write into or read its shared memory.
    cluster.sync();
}

size_t rnn_reg_smem(int B, int H, int G, int cl) {
    const int U = H / cl, R = G * U;
    const size_t bu4 = ((size_t)B * U + 3) & ~(size_t)3;
    const size_t f = 2 * (size_t)B * H + (size_t)B * R + bu4;
    return f * sizeof(float) + 4 * sizeof(uint64_t);
}

template <typename T, bool LSTM, int RPT>
int launch_rnn_reg_k(const RnnArgs& a, int64_t n, size_t smem, cudaStream_t st) {
    auto kern = rnn_reg_kernel<T, LSTM, RPT, 4>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
        return set_error(WIDEK_ERR_CUDA, "rnn: cannot reserve %zu bytes of shared memory", smem);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(n * a.cl));
    cfg.blockDim = dim3(kRegThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = a.cl;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, a, device_error_ptr());
    if (e != cudaSuccess) return set_error(WIDEK_ERR_CUDA, "rnn: launch failed: %s", cudaGetErrorString(e));
    return check_launch("widek_rnn_fwd (register-resident)");
}

// The register-resident kernel when H = 128 (KS = 4 words of k per lane part)
// and a cluster of cl CTAs leaves at most 128 gate rows per CTA (RPT <= 4).
template <typename T, bool LSTM>
int try_rnn_reg(RnnArgs a, int64_t n, cudaStream_t st, bool& used) {
    used = false;
    if (a.H != 128 || a.batch > 64) return WIDEK_OK;
    const int sms = sm_count(current_device());
    int cl = 0;
    for (int c : {8, 4, 2, 1}) {
        if (a.H % c || (int64_t)c * n > sms) continue;
        if (a.G * (a.H / c) <= 32 * 4) { cl = c; break; }
    }
    if (!cl) return WIDEK_OK;
    a.cl = cl;
    const int rpt = (a.G * (a.H / cl) + 31) / 32;
    const size_t smem = rnn_reg_smem(a.batch, a.H, a.G, cl);
    if (smem > 227 * 1024) return WIDEK_OK;
    used = true;
    switch (rpt) {
        case 1: return launch_rnn_reg_k<T, LSTM, 1>(a, n, smem, st);
        case 2: return launch_rnn_reg_k<T, LSTM, 2>(a, n, smem, st);
        case 3: return launch_rnn_reg_k<T, LSTM, 3>(a, n, smem, st);
        default: return launch_rnn_reg_k<T, LSTM, 4>(a, n, smem, st);
    }
}

constexpr size_t kMaxSmem = 227 * 1024;

size_t rnn_smem(int B, int H, int G, int cl, bool w_in_smem) {
    const int U = H / cl, R = G * U;
    size_t f = (w_in_smem ? (size_t)H * R : 0) + 2 * (size_t)B * H + (size_t)B * R + (size_t)B * U;
    return f * sizeof(float);
}

// 0: the register-resident kernel where it applies (default); 1: the
// shared-memory cluster kernel only. Set with widek_rnn_set_variant.
int g_rnn_variant = 0;

template <typename T, bool LSTM>
int launch_rnn(RnnArgs a, int64_t n, cudaStream_t st) {
    if (g_rnn_variant == 0) {
        bool used = false;
        const int rc = try_rnn_reg<T, LSTM>(a, n, st, used);
        if (used) return rc;
    }
    // Cluster of 1..8 CTAs per model (H divisible by it): the largest one for
    // which all models' clusters fit on the GPU at once (more SMs per model,
    // a shorter mat-vec per step), else the smallest whose weight slice fits
    // in shared memory; failing that, weights are read from global memory.
    const int sms = sm_count(current_device());
    int cl = 0;
    bool resident = false;
    for (int c : {8, 4, 2, 1}) {
        if (a.H % c || (int64_t)c * n > sms) continue;
        if (rnn_smem(a.batch, a.H, a.G, c, true) <= kMaxSmem) { cl = c; resident = true; break; }
    }
    for (int c : {1, 2, 4, 8}) {
        if (cl) break;
        if (a.H % c) continue;
        if (rnn_smem(a.batch, a.H, a.G, c, true) <= kMaxSmem) { cl = c; resident = true; break; }
    }
    if (!cl) {
        for (int c : {8, 4, 2, 1}) {
            if (a.H % c) continue;
            if (rnn_smem(a.batch, a.H, a.G, c, false) <= kMaxSmem) { cl = c; break; }
        }
    }
    if (!cl) return set_error(WIDEK_ERR_UNSUPPORTED, "rnn: batch=%d hidden=%d does not fit on chip", a.batch, a.H);
    a.cl = cl;
    a.w_in_smem = resident ? 1 : 0;
    const size_t smem = rnn_smem(a.batch, a.H, a.G, cl, resident);
    auto kern = rnn_cluster_kernel<T, LSTM>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
        return set_error(WIDEK_ERR_CUDA, "rnn: cannot reserve %zu bytes of shared memory", smem);
    const int rows = a.G * (a.H / cl);
    // Split-k factor of the resident vec4 mat-vec: the largest S in {8, 4, 2, 1}
    // dividing H/4 with S*rows <= 1024 threads (S = 1 keeps one row per thread).
    a.kparts = 1;
    if (resident && a.H % 4 == 0) {
        for (int sp : {8, 4, 2}) {
            if ((a.H / 4) % sp == 0 && sp * rows <= 1024) { a.kparts = sp; break; }
        }
    }
    int threads = ((rows * a.kparts + 31) / 32) * 32;
    const int pairs = a.batch * (a.H / cl);
    if (threads < pairs) threads = ((pairs + 31) / 32) * 32;
    if (threads > 1024) threads = 1024;     // the gate loop strides when pairs > 1024
    if (threads < 128) threads = 128;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(n * cl));
    cfg.blockDim = dim3((unsigned)threads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = cl;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, a);
    if (e != cudaSuccess) return set_error(WIDEK_ERR_CUDA, "rnn: launch failed: %s", cudaGetErrorString(e));
    return check_launch("widek_rnn_fwd");
}

struct RnnLaunch {
    RnnArgs a;
    int64_t n;
    bool lstm;
    cudaStream_t st;
    template <typename T>
    int run() {
        return lstm ? launch_rnn<T, true>(a, n, st) : launch_rnn<T, false>(a, n, st);
    }
};

int rnn_entry(bool lstm, const void* gates_x, const void* w_hh, const void* b_hh, const void* h0, const void* c0,
              void* out, void* h_n, void* c_n, int64_t n, int64_t batch, int64_t steps, int64_t hidden, int dtype,
              void* stream) {
    if (n < 0 || batch < 0 || steps < 0 || hidden < 0) return set_error(WIDEK_ERR_INVALID, "rnn: negative size");
    if (batch > 1024 || hidden > 4096 || steps > 0x7fffffff || n > 65535)
        return set_error(WIDEK_ERR_UNSUPPORTED, "rnn: batch=%lld hidden=%lld outside the supported range",
                         (long long)batch, (long long)hidden);
    if (n == 0 || batch == 0 || hidden == 0) return WIDEK_OK;
    if (!w_hh || !h_n || (steps > 0 && (!gates_x || !out)))
        return set_error(WIDEK_ERR_INVALID, "rnn: null pointer");
    const int g = lstm ? 4 : 3;
    RnnArgs a{gates_x, w_hh, b_hh, h0, c0, out, h_n, c_n, (int)batch, (int)steps, (int)hidden, g, 1, 1, 1,
              (int64_t)g * hidden * hidden, hidden, batch * steps * hidden, steps * hidden};
    RnnLaunch L{a, n, lstm, (cudaStream_t)stream};
    return dispatch_dtype(dtype, L);
}

// Whole forward: the input projection (CUDA-core grouped GEMM reading W_ih by
// stride) into the caller's workspace, then the recurrence (W_hh by stride).
int rnn_fwd_entry(bool lstm, const void* x, const void* w_ih, const void* w_hh, const void* b_ih, const void* b_hh,
                  const void* h0, const void* c0, void* out, void* h_n, void* c_n, const int64_t* wstrides,
                  void* workspace, size_t ws_bytes, int64_t n, int64_t batch, int64_t steps, int64_t input,
                  int64_t hidden, int in_layout, int out_layout, int dtype, void* stream) {
    if (n < 0 || batch < 0 || steps < 0 || hidden < 0 || input < 0)
        return set_error(WIDEK_ERR_INVALID, "rnn: negative size");
    if ((in_layout != WIDEK_LAYOUT_NFIRST && in_layout != WIDEK_LAYOUT_PACKED) ||
        (out_layout != WIDEK_LAYOUT_NFIRST && out_layout != WIDEK_LAYOUT_PACKED))
        return set_error(WIDEK_ERR_INVALID, "rnn: layouts must be N-first or packed");
    if (batch > 1024 || hidden > 4096 || steps > 0x7fffffff || n > 65535)
        return set_error(WIDEK_ERR_UNSUPPORTED, "rnn: batch=%lld hidden=%lld outside the supported range",
                         (long long)batch, (long long)hidden);
    if (n == 0 || batch == 0 || hidden == 0) return WIDEK_OK;
    if (!w_hh || !h_n || (steps > 0 && (!x || !out || !w_ih))) return set_error(WIDEK_ERR_INVALID, "rnn: null pointer");
    const int g = lstm ? 4 : 3;
    const int64_t ims = wstrides ? wstrides[0] : (int64_t)g * hidden * input;
    const int64_t irs = wstrides ? wstrides[1] : input;
    const int64_t hms = wstrides ? wstrides[2] : (int64_t)g * hidden * hidden;
    const int64_t hrs = wstrides ? wstrides[3] : hidden;
    if (ims < 0 || irs < input || hms < 0 || hrs < hidden)
        return set_error(WIDEK_ERR_INVALID, "rnn: weight strides (%lld, %lld, %lld, %lld) overlap the rows",
                         (long long)ims, (long long)irs, (long long)hms, (long long)hrs);
    const size_t need = (size_t)(n * batch * steps * g * hidden) * dtype_size(dtype);
    if (steps > 0 && (!workspace || ws_bytes < need))
        return set_error(WIDEK_ERR_INVALID, "rnn: workspace of %zu bytes needed, %zu given", need, ws_bytes);
    if (steps > 0) {
        // x rows (b, t) of model i: N-first at i*batch*T*I + (b*T + t)*I,
        // packed [batch, n*T, I] at (b*n + i)*T*I + t*I
        const bool pin = in_layout == WIDEK_LAYOUT_PACKED;
        const int64_t xms = pin ? steps * input : batch * steps * input;
        const int64_t xbs = pin ? n * steps * input : steps * input;
        const int64_t gsz = (int64_t)g * hidden;
        // fp32: the split-operand tensor-core GEMM where it fits, else the
        // CUDA-core kernel (both write the dense [n, batch*T, G*H] gates)
        int rc = WIDEK_ERR_UNSUPPORTED;
        if (dtype == WIDEK_F32)
            rc = linear_f32x3_strided(static_cast<const float*>(x), static_cast<const float*>(w_ih),
                                      static_cast<const float*>(b_ih), static_cast<float*>(workspace), n,
                                      batch * steps, input, gsz, ims, irs, xms, xbs, steps, batch * steps * gsz,
                                      steps * gsz, (cudaStream_t)stream);
        if (rc == WIDEK_ERR_UNSUPPORTED)
            rc = linear_simt_strided(x, w_ih, b_ih, workspace, n, batch * steps, input, gsz, ims, irs, dtype,
                                     WIDEK_ACT_NONE, (cudaStream_t)stream, xms, xbs, steps);
        if (rc) return rc;
    }
    const bool pout = out_layout == WIDEK_LAYOUT_PACKED;
    RnnArgs a{steps > 0 ? workspace : nullptr, w_hh, b_hh, h0, c0, out, h_n, c_n, (int)batch, (int)steps,
              (int)hidden, g, 1, 1, 1, hms, hrs, pout ? steps * hidden : batch * steps * hidden,
              pout ? n * steps * hidden : steps * hidden};
    RnnLaunch L{a, n, lstm, (cudaStream_t)stream};
    return dispatch_dtype(dtype, L);
}

}  // namespace
}  // namespace widek

extern "C" {

int widek_rnn_set_variant(int variant) {
    if (variant < 0 || variant > 1) return widek::set_error(WIDEK_ERR_INVALID, "rnn: unknown variant %d", variant);
    widek::g_rnn_variant = variant;
    return WIDEK_OK;
}

int widek_gru_recurrence(const void* gates_x, const void* w_hh, const void* b_hh, const void* h0, void* out,
                         void* h_n, int64_t n, int64_t batch, int64_t steps, int64_t hidden, int dtype,
                         void* stream) {
    return widek::rnn_entry(false, gates_x, w_hh, b_hh, h0, nullptr, out, h_n, nullptr, n, batch, steps, hidden,
                            dtype, stream);
}

int widek_lstm_recurrence(const void* gates_x, const void* w_hh, const void* b_hh, const void* h0, const void* c0,
                          void* out, void* h_n, void* c_n, int64_t n, int64_t batch, int64_t steps, int64_t hidden,
                          int dtype, void* stream) {
    return widek::rnn_entry(true, gates_x, w_hh, b_hh, h0, c0, out, h_n, c_n, n, batch, steps, hidden, dtype,
                            stream);
}

size_t widek_rnn_workspace(int lstm, int64_t n, int64_t batch, int64_t steps, int64_t hidden, int dtype) {
    if (n < 0 || batch < 0 || steps < 0 || hidden < 0) return 0;
    return (size_t)(n * batch * steps * (lstm ? 4 : 3) * hidden) * widek::dtype_size(dtype);
}

int widek_gru_fwd_ex(const void* x, const void* w_ih, const void* w_hh, const void* b_ih, const void* b_hh,
                     const void* h0, void* out, void* h_n, const int64_t* w_strides, void* workspace,
                     size_t workspace_bytes, int64_t n, int64_t batch, int64_t steps, int64_t input, int64_t hidden,
                     int in_layout, int out_layout, int dtype, void* stream) {
    return widek::rnn_fwd_entry(false, x, w_ih, w_hh, b_ih, b_hh, h0, nullptr, out, h_n, nullptr, w_strides,
                                workspace, workspace_bytes, n, batch, steps, input, hidden, in_layout, out_layout,
                                dtype, stream);
}

int widek_lstm_fwd_ex(const void* x, const void* w_ih, const void* w_hh, const void* b_ih, const void* b_hh,
                      const void* h0, const void* c0, void* out, void* h_n, void* c_n, const int64_t* w_strides,
                      void* workspace, size_t workspace_bytes, int64_t n, int64_t batch, int64_t steps,
                      int64_t input, int64_t hidden, int in_layout, int out_layout, int dtype, void* stream) {
    return widek::rnn_fwd_entry(true, x, w_ih, w_hh, b_ih, b_hh, h0, c0, out, h_n, c_n, w_strides, workspace,
                                workspace_bytes, n, batch, steps, input, hidden, in_layout, out_layout, dtype,
                                stream);
}

int widek_gru_fwd(const void* x, const void* w_ih, const void* w_hh, const void* b_ih, const void* b_hh,
                  const void* h0, void* out, void* h_n, const int64_t* w_strides, void* workspace,
                  size_t workspace_bytes, int64_t n, int64_t batch, int64_t steps, int64_t input, int64_t hidden,
                  int dtype, void* stream) {
    return widek_gru_fwd_ex(x, w_ih, w_hh, b_ih, b_hh, h0, out, h_n, w_strides, workspace, workspace_bytes, n, batch,
                            steps, input, hidden, WIDEK_LAYOUT_NFIRST, WIDEK_LAYOUT_NFIRST, dtype, stream);
}

int widek_lstm_fwd(const void* x, const void* w_ih, const void* w_hh, const void* b_ih, const void* b_hh,
                   const void* h0, const void* c0, void* out, void* h_n, void* c_n, const int64_t* w_strides,
                   void* workspace, size_t workspace_bytes, int64_t n, int64_t batch, int64_t steps, int64_t input,
                   int64_t hidden, int dtype, void* stream) {
    return widek_lstm_fwd_ex(x, w_ih, w_hh, b_ih, b_hh, h0, c0, out, h_n, c_n, w_strides, workspace, workspace_bytes,
                             n, batch, steps, input, hidden, WIDEK_LAYOUT_NFIRST, WIDEK_LAYOUT_NFIRST, dtype, stream);
}

}  // extern "C"
