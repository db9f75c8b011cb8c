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
// (up to 8 CTAs), resident weights are stored four k at a time so that the
// mat-vec reads 16-byte words of W and h, and the next step's input-gate
// values are loaded into registers one step ahead.
// When the weight slice does not fit in shared memory for any cluster size,
// the kernel reads W_hh rows from global memory (L2) instead.
#include <cooperative_groups.h>

#include "common.cuh"

namespace cg = cooperative_groups;

namespace widek {
namespace {

__device__ __forceinline__ float sigmoidf_(float x) { return 1.f / (1.f + expf(-x)); }

struct RnnArgs {
    const void* gx;      // [n, batch, T, G*H]
    const void* w_hh;    // [n, G*H, H]
    const void* b_hh;    // [n, G*H] or null
    const void* h0;      // [n, batch, H] or null
    const void* c0;      // [n, batch, H] or null (LSTM)
    void* out;           // [n, batch, T, H]
    void* hn;            // [n, batch, H]
    void* cn;            // [n, batch, H] or null (LSTM)
    int batch, T, H, G, cl, w_in_smem;
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
    const T* w = static_cast<const T*>(a.w_hh) + (size_t)model * G * H * H;
    const T* bh = a.b_hh ? static_cast<const T*>(a.b_hh) + (size_t)model * G * H : nullptr;
    T* out = static_cast<T*>(a.out) + (size_t)model * B * a.T * H;

    // global row of local row lr = g * U + j
    auto grow = [&](int lr) { return (lr / U) * H + q * U + (lr % U); };

    // Resident weights: [H/4][R][4] (four consecutive k of a row in one
    // 16-byte word) when H % 4 == 0, else k-major [H][R].
    const bool vec4 = a.w_in_smem && (H % 4 == 0);
    if (a.w_in_smem) {
        for (int i = threadIdx.x; i < R * H; i += blockDim.x) {
            const int lr = i / H, k = i % H;
            const float v = to_f<T>(w[(size_t)grow(lr) * H + k]);
            if (vec4) Ws[((size_t)(k >> 2) * R + lr) * 4 + (k & 3)] = v;
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
    if (pre && (int)threadIdx.x < bu && a.T > 0) load_gx(threadIdx.x, 0, gx_next);

    for (int t = 0; t < a.T; ++t) {
        const float* hc = hbuf + (size_t)(t & 1) * B * H;
        float* hn_local = hbuf + (size_t)((t + 1) & 1) * B * H;
        float gx_cur[4] = {gx_next[0], gx_next[1], gx_next[2], gx_next[3]};
        if (pre && (int)threadIdx.x < bu && t + 1 < a.T) load_gx(threadIdx.x, t + 1, gx_next);
        // 1. recurrent mat-vec: rows x batch
        for (int lr = threadIdx.x; lr < R; lr += blockDim.x) {
            const float bias = bh ? to_f<T>(bh[grow(lr)]) : 0.f;
            for (int b0 = 0; b0 < B; b0 += 4) {
                float acc[4];
#pragma unroll
                for (int bb = 0; bb < 4; ++bb) acc[bb] = bias;
                const int nb = B - b0 < 4 ? B - b0 : 4;
                if (vec4) {
                    // 16-byte weight words (conflict-free across the warp) and
                    // 16-byte broadcasts of four h values per batch row.
                    const float4* W4 = reinterpret_cast<const float4*>(Ws);
#pragma unroll 2
                    for (int k4 = 0; k4 < H / 4; ++k4) {
                        const float4 wv = W4[(size_t)k4 * R + lr];
#pragma unroll
                        for (int bb = 0; bb < 4; ++bb) {
                            if (bb < nb) {
                                const float4 hv = reinterpret_cast<const float4*>(hc + (size_t)(b0 + bb) * H)[k4];
                                float s = acc[bb];
                                s = fmaf(wv.x, hv.x, s);
                                s = fmaf(wv.y, hv.y, s);
                                s = fmaf(wv.z, hv.z, s);
                                s = fmaf(wv.w, hv.w, s);
                                acc[bb] = s;
                            }
                        }
                    }
                } else if (a.w_in_smem) {
#pragma unroll 4
                    for (int k = 0; k < H; ++k) {
                        const float wv = Ws[(size_t)k * R + lr];
#pragma unroll
                        for (int bb = 0; bb < 4; ++bb)
                            if (bb < nb) acc[bb] = fmaf(wv, hc[(size_t)(b0 + bb) * H + k], acc[bb]);
                    }
                } else {
                    const T* wr = w + (size_t)grow(lr) * H;
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
            out[((size_t)b * a.T + t) * H + ju] = hs;
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

constexpr size_t kMaxSmem = 227 * 1024;

size_t rnn_smem(int B, int H, int G, int cl, bool w_in_smem) {
    const int U = H / cl, R = G * U;
    size_t f = (w_in_smem ? (size_t)H * R : 0) + 2 * (size_t)B * H + (size_t)B * R + (size_t)B * U;
    return f * sizeof(float);
}

template <typename T, bool LSTM>
int launch_rnn(RnnArgs a, int64_t n, cudaStream_t st) {
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
    int threads = ((rows + 31) / 32) * 32;
    const int pairs = a.batch * (a.H / cl);
    if (threads < pairs) threads = ((pairs + 31) / 32) * 32;
    if (threads > 1024) threads = 1024;     // the gate loop strides when pairs > 1024
    if (threads < 128) threads = 128;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(n * cl));
    cfg.blockDim = dim3((unsigned)threads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = cl;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
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
    RnnArgs a{gates_x, w_hh, b_hh, h0, c0, out, h_n, c_n, (int)batch, (int)steps, (int)hidden, lstm ? 4 : 3, 1, 1};
    RnnLaunch L{a, n, lstm, (cudaStream_t)stream};
    return dispatch_dtype(dtype, L);
}

}  // namespace
}  // namespace widek

extern "C" {

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

}  // extern "C"
