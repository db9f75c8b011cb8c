// Chains of small wide Linear layers in one launch.
//
// A TracedWideModel of N small MLPs (e.g. Linear 64->128, ReLU, Linear 128->64)
// is a chain of wide Linears whose per-model weights and activations fit in
// one SM's shared memory. Run as separate GEMM launches (plus the boundary
// unpack and pack) it is launch- and latency-bound; here one CTA per model
// (per block of its batch rows) runs the whole chain:
//   * the CTA's input rows are read straight from the N-first [N, B, D0] or
//     the packed [B, N*D0] layout (the boundary unpack is fused);
//   * weights [Dout, Din] and biases go to shared memory as fp32 -- all
//     layers at once when they fit ("resident", one load phase with every
//     global load in flight together), else one layer at a time. A weight
//     and activation row is padded to a stride of an odd number of 16-byte
//     chunks, so float4 loads of 8 (4) consecutive rows hit different bank
//     groups;
//   * each warp tile is 16 batch rows x 8U outputs (U = 4, 2 or 1, the
//     widest that still gives all 16 warps a tile); per 4-wide k step a lane
//     loads 4 activation float4s and U weight float4s (one shared-memory
//     wavefront each) and runs 16U fp32 FMAs;
//   * activations stay in shared memory as fp32 between layers, rounded
//     through the storage dtype at each layer output as a layer-by-layer run
//     stores them;
//   * the result rows are written in the N-first or packed layout (the
//     boundary pack is fused).
// fp32 arithmetic for every storage dtype (no TF32).
//
// Replaces the per-layer path of wide_compiler/core/traced_wide.py:450-532
// (boundary unpack :467-468, one WideLinear per node with its einsum and bias
// add wide_compiler/core/primitives/wide_linear.py:165-168, the activation
// node, boundary pack :528-529) for chains whose weights fit on chip.
#include <type_traits>

#include "common.cuh"
#include "sm100_ptx.cuh"

namespace widek {
namespace {

constexpr int kChainMax = 8;
constexpr int kChainThreads = 512;
constexpr int kChainWarps = kChainThreads / 32;
constexpr int kTileRows = 16;                    // batch rows per warp tile (4 row groups x 4)
constexpr int64_t kChainSmemMax = 227 * 1024;

struct ChainArgs {
    const void* x;
    void* y;
    const void* w[kChainMax];
    const void* b[kChainMax];
    int dims[kChainMax + 1];
    int act[kChainMax];
    int wstride[kChainMax];   // padded weight row stride (floats)
    int w_off[kChainMax];     // weight offset of layer l in the weight region (floats)
    int b_off[kChainMax];     // bias offset of layer l in the bias region (floats)
    int layers, batch, n, in_packed, out_packed;
    int rows;                 // batch rows per CTA (blockIdx.y selects the block)
    int as;                   // activation row stride (floats, multiple of 4)
    int act_floats;           // one activation buffer: round4(rows) * as
    int w_floats, b_floats;   // weight / bias region sizes
    int resident;             // every layer's weights are loaded up front
    uint32_t vec;             // 16-byte row access: bit 0 x, 1 + l weight l, 9 + l bias l, 17 y
};

__host__ __device__ inline int round4(int v) { return (v + 3) & ~3; }

// Row stride of a [Dout, Din] fp32 weight tile: Din rounded up to 16-byte
// chunks, and an odd number of chunks (conflict-free quarter-warp float4s).
__host__ __device__ inline int chain_wstride(int din) {
    const int s = round4(din);
    return ((s >> 2) & 1) ? s : s + 4;
}

constexpr int kVecX = 0, kVecW = 1, kVecB = 9, kVecY = 17;
constexpr int kLoadBatch = 4;   // loads a thread issues before it stores them

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
    const uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem) : "memory");
}

__device__ __forceinline__ void cp_async_wait_all() {
    asm volatile("cp.async.commit_group;\n\tcp.async.wait_all;" ::: "memory");
}

// Copies `nrows` rows of `len` elements of T (row r at row(r) in global
// memory) into fp32 shared rows of stride `ds`, zero-filling the padding
// columns [len, round4(len)). With `vec` (16-byte aligned rows, len * sizeof(T)
// a multiple of 16): fp32 rows go by cp.async (no registers, every copy in
// flight at once; complete after cp_async_wait_all), 16-bit rows by 16-byte
// loads, kLoadBatch per thread issued before they are converted and stored.
template <typename T, typename RowFn>
__device__ __forceinline__ void chain_rows_in(float* dst, int ds, int nrows, int len, RowFn row, bool vec) {
    constexpr int V = 16 / sizeof(T);
    if (vec) {
        const int cpr = len / V;
        const int total = nrows * cpr;
        if constexpr (sizeof(T) == 4) {
            for (int c = threadIdx.x; c < total; c += kChainThreads) {
                const int r = c / cpr, q = c - r * cpr;
                cp_async16(dst + r * ds + q * V, row(r) + q * V);
            }
        } else {
            for (int base = threadIdx.x; base < total; base += kLoadBatch * kChainThreads) {
                uint4 raw[kLoadBatch];
#pragma unroll
                for (int j = 0; j < kLoadBatch; ++j) {
                    const int c = base + j * kChainThreads;
                    if (c < total) {
                        const int r = c / cpr, q = c - r * cpr;
                        raw[j] = __ldg(reinterpret_cast<const uint4*>(row(r) + q * V));
                    }
                }
#pragma unroll
                for (int j = 0; j < kLoadBatch; ++j) {
                    const int c = base + j * kChainThreads;
                    if (c < total) {
                        const int r = c / cpr, q = c - r * cpr;
                        const T* e = reinterpret_cast<const T*>(&raw[j]);
                        float* d = dst + r * ds + q * V;
#pragma unroll
                        for (int t = 0; t < V; t += 4)
                            *reinterpret_cast<float4*>(d + t) =
                                make_float4(to_f<T>(e[t]), to_f<T>(e[t + 1]), to_f<T>(e[t + 2]), to_f<T>(e[t + 3]));
                    }
                }
            }
        }
        return;
    }
    const int len4 = round4(len);
    const int total = nrows * len4;
    for (int base = threadIdx.x; base < total; base += kLoadBatch * kChainThreads) {
        float v[kLoadBatch];
#pragma unroll
        for (int j = 0; j < kLoadBatch; ++j) {
            const int c = base + j * kChainThreads;
            v[j] = 0.f;
            if (c < total) {
                const int r = c / len4, k = c - r * len4;
                if (k < len) v[j] = to_f<T>(row(r)[k]);
            }
        }
#pragma unroll
        for (int j = 0; j < kLoadBatch; ++j) {
            const int c = base + j * kChainThreads;
            if (c < total) {
                const int r = c / len4, k = c - r * len4;
                dst[r * ds + k] = v[j];
            }
        }
    }
}

// Writes `nrows` fp32 shared rows (stride ss) as rows of `len` elements of T.
template <typename T, typename RowFn>
__device__ __forceinline__ void chain_rows_out(const float* src, int ss, int nrows, int len, RowFn row, bool vec) {
    constexpr int V = 16 / sizeof(T);
    if (vec) {
        const int cpr = len / V;
        for (int c = threadIdx.x; c < nrows * cpr; c += kChainThreads) {
            const int r = c / cpr, q = c - r * cpr;
            float f[V];
#pragma unroll
            for (int t = 0; t < V; t += 4) {
                const float4 p = *reinterpret_cast<const float4*>(src + r * ss + q * V + t);
                f[t] = p.x;
                f[t + 1] = p.y;
                f[t + 2] = p.z;
                f[t + 3] = p.w;
            }
            store16<T>(row(r) + q * V, f);
        }
        return;
    }
    for (int c = threadIdx.x; c < nrows * len; c += kChainThreads) {
        const int r = c / len, k = c - r * len;
        row(r)[k] = from_f<T>(src[r * ss + k]);
    }
}

template <typename T>
__device__ __forceinline__ void chain_load_layer(const ChainArgs& a, int l, int model, float* Ws, float* bs) {
    const int din = a.dims[l], dout = a.dims[l + 1];
    const T* w = static_cast<const T*>(a.w[l]) + (size_t)model * dout * din;
    chain_rows_in<T>(Ws + a.w_off[l], a.wstride[l], dout, din, [&](int o) { return w + (size_t)o * din; },
                     (a.vec >> (kVecW + l)) & 1);
    float* bl = bs + a.b_off[l];
    if (a.b[l]) {
        const T* bias = static_cast<const T*>(a.b[l]) + (size_t)model * dout;
        chain_rows_in<T>(bl, 0, 1, dout, [&](int) { return bias; }, (a.vec >> (kVecB + l)) & 1);
    } else {
        for (int o = threadIdx.x; o < dout; o += kChainThreads) bl[o] = 0.f;
    }
}

// GELU (erf) out of line, so that the unrolled tiles stay small.
__device__ __noinline__ float chain_gelu(float v) { return gelu_erf(v); }

// One layer for this CTA's rows: nxt[r][o] = act(cur[r] . W[o] + bias[o]).
// A warp tile is 16 rows x 8U outputs; lane = 8 * rg + g computes rows
// rg + 4i (i < 4) and outputs g + 8j (j < U). Each float4 load of a k step
// touches 4 distinct activation rows (x) or 8 distinct weight rows (w), 16
// bytes each, in distinct bank groups (odd 16-byte-chunk row strides): one
// shared-memory wavefront per load, 4 + U loads per 16U FMAs.
template <typename T, int U>
__device__ __forceinline__ void chain_layer(const ChainArgs& a, int l, const float* cur, float* nxt,
                                            const float* W, const float* bias, int rows) {
    const int din = a.dims[l], dout = a.dims[l + 1], ws = a.wstride[l], as = a.as, act = a.act[l];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int rg = lane >> 3, g = lane & 7;
    const int row_tiles = (rows + kTileRows - 1) / kTileRows;
    const int out_tiles = (dout + 8 * U - 1) / (8 * U);
    const int k4n = round4(din) >> 2;
    const int dout4 = round4(dout);
    const int as4 = as >> 2, ws4 = ws >> 2;
    for (int job = warp; job < row_tiles * out_tiles; job += kChainWarps) {
        const int rt = job / out_tiles, ot = job - rt * out_tiles;
        const int b0 = rt * kTileRows + rg, o0 = ot * 8 * U + g;
        float acc[4][U];
        const float4* wr[U];
#pragma unroll
        for (int j = 0; j < U; ++j) {
            const int o = o0 + 8 * j;
            const float bv = o < dout ? bias[o] : 0.f;
#pragma unroll
            for (int i = 0; i < 4; ++i) acc[i][j] = bv;
            wr[j] = reinterpret_cast<const float4*>(W) + (o < dout ? o : dout - 1) * ws4;
        }
        // Rows past `rows` exist in the (16-row rounded) buffer; their sums
        // are never stored.
        const float4* xr = reinterpret_cast<const float4*>(cur) + b0 * as4;
#pragma unroll 4
        for (int k4 = 0; k4 < k4n; ++k4) {
            float4 xv[4], wv[U];
#pragma unroll
            for (int i = 0; i < 4; ++i) xv[i] = xr[4 * i * as4 + k4];
#pragma unroll
            for (int j = 0; j < U; ++j) wv[j] = wr[j][k4];
            // component by component: consecutive FMAs update different
            // accumulators
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < U; ++j) acc[i][j] = fmaf(xv[i].x, wv[j].x, acc[i][j]);
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < U; ++j) acc[i][j] = fmaf(xv[i].y, wv[j].y, acc[i][j]);
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < U; ++j) acc[i][j] = fmaf(xv[i].z, wv[j].z, acc[i][j]);
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < U; ++j) acc[i][j] = fmaf(xv[i].w, wv[j].w, acc[i][j]);
        }
        // activation: one uniform test per tile, branch-free per value
        if (act == WIDEK_ACT_RELU) {
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < U; ++j) acc[i][j] = acc[i][j] > 0.f ? acc[i][j] : 0.f;
        } else if (act == WIDEK_ACT_GELU) {
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < U; ++j) acc[i][j] = chain_gelu(acc[i][j]);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int r = b0 + 4 * i;
            if (r >= rows) break;
#pragma unroll
            for (int j = 0; j < U; ++j) {
                const int o = o0 + 8 * j;
                if (o < dout)
                    nxt[r * as + o] = to_f<T>(from_f<T>(acc[i][j]));
                else if (o < dout4)
                    nxt[r * as + o] = 0.f;     // zero padding read by the next layer's k loop
            }
        }
    }
}

// Outputs per lane for a layer: the widest tile that still gives every warp
// a tile (fewer FMAs per load below that, but no idle warps).
__device__ __forceinline__ int chain_pick_u(int rows, int dout) {
    const int row_tiles = (rows + kTileRows - 1) / kTileRows;
    if (row_tiles * ((dout + 31) / 32) >= kChainWarps) return 4;
    if (row_tiles * ((dout + 15) / 16) >= kChainWarps) return 2;
    return 1;
}

template <typename T>
__global__ void __launch_bounds__(kChainThreads) mlp_chain_kernel(ChainArgs a) {
    extern __shared__ __align__(16) float chain_sm[];
    const int model = blockIdx.x;
    const int row0 = blockIdx.y * a.rows;
    const int rows = min(a.rows, a.batch - row0);
    float* act0 = chain_sm;
    float* act1 = act0 + a.act_floats;
    float* Ws = act1 + a.act_floats;
    float* bs = Ws + a.w_floats;
    {
        const int d0 = a.dims[0];
        const T* x = static_cast<const T*>(a.x);
        const size_t n = a.n, B = a.batch;
        if (a.in_packed)
            chain_rows_in<T>(act0, a.as, rows, d0, [&](int r) { return x + ((size_t)(row0 + r) * n + model) * d0; },
                             (a.vec >> kVecX) & 1);
        else
            chain_rows_in<T>(act0, a.as, rows, d0, [&](int r) { return x + ((size_t)model * B + row0 + r) * d0; },
                             (a.vec >> kVecX) & 1);
    }
    if (a.resident)
        for (int l = 0; l < a.layers; ++l) chain_load_layer<T>(a, l, model, Ws, bs);
    cp_async_wait_all();
    float* cur = act0;
    float* nxt = act1;
    for (int l = 0; l < a.layers; ++l) {
        if (!a.resident) {
            __syncthreads();           // the previous layer is done reading Ws
            chain_load_layer<T>(a, l, model, Ws, bs);
            cp_async_wait_all();
        }
        __syncthreads();               // weights, biases and cur are in place
        const float* W = Ws + a.w_off[l];
        const float* bias = bs + a.b_off[l];
        const int u = chain_pick_u(rows, a.dims[l + 1]);
        if (u == 4)
            chain_layer<T, 4>(a, l, cur, nxt, W, bias, rows);
        else if (u == 2)
            chain_layer<T, 2>(a, l, cur, nxt, W, bias, rows);
        else
            chain_layer<T, 1>(a, l, cur, nxt, W, bias, rows);
        float* t = cur;
        cur = nxt;
        nxt = t;
    }
    __syncthreads();
    const int dl = a.dims[a.layers];
    T* y = static_cast<T*>(a.y);
    const size_t n = a.n, B = a.batch;
    if (a.out_packed)
        chain_rows_out<T>(cur, a.as, rows, dl, [&](int r) { return y + ((size_t)(row0 + r) * n + model) * dl; },
                          (a.vec >> kVecY) & 1);
    else
        chain_rows_out<T>(cur, a.as, rows, dl, [&](int r) { return y + ((size_t)model * B + row0 + r) * dl; },
                          (a.vec >> kVecY) & 1);
}

size_t chain_smem_bytes(const ChainArgs& a) {
    return ((size_t)2 * a.act_floats + a.w_floats + a.b_floats) * sizeof(float);
}

// Chooses the rows per CTA and the shared-memory plan; false if nothing fits.
bool chain_plan(ChainArgs& a, int sms) {
    int md4 = 0;
    int64_t w_all = 0, b_all = 0, w_max = 0, b_max = 0;
    for (int l = 0; l <= a.layers; ++l) md4 = md4 > round4(a.dims[l]) ? md4 : round4(a.dims[l]);
    for (int l = 0; l < a.layers; ++l) {
        a.wstride[l] = chain_wstride(a.dims[l]);
        const int64_t wf = (int64_t)a.dims[l + 1] * a.wstride[l], bf = round4(a.dims[l + 1]);
        w_all += wf;
        b_all += bf;
        w_max = w_max > wf ? w_max : wf;
        b_max = b_max > bf ? b_max : bf;
    }
    a.as = chain_wstride(md4);     // odd 16-byte chunks: conflict-free row-group loads
    // Rows per CTA: the whole batch, halved (to a multiple of the 16-row
    // warp tile) while the grid would leave more than half the SMs idle,
    // then (to a multiple of 4) until it fits.
    int rows = a.batch;
    while (rows > kTileRows && (int64_t)a.n * ((a.batch + rows - 1) / rows) * 2 <= sms)
        rows = ((rows + 1) / 2 + kTileRows - 1) / kTileRows * kTileRows;
    for (int pass = 0; pass < 2; ++pass) {
        const bool resident = pass == 0;
        const int64_t wf = resident ? w_all : w_max, bf = resident ? b_all : b_max;
        for (int r = rows;; r = round4((r + 1) / 2)) {
            const int64_t act = (int64_t)((r + kTileRows - 1) / kTileRows * kTileRows) * a.as;
            if ((2 * act + wf + bf) * 4 <= kChainSmemMax) {
                if ((a.batch + r - 1) / r > 65535) return false;
                a.rows = r;
                a.act_floats = (int)act;
                a.w_floats = (int)wf;
                a.b_floats = (int)bf;
                a.resident = resident ? 1 : 0;
                int wo = 0, bo = 0;
                for (int l = 0; l < a.layers; ++l) {
                    a.w_off[l] = resident ? wo : 0;
                    a.b_off[l] = resident ? bo : 0;
                    wo += a.dims[l + 1] * a.wstride[l];
                    bo += round4(a.dims[l + 1]);
                }
                return true;
            }
            if (r <= 4) break;
        }
    }
    return false;
}


// ---------------------------------------------------------------------------
// fp32 chains on the tensor cores (split bf16 operands)
//
// For fp32 chains whose layers are at most 128 wide (out) and 256 deep (in),
// with at most 256 batch rows per CTA, each layer runs as
//   D^T [dout x rows] = W [dout x din] . X^T
// on tcgen05: the weights are the A operand (M = 128; rows past dout are
// never written, and the accumulator rows they reach are dropped), the layer
// input the B operand (N = the batch rows rounded up to 16), so a small batch
// wastes little. Every fp32 operand is split into bf16 hi + lo parts and the
// product accumulated in fp32 TMEM as hi*hi + hi*lo + lo*hi (three MMAs per
// K step; each product within ~2^-17 of the fp32 one). The input rows and
// every layer's weights arrive up front as bulk copies into an fp32 staging
// area (one mbarrier), are split into the swizzled bf16 tiles, and the chain
// then costs per layer one MMA round trip and one epilogue: all 8 warps read
// the accumulator (one output feature per TMEM lane, 16 batch rows per
// read), add the bias, apply the activation and either write the next
// layer's split input tiles into shared memory or the result rows to global
// memory (N-first or packed; consecutive lanes = consecutive features, so
// the stores coalesce).
// ---------------------------------------------------------------------------
// Kernel choice for fp32 chains: 0 = the CUDA-core kernel (default), 1 =
// the tensor-core kernel wherever its plan fits. At cfg1 (32 rows x
// 64-128-64, the one size of that family whose fp32 staging plus bf16 tiles
// fit in shared memory) it takes 11.07 us against 10.76 us for the CUDA-core
// kernel: per CTA ~6 K cycles go to splitting the staged weights and ~2 K
// to each MMA round trip, against the ~4 K cycles the FFMA layers save.
// Set with widek_mlp_chain_set_variant (tests and measurements).
int g_chain_variant = 0;

constexpr int kTcThreads = 256;
constexpr int kTcMaxRows = 256;      // batch rows per CTA (N of the MMAs)
constexpr int kTcMaxIn = 256;        // din per layer (4 chunks of 64)
constexpr int kTcOut = 128;          // dout per layer (M of the MMAs)
constexpr int kTcLoadBatch = 16;

struct ChainTcPlan {
    int rows, np;                     // batch rows per CTA, N (rows rounded up to 16)
    int kc[kChainMax];                // 64-wide K chunks per layer
    uint32_t w_off[kChainMax];        // byte offset of layer l's hi tiles (lo tiles follow)
    uint32_t w_bytes, x_bytes, smem;  // weights region, one activation buffer (hi + lo), total
    uint32_t raw_w_off[kChainMax];    // fp32 staging of layer l's weights (bulk-copied) inside the raw region
    uint32_t raw_bytes;               // fp32 staging: input rows, then every layer's weights
    int tmem_cols;
};

__host__ __device__ inline uint32_t tc_tile_bytes(int rows) { return (uint32_t)rows * 128u; }   // [rows][64] bf16

bool chain_tc_plan(const ChainArgs& a, ChainTcPlan& p) {
    int max_kc = 0;
    uint32_t w = 0;
    for (int l = 0; l < a.layers; ++l) {
        if (a.dims[l + 1] > kTcOut || a.dims[l] > kTcMaxIn || a.dims[l] % 4 != 0) return false;
        p.kc[l] = (a.dims[l] + 63) / 64;
        max_kc = max_kc > p.kc[l] ? max_kc : p.kc[l];
        p.w_off[l] = w;
        w += 2u * (uint32_t)p.kc[l] * tc_tile_bytes(kTcOut);
    }
    if (a.dims[a.layers] % 4 != 0) return false;
    p.rows = a.batch < kTcMaxRows ? a.batch : kTcMaxRows;
    p.np = (p.rows + 15) / 16 * 16;
    p.w_bytes = w;
    p.x_bytes = 2u * (uint32_t)max_kc * tc_tile_bytes(p.np);
    uint32_t raw = (uint32_t)p.rows * a.dims[0] * 4;
    for (int l = 0; l < a.layers; ++l) {
        p.raw_w_off[l] = raw;
        raw += (uint32_t)a.dims[l + 1] * a.dims[l] * 4;
    }
    p.raw_bytes = raw;
    p.smem = 1024 + p.w_bytes + 2 * p.x_bytes + p.raw_bytes + 64;
    int c = 32;
    while (c < p.np) c <<= 1;
    p.tmem_cols = c;
    return p.smem <= (uint32_t)kChainSmemMax;
}

// Byte offset of element (r, kk) (kk < 64) in a 128-byte swizzled K-major
// bf16 tile: row r at r*128, 16-byte chunk kk/8 at chunk ^ (r % 8).
__device__ __forceinline__ uint32_t tc_off(int r, int kk) {
    return (uint32_t)(r * 128 + ((((kk >> 3) ^ (r & 7)) << 4) | ((kk & 7) << 1)));
}

__device__ __forceinline__ void tc_split4(uint8_t* hi, uint8_t* lo, uint32_t off, float4 v) {
    const float a4[4] = {v.x, v.y, v.z, v.w};
    uint32_t h2[2], l2[2];
#pragma unroll
    for (int q = 0; q < 2; ++q) {
        const __nv_bfloat162 h = __floats2bfloat162_rn(a4[2 * q], a4[2 * q + 1]);
        const float2 hf = __bfloat1622float2(h);
        const __nv_bfloat162 l = __floats2bfloat162_rn(a4[2 * q] - hf.x, a4[2 * q + 1] - hf.y);
        h2[q] = *reinterpret_cast<const uint32_t*>(&h);
        l2[q] = *reinterpret_cast<const uint32_t*>(&l);
    }
    *reinterpret_cast<uint2*>(hi + off) = make_uint2(h2[0], h2[1]);
    *reinterpret_cast<uint2*>(lo + off) = make_uint2(l2[0], l2[1]);
}

// Splits a [nrows][len] fp32 matrix staged densely in shared memory (row
// stride len) into kc 64-wide chunk tiles of prow rows at dst (lo tiles after
// the hi tiles); columns from len up to kc*64 become zeros. Rows from nrows
// to prow are left as they are: an MMA row (weights) or column (inputs) only
// reaches the accumulator row or column of the same index, which the
// epilogue drops. Four float4 per thread are loaded before any is stored.
__device__ __forceinline__ void tc_split_staged(uint8_t* dst, int kc, int prow, const float* raw, int nrows,
                                                int len) {
    const uint32_t tile = tc_tile_bytes(prow);
    const int per_row = kc * 16;                 // float4 per padded row
    const int total = nrows * per_row;
    for (int i0 = threadIdx.x; i0 < total; i0 += 4 * kTcThreads) {
        float4 v[4];
        int r[4], c4[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int i = i0 + u * kTcThreads;
            r[u] = i / per_row;
            c4[u] = i - r[u] * per_row;
            v[u] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (i < total && 4 * c4[u] < len)
                v[u] = *reinterpret_cast<const float4*>(raw + (size_t)r[u] * len + 4 * c4[u]);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            if (i0 + u * kTcThreads < total) {
                uint8_t* hi = dst + (uint32_t)(c4[u] >> 4) * tile;
                tc_split4(hi, hi + (uint32_t)kc * tile, tc_off(r[u], (c4[u] & 15) * 4), v[u]);
            }
        }
    }
}

// arr[i] for a kernel-parameter array by unrolled selects: a runtime index
// into a parameter array would otherwise copy the array to local memory.
template <typename T, int K>
__device__ __forceinline__ T pick(const T (&arr)[K], int i) {
    T v = arr[0];
#pragma unroll
    for (int u = 1; u < K; ++u) v = (i == u) ? arr[u] : v;
    return v;
}

__global__ void __launch_bounds__(kTcThreads, 1) mlp_chain_tc_kernel(ChainArgs a, ChainTcPlan p, int* err) {
    using namespace sm100;
    extern __shared__ uint8_t tc_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(tc_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* wreg = sm;
    uint8_t* const xbuf0 = sm + p.w_bytes;
    uint8_t* const xbuf1 = xbuf0 + p.x_bytes;
    uint8_t* rawp = sm + p.w_bytes + 2 * p.x_bytes;
    uint64_t* done = reinterpret_cast<uint64_t*>(rawp + p.raw_bytes);
    uint64_t* ld_bar = done + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 2);

    const int model = blockIdx.x;
    const int row0 = blockIdx.y * p.rows;
    const int rows = min(p.rows, a.batch - row0);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const size_t n = a.n, B = a.batch;
    const int d0 = a.dims[0];
    const float* x = static_cast<const float*>(a.x);

    if (tid == 0) {
        mbar_init(done, 1);
        mbar_init(ld_bar, 1);
        mbar_init_fence();
    }
    __syncthreads();
    // Input rows and every layer's weights as bulk copies into the fp32
    // staging area (one copy per weight matrix; the N-first input block is
    // contiguous, the packed input one copy per row), all in flight at once.
    if (warp == 0) {
        const uint64_t pol = l2_policy_evict_normal();
        if (lane == 0) {
            uint32_t bytes = (uint32_t)rows * d0 * 4;
            for (int l = 0; l < a.layers; ++l) bytes += (uint32_t)pick(a.dims, l + 1) * pick(a.dims, l) * 4;
            mbar_arrive_expect_tx(ld_bar, bytes);
            for (int l = 0; l < a.layers; ++l) {
                const int din = pick(a.dims, l), dout = pick(a.dims, l + 1);
                bulk_load(rawp + pick(p.raw_w_off, l), static_cast<const float*>(pick(a.w, l)) + (size_t)model * dout * din,
                          (uint32_t)dout * din * 4, ld_bar, pol);
            }
            if (!a.in_packed)
                bulk_load(rawp, x + ((size_t)model * B + row0) * d0, (uint32_t)rows * d0 * 4, ld_bar, pol);
        }
        __syncwarp();
        if (a.in_packed)
            for (int r = lane; r < rows; r += 32)
                bulk_load(rawp + (uint32_t)r * d0 * 4, x + ((size_t)(row0 + r) * n + model) * d0, (uint32_t)d0 * 4,
                          ld_bar, pol);
        tmem_alloc(tmem_slot, (uint32_t)p.tmem_cols);
        tmem_relinquish();
    }
    {
        const volatile int no_abort = 0;
        const bool got = mbar_wait(ld_bar, 0, &no_abort);
        if (!__syncthreads_and(got)) {
            // the copies did not land in time: report, and wait (bounded) before the CTA ends
            if (tid == 0) raise_device_error(err, DEV_ERR_GEMM_TIMEOUT);
            mbar_wait(ld_bar, 0, &no_abort);
            tc_fence_before();
            __syncthreads();
            if (warp == 0) { tc_fence_after(); tmem_dealloc(*tmem_slot, (uint32_t)p.tmem_cols); }
            return;
        }
    }
    // Split into the bf16 hi / lo tiles the MMAs read.
    tc_split_staged(xbuf0, p.kc[0], p.np, reinterpret_cast<const float*>(rawp), rows, d0);
    for (int l = 0; l < a.layers; ++l)
        tc_split_staged(wreg + pick(p.w_off, l), pick(p.kc, l), kTcOut, reinterpret_cast<const float*>(rawp + pick(p.raw_w_off, l)),
                        pick(a.dims, l + 1), pick(a.dims, l));
    fence_async_shared();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t idesc = idesc_f16(kTcOut, p.np, true);

    bool ok = true;
    for (int l = 0; l < a.layers && ok; ++l) {
        const int dout = pick(a.dims, l + 1);
        uint8_t* xin = (l & 1) ? xbuf1 : xbuf0;
        uint8_t* xout = (l & 1) ? xbuf0 : xbuf1;
        const int kc = pick(p.kc, l);
        if (tid == 0) {
            const uint32_t wt = tc_tile_bytes(kTcOut), xt = tc_tile_bytes(p.np);
            const uint8_t* wh = wreg + pick(p.w_off, l);
            const uint8_t* wl = wh + (uint32_t)kc * wt;
            const uint8_t* xh = xin;
            const uint8_t* xl = xin + (uint32_t)kc * xt;
            for (int c = 0; c < kc; ++c) {
                const uint64_t dwh = sdesc_kmajor_sw128(smem_addr(wh + c * wt)), dwl = sdesc_kmajor_sw128(smem_addr(wl + c * wt));
                const uint64_t dxh = sdesc_kmajor_sw128(smem_addr(xh + c * xt)), dxl = sdesc_kmajor_sw128(smem_addr(xl + c * xt));
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    umma_f16_ss(tmem, dwh + 2 * k, dxh + 2 * k, idesc, (c | k) != 0);
                    umma_f16_ss(tmem, dwh + 2 * k, dxl + 2 * k, idesc, 1);
                    umma_f16_ss(tmem, dwl + 2 * k, dxh + 2 * k, idesc, 1);
                }
            }
            umma_commit(done);
        }
        const volatile int no_abort = 0;
        const bool got = mbar_wait(done, (uint32_t)(l & 1), &no_abort);
        tc_fence_after();
        if (!__syncthreads_and(got)) { ok = false; break; }
        // Epilogue: all 8 warps; warp w reads TMEM lanes 32*(w%4).. (feature
        // o = TMEM lane) and every other 16-column (batch row) block, from
        // block w/4.
        {
            const int o = (warp & 3) * 32 + lane;
            const bool o_ok = o < dout;
            const float bo = (o_ok && pick(a.b, l)) ? static_cast<const float*>(pick(a.b, l))[(size_t)model * dout + o] : 0.f;
            const int act = pick(a.act, l);
            const bool last = l + 1 == a.layers;
            const uint32_t xt = tc_tile_bytes(p.np);
            const bool in_next = !last && (o >> 6) < pick(p.kc, l + 1);
            uint8_t* oh = xout + (uint32_t)(o >> 6) * xt;
            uint8_t* ol = xout + (uint32_t)pick(p.kc, last ? l : l + 1) * xt + (uint32_t)(o >> 6) * xt;
            float* y = static_cast<float*>(a.y);
#pragma unroll 1
            for (int c0 = (warp >> 2) * 16; c0 < p.np; c0 += 32) {
                uint32_t v[16];
                tmem_ld_32x32b_x16(tmem + (uint32_t)c0 + ((uint32_t)((warp & 3) * 32) << 16), v);
                tmem_ld_wait();
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const int r = c0 + j;
                    float f = __uint_as_float(v[j]) + bo;
                    if (act == WIDEK_ACT_RELU) f = f > 0.f ? f : 0.f;
                    else if (act == WIDEK_ACT_GELU) f = chain_gelu(f);
                    if (last) {
                        if (o_ok && r < rows) {
                            if (a.out_packed) y[((size_t)(row0 + r) * n + model) * dout + o] = f;
                            else y[((size_t)model * B + row0 + r) * dout + o] = f;
                        }
                    } else if (in_next) {
                        // next layer's input element (row r, k = o); features past dout
                        // and rows past the batch are zeros
                        const float fv = (o_ok && r < rows) ? f : 0.f;
                        const __nv_bfloat16 h = __float2bfloat16_rn(fv);
                        const __nv_bfloat16 lw = __float2bfloat16_rn(fv - __bfloat162float(h));
                        const uint32_t off = tc_off(r, o & 63);
                        *reinterpret_cast<__nv_bfloat16*>(oh + off) = h;
                        *reinterpret_cast<__nv_bfloat16*>(ol + off) = lw;
                    }
                }
            }
        }
        // The next layer's input tiles are written (generic proxy) before its MMAs read them.
        fence_async_shared();
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
    }
    if (!ok) raise_device_error(err, DEV_ERR_GEMM_TIMEOUT);
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, (uint32_t)p.tmem_cols);
    }
}

struct ChainLaunch {
    ChainArgs a;
    bool query;
    cudaStream_t st;
    template <typename T>
    int run() {
        if constexpr (std::is_same<T, float>::value) {
            // fp32: the tensor-core chain when selected and the layers and pointers fit it
            ChainTcPlan p{};
            bool aligned = query || (aligned16(a.x) && aligned16(a.y));
            for (int l = 0; l < a.layers && aligned && !query; ++l)
                aligned = aligned16(a.w[l]) && (!a.b[l] || aligned16(a.b[l]));
            if (g_chain_variant == 1 && aligned && chain_tc_plan(a, p)) {
                if (query) return WIDEK_OK;
                static bool attr_done[64] = {false};
                const int dev = current_device();
                if (dev >= 0 && dev < 64 && !attr_done[dev]) {
                    if (cudaFuncSetAttribute(mlp_chain_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)kChainSmemMax) != cudaSuccess)
                        return set_error(WIDEK_ERR_CUDA, "mlp_chain: cannot reserve shared memory");
                    attr_done[dev] = true;
                }
                const unsigned blocks = (unsigned)((a.batch + p.rows - 1) / p.rows);
                mlp_chain_tc_kernel<<<dim3((unsigned)a.n, blocks), kTcThreads, p.smem, st>>>(a, p,
                                                                                           device_error_ptr());
                return check_launch("widek_mlp_chain_fwd (tcgen05, split fp32)");
            }
        }
        if (!chain_plan(a, sm_count(current_device())))
            return query ? WIDEK_ERR_UNSUPPORTED
                         : set_error(WIDEK_ERR_UNSUPPORTED, "mlp_chain: the layers do not fit in shared memory");
        if (query) return WIDEK_OK;
        const size_t smem = chain_smem_bytes(a);
        auto rows16 = [](const void* p, int len) { return aligned16(p) && (len * sizeof(T)) % 16 == 0; };
        a.vec = 0;
        if (rows16(a.x, a.dims[0])) a.vec |= 1u << kVecX;
        if (rows16(a.y, a.dims[a.layers])) a.vec |= 1u << kVecY;
        for (int l = 0; l < a.layers; ++l) {
            if (rows16(a.w[l], a.dims[l])) a.vec |= 1u << (kVecW + l);
            if (a.b[l] && rows16(a.b[l], a.dims[l + 1])) a.vec |= 1u << (kVecB + l);
        }
        auto kern = mlp_chain_kernel<T>;
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
            return set_error(WIDEK_ERR_CUDA, "mlp_chain: cannot reserve %zu bytes of shared memory", smem);
        const unsigned blocks = (unsigned)((a.batch + a.rows - 1) / a.rows);
        kern<<<dim3((unsigned)a.n, blocks), kChainThreads, smem, st>>>(a);
        return check_launch("widek_mlp_chain_fwd");
    }
};

int chain_entry(const void* x, void* y, const void* const* weights, const void* const* biases, const int64_t* dims,
                const int* acts, int layers, int64_t n, int64_t batch, int in_layout, int out_layout, int dtype,
                bool query, void* stream) {
    if (layers < 1 || layers > kChainMax) return set_error(WIDEK_ERR_INVALID, "mlp_chain: 1..%d layers", kChainMax);
    if (!dims || !acts || (!query && (!weights || !biases)))
        return set_error(WIDEK_ERR_INVALID, "mlp_chain: null argument");
    if (n < 0 || batch < 0) return set_error(WIDEK_ERR_INVALID, "mlp_chain: negative size");
    if ((in_layout != WIDEK_LAYOUT_NFIRST && in_layout != WIDEK_LAYOUT_PACKED) ||
        (out_layout != WIDEK_LAYOUT_NFIRST && out_layout != WIDEK_LAYOUT_PACKED))
        return set_error(WIDEK_ERR_INVALID, "mlp_chain: layouts are N-first or packed");
    if (dtype != WIDEK_F32 && dtype != WIDEK_BF16 && dtype != WIDEK_F16)
        return set_error(WIDEK_ERR_INVALID, "unknown dtype code %d", dtype);
    ChainArgs a{};
    a.layers = layers;
    for (int l = 0; l <= layers; ++l) {
        if (dims[l] < 1) return set_error(WIDEK_ERR_INVALID, "mlp_chain: width %d is not positive", l);
        if (dims[l] > 4096) return set_error(WIDEK_ERR_UNSUPPORTED, "mlp_chain: width above 4096");
        a.dims[l] = (int)dims[l];
    }
    for (int l = 0; l < layers; ++l) {
        if (acts[l] < WIDEK_ACT_NONE || acts[l] > WIDEK_ACT_GELU)
            return set_error(WIDEK_ERR_INVALID, "mlp_chain: bad activation code %d", acts[l]);
        a.act[l] = acts[l];
    }
    if (n > 0x7fffffff || batch > 0x7fffffff) return set_error(WIDEK_ERR_UNSUPPORTED, "mlp_chain: batch or N too large");
    a.batch = (int)batch;
    a.n = (int)n;
    a.in_packed = in_layout == WIDEK_LAYOUT_PACKED;
    a.out_packed = out_layout == WIDEK_LAYOUT_PACKED;
    if (!query) {
        if (n == 0 || batch == 0) return WIDEK_OK;
        if (!x || !y) return set_error(WIDEK_ERR_INVALID, "mlp_chain: null pointer");
        for (int l = 0; l < layers; ++l) {
            if (!weights[l]) return set_error(WIDEK_ERR_INVALID, "mlp_chain: null weight %d", l);
            a.w[l] = weights[l];
            a.b[l] = biases[l];
        }
        a.x = x;
        a.y = y;
    } else if (n == 0 || batch == 0) {
        return WIDEK_OK;
    }
    ChainLaunch L{a, query, (cudaStream_t)stream};
    return dispatch_dtype(dtype, L);
}

}  // namespace
}  // namespace widek

extern "C" int widek_mlp_chain_fwd(const void* x, void* y, const void* const* weights, const void* const* biases,
                                   const int64_t* dims, const int* acts, int layers, int64_t n, int64_t batch,
                                   int in_layout, int out_layout, int dtype, void* stream) {
    return widek::chain_entry(x, y, weights, biases, dims, acts, layers, n, batch, in_layout, out_layout, dtype,
                              false, stream);
}

extern "C" int widek_mlp_chain_set_variant(int variant) {
    if (variant < 0 || variant > 1) return widek::set_error(WIDEK_ERR_INVALID, "mlp_chain: unknown variant %d", variant);
    widek::g_chain_variant = variant;
    return WIDEK_OK;
}

extern "C" int widek_mlp_chain_supported(const int64_t* dims, const int* acts, int layers, int64_t n, int64_t batch,
                                         int dtype) {
    return widek::chain_entry(nullptr, nullptr, nullptr, nullptr, dims, acts, layers, n, batch, WIDEK_LAYOUT_NFIRST,
                              WIDEK_LAYOUT_NFIRST, dtype, true, nullptr) == WIDEK_OK
               ? 1
               : 0;
}
