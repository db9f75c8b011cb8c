// Shared helpers for the widek kernels: error reporting across the C-ABI,
// dtype dispatch, vector load/store helpers and bounded device-side waits.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <stddef.h>

#include <cuda.h>

#include "../../include/widek.h"

namespace widek {

// ---------------------------------------------------------------------------
// Host-side error state (thread-local message, returned codes).
// ---------------------------------------------------------------------------
int set_error(int code, const char* fmt, ...);
int check_launch(const char* what);          // counts the launch; cudaGetLastError -> code
long long launch_count();                    // launches so far (process-wide)
int sm_count(int device);                    // cached multiprocessor count
int current_device();

// Encodes a tiled TMA descriptor (dims/strides innermost first; strides are
// for dims 1..rank-1, in bytes). Out-of-range box elements read as zero.
// elem_strides (optional, rank entries, each 1..8; entry 0 is ignored): the
// traversal step per dimension; a box of boxDim[i] elements then delivers
// ceil(boxDim[i] / elem_strides[i]) elements, densely packed in shared memory.
int encode_tmap_tiled(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base,
                      const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                      CUtensorMapSwizzle swizzle, const uint32_t* elem_strides = nullptr);

// Device-side error word: kernels that give up on a bounded wait, or that
// detect an out-of-contract index, record a code there instead of trapping.
// The host reads and clears it with widek_device_error(). Kernels receive its
// device address (per device, resolved once) as an ordinary argument.
int* device_error_ptr();

// CUDA-core grouped GEMM with a strided weight: y[i] = act(x[i] @ W_i^T +
// bias[i]) where W_i is the [o, k] matrix at w + i*w_ms with rows w_rs
// elements apart; x [n, m, k], y [n, m, o] dense (gemm_simt.cu).
// Optionally x is strided too: row r of model i at
// x + i*x_ms + (r / x_rpb)*x_bs + (r % x_rpb)*k (x_ms < 0: dense [n, m, k]),
// which reads the packed [B, n*T, k] boundary layout (x_ms = T*k,
// x_bs = n*T*k, x_rpb = T) in place; y likewise with y_ms / y_bs and the
// same row blocks (y_ms < 0: dense [n, m, o]).
// fp32 grouped GEMM on the tensor cores with split bf16 operands (three
// products per K step, gemm_f32x3.cu), same strided addressing as
// linear_simt_strided (x_ms >= 0 required; x_rpb rows per block). Returns
// WIDEK_ERR_UNSUPPORTED, launching nothing, when the shapes / alignment do
// not fit it.
int linear_f32x3_strided(const float* x, const float* w, const float* bias, float* y, int64_t n, int64_t m, int64_t k,
                         int64_t o, int64_t w_ms, int64_t w_rs, int64_t x_ms, int64_t x_bs, int64_t x_rpb,
                         int64_t y_ms, int64_t y_bs, cudaStream_t st);

// Grouped GEMM on the tcgen05 kernel of linear_sm100.cu, y[i] = A_i . B_i
// (bf16/f16, fp32 accumulate, dense y [n, M, N]) with either operand read
// MN-major: A is [n, M, K] (a_mn false) or [n, K, M] (a_mn true), B is
// [n, N, K] (b_mn false) or [n, K, N] (b_mn true). Returns
// WIDEK_ERR_UNSUPPORTED, launching nothing, when the dtype, the extents
// (contiguous extents multiples of 8) or the alignment do not fit.
int gemm_tc_mn(const void* a, const void* b, void* y, int64_t n, int64_t M, int64_t K, int64_t N, bool a_mn,
               bool b_mn, int dtype, cudaStream_t st);

int linear_simt_strided(const void* x, const void* w, const void* bias, void* y, int64_t n, int64_t m, int64_t k,
                        int64_t o, int64_t w_ms, int64_t w_rs, int dtype, int act, cudaStream_t st,
                        int64_t x_ms = -1, int64_t x_bs = 0, int64_t x_rpb = 0, int64_t y_ms = -1,
                        int64_t y_bs = 0);

__device__ __forceinline__ void raise_device_error(int* err, int code) {
    if (err) atomicCAS(err, 0, code);
}

// Codes written to the device error word.
enum DeviceError : int {
    DEV_ERR_NONE = 0,
    DEV_ERR_GEMM_TIMEOUT = 101,   // tcgen05 GEMM pipeline wait ran out
    DEV_ERR_RNN_TIMEOUT = 102,    // recurrent kernel cluster wait ran out
    DEV_ERR_ATTN_TIMEOUT = 103,
    DEV_ERR_CONV_TIMEOUT = 104,
    DEV_ERR_NORM_TIMEOUT = 105,   // BatchNorm ring wait ran out
    DEV_ERR_WAIT_PROBE = 106,     // widek_test_bounded_wait: its wait ran out (expected)
    DEV_ERR_INDEX = 110,          // an index input was out of range (skipped)
};

// ---------------------------------------------------------------------------
// dtype helpers
// ---------------------------------------------------------------------------
template <typename T> struct DT;
template <> struct DT<float> {
    static __device__ __forceinline__ float to_f(float v) { return v; }
    static __device__ __forceinline__ float from_f(float v) { return v; }
};
template <> struct DT<__nv_bfloat16> {
    static __device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
    static __device__ __forceinline__ __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
};
template <> struct DT<__half> {
    static __device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
    static __device__ __forceinline__ __half from_f(float v) { return __float2half_rn(v); }
};

template <typename T> __device__ __forceinline__ float to_f(T v) { return DT<T>::to_f(v); }
template <typename T> __device__ __forceinline__ T from_f(float v) { return DT<T>::from_f(v); }

inline size_t dtype_size(int dtype) {
    switch (dtype) {
        case WIDEK_F32: return 4;
        case WIDEK_BF16: return 2;
        case WIDEK_F16: return 2;
        default: return 0;
    }
}

// 16-byte vector of T: 4 floats or 8 halfs/bf16.
template <typename T> struct Vec16 {
    static constexpr int N = 16 / sizeof(T);
    T v[N];
};

template <typename T>
__device__ __forceinline__ void load16(const T* p, float* out) {
    uint4 raw = *reinterpret_cast<const uint4*>(p);
    const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
    for (int i = 0; i < 16 / (int)sizeof(T); ++i) out[i] = to_f<T>(e[i]);
}

template <typename T>
__device__ __forceinline__ void store16(T* p, const float* in) {
    uint4 raw;
    T* e = reinterpret_cast<T*>(&raw);
#pragma unroll
    for (int i = 0; i < 16 / (int)sizeof(T); ++i) e[i] = from_f<T>(in[i]);
    *reinterpret_cast<uint4*>(p) = raw;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float gelu_erf(float x) {
    // Exact (erf) GELU, the default of torch.nn.functional.gelu.
    return 0.5f * x * (1.0f + erff(x * 0.70710678118654752f));
}

__device__ __forceinline__ float apply_act(float v, int act) {
    if (act == WIDEK_ACT_RELU) return v > 0.f ? v : 0.f;
    if (act == WIDEK_ACT_GELU) return gelu_erf(v);
    return v;
}

// Nanosecond wall clock on the device; used to bound every spin-wait.
__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

// Upper bound for any single device-side wait (a pipeline stage, a cluster
// step). Far above any legitimate wait; reaching it means a logic error.
constexpr uint64_t kWaitLimitNs = 2000000000ull;   // 2 s

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace widek

// Calls launcher.template run<T>() for the storage type named by a dtype code.
template <typename L>
inline int dispatch_dtype(int dtype, L&& launcher) {
    switch (dtype) {
        case WIDEK_F32: return launcher.template run<float>();
        case WIDEK_BF16: return launcher.template run<__nv_bfloat16>();
        case WIDEK_F16: return launcher.template run<__half>();
        default: return widek::set_error(WIDEK_ERR_INVALID, "unknown dtype code %d", dtype);
    }
}
