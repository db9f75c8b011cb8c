// Library state behind the C-ABI: per-thread error messages, the device-side
// error word, and cached device attributes.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <atomic>
#include <mutex>

#include "common.cuh"
#include "sm100_ptx.cuh"

namespace widek {

__device__ int g_device_error = 0;

namespace {
int* g_err_ptr[64] = {nullptr};
thread_local char t_msg[512] = {0};
thread_local int t_code = 0;
std::mutex g_attr_mutex;
int g_sm_count[64] = {0};
}  // namespace

int set_error(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(t_msg, sizeof(t_msg), fmt, ap);
    va_end(ap);
    t_code = code;
    return code;
}

// Kernel launches issued by the library (every launch path ends in
// check_launch); read with widek_launch_count.
static std::atomic<long long> g_launches{0};

long long launch_count() { return g_launches.load(std::memory_order_relaxed); }

int check_launch(const char* what) {
    g_launches.fetch_add(1, std::memory_order_relaxed);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess)
        return set_error(WIDEK_ERR_CUDA, "%s: launch failed: %s", what, cudaGetErrorString(e));
    return WIDEK_OK;
}

int current_device() {
    int d = 0;
    cudaGetDevice(&d);
    return d;
}

int* device_error_ptr() {
    int d = current_device();
    if (d < 0 || d >= 64) return nullptr;
    std::lock_guard<std::mutex> lk(g_attr_mutex);
    if (!g_err_ptr[d]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_device_error) == cudaSuccess) g_err_ptr[d] = static_cast<int*>(p);
    }
    return g_err_ptr[d];
}

int sm_count(int device) {
    if (device < 0 || device >= 64) return 148;
    std::lock_guard<std::mutex> lk(g_attr_mutex);
    if (g_sm_count[device] == 0) {
        int v = 0;
        if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || v <= 0)
            v = 148;
        g_sm_count[device] = v;
    }
    return g_sm_count[device];
}

}  // namespace widek

extern "C" {

int widek_version(void) { return 100; }

int widek_last_error(char* buf, size_t len) {
    if (buf && len) {
        strncpy(buf, widek::t_msg, len - 1);
        buf[len - 1] = 0;
    }
    return widek::t_code;
}

int widek_device_error(int* code) {
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess)
        return widek::set_error(WIDEK_ERR_CUDA, "widek_device_error: %s", cudaGetErrorString(e));
    int v = 0;
    e = cudaMemcpyFromSymbol(&v, widek::g_device_error, sizeof(int));
    if (e != cudaSuccess)
        return widek::set_error(WIDEK_ERR_CUDA, "widek_device_error: %s", cudaGetErrorString(e));
    int zero = 0;
    e = cudaMemcpyToSymbol(widek::g_device_error, &zero, sizeof(int));
    if (e != cudaSuccess)
        return widek::set_error(WIDEK_ERR_CUDA, "widek_device_error: %s", cudaGetErrorString(e));
    if (code) *code = v;
    return WIDEK_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// TMA descriptor encoding through the driver entry point (no -lcuda needed).
// ---------------------------------------------------------------------------
#include <cudaTypedefs.h>

namespace widek {
namespace {
PFN_cuTensorMapEncodeTiled_v12000 g_encode_tiled = nullptr;
std::once_flag g_encode_once;
}  // namespace

int encode_tmap_tiled(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base,
                      const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                      CUtensorMapSwizzle swizzle, const uint32_t* elem_strides) {
    std::call_once(g_encode_once, []() {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_encode_tiled = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    });
    if (!g_encode_tiled) return set_error(WIDEK_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
    cuuint32_t estr[5] = {1, 1, 1, 1, 1};
    if (elem_strides)
        for (int i = 1; i < rank && i < 5; ++i) estr[i] = elem_strides[i];
    CUresult r = g_encode_tiled(map, dtype, (cuuint32_t)rank, const_cast<void*>(base),
                                reinterpret_cast<const cuuint64_t*>(dims),
                                reinterpret_cast<const cuuint64_t*>(strides_bytes),
                                reinterpret_cast<const cuuint32_t*>(box), estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(WIDEK_ERR_INVALID, "cuTensorMapEncodeTiled failed (CUresult %d)", (int)r);
    return WIDEK_OK;
}

}  // namespace widek

extern "C" long long widek_launch_count(void) { return widek::launch_count(); }

// ---------------------------------------------------------------------------
// Failure-path probe: a kernel whose mbarrier wait can never be satisfied
// (nothing arrives at the barrier) gives up after limit_ns, records
// DEV_ERR_WAIT_PROBE in the device error word and returns, as every bounded
// wait of the library does. Lets a test check, without any fault, that a
// wait that runs out ends the kernel and leaves the context usable.
// ---------------------------------------------------------------------------
namespace widek {
namespace {
__global__ void bounded_wait_probe_kernel(uint64_t limit_ns, int* err) {
    __shared__ uint64_t bar;
    __shared__ int abort_flag;
    if (threadIdx.x == 0) {
        sm100::mbar_init(&bar, 1);
        abort_flag = 0;
        sm100::mbar_init_fence();
    }
    __syncthreads();
    if (threadIdx.x == 0 && !sm100::mbar_wait_ns(&bar, 0, &abort_flag, limit_ns))
        raise_device_error(err, DEV_ERR_WAIT_PROBE);
    __syncthreads();
}
}  // namespace
}  // namespace widek

extern "C" int widek_test_bounded_wait(uint64_t limit_ns, void* stream) {
    using namespace widek;
    if (limit_ns == 0 || limit_ns > 1000000000ull)
        return set_error(WIDEK_ERR_INVALID, "widek_test_bounded_wait: limit %llu ns outside (0, 1 s]",
                         (unsigned long long)limit_ns);
    bounded_wait_probe_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(limit_ns, device_error_ptr());
    return check_launch("widek_test_bounded_wait");
}
