// runtime.cu -- library-wide host state: error messages, the device error
// word, per-device attributes and TMA tensor-map encoding.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "common.cuh"

namespace cb {

static constexpr int kMaxDevices = 64;

__device__ int g_device_error = 0;

static int *g_err_addr[kMaxDevices];
static std::once_flag g_err_once[kMaxDevices];

static thread_local char t_msg[512] = "";

void set_error(const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(t_msg, sizeof(t_msg), fmt, ap);
    va_end(ap);
}

int cuda_fail(cudaError_t e, const char *what) {
    set_error("%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
    return CB_ERR_CUDA;
}

static int current_device(int *dev) {
    cudaError_t e = cudaGetDevice(dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    if (*dev < 0 || *dev >= kMaxDevices) {
        set_error("device ordinal %d out of range", *dev);
        return CB_ERR_UNSUPPORTED;
    }
    return CB_OK;
}

int device_error_word(int **out) {
    int dev = 0;
    int st = current_device(&dev);
    if (st) return st;
    cudaError_t e = cudaSuccess;
    std::call_once(g_err_once[dev], [&] {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_device_error);
        g_err_addr[dev] = (e == cudaSuccess) ? static_cast<int *>(p) : nullptr;
    });
    if (!g_err_addr[dev]) return cuda_fail(e, "cudaGetSymbolAddress(device error word)");
    *out = g_err_addr[dev];
    return CB_OK;
}

static DeviceInfo g_info[kMaxDevices];
static std::once_flag g_info_once[kMaxDevices];

int device_info(DeviceInfo *out) {
    int dev = 0;
    int st = current_device(&dev);
    if (st) return st;
    // Bind the device's primary context to the calling thread: callers such
    // as autograd's backward threads may reach here with no current context,
    // and the driver-API tensor-map encoder needs one.
    cudaError_t se = cudaSetDevice(dev);
    if (se != cudaSuccess) return cuda_fail(se, "cudaSetDevice");
    cudaError_t err = cudaSuccess;
    std::call_once(g_info_once[dev], [&] {
        DeviceInfo d;
        err = cudaDeviceGetAttribute(&d.sm_count, cudaDevAttrMultiProcessorCount, dev);
        if (err == cudaSuccess)
            err = cudaDeviceGetAttribute(&d.max_smem_optin,
                                         cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
        g_info[dev] = d;
    });
    if (err != cudaSuccess) return cuda_fail(err, "cudaDeviceGetAttribute");
    if (g_info[dev].sm_count <= 0) {
        set_error("device %d attributes unavailable", dev);
        return CB_ERR_CUDA;
    }
    *out = g_info[dev];
    return CB_OK;
}

// cuTensorMapEncodeTiled is a driver-API call; fetch it through the runtime so
// the library does not link libcuda directly.
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                  const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                  const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

int make_tmap_lines(CUtensorMap *map, const void *base, uint64_t lines, uint32_t box_lines) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) {
        set_error("cuTensorMapEncodeTiled unavailable from the driver");
        return CB_ERR_CUDA;
    }
    cuuint64_t dims[2] = {32, lines};
    cuuint64_t strides[1] = {128};
    cuuint32_t box[2] = {32, box_lines};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void *>(base), dims,
                    strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_error("cuTensorMapEncodeTiled failed (CUresult %d)", (int)r);
        return CB_ERR_CUDA;
    }
    return CB_OK;
}

int make_tmap_2d(CUtensorMap *map, const void *base, uint64_t inner, uint64_t outer,
                 uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer,
                 CUtensorMapSwizzle swizzle) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) {
        set_error("cuTensorMapEncodeTiled unavailable from the driver");
        return CB_ERR_CUDA;
    }
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {row_bytes};
    cuuint32_t box[2] = {box_inner, box_outer};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void *>(base), dims,
                    strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_error("cuTensorMapEncodeTiled failed (CUresult %d)", (int)r);
        return CB_ERR_CUDA;
    }
    return CB_OK;
}

// One thread waits, bounded by `limit_us` microseconds, on an mbarrier that
// nothing arrives on; the bounded wait records `code` and returns.
__global__ void bounded_wait_selftest_kernel(uint32_t limit_us, int *err, int code) {
    __shared__ uint64_t bar;
    mbar_init(&bar, 1);
    fence_barrier_init();
    mbar_wait_bounded(&bar, 0, err, code, (uint64_t)limit_us * 1000ull);
}

}  // namespace cb

extern "C" int cb_selftest_bounded_wait(uint32_t limit_us, void *stream) {
    int *err = nullptr;
    int st = cb::device_error_word(&err);
    if (st) return st;
    cb::bounded_wait_selftest_kernel<<<1, 1, 0, static_cast<cudaStream_t>(stream)>>>(limit_us, err,
                                                                                      0x7f);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? CB_OK : cb::cuda_fail(e, "launch bounded_wait_selftest_kernel");
}

extern "C" const char *cb_last_error(void) { return cb::t_msg; }

extern "C" int cb_version(void) { return 100; }

extern "C" int cb_device_status(void *stream) {
    cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cb::cuda_fail(e, "cudaStreamSynchronize");
    int flag = 0;
    e = cudaMemcpyFromSymbol(&flag, cb::g_device_error, sizeof(int));
    if (e != cudaSuccess) return cb::cuda_fail(e, "cudaMemcpyFromSymbol");
    if (flag != 0) {
        int zero = 0;
        cudaMemcpyToSymbol(cb::g_device_error, &zero, sizeof(int));
        cb::set_error("device-side failure code %d (a bounded wait expired)", flag);
        return CB_ERR_DEVICE;
    }
    return CB_OK;
}
