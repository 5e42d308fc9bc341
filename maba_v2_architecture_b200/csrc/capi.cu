// Library-wide pieces of the C ABI: version, per-thread error message,
// descriptor validation helpers.
#include "common.cuh"
#include "sa_attention.cuh"

#include <string.h>

namespace maba {

static thread_local char g_last_error[1024] = "no error";

int set_error(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
    va_end(ap);
    return code;
}

int check_launch(const char* what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        return set_error(MABA_ERR_CUDA, "%s: CUDA error %s (%s)", what, cudaGetErrorName(e),
                         cudaGetErrorString(e));
    }
    return MABA_OK;
}

int expect_shape(const maba_tensor* t, const char* name, int ndim, const int64_t* shape) {
    if (!present(t)) return set_error(MABA_ERR_INVALID, "%s: tensor is required", name);
    if (t->ndim != ndim)
        return set_error(MABA_ERR_INVALID, "%s: expected %d dims, got %d", name, ndim, t->ndim);
    for (int i = 0; i < ndim; ++i) {
        if (shape[i] >= 0 && t->shape[i] != shape[i])
            return set_error(MABA_ERR_INVALID, "%s: dim %d is %lld, expected %lld", name, i,
                             (long long)t->shape[i], (long long)shape[i]);
        if (t->stride[i] < 0)
            return set_error(MABA_ERR_INVALID, "%s: negative stride in dim %d", name, i);
    }
    return MABA_OK;
}

int expect_dtype(const maba_tensor* t, const char* name, int dtype) {
    if (t->dtype != dtype)
        return set_error(MABA_ERR_DTYPE, "%s: dtype %s, expected %s", name, dtype_name(t->dtype),
                         dtype_name(dtype));
    return MABA_OK;
}

int sm_count() {
    static int cached[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    if (dev < 0 || dev >= 64) return 148;
    if (cached[dev] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
            n = 148;
        cached[dev] = n;
    }
    return cached[dev];
}

}  // namespace maba

extern "C" int maba_abi_version(void) { return MABA_ABI_VERSION; }

extern "C" const char* maba_last_error(void) { return maba::g_last_error; }

extern "C" int maba_selftest_wait_timeout(int64_t limit_cycles, void* stream) {
    if (limit_cycles <= 0) return maba::set_error(MABA_ERR_INVALID, "selftest_wait_timeout: limit must be positive");
    return maba::wait_timeout_selftest((long long)limit_cycles, static_cast<cudaStream_t>(stream));
}

extern "C" int maba_device_error(int32_t* out, void* stream) {
    if (out == nullptr) return maba::set_error(MABA_ERR_INVALID, "device_error: out is null");
    int v = 0;
    MABA_TRY(maba::device_error_take(static_cast<cudaStream_t>(stream), &v));
    *out = v;
    return MABA_OK;
}
