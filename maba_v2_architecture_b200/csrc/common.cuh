// Shared helpers for the sm_100a kernels of the Maba v2 hot path:
// element conversions, the per-thread error message behind maba_last_error(),
// descriptor checks and dtype dispatch.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <stdio.h>
#include <stdarg.h>

#include "../../include/maba_b200.h"

namespace maba {

// ---------------------------------------------------------------------------
// error reporting
// ---------------------------------------------------------------------------
int set_error(int code, const char* fmt, ...);
int check_launch(const char* what);

#define MABA_TRY(expr)                 \
    do {                               \
        int _rc = (expr);              \
        if (_rc != MABA_OK) return _rc; \
    } while (0)

// ---------------------------------------------------------------------------
// element conversions (device)
// ---------------------------------------------------------------------------
template <typename T> struct Cvt;
template <> struct Cvt<float> {
    __device__ __forceinline__ static float to_f(float x) { return x; }
    __device__ __forceinline__ static double to_d(float x) { return (double)x; }
    __device__ __forceinline__ static float from_f(float x) { return x; }
    __device__ __forceinline__ static float from_d(double x) { return (float)x; }
};
template <> struct Cvt<double> {
    __device__ __forceinline__ static float to_f(double x) { return (float)x; }
    __device__ __forceinline__ static double to_d(double x) { return x; }
    __device__ __forceinline__ static double from_f(float x) { return (double)x; }
    __device__ __forceinline__ static double from_d(double x) { return x; }
};
template <> struct Cvt<__half> {
    __device__ __forceinline__ static float to_f(__half x) { return __half2float(x); }
    __device__ __forceinline__ static double to_d(__half x) { return (double)__half2float(x); }
    __device__ __forceinline__ static __half from_f(float x) { return __float2half_rn(x); }
    __device__ __forceinline__ static __half from_d(double x) { return __float2half_rn((float)x); }
};
template <> struct Cvt<__nv_bfloat16> {
    __device__ __forceinline__ static float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
    __device__ __forceinline__ static double to_d(__nv_bfloat16 x) { return (double)__bfloat162float(x); }
    __device__ __forceinline__ static __nv_bfloat16 from_f(float x) { return __float2bfloat16_rn(x); }
    __device__ __forceinline__ static __nv_bfloat16 from_d(double x) { return __float2bfloat16_rn((float)x); }
};

// Load element as accumulator type ACC (float or double).
template <typename ACC, typename T>
__device__ __forceinline__ ACC load_as(const T* p) {
    if constexpr (sizeof(ACC) == 8) return Cvt<T>::to_d(*p);
    else return Cvt<T>::to_f(*p);
}
template <typename T, typename ACC>
__device__ __forceinline__ void store_from(T* p, ACC x) {
    if constexpr (sizeof(ACC) == 8) *p = Cvt<T>::from_d(x);
    else *p = Cvt<T>::from_f(x);
}

template <typename ACC> __device__ __forceinline__ ACC exp_acc(ACC x);
template <> __device__ __forceinline__ float exp_acc<float>(float x) { return expf(x); }
template <> __device__ __forceinline__ double exp_acc<double>(double x) { return exp(x); }
template <typename ACC> __device__ __forceinline__ ACC log_acc(ACC x);
template <> __device__ __forceinline__ float log_acc<float>(float x) { return logf(x); }
template <> __device__ __forceinline__ double log_acc<double>(double x) { return log(x); }

// ---------------------------------------------------------------------------
// descriptor helpers (host)
// ---------------------------------------------------------------------------
inline bool present(const maba_tensor* t) { return t != nullptr && t->data != nullptr; }

inline const char* dtype_name(int dt) {
    switch (dt) {
        case MABA_F32: return "float32";
        case MABA_F16: return "float16";
        case MABA_BF16: return "bfloat16";
        case MABA_F64: return "float64";
        case MABA_I64: return "int64";
        case MABA_I32: return "int32";
        default: return "unknown";
    }
}

inline bool is_float_dtype(int dt) {
    return dt == MABA_F32 || dt == MABA_F16 || dt == MABA_BF16 || dt == MABA_F64;
}

// Checks that tensor `t` (named `name`) is present, has ndim dims and the
// given shape (entries < 0 are wildcards).
int expect_shape(const maba_tensor* t, const char* name, int ndim, const int64_t* shape);
int expect_dtype(const maba_tensor* t, const char* name, int dtype);

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Number of SMs of the current device (cached per device).
int sm_count();

}  // namespace maba

// Dispatch a float dtype code onto a C++ type alias `T`.
#define MABA_DISPATCH_FLOAT(DT, NAME, ...)                                              \
    [&]() -> int {                                                                      \
        switch (DT) {                                                                   \
            case MABA_F32: { using T = float; return __VA_ARGS__(); }                   \
            case MABA_F16: { using T = __half; return __VA_ARGS__(); }                  \
            case MABA_BF16: { using T = __nv_bfloat16; return __VA_ARGS__(); }          \
            case MABA_F64: { using T = double; return __VA_ARGS__(); }                  \
            default:                                                                    \
                return ::maba::set_error(MABA_ERR_DTYPE, "%s: unsupported dtype %s",    \
                                         NAME, ::maba::dtype_name(DT));                 \
        }                                                                               \
    }()
