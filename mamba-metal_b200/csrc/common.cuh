// common.cuh -- shared device/host helpers for libmamba_b200.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <string>

#include "mamba.h"

namespace mb {

// ---- error reporting ------------------------------------------------------
// Thread-local last error text, surfaced by mamba_last_error().
void set_error(const std::string &msg);
const char *last_error();
void clear_error();

// ---- logging ----------------------------------------------------------------
// Lines "mamba-b200: ..." on stderr when the environment variable MAMBA_LOG
// is at least `level`: 0 (default) silent, 1 errors (every set_error), 2
// model set-up and graph captures, 3 one line per forward / step call.
int log_level();
void log_msg(int level, const char *fmt, ...) __attribute__((format(printf, 2, 3)));

#define MB_CUDA_TRY(expr)                                                          \
    do {                                                                           \
        cudaError_t _e = (expr);                                                   \
        if (_e != cudaSuccess) {                                                   \
            ::mb::set_error(std::string(#expr) + ": " + cudaGetErrorString(_e));   \
            return -1;                                                             \
        }                                                                          \
    } while (0)

#define MB_CHECK_ARG(cond, msg)                                                    \
    do {                                                                           \
        if (!(cond)) {                                                             \
            ::mb::set_error(msg);                                                  \
            return -1;                                                             \
        }                                                                          \
    } while (0)

// Launch status of the kernel just enqueued.
inline int launch_status(const char *what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        set_error(std::string(what) + ": " + cudaGetErrorString(e));
        return -1;
    }
    return 0;
}

// ---- element conversion ---------------------------------------------------
template <typename T> struct Elem;
template <> struct Elem<float> {
    static __device__ __forceinline__ float load(const float *p) { return *p; }
    static __device__ __forceinline__ float to_f32(float v) { return v; }
    static __device__ __forceinline__ float from_f32(float v) { return v; }
};
template <> struct Elem<__half> {
    static __device__ __forceinline__ float load(const __half *p) { return __half2float(*p); }
    static __device__ __forceinline__ float to_f32(__half v) { return __half2float(v); }
    static __device__ __forceinline__ __half from_f32(float v) { return __float2half_rn(v); }
};

template <typename T> __device__ __forceinline__ float ld_f32(const T *p) { return Elem<T>::load(p); }
template <typename T> __device__ __forceinline__ float cvt_f32(T v) { return Elem<T>::to_f32(v); }
template <typename T> __device__ __forceinline__ T cvt_out(float v) { return Elem<T>::from_f32(v); }

// softplus with the log1p form of selective_scan_cpu.hpp:21-23.
__device__ __forceinline__ float softplus_f(float x) { return x > 20.f ? x : log1pf(expf(x)); }

// SiLU(z) = z * sigmoid(z), the gate of mamba_block.metal:120.
__device__ __forceinline__ float silu_f(float z) { return z / (1.0f + expf(-z)); }

constexpr float kLog2e = 1.4426950408889634f;

inline size_t dtype_size(int dt) { return dt == MAMBA_F16 ? 2 : 4; }

inline int ceil_div(int a, int b) { return (a + b - 1) / b; }
inline int64_t ceil_div64(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Number of SMs of the current device (cached per device).
int device_sm_count();

}  // namespace mb
