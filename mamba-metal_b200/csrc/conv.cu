// conv.cu -- depthwise causal conv1d (full sequence and incremental).
//
// Full sequence (Sources/Kernels/causal_conv1d.metal:21-45, with the SiLU of
// MambaRuntime.cpp:96 fused into the epilogue):
//   y[b,t,d] = SiLU( sum_{k<K} w[d,k] * x[b, t-K+1+k, d] + bias[d] )
// One thread owns one channel and a run of TC consecutive timesteps; the
// K-1 previous inputs live in a register window, so each input element is
// read once (plus a K-1 halo per run) and every warp access is a contiguous
// row segment when channels are contiguous.  Memory-bound: per (t,d) it
// reads one x and writes one y.
//
// Incremental (causal_conv1d.metal:50-82): conv over conv_state
// (oldest..newest) and the current x, then shift-append x into the state.
#include "common.cuh"
#include "scan_math.cuh"

namespace mb {

namespace {

constexpr int kConvCH = 128;  // channels per CTA
constexpr int kConvTC = 64;   // timesteps per thread run

template <typename T, int K>
__global__ void __launch_bounds__(kConvCH)
    conv1d_kernel(const T *__restrict__ x, int64_t sx0, int64_t sx1, int64_t sx2,
                  const float *__restrict__ w, const float *__restrict__ bias, T *__restrict__ y,
                  int64_t sy0, int64_t sy1, int64_t sy2, int L, int D, int silu) {
    const int d = blockIdx.x * kConvCH + threadIdx.x;
    const int b = blockIdx.z;
    const int t0 = blockIdx.y * kConvTC;
    if (d >= D) return;
    const int t1 = min(L, t0 + kConvTC);
    float wk[K];
#pragma unroll
    for (int k = 0; k < K; ++k) wk[k] = w[(int64_t)d * K + k];
    const float bv = bias ? bias[d] : 0.f;
    const T *xb = x + (int64_t)b * sx0 + (int64_t)d * sx2;
    T *yb = y + (int64_t)b * sy0 + (int64_t)d * sy2;
    float win[K];  // win[k] = x[t - K + 1 + k]
#pragma unroll
    for (int k = 0; k < K - 1; ++k) {
        const int src = t0 - K + 1 + k;
        win[k] = src >= 0 ? ld_f32(xb + (int64_t)src * sx1) : 0.f;
    }
    for (int t = t0; t < t1; ++t) {
        win[K - 1] = ld_f32(xb + (int64_t)t * sx1);
        float acc = 0.f;
#pragma unroll
        for (int k = 0; k < K; ++k) acc = fmaf(win[k], wk[k], acc);
        acc += bv;
        if (silu) acc = silu_f(acc);
        yb[(int64_t)t * sy1] = cvt_out<T>(acc);
#pragma unroll
        for (int k = 0; k < K - 1; ++k) win[k] = win[k + 1];
    }
}

template <typename T, int K>
__global__ void conv1d_step_kernel(const T *__restrict__ x, int64_t xrs, const float *__restrict__ w,
                                   const float *__restrict__ bias, T *__restrict__ y, int64_t yrs,
                                   float *__restrict__ state, int D, int silu) {
    const int d = blockIdx.x * blockDim.x + threadIdx.x;
    const int b = blockIdx.y;
    if (d >= D) return;
    float *st = state + ((int64_t)b * D + d) * (K - 1);
    float win[K];
#pragma unroll
    for (int k = 0; k < K - 1; ++k) win[k] = st[k];
    win[K - 1] = ld_f32(x + (int64_t)b * xrs + d);
    float acc = 0.f;
#pragma unroll
    for (int k = 0; k < K; ++k) acc = fmaf(win[k], w[(int64_t)d * K + k], acc);
    if (bias) acc += bias[d];
    // FP16 activations: the full-sequence kernel's SiLU (one ex2 + Newton
    // reciprocal), so decode and forward apply the same function
    if (silu) acc = sizeof(T) == 4 ? silu_f(acc) : silu_fast(acc);
    y[(int64_t)b * yrs + d] = cvt_out<T>(acc);
#pragma unroll
    for (int k = 0; k < K - 1; ++k) st[k] = win[k + 1];
}


// Vectorised full-sequence conv for channel-contiguous tensors: each thread
// owns 4 adjacent channels, one vector load per row (8 bytes for FP16,
// 16 bytes for FP32).  Pack4<T> converts a row vector to and from FP32.
template <typename T> struct Pack4;
template <> struct Pack4<__half> {
    static constexpr int kVec = 4;
    using Raw = uint2;
    static __device__ __forceinline__ void unpack(const uint2 &r, float *f) {
        const __half2 *h = reinterpret_cast<const __half2 *>(&r);
        const float2 a = __half22float2(h[0]), b = __half22float2(h[1]);
        f[0] = a.x;
        f[1] = a.y;
        f[2] = b.x;
        f[3] = b.y;
    }
    static __device__ __forceinline__ uint2 pack(const float *f) {
        uint2 r;
        __half2 *h = reinterpret_cast<__half2 *>(&r);
        h[0] = __floats2half2_rn(f[0], f[1]);
        h[1] = __floats2half2_rn(f[2], f[3]);
        return r;
    }
};
template <> struct Pack4<float> {
    static constexpr int kVec = 4;
    using Raw = uint4;
    static __device__ __forceinline__ void unpack(const uint4 &r, float *f) {
        f[0] = __uint_as_float(r.x);
        f[1] = __uint_as_float(r.y);
        f[2] = __uint_as_float(r.z);
        f[3] = __uint_as_float(r.w);
    }
    static __device__ __forceinline__ uint4 pack(const float *f) {
        return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]),
                          __float_as_uint(f[3]));
    }
};

// Vectorised-kernel tiling: a thread convolves kConvVecTC timesteps of its
// channels, kConvRows rows per batch, with the next batch's loads issued
// before the current batch is computed.  Long runs amortise the per-thread
// weight loads and the K-1 halo rows; at [64, 4096, 4096] FP16 (read as the
// x half of xz) runs of 128 reached 4.4 TB/s against 4.0 for runs of 64
// and 2.9 for runs of 8.
#ifndef MAMBA_CONV_ROWS
#define MAMBA_CONV_ROWS 8
#endif
#ifndef MAMBA_CONV_VEC_TC
#define MAMBA_CONV_VEC_TC 128
#endif
constexpr int kConvRows = MAMBA_CONV_ROWS;
constexpr int kConvVecTC = MAMBA_CONV_VEC_TC;  // timesteps per thread run

template <typename T, int K, typename Pk>
__global__ void __launch_bounds__(kConvCH)
    conv1d_vec_kernel(const T *__restrict__ x, int64_t sx0, int64_t sx1, const float *__restrict__ w,
                      const float *__restrict__ bias, T *__restrict__ y, int64_t sy0, int64_t sy1, int L, int D,
                      int silu) {
    constexpr int VEC = Pk::kVec;
    using Raw = typename Pk::Raw;
    constexpr bool PRECISE = sizeof(T) == 4;
    const int d0 = (blockIdx.y * kConvCH + threadIdx.x) * VEC;
    const int b = blockIdx.z;
    const int t0 = blockIdx.x * kConvVecTC;
    if (d0 >= D) return;
    const int t1 = min(L, t0 + kConvVecTC);
    float wk[K][VEC], bv[VEC];
#pragma unroll
    for (int c = 0; c < VEC; ++c) {
#pragma unroll
        for (int k = 0; k < K; ++k) wk[k][c] = w[(int64_t)(d0 + c) * K + k];
        bv[c] = bias ? bias[d0 + c] : 0.f;
    }
    const T *xb = x + (int64_t)b * sx0 + d0;
    T *yb = y + (int64_t)b * sy0 + d0;
    float win[K][VEC];  // win[k] = x[t - K + 1 + k]
#pragma unroll
    for (int k = 0; k < K - 1; ++k) {
        const int src = t0 - K + 1 + k;
        if (src >= 0) {
            const Raw r = *reinterpret_cast<const Raw *>(xb + (int64_t)src * sx1);
            Pk::unpack(r, win[k]);
        } else {
#pragma unroll
            for (int c = 0; c < VEC; ++c) win[k][c] = 0.f;
        }
    }
    // Software pipeline: the next batch of rows is in flight while the
    // current one is convolved and stored.
    Raw raw[kConvRows];
#pragma unroll
    for (int r = 0; r < kConvRows; ++r)
        if (t0 + r < t1) raw[r] = *reinterpret_cast<const Raw *>(xb + (int64_t)(t0 + r) * sx1);
    for (int tb = t0; tb < t1; tb += kConvRows) {
        Raw cur[kConvRows];
#pragma unroll
        for (int r = 0; r < kConvRows; ++r) cur[r] = raw[r];
        const int tn = tb + kConvRows;
#pragma unroll
        for (int r = 0; r < kConvRows; ++r)
            if (tn + r < t1) raw[r] = *reinterpret_cast<const Raw *>(xb + (int64_t)(tn + r) * sx1);
#pragma unroll
        for (int r = 0; r < kConvRows; ++r) {
            if (tb + r >= t1) break;
            Pk::unpack(cur[r], win[K - 1]);
            float out[VEC];
#pragma unroll
            for (int c = 0; c < VEC; ++c) {
                float acc = 0.f;
#pragma unroll
                for (int k = 0; k < K; ++k) acc = fmaf(win[k][c], wk[k][c], acc);
                acc += bv[c];
                if (silu) acc = PRECISE ? silu_f(acc) : silu_fast(acc);
                out[c] = acc;
            }
            *reinterpret_cast<Raw *>(yb + (int64_t)(tb + r) * sy1) = Pk::pack(out);
#pragma unroll
            for (int k = 0; k < K - 1; ++k)
#pragma unroll
                for (int c = 0; c < VEC; ++c) win[k][c] = win[k + 1][c];
        }
    }
}

template <typename T, int K>
int launch_conv_k(const void *x, const int64_t *sx, const float *w, const float *bias, void *y,
                  const int64_t *sy, int batch, int L, int D, int silu, cudaStream_t st) {
    // FP16: 4 channels (8 bytes) per thread measured 2.5x faster than 8
    // channels (16 bytes), which held 145 registers and 3 CTAs per SM.
    using Pk = Pack4<T>;
    constexpr int VEC = Pk::kVec;
    constexpr int64_t VB = VEC * (int64_t)sizeof(T);  // vector bytes
    const bool vec = sx[2] == 1 && sy[2] == 1 && D % VEC == 0 &&
                     reinterpret_cast<uintptr_t>(x) % VB == 0 && reinterpret_cast<uintptr_t>(y) % VB == 0 &&
                     (sx[1] * (int64_t)sizeof(T)) % VB == 0 && (sy[1] * (int64_t)sizeof(T)) % VB == 0 &&
                     (sx[0] * (int64_t)sizeof(T)) % VB == 0 && (sy[0] * (int64_t)sizeof(T)) % VB == 0;
    if (vec) {
        dim3 grid(ceil_div(L, kConvVecTC), ceil_div(D / VEC, kConvCH), batch);
        conv1d_vec_kernel<T, K, Pk><<<grid, kConvCH, 0, st>>>(static_cast<const T *>(x), sx[0], sx[1], w, bias,
                                                               static_cast<T *>(y), sy[0], sy[1], L, D, silu);
        return launch_status("causal_conv1d (vectorised) kernel");
    }
    dim3 grid(ceil_div(D, kConvCH), ceil_div(L, kConvTC), batch);
    conv1d_kernel<T, K><<<grid, kConvCH, 0, st>>>(static_cast<const T *>(x), sx[0], sx[1], sx[2], w,
                                                   bias, static_cast<T *>(y), sy[0], sy[1], sy[2],
                                                   L, D, silu);
    return launch_status("causal_conv1d kernel");
}

template <typename T>
int launch_conv_t(const void *x, const int64_t *sx, const float *w, const float *bias, void *y,
                  const int64_t *sy, int batch, int L, int D, int K, int silu, cudaStream_t st) {
    switch (K) {
        case 1: return launch_conv_k<T, 1>(x, sx, w, bias, y, sy, batch, L, D, silu, st);
        case 2: return launch_conv_k<T, 2>(x, sx, w, bias, y, sy, batch, L, D, silu, st);
        case 3: return launch_conv_k<T, 3>(x, sx, w, bias, y, sy, batch, L, D, silu, st);
        case 4: return launch_conv_k<T, 4>(x, sx, w, bias, y, sy, batch, L, D, silu, st);
        case 5: return launch_conv_k<T, 5>(x, sx, w, bias, y, sy, batch, L, D, silu, st);
        case 6: return launch_conv_k<T, 6>(x, sx, w, bias, y, sy, batch, L, D, silu, st);
        case 7: return launch_conv_k<T, 7>(x, sx, w, bias, y, sy, batch, L, D, silu, st);
        case 8: return launch_conv_k<T, 8>(x, sx, w, bias, y, sy, batch, L, D, silu, st);
    }
    set_error("causal_conv1d: K must be in 1..8");
    return -1;
}

template <typename T, int K>
int launch_step_k(const void *x, int64_t xrs, const float *w, const float *bias, void *y, int64_t yrs,
                  float *state, int batch, int D, int silu, cudaStream_t st) {
    dim3 grid(ceil_div(D, 128), batch);
    conv1d_step_kernel<T, K><<<grid, 128, 0, st>>>(static_cast<const T *>(x), xrs, w, bias,
                                                    static_cast<T *>(y), yrs, state, D, silu);
    return launch_status("causal_conv1d_step kernel");
}

template <typename T>
int launch_step_t(const void *x, int64_t xrs, const float *w, const float *bias, void *y, int64_t yrs,
                  float *state, int batch, int D, int K, int silu, cudaStream_t st) {
    switch (K) {
        case 1: return launch_step_k<T, 1>(x, xrs, w, bias, y, yrs, state, batch, D, silu, st);
        case 2: return launch_step_k<T, 2>(x, xrs, w, bias, y, yrs, state, batch, D, silu, st);
        case 3: return launch_step_k<T, 3>(x, xrs, w, bias, y, yrs, state, batch, D, silu, st);
        case 4: return launch_step_k<T, 4>(x, xrs, w, bias, y, yrs, state, batch, D, silu, st);
        case 5: return launch_step_k<T, 5>(x, xrs, w, bias, y, yrs, state, batch, D, silu, st);
        case 6: return launch_step_k<T, 6>(x, xrs, w, bias, y, yrs, state, batch, D, silu, st);
        case 7: return launch_step_k<T, 7>(x, xrs, w, bias, y, yrs, state, batch, D, silu, st);
        case 8: return launch_step_k<T, 8>(x, xrs, w, bias, y, yrs, state, batch, D, silu, st);
    }
    set_error("causal_conv1d_step: K must be in 1..8");
    return -1;
}

}  // namespace

int causal_conv1d(const void *x, const int64_t *sx, const float *w, const float *bias, void *y,
                  const int64_t *sy, int batch, int L, int D, int K, int silu, int dtype,
                  cudaStream_t st) {
    MB_CHECK_ARG(batch >= 0 && L >= 0 && D >= 0, "causal_conv1d: negative size");
    MB_CHECK_ARG(batch <= 65535 && ceil_div(L, kConvTC) <= 65535, "causal_conv1d: grid too large");
    if (batch == 0 || L == 0 || D == 0) return 0;
    MB_CHECK_ARG(x && w && y && sx && sy, "causal_conv1d: null pointer");
    if (dtype == MAMBA_F32) return launch_conv_t<float>(x, sx, w, bias, y, sy, batch, L, D, K, silu, st);
    if (dtype == MAMBA_F16) return launch_conv_t<__half>(x, sx, w, bias, y, sy, batch, L, D, K, silu, st);
    set_error("causal_conv1d: bad dtype");
    return -1;
}

int causal_conv1d_step(const void *x, int64_t xrs, const float *w, const float *bias, void *y,
                       int64_t yrs, float *state, int batch, int D, int K, int silu, int dtype,
                       cudaStream_t st) {
    MB_CHECK_ARG(batch >= 0 && D >= 0, "causal_conv1d_step: negative size");
    if (batch == 0 || D == 0) return 0;
    MB_CHECK_ARG(x && w && y && state, "causal_conv1d_step: null pointer");
    if (dtype == MAMBA_F32) return launch_step_t<float>(x, xrs, w, bias, y, yrs, state, batch, D, K, silu, st);
    if (dtype == MAMBA_F16) return launch_step_t<__half>(x, xrs, w, bias, y, yrs, state, batch, D, K, silu, st);
    set_error("causal_conv1d_step: bad dtype");
    return -1;
}

}  // namespace mb
