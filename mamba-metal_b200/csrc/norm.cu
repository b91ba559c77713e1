// norm.cu -- RMSNorm (Sources/Kernels/rmsnorm.metal:11-81):
//   y = x * rsqrt(mean(x^2) + eps) * w
// One warp per row (one CTA per row when there are few rows): the row is
// read once into registers (up to
// kRowRegs * 32 * 4 elements; longer rows re-read from L2), squared and
// summed in FP32 with a butterfly reduction, then scaled and written in the
// output type.  HBM-bound: reads 4 or 2 bytes and writes 2 or 4 bytes per
// element.
#include "common.cuh"

namespace mb {

namespace {

constexpr int kRowRegs = 8;  // float4 chunks cached per lane (rows <= 1024 elems / lane pass)

template <typename Tin> struct Vec4;
template <> struct Vec4<float> {
    static __device__ __forceinline__ float4 load(const float *p) { return *reinterpret_cast<const float4 *>(p); }
};
template <> struct Vec4<__half> {
    static __device__ __forceinline__ float4 load(const __half *p) {
        const uint2 raw = *reinterpret_cast<const uint2 *>(p);
        const __half2 a = *reinterpret_cast<const __half2 *>(&raw.x);
        const __half2 b = *reinterpret_cast<const __half2 *>(&raw.y);
        const float2 fa = __half22float2(a), fb = __half22float2(b);
        return make_float4(fa.x, fa.y, fb.x, fb.y);
    }
};

template <typename Tout>
__device__ __forceinline__ void store4(Tout *p, float4 v);
template <>
__device__ __forceinline__ void store4<float>(float *p, float4 v) {
    *reinterpret_cast<float4 *>(p) = v;
}
template <>
__device__ __forceinline__ void store4<__half>(__half *p, float4 v) {
    __half2 a = __floats2half2_rn(v.x, v.y), b = __floats2half2_rn(v.z, v.w);
    uint2 raw;
    raw.x = *reinterpret_cast<uint32_t *>(&a);
    raw.y = *reinterpret_cast<uint32_t *>(&b);
    *reinterpret_cast<uint2 *>(p) = raw;
}

// Vectorised path: cols % 4 == 0 and 16-byte aligned rows.
template <typename Tin, typename Tout>
__global__ void rmsnorm_vec_kernel(const Tin *__restrict__ x, const float *__restrict__ w,
                                   Tout *__restrict__ y, int64_t rows, int cols, float eps) {
    const int lane = threadIdx.x & 31;
    const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (row >= rows) return;
    const Tin *xr = x + row * cols;
    Tout *yr = y + row * cols;
    const int nvec = cols >> 2;
    float4 cache[kRowRegs];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < kRowRegs; ++i) {
        const int v = lane + i * 32;
        if (v < nvec) {
            cache[i] = Vec4<Tin>::load(xr + 4 * v);
            ss = fmaf(cache[i].x, cache[i].x, ss);
            ss = fmaf(cache[i].y, cache[i].y, ss);
            ss = fmaf(cache[i].z, cache[i].z, ss);
            ss = fmaf(cache[i].w, cache[i].w, ss);
        }
    }
    for (int v = lane + kRowRegs * 32; v < nvec; v += 32) {
        const float4 c = Vec4<Tin>::load(xr + 4 * v);
        ss = fmaf(c.x, c.x, ss);
        ss = fmaf(c.y, c.y, ss);
        ss = fmaf(c.z, c.z, ss);
        ss = fmaf(c.w, c.w, ss);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float inv = rsqrtf(ss / (float)cols + eps);
    auto emit = [&](int v, float4 c) {
        float4 wv = w ? *reinterpret_cast<const float4 *>(w + 4 * v) : make_float4(1.f, 1.f, 1.f, 1.f);
        float4 o;
        o.x = (c.x * inv) * wv.x;
        o.y = (c.y * inv) * wv.y;
        o.z = (c.z * inv) * wv.z;
        o.w = (c.w * inv) * wv.w;
        store4<Tout>(yr + 4 * v, o);
    };
#pragma unroll
    for (int i = 0; i < kRowRegs; ++i) {
        const int v = lane + i * 32;
        if (v < nvec) emit(v, cache[i]);
    }
    for (int v = lane + kRowRegs * 32; v < nvec; v += 32) emit(v, Vec4<Tin>::load(xr + 4 * v));
}

// Scalar path for any cols.
template <typename Tin, typename Tout>
__global__ void rmsnorm_kernel(const Tin *__restrict__ x, const float *__restrict__ w,
                               Tout *__restrict__ y, int64_t rows, int cols, float eps) {
    const int lane = threadIdx.x & 31;
    const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (row >= rows) return;
    const Tin *xr = x + row * cols;
    Tout *yr = y + row * cols;
    float ss = 0.f;
    for (int i = lane; i < cols; i += 32) {
        const float v = cvt_f32(xr[i]);
        ss = fmaf(v, v, ss);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float inv = rsqrtf(ss / (float)cols + eps);
    for (int i = lane; i < cols; i += 32) {
        float v = cvt_f32(xr[i]) * inv;
        if (w) v *= w[i];
        yr[i] = cvt_out<Tout>(v);
    }
}

// Few rows (decode batches): one CTA per row, so a row's loads are spread
// over 256 threads instead of one warp and the grid still covers the SMs.
// Each thread caches up to kBlockRegs float4 chunks; longer rows re-read.
constexpr int kBlockThreads = 256;
constexpr int kBlockRegs = 4;

template <typename Tin, typename Tout>
__global__ void __launch_bounds__(kBlockThreads)
    rmsnorm_row_block_kernel(const Tin *__restrict__ x, const float *__restrict__ w, Tout *__restrict__ y,
                             int cols, float eps) {
    __shared__ float partial[kBlockThreads / 32];
    const int64_t row = blockIdx.x;
    const Tin *xr = x + row * cols;
    Tout *yr = y + row * cols;
    const int nvec = cols >> 2;
    float4 cache[kBlockRegs];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < kBlockRegs; ++i) {
        const int v = threadIdx.x + i * kBlockThreads;
        if (v < nvec) {
            cache[i] = Vec4<Tin>::load(xr + 4 * v);
            ss = fmaf(cache[i].x, cache[i].x, ss);
            ss = fmaf(cache[i].y, cache[i].y, ss);
            ss = fmaf(cache[i].z, cache[i].z, ss);
            ss = fmaf(cache[i].w, cache[i].w, ss);
        }
    }
    for (int v = threadIdx.x + kBlockRegs * kBlockThreads; v < nvec; v += kBlockThreads) {
        const float4 c = Vec4<Tin>::load(xr + 4 * v);
        ss = fmaf(c.x, c.x, ss);
        ss = fmaf(c.y, c.y, ss);
        ss = fmaf(c.z, c.z, ss);
        ss = fmaf(c.w, c.w, ss);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((threadIdx.x & 31) == 0) partial[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < kBlockThreads / 32; ++i) tot += partial[i];
    const float inv = rsqrtf(tot / (float)cols + eps);
    auto emit = [&](int v, float4 c) {
        c.x *= inv;
        c.y *= inv;
        c.z *= inv;
        c.w *= inv;
        if (w) {
            const float4 g = *reinterpret_cast<const float4 *>(w + 4 * v);
            c.x *= g.x;
            c.y *= g.y;
            c.z *= g.z;
            c.w *= g.w;
        }
        store4<Tout>(yr + 4 * v, c);
    };
#pragma unroll
    for (int i = 0; i < kBlockRegs; ++i) {
        const int v = threadIdx.x + i * kBlockThreads;
        if (v < nvec) emit(v, cache[i]);
    }
    for (int v = threadIdx.x + kBlockRegs * kBlockThreads; v < nvec; v += kBlockThreads)
        emit(v, Vec4<Tin>::load(xr + 4 * v));
}

template <typename Tin, typename Tout>
int launch_norm(const void *x, const float *w, void *y, int64_t rows, int cols, float eps,
                cudaStream_t st) {
    const int warps = 8;
    const int64_t blocks = ceil_div64(rows, warps);
    MB_CHECK_ARG(blocks <= 0x7fffffffLL, "rmsnorm: too many rows");
    // Rows of cols % 4 == 0 elements keep every row start 8- (half) or
    // 16-byte (float) aligned when the base pointers are 16-byte aligned.
    const bool vec = (cols % 4 == 0) && ((reinterpret_cast<uintptr_t>(x) % 16) == 0) &&
                     ((reinterpret_cast<uintptr_t>(y) % 16) == 0) &&
                     (w == nullptr || (reinterpret_cast<uintptr_t>(w) % 16) == 0);
    if (vec && rows <= 4LL * device_sm_count()) {
        rmsnorm_row_block_kernel<Tin, Tout><<<(unsigned)rows, kBlockThreads, 0, st>>>(
            static_cast<const Tin *>(x), w, static_cast<Tout *>(y), cols, eps);
        return launch_status("rmsnorm kernel");
    }
    if (vec)
        rmsnorm_vec_kernel<Tin, Tout><<<(unsigned)blocks, warps * 32, 0, st>>>(
            static_cast<const Tin *>(x), w, static_cast<Tout *>(y), rows, cols, eps);
    else
        rmsnorm_kernel<Tin, Tout><<<(unsigned)blocks, warps * 32, 0, st>>>(
            static_cast<const Tin *>(x), w, static_cast<Tout *>(y), rows, cols, eps);
    return launch_status("rmsnorm kernel");
}

}  // namespace

int rmsnorm(const void *x, const float *w, void *y, int64_t rows, int cols, float eps, int in_dt,
            int out_dt, cudaStream_t st) {
    MB_CHECK_ARG(rows >= 0 && cols >= 0, "rmsnorm: negative size");
    if (rows == 0 || cols == 0) return 0;
    MB_CHECK_ARG(x && y, "rmsnorm: null pointer");
    if (in_dt == MAMBA_F32 && out_dt == MAMBA_F32) return launch_norm<float, float>(x, w, y, rows, cols, eps, st);
    if (in_dt == MAMBA_F32 && out_dt == MAMBA_F16) return launch_norm<float, __half>(x, w, y, rows, cols, eps, st);
    if (in_dt == MAMBA_F16 && out_dt == MAMBA_F16) return launch_norm<__half, __half>(x, w, y, rows, cols, eps, st);
    if (in_dt == MAMBA_F16 && out_dt == MAMBA_F32) return launch_norm<__half, float>(x, w, y, rows, cols, eps, st);
    set_error("rmsnorm: bad dtype");
    return -1;
}

}  // namespace mb
