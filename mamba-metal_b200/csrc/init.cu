// init.cu -- weight preparation kernels.
//
// * Synthetic weights from a seed (mamba_init_weights_random).  Every element
//   is a pure function of (seed, tensor tag, layer, index): a splitmix64
//   hash gives two 32-bit uniforms, and normals come from the Box-Muller
//   transform, so the fill is reproducible and independent of launch shape.
// * Layout conversion for mamba_load_weights: the blob stores projections
//   as [K, N] FP32 (x @ W, Sources/Kernels/projection.metal:25-29); the GEMMs
//   read weights K-major as [N, K] in the activation type.  The inverse
//   conversion serves mamba_save_weights.
#include "common.cuh"

namespace mb {

namespace {

__device__ __forceinline__ uint64_t splitmix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

// Uniform in (0, 1]: 24 random bits.
__device__ __forceinline__ float u01(uint32_t r) { return ((r >> 8) + 1u) * (1.0f / 16777216.0f); }

enum Dist { kNormal = 0, kUniform = 1, kDtBias = 2 };

template <typename T>
__global__ void fill_kernel(T *out, int64_t n, uint64_t key, int dist, float p0, float p1) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const uint64_t r = splitmix64(key ^ ((uint64_t)i * 0xD1B54A32D192ED03ull));
    const float u1 = u01((uint32_t)r), u2 = u01((uint32_t)(r >> 32));
    float v;
    if (dist == kNormal) {
        // Box-Muller: p0 = mean, p1 = std.
        v = p0 + p1 * sqrtf(-2.f * logf(u1)) * cospif(2.f * u2);
    } else if (dist == kUniform) {
        v = p0 + (p1 - p0) * u1;
    } else {
        // dt ~ logU[p0, p1]; store softplus^-1(dt) = dt + log(-expm1(-dt)).
        const float lo = logf(p0), hi = logf(p1);
        const float dt = expf(lo + (hi - lo) * u1);
        v = dt + logf(-expm1f(-dt));
    }
    out[i] = cvt_out<T>(v);
}

__global__ void fill_A_kernel(float *A, int D, int N) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)D * N) return;
    A[i] = -(float)(i % N + 1);
}

__global__ void fill_const_kernel(float *p, int64_t n, float v) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) p[i] = v;
}

// dst[n, k] = src[k, n]  (src [K, N] FP32 row-major).
template <typename T>
__global__ void transpose_cast_kernel(const float *__restrict__ src, T *__restrict__ dst, int K, int N) {
    __shared__ float tile[32][33];
    const int k0 = blockIdx.y * 32, n0 = blockIdx.x * 32;
    for (int r = threadIdx.y; r < 32; r += blockDim.y) {
        const int k = k0 + r, n = n0 + threadIdx.x;
        if (k < K && n < N) tile[r][threadIdx.x] = src[(int64_t)k * N + n];
    }
    __syncthreads();
    for (int r = threadIdx.y; r < 32; r += blockDim.y) {
        const int n = n0 + r, k = k0 + threadIdx.x;
        if (n < N && k < K) dst[(int64_t)n * K + k] = cvt_out<T>(tile[threadIdx.x][r]);
    }
}

// dst[k, n] = src[n, k] widened to FP32 (src [N, K] in the activation type):
// the inverse of transpose_cast, for writing weights back out as a blob.
template <typename T>
__global__ void untranspose_widen_kernel(const T *__restrict__ src, float *__restrict__ dst, int K, int N) {
    __shared__ float tile[32][33];
    const int k0 = blockIdx.x * 32, n0 = blockIdx.y * 32;
    for (int r = threadIdx.y; r < 32; r += blockDim.y) {
        const int n = n0 + r, k = k0 + threadIdx.x;
        if (n < N && k < K) tile[r][threadIdx.x] = cvt_f32(src[(int64_t)n * K + k]);
    }
    __syncthreads();
    for (int r = threadIdx.y; r < 32; r += blockDim.y) {
        const int k = k0 + r, n = n0 + threadIdx.x;
        if (k < K && n < N) dst[(int64_t)k * N + n] = tile[threadIdx.x][r];
    }
}

}  // namespace

uint64_t fill_key(uint64_t seed, int layer, int tag) {
    // Host-side mirror of splitmix64 to derive a per-tensor key.
    uint64_t z = seed ^ (0xA24BAED4963EE407ull * (uint64_t)(layer + 1)) ^ ((uint64_t)tag << 56);
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

int fill_random(void *out, int dtype, int64_t n, uint64_t key, int dist, float p0, float p1,
                cudaStream_t st) {
    if (n <= 0) return 0;
    const int threads = 256;
    const unsigned blocks = (unsigned)ceil_div64(n, threads);
    if (dtype == MAMBA_F16)
        fill_kernel<__half><<<blocks, threads, 0, st>>>(static_cast<__half *>(out), n, key, dist, p0, p1);
    else
        fill_kernel<float><<<blocks, threads, 0, st>>>(static_cast<float *>(out), n, key, dist, p0, p1);
    return launch_status("fill kernel");
}

int fill_A(float *A, int D, int N, cudaStream_t st) {
    const int64_t n = (int64_t)D * N;
    if (n <= 0) return 0;
    fill_A_kernel<<<(unsigned)ceil_div64(n, 256), 256, 0, st>>>(A, D, N);
    return launch_status("fill_A kernel");
}

// 1/A per (channel, state), or 0 where |A| <= 1e-6: the same expression the
// scan and the decode kernels evaluate per CTA, computed once per weight load
// so the decode state update (read per token) does not divide.
__global__ void a_inverse_kernel(const float *__restrict__ A, float *__restrict__ Ainv, int64_t n) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) {
        const float a = A[i];
        Ainv[i] = fabsf(a) > 1e-6f ? 1.0f / a : 0.f;
    }
}

int a_inverse(const float *A, float *Ainv, int64_t n, cudaStream_t st) {
    if (n <= 0) return 0;
    a_inverse_kernel<<<(unsigned)ceil_div64(n, 256), 256, 0, st>>>(A, Ainv, n);
    return launch_status("a_inverse kernel");
}

int fill_const(float *p, int64_t n, float v, cudaStream_t st) {
    if (n <= 0) return 0;
    fill_const_kernel<<<(unsigned)ceil_div64(n, 256), 256, 0, st>>>(p, n, v);
    return launch_status("fill_const kernel");
}

int transpose_cast(const float *src, void *dst, int dtype, int K, int N, cudaStream_t st) {
    if (K <= 0 || N <= 0) return 0;
    dim3 grid(ceil_div(N, 32), ceil_div(K, 32)), block(32, 8);
    if (dtype == MAMBA_F16)
        transpose_cast_kernel<__half><<<grid, block, 0, st>>>(src, static_cast<__half *>(dst), K, N);
    else
        transpose_cast_kernel<float><<<grid, block, 0, st>>>(src, static_cast<float *>(dst), K, N);
    return launch_status("transpose_cast kernel");
}

int untranspose_widen(const void *src, float *dst, int dtype, int K, int N, cudaStream_t st) {
    if (K <= 0 || N <= 0) return 0;
    dim3 grid(ceil_div(K, 32), ceil_div(N, 32)), block(32, 8);
    if (dtype == MAMBA_F16)
        untranspose_widen_kernel<__half><<<grid, block, 0, st>>>(static_cast<const __half *>(src), dst, K, N);
    else
        untranspose_widen_kernel<float><<<grid, block, 0, st>>>(static_cast<const float *>(src), dst, K, N);
    return launch_status("untranspose_widen kernel");
}

}  // namespace mb
