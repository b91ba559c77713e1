// carries.cu -- two small public ops beside the scan:
//
//  * propagate_tile_carries: in-place exclusive scan of per-tile affine
//    carries (a, b), the job of propagate_tile_carries_f32
//    (Sources/Kernels/prefix_scan.metal:19-40) with the pair layout that
//    kernel intends: [num_tiles, width, 2], pair p of tile t at
//    (t*width + p)*2.  Tiles compose as compose(cur, acc) = (cur.a*acc.a,
//    cur.a*acc.b + cur.b) (prefix_scan.metal:12-14).
//  * gated_silu_mul: out = silu(gate) * up, the SwiGLU gate of
//    gated_silu_mul_f32/_f16 (Sources/Kernels/gated_mlp.metal:14-41).
//
// Both are HBM-bound streams: one pass, coalesced 8- or 16-byte accesses.
#include <algorithm>

#include "common.cuh"
#include "internal.h"
#include "scan_math.cuh"

namespace mb {
namespace {

constexpr int kCarryThreads = 256;

// One thread per lane p, walking the tiles in order.  The next tile's pair
// is loaded before the current one is overwritten, so a load is always in
// flight.  Products and sums are rounded separately (no FMA contraction),
// as in the CPU restatement, so results are bit-identical to it.
__global__ void __launch_bounds__(kCarryThreads)
    propagate_tile_carries_kernel(float2 *__restrict__ c, int num_tiles, int64_t width,
                                  float2 *__restrict__ total) {
    const int64_t p = (int64_t)blockIdx.x * kCarryThreads + threadIdx.x;
    if (p >= width) return;
    float acc_a = 1.f, acc_b = 0.f;
    float2 cur = num_tiles > 0 ? c[p] : make_float2(0.f, 0.f);
    for (int t = 0; t < num_tiles; ++t) {
        float2 nxt = cur;
        if (t + 1 < num_tiles) nxt = c[(int64_t)(t + 1) * width + p];
        c[(int64_t)t * width + p] = make_float2(acc_a, acc_b);
        const float na = __fmul_rn(cur.x, acc_a);
        const float nb = __fadd_rn(__fmul_rn(cur.x, acc_b), cur.y);
        acc_a = na;
        acc_b = nb;
        cur = nxt;
    }
    if (total) total[p] = make_float2(acc_a, acc_b);
}

constexpr int kGateThreads = 256;

// FP32: the reference's arithmetic (IEEE division, exp rounded once), four
// values per thread per iteration.  FP16: eight values per 16-byte access,
// fast SiLU in FP32, rounded once to FP16 as in gated_silu_mul_f16.
template <typename T, bool VEC>
__global__ void __launch_bounds__(kGateThreads)
    gated_silu_mul_kernel(const T *__restrict__ g, const T *__restrict__ u, T *__restrict__ out, int64_t n) {
    constexpr bool F32 = sizeof(T) == 4;
    const int64_t stride = (int64_t)gridDim.x * kGateThreads;
    int64_t i = (int64_t)blockIdx.x * kGateThreads + threadIdx.x;
    if (VEC) {
        constexpr int W = 16 / sizeof(T);
        const int64_t nv = n / W;
        for (int64_t v = i; v < nv; v += stride) {
            const uint4 rg = reinterpret_cast<const uint4 *>(g)[v];
            const uint4 ru = reinterpret_cast<const uint4 *>(u)[v];
            uint4 ro;
            if (F32) {
                const float *fg = reinterpret_cast<const float *>(&rg);
                const float *fu = reinterpret_cast<const float *>(&ru);
                float *fo = reinterpret_cast<float *>(&ro);
#pragma unroll
                for (int k = 0; k < 4; ++k) fo[k] = __fmul_rn(silu_exact(fg[k]), fu[k]);
            } else {
                const __half2 *hg = reinterpret_cast<const __half2 *>(&rg);
                const __half2 *hu = reinterpret_cast<const __half2 *>(&ru);
                __half2 *ho = reinterpret_cast<__half2 *>(&ro);
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const float2 a = __half22float2(hg[k]), b = __half22float2(hu[k]);
                    ho[k] = __floats2half2_rn(silu_fast(a.x) * b.x, silu_fast(a.y) * b.y);
                }
            }
            reinterpret_cast<uint4 *>(out)[v] = ro;
        }
        i += nv * W;  // the scalar loop below takes the tail after the vectors
    }
    for (; i < n; i += stride) {
        const float a = Elem<T>::to_f32(g[i]), b = Elem<T>::to_f32(u[i]);
        const float r = F32 ? __fmul_rn(silu_exact(a), b) : silu_fast(a) * b;
        out[i] = Elem<T>::from_f32(r);
    }
}

template <typename T>
int launch_gate(const void *g, const void *u, void *out, int64_t n, cudaStream_t st) {
    const bool vec = reinterpret_cast<uintptr_t>(g) % 16 == 0 && reinterpret_cast<uintptr_t>(u) % 16 == 0 &&
                     reinterpret_cast<uintptr_t>(out) % 16 == 0;
    const int64_t work = vec ? n / (16 / sizeof(T)) + 1 : n;
    const int64_t cap = (int64_t)device_sm_count() * 8;
    const unsigned grid = (unsigned)std::max<int64_t>(1, std::min(cap, (work + kGateThreads - 1) / kGateThreads));
    auto *gp = static_cast<const T *>(g);
    auto *up = static_cast<const T *>(u);
    auto *op = static_cast<T *>(out);
    if (vec)
        gated_silu_mul_kernel<T, true><<<grid, kGateThreads, 0, st>>>(gp, up, op, n);
    else
        gated_silu_mul_kernel<T, false><<<grid, kGateThreads, 0, st>>>(gp, up, op, n);
    return launch_status("gated_silu_mul kernel");
}

}  // namespace

int propagate_tile_carries(float *carries, int num_tiles, int64_t width, float *total, cudaStream_t st) {
    MB_CHECK_ARG(num_tiles >= 0 && width >= 0, "propagate_tile_carries: negative size");
    if (width == 0) return 0;
    MB_CHECK_ARG(num_tiles == 0 || carries, "propagate_tile_carries: null carries");
    MB_CHECK_ARG(reinterpret_cast<uintptr_t>(carries) % 8 == 0 && reinterpret_cast<uintptr_t>(total) % 8 == 0,
                 "propagate_tile_carries: pairs must be 8-byte aligned");
    if (num_tiles == 0 && !total) return 0;
    const unsigned grid = (unsigned)((width + kCarryThreads - 1) / kCarryThreads);
    MB_CHECK_ARG((width + kCarryThreads - 1) / kCarryThreads <= 0x7fffffff, "propagate_tile_carries: too wide");
    propagate_tile_carries_kernel<<<grid, kCarryThreads, 0, st>>>(reinterpret_cast<float2 *>(carries), num_tiles,
                                                                   width, reinterpret_cast<float2 *>(total));
    return launch_status("propagate_tile_carries kernel");
}

int gated_silu_mul(const void *gate, const void *up, void *out, int64_t n, int dtype, cudaStream_t st) {
    MB_CHECK_ARG(n >= 0, "gated_silu_mul: negative size");
    if (n == 0) return 0;
    MB_CHECK_ARG(gate && up && out, "gated_silu_mul: null pointer");
    if (dtype == MAMBA_F32) return launch_gate<float>(gate, up, out, n, st);
    if (dtype == MAMBA_F16) return launch_gate<__half>(gate, up, out, n, st);
    set_error("gated_silu_mul: bad dtype");
    return -1;
}

}  // namespace mb
