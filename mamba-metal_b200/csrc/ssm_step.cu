// ssm_step.cu -- single-token SSM state update for decode
// (Sources/Kernels/state_update.metal:15-57), with softplus always applied
// as in the reference oracle (Sources/CPURef/selective_scan_cpu.cpp:20),
// the dt bias added before it, and the SiLU(z) gate fused:
//   dt = softplus(delta + dt_bias)
//   h[n] = exp(dt*A[d,n]) * h[n] + (exp(dt*A)-1)/A * B[n] * x
//   y = (sum_n C[n]*h[n] + D*x) * SiLU(z)
// One thread per (b, d); its N FP32 states are a contiguous run, so a warp
// reads and writes 2 KB of state with 16-byte vector accesses.  The update
// is the same scan_step the full-sequence scan runs, so T decode steps
// reproduce a T-token forward.  HBM-bound on the state read-modify-write
// (8*N bytes per (b, d)).
#include <type_traits>

#include "common.cuh"
#include "scan_math.cuh"
#include "tma.cuh"

namespace mb {

__device__ unsigned int g_step_error = 0;

namespace {

template <int NS, typename Tx, typename Tdt, typename Tbc>
__global__ void __launch_bounds__(128)
    ssm_step_kernel(const Tx *__restrict__ x, int64_t xrs, const Tdt *__restrict__ delta, int64_t drs,
                    const float *__restrict__ dt_bias, const Tbc *__restrict__ Bm,
                    const Tbc *__restrict__ Cm, int64_t bcrs, const float *__restrict__ A,
                    const float *__restrict__ Dskip, const Tx *__restrict__ z, int64_t zrs,
                    Tx *__restrict__ y, int64_t yrs, float *__restrict__ state, int D, int N, int aligned) {
    constexpr bool PRECISE = std::is_same<Tx, float>::value;
    __shared__ __align__(16) float sBC[2 * NS];  // B[0..NS) then C[0..NS)
    const int b = blockIdx.y;
    const int d = blockIdx.x * blockDim.x + threadIdx.x;
    if (threadIdx.x < 2 * NS) {
        const int j = threadIdx.x;
        float v = 0.f;
        if (j < NS) {
            if (j < N) v = ld_f32(Bm + (int64_t)b * bcrs + j);
        } else if (j - NS < N) {
            v = ld_f32(Cm + (int64_t)b * bcrs + (j - NS));
        }
        sBC[j] = v;
    }
    __syncthreads();
    if (d >= D) return;
    float2 Ac[NS / 2], kI[NS / 2], h[NS / 2], P[NS / 2];
    const bool small = load_channel_consts<NS, PRECISE>(A, d, N, true, Ac, kI);
    float *hp = state + ((int64_t)b * D + d) * N;
    const bool vec = aligned && (NS == N) && (NS % 4 == 0);
    if (vec) {
#pragma unroll
        for (int i = 0; i < NS / 4; ++i) {
            const float4 v = reinterpret_cast<const float4 *>(hp)[i];
            h[2 * i] = make_float2(v.x, v.y);
            h[2 * i + 1] = make_float2(v.z, v.w);
        }
    } else {
#pragma unroll
        for (int q = 0; q < NS / 2; ++q) {
            h[q].x = 2 * q < N ? hp[2 * q] : 0.f;
            h[q].y = 2 * q + 1 < N ? hp[2 * q + 1] : 0.f;
        }
    }
    const float xv = ld_f32(x + (int64_t)b * xrs + d);
    float draw = ld_f32(delta + (int64_t)b * drs + d);
    if (dt_bias) draw = __fadd_rn(draw, dt_bias[d]);
    const float dt = scan_softplus<PRECISE>(draw);
    const float s = small ? scan_step<NS, false, PRECISE, true>(xv, dt, sBC, h, Ac, kI, P)
                          : scan_step<NS, false, PRECISE, false>(xv, dt, sBC, h, Ac, kI, P);
    if (vec) {
#pragma unroll
        for (int i = 0; i < NS / 4; ++i)
            reinterpret_cast<float4 *>(hp)[i] = make_float4(h[2 * i].x, h[2 * i].y, h[2 * i + 1].x, h[2 * i + 1].y);
    } else {
#pragma unroll
        for (int q = 0; q < NS / 2; ++q) {
            if (2 * q < N) hp[2 * q] = h[q].x;
            if (2 * q + 1 < N) hp[2 * q + 1] = h[q].y;
        }
    }
    const float dsk = Dskip ? Dskip[d] : 0.f;
    const float gate = z ? scan_silu<PRECISE>(ld_f32(z + (int64_t)b * zrs + d)) : 1.f;
    y[(int64_t)b * yrs + d] = cvt_out<Tx>(scan_output<PRECISE>(s, dsk, xv, gate));
}

// FP16 fast path: four threads per channel, each owning NS/4 consecutive
// states, so lane l of a warp reads and writes bytes [16 l, 16 l + 16) of a
// contiguous 512-byte run (full coalescing).  Each thread serves R batch
// rows of its channel: A and 1/A are loaded once, and the R state vectors
// are all in flight before any is used (with one row per thread too few
// bytes are in flight per SM to cover HBM latency).  Each state sees exactly
// the per-state operations of scan_step (fast mode); the four partial sums
// of C*h are combined with two butterfly shuffles.
template <int NS, int R, typename Tx, typename Tdt, typename Tbc>
__global__ void __launch_bounds__(128)
    ssm_step_quad_kernel(const Tx *__restrict__ x, int64_t xrs, const Tdt *__restrict__ delta, int64_t drs,
                         const float *__restrict__ dt_bias, const Tbc *__restrict__ Bm,
                         const Tbc *__restrict__ Cm, int64_t bcrs, const float *__restrict__ A,
                         const float *__restrict__ Dskip, const Tx *__restrict__ z, int64_t zrs,
                         Tx *__restrict__ y, int64_t yrs, float *__restrict__ state, int batch, int D, int N,
                         int aligned) {
    constexpr int S = NS / 4;  // states per thread
    static_assert(R * 2 * NS <= 128, "B/C staging uses one thread per value");
    __shared__ __align__(16) float sBC[R][2 * NS];
    const int b0 = blockIdx.y * R;
    const int q = threadIdx.x & 3;
    const int d = blockIdx.x * 32 + (threadIdx.x >> 2);
    if (threadIdx.x < R * 2 * NS) {
        const int r = threadIdx.x / (2 * NS), j = threadIdx.x % (2 * NS);
        const int b = b0 + r;
        float v = 0.f;
        if (b < batch) {
            if (j < NS) {
                if (j < N) v = ld_f32(Bm + (int64_t)b * bcrs + j);
            } else if (j - NS < N) {
                v = ld_f32(Cm + (int64_t)b * bcrs + (j - NS));
            }
        }
        sBC[r][j] = v;
    }
    // Lanes of channels past D (and rows past the batch) stay to the end
    // (every lane of the warp takes part in the shuffles below); only their
    // memory accesses are skipped.
    const bool valid = d < D;
    const int dd = valid ? d : 0;
    // 16-byte vector accesses to A and the state when both are 16-byte
    // aligned (checked on the host) and the state rows are exactly NS long.
    const bool vec = aligned && (NS == N) && (S == 4);
    float ac[S], kI[S];
    if (vec) {
        const float4 a4 = valid ? *reinterpret_cast<const float4 *>(A + (int64_t)dd * N + q * S)
                                : make_float4(0.f, 0.f, 0.f, 0.f);
        const float av[4] = {a4.x, a4.y, a4.z, a4.w};
#pragma unroll
        for (int j = 0; j < S; ++j) {
            ac[j] = av[j & 3] * kLog2e;
            kI[j] = fabsf(av[j & 3]) > 1e-6f ? 1.0f / av[j & 3] : 0.f;
        }
    } else {
#pragma unroll
        for (int j = 0; j < S; ++j) {
            const int n = q * S + j;
            const float a = (valid && n < N) ? A[(int64_t)dd * N + n] : 0.f;
            ac[j] = a * kLog2e;
            kI[j] = fabsf(a) > 1e-6f ? 1.0f / a : 0.f;
        }
    }
    float h[R][S], xv[R], draw[R];
    bool rv[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const int b = b0 + r;
        rv[r] = valid && b < batch;
        const int bb = rv[r] ? b : 0;
        const float *hp = state + ((int64_t)bb * D + dd) * N + q * S;
#pragma unroll
        for (int j = 0; j < S; ++j) h[r][j] = 0.f;
        if (rv[r]) {
            if (vec) {
                const float4 v = *reinterpret_cast<const float4 *>(hp);
                h[r][0] = v.x;
                h[r][S > 1 ? 1 : 0] = v.y;
                h[r][S > 2 ? 2 : 0] = v.z;
                h[r][S > 3 ? 3 : 0] = v.w;
            } else {
#pragma unroll
                for (int j = 0; j < S; ++j) h[r][j] = q * S + j < N ? hp[j] : 0.f;
            }
        }
        xv[r] = rv[r] ? ld_f32(x + (int64_t)bb * xrs + dd) : 0.f;
        draw[r] = rv[r] ? ld_f32(delta + (int64_t)bb * drs + dd) : 0.f;
    }
    const float bias = (dt_bias && valid) ? dt_bias[dd] : 0.f;
    __syncthreads();  // sBC
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const float dt = softplus_fast(dt_bias ? __fadd_rn(draw[r], bias) : draw[r]);
        float yp = 0.f;
#pragma unroll
        for (int j = 0; j < S; ++j) {
            const int n = q * S + j;
            const float a = ex2_approx(dt * ac[j]);
            h[r][j] = state_update(a, xv[r] * sBC[r][n], kI[j], dt, h[r][j]);
            yp = fmaf(sBC[r][NS + n], h[r][j], yp);
        }
        yp += __shfl_xor_sync(0xffffffffu, yp, 1);
        yp += __shfl_xor_sync(0xffffffffu, yp, 2);
        if (!rv[r]) continue;
        const int b = b0 + r;
        float *hp = state + ((int64_t)b * D + d) * N + q * S;
        if (vec) {
            *reinterpret_cast<float4 *>(hp) =
                make_float4(h[r][0], h[r][S > 1 ? 1 : 0], h[r][S > 2 ? 2 : 0], h[r][S > 3 ? 3 : 0]);
        } else {
#pragma unroll
            for (int j = 0; j < S; ++j)
                if (q * S + j < N) hp[j] = h[r][j];
        }
        if (q == 0) {
            const float dsk = Dskip ? Dskip[d] : 0.f;
            const float gate = z ? silu_fast(ld_f32(z + (int64_t)b * zrs + d)) : 1.f;
            y[(int64_t)b * yrs + d] = cvt_out<Tx>(fmaf(dsk, xv[r], yp) * gate);
        }
    }
}

// Bulk-copy variant of the kernel above for the common decode layout (FP16
// activations, exactly 16 FP32 states per channel, 32-channel blocks
// aligned): a CTA serves 32 channels x RB batch rows.  One thread issues RB
// bulk copies of the CTA's 2 KB state run of each row into shared memory
// (each completing on its own mbarrier), so RB x 2 KB per CTA and twelve
// CTAs per SM are in flight at once instead of 16 B per thread; the rows
// are updated in shared memory as they land (the same per-state operations
// as above, so decode still equals the scan bit for bit) and go back with
// bulk stores.  x, delta, z of all rows are loaded before the first wait.
constexpr unsigned kErrStepTimeout = 32u;  // bit 5 of the device status

template <int RB, typename Tx, typename Tdt, typename Tbc>
__global__ void __launch_bounds__(128, 12)
    ssm_step_bulk_kernel(const Tx *__restrict__ x, int64_t xrs, const Tdt *__restrict__ delta, int64_t drs,
                         const float *__restrict__ dt_bias, const Tbc *__restrict__ Bm,
                         const Tbc *__restrict__ Cm, int64_t bcrs, const float *__restrict__ A,
                         const float *__restrict__ Dskip, const Tx *__restrict__ z, int64_t zrs,
                         Tx *__restrict__ y, int64_t yrs, float *__restrict__ state, int batch, int D,
                         const float *__restrict__ A_inv) {
    constexpr int NS = 16, S = 4, kRowFloats = 32 * NS;  // one row's state run: 32 channels x 16 states
    extern __shared__ __align__(128) unsigned char smem[];
    float *sst = reinterpret_cast<float *>(smem);  // [RB][32][16]
    float *sBC = sst + RB * kRowFloats;            // [RB][2*NS]: B then C
    uint64_t *bars = reinterpret_cast<uint64_t *>(sBC + RB * 2 * NS);
    const int tid = threadIdx.x, q = tid & 3, cl = tid >> 2;
    const int d0 = blockIdx.x * 32, d = d0 + cl;
    const int b0 = blockIdx.y * RB;
    const int nr = min(RB, batch - b0);
    if (tid == 0) {
        for (int r = 0; r < RB; ++r) mbar_init(&bars[r], 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (tid == 0) {
        for (int r = 0; r < nr; ++r) {
            mbar_arrive_expect_tx(&bars[r], kRowFloats * 4);
            bulk_load(sst + r * kRowFloats, state + ((int64_t)(b0 + r) * D + d0) * NS, kRowFloats * 4, &bars[r]);
        }
    }
    for (int e = tid; e < nr * 2 * NS; e += 128) {
        const int r = e / (2 * NS), j = e % (2 * NS);
        const Tbc *src = j < NS ? Bm + (int64_t)(b0 + r) * bcrs + j : Cm + (int64_t)(b0 + r) * bcrs + (j - NS);
        sBC[r * 2 * NS + j] = ld_f32(src);
    }
    const float4 a4 = *reinterpret_cast<const float4 *>(A + (int64_t)d * NS + q * S);
    const float av[4] = {a4.x, a4.y, a4.z, a4.w};
    float ac[S], kI[S];
    if (A_inv) {
        // precomputed by the model at weight load (same expression, same bits)
        const float4 k4 = *reinterpret_cast<const float4 *>(A_inv + (int64_t)d * NS + q * S);
        kI[0] = k4.x;
        kI[1] = k4.y;
        kI[2] = k4.z;
        kI[3] = k4.w;
    }
#pragma unroll
    for (int j = 0; j < S; ++j) {
        ac[j] = av[j] * kLog2e;
        if (!A_inv) kI[j] = fabsf(av[j]) > 1e-6f ? 1.0f / av[j] : 0.f;
    }
    const float bias = dt_bias ? dt_bias[d] : 0.f;
    const float dsk = Dskip ? Dskip[d] : 0.f;
    // Lane q of a channel's quad evaluates softplus(delta) and SiLU(z) of
    // row q only (one each instead of four); the rows' dt values reach the
    // other lanes by shuffle, and lane q writes row q's output.
    static_assert(RB <= 4, "one row per lane of the quad");
    float xv[RB];
#pragma unroll
    for (int r = 0; r < RB; ++r) xv[r] = ld_f32(x + (int64_t)(b0 + (r < nr ? r : 0)) * xrs + d);
    const int bq = b0 + (q < nr ? q : 0);
    const float draw_q = ld_f32(delta + (int64_t)bq * drs + d);
    const float zq = z ? ld_f32(z + (int64_t)bq * zrs + d) : 0.f;
    __syncthreads();  // sBC
    const float dt_q = softplus_fast(dt_bias ? __fadd_rn(draw_q, bias) : draw_q);
    const float gate_q = z ? silu_fast(zq) : 1.f;
    const int quad0 = (tid & 31) & ~3;
    bool ok = true;
#pragma unroll
    for (int r = 0; r < RB; ++r) {
        if (r >= nr) break;
        // warp-uniform verdict: the shuffles below need every lane
        if (!__all_sync(0xffffffffu, mbar_wait_bounded(&bars[r], 0u))) {
            ok = false;
            break;
        }
        float *hp = sst + r * kRowFloats + cl * NS + q * S;
        const float4 hv = *reinterpret_cast<const float4 *>(hp);
        float h[S] = {hv.x, hv.y, hv.z, hv.w};
        const float dt = __shfl_sync(0xffffffffu, dt_q, quad0 + r);
        const float *bc = sBC + r * 2 * NS;
        float yp = 0.f;
#pragma unroll
        for (int j = 0; j < S; ++j) {
            const int n = q * S + j;
            const float a = ex2_approx(dt * ac[j]);
            h[j] = state_update(a, xv[r] * bc[n], kI[j], dt, h[j]);
            yp = fmaf(bc[NS + n], h[j], yp);
        }
        *reinterpret_cast<float4 *>(hp) = make_float4(h[0], h[1], h[2], h[3]);
        yp += __shfl_xor_sync(0xffffffffu, yp, 1);
        yp += __shfl_xor_sync(0xffffffffu, yp, 2);
        if (q == r) y[(int64_t)(b0 + r) * yrs + d] = cvt_out<Tx>(fmaf(dsk, xv[r], yp) * gate_q);
    }
    fence_proxy_async_smem();  // the updated rows are read by the bulk stores
    const bool aborted = __syncthreads_or(!ok);
    if (tid == 0) {
        if (aborted) {
            atomicOr(&g_step_error, kErrStepTimeout);
            // copies still landing in this CTA's shared memory finish first
            for (int r = 0; r < nr; ++r) mbar_wait_bounded(&bars[r], 0u);
        } else {
            for (int r = 0; r < nr; ++r)
                bulk_store(state + ((int64_t)(b0 + r) * D + d0) * NS, sst + r * kRowFloats, kRowFloats * 4);
            bulk_commit_group();
            bulk_wait_group_read<0>();
        }
    }
}

// Rows per CTA and resident CTAs, measured on the 64-layer decode (batch 256,
// 5120 channels): 4 rows with 12 CTAs per SM 43.5 us per layer; 8 rows / 8
// CTAs 48.0; 4 / 16 48.6; 2 / 16 49.2; 16 rows 57.6; the four-lanes kernel
// above 52.
constexpr int kStepBulkRows = 4;

template <int NS, typename Tx, typename Tdt, typename Tbc>
int launch_step(const void *x, int64_t xrs, const void *delta, int64_t drs, const float *dt_bias,
                const void *B, const void *C, int64_t bcrs, const float *A, const float *Dskip,
                const void *z, int64_t zrs, void *y, int64_t yrs, float *state, int batch, int D,
                int N, cudaStream_t st, const float *A_inv) {
    const int aligned = reinterpret_cast<uintptr_t>(A) % 16 == 0 && reinterpret_cast<uintptr_t>(state) % 16 == 0;
    if (!std::is_same<Tx, float>::value) {
        // Four threads per channel, 32 channels per CTA, R batch rows per
        // thread (fewer rows when the batch is small, to keep CTAs many).
#ifndef MAMBA_STEP_ROWS
#define MAMBA_STEP_ROWS 4
#endif
        constexpr int R = MAMBA_STEP_ROWS;
        if (NS == 16 && N == 16 && aligned && D % 32 == 0 &&
            (int64_t)(D / 32) * ceil_div(batch, kStepBulkRows) >= device_sm_count()) {
            constexpr int RB = kStepBulkRows;
            const int smem = RB * 32 * 16 * 4 + RB * 2 * 16 * 4 + RB * 8;
            dim3 grid(D / 32, ceil_div(batch, RB));
            ssm_step_bulk_kernel<RB, Tx, Tdt, Tbc><<<grid, 128, smem, st>>>(
                static_cast<const Tx *>(x), xrs, static_cast<const Tdt *>(delta), drs, dt_bias,
                static_cast<const Tbc *>(B), static_cast<const Tbc *>(C), bcrs, A, Dskip,
                static_cast<const Tx *>(z), zrs, static_cast<Tx *>(y), yrs, state, batch, D,
                A_inv && reinterpret_cast<uintptr_t>(A_inv) % 16 == 0 ? A_inv : nullptr);
            return launch_status("ssm_step (bulk copies) kernel");
        }
        const bool many = (int64_t)ceil_div(D, 32) * ceil_div(batch, R) >= 2LL * device_sm_count();
        if (many) {
            dim3 grid(ceil_div(D, 32), ceil_div(batch, R));
            ssm_step_quad_kernel<NS, R, Tx, Tdt, Tbc><<<grid, 128, 0, st>>>(
                static_cast<const Tx *>(x), xrs, static_cast<const Tdt *>(delta), drs, dt_bias,
                static_cast<const Tbc *>(B), static_cast<const Tbc *>(C), bcrs, A, Dskip,
                static_cast<const Tx *>(z), zrs, static_cast<Tx *>(y), yrs, state, batch, D, N, aligned);
        } else {
            dim3 grid(ceil_div(D, 32), batch);
            ssm_step_quad_kernel<NS, 1, Tx, Tdt, Tbc><<<grid, 128, 0, st>>>(
                static_cast<const Tx *>(x), xrs, static_cast<const Tdt *>(delta), drs, dt_bias,
                static_cast<const Tbc *>(B), static_cast<const Tbc *>(C), bcrs, A, Dskip,
                static_cast<const Tx *>(z), zrs, static_cast<Tx *>(y), yrs, state, batch, D, N, aligned);
        }
        return launch_status("ssm_step kernel");
    }
    dim3 grid(ceil_div(D, 128), batch);
    ssm_step_kernel<NS, Tx, Tdt, Tbc><<<grid, 128, 0, st>>>(
        static_cast<const Tx *>(x), xrs, static_cast<const Tdt *>(delta), drs, dt_bias,
        static_cast<const Tbc *>(B), static_cast<const Tbc *>(C), bcrs, A, Dskip,
        static_cast<const Tx *>(z), zrs, static_cast<Tx *>(y), yrs, state, D, N, aligned);
    return launch_status("ssm_step kernel");
}

template <typename Tx, typename Tdt, typename Tbc>
int launch_step_ns(const void *x, int64_t xrs, const void *delta, int64_t drs, const float *dt_bias,
                   const void *B, const void *C, int64_t bcrs, const float *A, const float *Dskip,
                   const void *z, int64_t zrs, void *y, int64_t yrs, float *state, int batch, int D,
                   int N, cudaStream_t st, const float *A_inv) {
    if (N <= 4)
        return launch_step<4, Tx, Tdt, Tbc>(x, xrs, delta, drs, dt_bias, B, C, bcrs, A, Dskip, z, zrs, y,
                                            yrs, state, batch, D, N, st, A_inv);
    if (N <= 8)
        return launch_step<8, Tx, Tdt, Tbc>(x, xrs, delta, drs, dt_bias, B, C, bcrs, A, Dskip, z, zrs, y,
                                            yrs, state, batch, D, N, st, A_inv);
    return launch_step<16, Tx, Tdt, Tbc>(x, xrs, delta, drs, dt_bias, B, C, bcrs, A, Dskip, z, zrs, y,
                                         yrs, state, batch, D, N, st, A_inv);
}

}  // namespace

int ssm_step(const void *x, int64_t xrs, const void *delta, int64_t drs, const float *dt_bias,
             const void *B, const void *C, int64_t bcrs, const float *A, const float *Dskip,
             const void *z, int64_t zrs, void *y, int64_t yrs, float *state, int batch, int D, int N,
             int xd, int dd, int bd, cudaStream_t st, const float *A_inv) {
    MB_CHECK_ARG(batch >= 0 && D >= 0, "ssm_step: negative size");
    MB_CHECK_ARG(N >= 1 && N <= 16, "ssm_step: dstate must be in 1..16");
    MB_CHECK_ARG(batch <= 65535, "ssm_step: batch > 65535");
    if (batch == 0 || D == 0) return 0;
    MB_CHECK_ARG(x && delta && B && C && A && y && state, "ssm_step: null pointer");
    if (xd == MAMBA_F32 && dd == MAMBA_F32 && bd == MAMBA_F32)
        return launch_step_ns<float, float, float>(x, xrs, delta, drs, dt_bias, B, C, bcrs, A, Dskip, z, zrs,
                                                   y, yrs, state, batch, D, N, st, A_inv);
    if (xd == MAMBA_F16 && dd == MAMBA_F16 && bd == MAMBA_F16)
        return launch_step_ns<__half, __half, __half>(x, xrs, delta, drs, dt_bias, B, C, bcrs, A, Dskip, z,
                                                      zrs, y, yrs, state, batch, D, N, st, A_inv);
    if (xd == MAMBA_F16 && dd == MAMBA_F32 && bd == MAMBA_F16)
        return launch_step_ns<__half, float, __half>(x, xrs, delta, drs, dt_bias, B, C, bcrs, A, Dskip, z,
                                                     zrs, y, yrs, state, batch, D, N, st, A_inv);
    if (xd == MAMBA_F16 && dd == MAMBA_F32 && bd == MAMBA_F32)
        return launch_step_ns<__half, float, float>(x, xrs, delta, drs, dt_bias, B, C, bcrs, A, Dskip, z,
                                                    zrs, y, yrs, state, batch, D, N, st, A_inv);
    set_error("ssm_step: unsupported dtype combination");
    return -1;
}

unsigned step_error_flags(bool clear) {
    unsigned v = 0;
    if (cudaMemcpyFromSymbol(&v, g_step_error, sizeof(v)) != cudaSuccess) return ~0u;
    if (clear && v) {
        const unsigned z = 0;
        cudaMemcpyToSymbol(g_step_error, &z, sizeof(z));
    }
    return v;
}

}  // namespace mb
