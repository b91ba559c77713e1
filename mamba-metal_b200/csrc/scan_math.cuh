// scan_math.cuh -- per-timestep arithmetic of the selective scan, shared by
// the full-sequence kernels and kept identical to the decode step.
//
// Two precision modes:
//  * PRECISE (FP32 inputs): the reference oracle's own sequence of FP32
//    operations (Sources/CPURef/selective_scan_cpu.cpp:17-41, each product
//    and sum rounded separately, IEEE division, states in order n = 0..N-1),
//    with exp, log1p and the SiLU exponential evaluated in double precision
//    and rounded once to FP32, i.e. correctly rounded like the libm calls the
//    oracle makes.  The zero-order hold's (a - 1) is ill-conditioned when
//    dt*A is small, so matching the oracle's rounding matters here.
//  * fast (FP16 inputs, 2e-3 budget): single-instruction ex2.approx, short
//    softplus/SiLU forms, and packed f32x2 arithmetic (two states per
//    instruction).
#pragma once

#include <cuda_fp16.h>

#include "common.cuh"

namespace mb {

constexpr float kLn2 = 0.69314718055994531f;

__device__ __forceinline__ float ex2_approx(float v) {
    float r;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(v));
    return r;
}

__device__ __forceinline__ float lg2_approx(float v) {
    float r;
    asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(v));
    return r;
}

__device__ __forceinline__ float rcp_approx(float v) {
    float r;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(v));
    return r;
}

// softplus(x) = max(x, 0) + log1p(e), e = exp(-|x|) in (0, 1], with one
// ex2 and log1p(e) = e * q(e), where q interpolates log1p(e)/e at the eight
// Chebyshev nodes of [0, 1] (max relative error 3.3e-7 in FP32 Horner form).
// For x > 20 the result rounds to x, as in selective_scan_cpu.hpp:21-23.
__device__ __forceinline__ float softplus_fast(float x) {
    const float e = ex2_approx(-fabsf(x) * kLog2e);
    float q = -8.371152915e-03f;
    q = fmaf(q, e, 4.349390045e-02f);
    q = fmaf(q, e, -1.068500280e-01f);
    q = fmaf(q, e, 1.768747717e-01f);
    q = fmaf(q, e, -2.447477430e-01f);
    q = fmaf(q, e, 3.327192962e-01f);
    q = fmaf(q, e, -4.999717474e-01f);
    q = fmaf(q, e, 9.999997616e-01f);
    return fmaf(e, q, fmaxf(x, 0.f));
}

// 1/v for v in [1, 2^120] on the FMA pipe: the exponent-negating integer
// seed (relative error <= 5.1%) refined by two Newton steps
// r <- r + r * (1 - v * r) (relative error <= 6.6e-6).
__device__ __forceinline__ float rcp_newton2(float v) {
    float r = __int_as_float(0x7EF311C7 - __float_as_int(v));
    r = fmaf(r, fmaf(-v, r, 1.f), r);
    r = fmaf(r, fmaf(-v, r, 1.f), r);
    return r;
}

// 2^v on the FMA pipe instead of the special-function unit: Cody-Waite
// reduction v = j + f (j = round(v) by the 1.5 * 2^23 magic add, |f| <= 1/2),
// 2^f = 1 + f q(f) with q interpolating (2^f - 1)/f at the five Chebyshev
// nodes of [-1/2, 1/2] (coefficients computed here in FP64, rounded to FP32;
// max relative error of the FP32 evaluation 2.6e-7), and j added to the
// exponent field as an integer.  v is clamped to [-125, 127], so the result
// stays a normal number (2^-125 where ex2.approx.ftz would flush to 0).
__device__ __forceinline__ float ex2_fma(float v) {
    v = fminf(fmaxf(v, -125.f), 127.f);
    const float t = v + 12582912.f;
    const float f = v - (t - 12582912.f);
    float q = 1.338130212e-03f;
    q = fmaf(q, f, 9.666368365e-03f);
    q = fmaf(q, f, 5.550381169e-02f);
    q = fmaf(q, f, 2.402234972e-01f);
    q = fmaf(q, f, 6.931471825e-01f);
    const float p = fmaf(q, f, 1.f);
    return __int_as_float(__float_as_int(p) + (__float_as_int(t) << 23));
}

#ifndef MAMBA_SCAN_FMA_EXP
#define MAMBA_SCAN_FMA_EXP 0
#endif
// State exponentials of the one-thread scan's fast path: the last state of
// each channel on the FMA pipe (ex2_fma) when built with
// MAMBA_SCAN_FMA_EXP=1, else all on the special-function unit.  Off by
// default: with it the scan of batch 64 x L 4096 x 4096 channels took 6.16 ms
// against 5.90 (the FMA pipe and issue slots, already ~55-60% busy, became
// the limit).  The decode kernels and the four-lane scan always use
// ex2.approx, so with the flag set their states no longer equal the scan's
// bit for bit.
__device__ __forceinline__ float state_ex2(float v, bool last_state) {
    return (MAMBA_SCAN_FMA_EXP && last_state) ? ex2_fma(v) : ex2_approx(v);
}

// SiLU(z) = z / (1 + exp(-z)) with one ex2 and a Newton reciprocal.
__device__ __forceinline__ float silu_fast(float z) {
    return z * rcp_newton2(1.f + ex2_approx(fminf(-z * kLog2e, 120.f)));
}

// Correctly rounded FP32 exp / log1p (evaluated in FP64, rounded once).
__device__ __forceinline__ float exp_cr(float x) { return __double2float_rn(exp((double)x)); }
__device__ __forceinline__ float log1p_cr(float x) { return __double2float_rn(log1p((double)x)); }

// selective_scan_cpu.hpp:21-23: x > 20 ? x : log1p(exp(x)).
__device__ __forceinline__ float softplus_exact(float x) { return x > 20.f ? x : log1p_cr(exp_cr(x)); }

// mamba_block.metal:120: z / (1 + exp(-z)).
__device__ __forceinline__ float silu_exact(float z) { return __fdiv_rn(z, __fadd_rn(1.0f, exp_cr(-z))); }

template <bool PRECISE>
__device__ __forceinline__ float scan_softplus(float x) {
    return PRECISE ? softplus_exact(x) : softplus_fast(x);
}

template <bool PRECISE>
__device__ __forceinline__ float scan_silu(float z) {
    return PRECISE ? silu_exact(z) : silu_fast(z);
}

// Per-channel constants of NS states packed in pairs: Ac = A (PRECISE) or
// A*log2(e) (fast); kI = 1/A, or 0 where |A| <= 1e-6 (the dt*B branch of
// selective_scan_cpu.cpp:28-30) and for padding states n >= N.
template <int NS, bool PRECISE>
__device__ __forceinline__ bool load_channel_consts(const float *__restrict__ A, int64_t row, int N,
                                                    bool valid, float2 *Ac, float2 *kI) {
    bool small = false;
#pragma unroll
    for (int p = 0; p < NS / 2; ++p) {
        float a[2], c[2], k[2];
#pragma unroll
        for (int q = 0; q < 2; ++q) {
            const int n = 2 * p + q;
            a[q] = (valid && n < N) ? A[row * N + n] : 0.f;
            c[q] = PRECISE ? a[q] : a[q] * kLog2e;
            const bool big = fabsf(a[q]) > 1e-6f;
            k[q] = big ? __frcp_rn(a[q]) : 0.f;  // correctly rounded, as 1.0f / a
            small |= (valid && n < N && !big);
        }
        Ac[p] = make_float2(c[0], c[1]);
        kI[p] = make_float2(k[0], k[1]);
    }
    return small;
}

// PRECISE timestep: selective_scan_cpu.cpp:21-37 operation by operation.
// Padding states (A = 0, B = C = 0) keep h = 0 and add +0 to y.
template <int NS, bool SUMMARY>
__device__ __forceinline__ float scan_step_exact(float xv, float dt, const float *__restrict__ bc, float2 *h,
                                                 const float2 *Ac, const float2 *kI, float2 *P) {
    float yt = 0.f;
#pragma unroll
    for (int n = 0; n < NS; ++n) {
        const float a = (n & 1) ? Ac[n / 2].y : Ac[n / 2].x;
        const bool big = ((n & 1) ? kI[n / 2].y : kI[n / 2].x) != 0.f;
        const float exp_da = exp_cr(__fmul_rn(dt, a));
        const float Bn = bc[n];
        const float Bbar = big ? __fmul_rn(__fdiv_rn(__fsub_rn(exp_da, 1.f), a), Bn) : __fmul_rn(dt, Bn);
        float &ht = (n & 1) ? h[n / 2].y : h[n / 2].x;
        ht = __fadd_rn(__fmul_rn(exp_da, ht), __fmul_rn(Bbar, xv));
        if (SUMMARY) {
            float &pt = (n & 1) ? P[n / 2].y : P[n / 2].x;
            pt = __fmul_rn(pt, exp_da);
        } else {
            yt = __fadd_rn(yt, __fmul_rn(bc[NS + n], ht));
        }
    }
    return yt;
}

// One state of the fast path: h' = a h + b with b = (a - 1)/A * w (w = B x)
// or b = dt * w where |A| <= 1e-6 (kI == 0).  The zero-order-hold form is
// evaluated as h + (a - 1)(h + w/A).
__device__ __forceinline__ float state_update(float a, float w, float kI, float dt, float h) {
    return kI != 0.f ? fmaf(a - 1.f, fmaf(w, kI, h), h) : fmaf(a, h, dt * w);
}

// One timestep for one channel.  bc points at the step's B[0..NS) and
// C[0..NS) (FP32, 16-byte aligned).  Updates h (and P = prod a in summary
// mode); returns sum_n C[n] * h[n] (output mode).
template <int NS, bool SUMMARY, bool PRECISE, bool SMALLA>
__device__ __forceinline__ float scan_step(float xv, float dt, const float *__restrict__ bc, float2 *h,
                                           const float2 *Ac, const float2 *kI, float2 *P) {
    if (PRECISE) return scan_step_exact<NS, SUMMARY>(xv, dt, bc, h, Ac, kI, P);
    const float4 *bq = reinterpret_cast<const float4 *>(bc);
    const float2 dt2 = make_float2(dt, dt), x2 = make_float2(xv, xv);
    float2 yacc = make_float2(0.f, 0.f);
#pragma unroll
    for (int q = 0; q < NS / 4; ++q) {
        const float4 Bv = bq[q];
        float4 Cv = make_float4(0.f, 0.f, 0.f, 0.f);
        if (!SUMMARY) Cv = bq[NS / 4 + q];
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
            const int p = 2 * q + hh;
            const float2 Bp = hh ? make_float2(Bv.z, Bv.w) : make_float2(Bv.x, Bv.y);
            const float2 dA = __fmul2_rn(dt2, Ac[p]);
            float2 a;
            if (PRECISE) {
                a.x = expf(dA.x);
                a.y = expf(dA.y);
            } else {
                a.x = ex2_approx(dA.x);
                a.y = state_ex2(dA.y, p == NS / 2 - 1);
            }
            const float2 w = __fmul2_rn(x2, Bp);
            if (SMALLA) {
                h[p].x = state_update(a.x, w.x, kI[p].x, dt, h[p].x);
                h[p].y = state_update(a.y, w.y, kI[p].y, dt, h[p].y);
            } else {
                // h' = a h + (a - 1) k = h + (a - 1)(h + k): no negated operand,
                // and the (a - 1) product stays well conditioned.
                const float2 sk = __ffma2_rn(w, kI[p], h[p]);
                h[p] = __ffma2_rn(__fadd2_rn(a, make_float2(-1.f, -1.f)), sk, h[p]);
            }
            if (SUMMARY) {
                P[p] = __fmul2_rn(P[p], a);
            } else {
                const float2 Cp = hh ? make_float2(Cv.z, Cv.w) : make_float2(Cv.x, Cv.y);
                yacc = __ffma2_rn(Cp, h[p], yacc);
            }
        }
    }
    return yacc.x + yacc.y;
}

// y = (s + D*x) * gate, in the oracle's rounding for PRECISE
// (selective_scan_cpu.cpp:38, mamba_block.metal:118-121).
template <bool PRECISE>
__device__ __forceinline__ float scan_output(float s, float dskip, float xv, float gate) {
    if (PRECISE) return __fmul_rn(__fadd_rn(s, __fmul_rn(dskip, xv)), gate);
    return fmaf(dskip, xv, s) * gate;
}

}  // namespace mb
