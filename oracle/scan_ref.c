/*
 * oracle/scan_ref.c -- CPU restatement of the reference selective scan.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker: only tests/,
 * __graft_entry__.smoke() and bench.py's CPU-baseline leg load it.  The
 * product library (libmamba_b200.so) never links or calls it.
 *
 * What it restates (reference = SNAPKITTYWEST/mamba-metal):
 *   oracle_selective_scan      Sources/CPURef/selective_scan_cpu.cpp:7-45
 *                              (sequential exact-ZOH scan, t -> d -> n loop
 *                              order, softplus via log1p,
 *                              Sources/CPURef/selective_scan_cpu.hpp:21-23)
 *   oracle_scan_general        the same per-element arithmetic, generalised to
 *                              a batch, arbitrary strides, an optional dt bias
 *                              (added before softplus), an optional initial
 *                              state, and the SiLU(z) output gate of
 *                              Sources/Kernels/mamba_block.metal:118-121.
 *                              The loop over channels is hoisted outside the
 *                              loop over time; each (b,d,n) recurrence is
 *                              evaluated with exactly the same operations in
 *                              the same order, so results are bit-identical
 *                              to the reference loop order.
 *   oracle_affine_compose      Sources/CPURef/selective_scan_cpu.hpp:17-19
 *   oracle_scan_chunk_*        the chunk-carry monoid used by the multi-chunk
 *                              and sequence-sharded scans (the intent of
 *                              Sources/Kernels/prefix_scan.metal:19-40 with
 *                              its pair-layout bug fixed): chunk summaries
 *                              (prod a, h_end from zero) and their exclusive
 *                              composition.
 *   oracle_propagate_tile_carries
 *                              Sources/Kernels/prefix_scan.metal:19-40 (in-place
 *                              exclusive scan of interleaved (a, b) tile
 *                              carries, layout bug fixed)
 *   oracle_gated_silu_mul      Sources/Kernels/gated_mlp.metal:14-41
 *
 * Parity pin: tests/test_oracle.py checks oracle_selective_scan bit-exactly
 * against golden vectors written by the reference's own selective_scan_cpu
 * (tests/golden/), including the reference test suite's known answers.
 *
 * Build with -ffp-contract=off (no FMA contraction) so every product and sum
 * is rounded exactly as in the reference build.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

static inline float oracle_softplus(float x)
{
    /* selective_scan_cpu.hpp:21-23 */
    return x > 20.f ? x : log1pf(expf(x));
}

static inline float oracle_silu(float z)
{
    /* mamba_block.metal:120 */
    return z / (1.0f + expf(-z));
}

/* (a2,b2) o (a1,b1) = (a2*a1, a2*b1 + b2); selective_scan_cpu.hpp:17-19 */
void oracle_affine_compose(float a2, float b2, float a1, float b1,
                           float *a_out, float *b_out)
{
    *a_out = a2 * a1;
    *b_out = a2 * b1 + b2;
}

/*
 * Exact restatement of selective_scan_cpu (selective_scan_cpu.cpp:7-45).
 * x, delta: [L, D]; B, C: [L, N]; A: [D, N]; Dskip: [D]; y: [L, D];
 * state_out: [D, N] or NULL.  delta is the raw value; softplus is applied.
 */
int oracle_selective_scan(const float *x, const float *delta,
                          const float *B, const float *C,
                          const float *A, const float *Dskip,
                          float *y, float *state_out,
                          int L, int D, int N)
{
    float *h = (float *)calloc((size_t)D * N, sizeof(float));
    if (!h) return -1;
    for (int t = 0; t < L; ++t) {
        for (int d = 0; d < D; ++d) {
            float xt = x[(size_t)t * D + d];
            float dt = oracle_softplus(delta[(size_t)t * D + d]);
            float yt = 0.f;
            for (int n = 0; n < N; ++n) {
                float a = A[(size_t)d * N + n];
                float da = dt * a;
                float exp_da = expf(da);
                float Bn = B[(size_t)t * N + n];
                float Bbar = (fabsf(a) > 1e-6f) ? ((exp_da - 1.f) / a) * Bn
                                                : dt * Bn;
                float *ht = &h[(size_t)d * N + n];
                *ht = exp_da * (*ht) + Bbar * xt;
                float Cn = C[(size_t)t * N + n];
                yt += Cn * (*ht);
            }
            yt += Dskip[d] * xt;
            y[(size_t)t * D + d] = yt;
        }
    }
    if (state_out) memcpy(state_out, h, sizeof(float) * (size_t)D * N);
    free(h);
    return 0;
}

/*
 * General batched scan over fp32 arrays with element strides.
 *   x, delta, z, y : strides {batch, time, channel}
 *   B, C           : strides {batch, time, state}
 *   A [D,N], Dskip [D], dt_bias [D] (or NULL), h0 [batch,D,N] (or NULL)
 *   z NULL => no gate.  state_out [batch,D,N] or NULL.
 * Per (b,d): the recurrence over t of selective_scan_cpu.cpp:17-41, then
 * y *= SiLU(z) when z is given (mamba_block.metal:118-121).
 * nthreads > 1 splits the independent (b,d) channels across OpenMP threads;
 * results do not depend on the thread count.
 */
int oracle_scan_general(const float *x, const int64_t *sx,
                        const float *delta, const int64_t *sdt,
                        const float *B, const int64_t *sB,
                        const float *C, const int64_t *sC,
                        const float *A, const float *Dskip,
                        const float *dt_bias,
                        const float *z, const int64_t *sz,
                        const float *h0,
                        float *y, const int64_t *sy,
                        float *state_out,
                        int batch, int L, int D, int N, int nthreads)
{
    if (N > 256) return -1;
    const int64_t total = (int64_t)batch * D;
#ifdef _OPENMP
    if (nthreads < 1) nthreads = 1;
#pragma omp parallel for schedule(dynamic, 4) num_threads(nthreads)
#endif
    for (int64_t bd = 0; bd < total; ++bd) {
        const int b = (int)(bd / D), d = (int)(bd % D);
        float h[256];
        float Ad[256];
        for (int n = 0; n < N; ++n) {
            h[n] = h0 ? h0[((int64_t)b * D + d) * N + n] : 0.f;
            Ad[n] = A[(int64_t)d * N + n];
        }
        const float bias = dt_bias ? dt_bias[d] : 0.f;
        for (int t = 0; t < L; ++t) {
            const float xt = x[b * sx[0] + t * sx[1] + d * sx[2]];
            float draw = delta[b * sdt[0] + t * sdt[1] + d * sdt[2]];
            if (dt_bias) draw = draw + bias;
            const float dt = oracle_softplus(draw);
            float yt = 0.f;
            for (int n = 0; n < N; ++n) {
                float a = Ad[n];
                float da = dt * a;
                float exp_da = expf(da);
                float Bn = B[b * sB[0] + t * sB[1] + n * sB[2]];
                float Bbar = (fabsf(a) > 1e-6f) ? ((exp_da - 1.f) / a) * Bn
                                                : dt * Bn;
                h[n] = exp_da * h[n] + Bbar * xt;
                float Cn = C[b * sC[0] + t * sC[1] + n * sC[2]];
                yt += Cn * h[n];
            }
            yt += Dskip[d] * xt;
            if (z) {
                const float zt = z[b * sz[0] + t * sz[1] + d * sz[2]];
                yt = yt * oracle_silu(zt);
            }
            y[b * sy[0] + t * sy[1] + d * sy[2]] = yt;
        }
        if (state_out)
            for (int n = 0; n < N; ++n)
                state_out[((int64_t)b * D + d) * N + n] = h[n];
    }
    return 0;
}

/*
 * Chunk summary of the affine recurrence over t in [t0, t1) for every
 * (b,d,n): P = prod_t a_t and H = h_{t1-1} started from h = 0, where
 * a_t = exp(softplus(delta+bias)*A) and the input term is the exact-ZOH
 * Bbar*x of selective_scan_cpu.cpp:24-33.  The pair (P, H) is the affine map
 * h -> P*h + H that the chunk applies to its incoming state.
 * Outputs P, H: [batch, D, N].
 */
int oracle_scan_chunk_summary(const float *x, const int64_t *sx,
                              const float *delta, const int64_t *sdt,
                              const float *B, const int64_t *sB,
                              const float *A, const float *dt_bias,
                              float *P, float *H,
                              int batch, int t0, int t1, int D, int N)
{
    if (N > 256) return -1;
    for (int b = 0; b < batch; ++b)
        for (int d = 0; d < D; ++d) {
            float p[256], h[256];
            for (int n = 0; n < N; ++n) { p[n] = 1.f; h[n] = 0.f; }
            const float bias = dt_bias ? dt_bias[d] : 0.f;
            for (int t = t0; t < t1; ++t) {
                const float xt = x[b * sx[0] + t * sx[1] + d * sx[2]];
                float draw = delta[b * sdt[0] + t * sdt[1] + d * sdt[2]];
                if (dt_bias) draw = draw + bias;
                const float dt = oracle_softplus(draw);
                for (int n = 0; n < N; ++n) {
                    float a = A[(int64_t)d * N + n];
                    float exp_da = expf(dt * a);
                    float Bn = B[b * sB[0] + t * sB[1] + n * sB[2]];
                    float Bbar = (fabsf(a) > 1e-6f) ? ((exp_da - 1.f) / a) * Bn
                                                    : dt * Bn;
                    /* (exp_da, Bbar*x) o (p, h) */
                    float na, nb;
                    oracle_affine_compose(exp_da, Bbar * xt, p[n], h[n], &na, &nb);
                    p[n] = na;
                    h[n] = nb;
                }
            }
            for (int n = 0; n < N; ++n) {
                P[((int64_t)b * D + d) * N + n] = p[n];
                H[((int64_t)b * D + d) * N + n] = h[n];
            }
        }
    return 0;
}

/*
 * Exclusive composition of G chunk summaries (P_g, H_g), each [count]
 * floats, laid out [G, count].  h_in[g] = state entering chunk g, starting
 * from h0 (or zero when h0 is NULL).  Optionally writes the final state.
 */
int oracle_scan_chunk_combine(const float *P, const float *H, int G,
                              int64_t count, const float *h0,
                              float *h_in, float *h_final)
{
    for (int64_t i = 0; i < count; ++i) {
        float h = h0 ? h0[i] : 0.f;
        for (int g = 0; g < G; ++g) {
            if (h_in) h_in[(int64_t)g * count + i] = h;
            h = P[(int64_t)g * count + i] * h + H[(int64_t)g * count + i];
        }
        if (h_final) h_final[i] = h;
    }
    return 0;
}

/* Causal depthwise conv, restating causal_conv1d.metal:34-44, with the SiLU
 * of MambaRuntime.cpp:96 optionally applied.  x, y: strides {b, t, d};
 * w [D, K]; bias [D] or NULL. */
int oracle_causal_conv1d(const float *x, const int64_t *sx,
                         const float *w, const float *bias,
                         float *y, const int64_t *sy,
                         int batch, int L, int D, int K, int silu)
{
    for (int b = 0; b < batch; ++b)
        for (int t = 0; t < L; ++t)
            for (int d = 0; d < D; ++d) {
                float acc = 0.f;
                for (int k = 0; k < K; ++k) {
                    int src = t - K + 1 + k;
                    if (src >= 0)
                        acc += x[b * sx[0] + (int64_t)src * sx[1] + d * sx[2]] *
                               w[(int64_t)d * K + k];
                }
                if (bias) acc += bias[d];
                if (silu) acc = acc / (1.0f + expf(-acc));
                y[b * sy[0] + (int64_t)t * sy[1] + d * sy[2]] = acc;
            }
    return 0;
}

/* Incremental conv step, restating causal_conv1d.metal:59-81: conv over the
 * state (oldest..newest) plus the current x, then shift-append.
 * x_t, y_t: [batch, D]; conv_state [batch, D, K-1] updated in place. */
int oracle_causal_conv1d_step(const float *x_t, const float *w,
                              const float *bias, float *y_t,
                              float *conv_state, int batch, int D, int K,
                              int silu)
{
    for (int b = 0; b < batch; ++b)
        for (int d = 0; d < D; ++d) {
            float *st = conv_state + ((int64_t)b * D + d) * (K - 1);
            float acc = 0.f;
            for (int k = 0; k < K - 1; ++k) acc += st[k] * w[(int64_t)d * K + k];
            const float xt = x_t[(int64_t)b * D + d];
            acc += xt * w[(int64_t)d * K + (K - 1)];
            if (bias) acc += bias[d];
            if (silu) acc = acc / (1.0f + expf(-acc));
            y_t[(int64_t)b * D + d] = acc;
            for (int k = 0; k + 1 < K - 1; ++k) st[k] = st[k + 1];
            if (K > 1) st[K - 2] = xt;
        }
    return 0;
}

/* Single-token SSM update, restating state_update.metal:31-56 with softplus
 * always applied (as in selective_scan_cpu.cpp:20), optional dt bias and
 * SiLU(z) gate.  x,delta,z,y: [batch, D]; B,C: strides {b, n};
 * state [batch, D, N] updated in place. */
int oracle_ssm_step(const float *x, const float *delta, const float *dt_bias,
                    const float *B, const float *C, int64_t sBb, int64_t sCb,
                    const float *A, const float *Dskip, const float *z,
                    float *y, float *state, int batch, int D, int N)
{
    for (int b = 0; b < batch; ++b)
        for (int d = 0; d < D; ++d) {
            const float xt = x[(int64_t)b * D + d];
            float draw = delta[(int64_t)b * D + d];
            if (dt_bias) draw = draw + dt_bias[d];
            const float dt = oracle_softplus(draw);
            float yt = 0.f;
            for (int n = 0; n < N; ++n) {
                float a = A[(int64_t)d * N + n];
                float exp_da = expf(dt * a);
                float Bn = B[b * sBb + n];
                float Bbar = (fabsf(a) > 1e-6f) ? ((exp_da - 1.f) / a) * Bn
                                                : dt * Bn;
                float *hp = &state[((int64_t)b * D + d) * N + n];
                *hp = exp_da * (*hp) + Bbar * xt;
                yt += C[b * sCb + n] * (*hp);
            }
            yt += Dskip[d] * xt;
            if (z) yt = yt * oracle_silu(z[(int64_t)b * D + d]);
            y[(int64_t)b * D + d] = yt;
        }
    return 0;
}

/* RMSNorm, restating rmsnorm.metal:26-44 with a sequential fp32 sum:
 * y = x * rsqrt(mean(x^2) + eps) * w.  x,y: [rows, N] row-major. */
int oracle_rmsnorm(const float *x, const float *w, float *y, int64_t rows,
                   int N, float eps)
{
    for (int64_t r = 0; r < rows; ++r) {
        const float *xr = x + r * N;
        double ss = 0.0;
        for (int i = 0; i < N; ++i) ss += (double)xr[i] * xr[i];
        const float inv = (float)(1.0 / sqrt(ss / N + (double)eps));
        for (int i = 0; i < N; ++i) {
            float v = xr[i] * inv;
            if (w) v *= w[i];
            y[r * N + i] = v;
        }
    }
    return 0;
}

/* Exclusive propagation of tile carries, restating the intent of
 * propagate_tile_carries_f32 (prefix_scan.metal:19-40) with its pair layout
 * fixed: carries is [num_tiles, width, 2], pair p of tile t at
 * (t*width + p)*2 as (a, b).  In place, tile t's pair becomes the
 * composition of tiles 0..t-1 (identity (1, 0) for tile 0), composed as
 * compose(cur, acc) (prefix_scan.metal:12-14, selective_scan_cpu.hpp:17-19).
 * total ([width, 2]) receives the composition of all tiles when not NULL. */
int oracle_propagate_tile_carries(float *carries, int num_tiles, int64_t width,
                                  float *total)
{
    for (int64_t p = 0; p < width; ++p) {
        float acc_a = 1.0f, acc_b = 0.0f;
        for (int t = 0; t < num_tiles; ++t) {
            float *pr = carries + ((int64_t)t * width + p) * 2;
            const float a = pr[0], b = pr[1];
            float na, nb;
            oracle_affine_compose(a, b, acc_a, acc_b, &na, &nb);
            pr[0] = acc_a;
            pr[1] = acc_b;
            acc_a = na;
            acc_b = nb;
        }
        if (total) {
            total[2 * p] = acc_a;
            total[2 * p + 1] = acc_b;
        }
    }
    return 0;
}

/* SwiGLU gate, restating gated_silu_mul_f32 (gated_mlp.metal:14-26):
 * out = g / (1 + exp(-g)) * u, elementwise over n values. */
int oracle_gated_silu_mul(const float *gate, const float *up, float *out, int64_t n)
{
    for (int64_t i = 0; i < n; ++i) {
        const float g = gate[i];
        const float s = g / (1.0f + expf(-g));
        out[i] = s * up[i];
    }
    return 0;
}
