// scan.cu -- fused selective scan for sm_100a.
//
// Maths (per batch row b, channel d, time t, state n), as in the reference
// oracle Sources/CPURef/selective_scan_cpu.cpp:17-41 and the gated variant
// Sources/Kernels/mamba_block.metal:67-122:
//   dt = softplus(delta + dt_bias)
//   a  = exp(dt * A[d,n])                (zero-order hold)
//   b  = (a - 1) / A[d,n] * B[t,n] * x   (dt * B * x when |A| <= 1e-6)
//   h  = a * h + b                        (FP32 state)
//   y  = sum_n C[t,n] * h + D[d] * x,  then y *= SiLU(z) when a gate is given
//
// Decomposition.  One thread owns one (b, d) channel and keeps its N states
// in registers; it walks time sequentially, so each (t, d, n) costs exactly
// one exponential and no scan-operator overhead.  A CTA covers CH adjacent
// channels of one batch row and one time chunk; per tile of TT timesteps the
// CTA stages x, delta, z (CH channels wide) and B, C (shared by all channels)
// in shared memory, so every global access is coalesced along whichever of
// the channel or time axes is contiguous.
//
// When batch * ceil(D / CH) CTAs are too few to fill the GPU, time is split
// into chunks (the carry propagation the reference intended in
// Sources/Kernels/prefix_scan.metal:19-40):
//   phase 1  each chunk computes its summary (P = prod a, H = h_end from 0),
//   phase 2  a combine kernel composes the summaries into the state entering
//            each chunk,
//   phase 3  each chunk rescans from its entering state and writes y.
// The same (P, H) monoid carries state across GPUs in sequence-sharded mode.
#include "common.cuh"

#include <algorithm>

namespace mb {

namespace {

constexpr int kScanCH = 128;  // channels (= threads) per CTA
constexpr int kScanTT = 32;   // timesteps per shared-memory tile

enum ScanMode { kModeOutput = 0, kModeSummary = 1 };

struct ScanKParams {
    const void *x, *delta, *B, *C, *z;
    const float *A, *Dskip, *dt_bias;
    const float *h_init;  // [batch, nchunks, D, N] entering states, or NULL
    void *y;
    float *final_state;   // [batch, D, N] or NULL
    float *sumP, *sumH;   // [batch, nchunks, D, N] (summary mode)
    int batch, L, D, N, nchunks, chunk_len;
    int64_t sx[3], sdt[3], sB[3], sC[3], sz[3], sy[3];
};

__device__ __forceinline__ float ex2_approx(float v) {
    float r;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(v));
    return r;
}

// Stage a [TT, CH] tile of a per-channel tensor into shared memory (row tt,
// column c).  Channel-contiguous tensors are read one row per warp pass;
// otherwise consecutive threads read consecutive timesteps of one channel.
template <typename T, int CH, int TT>
__device__ __forceinline__ void stage_tile(T *s, const T *g, const int64_t *st, int b, int t0,
                                           int nt, int d0, int D) {
    const int tid = threadIdx.x;
    const T *gb = g + (int64_t)b * st[0];
    if (st[2] == 1) {
        const int d = d0 + tid;
        if (d < D) {
            const T *gp = gb + (int64_t)t0 * st[1] + d;
            for (int tt = 0; tt < nt; ++tt) s[tt * CH + tid] = gp[(int64_t)tt * st[1]];
        }
    } else {
        for (int e = tid; e < TT * CH; e += CH) {
            const int c = e / TT, tt = e % TT;
            if (tt < nt && d0 + c < D)
                s[tt * CH + c] = gb[(int64_t)(t0 + tt) * st[1] + (int64_t)(d0 + c) * st[2]];
        }
    }
}

template <int NS, int CH, int TT, typename Tx, typename Tdt, typename Tbc, int MODE>
__global__ void __launch_bounds__(CH) scan_kernel(const ScanKParams p) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    float *sB = reinterpret_cast<float *>(smem_raw);  // [TT][NS]
    float *sC = sB + TT * NS;                          // [TT][NS]
    Tx *sX = reinterpret_cast<Tx *>(sC + TT * NS);     // [TT][CH]
    Tx *sZ = sX + TT * CH;                             // [TT][CH]
    Tdt *sDt = reinterpret_cast<Tdt *>(sZ + TT * CH);  // [TT][CH]

    const int tid = threadIdx.x;
    const int b = blockIdx.z, chunk = blockIdx.y;
    const int d0 = blockIdx.x * CH, d = d0 + tid;
    const bool dvalid = d < p.D;
    const int N = p.N;
    const int t_begin = chunk * p.chunk_len;
    const int t_end = min(p.L, t_begin + p.chunk_len);

    float A2[NS], kI[NS], h[NS], P[NS];
    bool small = false;
#pragma unroll
    for (int n = 0; n < NS; ++n) {
        const float a = (dvalid && n < N) ? p.A[(int64_t)d * N + n] : 0.f;
        A2[n] = a * kLog2e;
        const bool big = fabsf(a) > 1e-6f;
        kI[n] = big ? 1.0f / a : 0.f;
        small |= (dvalid && n < N && !big);
        h[n] = 0.f;
        P[n] = 1.f;
    }
    const int64_t st_off = (((int64_t)b * p.nchunks + chunk) * p.D + d) * N;
    if (MODE == kModeOutput && p.h_init && dvalid) {
#pragma unroll
        for (int n = 0; n < NS; ++n)
            if (n < N) h[n] = p.h_init[st_off + n];
    }
    const bool has_bias = p.dt_bias != nullptr;
    const float bias = (has_bias && dvalid) ? p.dt_bias[d] : 0.f;
    const float dskip = (p.Dskip && dvalid) ? p.Dskip[d] : 0.f;
    const bool any_small = __syncthreads_or(small);
    const bool has_z = (MODE == kModeOutput) && p.z != nullptr;

    const Tx *gx = static_cast<const Tx *>(p.x);
    const Tdt *gdt = static_cast<const Tdt *>(p.delta);
    const Tx *gz = static_cast<const Tx *>(p.z);
    const Tbc *gB = static_cast<const Tbc *>(p.B);
    const Tbc *gC = static_cast<const Tbc *>(p.C);
    Tx *gy = static_cast<Tx *>(p.y);

    for (int t0 = t_begin; t0 < t_end; t0 += TT) {
        const int nt = min(TT, t_end - t0);
        stage_tile<Tx, CH, TT>(sX, gx, p.sx, b, t0, nt, d0, p.D);
        stage_tile<Tdt, CH, TT>(sDt, gdt, p.sdt, b, t0, nt, d0, p.D);
        if (has_z) stage_tile<Tx, CH, TT>(sZ, gz, p.sz, b, t0, nt, d0, p.D);
        for (int e = tid; e < TT * NS; e += CH) {
            const int tt = e / NS, n = e % NS;
            float bv = 0.f, cv = 0.f;
            if (tt < nt && n < N) {
                const int64_t t = t0 + tt;
                bv = ld_f32(gB + (int64_t)b * p.sB[0] + t * p.sB[1] + (int64_t)n * p.sB[2]);
                if (MODE == kModeOutput)
                    cv = ld_f32(gC + (int64_t)b * p.sC[0] + t * p.sC[1] + (int64_t)n * p.sC[2]);
            }
            sB[e] = bv;
            sC[e] = cv;
        }
        __syncthreads();
        if (dvalid) {
            for (int tt = 0; tt < nt; ++tt) {
                const float xv = cvt_f32(sX[tt * CH + tid]);
                float draw = cvt_f32(sDt[tt * CH + tid]);
                if (has_bias) draw = draw + bias;
                const float dt = softplus_f(draw);
                const float *Bt = sB + tt * NS;
                const float *Ct = sC + tt * NS;
                float y0 = 0.f, y1 = 0.f;
#pragma unroll
                for (int n = 0; n < NS; ++n) {
                    const float a = ex2_approx(dt * A2[n]);
                    const float w = xv * Bt[n];
                    float bb;
                    if (any_small && kI[n] == 0.f) {
                        bb = dt * w;
                    } else {
                        const float k = w * kI[n];
                        bb = fmaf(a, k, -k);
                    }
                    h[n] = fmaf(a, h[n], bb);
                    if (MODE == kModeSummary) {
                        P[n] *= a;
                    } else {
                        if (n & 1) y1 = fmaf(Ct[n], h[n], y1);
                        else y0 = fmaf(Ct[n], h[n], y0);
                    }
                }
                if (MODE == kModeOutput) {
                    float yv = fmaf(dskip, xv, y0 + y1);
                    if (has_z) yv *= silu_f(cvt_f32(sZ[tt * CH + tid]));
                    gy[(int64_t)b * p.sy[0] + (int64_t)(t0 + tt) * p.sy[1] + (int64_t)d * p.sy[2]] =
                        cvt_out<Tx>(yv);
                }
            }
        }
        __syncthreads();
    }

    if (!dvalid) return;
    if (MODE == kModeSummary) {
#pragma unroll
        for (int n = 0; n < NS; ++n)
            if (n < N) {
                p.sumP[st_off + n] = P[n];
                p.sumH[st_off + n] = h[n];
            }
    } else if (p.final_state && t_end == p.L) {
        float *fs = p.final_state + ((int64_t)b * p.D + d) * N;
#pragma unroll
        for (int n = 0; n < NS; ++n)
            if (n < N) fs[n] = h[n];
    }
}

// Phase 2: compose the chunk summaries of every (b, d, n) in time order.
// On entry H/P hold the summaries [batch, nchunks, D*N]; when write_hin is
// set, H is overwritten in place with the state entering each chunk.
__global__ void scan_combine_kernel(const float *__restrict__ P, float *__restrict__ H,
                                    const float *__restrict__ h0, int nchunks, int64_t DN,
                                    int64_t total, int write_hin, float *__restrict__ P_total,
                                    float *__restrict__ H_total) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= total) return;
    const int64_t b = i / DN, r = i % DN;
    float h = h0 ? h0[i] : 0.f;
    float pt = 1.f;
    for (int c = 0; c < nchunks; ++c) {
        const int64_t idx = (b * nchunks + c) * DN + r;
        const float pc = P[idx], hc = H[idx];
        if (write_hin) H[idx] = h;
        h = pc * h + hc;
        pt *= pc;
    }
    if (H_total) H_total[i] = h;
    if (P_total) P_total[i] = pt;
}

// Sequence-sharded mode: state entering rank `rank` from the gathered
// per-rank summaries PH[world][2][count].
__global__ void scan_compose_prefix_kernel(const float *__restrict__ PH, int rank, int64_t count,
                                           const float *__restrict__ h0, float *__restrict__ h_in) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= count) return;
    float h = h0 ? h0[i] : 0.f;
    for (int g = 0; g < rank; ++g) {
        const float *Pg = PH + (int64_t)g * 2 * count;
        h = Pg[i] * h + Pg[count + i];
    }
    h_in[i] = h;
}

template <int NS, typename Tx, typename Tdt, typename Tbc, int MODE>
int launch_scan(const ScanKParams &kp, cudaStream_t st) {
    constexpr int CH = kScanCH, TT = kScanTT;
    auto kern = scan_kernel<NS, CH, TT, Tx, Tdt, Tbc, MODE>;
    const size_t smem = (size_t)TT * NS * 4 * 2 + (size_t)TT * CH * (2 * sizeof(Tx) + sizeof(Tdt));
    MB_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    dim3 grid(ceil_div(kp.D, CH), kp.nchunks, kp.batch);
    kern<<<grid, CH, smem, st>>>(kp);
    return launch_status("selective_scan kernel");
}

template <typename Tx, typename Tdt, typename Tbc, int MODE>
int launch_scan_ns(const ScanKParams &kp, cudaStream_t st) {
    if (kp.N <= 4) return launch_scan<4, Tx, Tdt, Tbc, MODE>(kp, st);
    if (kp.N <= 8) return launch_scan<8, Tx, Tdt, Tbc, MODE>(kp, st);
    return launch_scan<16, Tx, Tdt, Tbc, MODE>(kp, st);
}

template <int MODE>
int launch_scan_dtypes(const ScanKParams &kp, int xd, int dd, int bd, cudaStream_t st) {
    if (xd == MAMBA_F32 && dd == MAMBA_F32 && bd == MAMBA_F32)
        return launch_scan_ns<float, float, float, MODE>(kp, st);
    if (xd == MAMBA_F16 && dd == MAMBA_F16 && bd == MAMBA_F16)
        return launch_scan_ns<__half, __half, __half, MODE>(kp, st);
    if (xd == MAMBA_F16 && dd == MAMBA_F32 && bd == MAMBA_F16)
        return launch_scan_ns<__half, float, __half, MODE>(kp, st);
    if (xd == MAMBA_F16 && dd == MAMBA_F32 && bd == MAMBA_F32)
        return launch_scan_ns<__half, float, float, MODE>(kp, st);
    set_error("selective_scan: unsupported dtype combination (x, delta, B/C)");
    return -1;
}

// Time-chunk length for these dims.  One chunk per channel when the
// channel CTAs alone fill the GPU; otherwise split time so that about eight
// CTAs per SM exist, keeping chunks >= 128 steps.
int choose_chunk_len(int batch, int L, int D, int requested) {
    if (L <= 0) return 1;
    if (requested > 0) {
        const int c = ceil_div(requested, kScanTT) * kScanTT;
        return std::min(c, L);
    }
    const int64_t ctas = (int64_t)batch * ceil_div(D, kScanCH);
    const int sms = device_sm_count();
    if (ctas >= 4LL * sms) return L;
    const int64_t want = ceil_div64(8LL * sms, ctas);
    const int64_t maxc = std::max<int64_t>(1, L / 128);
    const int64_t nc = std::min(want, maxc);
    if (nc <= 1) return L;
    const int clen = (int)(ceil_div64(ceil_div64(L, nc), kScanTT) * kScanTT);
    return std::min(clen, L);
}

int validate(const MambaScanArgs *a) {
    MB_CHECK_ARG(a != nullptr, "selective_scan: null args");
    MB_CHECK_ARG(a->batch >= 0 && a->seqlen >= 0 && a->dim >= 0, "selective_scan: negative size");
    MB_CHECK_ARG(a->dstate >= 1 && a->dstate <= 16, "selective_scan: dstate must be in 1..16");
    MB_CHECK_ARG(a->batch <= 65535, "selective_scan: batch > 65535");
    if (a->batch == 0 || a->dim == 0) return 0;
    MB_CHECK_ARG(a->A != nullptr, "selective_scan: A is NULL");
    if (a->seqlen > 0) {
        MB_CHECK_ARG(a->x && a->delta && a->B, "selective_scan: x, delta and B are required");
    }
    return 0;
}

ScanKParams make_params(const MambaScanArgs *a, int chunk_len) {
    ScanKParams kp{};
    kp.x = a->x;
    kp.delta = a->delta;
    kp.B = a->B;
    kp.C = a->C;
    kp.z = a->z;
    kp.A = a->A;
    kp.Dskip = a->D;
    kp.dt_bias = a->dt_bias;
    kp.y = a->y;
    kp.final_state = a->final_state;
    kp.batch = a->batch;
    kp.L = a->seqlen;
    kp.D = a->dim;
    kp.N = a->dstate;
    kp.chunk_len = chunk_len;
    kp.nchunks = a->seqlen > 0 ? ceil_div(a->seqlen, chunk_len) : 1;
    for (int i = 0; i < 3; ++i) {
        kp.sx[i] = a->x_stride[i];
        kp.sdt[i] = a->delta_stride[i];
        kp.sB[i] = a->B_stride[i];
        kp.sC[i] = a->C_stride[i];
        kp.sz[i] = a->z_stride[i];
        kp.sy[i] = a->y_stride[i];
    }
    return kp;
}

int launch_combine(const float *P, float *H, const float *h0, int nchunks, int64_t DN, int batch,
                   int write_hin, float *P_total, float *H_total, cudaStream_t st) {
    const int64_t total = (int64_t)batch * DN;
    if (total == 0) return 0;
    const int threads = 256;
    scan_combine_kernel<<<(unsigned)ceil_div64(total, threads), threads, 0, st>>>(
        P, H, h0, nchunks, DN, total, write_hin, P_total, H_total);
    return launch_status("scan_combine kernel");
}

}  // namespace

size_t scan_workspace_bytes(const MambaScanArgs *a) {
    if (!a || a->batch <= 0 || a->dim <= 0 || a->seqlen <= 0) return 0;
    const int clen = choose_chunk_len(a->batch, a->seqlen, a->dim, a->chunk_len);
    const int nc = ceil_div(a->seqlen, clen);
    if (nc <= 1) return 0;
    return 2 * sizeof(float) * (size_t)a->batch * nc * a->dim * a->dstate;
}

int selective_scan(const MambaScanArgs *a, void *ws, size_t ws_bytes, cudaStream_t st) {
    if (validate(a)) return -1;
    if (a->batch == 0 || a->dim == 0) return 0;
    if (a->seqlen > 0) MB_CHECK_ARG(a->y && a->C, "selective_scan: y and C are required");
    const int clen = choose_chunk_len(a->batch, a->seqlen, a->dim, a->chunk_len);
    ScanKParams kp = make_params(a, clen);
    const int64_t DN = (int64_t)a->dim * a->dstate;
    if (kp.nchunks == 1) {
        kp.h_init = a->initial_state;
        return launch_scan_dtypes<kModeOutput>(kp, a->x_dtype, a->delta_dtype, a->bc_dtype, st);
    }
    const size_t need = scan_workspace_bytes(a);
    MB_CHECK_ARG(ws != nullptr && ws_bytes >= need, "selective_scan: workspace too small");
    float *sumP = static_cast<float *>(ws);
    float *sumH = sumP + (size_t)a->batch * kp.nchunks * DN;
    ScanKParams k1 = kp;
    k1.sumP = sumP;
    k1.sumH = sumH;
    if (launch_scan_dtypes<kModeSummary>(k1, a->x_dtype, a->delta_dtype, a->bc_dtype, st)) return -1;
    if (launch_combine(sumP, sumH, a->initial_state, kp.nchunks, DN, a->batch, 1, nullptr, nullptr, st))
        return -1;
    kp.h_init = sumH;
    return launch_scan_dtypes<kModeOutput>(kp, a->x_dtype, a->delta_dtype, a->bc_dtype, st);
}

int scan_summary(const MambaScanArgs *a, float *P, float *H, void *ws, size_t ws_bytes,
                 cudaStream_t st) {
    if (validate(a)) return -1;
    if (a->batch == 0 || a->dim == 0) return 0;
    MB_CHECK_ARG(P && H, "scan_summary: P and H are required");
    const int64_t DN = (int64_t)a->dim * a->dstate;
    if (a->seqlen == 0) {
        // Empty slice: the identity map (P = 1, H = 0); a combine over zero
        // chunks writes exactly that.
        return launch_combine(nullptr, nullptr, nullptr, 0, DN, a->batch, 0, P, H, st);
    }
    const int clen = choose_chunk_len(a->batch, a->seqlen, a->dim, a->chunk_len);
    ScanKParams kp = make_params(a, clen);
    if (kp.nchunks == 1) {
        kp.sumP = P;
        kp.sumH = H;
        return launch_scan_dtypes<kModeSummary>(kp, a->x_dtype, a->delta_dtype, a->bc_dtype, st);
    }
    const size_t need = scan_workspace_bytes(a);
    MB_CHECK_ARG(ws != nullptr && ws_bytes >= need, "scan_summary: workspace too small");
    float *sumP = static_cast<float *>(ws);
    float *sumH = sumP + (size_t)a->batch * kp.nchunks * DN;
    kp.sumP = sumP;
    kp.sumH = sumH;
    if (launch_scan_dtypes<kModeSummary>(kp, a->x_dtype, a->delta_dtype, a->bc_dtype, st)) return -1;
    return launch_combine(sumP, sumH, nullptr, kp.nchunks, DN, a->batch, 0, P, H, st);
}

int scan_compose_prefix(const float *PH, int world, int rank, int64_t count, const float *h0,
                        float *h_in, cudaStream_t st) {
    MB_CHECK_ARG(PH && h_in, "scan_compose_prefix: null buffer");
    MB_CHECK_ARG(world >= 1 && rank >= 0 && rank < world, "scan_compose_prefix: bad rank");
    if (count <= 0) return 0;
    const int threads = 256;
    scan_compose_prefix_kernel<<<(unsigned)ceil_div64(count, threads), threads, 0, st>>>(
        PH, rank, count, h0, h_in);
    return launch_status("scan_compose_prefix kernel");
}

}  // namespace mb
