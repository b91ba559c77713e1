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
// in registers; it walks time sequentially, so each (t, d, n) costs one
// exponential and no scan-operator overhead.  A CTA covers CH = 128 adjacent
// channels of one batch row and one time chunk.
//
// Staging.  When x, delta and z are channel-contiguous with 16-byte aligned
// rows (the layout of the model's activations), a 3-stage TMA pipeline
// brings [16 timesteps x 128 channels] tiles of each, and the [16 x N] tiles
// of B and C, into shared memory (cp.async.bulk.tensor, completion on an
// mbarrier), so the compute threads issue no global loads; each B/C tile is
// converted once per CTA into an FP32 double buffer read with broadcast
// loads.  B/C layouts TMA cannot describe are prefetched through registers.
// Any other layout goes through the generic kernel, which stages tiles with
// cooperative loads along whichever axis is contiguous.
//
// When batch * ceil(D / CH) CTAs are too few to fill the GPU, time is split
// into chunks (the carry propagation the reference intended in
// Sources/Kernels/prefix_scan.metal:19-40):
//   phase 1  each chunk computes its summary (P = prod a, H = h_end from 0),
//   phase 2  a combine kernel composes the summaries into the state entering
//            each chunk,
//   phase 3  each chunk rescans from its entering state and writes y.
// The same (P, H) monoid carries state across GPUs in sequence-sharded mode.
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>
#include <string>
#include <type_traits>
#include <vector>

#include "common.cuh"
#include "internal.h"
#include "scan_math.cuh"
#include "tma.cuh"
#include "umma.cuh"

namespace mb {

__device__ unsigned int g_device_error = 0;

namespace {

constexpr int kScanCH = 128;    // channels (= threads) per CTA
constexpr int kGenTT = 32;      // generic kernel: timesteps per tile
constexpr int kTmaTT = 16;      // TMA kernel: timesteps per tile
#ifndef MAMBA_SCAN_STAGES
#define MAMBA_SCAN_STAGES 3
#endif
constexpr int kTmaStages = MAMBA_SCAN_STAGES;  // TMA pipeline depth
// 4 resident CTAs (16 warps, up to 128 registers per thread) measured
// faster than 5 (96 registers) or 3: at [64, 4096, 4096] FP16 5.93 ms vs
// 6.23 and 6.20 ms.
#ifndef MAMBA_SCAN_MINCTAS
#define MAMBA_SCAN_MINCTAS 4
#endif
constexpr int kTmaMinCtas = MAMBA_SCAN_MINCTAS;  // resident CTAs per SM the TMA kernel is built for
// Register batch of 4 timesteps (softplus/SiLU of the batch, then its
// recurrences): 5.93 ms against 6.03 (8), 6.22 (2), 6.54 (16).
#ifndef MAMBA_SCAN_SUBTT
#define MAMBA_SCAN_SUBTT 4
#endif
constexpr int kSubTT = MAMBA_SCAN_SUBTT;  // timesteps per register batch inside a tile
constexpr int kChunkAlign = 32; // chunk lengths are multiples of both tile sizes

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

// ---- shared per-tile loop ------------------------------------------------------
// TT timesteps of one channel.  First the per-timestep scalars (softplus of
// delta, SiLU of the gate) for the whole tile -- independent chains, so the
// special-function pipe stays busy -- then the state recurrence, whose only
// serial dependence between timesteps is one packed FMA per state pair.
template <int NS, int CH, int TT, bool SUMMARY, bool PRECISE, bool SMALLA, bool FULL, typename Tx, typename Tdt>
__device__ __forceinline__ void run_tile(const ScanKParams &p, int nt, int t0, int b, int d,
                                         const Tx *__restrict__ sX, const Tdt *__restrict__ sDt,
                                         const Tx *__restrict__ sZ, const float *__restrict__ sBC,
                                         bool has_bias, float bias, float dskip, bool has_z, float2 *h,
                                         const float2 *Ac, const float2 *kI, float2 *P) {
    const int tid = threadIdx.x;
    float dtv[TT], gv[TT];
#pragma unroll
    for (int tt = 0; tt < TT; ++tt) {
        float draw = cvt_f32(sDt[tt * CH + tid]);
        if (has_bias) draw = __fadd_rn(draw, bias);
        dtv[tt] = scan_softplus<PRECISE>(draw);
        gv[tt] = 1.f;
        if (!SUMMARY && has_z) gv[tt] = scan_silu<PRECISE>(cvt_f32(sZ[tt * CH + tid]));
    }
    Tx *gy = static_cast<Tx *>(p.y) + (int64_t)b * p.sy[0] + (int64_t)t0 * p.sy[1] + (int64_t)d * p.sy[2];
#pragma unroll
    for (int tt = 0; tt < TT; ++tt) {
        if (FULL || tt < nt) {
            const float xv = cvt_f32(sX[tt * CH + tid]);
            const float s = scan_step<NS, SUMMARY, PRECISE, SMALLA>(xv, dtv[tt], sBC + tt * 2 * NS, h, Ac, kI, P);
            if (!SUMMARY) gy[(int64_t)tt * p.sy[1]] = cvt_out<Tx>(scan_output<PRECISE>(s, dskip, xv, gv[tt]));
        }
    }
}

// A tile of any length in sub-tiles of SUB timesteps; a full tile of TILE
// timesteps takes a fully unrolled path with every bound known at compile
// time (no per-step predicates).
template <int NS, int CH, int SUB, int TILE, bool SUMMARY, bool PRECISE, bool SMALLA, typename Tx, typename Tdt>
__device__ __forceinline__ void run_steps(const ScanKParams &p, int nt, int t0, int b, int d,
                                          const Tx *__restrict__ sX, const Tdt *__restrict__ sDt,
                                          const Tx *__restrict__ sZ, const float *__restrict__ sBC,
                                          bool has_bias, float bias, float dskip, bool has_z, float2 *h,
                                          const float2 *Ac, const float2 *kI, float2 *P) {
    static_assert(TILE % SUB == 0, "whole sub-tiles");
    if (nt == TILE) {
#pragma unroll
        for (int s0 = 0; s0 < TILE; s0 += SUB)
            run_tile<NS, CH, SUB, SUMMARY, PRECISE, SMALLA, true>(
                p, SUB, t0 + s0, b, d, sX + s0 * CH, sDt + s0 * CH, sZ + s0 * CH, sBC + s0 * 2 * NS, has_bias,
                bias, dskip, has_z, h, Ac, kI, P);
        return;
    }
    for (int s0 = 0; s0 < nt; s0 += SUB)
        run_tile<NS, CH, SUB, SUMMARY, PRECISE, SMALLA, false>(
            p, min(SUB, nt - s0), t0 + s0, b, d, sX + s0 * CH, sDt + s0 * CH, sZ + s0 * CH, sBC + s0 * 2 * NS,
            has_bias, bias, dskip, has_z, h, Ac, kI, P);
}

// B and C of one tile as FP32 [TT][2*NS] (B[0..NS) then C[0..NS) per
// timestep; zero beyond N, beyond the chunk, and C in summary mode).
template <int NS, int CH, int TT, typename Tbc, bool SUMMARY>
struct BCTile {
    static constexpr int kElems = TT * 2 * NS;
    static constexpr int kPer = (kElems + CH - 1) / CH;
    float v[kPer];
    __device__ __forceinline__ void load(const ScanKParams &p, int b, int t0, int t_end) {
        const Tbc *gB = static_cast<const Tbc *>(p.B);
        const Tbc *gC = static_cast<const Tbc *>(p.C);
#pragma unroll
        for (int i = 0; i < kPer; ++i) {
            const int e = threadIdx.x + i * CH;
            float val = 0.f;
            if (e < kElems) {
                const int tt = e / (2 * NS), j = e % (2 * NS);
                const int64_t t = t0 + tt;
                if (t < t_end) {
                    if (j < NS) {
                        if (j < p.N) val = ld_f32(gB + (int64_t)b * p.sB[0] + t * p.sB[1] + (int64_t)j * p.sB[2]);
                    } else if (!SUMMARY && j - NS < p.N) {
                        val = ld_f32(gC + (int64_t)b * p.sC[0] + t * p.sC[1] + (int64_t)(j - NS) * p.sC[2]);
                    }
                }
            }
            v[i] = val;
        }
    }
    __device__ __forceinline__ void store(float *dst) const {
#pragma unroll
        for (int i = 0; i < kPer; ++i) {
            const int e = threadIdx.x + i * CH;
            if (e < kElems) dst[e] = v[i];
        }
    }
};

// Stage a [TT, CH] tile of a per-channel tensor into shared memory (row tt,
// column c).  Channel-contiguous tensors are read one row per pass;
// otherwise consecutive threads read consecutive timesteps of one channel.
template <typename T, int CH, int TT>
__device__ __forceinline__ void stage_tile(T *s, const T *g, const int64_t *st, int b, int t0, int nt,
                                           int d0, int D) {
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

template <int NS>
__device__ __forceinline__ void write_epilogue(const ScanKParams &p, bool summary, int b, int chunk, int d,
                                               int t_end, const float2 *h, const float2 *P) {
    const int N = p.N;
    if (summary) {
        const int64_t off = (((int64_t)b * p.nchunks + chunk) * p.D + d) * N;
#pragma unroll
        for (int q = 0; q < NS / 2; ++q) {
            if (2 * q < N) {
                p.sumP[off + 2 * q] = P[q].x;
                p.sumH[off + 2 * q] = h[q].x;
            }
            if (2 * q + 1 < N) {
                p.sumP[off + 2 * q + 1] = P[q].y;
                p.sumH[off + 2 * q + 1] = h[q].y;
            }
        }
    } else if (p.final_state && t_end == p.L) {
        float *fs = p.final_state + ((int64_t)b * p.D + d) * N;
#pragma unroll
        for (int q = 0; q < NS / 2; ++q) {
            if (2 * q < N) fs[2 * q] = h[q].x;
            if (2 * q + 1 < N) fs[2 * q + 1] = h[q].y;
        }
    }
}

template <int NS>
__device__ __forceinline__ void load_initial_state(const ScanKParams &p, int b, int chunk, int d, float2 *h,
                                                   float2 *P) {
#pragma unroll
    for (int q = 0; q < NS / 2; ++q) {
        h[q] = make_float2(0.f, 0.f);
        P[q] = make_float2(1.f, 1.f);
    }
    if (p.h_init) {
        const int N = p.N;
        const float *src = p.h_init + (((int64_t)b * p.nchunks + chunk) * p.D + d) * N;
#pragma unroll
        for (int q = 0; q < NS / 2; ++q) {
            if (2 * q < N) h[q].x = src[2 * q];
            if (2 * q + 1 < N) h[q].y = src[2 * q + 1];
        }
    }
}

// ---- generic kernel (any strides) ------------------------------------------
template <int NS, int CH, int TT, typename Tx, typename Tdt, typename Tbc, int MODE>
__global__ void __launch_bounds__(CH) scan_generic_kernel(const ScanKParams p) {
    constexpr bool PRECISE = std::is_same<Tx, float>::value;
    constexpr bool SUMMARY = MODE == kModeSummary;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    float *sBC = reinterpret_cast<float *>(smem_raw);  // [TT][2*NS]
    Tx *sX = reinterpret_cast<Tx *>(sBC + TT * 2 * NS);  // [TT][CH]
    Tx *sZ = sX + TT * CH;                               // [TT][CH]
    Tdt *sDt = reinterpret_cast<Tdt *>(sZ + TT * CH);    // [TT][CH]

    const int tid = threadIdx.x;
    const int b = blockIdx.z, chunk = blockIdx.y;
    const int d0 = blockIdx.x * CH, d = d0 + tid;
    const bool dvalid = d < p.D;
    const int t_begin = chunk * p.chunk_len;
    const int t_end = min(p.L, t_begin + p.chunk_len);

    float2 Ac[NS / 2], kI[NS / 2], h[NS / 2], P[NS / 2];
    const bool small = load_channel_consts<NS, PRECISE>(p.A, d, p.N, dvalid, Ac, kI);
    if (dvalid && !SUMMARY) load_initial_state<NS>(p, b, chunk, d, h, P);
    else load_initial_state<NS>(ScanKParams{}, 0, 0, 0, h, P);
    const bool has_bias = p.dt_bias != nullptr;
    const float bias = (has_bias && dvalid) ? p.dt_bias[d] : 0.f;
    const float dskip = (p.Dskip && dvalid) ? p.Dskip[d] : 0.f;
    const bool any_small = __syncthreads_or(small);
    const bool has_z = !SUMMARY && p.z != nullptr;

    for (int t0 = t_begin; t0 < t_end; t0 += TT) {
        const int nt = min(TT, t_end - t0);
        stage_tile<Tx, CH, TT>(sX, static_cast<const Tx *>(p.x), p.sx, b, t0, nt, d0, p.D);
        stage_tile<Tdt, CH, TT>(sDt, static_cast<const Tdt *>(p.delta), p.sdt, b, t0, nt, d0, p.D);
        if (has_z) stage_tile<Tx, CH, TT>(sZ, static_cast<const Tx *>(p.z), p.sz, b, t0, nt, d0, p.D);
        {
            BCTile<NS, CH, TT, Tbc, SUMMARY> bc;
            bc.load(p, b, t0, t_end);
            bc.store(sBC);
        }
        __syncthreads();
        if (dvalid) {
            if (any_small)
                run_steps<NS, CH, kSubTT, TT, SUMMARY, PRECISE, true>(p, nt, t0, b, d, sX, sDt, sZ, sBC, has_bias,
                                                               bias, dskip, has_z, h, Ac, kI, P);
            else
                run_steps<NS, CH, kSubTT, TT, SUMMARY, PRECISE, false>(p, nt, t0, b, d, sX, sDt, sZ, sBC, has_bias, bias,
                                                            dskip, has_z, h, Ac, kI, P);
        }
        __syncthreads();
    }
    if (dvalid) write_epilogue<NS>(p, SUMMARY, b, chunk, d, t_end, h, P);
}

// ---- TMA-pipelined kernel (channel-contiguous, 16-byte aligned rows) ---------
template <int NS, int CH, int TT, int ST, typename Tx, typename Tdt, typename Tbc>
struct TmaLayout {
    static constexpr int align128(int v) { return (v + 127) / 128 * 128; }
    static constexpr int kXB = TT * CH * (int)sizeof(Tx);            // x or z tile
    static constexpr int kDB = TT * CH * (int)sizeof(Tdt);           // delta tile
    static constexpr int kBCB = align128(TT * NS * (int)sizeof(Tbc)); // raw B or C tile
    static constexpr int kOffD = kXB, kOffZ = kXB + kDB, kOffB = 2 * kXB + kDB, kOffC = kOffB + kBCB;
    static constexpr int kStage = kOffC + kBCB;                       // x | delta | z | B | C
    static constexpr int kBC = 2 * TT * 2 * NS * 4;                   // double-buffered FP32 B/C
    static constexpr int kBytes = ST * kStage + kBC + ST * 8;
    static_assert(kXB % 128 == 0 && kDB % 128 == 0, "TMA tiles must stay 128-byte aligned");
};

// Convert the raw B and C tiles of one stage into the FP32 [TT][2*NS] layout
// the recurrence reads (zero beyond N and beyond the chunk end).
template <int NS, int CH, int TT, typename Tbc, bool SUMMARY>
__device__ __forceinline__ void convert_bc(const Tbc *__restrict__ rawB, const Tbc *__restrict__ rawC,
                                           float *__restrict__ dst, int N, int t0, int t_end) {
    constexpr int kElems = TT * 2 * NS;
#pragma unroll
    for (int k = 0; k < (kElems + CH - 1) / CH; ++k) {
        const int e = threadIdx.x + k * CH;
        if (e < kElems) {
            const int tt = e / (2 * NS), j = e % (2 * NS);
            const int n = j < NS ? j : j - NS;
            float v = 0.f;
            if (n < N && t0 + tt < t_end && (j < NS || !SUMMARY))
                v = cvt_f32(j < NS ? rawB[tt * N + n] : rawC[tt * N + n]);
            dst[e] = v;
        }
    }
}

// BCTMA: B and C also arrive by TMA (when their layout allows it);
// otherwise each thread prefetches its share through registers.
template <int NS, int CH, int TT, int ST, typename Tx, typename Tdt, typename Tbc, int MODE, bool BCTMA>
__global__ void __launch_bounds__(CH, kTmaMinCtas)
    scan_tma_kernel(const ScanKParams p, const __grid_constant__ CUtensorMap tmx,
                    const __grid_constant__ CUtensorMap tmdt, const __grid_constant__ CUtensorMap tmz,
                    const __grid_constant__ CUtensorMap tmB, const __grid_constant__ CUtensorMap tmC) {
    constexpr bool PRECISE = std::is_same<Tx, float>::value;
    constexpr bool SUMMARY = MODE == kModeSummary;
    using Lay = TmaLayout<NS, CH, TT, ST, Tx, Tdt, Tbc>;
    extern __shared__ __align__(128) unsigned char smem[];
    float *bcf = reinterpret_cast<float *>(smem + ST * Lay::kStage);                    // [2][TT][2*NS]
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + ST * Lay::kStage + Lay::kBC);  // [ST]

    const int tid = threadIdx.x;
    const int b = blockIdx.z, chunk = blockIdx.y;
    const int d0 = blockIdx.x * CH, d = d0 + tid;
    const bool dvalid = d < p.D;
    const int N = p.N;
    const int t_begin = chunk * p.chunk_len;
    const int t_end = min(p.L, t_begin + p.chunk_len);
    const int ntiles = t_end > t_begin ? (t_end - t_begin + TT - 1) / TT : 0;
    const bool has_z = !SUMMARY && p.z != nullptr;
    const uint32_t bc_box = (uint32_t)(N * TT * (int)sizeof(Tbc));
    const uint32_t tx_bytes = Lay::kXB + Lay::kDB + (has_z ? Lay::kXB : 0) +
                              (BCTMA ? bc_box * (SUMMARY ? 1u : 2u) : 0u);

    float2 Ac[NS / 2], kI[NS / 2], h[NS / 2], P[NS / 2];
    const bool small = load_channel_consts<NS, PRECISE>(p.A, d, N, dvalid, Ac, kI);
    if (dvalid && !SUMMARY) load_initial_state<NS>(p, b, chunk, d, h, P);
    else load_initial_state<NS>(ScanKParams{}, 0, 0, 0, h, P);
    const bool has_bias = p.dt_bias != nullptr;
    const float bias = (has_bias && dvalid) ? p.dt_bias[d] : 0.f;
    const float dskip = (p.Dskip && dvalid) ? p.Dskip[d] : 0.f;

    if (tid == 0) {
        prefetch_tensormap(&tmx);
        prefetch_tensormap(&tmdt);
        if (has_z) prefetch_tensormap(&tmz);
        if (BCTMA) {
            prefetch_tensormap(&tmB);
            if (!SUMMARY) prefetch_tensormap(&tmC);
        }
        for (int s = 0; s < ST; ++s) mbar_init(&bars[s], 1);
        fence_mbar_init();
    }
    const bool any_small = __syncthreads_or(small);

    auto issue = [&](int tile, int s) {
        unsigned char *stg = smem + s * Lay::kStage;
        const int t = t_begin + tile * TT;
        mbar_arrive_expect_tx(&bars[s], tx_bytes);
        tma_load_3d(stg, &tmx, &bars[s], d0, t, b);
        tma_load_3d(stg + Lay::kOffD, &tmdt, &bars[s], d0, t, b);
        if (has_z) tma_load_3d(stg + Lay::kOffZ, &tmz, &bars[s], d0, t, b);
        if (BCTMA) {
            tma_load_3d(stg + Lay::kOffB, &tmB, &bars[s], 0, t, b);
            if (!SUMMARY) tma_load_3d(stg + Lay::kOffC, &tmC, &bars[s], 0, t, b);
        }
    };
    auto stage_bc = [&](int s, int t0, float *dst) {
        const unsigned char *stg = smem + s * Lay::kStage;
        convert_bc<NS, CH, TT, Tbc, SUMMARY>(reinterpret_cast<const Tbc *>(stg + Lay::kOffB),
                                             reinterpret_cast<const Tbc *>(stg + Lay::kOffC), dst, N, t0, t_end);
    };
    if (tid == 0)
        for (int s = 0; s < min(ST, ntiles); ++s) issue(s, s);

    BCTile<NS, CH, TT, Tbc, SUMMARY> bc;
    bool ok0 = true;
    if (ntiles > 0) {
        if (BCTMA) {
            ok0 = mbar_wait_bounded(&bars[0], 0u);
            if (ok0) stage_bc(0, t_begin, bcf);
        } else {
            bc.load(p, b, t_begin, t_end);
            bc.store(bcf);
        }
    }
    int i = 0;
    bool aborted = __syncthreads_or(!ok0);
    for (; !aborted && i < ntiles; ++i) {
        const int s = i % ST;
        const int t0 = t_begin + i * TT;
        const int nt = min(TT, t_end - t0);
        if (!BCTMA && i + 1 < ntiles) bc.load(p, b, t0 + TT, t_end);
        bool ok = mbar_wait_bounded(&bars[s], (uint32_t)((i / ST) & 1));
        if (ok && dvalid) {
            const unsigned char *stg = smem + s * Lay::kStage;
            const Tx *sX = reinterpret_cast<const Tx *>(stg);
            const Tdt *sDt = reinterpret_cast<const Tdt *>(stg + Lay::kOffD);
            const Tx *sZ = reinterpret_cast<const Tx *>(stg + Lay::kOffZ);
            const float *sBC = bcf + (i & 1) * TT * 2 * NS;
            if (any_small)
                run_steps<NS, CH, kSubTT, TT, SUMMARY, PRECISE, true>(p, nt, t0, b, d, sX, sDt, sZ, sBC, has_bias,
                                                                   bias, dskip, has_z, h, Ac, kI, P);
            else
                run_steps<NS, CH, kSubTT, TT, SUMMARY, PRECISE, false>(p, nt, t0, b, d, sX, sDt, sZ, sBC, has_bias,
                                                                    bias, dskip, has_z, h, Ac, kI, P);
        }
        if (i + 1 < ntiles) {
            float *next = bcf + ((i + 1) & 1) * TT * 2 * NS;
            if (BCTMA) {
                const int s1 = (i + 1) % ST;
                const bool ok1 = mbar_wait_bounded(&bars[s1], (uint32_t)(((i + 1) / ST) & 1));
                if (ok1) stage_bc(s1, t0 + TT, next);
                ok = ok && ok1;
            } else {
                bc.store(next);
            }
        }
        // One barrier per tile: the stage and the B/C buffer are free again,
        // and a timed-out wait anywhere in the CTA aborts all of it.
        if (__syncthreads_or(!ok)) {
            aborted = true;
            break;
        }
        if (tid == 0 && i + ST < ntiles) issue(i + ST, s);
    }
    if (aborted) {
        if (tid == 0) {
            atomicOr(&g_device_error, kErrTmaTimeout);
            // Let copies still in flight into this CTA's shared memory land
            // (each wait bounded) before the CTA exits.
            for (int j = i; j < min(i + ST, ntiles); ++j)
                mbar_wait_bounded(&bars[j % ST], (uint32_t)((j / ST) & 1));
        }
        __syncthreads();
        return;
    }
    if (dvalid) write_epilogue<NS>(p, SUMMARY, b, chunk, d, t_end, h, P);
}

// ---- the scan with dt_proj on the tensor cores --------------------------------
// The layer's dt_proj (draw = dt_r @ W_dt^T, K = dt_rank <= 128) folded into
// the one-thread TMA scan, so the [T, d_inner] draw tensor is never written
// to or read from HBM.  Per CTA (128 channels): W_dt's 128 rows live in TMEM
// (lane = channel, K along columns, two FP16 per column), loaded once.  Per
// 16-step tile the TMA ring brings the dt_r tile [16 x dt_rank] (FP16,
// 128-byte swizzle) in place of the delta tile; one thread issues
// tcgen05.mma (M 128 channels, N 16 steps, A from TMEM, B from shared
// memory) into one of three 16-column TMEM accumulators, two tiles ahead
// of its use, and each thread reads its channel's 16 values with tcgen05.ld,
// rounds them to FP16 (the values the separate GEMM would store) and writes
// them over the consumed dt_r tile, where the unchanged recurrence reads
// them as its delta tile.  Every wait is bounded; TMEM is freed on every
// path.
template <int ST>
struct DtLayout {
    static constexpr int RS = ST + 1;                  // dt_r slots: one tile ahead of the main ring
    static constexpr int kXB = kTmaTT * kScanCH * 2;   // x or z tile, FP16
    static constexpr int kBCB = kTmaTT * 16 * 2;       // B or C tile, FP16
    static constexpr int kOffZ = kXB, kOffB = 2 * kXB, kOffC = kOffB + kBCB;
    static constexpr int kStage = kOffC + kBCB;        // x | z | B | C
    static constexpr int kDR = 2 * kTmaTT * 128;       // dt_r: two [16 x 64] FP16 boxes; later the FP16 draw tile
    static constexpr int kOffDR = 0;                   // dt_r slots first (1 KB aligned for the swizzle)
    static constexpr int kOffStages = RS * kDR;
    static constexpr int kBC = 2 * kTmaTT * 2 * 16 * 4;  // double-buffered FP32 B/C
    static constexpr int kOffBC = kOffStages + ST * kStage;
    static constexpr int kOffBars = kOffBC + kBC;
    static constexpr int kBytes = 1024 + kOffBars + (ST + RS + 3 + 1) * 8 + 16;
    static_assert(kDR == kTmaTT * kScanCH * 2, "the draw tile reuses its dt_r slot");
    static_assert(kStage % 128 == 0, "TMA destinations stay 128-byte aligned");
};
constexpr int kDtMaxRank = 128;
constexpr int kDtTmemCols = 128;  // W_dt (64 columns) + three 16-column accumulators

template <int ST>
__global__ void __launch_bounds__(kScanCH, kTmaMinCtas)
    scan_dtmma_kernel(const ScanKParams p, const __grid_constant__ CUtensorMap tmx,
                      const __grid_constant__ CUtensorMap tmdr, const __grid_constant__ CUtensorMap tmz,
                      const __grid_constant__ CUtensorMap tmB, const __grid_constant__ CUtensorMap tmC,
                      const __half *__restrict__ wdt, int R) {
    constexpr int NS = 16, CH = kScanCH, TT = kTmaTT;
    using Lay = DtLayout<ST>;
    constexpr int RS = Lay::RS;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *dr_slots = smem + Lay::kOffDR;                             // [RS] dt_r boxes / draw tiles
    uint8_t *stages = smem + Lay::kOffStages;                           // [ST] x | z | B | C
    float *bcf = reinterpret_cast<float *>(smem + Lay::kOffBC);         // [2][TT][2*NS]
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + Lay::kOffBars);  // [ST] main copies landed
    uint64_t *dbars = bars + ST;                                        // [RS] dt_r copies landed
    uint64_t *mbars = dbars + RS;                                       // [3] draw accumulator ready
    uint64_t *drain = mbars + 3;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);

    const int tid = threadIdx.x, warp = tid >> 5;
    const int b = blockIdx.z;
    const int d0 = blockIdx.x * CH, d = d0 + tid;
    const bool dvalid = d < p.D;
    const int N = p.N, L = p.L;
    const int ntiles = (L + TT - 1) / TT;
    const bool has_z = p.z != nullptr;
    const int nkb = (R + 63) / 64;  // 64-wide K boxes of dt_r (zero past dt_rank)
    const uint32_t tx_main = Lay::kXB + (has_z ? Lay::kXB : 0) + 2u * (uint32_t)(N * TT * 2);
    const uint32_t tx_dr = (uint32_t)(nkb * TT * 128);
    constexpr uint32_t idesc = idesc_f16_f32acc(128, TT);

    float2 Ac[NS / 2], kI[NS / 2], h[NS / 2], P[NS / 2];
    const bool small = load_channel_consts<NS, false>(p.A, d, N, dvalid, Ac, kI);
    if (dvalid) load_initial_state<NS>(p, b, 0, d, h, P);
    else load_initial_state<NS>(ScanKParams{}, 0, 0, 0, h, P);
    const bool has_bias = p.dt_bias != nullptr;
    const float bias = (has_bias && dvalid) ? p.dt_bias[d] : 0.f;
    const float dskip = (p.Dskip && dvalid) ? p.Dskip[d] : 0.f;

    if (tid == 0) {
        prefetch_tensormap(&tmx);
        prefetch_tensormap(&tmdr);
        if (has_z) prefetch_tensormap(&tmz);
        prefetch_tensormap(&tmB);
        prefetch_tensormap(&tmC);
        for (int s = 0; s < ST; ++s) mbar_init(&bars[s], 1);
        for (int s = 0; s < RS; ++s) mbar_init(&dbars[s], 1);
        for (int s = 0; s < 3; ++s) mbar_init(&mbars[s], 1);
        mbar_init(drain, 1);
        fence_mbar_init();
    }
    if (warp == 0) {
        tmem_alloc(tmem_slot, kDtTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    const bool any_small = __syncthreads_or(small);
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    // this channel's row of W_dt (K-major, zero past dt_rank) as 64 columns of
    // packed FP16 pairs, 16 columns at a time
    {
        const uint4 *src = reinterpret_cast<const uint4 *>(wdt + (int64_t)(dvalid ? d : 0) * R);
#pragma unroll
        for (int c4 = 0; c4 < 4; ++c4) {
            uint32_t wr[16];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int g = 4 * c4 + i;  // 8 FP16 per 16-byte load
                const uint4 v = (dvalid && 8 * g < R) ? src[g] : make_uint4(0u, 0u, 0u, 0u);
                wr[4 * i] = v.x;
                wr[4 * i + 1] = v.y;
                wr[4 * i + 2] = v.z;
                wr[4 * i + 3] = v.w;
            }
            tmem_st_32x32b_x16(tmem + lane_base + 16 * c4, wr);
        }
    }
    tmem_wait_st();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();

    auto issue = [&](int tile) {
        const int s = tile % ST;
        uint8_t *stg = stages + s * Lay::kStage;
        const int t = tile * TT;
        mbar_arrive_expect_tx(&bars[s], tx_main);
        tma_load_3d(stg, &tmx, &bars[s], d0, t, b);
        if (has_z) tma_load_3d(stg + Lay::kOffZ, &tmz, &bars[s], d0, t, b);
        tma_load_3d(stg + Lay::kOffB, &tmB, &bars[s], 0, t, b);
        tma_load_3d(stg + Lay::kOffC, &tmC, &bars[s], 0, t, b);
    };
    auto issue_dr = [&](int tile) {
        const int r = tile % RS;
        mbar_arrive_expect_tx(&dbars[r], tx_dr);
        for (int kb = 0; kb < nkb; ++kb)
            tma_load_3d(dr_slots + r * Lay::kDR + kb * TT * 128, &tmdr, &dbars[r], kb * 64, tile * TT, b);
    };
    // One thread: the draw tile of `tile` into accumulator tile % 3, once its
    // dt_r boxes have landed.
    auto issue_mma = [&](int tile) -> bool {
        const int r = tile % RS;
        if (!mbar_wait_bounded(&dbars[r], (uint32_t)((tile / RS) & 1))) return false;
        tc_fence_after();
        const uint32_t b_addr = smem_u32(dr_slots + r * Lay::kDR);
        const uint32_t d_tmem = tmem + 64 + 16 * (tile % 3);
        for (int kk = 0; kk < 4 * nkb; ++kk)
            umma_f16_ts(d_tmem, tmem + 8 * kk, smem_desc_sw128(b_addr + (kk >> 2) * TT * 128 + (kk & 3) * 32), idesc,
                        kk != 0);
        umma_commit(&mbars[tile % 3]);
        return true;
    };
    auto stage_bc = [&](int tile, float *dst) {
        const uint8_t *stg = stages + (tile % ST) * Lay::kStage;
        convert_bc<NS, CH, TT, __half, false>(reinterpret_cast<const __half *>(stg + Lay::kOffB),
                                              reinterpret_cast<const __half *>(stg + Lay::kOffC), dst, N, tile * TT,
                                              L);
    };
    bool ok0 = true;
    if (tid == 0) {
        for (int t = 0; t < min(RS, ntiles); ++t) issue_dr(t);
        for (int t = 0; t < min(ST, ntiles); ++t) issue(t);
        for (int t = 0; t < min(2, ntiles); ++t) ok0 = ok0 && issue_mma(t);
    }
    if (ntiles > 0) {
        ok0 = ok0 && mbar_wait_bounded(&bars[0], 0u);
        if (ok0) stage_bc(0, bcf);
    }
    int i = 0;
    bool aborted = __syncthreads_or(!ok0);
    for (; !aborted && i < ntiles; ++i) {
        const int s = i % ST;
        const int t0 = i * TT;
        const int nt = min(TT, L - t0);
        bool ok = mbar_wait_bounded(&bars[s], (uint32_t)((i / ST) & 1)) &&
                  mbar_wait_bounded(&mbars[i % 3], (uint32_t)((i / 3) & 1));
        ok = __all_sync(0xffffffffu, ok);  // the TMEM load below is warp-collective
        if (ok) {
            tc_fence_after();
            uint32_t v[16];
            tmem_ld_32x32b_x16(tmem + lane_base + 64 + 16 * (i % 3), v);
            tmem_wait_ld();
            // over the consumed dt_r boxes: this thread's column of the FP16 draw tile
            __half *sD = reinterpret_cast<__half *>(dr_slots + (i % RS) * Lay::kDR);
#pragma unroll
            for (int tt = 0; tt < TT; ++tt) sD[tt * CH + tid] = __float2half_rn(__uint_as_float(v[tt]));
            if (dvalid) {
                const uint8_t *stg = stages + s * Lay::kStage;
                const __half *sX = reinterpret_cast<const __half *>(stg);
                const __half *sZ = reinterpret_cast<const __half *>(stg + Lay::kOffZ);
                const float *sBC = bcf + (i & 1) * TT * 2 * NS;
                if (any_small)
                    run_steps<NS, CH, kSubTT, TT, false, false, true>(p, nt, t0, b, d, sX, sD, sZ, sBC, has_bias,
                                                                     bias, dskip, has_z, h, Ac, kI, P);
                else
                    run_steps<NS, CH, kSubTT, TT, false, false, false>(p, nt, t0, b, d, sX, sD, sZ, sBC, has_bias,
                                                                      bias, dskip, has_z, h, Ac, kI, P);
            }
        }
        if (i + 1 < ntiles) {
            float *next = bcf + ((i + 1) & 1) * TT * 2 * NS;
            const bool ok1 = mbar_wait_bounded(&bars[(i + 1) % ST], (uint32_t)(((i + 1) / ST) & 1));
            if (ok1) stage_bc(i + 1, next);
            ok = ok && ok1;
        }
        // two tiles ahead: its dt_r boxes were issued two tiles ago
        if (tid == 0 && i + 2 < ntiles) ok = ok && issue_mma(i + 2);
        // the stage, the draw tile and this tile's accumulator are reused next
        fence_proxy_async_smem();
        tc_fence_before();
        if (__syncthreads_or(!ok)) {
            aborted = true;
            break;
        }
        tc_fence_after();
        if (tid == 0) {
            if (i + ST < ntiles) issue(i + ST);
            if (i + RS < ntiles) issue_dr(i + RS);
        }
    }
    if (tid == 0) {
        // every issued MMA has finished before TMEM is freed
        umma_commit(drain);
        if (!mbar_wait_bounded(drain, 0u)) aborted = true;
        if (aborted) {
            atomicOr(&g_device_error, kErrTmaTimeout);
            // copies still landing in this CTA's shared memory finish first
            for (int j = i; j < min(i + ST, ntiles); ++j) mbar_wait_bounded(&bars[j % ST], (uint32_t)((j / ST) & 1));
            for (int j = i; j < min(i + RS, ntiles); ++j) mbar_wait_bounded(&dbars[j % RS], (uint32_t)((j / RS) & 1));
        }
    }
    tc_fence_before();
    aborted = __syncthreads_or(aborted);
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, kDtTmemCols);
    }
    if (!aborted && dvalid) write_epilogue<NS>(p, false, b, 0, d, L, h, P);
}

// ---- four lanes per channel (few channels, single pass) ----------------------
// For problems with fewer 128-channel CTAs than SMs, one thread per channel
// is bound by the latency of a timestep, and splitting time into chunks
// doubles the work.  Here four lanes share a channel, each holding NS/4 of
// its states, so a timestep's exponentials are spread over four lanes and
// four times as many warps are in flight.  A CTA serves 32 channels of one
// batch row; tiles of x, delta, z ([TT steps x 32 channels]) and B, C come
// through the same 3-stage TMA ring as the one-thread kernel, B and C
// converted once per tile to FP32.  Each lane evaluates the timestep's
// softplus and SiLU itself (no exchange needed), updates its states with
// state_update (the fast path of the one-thread kernel) and the four partial
// sums of C*h are combined with two butterfly shuffles.  Output mode only.
constexpr int kQuadCPB = 32;  // channels per CTA

// One timestep of one lane's S states (S even: packed pairs, as scan_step):
// bq, cq point at this lane's B and C values in the FP32 tile.
template <int S, bool SMALLA>
__device__ __forceinline__ float quad_states(float x, float dt, const float *__restrict__ bq,
                                             const float *__restrict__ cq, float2 *h, const float2 *ac,
                                             const float2 *kI) {
    static_assert(S % 2 == 0, "packed pairs");
    float2 Bv[S / 2], Cv[S / 2];
    if (S == 4) {
        const float4 b4 = *reinterpret_cast<const float4 *>(bq), c4 = *reinterpret_cast<const float4 *>(cq);
        Bv[0] = make_float2(b4.x, b4.y);
        Bv[S / 2 - 1] = make_float2(b4.z, b4.w);
        Cv[0] = make_float2(c4.x, c4.y);
        Cv[S / 2 - 1] = make_float2(c4.z, c4.w);
    } else {
#pragma unroll
        for (int p = 0; p < S / 2; ++p) {
            Bv[p] = reinterpret_cast<const float2 *>(bq)[p];
            Cv[p] = reinterpret_cast<const float2 *>(cq)[p];
        }
    }
    const float2 dt2 = make_float2(dt, dt), x2 = make_float2(x, x);
    float2 y = make_float2(0.f, 0.f);
#pragma unroll
    for (int p = 0; p < S / 2; ++p) {
        const float2 dA = __fmul2_rn(dt2, ac[p]);
        const float2 a = make_float2(ex2_approx(dA.x), ex2_approx(dA.y));
        const float2 w = __fmul2_rn(x2, Bv[p]);
        if (SMALLA) {
            h[p].x = state_update(a.x, w.x, kI[p].x, dt, h[p].x);
            h[p].y = state_update(a.y, w.y, kI[p].y, dt, h[p].y);
        } else {
            const float2 sk = __ffma2_rn(w, kI[p], h[p]);
            h[p] = __ffma2_rn(__fadd2_rn(a, make_float2(-1.f, -1.f)), sk, h[p]);
        }
        y = __ffma2_rn(Cv[p], h[p], y);
    }
    return y.x + y.y;
}

template <int NS, int TT, int ST, typename Tx, typename Tdt, typename Tbc>
__global__ void __launch_bounds__(128, 4)
    scan_quad_kernel(const ScanKParams p, const __grid_constant__ CUtensorMap tmx,
                     const __grid_constant__ CUtensorMap tmdt, const __grid_constant__ CUtensorMap tmz,
                     const __grid_constant__ CUtensorMap tmB, const __grid_constant__ CUtensorMap tmC) {
    constexpr int S = NS / 4, CPB = kQuadCPB;
    using Lay = TmaLayout<NS, CPB, TT, ST, Tx, Tdt, Tbc>;
    extern __shared__ __align__(128) unsigned char smem[];
    float *bcf = reinterpret_cast<float *>(smem + ST * Lay::kStage);                    // [2][TT][2*NS]
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + ST * Lay::kStage + Lay::kBC);  // [ST]

    const int tid = threadIdx.x, q = tid & 3, c = tid >> 2, qbase = (tid & 31) & ~3;
    const int b = blockIdx.y;
    const int d0 = blockIdx.x * CPB, d = d0 + c;
    const bool valid = d < p.D;
    const int dd = valid ? d : 0;
    const int N = p.N, L = p.L;
    const int ntiles = (L + TT - 1) / TT;
    const bool has_z = p.z != nullptr;
    const uint32_t bc_box = (uint32_t)(N * TT * (int)sizeof(Tbc));
    const uint32_t tx_bytes = Lay::kXB + Lay::kDB + (has_z ? Lay::kXB : 0) + 2u * bc_box;

    static_assert(S % 2 == 0, "4 lanes x an even number of states");
    float2 ac[S / 2], kI[S / 2], h[S / 2];
    bool small = false;
#pragma unroll
    for (int j = 0; j < S; ++j) {
        const int n = q * S + j;
        const float a = (valid && n < N) ? p.A[(int64_t)dd * N + n] : 0.f;
        const float ki = fabsf(a) > 1e-6f ? __frcp_rn(a) : 0.f;
        const float h0 = (valid && n < N && p.h_init) ? p.h_init[((int64_t)b * p.D + dd) * N + n] : 0.f;
        small |= valid && n < N && ki == 0.f;
        if (j & 1) {
            ac[j / 2].y = a * kLog2e;
            kI[j / 2].y = ki;
            h[j / 2].y = h0;
        } else {
            ac[j / 2].x = a * kLog2e;
            kI[j / 2].x = ki;
            h[j / 2].x = h0;
        }
    }
    const bool has_bias = p.dt_bias != nullptr;
    const float bias = (has_bias && valid) ? p.dt_bias[dd] : 0.f;
    const float dskip = (p.Dskip && valid) ? p.Dskip[dd] : 0.f;
    Tx *gy = static_cast<Tx *>(p.y) + (int64_t)b * p.sy[0] + (int64_t)dd * p.sy[2];

    if (tid == 0) {
        prefetch_tensormap(&tmx);
        prefetch_tensormap(&tmdt);
        if (has_z) prefetch_tensormap(&tmz);
        prefetch_tensormap(&tmB);
        prefetch_tensormap(&tmC);
        for (int s = 0; s < ST; ++s) mbar_init(&bars[s], 1);
        fence_mbar_init();
    }
    // A state with |A| <= 1e-6 anywhere in the CTA selects the per-state
    // branch of the update (uniform, so the packed form serves the rest).
    const bool any_small = __syncthreads_or(small);

    auto issue = [&](int tile, int s) {
        unsigned char *stg = smem + s * Lay::kStage;
        const int t = tile * TT;
        mbar_arrive_expect_tx(&bars[s], tx_bytes);
        tma_load_3d(stg, &tmx, &bars[s], d0, t, b);
        tma_load_3d(stg + Lay::kOffD, &tmdt, &bars[s], d0, t, b);
        if (has_z) tma_load_3d(stg + Lay::kOffZ, &tmz, &bars[s], d0, t, b);
        tma_load_3d(stg + Lay::kOffB, &tmB, &bars[s], 0, t, b);
        tma_load_3d(stg + Lay::kOffC, &tmC, &bars[s], 0, t, b);
    };
    auto stage_bc = [&](int s, int t0, float *dst) {
        const unsigned char *stg = smem + s * Lay::kStage;
        convert_bc<NS, 128, TT, Tbc, false>(reinterpret_cast<const Tbc *>(stg + Lay::kOffB),
                                            reinterpret_cast<const Tbc *>(stg + Lay::kOffC), dst, N, t0, L);
    };
    if (tid == 0)
        for (int s = 0; s < min(ST, ntiles); ++s) issue(s, s);

    bool ok0 = true;
    if (ntiles > 0) {
        ok0 = mbar_wait_bounded(&bars[0], 0u);
        if (ok0) stage_bc(0, 0, bcf);
    }
    int i = 0;
    bool aborted = __syncthreads_or(!ok0);
    for (; !aborted && i < ntiles; ++i) {
        const int s = i % ST;
        const int t0 = i * TT;
        const int nt = min(TT, L - t0);
        // warp-uniform verdict: the shuffles below need every lane
        bool ok = __all_sync(0xffffffffu, mbar_wait_bounded(&bars[s], (uint32_t)((i / ST) & 1)));
        if (ok) {
            const unsigned char *stg = smem + s * Lay::kStage;
            const Tx *sX = reinterpret_cast<const Tx *>(stg);
            const Tdt *sDt = reinterpret_cast<const Tdt *>(stg + Lay::kOffD);
            const Tx *sZ = reinterpret_cast<const Tx *>(stg + Lay::kOffZ);
            const float *sBC = bcf + (i & 1) * TT * 2 * NS;
            // Groups of four timesteps: lane q evaluates x, softplus(delta)
            // and SiLU(z) of timestep q of the group (one each, so the quad
            // does no redundant special-function work) and the quad shares
            // them by shuffle; then the four recurrences, whose C*h sums are
            // reduced after the group, off the state's dependency chain.
            auto group = [&](const int g0, const int lim, auto small_tag) {
                constexpr bool SMALLA = decltype(small_tag)::value;
                const int sq = g0 + q;  // < TT: TT is a multiple of 4
                const float xq = cvt_f32(sX[sq * CPB + c]);
                float drq = cvt_f32(sDt[sq * CPB + c]);
                if (has_bias) drq = __fadd_rn(drq, bias);
                const float dq = softplus_fast(drq);
                const float gq = has_z ? silu_fast(cvt_f32(sZ[sq * CPB + c])) : 1.f;
                float xs[4], ds[4], gs[4], yp[4];
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    xs[k] = __shfl_sync(0xffffffffu, xq, qbase | k);
                    ds[k] = __shfl_sync(0xffffffffu, dq, qbase | k);
                    gs[k] = __shfl_sync(0xffffffffu, gq, qbase | k);
                }
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    yp[k] = 0.f;
                    if (g0 + k < lim) {  // uniform across the CTA
                        const float *bc = sBC + (g0 + k) * 2 * NS + q * S;
                        yp[k] = quad_states<S, SMALLA>(xs[k], ds[k], bc, bc + NS, h, ac, kI);
                    }
                }
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    yp[k] += __shfl_xor_sync(0xffffffffu, yp[k], 1);
                    yp[k] += __shfl_xor_sync(0xffffffffu, yp[k], 2);
                }
                // lane k of the quad stores timestep k of the group
                float yo = yp[0], xo = xs[0], go = gs[0];
#pragma unroll
                for (int k = 1; k < 4; ++k)
                    if (q == k) {
                        yo = yp[k];
                        xo = xs[k];
                        go = gs[k];
                    }
                if (valid && g0 + q < lim) gy[(int64_t)(t0 + g0 + q) * p.sy[1]] = cvt_out<Tx>(fmaf(dskip, xo, yo) * go);
            };
            using Small = std::integral_constant<bool, true>;
            using Packed = std::integral_constant<bool, false>;
            if (nt == TT && !any_small) {
                // full tile: every offset and bound is a compile-time constant
#pragma unroll
                for (int g0 = 0; g0 < TT; g0 += 4) group(g0, TT, Packed{});
            } else if (any_small) {
                for (int g0 = 0; g0 < nt; g0 += 4) group(g0, nt, Small{});
            } else {
                for (int g0 = 0; g0 < nt; g0 += 4) group(g0, nt, Packed{});
            }
        }
        if (i + 1 < ntiles) {
            float *next = bcf + ((i + 1) & 1) * TT * 2 * NS;
            const int s1 = (i + 1) % ST;
            const bool ok1 = mbar_wait_bounded(&bars[s1], (uint32_t)(((i + 1) / ST) & 1));
            if (ok1) stage_bc(s1, t0 + TT, next);
            ok = ok && ok1;
        }
        if (__syncthreads_or(!ok)) {
            aborted = true;
            break;
        }
        if (tid == 0 && i + ST < ntiles) issue(i + ST, s);
    }
    if (aborted) {
        if (tid == 0) {
            atomicOr(&g_device_error, kErrTmaTimeout);
            for (int j = i; j < min(i + ST, ntiles); ++j)
                mbar_wait_bounded(&bars[j % ST], (uint32_t)((j / ST) & 1));
        }
        __syncthreads();
        return;
    }
    if (p.final_state && valid) {
#pragma unroll
        for (int j = 0; j < S; ++j)
            if (q * S + j < N)
                p.final_state[((int64_t)b * p.D + d) * N + q * S + j] = (j & 1) ? h[j / 2].y : h[j / 2].x;
    }
}

// ---- phase 2 and the cross-rank composition -----------------------------------
// Compose the chunk summaries of every (b, d, n) in time order.  On entry
// H/P hold the summaries [batch, nchunks, D*N]; when write_hin is set, H is
// overwritten in place with the state entering each chunk.
__global__ void scan_combine_kernel(const float *__restrict__ P, float *__restrict__ H,
                                    const float *__restrict__ h0, int nchunks, int64_t DN, int64_t total,
                                    int write_hin, float *__restrict__ P_total, float *__restrict__ H_total) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= total) return;
    const int64_t b = i / DN, r = i % DN;
    float h = h0 ? h0[i] : 0.f;
    float pt = 1.f;
    // Loads for 8 chunks are issued before the dependent combine chain, so
    // the walk is not one HBM round trip per chunk.
    constexpr int kAhead = 8;
    for (int c0 = 0; c0 < nchunks; c0 += kAhead) {
        float pc[kAhead], hc[kAhead];
#pragma unroll
        for (int j = 0; j < kAhead; ++j) {
            if (c0 + j < nchunks) {
                const int64_t idx = (b * nchunks + c0 + j) * DN + r;
                pc[j] = P[idx];
                hc[j] = H[idx];
            }
        }
#pragma unroll
        for (int j = 0; j < kAhead; ++j) {
            if (c0 + j < nchunks) {
                if (write_hin) H[(b * nchunks + c0 + j) * DN + r] = h;
                h = pc[j] * h + hc[j];
                pt *= pc[j];
            }
        }
    }
    if (H_total) H_total[i] = h;
    if (P_total) P_total[i] = pt;
}

// State entering rank `rank` from the gathered summaries PH[world][2][count].
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

// ---- host side ------------------------------------------------------------------
}  // namespace

// The driver's tensor-map encoder, looked up once per process.
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    });
    return fn;
}

namespace {

// 3-D map over a [batch, L, dim0] tensor with stride 1 along dim0; box
// [1, TT, box0].  False when the layout does not meet the TMA rules
// (16-byte aligned base, 16-byte multiple strides and box rows), in which
// case another staging path is used.
bool encode_map(CUtensorMap *m, const void *ptr, int dtype, int dim0, int L, int B, const int64_t *st, int box0) {
    auto fn = tensor_map_encoder();
    if (!fn || !ptr || st[2] != 1) return false;
    const int64_t es = dtype == MAMBA_F16 ? 2 : 4;
    if (reinterpret_cast<uintptr_t>(ptr) % 16 || (box0 * es) % 16) return false;
    const int64_t row = st[1] * es;
    int64_t bat = st[0] * es;
    if (row <= 0 || row % 16 || row < dim0 * es) return false;
    if (B == 1) bat = row * std::max(L, 1);
    if (bat <= 0 || bat % 16) return false;
    cuuint64_t dims[3] = {(cuuint64_t)dim0, (cuuint64_t)L, (cuuint64_t)B};
    cuuint64_t strides[2] = {(cuuint64_t)row, (cuuint64_t)bat};
    cuuint32_t box[3] = {(cuuint32_t)box0, (cuuint32_t)kTmaTT, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    const CUresult r = fn(m, dtype == MAMBA_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
                          3, const_cast<void *>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                          CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

template <int NS, typename Tx, typename Tdt, typename Tbc, int MODE, bool BCTMA>
int launch_tma(const ScanKParams &kp, const CUtensorMap *maps, cudaStream_t st) {
    constexpr int CH = kScanCH, TT = kTmaTT, ST = kTmaStages;
    auto kern = scan_tma_kernel<NS, CH, TT, ST, Tx, Tdt, Tbc, MODE, BCTMA>;
    const int smem = TmaLayout<NS, CH, TT, ST, Tx, Tdt, Tbc>::kBytes;
    MB_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    MB_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100));
    dim3 grid(ceil_div(kp.D, CH), kp.nchunks, kp.batch);
    kern<<<grid, CH, smem, st>>>(kp, maps[0], maps[1], maps[2], maps[3], maps[4]);
    return launch_status("selective_scan (TMA) kernel");
}

template <int NS, typename Tx, typename Tdt, typename Tbc, int MODE>
int launch_generic(const ScanKParams &kp, cudaStream_t st) {
    constexpr int CH = kScanCH, TT = kGenTT;
    auto kern = scan_generic_kernel<NS, CH, TT, Tx, Tdt, Tbc, MODE>;
    const size_t smem = (size_t)TT * 2 * NS * 4 + (size_t)TT * CH * (2 * sizeof(Tx) + sizeof(Tdt));
    MB_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    dim3 grid(ceil_div(kp.D, CH), kp.nchunks, kp.batch);
    kern<<<grid, CH, smem, st>>>(kp);
    return launch_status("selective_scan kernel");
}

template <int NS, typename Tx, typename Tdt, typename Tbc, int MODE>
int launch_scan_ns(const ScanKParams &kp, int xd, int dd, int bd, cudaStream_t st) {
    CUtensorMap maps[5];  // x, delta, z, B, C
    const bool want_z = MODE == kModeOutput && kp.z != nullptr;
    const bool tma = kp.L > 0 && encode_map(&maps[0], kp.x, xd, kp.D, kp.L, kp.batch, kp.sx, kScanCH) &&
                     encode_map(&maps[1], kp.delta, dd, kp.D, kp.L, kp.batch, kp.sdt, kScanCH) &&
                     (!want_z || encode_map(&maps[2], kp.z, xd, kp.D, kp.L, kp.batch, kp.sz, kScanCH));
    if (!tma) return launch_generic<NS, Tx, Tdt, Tbc, MODE>(kp, st);
    if (!want_z) maps[2] = maps[0];  // unused by the kernel
    const bool bc_tma = kp.N == NS && encode_map(&maps[3], kp.B, bd, kp.N, kp.L, kp.batch, kp.sB, kp.N) &&
                        (MODE == kModeSummary || encode_map(&maps[4], kp.C, bd, kp.N, kp.L, kp.batch, kp.sC, kp.N));
    if (bc_tma) {
        if (MODE == kModeSummary) maps[4] = maps[3];  // unused by the kernel
        return launch_tma<NS, Tx, Tdt, Tbc, MODE, true>(kp, maps, st);
    }
    maps[3] = maps[4] = maps[0];  // unused by the kernel
    return launch_tma<NS, Tx, Tdt, Tbc, MODE, false>(kp, maps, st);
}

template <typename Tx, typename Tdt, typename Tbc, int MODE>
int launch_scan_n(const ScanKParams &kp, int xd, int dd, int bd, cudaStream_t st) {
    if (kp.N <= 4) return launch_scan_ns<4, Tx, Tdt, Tbc, MODE>(kp, xd, dd, bd, st);
    if (kp.N <= 8) return launch_scan_ns<8, Tx, Tdt, Tbc, MODE>(kp, xd, dd, bd, st);
    return launch_scan_ns<16, Tx, Tdt, Tbc, MODE>(kp, xd, dd, bd, st);
}

template <int MODE>
int launch_scan_dtypes(const ScanKParams &kp, int xd, int dd, int bd, cudaStream_t st) {
    if (xd == MAMBA_F32 && dd == MAMBA_F32 && bd == MAMBA_F32)
        return launch_scan_n<float, float, float, MODE>(kp, xd, dd, bd, st);
    if (xd == MAMBA_F16 && dd == MAMBA_F16 && bd == MAMBA_F16)
        return launch_scan_n<__half, __half, __half, MODE>(kp, xd, dd, bd, st);
    if (xd == MAMBA_F16 && dd == MAMBA_F32 && bd == MAMBA_F16)
        return launch_scan_n<__half, float, __half, MODE>(kp, xd, dd, bd, st);
    if (xd == MAMBA_F16 && dd == MAMBA_F32 && bd == MAMBA_F32)
        return launch_scan_n<__half, float, float, MODE>(kp, xd, dd, bd, st);
    set_error("selective_scan: unsupported dtype combination (x, delta, B/C)");
    return -1;
}

// Time-chunk length for these dims.  One chunk per channel when the
// channel CTAs alone fill the GPU; otherwise split time so that about eight
// CTAs per SM exist, keeping chunks >= 128 steps.
int choose_chunk_len(int batch, int L, int D, int requested) {
    if (L <= 0) return 1;
    if (requested > 0) {
        const int c = ceil_div(requested, kChunkAlign) * kChunkAlign;
        return std::min(c, L);
    }
    // One pass over time costs L steps of one CTA's latency (about 360 SM
    // cycles per step when a warp has its scheduler to itself); splitting
    // time into chunks doubles the work (summary + rescan) but spreads it
    // over idle SMs.  Measured on B200 (FP16, N 16): with at least one CTA
    // per SM the single pass wins (batch 16 x 4096 channels, L 4096:
    // 1.79 ms vs 2.75-2.90 ms chunked); below that chunking wins (batch 8
    // x 1536 channels, L 2048: 0.32-0.33 vs 0.39 ms; batch 1 x 2048,
    // L 131072: 2.8 vs 24 ms).
    const int64_t ctas = (int64_t)batch * ceil_div(D, kScanCH);
    const int sms = device_sm_count();
    if (ctas >= sms) return L;
    const int64_t want = ceil_div64(8LL * sms, ctas);
    const int64_t maxc = std::max<int64_t>(1, L / 128);
    const int64_t nc = std::min(want, maxc);
    if (nc <= 1) return L;
    const int clen = (int)(ceil_div64(ceil_div64(L, nc), kChunkAlign) * kChunkAlign);
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

int launch_combine(const float *P, float *H, const float *h0, int nchunks, int64_t DN, int batch, int write_hin,
                   float *P_total, float *H_total, cudaStream_t st) {
    const int64_t total = (int64_t)batch * DN;
    if (total == 0) return 0;
    const int threads = 256;
    scan_combine_kernel<<<(unsigned)ceil_div64(total, threads), threads, 0, st>>>(P, H, h0, nchunks, DN, total,
                                                                                 write_hin, P_total, H_total);
    return launch_status("scan_combine kernel");
}

}  // namespace

namespace {

// The four-lanes-per-channel pass serves FP16 problems that would otherwise
// be split into time chunks (fewer 128-channel CTAs than SMs) but have at
// least one 32-channel CTA per SM, in the layout its TMA tiles need
// (channel-contiguous rows, 16-byte aligned; B and C with exactly 8 or 16
// states).  Other problems keep the chunked path.
bool quad_rows_ok(const void *ptr, const int64_t *st, int es, int dim0, int batch) {
    if (!ptr) return true;  // not given: checked where it is required
    if (st[2] != 1 || reinterpret_cast<uintptr_t>(ptr) % 16) return false;
    const int64_t row = st[1] * es, bat = st[0] * es;
    return row > 0 && row % 16 == 0 && row >= (int64_t)dim0 * es && (batch == 1 || (bat > 0 && bat % 16 == 0));
}

bool use_quad(const MambaScanArgs *a) {
    if (a->chunk_len > 0 || a->seqlen <= 0 || a->x_dtype != MAMBA_F16) return false;
    if (a->dstate != 8 && a->dstate != 16) return false;
    const int sms = device_sm_count();
    const int64_t ctas = (int64_t)a->batch * ceil_div(a->dim, kScanCH);
    const int64_t quads = (int64_t)a->batch * ceil_div(a->dim, kQuadCPB);
    if (ctas >= sms || quads < sms) return false;
    const int xs = 2, ds = a->delta_dtype == MAMBA_F16 ? 2 : 4, bs = a->bc_dtype == MAMBA_F16 ? 2 : 4;
    return quad_rows_ok(a->x, a->x_stride, xs, a->dim, a->batch) &&
           quad_rows_ok(a->delta, a->delta_stride, ds, a->dim, a->batch) &&
           quad_rows_ok(a->z, a->z_stride, xs, a->dim, a->batch) &&
           quad_rows_ok(a->B, a->B_stride, bs, a->dstate, a->batch) &&
           quad_rows_ok(a->C, a->C_stride, bs, a->dstate, a->batch);
}

template <int NS, typename Tdt, typename Tbc>
int launch_quad_t(const ScanKParams &kp, int dd, int bd, cudaStream_t st) {
    constexpr int TT = kTmaTT, ST = kTmaStages;
    CUtensorMap maps[5];
    const bool ok = encode_map(&maps[0], kp.x, MAMBA_F16, kp.D, kp.L, kp.batch, kp.sx, kQuadCPB) &&
                    encode_map(&maps[1], kp.delta, dd, kp.D, kp.L, kp.batch, kp.sdt, kQuadCPB) &&
                    (!kp.z || encode_map(&maps[2], kp.z, MAMBA_F16, kp.D, kp.L, kp.batch, kp.sz, kQuadCPB)) &&
                    encode_map(&maps[3], kp.B, bd, kp.N, kp.L, kp.batch, kp.sB, kp.N) &&
                    encode_map(&maps[4], kp.C, bd, kp.N, kp.L, kp.batch, kp.sC, kp.N);
    MB_CHECK_ARG(ok, "selective_scan: tensor map encoding failed");
    if (!kp.z) maps[2] = maps[0];  // unused by the kernel
    auto kern = scan_quad_kernel<NS, TT, ST, __half, Tdt, Tbc>;
    const int smem = TmaLayout<NS, kQuadCPB, TT, ST, __half, Tdt, Tbc>::kBytes;
    MB_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    dim3 grid(ceil_div(kp.D, kQuadCPB), kp.batch);
    kern<<<grid, 128, smem, st>>>(kp, maps[0], maps[1], maps[2], maps[3], maps[4]);
    return launch_status("selective scan (4 lanes per channel) kernel");
}

template <int NS>
int launch_quad_ns(const ScanKParams &kp, int dd, int bd, cudaStream_t st) {
    if (dd == MAMBA_F16 && bd == MAMBA_F16) return launch_quad_t<NS, __half, __half>(kp, dd, bd, st);
    if (dd == MAMBA_F32 && bd == MAMBA_F16) return launch_quad_t<NS, float, __half>(kp, dd, bd, st);
    if (dd == MAMBA_F32 && bd == MAMBA_F32) return launch_quad_t<NS, float, float>(kp, dd, bd, st);
    set_error("selective_scan: unsupported dtype combination (x, delta, B/C)");
    return -1;
}

int launch_quad(const ScanKParams &kp, const MambaScanArgs *a, cudaStream_t st) {
    if (a->dstate == 8) return launch_quad_ns<8>(kp, a->delta_dtype, a->bc_dtype, st);
    return launch_quad_ns<16>(kp, a->delta_dtype, a->bc_dtype, st);
}

}  // namespace

namespace {

// 3-D map of dt_r (the first dt_rank columns of x_proj's output): dims
// {dt_rank, L, batch}, box [64 x 16 steps], 128-byte swizzle (the K-major
// B-operand layout of tcgen05.mma); columns past dt_rank read zeros.
bool encode_dt_r(CUtensorMap *m, const void *ptr, int R, int L, int B, const int64_t *st) {
    auto fn = tensor_map_encoder();
    if (!fn || !ptr || reinterpret_cast<uintptr_t>(ptr) % 16) return false;
    const int64_t row = st[1] * 2;
    int64_t bat = st[0] * 2;
    if (row <= 0 || row % 16 || row < (int64_t)R * 2) return false;
    if (B == 1) bat = row * std::max(L, 1);
    if (bat <= 0 || bat % 16) return false;
    cuuint64_t dims[3] = {(cuuint64_t)R, (cuuint64_t)L, (cuuint64_t)B};
    cuuint64_t strides[2] = {(cuuint64_t)row, (cuuint64_t)bat};
    cuuint32_t box[3] = {64, (cuuint32_t)kTmaTT, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void *>(ptr), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

bool scan_dtproj_supported(const MambaScanArgs *a, int R) {
    if (!a || a->batch <= 0 || a->dim <= 0 || a->seqlen <= 0) return false;
    if (a->x_dtype != MAMBA_F16 || a->bc_dtype != MAMBA_F16 || a->dstate != 16 || a->chunk_len > 0) return false;
    if (R < 8 || R > kDtMaxRank || R % 8) return false;
    return (int64_t)a->batch * ceil_div(a->dim, kScanCH) >= device_sm_count();
}

int selective_scan_dtproj(const MambaScanArgs *a, const void *dt_r, const int64_t *dr_stride, const void *w_dt,
                          int R, cudaStream_t st) {
    if (validate(a)) return -1;
    if (a->batch == 0 || a->dim == 0 || a->seqlen == 0) return selective_scan(a, nullptr, 0, st);
    MB_CHECK_ARG(dt_r && w_dt && dr_stride && a->y && a->C, "selective_scan_dtproj: null pointer");
    MB_CHECK_ARG(a->x_dtype == MAMBA_F16 && a->bc_dtype == MAMBA_F16 && a->dstate == 16,
                 "selective_scan_dtproj: needs FP16 x, z, B, C and 16 states");
    MB_CHECK_ARG(R >= 8 && R <= kDtMaxRank && R % 8 == 0,
                 "selective_scan_dtproj: dt_rank must be a multiple of 8 in 8..128");
    MB_CHECK_ARG(reinterpret_cast<uintptr_t>(w_dt) % 16 == 0, "selective_scan_dtproj: w_dt must be 16-byte aligned");
    MB_CHECK_ARG(a->chunk_len == 0 && scan_dtproj_supported(a, R),
                 "selective_scan_dtproj: needs batch * ceil(dim / 128) >= the SM count (one pass over time)");
    int dev = 0, major = 0;
    MB_CUDA_TRY(cudaGetDevice(&dev));
    MB_CUDA_TRY(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev));
    MB_CHECK_ARG(major == 10, "selective_scan_dtproj: needs a compute capability 10.x GPU (tcgen05)");
    ScanKParams kp = make_params(a, a->seqlen);
    kp.h_init = a->initial_state;
    CUtensorMap maps[5];  // x, dt_r, z, B, C
    const bool ok = encode_map(&maps[0], kp.x, MAMBA_F16, kp.D, kp.L, kp.batch, kp.sx, kScanCH) &&
                    encode_dt_r(&maps[1], dt_r, R, kp.L, kp.batch, dr_stride) &&
                    (!kp.z || encode_map(&maps[2], kp.z, MAMBA_F16, kp.D, kp.L, kp.batch, kp.sz, kScanCH)) &&
                    encode_map(&maps[3], kp.B, MAMBA_F16, kp.N, kp.L, kp.batch, kp.sB, kp.N) &&
                    encode_map(&maps[4], kp.C, MAMBA_F16, kp.N, kp.L, kp.batch, kp.sC, kp.N);
    MB_CHECK_ARG(ok, "selective_scan_dtproj: a tensor does not meet the TMA layout rules "
                     "(channel-contiguous 16-byte aligned rows)");
    if (!kp.z) maps[2] = maps[0];  // unused by the kernel
    constexpr int ST = kTmaStages;
    auto kern = scan_dtmma_kernel<ST>;
    const int smem = DtLayout<ST>::kBytes;
    MB_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    MB_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100));
    dim3 grid(ceil_div(kp.D, kScanCH), 1, kp.batch);
    kern<<<grid, kScanCH, smem, st>>>(kp, maps[0], maps[1], maps[2], maps[3], maps[4],
                                      static_cast<const __half *>(w_dt), R);
    return launch_status("selective scan with dt_proj (tcgen05) kernel");
}

// Carry scratch of the time-chunked path for these args (whether or not a
// single pass would be chosen instead).
size_t chunked_workspace_bytes(const MambaScanArgs *a) {
    if (!a || a->batch <= 0 || a->dim <= 0 || a->seqlen <= 0) return 0;
    const int clen = choose_chunk_len(a->batch, a->seqlen, a->dim, a->chunk_len);
    const int nc = ceil_div(a->seqlen, clen);
    if (nc <= 1) return 0;
    return 2 * sizeof(float) * (size_t)a->batch * nc * a->dim * a->dstate;
}

size_t scan_workspace_bytes(const MambaScanArgs *a) {
    if (!a || a->batch <= 0 || a->dim <= 0 || a->seqlen <= 0) return 0;
    if (use_quad(a)) return 0;
    const int clen = choose_chunk_len(a->batch, a->seqlen, a->dim, a->chunk_len);
    const int nc = ceil_div(a->seqlen, clen);
    if (nc <= 1) return 0;
    return 2 * sizeof(float) * (size_t)a->batch * nc * a->dim * a->dstate;
}

int selective_scan(const MambaScanArgs *a, void *ws, size_t ws_bytes, cudaStream_t st) {
    if (validate(a)) return -1;
    if (a->batch == 0 || a->dim == 0) return 0;
    if (a->seqlen > 0) MB_CHECK_ARG(a->y && a->C, "selective_scan: y and C are required");
    if (use_quad(a)) {
        ScanKParams kp = make_params(a, a->seqlen);
        kp.h_init = a->initial_state;
        return launch_quad(kp, a, st);
    }
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
    if (launch_combine(sumP, sumH, a->initial_state, kp.nchunks, DN, a->batch, 1, nullptr, nullptr, st)) return -1;
    kp.h_init = sumH;
    return launch_scan_dtypes<kModeOutput>(kp, a->x_dtype, a->delta_dtype, a->bc_dtype, st);
}

int scan_summary(const MambaScanArgs *a, float *P, float *H, void *ws, size_t ws_bytes, cudaStream_t st) {
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
    const size_t need = chunked_workspace_bytes(a);
    MB_CHECK_ARG(ws != nullptr && ws_bytes >= need, "scan_summary: workspace too small");
    float *sumP = static_cast<float *>(ws);
    float *sumH = sumP + (size_t)a->batch * kp.nchunks * DN;
    kp.sumP = sumP;
    kp.sumH = sumH;
    if (launch_scan_dtypes<kModeSummary>(kp, a->x_dtype, a->delta_dtype, a->bc_dtype, st)) return -1;
    return launch_combine(sumP, sumH, nullptr, kp.nchunks, DN, a->batch, 0, P, H, st);
}

// Sequence-sharded mode in two passes over the slice (instead of a summary
// pass followed by a full chunked scan, which would repeat the chunk
// summaries).  Pass 1 leaves the chunk summaries in `ws` and writes the
// slice's total map to P_tot / H_tot; pass 2 combines the stored summaries
// from the entering state a->initial_state and runs the output pass.  Both
// use the chunking choose_chunk_len gives these args, so `ws` (of
// scan_workspace_bytes(a) bytes) carries the summaries between them.
int scan_seqpar_pass1(const MambaScanArgs *a, float *P_tot, float *H_tot, void *ws, size_t ws_bytes,
                      cudaStream_t st) {
    if (validate(a)) return -1;
    if (a->batch == 0 || a->dim == 0) return 0;
    const int64_t DN = (int64_t)a->dim * a->dstate;
    if (a->seqlen == 0) return launch_combine(nullptr, nullptr, nullptr, 0, DN, a->batch, 0, P_tot, H_tot, st);
    const int clen = choose_chunk_len(a->batch, a->seqlen, a->dim, a->chunk_len);
    ScanKParams kp = make_params(a, clen);
    if (kp.nchunks == 1) {
        kp.sumP = P_tot;
        kp.sumH = H_tot;
        return launch_scan_dtypes<kModeSummary>(kp, a->x_dtype, a->delta_dtype, a->bc_dtype, st);
    }
    MB_CHECK_ARG(ws != nullptr && ws_bytes >= chunked_workspace_bytes(a), "scan_seqpar: workspace too small");
    kp.sumP = static_cast<float *>(ws);
    kp.sumH = kp.sumP + (size_t)a->batch * kp.nchunks * DN;
    if (launch_scan_dtypes<kModeSummary>(kp, a->x_dtype, a->delta_dtype, a->bc_dtype, st)) return -1;
    return launch_combine(kp.sumP, kp.sumH, nullptr, kp.nchunks, DN, a->batch, 0, P_tot, H_tot, st);
}

int scan_seqpar_pass2(const MambaScanArgs *a, void *ws, size_t ws_bytes, cudaStream_t st) {
    if (validate(a)) return -1;
    if (a->batch == 0 || a->dim == 0) return 0;
    if (a->seqlen == 0) return selective_scan(a, nullptr, 0, st);
    MB_CHECK_ARG(a->y && a->C, "selective_scan: y and C are required");
    const int clen = choose_chunk_len(a->batch, a->seqlen, a->dim, a->chunk_len);
    ScanKParams kp = make_params(a, clen);
    if (kp.nchunks == 1) {
        kp.h_init = a->initial_state;
        return launch_scan_dtypes<kModeOutput>(kp, a->x_dtype, a->delta_dtype, a->bc_dtype, st);
    }
    MB_CHECK_ARG(ws != nullptr && ws_bytes >= chunked_workspace_bytes(a), "scan_seqpar: workspace too small");
    const int64_t DN = (int64_t)a->dim * a->dstate;
    float *sumP = static_cast<float *>(ws);
    float *sumH = sumP + (size_t)a->batch * kp.nchunks * DN;
    if (launch_combine(sumP, sumH, a->initial_state, kp.nchunks, DN, a->batch, 1, nullptr, nullptr, st)) return -1;
    kp.h_init = sumH;
    return launch_scan_dtypes<kModeOutput>(kp, a->x_dtype, a->delta_dtype, a->bc_dtype, st);
}

int scan_compose_prefix(const float *PH, int world, int rank, int64_t count, const float *h0, float *h_in,
                        cudaStream_t st) {
    MB_CHECK_ARG(PH && h_in, "scan_compose_prefix: null buffer");
    MB_CHECK_ARG(world >= 1 && rank >= 0 && rank < world, "scan_compose_prefix: bad rank");
    if (count <= 0) return 0;
    const int threads = 256;
    scan_compose_prefix_kernel<<<(unsigned)ceil_div64(count, threads), threads, 0, st>>>(PH, rank, count, h0,
                                                                                          h_in);
    return launch_status("scan_compose_prefix kernel");
}

// ---- no-allocation entry point ------------------------------------------------
// Scratch for mamba_selective_scan_noalloc: a fixed 32 MiB array in the
// module's global memory.  Every device that loads this library holds it
// until the process exits.  In host code `g_noalloc_scratch` is only a
// host-side stand-in for the symbol, so its device address is looked up once
// per device with cudaGetSymbolAddress and that address is what the kernels
// receive.
constexpr size_t kNoAllocScratchBytes = size_t(32) << 20;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

namespace {

// The calling thread's current driver context, through the runtime's
// driver entry point (the library links only the runtime).
CUcontext current_context() {
    using GetCtx = CUresult (*)(CUcontext *);
    static GetCtx fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<GetCtx>(f);
    });
    CUcontext c = nullptr;
    if (!fn || fn(&c) != CUDA_SUCCESS) return nullptr;
    return c;
}

// Device address of g_noalloc_scratch on the current device, resolved with
// that device current on the first call there.  The address is cached with
// the context it was resolved in: after a device reset the module is loaded
// again in a new context, possibly elsewhere, and the address is looked up
// again.  (A thread that has not yet touched the device reports no context;
// the lookup itself then makes the primary context current.)
int noalloc_scratch(void **out) {
    static std::mutex mu;
    struct Slot {
        CUcontext ctx = nullptr;
        void *ptr = nullptr;
    };
    static std::vector<Slot> cache;
    int dev = 0;
    MB_CUDA_TRY(cudaGetDevice(&dev));
    const CUcontext ctx = current_context();
    std::lock_guard<std::mutex> lk(mu);
    if ((int)cache.size() <= dev) cache.resize(dev + 1);
    Slot &sl = cache[dev];
    if (!sl.ptr || !ctx || sl.ctx != ctx) {
        void *p = nullptr;
        MB_CUDA_TRY(cudaGetSymbolAddress(&p, g_noalloc_scratch));
        sl.ptr = p;
        sl.ctx = ctx;
    }
    *out = sl.ptr;
    return 0;
}

}  // namespace

int selective_scan_noalloc(const MambaScanArgs *a, cudaStream_t st) {
    if (validate(a)) return -1;
    const size_t need = scan_workspace_bytes(a);
    if (need > kNoAllocScratchBytes) {
        set_error("selective_scan_noalloc: these sizes need " + std::to_string(need) +
                  " bytes of scratch, above the static maximum of " + std::to_string(kNoAllocScratchBytes) +
                  " bytes; call mamba_selective_scan with a workspace instead");
        return -1;
    }
    void *ws = nullptr;
    if (need > 0 && noalloc_scratch(&ws)) return -1;
    return selective_scan(a, ws, need > 0 ? kNoAllocScratchBytes : 0, st);
}

namespace {

// A bounded mbarrier wait that nothing completes: the CTA's one thread
// initialises a barrier expecting one arrival, makes none, waits with the
// given limit through the same helper the pipelines use, and on timeout
// records kErrWaitSelftest in the device status and returns.
constexpr unsigned kErrWaitSelftest = 8u;

__global__ void bounded_wait_selftest_kernel(uint64_t limit_ns, int *waited_out) {
    __shared__ uint64_t bar;
    if (threadIdx.x != 0) return;
    mbar_init(&bar, 1);
    fence_mbar_init();
    const bool ok = mbar_wait_bounded(&bar, 0u, limit_ns);
    *waited_out = ok ? 0 : 1;
    if (!ok) atomicOr(&g_device_error, kErrWaitSelftest);
}

}  // namespace

int bounded_wait_selftest(unsigned limit_us, cudaStream_t st) {
    MB_CHECK_ARG(limit_us > 0 && limit_us <= 1000000u, "bounded_wait_selftest: limit must be in (0, 1 s]");
    int *flag = nullptr;
    MB_CUDA_TRY(cudaMallocAsync(&flag, sizeof(int), st));
    MB_CUDA_TRY(cudaMemsetAsync(flag, 0, sizeof(int), st));
    bounded_wait_selftest_kernel<<<1, 32, 0, st>>>((uint64_t)limit_us * 1000ull, flag);
    if (launch_status("bounded-wait selftest kernel")) return -1;
    int h = 0;
    MB_CUDA_TRY(cudaMemcpyAsync(&h, flag, sizeof(int), cudaMemcpyDeviceToHost, st));
    MB_CUDA_TRY(cudaFreeAsync(flag, st));
    MB_CUDA_TRY(cudaStreamSynchronize(st));
    MB_CHECK_ARG(h == 1, "bounded_wait_selftest: the wait did not report a timeout");
    return 0;
}

unsigned device_error_flags(bool clear) {
    unsigned v = 0;
    if (cudaMemcpyFromSymbol(&v, g_device_error, sizeof(v)) != cudaSuccess) return ~0u;
    if (clear && v) {
        const unsigned z = 0;
        cudaMemcpyToSymbol(g_device_error, &z, sizeof(z));
    }
    return v;
}

}  // namespace mb
