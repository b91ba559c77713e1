// gemm_tc.cu -- the Mamba block's projections on the fifth-generation
// tensor cores: C = A @ W^T with FP16 operands and FP32 accumulation, the
// job of linear_f16 (Sources/Kernels/projection.metal:32-49) for the
// in_proj, x_proj, dt_proj and out_proj GEMMs of the layer graph
// (Sources/Mamba/MambaRuntime.cpp:93-101).
//
//   A  FP16 [M, K] rows of lda elements (activations, K-major)
//   W  FP16 [N, K] (the reference's [K, N] weight transposed once at load)
//   C  [M, N] rows of ldc elements; epilogues (bias: optional FP32 [N]):
//        kProjF16     C (FP16)  = acc + bias      (in_proj, x_proj, dt_proj)
//        kProjF32Add  C (FP32) += acc + bias      (out_proj into the residual)
//        kProjF32     C (FP32)  = acc + bias
//
// Structure: a persistent kernel run by CTA pairs (thread-block clusters of
// two, cta_group::2).  A pair owns a 256 x BN output tile (BN <= 256): each
// CTA loads 128 rows of A and BN/2 rows of W per 64-wide K block by TMA
// (128-byte swizzle) into its own 5-stage ring (4 with the conv), and one thread of the even
// CTA issues tcgen05.mma with M = 256 that reads both CTAs' shared memory
// and accumulates in both CTAs' TMEM (each CTA gets its 128 rows).  Per SM
// and K block that is 32 KB of operands for a 128 x 256 x 64 slab, two
// thirds of what one CTA alone would load for the same slab.  TMEM holds two
// accumulators, so the epilogue of one tile overlaps the MMAs of the next.
//
// Roles (64 + 32 * epilogue warps threads per CTA):
//   warp 0 lane 0  TMA producer.  Its copies complete on the even CTA's
//                  stage barrier, which expects the bytes of both CTAs.
//   warp 1         TMEM owner (both CTAs); in the even CTA one lane issues
//                  the MMAs and commits them to both CTAs' barriers.
//   warps 2..      epilogue (8 warps; 4 for the conv-fused variant): warp w
//                  reads TMEM lane quarter w % 4, i.e. 32 rows, and a share
//                  of the column chunks: TMEM -> registers -> a
//                  128-byte-swizzled shared-memory box of 32 rows -> bulk
//                  tensor store (or bulk tensor add for the residual),
//                  double-buffered per warp; then the warp releases the
//                  accumulator to the even CTA's MMA thread.
// Every mbarrier wait is bounded (2 s); on timeout the role stops, bit 4 of
// the device status is set, and both CTAs still reach the final cluster
// barrier, so TMEM is freed and neither CTA exits while its peer may touch
// its shared memory.
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>
#include <vector>

#include "common.cuh"
#include "internal.h"
#include "scan_math.cuh"
#include "tma.cuh"
#include "umma.cuh"

namespace mb {

__device__ unsigned int g_proj_error = 0;

namespace {

constexpr int kPBK = 64;                          // K per stage: one 128-byte swizzle row
constexpr int kPUK = 16;                          // K per MMA
// Plain epilogues: 8 epilogue warps (two per TMEM lane quarter, splitting
// the tile's column chunks) and 5 stages.  The conv-fused epilogue: 4 warps
// (its halo exchange pairs warps by quarter) and 4 stages, making room for
// the conv input tile.
template <bool CONV>
struct ProjCfg {
    static constexpr int kStages = CONV ? 4 : 5;
    static constexpr int kEpiWarps = CONV ? 4 : 8;
    static constexpr int kThreads = 64 + 32 * kEpiWarps;
};
constexpr int kPAccCols = 256;                    // TMEM columns per accumulator
constexpr int kPTmemCols = 2 * kPAccCols;
constexpr int kPStageA = 128 * kPBK * 2;          // 16 KB: this CTA's 128 rows of A
constexpr int kPStageB = 128 * kPBK * 2;          // 16 KB: up to 128 rows of W
constexpr int kPStage = kPStageA + kPStageB;
constexpr int kPEpiBox = 32 * 128;                // 4 KB: 32 rows x 128 bytes
constexpr int kPXPitch = 68;                      // bytes per row of the conv input tile (32 FP16 + pad)
constexpr int kPXchBytes = 2 * 128 * kPXPitch;    // conv input tile [128 rows][32 cols] FP16, double-buffered
template <bool CONV>
constexpr int proj_smem_bytes() {
    return ProjCfg<CONV>::kStages * kPStage + ProjCfg<CONV>::kEpiWarps * 2 * kPEpiBox + (CONV ? kPXchBytes : 0) +
           1024 /* alignment */ + 256 /* barriers */;
}
static_assert(proj_smem_bytes<false>() <= 232448 && proj_smem_bytes<true>() <= 232448, "shared memory");
constexpr unsigned kErrProjTimeout = 16u;

struct ProjParams {
    const float *bias;              // [N] FP32 added to every row, or NULL
    const float *conv_w, *conv_b;   // conv-fused in_proj: [D, 4] and [D] FP32
    int M, N, K;
    int BN;          // output columns per tile (multiple of 16, <= 256)
    int m_tiles, n_tiles, kblocks;
    int mode;
    int halo;        // rows each CTA computes ahead of its first output row (3 when the conv is fused)
    int L;           // conv-fused: sequence length (the conv restarts at every multiple of L)
    int x_tiles;     // conv-fused: column tiles 0..x_tiles-1 hold the conv input x, the rest z
    int up_row0;     // gated (SwiGLU): first W row of the up projection (h); 0 otherwise
    uint32_t idesc;
    uint32_t tx_bytes;  // operand bytes of one stage, both CTAs
};

__device__ __forceinline__ bool warp_wait_p(uint64_t *bar, uint32_t parity) {
    int ok = 0;
    if ((threadIdx.x & 31) == 0) ok = mbar_wait_bounded(bar, parity) ? 1 : 0;
    return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

__device__ __forceinline__ uint32_t pack_half2(uint32_t a, uint32_t b) {
    const __half2 h = __floats2half2_rn(__uint_as_float(a), __uint_as_float(b));
    return *reinterpret_cast<const uint32_t *>(&h);
}
__device__ __forceinline__ uint32_t pack_half2f(float a, float b) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t *>(&h);
}

// Row `r` of a 32-row box of 128-byte rows with the TMA 128-byte swizzle:
// 16-byte chunk j lands at chunk j ^ (r % 8).
__device__ __forceinline__ void st_swizzled(uint8_t *box, int r, int j, uint4 v) {
    *reinterpret_cast<uint4 *>(box + r * 128 + ((j ^ (r & 7)) << 4)) = v;
}

// The four epilogue warps (threads 64..191) synchronise among themselves.
__device__ __forceinline__ void epilogue_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// Same barrier, returning whether `ok` holds in every epilogue thread, so
// that the warps leave their tile loop together (a warp that left alone
// would strand the others at the next barrier).
__device__ __forceinline__ bool epilogue_all(bool ok) {
    uint32_t r;
    asm volatile(
        "{\n"
        " .reg .pred p, q;\n"
        " setp.ne.u32 p, %1, 0;\n"
        " bar.red.and.pred q, 1, 128, p;\n"
        " selp.u32 %0, 1, 0, q;\n"
        "}\n"
        : "=r"(r)
        : "r"((uint32_t)ok)
        : "memory");
    return r != 0;
}

// Conv (width 4) + bias + SiLU down one column of 32 rows of the shared
// FP16 tile (element (r, col) at xc[r * kPXPitch / 2]), rows r0 .. r0+31,
// window (w0, w1, w2) = the three rows before r0; the FP16 result of row i
// goes to row (i - SKIP) & 31 of the 128-byte-swizzled output box (rows
// SKIP-1 .. below 0 wrap to rows the store never reads).  `off[k]` is this
// lane's byte offset within a box row whose swizzle phase is k.  FAST: no
// sequence starts inside the window; otherwise the window restarts (zeros)
// at every row whose sequence position t is 0.
template <int SKIP, bool FAST>
__device__ __forceinline__ void conv_column(const __half *__restrict__ xc, int r0, float w0, float w1, float w2,
                                            const float4 wv, float bj, uint8_t *box, const uint32_t (&off)[8], int t,
                                            int L) {
#pragma unroll
    for (int i = 0; i < 32; ++i) {
        const float x3 = __half2float(xc[(r0 + i) * (kPXPitch / 2)]);
        if (!FAST) {
            if (t == 0) w0 = w1 = w2 = 0.f;
            t = (t + 1 == L) ? 0 : t + 1;
        }
        float acc = fmaf(w0, wv.x, 0.f);
        acc = fmaf(w1, wv.y, acc);
        acc = fmaf(w2, wv.z, acc);
        acc = fmaf(x3, wv.w, acc);
        acc += bj;
        const int sr = (i - SKIP) & 31;
        *reinterpret_cast<__half *>(box + sr * 128 + off[sr & 7]) = __float2half_rn(silu_fast(acc));
        w0 = w1;
        w1 = w2;
        w2 = x3;
    }
}

template <bool CONV>
__global__ void __launch_bounds__(ProjCfg<CONV>::kThreads, 1)
    proj_gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                     const __grid_constant__ CUtensorMap map_c, const __grid_constant__ CUtensorMap map_c_short,
                     const __grid_constant__ CUtensorMap map_z, const __grid_constant__ CUtensorMap map_z_short,
                     const ProjParams p) {
    constexpr int kPStages = ProjCfg<CONV>::kStages;
    constexpr int kEpiWarps = ProjCfg<CONV>::kEpiWarps;
    constexpr int kEpiBytes = kEpiWarps * 2 * kPEpiBox;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *epi = smem + kPStages * kPStage;
    uint8_t *xch = epi + kEpiBytes;  // conv input tiles
    uint64_t *full = reinterpret_cast<uint64_t *>(epi + kEpiBytes + (CONV ? kPXchBytes : 0));
    uint64_t *empty = full + kPStages;
    uint64_t *tfull = empty + kPStages;
    uint64_t *tempty = tfull + 2;
    uint64_t *drain = tempty + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);

    const uint32_t rank = cluster_ctarank();  // 0: the pair's MMA issuer
    const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tiles = p.m_tiles * p.n_tiles;
    // Row geometry: a CTA computes 128 rows starting `halo` rows before its
    // first output row; a pair advances by 2 * (128 - halo) rows per tile.
    const int rstep = 128 - p.halo;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kPStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], 2 * kEpiWarps);  // every epilogue warp of both CTAs
        }
        mbar_init(drain, 1);
        fence_mbar_init();
        prefetch_tensormap(&map_a);
        prefetch_tensormap(&map_b);
        prefetch_tensormap(&map_c);
    }
    if (warp == 1) {
        tmem_alloc_pair(tmem_slot, kPTmemCols);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    cluster_sync();  // both CTAs' barriers initialised, TMEM allocated
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    bool ok = true;
    if (warp == 0) {
        if (lane == 0) {
            const uint32_t full0 = mapa_shared(smem_u32(&full[0]), 0);  // stage barriers of the even CTA
            const int half = p.BN >> 1;
            uint32_t it = 0;
            for (int tile = pair; tile < tiles && ok; tile += npairs) {
                const int mt = tile / p.n_tiles, nt = tile % p.n_tiles;
                // may be negative for the first tile (the halo): those rows read zeros
                const int arow = mt * 2 * rstep + (int)rank * rstep - p.halo;
                // gated: the even CTA loads the tile's 128 gate rows, the odd
                // one the matching 128 up rows, so accumulator columns 0..127
                // are gate and 128..255 up for the same 128 outputs
                const int brow = p.up_row0 ? (rank ? p.up_row0 : 0) + nt * half : nt * p.BN + (int)rank * half;
                for (int kb = 0; kb < p.kblocks; ++kb, ++it) {
                    const uint32_t s = it % kPStages, ph = (it / kPStages) & 1;
                    if (!mbar_wait_bounded(&empty[s], ph ^ 1)) {
                        ok = false;
                        break;
                    }
                    if (rank == 0) mbar_arrive_expect_tx(&full[s], p.tx_bytes);
                    uint8_t *a = smem + s * kPStage;
                    tma_load_2d_pair(a, &map_a, full0 + s * 8, kb * kPBK, arow);
                    tma_load_2d_pair(a + kPStageA, &map_b, full0 + s * 8, kb * kPBK, brow);
                }
            }
            // The even CTA sees every copy of both CTAs land before it exits.
            if (rank == 0) {
                const uint32_t first = it > (uint32_t)kPStages ? it - kPStages : 0;
                for (uint32_t j = first; j < it; ++j)
                    if (!mbar_wait_bounded_cluster(&full[j % kPStages], (j / kPStages) & 1)) ok = false;
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && rank == 0) {
            uint32_t it = 0, tcount = 0;
            for (int tile = pair; tile < tiles && ok; tile += npairs, ++tcount) {
                const uint32_t b = tcount & 1, tph = (tcount >> 1) & 1;
                if (!mbar_wait_bounded_cluster(&tempty[b], tph ^ 1)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem + b * kPAccCols;
                for (int kb = 0; kb < p.kblocks; ++kb, ++it) {
                    const uint32_t s = it % kPStages, ph = (it / kPStages) & 1;
                    if (!mbar_wait_bounded_cluster(&full[s], ph)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(smem + s * kPStage);
                    const uint32_t b_addr = a_addr + kPStageA;
#pragma unroll
                    for (int k = 0; k < kPBK / kPUK; ++k)
                        umma_f16_pair(d_tmem, smem_desc_sw128(a_addr + k * kPUK * 2),
                                      smem_desc_sw128(b_addr + k * kPUK * 2), p.idesc, (kb | k) != 0);
                    umma_commit_pair(&empty[s], 0x3);  // the stage is free in both CTAs once read
                }
                if (!ok) break;
                umma_commit_pair(&tfull[b], 0x3);  // accumulator b holds the finished tile
            }
            // Every issued MMA completes before TMEM may be freed.
            umma_commit_pair(drain, 0x1);
            if (!mbar_wait_bounded(drain, 0)) ok = false;
        }
    } else {
        // Epilogue: warp w reads TMEM lanes 32*(w%4) .. +31, i.e. rows
        // 32*(w%4) .. +31 of this CTA's 128.  In the first quarter the rows
        // before `halo` are not outputs: that warp stores a shorter box
        // (map *_short) from shared-memory row 0 = tile row `halo`.
        const int quarter = warp & 3;
        const int egroup = (warp - 2) >> 2;  // column-chunk group: chunks egroup, egroup + groups, ...
        constexpr int kGroups = kEpiWarps / 4;
        const int skip = quarter == 0 ? p.halo : 0;
        const int srow = lane - skip;  // this lane's row in the staged box (< 0: not stored)
        uint8_t *boxes = epi + (warp - 2) * 2 * kPEpiBox;  // this warp's two staging boxes
        const uint32_t tempty0 = mapa_shared(smem_u32(&tempty[0]), 0);
        const bool gated = !CONV && p.up_row0 != 0;
        const bool f16 = p.mode == kProjF16;
        const int cstep = f16 ? 64 : 32;
        const int ccols = gated ? p.BN / 2 : p.BN;  // output columns of a tile
        uint32_t tcount = 0, nbox = 0, nchunk = 0;
        for (int tile = pair; tile < tiles; tile += npairs, ++tcount) {
            const uint32_t b = tcount & 1, tph = (tcount >> 1) & 1;
            bool have = warp_wait_p(&tfull[b], tph);
            if (CONV) have = epilogue_all(have);
            if (!have) {
                ok = false;
                break;
            }
            tc_fence_after();
            const int mt = tile / p.n_tiles, nt = tile % p.n_tiles;
            const int wrow = mt * 2 * rstep + (int)rank * rstep - p.halo + quarter * 32;  // this warp's first row
            const int out_row = wrow + skip;                                                // first stored row
            const bool conv_tile = CONV && nt < p.x_tiles;
            const int ncol = CONV ? (conv_tile ? nt : nt - p.x_tiles) * p.BN : nt * ccols;
            const CUtensorMap *mfull = (CONV && !conv_tile) ? &map_z : &map_c;
            const CUtensorMap *mshort = (CONV && !conv_tile) ? &map_z_short : &map_c_short;
            const CUtensorMap *mstore = skip ? mshort : mfull;
            const int ncols = (CONV || gated) ? p.N / 2 : p.N;  // columns of the tensor being stored
            // sequence position of this warp's first row (the conv restarts
            // at t = 0; halo rows before the first token count as t < 0)
            int tpos0 = 0;
            if (conv_tile) tpos0 = ((wrow % p.L) + p.L) % p.L;
            // no sequence start among the rows this warp's windows read: for
            // the first quarter rows 1..31 (its rows 0..2 are not stored),
            // for the others rows -3..31
            const bool fast_rows = quarter == 0 ? (p.L >= 32 && tpos0 + 31 < p.L) : (tpos0 >= 3 && tpos0 + 31 < p.L);
            const uint32_t tl = tmem + ((uint32_t)(quarter * 32) << 16) + b * kPAccCols;
            for (int c = egroup * cstep; c < ccols; c += kGroups * cstep) {
                const int col = ncol + c;
                uint32_t v0[32];
                uint32_t pk[32];  // FP16 output: 64 columns as 32 packed pairs
                if (CONV && conv_tile) {
                    // Causal conv (width 4) + bias + SiLU, the arithmetic of the
                    // library's conv kernel (conv.cu), on two 32-column halves.
                    // Each warp writes its 32 rows of FP16-rounded x (the values
                    // the unfused path stores) into a shared tile; then lane l
                    // walks column l down the warp's rows with a 3-row window
                    // that starts in the previous warp's rows and restarts at
                    // every sequence start.  Taps oldest first, fma, then the
                    // bias, as conv.cu does.
                    uint8_t *box = boxes + (nbox & 1) * kPEpiBox;
                    if (lane == 0) bulk_wait_group_read<1>();
                    __syncwarp();
#pragma unroll 1
                    for (int hlf = 0; hlf < 2; ++hlf) {
                        tmem_ld_32x32b_x32(tl + c + 32 * hlf, v0);
                        tmem_wait_ld();
                        uint8_t *X = xch + (nchunk & 1) * (128 * kPXPitch);
                        uint8_t *xrow = X + (quarter * 32 + lane) * kPXPitch;
#pragma unroll
                        for (int j = 0; j < 16; ++j)
                            *reinterpret_cast<uint32_t *>(xrow + 4 * j) = pack_half2(v0[2 * j], v0[2 * j + 1]);
                        epilogue_bar();
                        const int cc = col + 32 * hlf + lane;  // this lane's channel
                        const float4 wv = __ldg(reinterpret_cast<const float4 *>(p.conv_w) + min(cc, ncols - 1));
                        const float bj = __ldg(p.conv_b + min(cc, ncols - 1));
                        const __half *xc = reinterpret_cast<const __half *>(X) + lane;  // column `lane`
                        uint32_t off[8];
#pragma unroll
                        for (int k = 0; k < 8; ++k) off[k] = ((((32 * hlf + lane) >> 3) ^ k) << 4) + ((lane & 7) << 1);
                        const int r0 = quarter * 32;
                        // window rows r0-3 .. r0-1, zero before the sequence start
                        float w0 = 0.f, w1 = 0.f, w2 = 0.f;
                        if (quarter > 0) {
                            if (tpos0 >= 3) w0 = __half2float(xc[(r0 - 3) * (kPXPitch / 2)]);
                            if (tpos0 >= 2) w1 = __half2float(xc[(r0 - 2) * (kPXPitch / 2)]);
                            if (tpos0 >= 1) w2 = __half2float(xc[(r0 - 1) * (kPXPitch / 2)]);
                        }
                        if (quarter == 0) {
                            if (fast_rows)
                                conv_column<3, true>(xc, r0, w0, w1, w2, wv, bj, box, off, tpos0, p.L);
                            else
                                conv_column<3, false>(xc, r0, w0, w1, w2, wv, bj, box, off, tpos0, p.L);
                        } else {
                            if (fast_rows)
                                conv_column<0, true>(xc, r0, w0, w1, w2, wv, bj, box, off, tpos0, p.L);
                            else
                                conv_column<0, false>(xc, r0, w0, w1, w2, wv, bj, box, off, tpos0, p.L);
                        }
                        ++nchunk;
                    }
                    if (col >= ncols || out_row >= p.M) continue;
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) {
                        tma_store_2d(mstore, box, col, out_row);
                        bulk_commit_group();
                    }
                    ++nbox;
                    continue;
                } else if (!CONV && gated) {
                    // silu(gate) * up, 32 outputs at a time (gate at column
                    // c, up at column 128 + c of the accumulator)
#pragma unroll
                    for (int hlf = 0; hlf < 2; ++hlf) {
                        uint32_t g[32];
                        tmem_ld_32x32b_x32(tl + c + 32 * hlf, g);
                        tmem_ld_32x32b_x32(tl + ccols + c + 32 * hlf, v0);
                        tmem_wait_ld();
#pragma unroll
                        for (int j = 0; j < 16; ++j)
                            pk[16 * hlf + j] = pack_half2f(silu_fast(__uint_as_float(g[2 * j])) * __uint_as_float(v0[2 * j]),
                                                           silu_fast(__uint_as_float(g[2 * j + 1])) *
                                                               __uint_as_float(v0[2 * j + 1]));
                    }
                } else {
                    uint32_t v1[32];
                    tmem_ld_32x32b_x32(tl + c, v0);
                    if (f16) tmem_ld_32x32b_x32(tl + c + 32, v1);
                    tmem_wait_ld();
                    if (f16) {
                        if (p.bias) {
#pragma unroll
                            for (int j = 0; j < 32; ++j) {
                                if (col + j < ncols)
                                    v0[j] = __float_as_uint(__uint_as_float(v0[j]) + p.bias[col + j]);
                                if (col + 32 + j < ncols)
                                    v1[j] = __float_as_uint(__uint_as_float(v1[j]) + p.bias[col + 32 + j]);
                            }
                        }
#pragma unroll
                        for (int j = 0; j < 16; ++j) {
                            pk[j] = pack_half2(v0[2 * j], v0[2 * j + 1]);
                            pk[16 + j] = pack_half2(v1[2 * j], v1[2 * j + 1]);
                        }
                    } else if (p.bias) {
#pragma unroll
                        for (int j = 0; j < 32; ++j)
                            if (col + j < ncols) v0[j] = __float_as_uint(__uint_as_float(v0[j]) + p.bias[col + j]);
                    }
                }
                if (col >= ncols || out_row >= p.M) continue;  // nothing of this box is inside C
                uint8_t *box = boxes + (nbox & 1) * kPEpiBox;
                // the bulk store that last read this box has finished reading it
                if (lane == 0) bulk_wait_group_read<1>();
                __syncwarp();
                if (srow >= 0) {
                    if (f16) {
#pragma unroll
                        for (int j = 0; j < 8; ++j)
                            st_swizzled(box, srow, j, make_uint4(pk[4 * j], pk[4 * j + 1], pk[4 * j + 2], pk[4 * j + 3]));
                    } else {
#pragma unroll
                        for (int j = 0; j < 8; ++j)
                            st_swizzled(box, srow, j, make_uint4(v0[4 * j], v0[4 * j + 1], v0[4 * j + 2], v0[4 * j + 3]));
                    }
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    if (p.mode == kProjF32Add)
                        tma_reduce_add_2d(mstore, box, col, out_row);
                    else
                        tma_store_2d(mstore, box, col, out_row);
                    bulk_commit_group();
                }
                ++nbox;
            }
            // accumulator b is read: hand it back to the even CTA's MMA thread
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                if (rank == 0)
                    mbar_arrive(&tempty[b]);
                else
                    mbar_arrive_cluster(tempty0 + b * 8);
            }
        }
        if (lane == 0) bulk_wait_group_all();
        __syncwarp();
    }
    if (!ok) atomicOr(&g_proj_error, kErrProjTimeout);
    tc_fence_before();
    cluster_sync();  // nothing of either CTA touches TMEM or the peer's shared memory after this
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem, kPTmemCols);
    }
}

// 2-D map over a row-major [rows, cols] matrix (row stride ld elements) with
// box [box_rows, box_cols] and the 128-byte swizzle; loads outside the
// matrix read zeros, stores outside it are dropped.
bool encode_2d(CUtensorMap *m, CUtensorMapDataType t, int esize, const void *ptr, int64_t rows, int64_t cols,
               int64_t ld, int box_cols, int box_rows) {
    auto enc = tensor_map_encoder();
    if (!enc) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)(ld * esize)};
    const cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return enc(m, t, 2, const_cast<void *>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
               CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Per-device launch facts: the shared-memory opt-in and how many CTA pairs
// of this kernel fit on the GPU at once (clusters must sit inside one GPC).
struct DevInfo {
    bool ready = false;
    int pairs = 0;
};

template <bool CONV>
int device_info(DevInfo &out) {
    static std::mutex mu;
    static std::vector<DevInfo> cache;
    int dev = 0;
    MB_CUDA_TRY(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> lk(mu);
    if ((int)cache.size() <= dev) cache.resize(dev + 1);
    DevInfo &d = cache[dev];
    if (!d.ready) {
        MB_CUDA_TRY(cudaFuncSetAttribute(proj_gemm_kernel<CONV>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         proj_smem_bytes<CONV>()));
        cudaLaunchConfig_t cfg{};
        cudaLaunchAttribute attr{};
        attr.id = cudaLaunchAttributeClusterDimension;
        attr.val.clusterDim.x = 2;
        attr.val.clusterDim.y = 1;
        attr.val.clusterDim.z = 1;
        cfg.gridDim = dim3(2 * 148, 1, 1);
        cfg.blockDim = dim3(ProjCfg<CONV>::kThreads, 1, 1);
        cfg.dynamicSmemBytes = proj_smem_bytes<CONV>();
        cfg.attrs = &attr;
        cfg.numAttrs = 1;
        int n = 0;
        MB_CUDA_TRY(cudaOccupancyMaxActiveClusters(&n, proj_gemm_kernel<CONV>, &cfg));
        MB_CHECK_ARG(n > 0, "proj_gemm: no CTA pair fits on this GPU");
        d.pairs = n;
        d.ready = true;
    }
    out = d;
    return 0;
}

int check_tc_device(const char *what) {
    int dev = 0, major = 0;
    MB_CUDA_TRY(cudaGetDevice(&dev));
    MB_CUDA_TRY(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev));
    MB_CHECK_ARG(major == 10, std::string(what) + ": needs a compute capability 10.x GPU (tcgen05)");
    return 0;
}

template <bool CONV>
int launch_proj(const CUtensorMap *maps, const ProjParams &p, cudaStream_t st) {
    DevInfo info;
    if (device_info<CONV>(info)) return -1;
    const int64_t tiles = (int64_t)p.m_tiles * p.n_tiles;
    MB_CHECK_ARG(tiles <= 0x7fffffff, "proj_gemm: too many tiles");
    const int pairs = (int)std::min<int64_t>(tiles, info.pairs);
    cudaLaunchConfig_t cfg{};
    cudaLaunchAttribute attr{};
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = 2;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.gridDim = dim3(2 * pairs, 1, 1);
    cfg.blockDim = dim3(ProjCfg<CONV>::kThreads, 1, 1);
    cfg.dynamicSmemBytes = proj_smem_bytes<CONV>();
    cfg.stream = st;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    MB_CUDA_TRY(cudaLaunchKernelEx(&cfg, proj_gemm_kernel<CONV>, maps[0], maps[1], maps[2], maps[3], maps[4],
                                   maps[5], p));
    return launch_status("projection GEMM (tcgen05, CTA pairs) kernel");
}

}  // namespace

int proj_gemm(const void *A, int64_t lda, const void *W, const float *bias, void *C, int64_t ldc, int64_t M, int N,
              int K, int mode, cudaStream_t st) {
    MB_CHECK_ARG(M >= 0 && N > 0 && K > 0, "proj_gemm: bad sizes");
    if (M == 0) return 0;
    MB_CHECK_ARG(A && W && C, "proj_gemm: null pointer");
    MB_CHECK_ARG(mode == kProjF16 || mode == kProjF32Add || mode == kProjF32, "proj_gemm: bad epilogue mode");
    MB_CHECK_ARG(K % 8 == 0 && lda % 8 == 0 && lda >= K, "proj_gemm: K and lda must be multiples of 8, lda >= K");
    const int cs = mode == kProjF16 ? 2 : 4;
    MB_CHECK_ARG(ldc >= N && (ldc * cs) % 16 == 0, "proj_gemm: ldc must be >= N with 16-byte aligned rows");
    MB_CHECK_ARG(reinterpret_cast<uintptr_t>(A) % 16 == 0 && reinterpret_cast<uintptr_t>(W) % 16 == 0 &&
                     reinterpret_cast<uintptr_t>(C) % 16 == 0,
                 "proj_gemm: pointers must be 16-byte aligned");
    MB_CHECK_ARG(M <= (int64_t)0x7fffffff - 256, "proj_gemm: too many rows");
    if (check_tc_device("proj_gemm")) return -1;

    ProjParams p{};
    p.bias = bias;
    p.M = (int)M;
    p.N = N;
    p.K = K;
    p.BN = N <= 256 ? (N + 15) / 16 * 16 : 256;
    p.m_tiles = (int)((M + 255) / 256);
    p.n_tiles = (N + p.BN - 1) / p.BN;
    p.kblocks = (K + kPBK - 1) / kPBK;
    p.mode = mode;
    p.halo = 0;
    p.idesc = idesc_f16_f32acc(256, p.BN);
    p.tx_bytes = (uint32_t)(2 * (kPStageA + (p.BN / 2) * kPBK * 2));

    CUtensorMap maps[6];
    const bool enc_ok =
        encode_2d(&maps[0], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, A, M, K, lda, kPBK, 128) &&
        encode_2d(&maps[1], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, W, N, K, K, kPBK, p.BN / 2) &&
        (mode == kProjF16 ? encode_2d(&maps[2], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, C, M, N, ldc, 64, 32)
                          : encode_2d(&maps[2], CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, C, M, N, ldc, 32, 32));
    MB_CHECK_ARG(enc_ok, "proj_gemm: tensor map encoding failed");
    maps[3] = maps[4] = maps[5] = maps[2];  // no halo, no second output
    return launch_proj<false>(maps, p, st);
}

int proj_gemm_gated(const void *x, const void *w, void *out, int64_t T, int d, int h, cudaStream_t st) {
    MB_CHECK_ARG(T >= 0 && d > 0 && h > 0, "gated_mlp_up: bad sizes");
    if (T == 0) return 0;
    MB_CHECK_ARG(x && w && out, "gated_mlp_up: null pointer");
    MB_CHECK_ARG(d % 8 == 0 && h % 8 == 0, "gated_mlp_up: d and h must be multiples of 8");
    MB_CHECK_ARG(reinterpret_cast<uintptr_t>(x) % 16 == 0 && reinterpret_cast<uintptr_t>(w) % 16 == 0 &&
                     reinterpret_cast<uintptr_t>(out) % 16 == 0,
                 "gated_mlp_up: pointers must be 16-byte aligned");
    MB_CHECK_ARG(T <= (int64_t)0x7fffffff - 256 && h <= 0x3fffffff - 256, "gated_mlp_up: too large");
    if (check_tc_device("gated_mlp_up")) return -1;
    ProjParams p{};
    p.M = (int)T;
    p.N = 2 * h;
    p.K = d;
    p.BN = 256;  // 128 gate + 128 up columns -> 128 outputs
    p.m_tiles = (int)((T + 255) / 256);
    p.n_tiles = (h + 127) / 128;
    p.kblocks = (d + kPBK - 1) / kPBK;
    p.mode = kProjF16;
    p.halo = 0;
    p.up_row0 = h;
    p.idesc = idesc_f16_f32acc(256, 256);
    p.tx_bytes = (uint32_t)(2 * (kPStageA + kPStageB));
    CUtensorMap maps[6];
    const auto F16 = CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    // The last gate box of an h that is not a multiple of 128 reads up rows:
    // those columns are beyond h and never stored.
    const bool enc_ok = encode_2d(&maps[0], F16, 2, x, T, d, d, kPBK, 128) &&
                        encode_2d(&maps[1], F16, 2, w, 2 * (int64_t)h, d, d, kPBK, 128) &&
                        encode_2d(&maps[2], F16, 2, out, T, h, h, 64, 32);
    MB_CHECK_ARG(enc_ok, "gated_mlp_up: tensor map encoding failed");
    maps[3] = maps[4] = maps[5] = maps[2];
    return launch_proj<false>(maps, p, st);
}

bool proj_conv_supported(int64_t T, int L, int D, int Mdim, int K) {
    return K == 4 && D % 256 == 0 && Mdim % 8 == 0 && L > 0 && T > 0 && T % L == 0 && T <= 0x7fff0000LL;
}

int proj_gemm_conv(const void *A, const void *W, const float *conv_w, const float *conv_b, void *u, void *z,
                   int64_t ldz, int64_t T, int L, int D, int Mdim, int K, cudaStream_t st) {
    MB_CHECK_ARG(T >= 0, "proj_gemm_conv: bad sizes");
    if (T == 0) return 0;
    MB_CHECK_ARG(A && W && conv_w && conv_b && u && z, "proj_gemm_conv: null pointer");
    MB_CHECK_ARG(proj_conv_supported(T, L, D, Mdim, K),
                 "proj_gemm_conv: needs d_conv 4, d_inner a multiple of 256, d_model a multiple of 8");
    MB_CHECK_ARG(ldz >= D && ldz % 8 == 0, "proj_gemm_conv: z row stride");
    MB_CHECK_ARG(reinterpret_cast<uintptr_t>(A) % 16 == 0 && reinterpret_cast<uintptr_t>(W) % 16 == 0 &&
                     reinterpret_cast<uintptr_t>(u) % 16 == 0 && reinterpret_cast<uintptr_t>(z) % 16 == 0 &&
                     reinterpret_cast<uintptr_t>(conv_w) % 16 == 0,
                 "proj_gemm_conv: pointers must be 16-byte aligned");
    if (check_tc_device("proj_gemm_conv")) return -1;
    const int halo = K - 1;
    ProjParams p{};
    p.conv_w = conv_w;
    p.conv_b = conv_b;
    p.M = (int)T;
    p.N = 2 * D;
    p.K = Mdim;
    p.BN = 256;
    p.m_tiles = (int)((T + 2 * (128 - halo) - 1) / (2 * (128 - halo)));
    p.n_tiles = 2 * D / p.BN;
    p.kblocks = (Mdim + kPBK - 1) / kPBK;
    p.mode = kProjF16;
    p.halo = halo;
    p.L = L;
    p.x_tiles = D / p.BN;
    p.idesc = idesc_f16_f32acc(256, p.BN);
    p.tx_bytes = (uint32_t)(2 * (kPStageA + (p.BN / 2) * kPBK * 2));
    CUtensorMap maps[6];
    const auto F16 = CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    const bool enc_ok = encode_2d(&maps[0], F16, 2, A, T, Mdim, Mdim, kPBK, 128) &&
                        encode_2d(&maps[1], F16, 2, W, 2 * (int64_t)D, Mdim, Mdim, kPBK, p.BN / 2) &&
                        encode_2d(&maps[2], F16, 2, u, T, D, D, 64, 32) &&
                        encode_2d(&maps[3], F16, 2, u, T, D, D, 64, 32 - halo) &&
                        encode_2d(&maps[4], F16, 2, z, T, D, ldz, 64, 32) &&
                        encode_2d(&maps[5], F16, 2, z, T, D, ldz, 64, 32 - halo);
    MB_CHECK_ARG(enc_ok, "proj_gemm_conv: tensor map encoding failed");
    return launch_proj<true>(maps, p, st);
}

unsigned proj_error_flags(bool clear) {
    unsigned v = 0;
    if (cudaMemcpyFromSymbol(&v, g_proj_error, sizeof(v)) != cudaSuccess) return ~0u;
    if (clear && v) {
        const unsigned z = 0;
        cudaMemcpyToSymbol(g_proj_error, &z, sizeof(z));
    }
    return v;
}

}  // namespace mb
