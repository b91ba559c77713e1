// gated_mlp.cu -- the SwiGLU up-projection of a gated MLP as one tensor-core
// kernel: out = silu(x @ W_gate^T) * (x @ W_up^T).
//
// The reference computes the two projections with its linear kernel and
// then applies gated_silu_mul (Sources/Kernels/gated_mlp.metal:12-41).  Here
// both projections run in one tcgen05 MMA stream and the gate is applied in
// the epilogue, straight out of tensor memory: the [tokens, 2h] FP32/FP16
// pre-activations never reach HBM.
//
// Layout: x FP16 [tokens, d] row-major; w FP16 [2h, d] (rows 0..h-1 are
// W_gate, rows h..2h-1 are W_up: the nn.Linear layout, K-major); out FP16
// [tokens, h].  FP32 accumulation.
//
// Kernel structure (persistent, one CTA per SM, 192 threads):
//   warp 0, one lane   TMA producer: per 64-wide K block, a [128 x 64] tile
//                      of x and the [128 x 64] tiles of W_gate and W_up rows
//                      of the output column block, into a 4-stage ring.
//   warp 1             owns TMEM (512 columns = two accumulators of
//                      128 lanes x 256 columns); one lane issues the MMAs:
//                      M 128, N 256 (gate columns 0..127, up columns
//                      128..255), K 16, four per K block.
//   warps 2-5          epilogue: each thread owns one output row (its TMEM
//                      lane), reads gate and up columns 32 at a time, writes
//                      silu(g) * u as FP16.  The second accumulator lets the
//                      epilogue of one tile overlap the MMAs of the next.
// Every wait is bounded; on timeout a role stops, the error flag is set, and
// the CTA still waits (bounded) for its copies and MMAs in flight and frees
// its TMEM before returning.
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdlib>
#include <mutex>
#include <vector>

#include "common.cuh"
#include "internal.h"
#include "scan_math.cuh"
#include "tma.cuh"
#include "umma.cuh"

namespace mb {

__device__ unsigned int g_gemm_error = 0;

namespace {

constexpr int kBM = 128;                   // output rows per tile (TMEM lanes)
constexpr int kBN = 128;                   // output columns per tile
constexpr int kBK = 64;                    // K per stage: one 128-byte swizzle row
constexpr int kUK = 16;                    // K per MMA instruction
constexpr int kStages = 4;
constexpr int kUmmaN = 2 * kBN;            // gate and up in one MMA
constexpr int kABytes = kBM * kBK * 2;     // 16 KB
constexpr int kBHalfBytes = kBN * kBK * 2; // 16 KB
constexpr int kStageBytes = kABytes + 2 * kBHalfBytes;
constexpr int kTmemCols = 2 * kUmmaN;      // 512: the whole TMEM of the SM
constexpr int kThreads = 192;
constexpr int kEpiThreads = 128;
constexpr int kSmemBytes = kStages * kStageBytes + 1024 /* alignment */ + 256 /* barriers */;
constexpr unsigned kErrGemmTimeout = 2u;

static_assert(kBM == 128 && kUmmaN % 16 == 0 && kUmmaN <= 256, "MMA shape");

__device__ __forceinline__ float bits_f32(uint32_t v) { return __uint_as_float(v); }

__device__ __forceinline__ bool warp_wait(uint64_t *bar, uint32_t parity) {
    // One lane polls; the verdict is shared so the warp stays converged for
    // the warp-collective TMEM loads that follow.
    int ok = 0;
    if ((threadIdx.x & 31) == 0) ok = mbar_wait_bounded(bar, parity) ? 1 : 0;
    return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

__global__ void __launch_bounds__(kThreads, 1)
    gated_mlp_up_kernel(const __grid_constant__ CUtensorMap map_x, const __grid_constant__ CUtensorMap map_w,
                        __half *__restrict__ out, int64_t T, int H, int K, int m_blocks, int n_blocks) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + kStages * kStageBytes);
    uint64_t *empty = full + kStages;
    uint64_t *tfull = empty + kStages;
    uint64_t *tempty = tfull + 2;
    uint64_t *drain = tempty + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int num_tiles = m_blocks * n_blocks;
    const int kblocks = (K + kBK - 1) / kBK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], kEpiThreads);
        }
        mbar_init(drain, 1);
        fence_mbar_init();
        prefetch_tensormap(&map_x);
        prefetch_tensormap(&map_w);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    bool ok = true;
    if (warp == 0) {
        if (lane == 0) {
            uint32_t it = 0;
            for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
                const int mb_ = tile / n_blocks, nb = tile % n_blocks;
                for (int kb = 0; kb < kblocks; ++kb, ++it) {
                    const uint32_t s = it % kStages, ph = (it / kStages) & 1;
                    if (!mbar_wait_bounded(&empty[s], ph ^ 1)) {
                        ok = false;
                        break;
                    }
                    uint8_t *a = smem + s * kStageBytes;
                    uint8_t *b = a + kABytes;
                    mbar_arrive_expect_tx(&full[s], kStageBytes);
                    tma_load_2d(a, &map_x, &full[s], kb * kBK, mb_ * kBM);
                    tma_load_2d(b, &map_w, &full[s], kb * kBK, nb * kBN);
                    tma_load_2d(b + kBHalfBytes, &map_w, &full[s], kb * kBK, H + nb * kBN);
                }
            }
            // Every issued copy lands before the CTA may exit.
            const uint32_t first = it > (uint32_t)kStages ? it - kStages : 0;
            for (uint32_t j = first; j < it; ++j)
                if (!mbar_wait_bounded(&full[j % kStages], (j / kStages) & 1)) ok = false;
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t idesc = idesc_f16_f32acc(kBM, kUmmaN);
            uint32_t it = 0, tcount = 0;
            for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++tcount) {
                const uint32_t b = tcount & 1, tph = (tcount >> 1) & 1;
                if (!mbar_wait_bounded(&tempty[b], tph ^ 1)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem + b * kUmmaN;
                for (int kb = 0; kb < kblocks; ++kb, ++it) {
                    const uint32_t s = it % kStages, ph = (it / kStages) & 1;
                    if (!mbar_wait_bounded(&full[s], ph)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(smem + s * kStageBytes);
                    const uint32_t b_addr = a_addr + kABytes;
#pragma unroll
                    for (int k = 0; k < kBK / kUK; ++k)
                        umma_f16(d_tmem, smem_desc_sw128(a_addr + k * kUK * 2), smem_desc_sw128(b_addr + k * kUK * 2),
                                 idesc, (kb | k) != 0);
                    umma_commit(&empty[s]);  // the stage is free once these MMAs have read it
                }
                if (!ok) break;
                umma_commit(&tfull[b]);  // accumulator b holds the finished tile
            }
            // Every issued MMA completes before TMEM may be freed.
            umma_commit(drain);
            if (!mbar_wait_bounded(drain, 0)) ok = false;
        }
    } else {
        // Epilogue: warp w may access TMEM lanes 32*(w%4) .. 32*(w%4)+31.
        const int quarter = warp & 3;
        const int r = quarter * 32 + lane;
        uint32_t tcount = 0;
        for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++tcount) {
            const uint32_t b = tcount & 1, tph = (tcount >> 1) & 1;
            if (!warp_wait(&tfull[b], tph)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const int mb_ = tile / n_blocks, nb = tile % n_blocks;
            const int64_t row = (int64_t)mb_ * kBM + r;
            const uint32_t tl = tmem + ((uint32_t)(quarter * 32) << 16) + b * kUmmaN;
            __half *orow = out + row * H;
#pragma unroll 1
            for (int c = 0; c < kBN; c += 32) {
                uint32_t g[32], u[32];
                tmem_ld_32x32b_x32(tl + c, g);
                tmem_ld_32x32b_x32(tl + kBN + c, u);
                tmem_wait_ld();
                const int col0 = nb * kBN + c;
                if (row < T) {
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        if (col0 + 8 * q >= H) break;
                        uint4 v;
                        __half2 *hv = reinterpret_cast<__half2 *>(&v);
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            const int e = 8 * q + 2 * j;
                            hv[j] = __floats2half2_rn(silu_fast(bits_f32(g[e])) * bits_f32(u[e]),
                                                      silu_fast(bits_f32(g[e + 1])) * bits_f32(u[e + 1]));
                        }
                        *reinterpret_cast<uint4 *>(orow + col0 + 8 * q) = v;
                    }
                }
            }
            tc_fence_before();
            mbar_arrive(&tempty[b]);
        }
    }
    if (!ok) atomicOr(&g_gemm_error, kErrGemmTimeout);
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

// 2-D map over a row-major FP16 [rows, cols] matrix, box [128 rows, 64 cols],
// 128-byte swizzle, zero fill outside the matrix.
bool encode_kmajor(CUtensorMap *m, const void *ptr, int64_t rows, int cols) {
    auto enc = tensor_map_encoder();
    if (!enc) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
    const cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)kBM};
    const cuuint32_t estr[2] = {1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(ptr), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

int gated_mlp_up(const void *x, const void *w, void *out, int64_t T, int d, int h, cudaStream_t st) {
    MB_CHECK_ARG(T >= 0 && d > 0 && h > 0, "gated_mlp_up: bad sizes");
    if (T == 0) return 0;
    // The CTA-pair projection GEMM with a SwiGLU epilogue (gemm_tc.cu) is the
    // default; MAMBA_MLP_PAIR=0 selects this file's one-CTA kernel.
    static const bool pair = [] {
        const char *e = std::getenv("MAMBA_MLP_PAIR");
        return !e || std::atoi(e) != 0;
    }();
    if (pair) return proj_gemm_gated(x, w, out, T, d, h, st);
    MB_CHECK_ARG(x && w && out, "gated_mlp_up: null pointer");
    MB_CHECK_ARG(d % 8 == 0 && h % 8 == 0, "gated_mlp_up: d and h must be multiples of 8");
    MB_CHECK_ARG(reinterpret_cast<uintptr_t>(x) % 16 == 0 && reinterpret_cast<uintptr_t>(w) % 16 == 0 &&
                     reinterpret_cast<uintptr_t>(out) % 16 == 0,
                 "gated_mlp_up: pointers must be 16-byte aligned");
    MB_CHECK_ARG(T <= (int64_t)0x7fffffff - kBM && (int64_t)2 * h <= 0x7fffffff - kBN,
                 "gated_mlp_up: too large");
    int dev = 0;
    MB_CUDA_TRY(cudaGetDevice(&dev));
    int major = 0;
    MB_CUDA_TRY(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev));
    MB_CHECK_ARG(major == 10, "gated_mlp_up: needs a compute capability 10.x GPU (tcgen05)");
    CUtensorMap mx, mw;
    MB_CHECK_ARG(encode_kmajor(&mx, x, T, d) && encode_kmajor(&mw, w, 2 * (int64_t)h, d),
                 "gated_mlp_up: tensor map encoding failed");
    {
        // the shared-memory opt-in is per device
        static std::mutex mu;
        static std::vector<char> done;
        std::lock_guard<std::mutex> lk(mu);
        if ((int)done.size() <= dev) done.resize(dev + 1, 0);
        if (!done[dev]) {
            MB_CUDA_TRY(
                cudaFuncSetAttribute(gated_mlp_up_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes));
            done[dev] = 1;
        }
    }
    const int m_blocks = (int)((T + kBM - 1) / kBM), n_blocks = (h + kBN - 1) / kBN;
    const int64_t tiles = (int64_t)m_blocks * n_blocks;
    MB_CHECK_ARG(tiles <= 0x7fffffff, "gated_mlp_up: too many tiles");
    const int grid = (int)std::min<int64_t>(tiles, device_sm_count());
    gated_mlp_up_kernel<<<grid, kThreads, kSmemBytes, st>>>(mx, mw, static_cast<__half *>(out), T, h, d, m_blocks,
                                                            n_blocks);
    return launch_status("gated_mlp_up kernel");
}

unsigned gemm_error_flags(bool clear) {
    unsigned v = 0;
    if (cudaMemcpyFromSymbol(&v, g_gemm_error, sizeof(v)) != cudaSuccess) return ~0u;
    if (clear && v) {
        const unsigned z = 0;
        cudaMemcpyToSymbol(g_gemm_error, &z, sizeof(z));
    }
    return v;
}

}  // namespace mb
