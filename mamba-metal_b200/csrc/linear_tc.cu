// linear_tc.cu -- y = x @ W^T (+ bias) on the tensor cores (tcgen05), the job
// of linear_f32/_f16 (Sources/Kernels/projection.metal:13-49) for FP16
// operands, with FP32 accumulation and three epilogues:
//   mode 0  y (FP16)  = acc + bias
//   mode 1  y (FP32) += acc + bias     (the FP32 residual stream: beta = 1)
//   mode 2  y (FP32)  = acc + bias
// x FP16 [M, K] with row stride ldx elements; W FP16 [N, K] (K-major: the
// reference's [K, N] weight transposed once at load); y row stride ldy.
//
// Built for the decode-sized projections (M = the decode batch, a few
// hundred rows), where a library GEMM's large tiles leave most SMs idle:
// one CTA computes a [256 x BN] block of y (two 128-lane TMEM accumulators)
// over a range of K; the K range is split so that the grid covers the SMs.
// Splits write FP32 partials to a workspace and a second, fully parallel
// kernel sums them in split order and applies the epilogue, so results do
// not depend on the order in which CTAs run.
//
// Roles (192 threads): warp 0 lane 0 issues the TMA loads (x tile
// [rows x 64], W tile [BN x 64], 128-byte swizzle, 4-stage ring); warp 1
// owns TMEM and one lane issues tcgen05.mma (M 128, N BN, K 16; one or two
// per 16-wide K step); warps 2-5 run the epilogue out of TMEM.  Every wait
// is bounded (2 s); on timeout the CTA stops, records bit 2 of the device
// status, drains its copies and MMAs and frees its TMEM.
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>
#include <vector>

#include "common.cuh"
#include "internal.h"
#include "tma.cuh"
#include "umma.cuh"

namespace mb {

__device__ unsigned int g_linear_error = 0;

namespace {

constexpr int kLBK = 64;          // K per stage (one 128-byte swizzle row)
constexpr int kLUK = 16;          // K per MMA
constexpr int kLStages = 4;
constexpr int kLThreads = 192;
constexpr unsigned kErrLinearTimeout = 4u;

struct LinearParams {
    void *y;
    int64_t ldy;
    float *ws;        // [splits][M][N] FP32 partials (splits > 1)
    const float *bias;
    int M, N, K;
    int a_rows;       // rows per x tile: 128 (M <= 128) or 256
    int m_tiles, n_tiles, splits, kb_per_split, kblocks;
    int mode;
};

template <int BN>
constexpr int stage_bytes() {
    return 256 * kLBK * 2 + BN * kLBK * 2;
}
template <int BN>
constexpr int smem_bytes() {
    return kLStages * stage_bytes<BN>() + 1024 + 256;
}

__device__ __forceinline__ bool warp_wait_l(uint64_t *bar, uint32_t parity) {
    int ok = 0;
    if ((threadIdx.x & 31) == 0) ok = mbar_wait_bounded(bar, parity) ? 1 : 0;
    return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

// Final epilogue for 8 consecutive columns of one row.
__device__ __forceinline__ void finish8(const LinearParams &p, int64_t row, int col, float *v) {
    if (p.bias) {
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] += p.bias[col + j];
    }
    if (p.mode == 0) {
        uint4 o;
        __half2 *h = reinterpret_cast<__half2 *>(&o);
#pragma unroll
        for (int j = 0; j < 4; ++j) h[j] = __floats2half2_rn(v[2 * j], v[2 * j + 1]);
        *reinterpret_cast<uint4 *>(static_cast<__half *>(p.y) + row * p.ldy + col) = o;
    } else {
        float4 *dst = reinterpret_cast<float4 *>(static_cast<float *>(p.y) + row * p.ldy + col);
        float4 a = make_float4(v[0], v[1], v[2], v[3]), b = make_float4(v[4], v[5], v[6], v[7]);
        if (p.mode == 1) {
            const float4 r0 = dst[0], r1 = dst[1];
            a = make_float4(r0.x + a.x, r0.y + a.y, r0.z + a.z, r0.w + a.w);
            b = make_float4(r1.x + b.x, r1.y + b.y, r1.z + b.z, r1.w + b.w);
        }
        dst[0] = a;
        dst[1] = b;
    }
}

template <int BN>
__global__ void __launch_bounds__(kLThreads, 1)
    linear_tc_kernel(const __grid_constant__ CUtensorMap map_x, const __grid_constant__ CUtensorMap map_w,
                     const LinearParams p) {
    constexpr int kStage = stage_bytes<BN>();
    constexpr int kA = 256 * kLBK * 2;  // x region of a stage (fits 256 rows)
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + kLStages * kStage);
    uint64_t *empty = full + kLStages;
    uint64_t *accb = empty + kLStages;
    uint64_t *drain = accb + 1;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int u = blockIdx.x;
    const int split = u % p.splits, tile = u / p.splits;
    const int nt = tile % p.n_tiles, mt = tile / p.n_tiles;
    const int kb0 = split * p.kb_per_split;
    const int kb1 = min(p.kblocks, kb0 + p.kb_per_split);
    const int nkb = kb1 - kb0;
    // CTAs start their K walk at different blocks, so that the x tile of one
    // K block is not requested by every SM at once (one L2 slice would
    // serve them all).
    const int rot = nkb > 1 ? (int)(((unsigned)u * 7u) % (unsigned)nkb) : 0;
    const int row0 = mt * p.a_rows;
    const int mh = (p.M - row0 > 128 && p.a_rows == 256) ? 2 : 1;  // 128-row halves with rows
    const uint32_t tx_bytes = (uint32_t)(p.a_rows * kLBK * 2 + BN * kLBK * 2);

    if (threadIdx.x == 0) {
        for (int s = 0; s < kLStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(accb, 1);
        mbar_init(drain, 1);
        fence_mbar_init();
        prefetch_tensormap(&map_x);
        prefetch_tensormap(&map_w);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, 2 * BN);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    bool ok = true;
    if (warp == 0) {
        if (lane == 0) {
            int i = 0;
            for (; i < nkb; ++i) {
                const uint32_t s = i % kLStages, ph = (i / kLStages) & 1;
                if (!mbar_wait_bounded(&empty[s], ph ^ 1)) {
                    ok = false;
                    break;
                }
                uint8_t *a = smem + s * kStage;
                mbar_arrive_expect_tx(&full[s], tx_bytes);
                const int kb = kb0 + (i + rot) % nkb;
                tma_load_2d(a, &map_x, &full[s], kb * kLBK, row0);
                tma_load_2d(a + kA, &map_w, &full[s], kb * kLBK, nt * BN);
            }
            for (int j = i > kLStages ? i - kLStages : 0; j < i; ++j)
                if (!mbar_wait_bounded(&full[j % kLStages], (j / kLStages) & 1)) ok = false;
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t idesc = idesc_f16_f32acc(128, BN);
            for (int i = 0; i < nkb; ++i) {
                const uint32_t s = i % kLStages, ph = (i / kLStages) & 1;
                if (!mbar_wait_bounded(&full[s], ph)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t a_addr = smem_u32(smem + s * kStage);
                const uint32_t b_addr = a_addr + kA;
#pragma unroll
                for (int k = 0; k < kLBK / kLUK; ++k) {
                    const uint64_t bdesc = smem_desc_sw128(b_addr + k * kLUK * 2);
                    for (int h = 0; h < mh; ++h)
                        umma_f16(tmem + h * BN, smem_desc_sw128(a_addr + h * 128 * 128 + k * kLUK * 2), bdesc, idesc,
                                 (i | k) != 0);
                }
                umma_commit(&empty[s]);
            }
            umma_commit(accb);  // also reached on the error path: completes when issued MMAs do
            umma_commit(drain);
            if (!mbar_wait_bounded(drain, 0)) ok = false;
        }
    } else {
        const int quarter = warp & 3;
        const int r = quarter * 32 + lane;
        const bool have = warp_wait_l(accb, 0);
        if (!have) ok = false;
        tc_fence_after();
        const int ncol0 = nt * BN;
        // partial or final values straight out of TMEM
        if (have) {
            for (int h = 0; h < mh; ++h) {
                const int64_t row = (int64_t)row0 + h * 128 + r;
                const uint32_t tl = tmem + ((uint32_t)(quarter * 32) << 16) + h * BN;
#pragma unroll 1
                for (int c = 0; c < BN; c += 32) {
                    uint32_t v[32];
                    tmem_ld_32x32b_x32(tl + c, v);
                    tmem_wait_ld();
                    if (row >= p.M) continue;
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const int col = ncol0 + c + 8 * q;
                        if (col >= p.N) break;
                        float f[8];
#pragma unroll
                        for (int j = 0; j < 8; ++j) f[j] = __uint_as_float(v[8 * q + j]);
                        if (p.splits == 1) {
                            finish8(p, row, col, f);
                        } else {
                            float4 *dst = reinterpret_cast<float4 *>(
                                p.ws + ((int64_t)split * p.M + row) * p.N + col);
                            dst[0] = make_float4(f[0], f[1], f[2], f[3]);
                            dst[1] = make_float4(f[4], f[5], f[6], f[7]);
                        }
                    }
                }
            }
        }
    }
    if (!ok) atomicOr(&g_linear_error, kErrLinearTimeout);
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 2 * BN);
    }
}

// Sum of the K-split partials in split order, then the epilogue; one thread
// per 8 consecutive outputs (coalesced 32-byte partial reads).
__global__ void __launch_bounds__(256) linear_reduce_kernel(const LinearParams p) {
    const int64_t g = (int64_t)blockIdx.x * 256 + threadIdx.x;
    const int groups = p.N / 8;
    if (g >= (int64_t)p.M * groups) return;
    const int64_t row = g / groups;
    const int col = (int)(g % groups) * 8;
    float f[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    const int64_t split_stride = (int64_t)p.M * p.N;
    const float *base = p.ws + row * p.N + col;
    // Loads of 4 splits are issued before their sums, so the walk over the
    // splits is not one L2 round trip per split; the sum order stays 0, 1, ...
    for (int s0 = 0; s0 < p.splits; s0 += 4) {
        float4 a[4], b[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            if (s0 + j < p.splits) {
                const float4 *src = reinterpret_cast<const float4 *>(base + (s0 + j) * split_stride);
                a[j] = src[0];
                b[j] = src[1];
            }
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            if (s0 + j < p.splits) {
                f[0] += a[j].x;
                f[1] += a[j].y;
                f[2] += a[j].z;
                f[3] += a[j].w;
                f[4] += b[j].x;
                f[5] += b[j].y;
                f[6] += b[j].z;
                f[7] += b[j].w;
            }
        }
    }
    finish8(p, row, col, f);
}

bool encode_rows(CUtensorMap *m, const void *ptr, int64_t rows, int cols, int64_t ld, int box_rows) {
    auto enc = tensor_map_encoder();
    if (!enc) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
    const cuuint32_t box[2] = {(cuuint32_t)kLBK, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(ptr), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

struct Plan {
    int bn, a_rows, m_tiles, n_tiles, splits, kb_per_split, kblocks;
};

Plan make_plan(int64_t M, int N, int K, int sms) {
    Plan pl{};
    pl.a_rows = M <= 128 ? 128 : 256;
    pl.m_tiles = (int)((M + pl.a_rows - 1) / pl.a_rows);
    pl.kblocks = (K + kLBK - 1) / kLBK;
    // 128-column blocks re-read the x tile half as often as 64-column ones;
    // narrower blocks only when K is too short to split.
    pl.bn = N > 64 ? 128 : 64;
    pl.n_tiles = (N + pl.bn - 1) / pl.bn;
    if (pl.bn == 128 && (int64_t)pl.m_tiles * pl.n_tiles < sms && pl.kblocks < 8) {
        pl.bn = 64;
        pl.n_tiles = (N + 63) / 64;
    }
    const int64_t tiles = (int64_t)pl.m_tiles * pl.n_tiles;
    int splits = 1;
    if (tiles < sms) {
        // as many splits as keep the grid within one CTA per SM (the
        // kernel holds a whole SM's shared memory), at least 2 K blocks each
        const int64_t fit = sms / tiles;
        const int cap = std::max(1, std::min(32, pl.kblocks / 2));
        splits = (int)std::max<int64_t>(1, std::min<int64_t>(fit, cap));
    }
    pl.kb_per_split = (pl.kblocks + splits - 1) / splits;
    pl.splits = (pl.kblocks + pl.kb_per_split - 1) / pl.kb_per_split;
    return pl;
}

template <int BN>
int launch_bn(const CUtensorMap &mx, const CUtensorMap &mw, const LinearParams &p, int grid, cudaStream_t st) {
    static std::mutex mu;
    static std::vector<char> done;
    int dev = 0;
    MB_CUDA_TRY(cudaGetDevice(&dev));
    {
        std::lock_guard<std::mutex> lk(mu);
        if ((int)done.size() <= dev) done.resize(dev + 1, 0);
        if (!done[dev]) {
            MB_CUDA_TRY(cudaFuncSetAttribute(linear_tc_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             smem_bytes<BN>()));
            done[dev] = 1;
        }
    }
    linear_tc_kernel<BN><<<grid, kLThreads, smem_bytes<BN>(), st>>>(mx, mw, p);
    if (launch_status("linear (tcgen05) kernel")) return -1;
    if (p.splits > 1) {
        const int64_t work = (int64_t)p.M * (p.N / 8);
        linear_reduce_kernel<<<(unsigned)((work + 255) / 256), 256, 0, st>>>(p);
        return launch_status("linear split-K reduction kernel");
    }
    return 0;
}

}  // namespace

size_t linear_workspace_bytes(int64_t M, int N, int K) {
    if (M <= 0 || N <= 0 || K <= 0 || M > kProjMinRows) return 0;
    const Plan pl = make_plan(M, N, K, device_sm_count());
    if (pl.splits <= 1) return 0;
    return (size_t)pl.splits * (size_t)M * (size_t)N * sizeof(float);
}

int linear_tc(const void *x, int64_t ldx, const void *w, const float *bias, void *y, int64_t ldy, int64_t M, int N,
              int K, int mode, void *ws, size_t ws_bytes, cudaStream_t st) {
    MB_CHECK_ARG(M >= 0 && N > 0 && K > 0, "linear: bad sizes");
    if (M == 0) return 0;
    MB_CHECK_ARG(x && w && y, "linear: null pointer");
    MB_CHECK_ARG(mode >= 0 && mode <= 2, "linear: bad mode");
    MB_CHECK_ARG(K % 8 == 0 && N % 8 == 0, "linear: K and N must be multiples of 8");
    MB_CHECK_ARG(ldy >= N && ldy % 8 == 0, "linear: ldy must be >= N and a multiple of 8");
    MB_CHECK_ARG(ldx >= K && ldx % 8 == 0, "linear: ldx must be >= K and a multiple of 8");
    MB_CHECK_ARG(reinterpret_cast<uintptr_t>(x) % 16 == 0 && reinterpret_cast<uintptr_t>(w) % 16 == 0 &&
                     reinterpret_cast<uintptr_t>(y) % 16 == 0,
                 "linear: pointers must be 16-byte aligned");
    MB_CHECK_ARG(M <= (int64_t)0x7fffffff - 256, "linear: too many rows");
    // Many rows: the CTA-pair GEMM (gemm_tc.cu) without K splits.
    if (M > kProjMinRows) return proj_gemm(x, ldx, w, bias, y, ldy, M, N, K, mode, st);
    int dev = 0, major = 0;
    MB_CUDA_TRY(cudaGetDevice(&dev));
    MB_CUDA_TRY(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev));
    MB_CHECK_ARG(major == 10, "linear: needs a compute capability 10.x GPU (tcgen05)");
    const Plan pl = make_plan(M, N, K, device_sm_count());
    const int64_t units = (int64_t)pl.m_tiles * pl.n_tiles * pl.splits;
    MB_CHECK_ARG(units <= 0x7fffffff, "linear: too many tiles");
    LinearParams p{};
    p.y = y;
    p.ldy = ldy;
    p.bias = bias;
    p.M = (int)M;
    p.N = N;
    p.K = K;
    p.a_rows = pl.a_rows;
    p.m_tiles = pl.m_tiles;
    p.n_tiles = pl.n_tiles;
    p.splits = pl.splits;
    p.kb_per_split = pl.kb_per_split;
    p.kblocks = pl.kblocks;
    p.mode = mode;
    if (pl.splits > 1) {
        const size_t need = linear_workspace_bytes(M, N, K);
        MB_CHECK_ARG(ws && ws_bytes >= need, "linear: workspace too small (see mamba_linear_workspace)");
        MB_CHECK_ARG(reinterpret_cast<uintptr_t>(ws) % 16 == 0, "linear: workspace must be 16-byte aligned");
        p.ws = static_cast<float *>(ws);
    }
    CUtensorMap mx, mw;
    MB_CHECK_ARG(encode_rows(&mx, x, M, K, ldx, pl.a_rows) && encode_rows(&mw, w, N, K, K, pl.bn),
                 "linear: tensor map encoding failed");
    if (pl.bn == 128) return launch_bn<128>(mx, mw, p, (int)units, st);
    return launch_bn<64>(mx, mw, p, (int)units, st);
}

unsigned linear_error_flags(bool clear) {
    unsigned v = 0;
    if (cudaMemcpyFromSymbol(&v, g_linear_error, sizeof(v)) != cudaSuccess) return ~0u;
    if (clear && v) {
        const unsigned z = 0;
        cudaMemcpyToSymbol(g_linear_error, &z, sizeof(z));
    }
    return v;
}

}  // namespace mb
