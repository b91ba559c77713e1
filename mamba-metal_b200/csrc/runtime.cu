// runtime.cu -- the model runtime behind the C API.
//
// Replaces mamba::MambaRuntime (Sources/Mamba/MambaRuntime.hpp:27-64,
// MambaRuntime.cpp:18-119) and its Metal device/buffer/pipeline layer
// (Sources/Runtime/*) with a thin CUDA layer: one device, one stream and one
// cuBLAS handle per model; weights resident in HBM in one allocation; an
// activation arena sized for the largest batch*seq_len seen.
//
// Layer graph (the sequence written at MambaRuntime.cpp:93-101), tokens
// row-major [T = batch*seq_len, features]:
//   normed = RMSNorm(h)                            [T, d_model]   act
//   xz     = normed @ in_proj                      [T, 2*d_inner] act
//   u      = SiLU(causal_conv1d(xz[:, :d_inner]))  [T, d_inner]   act
//   xdbc   = u @ x_proj                            [T, R + 2N]    act
//   draw   = xdbc[:, :R] @ dt_proj                 [T, d_inner]   act
//   y      = scan(u, draw + dt_bias, B, C, z = xz[:, d_inner:])  act
//   h     += y @ out_proj                          [T, d_model]   FP32
// The residual stream h stays FP32; activations use cfg.dtype.
#include <cublas_v2.h>

#include <nvtx3/nvToolsExt.h>

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "common.cuh"
#include "internal.h"

namespace mb {

// ---- errors ---------------------------------------------------------------
namespace {
thread_local std::string g_last_error;
}
int log_level() {
    static const int level = [] {
        const char *e = std::getenv("MAMBA_LOG");
        return e ? std::max(0, std::atoi(e)) : 0;
    }();
    return level;
}
void log_msg(int level, const char *fmt, ...) {
    if (log_level() < level) return;
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    std::vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    std::fprintf(stderr, "mamba-b200: %s\n", buf);
}
void set_error(const std::string &msg) {
    g_last_error = msg;
    log_msg(1, "error: %s", msg.c_str());
}
const char *last_error() { return g_last_error.c_str(); }
void clear_error() { g_last_error.clear(); }

int device_sm_count() {
    static std::mutex mu;
    static std::vector<int> cache;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    std::lock_guard<std::mutex> lk(mu);
    if ((int)cache.size() <= dev) cache.resize(dev + 1, 0);
    if (cache[dev] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        cache[dev] = n;
    }
    return cache[dev];
}

namespace {

constexpr float kNormEps = 1e-5f;
constexpr size_t kAlign = 256;
constexpr size_t kCublasWs = 32u << 20;

size_t align_up(size_t v) { return (v + kAlign - 1) / kAlign * kAlign; }

// Sets a device for the scope and restores the caller's device after.
struct DeviceGuard {
    int prev = -1;
    bool ok = false;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        ok = (prev == dev) || cudaSetDevice(dev) == cudaSuccess;
    }
    ~DeviceGuard() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

// Move-only device allocation (replaces MetalBuffer, Sources/Runtime/MetalBuffer.hpp:7-28;
// no unified memory: the host reaches it through explicit copies).
struct DeviceBuffer {
    void *ptr = nullptr;
    size_t bytes = 0;
    DeviceBuffer() = default;
    DeviceBuffer(const DeviceBuffer &) = delete;
    DeviceBuffer &operator=(const DeviceBuffer &) = delete;
    ~DeviceBuffer() { release(); }
    void release() {
        if (ptr) cudaFree(ptr);
        ptr = nullptr;
        bytes = 0;
    }
    int reserve(size_t n) {
        if (n <= bytes) return 0;
        release();
        if (cudaMalloc(&ptr, n) != cudaSuccess) {
            cudaGetLastError();
            ptr = nullptr;
            set_error("cudaMalloc of " + std::to_string(n) + " bytes failed");
            return -1;
        }
        bytes = n;
        return 0;
    }
};

struct LayerWeights {
    void *w_in_t = nullptr;   // [2D, M]    act  (in_proj^T)
    void *w_x_t = nullptr;    // [R+2N, D]  act  (x_proj^T)
    void *w_dt_t = nullptr;   // [D, R]     act  (dt_proj^T)
    void *w_out_t = nullptr;  // [M, D]     act  (out_proj^T)
    float *conv_w = nullptr;  // [D, K]
    float *conv_b = nullptr;  // [D]
    float *A = nullptr;       // [D, N]
    float *A_inv = nullptr;   // [D, N] 1/A (0 where |A| <= 1e-6), derived at load
    float *Dskip = nullptr;   // [D]
    float *norm_w = nullptr;  // [M]
    float *dt_bias = nullptr; // [D]
};

// Per-operation CUDA-event timing (mamba_profile_*).  Events come from a
// pool that is reused after every mamba_profile_enable.
struct Profiler {
    bool on = false;
    // MAMBA_DEBUG=1: every operation's stream is synchronised and checked
    // (CUDA error, device status flags) right after it; the first failure
    // names the operation and layer and makes the call return -1.
    bool debug = false;
    bool debug_failed = false;
    int layer = -1;
    std::vector<cudaEvent_t> pool;
    size_t used = 0;
    struct Rec {
        int op;
        cudaEvent_t a, b;
        int kernels;
    };
    std::vector<Rec> recs;
    ~Profiler() {
        for (cudaEvent_t e : pool) cudaEventDestroy(e);
    }
    cudaEvent_t take() {
        if (used == pool.size()) {
            cudaEvent_t e = nullptr;
            if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
            pool.push_back(e);
        }
        return pool[used++];
    }
    void reset() {
        used = 0;
        recs.clear();
    }
};

const char *op_name(int op) {
    static const char *names[MAMBA_OP_COUNT] = {"rmsnorm", "in_proj", "conv", "x_proj",
                                                "dt_proj", "scan",    "out_proj"};
    return op >= 0 && op < MAMBA_OP_COUNT ? names[op] : "op";
}

// Brackets one operation: an NVTX range named after it, an event pair while
// profiling is on, and the MAMBA_DEBUG check after it.
struct OpScope {
    Profiler &p;
    int op;
    cudaStream_t st;
    int kernels;  // this library's kernels in the operation (may be set after construction)
    cudaEvent_t a = nullptr;
    OpScope(Profiler &p_, int op_, cudaStream_t s, int k) : p(p_), op(op_), st(s), kernels(k) {
        nvtxRangePushA(op_name(op));
        if (p.on && (a = p.take())) cudaEventRecord(a, st);
    }
    ~OpScope() {
        nvtxRangePop();
        if (p.debug && !p.debug_failed) debug_check();
        if (!p.on || !a) return;
        cudaEvent_t b = p.take();
        if (b && cudaEventRecord(b, st) == cudaSuccess) p.recs.push_back({op, a, b, kernels});
    }
    void debug_check() {
        cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
        if (cudaStreamIsCapturing(st, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) return;
        const cudaError_t e1 = cudaStreamSynchronize(st);
        const cudaError_t e2 = cudaGetLastError();
        const unsigned flags = mamba_device_status(0);
        if (e1 == cudaSuccess && e2 == cudaSuccess && flags == 0) return;
        p.debug_failed = true;
        char buf[256];
        std::snprintf(buf, sizeof(buf), "MAMBA_DEBUG: operation %s of layer %d failed: %s (device status 0x%x)",
                      op_name(op), p.layer, cudaGetErrorString(e1 != cudaSuccess ? e1 : e2), flags);
        set_error(buf);
    }
};

// NVTX range over one layer; also tells the debug check which layer runs.
struct LayerScope {
    Profiler &p;
    LayerScope(Profiler &p_, int l) : p(p_) {
        p.layer = l;
        char name[32];
        std::snprintf(name, sizeof(name), "mamba layer %d", l);
        nvtxRangePushA(name);
    }
    ~LayerScope() {
        nvtxRangePop();
        p.layer = -1;
    }
};

// One decode step of every layer captured as a CUDA graph, replayed while
// the state buffers, token/output pointers, arena and stream stay the same.
struct StepGraph {
    const float *conv = nullptr, *ssm = nullptr;
    int batch = -1;
    const float *in = nullptr;
    float *out = nullptr;
    cudaStream_t st = nullptr;
    const void *arena = nullptr;
    cudaGraphExec_t exec = nullptr;
    void reset() {
        if (exec) cudaGraphExecDestroy(exec);
        exec = nullptr;
        batch = -1;
    }
    ~StepGraph() { reset(); }
};

}  // namespace

struct Model {
    MambaConfig cfg{};
    int M = 0, D = 0, N = 0, K = 0, R = 0, XD = 0;
    int act = MAMBA_F16;
    int dev = 0;
    cudaStream_t stream = nullptr;
    cublasHandle_t cublas = nullptr;
    DeviceBuffer cublas_ws;
    DeviceBuffer weights;
    std::vector<LayerWeights> layers;
    // forward arena
    DeviceBuffer arena;
    int64_t arena_tokens = 0;
    DeviceBuffer io;  // host-API staging for forward/step
    // step arena
    DeviceBuffer step_arena;
    int64_t step_rows = 0;
    // caller-provided stream (mamba_set_stream) and tracing
    cudaStream_t user_stream = nullptr;
    Profiler prof;
    // decode graph (MAMBA_STEP_GRAPH=0 disables)
    StepGraph step_graph;
    bool use_graphs = true;

    cudaStream_t cur_stream() const { return user_stream ? user_stream : stream; }

    ~Model() {
        if (stream) cudaStreamSynchronize(stream);
        if (h2d) cudaStreamSynchronize(h2d);
        if (d2h) cudaStreamSynchronize(d2h);
        step_graph.reset();
        if (cublas) cublasDestroy(cublas);
        for (cudaEvent_t e : io_events) cudaEventDestroy(e);
        if (h2d) cudaStreamDestroy(h2d);
        if (d2h) cudaStreamDestroy(d2h);
        if (stream) cudaStreamDestroy(stream);
    }

    size_t act_size() const { return dtype_size(act); }

    size_t layer_bytes() const {
        const size_t a = act_size();
        size_t s = 0;
        s += align_up((size_t)2 * D * M * a);
        s += align_up((size_t)XD * D * a);
        s += align_up((size_t)D * R * a);
        s += align_up((size_t)M * D * a);
        s += align_up((size_t)D * K * 4);
        s += align_up((size_t)D * 4);
        s += align_up((size_t)D * N * 4);
        s += align_up((size_t)D * N * 4);  // A_inv
        s += align_up((size_t)D * 4);
        s += align_up((size_t)M * 4);
        s += align_up((size_t)D * 4);
        return s;
    }

    int init(const MambaConfig &c) {
        cfg = c;
        M = c.d_model;
        D = c.expand * c.d_model;
        N = c.d_state;
        K = c.d_conv;
        R = (c.d_model + 15) / 16;
        XD = R + 2 * N;
        act = c.dtype;
        MB_CUDA_TRY(cudaGetDevice(&dev));
        cudaDeviceProp prop;
        MB_CUDA_TRY(cudaGetDeviceProperties(&prop, dev));
        MB_CHECK_ARG(prop.major == 10, std::string("mamba_create: device '") + prop.name +
                                           "' is not sm_100 (compute capability 10.x required)");
        MB_CUDA_TRY(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));
        if (const char *g = std::getenv("MAMBA_STEP_GRAPH")) use_graphs = std::atoi(g) != 0;
        if (const char *t = std::getenv("MAMBA_TC_LINEAR")) tc_linear = std::atoi(t) != 0;
        if (const char *h = std::getenv("MAMBA_HOST_CHUNKS")) host_chunks = std::max(0, std::atoi(h));
        if (const char *pj = std::getenv("MAMBA_PROJ")) proj_tc = std::atoi(pj) != 0;
        if (const char *cf = std::getenv("MAMBA_CONV_FUSE")) conv_fuse = std::atoi(cf) != 0;
        if (const char *df = std::getenv("MAMBA_DT_FUSE")) dt_fuse = std::atoi(df) != 0;
        if (const char *dbg = std::getenv("MAMBA_DEBUG")) prof.debug = std::atoi(dbg) != 0;
        log_msg(2, "model on device %d (%s, %d SMs): d_model %d, d_inner %d, d_state %d, d_conv %d, dt_rank %d, "
                   "%d layers, %s activations; projections on %s; debug checks %s",
                dev, prop.name, prop.multiProcessorCount, M, D, N, K, R, c.n_layer, act == MAMBA_F16 ? "FP16" : "FP32",
                proj_tc && act == MAMBA_F16 ? "the CTA-pair tcgen05 GEMM (> 512 rows)" : "cuBLAS",
                prof.debug ? "on" : "off");
        if (cublasCreate(&cublas) != CUBLAS_STATUS_SUCCESS) {
            set_error("cublasCreate failed");
            return -1;
        }
        if (cublas_ws.reserve(kCublasWs)) return -1;
        if (cublasSetWorkspace(cublas, cublas_ws.ptr, kCublasWs) != CUBLAS_STATUS_SUCCESS) {
            set_error("cublasSetWorkspace failed");
            return -1;
        }
        const size_t lb = layer_bytes();
        if (weights.reserve(lb * c.n_layer)) return -1;
        MB_CUDA_TRY(cudaMemsetAsync(weights.ptr, 0, lb * c.n_layer, stream));
        layers.resize(c.n_layer);
        const size_t a = act_size();
        for (int l = 0; l < c.n_layer; ++l) {
            char *p = static_cast<char *>(weights.ptr) + lb * l;
            auto take = [&](size_t bytes) {
                char *q = p;
                p += align_up(bytes);
                return q;
            };
            LayerWeights &w = layers[l];
            w.w_in_t = take((size_t)2 * D * M * a);
            w.w_x_t = take((size_t)XD * D * a);
            w.w_dt_t = take((size_t)D * R * a);
            w.w_out_t = take((size_t)M * D * a);
            w.conv_w = reinterpret_cast<float *>(take((size_t)D * K * 4));
            w.conv_b = reinterpret_cast<float *>(take((size_t)D * 4));
            w.A = reinterpret_cast<float *>(take((size_t)D * N * 4));
            w.A_inv = reinterpret_cast<float *>(take((size_t)D * N * 4));
            w.Dskip = reinterpret_cast<float *>(take((size_t)D * 4));
            w.norm_w = reinterpret_cast<float *>(take((size_t)M * 4));
            w.dt_bias = reinterpret_cast<float *>(take((size_t)D * 4));
        }
        MB_CUDA_TRY(cudaStreamSynchronize(stream));
        return 0;
    }

    // C[rows, n] (ldc) = A[rows, k] (lda) @ W where W is stored as Wt [n, k];
    // beta = 1 accumulates into C (used for the residual).  C may be FP32
    // while A/W are FP16 (FP32 accumulation in every case).
    // The projections run on cuBLAS.  MAMBA_TC_LINEAR=1 sends few-row FP16
    // projections (decode batches, short forwards) to this library's
    // tcgen05 linear kernel instead; at the decode shapes (256 rows) it is
    // measured 2-3x slower than cuBLAS (its K splits cannot balance the
    // output blocks over 148 SMs), so it is off by default.
    static constexpr int64_t kTcRows = kProjMinRows;
    bool tc_linear = false;  // read from MAMBA_TC_LINEAR when the model is created
    bool tc_linear_enabled() const { return tc_linear; }
    bool use_tc(int64_t rows, int n, int k, int lda, int ldc) const {
        return act == MAMBA_F16 && rows <= kTcRows && tc_linear_enabled() && n % 8 == 0 && k % 8 == 0 &&
               lda % 8 == 0 && ldc % 8 == 0;
    }
    // Workspace for the split-K partials of every projection of one layer.
    size_t linear_ws_need(int64_t rows) const {
        size_t w = 0;
        const int shapes[4][4] = {{2 * D, M, M, 2 * D}, {XD, D, D, XD}, {D, R, XD, D}, {M, D, D, M}};
        for (const auto &sh : shapes)
            if (use_tc(rows, sh[0], sh[1], sh[2], sh[3])) w = std::max(w, linear_workspace_bytes(rows, sh[0], sh[1]));
        return w;
    }

    // FP16 projections of more than kTcRows rows (forward passes) run on this
    // library's CTA-pair tcgen05 GEMM (gemm_tc.cu); MAMBA_PROJ=0 sends them
    // to cuBLAS instead (for comparisons).
    bool proj_tc = true;
    int last_gemm_kernels = 0;  // this library's kernels launched by the last gemm()
    // in_proj and the causal conv as one kernel (mamba_in_proj_conv) when
    // MAMBA_CONV_FUSE=1.  Off by default: at the 48-layer workload the fused
    // kernel takes 8.9 ms per layer against 6.0 + 1.3 ms for the GEMM and the
    // separate conv, because the conv in the epilogue (one warp per SM
    // sub-partition, ~21 instructions per element) outlasts the MMAs of the
    // next tile.
    bool conv_fuse = false;
    bool fuse_conv(int64_t T, int L) const {
        return conv_fuse && proj_tc && act == MAMBA_F16 && T > kTcRows && proj_conv_supported(T, L, D, M, K);
    }

    // dt_proj folded into the scan (selective_scan_dtproj) when
    // MAMBA_DT_FUSE=1, wherever that kernel applies: FP16, 16 states,
    // dt_rank a multiple of 8 up to 128, x_proj rows 16-byte aligned, one
    // 128-channel CTA per SM or more.  Off by default: at the 48-layer
    // workload the fused scan takes 9.3 ms per layer against 7.4 + 0.66 ms
    // for the scan and the separate GEMM (the per-tile MMA issue and TMEM
    // read sit on the path of warps that each carry 32 channels).
    bool dt_fuse = false;
    bool fuse_dt(const MambaScanArgs &sa) const {
        return dt_fuse && act == MAMBA_F16 && (XD * 2) % 16 == 0 && scan_dtproj_supported(&sa, R);
    }

    bool use_proj(int64_t rows, int k, int lda, int ldc, int c_dtype) const {
        return proj_tc && act == MAMBA_F16 && rows > kTcRows && k % 8 == 0 && lda % 8 == 0 &&
               (ldc * (c_dtype == MAMBA_F16 ? 2 : 4)) % 16 == 0;
    }

    int gemm(cudaStream_t st, int64_t rows, int n, int k, const void *A, int lda, const void *Wt,
             void *C, int ldc, int c_dtype, float beta, void *lws, size_t lws_bytes) {
        last_gemm_kernels = 0;
        if (rows == 0 || n == 0) return 0;
        MB_CHECK_ARG(rows <= 0x7fffffffLL, "gemm: too many rows");
        const bool aligned = reinterpret_cast<uintptr_t>(A) % 16 == 0 && reinterpret_cast<uintptr_t>(Wt) % 16 == 0 &&
                             reinterpret_cast<uintptr_t>(C) % 16 == 0;
        const bool beta_ok = beta == 0.f || (beta == 1.f && c_dtype == MAMBA_F32);
        if (aligned && beta_ok && use_proj(rows, k, lda, ldc, c_dtype)) {
            const int mode = c_dtype == MAMBA_F16 ? kProjF16 : (beta == 1.f ? kProjF32Add : kProjF32);
            last_gemm_kernels = 1;
            return proj_gemm(A, lda, Wt, nullptr, C, ldc, rows, n, k, mode, st);
        }
        if (aligned && use_tc(rows, n, k, lda, ldc) && beta_ok) {
            const int mode = c_dtype == MAMBA_F16 ? 0 : (beta == 1.f ? 1 : 2);
            last_gemm_kernels = linear_workspace_bytes(rows, n, k) ? 2 : 1;
            return linear_tc(A, lda, Wt, nullptr, C, ldc, rows, n, k, mode, lws, lws_bytes, st);
        }
        const cudaDataType at = act == MAMBA_F16 ? CUDA_R_16F : CUDA_R_32F;
        const cudaDataType ct = c_dtype == MAMBA_F16 ? CUDA_R_16F : CUDA_R_32F;
        const float alpha = 1.f;
        if (cublasSetStream(cublas, st) != CUBLAS_STATUS_SUCCESS) {
            set_error("cublasSetStream failed");
            return -1;
        }
        const cublasStatus_t s =
            cublasGemmEx(cublas, CUBLAS_OP_T, CUBLAS_OP_N, n, (int)rows, k, &alpha, Wt, at, k, A, at,
                         lda, &beta, C, ct, ldc, CUBLAS_COMPUTE_32F, CUBLAS_GEMM_DEFAULT);
        if (s != CUBLAS_STATUS_SUCCESS) {
            set_error("cublasGemmEx failed with status " + std::to_string((int)s));
            return -1;
        }
        return 0;
    }

    struct Arena {
        void *normed, *xz, *u, *xdbc, *draw, *y, *scan_ws, *lin_ws;
        size_t scan_ws_bytes, lin_ws_bytes;
    };

    MambaScanArgs scan_args(const LayerWeights &w, const Arena &ar, int batch, int L) const {
        MambaScanArgs s{};
        const size_t a = act_size();
        s.x = ar.u;
        s.delta = ar.draw;
        s.B = static_cast<const char *>(ar.xdbc) + (size_t)R * a;
        s.C = static_cast<const char *>(ar.xdbc) + (size_t)(R + N) * a;
        s.A = w.A;
        s.D = w.Dskip;
        s.y = ar.y;
        s.final_state = nullptr;
        s.z = static_cast<const char *>(ar.xz) + (size_t)D * a;
        s.dt_bias = w.dt_bias;
        s.initial_state = nullptr;
        s.batch = batch;
        s.seqlen = L;
        s.dim = D;
        s.dstate = N;
        s.x_dtype = act;
        s.delta_dtype = act;
        s.bc_dtype = act;
        s.chunk_len = 0;
        const int64_t Ld = L;
        const int64_t xs[3] = {Ld * D, D, 1};
        const int64_t bcs[3] = {Ld * XD, XD, 1};
        const int64_t zs[3] = {Ld * 2 * D, 2 * D, 1};
        for (int i = 0; i < 3; ++i) {
            s.x_stride[i] = xs[i];
            s.delta_stride[i] = xs[i];
            s.y_stride[i] = xs[i];
            s.B_stride[i] = bcs[i];
            s.C_stride[i] = bcs[i];
            s.z_stride[i] = zs[i];
        }
        return s;
    }

    int ensure_arena(int batch, int L, Arena &ar) {
        const int64_t T = (int64_t)batch * L;
        const size_t a = act_size();
        Arena probe{};
        MambaScanArgs sa = scan_args(layers.empty() ? LayerWeights{} : layers[0], probe, batch, L);
        const size_t ws = scan_workspace_bytes(&sa);
        const size_t lws = linear_ws_need(T);
        size_t need = align_up(T * M * a) + align_up(T * 2 * D * a) + align_up(T * D * a) +
                      align_up(T * XD * a) + align_up(T * D * a) + align_up(T * D * a) + align_up(ws) +
                      align_up(lws);
        if (need > arena.bytes) {
            // Work queued on either stream may still read the old arena.
            MB_CUDA_TRY(cudaStreamSynchronize(stream));
            MB_CUDA_TRY(cudaStreamSynchronize(cur_stream()));
            if (arena.reserve(need)) return -1;
        }
        char *p = static_cast<char *>(arena.ptr);
        auto take = [&](size_t bytes) {
            char *q = p;
            p += align_up(bytes);
            return (void *)q;
        };
        ar.normed = take(T * M * a);
        ar.xz = take(T * 2 * D * a);
        ar.u = take(T * D * a);
        ar.xdbc = take(T * XD * a);
        ar.draw = take(T * D * a);
        ar.y = take(T * D * a);
        ar.scan_ws = ws ? take(ws) : nullptr;
        ar.scan_ws_bytes = ws;
        ar.lin_ws = lws ? take(lws) : nullptr;
        ar.lin_ws_bytes = lws;
        return 0;
    }

    int forward_device(const float *in, float *out, int batch, int L, cudaStream_t st) {
        MB_CHECK_ARG(batch >= 0 && L >= 0, "forward: negative batch or seq_len");
        const int64_t T = (int64_t)batch * L;
        if (T == 0) return 0;
        MB_CHECK_ARG(in && out, "forward: null pointer");
        if (!st) st = cur_stream();
        if (in != out) MB_CUDA_TRY(cudaMemcpyAsync(out, in, sizeof(float) * T * M, cudaMemcpyDeviceToDevice, st));
        return forward_layers(out, batch, L, 0, (int)layers.size(), st);
    }

    // Layers [l0, l1) on the FP32 residual stream out [batch, L, M], in place.
    // Every op is independent across batch rows, so a row range run alone
    // gives the same bits as inside the whole batch (as long as both take the
    // same kernels: more than 512 rows per GEMM).
    int forward_layers(float *out, int batch, int L, int l0, int l1, cudaStream_t st) {
        const int64_t T = (int64_t)batch * L;
        Arena ar{};
        if (ensure_arena(batch, L, ar)) return -1;
        const int64_t Ld = L;
        const int64_t xs[3] = {Ld * 2 * D, 2 * D, 1};
        const int64_t us[3] = {Ld * D, D, 1};
        prof.debug_failed = false;
        for (int li = l0; li < l1; ++li) {
            if (prof.debug_failed) return -1;
            LayerScope layer_scope(prof, li);
            const LayerWeights &w = layers[li];
            {
                OpScope o(prof, MAMBA_OP_RMSNORM, st, 1);
                if (rmsnorm(out, w.norm_w, ar.normed, T, M, kNormEps, MAMBA_F32, act, st)) return -1;
            }
            if (fuse_conv(T, L)) {
                // in_proj with the causal conv + SiLU in its epilogue: writes
                // u and the z half of xz; the x half is never stored.
                OpScope o(prof, MAMBA_OP_IN_PROJ, st, 1);
                if (proj_gemm_conv(ar.normed, w.w_in_t, w.conv_w, w.conv_b, ar.u,
                                   static_cast<char *>(ar.xz) + (size_t)D * act_size(), 2 * D, T, L, D, M, K, st))
                    return -1;
            } else {
                {
                    OpScope o(prof, MAMBA_OP_IN_PROJ, st, 0);
                    if (gemm(st, T, 2 * D, M, ar.normed, M, w.w_in_t, ar.xz, 2 * D, act, 0.f, ar.lin_ws,
                             ar.lin_ws_bytes))
                        return -1;
                    o.kernels = last_gemm_kernels;
                }
                {
                    OpScope o(prof, MAMBA_OP_CONV, st, 1);
                    if (causal_conv1d(ar.xz, xs, w.conv_w, w.conv_b, ar.u, us, batch, L, D, K, 1, act, st))
                        return -1;
                }
            }
            {
                OpScope o(prof, MAMBA_OP_X_PROJ, st, 0);
                if (gemm(st, T, XD, D, ar.u, D, w.w_x_t, ar.xdbc, XD, act, 0.f, ar.lin_ws, ar.lin_ws_bytes))
                    return -1;
                o.kernels = last_gemm_kernels;
            }
            MambaScanArgs sa = scan_args(w, ar, batch, L);
            const bool fdt = fuse_dt(sa);
            if (!fdt) {
                OpScope o(prof, MAMBA_OP_DT_PROJ, st, 0);
                if (gemm(st, T, D, R, ar.xdbc, XD, w.w_dt_t, ar.draw, D, act, 0.f, ar.lin_ws, ar.lin_ws_bytes))
                    return -1;
                o.kernels = last_gemm_kernels;
            }
            if (fdt) {
                // dt_proj inside the scan (tcgen05 from TMEM-resident W_dt)
                OpScope o(prof, MAMBA_OP_SCAN, st, 1);
                const int64_t dr_stride[2] = {(int64_t)L * XD, XD};
                if (selective_scan_dtproj(&sa, ar.xdbc, dr_stride, w.w_dt_t, R, st)) return -1;
            } else {
                OpScope o(prof, MAMBA_OP_SCAN, st, ar.scan_ws_bytes ? 3 : 1);
                if (selective_scan(&sa, ar.scan_ws, ar.scan_ws_bytes, st)) return -1;
            }
            {
                OpScope o(prof, MAMBA_OP_OUT_PROJ, st, 0);
                if (gemm(st, T, M, D, ar.y, D, w.w_out_t, out, M, MAMBA_F32, 1.f, ar.lin_ws, ar.lin_ws_bytes))
                    return -1;
                o.kernels = last_gemm_kernels;
            }
        }
        return prof.debug_failed ? -1 : 0;
    }

    // Host-buffer forward.  Large inputs are cut into row chunks uploaded and
    // downloaded on copy streams while other rows compute, so the PCIe
    // transfers hide behind the layers (overlap needs pinned host memory;
    // pageable buffers are staged by the driver).  With at least
    // 2 * kEdgeLayers layers the row chunks (batch/8 rows each) only drive
    // the edge layers: the first kEdgeLayers layers run per chunk as its
    // upload lands, the layers between run once on the whole batch, and the
    // last kEdgeLayers run per chunk, each chunk's download issued as soon as
    // it is done.  Only the first chunk's upload and the last chunk's
    // download are exposed, and only the edge layers run at the chunk's
    // smaller batch (whose scan fills fewer SMs).  Shallower stacks (and
    // forced chunk counts, MAMBA_HOST_CHUNKS) run whole-stack forwards over
    // the chunks: [c, batch - 2c, c] rows, c ~ batch/8.
    static constexpr size_t kChunkedHostBytes = 64u << 20;
    static constexpr int kEdgeLayers = 2;
    int host_chunks = 0;  // MAMBA_HOST_CHUNKS: forced chunk count (0 = automatic)
    cudaStream_t h2d = nullptr, d2h = nullptr;
    std::vector<cudaEvent_t> io_events;

    int forward_host(const float *in, float *out, int batch, int L) {
        MB_CHECK_ARG(batch >= 0 && L >= 0, "forward: negative batch or seq_len");
        const int64_t T = (int64_t)batch * L;
        if (T == 0) return 0;
        MB_CHECK_ARG(in && out, "forward: null pointer");
        const size_t bytes = sizeof(float) * T * M;
        cudaStream_t st = cur_stream();
        MB_CUDA_TRY(cudaStreamSynchronize(st));
        if (io.reserve(bytes)) return -1;
        float *d = static_cast<float *>(io.ptr);
        int chunks = host_chunks > 0 ? host_chunks : (bytes >= kChunkedHostBytes ? 2 : 1);
        chunks = std::max(1, std::min(chunks, batch));
        log_msg(3, "forward: batch %d x L %d from host buffers (%zu bytes each way), %s", batch, L, bytes,
                chunks == 1 ? "one call" : "row chunks overlapped with the copies");
        if (chunks == 1) {
            MB_CUDA_TRY(cudaMemcpyAsync(d, in, bytes, cudaMemcpyHostToDevice, st));
            if (forward_device(d, d, batch, L, st)) return -1;
            MB_CUDA_TRY(cudaMemcpyAsync(out, d, bytes, cudaMemcpyDeviceToHost, st));
            MB_CUDA_TRY(cudaStreamSynchronize(st));
            return 0;
        }
        if (!h2d) MB_CUDA_TRY(cudaStreamCreateWithFlags(&h2d, cudaStreamNonBlocking));
        if (!d2h) MB_CUDA_TRY(cudaStreamCreateWithFlags(&d2h, cudaStreamNonBlocking));
        // Row ranges: forced chunk counts split evenly; automatic: batch/8
        // rows per chunk for the edge-layer schedule, else [c, batch - 2c, c].
        const int nl = (int)layers.size();
        const bool edges = host_chunks == 0 && batch >= 3 && nl >= 2 * kEdgeLayers;
        std::vector<int> starts;
        if (host_chunks > 0 || batch < 3) {
            const int rows = (batch + chunks - 1) / chunks;
            for (int r0 = 0; r0 < batch; r0 += rows) starts.push_back(r0);
        } else if (edges) {
            const int c = std::max(1, batch / 8);
            for (int r0 = 0; r0 < batch; r0 += c) starts.push_back(r0);
        } else {
            const int c = std::max(1, batch / 8);
            starts = {0, c, batch - c};
        }
        starts.push_back(batch);
        chunks = (int)starts.size() - 1;
        while ((int)io_events.size() < 2 * chunks) {
            cudaEvent_t e;
            MB_CUDA_TRY(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
            io_events.push_back(e);
        }
        const size_t row_elems = (size_t)L * M;
        // Errors inside the loops stop further enqueues but never return
        // early: the copies already queued read `in` and write `out`, so all
        // three streams are drained before returning, error or not.
        int err = 0;
        auto note = [&](cudaError_t e, const char *what) {
            if (e != cudaSuccess && !err) {
                set_error(std::string("forward: ") + what + ": " + cudaGetErrorString(e));
                err = -1;
            }
        };
        int uploaded = 0;
        for (int k = 0; k < chunks && !err; ++k) {
            const int r0 = starts[k], nr = starts[k + 1] - r0;
            if (nr <= 0) break;
            note(cudaMemcpyAsync(d + r0 * row_elems, in + r0 * row_elems, sizeof(float) * nr * row_elems,
                                 cudaMemcpyHostToDevice, h2d),
                 "host-to-device copy");
            if (!err) note(cudaEventRecord(io_events[2 * k], h2d), "event record");
            if (!err) uploaded = k + 1;
        }
        // Compute on st; chunk k's download waits for the event after its
        // last layer.
        auto download = [&](int k) {
            const int r0 = starts[k], nr = starts[k + 1] - r0;
            note(cudaEventRecord(io_events[2 * k + 1], st), "event record");
            if (!err) note(cudaStreamWaitEvent(d2h, io_events[2 * k + 1], 0), "stream wait");
            if (!err)
                note(cudaMemcpyAsync(out + r0 * row_elems, d + r0 * row_elems, sizeof(float) * nr * row_elems,
                                     cudaMemcpyDeviceToHost, d2h),
                     "device-to-host copy");
        };
        if (edges) {
            // The arena at full size first, so no chunk call regrows it.
            Arena full{};
            if (uploaded < chunks || ensure_arena(batch, L, full)) err = -1;
            for (int k = 0; k < chunks && !err; ++k) {
                const int r0 = starts[k], nr = starts[k + 1] - r0;
                note(cudaStreamWaitEvent(st, io_events[2 * k], 0), "stream wait");
                if (!err && forward_layers(d + r0 * row_elems, nr, L, 0, kEdgeLayers, st)) err = -1;
            }
            if (!err && forward_layers(d, batch, L, kEdgeLayers, nl - kEdgeLayers, st)) err = -1;
            for (int k = 0; k < chunks && !err; ++k) {
                const int r0 = starts[k], nr = starts[k + 1] - r0;
                if (forward_layers(d + r0 * row_elems, nr, L, nl - kEdgeLayers, nl, st)) err = -1;
                if (!err) download(k);
            }
        } else {
            for (int k = 0; k < uploaded && !err; ++k) {
                const int r0 = starts[k], nr = starts[k + 1] - r0;
                if (nr <= 0) break;
                float *dk = d + r0 * row_elems;
                note(cudaStreamWaitEvent(st, io_events[2 * k], 0), "stream wait");
                if (err) break;
                if (forward_device(dk, dk, nr, L, st)) {
                    err = -1;
                    break;
                }
                download(k);
            }
        }
        const cudaError_t e1 = cudaStreamSynchronize(h2d);
        const cudaError_t e2 = cudaStreamSynchronize(st);
        const cudaError_t e3 = cudaStreamSynchronize(d2h);
        if (err) return -1;
        MB_CUDA_TRY(e1);
        MB_CUDA_TRY(e2);
        MB_CUDA_TRY(e3);
        return 0;
    }
};

}  // namespace mb

// ---- state handle -----------------------------------------------------------
struct MambaStateHandle {
    int dev = 0;
    int batch = 0, n_layer = 0, D = 0, N = 0, K = 0;
    float *conv = nullptr;  // [n_layer, batch, D, K-1]
    float *ssm = nullptr;   // [n_layer, batch, D, N]
    size_t conv_elems() const { return (size_t)n_layer * batch * D * (K - 1); }
    size_t ssm_elems() const { return (size_t)n_layer * batch * D * N; }
    ~MambaStateHandle() {
        mb::DeviceGuard g(dev);
        if (conv) cudaFree(conv);
        if (ssm) cudaFree(ssm);
    }
};

struct MambaModel {
    std::unique_ptr<mb::Model> rt;
};

namespace mb {

struct StepArena {
    void *normed, *xz, *u, *xdbc, *draw, *y, *lin_ws;
    size_t lin_ws_bytes;
};

static int ensure_step_arena(Model &m, int rows, StepArena &ar) {
    const size_t a = m.act_size();
    const int64_t T = rows;
    const size_t lws = m.linear_ws_need(T);
    const size_t need = align_up(T * m.M * a) + align_up(T * 2 * m.D * a) + align_up(T * m.D * a) +
                        align_up(T * m.XD * a) + align_up(T * m.D * a) + align_up(T * m.D * a) + align_up(lws);
    if (need > m.step_arena.bytes) {
        MB_CUDA_TRY(cudaStreamSynchronize(m.stream));
        MB_CUDA_TRY(cudaStreamSynchronize(m.cur_stream()));
        if (m.step_arena.reserve(need)) return -1;
    }
    char *p = static_cast<char *>(m.step_arena.ptr);
    auto take = [&](size_t bytes) {
        char *q = p;
        p += align_up(bytes);
        return (void *)q;
    };
    ar.normed = take(T * m.M * a);
    ar.xz = take(T * 2 * m.D * a);
    ar.u = take(T * m.D * a);
    ar.xdbc = take(T * m.XD * a);
    ar.draw = take(T * m.D * a);
    ar.y = take(T * m.D * a);
    ar.lin_ws = lws ? take(lws) : nullptr;
    ar.lin_ws_bytes = lws;
    return 0;
}

// Enqueues one decode step of every layer on `st` (the arena is ready).
static int step_enqueue(Model &m, MambaStateHandle &s, const float *tok, float *out, cudaStream_t st,
                        const StepArena &ar) {
    const int Bt = s.batch;
    if (tok != out)
        MB_CUDA_TRY(cudaMemcpyAsync(out, tok, sizeof(float) * Bt * m.M, cudaMemcpyDeviceToDevice, st));
    const size_t a = m.act_size();
    const int D = m.D, N = m.N, K = m.K, R = m.R, XD = m.XD;
    Profiler &pf = m.prof;
    pf.debug_failed = false;
    for (int l = 0; l < m.cfg.n_layer; ++l) {
        if (pf.debug_failed) return -1;
        LayerScope layer_scope(pf, l);
        const LayerWeights &w = m.layers[l];
        float *conv_state = s.conv + (size_t)l * Bt * D * (K - 1);
        float *ssm_state = s.ssm + (size_t)l * Bt * D * N;
        {
            OpScope o(pf, MAMBA_OP_RMSNORM, st, 1);
            if (rmsnorm(out, w.norm_w, ar.normed, Bt, m.M, kNormEps, MAMBA_F32, m.act, st)) return -1;
        }
        {
            OpScope o(pf, MAMBA_OP_IN_PROJ, st, 0);
            if (m.gemm(st, Bt, 2 * D, m.M, ar.normed, m.M, w.w_in_t, ar.xz, 2 * D, m.act, 0.f, ar.lin_ws,
                       ar.lin_ws_bytes))
                return -1;
            o.kernels = m.last_gemm_kernels;
        }
        {
            OpScope o(pf, MAMBA_OP_CONV, st, 1);
            if (causal_conv1d_step(ar.xz, 2 * D, w.conv_w, w.conv_b, ar.u, D, conv_state, Bt, D, K, 1, m.act,
                                   st))
                return -1;
        }
        {
            OpScope o(pf, MAMBA_OP_X_PROJ, st, 0);
            if (m.gemm(st, Bt, XD, D, ar.u, D, w.w_x_t, ar.xdbc, XD, m.act, 0.f, ar.lin_ws, ar.lin_ws_bytes))
                return -1;
            o.kernels = m.last_gemm_kernels;
        }
        {
            OpScope o(pf, MAMBA_OP_DT_PROJ, st, 0);
            if (m.gemm(st, Bt, D, R, ar.xdbc, XD, w.w_dt_t, ar.draw, D, m.act, 0.f, ar.lin_ws, ar.lin_ws_bytes))
                return -1;
            o.kernels = m.last_gemm_kernels;
        }
        {
            OpScope o(pf, MAMBA_OP_SCAN, st, 1);
            const char *xdbc = static_cast<const char *>(ar.xdbc);
            if (ssm_step(ar.u, D, ar.draw, D, w.dt_bias, xdbc + (size_t)R * a, xdbc + (size_t)(R + N) * a, XD,
                         w.A, w.Dskip, static_cast<const char *>(ar.xz) + (size_t)D * a, 2 * D, ar.y, D,
                         ssm_state, Bt, D, N, m.act, m.act, m.act, st, w.A_inv))
                return -1;
        }
        {
            OpScope o(pf, MAMBA_OP_OUT_PROJ, st, 0);
            if (m.gemm(st, Bt, m.M, D, ar.y, D, w.w_out_t, out, m.M, MAMBA_F32, 1.f, ar.lin_ws, ar.lin_ws_bytes))
                return -1;
            o.kernels = m.last_gemm_kernels;
        }
    }
    return pf.debug_failed ? -1 : 0;
}

static int step_device(Model &m, MambaStateHandle &s, const float *tok, float *out, cudaStream_t st) {
    MB_CHECK_ARG(tok && out, "step: null pointer");
    MB_CHECK_ARG(s.dev == m.dev && s.n_layer == m.cfg.n_layer && s.D == m.D && s.N == m.N && s.K == m.K,
                 "step: state does not belong to this model's configuration");
    const int Bt = s.batch;
    if (Bt == 0) return 0;
    if (!st) st = m.cur_stream();
    StepArena ar{};
    if (ensure_step_arena(m, Bt, ar)) return -1;  // any allocation happens before a capture
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    MB_CUDA_TRY(cudaStreamIsCapturing(st, &cs));
    // Plain launches when graphs are off, while profiling (events per
    // operation), or when the caller is capturing the stream itself.
    log_msg(3, "step: batch %d, %d layers", Bt, m.cfg.n_layer);
    if (!m.use_graphs || m.prof.on || m.prof.debug || cs != cudaStreamCaptureStatusNone)
        return step_enqueue(m, s, tok, out, st, ar);
    StepGraph &g = m.step_graph;
    const bool hit = g.exec && g.conv == s.conv && g.ssm == s.ssm && g.batch == Bt && g.in == tok && g.out == out &&
                     g.st == st && g.arena == m.step_arena.ptr;
    if (!hit) {
        g.reset();
        log_msg(2, "step: capturing the %d-layer decode step as a CUDA graph (batch %d)", m.cfg.n_layer, Bt);
        MB_CUDA_TRY(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
        const int rc = step_enqueue(m, s, tok, out, st, ar);
        cudaGraph_t graph = nullptr;
        const cudaError_t e = cudaStreamEndCapture(st, &graph);
        if (rc || e != cudaSuccess || !graph) {
            if (graph) cudaGraphDestroy(graph);
            if (!rc) set_error(std::string("step: graph capture failed: ") + cudaGetErrorString(e));
            return -1;
        }
        const cudaError_t ei = cudaGraphInstantiate(&g.exec, graph, 0);
        cudaGraphDestroy(graph);
        if (ei != cudaSuccess) {
            g.exec = nullptr;
            set_error(std::string("step: graph instantiation failed: ") + cudaGetErrorString(ei));
            return -1;
        }
        g.conv = s.conv;
        g.ssm = s.ssm;
        g.batch = Bt;
        g.in = tok;
        g.out = out;
        g.st = st;
        g.arena = m.step_arena.ptr;
    }
    MB_CUDA_TRY(cudaGraphLaunch(g.exec, st));
    return 0;
}

// ---- weights -----------------------------------------------------------------
namespace {

constexpr char kBlobMagic[8] = {'M', 'A', 'M', 'B', 'A', 'B', '2', 0};
constexpr uint32_t kBlobVersion = 1;
constexpr uint32_t kBlobHeader = 64;

bool config_valid(const MambaConfig *c, std::string &why) {
    if (!c) {
        why = "null config";
        return false;
    }
    if (c->d_model <= 0 || c->expand <= 0 || c->n_layer <= 0) {
        why = "d_model, expand and n_layer must be positive";
        return false;
    }
    if (c->d_state < 1 || c->d_state > 16) {
        why = "d_state must be in 1..16";
        return false;
    }
    if (c->d_conv < 1 || c->d_conv > 8) {
        why = "d_conv must be in 1..8";
        return false;
    }
    if (c->dtype != MAMBA_F32 && c->dtype != MAMBA_F16) {
        why = "dtype must be MAMBA_F32 or MAMBA_F16";
        return false;
    }
    if ((int64_t)c->expand * c->d_model > (1 << 24)) {
        why = "d_inner too large";
        return false;
    }
    return true;
}

size_t layer_floats(const MambaConfig &c) {
    const size_t M = c.d_model, D = (size_t)c.expand * c.d_model, N = c.d_state, K = c.d_conv;
    const size_t R = (M + 15) / 16;
    return M * 2 * D + D * K + D + D * (R + 2 * N) + R * D + D * N + D + D * M + M + D;
}

}  // namespace

static int load_weights(Model &m, const void *data, size_t size) {
    MB_CHECK_ARG(data != nullptr, "load_weights: null blob");
    MB_CHECK_ARG(size >= kBlobHeader, "load_weights: blob shorter than its 64-byte header");
    const char *p = static_cast<const char *>(data);
    MB_CHECK_ARG(std::memcmp(p, kBlobMagic, 8) == 0, "load_weights: bad magic (expected MAMBAB2)");
    uint32_t ver, hdr;
    std::memcpy(&ver, p + 8, 4);
    std::memcpy(&hdr, p + 12, 4);
    MB_CHECK_ARG(ver == kBlobVersion && hdr == kBlobHeader, "load_weights: unsupported blob version");
    MambaConfig bc;
    std::memcpy(&bc, p + 16, sizeof(bc));
    MB_CHECK_ARG(std::memcmp(&bc, &m.cfg, sizeof(bc)) == 0, "load_weights: blob config differs from the model's");
    int32_t r;
    std::memcpy(&r, p + 40, 4);
    MB_CHECK_ARG(r == m.R, "load_weights: blob dt_rank differs");
    const size_t per = layer_floats(m.cfg);
    MB_CHECK_ARG(size == kBlobHeader + per * 4 * (size_t)m.cfg.n_layer, "load_weights: blob size mismatch");
    DeviceBuffer stage;
    if (stage.reserve(per * 4)) return -1;
    const int M = m.M, D = m.D, N = m.N, K = m.K, R = m.R, XD = m.XD;
    cudaStream_t st = m.stream;
    for (int l = 0; l < m.cfg.n_layer; ++l) {
        const float *src = reinterpret_cast<const float *>(p + kBlobHeader) + per * l;
        MB_CUDA_TRY(cudaMemcpyAsync(stage.ptr, src, per * 4, cudaMemcpyHostToDevice, st));
        const float *s = static_cast<const float *>(stage.ptr);
        LayerWeights &w = m.layers[l];
        if (transpose_cast(s, w.w_in_t, m.act, M, 2 * D, st)) return -1;
        s += (size_t)M * 2 * D;
        MB_CUDA_TRY(cudaMemcpyAsync(w.conv_w, s, (size_t)D * K * 4, cudaMemcpyDeviceToDevice, st));
        s += (size_t)D * K;
        MB_CUDA_TRY(cudaMemcpyAsync(w.conv_b, s, (size_t)D * 4, cudaMemcpyDeviceToDevice, st));
        s += D;
        if (transpose_cast(s, w.w_x_t, m.act, D, XD, st)) return -1;
        s += (size_t)D * XD;
        if (transpose_cast(s, w.w_dt_t, m.act, R, D, st)) return -1;
        s += (size_t)R * D;
        MB_CUDA_TRY(cudaMemcpyAsync(w.A, s, (size_t)D * N * 4, cudaMemcpyDeviceToDevice, st));
        if (a_inverse(w.A, w.A_inv, (int64_t)D * N, st)) return -1;
        s += (size_t)D * N;
        MB_CUDA_TRY(cudaMemcpyAsync(w.Dskip, s, (size_t)D * 4, cudaMemcpyDeviceToDevice, st));
        s += D;
        if (transpose_cast(s, w.w_out_t, m.act, D, M, st)) return -1;
        s += (size_t)D * M;
        MB_CUDA_TRY(cudaMemcpyAsync(w.norm_w, s, (size_t)M * 4, cudaMemcpyDeviceToDevice, st));
        s += M;
        MB_CUDA_TRY(cudaMemcpyAsync(w.dt_bias, s, (size_t)D * 4, cudaMemcpyDeviceToDevice, st));
        // The staging buffer is reused by the next layer.
        MB_CUDA_TRY(cudaStreamSynchronize(st));
    }
    return 0;
}

// Writes the model's weights as a blob that load_weights accepts: projections
// widened back to FP32 [K, N] (exactly the values the GEMMs use, i.e. already
// rounded to the activation type), per-channel vectors copied as stored.
static int save_weights(Model &m, void *data, size_t size) {
    MB_CHECK_ARG(data != nullptr, "save_weights: null blob");
    const size_t per = layer_floats(m.cfg);
    MB_CHECK_ARG(size == kBlobHeader + per * 4 * (size_t)m.cfg.n_layer,
                 "save_weights: blob size differs from mamba_weights_blob_size");
    char *p = static_cast<char *>(data);
    std::memset(p, 0, kBlobHeader);
    std::memcpy(p, kBlobMagic, 8);
    std::memcpy(p + 8, &kBlobVersion, 4);
    std::memcpy(p + 12, &kBlobHeader, 4);
    std::memcpy(p + 16, &m.cfg, sizeof(MambaConfig));
    const int32_t r = m.R;
    std::memcpy(p + 40, &r, 4);
    DeviceBuffer stage;
    if (stage.reserve(per * 4)) return -1;
    const int M = m.M, D = m.D, N = m.N, K = m.K, R = m.R, XD = m.XD;
    cudaStream_t st = m.stream;
    for (int l = 0; l < m.cfg.n_layer; ++l) {
        float *s = static_cast<float *>(stage.ptr);
        const LayerWeights &w = m.layers[l];
        if (untranspose_widen(w.w_in_t, s, m.act, M, 2 * D, st)) return -1;
        s += (size_t)M * 2 * D;
        MB_CUDA_TRY(cudaMemcpyAsync(s, w.conv_w, (size_t)D * K * 4, cudaMemcpyDeviceToDevice, st));
        s += (size_t)D * K;
        MB_CUDA_TRY(cudaMemcpyAsync(s, w.conv_b, (size_t)D * 4, cudaMemcpyDeviceToDevice, st));
        s += D;
        if (untranspose_widen(w.w_x_t, s, m.act, D, XD, st)) return -1;
        s += (size_t)D * XD;
        if (untranspose_widen(w.w_dt_t, s, m.act, R, D, st)) return -1;
        s += (size_t)R * D;
        MB_CUDA_TRY(cudaMemcpyAsync(s, w.A, (size_t)D * N * 4, cudaMemcpyDeviceToDevice, st));
        s += (size_t)D * N;
        MB_CUDA_TRY(cudaMemcpyAsync(s, w.Dskip, (size_t)D * 4, cudaMemcpyDeviceToDevice, st));
        s += D;
        if (untranspose_widen(w.w_out_t, s, m.act, D, M, st)) return -1;
        s += (size_t)D * M;
        MB_CUDA_TRY(cudaMemcpyAsync(s, w.norm_w, (size_t)M * 4, cudaMemcpyDeviceToDevice, st));
        s += M;
        MB_CUDA_TRY(cudaMemcpyAsync(s, w.dt_bias, (size_t)D * 4, cudaMemcpyDeviceToDevice, st));
        char *dst = p + kBlobHeader + per * 4 * (size_t)l;
        MB_CUDA_TRY(cudaMemcpyAsync(dst, stage.ptr, per * 4, cudaMemcpyDeviceToHost, st));
        // The staging buffer is reused by the next layer.
        MB_CUDA_TRY(cudaStreamSynchronize(st));
    }
    return 0;
}

enum Tag { kTagIn = 1, kTagConvW, kTagConvB, kTagX, kTagDt, kTagOut, kTagDtBias };

static int init_random(Model &m, uint64_t seed) {
    cudaStream_t st = m.stream;
    const int M = m.M, D = m.D, N = m.N, K = m.K, R = m.R, XD = m.XD;
    for (int l = 0; l < m.cfg.n_layer; ++l) {
        LayerWeights &w = m.layers[l];
        if (fill_random(w.w_in_t, m.act, (int64_t)2 * D * M, fill_key(seed, l, kTagIn), 0, 0.f, 0.02f, st)) return -1;
        if (fill_random(w.conv_w, MAMBA_F32, (int64_t)D * K, fill_key(seed, l, kTagConvW), 1, -0.5f, 0.5f, st)) return -1;
        if (fill_random(w.conv_b, MAMBA_F32, D, fill_key(seed, l, kTagConvB), 1, -0.5f, 0.5f, st)) return -1;
        if (fill_random(w.w_x_t, m.act, (int64_t)XD * D, fill_key(seed, l, kTagX), 0, 0.f, 0.02f, st)) return -1;
        if (fill_random(w.w_dt_t, m.act, (int64_t)D * R, fill_key(seed, l, kTagDt), 0, 0.f, 0.02f, st)) return -1;
        if (fill_random(w.w_out_t, m.act, (int64_t)M * D, fill_key(seed, l, kTagOut), 0, 0.f, 0.02f, st)) return -1;
        if (fill_random(w.dt_bias, MAMBA_F32, D, fill_key(seed, l, kTagDtBias), 2, 1e-3f, 1e-1f, st)) return -1;
        if (fill_A(w.A, D, N, st)) return -1;
        if (a_inverse(w.A, w.A_inv, (int64_t)D * N, st)) return -1;
        if (fill_const(w.Dskip, D, 1.f, st)) return -1;
        if (fill_const(w.norm_w, M, 1.f, st)) return -1;
    }
    MB_CUDA_TRY(cudaStreamSynchronize(st));
    return 0;
}

}  // namespace mb

// ============================================================================
// C API
// ============================================================================
using mb::set_error;

extern "C" {

MambaModel *mamba_create(const MambaConfig *cfg) {
    mb::clear_error();
    std::string why;
    if (!mb::config_valid(cfg, why)) {
        set_error("mamba_create: " + why);
        return nullptr;
    }
    auto *m = new MambaModel;
    m->rt = std::make_unique<mb::Model>();
    if (m->rt->init(*cfg)) {
        delete m;
        return nullptr;
    }
    return m;
}

void mamba_destroy(MambaModel *m) {
    if (!m) return;
    if (m->rt) {
        mb::DeviceGuard g(m->rt->dev);
        m->rt.reset();
    }
    delete m;
}

int mamba_load_weights(MambaModel *m, const void *data, size_t size) {
    mb::clear_error();
    if (!m || !m->rt) {
        set_error("mamba_load_weights: null model");
        return -1;
    }
    mb::DeviceGuard g(m->rt->dev);
    return mb::load_weights(*m->rt, data, size) ? -1 : 0;
}

int mamba_forward(MambaModel *m, const float *input, float *output, int batch, int seq_len) {
    mb::clear_error();
    if (!m || !m->rt) {
        set_error("mamba_forward: null model");
        return -1;
    }
    mb::DeviceGuard g(m->rt->dev);
    return m->rt->forward_host(input, output, batch, seq_len) ? -1 : 0;
}

MambaStateHandle *mamba_create_state(MambaModel *m, int batch) {
    mb::clear_error();
    if (!m || !m->rt) {
        set_error("mamba_create_state: null model");
        return nullptr;
    }
    if (batch < 0 || batch > 65535) {
        set_error("mamba_create_state: batch must be in 0..65535");
        return nullptr;
    }
    mb::Model &rt = *m->rt;
    mb::DeviceGuard g(rt.dev);
    auto *s = new MambaStateHandle;
    s->dev = rt.dev;
    s->batch = batch;
    s->n_layer = rt.cfg.n_layer;
    s->D = rt.D;
    s->N = rt.N;
    s->K = rt.K;
    const size_t cb = std::max<size_t>(s->conv_elems(), 1) * 4, sb = std::max<size_t>(s->ssm_elems(), 1) * 4;
    if (cudaMalloc(&s->conv, cb) != cudaSuccess || cudaMalloc(&s->ssm, sb) != cudaSuccess) {
        cudaGetLastError();
        set_error("mamba_create_state: cudaMalloc failed");
        delete s;
        return nullptr;
    }
    if (cudaMemset(s->conv, 0, cb) != cudaSuccess || cudaMemset(s->ssm, 0, sb) != cudaSuccess) {
        set_error("mamba_create_state: cudaMemset failed");
        delete s;
        return nullptr;
    }
    return s;
}

void mamba_reset_state(MambaStateHandle *s) {
    if (!s) return;
    mb::DeviceGuard g(s->dev);
    if (s->conv) cudaMemset(s->conv, 0, std::max<size_t>(s->conv_elems(), 1) * 4);
    if (s->ssm) cudaMemset(s->ssm, 0, std::max<size_t>(s->ssm_elems(), 1) * 4);
}

int mamba_step(MambaModel *m, MambaStateHandle *s, const float *token, float *out) {
    mb::clear_error();
    if (!m || !m->rt || !s) {
        set_error("mamba_step: null model or state");
        return -1;
    }
    mb::Model &rt = *m->rt;
    mb::DeviceGuard g(rt.dev);
    if (!token || !out) {
        set_error("mamba_step: null pointer");
        return -1;
    }
    const size_t bytes = sizeof(float) * (size_t)s->batch * rt.M;
    if (bytes == 0) return 0;
    cudaStream_t st_ = rt.cur_stream();
    if (cudaStreamSynchronize(st_) != cudaSuccess || rt.io.reserve(bytes)) {
        if (!*mb::last_error()) set_error("mamba_step: device error");
        return -1;
    }
    float *d = static_cast<float *>(rt.io.ptr);
    if (cudaMemcpyAsync(d, token, bytes, cudaMemcpyHostToDevice, st_) != cudaSuccess) {
        set_error("mamba_step: host-to-device copy failed");
        return -1;
    }
    if (mb::step_device(rt, *s, d, d, st_)) return -1;
    if (cudaMemcpyAsync(out, d, bytes, cudaMemcpyDeviceToHost, st_) != cudaSuccess ||
        cudaStreamSynchronize(st_) != cudaSuccess) {
        set_error("mamba_step: device-to-host copy failed");
        return -1;
    }
    return 0;
}

void mamba_destroy_state(MambaStateHandle *s) { delete s; }

const char *mamba_last_error(void) { return mb::last_error(); }

unsigned mamba_device_status(int clear) {
    const unsigned scan = mb::device_error_flags(clear != 0);
    const unsigned gemm = mb::gemm_error_flags(clear != 0);
    const unsigned lin = mb::linear_error_flags(clear != 0);
    const unsigned proj = mb::proj_error_flags(clear != 0);
    const unsigned step = mb::step_error_flags(clear != 0);
    return (scan == ~0u || gemm == ~0u || lin == ~0u || proj == ~0u || step == ~0u) ? ~0u
                                                                                       : (scan | gemm | lin | proj | step);
}

int mamba_selftest_bounded_wait(unsigned limit_us, void *stream) {
    mb::clear_error();
    return mb::bounded_wait_selftest(limit_us, static_cast<cudaStream_t>(stream)) ? -1 : 0;
}

int mamba_dt_rank(const MambaConfig *cfg) { return cfg ? (cfg->d_model + 15) / 16 : -1; }

size_t mamba_weights_blob_size(const MambaConfig *cfg) {
    std::string why;
    if (!mb::config_valid(cfg, why)) return 0;
    return mb::kBlobHeader + mb::layer_floats(*cfg) * 4 * (size_t)cfg->n_layer;
}

int mamba_init_weights_random(MambaModel *m, uint64_t seed) {
    mb::clear_error();
    if (!m || !m->rt) {
        set_error("mamba_init_weights_random: null model");
        return -1;
    }
    mb::DeviceGuard g(m->rt->dev);
    return mb::init_random(*m->rt, seed) ? -1 : 0;
}

int mamba_save_weights(MambaModel *m, void *blob, size_t size) {
    mb::clear_error();
    if (!m || !m->rt) {
        set_error("mamba_save_weights: null model");
        return -1;
    }
    mb::DeviceGuard g(m->rt->dev);
    // Weights may still be written by work queued on the caller's stream.
    if (cudaStreamSynchronize(m->rt->cur_stream()) != cudaSuccess) {
        set_error("mamba_save_weights: stream error");
        return -1;
    }
    return mb::save_weights(*m->rt, blob, size) ? -1 : 0;
}

int mamba_forward_device(MambaModel *m, const float *input, float *output, int batch, int seq_len,
                         void *stream) {
    mb::clear_error();
    if (!m || !m->rt) {
        set_error("mamba_forward_device: null model");
        return -1;
    }
    mb::DeviceGuard g(m->rt->dev);
    return m->rt->forward_device(input, output, batch, seq_len, static_cast<cudaStream_t>(stream)) ? -1 : 0;
}

int mamba_step_device(MambaModel *m, MambaStateHandle *s, const float *token, float *out, void *stream) {
    mb::clear_error();
    if (!m || !m->rt || !s) {
        set_error("mamba_step_device: null model or state");
        return -1;
    }
    mb::DeviceGuard g(m->rt->dev);
    return mb::step_device(*m->rt, *s, token, out, static_cast<cudaStream_t>(stream)) ? -1 : 0;
}

int mamba_state_batch(const MambaStateHandle *s) { return s ? s->batch : -1; }

int mamba_state_buffers(MambaStateHandle *s, int layer, float **conv_state, float **ssm_state) {
    if (!s || layer < 0 || layer >= s->n_layer) {
        set_error("mamba_state_buffers: bad state or layer");
        return -1;
    }
    if (conv_state) *conv_state = s->conv + (size_t)layer * s->batch * s->D * (s->K - 1);
    if (ssm_state) *ssm_state = s->ssm + (size_t)layer * s->batch * s->D * s->N;
    return 0;
}

int mamba_set_stream(MambaModel *m, void *stream) {
    mb::clear_error();
    if (!m || !m->rt) {
        set_error("mamba_set_stream: null model");
        return -1;
    }
    m->rt->user_stream = static_cast<cudaStream_t>(stream);
    return 0;
}

int mamba_profile_enable(MambaModel *m, int on) {
    mb::clear_error();
    if (!m || !m->rt) {
        set_error("mamba_profile_enable: null model");
        return -1;
    }
    mb::DeviceGuard g(m->rt->dev);
    if (cudaStreamSynchronize(m->rt->cur_stream()) != cudaSuccess) {
        set_error("mamba_profile_enable: stream error");
        return -1;
    }
    m->rt->prof.reset();
    m->rt->prof.on = on != 0;
    return 0;
}

int mamba_profile_read(MambaModel *m, int op, double *total_ms, int64_t *calls, int64_t *kernels) {
    mb::clear_error();
    if (!m || !m->rt || op < 0 || op >= MAMBA_OP_COUNT) {
        set_error("mamba_profile_read: bad model or op");
        return -1;
    }
    mb::DeviceGuard g(m->rt->dev);
    double tot = 0.0;
    int64_t n = 0, k = 0;
    for (const auto &r : m->rt->prof.recs) {
        if (r.op != op) continue;
        float ms = 0.f;
        if (cudaEventSynchronize(r.b) != cudaSuccess || cudaEventElapsedTime(&ms, r.a, r.b) != cudaSuccess) {
            set_error("mamba_profile_read: event query failed");
            return -1;
        }
        tot += ms;
        ++n;
        k += r.kernels;
    }
    if (total_ms) *total_ms = tot;
    if (calls) *calls = n;
    if (kernels) *kernels = k;
    return 0;
}

// ---- Part 3: kernels on device pointers --------------------------------------
size_t mamba_selective_scan_workspace(const MambaScanArgs *a) { return mb::scan_workspace_bytes(a); }

size_t mamba_scan_summary_workspace(const MambaScanArgs *a) { return mb::chunked_workspace_bytes(a); }

int mamba_selective_scan(const MambaScanArgs *a, void *workspace, size_t workspace_bytes, void *stream) {
    mb::clear_error();
    return mb::selective_scan(a, workspace, workspace_bytes, static_cast<cudaStream_t>(stream)) ? -1 : 0;
}

int mamba_selective_scan_dtproj(const MambaScanArgs *a, const void *dt_r, const int64_t *dt_r_stride, const void *w_dt,
                                int dt_rank, void *stream) {
    mb::clear_error();
    return mb::selective_scan_dtproj(a, dt_r, dt_r_stride, w_dt, dt_rank, static_cast<cudaStream_t>(stream)) ? -1 : 0;
}

int mamba_selective_scan_noalloc(const MambaScanArgs *a, void *stream) {
    mb::clear_error();
    return mb::selective_scan_noalloc(a, static_cast<cudaStream_t>(stream)) ? -1 : 0;
}

int mamba_scan_summary(const MambaScanArgs *a, float *P, float *H, void *workspace, size_t workspace_bytes,
                       void *stream) {
    mb::clear_error();
    return mb::scan_summary(a, P, H, workspace, workspace_bytes, static_cast<cudaStream_t>(stream)) ? -1 : 0;
}

int mamba_scan_compose_prefix(const float *PH, int world, int rank, int64_t count, const float *h0,
                              float *h_in, void *stream) {
    mb::clear_error();
    return mb::scan_compose_prefix(PH, world, rank, count, h0, h_in, static_cast<cudaStream_t>(stream)) ? -1
                                                                                                         : 0;
}

size_t mamba_selective_scan_seqpar_workspace(const MambaScanArgs *a, int world) {
    return mb::seqpar_workspace_bytes(a, world);
}

int mamba_selective_scan_seqpar(const MambaScanArgs *a, void *nccl_comm, int world, int rank, void *workspace,
                                size_t workspace_bytes, void *stream) {
    mb::clear_error();
    return mb::seqpar_scan(a, nccl_comm, world, rank, workspace, workspace_bytes, static_cast<cudaStream_t>(stream))
               ? -1
               : 0;
}

int mamba_nccl_unique_id(void *id128) {
    mb::clear_error();
    return mb::nccl_unique_id(id128) ? -1 : 0;
}

int mamba_nccl_comm_create(const void *id128, int world, int rank, void **comm) {
    mb::clear_error();
    return mb::nccl_comm_create(id128, world, rank, comm) ? -1 : 0;
}

int mamba_nccl_comm_destroy(void *comm) {
    mb::clear_error();
    return mb::nccl_comm_destroy(comm) ? -1 : 0;
}

int mamba_causal_conv1d(const void *x, const int64_t *x_stride, const float *w, const float *bias, void *y,
                        const int64_t *y_stride, int batch, int seqlen, int dim, int K, int silu, int dtype,
                        void *stream) {
    mb::clear_error();
    return mb::causal_conv1d(x, x_stride, w, bias, y, y_stride, batch, seqlen, dim, K, silu, dtype,
                             static_cast<cudaStream_t>(stream))
               ? -1
               : 0;
}

int mamba_causal_conv1d_step(const void *x_t, int64_t x_row_stride, const float *w, const float *bias,
                             void *y_t, int64_t y_row_stride, float *conv_state, int batch, int dim, int K,
                             int silu, int dtype, void *stream) {
    mb::clear_error();
    return mb::causal_conv1d_step(x_t, x_row_stride, w, bias, y_t, y_row_stride, conv_state, batch, dim, K,
                                  silu, dtype, static_cast<cudaStream_t>(stream))
               ? -1
               : 0;
}

int mamba_ssm_step(const void *x, int64_t x_row_stride, const void *delta, int64_t delta_row_stride,
                   const float *dt_bias, const void *B, const void *C, int64_t bc_row_stride, const float *A,
                   const float *D, const void *z, int64_t z_row_stride, void *y, int64_t y_row_stride,
                   float *state, int batch, int dim, int dstate, int x_dtype, int delta_dtype, int bc_dtype,
                   void *stream) {
    mb::clear_error();
    return mb::ssm_step(x, x_row_stride, delta, delta_row_stride, dt_bias, B, C, bc_row_stride, A, D, z,
                        z_row_stride, y, y_row_stride, state, batch, dim, dstate, x_dtype, delta_dtype,
                        bc_dtype, static_cast<cudaStream_t>(stream))
               ? -1
               : 0;
}

int mamba_rmsnorm(const void *x, const float *w, void *y, int64_t rows, int cols, float eps, int in_dtype,
                  int out_dtype, void *stream) {
    mb::clear_error();
    return mb::rmsnorm(x, w, y, rows, cols, eps, in_dtype, out_dtype, static_cast<cudaStream_t>(stream)) ? -1
                                                                                                        : 0;
}

int mamba_propagate_tile_carries(float *carries, int num_tiles, int64_t width, float *total, void *stream) {
    mb::clear_error();
    return mb::propagate_tile_carries(carries, num_tiles, width, total, static_cast<cudaStream_t>(stream)) ? -1 : 0;
}

size_t mamba_linear_workspace(int64_t rows, int n, int k) { return mb::linear_workspace_bytes(rows, n, k); }

int mamba_linear(const void *x, int64_t ldx, const void *w, const float *bias, void *y, int64_t ldy, int64_t rows,
                 int n, int k, int mode, void *workspace, size_t workspace_bytes, void *stream) {
    mb::clear_error();
    return mb::linear_tc(x, ldx, w, bias, y, ldy, rows, n, k, mode, workspace, workspace_bytes,
                         static_cast<cudaStream_t>(stream))
               ? -1
               : 0;
}

int mamba_in_proj_conv(const void *x, const void *w_in, const float *conv_w, const float *conv_b, void *u, void *z,
                       int64_t z_row_stride, int batch, int seqlen, int d_model, int d_inner, int d_conv,
                       void *stream) {
    mb::clear_error();
    if (batch < 0 || seqlen < 0) {
        set_error("mamba_in_proj_conv: negative batch or seqlen");
        return -1;
    }
    const int64_t T = (int64_t)batch * seqlen;
    if (T == 0) return 0;
    return mb::proj_gemm_conv(x, w_in, conv_w, conv_b, u, z, z_row_stride, T, seqlen, d_inner, d_model, d_conv,
                              static_cast<cudaStream_t>(stream))
               ? -1
               : 0;
}

int mamba_gated_mlp_up(const void *x, const void *w_gate_up, void *out, int64_t tokens, int d, int h,
                       void *stream) {
    mb::clear_error();
    return mb::gated_mlp_up(x, w_gate_up, out, tokens, d, h, static_cast<cudaStream_t>(stream)) ? -1 : 0;
}

int mamba_gated_silu_mul(const void *gate, const void *up, void *out, int64_t n, int dtype, void *stream) {
    mb::clear_error();
    return mb::gated_silu_mul(gate, up, out, n, dtype, static_cast<cudaStream_t>(stream)) ? -1 : 0;
}

}  // extern "C"
