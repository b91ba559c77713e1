/*
 * mamba.h -- C ABI of libmamba_b200.so, the B200 (sm_100a) implementation of
 * the mamba-metal selective-scan path.
 *
 * Part 1 is the reference's C API, symbol for symbol, with the same
 * signatures, argument meaning and error convention (int 0 = success,
 * -1 = failure; NULL from the create functions on failure).  It replaces
 * Sources/Mamba/MambaRuntime.hpp:69-85 of SNAPKITTYWEST/mamba-metal.
 * Part 2 holds extensions (device-pointer entry points, weight blob helpers,
 * error text).  Part 3 exposes the individual kernels on device pointers, in
 * the buffer order of the reference's Metal kernels, for callers that drive
 * their own layer graph and for the parity tests.
 *
 * Pure C: no C++ or PyTorch types cross this boundary.  All "stream"
 * arguments are cudaStream_t values passed as void*; NULL selects the
 * model's own stream (Part 1/2) or the legacy default stream (Part 3).
 */
#ifndef MAMBA_B200_H
#define MAMBA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------------ */
/* Part 1: the reference C API                                              */
/* ------------------------------------------------------------------------ */

/* Element type.  Replaces enum class DType { F32, F16 }
 * (Sources/Mamba/MambaConfig.hpp:6); same values. */
typedef enum MambaDType { MAMBA_F32 = 0, MAMBA_F16 = 1 } MambaDType;

/* Model hyper-parameters.  Layout-compatible with mamba::MambaConfig
 * (Sources/Mamba/MambaConfig.hpp:8-18): 24 bytes, n_layer at offset 16,
 * dtype at offset 20.  d_inner = expand * d_model; dt_rank is derived as
 * ceil(d_model / 16).  dtype selects the activation and GEMM-weight type;
 * the SSM state is always FP32. */
typedef struct MambaConfig {
    int32_t d_model;
    int32_t d_state; /* N, 1..16 */
    int32_t d_conv;  /* K, 1..8  */
    int32_t expand;
    int32_t n_layer;
    int32_t dtype; /* MambaDType */
} MambaConfig;

typedef struct MambaModel MambaModel;             /* MambaRuntime.hpp:71 */
typedef struct MambaStateHandle MambaStateHandle; /* MambaRuntime.hpp:72 */

/* Replaces mamba_create (MambaRuntime.hpp:74, MambaRuntime.cpp:134-143).
 * Binds the calling thread's current CUDA device (must be sm_100), creates
 * the model's stream and allocates zero weights.  NULL on failure. */
MambaModel *mamba_create(const MambaConfig *cfg);

/* Replaces mamba_destroy (MambaRuntime.hpp:75, MambaRuntime.cpp:145-147).
 * Does not free state handles (as in the reference); they stay valid. */
void mamba_destroy(MambaModel *m);

/* Replaces mamba_load_weights (MambaRuntime.hpp:77, stub at
 * MambaRuntime.cpp:59-67).  Parses the weight blob format documented in
 * Part 2 (64-byte header, then per-layer FP32 tensors in MambaWeights order,
 * MambaRuntime.hpp:13-25, plus dt_bias).  0 / -1. */
int mamba_load_weights(MambaModel *m, const void *data, size_t size);

/* Replaces mamba_forward (MambaRuntime.hpp:78, MambaRuntime.cpp:154-157).
 * input/output: HOST FP32 [batch, seq_len, d_model].  Runs every layer
 * (RMSNorm -> in_proj -> causal conv + SiLU -> x_proj -> dt_proj ->
 * selective scan with SiLU(z) gate -> out_proj + residual) and returns when
 * the output is in host memory.  input and output may alias.  0 / -1. */
int mamba_forward(MambaModel *m, const float *input, float *output, int batch, int seq_len);

/* Replaces mamba_create_state (MambaRuntime.hpp:80, MambaRuntime.cpp:69-78).
 * FP32 conv_state [n_layer, batch, d_inner, d_conv-1] and ssm_state
 * [n_layer, batch, d_inner, d_state] on the model's device, zeroed. */
MambaStateHandle *mamba_create_state(MambaModel *m, int batch);

/* Replaces mamba_reset_state (MambaRuntime.hpp:81, MambaRuntime.cpp:80-90). */
void mamba_reset_state(MambaStateHandle *s);

/* Replaces mamba_step (MambaRuntime.hpp:82, MambaRuntime.cpp:170-173).
 * token/out: HOST FP32 [batch, d_model] where batch is the state's batch
 * (the reference drops the batch and steps one row; this implementation
 * steps every row of the state).  Updates the state in place.  0 / -1. */
int mamba_step(MambaModel *m, MambaStateHandle *s, const float *token, float *out);

/* Replaces mamba_destroy_state (MambaRuntime.hpp:83, MambaRuntime.cpp:175-177). */
void mamba_destroy_state(MambaStateHandle *s);

/* ------------------------------------------------------------------------ */
/* Part 2: extensions                                                       */
/* ------------------------------------------------------------------------ */

/* Text of the last failure on the calling thread ("" if none).  The
 * reference only prints to stderr (MambaRuntime.cpp:42,65). */
const char *mamba_last_error(void);

/* Error flags raised by kernels on the current device since the last
 * clear (0 = none).  Bit 0: a shared-memory pipeline wait inside the
 * selective scan exceeded its 2-second bound, so that call stopped early and
 * its outputs are invalid.  Bit 1: the same for a wait inside the one-CTA
 * SwiGLU kernel (mamba_gated_mlp_up with MAMBA_MLP_PAIR=0).  Bit 2: the same
 * for mamba_linear (and the decode projections that use it).  Bit 3: set by
 * mamba_selftest_bounded_wait.  Bit 4: the same as bit 0 for the CTA-pair
 * projection GEMM (the model's forward projections, mamba_linear above 512
 * rows, mamba_gated_mlp_up by default).  Bit 5: the same for
 * the decode state update's bulk-copy waits (mamba_ssm_step, mamba_step).
 * Waits for the device; clear != 0 resets them. */
unsigned mamba_device_status(int clear);

/* Health check of the device-side failure path: launches one thread that
 * waits, through the same bounded mbarrier wait the kernels use, on a
 * barrier nothing completes, with a limit of limit_us microseconds
 * (1..1000000).  Returns 0 when the wait gave up on time and reported it
 * (bit 3 of mamba_device_status is then set; the context stays usable),
 * -1 otherwise. */
int mamba_selftest_bounded_wait(unsigned limit_us, void *stream);

/* dt_rank used for a config: ceil(d_model / 16). */
int mamba_dt_rank(const MambaConfig *cfg);

/* Weight blob layout accepted by mamba_load_weights:
 *   bytes 0..7   magic "MAMBAB2\0"
 *   bytes 8..11  uint32 version (1)
 *   bytes 12..15 uint32 header size (64)
 *   bytes 16..39 MambaConfig (must equal the model's)
 *   bytes 40..43 int32 dt_rank (must equal mamba_dt_rank)
 *   bytes 44..63 zero
 *   then for each layer, FP32 row-major, in this order:
 *     in_proj [d_model, 2*d_inner], conv1d [d_inner, d_conv],
 *     conv_bias [d_inner], x_proj [d_inner, dt_rank + 2*d_state],
 *     dt_proj [dt_rank, d_inner], A [d_inner, d_state] (negative, i.e.
 *     -exp(A_log)), D [d_inner], out_proj [d_inner, d_model],
 *     norm_weight [d_model], dt_bias [d_inner]. */
size_t mamba_weights_blob_size(const MambaConfig *cfg);

/* Fills every weight on the device from a seed (synthetic checkpoints):
 * linear ~ N(0, 0.02), conv1d and conv_bias ~ U(-0.5, 0.5),
 * dt_bias = softplus^-1(dt) with dt ~ logU[1e-3, 1e-1],
 * A[d,n] = -(n+1), D = 1, norm_weight = 1.  0 / -1. */
int mamba_init_weights_random(MambaModel *m, uint64_t seed);

/* Writes the model's weights into a host buffer of exactly
 * mamba_weights_blob_size(cfg) bytes, in the blob format above, so that
 * mamba_load_weights on a model of the same config reproduces this model
 * bit for bit.  Projections come back as the values the GEMMs use (already
 * rounded to the activation type), widened to FP32.  No counterpart in the
 * reference, which has no way to read weights back (checkpoint save; also
 * lets a CPU reference run on the weights of mamba_init_weights_random).
 * Waits for the model's stream.  0 / -1. */
int mamba_save_weights(MambaModel *m, void *blob, size_t size);

/* Device-pointer forward: input/output are DEVICE FP32 [batch, seq_len,
 * d_model] on the model's device (may alias).  Enqueued on `stream` (NULL =
 * the model's stream); does not synchronize. */
int mamba_forward_device(MambaModel *m, const float *input, float *output, int batch,
                         int seq_len, void *stream);

/* Device-pointer decode step: token/out DEVICE FP32 [batch, d_model].
 * Enqueued on `stream` (NULL = the model's stream); does not synchronize. */
int mamba_step_device(MambaModel *m, MambaStateHandle *s, const float *token, float *out,
                      void *stream);

/* Batch of the state handle, or -1. */
int mamba_state_batch(const MambaStateHandle *s);

/* Device pointers of a state's FP32 buffers for one layer (for export,
 * import and tests).  0 / -1. */
int mamba_state_buffers(MambaStateHandle *s, int layer, float **conv_state, float **ssm_state);

/* Use `stream` (a cudaStream_t on the model's device, owned by the caller)
 * for every later call on this model, including the host-pointer
 * mamba_forward / mamba_step; NULL returns to the model's own stream. */
int mamba_set_stream(MambaModel *m, void *stream);

/* Per-operation timing of the layer graph (tracing).  While enabled, the
 * runtime records a CUDA event pair around every operation it enqueues;
 * mamba_profile_read sums the event times of one operation over all
 * recorded calls (waiting for the last event).  Operations: */
typedef enum MambaOp {
    MAMBA_OP_RMSNORM = 0,
    MAMBA_OP_IN_PROJ = 1,
    MAMBA_OP_CONV = 2,
    MAMBA_OP_X_PROJ = 3,
    MAMBA_OP_DT_PROJ = 4,
    MAMBA_OP_SCAN = 5, /* selective scan (forward) or SSM update (step) */
    MAMBA_OP_OUT_PROJ = 6,
    MAMBA_OP_COUNT = 7
} MambaOp;
int mamba_profile_enable(MambaModel *m, int on); /* clears the records */
/* total_ms: summed duration; calls: recorded operations; kernels: kernels
 * of this library launched by those operations (0 for library GEMMs). */
int mamba_profile_read(MambaModel *m, int op, double *total_ms, int64_t *calls, int64_t *kernels);

/* ------------------------------------------------------------------------ */
/* Part 3: kernels on device pointers                                       */
/* ------------------------------------------------------------------------ */

/* Arguments of the fused selective scan.  Buffer order follows
 * selective_scan_f32 (Sources/Kernels/selective_scan.metal:84-93: x, delta,
 * B, C, A, D, y, final_state) with the gate of
 * fused_selective_scan_gate_f32 (Sources/Kernels/mamba_block.metal:36-45)
 * and the dims of ScanParams (selective_scan.metal:32-38).
 * Per (b, t, d):  dt = softplus(delta + dt_bias);
 *   for n: a = exp(dt*A[d,n]); Bbar = (a-1)/A[d,n]*B  (dt*B when
 *   |A| <= 1e-6); h = a*h + Bbar*x;  y = sum_n C*h + D*x;
 *   if z: y *= SiLU(z).   (Sources/CPURef/selective_scan_cpu.cpp:17-41)
 * Strides are in elements: {batch, time, channel} for x, delta, z, y and
 * {batch, time, state} for B, C.  dtypes: x, z and y share x_dtype.
 * Supported (x, delta, B/C): (F32,F32,F32), (F16,F16,F16), (F16,F32,F16),
 * (F16,F32,F32). */
typedef struct MambaScanArgs {
    const void *x;
    const void *delta;
    const void *B;
    const void *C;
    const float *A;             /* [dim, dstate] */
    const float *D;             /* [dim] or NULL (no skip term) */
    void *y;
    float *final_state;         /* [batch, dim, dstate] or NULL */
    const void *z;              /* gate or NULL */
    const float *dt_bias;       /* [dim] or NULL */
    const float *initial_state; /* [batch, dim, dstate] or NULL (zeros) */
    int32_t batch, seqlen, dim, dstate;
    int32_t x_dtype, delta_dtype, bc_dtype;
    int32_t chunk_len;          /* time chunk per CTA; 0 = automatic */
    int64_t x_stride[3], delta_stride[3], B_stride[3], C_stride[3], z_stride[3], y_stride[3];
} MambaScanArgs;

/* Scratch bytes mamba_selective_scan needs for these args (the per-chunk
 * carries of a sequence split into several time chunks); 0 when the scan
 * runs as one chunk per channel. */
size_t mamba_selective_scan_workspace(const MambaScanArgs *a);

/* Fused selective scan (selective_scan.metal:84-244 and
 * mamba_block.metal:36-128, with the cross-chunk carry that
 * prefix_scan.metal:19-40 intended).  workspace: device memory of at least
 * mamba_selective_scan_workspace(a) bytes (may be NULL when that is 0).
 * 0 / -1 (see mamba_last_error). */
int mamba_selective_scan(const MambaScanArgs *a, void *workspace, size_t workspace_bytes,
                         void *stream);

/* The fused selective scan with the layer's dt_proj computed inside it
 * (linear_f16 of projection.metal:32-49 for dt_proj, MambaRuntime.cpp:98,
 * folded into selective_scan.metal:84-244): delta = dt_r @ w_dt^T with FP32
 * accumulation on the tensor cores, rounded to FP16 (the value a separate
 * FP16 GEMM would store), then dt = softplus(delta + dt_bias) as in
 * mamba_selective_scan; a->delta is ignored.  dt_r FP16 [batch, seqlen,
 * dt_rank] with element strides dt_r_stride = {batch, time} (channel stride
 * 1; e.g. the first dt_rank columns of x_proj's output); w_dt FP16
 * [dim, dt_rank] (dt_proj transposed, K-major).  Requires FP16 x, z, B, C,
 * 16 states, dt_rank a multiple of 8 up to 128, channel-contiguous 16-byte
 * aligned rows, batch * ceil(dim / 128) >= the GPU's SM count (one pass
 * over time, no workspace), a compute capability 10.x GPU.  0 / -1. */
int mamba_selective_scan_dtproj(const MambaScanArgs *a, const void *dt_r, const int64_t *dt_r_stride, const void *w_dt,
                                int dt_rank, void *stream);

/* The fused selective scan without a caller workspace: it allocates no
 * device memory (no cudaMalloc, cudaFree or allocating library call).  No
 * counterpart in the reference.  For callers that cannot allocate device
 * memory or pass scratch to us: hosts whose interface has no slot for a
 * workspace pointer (for instance ones that bind only the Metal kernels'
 * buffer list), and processes that fix their device-memory budget at start-up
 * and forbid allocations afterwards.  When the sequence is split into time
 * chunks, the chunk carries live in one static 32 MiB array in the library's
 * device globals, which every GPU that loads the library holds until the
 * process exits; args needing more than that (see
 * mamba_selective_scan_workspace) are rejected with -1 and a message.  The
 * first call on a device looks up that array's address (once per device), so
 * make that first call before any stream capture.  All calls share the one
 * array and nothing in it carries over between calls (every slot a call reads
 * is written earlier by the same call), but calls that overlap on the GPU
 * (other streams, other host threads on the same device) race on it:
 * serialise them.  When the 32 MiB is committed: with CUDA's default lazy
 * module loading (CUDA_MODULE_LOADING=LAZY), on a device the first time
 * this library's scan code is used there -- the first scan call of any
 * kind, or the first symbol lookup -- not at process start.  A caller that
 * fixes its device-memory budget at start-up should make one small scan call
 * (this one, with batch 1 and a short sequence) on each device during
 * start-up, or run with CUDA_MODULE_LOADING=EAGER so the array is committed
 * when the library's module is loaded.  A device reset (cudaDeviceReset)
 * between calls is handled: the address is looked up again in the new
 * context.  Results equal mamba_selective_scan's, bit for bit, for the same
 * args.  0 / -1. */
int mamba_selective_scan_noalloc(const MambaScanArgs *a, void *stream);

/* Sequence-sharded mode, step 1: summary of this rank's slice of the
 * sequence: for every (b, d, n) the affine map h -> P*h + H that the slice
 * applies to its incoming state.  P, H: DEVICE FP32 [batch, dim, dstate].
 * y, z, C and the initial/final state in `a` are ignored.  workspace: at
 * least mamba_scan_summary_workspace(a) bytes (0: may be NULL). */
size_t mamba_scan_summary_workspace(const MambaScanArgs *a);
int mamba_scan_summary(const MambaScanArgs *a, float *P, float *H, void *workspace,
                       size_t workspace_bytes, void *stream);

/* Sequence-sharded mode, step 2: given the summaries of all ranks gathered
 * as PH[world][2][count] (P then H, count = batch*dim*dstate), compose the
 * state entering rank `rank`: h_in = S_{rank-1} o ... o S_0 (h0), with h0 =
 * NULL meaning zeros.  h_in: DEVICE FP32 [count].  Step 3 is
 * mamba_selective_scan with initial_state = h_in. */
int mamba_scan_compose_prefix(const float *PH, int world, int rank, int64_t count,
                              const float *h0, float *h_in, void *stream);

/* Sequence-sharded mode as one call over NCCL: rank `rank` of `world`
 * holds time slice `rank` of every sequence in `a` (x, delta, z, B, C, y of
 * its slice; a->initial_state, if given, is the state entering slice 0 and
 * must be the same on every rank).  On `stream` it computes its slice's
 * summary, exchanges all summaries with one ncclAllGather of
 * 2*batch*dim*dstate floats (the GPU-granularity carry exchange that
 * prefix_scan.metal:19-40 does for tiles), composes the state entering its
 * slice (mamba_scan_compose_prefix) and rescans the slice from it, writing
 * y and a->final_state (on the last rank: the sequence's final state).
 * nccl_comm is an ncclComm_t of exactly `world` ranks in which this process
 * is `rank` (e.g. from mamba_nccl_comm_create).  Every rank must make the
 * call (it contains a collective).  workspace: 256-byte aligned device
 * memory of mamba_selective_scan_seqpar_workspace(a, world) bytes.  NCCL is
 * loaded at run time (libnccl.so.2); without it the call fails with -1.
 * 0 / -1. */
size_t mamba_selective_scan_seqpar_workspace(const MambaScanArgs *a, int world);
int mamba_selective_scan_seqpar(const MambaScanArgs *a, void *nccl_comm, int world, int rank, void *workspace,
                                size_t workspace_bytes, void *stream);

/* NCCL communicator helpers for the call above: one rank creates a 128-byte
 * id, the caller distributes it (any channel), and every rank creates its
 * communicator on its current device.  0 / -1. */
int mamba_nccl_unique_id(void *id128);
int mamba_nccl_comm_create(const void *id128, int world, int rank, void **comm);
int mamba_nccl_comm_destroy(void *comm);

/* Depthwise causal conv (causal_conv1d.metal:21-45), width K, optional
 * bias and SiLU.  x, y strides {batch, time, channel}; w [dim, K] FP32;
 * bias [dim] FP32 or NULL.  x and y share `dtype`. */
int mamba_causal_conv1d(const void *x, const int64_t *x_stride, const float *w,
                        const float *bias, void *y, const int64_t *y_stride, int batch,
                        int seqlen, int dim, int K, int silu, int dtype, void *stream);

/* Incremental conv (causal_conv1d.metal:50-82): conv over conv_state
 * (oldest..newest) and x_t, then shift-append x_t.  x_t/y_t rows of
 * `x_row_stride`/`y_row_stride` elements per batch row, channel stride 1;
 * conv_state FP32 [batch, dim, K-1] updated in place. */
int mamba_causal_conv1d_step(const void *x_t, int64_t x_row_stride, const float *w,
                             const float *bias, void *y_t, int64_t y_row_stride,
                             float *conv_state, int batch, int dim, int K, int silu,
                             int dtype, void *stream);

/* Single-token SSM update (state_update.metal:15-57, softplus always
 * applied as in selective_scan_cpu.cpp:20), with optional dt_bias and
 * SiLU(z) gate.  x, delta, z, y: rows of the given row strides (channel
 * stride 1); B, C: rows of bc_row_stride elements (state stride 1);
 * state FP32 [batch, dim, dstate] in place.  x, z, y share x_dtype;
 * delta has delta_dtype; B/C have bc_dtype. */
int mamba_ssm_step(const void *x, int64_t x_row_stride, const void *delta,
                   int64_t delta_row_stride, const float *dt_bias, const void *B,
                   const void *C, int64_t bc_row_stride, const float *A, const float *D,
                   const void *z, int64_t z_row_stride, void *y, int64_t y_row_stride,
                   float *state, int batch, int dim, int dstate, int x_dtype,
                   int delta_dtype, int bc_dtype, void *stream);

/* RMSNorm (rmsnorm.metal:11-81): y = x * rsqrt(mean(x^2) + eps) * w.
 * x [rows, cols] of in_dtype, y [rows, cols] of out_dtype, w FP32 [cols]
 * or NULL. */
int mamba_rmsnorm(const void *x, const float *w, void *y, int64_t rows, int cols, float eps,
                  int in_dtype, int out_dtype, void *stream);

/* Exclusive propagation of per-tile affine carries: the job of
 * propagate_tile_carries_f32 (prefix_scan.metal:19-40), with the pair layout
 * that kernel documents and its indexing fixed.  carries FP32
 * [num_tiles, width, 2], pair p of tile t at (t*width + p)*2 as (a, b);
 * in place, tile t's pair becomes the composition of tiles 0..t-1
 * ((1, 0) for tile 0), composed as (a2, b2) o (a1, b1) =
 * (a2*a1, a2*b1 + b2) (prefix_scan.metal:12-14).  total FP32 [width, 2]
 * (or NULL) receives the composition of all tiles.  8-byte aligned. */
int mamba_propagate_tile_carries(float *carries, int num_tiles, int64_t width, float *total,
                                 void *stream);

/* SwiGLU gate (gated_silu_mul_f32/_f16, gated_mlp.metal:14-41):
 * out[i] = silu(gate[i]) * up[i] for n elements of dtype (MAMBA_F32 or
 * MAMBA_F16; FP16 computes in FP32 and rounds once). */
int mamba_gated_silu_mul(const void *gate, const void *up, void *out, int64_t n, int dtype,
                         void *stream);

/* Linear layer on the tensor cores (linear_f16, projection.metal:32-49):
 *   mode 0: y (FP16)  = x @ w^T + bias
 *   mode 1: y (FP32) += x @ w^T + bias   (accumulate into an FP32 buffer)
 *   mode 2: y (FP32)  = x @ w^T + bias
 * x FP16 [rows, k] with row stride ldx elements; w FP16 [n, k] (the
 * reference's [k, n] weight transposed, i.e. K-major); bias FP32 [n] or
 * NULL; y row stride ldy elements.  FP32 accumulation.  k and n multiples
 * of 8, ldx and ldy multiples of 8, pointers 16-byte aligned.  Up to 512
 * rows (decode sizes): one CTA per 256-row block, K split across CTAs when
 * the output blocks cannot fill the GPU, which needs a workspace of
 * mamba_linear_workspace(rows, n, k) bytes (0 when no split is made;
 * 16-byte aligned) for the FP32 partials, summed in split order by a second
 * kernel (results do not depend on CTA timing).  Calls sharing a workspace
 * must not overlap on the GPU.  Above 512 rows: the persistent CTA-pair
 * kernel the model's forward projections use (256 x 256 tiles, M = 256
 * pair MMAs, bulk tensor stores; mode 1 adds with bulk tensor adds), no
 * workspace.  Needs a compute capability 10.x GPU. */
size_t mamba_linear_workspace(int64_t rows, int n, int k);
int mamba_linear(const void *x, int64_t ldx, const void *w, const float *bias, void *y, int64_t ldy, int64_t rows,
                 int n, int k, int mode, void *workspace, size_t workspace_bytes, void *stream);

/* in_proj with the causal conv fused into its epilogue (the first three
 * steps of the layer graph after RMSNorm, MambaRuntime.cpp:94-96:
 * linear_f16, projection.metal:32-49, then causal_conv1d_f16 + SiLU,
 * causal_conv1d.metal:85-100, on its x half), one tensor-core kernel:
 *   xz = x @ w_in^T (FP32 accumulation, rounded to FP16),
 *   u  = SiLU(conv(xz[:, :d_inner]) + conv_b),   z = xz[:, d_inner:]
 * where the conv is causal along each sequence of `seqlen` tokens (zero
 * before its start), taps oldest first.  x FP16 [batch*seqlen, d_model];
 * w_in FP16 [2*d_inner, d_model] (in_proj transposed); conv_w FP32
 * [d_inner, 4]; conv_b FP32 [d_inner]; u FP16 [batch*seqlen, d_inner];
 * z FP16 rows of z_row_stride elements (the x half of xz is never written).
 * Requires d_conv = 4, d_inner a multiple of 256, d_model a multiple of 8,
 * 16-byte aligned pointers, a compute capability 10.x GPU.  Results equal
 * mamba_linear (mode 0) followed by mamba_causal_conv1d (silu = 1) bit for
 * bit.  0 / -1. */
int mamba_in_proj_conv(const void *x, const void *w_in, const float *conv_w, const float *conv_b, void *u, void *z,
                       int64_t z_row_stride, int batch, int seqlen, int d_model, int d_inner, int d_conv,
                       void *stream);

/* Fused SwiGLU up-projection on the tensor cores (no reference
 * counterpart as one op: the reference's linear_f16 twice, then
 * gated_silu_mul_f16, gated_mlp.metal:12-41):
 *   out = silu(x @ w_gate^T) * (x @ w_up^T)
 * x FP16 [tokens, d] row-major; w_gate_up FP16 [2h, d] with w_gate in rows
 * 0..h-1 and w_up in rows h..2h-1 (the nn.Linear weight layout); out FP16
 * [tokens, h].  FP32 accumulation; the gate is applied to the FP32
 * accumulators and rounded once.  d and h multiples of 8, pointers 16-byte
 * aligned.  Needs a compute capability 10.x GPU.  Runs on the CTA-pair
 * projection GEMM (gate rows in one CTA of the pair, the matching up rows in
 * the other); MAMBA_MLP_PAIR=0 selects the one-CTA kernel instead. */
int mamba_gated_mlp_up(const void *x, const void *w_gate_up, void *out, int64_t tokens, int d, int h,
                       void *stream);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* MAMBA_B200_H */
