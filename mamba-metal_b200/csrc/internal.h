// internal.h -- declarations shared between the .cu translation units.
#pragma once

#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstdint>

#include "mamba.h"

namespace mb {

// scan.cu
size_t scan_workspace_bytes(const MambaScanArgs *a);
size_t chunked_workspace_bytes(const MambaScanArgs *a);
int selective_scan(const MambaScanArgs *a, void *ws, size_t ws_bytes, cudaStream_t st);
int scan_summary(const MambaScanArgs *a, float *P, float *H, void *ws, size_t ws_bytes,
                 cudaStream_t st);
int scan_compose_prefix(const float *PH, int world, int rank, int64_t count, const float *h0,
                        float *h_in, cudaStream_t st);
int scan_seqpar_pass1(const MambaScanArgs *a, float *P_tot, float *H_tot, void *ws, size_t ws_bytes,
                      cudaStream_t st);
int scan_seqpar_pass2(const MambaScanArgs *a, void *ws, size_t ws_bytes, cudaStream_t st);
unsigned device_error_flags(bool clear);
int bounded_wait_selftest(unsigned limit_us, cudaStream_t st);
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder();
int selective_scan_noalloc(const MambaScanArgs *a, cudaStream_t st);
bool scan_dtproj_supported(const MambaScanArgs *a, int R);
int selective_scan_dtproj(const MambaScanArgs *a, const void *dt_r, const int64_t *dr_stride, const void *w_dt,
                          int R, cudaStream_t st);

// seqpar.cu
size_t seqpar_workspace_bytes(const MambaScanArgs *a, int world);
int seqpar_scan(const MambaScanArgs *a, void *comm, int world, int rank, void *ws, size_t ws_bytes,
                cudaStream_t st);
int nccl_unique_id(void *id);
int nccl_comm_create(const void *id, int world, int rank, void **comm);
int nccl_comm_destroy(void *comm);

// conv.cu
int causal_conv1d(const void *x, const int64_t *sx, const float *w, const float *bias, void *y,
                  const int64_t *sy, int batch, int L, int D, int K, int silu, int dtype,
                  cudaStream_t st);
int causal_conv1d_step(const void *x, int64_t xrs, const float *w, const float *bias, void *y,
                       int64_t yrs, float *state, int batch, int D, int K, int silu, int dtype,
                       cudaStream_t st);

// norm.cu
int rmsnorm(const void *x, const float *w, void *y, int64_t rows, int cols, float eps, int in_dt,
            int out_dt, cudaStream_t st);

// ssm_step.cu
int ssm_step(const void *x, int64_t xrs, const void *delta, int64_t drs, const float *dt_bias,
             const void *B, const void *C, int64_t bcrs, const float *A, const float *Dskip,
             const void *z, int64_t zrs, void *y, int64_t yrs, float *state, int batch, int D, int N,
             int xd, int dd, int bd, cudaStream_t st, const float *A_inv = nullptr);
unsigned step_error_flags(bool clear);

// carries.cu
int propagate_tile_carries(float *carries, int num_tiles, int64_t width, float *total, cudaStream_t st);
int gated_silu_mul(const void *gate, const void *up, void *out, int64_t n, int dtype, cudaStream_t st);

// gated_mlp.cu
int gated_mlp_up(const void *x, const void *w_gate_up, void *out, int64_t tokens, int d, int h, cudaStream_t st);
unsigned gemm_error_flags(bool clear);

// gemm_tc.cu
enum ProjMode { kProjF16 = 0, kProjF32Add = 1, kProjF32 = 2 };
// SwiGLU up-projection on the CTA-pair GEMM: out [T, h] FP16 =
// silu(x Wg^T) * (x Wu^T), w = [Wg; Wu] FP16 [2h, d] (gate rows first).
int proj_gemm_gated(const void *x, const void *w_gate_up, void *out, int64_t T, int d, int h, cudaStream_t st);
int proj_gemm(const void *A, int64_t lda, const void *W, const float *bias, void *C, int64_t ldc, int64_t M, int N,
              int K, int mode, cudaStream_t st);
constexpr int64_t kProjMinRows = 512;  // mamba_linear uses the CTA-pair GEMM above this many rows
// in_proj with the causal conv + SiLU fused into its epilogue:
// u = SiLU(conv(x)) [T, D] and z [T, D] (row stride ldz) from A [T, Mdim]
// and W = in_proj^T [2D, Mdim]; T = batch * L tokens, sequences of L.
bool proj_conv_supported(int64_t T, int L, int D, int Mdim, int K);
int proj_gemm_conv(const void *A, const void *W, const float *conv_w, const float *conv_b, void *u, void *z,
                   int64_t ldz, int64_t T, int L, int D, int Mdim, int K, cudaStream_t st);
unsigned proj_error_flags(bool clear);

// linear_tc.cu
size_t linear_workspace_bytes(int64_t M, int N, int K);
int linear_tc(const void *x, int64_t ldx, const void *w, const float *bias, void *y, int64_t ldy, int64_t M, int N,
              int K, int mode, void *ws, size_t ws_bytes, cudaStream_t st);
unsigned linear_error_flags(bool clear);

// init.cu
uint64_t fill_key(uint64_t seed, int layer, int tag);
int fill_random(void *out, int dtype, int64_t n, uint64_t key, int dist, float p0, float p1,
                cudaStream_t st);
int fill_A(float *A, int D, int N, cudaStream_t st);
int a_inverse(const float *A, float *Ainv, int64_t n, cudaStream_t st);
int fill_const(float *p, int64_t n, float v, cudaStream_t st);
int transpose_cast(const float *src, void *dst, int dtype, int K, int N, cudaStream_t st);
int untranspose_widen(const void *src, float *dst, int dtype, int K, int N, cudaStream_t st);

}  // namespace mb
