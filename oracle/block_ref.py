"""CPU block reference -- TEST INFRASTRUCTURE ONLY (the checker).

numpy restatement of the Mamba layer graph the reference describes at
Sources/Mamba/MambaRuntime.cpp:93-101 (RMSNorm -> in_proj -> causal conv ->
SiLU -> x_proj -> dt/B/C -> selective scan -> SiLU(z) gate -> out_proj ->
residual), built from the kernel maths of Sources/Kernels/rmsnorm.metal:26-44,
projection.metal:25-29 (y = x @ W), causal_conv1d.metal:34-44 and the scan
oracle (oracle.scan, restating selective_scan_cpu.cpp:7-45), plus the decode
step (causal_conv1d.metal:59-81, state_update.metal:31-56 with softplus
always applied).

Activations are rounded to the activation dtype at exactly the points where
the CUDA path stores them (RMSNorm output, every projection output, conv
output, scan output) and GEMM weights are rounded to it as well, so GPU and
CPU see identical operands; the residual stream stays FP32.  GEMMs
accumulate in FP32.
"""
import os

import numpy as np

import oracle

F32, F16 = 0, 1
EPS = 1e-5


def rnd(a, act):
    a = np.asarray(a, dtype=np.float32)
    return a.astype(np.float16).astype(np.float32) if act == F16 else a


def _mm(a, w):
    return np.matmul(np.ascontiguousarray(a, np.float32), np.ascontiguousarray(w, np.float32))


def _scan_with_reference(u, draw, Bm, Cm, w, z):
    """The scan step through the reference's own selective_scan_cpu
    (oracle/_ref): it takes the biased delta and has no gate, so the dt bias
    is added before and SiLU(z) applied after, as the gated restatement does."""
    delta = (draw + w["dt_bias"][None, None, :]).astype(np.float32)
    y, _ = oracle.ref_scan_batched(u, delta, Bm, Cm, w["A"], w["D"],
                                   nthreads=os.cpu_count() or 1)
    return y * (z / (np.float32(1) + np.exp(-z)))


def block_forward(h, w, cfg, act, scan_impl="oracle"):
    """h: FP32 [batch, L, d_model] -> FP32 [batch, L, d_model].
    scan_impl "reference" runs the scan step through the reference's own
    compiled selective_scan_cpu instead of the restatement."""
    bsz, L, M = h.shape
    D, N, R = cfg.d_inner, cfg.d_state, cfg.dt_rank
    T = bsz * L
    hn = rnd(oracle.rmsnorm(h.reshape(T, M), w["norm_weight"], EPS), act)
    xz = rnd(_mm(hn, rnd(w["in_proj"], act)), act).reshape(bsz, L, 2 * D)
    x, z = xz[..., :D], xz[..., D:]
    u = rnd(oracle.causal_conv1d(x, w["conv1d"], w["conv_bias"], silu=True), act)
    xdbc = rnd(_mm(u.reshape(T, D), rnd(w["x_proj"], act)), act).reshape(bsz, L, R + 2 * N)
    dt_r, Bm, Cm = xdbc[..., :R], xdbc[..., R:R + N], xdbc[..., R + N:]
    draw = rnd(_mm(dt_r.reshape(T, R), rnd(w["dt_proj"], act)), act).reshape(bsz, L, D)
    if scan_impl == "reference":
        y = _scan_with_reference(u, draw, Bm, Cm, w, z)
    else:
        y, _ = oracle.scan(u, draw, Bm, Cm, w["A"], w["D"], z=z, dt_bias=w["dt_bias"])
    y = rnd(y, act)
    return h + _mm(y.reshape(T, D), rnd(w["out_proj"], act)).reshape(bsz, L, M)


def model_forward(h, layers, cfg, act):
    h = np.asarray(h, np.float32)
    for w in layers:
        h = block_forward(h, w, cfg, act)
    return h


def new_state(cfg, batch):
    D, N, K = cfg.d_inner, cfg.d_state, cfg.d_conv
    conv = [np.zeros((batch, D, K - 1), np.float32) for _ in range(cfg.n_layer)]
    ssm = [np.zeros((batch, D, N), np.float32) for _ in range(cfg.n_layer)]
    return conv, ssm


def block_step(h_t, w, conv_state, ssm_state, cfg, act):
    """h_t: FP32 [batch, d_model]; states updated in place."""
    D, N, R = cfg.d_inner, cfg.d_state, cfg.dt_rank
    hn = rnd(oracle.rmsnorm(h_t, w["norm_weight"], EPS), act)
    xz = rnd(_mm(hn, rnd(w["in_proj"], act)), act)
    x, z = xz[:, :D], xz[:, D:]
    u = rnd(oracle.causal_conv1d_step(x, w["conv1d"], w["conv_bias"], conv_state, silu=True), act)
    xdbc = rnd(_mm(u, rnd(w["x_proj"], act)), act)
    dt_r, Bm, Cm = xdbc[:, :R], xdbc[:, R:R + N], xdbc[:, R + N:]
    draw = rnd(_mm(dt_r, rnd(w["dt_proj"], act)), act)
    y = oracle.ssm_step(u, draw, Bm, Cm, w["A"], w["D"], ssm_state, z=z, dt_bias=w["dt_bias"])
    y = rnd(y, act)
    return h_t + _mm(y, rnd(w["out_proj"], act))


def model_decode(h_seq, layers, cfg, act, state=None):
    """T decode steps from `state` (zeros when None): h_seq FP32 [batch, T,
    d_model] -> outputs [batch, T, d_model].  The same arithmetic as calling
    model_step T times (conv and SSM updates via the step restatements, token
    by token), ordered layer by layer: a layer's projections act row-wise,
    so they run on all T tokens at once and each layer's weights are read
    once instead of T times."""
    h = np.array(h_seq, dtype=np.float32, copy=True)
    bsz, T, M = h.shape
    D, N, R = cfg.d_inner, cfg.d_state, cfg.dt_rank
    conv, ssm = state if state is not None else new_state(cfg, bsz)
    for l, w in enumerate(layers):
        hn = rnd(oracle.rmsnorm(h.reshape(bsz * T, M), w["norm_weight"], EPS), act)
        xz = rnd(_mm(hn, rnd(w["in_proj"], act)), act).reshape(bsz, T, 2 * D)
        u = np.empty((bsz, T, D), np.float32)
        for t in range(T):
            u[:, t] = rnd(oracle.causal_conv1d_step(xz[:, t, :D], w["conv1d"], w["conv_bias"], conv[l],
                                                    silu=True), act)
        xdbc = rnd(_mm(u.reshape(bsz * T, D), rnd(w["x_proj"], act)), act).reshape(bsz, T, R + 2 * N)
        draw = rnd(_mm(xdbc[..., :R].reshape(bsz * T, R), rnd(w["dt_proj"], act)), act).reshape(bsz, T, D)
        y = np.empty((bsz, T, D), np.float32)
        for t in range(T):
            y[:, t] = oracle.ssm_step(u[:, t], draw[:, t], xdbc[:, t, R:R + N], xdbc[:, t, R + N:], w["A"],
                                      w["D"], ssm[l], z=xz[:, t, D:], dt_bias=w["dt_bias"])
        y = rnd(y, act)
        h = h + _mm(y.reshape(bsz * T, D), rnd(w["out_proj"], act)).reshape(bsz, T, M)
    return h


def model_step(h_t, layers, state, cfg, act):
    conv, ssm = state
    h_t = np.asarray(h_t, np.float32)
    for l, w in enumerate(layers):
        h_t = block_step(h_t, w, conv[l], ssm[l], cfg, act)
    return h_t
