"""CPU oracle for the selective-scan path -- TEST INFRASTRUCTURE ONLY.

This package is the checker.  Only tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline leg import it; the product (libmamba_b200.so and the
mamba_b200 binding) never does.

* liboracle.so (oracle/scan_ref.c): C restatement of the reference's
  selective_scan_cpu (Sources/CPURef/selective_scan_cpu.cpp:7-45) and its
  generalisations (batch, strides, dt bias, initial state, SiLU gate, chunk
  summaries), plus conv, conv step, SSM step and RMSNorm restatements.
* libref_scan.so (oracle/_ref/): the reference's own selective_scan_cpu,
  compiled from the reference tree by oracle/build_oracle.py.
* oracle.block_ref: numpy restatement of the Mamba block graph
  (Sources/Mamba/MambaRuntime.cpp:93-101) and of the decode step, with
  activations rounded at the same points as the CUDA path.
"""
import ctypes
import os

import numpy as np

from . import build_oracle

HERE = os.path.dirname(os.path.abspath(__file__))
_c = ctypes.c_int
_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_f = ctypes.c_float

_lib = None
_ref = None


def lib():
    """The C restatement (built on demand where gcc exists)."""
    global _lib
    if _lib is None:
        path = os.path.join(build_oracle.BUILD, "liboracle.so")
        if not os.path.exists(path):
            build_oracle.build_restatement()
        L = ctypes.CDLL(path)
        L.oracle_selective_scan.argtypes = [_p] * 8 + [_c, _c, _c]
        L.oracle_scan_general.argtypes = [_p] * 17 + [_c] * 5
        L.oracle_scan_chunk_summary.argtypes = [_p] * 10 + [_c] * 5
        L.oracle_scan_chunk_combine.argtypes = [_p, _p, _c, _i64, _p, _p, _p]
        L.oracle_causal_conv1d.argtypes = [_p] * 6 + [_c] * 5
        L.oracle_causal_conv1d_step.argtypes = [_p] * 5 + [_c] * 4
        L.oracle_ssm_step.argtypes = [_p] * 5 + [_i64, _i64] + [_p] * 5 + [_c] * 3
        L.oracle_rmsnorm.argtypes = [_p, _p, _p, _i64, _c, _f]
        L.oracle_affine_compose.argtypes = [_f, _f, _f, _f, _p, _p]
        L.oracle_propagate_tile_carries.argtypes = [_p, _c, _i64, _p]
        L.oracle_gated_silu_mul.argtypes = [_p, _p, _p, _i64]
        _lib = L
    return _lib


def ref_lib():
    """The reference's own selective_scan_cpu, or None if it was not built."""
    global _ref
    if _ref is None:
        path = os.path.join(HERE, "_ref", "libref_scan.so")
        if not os.path.exists(path):
            build_oracle.build_reference()
        if not os.path.exists(path):
            return None
        L = ctypes.CDLL(path)
        L.ref_selective_scan_cpu.argtypes = [_p] * 8 + [_c, _c, _c]
        L.ref_scan_batched_mt.argtypes = [_p] * 8 + [_c] * 5
        _ref = L
    return _ref


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _ptr(a):
    return None if a is None else a.ctypes.data


def _estrides(a):
    return (_i64 * len(a.shape))(*[s // a.itemsize for s in a.strides])


# --- reference-exact single-sequence scan -----------------------------------
def selective_scan(x, delta, B, C, A, Dskip, use_reference=False):
    """x, delta [L, D]; B, C [L, N]; A [D, N]; Dskip [D] -> (y [L, D], h [D, N])."""
    x, delta, B, C, A, Dskip = map(_f32, (x, delta, B, C, A, Dskip))
    L, D = x.shape
    N = A.shape[1]
    y = np.empty((L, D), np.float32)
    h = np.empty((D, N), np.float32)
    if use_reference:
        r = ref_lib()
        if r is None:
            raise RuntimeError("reference oracle library not built")
        r.ref_selective_scan_cpu(*map(_ptr, (x, delta, B, C, A, Dskip, y, h)), L, D, N)
    else:
        lib().oracle_selective_scan(*map(_ptr, (x, delta, B, C, A, Dskip, y, h)), L, D, N)
    return y, h


def ref_scan_batched(x, delta, B, C, A, Dskip, nthreads=1):
    """Reference selective_scan_cpu over a batch: x, delta [b, L, D];
    B, C [b, L, N] -> (y [b, L, D], h [b, D, N]), split over host threads."""
    x, delta, B, C, A, Dskip = map(_f32, (x, delta, B, C, A, Dskip))
    b, L, D = x.shape
    N = A.shape[1]
    y = np.empty_like(x)
    h = np.empty((b, D, N), np.float32)
    r = ref_lib()
    if r is None:
        raise RuntimeError("reference oracle library not built")
    r.ref_scan_batched_mt(*map(_ptr, (x, delta, B, C, A, Dskip, y, h)), b, L, D, N, nthreads)
    return y, h


# --- generalised scan ----------------------------------------------------------
def scan(x, delta, B, C, A, Dskip=None, z=None, dt_bias=None, h0=None, nthreads=None):
    """Batched scan on FP32 numpy views of any strides.

    x, delta, z: [batch, L, D]; B, C: [batch, L, N]; returns
    (y [batch, L, D] contiguous, h_final [batch, D, N])."""
    arrs = [x, delta, B, C, z]
    for a in arrs:
        if a is not None and a.dtype != np.float32:
            raise TypeError("oracle.scan expects float32 arrays")
    bsz, L, D = x.shape
    N = A.shape[1]
    A = _f32(A)
    Dskip = _f32(Dskip if Dskip is not None else np.zeros(D, np.float32))
    dt_bias = None if dt_bias is None else _f32(dt_bias)
    h0 = None if h0 is None else _f32(h0)
    y = np.empty((bsz, L, D), np.float32)
    hN = np.empty((bsz, D, N), np.float32)
    nthreads = nthreads or os.cpu_count() or 1
    zz = z if z is not None else x
    rc = lib().oracle_scan_general(
        _ptr(x), _estrides(x), _ptr(delta), _estrides(delta), _ptr(B), _estrides(B), _ptr(C),
        _estrides(C), _ptr(A), _ptr(Dskip), _ptr(dt_bias), _ptr(z), _estrides(zz), _ptr(h0),
        _ptr(y), _estrides(y), _ptr(hN), bsz, L, D, N, nthreads)
    assert rc == 0
    return y, hN


def scan_chunk_summary(x, delta, B, A, dt_bias=None, t0=0, t1=None):
    """(P, H) [batch, D, N] of the affine map over t in [t0, t1)."""
    bsz, L, D = x.shape
    N = A.shape[1]
    t1 = L if t1 is None else t1
    P = np.empty((bsz, D, N), np.float32)
    H = np.empty((bsz, D, N), np.float32)
    A = _f32(A)
    dt_bias = None if dt_bias is None else _f32(dt_bias)
    rc = lib().oracle_scan_chunk_summary(
        _ptr(x), _estrides(x), _ptr(delta), _estrides(delta), _ptr(B), _estrides(B), _ptr(A),
        _ptr(dt_bias), _ptr(P), _ptr(H), bsz, t0, t1, D, N)
    assert rc == 0
    return P, H


def scan_chunk_combine(P, H, h0=None):
    """P, H: [G, count]; returns (h_in [G, count], h_final [count])."""
    P, H = _f32(P), _f32(H)
    G, count = P.shape
    h_in = np.empty((G, count), np.float32)
    hf = np.empty(count, np.float32)
    h0 = None if h0 is None else _f32(h0).reshape(-1)
    lib().oracle_scan_chunk_combine(_ptr(P), _ptr(H), G, count, _ptr(h0), _ptr(h_in), _ptr(hf))
    return h_in, hf


def affine_compose(t2, t1):
    a, b = _f(), _f()
    lib().oracle_affine_compose(t2[0], t2[1], t1[0], t1[1], ctypes.byref(a), ctypes.byref(b))
    return a.value, b.value


def propagate_tile_carries(carries):
    """carries [num_tiles, width, 2] FP32 (a, b) pairs -> (exclusive prefixes
    of the same shape, inclusive total [width, 2]); prefix_scan.metal:19-40."""
    c = np.array(carries, dtype=np.float32, order="C", copy=True)
    nt, width = c.shape[0], c.shape[1]
    total = np.empty((width, 2), np.float32)
    lib().oracle_propagate_tile_carries(_ptr(c), nt, width, _ptr(total))
    return c, total


def gated_silu_mul(gate, up):
    """silu(gate) * up elementwise in FP32 (gated_mlp.metal:14-26)."""
    g, u = _f32(gate), _f32(up)
    assert g.shape == u.shape
    out = np.empty_like(g)
    lib().oracle_gated_silu_mul(_ptr(g), _ptr(u), _ptr(out), g.size)
    return out


def linear(x, w, bias=None):
    """y = x @ w^T + bias in float64 (linear_f32/_f16, projection.metal:25-29,
    whose W is [K, N]; here w is that matrix transposed, [N, K])."""
    y = np.asarray(x, np.float64) @ np.asarray(w, np.float64).T
    if bias is not None:
        y = y + np.asarray(bias, np.float64)
    return y


def gated_mlp_up(x, w_gate, w_up):
    """silu(x @ w_gate^T) * (x @ w_up^T) with FP32 products (the two
    projections gated_mlp.metal:13 assumes done, then its gate).
    x [T, D]; w_gate, w_up [H, D]."""
    x, wg, wu = (np.asarray(a, dtype=np.float64) for a in (x, w_gate, w_up))
    g = (x @ wg.T).astype(np.float32)
    u = (x @ wu.T).astype(np.float32)
    return gated_silu_mul(g, u)


def causal_conv1d(x, w, bias=None, silu=True):
    """x: [batch, L, D] FP32 view -> y [batch, L, D]."""
    bsz, L, D = x.shape
    K = w.shape[1]
    y = np.empty((bsz, L, D), np.float32)
    w = _f32(w)
    bias = None if bias is None else _f32(bias)
    lib().oracle_causal_conv1d(_ptr(x), _estrides(x), _ptr(w), _ptr(bias), _ptr(y), _estrides(y),
                               bsz, L, D, K, int(silu))
    return y


def causal_conv1d_step(x_t, w, bias, conv_state, silu=True):
    """x_t [batch, D]; conv_state [batch, D, K-1] FP32 updated in place."""
    # Every array handed to C by address stays bound to a local name until
    # the call returns (a temporary would be freed before the call runs).
    x_t = _f32(x_t)
    w = _f32(w)
    bias = None if bias is None else _f32(bias)
    bsz, D = x_t.shape
    K = w.shape[1]
    y = np.empty((bsz, D), np.float32)
    assert conv_state.dtype == np.float32 and conv_state.flags.c_contiguous
    lib().oracle_causal_conv1d_step(_ptr(x_t), _ptr(w), _ptr(bias), _ptr(y), _ptr(conv_state),
                                    bsz, D, K, int(silu))
    return y


def ssm_step(x, delta, B, C, A, Dskip, state, z=None, dt_bias=None):
    """x, delta, z [batch, D]; B, C [batch, N]; state [batch, D, N] in place."""
    x, delta, B, C, A, Dskip = map(_f32, (x, delta, B, C, A, Dskip))
    z = None if z is None else _f32(z)
    dt_bias = None if dt_bias is None else _f32(dt_bias)
    bsz, D = x.shape
    N = A.shape[1]
    y = np.empty((bsz, D), np.float32)
    assert state.dtype == np.float32 and state.flags.c_contiguous
    lib().oracle_ssm_step(_ptr(x), _ptr(delta), _ptr(dt_bias), _ptr(B), _ptr(C), B.strides[0] // 4,
                          C.strides[0] // 4, _ptr(A), _ptr(Dskip), _ptr(z), _ptr(y), _ptr(state),
                          bsz, D, N)
    return y


def rmsnorm(x, w=None, eps=1e-5):
    x = _f32(x)
    w = None if w is None else _f32(w)
    rows, cols = x.shape
    y = np.empty_like(x)
    lib().oracle_rmsnorm(_ptr(x), _ptr(w), _ptr(y), rows, cols, eps)
    return y


def normwise_rel_err(a, b):
    """max|a - b| / max|b| (the parity metric; b is the oracle)."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    den = np.max(np.abs(b)) if b.size else 0.0
    num = np.max(np.abs(a - b)) if b.size else 0.0
    return float(num / den) if den > 0 else float(num)
