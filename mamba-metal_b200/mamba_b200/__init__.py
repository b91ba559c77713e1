"""Python binding of libmamba_b200.so over its C ABI (include/mamba.h).

The library is the product: every call below goes through ctypes into the
CUDA code.  PyTorch is used only to own device memory and streams for the
tensor-level helpers; the model-level class works on numpy/host buffers.
There is no CPU fallback: importing this module fails loudly when the
built library is missing.

Reference interface mirrored (SNAPKITTYWEST/mamba-metal):
  Model            mamba_create / mamba_load_weights / mamba_forward /
                   mamba_create_state / mamba_step ...
                   (Sources/Mamba/MambaRuntime.hpp:69-85)
  selective_scan   selective_scan_f32/_f16 + fused gate
                   (Sources/Kernels/selective_scan.metal:84-93,
                   Sources/Kernels/mamba_block.metal:36-45)
  causal_conv1d, causal_conv1d_step, ssm_step, rmsnorm
                   (Sources/Kernels/causal_conv1d.metal, state_update.metal,
                   rmsnorm.metal)
"""
import ctypes
import os
import struct

import numpy as np

PKG_DIR = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
# MAMBA_B200_LIB selects another build of the same library (e.g. a tuning
# variant); by default the in-tree build is loaded.
LIB_PATH = os.environ.get("MAMBA_B200_LIB") or os.path.join(PKG_DIR, "lib", "libmamba_b200.so")

F32 = 0
F16 = 1

# MambaOp order of include/mamba.h
OP_NAMES = ("rmsnorm", "in_proj", "conv", "x_proj", "dt_proj", "scan", "out_proj")

c_int = ctypes.c_int
c_i64 = ctypes.c_int64
c_size = ctypes.c_size_t
c_void_p = ctypes.c_void_p
c_float = ctypes.c_float
c_float_p = ctypes.POINTER(ctypes.c_float)


class MambaConfig(ctypes.Structure):
    """Layout-compatible with mamba::MambaConfig (Sources/Mamba/MambaConfig.hpp:8-18)."""
    _fields_ = [("d_model", ctypes.c_int32), ("d_state", ctypes.c_int32),
                ("d_conv", ctypes.c_int32), ("expand", ctypes.c_int32),
                ("n_layer", ctypes.c_int32), ("dtype", ctypes.c_int32)]

    @property
    def d_inner(self):
        return self.expand * self.d_model

    @property
    def dt_rank(self):
        return (self.d_model + 15) // 16


class MambaScanArgs(ctypes.Structure):
    _fields_ = [("x", c_void_p), ("delta", c_void_p), ("B", c_void_p), ("C", c_void_p),
                ("A", c_void_p), ("D", c_void_p), ("y", c_void_p), ("final_state", c_void_p),
                ("z", c_void_p), ("dt_bias", c_void_p), ("initial_state", c_void_p),
                ("batch", ctypes.c_int32), ("seqlen", ctypes.c_int32), ("dim", ctypes.c_int32),
                ("dstate", ctypes.c_int32), ("x_dtype", ctypes.c_int32),
                ("delta_dtype", ctypes.c_int32), ("bc_dtype", ctypes.c_int32),
                ("chunk_len", ctypes.c_int32),
                ("x_stride", c_i64 * 3), ("delta_stride", c_i64 * 3), ("B_stride", c_i64 * 3),
                ("C_stride", c_i64 * 3), ("z_stride", c_i64 * 3), ("y_stride", c_i64 * 3)]


# Every symbol include/mamba.h declares, with its ctypes prototype.
_PROTOTYPES = {
    "mamba_create": (c_void_p, [ctypes.POINTER(MambaConfig)]),
    "mamba_destroy": (None, [c_void_p]),
    "mamba_load_weights": (c_int, [c_void_p, c_void_p, c_size]),
    "mamba_forward": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int]),
    "mamba_create_state": (c_void_p, [c_void_p, c_int]),
    "mamba_reset_state": (None, [c_void_p]),
    "mamba_step": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p]),
    "mamba_destroy_state": (None, [c_void_p]),
    "mamba_last_error": (ctypes.c_char_p, []),
    "mamba_device_status": (ctypes.c_uint, [c_int]),
    "mamba_dt_rank": (c_int, [ctypes.POINTER(MambaConfig)]),
    "mamba_weights_blob_size": (c_size, [ctypes.POINTER(MambaConfig)]),
    "mamba_init_weights_random": (c_int, [c_void_p, ctypes.c_uint64]),
    "mamba_save_weights": (c_int, [c_void_p, c_void_p, c_size]),
    "mamba_forward_device": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_void_p]),
    "mamba_step_device": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p]),
    "mamba_state_batch": (c_int, [c_void_p]),
    "mamba_state_buffers": (c_int, [c_void_p, c_int, ctypes.POINTER(c_void_p),
                                    ctypes.POINTER(c_void_p)]),
    "mamba_set_stream": (c_int, [c_void_p, c_void_p]),
    "mamba_profile_enable": (c_int, [c_void_p, c_int]),
    "mamba_profile_read": (c_int, [c_void_p, c_int, ctypes.POINTER(ctypes.c_double),
                                   ctypes.POINTER(c_i64), ctypes.POINTER(c_i64)]),
    "mamba_selective_scan_workspace": (c_size, [ctypes.POINTER(MambaScanArgs)]),
    "mamba_scan_summary_workspace": (c_size, [ctypes.POINTER(MambaScanArgs)]),
    "mamba_selective_scan": (c_int, [ctypes.POINTER(MambaScanArgs), c_void_p, c_size, c_void_p]),
    "mamba_selective_scan_noalloc": (c_int, [ctypes.POINTER(MambaScanArgs), c_void_p]),
    "mamba_selective_scan_dtproj": (c_int, [ctypes.POINTER(MambaScanArgs), c_void_p, ctypes.POINTER(c_i64), c_void_p,
                                            c_int, c_void_p]),
    "mamba_scan_summary": (c_int, [ctypes.POINTER(MambaScanArgs), c_void_p, c_void_p, c_void_p,
                                   c_size, c_void_p]),
    "mamba_selective_scan_seqpar_workspace": (c_size, [ctypes.POINTER(MambaScanArgs), c_int]),
    "mamba_selective_scan_seqpar": (c_int, [ctypes.POINTER(MambaScanArgs), c_void_p, c_int, c_int, c_void_p, c_size,
                                            c_void_p]),
    "mamba_nccl_unique_id": (c_int, [c_void_p]),
    "mamba_nccl_comm_create": (c_int, [c_void_p, c_int, c_int, ctypes.POINTER(c_void_p)]),
    "mamba_nccl_comm_destroy": (c_int, [c_void_p]),
    "mamba_scan_compose_prefix": (c_int, [c_void_p, c_int, c_int, c_i64, c_void_p, c_void_p,
                                          c_void_p]),
    "mamba_causal_conv1d": (c_int, [c_void_p, ctypes.POINTER(c_i64), c_void_p, c_void_p, c_void_p,
                                    ctypes.POINTER(c_i64), c_int, c_int, c_int, c_int, c_int,
                                    c_int, c_void_p]),
    "mamba_causal_conv1d_step": (c_int, [c_void_p, c_i64, c_void_p, c_void_p, c_void_p, c_i64,
                                         c_void_p, c_int, c_int, c_int, c_int, c_int, c_void_p]),
    "mamba_ssm_step": (c_int, [c_void_p, c_i64, c_void_p, c_i64, c_void_p, c_void_p, c_void_p,
                               c_i64, c_void_p, c_void_p, c_void_p, c_i64, c_void_p, c_i64,
                               c_void_p, c_int, c_int, c_int, c_int, c_int, c_int, c_void_p]),
    "mamba_rmsnorm": (c_int, [c_void_p, c_void_p, c_void_p, c_i64, c_int, c_float, c_int, c_int,
                              c_void_p]),
    "mamba_propagate_tile_carries": (c_int, [c_void_p, c_int, c_i64, c_void_p, c_void_p]),
    "mamba_gated_silu_mul": (c_int, [c_void_p, c_void_p, c_void_p, c_i64, c_int, c_void_p]),
    "mamba_gated_mlp_up": (c_int, [c_void_p, c_void_p, c_void_p, c_i64, c_int, c_int, c_void_p]),
    "mamba_in_proj_conv": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_i64, c_int, c_int,
                                   c_int, c_int, c_int, c_void_p]),
    "mamba_linear_workspace": (c_size, [c_i64, c_int, c_int]),
    "mamba_selftest_bounded_wait": (c_int, [ctypes.c_uint, c_void_p]),
    "mamba_linear": (c_int, [c_void_p, c_i64, c_void_p, c_void_p, c_void_p, c_i64, c_i64, c_int, c_int, c_int,
                             c_void_p, c_size, c_void_p]),
}

_lib = None


def lib():
    """Load libmamba_b200.so (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError("libmamba_b200.so not built (%s); run "
                               "python mamba-metal_b200/build.py" % LIB_PATH)
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in _PROTOTYPES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


class MambaError(RuntimeError):
    pass


def _check(rc, what):
    if rc != 0:
        raise MambaError("%s failed: %s" % (what, lib().mamba_last_error().decode()))


def last_error():
    return lib().mamba_last_error().decode()


def device_status(clear=True):
    """Kernel error flags on the current device (0 = none)."""
    return lib().mamba_device_status(int(clear))


# ---------------------------------------------------------------------------
# Weight blob (format in include/mamba.h, Part 2)
# ---------------------------------------------------------------------------
LAYER_TENSORS = ("in_proj", "conv1d", "conv_bias", "x_proj", "dt_proj", "A", "D", "out_proj",
                 "norm_weight", "dt_bias")


def layer_shapes(cfg):
    M, D, N, K, R = cfg.d_model, cfg.d_inner, cfg.d_state, cfg.d_conv, cfg.dt_rank
    return {"in_proj": (M, 2 * D), "conv1d": (D, K), "conv_bias": (D,), "x_proj": (D, R + 2 * N),
            "dt_proj": (R, D), "A": (D, N), "D": (D,), "out_proj": (D, M), "norm_weight": (M,),
            "dt_bias": (D,)}


def make_weight_blob(cfg, layers):
    """Serialise per-layer FP32 numpy weights (dicts keyed by LAYER_TENSORS)."""
    shapes = layer_shapes(cfg)
    header = b"MAMBAB2\0" + struct.pack("<II", 1, 64) + bytes(cfg) + \
        struct.pack("<i", cfg.dt_rank) + b"\0" * 20
    assert len(header) == 64
    parts = [header]
    for lw in layers:
        for name in LAYER_TENSORS:
            a = np.ascontiguousarray(lw[name], dtype=np.float32)
            if a.shape != shapes[name]:
                raise ValueError("%s has shape %s, expected %s" % (name, a.shape, shapes[name]))
            parts.append(a.tobytes())
    return b"".join(parts)


def weights_from_blob(cfg, blob):
    """Per-layer dicts of FP32 numpy views into a weight blob (the inverse of
    make_weight_blob; no copies).  blob: bytes, bytearray or a uint8 array."""
    shapes = layer_shapes(cfg)
    buf = np.frombuffer(blob, dtype=np.uint8)
    if bytes(buf[:8]) != b"MAMBAB2\0":
        raise ValueError("not a weight blob (bad magic)")
    per = sum(int(np.prod(shapes[n])) for n in LAYER_TENSORS)
    floats = buf[64:].view(np.float32)
    if floats.size != per * cfg.n_layer:
        raise ValueError("blob holds %d floats, config needs %d" % (floats.size, per * cfg.n_layer))
    layers = []
    off = 0
    for _ in range(cfg.n_layer):
        lw = {}
        for name in LAYER_TENSORS:
            n = int(np.prod(shapes[name]))
            lw[name] = floats[off:off + n].reshape(shapes[name])
            off += n
        layers.append(lw)
    return layers


def random_layer_weights(cfg, rng):
    """Synthetic FP32 weights with the documented distributions (numpy RNG):
    linear ~ N(0, 0.02); conv1d, conv_bias ~ U(-0.5, 0.5);
    dt_bias = softplus^-1(dt), dt ~ logU[1e-3, 1e-1]; A[d, n] = -(n+1);
    D = 1; norm_weight = 1."""
    s = layer_shapes(cfg)
    D, N = cfg.d_inner, cfg.d_state
    w = {}
    w["in_proj"] = rng.normal(0, 0.02, s["in_proj"]).astype(np.float32)
    w["conv1d"] = rng.uniform(-0.5, 0.5, s["conv1d"]).astype(np.float32)
    w["conv_bias"] = rng.uniform(-0.5, 0.5, s["conv_bias"]).astype(np.float32)
    w["x_proj"] = rng.normal(0, 0.02, s["x_proj"]).astype(np.float32)
    w["dt_proj"] = rng.normal(0, 0.02, s["dt_proj"]).astype(np.float32)
    w["A"] = np.tile(-np.arange(1, N + 1, dtype=np.float32), (D, 1))
    w["D"] = np.ones(D, np.float32)
    w["out_proj"] = rng.normal(0, 0.02, s["out_proj"]).astype(np.float32)
    w["norm_weight"] = np.ones(cfg.d_model, np.float32)
    dt = np.exp(rng.uniform(np.log(1e-3), np.log(1e-1), D))
    w["dt_bias"] = (dt + np.log(-np.expm1(-dt))).astype(np.float32)
    return w


# ---------------------------------------------------------------------------
# Model-level API (reference C API)
# ---------------------------------------------------------------------------
class Model:
    """Owns a MambaModel* (mamba_create ... mamba_destroy)."""

    def __init__(self, d_model, d_state=16, d_conv=4, expand=2, n_layer=1, dtype=F16):
        self.cfg = MambaConfig(d_model, d_state, d_conv, expand, n_layer, dtype)
        self._lib = lib()  # kept for close() during interpreter shutdown
        self._h = self._lib.mamba_create(ctypes.byref(self.cfg))
        if not self._h:
            raise MambaError("mamba_create failed: " + last_error())

    def close(self):
        if getattr(self, "_h", None):
            self._lib.mamba_destroy(self._h)
            self._h = None

    def __del__(self):
        self.close()

    @property
    def handle(self):
        return self._h

    def load_weights(self, blob):
        if isinstance(blob, np.ndarray):
            blob = np.ascontiguousarray(blob, dtype=np.uint8)
            _check(lib().mamba_load_weights(self._h, blob.ctypes.data, blob.nbytes), "mamba_load_weights")
            return
        buf = ctypes.create_string_buffer(blob, len(blob)) if isinstance(blob, bytes) else blob
        _check(lib().mamba_load_weights(self._h, buf, len(blob)), "mamba_load_weights")

    def init_random(self, seed):
        _check(lib().mamba_init_weights_random(self._h, seed), "mamba_init_weights_random")

    def save_weights(self):
        """The model's weights as a blob (mamba_save_weights): a numpy uint8
        array that load_weights and weights_from_blob accept."""
        size = lib().mamba_weights_blob_size(ctypes.byref(self.cfg))
        if size == 0:
            raise MambaError("mamba_weights_blob_size: bad config")
        blob = np.empty(size, dtype=np.uint8)
        _check(lib().mamba_save_weights(self._h, blob.ctypes.data, size), "mamba_save_weights")
        return blob

    def forward(self, x, out=None):
        """Host FP32 [batch, L, d_model] numpy in, numpy out (mamba_forward)."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        b, L, m = x.shape
        assert m == self.cfg.d_model
        if out is None:
            out = np.empty_like(x)
        _check(lib().mamba_forward(self._h, x.ctypes.data, out.ctypes.data, b, L), "mamba_forward")
        return out

    def forward_ptr(self, in_ptr, out_ptr, batch, L):
        """mamba_forward on raw host pointers (e.g. pinned torch tensors)."""
        _check(lib().mamba_forward(self._h, in_ptr, out_ptr, batch, L), "mamba_forward")

    def forward_device(self, in_ptr, out_ptr, batch, L, stream=0):
        _check(lib().mamba_forward_device(self._h, in_ptr, out_ptr, batch, L, stream),
               "mamba_forward_device")

    def create_state(self, batch):
        return State(self, batch)

    def set_stream(self, stream):
        """Run later calls (host API included) on a caller stream handle."""
        _check(lib().mamba_set_stream(self._h, stream or None), "mamba_set_stream")

    def profile(self, on=True):
        _check(lib().mamba_profile_enable(self._h, int(on)), "mamba_profile_enable")

    def profile_read(self):
        """{op_name: (total_ms, calls, kernels)} of the recorded operations."""
        out = {}
        for i, name in enumerate(OP_NAMES):
            ms, calls, kern = ctypes.c_double(), c_i64(), c_i64()
            _check(lib().mamba_profile_read(self._h, i, ctypes.byref(ms), ctypes.byref(calls),
                                            ctypes.byref(kern)), "mamba_profile_read")
            out[name] = (ms.value, calls.value, kern.value)
        return out


class State:
    def __init__(self, model, batch):
        self.model = model
        self._lib = lib()
        self._h = self._lib.mamba_create_state(model.handle, batch)
        if not self._h:
            raise MambaError("mamba_create_state failed: " + last_error())
        self.batch = batch

    def reset(self):
        lib().mamba_reset_state(self._h)

    def close(self):
        if getattr(self, "_h", None):
            self._lib.mamba_destroy_state(self._h)
            self._h = None

    def __del__(self):
        self.close()

    @property
    def handle(self):
        return self._h

    def step(self, token, out=None):
        """Host FP32 [batch, d_model] -> [batch, d_model] (mamba_step)."""
        token = np.ascontiguousarray(token, dtype=np.float32)
        if out is None:
            out = np.empty_like(token)
        _check(lib().mamba_step(self.model.handle, self._h, token.ctypes.data, out.ctypes.data),
               "mamba_step")
        return out

    def step_device(self, in_ptr, out_ptr, stream=0):
        _check(lib().mamba_step_device(self.model.handle, self._h, in_ptr, out_ptr, stream),
               "mamba_step_device")

    def buffers(self, layer):
        c, s = c_void_p(), c_void_p()
        _check(lib().mamba_state_buffers(self._h, layer, ctypes.byref(c), ctypes.byref(s)),
               "mamba_state_buffers")
        return c.value, s.value

    def tensors(self, layer):
        """Zero-copy torch views of one layer's FP32 state on the device:
        (conv_state [batch, d_inner, d_conv-1], ssm_state [batch, d_inner,
        d_state]).  Valid while this state handle lives."""
        cfg = self.model.cfg
        c, s = self.buffers(layer)
        return (_device_view(c, (self.batch, cfg.d_inner, cfg.d_conv - 1)),
                _device_view(s, (self.batch, cfg.d_inner, cfg.d_state)))


# ---------------------------------------------------------------------------
# Kernel-level helpers on torch CUDA tensors
# ---------------------------------------------------------------------------
def _torch():
    import torch
    return torch


def _dt(t):
    torch = _torch()
    if t.dtype == torch.float32:
        return F32
    if t.dtype == torch.float16:
        return F16
    raise TypeError("unsupported dtype %s" % t.dtype)


def _ptr(t):
    return None if t is None else t.data_ptr()


class _CudaArray:
    """Describes library-owned device memory through __cuda_array_interface__
    so torch can view it without a copy."""

    def __init__(self, ptr, shape, typestr):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr,
                                         "data": (ptr, False), "version": 2, "strides": None}


def _device_view(ptr, shape, typestr="<f4"):
    torch = _torch()
    return torch.as_tensor(_CudaArray(ptr, shape, typestr), device="cuda")


def _stream(stream):
    torch = _torch()
    if stream is None:
        return torch.cuda.current_stream().cuda_stream
    return stream.cuda_stream if hasattr(stream, "cuda_stream") else stream


def _strides3(t):
    s = t.stride()
    return (c_i64 * 3)(s[0], s[1], s[2])


def _scan_args(x, delta, A, B, C, D, z, dt_bias, h0, y, hN, chunk_len):
    bsz, L, dim = x.shape
    N = A.shape[1]
    a = MambaScanArgs()
    a.x, a.delta, a.B, a.C = _ptr(x), _ptr(delta), _ptr(B), _ptr(C)
    a.A, a.D, a.y, a.final_state = _ptr(A), _ptr(D), _ptr(y), _ptr(hN)
    a.z, a.dt_bias, a.initial_state = _ptr(z), _ptr(dt_bias), _ptr(h0)
    a.batch, a.seqlen, a.dim, a.dstate = bsz, L, dim, N
    a.x_dtype, a.delta_dtype, a.bc_dtype = _dt(x), _dt(delta), _dt(B)
    a.chunk_len = chunk_len
    a.x_stride = _strides3(x)
    a.delta_stride = _strides3(delta)
    a.B_stride = _strides3(B)
    a.C_stride = _strides3(C if C is not None else B)
    a.z_stride = _strides3(z if z is not None else x)
    a.y_stride = _strides3(y if y is not None else x)
    return a


def selective_scan(x, delta, A, B, C, D=None, z=None, dt_bias=None, initial_state=None,
                   return_final_state=False, chunk_len=0, y=None, stream=None):
    """Fused selective scan (mamba_selective_scan).

    x, delta, z: [batch, L, dim] views (any strides); B, C: [batch, L, N];
    A: FP32 [dim, N]; D, dt_bias: FP32 [dim]; initial_state FP32
    [batch, dim, N].  delta is raw (softplus applied in the kernel).
    Returns y (x's dtype) and, if asked, the FP32 final state."""
    torch = _torch()
    bsz, L, dim = x.shape
    N = A.shape[1]
    if y is None:
        y = torch.empty((bsz, L, dim), dtype=x.dtype, device=x.device)
    hN = torch.empty((bsz, dim, N), dtype=torch.float32, device=x.device) \
        if return_final_state else None
    a = _scan_args(x, delta, A, B, C, D, z, dt_bias, initial_state, y, hN, chunk_len)
    ws_bytes = lib().mamba_selective_scan_workspace(ctypes.byref(a))
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=x.device) if ws_bytes else None
    _check(lib().mamba_selective_scan(ctypes.byref(a), _ptr(ws), ws_bytes, _stream(stream)),
           "mamba_selective_scan")
    return (y, hN) if return_final_state else y


def selective_scan_dtproj(x, dt_r, w_dt, A, B, C, D=None, z=None, dt_bias=None, initial_state=None,
                          return_final_state=False, y=None, stream=None):
    """Selective scan with delta = dt_r @ w_dt^T computed inside
    (mamba_selective_scan_dtproj).  x, z: FP16 [batch, L, dim]; dt_r: FP16
    [batch, L, dt_rank] view with channel stride 1; w_dt: FP16 [dim, dt_rank]
    contiguous; B, C FP16 [batch, L, 16]."""
    torch = _torch()
    bsz, L, dim = x.shape
    N = A.shape[1]
    assert dt_r.stride(2) == 1 and w_dt.is_contiguous() and w_dt.shape[0] == dim
    if y is None:
        y = torch.empty((bsz, L, dim), dtype=x.dtype, device=x.device)
    hN = torch.empty((bsz, dim, N), dtype=torch.float32, device=x.device) if return_final_state else None
    a = _scan_args(x, x, A, B, C, D, z, dt_bias, initial_state, y, hN, 0)
    a.delta_dtype = F16
    st = (c_i64 * 2)(dt_r.stride(0), dt_r.stride(1))
    _check(lib().mamba_selective_scan_dtproj(ctypes.byref(a), _ptr(dt_r), st, _ptr(w_dt), w_dt.shape[1],
                                             _stream(stream)), "mamba_selective_scan_dtproj")
    return (y, hN) if return_final_state else y


def scan_workspace_bytes(x, delta, A, B, chunk_len=0):
    a = _scan_args(x, delta, A, B, None, None, None, None, None, None, None, chunk_len)
    return lib().mamba_selective_scan_workspace(ctypes.byref(a))


def scan_summary(x, delta, A, B, dt_bias=None, chunk_len=0, stream=None):
    """(P, H) of this sequence slice: FP32 [batch, dim, N] each."""
    torch = _torch()
    bsz, L, dim = x.shape
    N = A.shape[1]
    P = torch.empty((bsz, dim, N), dtype=torch.float32, device=x.device)
    H = torch.empty_like(P)
    a = _scan_args(x, delta, A, B, None, None, None, dt_bias, None, None, None, chunk_len)
    ws_bytes = lib().mamba_scan_summary_workspace(ctypes.byref(a))
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=x.device) if ws_bytes else None
    _check(lib().mamba_scan_summary(ctypes.byref(a), _ptr(P), _ptr(H), _ptr(ws), ws_bytes,
                                    _stream(stream)), "mamba_scan_summary")
    return P, H


def scan_compose_prefix(PH, rank, h0=None, stream=None):
    """PH: FP32 [world, 2, count] gathered summaries -> h_in FP32 [count]."""
    torch = _torch()
    world, two, count = PH.shape
    assert two == 2 and PH.is_contiguous()
    h_in = torch.empty(count, dtype=torch.float32, device=PH.device)
    _check(lib().mamba_scan_compose_prefix(_ptr(PH), world, rank, count, _ptr(h0), _ptr(h_in),
                                           _stream(stream)), "mamba_scan_compose_prefix")
    return h_in


def causal_conv1d(x, w, bias=None, silu=True, y=None, stream=None):
    """x: [batch, L, dim] view (any strides); w FP32 [dim, K]."""
    torch = _torch()
    bsz, L, dim = x.shape
    if y is None:
        y = torch.empty((bsz, L, dim), dtype=x.dtype, device=x.device)
    _check(lib().mamba_causal_conv1d(_ptr(x), _strides3(x), _ptr(w), _ptr(bias), _ptr(y),
                                     _strides3(y), bsz, L, dim, w.shape[1], int(silu), _dt(x),
                                     _stream(stream)), "mamba_causal_conv1d")
    return y


def causal_conv1d_step(x_t, w, bias, conv_state, silu=True, y=None, stream=None):
    """x_t: [batch, dim] (row stride any, channel stride 1); conv_state FP32
    [batch, dim, K-1] updated in place."""
    torch = _torch()
    bsz, dim = x_t.shape
    assert x_t.stride(1) == 1
    if y is None:
        y = torch.empty((bsz, dim), dtype=x_t.dtype, device=x_t.device)
    _check(lib().mamba_causal_conv1d_step(_ptr(x_t), x_t.stride(0), _ptr(w), _ptr(bias), _ptr(y),
                                          y.stride(0), _ptr(conv_state), bsz, dim, w.shape[1],
                                          int(silu), _dt(x_t), _stream(stream)),
           "mamba_causal_conv1d_step")
    return y


def ssm_step(x, delta, A, B, C, state, D=None, z=None, dt_bias=None, y=None, stream=None):
    """One decode step: x, delta, z [batch, dim]; B, C [batch, N];
    state FP32 [batch, dim, N] updated in place."""
    torch = _torch()
    bsz, dim = x.shape
    N = A.shape[1]
    assert B.stride(0) == C.stride(0) and B.stride(1) == 1 and C.stride(1) == 1
    if y is None:
        y = torch.empty((bsz, dim), dtype=x.dtype, device=x.device)
    _check(lib().mamba_ssm_step(_ptr(x), x.stride(0), _ptr(delta), delta.stride(0), _ptr(dt_bias),
                                _ptr(B), _ptr(C), B.stride(0), _ptr(A), _ptr(D), _ptr(z),
                                z.stride(0) if z is not None else 0, _ptr(y), y.stride(0),
                                _ptr(state), bsz, dim, N, _dt(x), _dt(delta), _dt(B),
                                _stream(stream)), "mamba_ssm_step")
    return y


def rmsnorm(x, w=None, eps=1e-5, out_dtype=None, y=None, stream=None):
    """x: contiguous [rows, cols]; w FP32 [cols] or None."""
    torch = _torch()
    rows, cols = x.shape
    assert x.is_contiguous()
    if y is None:
        y = torch.empty((rows, cols), dtype=out_dtype or x.dtype, device=x.device)
    _check(lib().mamba_rmsnorm(_ptr(x), _ptr(w), _ptr(y), rows, cols, eps, _dt(x), _dt(y),
                               _stream(stream)), "mamba_rmsnorm")
    return y


def propagate_tile_carries(carries, total=None, stream=None):
    """carries: contiguous FP32 [num_tiles, width, 2] (a, b) pairs, replaced in
    place by their exclusive prefixes; returns the inclusive total
    [width, 2] (prefix_scan.metal:19-40)."""
    torch = _torch()
    assert carries.is_contiguous() and carries.dtype == torch.float32 and carries.shape[-1] == 2
    nt, width = carries.shape[0], carries.shape[1]
    if total is None:
        total = torch.empty((width, 2), dtype=torch.float32, device=carries.device)
    _check(lib().mamba_propagate_tile_carries(_ptr(carries), nt, width, _ptr(total), _stream(stream)),
           "mamba_propagate_tile_carries")
    return total


def linear(x, w, bias=None, y=None, mode=0, workspace=None, stream=None):
    """y = x @ w^T (+ bias) on the tensor cores.  x FP16 [rows, k] (row
    stride any multiple of 8); w FP16 [n, k]; mode 0 -> y FP16, 1 -> y FP32
    += result, 2 -> y FP32 = result.  A workspace is allocated when none is
    given and the call splits K."""
    torch = _torch()
    assert x.dtype == torch.float16 and w.dtype == torch.float16
    assert x.stride(1) == 1 and w.is_contiguous()
    rows, k = x.shape
    n = w.shape[0]
    if y is None:
        y = torch.empty((rows, n), dtype=torch.float16 if mode == 0 else torch.float32, device=x.device)
    need = lib().mamba_linear_workspace(rows, n, k)
    if need and workspace is None:
        workspace = torch.empty(need, dtype=torch.uint8, device=x.device)
    ws_ptr, ws_len = (_ptr(workspace), workspace.numel()) if workspace is not None else (None, 0)
    _check(lib().mamba_linear(_ptr(x), x.stride(0), _ptr(w), _ptr(bias), _ptr(y), y.stride(0), rows, n, k, mode,
                              ws_ptr, ws_len, _stream(stream)), "mamba_linear")
    return y


def in_proj_conv(x, w_in, conv_w, conv_b, batch, seqlen, u=None, z=None, stream=None):
    """in_proj with the causal conv + SiLU fused (mamba_in_proj_conv).
    x FP16 [batch*seqlen, d_model]; w_in FP16 [2*d_inner, d_model]; conv_w
    FP32 [d_inner, 4]; conv_b FP32 [d_inner].  Returns (u, z), FP16
    [batch*seqlen, d_inner] each (z may be a strided view)."""
    torch = _torch()
    T, dm = x.shape
    D = w_in.shape[0] // 2
    assert x.is_contiguous() and w_in.is_contiguous() and T == batch * seqlen
    if u is None:
        u = torch.empty((T, D), dtype=torch.float16, device=x.device)
    if z is None:
        z = torch.empty((T, D), dtype=torch.float16, device=x.device)
    assert z.stride(1) == 1
    _check(lib().mamba_in_proj_conv(_ptr(x), _ptr(w_in), _ptr(conv_w), _ptr(conv_b), _ptr(u), _ptr(z), z.stride(0),
                                    batch, seqlen, dm, D, conv_w.shape[1], _stream(stream)), "mamba_in_proj_conv")
    return u, z


def gated_mlp_up(x, w_gate_up, out=None, stream=None):
    """silu(x @ w_gate^T) * (x @ w_up^T) on the tensor cores.  x FP16
    [tokens, d]; w_gate_up FP16 [2h, d] (gate rows, then up rows)."""
    torch = _torch()
    assert x.dtype == torch.float16 and w_gate_up.dtype == torch.float16
    assert x.is_contiguous() and w_gate_up.is_contiguous()
    tokens, d = x.shape
    h = w_gate_up.shape[0] // 2
    assert w_gate_up.shape == (2 * h, d)
    if out is None:
        out = torch.empty((tokens, h), dtype=torch.float16, device=x.device)
    _check(lib().mamba_gated_mlp_up(_ptr(x), _ptr(w_gate_up), _ptr(out), tokens, d, h, _stream(stream)),
           "mamba_gated_mlp_up")
    return out


def gated_silu_mul(gate, up, out=None, stream=None):
    """silu(gate) * up elementwise (contiguous, same dtype)."""
    assert gate.is_contiguous() and up.is_contiguous() and gate.shape == up.shape
    if out is None:
        out = _torch().empty_like(gate)
    _check(lib().mamba_gated_silu_mul(_ptr(gate), _ptr(up), _ptr(out), gate.numel(), _dt(gate),
                                      _stream(stream)), "mamba_gated_silu_mul")
    return out
