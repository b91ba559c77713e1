"""GPU parity of the fused selective scan (C ABI mamba_selective_scan) against
the oracle.  Tolerances (normwise max|gpu - ref| / max|ref|): 1e-5 for the
FP32 path, 2e-3 for FP16-input paths.
"""
import os

import numpy as np
import pytest
import torch

import mamba_b200 as mb
import oracle
from test_oracle import GOLDEN, load_golden

pytestmark = pytest.mark.gpu

TOL32 = 1e-5
TOL16 = 2e-3


def scan_inputs(seed, bsz, L, D, N):
    """Standalone-scan workload distributions: x, B, C, z ~ N(0,1),
    delta_raw ~ N(-4.6, 0.5) (softplus gives dt ~ 1e-3..1e-1),
    A[d, n] = -(n+1), D = 1."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((bsz, L, D)).astype(np.float32)
    dr = rng.normal(-4.6, 0.5, (bsz, L, D)).astype(np.float32)
    B = rng.standard_normal((bsz, L, N)).astype(np.float32)
    C = rng.standard_normal((bsz, L, N)).astype(np.float32)
    z = rng.standard_normal((bsz, L, D)).astype(np.float32)
    A = np.tile(-np.arange(1, N + 1, dtype=np.float32), (D, 1))
    Dk = np.ones(D, np.float32)
    return x, dr, B, C, z, A, Dk


def dev(a, dtype=torch.float32, time_major=True):
    """numpy [b, L, F] -> CUDA tensor viewed as [b, L, F]; time_major=False
    stores it as [b, F, L] in memory (the layout of the standalone-scan
    workload) and returns the transposed view."""
    t = torch.from_numpy(np.ascontiguousarray(a))
    if not time_major:
        t = t.transpose(1, 2).contiguous().transpose(1, 2)
    return t.to("cuda", dtype)


def r16(a):
    return a.astype(np.float16).astype(np.float32)


def err(gpu, ref):
    return oracle.normwise_rel_err(gpu.float().cpu().numpy(), ref)


def test_standalone_scan_workload_fp32(cuda):
    """B=1, d_inner=1024, N=16, L=256, FP32; x, delta, z in [B, D, L] and
    B, C in [B, N, L] memory layout; gated output and final state."""
    x, dr, B, C, z, A, Dk = scan_inputs(0, 1, 256, 1024, 16)
    y_ref, h_ref = oracle.scan(x, dr, B, C, A, Dk, z=z)
    y, h = mb.selective_scan(dev(x, time_major=False), dev(dr, time_major=False), dev(A),
                             dev(B, time_major=False), dev(C, time_major=False), D=dev(Dk),
                             z=dev(z, time_major=False), return_final_state=True)
    torch.cuda.synchronize()
    assert err(y, y_ref) < TOL32
    assert err(h, h_ref) < TOL32


def test_matches_reference_selective_scan_cpu(cuda):
    """Ungated scan against the reference's own compiled selective_scan_cpu."""
    if oracle.ref_lib() is None:
        pytest.skip("reference oracle library not built")
    x, dr, B, C, _, A, Dk = scan_inputs(1, 1, 256, 512, 16)
    y_ref, h_ref = oracle.selective_scan(x[0], dr[0], B[0], C[0], A, Dk, use_reference=True)
    y, h = mb.selective_scan(dev(x), dev(dr), dev(A), dev(B), dev(C), D=dev(Dk),
                             return_final_state=True)
    torch.cuda.synchronize()
    assert err(y[0], y_ref) < TOL32
    assert err(h[0], h_ref) < TOL32


GOLD = sorted(f for f in os.listdir(GOLDEN) if f.endswith(".bin"))


@pytest.mark.parametrize("name", GOLD)
def test_golden_vectors(cuda, name):
    """Every golden case (outputs written by the reference itself)."""
    g = load_golden(os.path.join(GOLDEN, name))
    x, dr, B, C = (g[k][None] for k in ("x", "delta", "B", "C"))
    y, h = mb.selective_scan(dev(x), dev(dr), dev(g["A"]), dev(B), dev(C), D=dev(g["Dskip"]),
                             return_final_state=True)
    torch.cuda.synchronize()
    if np.abs(g["y"]).max() == 0:
        assert float(y.abs().max()) == 0.0
        return
    assert err(y[0], g["y"]) < TOL32
    assert err(h[0], g["state"]) < TOL32


def test_small_A_branch_and_softplus_branches(cuda):
    """|A| <= 1e-6 takes Bbar = dt*B (selective_scan_cpu.cpp:28-30); delta
    above 20 bypasses softplus; checked channel by channel."""
    rng = np.random.default_rng(5)
    bsz, L, D, N = 2, 45, 12, 6
    x = rng.uniform(-1, 1, (bsz, L, D)).astype(np.float32)
    dr = rng.normal(-3, 1.5, (bsz, L, D)).astype(np.float32)
    dr[:, ::7, :] = 25.0
    dr[:, 3::11, :] = -40.0
    B = rng.uniform(-1, 1, (bsz, L, N)).astype(np.float32)
    C = rng.uniform(-1, 1, (bsz, L, N)).astype(np.float32)
    avals = np.array([0.0, 1e-6, -1e-6, -1e-7, -0.5, -3.0], np.float32)
    A = np.stack([np.roll(avals, d) for d in range(D)]).astype(np.float32)
    Dk = rng.uniform(-1, 1, D).astype(np.float32)
    y_ref, h_ref = oracle.scan(x, dr, B, C, A, Dk)
    y, h = mb.selective_scan(dev(x), dev(dr), dev(A), dev(B), dev(C), D=dev(Dk),
                             return_final_state=True)
    torch.cuda.synchronize()
    yg = y.cpu().numpy()
    for d in range(D):
        assert oracle.normwise_rel_err(yg[:, :, d], y_ref[:, :, d]) < TOL32, d
    assert err(h, h_ref) < TOL32


@pytest.mark.parametrize("chunk_len", [0, 32, 64, 96, 2048])
def test_chunked_time_carries(cuda, chunk_len):
    """The multi-chunk path (chunk summaries, combine, rescan) equals the
    oracle for any chunk length, with an initial state and dt bias."""
    x, dr, B, C, z, A, Dk = scan_inputs(2, 2, 700, 256, 16)
    rng = np.random.default_rng(7)
    bias = rng.normal(0, 0.5, 256).astype(np.float32)
    h0 = (rng.standard_normal((2, 256, 16)) * 0.3).astype(np.float32)
    y_ref, h_ref = oracle.scan(x, dr, B, C, A, Dk, z=z, dt_bias=bias, h0=h0)
    y, h = mb.selective_scan(dev(x), dev(dr), dev(A), dev(B), dev(C), D=dev(Dk), z=dev(z),
                             dt_bias=dev(bias), initial_state=dev(h0), return_final_state=True,
                             chunk_len=chunk_len)
    torch.cuda.synchronize()
    assert err(y, y_ref) < TOL32
    assert err(h, h_ref) < TOL32


DTYPES = [(torch.float16, torch.float16, torch.float16),
          (torch.float16, torch.float32, torch.float16),
          (torch.float16, torch.float32, torch.float32)]


@pytest.mark.parametrize("dts", DTYPES, ids=["f16-f16-f16", "f16-f32-f16", "f16-f32-f32"])
def test_fp16_inputs(cuda, dts):
    """FP16 x/z (and delta, B/C where chosen), FP32 state and arithmetic; the
    oracle sees the same FP16-rounded values widened to FP32."""
    tx, tdt, tbc = dts
    x, dr, B, C, z, A, Dk = scan_inputs(3, 3, 300, 384, 16)
    x, z = r16(x), r16(z)
    if tdt == torch.float16:
        dr = r16(dr)
    if tbc == torch.float16:
        B, C = r16(B), r16(C)
    y_ref, h_ref = oracle.scan(x, dr, B, C, A, Dk, z=z)
    y, h = mb.selective_scan(dev(x, tx), dev(dr, tdt), dev(A), dev(B, tbc), dev(C, tbc),
                             D=dev(Dk), z=dev(z, tx), return_final_state=True)
    torch.cuda.synchronize()
    assert y.dtype == torch.float16
    assert err(y, y_ref) < TOL16
    assert err(h, h_ref) < 1e-5


@pytest.mark.parametrize("shape", [(1, 1, 8, 16), (3, 37, 13, 5), (2, 129, 130, 8),
                                   (1, 33, 1, 1), (4, 64, 200, 4)])
def test_ragged_shapes(cuda, shape):
    bsz, L, D, N = shape
    x, dr, B, C, z, A, Dk = scan_inputs(4, bsz, L, D, N)
    y_ref, h_ref = oracle.scan(x, dr, B, C, A, Dk, z=z)
    y, h = mb.selective_scan(dev(x), dev(dr), dev(A), dev(B), dev(C), D=dev(Dk), z=dev(z),
                             return_final_state=True)
    torch.cuda.synchronize()
    assert err(y, y_ref) < TOL32
    assert err(h, h_ref) < TOL32


def test_empty_sequence_passes_state_through(cuda):
    x, dr, B, C, z, A, Dk = scan_inputs(5, 2, 0, 64, 16)
    h0 = np.random.default_rng(0).standard_normal((2, 64, 16)).astype(np.float32)
    y, h = mb.selective_scan(dev(x), dev(dr), dev(A), dev(B), dev(C), D=dev(Dk),
                             initial_state=dev(h0), return_final_state=True)
    torch.cuda.synchronize()
    assert y.numel() == 0
    assert np.array_equal(h.cpu().numpy(), h0)


def test_deterministic(cuda):
    x, dr, B, C, z, A, Dk = scan_inputs(6, 2, 500, 512, 16)
    args = (dev(x, torch.float16), dev(dr, torch.float16), dev(A), dev(B, torch.float16),
            dev(C, torch.float16))
    y1 = mb.selective_scan(*args, D=dev(Dk), z=dev(z, torch.float16))
    y2 = mb.selective_scan(*args, D=dev(Dk), z=dev(z, torch.float16))
    torch.cuda.synchronize()
    assert torch.equal(y1, y2)


def test_summary_and_compose_emulate_sequence_sharding(cuda):
    """Sequence-sharded mode on one GPU: G slices, per-slice summaries,
    prefix composition, rescan from the entering state == one long scan."""
    G = 4
    x, dr, B, C, z, A, Dk = scan_inputs(8, 1, 4 * 333, 256, 16)
    y_ref, h_ref = oracle.scan(x, dr, B, C, A, Dk, z=z)
    Ls = 333
    sl = [slice(g * Ls, (g + 1) * Ls) for g in range(G)]
    dA, dDk = dev(A), dev(Dk)
    PH = []
    for s in sl:
        P, H = mb.scan_summary(dev(x[:, s]), dev(dr[:, s]), dA, dev(B[:, s]))
        PH.append(torch.stack([P.reshape(-1), H.reshape(-1)]))
    PH = torch.stack(PH).contiguous()
    ys = []
    for g, s in enumerate(sl):
        h_in = mb.scan_compose_prefix(PH, g).reshape(1, 256, 16)
        y, h = mb.selective_scan(dev(x[:, s]), dev(dr[:, s]), dA, dev(B[:, s]), dev(C[:, s]),
                                 D=dDk, z=dev(z[:, s]), initial_state=h_in, return_final_state=True)
        ys.append(y)
    torch.cuda.synchronize()
    assert err(torch.cat(ys, 1), y_ref) < TOL32
    assert err(h, h_ref) < TOL32


def test_workspace_too_small_is_an_error(cuda):
    import ctypes
    x, dr, B, C, z, A, Dk = scan_inputs(9, 1, 4096, 128, 16)
    tx, tdr, tA, tB, tC = dev(x), dev(dr), dev(A), dev(B), dev(C)
    y = torch.empty_like(tx)
    a = mb._scan_args(tx, tdr, tA, tB, tC, None, None, None, None, y, None, 64)
    need = mb.lib().mamba_selective_scan_workspace(ctypes.byref(a))
    assert need > 0
    assert mb.lib().mamba_selective_scan(ctypes.byref(a), None, 0, None) == -1
    assert "workspace" in mb.last_error()


QUAD_CASES = [
    # (N, delta dtype, B/C dtype, time_major)
    (16, torch.float16, torch.float16, True),    # vector B/C loads
    (16, torch.float32, torch.float32, True),
    (8, torch.float16, torch.float16, True),     # fewer states per lane
    (4, torch.float32, torch.float32, True),     # one state per lane: chunked path instead
    (5, torch.float32, torch.float16, True),     # not 4/8/16 states: chunked path instead
    (16, torch.float16, torch.float16, False),   # [B, D, L] storage: chunked path instead
]


@pytest.mark.parametrize("N,tdt,tbc,time_major", QUAD_CASES)
def test_four_lanes_per_channel_pass(cuda, N, tdt, tbc, time_major):
    """Batch 5 x 1024 channels: fewer 128-channel CTAs than SMs but enough
    32-channel ones, so the single pass with four lanes per channel runs (no
    workspace) where its TMA layout holds; gated output, dt bias, initial and
    final state vs the oracle, over a length that is not a multiple of the
    16-step tiles."""
    bsz, L, D = 5, 301, 1024
    x, dr, B, C, z, A, Dk = scan_inputs(31, bsz, L, D, N)
    rng = np.random.default_rng(8)
    bias = rng.normal(0, 0.5, D).astype(np.float32)
    h0 = (rng.standard_normal((bsz, D, N)) * 0.3).astype(np.float32)
    x, z = r16(x), r16(z)
    if tdt == torch.float16:
        dr = r16(dr)
    if tbc == torch.float16:
        B, C = r16(B), r16(C)
    tx, tdr = dev(x, torch.float16, time_major), dev(dr, tdt, time_major)
    tB, tC, tz = dev(B, tbc, time_major), dev(C, tbc, time_major), dev(z, torch.float16, time_major)
    bc_row_bytes = N * (2 if tbc == torch.float16 else 4)
    quad = N in (8, 16) and time_major and bc_row_bytes % 16 == 0
    assert (mb.scan_workspace_bytes(tx, tdr, dev(A), tB) == 0) == quad
    y_ref, h_ref = oracle.scan(x, dr, B, C, A, Dk, z=z, dt_bias=bias, h0=h0)
    y, h = mb.selective_scan(tx, tdr, dev(A), tB, tC, D=dev(Dk), z=tz, dt_bias=dev(bias),
                             initial_state=dev(h0), return_final_state=True)
    torch.cuda.synchronize()
    assert mb.device_status() == 0
    assert err(y, y_ref) < TOL16
    assert err(h, h_ref) < TOL32


def test_zero_length_and_empty_problems(cuda):
    """L = 0: no output rows, the final state is the initial state (zero when
    none is given).  batch 0 or dim 0: nothing to do, no error."""
    N, D = 16, 64
    A = dev(np.tile(-np.arange(1, N + 1, dtype=np.float32), (D, 1)))
    e = torch.empty((2, 0, D), device="cuda")
    eB = torch.empty((2, 0, N), device="cuda")
    h0 = torch.randn((2, D, N), device="cuda")
    y, h = mb.selective_scan(e, e, A, eB, eB, initial_state=h0, return_final_state=True)
    torch.cuda.synchronize()
    assert y.shape == (2, 0, D)
    assert torch.equal(h, h0)
    _, h = mb.selective_scan(e, e, A, eB, eB, return_final_state=True)
    torch.cuda.synchronize()
    assert torch.count_nonzero(h) == 0
    z0 = torch.empty((0, 5, D), device="cuda")
    y0 = mb.selective_scan(z0, z0, A, torch.empty((0, 5, N), device="cuda"), torch.empty((0, 5, N), device="cuda"))
    torch.cuda.synchronize()
    assert y0.shape == (0, 5, D)
    assert mb.device_status() == 0


def test_summary_on_a_four_lane_shape_sizes_its_own_workspace(cuda):
    """Where the scan itself takes the four-lane single pass (no workspace),
    the slice summary still splits time into chunks: its scratch comes from
    mamba_scan_summary_workspace, and the summary's H (the map applied to a
    zero state) equals the scan's final state from zero."""
    import ctypes
    bsz, L, D, N = 5, 1000, 1024, 16
    x, dr, B, C, z, A, Dk = scan_inputs(41, bsz, L, D, N)
    tx, tdr, tA = dev(r16(x), torch.float16), dev(r16(dr), torch.float16), dev(A)
    tB, tC = dev(r16(B), torch.float16), dev(r16(C), torch.float16)
    assert mb.scan_workspace_bytes(tx, tdr, tA, tB) == 0  # the scan runs four lanes per channel
    a = mb._scan_args(tx, tdr, tA, tB, None, None, None, None, None, None, None, 0)
    assert mb.lib().mamba_scan_summary_workspace(ctypes.byref(a)) > 0
    P, H = mb.scan_summary(tx, tdr, tA, tB)
    _, h = mb.selective_scan(tx, tdr, tA, tB, tC, D=dev(Dk), return_final_state=True)
    torch.cuda.synchronize()
    assert mb.device_status() == 0
    assert err(H, h.cpu().numpy()) < TOL32
