"""GPU parity of conv, conv step, SSM step and RMSNorm kernels (through the
C ABI) against the oracle restatements."""
import numpy as np
import pytest
import torch

import mamba_b200 as mb
import oracle
from test_scan_gpu import TOL16, TOL32, dev, err, r16, scan_inputs

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("K", [2, 3, 4])
@pytest.mark.parametrize("dtype", [torch.float32, torch.float16])
def test_causal_conv1d(cuda, K, dtype):
    """x read as the first half of an interleaved [b, L, 2D] buffer (the
    in_proj output layout), SiLU fused."""
    rng = np.random.default_rng(K)
    bsz, L, D = 3, 150, 200
    xz = rng.standard_normal((bsz, L, 2 * D)).astype(np.float32)
    if dtype == torch.float16:
        xz = r16(xz)
    w = rng.uniform(-0.5, 0.5, (D, K)).astype(np.float32)
    b = rng.uniform(-0.5, 0.5, D).astype(np.float32)
    y_ref = oracle.causal_conv1d(xz[..., :D], w, b, silu=True)
    txz = dev(xz, dtype)
    y = mb.causal_conv1d(txz[..., :D], dev(w), dev(b), silu=True)
    torch.cuda.synchronize()
    assert err(y, y_ref) < (TOL32 if dtype == torch.float32 else TOL16)


def test_causal_conv1d_time_contiguous_no_bias(cuda):
    rng = np.random.default_rng(11)
    x = rng.standard_normal((2, 77, 33)).astype(np.float32)
    w = rng.uniform(-0.5, 0.5, (33, 4)).astype(np.float32)
    y_ref = oracle.causal_conv1d(x, w, None, silu=False)
    y = mb.causal_conv1d(dev(x, time_major=False), dev(w), None, silu=False)
    torch.cuda.synchronize()
    assert err(y, y_ref) < TOL32


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16])
def test_conv_step_sequence(cuda, dtype):
    rng = np.random.default_rng(12)
    bsz, L, D, K = 4, 10, 96, 4
    x = rng.standard_normal((bsz, L, D)).astype(np.float32)
    if dtype == torch.float16:
        x = r16(x)
    w = rng.uniform(-0.5, 0.5, (D, K)).astype(np.float32)
    b = rng.uniform(-0.5, 0.5, D).astype(np.float32)
    st_ref = np.zeros((bsz, D, K - 1), np.float32)
    st = torch.zeros((bsz, D, K - 1), device="cuda")
    tx, tw, tb = dev(x, dtype), dev(w), dev(b)
    for t in range(L):
        yr = oracle.causal_conv1d_step(x[:, t], w, b, st_ref, silu=True)
        y = mb.causal_conv1d_step(tx[:, t], tw, tb, st, silu=True)
        torch.cuda.synchronize()
        assert err(y, yr) < (TOL32 if dtype == torch.float32 else TOL16)
    assert np.array_equal(st.cpu().numpy(), st_ref)


@pytest.mark.parametrize("dtype,D,N", [(torch.float32, 160, 16), (torch.float16, 160, 16),
                                       (torch.float16, 100, 16), (torch.float16, 70, 8),
                                       (torch.float16, 33, 5)])
def test_ssm_step_sequence(cuda, dtype, D, N):
    """T decode updates equal the oracle step (and so the scan); FP16 runs
    the four-threads-per-channel kernel, including channel counts that leave
    part of a warp without a channel."""
    bsz, L = 5, 12
    x, dr, B, C, z, A, Dk = scan_inputs(13, bsz, L, D, N)
    bias = np.random.default_rng(0).normal(0, 0.5, D).astype(np.float32)
    if dtype == torch.float16:
        x, dr, B, C, z = map(r16, (x, dr, B, C, z))
    st_ref = np.zeros((bsz, D, N), np.float32)
    st = torch.zeros((bsz, D, N), device="cuda")
    tA, tD, tb = dev(A), dev(Dk), dev(bias)
    tx, tdr, tB, tC, tz = (dev(a, dtype) for a in (x, dr, B, C, z))
    for t in range(L):
        yr = oracle.ssm_step(x[:, t], dr[:, t], B[:, t], C[:, t], A, Dk, st_ref, z=z[:, t],
                             dt_bias=bias)
        y = mb.ssm_step(tx[:, t], tdr[:, t], tA, tB[:, t], tC[:, t], st, D=tD, z=tz[:, t],
                        dt_bias=tb)
        torch.cuda.synchronize()
        assert err(y, yr) < (TOL32 if dtype == torch.float32 else TOL16)
    assert err(st, st_ref) < TOL32


def test_fp16_decode_states_match_scan_bitwise(cuda):
    """The FP16 decode kernel applies the scan's per-state operations, so T
    steps leave exactly the scan's final state."""
    bsz, L, D, N = 3, 30, 256, 16
    x, dr, B, C, z, A, Dk = scan_inputs(15, bsz, L, D, N)
    h16 = lambda a: dev(a, torch.float16)  # noqa: E731
    tx, tdr, tB, tC, tz = h16(x), h16(dr), h16(B), h16(C), h16(z)
    tA, tD = dev(A), dev(Dk)
    y_scan, h_scan = mb.selective_scan(tx, tdr, tA, tB, tC, D=tD, z=tz, return_final_state=True)
    st = torch.zeros((bsz, D, N), device="cuda")
    ys = [mb.ssm_step(tx[:, t], tdr[:, t], tA, tB[:, t], tC[:, t], st, D=tD, z=tz[:, t]) for t in range(L)]
    torch.cuda.synchronize()
    assert torch.equal(st, h_scan)
    assert err(torch.stack(ys, 1), y_scan.float().cpu().numpy()) < 2e-3


def test_ssm_step_matches_scan_final_state(cuda):
    bsz, L, D, N = 2, 40, 64, 8
    x, dr, B, C, z, A, Dk = scan_inputs(14, bsz, L, D, N)
    tx, tdr, tA, tB, tC, tz, tD = dev(x), dev(dr), dev(A), dev(B), dev(C), dev(z), dev(Dk)
    y_scan, h_scan = mb.selective_scan(tx, tdr, tA, tB, tC, D=tD, z=tz, return_final_state=True)
    st = torch.zeros((bsz, D, N), device="cuda")
    ys = [mb.ssm_step(tx[:, t], tdr[:, t], tA, tB[:, t], tC[:, t], st, D=tD, z=tz[:, t])
          for t in range(L)]
    torch.cuda.synchronize()
    # same arithmetic sequence in both kernels
    assert torch.allclose(torch.stack(ys, 1), y_scan, rtol=1e-6, atol=1e-6)
    assert torch.allclose(st, h_scan, rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("cols", [768, 2048, 2560, 100, 4100])
@pytest.mark.parametrize("out", [torch.float32, torch.float16])
def test_rmsnorm(cuda, cols, out):
    rng = np.random.default_rng(cols)
    rows = 257
    x = (rng.standard_normal((rows, cols)) * 3).astype(np.float32)
    w = rng.uniform(0.5, 1.5, cols).astype(np.float32)
    y_ref = oracle.rmsnorm(x, w, 1e-5)
    y = mb.rmsnorm(dev(x), dev(w), 1e-5, out_dtype=out)
    torch.cuda.synchronize()
    assert err(y, y_ref) < (1e-6 if out == torch.float32 else 1e-3)


def test_rmsnorm_fp16_input_no_weight(cuda):
    rng = np.random.default_rng(3)
    x = r16(rng.standard_normal((64, 512)).astype(np.float32))
    y_ref = oracle.rmsnorm(x, None, 1e-5)
    y = mb.rmsnorm(dev(x, torch.float16), None, 1e-5)
    torch.cuda.synchronize()
    assert err(y, y_ref) < 1e-3


@pytest.mark.parametrize("nt,width", [(1, 1), (5, 300), (64, 4096), (0, 7), (129, 33)])
def test_propagate_tile_carries_bitwise(cuda, nt, width):
    """Exclusive carry propagation equals the oracle bit for bit (same
    separately rounded products and sums)."""
    rng = np.random.default_rng(nt * 1000 + width)
    car = np.stack([rng.uniform(0.5, 1.0, (nt, width)), rng.standard_normal((nt, width))], -1)
    car = car.astype(np.float32)
    ex_ref, tot_ref = oracle.propagate_tile_carries(car)
    c = torch.from_numpy(car).cuda()
    tot = mb.propagate_tile_carries(c)
    torch.cuda.synchronize()
    assert np.array_equal(c.cpu().numpy(), ex_ref)
    assert np.array_equal(tot.cpu().numpy(), tot_ref)


def test_propagate_tile_carries_rejects_misaligned(cuda):
    c = torch.zeros(2 * 4 * 2 + 1, device="cuda")
    L = mb.lib()
    assert L.mamba_propagate_tile_carries(c.data_ptr() + 4, 2, 4, None, None) == -1
    assert "aligned" in mb.last_error()


@pytest.mark.parametrize("n", [1, 7, 4096, 100003])
@pytest.mark.parametrize("dtype,tol", [(torch.float32, 1e-6), (torch.float16, 1e-3)])
def test_gated_silu_mul(cuda, n, dtype, tol):
    rng = np.random.default_rng(n)
    g = (rng.standard_normal(n) * 4).astype(np.float32)
    u = rng.standard_normal(n).astype(np.float32)
    if dtype == torch.float16:
        g, u = r16(g), r16(u)
    want = oracle.gated_silu_mul(g, u)
    tg, tu = dev(g, dtype), dev(u, dtype)
    out = mb.gated_silu_mul(tg, tu)
    # unaligned views take the scalar path
    out_off = mb.gated_silu_mul(tg[1:], tu[1:]) if n > 1 else None
    torch.cuda.synchronize()
    assert err(out, want) < tol
    if out_off is not None:
        assert err(out_off, want[1:]) < tol


@pytest.mark.parametrize("misalign", [False, True])
def test_ssm_step_multirow_kernel(cuda, misalign):
    """Large enough to take the several-rows-per-thread FP16 decode kernel:
    2048 channels x batch 19 (the last row group holds 3 rows).  With A and
    the state 4 bytes off a 16-byte boundary the kernel uses scalar accesses
    and must give the same results."""
    bsz, L, D, N = 19, 3, 2048, 16
    x, dr, B, C, z, A, Dk = scan_inputs(21, bsz, L, D, N)
    x, dr, B, C, z = map(r16, (x, dr, B, C, z))
    bias = np.random.default_rng(1).normal(0, 0.5, D).astype(np.float32)
    st_ref = np.zeros((bsz, D, N), np.float32)
    tA_buf = torch.zeros(D * N + 1, device="cuda")
    st_buf = torch.zeros(bsz * D * N + 1, device="cuda")
    off = 1 if misalign else 0
    tA = tA_buf[off:off + D * N].view(D, N)
    tA.copy_(torch.from_numpy(A))
    st = st_buf[off:off + bsz * D * N].view(bsz, D, N)
    tD, tb = dev(Dk), dev(bias)
    tx, tdr, tB, tC, tz = (dev(a, torch.float16) for a in (x, dr, B, C, z))
    for t in range(L):
        yr = oracle.ssm_step(x[:, t], dr[:, t], B[:, t], C[:, t], A, Dk, st_ref, z=z[:, t], dt_bias=bias)
        y = mb.ssm_step(tx[:, t], tdr[:, t], tA, tB[:, t], tC[:, t], st, D=tD, z=tz[:, t], dt_bias=tb)
        torch.cuda.synchronize()
        assert err(y, yr) < TOL16
    assert err(st, st_ref) < TOL32


@pytest.mark.parametrize("bsz", [40, 42])
def test_ssm_step_bulk_copy_kernel(cuda, bsz):
    """Enough 32-channel x 4-row blocks to take the bulk-copy FP16 decode
    kernel (3072 channels; batch 42 leaves a last row group of 2): the
    outputs match the oracle step, and T steps leave exactly the scan's final
    state (the per-state operations are the scan's)."""
    L, D, N = 6, 3072, 16
    x, dr, B, C, z, A, Dk = scan_inputs(23, bsz, L, D, N)
    x, dr, B, C, z = map(r16, (x, dr, B, C, z))
    bias = np.random.default_rng(2).normal(0, 0.5, D).astype(np.float32)
    st_ref = np.zeros((bsz, D, N), np.float32)
    st = torch.zeros((bsz, D, N), device="cuda")
    tA, tD, tb = dev(A), dev(Dk), dev(bias)
    tx, tdr, tB, tC, tz = (dev(a, torch.float16) for a in (x, dr, B, C, z))
    ys = []
    for t in range(L):
        yr = oracle.ssm_step(x[:, t], dr[:, t], B[:, t], C[:, t], A, Dk, st_ref, z=z[:, t], dt_bias=bias)
        y = mb.ssm_step(tx[:, t], tdr[:, t], tA, tB[:, t], tC[:, t], st, D=tD, z=tz[:, t], dt_bias=tb)
        torch.cuda.synchronize()
        assert err(y, yr) < TOL16
        ys.append(y)
    assert mb.device_status() == 0
    assert err(st, st_ref) < TOL32
    y_scan, h_scan = mb.selective_scan(tx, tdr, tA, tB, tC, D=tD, z=tz, dt_bias=tb, return_final_state=True)
    torch.cuda.synchronize()
    assert torch.equal(st, h_scan)
    # y sums C*h in another order (four lanes' partial sums), so not bitwise
    assert err(torch.stack(ys, 1), y_scan.float().cpu().numpy()) < TOL16
