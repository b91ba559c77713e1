"""GPU parity at the shapes of the workloads the benchmarks are quoted on.

* Stack forward (48 layers, d_model 2048, d_inner 4096, d_state 16, d_conv
  4, dt_rank 128, batch 64, L 4096, FP16 activations): the full-size forward
  runs on the GPU; because every op is causal in time, the first 256 tokens
  of rows 0 and 63 are checked against the CPU block reference on the same
  weights (read back with mamba_save_weights).  At full length the batch-64
  rows are checked against the same rows run on their own (other kernel
  paths), i.e. batch-shard invariance.
* Decode (64 layers, d_model 2560, d_inner 5120, dt_rank 160, batch 256):
  16 steps from zero state at batch 256; rows 0 and 255 against the CPU
  decode reference.
* Long scan (batch 1, d_inner 2048, d_state 16, L 131072; x, B, C, z FP16,
  delta FP32): the whole sequence against the oracle.

Tolerance (normwise max|gpu - ref| / max|ref|): 2e-3 for FP16-input paths,
1e-5 for the FP32 state of the scan.
"""
import numpy as np
import pytest
import torch

import mamba_b200 as mb
import oracle
from oracle import block_ref

pytestmark = pytest.mark.gpu

TOL16 = 2e-3


def _seeded_randn(shape, seed):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    return torch.randn(shape, device="cuda", dtype=torch.float32, generator=g)


def test_stack_workload_prefix_and_shard_invariance(cuda):
    cfg = mb.MambaConfig(2048, 16, 4, 2, 48, mb.F16)
    m = mb.Model(2048, 16, 4, 2, 48, mb.F16)
    m.init_random(1234)
    layers = mb.weights_from_blob(cfg, m.save_weights())
    x = _seeded_randn((64, 4096, 2048), 1000)
    out = torch.empty_like(x)
    m.forward_device(x.data_ptr(), out.data_ptr(), 64, 4096)
    torch.cuda.synchronize()
    assert mb.device_status() == 0
    assert bool(torch.isfinite(out).all())
    rows = [0, 63]
    h = x[rows, :256].cpu().numpy()
    ref = block_ref.model_forward(h, layers, cfg, block_ref.F16)
    got = out[rows, :256].cpu().numpy()
    e = oracle.normwise_rel_err(got - h, ref - h)
    print("stack prefix parity (2 rows x 256 tokens, 48 layers): %.3e" % e)
    assert e < TOL16
    # Full length: rows 0..7 alone (the per-rank batch at 8 GPUs) and row 0
    # alone (batch 1) against the same rows of the batch-64 forward.
    for lo, hi in ((0, 8), (0, 1)):
        xs = x[lo:hi].contiguous()
        os_ = torch.empty_like(xs)
        m.forward_device(xs.data_ptr(), os_.data_ptr(), hi - lo, 4096)
        torch.cuda.synchronize()
        d = (os_ - out[lo:hi]).abs().max().item() / (out[lo:hi] - xs).abs().max().item()
        print("batch %d vs batch 64 rows, full length: %.3e" % (hi - lo, d))
        assert d < TOL16


def test_decode_workload_rows(cuda):
    cfg = mb.MambaConfig(2560, 16, 4, 2, 64, mb.F16)
    m = mb.Model(2560, 16, 4, 2, 64, mb.F16)
    m.init_random(4321)
    blob = m.save_weights()
    layers = mb.weights_from_blob(cfg, blob)
    st = m.create_state(256)
    T = 16
    toks = np.random.default_rng(500).standard_normal((T, 256, 2560)).astype(np.float32)
    outs = np.stack([st.step(toks[t]) for t in range(T)], 1)  # [256, T, 2560]
    assert mb.device_status() == 0
    rows = [0, 255]
    h = np.ascontiguousarray(toks[:, rows].transpose(1, 0, 2))
    state = block_ref.new_state(cfg, 2)
    ref = block_ref.model_decode(h, layers, cfg, block_ref.F16, state=state)
    e = oracle.normwise_rel_err(outs[rows] - h, ref - h)
    print("decode parity (2 rows x %d steps, 64 layers): %.3e" % (T, e))
    assert e < TOL16
    # the SSM state of the last layer after T steps, rows 0 and 255
    _, ssm = st.tensors(63)
    es = oracle.normwise_rel_err(ssm[rows].cpu().numpy(), state[1][63])
    print("decode state parity (layer 63): %.3e" % es)
    assert es < TOL16


def test_long_scan_workload_full_sequence(cuda):
    L, D, N = 131072, 2048, 16
    rng = np.random.default_rng(77)
    x = rng.standard_normal((1, L, D), dtype=np.float32).astype(np.float16)
    z = rng.standard_normal((1, L, D), dtype=np.float32).astype(np.float16)
    dr = (rng.standard_normal((1, L, D), dtype=np.float32) * np.float32(0.5) - np.float32(4.6))
    B = rng.standard_normal((1, L, N), dtype=np.float32).astype(np.float16)
    C = rng.standard_normal((1, L, N), dtype=np.float32).astype(np.float16)
    A = np.tile(-np.arange(1, N + 1, dtype=np.float32), (D, 1))
    Dk = np.ones(D, np.float32)
    t = lambda a: torch.from_numpy(a).cuda()  # noqa: E731
    y, h = mb.selective_scan(t(x), t(dr), t(A), t(B), t(C), D=t(Dk), z=t(z), return_final_state=True)
    torch.cuda.synchronize()
    assert mb.device_status() == 0
    # channel-major copies so each oracle thread walks one channel contiguously
    cm = lambda a: np.ascontiguousarray(a.astype(np.float32).transpose(0, 2, 1)).transpose(0, 2, 1)  # noqa: E731
    y_ref, h_ref = oracle.scan(cm(x), cm(dr), B.astype(np.float32), C.astype(np.float32), A, Dk, z=cm(z))
    ey = oracle.normwise_rel_err(y.float().cpu().numpy(), y_ref)
    eh = oracle.normwise_rel_err(h.cpu().numpy(), h_ref)
    print("long scan parity: y %.3e, final state %.3e" % (ey, eh))
    assert ey < TOL16
    assert eh < 1e-5
