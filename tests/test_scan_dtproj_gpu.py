"""GPU parity of mamba_selective_scan_dtproj: the selective scan with the
layer's dt_proj (delta = dt_r @ w_dt^T) computed inside it on the tensor
cores, against the separate path (mamba_linear, mode 0, then
mamba_selective_scan) on the same FP16 operands and against the oracle.

Both round delta to FP16; the tensor-core products may round a delta value
differently in rare cases, so the comparison is normwise: 2e-3 on y (the
FP16-input bound), 1e-4 on the FP32 final state."""
import numpy as np
import pytest
import torch

import mamba_b200 as mb
import oracle
from oracle import block_ref

pytestmark = pytest.mark.gpu


def _rel(a, b):
    a, b = a.double(), b.double()
    return float((a - b).abs().max() / b.abs().max())


# (batch, L, dim, dt_rank): the layer shapes of the stack workload's per-rank
# batches need one 128-channel CTA per SM; ragged last tile; dt_rank of one
# partial 64-wide K box, of two boxes, and of two full boxes.
CASES = [(3, 300, 6400, 128), (10, 129, 2048, 48), (2, 200, 9600, 80)]


@pytest.mark.parametrize("bsz,L,D,R", CASES)
def test_dtproj_scan_matches_separate_gemm_and_scan(cuda, bsz, L, D, R):
    N = 16
    XD = R + 2 * N
    rng = np.random.default_rng(bsz * L + R)
    f16 = lambda a: torch.from_numpy(np.asarray(a, np.float32)).to("cuda", torch.float16)  # noqa: E731
    x = f16(rng.standard_normal((bsz, L, D)))
    z = f16(rng.standard_normal((bsz, L, D)))
    xdbc = f16(rng.standard_normal((bsz, L, XD)) * np.concatenate([np.full(R, 0.3), np.ones(2 * N)]))
    w_dt = f16(rng.normal(0, 0.4, (D, R)))
    A = torch.from_numpy(np.tile(-np.arange(1, N + 1, dtype=np.float32), (D, 1))).cuda()
    Dk = torch.ones(D, device="cuda")
    bias = torch.from_numpy(rng.normal(-4.6, 0.5, D).astype(np.float32)).cuda()
    h0 = torch.from_numpy((rng.standard_normal((bsz, D, N)) * 0.2).astype(np.float32)).cuda()
    dt_r, B, C = xdbc[..., :R], xdbc[..., R:R + N], xdbc[..., R + N:]
    y1, h1 = mb.selective_scan_dtproj(x, dt_r, w_dt, A, B, C, D=Dk, z=z, dt_bias=bias, initial_state=h0,
                                      return_final_state=True)
    draw = mb.linear(xdbc.reshape(bsz * L, XD)[:, :R], w_dt, mode=0).view(bsz, L, D)
    y2, h2 = mb.selective_scan(x, draw, A, B, C, D=Dk, z=z, dt_bias=bias, initial_state=h0,
                               return_final_state=True)
    torch.cuda.synchronize()
    assert mb.device_status() == 0
    assert _rel(y1, y2) < 2e-3
    assert _rel(h1, h2) < 1e-4
    # and the oracle on the FP16 delta the separate GEMM produced
    c = lambda t: t.float().cpu().numpy()  # noqa: E731
    y_ref, h_ref = oracle.scan(c(x), c(draw), c(B).copy(), c(C).copy(), c(A), c(Dk), z=c(z), dt_bias=c(bias),
                               h0=c(h0))
    assert oracle.normwise_rel_err(c(y1), y_ref) < 2e-3
    assert oracle.normwise_rel_err(c(h1), h_ref) < 1e-4


def test_dtproj_scan_rejects_unsupported_shapes(cuda):
    x = torch.zeros((1, 32, 256), dtype=torch.float16, device="cuda")  # 2 CTAs: fewer than the SMs
    xdbc = torch.zeros((1, 32, 64 + 32), dtype=torch.float16, device="cuda")
    w = torch.zeros((256, 64), dtype=torch.float16, device="cuda")
    A = -torch.ones((256, 16), device="cuda")
    with pytest.raises(mb.MambaError, match="SM count"):
        mb.selective_scan_dtproj(x, xdbc[..., :64], w, A, xdbc[..., 64:80], xdbc[..., 80:], z=x)


def test_model_forward_with_dt_fused_scan(cuda, monkeypatch):
    """A layer shape where the model can fold dt_proj into the scan (d_inner
    2048 x batch 10 = 160 channel CTAs), with MAMBA_DT_FUSE=1: the forward
    matches the forward with the separate GEMM (the default) and the CPU
    block reference."""
    rng = np.random.default_rng(120)
    cfg = mb.MambaConfig(1024, 16, 4, 2, 1, mb.F16)
    layers = [mb.random_layer_weights(cfg, rng)]
    blob = mb.make_weight_blob(cfg, layers)
    monkeypatch.setenv("MAMBA_DT_FUSE", "0")
    sep = mb.Model(1024, 16, 4, 2, 1, mb.F16)
    monkeypatch.setenv("MAMBA_DT_FUSE", "1")
    fused = mb.Model(1024, 16, 4, 2, 1, mb.F16)
    sep.load_weights(blob)
    fused.load_weights(blob)
    h = rng.standard_normal((10, 96, 1024)).astype(np.float32)
    fused.profile(True)
    a = fused.forward(h)
    prof = fused.profile_read()
    fused.profile(False)
    assert prof["dt_proj"][1] == 0  # no separate dt_proj ran
    b = sep.forward(h)
    assert oracle.normwise_rel_err(a - h, b - h) < 2e-3
    ref = block_ref.model_forward(h, layers, cfg, block_ref.F16)
    assert oracle.normwise_rel_err(a - h, ref - h) < 2e-3
