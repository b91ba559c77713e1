"""GPU parity of mamba_in_proj_conv: in_proj with the causal conv + SiLU
fused into the tensor-core GEMM's epilogue.

Against the oracle (float64 product rounded to FP16, then the conv
restatement on those values): normwise 2e-3.  Against the unfused library
path (mamba_linear, then mamba_causal_conv1d): bit for bit, since both run
the same MMAs and the same conv arithmetic on the same FP16 values."""
import numpy as np
import pytest
import torch

import mamba_b200 as mb
import oracle

pytestmark = pytest.mark.gpu


def _case(seed, batch, L, dm, D):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((batch * L, dm)).astype(np.float16)
    w = (rng.standard_normal((2 * D, dm)) / np.sqrt(dm)).astype(np.float16)
    cw = rng.uniform(-0.5, 0.5, (D, 4)).astype(np.float32)
    cb = rng.uniform(-0.5, 0.5, D).astype(np.float32)
    return x, w, cw, cb


# (batch, L, d_model, d_inner): sequence starts inside row tiles; a ragged
# last tile; short sequences (many starts per tile); one-token sequences.
# Every case has more than 512 rows, where mamba_linear runs the same
# CTA-pair GEMM (below that it splits K, which changes summation order).
CASES = [(3, 700, 256, 512), (20, 37, 128, 256), (600, 1, 64, 256), (1, 4096, 512, 1024), (3, 250, 256, 256)]


@pytest.mark.parametrize("batch,L,dm,D", CASES)
def test_in_proj_conv_matches_oracle_and_unfused_path(cuda, batch, L, dm, D):
    x, w, cw, cb = _case(batch * L + D, batch, L, dm, D)
    tx, tw, tcw, tcb = (torch.from_numpy(a).cuda() for a in (x, w, cw, cb))
    xz_full = torch.full((batch * L, 2 * D), float("nan"), dtype=torch.float16, device="cuda")
    u, z = mb.in_proj_conv(tx, tw, tcw, tcb, batch, L, z=xz_full[:, D:])
    # unfused: GEMM, then conv on the x half
    xz = mb.linear(tx, tw, mode=0)
    u2 = mb.causal_conv1d(xz[:, :D].view(batch, L, D), tcw, tcb, silu=True)
    torch.cuda.synchronize()
    assert mb.device_status() == 0
    assert torch.equal(z, xz[:, D:])
    assert torch.equal(u, u2.view(batch * L, D))
    assert torch.isnan(xz_full[:, :D]).all()  # the x half is never written
    xz_ref = oracle.linear(x, w).astype(np.float32).astype(np.float16).astype(np.float32)
    u_ref = oracle.causal_conv1d(xz_ref[:, :D].reshape(batch, L, D), cw, cb, silu=True).reshape(batch * L, D)
    assert oracle.normwise_rel_err(z.float().cpu().numpy(), xz_ref[:, D:]) < 2e-3
    assert oracle.normwise_rel_err(u.float().cpu().numpy(), u_ref) < 2e-3


def test_in_proj_conv_rejects_unsupported_shapes(cuda):
    x, w, cw, cb = _case(1, 2, 64, 64, 128)  # d_inner 128: not a multiple of 256
    tx, tw, tcw, tcb = (torch.from_numpy(a).cuda() for a in (x, w, cw, cb))
    with pytest.raises(mb.MambaError, match="multiple of 256"):
        mb.in_proj_conv(tx, tw, tcw, tcb, 2, 64)
