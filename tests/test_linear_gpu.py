"""GPU parity of mamba_linear (tcgen05 linear layer, split-K with a serial
fix-up) against the oracle's float64 product of the same FP16 operands.

Tolerance: normwise 2e-3 for FP16 output (one rounding), 1e-5 for the FP32
outputs (FP32 accumulation of exact FP16 products)."""
import ctypes

import numpy as np
import pytest
import torch

import mamba_b200 as mb
import oracle

pytestmark = pytest.mark.gpu


def _case(seed, rows, n, k, bias):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((rows, k)).astype(np.float16)
    w = (rng.standard_normal((n, k)) / np.sqrt(k)).astype(np.float16)
    b = rng.standard_normal(n).astype(np.float32) if bias else None
    return x, w, b


def _dev(a):
    return None if a is None else torch.from_numpy(a).cuda()


SHAPES = [
    (5, 96, 64),          # one K block, few rows
    (256, 10240, 2560),   # decode in_proj (batch 256, d_model 2560)
    (256, 192, 5120),     # decode x_proj: narrow output, long K, many splits
    (256, 5120, 160),     # decode dt_proj: K tail (2.5 blocks)
    (300, 200, 136),      # two row tiles (the second ragged), ragged columns
    (1, 8, 8),            # smallest legal sizes
    (8192, 1024, 128),    # above 512 rows: the CTA-pair kernel
    (4096, 8192, 2048),   # in_proj-like: 512 tiles over the persistent CTA pairs
    (1000, 160, 4096),    # x_proj-like: one 160-column tile, ragged last row block
    (777, 4096, 128),     # dt_proj-like: two K blocks per tile
    (520, 200, 136),      # ragged columns (tile 208) and K tail, 8 rows in the last block
]


@pytest.mark.parametrize("rows,n,k", SHAPES)
@pytest.mark.parametrize("bias", [False, True])
def test_linear_fp16_out(cuda, rows, n, k, bias):
    x, w, b = _case(rows + n + k, rows, n, k, bias)
    y = mb.linear(_dev(x), _dev(w), bias=_dev(b), mode=0)
    torch.cuda.synchronize()
    assert mb.device_status() == 0
    ref = oracle.linear(x, w, b)
    assert oracle.normwise_rel_err(y.float().cpu().numpy(), ref) < 2e-3


@pytest.mark.parametrize("rows,n,k", [(256, 2560, 5120), (37, 64, 1024), (300, 200, 136), (600, 2048, 4096),
                                      (1030, 96, 200)])
def test_linear_fp32_accumulate_and_store(cuda, rows, n, k):
    """mode 1 adds into an FP32 buffer (the residual stream of out_proj);
    mode 2 overwrites it."""
    x, w, b = _case(7 * rows + n, rows, n, k, True)
    resid = np.random.default_rng(1).standard_normal((rows, n)).astype(np.float32)
    y = torch.from_numpy(resid.copy()).cuda()
    mb.linear(_dev(x), _dev(w), bias=_dev(b), y=y, mode=1)
    y2 = torch.full((rows, n), float("nan"), device="cuda")
    mb.linear(_dev(x), _dev(w), bias=_dev(b), y=y2, mode=2)
    torch.cuda.synchronize()
    ref = oracle.linear(x, w, b)
    assert oracle.normwise_rel_err(y.cpu().numpy(), ref + resid) < 1e-5
    assert oracle.normwise_rel_err(y2.cpu().numpy(), ref) < 1e-5


def test_linear_split_k_is_deterministic_and_reusable(cuda):
    """The split-K fix-up sums partials in split order: repeated calls on one
    workspace give identical bits, and the workspace stays usable."""
    rows, n, k = 256, 192, 5120
    L = mb.lib()
    need = L.mamba_linear_workspace(rows, n, k)
    assert need > 0  # this shape splits K
    ws = torch.zeros(need, dtype=torch.uint8, device="cuda")
    x, w, _ = _case(3, rows, n, k, False)
    tx, tw = _dev(x), _dev(w)
    outs = [mb.linear(tx, tw, workspace=ws, mode=2) for _ in range(4)]
    torch.cuda.synchronize()
    for o in outs[1:]:
        assert torch.equal(o, outs[0])
    assert oracle.normwise_rel_err(outs[0].cpu().numpy(), oracle.linear(x, w)) < 1e-5
    wide = torch.zeros((rows, k + 64), dtype=torch.float16, device="cuda")
    wide[:, :k] = tx
    o = mb.linear(wide[:, :k], tw, workspace=ws, mode=2)
    torch.cuda.synchronize()
    assert torch.equal(o, outs[0])


def test_linear_rejects_bad_arguments(cuda):
    L = mb.lib()
    x = torch.zeros((4, 12), dtype=torch.float16, device="cuda")
    w = torch.zeros((8, 12), dtype=torch.float16, device="cuda")
    y = torch.zeros((4, 8), dtype=torch.float16, device="cuda")
    assert L.mamba_linear(x.data_ptr(), 12, w.data_ptr(), None, y.data_ptr(), 8, 4, 8, 12, 0, None, 0, None) == -1
    assert "multiples of 8" in mb.last_error()
    x = torch.zeros((256, 5120), dtype=torch.float16, device="cuda")
    w = torch.zeros((192, 5120), dtype=torch.float16, device="cuda")
    y = torch.zeros((256, 192), dtype=torch.float16, device="cuda")
    assert L.mamba_linear(x.data_ptr(), 5120, w.data_ptr(), None, y.data_ptr(), 192, 256, 192, 5120, 0, None, 0,
                          None) == -1
    assert "workspace" in mb.last_error()
    assert L.mamba_linear(x.data_ptr(), 5120, w.data_ptr(), None, y.data_ptr(), 192, 256, 192, 5120, 3, None, 0,
                          None) == -1
    assert "mode" in mb.last_error()


def test_pair_gemm_strided_operand_and_determinism(cuda):
    """Above 512 rows (the CTA-pair kernel): x read with a row stride wider
    than K (dt_proj reads the first dt_rank columns of x_proj's output), and
    repeated calls give identical bits."""
    rows, n, k, ld = 2304, 4096, 128, 160
    rng = np.random.default_rng(12)
    full = rng.standard_normal((rows, ld)).astype(np.float16)
    w = (rng.standard_normal((n, k)) / np.sqrt(k)).astype(np.float16)
    tx, tw = _dev(full), _dev(w)
    ys = [mb.linear(tx[:, :k], tw, mode=0) for _ in range(3)]
    torch.cuda.synchronize()
    assert mb.device_status() == 0
    for y in ys[1:]:
        assert torch.equal(y, ys[0])
    ref = oracle.linear(full[:, :k], w)
    assert oracle.normwise_rel_err(ys[0].float().cpu().numpy(), ref) < 2e-3
