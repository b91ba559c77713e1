"""mamba_selective_scan_noalloc: the selective scan for callers that cannot
allocate device memory or hand the library a workspace.

It must give the same results as mamba_selective_scan (which takes a caller
workspace) through the C ABI, on consecutive calls that reuse the library's
static scratch, and reject sizes whose chunk carries exceed that scratch.
This file is collected last so that a failing run stopping at the first
failure has already run every other test.
"""
import ctypes

import numpy as np
import pytest
import torch

import mamba_b200 as mb

pytestmark = pytest.mark.gpu

STATIC_SCRATCH_BYTES = 32 << 20


def _inputs(seed, bsz, L, D, N, dtype):
    g = torch.Generator(device="cpu")
    g.manual_seed(seed)
    x = torch.randn((bsz, L, D), generator=g).to("cuda", dtype)
    z = torch.randn((bsz, L, D), generator=g).to("cuda", dtype)
    dr = (torch.randn((bsz, L, D), generator=g) * 0.5 - 4.6).to("cuda", dtype)
    B = torch.randn((bsz, L, N), generator=g).to("cuda", dtype)
    C = torch.randn((bsz, L, N), generator=g).to("cuda", dtype)
    A = -torch.arange(1, N + 1, dtype=torch.float32).repeat(D, 1).contiguous().cuda()
    Dk = torch.ones(D, device="cuda")
    bias = (torch.randn(D, generator=g) * 0.3).cuda()
    h0 = (torch.randn((bsz, D, N), generator=g) * 0.1).cuda()
    return x, dr, A, B, C, Dk, z, bias, h0


def _args(x, dr, A, B, C, Dk, z, bias, h0, y, hN):
    return mb._scan_args(x, dr, A, B, C, Dk, z, bias, h0, y, hN, 0)


def _run_pair(inputs):
    """The same scan through both entry points; returns both outputs."""
    L = mb.lib()
    x, dr, A, B, C, Dk, z, bias, h0 = inputs
    y_ws, h_ws = torch.empty_like(x), torch.empty_like(h0)
    y_na, h_na = torch.full_like(x, float("nan")), torch.full_like(h0, float("nan"))
    a_ws = _args(x, dr, A, B, C, Dk, z, bias, h0, y_ws, h_ws)
    a_na = _args(x, dr, A, B, C, Dk, z, bias, h0, y_na, h_na)
    need = L.mamba_selective_scan_workspace(ctypes.byref(a_ws))
    assert 0 < need <= STATIC_SCRATCH_BYTES, need  # the chunked path, which uses scratch
    ws = torch.empty(need, dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    assert L.mamba_selective_scan(ctypes.byref(a_ws), ws.data_ptr(), need, stream) == 0, mb.last_error()
    assert L.mamba_selective_scan_noalloc(ctypes.byref(a_na), stream) == 0, mb.last_error()
    torch.cuda.synchronize()
    assert mb.device_status() == 0
    return (y_ws, h_ws), (y_na, h_na)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16])
def test_noalloc_matches_workspace_entry_point_on_consecutive_calls(dtype):
    # batch 1 x 256 channels is too few CTAs to fill the GPU, so time is split
    # into chunks and the carries go through scratch memory.  Both entry
    # points run the same kernels with the same chunk length, so the results
    # must agree bit for bit (a wrong offset into the scratch array or a carry
    # left over from the previous call would show up here).
    for seed in (11, 12):  # two calls in a row, different data
        (y_ws, h_ws), (y_na, h_na) = _run_pair(_inputs(seed, 1, 4096, 256, 16, dtype))
        assert torch.isfinite(y_na.float()).all()
        assert torch.equal(y_na, y_ws)
        assert torch.equal(h_na, h_ws)


def test_noalloc_rejects_sizes_beyond_its_static_scratch():
    L = mb.lib()
    x, dr, A, B, C, Dk, z, bias, h0 = _inputs(13, 1, 8, 4096, 16, torch.float16)
    y = torch.empty_like(x)
    a = _args(x, dr, A, B, C, Dk, z, bias, None, y, None)
    a.seqlen = 1 << 17  # checked on the host before any device access
    a.chunk_len = 32
    need = L.mamba_selective_scan_workspace(ctypes.byref(a))
    assert need > STATIC_SCRATCH_BYTES
    assert L.mamba_selective_scan_noalloc(ctypes.byref(a), None) == -1
    msg = mb.last_error()
    assert "static maximum" in msg and str(STATIC_SCRATCH_BYTES) in msg
