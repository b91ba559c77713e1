"""GPU tests of the sequence-sharded scan as one library call,
mamba_selective_scan_seqpar (summary -> ncclAllGather -> compose -> rescan
on the caller's stream).

* world 1 (one GPU, an NCCL communicator of one rank): bit for bit the
  plain scan with the same initial state.
* world 2 (run when two GPUs are visible; one process per GPU, NCCL):
  the concatenated slices equal the one-GPU scan of the whole sequence
  within the tolerance of each input type (the chunking differs), and the
  last rank's final state equals the whole sequence's.
"""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import mamba_b200 as mb

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs(seed, L, D, N, dt):
    g = torch.Generator(device="cpu")
    g.manual_seed(seed)
    x = torch.randn((1, L, D), generator=g).to(dt)
    z = torch.randn((1, L, D), generator=g).to(dt)
    dr = (torch.randn((1, L, D), generator=g) * 0.5 - 4.6).float()
    B = torch.randn((1, L, N), generator=g).to(dt)
    C = torch.randn((1, L, N), generator=g).to(dt)
    A = -torch.arange(1, N + 1, dtype=torch.float32).repeat(D, 1).contiguous()
    Dk = torch.ones(D)
    bias = torch.randn(D, generator=g) * 0.3
    h0 = torch.randn((1, D, N), generator=g) * 0.2
    return x, dr, A, B, C, Dk, z, bias, h0


@pytest.mark.parametrize("dt", [torch.float32, torch.float16])
def test_seqpar_world1_equals_plain_scan(cuda, dt):
    from mamba_b200.seqpar import NcclComm, sequence_parallel_scan_nccl
    dist.init_process_group("gloo", init_method="tcp://127.0.0.1:%d" % _port(), rank=0, world_size=1,
                            timeout=datetime.timedelta(seconds=60))
    try:
        comm = NcclComm()
        try:
            x, dr, A, B, C, Dk, z, bias, h0 = (t.cuda() for t in _inputs(3, 3000, 512, 16, dt))
            y1, h1 = sequence_parallel_scan_nccl(comm, x, dr, A, B, C, D=Dk, z=z, dt_bias=bias, h0=h0)
            y2, h2 = mb.selective_scan(x, dr, A, B, C, D=Dk, z=z, dt_bias=bias, initial_state=h0,
                                       return_final_state=True)
            torch.cuda.synchronize()
            assert mb.device_status() == 0
            assert torch.equal(y1, y2)
            assert torch.equal(h1, h2)
        finally:
            comm.close()
    finally:
        dist.destroy_process_group()


def _worker(rank, world, port, dt_name, q):
    import sys
    for p in (ROOT, os.path.join(ROOT, "mamba-metal_b200")):
        sys.path.insert(0, p)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method="tcp://127.0.0.1:%d" % port, rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        import mamba_b200 as mbw
        from mamba_b200.seqpar import NcclComm, sequence_parallel_scan_nccl
        dt = getattr(torch, dt_name)
        L = 4096 * world
        x, dr, A, B, C, Dk, z, bias, h0 = (t.cuda() for t in _inputs(4, L, 512, 16, dt))
        Ls = L // world
        s = slice(rank * Ls, (rank + 1) * Ls)
        comm = NcclComm()
        try:
            y, h = sequence_parallel_scan_nccl(comm, x[:, s].contiguous(), dr[:, s].contiguous(), A,
                                               B[:, s].contiguous(), C[:, s].contiguous(), D=Dk,
                                               z=z[:, s].contiguous(), dt_bias=bias, h0=h0)
            torch.cuda.synchronize()
            status = mbw.device_status()
        finally:
            comm.close()
        if rank == 0 or rank == world - 1:
            yf, hf = mbw.selective_scan(x, dr, A, B, C, D=Dk, z=z, dt_bias=bias, initial_state=h0,
                                        return_final_state=True)
            torch.cuda.synchronize()
            ref_y = yf[:, s].float()
            ey = float((y.float() - ref_y).abs().max() / ref_y.abs().max())
            eh = float((h - hf).abs().max() / hf.abs().max())
            q.put((rank, status, ey, eh))
        else:
            q.put((rank, status, 0.0, 0.0))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two visible GPUs")
@pytest.mark.parametrize("dt_name,tol", [("float32", 1e-5), ("float16", 2e-3)])
def test_seqpar_two_gpus_matches_one_gpu_scan(cuda, dt_name, tol):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, dt_name, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, status, ey, eh in res:
        assert status == 0
        assert ey < tol, (rank, ey)
        if rank == world - 1:
            assert eh < 1e-5, eh
