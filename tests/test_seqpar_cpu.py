"""Sequence-sharded scan logic on CPU ranks (gloo, world sizes 2 and 3).

mamba_b200.seqpar.sequence_parallel_scan is run unchanged; its three compute
steps come from the oracle here (the GPU run uses the CUDA kernels), so this
tests the partition / all-gather / prefix-composition / rescan plumbing
without a GPU.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


class OracleOps:
    @staticmethod
    def summary(x, delta, A, B, dt_bias, chunk_len=0):
        import oracle
        P, H = oracle.scan_chunk_summary(x.numpy(), delta.numpy(), B.numpy(), A.numpy(),
                                         dt_bias=None if dt_bias is None else dt_bias.numpy())
        return torch.from_numpy(P), torch.from_numpy(H)

    @staticmethod
    def compose(PH, rank, h0):
        h = torch.zeros(PH.shape[2]) if h0 is None else h0.reshape(-1).clone()
        for g in range(rank):
            h = PH[g, 0] * h + PH[g, 1]
        return h

    @staticmethod
    def scan(x, delta, A, B, C, D, z, dt_bias, h_in, chunk_len=0):
        import oracle
        y, h = oracle.scan(x.numpy(), delta.numpy(), B.numpy(), C.numpy(), A.numpy(),
                           D.numpy(), z=z.numpy(), dt_bias=dt_bias.numpy(),
                           h0=h_in.numpy(), nthreads=1)
        return torch.from_numpy(y), torch.from_numpy(h)


def _inputs(L, D=16, N=8):
    rng = np.random.default_rng(21)
    x = rng.standard_normal((1, L, D)).astype(np.float32)
    dr = rng.normal(-4.6, 0.5, (1, L, D)).astype(np.float32)
    B = rng.standard_normal((1, L, N)).astype(np.float32)
    C = rng.standard_normal((1, L, N)).astype(np.float32)
    z = rng.standard_normal((1, L, D)).astype(np.float32)
    A = np.tile(-np.arange(1, N + 1, dtype=np.float32), (D, 1))
    Dk = np.ones(D, np.float32)
    bias = rng.normal(0, 0.3, D).astype(np.float32)
    h0 = (rng.standard_normal((1, D, N)) * 0.2).astype(np.float32)
    return x, dr, B, C, z, A, Dk, bias, h0


def _worker(rank, world, port, L, q):
    import sys
    for p in (ROOT, os.path.join(ROOT, "mamba-metal_b200")):
        sys.path.insert(0, p)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        from mamba_b200.seqpar import sequence_parallel_scan
        x, dr, B, C, z, A, Dk, bias, h0 = _inputs(L)
        bounds = np.linspace(0, L, world + 1).astype(int)
        s = slice(bounds[rank], bounds[rank + 1])
        t = torch.from_numpy
        y, h = sequence_parallel_scan(t(np.ascontiguousarray(x[:, s])),
                                      t(np.ascontiguousarray(dr[:, s])), t(A),
                                      t(np.ascontiguousarray(B[:, s])),
                                      t(np.ascontiguousarray(C[:, s])), D=t(Dk),
                                      z=t(np.ascontiguousarray(z[:, s])), dt_bias=t(bias),
                                      h0=t(h0), ops=OracleOps)
        q.put((rank, y.numpy(), h.numpy()))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world,L", [(2, 64), (3, 100)])
def test_sequence_parallel_scan_gloo(world, L):
    import sys
    sys.path.insert(0, ROOT)
    import oracle
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, L, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        r, y, h = q.get(timeout=120)
        results[r] = (y, h)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    x, dr, B, C, z, A, Dk, bias, h0 = _inputs(L)
    y_ref, h_ref = oracle.scan(x, dr, B, C, A, Dk, z=z, dt_bias=bias, h0=h0)
    y = np.concatenate([results[r][0] for r in range(world)], axis=1)
    assert oracle.normwise_rel_err(y, y_ref) < 1e-5
    assert oracle.normwise_rel_err(results[world - 1][1], h_ref) < 1e-5


def _failing_worker(rank, world, port, q):
    """Rank 1 leaves before the carry exchange (between steps, nothing in
    flight); rank 0 must come back with an error from its collective within
    the short process-group timeout instead of waiting forever."""
    import sys
    for p in (ROOT, os.path.join(ROOT, "mamba-metal_b200")):
        sys.path.insert(0, p)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    import time
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    def report(msg):
        q.put((rank, msg))
        q.close()
        q.join_thread()  # the message is out before the process ends

    if rank == 1:
        report("left")
        os._exit(0)  # leaves without taking part in the exchange
    from mamba_b200.seqpar import sequence_parallel_scan
    x, dr, B, C, z, A, Dk, bias, h0 = _inputs(32)
    t = torch.from_numpy
    t0 = time.monotonic()
    try:
        sequence_parallel_scan(t(np.ascontiguousarray(x[:, :16])), t(np.ascontiguousarray(dr[:, :16])), t(A),
                               t(np.ascontiguousarray(B[:, :16])), t(np.ascontiguousarray(C[:, :16])), D=t(Dk),
                               z=t(np.ascontiguousarray(z[:, :16])), dt_bias=t(bias), h0=t(h0), ops=OracleOps)
        report("returned")
    except Exception as e:  # the collective reports the missing peer
        report("error after %.1f s: %s" % (time.monotonic() - t0, type(e).__name__))
    os._exit(0)


def test_missing_rank_is_reported_not_hung():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=60) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
    assert got[1] == "left"
    assert got[0].startswith("error after"), got[0]
