"""Sequence-sharded selective scan across ranks (one process per GPU).

Rank r holds time slice r of every sequence.  The scan recurrence
h_t = a_t * h_{t-1} + b_t is an affine map per (b, d, n); a slice applies the
composed map h -> P*h + H to its incoming state (the carry monoid of
Sources/CPURef/selective_scan_cpu.hpp:12-19, applied at GPU granularity as
Sources/Kernels/prefix_scan.metal:19-40 intended for tiles).  So:

  1. each rank computes its slice summary (P, H)         [batch, dim, N] FP32
  2. one all-gather of the summaries (the only exchange; 2*batch*dim*N*4 B)
  3. each rank composes the summaries of ranks < r into its entering state
  4. each rank rescans its slice from that state and writes its y

The final state of the whole sequence is the final state of the last rank.
Every rank runs the same collective in the same order.

Two entry points:
  sequence_parallel_scan_nccl  the library call mamba_selective_scan_seqpar:
                               all four steps on the GPU stream, the exchange
                               an ncclAllGather on a communicator the library
                               creates (NcclComm).  The product path.
  sequence_parallel_scan       the same steps orchestrated here over any
                               torch.distributed group; `ops` supplies the
                               compute steps (LibOps: the CUDA kernels; the
                               CPU tests pass the oracle), so the plumbing is
                               testable on gloo ranks without a GPU.
"""
import ctypes

import torch
import torch.distributed as dist

from . import _check, _ptr, _scan_args, _stream, lib, scan_compose_prefix, scan_summary, selective_scan


class NcclComm:
    """An NCCL communicator over the ranks of a torch.distributed group,
    created by the library (mamba_nccl_comm_create) on the current device.
    Rank 0 makes the 128-byte id; the group broadcasts it."""

    def __init__(self, group=None):
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        uid = torch.zeros(128, dtype=torch.uint8)
        if self.rank == 0:
            _check(lib().mamba_nccl_unique_id(uid.data_ptr()), "mamba_nccl_unique_id")
        dev = "cuda" if dist.get_backend(group) == "nccl" else "cpu"
        t = uid.to(dev)
        dist.broadcast(t, src=dist.get_global_rank(group, 0) if group is not None else 0, group=group)
        uid = t.cpu().contiguous()
        c = ctypes.c_void_p()
        _check(lib().mamba_nccl_comm_create(uid.data_ptr(), self.world, self.rank, ctypes.byref(c)),
               "mamba_nccl_comm_create")
        self.handle = c.value

    def close(self):
        if getattr(self, "handle", None):
            lib().mamba_nccl_comm_destroy(self.handle)
            self.handle = None


def sequence_parallel_scan_nccl(comm, x, delta, A, B, C, D=None, z=None, dt_bias=None, h0=None, y=None,
                                workspace=None, stream=None):
    """This rank's slice through mamba_selective_scan_seqpar; returns
    (y_local, final_state_of_slice).  Shapes as sequence_parallel_scan."""
    bsz, L, dim = x.shape
    N = A.shape[1]
    if y is None:
        y = torch.empty((bsz, L, dim), dtype=x.dtype, device=x.device)
    hN = torch.empty((bsz, dim, N), dtype=torch.float32, device=x.device)
    a = _scan_args(x, delta, A, B, C, D, z, dt_bias, h0, y, hN, 0)
    need = lib().mamba_selective_scan_seqpar_workspace(ctypes.byref(a), comm.world)
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(max(need, 256), dtype=torch.uint8, device=x.device)
    _check(lib().mamba_selective_scan_seqpar(ctypes.byref(a), comm.handle, comm.world, comm.rank, _ptr(workspace),
                                             workspace.numel(), _stream(stream)), "mamba_selective_scan_seqpar")
    return y, hN


class LibOps:
    """The product implementation: CUDA kernels via the C ABI."""

    @staticmethod
    def summary(x, delta, A, B, dt_bias, chunk_len=0):
        return scan_summary(x, delta, A, B, dt_bias=dt_bias, chunk_len=chunk_len)

    @staticmethod
    def compose(PH, rank, h0):
        return scan_compose_prefix(PH, rank, h0=h0)

    @staticmethod
    def scan(x, delta, A, B, C, D, z, dt_bias, h_in, chunk_len=0):
        return selective_scan(x, delta, A, B, C, D=D, z=z, dt_bias=dt_bias, initial_state=h_in,
                              return_final_state=True, chunk_len=chunk_len)


def sequence_parallel_scan(x, delta, A, B, C, D=None, z=None, dt_bias=None, h0=None, group=None,
                           ops=LibOps, chunk_len=0):
    """Scan this rank's time slice; returns (y_local, final_state_of_slice).

    x, delta, z: [batch, L_local, dim]; B, C: [batch, L_local, N];
    h0: FP32 [batch, dim, N] state before rank 0's slice (or None = zeros)."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    bsz, _, dim = x.shape
    N = A.shape[1]
    P, H = ops.summary(x, delta, A, B, dt_bias, chunk_len)
    local = torch.stack([P.reshape(-1), H.reshape(-1)]).contiguous()
    gathered = [torch.empty_like(local) for _ in range(world)]
    dist.all_gather(gathered, local, group=group)
    PH = torch.stack(gathered).contiguous()
    h_in = ops.compose(PH, rank, h0).reshape(bsz, dim, N)
    return ops.scan(x, delta, A, B, C, D, z, dt_bias, h_in, chunk_len)
