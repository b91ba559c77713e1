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
Every rank runs the same collective in the same order.  `ops` supplies the
three compute steps: LibOps runs them through libmamba_b200 on the GPU;
tests may pass other implementations of the same interface.
"""
import torch
import torch.distributed as dist

from . import scan_compose_prefix, scan_summary, selective_scan


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
