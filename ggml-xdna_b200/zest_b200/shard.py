"""Partitioning a layer's MUL_MATs across GPUs.

N-sharding: each rank converts and multiplies its slab of weight rows
(output columns); an all-gather of the slab outputs over NCCL (gloo on CPU)
rebuilds ggml's row-major [M][N] on every rank.

K-sharding (the tensor-parallel block): a projection whose input is already
split by columns across the ranks (the FFN's down projection after N-sharded
gate/up) multiplies each rank's column slab of the input by the same column
slab of the weight; the ranks' partial products add up to the full product
in one all-reduce, of [M][N] instead of the gather of every projection.

The reference runs on one NPU and has no counterpart; these are the
partitionings its GEMM admits.
"""
from __future__ import annotations

GRANULE = 128  # rows per shard granule: whole GEMM tile rows, and 16-row pack units


def shard_rows(N: int, world: int, rank: int, granule: int = GRANULE) -> tuple[int, int]:
    """This rank's slab [row0, row0 + n) of N weight rows, in whole granules
    spread as evenly as they go (the last slab takes the ragged end)."""
    g = (N + granule - 1) // granule
    lo = g * rank // world * granule
    hi = min(N, g * (rank + 1) // world * granule)
    return lo, max(0, hi - lo)


def slab_width(N: int, world: int, granule: int = GRANULE) -> int:
    """The widest slab: every rank's output is padded to it for the gather."""
    return max(shard_rows(N, world, r, granule)[1] for r in range(world))


def gather_slabs(slab_out, full_out, world: int, N: int, group=None, granule: int = GRANULE, wire=None):
    """slab_out: this rank's [M][slab_width] output (columns past its slab
    unused); full_out: [M][N]. All-gathers the slabs and writes them into
    their columns of full_out. wire: the dtype the slabs cross the link in
    (default: their own). torch.bfloat16 halves an f32 gather and loses
    nothing when the values are bf16-rounded already, as the GEMM's default
    output is (GGML_XDNA_OUT16=1). Collective: every rank calls it, in order."""
    import torch
    import torch.distributed as dist

    M, w = slab_out.shape
    send = slab_out.contiguous() if wire is None else slab_out.to(wire).contiguous()
    flat = torch.empty((world * M, w), dtype=send.dtype, device=slab_out.device)
    dist.all_gather_into_tensor(flat, send, group=group)
    gathered = flat.view(world, M, w)
    for r in range(world):
        lo, n = shard_rows(N, world, r, granule)
        if n:
            full_out[:, lo:lo + n].copy_(gathered[r, :, :n])
    return full_out


K_GRANULE = 64  # columns per K-shard granule: the GEMM's k-block and the pack's tile


def shard_cols(K: int, world: int, rank: int, granule: int = K_GRANULE) -> tuple[int, int]:
    """This rank's slab [k0, k0 + k) of K reduction columns, in whole
    granules spread as evenly as they go."""
    return shard_rows(K, world, rank, granule)


def all_reduce_rows(partial, row0: int, rows: int, group=None, async_op: bool = True):
    """Sums rows [row0, row0 + rows) of every rank's partial [M][N] product
    in place (NCCL, or gloo on CPU). Collective: every rank calls it, in
    order; returns the work handle when async_op."""
    import torch.distributed as dist
    return dist.all_reduce(partial[row0:row0 + rows], op=dist.ReduceOp.SUM, group=group, async_op=async_op)


def any_rank(flag: bool, group=None) -> bool:
    """Whether `flag` holds on any rank of the group (this rank's own flag
    when no process group is up): ranks take an error path together, so none
    is left waiting in a collective that a failing rank skipped. Collective:
    every rank calls it, in order."""
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()):
        return bool(flag)
    dev = "cuda" if dist.get_backend(group) == "nccl" else "cpu"
    t = torch.tensor([1 if flag else 0], dtype=torch.int32, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return bool(t.item())
