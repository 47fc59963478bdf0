"""Selective scan across the GPUs of one node: shard by batch, gather the output.

The reference parallelises only over (batch, d_inner) rows with OpenMP
(src/native/cpp/selective_scan.cc:232-234); rows are independent and there is
no reduction. Across GPUs the same property means each rank scans its own
slice of rows and no data moves until the caller wants the whole output on
one rank:

* shard_plan() splits the batch axis across ranks (d_inner when the batch is
  smaller than the number of ranks, in which case each rank takes matching
  A[d] and D[d] rows and the full B/C);
* scan_shard() runs the CUDA kernel on a rank's slice;
* gather_output() is the one collective: the shards go to rank 0 (NCCL on
  GPUs, gloo on CPU tensors), padded to the largest shard so a single gather
  call carries uneven splits.

One process per GPU; the process group is set up by the caller (e.g. under
torch.distributed.run).
"""
from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class ShardPlan:
    axis: int        # 0: batch, 1: d_inner
    start: int
    stop: int
    sizes: tuple     # slice length of every rank, in rank order

    @property
    def length(self) -> int:
        return self.stop - self.start

    def slice_inputs(self, u, delta, A, B, C, D, z=None, delta_bias=None):
        """This rank's slice of global inputs (views; contiguous copies on d_inner)."""
        s = slice(self.start, self.stop)
        if self.axis == 0:
            return (u[s], delta[s], A, B[s], C[s], D, None if z is None else z[s], delta_bias)
        c = lambda t: t[:, s].contiguous()  # noqa: E731
        return (c(u), c(delta), A[s].contiguous(), B, C, D[s].contiguous(),
                None if z is None else c(z),
                None if delta_bias is None else delta_bias[s].contiguous())


def _split(n: int, parts: int):
    base, extra = divmod(n, parts)
    return tuple(base + (1 if r < extra else 0) for r in range(parts))


def shard_plan(batch: int, dim: int, world: int, rank: int) -> ShardPlan:
    """Batch shards when batch >= world, else d_inner shards; sizes differ by at most 1."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of {world}")
    axis = 0 if batch >= world else 1
    n = batch if axis == 0 else dim
    if n < world:
        raise ValueError(f"cannot split batch {batch} x d_inner {dim} over {world} ranks")
    sizes = _split(n, world)
    start = sum(sizes[:rank])
    return ShardPlan(axis, start, start + sizes[rank], sizes)


def scan_shard(op: str, plan: ShardPlan, u, delta, A, B, C, D, z=None, delta_bias=None,
               **kw):
    """Run the CUDA scan on this rank's slice (the arguments are already sliced)."""
    from . import cuda

    return cuda.selective_scan(op, u, delta, A, B, C, D, z, delta_bias=delta_bias, **kw)


def gather_output(out_local, plan: ShardPlan, group=None, dst: int = 0, out=None):
    """Collect every rank's output shard on rank `dst`; returns the full tensor there.

    With a batch split of equal shards and `out` (the full [batch, dim, seqlen]
    tensor, on `dst` only) the shards land directly in their slices of `out`.
    Otherwise shards are padded to the largest shard along the split axis so
    one gather carries uneven splits, and the result is concatenated. Other
    ranks return None.
    """
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    if plan.axis == 0 and len(set(plan.sizes)) == 1 and (out is not None or rank != dst):
        n = plan.sizes[0]
        bufs = [out.narrow(0, r * n, n) for r in range(world)] if rank == dst else None
        dist.gather(out_local.contiguous(), bufs, dst=dst, group=group)
        return out if rank == dst else None
    biggest = max(plan.sizes)
    if plan.length < biggest:
        pad_shape = list(out_local.shape)
        pad_shape[plan.axis] = biggest - plan.length
        out_local = torch.cat([out_local, out_local.new_zeros(pad_shape)], dim=plan.axis)
    out_local = out_local.contiguous()
    bufs = [torch.empty_like(out_local) for _ in range(world)] if rank == dst else None
    dist.gather(out_local, bufs, dst=dst, group=group)
    if rank != dst:
        return None
    parts = [b.narrow(plan.axis, 0, n) for b, n in zip(bufs, plan.sizes)]
    if out is not None:
        return torch.cat(parts, dim=plan.axis, out=out)
    return torch.cat(parts, dim=plan.axis)
