"""CPU (gloo, world size 2 and 3): the sharding plan and the output gather.

Each rank computes its shard's output with the oracle (the kernels need a GPU;
what is under test here is the host-side split and the collective), gathers to
rank 0, and rank 0 compares with the unsharded oracle result.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import scan_cases as sc
from mamba_onnx.distributed import shard_plan


def test_plan_covers_rows_exactly_once():
    for batch, dim, world in [(64, 5120, 8), (8, 5120, 8), (3, 100, 8), (10, 7, 4), (1, 9, 2)]:
        plans = [shard_plan(batch, dim, world, r) for r in range(world)]
        n = batch if plans[0].axis == 0 else dim
        covered = []
        for p in plans:
            covered.extend(range(p.start, p.stop))
        assert covered == list(range(n))
        assert max(p.sizes) - min(p.sizes) <= 1
    assert shard_plan(64, 5120, 8, 3).axis == 0
    assert shard_plan(4, 5120, 8, 3).axis == 1
    with pytest.raises(ValueError):
        shard_plan(1, 1, 2, 0)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, batch, dim, op, q, into_out=False):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from mamba_onnx.distributed import gather_output
        from oracle import oracle

        fused = oracle.OPS[op][1]
        u, delta, A, B, C, D, z = sc.reference_test_inputs(batch, dim, 24, fused, seed=13)
        plan = shard_plan(batch, dim, world, rank)
        t = lambda a: None if a is None else torch.from_numpy(a)  # noqa: E731
        lu, ld, lA, lB, lC, lD, lz, _ = plan.slice_inputs(t(u), t(delta), t(A), t(B), t(C),
                                                          t(D), t(z))
        n = lambda x: None if x is None else x.numpy()  # noqa: E731
        local = oracle.scan_f64(op, n(lu), n(ld), n(lA), n(lB), n(lC), n(lD), n(lz))
        out = torch.empty(batch, dim, 24, dtype=torch.float64) if into_out and rank == 0 else None
        full = gather_output(torch.from_numpy(local), plan, out=out)
        if out is not None:
            assert full is out
        if rank == 0:
            ref = oracle.scan_f64(op, u, delta, A, B, C, D, z)
            q.put(("ok", float(np.abs(full.numpy() - ref).max()), tuple(full.shape)))
    except Exception as e:  # noqa: BLE001
        q.put(("error", repr(e), None))
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,batch,dim,op,into_out", [
    (2, 4, 40, "SelectiveScanFused", False),   # batch split
    (2, 4, 40, "SelectiveScanFused", True),    # even batch split, straight into `out`
    (2, 1, 37, "SelectiveScanExact", False),   # d_inner split (batch < world), uneven
    (3, 5, 16, "SelectiveScan", False),        # uneven batch split
    (3, 5, 16, "SelectiveScan", True),         # uneven: padded gather, concatenated into `out`
])
def test_sharded_scan_gathers_to_rank0(world, batch, dim, op, into_out):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, batch, dim, op, q, into_out))
             for r in range(world)]
    for p in procs:
        p.start()
    status, err, shape = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
    assert status == "ok", err
    assert shape == (batch, dim, 24)
    assert err == 0.0
    assert all(p.exitcode == 0 for p in procs)
