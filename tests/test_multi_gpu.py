"""GPU, 2 ranks (NCCL): sharded scan + output gather equals the one-GPU result.

Skipped unless at least two CUDA devices are visible. Each rank scans its
batch (or d_inner) shard with the CUDA kernels; rank 0 gathers the shards
and compares them with the unsharded scan it runs itself.
"""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs(batch, dim, seqlen, device):
    g = torch.Generator(device=device).manual_seed(77)
    kw = dict(device=device, generator=g)
    u = torch.randn(batch, dim, seqlen, **kw)
    z = torch.randn(batch, dim, seqlen, **kw)
    delta = torch.randn(batch, dim, seqlen, **kw) * 0.5 - 3.0
    A = -torch.rand(dim, 16, **kw) - 0.5
    B = torch.randn(batch, seqlen, 16, **kw)
    C = torch.randn(batch, seqlen, 16, **kw)
    D = torch.randn(dim, **kw)
    return u, delta, A, B, C, D, z


def _worker(rank, world, port, batch, dim, seqlen, chunked, q):
    import torch.distributed as dist
    from datetime import timedelta

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=timedelta(seconds=60))
    try:
        from mamba_onnx import cuda
        from mamba_onnx.distributed import gather_output, shard_plan

        inputs = _inputs(batch, dim, seqlen, dev)  # every rank builds the same global tensors
        plan = shard_plan(batch, dim, world, rank)
        local = plan.slice_inputs(*inputs)
        out_local = cuda.selective_scan("SelectiveScanFused", *local[:7], delta_bias=local[7],
                                        chunked=chunked)
        full = gather_output(out_local, plan)
        if rank == 0:
            ref = cuda.selective_scan("SelectiveScanFused", *inputs, chunked=chunked)
            q.put(("ok", float((full - ref).abs().max().item()), tuple(full.shape)))
        dist.barrier()
    except Exception as e:  # noqa: BLE001
        q.put(("error", repr(e), None))
        raise
    finally:
        dist.destroy_process_group()


# The unchunked case (batch 16: 8 per rank) runs every row as one pass on both
# sides, so the bits agree whatever sequence split either shape would plan.
@pytest.mark.parametrize("batch,dim,seqlen,chunked", [(4, 256, 512, True), (1, 300, 256, True),
                                                      (16, 512, 1024, False)])
def test_sharded_scan_gathered_on_rank0(batch, dim, seqlen, chunked):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, batch, dim, seqlen, chunked, q))
             for r in range(2)]
    for p in procs:
        p.start()
    status, err, shape = q.get(timeout=180)
    for p in procs:
        p.join(timeout=60)
    assert status == "ok", err
    assert shape == (batch, dim, seqlen)
    assert err == 0.0  # the same rows through the same kernel: identical bits
    assert all(p.exitcode == 0 for p in procs)
