"""GPU: mamba_scan_launch_static_workspace, the scan for callers that cannot allocate.

Some hosts cannot give the library scratch memory (their memory planner owns
every device buffer, or their launch path must not call cudaMalloc). The
static-workspace entry point takes no workspace argument and uses an array
compiled into the library instead. These tests call it through the C ABI and
check that, on shapes that need scratch, it produces the same outputs as
mamba_scan_launch given a caller-allocated workspace, for two calls in a row
(the second call reuses the array the first one left behind).

This file is collected last so that a run stopping at the first failure has
run every other test first; it needs nothing from them.
"""

import numpy as np
import pytest
import torch

import scan_cases as sc
from mamba_onnx import cuda
from oracle import oracle

pytestmark = pytest.mark.gpu

# Tolerance of the other parity tests at these distributions.
RTOL = ATOL = 1e-5


def _args(u, delta, A, B, C, D, z, out):
    p = lambda t: None if t is None else t.data_ptr()  # noqa: E731
    batch, dim, seqlen = u.shape
    return cuda.ScanArgs(p(u), p(delta), p(A), p(B), p(C), p(D), p(z), None, None, p(out), None,
                         batch, dim, seqlen, A.shape[1])


def _inputs(op, batch, dim, seqlen, seed):
    fused = oracle.OPS[op][1]
    arrs = sc.config_inputs(batch, dim, seqlen, fused, seed=seed,
                            exact_dt_per_element=not fused)[:7]
    return [None if a is None else torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in arrs]


# Shapes that split sequences into chunks, so the scan needs scratch.
CASES = [
    ("SelectiveScanExact", 1, 2048, 4096),
    ("SelectiveScanFused", 1, 1536, 2048),
    ("SelectiveScanFusedExact", 2, 256, 1000),
]


@pytest.mark.parametrize("op,batch,dim,seqlen", CASES)
def test_static_workspace_matches_caller_workspace(op, batch, dim, seqlen):
    assert 0 < cuda.workspace_size(op, batch, dim, seqlen) <= 8 << 20
    u, delta, A, B, C, D, z = _inputs(op, batch, dim, seqlen, seed=21)
    stream = torch.cuda.current_stream().cuda_stream
    expected = cuda.selective_scan(op, u, delta, A, B, C, D, z)  # torch-allocated workspace
    for call in range(2):
        out = torch.full_like(u, float("nan"))
        rc = cuda.launch_static_workspace(cuda.OPS[op], _args(u, delta, A, B, C, D, z, out),
                                          stream)
        assert rc == 0, cuda.library().mamba_scan_last_error().decode()
        torch.cuda.synchronize()
        assert torch.isfinite(out).all(), f"call {call}"
        torch.testing.assert_close(out, expected, rtol=RTOL, atol=ATOL)


def test_static_workspace_after_a_different_shape():
    """A call does not depend on what the previous call left in the array:
    two shapes that both need scratch, back to back, each match the
    caller-workspace path."""
    assert cuda.workspace_size("SelectiveScanExact", 1, 1024, 8192) > 0
    assert cuda.workspace_size("SelectiveScan", 1, 512, 3000) > 0
    stream = torch.cuda.current_stream().cuda_stream
    first = _inputs("SelectiveScanExact", 1, 1024, 8192, seed=5)
    out1 = torch.empty_like(first[0])
    assert cuda.launch_static_workspace(1, _args(*first, out1), stream) == 0
    second = _inputs("SelectiveScan", 1, 512, 3000, seed=6)
    out2 = torch.empty_like(second[0])
    assert cuda.launch_static_workspace(0, _args(*second, out2), stream) == 0
    torch.cuda.synchronize()
    torch.testing.assert_close(out1, cuda.selective_scan("SelectiveScanExact", *first[:6]),
                               rtol=RTOL, atol=ATOL)
    torch.testing.assert_close(out2, cuda.selective_scan("SelectiveScan", *second[:6]),
                               rtol=RTOL, atol=ATOL)


def test_built_in_workspace_covers_every_shape_on_this_gpu():
    """The planner keeps split work within one wave of CTAs, so the scratch any
    shape needs is bounded by (CTAs per wave) x 4 KiB; on a B200 that is under
    the 8 MiB built in, and no shape is turned away."""
    worst = 0
    for op in cuda.OPS:
        for batch, dim in [(1, 32), (1, 2048), (2, 8000), (8, 5120), (9, 5120), (64, 5120)]:
            for seqlen in [65, 1000, 4096, 16384, 1 << 20]:
                worst = max(worst, cuda.workspace_size(op, batch, dim, seqlen))
    assert 0 < worst <= 8 << 20


def test_static_workspace_rejects_shapes_that_need_more():
    """Shapes needing more scratch than is built in get MAMBA_SCAN_ERR_WORKSPACE
    and nothing is launched (reachable only on GPUs with more SMs than a B200)."""
    shapes = [(op, b, d, l) for op in cuda.OPS for b, d in [(1, 32), (1, 4096), (3, 9000)]
              for l in [1 << 16, 1 << 20]]
    big = [s for s in shapes if cuda.workspace_size(*s) > 8 << 20]
    if not big:
        pytest.skip("no shape needs more than the built-in 8 MiB on this GPU")
    op, batch, dim, seqlen = big[0]
    # NULL tensors: were the size check ever to pass such a shape, the scan's
    # own NULL check would still refuse it before any launch
    args = cuda.ScanArgs(None, None, None, None, None, None, None, None, None, None, None,
                         batch, dim, seqlen, 16)
    assert cuda.launch_static_workspace(cuda.OPS[op], args, None) == 3
    assert "built-in workspace" in cuda.library().mamba_scan_last_error().decode()
