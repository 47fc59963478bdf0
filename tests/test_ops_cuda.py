"""GPU: the reference's test suite (tests/test_ops.py), run on the CUDA ops.

Same cases, same inputs (recipes of tests/test_ops.py, pinned by the golden
vectors), same tolerances; the op is driven the way ONNX Runtime's CUDA EP
drives it (through the library's RegisterCustomOps / KernelComputeV2 entries,
fake_ort/ort_shim.py). Each case is checked against
* out_torch32 — the reference test oracle (reference_selective_scan),
* the float64 restatement of the oracle, and
* out_cpp — the reference C++ plugin (tests/test_ops.py:280-294's
  cross-backend agreement, with this backend in place of zig).
"""
import numpy as np
import torch
import pytest

import golden_cases as gc
import mamba_onnx
import scan_cases as sc
from fake_ort import ort_shim
from mamba_onnx import cuda
from oracle import oracle

pytestmark = pytest.mark.gpu


def _run_onnx(op_name, use_fused, feed, use_v2=True):
    """tests/test_ops.py:136-144 with the CUDA execution provider."""
    opts = ort_shim.SessionOptions()
    mamba_onnx.register_custom_ops(opts, backend="cuda")
    model = ort_shim.make_model(op_name, use_fused, with_delta_bias="delta_bias" in feed)
    with ort_shim.InferenceSession(model, opts, providers=["CUDAExecutionProvider"],
                                   use_v2=use_v2) as sess:
        return sess.run(None, feed)[0]


def _feed(u, delta, A, B, C, D, z):
    """tests/test_ops.py:125-133."""
    feed = {"u": u, "delta": delta, "A": A, "B": B, "C": C, "D": D}
    if z is not None:
        feed["z"] = z
    return feed


def _check(case_name):
    case = gc.load(case_name)
    inputs = case.inputs()
    fused = oracle.OPS[case.op][1]
    out = _run_onnx(case.op, fused, _feed(*inputs))
    assert np.isfinite(out).all()
    got = case.select(out)
    # the reference test's own comparison (vs reference_selective_scan in fp32)
    np.testing.assert_allclose(got, case.out_torch32, rtol=case.tol, atol=case.tol)
    # float64 ground truth, all rows
    np.testing.assert_allclose(out, oracle.scan_f64(case.op, *inputs), rtol=case.tol,
                               atol=case.tol)
    return case, got


@pytest.mark.parametrize("op_name", [op for op, _, _ in sc.ALL_OPS])
def test_selective_scan(op_name):
    """tests/test_ops.py:156-171: every op, B=1, D=64, L=32, rtol=atol=1e-4."""
    _check(f"core_{op_name}")


@pytest.mark.parametrize("sid", sc.REFERENCE_SHAPE_IDS)
def test_shapes(sid):
    """tests/test_ops.py:178-203: SelectiveScan over four shapes, 1e-4."""
    _check(f"shape_{sid}")


@pytest.mark.parametrize("regime", sc.EDGE_REGIMES)
def test_numerical_edge_cases(regime):
    """tests/test_ops.py:210-248: zero input, A=-10, delta=2 (growing state), 1e-3."""
    _check(f"edge_{regime}")


def test_numerical_edge_cases_exact():
    """tests/test_ops.py:251-273: SelectiveScanExact with A=-5, 1e-3."""
    _check("edge_exact")


@pytest.mark.parametrize("op_name", [op for op, _, _ in sc.ALL_OPS])
def test_cross_backend_agreement(op_name):
    """tests/test_ops.py:280-294 (B=2, D=128, L=64): CUDA vs the reference C++, 1e-4."""
    case, got = _check(f"cross_{op_name}")
    np.testing.assert_allclose(got, case.out_cpp, rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("op_name", [op for op, _, _ in sc.ALL_OPS])
def test_config_1x1536x512(op_name):
    """The 1x1536x512 benchmark configuration (seed 0): vs float64 at every element.

    Every variant: normwise relative error <= 1e-5 against float64; elementwise
    allclose 1e-4 (Exact) or 1e-3 (approximate variants). Against the reference
    C++ output (sampled rows): normwise relative error <= 1e-3 — the C++ Exact
    variants themselves sit ~3e-4 from float64 here (their Taylor-5 exp).
    """
    case = gc.load(f"cfg0_{op_name}")
    inputs = case.inputs()
    fused, exact = oracle.OPS[op_name][1:]
    out = _run_onnx(op_name, fused, _feed(*inputs)).astype(np.float64)
    ref = oracle.scan_f64(op_name, *inputs)
    normrel = np.linalg.norm(out - ref) / np.linalg.norm(ref)
    assert normrel <= 1e-5, normrel
    tol = 1e-4 if exact else 1e-3
    np.testing.assert_allclose(out, ref, rtol=tol, atol=tol)
    got = case.select(out)
    cpp = case.out_cpp.astype(np.float64)
    assert np.linalg.norm(got - cpp) / np.linalg.norm(cpp) <= 1e-3


def test_void_compute_entry_matches_status_entry():
    case = gc.load("core_SelectiveScanFused")
    feed = _feed(*case.inputs())
    a = _run_onnx(case.op, True, feed, use_v2=True)
    b = _run_onnx(case.op, True, feed, use_v2=False)
    np.testing.assert_array_equal(a, b)


def test_optional_delta_bias_input():
    """8th input of the fused ops: equals folding the bias into delta on the host."""
    u, delta, A, B, C, D, z, bias = sc.config_inputs(2, 96, 160, True, seed=11, fold_bias=False)
    feed = _feed(u, delta, A, B, C, D, z)
    feed["delta_bias"] = bias
    with_bias = _run_onnx("SelectiveScanFused", True, feed)
    feed.pop("delta_bias")
    feed["delta"] = (delta + bias[None, :, None]).astype(np.float32)
    folded = _run_onnx("SelectiveScanFused", True, feed)
    np.testing.assert_allclose(with_bias, folded, rtol=1e-5, atol=1e-5)
    ref = oracle.scan_f64("SelectiveScanFused", u, delta, A, B, C, D, z, delta_bias=bias)
    np.testing.assert_allclose(with_bias, ref, rtol=1e-3, atol=1e-3)


def test_long_sequence_uses_workspace_and_releases_it():
    """A 1x64x4096 shape takes the chunked path; its ORT scratch is returned
    when the kernel is destroyed (the session closes)."""
    u, delta, A, B, C, D, z, _ = sc.config_inputs(1, 64, 4096, False, seed=4,
                                                  exact_dt_per_element=True)
    before = ort_shim.live_allocations()
    out = _run_onnx("SelectiveScanExact", False, _feed(u, delta, A, B, C, D, None))
    assert ort_shim.live_allocations() == before
    ref = oracle.scan_f64("SelectiveScanExact", u, delta, A, B, C, D)
    assert np.linalg.norm(out - ref) / np.linalg.norm(ref) <= 1e-5
    np.testing.assert_allclose(out, ref, rtol=1e-4, atol=1e-4)


def _dev_inputs(op, batch, dim, seqlen, seed):
    fused = oracle.OPS[op][1]
    arrs = sc.config_inputs(batch, dim, seqlen, fused, seed=seed,
                            exact_dt_per_element=not fused)[:7]
    return arrs, [None if a is None else torch.from_numpy(np.ascontiguousarray(a)).cuda()
                  for a in arrs]


def test_one_kernel_on_two_streams_keeps_separate_scratch():
    """ONNX Runtime keeps one kernel object per node and may run it on several
    streams at once (multi-stream execution, concurrent sessions runs). The
    chunked path's scratch must then not be shared: two shapes that split their
    sequences run interleaved on two streams, with nothing ordering one stream
    against the other, three times each through one kernel; every output
    matches the oracle, and the kernel holds one buffer per stream until
    KernelDestroy returns them."""
    op = "SelectiveScanExact"
    opts = ort_shim.SessionOptions()
    mamba_onnx.register_custom_ops(opts, backend="cuda")
    before = ort_shim.live_allocations()
    (a_np, a_dev), (b_np, b_dev) = (_dev_inputs(op, 1, 64, 4096, 31),
                                    _dev_inputs(op, 1, 96, 3000, 32))
    assert cuda.workspace_size(op, 1, 64, 4096) > 0 and cuda.workspace_size(op, 1, 96, 3000) > 0
    s1, s2 = torch.cuda.Stream(), torch.cuda.Stream()
    with ort_shim.InferenceSession(ort_shim.make_model(op, False), opts) as sess:
        outs = []
        for _ in range(3):
            oa = torch.full_like(a_dev[0], float("nan"))
            ob = torch.full_like(b_dev[0], float("nan"))
            sess.run_device(a_dev[:6], oa, s1)
            sess.run_device(b_dev[:6], ob, s2)
            outs.append((oa, ob))
        torch.cuda.synchronize()
        assert ort_shim.live_allocations() == before + 2
        for arrs, got in [(a_np, [o[0] for o in outs]), (b_np, [o[1] for o in outs])]:
            ref = oracle.scan_f64(op, *arrs[:6])
            for g in got:
                g = g.cpu().numpy()
                assert np.linalg.norm(g - ref) / np.linalg.norm(ref) <= 1e-5
                np.testing.assert_allclose(g, ref, rtol=1e-4, atol=1e-4)
    assert ort_shim.live_allocations() == before


def test_kernel_scratch_grows_for_a_larger_shape():
    """A larger shape on the same stream gets a larger buffer; the outgrown one
    stays allocated (work already enqueued may read it) until KernelDestroy."""
    op = "SelectiveScanFused"
    opts = ort_shim.SessionOptions()
    mamba_onnx.register_custom_ops(opts, backend="cuda")
    before = ort_shim.live_allocations()
    small_np, small = _dev_inputs(op, 1, 32, 1024, 41)
    big_np, big = _dev_inputs(op, 1, 256, 4096, 42)
    assert 0 < cuda.workspace_size(op, 1, 32, 1024) < cuda.workspace_size(op, 1, 256, 4096)
    with ort_shim.InferenceSession(ort_shim.make_model(op, True), opts) as sess:
        o_small, o_big = torch.empty_like(small[0]), torch.empty_like(big[0])
        sess.run_device(small, o_small)
        sess.run_device(big, o_big)
        sess.run_device(small, o_small)
        torch.cuda.synchronize()
        assert ort_shim.live_allocations() == before + 2
        for arrs, got in [(small_np, o_small), (big_np, o_big)]:
            ref = oracle.scan_f64(op, *arrs)
            np.testing.assert_allclose(got.cpu().numpy(), ref, rtol=1e-3, atol=1e-3)
    assert ort_shim.live_allocations() == before
