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
import pytest

import golden_cases as gc
import mamba_onnx
import scan_cases as sc
from fake_ort import ort_shim
from oracle import oracle

pytestmark = pytest.mark.gpu


def _run_onnx(op_name, use_fused, feed, use_v2=True):
    """tests/test_ops.py:136-144 with the CUDA execution provider."""
    opts = ort_shim.SessionOptions()
    mamba_onnx.register_custom_ops(opts, backend="cuda")
    model = ort_shim.make_model(op_name, use_fused, with_delta_bias="delta_bias" in feed)
    sess = ort_shim.InferenceSession(model, opts, providers=["CUDAExecutionProvider"],
                                     use_v2=use_v2)
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
    """A 1x64x4096 shape takes the chunked path; its ORT scratch is freed."""
    u, delta, A, B, C, D, z, _ = sc.config_inputs(1, 64, 4096, False, seed=4,
                                                  exact_dt_per_element=True)
    before = ort_shim.live_allocations()
    out = _run_onnx("SelectiveScanExact", False, _feed(u, delta, A, B, C, D, None))
    assert ort_shim.live_allocations() == before
    ref = oracle.scan_f64("SelectiveScanExact", u, delta, A, B, C, D)
    assert np.linalg.norm(out - ref) / np.linalg.norm(ref) <= 1e-5
    np.testing.assert_allclose(out, ref, rtol=1e-4, atol=1e-4)
