"""CPU: the oracle against the golden vectors of the reference's own tests.

Pins the two restatements in oracle/scan_oracle.c before they are trusted as
the checker for the CUDA path:
* float64 restatement vs the reference test oracle (reference_selective_scan,
  tests/test_ops.py:17-63) at each reference test's own tolerance;
* float32 restatement of the reference C++ numerics vs the compiled reference
  plugin's outputs, bit for bit;
* the compiled reference plugin (oracle/_ref) reproduces its golden outputs.
"""
import numpy as np
import pytest

import golden_cases as gc
import scan_cases as sc
from oracle import oracle


@pytest.mark.parametrize("name", gc.names())
def test_golden_inputs_regenerate(name):
    case = gc.load(name)
    assert sc.sha256_arrays(case.inputs()) == case.input_sha256


@pytest.mark.parametrize("name", gc.names())
def test_f64_oracle_matches_reference_test_oracle(name):
    """Float64 restatement vs the reference's torch oracle (fp32), at the test tolerance."""
    case = gc.load(name)
    u, delta, A, B, C, D, z = case.inputs()
    got = case.select(oracle.scan_f64(case.op, u, delta, A, B, C, D, z))
    np.testing.assert_allclose(got, case.out_torch32, rtol=case.tol, atol=case.tol)


@pytest.mark.parametrize("name", gc.names())
def test_f32_restatement_bit_exact_vs_reference_cpp(name):
    """Float32 restatement of cc:33-305 equals the compiled reference C++ exactly."""
    case = gc.load(name)
    got = case.select(oracle.scan_f32ref(case.op, *case.inputs()))
    np.testing.assert_array_equal(got, case.out_cpp)


@pytest.mark.skipif(not oracle.ref_available(), reason="reference plugin not built")
@pytest.mark.parametrize("name", gc.names())
def test_reference_plugin_reproduces_golden(name):
    case = gc.load(name)
    got = case.select(oracle.ref_run(case.op, *case.inputs(), n_threads=2))
    np.testing.assert_array_equal(got, case.out_cpp)


@pytest.mark.skipif(not oracle.ref_available(), reason="reference plugin not built")
def test_reference_plugin_registers_four_ops_and_rejects_dstate():
    assert oracle.ref_op_names() == [op for op, _, _ in sc.ALL_OPS]
    u, delta, A, B, C, D, _ = sc.reference_test_inputs(1, 8, 4, False)
    with pytest.raises(RuntimeError, match="dstate=16"):
        oracle.ref_run("SelectiveScan", u, delta, A[:, :8], B[..., :8], C[..., :8], D)


def test_reference_fast_exp_error_and_underflow_quirk():
    """cc:33-69: max relative error ~8.6e-5 on [-20, 0]; -inf below about -88.03."""
    x = np.linspace(-20.0, 0.0, 200001, dtype=np.float32)
    rel = np.abs(oracle.ref_fast_exp(x).astype(np.float64) / np.exp(x.astype(np.float64)) - 1)
    assert 5e-5 < rel.max() < 1e-4
    y = oracle.ref_fast_exp(np.array([-88.2, -100.0, -87.0], dtype=np.float32))
    assert np.isneginf(y[0]) and np.isneginf(y[1]) and y[2] > 0


@pytest.mark.parametrize("op", [op for op, _, _ in sc.ALL_OPS])
def test_f64_state_composition(op):
    """Scanning [0, L) equals scanning [0, k) then [k, L) from the carried state."""
    fused = oracle.OPS[op][1]
    u, delta, A, B, C, D, z = sc.reference_test_inputs(2, 16, 40, fused, seed=3)
    full, h_full = oracle.scan_f64(op, u, delta, A, B, C, D, z, return_state=True)
    k = 17
    sl = lambda a, ax: None if a is None else np.ascontiguousarray(np.take(a, range(k), axis=ax))  # noqa
    sr = lambda a, ax: None if a is None else np.ascontiguousarray(np.take(a, range(k, 40), axis=ax))  # noqa
    first, h_mid = oracle.scan_f64(op, sl(u, 2), sl(delta, 2), A, sl(B, 1), sl(C, 1), D, sl(z, 2),
                                   return_state=True)
    second, h_end = oracle.scan_f64(op, sr(u, 2), sr(delta, 2), A, sr(B, 1), sr(C, 1), D, sr(z, 2),
                                    h0=h_mid, return_state=True)
    np.testing.assert_allclose(np.concatenate([first, second], axis=2), full, rtol=1e-12,
                               atol=1e-12)
    np.testing.assert_allclose(h_end, h_full, rtol=1e-12, atol=1e-12)


def test_f64_rows_subset_and_delta_bias():
    u, delta, A, B, C, D, z, bias = sc.config_inputs(2, 40, 24, True, seed=5, fold_bias=False)
    rows = np.array([0, 7, 39, 40, 79])
    sub = oracle.scan_f64("SelectiveScanFused", u, delta, A, B, C, D, z, delta_bias=bias, rows=rows)
    folded = (delta + bias[None, :, None]).astype(np.float32)
    full = oracle.scan_f64("SelectiveScanFused", u, folded, A, B, C, D, z)
    np.testing.assert_allclose(sub, full.reshape(-1, 24)[rows], rtol=1e-6, atol=1e-6)
