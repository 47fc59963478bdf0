"""GPU: the Exact ops' exp modes (include/mamba_scan.h, MAMBA_SCAN_EXP_*).

* exp="reference" forms every exp the way the reference C++ backend does (its
  published Taylor-5 times 2^n method, selective_scan.cc:33-69, also inside
  softplus and SiLU, cc:137-148), so its output follows that backend's own
  numbers: within normwise 1e-5 of the backend's golden outputs (out_cpp of
  tests/golden, written by the compiled reference) on every golden case of
  the Exact ops, the 1x1536x512 benchmark configuration included, where the
  backend itself sits ~3e-4 from float64. This is the "rel <= 1e-5 against
  SelectiveScanExact" agreement. On a shape the planner splits into chunks,
  the same holds against the oracle's float32 restatement of the backend
  (bit-exact against it on the golden cases).
* exp="ieee" (CUDA's expf) and the default (SFU ex2.approx) follow the exact
  function: normwise within 1e-5 of the float64 oracle.
"""
import numpy as np
import pytest
import torch

import golden_cases as gc
import scan_cases as sc
from mamba_onnx import cuda
from oracle import oracle

pytestmark = pytest.mark.gpu

EXACT_OPS = ["SelectiveScanExact", "SelectiveScanFusedExact"]
EXACT_CASES = [n for n in gc.names() if gc.load(n).op in EXACT_OPS]


def _dev(a):
    return None if a is None else torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _run(op, inputs, **kw):
    u, delta, A, B, C, D, z = inputs[:7]
    return cuda.selective_scan(op, _dev(u), _dev(delta), _dev(A), _dev(B), _dev(C), _dev(D),
                               _dev(z) if "Fused" in op else None, **kw)


def _normrel(a, b):
    return float(np.linalg.norm(np.asarray(a, np.float64) - b) / np.linalg.norm(b))


@pytest.mark.parametrize("name", EXACT_CASES)
def test_reference_exp_follows_the_cpp_backend(name):
    case = gc.load(name)
    inputs = case.inputs()
    got = case.select(_run(case.op, inputs, exp="reference").cpu().numpy())
    assert _normrel(got, case.out_cpp.astype(np.float64)) <= 1e-5
    np.testing.assert_allclose(got, case.out_cpp, rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("op", EXACT_OPS)
def test_reference_exp_through_the_chunked_path(op):
    fused = oracle.OPS[op][1]
    inputs = sc.config_inputs(1, 256, 8192, fused, seed=12, exact_dt_per_element=not fused)[:7]
    assert cuda.workspace_size(op, 1, 256, 8192, exp="reference") > 0
    got = _run(op, inputs, exp="reference").cpu().numpy()
    cpp = oracle.scan_f32ref(op, *inputs).astype(np.float64)
    assert _normrel(got, cpp) <= 1e-5
    single = _run(op, inputs, exp="reference", chunked=False).cpu().numpy()
    assert _normrel(single, cpp) <= 1e-5


@pytest.mark.parametrize("exp", [None, "ieee"])
@pytest.mark.parametrize("op", EXACT_OPS)
@pytest.mark.parametrize("shape", [(1, 1536, 512), (1, 256, 8192)], ids=["1x1536x512", "1x256x8192"])
def test_accurate_exp_modes_follow_float64(op, exp, shape):
    fused = oracle.OPS[op][1]
    inputs = sc.config_inputs(*shape, fused, seed=0, exact_dt_per_element=not fused)[:7]
    got = _run(op, inputs, exp=exp).cpu().numpy()
    ref = oracle.scan_f64(op, *inputs)
    assert _normrel(got, ref) <= 1e-5
    np.testing.assert_allclose(got, ref, rtol=1e-4, atol=1e-4)
