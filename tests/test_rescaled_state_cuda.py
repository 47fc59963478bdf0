"""GPU: inputs that stress the linear ops' rescaled state.

SelectiveScan and SelectiveScanFused run their recurrence on g = h / w with
w = delta*u (|w| held at 1e-12 or above), so zero, tiny, denormal,
sign-flipping or widely ranging delta*u must leave the result unchanged. Each
case checks the output and the final state of all four ops against the
oracle's float64 restatement at the reference tests' tolerance
(rtol = atol = 1e-4, tests/test_ops.py:171), through the single-pass TMA path
(with a partial last tile), the chunked path and the plain-load path.
"""
import zlib

import numpy as np
import pytest
import torch

import scan_cases as sc
from mamba_onnx import cuda
from oracle import oracle

pytestmark = pytest.mark.gpu
OPS = [op for op, _, _ in sc.ALL_OPS]

# (batch, dim, seqlen): 200 = 12 tiles + 8 steps (TMA, partial last tile);
# 3000 steps over 48 rows -> chunked; 203 % 4 != 0 -> plain-load path
SHAPES = [(2, 64, 200), (1, 48, 3000), (2, 40, 203)]
CASES = ["zeros", "tiny", "sign_flip", "wide_range", "zero_delta"]


def _stress(case, u, delta, rng):
    u, delta = u.copy(), delta.copy()
    L = u.shape[2]
    if case == "zeros":
        u[..., ::5] = 0.0                 # every fifth step
        u[..., 0] = 0.0                   # first step (w_{-1} = 1 -> r = 1e12)
        u[..., L - 1] = 0.0               # last step (state leaves as 1e-12 * g)
        u[..., 15:17] = 0.0               # across a tile boundary
        u[:, ::7, :] = 0.0                # whole rows
    elif case == "tiny":
        mask = rng.random(u.shape) < 0.3
        mag = 10.0 ** rng.uniform(-45.0, -8.0, u.shape)  # includes float32 denormals
        u = np.where(mask, np.sign(u) * mag, u).astype(np.float32)
    elif case == "sign_flip":
        u = (np.abs(u) * np.where(np.arange(L) % 2 == 0, 1.0, -1.0)).astype(np.float32)
    elif case == "wide_range":
        u = (u * 10.0 ** rng.uniform(-6.0, 6.0, u.shape)).astype(np.float32)
    elif case == "zero_delta":
        delta[..., ::3] = 0.0
    return u, delta


def _dev(a):
    return None if a is None else torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("shape", SHAPES, ids=[f"{b}x{d}x{l}" for b, d, l in SHAPES])
@pytest.mark.parametrize("case", CASES)
@pytest.mark.parametrize("op", OPS)
def test_stressed_inputs_match_oracle(op, case, shape):
    fused = oracle.OPS[op][1]
    B, D, L = shape
    u, delta, A, Bm, C, Dv, z = sc.reference_test_inputs(B, D, L, fused, seed=11)
    rng = np.random.default_rng(zlib.crc32(repr((op, case, shape)).encode()))
    u, delta = _stress(case, u, delta, rng)
    h0 = (rng.standard_normal((B, D, 16)) * 0.5).astype(np.float32)
    h_last = torch.empty(B, D, 16, device="cuda")
    out = cuda.selective_scan(op, _dev(u), _dev(delta), _dev(A), _dev(Bm), _dev(C), _dev(Dv),
                              _dev(z), h0=_dev(h0), h_last=h_last)
    got = out.cpu().numpy()
    ref, h_ref = oracle.scan_f64(op, u, delta, A, Bm, C, Dv, z, h0=h0.reshape(-1, 16),
                                 return_state=True)
    assert np.isfinite(got).all()
    scale = max(1.0, float(np.abs(ref).max()) * 1e-3) if case == "wide_range" else 1.0
    np.testing.assert_allclose(got, ref, rtol=1e-4, atol=1e-4 * scale)
    np.testing.assert_allclose(h_last.cpu().numpy().reshape(-1, 16), h_ref, rtol=1e-4,
                               atol=1e-4 * scale)
