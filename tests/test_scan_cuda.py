"""GPU: the C ABI (include/mamba_scan.h) across shapes, code paths and properties.

Every comparison is against the oracle's float64 restatement. Tolerances:
rtol = atol = 1e-4 at the reference test distributions (the tolerance of
tests/test_ops.py:171), normwise relative error <= 1e-5 at the benchmark
distributions, plus elementwise 1e-4 (Exact variants) / 1e-3 (approximate
variants: SFU exp/log in softplus and silu).
"""
import numpy as np
import pytest
import torch

import scan_cases as sc
from mamba_onnx import cuda
from oracle import oracle

pytestmark = pytest.mark.gpu
OPS = [op for op, _, _ in sc.ALL_OPS]


def dev(a):
    return None if a is None else torch.from_numpy(np.ascontiguousarray(a)).cuda()


def run(op, inputs, **kw):
    u, delta, A, B, C, D, z = inputs[:7]
    out = cuda.selective_scan(op, dev(u), dev(delta), dev(A), dev(B), dev(C), dev(D),
                              dev(z) if "Fused" in op else None, **kw)
    return out


def ref_inputs(B, D, L, fused, seed=42):
    return sc.reference_test_inputs(B, D, L, fused, seed=seed)


SHAPES = [
    (1, 1, 1),       # one row, one step
    (1, 64, 1),      # tests/test_ops.py L=1
    (3, 33, 17),     # ragged rows and steps; L % 4 != 0 -> plain-load path
    (2, 48, 20),     # L % 16 != 0 -> partial last TMA tile
    (1, 100, 300),   # several tiles, ragged rows
    (2, 64, 1000),   # few rows, long L -> chunked (aggregate + emit)
    (1, 40, 2050),   # chunked with a ragged last chunk
    (5, 130, 64),
]


@pytest.mark.parametrize("shape", SHAPES, ids=[f"{b}x{d}x{l}" for b, d, l in SHAPES])
@pytest.mark.parametrize("op", OPS)
def test_matches_oracle(op, shape):
    fused = oracle.OPS[op][1]
    inputs = ref_inputs(*shape, fused)
    got = run(op, inputs).cpu().numpy()
    ref = oracle.scan_f64(op, *inputs)
    np.testing.assert_allclose(got, ref, rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("op", OPS)
def test_plain_load_path_equals_tma_path(op):
    """Misaligned (4-byte offset) inputs take the plain-load path: same bits."""
    fused = oracle.OPS[op][1]
    inputs = ref_inputs(2, 70, 96, fused, seed=5)
    a = run(op, inputs)

    def shifted(x):
        if x is None:
            return None
        buf = torch.empty(x.size + 1, dtype=torch.float32, device="cuda")
        view = buf[1:].view(x.shape)
        view.copy_(torch.from_numpy(np.ascontiguousarray(x)))
        return view

    u, delta, A, B, C, D, z = inputs
    b = cuda.selective_scan(op, shifted(u), shifted(delta), dev(A), shifted(B), shifted(C),
                            dev(D), shifted(z) if fused else None)
    torch.testing.assert_close(a, b, rtol=0, atol=0)


@pytest.mark.parametrize("op", OPS)
def test_chunked_equals_single_pass(op):
    fused = oracle.OPS[op][1]
    inputs = sc.config_inputs(1, 64, 3000, fused, seed=7, exact_dt_per_element=not fused)[:7]
    assert cuda.workspace_size(op, 1, 64, 3000) > 0
    a = run(op, inputs).double()
    b = run(op, inputs, chunked=False).double()
    assert ((a - b).norm() / b.norm()).item() <= 1e-5
    ref = oracle.scan_f64(op, *inputs)
    got = a.cpu().numpy()
    assert np.linalg.norm(got - ref) / np.linalg.norm(ref) <= 1e-5


@pytest.mark.parametrize("op", OPS)
def test_initial_and_final_state_compose(op):
    """Scan [0,L) == scan [0,k) then [k,L) from h_last; h_last matches the oracle."""
    fused = oracle.OPS[op][1]
    B, D, L, k = 2, 80, 777, 300
    u, delta, A, Bm, C, Dv, z = ref_inputs(B, D, L, fused, seed=9)
    h_full = torch.empty(B, D, 16, device="cuda")
    full = cuda.selective_scan(op, dev(u), dev(delta), dev(A), dev(Bm), dev(C), dev(Dv),
                               dev(z), h_last=h_full)
    sl = lambda a, ax, r: None if a is None else np.ascontiguousarray(np.take(a, r, axis=ax))  # noqa
    r1, r2 = range(k), range(k, L)
    h_mid = torch.empty(B, D, 16, device="cuda")
    first = cuda.selective_scan(op, dev(sl(u, 2, r1)), dev(sl(delta, 2, r1)), dev(A),
                                dev(sl(Bm, 1, r1)), dev(sl(C, 1, r1)), dev(Dv),
                                dev(sl(z, 2, r1)), h_last=h_mid)
    h_end = torch.empty(B, D, 16, device="cuda")
    second = cuda.selective_scan(op, dev(sl(u, 2, r2)), dev(sl(delta, 2, r2)), dev(A),
                                 dev(sl(Bm, 1, r2)), dev(sl(C, 1, r2)), dev(Dv),
                                 dev(sl(z, 2, r2)), h0=h_mid, h_last=h_end)
    torch.testing.assert_close(torch.cat([first, second], dim=2), full, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(h_end, h_full, rtol=1e-5, atol=1e-5)
    _, h_ref = oracle.scan_f64(op, u, delta, A, Bm, C, Dv, z, return_state=True)
    np.testing.assert_allclose(h_full.cpu().numpy().reshape(-1, 16), h_ref, rtol=1e-4,
                               atol=1e-4)


def test_zero_length_sequence_returns_initial_state():
    A = dev(-np.ones((8, 16), np.float32))
    Dv = dev(np.ones(8, np.float32))
    e3 = torch.empty(1, 8, 0, device="cuda")
    eb = torch.empty(1, 0, 16, device="cuda")
    h0 = torch.randn(1, 8, 16, device="cuda")
    h_last = torch.full((1, 8, 16), float("nan"), device="cuda")
    out = cuda.selective_scan("SelectiveScan", e3, e3, A, eb, eb, Dv, h0=h0, h_last=h_last)
    assert out.shape == (1, 8, 0)
    torch.testing.assert_close(h_last, h0, rtol=0, atol=0)


def test_delta_bias_equals_folded_bias():
    u, delta, A, B, C, D, z, bias = sc.config_inputs(1, 96, 256, True, seed=3, fold_bias=False)
    a = cuda.selective_scan("SelectiveScanFusedExact", dev(u), dev(delta), dev(A), dev(B),
                            dev(C), dev(D), dev(z), delta_bias=dev(bias))
    ref = oracle.scan_f64("SelectiveScanFusedExact", u, delta, A, B, C, D, z, delta_bias=bias)
    got = a.cpu().numpy()
    assert np.linalg.norm(got - ref) / np.linalg.norm(ref) <= 1e-5


def test_errors_are_reported_without_launching():
    u, delta, A, B, C, D, _ = ref_inputs(1, 64, 32, False)
    with pytest.raises(cuda.ScanError, match="dstate=16") as e:
        cuda.selective_scan("SelectiveScan", dev(u), dev(delta), dev(A[:, :8]), dev(B[..., :8]),
                            dev(C[..., :8]), dev(D))
    assert e.value.status == 2
    x = dev(u)
    with pytest.raises(cuda.ScanError, match="overlaps") as e:
        cuda.selective_scan("SelectiveScan", x, dev(delta), dev(A), dev(B), dev(C), dev(D), out=x)
    assert e.value.status == 4
    big = sc.config_inputs(1, 64, 3000, False, seed=1)[:7]
    with pytest.raises(cuda.ScanError, match="workspace") as e:
        run("SelectiveScan", big, workspace=torch.empty(16, dtype=torch.uint8, device="cuda"))
    assert e.value.status == 3


@pytest.mark.parametrize("op", OPS)
def test_deterministic(op):
    fused = oracle.OPS[op][1]
    inputs = sc.config_inputs(2, 256, 512, fused, seed=2)[:7]
    a, b = run(op, inputs), run(op, inputs)
    assert torch.equal(a, b)


# ---- full benchmark sizes: sampled rows vs float64, and size-free properties ----

def gpu_config(B, D, L, fused, seed, exact_dt_per_element=False):
    """Benchmark distributions drawn on the device (torch CUDA generator)."""
    g = torch.Generator(device="cuda").manual_seed(seed)
    kw = dict(device="cuda", generator=g)
    u = torch.randn(B, D, L, **kw)
    z = torch.randn(B, D, L, **kw) if fused else None
    Bm = torch.randn(B, L, 16, **kw)
    Cm = torch.randn(B, L, 16, **kw)
    lo, hi = np.log(1e-3), np.log(1e-1)
    dt = torch.exp(torch.rand(D, **kw) * (hi - lo) + lo)
    A = -torch.arange(1, 17, device="cuda", dtype=torch.float32).repeat(D, 1)
    Dv = torch.ones(D, device="cuda")
    if fused:
        delta = torch.randn(B, D, L, **kw) * 0.5 + torch.log(torch.expm1(dt))[None, :, None]
    elif exact_dt_per_element:
        delta = torch.exp(torch.rand(B, D, L, **kw) * (hi - lo) + lo)
    else:
        delta = dt[None, :, None].expand(B, D, L).contiguous()
    return u, delta, A, Bm, Cm, Dv, z


def check_rows(op, inputs, out, n_rows=48, seed=0):
    u, delta, A, Bm, Cm, Dv, z = inputs
    B, D, L = u.shape
    rows = np.random.default_rng(seed).choice(B * D, n_rows, replace=False)
    rows[:2] = [0, B * D - 1]
    errs, norms = 0.0, 0.0
    exact = oracle.OPS[op][2]
    for r in rows:
        b, d = divmod(int(r), D)
        sl = lambda t: t[b, d][None, None].cpu().numpy()  # noqa: E731
        ref = oracle.scan_f64(op, sl(u), sl(delta), A[d][None].cpu().numpy(),
                              Bm[b][None].cpu().numpy(), Cm[b][None].cpu().numpy(),
                              Dv[d][None].cpu().numpy(), sl(z) if z is not None else None)[0, 0]
        got = out[b, d].double().cpu().numpy()
        tol = 1e-4 if exact else 1e-3
        np.testing.assert_allclose(got, ref, rtol=tol, atol=tol)
        errs += float(np.sum((got - ref) ** 2))
        norms += float(np.sum(ref ** 2))
    assert (errs / norms) ** 0.5 <= 1e-5


def test_config_8x5120x2048_fused_rows():
    inputs = gpu_config(8, 5120, 2048, True, seed=1)
    out = cuda.selective_scan("SelectiveScanFused", *inputs)
    assert torch.isfinite(out).all()
    check_rows("SelectiveScanFused", inputs, out)


def test_config_64x5120x4096_fused_rows():
    """The multi-GPU configuration's whole batch (64 x 5120 x 4096, 21.5 GB of
    tensors) on one GPU: 48 sampled rows against the float64 oracle, the
    first and last row among them."""
    inputs = gpu_config(64, 5120, 4096, True, seed=3)
    out = cuda.selective_scan("SelectiveScanFused", *inputs)
    assert torch.isfinite(out).all()
    check_rows("SelectiveScanFused", inputs, out)
    del inputs, out
    torch.cuda.empty_cache()


def test_config_1x2048x16384_exact_rows_and_chunking():
    inputs = gpu_config(1, 2048, 16384, False, seed=2, exact_dt_per_element=True)
    out = cuda.selective_scan("SelectiveScanExact", *inputs[:6])
    assert torch.isfinite(out).all()
    check_rows("SelectiveScanExact", inputs, out, n_rows=24)
    single = cuda.selective_scan("SelectiveScanExact", *inputs[:6], chunked=False)
    assert ((out.double() - single.double()).norm() / single.double().norm()).item() <= 1e-5


@pytest.mark.parametrize("op", ["SelectiveScan", "SelectiveScanExact"])
def test_linearity_in_u_at_full_length(op):
    """Non-fused ops are linear in u for fixed delta: scan(a*u1 + b*u2) = a*scan(u1) + b*scan(u2)."""
    u1, delta, A, Bm, Cm, Dv, _ = gpu_config(1, 2048, 16384, False, seed=4,
                                            exact_dt_per_element=True)
    u2 = torch.randn_like(u1)
    y1 = cuda.selective_scan(op, u1, delta, A, Bm, Cm, Dv)
    y2 = cuda.selective_scan(op, u2, delta, A, Bm, Cm, Dv)
    y12 = cuda.selective_scan(op, (0.5 * u1 - 2.0 * u2).contiguous(), delta, A, Bm, Cm, Dv)
    comb = 0.5 * y1.double() - 2.0 * y2.double()
    assert ((y12.double() - comb).norm() / comb.norm()).item() <= 1e-5


def test_no_device_error_recorded():
    assert cuda.check_device_error() == 0


def test_bounded_wait_gives_up_and_the_context_survives():
    """A wait that cannot complete (announced bytes that no copy delivers)
    gives up after its limit and records MAMBA_SCAN_ERR_DEVICE_TIMEOUT; the
    next scan runs normally. No fault is involved."""
    import time

    assert cuda.check_device_error() == 0
    t0 = time.perf_counter()
    assert cuda.selftest_wait_timeout(20_000_000) == 0  # 20 ms
    assert cuda.check_device_error() == 6
    assert time.perf_counter() - t0 < 5.0
    assert cuda.check_device_error() == 0  # read clears it
    assert cuda.selftest_wait_timeout(0) == 1  # limit out of range: nothing launched
    u, delta, A, B, C, D, z = [None if a is None else dev(a) for a in
                               sc.config_inputs(1, 64, 256, True, seed=4)[:7]]
    out = cuda.selective_scan("SelectiveScanFused", u, delta, A, B, C, D, z)
    assert torch.isfinite(out).all()
    assert cuda.check_device_error() == 0
