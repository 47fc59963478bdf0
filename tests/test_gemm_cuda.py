"""Tensor-core 3xTF32 GEMM and its tf32 split (include/mamba_model_ops.h).

The GEMM serves the Mamba model's dense projections around the scan op; it
must be as accurate as an fp32 GEMM. Each case compares it with a float64
matmul of the same fp32 inputs: elementwise within 1e-5 of sum_k |a||b| (the
fp32 accumulation bound of a K <= 2048 reduction is ~1e-4 of that sum), and
normwise no further from float64 than 2x cuBLAS's own fp32 GEMM (TF32 off)
plus 1e-7.
"""
import pytest
import torch

from mamba_onnx import cuda

pytestmark = pytest.mark.gpu


def _rand(shape, seed, dev, scale=1.0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return (torch.randn(shape, generator=g) * scale).to(dev)


def test_split_parts_are_tf32_and_sum_to_x(cuda_device):
    x = _rand((37, 91), 0, cuda_device) * torch.logspace(-20, 20, 91, device=cuda_device)
    s = cuda.split_tf32(x)
    assert s.ld == 92 and (s.rows, s.cols) == (37, 91)
    hi, lo = s.hi[:, :91], s.lo[:, :91]
    low13 = (1 << 13) - 1
    assert int((hi.view(torch.int32) & low13).abs().sum()) == 0
    assert int((lo.view(torch.int32) & low13).abs().sum()) == 0
    x64 = x.double()
    err = (hi.double() + lo.double() - x64).abs()
    assert bool((err <= 2.0 ** -22 * x64.abs()).all())
    assert bool((lo.abs() <= 2.0 ** -11 * x.abs()).all())
    t = cuda.split_tf32(x.t().contiguous(), transpose=True)
    assert torch.equal(t.hi[:, :91], hi) and torch.equal(t.lo[:, :91], lo)


CASES = [
    # M, N, K, transpose_c, accumulate
    (128, 128, 32, False, False),
    (1, 1, 1, False, False),
    (5, 7, 3, True, False),
    (200, 300, 48, False, True),
    (130, 257, 100, True, True),
    (80, 1024, 1536, True, False),      # x_proj shape
    (3072, 1024, 768, False, False),    # in_proj: W [2D, d] x hn^T
    (768, 1024, 1536, True, True),      # out_proj into the residual [L, d]
    (1024, 2000, 768, False, False),    # an LM-head slice
    # 192-column tiles (chosen when they take fewer waves): ragged M, N, K
    (3000, 1000, 100, False, False),
    (2900, 900, 40, True, True),
    # CTA pairs with 256-column tiles (the LM head's choice): a pair whose
    # second CTA lies wholly past M, ragged N and K
    (300, 7500, 100, False, True),
    (1024, 3500, 768, True, False),
    # few rows, many columns: single CTAs with 192-column tiles
    (64, 19008, 40, False, False),
    # several waves of 256 x 256 pair tiles: ragged M, N, K; row-major C with
    # C_in, column-major C
    (1000, 20000, 100, False, True),
    (700, 15000, 64, True, False),
]


@pytest.mark.parametrize("M,N,K,tc,acc", CASES)
def test_gemm_matches_float64(cuda_device, M, N, K, tc, acc):
    dev = cuda_device
    a = _rand((M, K), 1 + M, dev)
    b = _rand((N, K), 2 + N, dev, scale=0.05)
    c0 = _rand((N, M) if tc else (M, N), 3 + K, dev)
    c = c0.clone() if acc else torch.full_like(c0, float("nan"))
    cuda.gemm_tf32x3(cuda.split_tf32(a), cuda.split_tf32(b), c, transpose_c=tc,
                     c_in=c if acc else None)
    ref = a.double() @ b.double().t()
    if tc:
        ref = ref.t()
    if acc:
        ref = ref + c0.double()
    bound = (a.double().abs() @ b.double().abs().t())
    bound = (bound.t() if tc else bound) + (c0.double().abs() if acc else 0)
    err = (c.double() - ref).abs()
    assert bool((err <= 1e-5 * bound + 1e-30).all()), float((err / (bound + 1e-30)).max())
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        cb = a @ b.t()
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    cb = (cb.t() if tc else cb) + (c0 if acc else 0)
    e_ours = float((c.double() - ref).norm() / ref.norm())
    e_cublas = float((cb.double() - ref).norm() / ref.norm())
    assert e_ours <= 2 * e_cublas + 1e-7, (e_ours, e_cublas)
    assert cuda.check_device_error() == 0


def test_gemm_c_in_distinct_from_c(cuda_device):
    dev = cuda_device
    a, b = _rand((70, 40), 4, dev), _rand((50, 40), 5, dev)
    c_in = _rand((70, 50), 6, dev)
    keep = c_in.clone()
    c = torch.empty_like(c_in)
    cuda.gemm_tf32x3(cuda.split_tf32(a), cuda.split_tf32(b), c, c_in=c_in)
    assert torch.equal(c_in, keep)
    ref = keep.double() + a.double() @ b.double().t()
    assert float((c.double() - ref).norm() / ref.norm()) < 1e-6


def test_gemm_transposed_operand_split(cuda_device):
    """B taken as the split transpose of a [K][N] activation (the model's y^T)."""
    dev = cuda_device
    a = _rand((96, 200), 7, dev)
    y = _rand((200, 333), 8, dev)  # [K][N]
    c = torch.empty(96, 333, device=dev)
    cuda.gemm_tf32x3(cuda.split_tf32(a), cuda.split_tf32(y, transpose=True), c)
    ref = a.double() @ y.double()
    assert float((c.double() - ref).norm() / ref.norm()) < 1e-6


def test_gemm_rejects_bad_arguments(cuda_device):
    dev = cuda_device
    a = cuda.split_tf32(_rand((8, 16), 1, dev))
    b = cuda.split_tf32(_rand((8, 12), 2, dev))
    with pytest.raises(ValueError):
        cuda.gemm_tf32x3(a, b, torch.empty(8, 8, device=dev))
    lib = cuda.library()
    rc = lib.mamba_gemm_tf32x3(a.hi.data_ptr(), a.lo.data_ptr(), 6, a.hi.data_ptr(),
                               a.lo.data_ptr(), 16, None, a.hi.data_ptr(), 8, 1, 8, 8, 16, None)
    assert rc != 0 and b"multiples of 4" in lib.mamba_scan_last_error()


def test_split_more_rows_than_one_grid(cuda_device):
    """Row counts past one launch's 65535-row grid (the tied embedding has 50280)."""
    x = _rand((70001, 6), 9, cuda_device)
    s = cuda.split_tf32(x)
    err = (s.hi[:, :6].double() + s.lo[:, :6].double() - x.double()).abs()
    assert bool((err <= 2.0 ** -22 * x.double().abs()).all())


def test_gemm_is_deterministic(cuda_device):
    """Two runs of the same product are bit-identical (CUDA-graph replay relies on it)."""
    dev = cuda_device
    a = cuda.split_tf32(_rand((768, 1536), 11, dev))
    b = cuda.split_tf32(_rand((1024, 1536), 12, dev))
    c1, c2 = torch.empty(768, 1024, device=dev), torch.empty(768, 1024, device=dev)
    cuda.gemm_tf32x3(a, b, c1)
    cuda.gemm_tf32x3(a, b, c2)
    assert torch.equal(c1, c2)
    assert cuda.check_device_error() == 0


SPLIT_CASES = [
    # M, N, K, transpose_c, accumulate: products with few output tiles,
    # whose K the GEMM splits across the SMs through a workspace
    (768, 1024, 1536, True, True),    # out_proj into the residual (C_in = C)
    (768, 1024, 1536, False, False),  # row-major C (the float4 reduction)
    (701, 999, 1500, False, True),    # ragged M, N, K, odd M * N: the scalar reduction
    (80, 1024, 1536, True, False),
    (64, 64, 4096, False, True),
]


@pytest.mark.parametrize("M,N,K,tc,acc", SPLIT_CASES)
def test_gemm_split_k_matches_float64(cuda_device, M, N, K, tc, acc):
    """Split K (partials in the workspace, fixed-order reduction): the same
    accuracy bounds as the unsplit product, bit-identical on a second run,
    and within fp32 rounding of the unsplit product."""
    dev = cuda_device
    need = cuda.gemm_workspace_size(M, N, K)
    assert need > 0, "the case must split"
    a = _rand((M, K), 21 + M, dev)
    b = _rand((N, K), 22 + N, dev, scale=0.05)
    c0 = _rand((N, M) if tc else (M, N), 23 + K, dev)
    ws = torch.full((need,), 0xFF, dtype=torch.uint8, device=dev)  # NaN garbage
    sa, sb = cuda.split_tf32(a), cuda.split_tf32(b)

    def run(workspace):
        c = c0.clone() if acc else torch.full_like(c0, float("nan"))
        cuda.gemm_tf32x3(sa, sb, c, transpose_c=tc, c_in=c if acc else None,
                         workspace=workspace)
        return c

    c = run(ws)
    ref = a.double() @ b.double().t()
    bound = a.double().abs() @ b.double().abs().t()
    if tc:
        ref, bound = ref.t(), bound.t()
    if acc:
        ref, bound = ref + c0.double(), bound + c0.double().abs()
    err = (c.double() - ref).abs()
    assert bool((err <= 1e-5 * bound + 1e-30).all()), float((err / (bound + 1e-30)).max())
    assert torch.equal(run(ws), c)
    unsplit = run(None)
    assert float((c.double() - unsplit.double()).abs().max()) <= \
        float((2e-6 * bound).max())
    with pytest.raises(RuntimeError, match="workspace"):
        run(ws[: need - 16])
    assert cuda.check_device_error() == 0


def test_gemm_split_k_strided_c_distinct_c_in_and_reused_workspace(cuda_device):
    """Split K into a C with padded rows (not the partials' compact layout:
    the element-wise reduction) from a C_in that is not C, then a different
    product through the same workspace: each result matches its unsplit
    product to fp32 rounding, and C_in is left untouched."""
    dev = cuda_device
    M, N, K = 768, 1000, 1536
    ws = torch.empty(max(cuda.gemm_workspace_size(M, N, K), cuda.gemm_workspace_size(80, 1024, 1536)),
                     dtype=torch.uint8, device=dev)
    assert cuda.gemm_workspace_size(M, N, K) > 0
    sa, sb = cuda.split_tf32(_rand((M, K), 31, dev)), cuda.split_tf32(_rand((N, K), 32, dev, 0.05))
    c_in = _rand((M, N + 5), 33, dev)[:, :N]  # row stride N + 5
    keep = c_in.clone()
    c = torch.full((M, N + 5), float("nan"), device=dev)[:, :N]  # C_in shares C's strides
    cuda.gemm_tf32x3(sa, sb, c, c_in=c_in, workspace=ws)
    assert torch.equal(c_in, keep)
    unsplit = torch.empty(M, N + 5, device=dev)[:, :N]
    cuda.gemm_tf32x3(sa, sb, unsplit, c_in=c_in)
    bound = (sa.hi[:, :K].double().abs() @ sb.hi[:, :K].double().abs().t()) + keep.double().abs()
    assert float(((c.double() - unsplit.double()).abs() / (bound + 1e-30)).max()) <= 2e-6
    # another product through the same workspace, which still holds the first one's partials
    sx, sy = cuda.split_tf32(_rand((80, 1536), 34, dev)), cuda.split_tf32(_rand((1024, 1536), 35, dev))
    c2 = torch.empty(1024, 80, device=dev)
    cuda.gemm_tf32x3(sx, sy, c2, transpose_c=True, workspace=ws)
    u2 = torch.empty_like(c2)
    cuda.gemm_tf32x3(sx, sy, u2, transpose_c=True)
    b2 = (sx.hi[:, :1536].double().abs() @ sy.hi[:, :1536].double().abs().t()).t()
    assert float(((c2.double() - u2.double()).abs() / (b2 + 1e-30)).max()) <= 2e-6
    assert cuda.check_device_error() == 0
