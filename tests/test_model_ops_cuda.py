"""GPU: the Mamba-block kernels (include/mamba_model_ops.h) against torch fp32.

RMSNorm and the causal depthwise convolution + SiLU are compared with the
torch expressions they replace in mamba_onnx/model.py, on the model's shapes
and on ragged shapes that take the scalar (non-float4) paths. Tolerance:
rtol = 1e-5, atol = 1e-6 (fp32, differences are summation order and the
rsqrt/exp rounding).
"""
import pytest
import torch
import torch.nn.functional as F

from mamba_onnx import cuda

pytestmark = pytest.mark.gpu


def _torch_rmsnorm(x, w, eps):
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w


@pytest.mark.parametrize("shape", [(1, 1024, 768), (3, 5, 13), (2, 7, 1000), (1, 1, 4)])
def test_rmsnorm_matches_torch(shape):
    g = torch.Generator(device="cuda").manual_seed(1)
    x = torch.randn(*shape, device="cuda", generator=g) * 3
    w = torch.randn(shape[-1], device="cuda", generator=g)
    got = cuda.rmsnorm(x, w, 1e-5)
    torch.testing.assert_close(got, _torch_rmsnorm(x, w, 1e-5), rtol=1e-5, atol=1e-6)


def test_rmsnorm_unaligned_input_takes_the_scalar_path():
    g = torch.Generator(device="cuda").manual_seed(2)
    buf = torch.randn(1 + 6 * 64, device="cuda", generator=g)
    x = buf[1:].view(6, 64)  # 4-byte offset: not 16-byte aligned
    w = torch.randn(64, device="cuda", generator=g)
    torch.testing.assert_close(cuda.rmsnorm(x, w, 1e-6), _torch_rmsnorm(x, w, 1e-6),
                               rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("shape", [(1, 1024, 768), (3, 7, 64), (5, 4)])
def test_rmsnorm_split_equals_rmsnorm_then_split(shape):
    """The fused norm + tf32 split writes exactly split_tf32(rmsnorm(x))."""
    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randn(*shape, device="cuda", generator=g) * 3
    w = torch.randn(shape[-1], device="cuda", generator=g)
    got = cuda.rmsnorm_split_tf32(x, w, 1e-5)
    want = cuda.split_tf32(cuda.rmsnorm(x, w, 1e-5).reshape(-1, shape[-1]))
    assert (got.rows, got.cols) == (want.rows, want.cols)
    assert torch.equal(got.hi, want.hi[:, :shape[-1]]) and torch.equal(got.lo, want.lo[:, :shape[-1]])
    with pytest.raises(RuntimeError, match="multiples of 4"):
        cuda.rmsnorm_split_tf32(torch.randn(2, 6, device="cuda"), torch.randn(6, device="cuda"), 1e-5)


def _torch_conv_silu(x, w, b):
    K, L = w.shape[-1], x.shape[-1]
    return F.silu(F.conv1d(x, w, b, padding=K - 1, groups=x.shape[1])[..., :L])


@pytest.mark.parametrize("batch,dim,seqlen,width", [
    (1, 1536, 1024, 4),  # Mamba-130m layer
    (2, 48, 2052, 4),    # width 4 on float4 rows: several 1024-step blocks, a partial last one
    (2, 100, 37, 4),     # ragged sequence: scalar stores
    (3, 17, 64, 1), (1, 8, 5, 8), (2, 33, 200, 3), (1, 4, 1, 4),
])
@pytest.mark.parametrize("with_bias", [True, False])
def test_causal_conv1d_silu_matches_torch(batch, dim, seqlen, width, with_bias):
    g = torch.Generator(device="cuda").manual_seed(3)
    # x is the first half of an in_proj-shaped output [B, 2D, L], as in the model
    xz = torch.randn(batch, 2 * dim, seqlen, device="cuda", generator=g)
    x = xz[:, :dim]
    w = torch.randn(dim, 1, width, device="cuda", generator=g) * 0.5
    b = torch.randn(dim, device="cuda", generator=g) if with_bias else None
    got = cuda.causal_conv1d_silu(x, w, b)
    torch.testing.assert_close(got, _torch_conv_silu(x, w, b), rtol=1e-5, atol=1e-6)


def test_model_layer_uses_the_kernels_and_matches_the_torch_path():
    """One MambaLayer forward on CUDA equals the same layer's torch glue."""
    from mamba_onnx.model import MambaConfig, MambaLM, add_out_proj

    cfg = MambaConfig(d_model=64, n_layer=1, vocab_size=50)
    m = MambaLM(cfg).init_random(seed=4).cuda()
    layer = m.layers[0]
    h = torch.randn(1, 96, 64, device="cuda")
    A = -torch.exp(layer.A_log)
    got = layer(h, A)
    # the same block with torch glue (the scan stays on the CUDA op)
    D, K = cfg.d_inner, cfg.d_conv
    xz = torch.matmul(layer.in_proj_weight, _torch_rmsnorm(h, layer.norm_weight, cfg.rms_eps)
                      .transpose(1, 2))
    x = _torch_conv_silu(xz[:, :D], layer.conv_weight, layer.conv_bias)
    delta, Bm, Cm = layer._ssm_inputs(x)
    y = cuda.selective_scan("SelectiveScanFusedExact", x, delta, A, Bm, Cm, layer.D,
                            xz[:, D:].contiguous(), delta_bias=layer.dt_proj_bias)
    ref = h + torch.matmul(y.transpose(1, 2), layer.out_proj_weight.t())
    torch.testing.assert_close(got, ref, rtol=1e-4, atol=1e-5)
    torch.testing.assert_close(add_out_proj(h, y, layer.out_proj_weight), ref, rtol=1e-5,
                               atol=1e-6)


XPROJ_CASES = [
    # batch, dim, seqlen, rank, dstate
    (1, 1536, 1024, 48, 16),   # Mamba-130m
    (2, 200, 77, 8, 16),       # ragged: dim not a multiple of 8 x 32, seqlen of 64
    (1, 96, 1, 48, 16),        # one token (decoding): one warp per output
    (4, 1536, 1, 48, 16),      # 4 decoding streams
    (2, 300, 8, 80, 16),       # 16 tokens, P = 112, warp-per-output path
    (3, 520, 130, 80, 16),     # rank + 2 dstate = 112: the 8-outputs-per-thread path
]


@pytest.mark.parametrize("batch,dim,seqlen,rank,dstate", XPROJ_CASES)
def test_x_proj_matches_float64(batch, dim, seqlen, rank, dstate):
    """x_proj (cluster-split over d_inner, partials added in rank order)
    against a float64 matmul of the same fp32 inputs: normwise 1e-6,
    elementwise within 1e-5 of sum |w||x|; repeated calls are bit-identical."""
    g = torch.Generator(device="cpu").manual_seed(batch * 7 + dim)
    x = torch.randn(batch, dim, seqlen, generator=g).cuda()
    wx = (torch.randn(rank + 2 * dstate, dim, generator=g) * 0.02).cuda()
    dt, Bm, Cm = cuda.x_proj(x, wx, rank, dstate)
    assert dt.is_contiguous() and Bm.is_contiguous() and Cm.is_contiguous()
    ref = torch.einsum("jd,bdt->btj", wx.double(), x.double())
    bound = torch.einsum("jd,bdt->btj", wx.double().abs(), x.double().abs())
    got = torch.cat([dt, Bm, Cm], dim=-1).double()
    assert ((got - ref).abs() <= 1e-5 * bound + 1e-30).all()
    assert float((got - ref).norm() / ref.norm()) < 1e-6
    dt2, B2, C2 = cuda.x_proj(x, wx, rank, dstate)
    assert torch.equal(dt, dt2) and torch.equal(Bm, B2) and torch.equal(Cm, C2)
    assert cuda.check_device_error() == 0


XPROJ_DELTA_CASES = [
    (1, 1536, 1024, 48, 16),   # Mamba-130m
    (2, 200, 77, 8, 16),       # ragged dim and seqlen
    (3, 520, 130, 80, 16),     # P = 112: 4 outputs per thread
    (1, 96, 5, 48, 16),        # five tokens: one cluster, mostly padding
    (2, 2048, 64, 64, 16),     # dt_rank 64 (Mamba-370m widths)
    (1, 300, 40, 96, 16),      # the largest dt_rank, P = 128
]


@pytest.mark.parametrize("batch,dim,seqlen,rank,dstate", XPROJ_DELTA_CASES)
def test_x_proj_delta_equals_x_proj_then_dt_proj(batch, dim, seqlen, rank, dstate):
    """x_proj with dt_proj fused behind it: delta within 2e-5 of the float64
    chain's sum of magnitudes. Above 16 tokens, where mamba_x_proj takes the
    same cluster kernel, B and C are bit-identical to mamba_x_proj's and
    delta to mamba_dt_proj of mamba_x_proj's dt (same sums in the same order);
    at 16 tokens or fewer mamba_x_proj sums in another order, and B and C are
    compared with the float64 product instead."""
    g = torch.Generator(device="cpu").manual_seed(batch * 13 + dim + rank)
    x = torch.randn(batch, dim, seqlen, generator=g).cuda()
    wx = (torch.randn(rank + 2 * dstate, dim, generator=g) * dim ** -0.5).cuda()
    wdt = (torch.randn(dim, rank, generator=g) * rank ** -0.5).cuda()
    delta, Bm, Cm = cuda.x_proj_delta(x, wx, wdt, rank, dstate)
    dt, B2, C2 = cuda.x_proj(x, wx, rank, dstate)
    if batch * seqlen > 16:
        assert torch.equal(Bm, B2) and torch.equal(Cm, C2)
        assert torch.equal(delta, cuda.dt_proj(dt, wdt))
    else:
        bc = torch.einsum("jd,bdt->btj", wx[rank:].double(), x.double())
        bc_bound = torch.einsum("jd,bdt->btj", wx[rank:].double().abs(), x.double().abs())
        got = torch.cat([Bm, Cm], dim=-1).double()
        assert ((got - bc).abs() <= 1e-5 * bc_bound + 1e-30).all()
    dt64 = torch.einsum("jd,bdt->btj", wx[:rank].double(), x.double())
    ref = torch.einsum("dk,btk->bdt", wdt.double(), dt64)
    bound = torch.einsum("dk,btk->bdt", wdt.double().abs(),
                         torch.einsum("jd,bdt->btj", wx[:rank].double().abs(), x.double().abs()))
    assert ((delta.double() - ref).abs() <= 2e-5 * bound + 1e-30).all()
    assert cuda.check_device_error() == 0


DTPROJ_CASES = [
    (1, 1536, 1024, 48),   # Mamba-130m
    (2, 5120, 300, 160),   # Mamba-2.8B widths, ragged seqlen (scalar tail stores)
    (3, 70, 130, 7),       # dim and seqlen off the 64 x 128 tile, rank off the 16-step
    (1, 64, 1, 48),        # one token
]


@pytest.mark.parametrize("batch,dim,seqlen,rank", DTPROJ_CASES)
def test_dt_proj_matches_float64(batch, dim, seqlen, rank):
    """dt_proj (delta[b, d, t] = sum_k W[d, k] dt[b, t, k]) against a float64
    matmul of the same fp32 inputs: elementwise within 1e-5 of sum |W||dt|,
    normwise 1e-6; repeated calls are bit-identical."""
    g = torch.Generator(device="cpu").manual_seed(batch * 11 + dim + rank)
    dt = torch.randn(batch, seqlen, rank, generator=g).cuda()
    w = (torch.randn(dim, rank, generator=g) * rank ** -0.5).cuda()
    delta = cuda.dt_proj(dt, w)
    ref = torch.einsum("dk,btk->bdt", w.double(), dt.double())
    bound = torch.einsum("dk,btk->bdt", w.double().abs(), dt.double().abs())
    got = delta.double()
    assert ((got - ref).abs() <= 1e-5 * bound + 1e-30).all()
    assert float((got - ref).norm() / ref.norm()) < 1e-6
    assert torch.equal(delta, cuda.dt_proj(dt, w))
    assert cuda.check_device_error() == 0


@pytest.mark.parametrize("batch,dim,width", [(1, 1536, 4), (3, 70, 4), (2, 33, 1), (2, 40, 8)])
def test_conv1d_step_matches_torch_over_several_steps(batch, dim, width):
    """Decoding steps of the causal convolution: the window shifts in the new
    input (read through a batch stride, as the x half of a one-token in_proj
    output) and y = silu(bias + w . window), for 5 consecutive steps."""
    g = torch.Generator(device="cpu").manual_seed(dim + width)
    state = torch.randn(batch, dim, width, generator=g).cuda()
    w = torch.randn(dim, 1, width, generator=g).cuda()
    bias = torch.randn(dim, generator=g).cuda()
    ref_state = state.clone()
    for step in range(5):
        xz = torch.randn(batch, 2 * dim, 1, generator=g).cuda()
        y = cuda.causal_conv1d_step(state, xz[:, :dim, 0], w, bias)
        ref_state = torch.cat([ref_state[..., 1:], xz[:, :dim]], dim=-1)
        ref = F.silu((ref_state * w[:, 0, :]).sum(-1) + bias)
        assert torch.equal(state, ref_state), step
        torch.testing.assert_close(y, ref, rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("batch,dim,rank", [(1, 1536, 48), (3, 200, 8), (2, 130, 64)])
def test_ssm_decode_step_matches_the_scan_op(batch, dim, rank):
    """The fused decode step (dt_proj, softplus, exp(delta A) update in place,
    C.h + D u, silu(z) gate) equals SelectiveScanFusedExact at seqlen 1 with
    h0/h_last and dt_proj computed by torch, for 3 consecutive steps
    (tolerance of the op's Exact tests: 1e-5 relative)."""
    g = torch.Generator(device="cpu").manual_seed(dim + rank)
    dev = torch.device("cuda", 0)
    N = 16
    rnd = lambda *s, sc=1.0: (torch.randn(*s, generator=g) * sc).to(dev)  # noqa: E731
    wdt, bias = rnd(dim, rank, sc=0.1), rnd(dim, sc=0.5) - 2.0
    A = -torch.arange(1, N + 1, dtype=torch.float32, device=dev).repeat(dim, 1) * \
        (rnd(dim, 1).abs() + 0.5)
    Dv = rnd(dim)
    state = rnd(batch, dim, N, sc=0.3)
    ref_state = state.clone()
    for step in range(3):
        u, dt = rnd(batch, dim), rnd(batch, rank)
        zz = rnd(batch, 2 * dim)[:, dim:]  # strided z, as the z half of in_proj's output
        Bm, Cm = rnd(batch, N), rnd(batch, N)
        y = cuda.ssm_decode_step(u, zz, dt, Bm, Cm, wdt, bias, A, Dv, state)
        delta = torch.matmul(dt, wdt.t()).unsqueeze(-1)  # [B, D, 1] before the bias
        new = torch.empty_like(ref_state)
        ref = cuda.selective_scan("SelectiveScanFusedExact", u.unsqueeze(-1).contiguous(), delta,
                                  A, Bm.unsqueeze(1).contiguous(), Cm.unsqueeze(1).contiguous(),
                                  Dv, zz.unsqueeze(-1).contiguous(), delta_bias=bias,
                                  h0=ref_state, h_last=new)
        ref_state = new
        torch.testing.assert_close(y, ref[..., 0], rtol=1e-5, atol=1e-6)
        torch.testing.assert_close(state, ref_state, rtol=1e-5, atol=1e-6)
    assert cuda.check_device_error() == 0


@pytest.mark.parametrize("batch,cols,rows", [(1, 768, 3072), (3, 64, 10), (2, 1024, 777)])
def test_rmsnorm_gemv_matches_float64(batch, cols, rows):
    """weight @ rmsnorm(x) for decoding tokens against float64: normwise 1e-6."""
    g = torch.Generator(device="cpu").manual_seed(cols + rows)
    x = torch.randn(batch, cols, generator=g).cuda()
    nw = (1 + 0.1 * torch.randn(cols, generator=g)).cuda()
    w = (torch.randn(rows, cols, generator=g) * 0.02).cuda()
    got = cuda.rmsnorm_gemv(x, nw, 1e-5, w)
    x64 = x.double()
    hn = x64 * torch.rsqrt(x64.pow(2).mean(-1, keepdim=True) + 1e-5) * nw.double()
    ref = hn @ w.double().t()
    assert float((got.double() - ref).norm() / ref.norm()) < 1e-6
    assert torch.equal(got, cuda.rmsnorm_gemv(x, nw, 1e-5, w))


@pytest.mark.parametrize("batch,cols,rows,res", [(1, 1536, 768, True), (3, 64, 10, False),
                                                 (2, 768, 50280, False)])
def test_gemv_matches_float64(batch, cols, rows, res):
    """(residual +) W x for decoding tokens (out_proj, the LM head) against float64."""
    g = torch.Generator(device="cpu").manual_seed(cols + rows)
    x = torch.randn(batch, cols, generator=g).cuda()
    w = (torch.randn(rows, cols, generator=g) * 0.02).cuda()
    r = torch.randn(batch, rows, generator=g).cuda() if res else None
    got = cuda.gemv(x, w, residual=r)
    ref = x.double() @ w.double().t() + (r.double() if res else 0)
    assert float((got.double() - ref).norm() / ref.norm()) < 1e-6
