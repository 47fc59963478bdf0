"""GPU: the Mamba language model with every selective scan on the CUDA op.

Oracle: transformers' MambaForCausalLM with the same weights. Without the
mamba-ssm kernels it runs MambaMixer.slow_forward: exact discretisation
exp(delta*A), softplus(dt_proj(x)), a sequential scan in torch. Our model
sends the scan through SelectiveScanFusedExact with dt_proj.bias as the
op's delta_bias.

At Mamba-130m depth (24 random-initialised blocks) fp32 rounding differences
of any origin (a different GEMM algorithm is enough) grow about 1000-fold
from the first block to the logits, so the 130m tests use the float64 run
of the transformers model as ground truth and require our fp32 logits to be
no further from it than transformers' own fp32 run is (with a 3x margin).
"""
import warnings

import pytest
import torch

from mamba_onnx.model import MambaConfig, MambaLM, mamba_130m

pytestmark = pytest.mark.gpu

transformers = pytest.importorskip("transformers")


def _hf(cfg: MambaConfig, seed: int, device):
    torch.manual_seed(seed)
    hf_cfg = transformers.MambaConfig(vocab_size=cfg.vocab_size, hidden_size=cfg.d_model,
                                      state_size=cfg.d_state, num_hidden_layers=cfg.n_layer,
                                      expand=cfg.expand, conv_kernel=cfg.d_conv,
                                      layer_norm_epsilon=cfg.rms_eps)
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        return transformers.MambaForCausalLM(hf_cfg).to(device).eval()


def _ids(vocab, L, seed, device, batch=1):
    g = torch.Generator(device=device).manual_seed(seed)
    return torch.randint(0, vocab, (batch, L), device=device, generator=g)


def _normrel(a, b):
    return ((a.double() - b.double()).norm() / b.double().norm()).item()


@torch.no_grad()
def _hf_logits(hf, ids):
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        return hf(ids).logits


def test_small_model_matches_transformers(cuda_device):
    cfg = MambaConfig(d_model=64, n_layer=2, vocab_size=100)
    hf = _hf(cfg, 1, cuda_device)
    ours = MambaLM(cfg).load_hf_state_dict(hf.state_dict()).to(cuda_device)
    for batch, L in [(1, 40), (3, 77), (2, 300)]:
        ids = _ids(cfg.vocab_size, L, batch + L, cuda_device, batch)
        assert _normrel(ours(ids), _hf_logits(hf, ids)) < 1e-5, (batch, L)


def test_batched_forward_equals_each_sequence_alone(cuda_device):
    """Mamba-130m widths (2 blocks), batch 3 x 256 tokens: out_proj splits K
    through one shared workspace per batch entry in turn, and the scans'
    chunk plans differ from the single-sequence ones; every sequence's logits
    must match its own batch-1 forward."""
    cfg = MambaConfig(n_layer=2)
    model = MambaLM(cfg).init_random(4).to(cuda_device)
    ids = _ids(cfg.vocab_size, 256, 11, cuda_device, batch=3)
    batched = model(ids)
    for b in range(3):
        alone = model(ids[b:b + 1])
        assert _normrel(batched[b:b + 1], alone) < 1e-5, b


@pytest.mark.parametrize("L", [64, 1024])
def test_mamba_130m_matches_transformers_float64(cuda_device, L):
    """L = 1024, batch 1 is the Mamba-130m forward workload (24 blocks)."""
    cfg = mamba_130m()
    hf = _hf(cfg, 2, cuda_device)
    ours = MambaLM(cfg).load_hf_state_dict(hf.state_dict()).to(cuda_device)
    ids = _ids(cfg.vocab_size, L, 7, cuda_device)
    got = ours(ids)
    ref32 = _hf_logits(hf, ids)
    ref64 = _hf_logits(hf.double(), ids)
    e_ours, e_hf32 = _normrel(got, ref64), _normrel(ref32, ref64)
    assert e_ours <= 3 * e_hf32 + 1e-6, (e_ours, e_hf32)
    assert _normrel(got, ref32) < 1e-3
    assert torch.isfinite(got).all()


@pytest.mark.parametrize("cfg", [MambaConfig(d_model=64, n_layer=2, vocab_size=100), mamba_130m()],
                         ids=["small", "130m"])
def test_prefill_then_decode_matches_forward(cuda_device, cfg):
    """Prompt of 100 tokens, then 24 single-token steps through the scan's
    h0/h_last: the logits equal those of one forward over all 124 tokens."""
    model = MambaLM(cfg).init_random(seed=11).to(cuda_device)
    ids = _ids(cfg.vocab_size, 124, 3, cuda_device, batch=2)
    full = model(ids)
    logits, state = model.prefill(ids[:, :100])
    tol = 1e-5 if cfg.n_layer == 2 else 1e-3
    assert _normrel(logits, full[:, :100]) < tol
    steps = torch.stack([model.step(ids[:, t], state) for t in range(100, 124)], dim=1)
    assert _normrel(steps, full[:, 100:]) < tol


def test_cuda_graph_replay_equals_eager(cuda_device):
    model = MambaLM(mamba_130m()).init_random(seed=0).to(cuda_device)
    ids, logits, graph = model.capture(1, 256)
    x = _ids(model.cfg.vocab_size, 256, 5, cuda_device)
    ids.copy_(x)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(logits, model(x))


def test_captured_decode_step_equals_eager(cuda_device):
    """Prefill a prompt, then decode 8 tokens with the CUDA-graphed step and
    with the eager step from the same state: identical logits."""
    model = MambaLM(mamba_130m()).init_random(seed=1).to(cuda_device)
    ids = _ids(model.cfg.vocab_size, 72, 6, cuda_device, batch=2)
    _, state = model.prefill(ids[:, :64])
    g_ids, g_logits, g_state, graph = model.capture_step(2)
    model.copy_state(g_state, state)
    for t in range(64, 72):
        g_ids.copy_(ids[:, t])
        graph.replay()
        eager = model.step(ids[:, t], state)
        torch.cuda.synchronize()
        assert torch.equal(g_logits, eager), t


@pytest.mark.parametrize("batch", [1, 3])
def test_persistent_decode_equals_the_kernel_chain(cuda_device, batch):
    """The one-kernel decoding step (mamba_decode_step: every block and the
    LM head in one cooperative launch) against the chain of per-block
    kernels from the same prefilled state: logits and both states equal bit
    for bit over 6 tokens, eagerly and replayed as a CUDA graph."""
    from mamba_onnx import cuda, model as M

    model = MambaLM(mamba_130m()).init_random(seed=4).to(cuda_device)
    ids = _ids(model.cfg.vocab_size, 40, 8, cuda_device, batch=batch)
    _, state = model.prefill(ids[:, :32])
    chain_state = model.new_state(batch)
    model.copy_state(chain_state, state)
    old = M.DECODE
    try:
        g_ids, g_logits, g_state, graph = model.capture_step(batch)
        model.copy_state(g_state, state)
        for t in range(32, 38):
            M.DECODE = "chain"
            ref = model.step(ids[:, t], chain_state)
            M.DECODE = "persistent"
            got = model.step(ids[:, t], state)
            g_ids.copy_(ids[:, t])
            graph.replay()
            torch.cuda.synchronize()
            assert torch.equal(got, ref), t
            assert torch.equal(g_logits, ref), t
            for a, b, c in zip(state.conv + state.ssm, chain_state.conv + chain_state.ssm,
                               g_state.conv + g_state.ssm):
                assert torch.equal(a, b) and torch.equal(c, b), t
    finally:
        M.DECODE = old
    assert cuda.check_device_error() == 0


def test_decode_barrier_gives_up_and_the_context_survives(cuda_device):
    """The decoding kernel's grid barrier bounded like its scan waits: a
    barrier that no other CTA joins gives up after 20 ms and records
    MAMBA_SCAN_ERR_DEVICE_TIMEOUT (no fault involved); a decoding step then
    runs normally."""
    import time

    from mamba_onnx import cuda

    scratch = torch.zeros(128, dtype=torch.uint8, device=cuda_device)
    assert cuda.check_device_error() == 0
    t0 = time.perf_counter()
    assert cuda.decode_selftest_barrier_timeout(20_000_000, scratch) == 0
    assert cuda.check_device_error() == 6
    assert time.perf_counter() - t0 < 5.0
    assert cuda.decode_selftest_barrier_timeout(0, scratch) == 1
    assert cuda.decode_selftest_barrier_timeout(20_000_000, scratch[:64]) == 3
    model = MambaLM(MambaConfig(d_model=64, n_layer=2, vocab_size=100)).init_random(seed=5)
    model = model.to(cuda_device)
    state = model.new_state(1)
    logits = model.step(torch.tensor([3], device=cuda_device), state)
    assert torch.isfinite(logits).all()
    assert cuda.check_device_error() == 0


def test_forward_with_scans_through_the_ort_op_entry(cuda_device):
    """The 130m forward with each of its 24 scans run through the library's
    ONNX Runtime custom-op entry (RegisterCustomOps, CreateKernelV2,
    KernelComputeV2 on the CUDA-EP host of tests/fake_ort, with dt_proj.bias
    as the op's optional delta_bias input) gives the same logits, bit for bit,
    as the forward calling the C ABI directly: the op layer adds nothing to
    the numbers. The 1x1536x1024 scans take the chunked path, so the kernel's
    per-stream scratch is exercised too."""
    import sys
    from pathlib import Path

    sys.path.insert(0, str(Path(__file__).resolve().parent))
    from fake_ort import ort_shim

    model = MambaLM(mamba_130m()).init_random(seed=2).to(cuda_device)
    x = _ids(model.cfg.vocab_size, 1024, 7, cuda_device)
    scan = ort_shim.OrtScan()
    try:
        via_op = model(x, scan=scan)
        direct = model(x)
        torch.cuda.synchronize()
        assert torch.equal(via_op, direct)
    finally:
        scan.close()
